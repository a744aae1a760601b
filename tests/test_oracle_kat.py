"""Known-answer and semantic tests of the oracle restatement, mirroring the reference's own unit tests
(garv901/kimi-k3-goalbox megabench/tests/test_kimi.py:25-109), on the same tiny geometry."""

import copy

import pytest
import torch

from oracle import kimi_oracle as ko
from tests.golden.make_golden import TINY

DEV = {"id": "kimi-k3-dev-l4-tp1-b8-s8192", "family": "kimi_k3_step", "gpus": 1, "tp": 1, "ep": 1,
       "params": {"layers": 4, "experts": 896, "topk": 16, "hidden": 7168, "latent_hidden": 3584,
                  "intermediate": 3072, "dense_intermediate": 33792, "first_dense": 1, "shared_experts": 2,
                  "q_heads": 96, "head_dim": 128, "q_lora_rank": 1536, "kv_lora_rank": 512, "qk_nope_dim": 128,
                  "qk_rope_dim": 64, "v_head_dim": 128, "vocab": 163840, "conv_kernel": 4,
                  "attn_res_block_size": 12, "context": 8192, "batch": 8}}


def tiny(batch=3):
    case = copy.deepcopy(DEV)
    case["params"].update(TINY, batch=batch)
    return case


def test_kda_matches_closed_form_transition():
    """test_kimi.py:25-41: S <- S diag(decay) (I - s(b) k k^T) + s(b) v k^T, eight steps."""
    torch.manual_seed(5)
    heads, dim = 3, 16
    state = torch.randn(heads, dim, dim)
    expected = state.clone()
    A, dt = torch.randn(heads), torch.randn(heads, dim)
    for _ in range(8):
        q, k, v, g = (torch.randn(heads, dim) for _ in range(4))
        b = torch.randn(heads)
        nq = q / (q.square().sum(-1, keepdim=True) + 1e-6).sqrt() / dim ** 0.5
        nk = k / (k.square().sum(-1, keepdim=True) + 1e-6).sqrt()
        decay = torch.exp(-5 * torch.sigmoid(torch.exp(A)[:, None] * (g + dt)))
        update = torch.eye(dim)[None] - b.sigmoid()[:, None, None] * nk[:, :, None] * nk[:, None, :]
        expected = torch.bmm(expected, torch.diag_embed(decay)) @ update + b.sigmoid()[:, None, None] * v[:, :, None] * nk[:, None, :]
        output, state = ko.kda_update(q, k, v, g, b, A, dt, state)
        torch.testing.assert_close(state, expected, rtol=2e-5, atol=2e-6)
        torch.testing.assert_close(output, (expected @ nq[:, :, None]).squeeze(-1), rtol=2e-5, atol=2e-6)


def test_synthetic_weights_match_declared_shapes():
    case = tiny()
    values = ko.synthetic_weights(case, 3, "cpu", 0)
    specs = ko.tensor_specs(case)
    assert set(values) == set(specs)
    for name, (shape, dtype, _, _) in specs.items():
        assert (tuple(values[name].shape), values[name].dtype) == (shape, dtype), name
    decoded = ko.decode_mxfp4(values["l1_gate_blocks"], values["l1_gate_scales"])
    rms = decoded.square().mean().sqrt().item()
    assert 0.3 < rms * case["params"]["latent_hidden"] ** 0.5 < 3


def test_batch_rows_equal_single_sequence():
    case = tiny(3)
    values = ko.make_inputs(case, 21, "cpu")
    values["reset"] = torch.tensor([False, True, False])
    batched = ko.reference(case, values, serial=True)
    one = copy.deepcopy(case)
    one["params"]["batch"] = 1
    for b in range(3):
        row = {n: (v[b:b + 1] if n in ("token", "reset") or n.endswith(("_cache", "_state")) else v)
               for n, v in values.items()}
        single = ko.reference(one, row, serial=True)
        torch.testing.assert_close(single["logits"][0], batched["logits"][b], rtol=2e-2, atol=2e-2)
        assert int(single["cache_length"][0]) == int(batched["cache_length"][b])


def test_reset_ignores_state_and_inputs_are_preserved():
    case = tiny(2)
    values = ko.make_inputs(case, 17, "cpu")
    values["reset"] = torch.tensor([True, False])
    before = ko.snapshot(values)
    actual = ko.reference(case, values, serial=True)
    ko.check_unchanged(values, before)
    assert actual["cache_length"].tolist() == [1, case["params"]["context"] + 1]
    changed = {n: (v + 10 if n.endswith(("_cache", "_state")) else v) for n, v in values.items()}
    other = ko.reference(case, changed, serial=True)
    assert torch.equal(actual["logits"][0], other["logits"][0])
    assert not torch.equal(actual["logits"][1], other["logits"][1])


def test_band_accepts_oracle_and_fp32_and_rejects_noise():
    case = tiny(2)
    values = ko.make_inputs(case, 5, "cpu")
    expected = ko.reference(case, values, serial=True)
    ko.compare(case, values, expected, {k: v.clone() for k, v in expected.items()}, serial=True)
    fp32 = ko.reference(case, values, serial=True, fp32=True)
    as_fp32 = {k: (fp32[k].to(v.dtype) if k not in ("expert_ids", "next_token") else v) for k, v in expected.items()}
    ko.compare(case, values, expected, as_fp32, serial=True)
    noisy = dict(expected, logits=expected["logits"] + 0.2 * expected["logits"].std() * torch.randn_like(expected["logits"]))
    with pytest.raises(AssertionError):
        ko.compare(case, values, expected, noisy, serial=True)
    ko.compare(case, values, expected, dict(expected, expert_ids=expected["expert_ids"].flip(-1)), serial=True)
    repeated = expected["expert_ids"].clone()
    repeated[1:, :, 1] = repeated[1:, :, 0]
    with pytest.raises(AssertionError):
        ko.compare(case, values, expected, dict(expected, expert_ids=repeated), serial=True)


def test_forced_routes_and_shortfall():
    case = tiny(2)
    values = ko.make_inputs(case, 9, "cpu")
    own = ko.reference(case, values, serial=True, fp32=True)
    forced = ko.reference(case, values, serial=True, fp32=True, routes=own["expert_ids"])
    assert torch.equal(own["logits"], forced["logits"])
    assert float(forced["route_shortfall"].max()) == 0.0
    worst = own["expert_ids"].clone()
    p = case["params"]
    for layer in range(p["first_dense"], p["layers"]):
        worst[layer] = torch.arange(p["experts"] - p["topk"], p["experts"])
    bad = ko.reference(case, values, serial=True, fp32=True, routes=worst)
    assert float(bad["route_shortfall"].max()) > ko.ROUTE_FLOOR


def test_mxfp4_decode_table_and_nan_scale():
    codes = torch.arange(256, dtype=torch.uint8).view(16, 16)
    scales = torch.full((16,), 127, dtype=torch.uint8)
    scales[3] = 255
    scales[4] = 120
    out = ko.decode_mxfp4(codes, scales)
    table = torch.tensor(ko.E2M1_VALUES)
    flat = torch.stack((codes & 15, codes >> 4), -1).flatten(-2).long()
    want = table[flat] * torch.pow(2.0, scales.float() - 127)[:, None]
    want[3] = torch.nan
    assert out.shape == (512,)
    torch.testing.assert_close(out.view(16, 32), want, equal_nan=True, rtol=0, atol=0)
