"""Multi-step decoding with in-place cache append (kk3_step_append), graded step by step against the oracle.

The reference chains decode steps by feeding one step's outputs back as the next step's state: the MLA latent
and rope rows it wrote become the cache, the KDA conv and recurrent states carry over
(garv901/kimi-k3-goalbox tools/verify_kimi_vs_hf.py:145-154). kk3_step_append does that in place: each row
attends its first lengths[b] cached positions plus the new token, appends its new MLA entries to the caches at
position lengths[b], updates the stacked KDA states in place, and reports cache_length = lengths + 1, which is
fed back as the next step's lengths.

Each step is graded with the reference's band rule (oracle/kimi_oracle.py:compare, kimi.py:370-462) against
the oracle run on exactly the state the kernel held before the step (the cache truncated to the row's length,
the states as the previous step left them), so every step of the chain is checked on identical inputs. Rows
with different lengths (a row reset mid-chain) are graded one row at a time; the step is row-independent
(the reference's own batch-independence test, megabench/tests/test_kimi.py:54-65).
"""

from __future__ import annotations

import pytest
import torch

from kimi_k3_goalbox_b200 import cases
from oracle import kimi_oracle as ko

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from kimi_k3_goalbox_b200.runtime import StepContext
    from tests import gpu_helpers as gh

CAPACITY = 8


def _stacked_states(case: dict, values: dict) -> tuple[torch.Tensor, torch.Tensor]:
    """Stack the per-layer KDA states into one tensor each and make the per-layer inputs views of it, so the
    step's state outputs (the stacked tensors) update the inputs in place."""
    kda = ko.kda_layer_ids(case)
    conv = torch.stack([values[f"l{l}_conv_state"] for l in kda])
    rec = torch.stack([values[f"l{l}_recurrent_state"] for l in kda])
    for i, l in enumerate(kda):
        values[f"l{l}_conv_state"] = conv[i]
        values[f"l{l}_recurrent_state"] = rec[i]
    return conv, rec


def _oracle_inputs(case: dict, values: dict, rows: list[int], length: int) -> tuple[dict, dict]:
    """The oracle's view of rows `rows` before the step: their caches truncated to `length` positions (at least
    one, so that reset rows still have a cache tensor), copies of their states, the shared weights."""
    sub = cases.variant(case, batch=len(rows), context=max(length, 1))
    idx = torch.tensor(rows, device=values["token"].device)
    per_row = {"token", "reset"} | {f"l{l}_{n}" for l in range(case["params"]["layers"])
                                    for n in ("kv_cache", "pe_cache", "conv_state", "recurrent_state")}
    out = {}
    for name, t in values.items():
        if name not in per_row:
            out[name] = t
        elif name.endswith(("kv_cache", "pe_cache")):
            out[name] = t.index_select(0, idx)[:, :max(length, 1)].clone()
        else:
            out[name] = t.index_select(0, idx).clone()
    return sub, out


def _slice_outputs(actual: dict, rows: list[int]) -> dict:
    idx = torch.tensor(rows, device=actual["logits"].device)
    out = {}
    for name, t in actual.items():
        if name in ("logits", "next_token", "cache_length"):
            out[name] = t.index_select(0, idx).clone()
        else:   # [layers, B, ...]
            out[name] = t.index_select(1, idx).clone() if t.numel() else t.clone()
    return out


def _grade_rows(case, values, actual, rows, length):
    sub, vals = _oracle_inputs(case, values, rows, length)
    expected = ko.reference(sub, vals, serial=True)
    return ko.compare(sub, vals, expected, _slice_outputs(actual, rows), serial=True)


@pytest.mark.parametrize("batch,seed", [(3, 31), (5, 29)])
def test_append_chain_matches_oracle_every_step(batch, seed):
    case = gh.small_case(batch, context=CAPACITY)
    p = case["params"]
    mla = ko.mla_layer_ids(case)
    with torch.inference_mode():
        values = ko.make_inputs(case, seed, "cuda")
        conv, rec = _stacked_states(case, values)
        ctx = StepContext(case)
        try:
            lengths = torch.zeros(batch, dtype=torch.int64, device="cuda")
            gen = torch.Generator(device="cuda").manual_seed(seed)
            for step in range(5):
                # step 0 starts every sequence; at step 3 row 1 starts a new sequence (ragged lengths after it)
                reset = torch.zeros(batch, dtype=torch.bool, device="cuda")
                if step == 0:
                    reset[:] = True
                elif step == 3:
                    reset[1] = True
                values["token"] = torch.randint(0, p["vocab"], (batch,), generator=gen, device="cuda")
                values["reset"] = reset
                before = {k: (v.clone() if k.endswith(("kv_cache", "pe_cache", "conv_state", "recurrent_state"))
                              or k in ("token", "reset") else v) for k, v in values.items()}
                outputs = ctx.allocate_outputs()
                outputs["conv_state"], outputs["recurrent_state"] = conv, rec
                ctx.step_append(values, outputs, lengths)
                torch.cuda.synchronize()
                ctx.check()
                actual = {k: v.clone() for k, v in outputs.items()}
                lens = lengths.tolist()
                want_len = [1 if reset[b] else lens[b] + 1 for b in range(batch)]
                assert actual["cache_length"].tolist() == want_len
                # the new MLA entries sit in the caches at each row's old length (0 after a reset)
                for i, l in enumerate(mla):
                    for b in range(batch):
                        pos = 0 if reset[b] else lens[b]
                        assert torch.equal(values[f"l{l}_kv_cache"][b, pos], actual["kv_write"][i, b])
                        assert torch.equal(values[f"l{l}_pe_cache"][b, pos], actual["pe_write"][i, b])
                # band rule per group of rows with the same cached length
                groups: dict[int, list[int]] = {}
                for b in range(batch):
                    groups.setdefault(0 if reset[b] else lens[b], []).append(b)
                for length, rows in sorted(groups.items()):
                    details = _grade_rows(case, before, actual, rows, length)
                    print(f"step {step} rows {rows} cached {length}: "
                          + ", ".join(f"{k}={v['worst_ratio']:.3f}" for k, v in details.items() if "worst_ratio" in v))
                lengths = outputs["cache_length"]   # fed back as the next step's lengths
        finally:
            ctx.close()


def test_append_rejects_a_full_cache():
    """A row whose length reaches the cache capacity makes the step fail cleanly (status KK3_ERR_DEVICE), and the
    failed step marks its integer outputs; the device stays usable."""
    case = gh.small_case(2, context=CAPACITY)
    with torch.inference_mode():
        values = ko.make_inputs(case, 3, "cuda")
        values["reset"] = torch.zeros(2, dtype=torch.bool, device="cuda")
        ctx = StepContext(case)
        try:
            lengths = torch.tensor([CAPACITY, 0], dtype=torch.int64, device="cuda")
            out = ctx.step_append(values, ctx.allocate_outputs(), lengths)
            torch.cuda.synchronize()
            assert ctx.status() == -5
            assert bool((out["next_token"] == -1).all()) and bool((out["cache_length"] == 0).all())
        finally:
            ctx.close()
        assert float(torch.ones(16, device="cuda").sum()) == 16.0
