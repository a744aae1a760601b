"""The oracle restatement reproduces the reference's own outputs bit for bit (CPU).

Fixtures in tests/golden were produced by running garv901/kimi-k3-goalbox's `megabench/tasks/kimi.py`
(reference, compare) on CPU; see tests/golden/make_golden.py.
"""

import hashlib
import os
import tempfile
from pathlib import Path

import pytest
import torch

from oracle import kimi_oracle as ko

GOLDEN = Path(__file__).resolve().parent / "golden"
SERIAL = ["tiny_b3_s21", "tiny_b1_s9", "small_b3_s7"]


def _digest(t):
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def _load(name):
    return torch.load(GOLDEN / f"{name}.pt", weights_only=False)


@pytest.mark.parametrize("name", SERIAL)
def test_generator_matches_reference_digests(name):
    fx = _load(name)
    values = ko.make_inputs(fx["case"], fx["seed"], "cpu", rank=0)
    assert set(values) == set(fx["inputs"])
    for key, want in fx["inputs"].items():
        assert _digest(values[key]) == want, key


@pytest.mark.parametrize("name", SERIAL)
def test_bf16_and_fp32_oracle_bit_exact(name):
    torch.set_num_threads(4)
    fx = _load(name)
    case = fx["case"]
    values = ko.make_inputs(case, fx["seed"], "cpu", rank=0)
    bf16 = ko.reference(case, values, serial=True)
    assert set(bf16) == set(fx["bf16"])
    for key, want in fx["bf16"].items():
        assert torch.equal(bf16[key], want), key
    fp32 = ko.reference(case, values, serial=True, fp32=True)
    for key, want in fx["fp32"].items():
        if key == "recurrent_state_digest":
            assert _digest(fp32["recurrent_state"]) == want
        elif key == "recurrent_state_sample":
            assert torch.equal(fp32["recurrent_state"].flatten()[::97], want)
        else:
            assert torch.equal(fp32[key], want), key
    forced = ko.reference(case, values, serial=True, fp32=True, routes=bf16["expert_ids"])
    assert torch.equal(forced["route_shortfall"], fx["forced_shortfall"])


@pytest.mark.parametrize("name", SERIAL)
def test_band_grader_matches_reference(name):
    fx = _load(name)
    case = fx["case"]
    values = ko.make_inputs(case, fx["seed"], "cpu", rank=0)
    bf16 = fx["bf16"]
    fp32 = ko.reference(case, values, serial=True, fp32=True)
    cands = {
        "oracle": {k: v.clone() for k, v in bf16.items()},
        "fp32": {k: (fp32[k].to(v.dtype) if k not in ("expert_ids", "next_token") else v) for k, v in bf16.items()},
        "noisy": dict(bf16, logits=fx["noisy_logits"]),
        "flipped": dict(bf16, expert_ids=bf16["expert_ids"].flip(-1)),
    }
    for label, cand in cands.items():
        want = fx["grades"][label]
        try:
            got = {"ok": True, "details": ko.compare(case, values, bf16, cand, serial=True)}
        except AssertionError as exc:
            got = {"ok": False, "error": str(exc)}
        assert got == want, label


def _tp_rank(rank, world, fx_path, out_dir, init):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        fx = torch.load(fx_path, weights_only=False)
        case = fx["case"]
        values = ko.make_inputs(case, fx["seed"], "cpu", rank=rank)
        out = ko.reference(case, values)
        grade = ko.compare(case, values, out, {k: v.clone() for k, v in out.items()})
        torch.save({"inputs": {k: _digest(v) for k, v in values.items()}, "bf16": out, "grade": grade},
                   os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_matches_reference():
    import torch.multiprocessing as mp
    path = GOLDEN / "tiny_tp2_b2_s5.pt"
    fx = torch.load(path, weights_only=False)
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_tp_rank, nprocs=2, args=(2, str(path), tmp, (Path(tmp) / "rdv").as_uri()))
        ranks = [torch.load(os.path.join(tmp, f"rank{r}.pt"), weights_only=False) for r in range(2)]
    for got, want in zip(ranks, fx["ranks"]):
        assert got["inputs"] == want["inputs"]
        for key, t in want["bf16"].items():
            assert torch.equal(got["bf16"][key], t), key
        assert got["grade"] == want["grade"]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_c_decode_matches_torch_decode_on_every_scale_byte(dtype):
    """oracle/mxfp4.c reproduces the torch restatement of quantization.py:40-51 bit for bit, for every E8M0
    byte (0: subnormal products, 254: overflow to inf, 255: NaN groups) and every code byte."""
    from kimi_k3_goalbox_b200 import build
    build.build(verbose=False)
    assert ko._c_decode_lib() is not None, "oracle/libkk3_oracle_mxfp4.so was not built"
    g = torch.Generator().manual_seed(5)
    codes = torch.randint(0, 256, (256, 3, 16), generator=g, dtype=torch.uint8)
    codes[:, 0] = torch.arange(256, dtype=torch.uint8)[:, None].expand(256, 16).flip(0)
    scales = torch.arange(256, dtype=torch.uint8)[:, None].expand(256, 3).contiguous()
    want = ko.decode_mxfp4(codes, scales).to(dtype)
    got = ko.decode_mxfp4_as(codes, scales, dtype)
    assert got.shape == want.shape and got.dtype == want.dtype
    nan = want.isnan()
    assert torch.equal(got.isnan(), nan)   # NaN groups agree; NaN payload bits are not part of the contract
    view = torch.int16 if dtype == torch.bfloat16 else torch.int32
    assert torch.equal(got.view(view)[~nan], want.view(view)[~nan])
