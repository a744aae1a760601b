"""Helpers shared by the GPU parity tests, smoke() and bench.py: geometries, the host mirror of the kernel's
phase program, and a per-phase comparison of scratch buffers against the oracle's trace."""

from __future__ import annotations

import copy

import torch

from kimi_k3_goalbox_b200 import cases
from kimi_k3_goalbox_b200.cases import is_mla  # noqa: F401
from kimi_k3_goalbox_b200.phase_profile import phase_program

# The smallest geometry the kernels accept: Kimi's fixed head dims, small everything else.
SMALL = {"layers": 5, "hidden": 256, "latent_hidden": 128, "intermediate": 128, "dense_intermediate": 256,
         "q_heads": 2, "head_dim": 128, "q_lora_rank": 128, "kv_lora_rank": 512, "qk_nope_dim": 128,
         "qk_rope_dim": 64, "v_head_dim": 128, "vocab": 512, "experts": 16, "topk": 4, "context": 16,
         "attn_res_block_size": 2}

# KK3_BUF_* ids (include/kk3.h kk3_debug_buffer_id)
BUF = {"prefix": 0, "xa": 1, "xm": 2, "attn_in": 3, "scores": 4, "latent": 5, "shared_act": 6, "x3": 7,
       "route_w": 8, "qkv": 9, "mla_q": 10, "absorbed": 11, "attn_lat": 12, "expert_sum": 13, "blocks": 14,
       "exchange": 15}


def small_case(batch=3, **over) -> dict:
    base = cases.get_case("kimi-k3-dev-l4-tp1-b8-s8192")
    return cases.variant(base, **(SMALL | {"batch": batch} | over))


def rank_equivalent(case_id: str, **over) -> dict:
    """A TP1 case with one TP rank's shard shapes: its arithmetic equals one rank of `case_id` with
    identity reductions (the survey's one-rank-equivalent method)."""
    c = cases.get_case(case_id)
    p, tp = dict(c["params"]), c["tp"]
    for key in ("q_heads", "vocab", "intermediate", "dense_intermediate"):
        p[key] //= tp
    p.update(over)
    p.pop("checkpoint", None)
    return dict(copy.deepcopy(c), id=c["id"] + "-rank-equivalent", gpus=1, tp=1, params=p)


def rel_l2(got: torch.Tensor, want: torch.Tensor) -> float:
    g, w = got.float().flatten(), want.float().flatten()
    return float((g - w).norm() / w.norm().clamp_min(1e-30))


def checkpoints(case: dict) -> list[tuple[int, str, str, torch.dtype, tuple]]:
    """(stop_phase, label, buffer, dtype, shape, trace key) for the per-phase comparison."""
    p = case["params"]
    B, h, lh, hr = p["batch"], p["hidden"], p["latent_hidden"], p["q_heads"] // case["tp"]
    out = []
    for i, (name, l) in enumerate(phase_program(p)):
        stop = i + 1
        if name == "embed":
            out.append((stop, "embed", "prefix", torch.bfloat16, (B, h), "embed"))
        elif name == "attn_prologue":
            out.append((stop, f"l{l} x_attn", "xa", torch.bfloat16, (B, h), f"l{l}_x_attn"))
        elif name == "kda":
            out.append((stop, f"l{l} kda out", "attn_in", torch.bfloat16, (B, hr * 128), f"l{l}_attn_in"))
        elif name == "mla_qb":
            out.append((stop, f"l{l} mla q", "mla_q", torch.bfloat16, (B, hr, 192), f"l{l}_q"))
        elif name == "mla_absorb":
            out.append((stop, f"l{l} absorbed", "absorbed", torch.bfloat16, (B, hr, 512), f"l{l}_absorbed"))
        elif name == "mla_combine":
            out.append((stop, f"l{l} attended", "absorbed", torch.bfloat16, (B, hr, 512), f"l{l}_attn_latent"))
            out.append((stop, f"l{l} mla out", "attn_in", torch.bfloat16, (B, hr * 128), f"l{l}_attn_in"))
        elif name == "mlp_prologue":
            out.append((stop, f"l{l} x_mlp", "xm", torch.bfloat16, (B, h), f"l{l}_x_mlp"))
        elif name == "moe_in":
            out.append((stop, f"l{l} latent", "latent", torch.bfloat16, (B, lh), f"l{l}_latent"))
        elif name == "moe_combine":
            out.append((stop, f"l{l} expert_sum", "expert_sum", torch.float32, (B, lh), f"l{l}_expert_sum_local"))
        elif name == "latent_up":
            out.append((stop, f"l{l} prefix", "prefix", torch.bfloat16, (B, h), f"l{l}_prefix"))
        elif name == "head_prologue":
            out.append((stop, "x_head", "xa", torch.bfloat16, (B, h), "x_head"))
    return out


def diagnose(ctx, case: dict, values: dict, trace: dict, limit: float = 0.05, verbose: bool = True) -> list:
    """Run the kernel phase by phase and compare scratch buffers with the oracle trace. Returns rows of
    (label, rel_l2). Diagnostic only: routing near-ties may legitimately change later layers."""
    rows = []
    for stop, label, buf, dtype, shape, key in checkpoints(case):
        if key not in trace:
            continue
        ctx.step(values, stop_phase=stop)
        torch.cuda.synchronize()
        ctx.check()
        got = ctx.debug_buffer(BUF[buf], dtype, shape)
        want = trace[key].to(got.device).reshape(shape)
        err = rel_l2(got, want)
        rows.append((label, err))
        if verbose:
            print(f"  {label:22s} rel_l2 = {err:.3e}{'   <-- large' if err > limit else ''}")
    return rows


def load_submission(path, contract: dict):
    """Import the candidate file by path and call its build(contract), as the reference harness does
    (megabench/harness/runner.py:53-69): a fresh module named megabench_candidate, the file's folder first on
    sys.path, build must be callable and must return a callable."""
    import importlib.util
    import sys
    from pathlib import Path

    path = Path(path).resolve()
    spec = importlib.util.spec_from_file_location("megabench_candidate", path)
    module = importlib.util.module_from_spec(spec)
    sys.path.insert(0, str(path.parent))
    spec.loader.exec_module(module)
    assert callable(getattr(module, "build", None)), "submission must export build(case)"
    runner = module.build(contract)
    assert callable(runner), "build(case) must return a callable run(inputs)"
    return runner


def audit_launches(fn, inputs: dict) -> list[str]:
    """Names of the GPU activities one call of fn(inputs) produces, recorded with torch.profiler the way the
    reference harness audits a candidate's launch budget (megabench/harness/benchmark.py:49-74)."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        fn(inputs)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    if not names:   # diagnostics for the assertion that follows: what the profiler did record
        print("profiler events:", [(e.name, str(e.device_type)) for e in prof.events()][:40])
    return names
