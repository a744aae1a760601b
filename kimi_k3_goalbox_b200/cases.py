"""Kimi K3 case geometry and the MegaBench case table (restated from garv901/kimi-k3-goalbox
megabench/cases.py:12-84), as plain dicts shaped like the reference's `Case.to_dict()`."""

from __future__ import annotations

import copy

# megabench/cases.py:48-55
KIMI = {"layers": 93, "experts": 896, "topk": 16, "hidden": 7168, "latent_hidden": 3584, "intermediate": 3072,
        "dense_intermediate": 33792, "first_dense": 1, "shared_experts": 2, "q_heads": 96, "head_dim": 128,
        "q_lora_rank": 1536, "kv_lora_rank": 512, "qk_nope_dim": 128, "qk_rope_dim": 64, "v_head_dim": 128,
        "vocab": 163840, "conv_kernel": 4, "attn_res_block_size": 12, "context": 8192}


def make_case(case_id: str, batch: int, *, layers: int = 93, gpus: int = 8, checkpoint: bool = True,
              suite: str = "p0", note: str = "", params: dict | None = None) -> dict:
    """megabench/cases.py:58-64: one Kimi case (TP = gpus, EP = 1, one launch per rank)."""
    p = KIMI | {"batch": batch, "layers": layers} | (params or {})
    if checkpoint:
        p["checkpoint"] = 1
    return {"id": case_id, "family": "kimi_k3_step", "model": "moonshotai/Kimi-K3", "phase": "decode",
            "params": p, "category": "frontier_hybrid", "suite": suite, "backend": "cuda", "gpus": gpus,
            "tp": gpus, "ep": 1, "max_gpu_launches": 1, "atol": 0.0, "rtol": 0.0, "bf16_rtol": 0.008,
            "ready": True, "note": note}


# megabench/cases.py:67-82
CASES = {c["id"]: c for c in (
    make_case("kimi-k3-tp8-b1-s8192", 1),
    make_case("kimi-k3-tp8-b8-s8192", 8),
    make_case("kimi-k3-tp8-b64-s8192", 64),
    make_case("kimi-k3-syn-l8-tp8-b1-s8192", 1, layers=8, checkpoint=False, suite="p1"),
    make_case("kimi-k3-syn-l8-tp8-b8-s8192", 8, layers=8, checkpoint=False, suite="p1"),
    make_case("kimi-k3-syn-l8-tp8-b64-s8192", 64, layers=8, checkpoint=False, suite="p1"),
    make_case("kimi-k3-dev-l4-tp1-b8-s8192", 8, layers=4, gpus=1, checkpoint=False, suite="p2"),
    make_case("kimi-k3-dev-l8-tp2-b8-s8192", 8, layers=8, gpus=2, checkpoint=False, suite="p2"),
)}


def get_case(case_id: str) -> dict:
    if case_id not in CASES:
        raise ValueError(f"unknown case {case_id}; known: {', '.join(CASES)}")
    return copy.deepcopy(CASES[case_id])


def variant(case: dict, *, tp: int | None = None, **params) -> dict:
    """A copy of `case` with other params and/or TP degree (like dataclasses.replace on a Case)."""
    out = copy.deepcopy(case)
    out["params"].update(params)
    if tp is not None:
        out["gpus"] = out["tp"] = tp
    suffix = "".join(f"-{k}{v}" for k, v in params.items()) + (f"-tp{tp}" if tp else "")
    out["id"] = case["id"] + suffix
    return out


def is_mla(params: dict, layer: int) -> bool:
    """megabench/tasks/kimi.py:44-45."""
    return (layer + 1) % 4 == 0 or layer == params["layers"] - 1
