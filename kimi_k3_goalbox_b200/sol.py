"""Per-rank HBM traffic floor of one Kimi K3 decode step, restated from garv901/kimi-k3-goalbox
megabench/sol.py:27-73 (the reference's speed-of-light model: useful bytes of the slowest rank)."""

from __future__ import annotations

from .cases import is_mla

BF16, FP32, INT64 = 2, 4, 8
REFERENCE_TB_S = 8.0   # sol.py:18


def _mxfp4_bytes(rows: int, cols: int) -> int:
    return rows * cols // 2 + rows * cols // 32


def floor_bytes(case: dict) -> dict:
    """Component byte counts and their total for the slowest rank (sol.py:39-68)."""
    p, tp = case["params"], case["tp"]
    B, h, lh, d, H = p["batch"], p["hidden"], p["latent_hidden"], p["head_dim"], p["q_heads"]
    qdim, ctx, E, k = H * d, p["context"], p["experts"], p["topk"]
    qr, kr, nr, rd, vd = p["q_lora_rank"], p["kv_lora_rank"], p["qk_nope_dim"], p["qk_rope_dim"], p["v_head_dim"]
    inter, shared = p["intermediate"] // tp, p["intermediate"] * p["shared_experts"] // tp
    mla = [l for l in range(p["layers"]) if is_mla(p, l)]
    kda = [l for l in range(p["layers"]) if not is_mla(p, l)]
    moe = p["layers"] - p["first_dense"]
    distinct = E * (1 - (1 - k / E) ** B)
    comps = {
        "kda_weights": len(kda) * BF16 * (5 * qdim // tp * h + d * h + qdim // tp * d + H // tp * h)
        + len(kda) * FP32 * 3 * qdim // tp * p["conv_kernel"],
        "mla_weights": len(mla) * BF16 * (qr * h + H // tp * (nr + rd) * qr + (kr + rd) * h + H // tp * (nr + vd) * kr
                                          + 2 * H // tp * vd * h),
        "dense_ffn": p["first_dense"] * 3 * BF16 * p["dense_intermediate"] // tp * h,
        "moe_dense_parts": moe * BF16 * (E * h + 2 * lh * h + 3 * shared * h),
        "routed_experts": int(moe * distinct * (2 * _mxfp4_bytes(inter, lh) + _mxfp4_bytes(lh, inter))),
        "norms_and_residual_mixers": p["layers"] * 6 * h * BF16,
        "lm_head": p["vocab"] // tp * h * BF16,
        "embedding_rows": B * h * BF16,
        "mla_cache_reads": B * len(mla) * ctx * (kr + rd) * BF16,
        "kda_state": len(kda) * B * (2 * H // tp * d * d * FP32 + 2 * 3 * qdim // tp * p["conv_kernel"] * BF16),
        "outputs": B * (p["vocab"] // tp * FP32 + INT64 * (2 + p["layers"] * k) + len(mla) * (kr + rd) * BF16),
    }
    comps = {n: int(v) for n, v in comps.items()}
    return {"components": comps, "minimum_bytes": sum(comps.values()), "distinct_experts": distinct}


def floor_us(case: dict, tb_s: float = REFERENCE_TB_S) -> float:
    return floor_bytes(case)["minimum_bytes"] / (tb_s * 1e12) * 1e6
