"""Seeded synthetic per-rank inputs in the reference's layout, generated on the device.

Restates the reference's generator (garv901/kimi-k3-goalbox megabench/tasks/kimi.py:56-69 draws,
:72-122 shapes, :125-144 weights, :164-182 state; per-tensor streams seeded by blake2b(seed:name),
megabench/tasks/distributed.py:25-26) so that bench.py and users get exactly the tensors the MegaBench
harness would hand to run() for the same seed and device. tests/test_synthetic.py pins it to the oracle.
"""

from __future__ import annotations

import hashlib

import torch

from .cases import is_mla


def stream_seed(seed: int, name: str) -> int:
    return int.from_bytes(hashlib.blake2b(f"{seed}:{name}".encode(), digest_size=8).digest(), "little")


def weight_specs(case: dict) -> dict:
    """name -> (shape, dtype, fan_in, split) for one rank (kimi.py:72-122)."""
    p, tp = case["params"], case["tp"]
    h, lh, d, H, L, V = p["hidden"], p["latent_hidden"], p["head_dim"], p["q_heads"], p["layers"], p["vocab"]
    hr, qd = H // tp, H * d // tp
    bf, f32, u8 = torch.bfloat16, torch.float32, torch.uint8
    out = {"embed": ((V // tp, h), bf, h, True), "lm_head": ((V // tp, h), bf, h, True), "fnorm": ((h,), bf, 0, False),
           "output_res_norm": ((h,), bf, 0, False), "output_res_proj": ((h,), bf, h, False)}
    for n in ("ln1", "ln2", "attention_res_norm", "mlp_res_norm"):
        out[n] = ((L, h), bf, 0, False)
    for n in ("attention_res_proj", "mlp_res_proj"):
        out[n] = ((L, h), bf, h, False)
    for l in range(L):
        x = f"l{l}_"
        if is_mla(p, l):
            qr, kr, nr, rd, vd = p["q_lora_rank"], p["kv_lora_rank"], p["qk_nope_dim"], p["qk_rope_dim"], p["v_head_dim"]
            out.update({x + "qa": ((qr, h), bf, h, False), x + "qb": ((hr * (nr + rd), qr), bf, qr, True),
                        x + "ka": ((kr + rd, h), bf, h, False), x + "kb": ((hr * (nr + vd), kr), bf, kr, True),
                        x + "o": ((h, hr * vd), bf, H * vd, True), x + "output_gate": ((hr * vd, h), bf, h, True),
                        x + "qn": ((qr,), bf, 0, False), x + "kn": ((kr,), bf, 0, False)})
        else:
            for n in ("q", "k", "v", "output_gate"):
                out[x + n] = ((qd, h), bf, h, True)
            out.update({x + "o": ((h, qd), bf, H * d, True), x + "fa": ((d, h), bf, h, False),
                        x + "fb": ((qd, d), bf, d, True), x + "beta": ((hr, h), bf, h, True),
                        x + "onorm": ((d,), f32, 0, False), x + "A_log": ((hr,), f32, 0, True),
                        x + "dt_bias": ((qd,), f32, 0, True),
                        x + "conv_weight": ((3, qd, p["conv_kernel"]), f32, p["conv_kernel"], True)})
        if l < p["first_dense"]:
            di = p["dense_intermediate"] // tp
            out.update({x + "gate": ((di, h), bf, h, True), x + "up": ((di, h), bf, h, True),
                        x + "down": ((h, di), bf, p["dense_intermediate"], True)})
        else:
            E, it = p["experts"], p["intermediate"] // tp
            sh = p["intermediate"] * p["shared_experts"] // tp
            out.update({x + "latent_down": ((lh, h), bf, h, False), x + "latent_up": ((h, lh), bf, lh, False),
                        x + "latent_norm": ((lh,), bf, 0, False), x + "router": ((E, h), bf, h, False),
                        x + "router_bias": ((E,), f32, 0, False),
                        x + "gate_blocks": ((E, it, lh // 32, 16), u8, lh, True),
                        x + "gate_scales": ((E, it, lh // 32), u8, 0, True),
                        x + "up_blocks": ((E, it, lh // 32, 16), u8, lh, True),
                        x + "up_scales": ((E, it, lh // 32), u8, 0, True),
                        x + "down_blocks": ((E, lh, it // 32, 16), u8, p["intermediate"], True),
                        x + "down_scales": ((E, lh, it // 32), u8, 0, True),
                        x + "shared_gate": ((sh, h), bf, h, True), x + "shared_up": ((sh, h), bf, h, True),
                        x + "shared_down": ((h, sh), bf, p["intermediate"] * p["shared_experts"], True)})
    return out


def _normal(seed, stream, shape, std, device, dtype=torch.bfloat16, mean=0.0):
    gen = torch.Generator(device=device).manual_seed(stream_seed(seed, stream))
    return (torch.randn(shape, generator=gen, device=device) * std + mean).to(dtype)


def _codes_and_scales(seed, stream, shape, fan_in, device):
    gen = torch.Generator(device=device).manual_seed(stream_seed(seed, stream))
    *lead, cols = shape
    codes = torch.randint(0, 256, (*lead, cols // 32, 16), generator=gen, device=device, dtype=torch.uint8)
    e = round(-torch.log2(torch.tensor(2.93 * fan_in ** 0.5)).item())
    return codes, (126 + e + torch.randint(0, 3, (*lead, cols // 32), generator=gen, device=device)).to(torch.uint8)


def make_inputs(case: dict, seed: int, device, rank: int = 0) -> dict:
    """Weights and state of one rank, identical to the reference's make_inputs for the same seed/device."""
    p, tp, B = case["params"], case["tp"], case["params"]["batch"]
    out = {}
    for name, (shape, dtype, fan_in, split) in weight_specs(case).items():
        stream = f"{name}@{rank}" if split else name
        if name.endswith("_scales"):
            continue
        if name.endswith("_blocks"):
            out[name], out[name[:-7] + "_scales"] = _codes_and_scales(seed, stream, shape[:-2] + (shape[-2] * 32,),
                                                                      fan_in, device)
        elif name.endswith("A_log"):
            out[name] = _normal(seed, stream, shape, 0.5, device, dtype)
        elif name.endswith("dt_bias"):
            out[name] = _normal(seed, stream, shape, 1.0, device, dtype, mean=-4.0)
        elif name.endswith("router_bias"):
            out[name] = _normal(seed, stream, shape, 0.01, device, dtype)
        elif fan_in == 0:
            out[name] = _normal(seed, stream, shape, 0.1, device, dtype, mean=1.0)
        else:
            out[name] = _normal(seed, stream, shape, fan_in ** -0.5, device, dtype)
    gen = torch.Generator(device=device).manual_seed(stream_seed(seed, "token"))
    out["token"] = torch.randint(0, p["vocab"], (B,), generator=gen, device=device)
    out["reset"] = torch.rand((B,), generator=gen, device=device) < 0.25
    out["reset"][0] = False
    if B == 1:
        out["reset"][0] = seed % 3 == 0
    hr, d = p["q_heads"] // tp, p["head_dim"]
    for l in range(p["layers"]):
        x = f"l{l}_"
        if is_mla(p, l):
            out[x + "kv_cache"] = _normal(seed, x + "kv_cache", (B, p["context"], p["kv_lora_rank"]), 1.0, device)
            out[x + "pe_cache"] = _normal(seed, x + "pe_cache", (B, p["context"], p["qk_rope_dim"]), 1.0, device)
        else:
            out[x + "conv_state"] = _normal(seed, f"{x}conv_state@{rank}", (B, 3, hr * d, p["conv_kernel"]), 1.0, device)
            out[x + "recurrent_state"] = _normal(seed, f"{x}recurrent@{rank}", (B, hr, d, d), 0.05, device, torch.float32)
    return out
