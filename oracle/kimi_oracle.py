"""TEST INFRASTRUCTURE ONLY: a restatement of the reference's Kimi K3 decode-step oracle.

The reference (garv901/kimi-k3-goalbox) specifies one decode step per tensor-parallel rank as a
PyTorch program in `megabench/tasks/kimi.py`, with helpers in `megabench/tasks/common.py`,
`megabench/tasks/quantization.py` and `megabench/tasks/distributed.py`. This module restates that
program with the same arithmetic (same dtypes, same rounding points, same torch reductions) so that,
on CPU, it reproduces the reference's outputs bit for bit (pinned by `tests/golden`). It is the
checker for the CUDA path and the timed CPU baseline; the product never calls it.

A `case` here is the dict the reference's `Case.to_dict()` produces (keys `id`, `gpus`, `tp`, `ep`,
`params`, ...).
"""

from __future__ import annotations

import hashlib

import torch
import torch.distributed as dist
import torch.nn.functional as F

# kimi.py:38-40 -- the oracle band constants
BAND = 2.0
FLOOR = 2e-3
ROUTE_FLOOR = 1e-3

# quantization.py:8-9 -- E2M1 code -> value (bit 3 is the sign)
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
               -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def stream_seed(seed: int, name: str) -> int:
    """Per-tensor generator seed: blake2b-64 of "seed:name", little endian (tasks/distributed.py:25-26)."""
    digest = hashlib.blake2b(f"{seed}:{name}".encode(), digest_size=8).digest()
    return int.from_bytes(digest, "little")


def _params(case) -> dict:
    return case["params"]


def is_mla(case, layer: int) -> bool:
    """Gated-MLA layers are 3, 7, 11, ... and the last layer (kimi.py:44-45)."""
    return (layer + 1) % 4 == 0 or layer == _params(case)["layers"] - 1


def mla_layer_ids(case) -> list[int]:
    return [l for l in range(_params(case)["layers"]) if is_mla(case, l)]


def kda_layer_ids(case) -> list[int]:
    return [l for l in range(_params(case)["layers"]) if not is_mla(case, l)]


def tensor_specs(case) -> dict:
    """Per-rank weight tensors: name -> (shape, dtype, fan_in, split over TP) (kimi.py:72-122)."""
    p, tp = _params(case), case["tp"]
    h, lh, d, H = p["hidden"], p["latent_hidden"], p["head_dim"], p["q_heads"]
    L, V = p["layers"], p["vocab"]
    qdim = H * d
    for n in (H, V, p["intermediate"], p["dense_intermediate"]):
        if n % tp:
            raise ValueError("Kimi attention heads, vocabulary and FFN intermediate must divide TP")
    if (p["intermediate"] // tp) % 32:
        raise ValueError("MXFP4 down-projection shards must align to groups of 32")
    bf, f32, u8 = torch.bfloat16, torch.float32, torch.uint8
    specs = {
        "embed": ((V // tp, h), bf, h, True),
        "lm_head": ((V // tp, h), bf, h, True),
        "fnorm": ((h,), bf, 0, False),
        "output_res_norm": ((h,), bf, 0, False),
        "output_res_proj": ((h,), bf, h, False),
    }
    for name in ("ln1", "ln2", "attention_res_norm", "mlp_res_norm"):
        specs[name] = ((L, h), bf, 0, False)
    for name in ("attention_res_proj", "mlp_res_proj"):
        specs[name] = ((L, h), bf, h, False)
    hr = H // tp
    for layer in range(L):
        pre = f"l{layer}_"
        if is_mla(case, layer):
            qr, kr = p["q_lora_rank"], p["kv_lora_rank"]
            nr, rd, vd = p["qk_nope_dim"], p["qk_rope_dim"], p["v_head_dim"]
            specs.update({
                pre + "qa": ((qr, h), bf, h, False),
                pre + "qb": ((hr * (nr + rd), qr), bf, qr, True),
                pre + "ka": ((kr + rd, h), bf, h, False),
                pre + "kb": ((hr * (nr + vd), kr), bf, kr, True),
                pre + "o": ((h, hr * vd), bf, H * vd, True),
                pre + "output_gate": ((hr * vd, h), bf, h, True),
                pre + "qn": ((qr,), bf, 0, False),
                pre + "kn": ((kr,), bf, 0, False),
            })
        else:
            for name in ("q", "k", "v", "output_gate"):
                specs[pre + name] = ((qdim // tp, h), bf, h, True)
            specs.update({
                pre + "o": ((h, qdim // tp), bf, qdim, True),
                pre + "fa": ((d, h), bf, h, False),
                pre + "fb": ((qdim // tp, d), bf, d, True),
                pre + "beta": ((hr, h), bf, h, True),
                pre + "onorm": ((d,), f32, 0, False),
                pre + "A_log": ((hr,), f32, 0, True),
                pre + "dt_bias": ((qdim // tp,), f32, 0, True),
                pre + "conv_weight": ((3, qdim // tp, p["conv_kernel"]), f32, p["conv_kernel"], True),
            })
        if layer < p["first_dense"]:
            inter = p["dense_intermediate"] // tp
            specs.update({
                pre + "gate": ((inter, h), bf, h, True),
                pre + "up": ((inter, h), bf, h, True),
                pre + "down": ((h, inter), bf, p["dense_intermediate"], True),
            })
        else:
            E, inter = p["experts"], p["intermediate"] // tp
            shared = p["intermediate"] * p["shared_experts"] // tp
            specs.update({
                pre + "latent_down": ((lh, h), bf, h, False),
                pre + "latent_up": ((h, lh), bf, lh, False),
                pre + "latent_norm": ((lh,), bf, 0, False),
                pre + "router": ((E, h), bf, h, False),
                pre + "router_bias": ((E,), f32, 0, False),
                pre + "gate_blocks": ((E, inter, lh // 32, 16), u8, lh, True),
                pre + "gate_scales": ((E, inter, lh // 32), u8, 0, True),
                pre + "up_blocks": ((E, inter, lh // 32, 16), u8, lh, True),
                pre + "up_scales": ((E, inter, lh // 32), u8, 0, True),
                pre + "down_blocks": ((E, lh, inter // 32, 16), u8, p["intermediate"], True),
                pre + "down_scales": ((E, lh, inter // 32), u8, 0, True),
                pre + "shared_gate": ((shared, h), bf, h, True),
                pre + "shared_up": ((shared, h), bf, h, True),
                pre + "shared_down": ((h, shared), bf, p["intermediate"] * p["shared_experts"], True),
            })
    return specs


def _gaussian(seed, stream, shape, std, device, dtype=torch.bfloat16, mean=0.0):
    """kimi.py:56-58: FP32 normal draws from a per-stream generator, scaled, shifted, then cast."""
    gen = torch.Generator(device=device).manual_seed(stream_seed(seed, stream))
    return (torch.randn(shape, generator=gen, device=device) * std + mean).to(dtype)


def _mxfp4_random(seed, stream, shape, fan_in, device):
    """kimi.py:61-69: uniform E2M1 bytes and E8M0 exponents near 1/(2.93*sqrt(fan_in))."""
    gen = torch.Generator(device=device).manual_seed(stream_seed(seed, stream))
    *lead, cols = shape
    codes = torch.randint(0, 256, (*lead, cols // 32, 16), generator=gen, device=device, dtype=torch.uint8)
    centre = round(-torch.log2(torch.tensor(2.93 * fan_in ** 0.5)).item())
    jitter = torch.randint(0, 3, (*lead, cols // 32), generator=gen, device=device)
    return codes, (127 + centre - 1 + jitter).to(torch.uint8)


def synthetic_weights(case, seed: int, device, rank: int) -> dict:
    """kimi.py:125-144: fresh seeded weights; split tensors use the stream `name@rank`."""
    out = {}
    for name, (shape, dtype, fan_in, split) in tensor_specs(case).items():
        stream = f"{name}@{rank}" if split else name
        if name.endswith("_scales"):
            continue
        if name.endswith("_blocks"):
            base = name[: -len("_blocks")]
            out[name], out[base + "_scales"] = _mxfp4_random(
                seed, stream, shape[:-2] + (shape[-2] * 32,), fan_in, device)
        elif name.endswith("A_log"):
            out[name] = _gaussian(seed, stream, shape, 0.5, device, dtype)
        elif name.endswith("dt_bias"):
            out[name] = _gaussian(seed, stream, shape, 1.0, device, dtype, mean=-4.0)
        elif name.endswith("router_bias"):
            out[name] = _gaussian(seed, stream, shape, 0.01, device, dtype)
        elif fan_in == 0:
            out[name] = _gaussian(seed, stream, shape, 0.1, device, dtype, mean=1.0)
        else:
            out[name] = _gaussian(seed, stream, shape, fan_in ** -0.5, device, dtype)
    return out


def make_state(case, seed: int, device, rank: int) -> dict:
    """kimi.py:164-182: tokens, reset flags, MLA latent/rope caches, KDA conv and recurrent states."""
    p, tp, B = _params(case), case["tp"], _params(case)["batch"]
    gen = torch.Generator(device=device).manual_seed(stream_seed(seed, "token"))
    state = {"token": torch.randint(0, p["vocab"], (B,), generator=gen, device=device),
             "reset": torch.rand((B,), generator=gen, device=device) < 0.25}
    state["reset"][0] = False
    if B == 1:
        state["reset"][0] = seed % 3 == 0
    hr, d = p["q_heads"] // tp, p["head_dim"]
    qdim = p["q_heads"] * d // tp
    for layer in range(p["layers"]):
        pre = f"l{layer}_"
        if is_mla(case, layer):
            state[pre + "kv_cache"] = _gaussian(seed, pre + "kv_cache", (B, p["context"], p["kv_lora_rank"]), 1.0, device)
            state[pre + "pe_cache"] = _gaussian(seed, pre + "pe_cache", (B, p["context"], p["qk_rope_dim"]), 1.0, device)
        else:
            state[pre + "conv_state"] = _gaussian(seed, f"{pre}conv_state@{rank}", (B, 3, qdim, p["conv_kernel"]), 1.0, device)
            state[pre + "recurrent_state"] = _gaussian(seed, f"{pre}recurrent@{rank}", (B, hr, d, d), 0.05, device, torch.float32)
    return state


def make_inputs(case, seed: int, device, rank: int = 0) -> dict:
    """kimi.py:185-191 (synthetic source only): weights | state for one rank."""
    if case["ep"] != 1 or case["gpus"] != case["tp"] or not 0 <= rank < case["gpus"]:
        raise ValueError("Kimi requires one TP group spanning all ranks")
    if _params(case).get("checkpoint"):
        raise ValueError("real-checkpoint cases are not generated by the oracle restatement")
    return synthetic_weights(case, seed, device, rank) | make_state(case, seed, device, rank)


def decode_mxfp4(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """quantization.py:40-51: E2M1 nibbles (low nibble first) times 2**(scale-127); scale 255 is NaN."""
    if codes.dtype != torch.uint8 or scales.dtype != torch.uint8:
        raise ValueError("MXFP4 blocks and E8M0 scales must be uint8")
    if codes.shape[:-1] != scales.shape or codes.shape[-1] != 16:
        raise ValueError("invalid MXFP4 block/scale geometry")
    table = torch.tensor(E2M1_VALUES, device=codes.device, dtype=torch.float32)
    nibbles = torch.stack((codes & 15, codes >> 4), dim=-1).flatten(-2)
    values = torch.ldexp(table[nibbles.long()], scales.int()[..., None] - 127)
    values = values.masked_fill(scales[..., None] == 255, torch.nan)
    return values.flatten(-2)


_C_DECODE = None


def _c_decode_lib():
    """The C restatement of the decode (oracle/mxfp4.c), built in-tree by kimi_k3_goalbox_b200/build.py; None
    when it has not been built (the torch restatement above is then used everywhere)."""
    global _C_DECODE
    if _C_DECODE is None:
        import ctypes
        from pathlib import Path
        path = Path(__file__).resolve().parent / "libkk3_oracle_mxfp4.so"
        _C_DECODE = False
        if path.exists():
            lib = ctypes.CDLL(str(path))
            for name in ("kk3o_decode_mxfp4_f32", "kk3o_decode_mxfp4_bf16"):
                getattr(lib, name).argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p]
                getattr(lib, name).restype = None
            _C_DECODE = lib
    return _C_DECODE or None


def decode_mxfp4_as(codes: torch.Tensor, scales: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """decode_mxfp4(codes, scales).to(dtype) for dtype FP32 or BF16. On CPU with the C decode built, the same
    bits come from oracle/mxfp4.c in one multithreaded pass (the torch form materialises int64 indices and
    several FP32 temporaries per value and dominates the oracle's CPU step); elsewhere the torch form."""
    lib = _c_decode_lib()
    if (lib is None or codes.device.type != "cpu" or dtype not in (torch.float32, torch.bfloat16)
            or codes.dtype != torch.uint8 or scales.dtype != torch.uint8
            or codes.shape[:-1] != scales.shape or codes.shape[-1] != 16):
        return decode_mxfp4(codes, scales).to(dtype)
    codes, scales = codes.contiguous(), scales.contiguous()
    out = torch.empty(scales.shape + (32,), dtype=dtype)
    fn = lib.kk3o_decode_mxfp4_f32 if dtype == torch.float32 else lib.kk3o_decode_mxfp4_bf16
    fn(codes.data_ptr(), scales.data_ptr(), scales.numel(), out.data_ptr())
    return out.flatten(-2)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """common.py:13-21 (plain form): FP32 normalise, cast to x's dtype, multiply by the weight in that dtype."""
    xf = x.float()
    scaled = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)
    return scaled.to(x.dtype) * weight.to(x.dtype)


def situ(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """kimi.py:194-196: 4*tanh(g/4)*sigmoid(g) * 25*tanh(u/25), in FP32."""
    g, u = gate.float(), up.float()
    return 4 * torch.tanh(g / 4) * g.sigmoid() * (25 * torch.tanh(u / 25))


def block_mix(prefix, blocks, norm, proj, cast):
    """kimi.py:199-204: softmax over [blocks..., prefix] of rms(v).(norm*proj), mixing in FP32."""
    stacked = torch.stack([*blocks, prefix]).float()
    keys = stacked * torch.rsqrt(stacked.square().mean(-1, keepdim=True) + 1e-5)
    logits = (keys * (norm.float() * proj.float())).sum(-1)
    weights = logits.softmax(0)
    return cast((weights[..., None] * stacked).sum(0))


def kda_update(q, k, v, g, beta, A_log, dt_bias, state):
    """kimi.py:207-215: one gated delta-rule token per row; state is V-first [.., H, V, K] in FP32."""
    qf = q.float() * torch.rsqrt(q.float().square().sum(-1, keepdim=True) + 1e-6) / q.shape[-1] ** 0.5
    kf = k.float() * torch.rsqrt(k.float().square().sum(-1, keepdim=True) + 1e-6)
    decay = (-5 * torch.sigmoid(A_log.float().exp()[:, None] * (g.float() + dt_bias.float()))).exp()
    s = state.float() * decay[..., None, :]
    err = v.float() - torch.einsum("...hvk,...hk->...hv", s, kf)
    s = s + torch.einsum("...hv,...hk->...hvk", err * beta.float().sigmoid()[..., None], kf)
    return torch.einsum("...hvk,...hk->...hv", s, qf), s


def _tp_sum(value, group):
    """kimi.py:343-347: FP32 SUM all-reduce, then back to the value's dtype."""
    acc = value.float().clone()
    dist.all_reduce(acc, group=group)
    return acc.to(value.dtype)


def _argmax_sharded(logits, offset, group, serial):
    """kimi.py:218-227: global argmax of vocabulary-sharded logits; the lowest index wins ties."""
    if serial:
        return logits.argmax(-1)
    best = logits.max(-1).values.clone()
    dist.all_reduce(best, op=dist.ReduceOp.MAX, group=group)
    index = torch.arange(logits.shape[-1], device=logits.device) + offset
    token = torch.where(logits == best[:, None], index, torch.iinfo(torch.int64).max).min(-1).values
    dist.all_reduce(token, op=dist.ReduceOp.MIN, group=group)
    return token


def _rank_context(case, serial, tp_rank, group):
    if serial:
        if (case["gpus"], case["tp"], case["ep"]) != (1, 1, 1):
            raise ValueError("serial validation requires unsharded geometry")
        return 0, None
    if tp_rank is None:
        tp_rank = dist.get_rank() % case["tp"]
    return tp_rank, group


class _Step:
    """Mutable state of one decode step while the oracle walks the layers (kimi.py:249-340)."""

    def __init__(self, case, values, serial, fp32, routes, tp_rank, group, trace):
        self.case, self.values, self.routes = case, values, routes
        self.serial = case["gpus"] == 1 if serial is None else serial
        self.tp_rank, self.group = _rank_context(case, self.serial, tp_rank, group)
        self.act = torch.float32 if fp32 else torch.bfloat16
        self.p = _params(case)
        self.device = values["token"].device
        self.trace = trace
        self.blocks, self.kv_out, self.pe_out, self.state_out = [], [], [], []
        self.conv_out, self.chosen, self.shortfall = [], [], []
        self.prefix = None
        self.keep = ~values["reset"]

    def cast(self, t):
        return t.to(self.act)

    def reduce(self, t):
        return t if self.serial else _tp_sum(t, self.group)

    def rec(self, key, t):
        if self.trace is not None:
            self.trace[key] = t.detach().clone()

    def proj(self, name, x):
        return self.cast(x) @ self.cast(self.values[name]).T


def _embed(st):
    """kimi.py:249-252: masked gather of this rank's vocabulary shard, TP sum."""
    chunk = st.p["vocab"] // st.case["tp"]
    offset = st.tp_rank * chunk
    token = st.values["token"]
    mine = (token >= offset) & (token < offset + chunk)
    rows = torch.where(mine[:, None], st.values["embed"][(token - offset).clamp(0, chunk - 1)], 0)
    st.prefix = st.cast(st.reduce(rows))
    st.rec("embed", st.prefix)


def _mla_attention(st, layer, x):
    """kimi.py:263-283 (gated MLA, absorbed latent form, no rotary)."""
    p, v, pre = st.p, st.values, f"l{layer}_"
    B, hr = p["batch"], p["q_heads"] // st.case["tp"]
    kr, nr, rd, vd = p["kv_lora_rank"], p["qk_nope_dim"], p["qk_rope_dim"], p["v_head_dim"]
    q = st.proj(pre + "qb", rms_norm(st.proj(pre + "qa", x), v[pre + "qn"], 1e-6)).view(B, hr, nr + rd)
    raw = st.proj(pre + "ka", x)
    latent = rms_norm(raw[:, :kr], v[pre + "kn"], 1e-6)
    pe = raw[:, kr:]
    st.kv_out.append(latent)
    st.pe_out.append(pe)
    kb = st.cast(v[pre + "kb"]).view(hr, nr + vd, kr)
    absorbed = torch.einsum("bhd,hdc->bhc", q[..., :nr], kb[:, :nr])
    st.rec(pre + "q", q)
    st.rec(pre + "absorbed", absorbed)
    rows = []
    for b in range(B):
        lat, pos = latent[b:b + 1], pe[b:b + 1]
        if st.keep[b]:
            lat = torch.cat((st.cast(v[pre + "kv_cache"][b]), lat))
            pos = torch.cat((st.cast(v[pre + "pe_cache"][b]), pos))
        scores = (absorbed[b].float() @ lat.float().T + q[b, :, nr:].float() @ pos.float().T) / (nr + rd) ** 0.5
        rows.append(st.cast(scores.softmax(-1)) @ lat)
    mixed = torch.stack(rows)
    st.rec(pre + "attn_latent", mixed)
    out = torch.einsum("bhc,hdc->bhd", mixed, kb[:, nr:]).flatten(1)
    out = out * st.proj(pre + "output_gate", x).sigmoid()
    st.rec(pre + "attn_in", out)
    return st.cast(st.reduce(st.proj(pre + "o", out)))


def _kda_attention(st, layer, x):
    """kimi.py:285-299 (short conv, f_a/f_b gate, beta, gated delta rule, gated per-head norm)."""
    p, v, pre = st.p, st.values, f"l{layer}_"
    B, hr, d = p["batch"], p["q_heads"] // st.case["tp"], p["head_dim"]
    raw = torch.stack([st.proj(pre + n, x) for n in ("q", "k", "v")], 1)
    old = v[pre + "conv_state"] * st.keep[:, None, None, None]
    window = torch.cat((st.cast(old[..., 1:]), raw[..., None]), -1)
    st.conv_out.append(window)
    q, k, val = st.cast(F.silu((window.float() * v[pre + "conv_weight"].float()).sum(-1))).view(B, 3, hr, d).unbind(1)
    gate = st.proj(pre + "fb", st.proj(pre + "fa", x)).view(B, hr, d)
    beta = st.proj(pre + "beta", x)
    state = v[pre + "recurrent_state"] * st.keep[:, None, None, None]
    out, new_state = kda_update(q, k, val, gate, beta, v[pre + "A_log"], v[pre + "dt_bias"].view(hr, d), state)
    st.state_out.append(new_state)
    out = st.cast(out).float()
    out = out * torch.rsqrt(out.square().mean(-1, keepdim=True) + 1e-5) * v[pre + "onorm"].float()
    out = st.cast(out * st.proj(pre + "output_gate", x).view(B, hr, d).float().sigmoid())
    st.rec(pre + "attn_in", out.flatten(1))
    return st.cast(st.reduce(st.proj(pre + "o", out.flatten(1))))


def _moe(st, layer, x):
    """kimi.py:307-328 (router, top-k with bias, MXFP4 routed experts in the latent space, shared experts)."""
    p, v, pre, act = st.p, st.values, f"l{layer}_", st.act
    B = p["batch"]
    scores = (x.float() @ v[pre + "router"].float().T).sigmoid()
    st.rec(pre + "scores", scores)
    biased = scores + v[pre + "router_bias"].float()
    top = biased.topk(p["topk"], -1).indices
    if st.routes is not None:
        top = st.routes[layer].to(device=st.device, dtype=torch.int64)
        kth = biased.topk(p["topk"], -1).values[:, -1]
        st.shortfall.append((kth - biased.gather(1, top).min(-1).values).clamp_min(0))
    w = scores.gather(1, top)
    w = w / (w.sum(-1, keepdim=True) + 1e-20)
    st.chosen.append(top.sort(-1).values)
    latent = st.proj(pre + "latent_down", x)
    st.rec(pre + "latent", latent)
    total = torch.zeros(B, p["latent_hidden"], device=st.device)
    for expert in top.unique().tolist():
        rows, slots = (top == expert).nonzero(as_tuple=True)

        def wt(kind, e=expert):
            return decode_mxfp4_as(v[f"{pre}{kind}_blocks"][e], v[f"{pre}{kind}_scales"][e], act)

        y = st.cast(st.cast(situ(latent[rows] @ wt("gate").T, latent[rows] @ wt("up").T)) @ wt("down").T)
        total.index_add_(0, rows, y.float() * w[rows, slots, None])
    st.rec(pre + "expert_sum_local", total)
    total = st.reduce(total)
    routed = st.proj(pre + "latent_up", rms_norm(st.cast(total), v[pre + "latent_norm"], 1e-5))
    shared = st.reduce(st.proj(pre + "shared_down", st.cast(situ(st.proj(pre + "shared_gate", x),
                                                                 st.proj(pre + "shared_up", x)))))
    st.rec(pre + "routed", routed)
    st.rec(pre + "shared", st.cast(shared))
    return routed + st.cast(shared)


def _layer(st, layer):
    """One decoder layer (kimi.py:256-329): block residual, attention, block residual, FFN."""
    p, v, pre = st.p, st.values, f"l{layer}_"
    hidden = block_mix(st.prefix, st.blocks, v["attention_res_norm"][layer], v["attention_res_proj"][layer],
                       st.cast) if st.blocks else st.prefix
    if layer % p["attn_res_block_size"] == 0:
        st.blocks.append(st.prefix)
        st.prefix = None
    x = rms_norm(hidden, v["ln1"][layer], 1e-5)
    st.rec(pre + "x_attn", x)
    attention = _mla_attention(st, layer, x) if is_mla(st.case, layer) else _kda_attention(st, layer, x)
    st.rec(pre + "attn", attention)
    st.prefix = attention if st.prefix is None else st.prefix + attention
    hidden = block_mix(st.prefix, st.blocks, v["mlp_res_norm"][layer], v["mlp_res_proj"][layer], st.cast)
    x = rms_norm(hidden, v["ln2"][layer], 1e-5)
    st.rec(pre + "x_mlp", x)
    if layer < p["first_dense"]:
        out = st.cast(st.reduce(st.proj(pre + "down", st.cast(situ(st.proj(pre + "gate", x), st.proj(pre + "up", x))))))
        st.chosen.append(torch.full((p["batch"], p["topk"]), -1, device=st.device, dtype=torch.int64))
        st.shortfall.append(torch.zeros(p["batch"], device=st.device))
    else:
        out = _moe(st, layer, x)
    st.rec(pre + "mlp", out)
    st.prefix = st.prefix + out
    st.rec(pre + "prefix", st.prefix)


def _head(st):
    """kimi.py:330-340: output block residual, final norm, LM head, greedy token, outputs."""
    p, v = st.p, st.values
    chunk = p["vocab"] // st.case["tp"]
    hidden = block_mix(st.prefix, st.blocks, v["output_res_norm"], v["output_res_proj"], st.cast)
    x = rms_norm(hidden, v["fnorm"], 1e-5)
    st.rec("x_head", x)
    logits = st.proj("lm_head", x).float()
    length = torch.where(v["reset"], 1, p["context"] + 1).to(torch.int64)
    stack = lambda items: torch.stack(items) if items else torch.zeros(0, device=st.device)
    result = {"logits": logits, "next_token": _argmax_sharded(logits, st.tp_rank * chunk, st.group, st.serial),
              "kv_write": stack(st.kv_out), "pe_write": stack(st.pe_out),
              "recurrent_state": stack(st.state_out), "conv_state": stack(st.conv_out),
              "expert_ids": torch.stack(st.chosen), "cache_length": length}
    if st.routes is not None:
        result["route_shortfall"] = torch.stack(st.shortfall)
    return result


def reference(case, values, *, serial=None, fp32=False, routes=None, tp_rank=None, group=None, trace=None):
    """One decode step for one rank (kimi.py:230-340).

    fp32=False is the BF16 serving oracle; fp32=True recomputes with FP32 activations. `routes`
    [L, B, topk] forces the MoE expert sets and adds `route_shortfall` [L, B]. `tp_rank`/`group`
    name this rank's TP position and process group when not serial (default: WORLD, rank % tp).
    `trace`, if a dict, receives per-layer intermediates (debugging aid for the CUDA path).
    """
    st = _Step(case, values, serial, fp32, routes, tp_rank, group, trace)
    _embed(st)
    for layer in range(st.p["layers"]):
        _layer(st, layer)
    return _head(st)


def timed_sample(case, values, part):
    """CPU-baseline sample: run one part of the BF16 step serially and return its wall time in seconds.
    `part` is 'embed+head' or a layer index; the blocks/prefix context is a plausible stand-in (the cost of a
    layer does not depend on it)."""
    import time
    st = _Step(case, values, True, False, None, 0, None, None)
    _embed(st)
    if part == "embed+head":
        t0 = time.perf_counter()
        _embed(st)
        st.blocks = [st.prefix]
        # no layer ran, so the per-layer route list the outputs stack is empty: one placeholder row set
        st.chosen = [torch.full((st.p["batch"], st.p["topk"]), -1, dtype=torch.int64, device=st.device)]
        _head(st)
        return time.perf_counter() - t0
    layer = int(part)
    st.blocks = [st.prefix]
    t0 = time.perf_counter()
    _layer(st, layer)
    return time.perf_counter() - t0


def _group_sum(t, group, serial):
    if not serial:
        dist.all_reduce(t, group=group)
    return t


def routes_valid(case, routes, expected) -> bool:
    """kimi.py:358-367: ids in range and distinct per row; dense layers carry -1 exactly as expected."""
    p, dense = _params(case), _params(case)["first_dense"]
    if not torch.equal(routes[:dense], expected[:dense]):
        return False
    moe = routes[dense:]
    if bool(((moe < 0) | (moe >= p["experts"])).any()):
        return False
    ordered = moe.sort(-1).values
    return not bool((ordered[..., 1:] == ordered[..., :-1]).any())


def compare(case, values, expected, actual, *, serial=None, tp_rank=None, group=None):
    """The oracle band grader (kimi.py:370-462). Returns details; raises AssertionError on failure."""
    if not isinstance(actual, dict) or set(actual) != set(expected):
        raise AssertionError(f"output keys: expected {sorted(expected)}, got "
                             f"{sorted(actual) if isinstance(actual, dict) else type(actual)}")
    for name, want in expected.items():
        got = actual[name]
        if not isinstance(got, torch.Tensor):
            raise AssertionError(f"{name}: output must be a Tensor")
        if got.shape != want.shape or got.dtype != want.dtype or got.device != want.device:
            raise AssertionError(f"{name}: expected {tuple(want.shape)} {want.dtype} on {want.device}, "
                                 f"got {tuple(got.shape)} {got.dtype} on {got.device}")
    serial = case["gpus"] == 1 if serial is None else serial
    tp_rank, group = _rank_context(case, serial, tp_rank, group)
    routes = actual["expert_ids"].long()
    ordered = routes.sort(-1).values
    checksum = (ordered * torch.arange(1, ordered.numel() + 1, device=ordered.device).view(ordered.shape)).sum()
    flags = torch.tensor([0 if routes_valid(case, routes, expected["expert_ids"]) else 1,
                          int(checksum), -int(checksum),
                          0 if torch.equal(routes.sort(-1).values, expected["expert_ids"]) else 1],
                         device=routes.device, dtype=torch.int64)
    if not serial:
        dist.all_reduce(flags, op=dist.ReduceOp.MAX, group=group)
    if flags[0] or int(flags[1]) != -int(flags[2]):
        raise AssertionError("expert_ids: ids out of range, repeated in a row, wrong in a dense layer, "
                             "or different between ranks")
    kw = dict(serial=serial, fp32=True, tp_rank=tp_rank, group=group)
    truth_o = reference(case, values, routes=expected["expert_ids"], **kw)
    truth_c = truth_o if not flags[3] else reference(case, values, routes=routes, **kw)
    details, failures = {}, []
    for name in ("logits", "kv_write", "pe_write", "recurrent_state", "conv_state"):
        ref_o, ref_c = truth_o[name].float(), truth_c[name].float()
        oracle, got = expected[name].float(), actual[name].float()
        rows = ref_o.shape[0] if name == "logits" else 1
        ref_o, ref_c, oracle, got = (t.reshape(rows, -1) for t in (ref_o, ref_c, oracle, got))
        if not torch.isfinite(got).all():
            failures.append(f"{name}: non-finite values")
        sums = torch.stack([(oracle - ref_o).square().sum(-1), ref_o.square().sum(-1),
                            (got - ref_c).square().sum(-1), ref_c.square().sum(-1)])
        sums = _group_sum(sums.double(), group, serial)
        oracle_err = (sums[0] / sums[1].clamp_min(1e-30)).sqrt()
        cand_err = (sums[2] / sums[3].clamp_min(1e-30)).sqrt()
        limit = BAND * oracle_err + FLOOR
        details[name] = {"candidate_rel_l2_max": float(cand_err.max()),
                         "oracle_rel_l2_max": float(oracle_err.max()),
                         "worst_ratio": float((cand_err / limit).max())}
        if bool((cand_err > limit).any()) or not torch.isfinite(cand_err).all():
            failures.append(f"{name}: {details[name]}")
    ref = truth_c["logits"].float()
    chunk = ref.shape[-1]
    offset = 0 if serial else tp_rank * chunk
    stats = torch.stack([ref.max(-1).values,
                         (expected["logits"].float() - truth_o["logits"].float()).abs().max(-1).values])
    if not serial:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX, group=group)
    token = actual["next_token"].long()
    mine = (token >= offset) & (token < offset + chunk)
    picked = torch.where(mine, ref.gather(1, (token - offset).clamp(0, chunk - 1)[:, None])[:, 0], -torch.inf)
    if not serial:
        dist.all_reduce(picked, op=dist.ReduceOp.MAX, group=group)
    bad = picked < stats[0] - 2 * stats[1]
    details["next_token"] = {"rows_outside_tie_margin": int(bad.sum()),
                             "rows_differing_from_fp32_argmax": int((token != truth_c["next_token"]).sum())}
    if bad.any():
        failures.append(f"next_token: {details['next_token']}")
    oracle_short = float(truth_o["route_shortfall"].max()) if truth_o["route_shortfall"].numel() else 0.0
    cand_short = truth_c["route_shortfall"]
    allowed = BAND * oracle_short + ROUTE_FLOOR
    details["expert_ids"] = {"candidate_max_shortfall": float(cand_short.max()) if cand_short.numel() else 0.0,
                             "oracle_max_shortfall": oracle_short, "allowed": allowed,
                             "sets_differing_from_oracle": int((routes.sort(-1).values != expected["expert_ids"]).any(-1).sum())}
    if cand_short.numel() and bool((cand_short > allowed).any()):
        failures.append(f"expert_ids: {details['expert_ids']}")
    mismatch = int((actual["cache_length"] != expected["cache_length"]).sum())
    details["cache_length"] = {"mismatched_elements": mismatch}
    if mismatch:
        failures.append(f"cache_length: {mismatch} mismatches")
    if failures:
        raise AssertionError("; ".join(failures))
    return details


def snapshot(inputs: dict) -> dict:
    """Input-mutation detector in the spirit of harness/correctness.py:13-45 (host copy or device checksums)."""
    out = {}
    for name, value in inputs.items():
        value = value.detach()
        nbytes = value.numel() * value.element_size()
        if nbytes <= 1 << 26 or not value.is_contiguous() or nbytes % 4:
            out[name] = value.to("cpu", copy=True)
            continue
        words = value.reshape(-1).view(torch.uint8).view(torch.int32)
        total = torch.zeros(2, dtype=torch.int64, device=value.device)
        step = 1 << 26
        weight = (torch.arange(step, device=value.device, dtype=torch.int64) % 65521) + 1
        for start in range(0, words.numel(), step):
            part = words[start:start + step].to(torch.int64)
            total[0] += part.sum()
            total[1] += (part * weight[:part.numel()]).sum()
        out[name] = total.cpu()
    return out


def check_unchanged(inputs: dict, before: dict) -> None:
    after = snapshot(inputs)
    for name in inputs:
        if not torch.equal(after[name], before[name]):
            raise AssertionError(f"candidate mutated input {name}")


def serial_rank_view(case):
    """A TP1 case dict that runs exactly one TP rank's arithmetic serially (reductions become identity)."""
    p, tp = dict(_params(case)), case["tp"]
    for key in ("q_heads", "vocab", "intermediate", "dense_intermediate"):
        p[key] //= tp
    return dict(case, id=case["id"] + "-rank-equivalent", gpus=1, tp=1, params=p)

