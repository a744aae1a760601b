"""ctypes binding of libkk3.so (include/kk3.h) and the per-rank decode-step runner.

This is the host side of the drop-in boundary: it maps the reference's per-rank input dict
(garv901/kimi-k3-goalbox megabench/tasks/kimi.py:72-122 weights, :164-182 state) onto the C ABI's
pointer table, allocates the reference-shaped outputs (:332-340) and enqueues one kernel launch on the
current CUDA stream. There is no fallback: if the library or a GPU is missing, it raises.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

from .cases import is_mla

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libkk3.so"

GLOBAL_SLOTS = 32
LAYER_SLOTS = 32
GLOBAL_NAMES = ["token", "reset", "embed", "lm_head", "fnorm", "output_res_norm", "output_res_proj", "ln1", "ln2",
                "attention_res_norm", "mlp_res_norm", "attention_res_proj", "mlp_res_proj"]
OUTPUT_NAMES = ["logits", "next_token", "kv_write", "pe_write", "recurrent_state", "conv_state", "expert_ids",
                "cache_length"]
OUTPUT_SLOT0 = 13
KDA_NAMES = ["q", "k", "v", "output_gate", "o", "fa", "fb", "beta", "onorm", "A_log", "dt_bias", "conv_weight",
             "conv_state", "recurrent_state"]
MLA_NAMES = ["qa", "qb", "ka", "kb", "o", "output_gate", "qn", "kn", "kv_cache", "pe_cache"]
DENSE_NAMES = ["gate", "up", "down"]
MOE_NAMES = ["latent_down", "latent_up", "latent_norm", "router", "router_bias", "gate_blocks", "gate_scales",
             "up_blocks", "up_scales", "down_blocks", "down_scales", "shared_gate", "shared_up", "shared_down"]
FFN_SLOT0 = 16

ERRORS = {0: "ok", -1: "bad argument or pointer table", -2: "geometry not supported by the sm_100a kernels",
          -3: "CUDA runtime call failed", -4: "in-kernel wait exceeded its bound", -5: "in-kernel check failed",
          -6: "tensor-parallel peers are not open", -7: "context failed earlier; rebuild it",
          -8: "geometry needs more scratch than the allocation-free entry point's static buffer"}


class Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "layers", "batch", "hidden", "latent_hidden", "inter_shard", "dense_inter_shard", "shared_inter_shard",
        "heads", "head_dim", "q_lora_rank", "kv_lora_rank", "qk_nope_dim", "qk_rope_dim", "v_head_dim",
        "vocab_shard", "experts", "topk", "context", "conv_kernel", "attn_res_block_size", "first_dense", "tp",
        "rank", "device")] + [("timeout_ns", ctypes.c_int64)]


COMM_PEER, COMM_HOST, COMM_PUSH = 0, 1, 2   # include/kk3.h KK3_COMM_*
GEMV_AUTO, GEMV_MMA = 0, 1     # include/kk3.h KK3_GEMV_*


def host_comm_segments(params: dict, tp: int) -> list[tuple[int, int, list[tuple[str, str, int]]]]:
    """Phase ranges of one step under the host transport (KK3_COMM_HOST), as the kernel runs them
    (csrc/kk3_kernel.cuh): (start_phase, stop_phase, exchanges to run after the range), stop_phase -1 = to the
    end. An exchange is (sub-region, "sum" | "gather", parity): "sum" all-reduces this rank's slot (FP32 sum,
    kimi.py:343-347), "gather" all-gathers the argmax keys (kimi.py:218-227). Exchanges alternate parity in
    program order, as the kernel's exchange counter does."""
    names = host_comm_program(params)
    points = {"embed": [("att", "sum")], "o_proj": [("att", "sum")], "dense_down": [("att", "sum")],
              "moe_combine_write": [("exp", "sum"), ("shd", "sum")], "argmax_write": [("key", "gather")]}
    segs, start, xi = [], 0, 0
    for i, name in enumerate(names):
        if name in points and tp > 1:
            segs.append((start, i + 1, [(region, kind, xi & 1) for region, kind in points[name]]))
            xi += 1
            start = i + 1
    segs.append((start, -1, []))
    return segs


def host_comm_program(params: dict) -> list[str]:
    """Grid phases of one step under the host transport, in kernel order: the peer program with the MoE
    combine and the argmax each split at their exchange (csrc/kk3_kernel.cuh)."""
    from .cases import is_mla
    L, fd = params["layers"], params["first_dense"]
    names = ["embed"]
    for l in range(L):
        names.append("attn_prologue")
        names += (["mla_proj", "mla_rows", "mla_qb", "mla_absorb", "mla_attend", "mla_combine"] if is_mla(params, l)
                  else ["kda_proj", "kda"])
        names += ["o_proj", "mlp_prologue"]
        names += (["dense_gate_up", "dense_down"] if l < fd else
                  ["moe_in", "experts_gate_up", "experts_down", "moe_combine_write", "moe_combine_read", "latent_up"])
    if L <= fd:
        names.append("fold")
    names += ["head_prologue", "lm_head", "argmax_write", "argmax_read"]
    return names


class _DeviceBytes:
    """A raw device range exposed through __cuda_array_interface__, so torch can alias it without a copy."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}


class KK3Error(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what}: kk3 error {code} ({ERRORS.get(code, 'unknown')})")
        self.code = code


_LIB = None


def load_library() -> ctypes.CDLL:
    """Load the in-tree libkk3.so (built by kimi_k3_goalbox_b200.build). Raises if it is missing."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m kimi_k3_goalbox_b200.build` first")
        lib = ctypes.CDLL(str(LIB_PATH))
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        lib.kk3_table_size.argtypes = [ctypes.POINTER(Config)]
        lib.kk3_init.argtypes = [ctypes.POINTER(Config), ctypes.POINTER(vp)]
        lib.kk3_ipc_handle.argtypes = [vp, vp]
        lib.kk3_open_peers.argtypes = [vp, vp]
        lib.kk3_step.argtypes = [vp, vp, i32, vp]
        lib.kk3_step_append.argtypes = [vp, vp, i32, vp, vp]
        lib.kk3_debug_step.argtypes = [vp, vp, i32, vp, i32]
        lib.kk3_debug_phases.argtypes = [vp, vp, i32, vp, i32, i32]
        lib.kk3_status.argtypes = [vp]
        lib.kk3_phase_count.argtypes = [vp]
        lib.kk3_error_string.argtypes = [i32]
        lib.kk3_error_string.restype = ctypes.c_char_p
        lib.kk3_free.argtypes = [vp]
        lib.kk3_free.restype = None
        lib.kk3_debug_buffer.argtypes = [vp, i32, ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_size_t)]
        lib.kk3_exchange_bytes.argtypes = [vp]
        lib.kk3_exchange_bytes.restype = ctypes.c_size_t
        lib.kk3_debug_set_peer.argtypes = [vp, i32, vp]
        lib.kk3_debug_copy.argtypes = [vp, i32, vp, ctypes.c_size_t]
        lib.kk3_debug_trace.argtypes = [vp, i32, ctypes.POINTER(ctypes.c_int), i32]
        lib.kk3_launch_config.argtypes = [vp, ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(ctypes.c_size_t)]
        lib.kk3_exchange_layout.argtypes = [vp, ctypes.POINTER(ctypes.c_longlong)]
        lib.kk3_set_comm_mode.argtypes = [vp, i32]
        lib.kk3_set_gemv_engine.argtypes = [vp, i32]
        _LIB = lib
    return _LIB


def padded_tiles(batch: int) -> int:
    """The step kernel's batch class: 8-column MMA n-tiles per batch (1, 2, 4 or 8 for B <= 8, 16, 32, 64)."""
    return 1 if batch <= 8 else 2 if batch <= 16 else 4 if batch <= 32 else 8


def rank_config(case: dict, rank: int, device: int, timeout_ns: int = 0) -> Config:
    """kk3_config for one TP rank of a reference case dict (megabench/tasks/kimi.py:72-122 divisions)."""
    p, tp = case["params"], case["tp"]
    if case.get("ep", 1) != 1 or case["gpus"] != tp:
        raise ValueError("Kimi requires one TP group spanning all ranks (megabench/tasks/kimi.py:187)")
    for n in (p["q_heads"], p["vocab"], p["intermediate"], p["dense_intermediate"]):
        if n % tp:
            raise ValueError("Kimi attention heads, vocabulary and FFN intermediate must divide TP")
    return Config(layers=p["layers"], batch=p["batch"], hidden=p["hidden"], latent_hidden=p["latent_hidden"],
                  inter_shard=p["intermediate"] // tp, dense_inter_shard=p["dense_intermediate"] // tp,
                  shared_inter_shard=p["intermediate"] * p["shared_experts"] // tp, heads=p["q_heads"] // tp,
                  head_dim=p["head_dim"], q_lora_rank=p["q_lora_rank"], kv_lora_rank=p["kv_lora_rank"],
                  qk_nope_dim=p["qk_nope_dim"], qk_rope_dim=p["qk_rope_dim"], v_head_dim=p["v_head_dim"],
                  vocab_shard=p["vocab"] // tp, experts=p["experts"], topk=p["topk"], context=p["context"],
                  conv_kernel=p["conv_kernel"], attn_res_block_size=p["attn_res_block_size"],
                  first_dense=p["first_dense"], tp=tp, rank=rank, device=device, timeout_ns=timeout_ns)


def table_layout(params: dict) -> list[tuple[int, str]]:
    """(slot, input name) pairs of the pointer table for one geometry (include/kk3.h enums)."""
    out = [(i, n) for i, n in enumerate(GLOBAL_NAMES)]
    for layer in range(params["layers"]):
        base = GLOBAL_SLOTS + layer * LAYER_SLOTS
        attn = MLA_NAMES if is_mla(params, layer) else KDA_NAMES
        out += [(base + i, f"l{layer}_{n}") for i, n in enumerate(attn)]
        ffn = DENSE_NAMES if layer < params["first_dense"] else MOE_NAMES
        out += [(base + FFN_SLOT0 + i, f"l{layer}_{n}") for i, n in enumerate(ffn)]
    return out


def output_specs(case: dict) -> dict:
    """Reference output shapes and dtypes for one rank (megabench/tasks/kimi.py:332-340)."""
    p, tp = case["params"], case["tp"]
    B, L, K = p["batch"], p["layers"], p["topk"]
    nmla = sum(is_mla(p, l) for l in range(L))
    nkda = L - nmla
    hr, d = p["q_heads"] // tp, p["head_dim"]
    f32, bf, i64 = torch.float32, torch.bfloat16, torch.int64
    return {
        "logits": ((B, p["vocab"] // tp), f32),
        "next_token": ((B,), i64),
        "kv_write": ((nmla, B, p["kv_lora_rank"]), bf) if nmla else ((0,), f32),
        "pe_write": ((nmla, B, p["qk_rope_dim"]), bf) if nmla else ((0,), f32),
        "recurrent_state": ((nkda, B, hr, d, d), f32) if nkda else ((0,), f32),
        "conv_state": ((nkda, B, 3, hr * d, p["conv_kernel"]), bf) if nkda else ((0,), f32),
        "expert_ids": ((L, B, K), i64),
        "cache_length": ((B,), i64),
    }


class StepContext:
    """One kk3 context: a rank's scratch, exchange buffer and launch state (kk3_init .. kk3_free)."""

    def __init__(self, case: dict, rank: int = 0, device: int | None = None, timeout_ns: int = 0):
        if not torch.cuda.is_available():
            raise RuntimeError("the Kimi K3 step needs a CUDA GPU (B200, sm_100a); no CPU fallback exists")
        self.lib = load_library()
        self.case = case
        self.params = case["params"]
        self.device = torch.cuda.current_device() if device is None else device
        self.cfg = rank_config(case, rank, self.device, timeout_ns)
        handle = ctypes.c_void_p()
        rc = self.lib.kk3_init(ctypes.byref(self.cfg), ctypes.byref(handle))
        if rc != 0:
            raise KK3Error(rc, "kk3_init")
        self.handle = handle
        self.layout = table_layout(self.params)
        self.nslots = GLOBAL_SLOTS + self.params["layers"] * LAYER_SLOTS
        self.table = (ctypes.c_void_p * self.nslots)()
        self.outspec = output_specs(case)
        self._cached_inputs: tuple | None = None

    # --- tensor parallel set-up -------------------------------------------------------------------
    def ipc_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(64)
        rc = self.lib.kk3_ipc_handle(self.handle, buf)
        if rc != 0:
            raise KK3Error(rc, "kk3_ipc_handle")
        return buf.raw

    def exchange_bytes(self) -> int:
        """Bytes of this rank's exchange buffer (flags + two parity regions)."""
        return int(self.lib.kk3_exchange_bytes(self.handle))

    def debug_set_peer(self, r: int, buf: torch.Tensor) -> None:
        """Single-process testing aid: use a device tensor of exchange_bytes() bytes as rank r's buffer."""
        if buf.numel() * buf.element_size() < self.exchange_bytes() or not buf.is_cuda:
            raise ValueError("peer buffer must be a device tensor of at least exchange_bytes() bytes")
        self._peer_keepalive = buf
        rc = self.lib.kk3_debug_set_peer(self.handle, r, ctypes.c_void_p(buf.data_ptr()))
        if rc != 0:
            raise KK3Error(rc, "kk3_debug_set_peer")

    def open_peers(self, handles: list[bytes]) -> None:
        blob = b"".join(handles)
        rc = self.lib.kk3_open_peers(self.handle, blob)
        if rc != 0:
            raise KK3Error(rc, "kk3_open_peers")

    # --- the step ----------------------------------------------------------------------------------
    def _bind_inputs(self, values: dict) -> None:
        """Fill the input slots (cached while the same tensor objects are passed)."""
        cached = self._cached_inputs
        if cached is not None and len(cached[0]) == len(self.layout):
            names = cached[1]
            objs = cached[0]
            if all(values[n] is t for n, t in zip(names, objs)):
                return
        dev = torch.device("cuda", self.device)
        objs, names = [], []
        for slot, name in self.layout:
            t = values.get(name)
            if t is None:
                raise ValueError(f"missing input {name}")
            if t.device != dev or not t.is_contiguous():
                raise ValueError(f"input {name} must be a contiguous tensor on {dev}")
            self.table[slot] = t.data_ptr()
            objs.append(t)
            names.append(name)
        self._check_inputs(values)
        self._cached_inputs = (tuple(objs), tuple(names))

    def _check_inputs(self, values: dict) -> None:
        p, B = self.params, self.params["batch"]
        if values["token"].dtype != torch.int64 or tuple(values["token"].shape) != (B,):
            raise ValueError("token must be int64 [B]")
        if values["reset"].dtype != torch.bool or tuple(values["reset"].shape) != (B,):
            raise ValueError("reset must be bool [B]")
        h = p["hidden"]
        if tuple(values["embed"].shape) != (p["vocab"] // self.case["tp"], h) or values["embed"].dtype != torch.bfloat16:
            raise ValueError("embed must be bf16 [vocab/tp, hidden]")

    def allocate_outputs(self) -> dict:
        dev = torch.device("cuda", self.device)
        return {n: torch.empty(shape, dtype=dt, device=dev) for n, (shape, dt) in self.outspec.items()}

    def bind_outputs(self, outputs: dict) -> None:
        for i, n in enumerate(OUTPUT_NAMES):
            self.table[OUTPUT_SLOT0 + i] = outputs[n].data_ptr() if outputs[n].numel() else None

    def status(self) -> int:
        return self.lib.kk3_status(self.handle)

    def check(self) -> None:
        rc = self.status()
        if rc != 0:
            raise KK3Error(rc, "decode-step kernel")

    def launch(self, stream: int | None = None, stop_phase: int = -1, start_phase: int = 0) -> None:
        if stream is None:
            stream = torch.cuda.current_stream(self.device).cuda_stream
        if start_phase > 0:
            rc = self.lib.kk3_debug_phases(self.handle, self.table, self.nslots, ctypes.c_void_p(stream), start_phase,
                                           stop_phase)
        elif stop_phase >= 0:
            rc = self.lib.kk3_debug_step(self.handle, self.table, self.nslots, ctypes.c_void_p(stream), stop_phase)
        else:
            rc = self.lib.kk3_step(self.handle, self.table, self.nslots, ctypes.c_void_p(stream))
        if rc != 0:
            raise KK3Error(rc, "kk3_step")

    def step(self, values: dict, outputs: dict | None = None, stop_phase: int = -1) -> dict:
        """Enqueue one step. Raises if an earlier step of this context reported a failure (the status word is
        read without synchronising, so a failure of the previous step is seen once its kernel has ended). A
        step that fails writes next_token = -1 and cache_length = 0 into its own outputs, so its failure is
        visible in what the caller reads back after synchronising."""
        self.check()
        self._bind_inputs(values)
        out = self.allocate_outputs() if outputs is None else outputs
        self.bind_outputs(out)
        self.launch(stop_phase=stop_phase)
        return out

    def step_append(self, values: dict, outputs: dict, lengths: torch.Tensor) -> dict:
        """One step that continues every sequence in place (include/kk3.h kk3_step_append): row b attends its
        first lengths[b] cached positions plus the new token, its new MLA entries are written into the cache
        inputs at position lengths[b] (0 after a reset), and cache_length = lengths + 1. `lengths` is a device
        int64 [B] tensor (the previous step's cache_length output works as is). The KDA state outputs may be the
        stacked tensor whose per-layer views are the state inputs (an in-place update)."""
        self.check()
        if lengths.dtype != torch.int64 or lengths.device != torch.device("cuda", self.device) or \
                tuple(lengths.shape) != (self.params["batch"],):
            raise ValueError("lengths must be a device int64 tensor [batch] on the context's device")
        self._bind_inputs(values)
        self.bind_outputs(outputs)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = self.lib.kk3_step_append(self.handle, self.table, self.nslots, ctypes.c_void_p(lengths.data_ptr()),
                                      ctypes.c_void_p(stream))
        if rc != 0:
            raise KK3Error(rc, "kk3_step_append")
        return outputs

    def phase_count(self) -> int:
        return self.lib.kk3_phase_count(self.handle)

    def debug_buffer(self, which: int, dtype: torch.dtype, shape: tuple) -> torch.Tensor:
        """Copy an internal scratch buffer (include/kk3.h kk3_debug_buffer_id) into a new tensor."""
        ptr, size = ctypes.c_void_p(), ctypes.c_size_t()
        rc = self.lib.kk3_debug_buffer(self.handle, which, ctypes.byref(ptr), ctypes.byref(size))
        if rc != 0:
            raise KK3Error(rc, "kk3_debug_buffer")
        out = torch.empty(shape, dtype=dtype, device=torch.device("cuda", self.device))
        nbytes = out.numel() * out.element_size()
        if nbytes > size.value:
            raise ValueError("debug buffer smaller than requested view")
        torch.cuda.synchronize(self.device)
        rc = self.lib.kk3_debug_copy(self.handle, which, ctypes.c_void_p(out.data_ptr()), nbytes)
        if rc != 0:
            raise KK3Error(rc, "kk3_debug_copy")
        return out

    def trace(self, enable: bool | None = None) -> list[int]:
        """Trace words: phase reached per CTA [1024], progress code per CTA [1024], marker per warp [4096];
        optionally switch publishing on/off."""
        buf = (ctypes.c_int * (2 * 1024 + 4096))()
        self.lib.kk3_debug_trace(self.handle, -1 if enable is None else int(enable), buf, len(buf))
        return list(buf)

    def launch_config(self) -> tuple[int, int, int]:
        g, t, s = ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
        self.lib.kk3_launch_config(self.handle, ctypes.byref(g), ctypes.byref(t), ctypes.byref(s))
        return g.value, t.value, s.value

    # --- the host-transport comparison baseline (KK3_COMM_HOST) -----------------------------------------
    def set_gemv_engine(self, engine: int) -> None:
        """GEMV_AUTO (tcgen05 projections above batch 16) or GEMV_MMA (mma.sync for every batch), include/kk3.h."""
        rc = self.lib.kk3_set_gemv_engine(self.handle, engine)
        if rc != 0:
            raise KK3Error(rc, "kk3_set_gemv_engine")

    def set_comm_mode(self, mode: int) -> None:
        rc = self.lib.kk3_set_comm_mode(self.handle, mode)
        if rc != 0:
            raise KK3Error(rc, "kk3_set_comm_mode")

    def exchange_slots(self) -> dict:
        """This rank's exchange buffer as torch views: {(parity, region): tensor [tp, n]}, one row per source
        rank, for the regions att (bf16, n = hidden x bp), exp (f32, n = batch x latent_hidden), shd (bf16, as
        att) and key (int64 view of the u64 keys, n = batch). bp is the batch padded to the kernel's n-tile width
        (8, 16, 32 or 64); the bf16 regions are channel-tiled ([hidden / 16][bp][16] per source), which the
        elementwise NCCL reductions of the host transport do not need to know."""
        if getattr(self, "_xviews", None) is None:
            ptr, size = ctypes.c_void_p(), ctypes.c_size_t()
            rc = self.lib.kk3_debug_buffer(self.handle, 15, ctypes.byref(ptr), ctypes.byref(size))   # KK3_BUF_EXCHANGE
            if rc != 0:
                raise KK3Error(rc, "kk3_debug_buffer")
            off = (ctypes.c_longlong * 8)()
            rc = self.lib.kk3_exchange_layout(self.handle, off)
            if rc != 0:
                raise KK3Error(rc, "kk3_exchange_layout")
            raw = torch.as_tensor(_DeviceBytes(ptr.value, size.value), device=torch.device("cuda", self.device))
            tp, B, p = self.case["tp"], self.params["batch"], self.params
            bp = 8 * padded_tiles(B)
            sizes = {"att": (p["hidden"] * bp, torch.bfloat16, 4), "exp": (B * p["latent_hidden"], torch.float32, 5),
                     "shd": (p["hidden"] * bp, torch.bfloat16, 6), "key": (B, torch.int64, 7)}
            views = {}
            for parity in (0, 1):
                for region, (n, dt, k) in sizes.items():
                    start = off[1 + parity] + off[k]
                    nbytes = tp * n * torch.empty(0, dtype=dt).element_size()
                    views[(parity, region)] = raw[start:start + nbytes].view(dt).view(tp, n)
            self._xraw, self._xviews = raw, views
        return self._xviews

    def launch_host_comm(self, group, stream: int | None = None) -> dict:
        """One step with the host transport: the kernel runs in phase ranges and NCCL reduces the partials
        between them, as the reference does (kimi.py:343-347: FP32 all-reduce of each partial, cast back;
        :218-227: the argmax keys are all-gathered and the kernel takes their maximum). Returns the launch
        counts of the step."""
        import torch.distributed as dist
        tp, rank = self.case["tp"], self.cfg.rank
        views = self.exchange_slots()
        segs = host_comm_segments(self.params, tp)
        counts = {"step_kernel_segments": len(segs), "nccl_collectives": 0, "torch_glue_kernels": 0}
        for start, stop, exchanges in segs:
            self.launch(stream, stop_phase=stop, start_phase=start)
            for region, kind, parity in exchanges:
                v = views[(parity, region)]
                if kind == "gather":
                    flat = v.view(-1)
                    mine = flat[rank * v.shape[1]:(rank + 1) * v.shape[1]].clone()
                    dist.all_gather_into_tensor(flat, mine, group=group)
                    counts["torch_glue_kernels"] += 1
                elif v.dtype == torch.float32:
                    dist.all_reduce(v[rank], group=group)
                else:
                    acc = v[rank].float()
                    dist.all_reduce(acc, group=group)
                    v[rank].copy_(acc)
                    counts["torch_glue_kernels"] += 2
                counts["nccl_collectives"] += 1
        return counts

    def close(self) -> None:
        self._cached_inputs = None   # the bound input tensors: let the caller's memory go with the context
        self._xviews = self._xraw = None
        if getattr(self, "handle", None):
            self.lib.kk3_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
