"""kk3_step_noalloc: the allocation-free TP1 decode step (scratch in a static device array), called through the
C ABI with ctypes and compared with the context path (kk3_init + kk3_step) on the same inputs.

The two paths run the same kernel with the same geometry plan on the same inputs, so their outputs should
agree bit for bit; the float comparison still allows a relative L2 distance of 1e-6. Two calls in a row check
that the zero-state the entry point restores before each launch is enough for a second step.
This file is collected last so that the entry point also runs after every other test in the same process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from kimi_k3_goalbox_b200 import cases, runtime, synthetic
from tests import gpu_helpers as gh

KK3_ERR_ARG, KK3_ERR_UNSUPPORTED, KK3_ERR_TOO_LARGE = -1, -2, -8
FLOAT_TOL = 1e-6   # relative L2 distance allowed for float outputs (integer outputs must match exactly)


@pytest.fixture(scope="module")
def lib():
    from kimi_k3_goalbox_b200 import build
    build.build(verbose=False)   # incremental: recompiles only stale translation units
    lib = runtime.load_library()
    vp = ctypes.c_void_p
    lib.kk3_step_noalloc.argtypes = [ctypes.POINTER(runtime.Config), vp, ctypes.c_int, vp, vp]
    return lib


def table_for(case: dict, values: dict, outputs: dict):
    """Pointer table in include/kk3.h slot order (the same layout the context path binds)."""
    p = case["params"]
    n = runtime.GLOBAL_SLOTS + p["layers"] * runtime.LAYER_SLOTS
    table = (ctypes.c_void_p * n)()
    for slot, name in runtime.table_layout(p):
        table[slot] = values[name].data_ptr()
    for i, name in enumerate(runtime.OUTPUT_NAMES):
        t = outputs[name]
        table[runtime.OUTPUT_SLOT0 + i] = t.data_ptr() if t.numel() else None
    return table, n


def noalloc_step(lib, case: dict, values: dict, error_word: torch.Tensor) -> dict:
    dev = values["token"].device
    outputs = {k: torch.empty(s, dtype=dt, device=dev) for k, (s, dt) in runtime.output_specs(case).items()}
    table, n = table_for(case, values, outputs)
    cfg = runtime.rank_config(case, 0, dev.index)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.kk3_step_noalloc(ctypes.byref(cfg), table, n, ctypes.c_void_p(stream),
                              ctypes.c_void_p(error_word.data_ptr()))
    assert rc == 0, lib.kk3_error_string(rc)
    return outputs


def assert_same(got: dict, want: dict) -> None:
    for key, w in want.items():
        g = got[key]
        assert g.shape == w.shape and g.dtype == w.dtype, key
        if w.numel() == 0:
            continue
        if w.dtype.is_floating_point:
            assert gh.rel_l2(g, w) <= FLOAT_TOL, (key, gh.rel_l2(g, w))
        else:
            assert torch.equal(g, w), key


@pytest.mark.gpu
@pytest.mark.parametrize("case", [gh.small_case(3), gh.small_case(12),
                                  gh.rank_equivalent("kimi-k3-syn-l8-tp8-b8-s8192", layers=4)],
                         ids=["small-b3", "small-b12-nt2", "tp8-rank-b8-l4"])
def test_noalloc_matches_context_step_twice(lib, case):
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    with torch.inference_mode():
        values = synthetic.make_inputs(case, 5, dev)
        ctx = runtime.StepContext(case, device=0)
        try:
            want = ctx.step(values)
            torch.cuda.synchronize()
            ctx.check()
        finally:
            ctx.close()
        error_word = torch.zeros(1, dtype=torch.int32, device=dev)
        for _ in range(2):
            got = noalloc_step(lib, case, values, error_word)
            torch.cuda.synchronize()
            assert int(error_word.item()) == 0
            assert_same(got, want)


@pytest.mark.gpu
def test_noalloc_rejects_geometry_beyond_its_static_scratch(lib):
    # the dev geometry at batch 64: its stream-K partial tiles alone take ~39 MB (the limit is 32 MiB); the
    # table is NULL, so a geometry that unexpectedly fitted would still stop at KK3_ERR_ARG, never launch
    case = cases.get_case("kimi-k3-dev-l4-tp1-b8-s8192")
    cfg = runtime.rank_config(case, 0, 0)
    cfg.batch = 64
    n = runtime.GLOBAL_SLOTS + case["params"]["layers"] * runtime.LAYER_SLOTS
    table = (ctypes.c_void_p * n)()
    rc = lib.kk3_step_noalloc(ctypes.byref(cfg), table, n, None, None)
    assert rc == KK3_ERR_TOO_LARGE
    assert b"32 MiB" in lib.kk3_error_string(rc)


def test_noalloc_rejects_tensor_parallel_configs(lib):
    """tp > 1 is refused before any CUDA call (runs without a GPU)."""
    case = cases.get_case("kimi-k3-syn-l8-tp8-b8-s8192")
    cfg = runtime.rank_config(case, 3, 0)
    n = runtime.GLOBAL_SLOTS + case["params"]["layers"] * runtime.LAYER_SLOTS
    table = (ctypes.c_void_p * n)()
    assert lib.kk3_step_noalloc(ctypes.byref(cfg), table, n, None, None) == KK3_ERR_UNSUPPORTED


def test_noalloc_rejects_misaligned_pointers(lib):
    """A tensor pointer off a 16-byte boundary is refused before any CUDA call (runs without a GPU); token
    ids and reset flags are read with scalar loads and may sit anywhere. The table holds placeholder
    addresses that are never dereferenced."""
    case = gh.small_case(3)
    cfg = runtime.rank_config(case, 0, 0)
    n = runtime.GLOBAL_SLOTS + case["params"]["layers"] * runtime.LAYER_SLOTS
    table = (ctypes.c_void_p * n)()
    table[2] = 0x10002   # KK3_EMBED, 2 bytes off
    assert lib.kk3_step_noalloc(ctypes.byref(cfg), table, n, None, None) == KK3_ERR_ARG
    lsl = runtime.GLOBAL_SLOTS + runtime.LAYER_SLOTS * 1 + 19   # layer 1, KK3_MOE_ROUTER
    table[2] = None
    table[lsl] = 0x10008
    assert lib.kk3_step_noalloc(ctypes.byref(cfg), table, n, None, None) == KK3_ERR_ARG
