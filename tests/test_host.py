"""CPU tests of the host side: the C-ABI library loads and exports every entry point include/kk3.h declares,
geometry validation, the pointer-table layout, output shapes, the HBM floor model, and the phase program."""

from __future__ import annotations

import ctypes
import json
import re
from pathlib import Path

import pytest
import torch

from kimi_k3_goalbox_b200 import cases, runtime, sol
from oracle import kimi_oracle as ko
from tests import gpu_helpers as gh

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"


@pytest.fixture(scope="module")
def lib():
    from kimi_k3_goalbox_b200 import build
    build.build(verbose=False)   # incremental: recompiles only stale translation units
    return runtime.load_library()


def declared_functions() -> list[str]:
    text = (ROOT / "include" / "kk3.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kk3_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 12
    for name in names:
        assert hasattr(lib, name), name


def test_error_strings_and_table_size(lib):
    assert lib.kk3_error_string(0) == b"ok"
    assert b"timeout" in lib.kk3_error_string(-4) or b"bound" in lib.kk3_error_string(-4)
    cfg = runtime.rank_config(cases.get_case("kimi-k3-syn-l8-tp8-b8-s8192"), 3, 0)
    assert lib.kk3_table_size(ctypes.byref(cfg)) == 32 + 8 * 32


@pytest.mark.parametrize("cid", ["kimi-k3-dev-l4-tp1-b8-s8192", "kimi-k3-syn-l8-tp8-b8-s8192"])
def test_check_table_requires_exactly_the_runtime_layout(lib, cid):
    """kk3_check_table (host only, no CUDA call) accepts a table whose used slots are the runtime's layout
    plus the outputs it binds, refuses it with KK3_ERR_ARG as soon as any one of them is NULL, and ignores
    NULL in every other slot. Placeholder addresses are never dereferenced."""
    case = cases.get_case(cid)
    p = case["params"]
    cfg = runtime.rank_config(case, 0, 0)
    n = runtime.GLOBAL_SLOTS + p["layers"] * runtime.LAYER_SLOTS
    vp = ctypes.c_void_p
    lib.kk3_check_table.argtypes = [ctypes.POINTER(runtime.Config), vp, ctypes.c_int]
    used = [slot for slot, _ in runtime.table_layout(p)]
    for i, (name, (shape, _)) in enumerate(runtime.output_specs(case).items()):
        if torch.Size(shape).numel():
            used.append(runtime.OUTPUT_SLOT0 + i)
    table = (vp * n)()
    for s in used:
        table[s] = 0x10000 + 16 * s
    assert lib.kk3_check_table(ctypes.byref(cfg), table, n) == 0
    for s in used:
        table[s] = None
        assert lib.kk3_check_table(ctypes.byref(cfg), table, n) == -1, s
        table[s] = 0x10000 + 16 * s
    table[used[-1]] = 0x10008   # misaligned
    assert lib.kk3_check_table(ctypes.byref(cfg), table, n) == -1
    assert lib.kk3_check_table(ctypes.byref(cfg), table, n - 1) == -1


def test_init_rejects_unsupported_geometry_without_a_gpu(lib):
    case = cases.variant(cases.get_case("kimi-k3-dev-l4-tp1-b8-s8192"), head_dim=64)
    cfg = runtime.rank_config(case, 0, 0)
    h = ctypes.c_void_p()
    assert lib.kk3_init(ctypes.byref(cfg), ctypes.byref(h)) == -2
    big = runtime.rank_config(cases.variant(cases.get_case("kimi-k3-dev-l4-tp1-b8-s8192"), batch=65), 0, 0)
    assert lib.kk3_init(ctypes.byref(big), ctypes.byref(h)) == -2


def test_rank_config_divides_by_tp():
    cfg = runtime.rank_config(cases.get_case("kimi-k3-syn-l8-tp8-b64-s8192"), 5, 2)
    assert (cfg.heads, cfg.vocab_shard, cfg.inter_shard, cfg.dense_inter_shard, cfg.shared_inter_shard) == \
        (12, 20480, 384, 4224, 768)
    assert (cfg.rank, cfg.tp, cfg.batch, cfg.device) == (5, 8, 64, 2)
    with pytest.raises(ValueError):
        runtime.rank_config(cases.variant(cases.get_case("kimi-k3-dev-l4-tp1-b8-s8192"), tp=7), 0, 0)


@pytest.mark.parametrize("case", [gh.small_case(3), cases.get_case("kimi-k3-dev-l4-tp1-b8-s8192"),
                                  cases.get_case("kimi-k3-syn-l8-tp8-b8-s8192"),
                                  cases.get_case("kimi-k3-dev-l8-tp2-b8-s8192")])
def test_table_layout_covers_every_input(case):
    specs = ko.tensor_specs(case)
    layout = runtime.table_layout(case["params"])
    names = [n for _, n in layout]
    slots = [s for s, _ in layout]
    assert len(set(slots)) == len(slots)
    state = {"token", "reset"} | {f"l{l}_{n}" for l in range(case["params"]["layers"])
                                  for n in (("kv_cache", "pe_cache") if ko.is_mla(case, l) else ("conv_state", "recurrent_state"))}
    assert set(names) == set(specs) | state
    assert max(slots) < runtime.GLOBAL_SLOTS + case["params"]["layers"] * runtime.LAYER_SLOTS
    out_slots = set(range(runtime.OUTPUT_SLOT0, runtime.OUTPUT_SLOT0 + len(runtime.OUTPUT_NAMES)))
    assert not out_slots & set(slots)


@pytest.mark.parametrize("name", ["tiny_b3_s21", "small_b3_s7"])
def test_output_specs_match_reference_outputs(name):
    fx = torch.load(GOLDEN / f"{name}.pt", weights_only=False)
    spec = runtime.output_specs(fx["case"])
    assert set(spec) == set(fx["bf16"])
    for key, (shape, dtype) in spec.items():
        assert tuple(fx["bf16"][key].shape) == tuple(shape) and fx["bf16"][key].dtype == dtype, key


def test_floor_model_matches_reference():
    want = json.loads((GOLDEN / "sol_reference.json").read_text())
    assert set(want) == set(cases.CASES)
    for case_id, ref in want.items():
        got = sol.floor_bytes(cases.get_case(case_id))
        assert got["minimum_bytes"] == ref["minimum_bytes"], case_id
        assert got["components"] == ref["components"], case_id


def test_phase_program_shape():
    p = gh.small_case(3)["params"]
    prog = gh.phase_program(p)
    assert prog[0] == ("embed", -1) and prog[-1] == ("argmax", -1)
    # 5 layers: layer 0 KDA+dense, 1-2 KDA+MoE, 3-4 MLA+MoE
    per_layer = {0: 1 + 2 + 2 + 2, 1: 1 + 2 + 2 + 5, 2: 1 + 2 + 2 + 5, 3: 1 + 6 + 2 + 5, 4: 1 + 6 + 2 + 5}
    assert len(prog) == 1 + sum(per_layer.values()) + 3


def test_submission_requires_cuda_and_fails_loudly():
    from kimi_k3_goalbox_b200.submission import build
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    with pytest.raises(RuntimeError):
        build(cases.get_case("kimi-k3-dev-l4-tp1-b8-s8192"))
