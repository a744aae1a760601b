"""The tensor-core (tcgen05 block-scaled) expert engine against the decode step's mma.sync engine.

`kimi_k3_goalbox_b200/_lib/kk3_tc_check` (built from csrc/kk3_tc_check.cu) runs both engines on one TP8 rank's
expert geometry (or, with arguments, TP1's) with random MXFP4 weights and bf16-valued latent rows, gate/up
then down, and prints one JSON line. The two engines sum the same exact products in a different FP32 order, so a few results may
differ by one bf16 (slot outputs) or FP16 (activations) ulp; everything else must be bit-identical.
"""

from __future__ import annotations

import json
import subprocess

import pytest

from kimi_k3_goalbox_b200 import build

IDENTICAL_MIN = 0.995      # fraction of bit-identical results
REL_DIFF_MAX = 2.0 ** -7   # largest difference relative to the largest value: one bf16 ulp


def test_checker_builds():
    """The checker cross-compiles for sm_100a with the library (no GPU needed)."""
    build.build(verbose=False)
    assert build.CHECK.exists()


@pytest.mark.parametrize("args", [["1", "100"], ["1", "0"], ["1", "384", "0"], ["1", "3072", "897"]])
def test_checker_rejects_bad_geometry(args):
    """expert_intermediate must be a positive multiple of 128 and distinct_experts in [1, 896]; the checker
    says so and exits 1 before touching the GPU."""
    build.build(verbose=False)
    res = subprocess.run([str(build.CHECK), *args], capture_output=True, text=True, timeout=60)
    assert res.returncode == 1
    assert "error" in json.loads(res.stdout.strip().splitlines()[-1])


@pytest.mark.gpu
def test_tensor_core_engine_matches_mma_sync_engine_tp1_all_experts():
    """The TP1 expert geometry (intermediate 3072) with all 896 experts distinct (no folding)."""
    build.build(verbose=False)
    res = subprocess.run([str(build.CHECK), "2", "3072", "896"], capture_output=True, text=True, timeout=300)
    out = json.loads(res.stdout.strip().splitlines()[-1])
    assert res.returncode == 0, out
    assert out["error_word"] == 0 and out["pairs"] == 128
    assert out["act_identical"] >= IDENTICAL_MIN and out["out_identical"] >= IDENTICAL_MIN, out
    assert out["act_max_rel_diff"] <= REL_DIFF_MAX and out["out_max_rel_diff"] <= REL_DIFF_MAX, out


@pytest.mark.gpu
def test_tensor_core_engine_matches_mma_sync_engine():
    build.build(verbose=False)
    res = subprocess.run([str(build.CHECK), "2"], capture_output=True, text=True, timeout=300)
    line = res.stdout.strip().splitlines()[-1]
    out = json.loads(line)
    assert res.returncode == 0, line
    assert out["error_word"] == 0
    assert out["pairs"] == 128 and out["chunks"] > 100
    assert out["act_identical"] >= IDENTICAL_MIN, out
    assert out["out_identical"] >= IDENTICAL_MIN, out
    assert out["act_max_rel_diff"] <= REL_DIFF_MAX, out
    assert out["out_max_rel_diff"] <= REL_DIFF_MAX, out
