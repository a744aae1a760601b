"""The submission driven through the reference harness's single-GPU protocol.

The harness (garv901/kimi-k3-goalbox megabench/harness/runner.py:53-69, :72-160) runs every case in a worker
process of its own. The worker imports the candidate file by path and calls build(case.to_dict()). For each trial
it generates inputs with the seeded generator, snapshots them, runs the BF16 oracle, calls run(inputs),
synchronises, checks that the inputs are unchanged and grades the outputs with the band rule (correctness.py,
kimi.py:370-462). It then times run() with CUDA events (benchmark.py:10-46) and audits one call's GPU launches
with torch.profiler (benchmark.py:49-74): a Kimi case passes the audit with 1 <= launches <= max_gpu_launches = 1
(megabench/cases.py:58-64). The reference package does not exist on the GPU machine, so tests/harness_worker.py
restates those steps, and this file runs it once per case in a child process; tests/tp_worker.py runs the same
protocol per rank for TP > 1.
"""

from __future__ import annotations

import gc
import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("which,seeds", [("small-b3", "7,21"), ("kimi-k3-dev-l4-tp1-b8-s8192", "1234")])
def test_harness_protocol(which, seeds):
    # the worker needs the GPU memory this process cached in earlier tests (as a fresh harness worker has it)
    gc.collect()
    torch.cuda.empty_cache()
    r = subprocess.run([sys.executable, str(ROOT / "tests" / "harness_worker.py"), "--case", which, "--seeds", seeds],
                       cwd=ROOT, capture_output=True, text=True, timeout=900)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-6000:]
    res = json.loads([line for line in r.stdout.splitlines() if line.startswith("{")][-1])
    print(f"[{res['case']}] trials {res['trials']}, cuda-event p50 {res['cuda_event_p50_ms'] * 1e3:.1f} us, "
          f"launches {res['launches']}")
    assert len(res["trials"]) == len(seeds.split(","))
    assert 1 <= len(res["launches"]) <= res["max_gpu_launches"], res["launches"]
    assert "kk3_step_kernel" in res["launches"][0], res["launches"]
