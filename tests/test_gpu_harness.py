"""The submission driven through the reference harness's single-GPU protocol.

The harness (garv901/kimi-k3-goalbox megabench/harness/runner.py:53-69, :72-160) imports the candidate file by
path and calls build(case.to_dict()). For each trial it generates inputs with the seeded generator, snapshots
them, runs the BF16 oracle, calls run(inputs), synchronises, checks that the inputs are unchanged and grades
the outputs with the band rule (correctness.py, kimi.py:370-462). It then times run() with CUDA events
(benchmark.py:10-46) and audits one call's GPU launches with torch.profiler (benchmark.py:49-74): a Kimi case
passes the audit with 1 <= launches <= max_gpu_launches = 1 (megabench/cases.py:58-64). The reference package
does not exist on the GPU machine, so these steps are restated here; tests/tp_worker.py runs the same protocol
per rank for TP > 1.
"""

from __future__ import annotations

import statistics
from pathlib import Path

import pytest
import torch

from kimi_k3_goalbox_b200 import cases
from oracle import kimi_oracle as ko

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from tests import gpu_helpers as gh

SUBMISSION = Path(__file__).resolve().parents[1] / "submission.py"


def _measure(fn, inputs: dict, warmup: int, reps: int) -> list[float]:
    """CUDA-event milliseconds of reps calls after warmup calls (benchmark.py:10-33)."""
    for _ in range(warmup):
        fn(inputs)
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn(inputs)
        end.record()
        end.synchronize()
        times.append(start.elapsed_time(end))
    return times


@pytest.mark.parametrize("which,seeds", [("small-b3", (7, 21)), ("kimi-k3-dev-l4-tp1-b8-s8192", (1234,))])
def test_harness_protocol(which, seeds):
    case = gh.small_case(3) if which == "small-b3" else cases.get_case(which)
    case["params"].pop("checkpoint", None)
    with torch.inference_mode():
        run = gh.load_submission(SUBMISSION, case)
        try:
            for seed in seeds:
                inputs = ko.make_inputs(case, seed, "cuda")
                originals = ko.snapshot(inputs)
                expected = ko.reference(case, inputs, serial=True)
                actual = run(inputs)
                torch.cuda.synchronize()
                ko.check_unchanged(inputs, originals)
                details = ko.compare(case, inputs, expected, actual, serial=True)
                print(f"[{case['id']} seed {seed}] " + ", ".join(
                    f"{k}={v['worst_ratio']:.3f}" for k, v in details.items() if "worst_ratio" in v))
                del inputs, originals, expected, actual
            perf_inputs = ko.make_inputs(case, 99, "cuda")
            times = _measure(run, perf_inputs, warmup=2, reps=5)
            assert all(t > 0 for t in times)
            # CUPTI records kernel activity into device buffers it allocates when a profiler session starts. With
            # torch's allocator cache holding nearly all of the GPU after the full-width oracle and the earlier
            # tests, the sessions recorded no GPU activity at all (the launch API call itself was recorded), so the
            # cache is released first
            import gc
            gc.collect()
            torch.cuda.empty_cache()
            names = gh.audit_launches(run, perf_inputs)
            print(f"[{case['id']}] cuda-event p50 {statistics.median(times) * 1e3:.1f} us, launches {names}")
            assert 1 <= len(names) <= case["max_gpu_launches"], names
            assert "kk3_step_kernel" in names[0], names
            run.ctx.check()
        finally:
            run.close()
