"""One case of the reference harness's single-GPU protocol, in a process of its own (run by
tests/test_gpu_harness.py), as the harness runs every case in its own worker (megabench/harness/runner.py:163-176,
:177-237). Prints one JSON line with the trial details, the timing and the audited launches."""

from __future__ import annotations

import argparse
import json
import statistics
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from kimi_k3_goalbox_b200 import cases  # noqa: E402
from oracle import kimi_oracle as ko  # noqa: E402
from tests import gpu_helpers as gh  # noqa: E402


def measure(fn, inputs: dict, warmup: int, reps: int) -> list[float]:
    """CUDA-event milliseconds of reps calls after warmup calls (megabench/harness/benchmark.py:10-33)."""
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


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True, help="a case id, or small-b3 for the small test geometry")
    ap.add_argument("--seeds", default="1234")
    args = ap.parse_args()
    case = gh.small_case(3) if args.case == "small-b3" else cases.get_case(args.case)
    case["params"].pop("checkpoint", None)
    trials = []
    with torch.inference_mode():
        run = gh.load_submission(ROOT / "submission.py", case)
        try:
            for seed in (int(x) for x in args.seeds.split(",")):
                inputs = ko.make_inputs(case, seed, "cuda")
                originals = ko.snapshot(inputs)
                expected = ko.reference(case, inputs, serial=True)
                actual = run(inputs)
                torch.cuda.synchronize()
                ko.check_unchanged(inputs, originals)
                details = ko.compare(case, inputs, expected, actual, serial=True)
                trials.append({"seed": seed, "worst_ratio": {k: round(v["worst_ratio"], 3) for k, v in details.items()
                                                             if "worst_ratio" in v}})
                del inputs, originals, expected, actual
            perf_inputs = ko.make_inputs(case, 99, "cuda")
            times = measure(run, perf_inputs, warmup=2, reps=5)
            names = gh.audit_launches(run, perf_inputs)
            run.ctx.check()
        finally:
            run.close()
    print(json.dumps({"case": case["id"], "trials": trials, "cuda_event_p50_ms": statistics.median(times),
                      "launches": names, "max_gpu_launches": case["max_gpu_launches"]}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
