"""One rank of the tensor-parallel GPU parity test (launched by tests/test_gpu_tp.py through torchrun).

Each rank imports submission.py by path and builds it with the reference's execution context (rank, tp_rank,
device, tp_group; megabench/harness/distributed.py:67-69, runner.py:53-69), runs the step twice, checks that
the inputs are unchanged, audits one call's GPU launches (exactly one kernel; harness/benchmark.py:49-74), and
grades its outputs with the oracle's band rule against the BF16 and FP32 oracle computed with real all-reduces
over the same process group (megabench/tasks/kimi.py:343-347). The second step must reproduce the first bit
for bit: the in-kernel exchange alternates parity regions and sequence numbers between steps.
"""

from __future__ import annotations

import argparse
import json
import os
import secrets
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from kimi_k3_goalbox_b200 import cases  # noqa: E402
from oracle import kimi_oracle as ko  # noqa: E402
from tests import gpu_helpers as gh  # noqa: E402


def make_case(spec: dict) -> dict:
    if spec["kind"] == "small":
        # per rank: 128 expert rows (the expert engine needs shards of 128), 64 dense rows, one head or more
        tp = spec["tp"]
        return cases.variant(gh.small_case(spec["batch"], intermediate=128 * tp, dense_intermediate=max(256, 64 * tp),
                                           q_heads=max(2, tp)), tp=tp)
    base = cases.get_case(spec["case"])
    return cases.variant(base, tp=spec.get("tp"), **spec.get("params", {}))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--spec", required=True, help="JSON case spec")
    ap.add_argument("--seed", type=int, default=None, help="default: a fresh seed per run (printed)")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    spec = json.loads(args.spec)
    case = make_case(spec)
    case["params"].pop("checkpoint", None)
    assert case["tp"] == world, (case["tp"], world)
    group = dist.group.WORLD
    # a fresh seed per run, drawn on rank 0 and broadcast (megabench/harness/distributed.py:33-36)
    seed = [args.seed if args.seed is not None else secrets.randbits(32)]
    dist.broadcast_object_list(seed, src=0)
    args.seed = int(seed[0])
    try:
        with torch.inference_mode():
            values = ko.make_inputs(case, args.seed, device, rank)
            execution = {"rank": rank, "world_size": world, "tp_rank": rank, "ep_rank": 0, "backend": "nccl",
                         "device": str(device), "tp_group": group, "ep_group": None}
            run = gh.load_submission(ROOT / "submission.py", dict(case, execution=execution))
            if spec.get("comm"):   # another in-kernel exchange transport (include/kk3.h KK3_COMM_*)
                run.ctx.set_comm_mode(spec["comm"])
            originals = ko.snapshot(values)
            first = {k: v.clone() for k, v in run(values).items()}
            second = run(values)
            torch.cuda.synchronize()
            run.ctx.check()
            ko.check_unchanged(values, originals)
            # one call is one GPU launch on every rank (megabench/harness/benchmark.py:49-74, budget 1)
            launches = gh.audit_launches(run, values)
            assert len(launches) == case["max_gpu_launches"] == 1 and "kk3_step_kernel" in launches[0], launches
            expected = ko.reference(case, values, serial=False, tp_rank=rank, group=group)
            try:
                details = ko.compare(case, values, expected, first, serial=False, tp_rank=rank, group=group)
            except AssertionError as exc:
                print(f"rank {rank} FAIL: seed {args.seed}: {exc}", flush=True)
                raise
            for key, t in first.items():
                assert torch.equal(t, second[key]), f"rank {rank}: second step differs in {key}"
            run.close()
        print(f"rank {rank} ok: seed {args.seed}", {k: (v.get("worst_ratio", v) if isinstance(v, dict) else v) for k, v in details.items()},
              flush=True)
    finally:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
