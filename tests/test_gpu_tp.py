"""Tensor-parallel GPU tests: the in-kernel one-shot exchange over NVLink peer memory.

- test_tp_band_multi_gpu: TP2, TP4 and TP8 ranks on as many GPUs (torchrun, NCCL only for set-up), each graded
  with the band rule against the oracle computed with real all-reduces, on fresh seeds; a spec is skipped on
  a box with fewer GPUs than its TP degree.
- test_exchange_wait_times_out: failure detection on one GPU without a fault. A TP2 context's peer buffer is
  a zeroed allocation that no rank ever writes, so the first exchange wait runs out its (short) bound; the
  kernel must report KK3_ERR_TIMEOUT through the status word, write next_token = -1 and cache_length = 0 into
  the step's outputs, leave the device usable, and the context must refuse further steps.
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from kimi_k3_goalbox_b200 import cases, runtime
from oracle import kimi_oracle as ko
from tests import gpu_helpers as gh

ROOT = Path(__file__).resolve().parents[1]
KK3_ERR_TIMEOUT, KK3_ERR_FAILED = -4, -7


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


# Every spec runs as tp ranks on tp GPUs; each rank is graded against the oracle with real all-reduces. The small
# geometry runs with a fixed seed (its 16 experts make the band's routing floor tighter than BF16 noise on some
# seeds, see test_gpu_parity.test_fresh_seeds_full_width); the full-width cases draw a fresh seed per run.
TP_SPECS = [
    ({"kind": "small", "batch": 3, "tp": 2, "seed": 11}, "small-b3-tp2"),
    ({"kind": "case", "case": "kimi-k3-dev-l8-tp2-b8-s8192"}, "dev-l8-tp2-b8"),
    ({"kind": "small", "batch": 5, "tp": 4, "seed": 11}, "small-b5-tp4"),
    ({"kind": "case", "case": "kimi-k3-dev-l4-tp1-b8-s8192", "tp": 4}, "dev-l4-tp4-b8"),
    ({"kind": "small", "batch": 3, "tp": 8, "seed": 11}, "small-b3-tp8"),
    ({"kind": "case", "case": "kimi-k3-syn-l8-tp8-b1-s8192"}, "syn-l8-tp8-b1"),
    ({"kind": "case", "case": "kimi-k3-syn-l8-tp8-b8-s8192"}, "syn-l8-tp8-b8"),
    ({"kind": "case", "case": "kimi-k3-syn-l8-tp8-b64-s8192"}, "syn-l8-tp8-b64"),
    # the push transport (KK3_COMM_PUSH = 2): the projections' partials pushed in per-CTA chunks
    ({"kind": "small", "batch": 3, "tp": 2, "seed": 11, "comm": 2}, "small-b3-tp2-push"),
    ({"kind": "case", "case": "kimi-k3-dev-l8-tp2-b8-s8192", "comm": 2}, "dev-l8-tp2-b8-push"),
    ({"kind": "case", "case": "kimi-k3-syn-l8-tp8-b8-s8192", "comm": 2}, "syn-l8-tp8-b8-push"),
]


def worker_report(out: str) -> str:
    """The workers' own output (FAIL lines with their seed, tracebacks) without torchrun's per-rank failure
    summaries, which would otherwise fill the assertion message."""
    noise = ("torch/distributed/elastic", "error_file", "traceback :", "elastic/errors.html", "Sending process",
             "ChildFailedError", "exitcode", "<N/A>", "[1]:", "[2]:", "[3]:", "[4]:", "[5]:", "[6]:", "[7]:", "====")
    return "\n".join(line for line in out.splitlines() if not any(n in line for n in noise))[-8000:]


def spec_tp(spec: dict) -> int:
    if "tp" in spec:
        return spec["tp"]
    return cases.get_case(spec["case"])["tp"]


@pytest.mark.gpu
@pytest.mark.parametrize("spec", [s for s, _ in TP_SPECS], ids=[i for _, i in TP_SPECS])
def test_tp_band_multi_gpu(spec):
    tp = spec_tp(spec)
    if gpus() < tp:
        pytest.skip(f"needs {tp} GPUs")
    # the ranks run in child processes on GPUs 0..tp-1: give back what earlier tests of this process cached on
    # GPU 0 (the full-width cases leave ~120 GB in torch's allocator cache)
    import gc
    gc.collect()
    torch.cuda.empty_cache()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1")
    cmd = ["timeout", "-k", "30", "900", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={tp}", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           str(ROOT / "tests" / "tp_worker.py"), "--spec", json.dumps(spec)] + \
          (["--seed", str(spec["seed"])] if "seed" in spec else [])
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=1000)
    out = r.stdout + r.stderr
    assert r.returncode == 0, worker_report(out)
    assert out.count("ok:") == tp, worker_report(out)
    print("\n".join(line for line in out.splitlines() if "ok:" in line))


@pytest.mark.gpu
def test_exchange_wait_times_out():
    torch.cuda.set_device(0)
    case = cases.variant(gh.small_case(2, intermediate=256), tp=2)
    with torch.inference_mode():
        values = ko.make_inputs(case, 3, "cuda:0", 0)
        ctx = runtime.StepContext(case, rank=0, device=0, timeout_ns=50_000_000)
        try:
            peer = torch.zeros(ctx.exchange_bytes(), dtype=torch.uint8, device="cuda:0")
            ctx.debug_set_peer(1, peer)
            out = ctx.step(values)
            torch.cuda.synchronize()          # the kernel must end by itself
            assert ctx.status() == KK3_ERR_TIMEOUT
            # the failed step marks its own integer outputs as invalid
            assert bool((out["next_token"] == -1).all()) and bool((out["cache_length"] == 0).all())
            with pytest.raises(runtime.KK3Error) as err:
                ctx.step(values)
            assert err.value.code in (KK3_ERR_TIMEOUT, KK3_ERR_FAILED)
        finally:
            ctx.close()
        # the device is still usable
        x = torch.ones(1024, device="cuda:0")
        assert float(x.sum()) == 1024.0
