"""Tensor-parallel GPU tests: the in-kernel one-shot exchange over NVLink peer memory.

- test_tp2_band_two_gpus: two ranks on two GPUs (torchrun, NCCL only for set-up), each graded with the band
  rule against the oracle computed with real all-reduces; skipped on a box with fewer than two GPUs.
- test_exchange_wait_times_out: failure detection on one GPU without a fault. A TP2 context's peer buffer is
  a zeroed allocation that no rank ever writes, so the first exchange wait runs out its (short) bound; the
  kernel must report KK3_ERR_TIMEOUT through the status word, leave the device usable, and the context must
  refuse further steps.
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


def two_gpus() -> bool:
    return torch.cuda.is_available() and torch.cuda.device_count() >= 2


@pytest.mark.gpu
@pytest.mark.skipif(not two_gpus(), reason="needs two GPUs")
@pytest.mark.parametrize("spec", [{"kind": "small", "batch": 3, "tp": 2},
                                  {"kind": "case", "case": "kimi-k3-dev-l8-tp2-b8-s8192", "params": {"layers": 4}}],
                         ids=["small-b3-tp2", "dev-l4-tp2-b8"])
def test_tp2_band_two_gpus(spec):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           str(ROOT / "tests" / "tp_worker.py"), "--spec", json.dumps(spec)]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=700)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert out.count("ok:") == 2, out[-4000:]


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
            ctx.step(values)
            torch.cuda.synchronize()          # the kernel must end by itself
            assert ctx.status() == KK3_ERR_TIMEOUT
            with pytest.raises(runtime.KK3Error) as err:
                ctx.step(values)
            assert err.value.code in (KK3_ERR_TIMEOUT, KK3_ERR_FAILED)
        finally:
            ctx.close()
        # the device is still usable
        x = torch.ones(1024, device="cuda:0")
        assert float(x.sum()) == 1024.0
