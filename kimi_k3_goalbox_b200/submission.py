"""MegaBench submission interface for the B200 Kimi K3 decode step.

Mirrors the reference's plugin contract (garv901/kimi-k3-goalbox megabench/harness/runner.py:53-69,
megabench/integrations/make_kimi_workspace.py:37-44): `build(case: dict) -> run`, where
`run(inputs: dict[str, Tensor]) -> dict[str, Tensor]` computes this rank's outputs of
`megabench/tasks/kimi.py:reference` with one cooperative kernel launch on the current CUDA stream.

For multi-GPU cases `case['execution']` carries rank, world_size, tp_rank, device and the live
`tp_group` (megabench/harness/distributed.py:67-69); build() uses tp_group once to all-gather the CUDA IPC
handles of the per-rank exchange buffers, after which the step communicates only through NVLink peer
memory inside the kernel (no NCCL call inside run()).
"""

from __future__ import annotations

import torch

from .runtime import StepContext


class Runner:
    """The callable returned by build(); one per rank."""

    def __init__(self, case: dict):
        if case.get("family", "kimi_k3_step") != "kimi_k3_step":
            raise NotImplementedError(f"{case.get('id')}: only the kimi_k3_step family is implemented")
        execution = case.get("execution")
        if execution is not None:
            device = torch.device(execution["device"])
            rank = int(execution["tp_rank"])
        else:
            device = torch.device("cuda", torch.cuda.current_device())
            rank = 0
        if device.type != "cuda":
            raise RuntimeError("the Kimi K3 step runs on CUDA devices only (no CPU fallback)")
        torch.cuda.set_device(device)
        self.case = {k: v for k, v in case.items() if k != "execution"}
        self.ctx = StepContext(self.case, rank=rank, device=device.index)
        if case["tp"] > 1:
            import torch.distributed as dist
            group = execution["tp_group"]
            handles = [None] * case["tp"]
            dist.all_gather_object(handles, self.ctx.ipc_handle(), group=group)
            self.ctx.open_peers(handles)
            dist.barrier(group=group)

    def __call__(self, inputs: dict) -> dict:
        return self.ctx.step(inputs)

    def close(self) -> None:
        self.ctx.close()


def build(case: dict) -> Runner:
    """Reference plugin entry point (megabench/harness/runner.py:60-66)."""
    return Runner(case)
