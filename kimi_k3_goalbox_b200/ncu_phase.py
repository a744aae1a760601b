"""Run selected phases of the decode-step kernel (or whole steps) in isolation inside a profiler capture window.

    ncu --profile-from-start off --clock-control none -k regex:kk3_step_kernel ... \
        python -m kimi_k3_goalbox_b200.ncu_phase --case ID [--rank-equivalent] [--layers L] --phase NAME[:LAYER] ...

Fills the scratch buffers with two full steps, then, between cudaProfilerStart/Stop, launches each requested
phase alone (kk3_debug_phases) once, after evicting L2 with a 1 GiB write. The same pattern as the reference's
capture of one warm step (megabench/integrations/ncu_profile_case.py:47-52), narrowed to one phase.
"""

from __future__ import annotations

import argparse
import sys

import torch

from . import cases, synthetic
from .phase_profile import phase_program
from .runtime import StepContext


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--case", default="kimi-k3-syn-l8-tp8-b8-s8192")
    ap.add_argument("--rank-equivalent", action="store_true")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--phase", action="append", required=True,
                    help="NAME or NAME:LAYER (first match if no layer), or 'step' for one whole step")
    args = ap.parse_args(argv)
    case = cases.get_case(args.case)
    case["params"].pop("checkpoint", None)
    if args.rank_equivalent and case["tp"] > 1:
        for key in ("q_heads", "vocab", "intermediate", "dense_intermediate"):
            case["params"][key] //= case["tp"]
        case.update(gpus=1, tp=1)
    if args.layers:
        case["params"]["layers"] = args.layers
    if args.batch:
        case["params"]["batch"] = args.batch
    prog = phase_program(case["params"])
    picks = []
    for spec in args.phase:
        if spec == "step":
            picks.append(-1)
            continue
        name, _, layer = spec.partition(":")
        idx = [i for i, (n, l) in enumerate(prog) if n == name and (not layer or l == int(layer))]
        if not idx:
            raise SystemExit(f"no phase {spec} in this geometry")
        picks.append(idx[0])
    dev = torch.device("cuda", 0)
    with torch.inference_mode():
        values = synthetic.make_inputs(case, 1, dev)
        ctx = StepContext(case)
        out = ctx.allocate_outputs()
        ctx._bind_inputs(values)
        ctx.bind_outputs(out)
        stream = torch.cuda.current_stream().cuda_stream
        for _ in range(2):
            ctx.launch(stream)
        torch.cuda.synchronize()
        ctx.check()
        flush = torch.empty(64 << 22, dtype=torch.float32, device=dev)
        torch.cuda.cudart().cudaProfilerStart()
        for i in picks:
            flush.zero_()
            if i < 0:
                ctx.launch(stream)
            else:
                ctx.launch(stream, stop_phase=i + 1 if i + 1 < len(prog) else -1, start_phase=i)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        ctx.check()
        ctx.close()
    print("captured:", [f"{prog[i][0]}:{prog[i][1]} (#{i})" if i >= 0 else "whole step" for i in picks])
    return 0


if __name__ == "__main__":
    sys.exit(main())
