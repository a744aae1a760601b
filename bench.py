"""Benchmark: Kimi K3 decode-step latency per rank on B200 (one cooperative kernel launch per rank per step).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--case ID] [--batch B]

Default workload: kimi-k3-dev-l4-tp1-b8-s8192 at N=1 (the only single-GPU case of the reference's table);
at N>1 the same model (4 layers, full width, batch 8, context 8192) at TP=N, one rank per GPU over NCCL
(torchrun), i.e. strong scaling of a fixed model. `--case` selects any case of the table instead
(e.g. kimi-k3-syn-l8-tp8-b8-s8192 with --gpus 8). Synthetic seeded weights and state on the device
(the reference's generator); inputs (>= 14 GB per GPU at the default) are larger than the 126 MB L2,
so no flush runs between steps.

`value` is the device time of one step (CUDA events on the launching stream, max over ranks): pure kernel
time with inputs resident. `e2e` is the same metric through the public API (`submission.build(case)` ->
`run(inputs)`), with the step's per-sequence inputs (token, reset) copied host->device from pinned memory
and the result (next_token) copied back inside the timed region.
`--impl reference` times the reference algorithm (the oracle restatement, BF16, torch on the host cores)
on a bounded per-layer sample of the same workload, on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from kimi_k3_goalbox_b200 import cases, sol  # noqa: E402

DEFAULT_CASE = "kimi-k3-dev-l4-tp1-b8-s8192"
FALLBACK_HBM_GBS = 6650.0


def pick_case(args, n: int) -> dict:
    if args.case:
        case = cases.get_case(args.case)
    else:
        case = cases.get_case(DEFAULT_CASE)
        if n != 1:
            case = cases.variant(case, tp=n)
    if getattr(args, "rank_equivalent", False) and case["tp"] > 1 and n == 1:
        # one TP rank's shard shapes as a TP1 geometry: the same arithmetic and bytes as one rank of the case,
        # with identity reductions
        tp = case["tp"]
        params = dict(case["params"])
        for key in ("q_heads", "vocab", "intermediate", "dense_intermediate"):
            params[key] //= tp
        case = dict(case, id=case["id"] + "-rank-equivalent", gpus=1, tp=1, params=params)
    elif args.case and case["tp"] != n:
        case = cases.variant(case, tp=n)
    if args.batch:
        case = cases.variant(case, batch=args.batch)
    case["params"].pop("checkpoint", None)
    return case


def peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def traffic_for(case_id: str):
    path = ROOT / "profiles" / "step_kernel_traffic.json"
    if path.exists():
        try:
            return json.loads(path.read_text()).get(case_id)
        except Exception:
            return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 50 ms with timestamps. The sampler starts before
    the warm-up (nvidia-smi needs a moment to start); only samples inside [mark_start, mark_end], the timed
    region, enter the summary."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.t0 = self.t1 = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)   # let the sample that covers the end of the timed region arrive
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        from datetime import datetime
        sm, mx, reasons, power = [], None, set(), []
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                clk, mxv = float(parts[2]), float(parts[3])
            except ValueError:
                continue
            # a sample reports the state just before its timestamp: keep those inside the timed window
            if self.t0 is None or self.t1 is None or not (self.t0 <= ts <= self.t1 + 0.05):
                continue
            sm.append(clk)
            mx = mxv
            try:
                power.append(float(parts[4]))
            except ValueError:
                pass
            for name, val in zip(names, parts[6:10]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


def init_dist(n: int):
    if n == 1:
        return 0, 0
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return rank, local


def max_over_ranks(x: float, n: int) -> float:
    if n == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(n: int):
    if n > 1:
        dist.barrier()
    torch.cuda.synchronize()


def run_b200(args, n: int, rank: int, local: int) -> dict | None:
    from kimi_k3_goalbox_b200 import synthetic
    from kimi_k3_goalbox_b200.runtime import StepContext
    from kimi_k3_goalbox_b200.submission import build

    case = pick_case(args, n)
    p = case["params"]
    device = torch.device("cuda", local)
    seed = args.seed
    with torch.inference_mode():
        values = synthetic.make_inputs(case, seed, device, rank=rank)
        torch.cuda.synchronize()
        # --- kernel-only timing (inputs resident, table bound once)
        exec_info = None
        if n > 1:
            exec_info = {"rank": rank, "world_size": n, "tp_rank": rank, "ep_rank": 0, "backend": "nccl",
                         "device": str(device), "tp_group": dist.group.WORLD, "ep_group": None}
        runner = build(dict(case, execution=exec_info) if exec_info else case)
        ctx: StepContext = runner.ctx
        outputs = ctx.allocate_outputs()
        ctx._bind_inputs(values)
        ctx.bind_outputs(outputs)
        stream = torch.cuda.current_stream(device)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        t_all0, t_all1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            for _ in range(args.warmup):
                ctx.launch(stream.cuda_stream)
            torch.cuda.synchronize()
            barrier(n)
            ctx.check()
            barrier(n)
            clocks.mark_start()
            t_all0.record(stream)
            for i in range(args.steps):
                starts[i].record(stream)
                ctx.launch(stream.cuda_stream)
                ends[i].record(stream)
            t_all1.record(stream)
            torch.cuda.synchronize()
            clocks.mark_end()
        barrier(n)
        ctx.check()
        per_step = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        total_ms = max_over_ranks(t_all0.elapsed_time(t_all1), n)
        p50_ms = max_over_ranks(statistics.median(per_step), n)
        ms_per_step = total_ms / args.steps

        # --- end to end through the public API: H2D of token/reset, run(), D2H of next_token
        tok_h = values["token"].cpu().pin_memory()
        rst_h = values["reset"].cpu().pin_memory()
        nxt_h = torch.empty(p["batch"], dtype=torch.int64).pin_memory()
        tok_d, rst_d = values["token"], values["reset"]
        for _ in range(args.warmup):
            tok_d.copy_(tok_h, non_blocking=True)
            rst_d.copy_(rst_h, non_blocking=True)
            out = runner(values)
            nxt_h.copy_(out["next_token"], non_blocking=True)
        barrier(n)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            tok_d.copy_(tok_h, non_blocking=True)
            rst_d.copy_(rst_h, non_blocking=True)
            out = runner(values)
            nxt_h.copy_(out["next_token"], non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(n)
        ctx.check()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1), n) / args.steps
        runner.close()

    if rank != 0:
        return None
    fl = sol.floor_bytes(case)
    nbytes = fl["minimum_bytes"]
    peak, peak_src = peaks()
    achieved = nbytes / (ms_per_step * 1e-3) / 1e9
    B = p["batch"]
    return {
        "metric": "decode-step latency per rank (worst rank, CUDA events)",
        "value": round(ms_per_step * 1000.0, 2),
        "unit": "us",
        "n_gpus": n,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16 activations, mxfp4 experts, fp32 accumulate/state",
        "data": "synthetic (reference seeded generator, seed %d)" % seed,
        "config": {"workload": case["id"], "tp": case["tp"], "batch": B, "layers": p["layers"],
                   "context": p["context"], "parallelism": f"tp{case['tp']}",
                   "l2": "inputs %.1f GB per rank > 126 MB L2; no flush" % (nbytes / 1e9)},
        "p50_us": round(p50_ms * 1000.0, 2),
        "hbm_floor_us": {"at_8.0_TBps": round(nbytes / 8.0e12 * 1e6, 1),
                         f"at_{peak_src}_{peak / 1000:.3f}_TBps": round(nbytes / (peak * 1e9) * 1e6, 1)},
        "pct_of_floor_8TBps": round(100.0 * (nbytes / 8.0e12) / (ms_per_step * 1e-3), 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic_for(case["id"]),
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else "fallback",
                     "algorithmic_bytes_per_launch": nbytes},
        "e2e": {"value": round(e2e_ms * 1000.0, 2), "unit": "us", "h2d_bytes_per_step": B * 8 + B,
                "d2h_bytes_per_step": B * 8},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }


def run_reference(args, n: int) -> dict:
    """The reference algorithm (oracle restatement) on the host cores, per-layer samples of the workload."""
    from oracle import kimi_oracle as ko
    case = pick_case(args, n)
    if case["tp"] != 1:
        case = ko.serial_rank_view(case)   # one rank's arithmetic, reductions local
    p = case["params"]
    torch.set_num_threads(os.cpu_count() or 1)
    t0 = time.perf_counter()
    values = fast_cpu_inputs(case)
    gen_s = time.perf_counter() - t0
    parts = ["embed+head"] + list(range(p["layers"]))
    times = {str(x): [] for x in parts}
    with torch.inference_mode():
        for i in range(args.warmup + args.steps):
            part = parts[i % len(parts)]
            dt = ko.timed_sample(case, values, part)
            if i >= args.warmup:
                times[str(part)].append(dt)
        # parts never sampled in the timed window are sampled once more
        for part in parts:
            if not times[str(part)]:
                times[str(part)].append(ko.timed_sample(case, values, part))
    step_s = sum(statistics.median(v) for v in times.values())
    return {
        "metric": "decode-step latency per rank (worst rank, CUDA events)",
        "impl": "reference",
        "value": round(step_s * 1e6, 1),
        "unit": "us",
        "n_gpus": n,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_s * 1e3, 3),
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16 activations, mxfp4 experts (decoded to bf16), fp32 accumulate/state",
        "data": "synthetic (random fill with the reference's shapes and distributions)",
        "config": {"workload": pick_case(args, n)["id"], "tp": pick_case(args, n)["tp"], "batch": p["batch"],
                   "layers": p["layers"], "context": p["context"], "parallelism": "cpu"},
        "cpu_baseline": {"value": round(step_s * 1e6, 1), "unit": "us", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": "one decoder layer (or embed+head) per step, cycling; value = sum of per-part medians"
                                   f"; input fill {gen_s:.1f} s untimed"},
        "e2e": {"value": round(step_s * 1e6, 1), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "per_part_s": {k: round(statistics.median(v), 4) for k, v in times.items()},
    }


def fast_cpu_inputs(case: dict) -> dict:
    """CPU inputs with the reference's shapes, dtypes and value distributions, filled by tiling one random
    block (the oracle's cost does not depend on the exact values; seeded generation of ~15 GB on CPU would
    take minutes)."""
    from oracle import kimi_oracle as ko
    g = torch.Generator().manual_seed(0)
    block = torch.randn(1 << 22, generator=g)
    codes = torch.randint(0, 256, (1 << 22,), generator=g, dtype=torch.uint8)
    converted: dict = {}

    def tile(t, src):
        flat = t.view(-1)
        for s in range(0, flat.numel(), src.numel()):
            n = min(src.numel(), flat.numel() - s)
            flat[s:s + n].copy_(src[:n])
        return t

    def fill(shape, std, mean, dtype):
        key = (std, mean, dtype)
        if key not in converted:
            converted[key] = (block * std + mean).to(dtype)
        return tile(torch.empty(shape, dtype=dtype), converted[key])

    vals = {}
    p = case["params"]
    for name, (shape, dtype, fan_in, _) in ko.tensor_specs(case).items():
        if name.endswith("_blocks"):
            vals[name] = tile(torch.empty(shape, dtype=torch.uint8), codes)
        elif name.endswith("_scales"):
            e = round(-torch.log2(torch.tensor(2.93 * (p["latent_hidden"] if "down" not in name else p["intermediate"]) ** 0.5)).item())
            vals[name] = (126 + e + torch.randint(0, 3, shape, generator=g)).to(torch.uint8)
        elif name.endswith("A_log"):
            vals[name] = fill(shape, 0.5, 0.0, dtype)
        elif name.endswith("dt_bias"):
            vals[name] = fill(shape, 1.0, -4.0, dtype)
        elif name.endswith("router_bias"):
            vals[name] = fill(shape, 0.01, 0.0, dtype)
        elif fan_in == 0:
            vals[name] = fill(shape, 0.1, 1.0, dtype)
        else:
            vals[name] = fill(shape, fan_in ** -0.5, 0.0, dtype)
    state = ko.make_state(dict(case, params=dict(p, context=1)), 0, "cpu", 0)
    B = p["batch"]
    vals["token"] = state["token"]
    vals["reset"] = torch.zeros(B, dtype=torch.bool)
    hr, d = p["q_heads"] // case["tp"], p["head_dim"]
    for l in range(p["layers"]):
        x = f"l{l}_"
        if ko.is_mla(case, l):
            vals[x + "kv_cache"] = fill((B, p["context"], p["kv_lora_rank"]), 1.0, 0.0, torch.bfloat16)
            vals[x + "pe_cache"] = fill((B, p["context"], p["qk_rope_dim"]), 1.0, 0.0, torch.bfloat16)
        else:
            vals[x + "conv_state"] = fill((B, 3, hr * d, p["conv_kernel"]), 1.0, 0.0, torch.bfloat16)
            vals[x + "recurrent_state"] = fill((B, hr, d, d), 0.05, 0.0, torch.float32)
    return vals


def cpu_baseline_line(args, n: int) -> dict:
    """A short reference-arm measurement attached to the b200 line (rank 0, N=1)."""
    sub = argparse.Namespace(**vars(args))
    sub.steps, sub.warmup = args.cpu_steps, 0
    ref = run_reference(sub, n)
    return ref["cpu_baseline"]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--case", default=None)
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--rank-equivalent", action="store_true",
                    help="N=1 only: time one TP rank of --case (its shard shapes as a TP1 geometry)")
    ap.add_argument("--seed", type=int, default=20261201)
    ap.add_argument("--cpu-steps", type=int, default=5, help="samples of the attached cpu_baseline (N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    n = args.gpus
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}: launch N>1 with torch.distributed.run")
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank == 0:
            print(json.dumps(run_reference(args, n)), flush=True)
        return 0
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    rank, local = init_dist(n)
    try:
        line = run_b200(args, n, rank, local)
        if rank == 0 and line is not None:
            if n == 1 and not args.no_cpu_baseline:
                line["cpu_baseline"] = cpu_baseline_line(args, n)
            print(json.dumps(line), flush=True)
    finally:
        if n > 1:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
