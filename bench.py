"""Benchmark: Kimi K3 decode-step latency per rank on B200 (one cooperative kernel launch per rank per step).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--case ID] [--batch B]

Default workload: kimi-k3-dev-l4-tp1-b8-s8192 at N=1 (the only single-GPU case of the reference's table);
at N>1 the same model (4 layers, full width, batch 8, context 8192) at TP=N, one rank per GPU over NCCL
(torchrun), i.e. strong scaling of a fixed model. `--case` selects any case of the table instead
(e.g. kimi-k3-syn-l8-tp8-b8-s8192 with --gpus 8). Synthetic seeded weights and state on the device
(the reference's generator, a fresh seed per run as the reference's harness draws one per trial); inputs
(>= 14 GB per GPU at the default) are larger than the 126 MB L2, so no flush runs between steps.

Legs of one run, in order:
- parity (checker, untimed): one step through the public `run(inputs)` on fresh-seed inputs, graded with the
  reference's band rule against the BF16 and FP32 oracle computed on the same device tensors, with real
  NCCL all-reduces at N>1 (the reference's `_reduce`/`_greedy` collectives). The oracle is the checker
  here, never the thing measured.
- `value`: device time of K steps (CUDA events on the launching stream, max over ranks), inputs resident.
- `e2e`: the same metric through `submission.build(case)` -> `run(inputs)`, with the step's per-sequence
  inputs (token, reset) copied host->device from pinned memory and next_token copied back, inside the
  timed region.
- extras: at N=8 the north-star cases kimi-k3-syn-l8-tp8-b{1,8,64}-s8192 at real TP8 (parity + latency); at
  N=1 the deep stack (one TP8 rank of syn b8 at the deepest layer count that fits, per layer x 93).
- `--impl reference` times whole steps of the reference algorithm (the oracle restatement, BF16, torch on
  the host cores) on the same workload, on rank 0 only.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import secrets
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

# Inputs of tens to ~170 GB per GPU are generated, freed and generated again in one process: expandable
# segments keep the caching allocator from pinning freed space behind live tensors (set before CUDA starts).
os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from kimi_k3_goalbox_b200 import cases, sol  # noqa: E402

DEFAULT_CASE = "kimi-k3-dev-l4-tp1-b8-s8192"
NORTH_STAR = ["kimi-k3-syn-l8-tp8-b1-s8192", "kimi-k3-syn-l8-tp8-b8-s8192", "kimi-k3-syn-l8-tp8-b64-s8192"]
DEEP_CASE = "kimi-k3-syn-l8-tp8-b8-s8192"
DEEP_LAYERS = (84, 80, 76)           # deepest first; the first whose inputs fit with a margin is used
DEEP_MARGIN = 10 << 30               # bytes left free for the CUDA context, scratch and allocator slack
FALLBACK_HBM_GBS = 6650.0
METRIC = "decode-step latency per rank (worst rank, CUDA events)"


def pick_case(args, n: int) -> dict:
    if args.case:
        case = cases.get_case(args.case)
    else:
        case = cases.get_case(DEFAULT_CASE)
        if n != 1:
            case = cases.variant(case, tp=n)
    if getattr(args, "rank_equivalent", False) and case["tp"] > 1 and n == 1:
        case = rank_equivalent(case)
    elif args.case and case["tp"] != n:
        case = cases.variant(case, tp=n)
    if args.batch:
        case = cases.variant(case, batch=args.batch)
    case["params"].pop("checkpoint", None)
    return case


def plain_case(case_id: str) -> dict:
    """A case of the table with synthetic weights (the checkpoint flag dropped)."""
    case = cases.get_case(case_id)
    case["params"].pop("checkpoint", None)
    return case


def rank_equivalent(case: dict) -> dict:
    """One TP rank's shard shapes as a TP1 geometry: the same arithmetic and bytes as one rank of the case,
    with identity reductions (the survey's one-rank-equivalent method)."""
    tp = case["tp"]
    params = dict(case["params"])
    for key in ("q_heads", "vocab", "intermediate", "dense_intermediate"):
        params[key] //= tp
    params.pop("checkpoint", None)
    return dict(case, id=case["id"] + "-rank-equivalent", gpus=1, tp=1, params=params)


def config_for(case: dict, n: int) -> dict:
    """The `config` object of both arms (the same dict, so the two lines name the same workload)."""
    p = case["params"]
    nbytes = sol.floor_bytes(case)["minimum_bytes"]
    return {"workload": case["id"], "tp": case["tp"], "batch": p["batch"], "layers": p["layers"],
            "context": p["context"], "parallelism": f"tp{case['tp']}", "n_gpus": n,
            "l2": "inputs %.1f GB per rank > 126 MB L2; no flush" % (nbytes / 1e9)}


def peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def traffic_for(case_id: str):
    """DRAM bytes (read + write) of one step-kernel launch of this workload, from the committed ncu summary
    (profiles/step_kernel_traffic.json); None when no capture of this workload exists."""
    path = ROOT / "profiles" / "step_kernel_traffic.json"
    if path.exists():
        try:
            v = json.loads(path.read_text()).get(case_id)
            return v if isinstance(v, (int, float)) else None
        except Exception:
            return None
    return None


# ---------------------------------------------------------------------------------------------------------
# clocks during the timed region


# The sampler loop, run as its own process: it polls NVML every ~1 ms and prints one line per sample
# (time, SM MHz, max SM MHz, power W, clock-event reason bits) until its stdin closes. A process, not a thread:
# in torchrun ranks a polling thread starved (no sample in a whole run), and a process shares nothing with the
# rank's interpreter.
_POLL_SRC = r"""
import sys, time, select
import pynvml
pynvml.nvmlInit()
bus, index, path = sys.argv[1], int(sys.argv[2]), sys.argv[3]
try:
    h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
except Exception:
    h = pynvml.nvmlDeviceGetHandleByIndex(index)
try:
    mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
except Exception:
    mx = float("nan")
with open(path, "w") as out:
    i, pw, ready = 0, float("nan"), False
    while True:
        try:
            sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
            rs = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
            if i % 8 == 0:   # power is the slowest query: every 8th sample
                pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
            out.write(f"{time.time():.6f},{sm},{mx},{pw},{rs}\n")
        except Exception as exc:
            out.write(f"error,{type(exc).__name__}: {exc}\n")
        i += 1
        if not ready:   # NVML is warm once the first sample is written
            print("ready", flush=True)
            ready = True
        r, _, _ = select.select([sys.stdin], [], [], 0.001)
        if r:
            break
"""


class ClockSampler:
    """SM clock, max clock, power and clock-event (throttle) reasons of this rank's GPU, sampled during the
    timed region by a separate process that polls NVML every ~1 ms (the steps are milliseconds long, so an
    nvidia-smi loop at its 50 ms floor would see no sample inside a 20-step window); without NVML it falls back
    to `nvidia-smi -lms 50`. The poller writes its samples to a file (a pipe that nobody reads while the steps
    run would fill up and stall it) and stops when its standard input closes. Only samples inside
    [mark_start, mark_end] enter the summary."""

    # nvmlClocksEventReasons bits (nvml.h)
    REASONS = {0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index: int, bus: str | None = None):
        self.device_index = device_index
        self.bus = bus   # PCI bus id of the GPU (default: from torch's device properties)
        self.samples: list[tuple[float, float, float, float, int]] = []   # (t, sm, max, power_w, reasons)
        self.t0 = self.t1 = None
        self.source = None
        self._proc = None
        self._smi = False
        self._path = None
        self.error = None

    def __enter__(self):
        try:
            import pynvml  # noqa: F401  (the poller needs it)
            bus = self.bus
            if bus is None:
                prop = torch.cuda.get_device_properties(self.device_index)
                bus = f"{prop.pci_domain_id:08x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
            fd, self._path = tempfile.mkstemp(prefix="kk3_clocks_", suffix=".csv")
            os.close(fd)
            self._proc = subprocess.Popen([sys.executable, "-c", _POLL_SRC, bus, str(self.device_index), self._path],
                                          stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                          text=True)
            first = self._proc.stdout.readline().strip()   # NVML up before the timed region starts
            if first != "ready":
                raise RuntimeError(f"poller did not start: {first!r}")
            self.source = "nvml process (1 ms poll)"
        except Exception as exc:
            self.error = f"nvml poller: {type(exc).__name__}: {exc}"
            if self._proc is not None:
                self._proc.kill()
            try:
                fields = "timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active"
                self._proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                     "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self._smi = True
                self.source = "nvidia-smi (50 ms)"
            except Exception:
                self._proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def __exit__(self, *exc):
        if self._proc is None:
            return
        time.sleep(0.01)
        out = ""
        try:
            if self._smi:
                time.sleep(0.1)
                self._proc.terminate()
            out, _ = self._proc.communicate(timeout=10)   # closes the poller's standard input: its stop signal
        except Exception as exc:
            self.error = f"clock sampler stop: {type(exc).__name__}: {exc}"
            self._proc.kill()
            self._proc.communicate()
        if self._path is not None:
            try:
                with open(self._path) as f:
                    out = f.read()
            finally:
                os.unlink(self._path)
        from datetime import datetime
        for line in out.splitlines():
            parts = [x.strip() for x in line.split(",")]
            try:
                if parts[0] == "error":
                    self.error = ",".join(parts[1:])[:200]
                    continue
                ts = (datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp() if self._smi
                      else float(parts[0]))
                rs = int(parts[4], 16) if self._smi else int(parts[4])
                self.samples.append((ts, float(parts[1]), float(parts[2]), float(parts[3]), rs))
            except Exception:
                continue

    def summary(self) -> dict:
        inside = [s for s in self.samples if self.t0 is not None and self.t1 is not None and self.t0 <= s[0] <= self.t1]
        reasons = set()
        for s in inside:
            for bit, name in self.REASONS.items():
                if s[4] & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median([s[1] for s in inside]) if inside else None,
                "sm_max_mhz": inside[0][2] if inside else None, "reasons": sorted(reasons), "samples": len(inside),
                "power_w_max": max((s[3] for s in inside if s[3] == s[3]), default=None), "source": self.source,
                "samples_total": len(self.samples), "error": self.error}


def merge_clocks(summaries: list[dict]) -> dict:
    """Clocks over ranks: the lowest per-rank median, every reason seen on any rank, all samples."""
    got = [s for s in summaries if s.get("sm_mhz") is not None]
    out = {"sm_mhz": min(s["sm_mhz"] for s in got) if got else None,
           "sm_max_mhz": max(s["sm_max_mhz"] for s in got) if got else None,
           "reasons": sorted({r for s in summaries for r in s.get("reasons", [])}),
           "samples": sum(s.get("samples", 0) for s in summaries),
           "power_w_max": max((s["power_w_max"] for s in got if s.get("power_w_max") is not None), default=None),
           "source": summaries[0].get("source") if summaries else None}
    if len(summaries) > 1:
        out["per_rank_sm_mhz"] = [s.get("sm_mhz") for s in summaries]
        out["per_rank_samples"] = [(s.get("samples"), s.get("samples_total")) for s in summaries]
    errors = [s.get("error") for s in summaries if s.get("error")]
    if errors:
        out["errors"] = errors[:2]
    return out


# ---------------------------------------------------------------------------------------------------------
# distributed plumbing


def init_dist(n: int):
    if n == 1:
        return 0, 0
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    return rank, local


def max_over_ranks(x: float, n: int) -> float:
    if n == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather(obj, n: int) -> list:
    if n == 1:
        return [obj]
    out = [None] * n
    dist.all_gather_object(out, obj)
    return out


def barrier(n: int):
    if n > 1:
        dist.barrier()
    torch.cuda.synchronize()


def fresh_seed(args, n: int) -> int:
    """The harness draws secrets.randbits(32) on rank 0 per trial and broadcasts it
    (megabench/harness/distributed.py:33-36); --seed fixes it instead."""
    if args.seed is not None:
        return args.seed
    values = [secrets.randbits(32)]
    if n > 1:
        dist.broadcast_object_list(values, src=0)
    return int(values[0])


def execution_for(case: dict, n: int, rank: int, device) -> dict | None:
    if n == 1:
        return None
    return {"rank": rank, "world_size": n, "tp_rank": rank, "ep_rank": 0, "backend": "nccl", "device": str(device),
            "tp_group": dist.group.WORLD, "ep_group": None}


# ---------------------------------------------------------------------------------------------------------
# the legs


def parity_leg(case: dict, values: dict, runner, n: int, rank: int, seed: int) -> dict:
    """Checker leg (untimed): one step through run(), graded by the reference's band rule
    (megabench/tasks/kimi.py:370-462) against the BF16 and FP32 oracle on the same device tensors, with real
    all-reduces over the process group at N>1 (kimi.py:343-347, :218-227). Every rank takes the same
    collective steps; the outcome is agreed over ranks."""
    from oracle import kimi_oracle as ko
    t0 = time.perf_counter()
    serial = n == 1
    group = None if serial else dist.group.WORLD
    error, details = None, None
    try:
        before = ko.snapshot(values)
        actual = runner(values)
        torch.cuda.synchronize()
        runner.ctx.check()
        actual = {k: v.clone() for k, v in actual.items()}
        ko.check_unchanged(values, before)
    except Exception as exc:   # the step itself failed: no grading collectives are entered by anyone
        error = f"step: {type(exc).__name__}: {exc}"
    errors = gather(error, n)
    if any(errors):
        return {"seed": seed, "pass": False, "reason": "; ".join(e for e in errors if e)[:500]}
    try:
        expected = ko.reference(case, values, serial=serial, tp_rank=rank, group=group)
        details = ko.compare(case, values, expected, actual, serial=serial, tp_rank=rank, group=group)
    except AssertionError as exc:
        error = f"band: {exc}"
    except Exception as exc:
        error = f"grader: {type(exc).__name__}: {exc}"
    errors = gather(error, n)
    torch.cuda.synchronize()
    out = {"seed": seed, "pass": not any(errors), "grader": "oracle band rule (kimi.py:370-462)",
           "collectives": "none (serial)" if serial else f"NCCL all-reduce over {n} ranks", "seconds": None}
    if any(errors):
        out["reason"] = "; ".join(e for e in errors if e)[:500]
    else:
        out["worst_ratio"] = {k: round(v["worst_ratio"], 4) for k, v in details.items() if "worst_ratio" in v}
        out["next_token"] = details["next_token"]
        out["expert_sets_differing_from_oracle"] = details["expert_ids"]["sets_differing_from_oracle"]
        out["cache_length_mismatches"] = details["cache_length"]["mismatched_elements"]
    out["seconds"] = round(time.perf_counter() - t0, 1)
    return out


def time_steps(ctx, stream, steps: int, warmup: int, n: int, clocks: ClockSampler | None = None) -> tuple:
    """Warm up, then time exactly `steps` launches: (total ms of the region, per-step ms list), this rank."""
    for _ in range(warmup):
        ctx.launch(stream.cuda_stream)
    barrier(n)
    ctx.check()
    barrier(n)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clocks:
        clocks.mark_start()
    t0.record(stream)
    for i in range(steps):
        starts[i].record(stream)
        ctx.launch(stream.cuda_stream)
        ends[i].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    if clocks:
        clocks.mark_end()
    barrier(n)
    ctx.check()
    return t0.elapsed_time(t1), [s.elapsed_time(e) for s, e in zip(starts, ends)]


def phase_breakdown(ctx, stream, n: int) -> dict:
    """In-step phase times (CTA 0's %globaltimer stamps after every grid barrier) of the last of three
    back-to-back steps after a barrier, so that the ranks' launch skew does not land in the first exchange
    wait: per phase the slowest rank, summed by phase name over the layers (largest first). Untimed."""
    from kimi_k3_goalbox_b200 import phase_profile
    barrier(n)
    for _ in range(3):
        ctx.launch(stream.cuda_stream)
    torch.cuda.synchronize()
    ctx.check()
    rows = phase_profile.step_phase_times(ctx)
    per_rank = gather(rows, n)
    worst = []
    for i, r in enumerate(rows):
        k = max(range(n), key=lambda q: per_rank[q][i]["us"])
        worst.append(per_rank[k][i])
    out = phase_profile.summarize(worst)
    out["method"] = ("in-step %globaltimer stamps of the last of 3 back-to-back steps; per phase the slowest rank; "
                     "work = until the last CTA arrived")
    return out


def host_comm_leg(args, ctx, stream, n: int) -> dict:
    """The comparison baseline at N>1: the same kernel in phase ranges with the reference's NCCL collectives
    between them (FP32 all-reduce of each partial, kimi.py:343-347; all-gather of the argmax keys, :218-227)
    instead of the in-kernel one-shot peer exchange. Same inputs and outputs as the timed fused steps; one step
    is compared with a fused step first."""
    from kimi_k3_goalbox_b200 import runtime
    from kimi_k3_goalbox_b200 import phase_profile
    group = dist.group.WORLD
    fused = ctx.allocate_outputs()
    ctx.bind_outputs(fused)
    barrier(n)
    for _ in range(3):
        ctx.launch(stream.cuda_stream)
    torch.cuda.synchronize()
    ctx.check()
    fused_rows = phase_profile.step_phase_times(ctx)
    host = ctx.allocate_outputs()
    ctx.bind_outputs(host)
    ctx.set_comm_mode(runtime.COMM_HOST)
    try:
        counts = ctx.launch_host_comm(group, stream.cuda_stream)
        torch.cuda.synchronize()
        ctx.check()
        diff = float((host["logits"] - fused["logits"]).abs().max())
        same_tokens = bool(torch.equal(host["next_token"], fused["next_token"]))
        same_routes = bool(torch.equal(host["expert_ids"], fused["expert_ids"]))
        for _ in range(args.warmup):
            ctx.launch_host_comm(group, stream.cuda_stream)
        barrier(n)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            ctx.launch_host_comm(group, stream.cuda_stream)
        t1.record(stream)
        torch.cuda.synchronize()
        barrier(n)
        ctx.check()
        host_rows = host_phase_times(ctx, runtime)
    finally:
        ctx.set_comm_mode(runtime.COMM_PEER)
    ms = max_over_ranks(t0.elapsed_time(t1), n) / args.steps
    # the phases whose epilogue stores the partial into every rank's slot (fused) or only into its own (host):
    # their in-step time with each transport (slowest rank), the store cost of the peer exchange
    compare = {}
    for name in ("o_proj", "dense_down", "experts_down", "embed"):
        f = [r["us"] for r in fused_rows if r["name"] == name]
        h = [r["us"] for r in host_rows if r["name"] == name and r["us"] is not None]
        if f and h:
            compare[name] = {"fused_us": round(sum(f), 1), "host_us": round(sum(h), 1), "count": len(f)}
    per_rank = gather(compare, n)
    for name in compare:
        for k in ("fused_us", "host_us"):
            compare[name][k] = max(pr[name][k] for pr in per_rank)
    flags = torch.tensor([diff, float(not same_tokens), float(not same_routes)], device="cuda", dtype=torch.float64)
    dist.all_reduce(flags, op=dist.ReduceOp.MAX)
    return {"us": round(ms * 1000.0, 2), "launches_per_step": counts,
            "transport": "NCCL all-reduce (FP32) per partial + all-gather of argmax keys, between phase-range launches",
            "vs_fused": {"max_abs_logit_diff": float(flags[0]), "next_token_equal": not bool(flags[1]),
                         "expert_ids_equal": not bool(flags[2])},
            "exchange_store_phases": compare,
            "note": "same kernel; exchanges by NCCL on the host instead of in-kernel NVLink peer stores"}


def push_comm_leg(args, ctx, stream, n: int) -> dict:
    """The in-kernel push transport (include/kk3.h KK3_COMM_PUSH) on the same inputs: one step compared with a
    fused (peer-transport) step, K timed steps (max over ranks) and its in-step phase breakdown. One launch per
    step, no host collective."""
    from kimi_k3_goalbox_b200 import runtime
    fused = ctx.allocate_outputs()
    ctx.bind_outputs(fused)
    ctx.launch(stream.cuda_stream)
    torch.cuda.synchronize()
    ctx.check()
    pushed = ctx.allocate_outputs()
    ctx.bind_outputs(pushed)
    ctx.set_comm_mode(runtime.COMM_PUSH)
    try:
        ctx.launch(stream.cuda_stream)
        torch.cuda.synchronize()
        ctx.check()
        same = all(torch.equal(pushed[k], fused[k]) for k in fused)
        total_ms, _ = time_steps(ctx, stream, args.steps, args.warmup, n, None)
        phases = phase_breakdown(ctx, stream, n)
    finally:
        ctx.set_comm_mode(runtime.COMM_PEER)
    flag = torch.tensor([0.0 if same else 1.0], device="cuda", dtype=torch.float64)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX)
    return {"us": round(max_over_ranks(total_ms, n) / args.steps * 1000.0, 2), "launches_per_step": 1,
            "outputs_identical_to_fused": not bool(flag[0]), "phase_breakdown": phases,
            "transport": "partials of the projections stored locally, pushed by every CTA at the start of the "
                         "reading phase (coalesced 16-byte pieces, one flag per source and CTA)"}


def host_phase_times(ctx, runtime) -> list[dict]:
    """In-step phase times of the last host-transport step: the phases inside a launch range (a range's first
    phase is left out, its stamp difference spans the NCCL collective before it)."""
    names = runtime.host_comm_program(ctx.params)
    ts = ctx.debug_buffer(16, torch.int64, (len(names) + 1,)).cpu().tolist()
    starts = {start for start, _, _ in runtime.host_comm_segments(ctx.params, ctx.case["tp"])}
    return [{"name": nm, "us": None if i in starts else (ts[i + 1] - ts[i]) / 1e3} for i, nm in enumerate(names)]


def build_runner(case: dict, n: int, rank: int, device):
    from kimi_k3_goalbox_b200.submission import build
    exec_info = execution_for(case, n, rank, device)
    return build(dict(case, execution=exec_info) if exec_info else case)


def measure_case(args, case: dict, n: int, rank: int, local: int, *, parity: bool, seed: int) -> dict:
    """Extra workload: fresh inputs, optional parity leg, K timed steps (max over ranks). Returns the entry."""
    from kimi_k3_goalbox_b200 import synthetic
    device = torch.device("cuda", local)
    entry = {"workload": case["id"], "tp": case["tp"], "batch": case["params"]["batch"],
             "layers": case["params"]["layers"]}
    with torch.inference_mode():
        values = synthetic.make_inputs(case, seed, device, rank=rank)
        torch.cuda.synchronize()
        runner = build_runner(case, n, rank, device)
        try:
            if parity:
                entry["parity"] = parity_leg(case, values, runner, n, rank, seed)
            ctx = runner.ctx
            outputs = ctx.allocate_outputs()
            ctx._bind_inputs(values)
            ctx.bind_outputs(outputs)
            stream = torch.cuda.current_stream(device)
            total_ms, per_step = time_steps(ctx, stream, args.steps, args.warmup, n)
        finally:
            barrier(n)
            runner.close()
    ms = max_over_ranks(total_ms / args.steps, n)
    p50 = max_over_ranks(statistics.median(per_step), n)
    nbytes = sol.floor_bytes(case)["minimum_bytes"]
    peak, _ = peaks()
    entry.update({"us": round(ms * 1000.0, 2), "p50_us": round(p50 * 1000.0, 2),
                  "floor_us_at_8TBps": round(nbytes / 8.0e12 * 1e6, 1),
                  "pct_of_floor_8TBps": round(100.0 * (nbytes / 8.0e12) / (ms * 1e-3), 1),
                  "frac_of_measured_hbm": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4),
                  "algorithmic_bytes": nbytes, "launches_per_step": 1, "seed": seed})
    del values, runner
    gc.collect()
    torch.cuda.empty_cache()
    return entry


def deep_stack(args, local: int) -> dict:
    """One TP8 rank of syn b8 (rank-equivalent TP1 geometry) at the deepest layer count whose inputs fit this
    GPU's free memory with a margin; per-layer latency extrapolated to the full model's 93 layers
    (megabench/sol.py:27-73 floor, README.md:157: 93 layers need ~200 GB per rank)."""
    free, total = torch.cuda.mem_get_info(local)
    base = cases.get_case(DEEP_CASE)
    chosen = None
    for L in DEEP_LAYERS:
        case = rank_equivalent(cases.variant(base, layers=L))
        from kimi_k3_goalbox_b200 import synthetic
        need = sum(torch.Size(s).numel() * torch.empty(0, dtype=dt).element_size()
                   for s, dt, _, _ in synthetic.weight_specs(case).values())
        p = case["params"]
        for l in range(L):
            if cases.is_mla(p, l):
                need += p["batch"] * p["context"] * (p["kv_lora_rank"] + p["qk_rope_dim"]) * 2
            else:
                need += p["batch"] * (3 * p["q_heads"] * p["head_dim"] * 4 * 2 + p["q_heads"] * 128 * 128 * 4)
        if need + DEEP_MARGIN <= free:
            chosen = (L, case, need)
            break
    if chosen is None:
        return {"skipped": f"no layer count in {DEEP_LAYERS} fits {free / 2**30:.1f} GiB free",
                "torch_allocated_gib": round(torch.cuda.memory_allocated(local) / 2**30, 2),
                "torch_reserved_gib": round(torch.cuda.memory_reserved(local) / 2**30, 2)}
    L, case, need = chosen
    seed = args.seed if args.seed is not None else secrets.randbits(32)
    e = measure_case(args, case, 1, 0, local, parity=False, seed=seed)
    full = rank_equivalent(cases.variant(base, layers=93))
    floor93 = sol.floor_bytes(full)["minimum_bytes"]
    per_layer = e["us"] / L
    e.update({"inputs_gib": round(need / 2**30, 1), "free_gib_before": round(free / 2**30, 1),
              "per_layer_us": round(per_layer, 2), "extrapolated_93_layers_us": round(per_layer * 93, 1),
              "floor_93_layers_us_at_8TBps": round(floor93 / 8.0e12 * 1e6, 1),
              "pct_of_floor_93_8TBps": round(100.0 * (floor93 / 8.0e12) / (per_layer * 93 * 1e-6), 1),
              "note": "per layer = step / L (embedding and head included); no parity leg at this depth"})
    return e


def run_b200(args, n: int, rank: int, local: int) -> dict | None:
    from kimi_k3_goalbox_b200 import synthetic
    from kimi_k3_goalbox_b200.runtime import StepContext

    case = pick_case(args, n)
    p = case["params"]
    device = torch.device("cuda", local)
    seed = fresh_seed(args, n)
    with torch.inference_mode():
        values = synthetic.make_inputs(case, seed, device, rank=rank)
        torch.cuda.synchronize()
        runner = build_runner(case, n, rank, device)
        parity = parity_leg(case, values, runner, n, rank, seed) if not args.no_parity else None
        # --- kernel-only timing (inputs resident, table bound once)
        ctx: StepContext = runner.ctx
        outputs = ctx.allocate_outputs()
        ctx._bind_inputs(values)
        ctx.bind_outputs(outputs)
        stream = torch.cuda.current_stream(device)
        with ClockSampler(local) as clocks:
            total_ms, per_step = time_steps(ctx, stream, args.steps, args.warmup, n, clocks)
        clock_summary = merge_clocks(gather(clocks.summary(), n))
        phases = phase_breakdown(ctx, stream, n)
        total_ms = max_over_ranks(total_ms, n)
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
        nccl = host_comm_leg(args, ctx, stream, n) if n > 1 and not args.no_nccl else None
        push = push_comm_leg(args, ctx, stream, n) if n > 1 else None
        runner.close()
        host_values = None
        if rank == 0 and n == 1 and not args.no_cpu_baseline:
            host_values = {k: v.cpu() for k, v in values.items()}   # for the cpu_baseline leg
        del values, outputs, out, runner, ctx, tok_d, rst_d
        gc.collect()
        torch.cuda.empty_cache()

    extras = {}
    if not args.no_extras:
        if n == 8 and args.case is None:
            extras["north_star_tp8"] = [measure_case(args, plain_case(cid), n, rank, local, parity=not args.no_parity,
                                                     seed=fresh_seed(args, n)) for cid in NORTH_STAR]
        elif args.north_star_layers and n > 1 and args.case is None:
            # validation of the north-star leg on fewer GPUs: the same cases at TP = N with fewer layers
            extras["north_star_reduced"] = [
                measure_case(args, cases.variant(plain_case(cid), tp=n, layers=args.north_star_layers), n, rank, local,
                             parity=not args.no_parity, seed=fresh_seed(args, n)) for cid in NORTH_STAR]
        if n == 1 and args.case is None:
            extras["deep_stack"] = deep_stack(args, local)

    if rank != 0:
        return None
    fl = sol.floor_bytes(case)
    nbytes = fl["minimum_bytes"]
    peak, peak_src = peaks()
    achieved = nbytes / (ms_per_step * 1e-3) / 1e9
    B = p["batch"]
    line = {
        "metric": METRIC,
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
        "data": "synthetic (reference seeded generator, fresh seed %d)" % seed,
        "config": config_for(case, n),
        "p50_us": round(p50_ms * 1000.0, 2),
        "hbm_floor_us": {"at_8.0_TBps": round(nbytes / 8.0e12 * 1e6, 1),
                         f"at_{peak_src}_{peak / 1000:.3f}_TBps": round(nbytes / (peak * 1e9) * 1e6, 1)},
        "pct_of_floor_8TBps": round(100.0 * (nbytes / 8.0e12) / (ms_per_step * 1e-3), 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic_for(case["id"]),
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else "fallback",
                     "algorithmic_bytes_per_launch": nbytes,
                     "kernel": "kk3_step_kernel (the whole step is one launch)"},
        "parity": parity,
        "phase_breakdown": phases,
        "nccl_allreduce_variant": nccl,
        "push_exchange_variant": push,
        "e2e": {"value": round(e2e_ms * 1000.0, 2), "unit": "us", "h2d_bytes_per_step": B * 8 + B,
                "d2h_bytes_per_step": B * 8},
        "gpu_launches": args.steps,
        "clocks": clock_summary,
    }
    line.update(extras)
    if host_values is not None:
        line["cpu_baseline"] = cpu_baseline_line(args, n, case, host_values)
    return line


# ---------------------------------------------------------------------------------------------------------
# the reference arm: whole steps of the oracle restatement on the host cores


def host_inputs(case: dict, seed: int) -> tuple[dict, str]:
    """The workload's inputs in host memory: generated with the reference's seeded generator on the GPU
    when one is present (seconds) and copied to the host, else on the host (minutes)."""
    from oracle import kimi_oracle as ko
    if torch.cuda.is_available():
        with torch.inference_mode():
            vals = ko.make_inputs(case, seed, "cuda:0")
            out = {k: v.cpu() for k, v in vals.items()}
            del vals
            torch.cuda.empty_cache()
        return out, "seeded generator on cuda:0, copied to host"
    return ko.make_inputs(case, seed, "cpu"), "seeded generator on the host"


def time_reference_steps(case: dict, values: dict, steps: int, warmup: int) -> tuple[list[float], int]:
    from oracle import kimi_oracle as ko
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    times = []
    with torch.inference_mode():
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            ko.reference(case, values, serial=True)
            dt = time.perf_counter() - t0
            if i >= warmup:
                times.append(dt)
    return times, torch.get_num_threads()


def run_reference(args, n: int) -> dict:
    """`--impl reference`: whole BF16 oracle steps (the reference algorithm, kimi.py:230-340) on the host cores,
    on the arm's workload. At TP>1 one rank's arithmetic runs serially (its shard shapes, local reductions)."""
    from oracle import kimi_oracle as ko
    case = pick_case(args, n)
    serial_case = ko.serial_rank_view(case) if case["tp"] != 1 else case
    seed = args.seed if args.seed is not None else secrets.randbits(32)
    t0 = time.perf_counter()
    values, how = host_inputs(serial_case, seed)
    gen_s = time.perf_counter() - t0
    times, cores = time_reference_steps(serial_case, values, args.steps, args.warmup)
    total_s = sum(times)
    step_us = total_s / len(times) * 1e6
    sample = (f"{args.steps} whole decode steps after {args.warmup} warm-up steps, BF16 oracle restatement "
              f"(MXFP4 decode in C, bit-identical to the reference's torch decode); inputs: {how} in {gen_s:.0f} s, "
              "untimed" + ("; one TP rank's arithmetic serially (reductions local)" if case["tp"] != 1 else ""))
    return {
        "metric": METRIC, "impl": "reference", "value": round(step_us, 1), "unit": "us", "n_gpus": n,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_us / 1000.0, 3),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 activations, mxfp4 experts (decoded to bf16), fp32 accumulate/state",
        "data": "synthetic (reference seeded generator, seed %d)" % seed,
        "config": config_for(case, n),
        "p50_us": round(statistics.median(times) * 1e6, 1),
        "cpu_baseline": {"value": round(step_us, 1), "unit": "us", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(step_us, 1), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "timed_region_s": round(total_s, 1),
    }


def cpu_baseline_line(args, n: int, case: dict, host_values: dict) -> dict:
    """The cpu_baseline object of the b200 line (rank 0, N=1): a bounded sample of whole oracle steps on the
    same inputs (already in host memory), timed on the host cores."""
    times, cores = time_reference_steps(case, host_values, args.cpu_steps, 1)
    step_us = statistics.median(times) * 1e6
    return {"value": round(step_us, 1), "unit": "us", "cores": cores, "kind": "port",
            "sample": f"median of {args.cpu_steps} whole BF16 oracle steps (after 1 warm-up) on this run's inputs; "
                      "MXFP4 decode in C, bit-identical to the reference's torch decode"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--case", default=None)
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--rank-equivalent", action="store_true",
                    help="N=1 only: time one TP rank of --case (its shard shapes as a TP1 geometry)")
    ap.add_argument("--seed", type=int, default=None, help="fixed input seed (default: a fresh one per run)")
    ap.add_argument("--cpu-steps", type=int, default=3, help="whole oracle steps in the attached cpu_baseline (N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the checker leg")
    ap.add_argument("--no-extras", action="store_true", help="skip the north-star (N=8) and deep-stack (N=1) keys")
    ap.add_argument("--no-nccl", action="store_true", help="N>1: skip the plain-NCCL comparison variant")
    ap.add_argument("--north-star-layers", type=int, default=0,
                    help="N in 2..7: also run the north-star cases at TP = N with this many layers (validation)")
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
            print(json.dumps(line), flush=True)
    finally:
        if n > 1:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
