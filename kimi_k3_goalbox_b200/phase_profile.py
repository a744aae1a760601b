"""Per-phase timing of the persistent decode-step kernel.

    python -m kimi_k3_goalbox_b200.phase_profile [--case ID] [--batch B] [--reps N] [--json out.json]

The step is one cooperative launch walking a fixed program of grid-wide phases. CTA 0 stamps %globaltimer at
kernel start and after every grid barrier (KK3_BUF_PHASE_TS), so one full step yields the in-step time of
every phase including its barrier and tail. For comparison each phase is also timed alone:
kk3_debug_phases(start, stop) runs only phases [start, stop) (skipped phases do no work and no barrier), so
phase i alone costs t([i, i+1)) - t(no phase) (CUDA events, median of N repetitions). Each phase also gets its algorithmic HBM
bytes (weights, cache and state it must read or write once), so the table reports achieved GB/s per phase
(the reference measures per-kernel GB/s with Nsight Compute, megabench/integrations/ncu_profile_case.py).
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys

import torch

from . import cases, synthetic
from .cases import is_mla
from .runtime import StepContext


def phase_program(params: dict) -> list[tuple[str, int]]:
    """Grid-phase sequence of the step kernel (csrc/kk3_kernel.cuh): index i ends at stop_phase i+1."""
    L, fd = params["layers"], params["first_dense"]
    prog = [("embed", -1)]
    for l in range(L):
        prog.append(("attn_prologue", l))
        if is_mla(params, l):
            prog += [("mla_proj", l), ("mla_rows", l), ("mla_qb", l), ("mla_absorb", l), ("mla_attend", l),
                     ("mla_combine", l)]
        else:
            prog += [("kda_proj", l), ("kda", l)]
        prog += [("o_proj", l), ("mlp_prologue", l)]
        if l < fd:
            prog += [("dense_gate_up", l), ("dense_down", l)]
        else:
            prog += [("moe_in", l), ("experts_gate_up", l), ("experts_down", l), ("moe_combine", l),
                     ("latent_up", l)]
    if L <= fd:
        prog.append(("fold", -1))
    prog += [("head_prologue", -1), ("lm_head", -1), ("argmax", -1)]
    return prog


def phase_bytes(case: dict, distinct_experts: float | None = None) -> list[int]:
    """Algorithmic HBM bytes of each phase (same accounting as the reference's floor model, split by phase)."""
    p, tp = case["params"], case["tp"]
    B, h, lh, d, H = p["batch"], p["hidden"], p["latent_hidden"], p["head_dim"], p["q_heads"]
    hr, qd = H // tp, H * d // tp
    qr, kr, nr, rd, vd = p["q_lora_rank"], p["kv_lora_rank"], p["qk_nope_dim"], p["qk_rope_dim"], p["v_head_dim"]
    E, k, ctx = p["experts"], p["topk"], p["context"]
    inter, sh, di = p["intermediate"] // tp, p["intermediate"] * p["shared_experts"] // tp, p["dense_intermediate"] // tp
    dist = distinct_experts if distinct_experts is not None else E * (1 - (1 - k / E) ** B)
    fp4 = lambda r, c: r * c // 2 + r * c // 32
    out = []
    for name, l in phase_program(p):
        b = 0
        if name == "embed":
            b = B * h * 2
        elif name == "kda_proj":
            b = 2 * h * (4 * qd + d + hr)
        elif name == "kda":
            b = 2 * qd * d + B * (2 * hr * d * d * 4 + 2 * 3 * qd * 4 * 2) + 3 * qd * 4 * 4
        elif name == "mla_proj":
            b = 2 * h * (qr + kr + rd + hr * vd)
        elif name == "mla_qb":
            b = 2 * hr * (nr + rd) * qr
        elif name == "mla_absorb":
            b = 2 * hr * nr * kr
        elif name == "mla_attend":
            b = B * ctx * (kr + rd) * 2
        elif name == "mla_combine":
            b = 2 * hr * vd * kr
        elif name == "o_proj":
            b = 2 * h * hr * vd
        elif name == "dense_gate_up":
            b = 2 * 2 * di * h
        elif name == "dense_down":
            b = 2 * h * di
        elif name == "moe_in":
            b = 2 * h * (E + lh + 2 * sh)
        elif name == "experts_gate_up":
            b = int(dist * 2 * fp4(inter, lh))
        elif name == "experts_down":
            b = 2 * h * sh + int(dist * fp4(lh, inter))
        elif name == "latent_up":
            b = 2 * h * lh
        elif name == "lm_head":
            b = 2 * (p["vocab"] // tp) * h + B * (p["vocab"] // tp) * 4
        out.append(b)
    return out


def step_phase_times(ctx) -> list[dict]:
    """In-step time of every grid phase of the step that ran last on `ctx` (synchronised by the caller), from the
    %globaltimer stamps CTA 0 writes after every grid barrier: per phase its name, layer, time, the part until
    the last CTA arrived at the barrier ("work") and the barrier after it."""
    prog = phase_program(ctx.params)
    n = len(prog)
    ts = ctx.debug_buffer(16, torch.int64, (n + 1,)).cpu().tolist()
    grid = ctx.launch_config()[0]
    narr = min(n - 1, 256)
    arr = ctx.debug_buffer(17, torch.int64, (narr, grid)).cpu()
    out = []
    for i, (name, layer) in enumerate(prog):
        row = {"name": name, "layer": layer, "us": (ts[i + 1] - ts[i]) / 1e3}
        if i < narr:
            last = int(arr[i].max())
            row["work_us"] = (last - ts[i]) / 1e3
            row["barrier_us"] = (ts[i + 1] - last) / 1e3
        out.append(row)
    return out


def summarize(rows: list[dict], top: int = 10) -> dict:
    """Per phase name: total in-step time over the layers (and its work / barrier split), largest first."""
    agg: dict[str, dict] = {}
    for r in rows:
        a = agg.setdefault(r["name"], {"us": 0.0, "work_us": 0.0, "barrier_us": 0.0, "count": 0})
        a["us"] += r["us"]
        a["work_us"] += r.get("work_us") or 0.0
        a["barrier_us"] += r.get("barrier_us") or 0.0
        a["count"] += 1
    total = sum(r["us"] for r in rows)
    order = sorted(agg.items(), key=lambda kv: -kv[1]["us"])[:top]
    return {"step_us": round(total, 1), "phases": len(rows),
            "barrier_us_total": round(sum(r.get("barrier_us") or 0.0 for r in rows), 1),
            "top": [{"name": k, "us": round(v["us"], 1), "share": round(v["us"] / total, 3) if total else None,
                     "work_us": round(v["work_us"], 1), "barrier_us": round(v["barrier_us"], 1), "count": v["count"]}
                    for k, v in order]}


def profile(case: dict, reps: int = 5, seed: int = 1, device: int = 0) -> list[dict]:
    torch.cuda.set_device(device)
    with torch.inference_mode():
        values = synthetic.make_inputs(case, seed, torch.device("cuda", device))
        ctx = StepContext(case, device=device)
        try:
            out = ctx.allocate_outputs()
            ctx._bind_inputs(values)
            ctx.bind_outputs(out)
            prog = phase_program(case["params"])
            stream = torch.cuda.current_stream()
            for _ in range(3):
                ctx.launch(stream.cuda_stream)
            torch.cuda.synchronize()
            ctx.check()
            flush = torch.empty(64 << 22, dtype=torch.float32, device=torch.device("cuda", device))   # 1 GiB > L2

            def timed(start, stop):
                ts = []
                for _ in range(reps):
                    flush.zero_()   # evict the 126 MB L2 so an isolated phase streams its weights from HBM
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record(stream)
                    ctx.launch(stream.cuda_stream, stop_phase=stop, start_phase=start)
                    e.record(stream)
                    e.synchronize()
                    ts.append(s.elapsed_time(e) * 1000.0)
                return statistics.median(ts)

            full = timed(0, -1)
            # in-step breakdown: globaltimer stamps written at every grid barrier of one full step
            flush.zero_()
            ctx.launch(stream.cuda_stream)
            torch.cuda.synchronize()
            ts = ctx.debug_buffer(16, torch.int64, (len(prog) + 1,)).cpu().tolist()
            instep = [(ts[i + 1] - ts[i]) / 1000.0 for i in range(len(prog))]
            grid = ctx.launch_config()[0]
            sub = ctx.debug_buffer(18, torch.int64, (256, 16)).cpu()
            narr = min(len(prog) - 1, 256)
            arr = ctx.debug_buffer(17, torch.int64, (narr, grid)).cpu()
            wts = ctx.debug_buffer(19, torch.int64, (narr, grid, 16)).cpu()
            # per phase: slowest CTA's arrival after the phase began, and barrier latency after it
            work, barrier, last_cta, spread = [], [], [], []
            for i in range(len(prog)):
                if i < narr:
                    row = arr[i]
                    last = int(row.max())
                    work.append((last - ts[i]) / 1000.0)
                    barrier.append((ts[i + 1] - last) / 1000.0)
                    last_cta.append(int(row.argmax()))
                    rel = ((row - ts[i]).double() / 1000.0).sort().values
                    q = lambda f: round(float(rel[min(len(rel) - 1, int(f * (len(rel) - 1)))]), 2)
                    order = ((row - ts[i]).double()).argsort(descending=True)[:8].tolist()
                    spread.append({"p10": q(0.1), "p50": q(0.5), "p90": q(0.9), "max": q(1.0), "latest": order})
                else:
                    work.append(None)
                    barrier.append(None)
                    last_cta.append(None)
                    spread.append(None)
            empty = timed(len(prog) + 1, -1)      # walks the program, runs no phase: launch cost
            alone = [max(timed(i, i + 1 if i + 1 < len(prog) else -1) - empty, 1e-3) for i in range(len(prog))]
            ctx.check()
        finally:
            ctx.close()
    nbytes = phase_bytes(case)
    subinfo = {}
    for i, (name, layer) in enumerate(prog[:256]):
        st = sub[i].tolist()
        base = ts[i]
        if name == "attn_prologue" and st[0]:
            subinfo[f"{name}:{layer}"] = {"after_wait": (st[0] - base) / 1e3, "stats": (st[1] - base) / 1e3,
                                          "red1": (st[2] - base) / 1e3, "mix": (st[3] - base) / 1e3,
                                          "red2": (st[4] - base) / 1e3, "store": (st[5] - base) / 1e3,
                                          "done": (st[6] - base) / 1e3, "phase_end": (ts[i + 1] - base) / 1e3}
        if name == "mla_attend" and st[0]:
            subinfo[f"{name}:{layer}"] = {k: (st[i] - base) / 1e3 for i, k in enumerate(
                ["start", "q_ready", "t0_data", "t0_scores", "t0_softmax", "t0_pv", "t1_data", "t1_scores",
                 "t1_softmax", "t1_pv", "item_end"]) if st[i]} | {"subtiles": st[11],
                                                                  "phase_end": (ts[i + 1] - base) / 1e3}
        if name == "mla_combine" and st[0]:
            subinfo[f"{name}:{layer}"] = {k: (st[j] - base) / 1e3 for j, k in enumerate(
                ["start", "weights", "latent", "values_pass0", "values_pass1"]) if st[j]} | {
                "phase_end": (ts[i + 1] - base) / 1e3}
        if name == "experts_gate_up" and st[15]:
            subinfo[f"{name}:{layer}"] = {"raw5": st[5], "raw6": st[6], "raw7": st[7], "raw8": st[8],
                                          "staged": (st[9] - base) / 1e3, "warp0_keys": (st[10] - base) / 1e3,
                                          "warp0_threshold": (st[12] - base) / 1e3, "warp0_row": (st[13] - base) / 1e3,
                                          "all_rows": (st[14] - base) / 1e3, "grouped": (st[15] - base) / 1e3,
                                          "phase_end": (ts[i + 1] - base) / 1e3}
        if name == "kda" and st[0]:
            subinfo[f"{name}:{layer}"] = {k: (st[j] - base) / 1e3 for j, k in enumerate(
                ["item_start", "loads_fa", "conv_gate", "norms", "state", "item_end"]) if st[j]} | {
                "phase_end": (ts[i + 1] - base) / 1e3}
        if name == "experts_down" and st[0]:
            subinfo[f"{name}:{layer}"] = {"shared_down_cta0": (st[0] - base) / 1e3, "staged_cta0": (st[1] - base) / 1e3,
                                          "phase_end": (ts[i + 1] - base) / 1e3}
        if name in ("kda_proj", "mla_proj", "moe_in") and st[8]:
            subinfo[f"{name}:{layer}"] = {"warp0_start": (st[8] - base) / 1e3, "first_data": (st[9] - base) / 1e3,
                                          "warp0_end": (st[10] - base) / 1e3, "units": st[11],
                                          "phase_end": (ts[i + 1] - base) / 1e3}
    # engine warps (GEMV / experts): when each warp finished, relative to the phase start; entries outside the
    # phase's window are stale (warps without work in this phase)
    for i, (name, layer) in enumerate(prog[:narr]):
        lo, hi = ts[i], ts[i + 1]
        wend = wts[i].double()
        valid = (wend >= lo) & (wend <= hi)
        if int(valid.sum()) < 64:
            continue
        wrel = torch.where(valid, (wend - lo) / 1e3, torch.full_like(wend, float("nan")))
        wsorted = wrel[valid].sort().values
        wq = lambda f: round(float(wsorted[min(len(wsorted) - 1, int(f * (len(wsorted) - 1)))]), 2)
        wspread = (torch.nan_to_num(wrel, nan=-1e9).max(1).values - torch.nan_to_num(wrel, nan=1e9).min(1).values)
        wspread = wspread[valid.any(1)]
        by_warp = [round(float(wrel[:, k][valid[:, k]].mean()), 1) if bool(valid[:, k].any()) else None
                   for k in range(16)]
        subinfo[f"warps {name}:{layer}"] = {"end_p10": wq(0.1), "end_p50": wq(0.5), "end_p90": wq(0.9),
                                            "end_max": wq(1.0), "cta_spread_mean": round(float(wspread.mean()), 2),
                                            "mean_end_by_warp": by_warp}
    rows = [{"phase": -2, "name": "sub_stamps", "layer": -1, "us": 0.0, "bytes": 0, "GBps": None, "info": subinfo},{"phase": -1, "name": "full_step", "layer": -1, "us": round(full, 2), "bytes": 0, "GBps": None},
            {"phase": -1, "name": "empty_launch", "layer": -1, "us": round(empty, 2), "bytes": 0, "GBps": None}]
    for i, (name, layer) in enumerate(prog):
        dt = instep[i]
        rows.append({"phase": i, "name": name, "layer": layer, "us": round(dt, 2), "alone_us": round(alone[i], 2),
                     "work_us": None if work[i] is None else round(work[i], 2),
                     "barrier_us": None if barrier[i] is None else round(barrier[i], 2), "last_cta": last_cta[i],
                     "cta_done_us": spread[i],
                     "bytes": nbytes[i], "GBps": round(nbytes[i] / (dt * 1e-6) / 1e9, 1) if nbytes[i] and dt > 0 else None})
    return rows


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--case", default="kimi-k3-dev-l4-tp1-b8-s8192")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--rank-equivalent", action="store_true", help="one TP rank of --case as a TP1 geometry")
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--json", default=None)
    args = ap.parse_args(argv)
    case = cases.get_case(args.case)
    case["params"].pop("checkpoint", None)
    if args.rank_equivalent and case["tp"] > 1:
        tp = case["tp"]
        for key in ("q_heads", "vocab", "intermediate", "dense_intermediate"):
            case["params"][key] //= tp
        case.update(gpus=1, tp=1, id=case["id"] + "-rank-equivalent")
    elif case["tp"] > 1:
        raise SystemExit("multi-rank cases: pass --rank-equivalent (one rank's shapes on one GPU)")
    if args.batch:
        case = cases.variant(case, batch=args.batch)
    rows = profile(case, args.reps)
    subrow, head, rows = rows[0], rows[1:3], rows[3:]
    for k, v in [kv for kv in subrow["info"].items() if kv[0].startswith(("mla_attend", "mla_combine", "experts_gate_up", "experts_down:1", "attn_prologue:2", "moe_in:1", "kda:", "warps ")) and (not kv[0].startswith("warps ") or kv[0].endswith(":1"))]:
        print("  sub-phase", k, {kk: (round(vv, 2) if isinstance(vv, float) else vv) for kk, vv in v.items()})
    total = sum(r["us"] for r in rows)
    print(f"{case['id']}: full step {head[0]['us']:.1f} us (events), empty launch {head[1]['us']:.1f} us, "
          f"in-step phases sum to {total:.1f} us (globaltimer), alone-sum {sum(r['alone_us'] for r in rows):.1f} us")
    agg: dict[str, list] = {}
    for r in rows:
        a = agg.setdefault(r["name"], [0.0, 0, 0.0, 0.0, 0, 0.0, 0.0])
        a[0] += r["us"]
        a[1] += r["bytes"]
        if r["work_us"] is not None:
            a[2] += r["work_us"]
            a[3] += r["barrier_us"]
            a[4] += 1
            a[5] += r["cta_done_us"]["p10"]
            a[6] += r["cta_done_us"]["p50"]
    print(f"  {'phase':18s} {'in-step':>9s}  {'share':>5s}  {'GB/s':>13s}  {'CTA done p10/p50/max':>22s}  {'barrier':>8s}")
    for name, (us, b, wk, br, n, p10, p50) in sorted(agg.items(), key=lambda kv: -kv[1][0]):
        gbps = f"{b / (us * 1e-6) / 1e9:8.1f} GB/s" if b and us > 0 else "        -     "
        extra = f"  {p10 / n:6.1f} /{p50 / n:6.1f} /{wk / n:6.1f} us  {br / n:6.2f} us (mean of {n})" if n else ""
        print(f"  {name:18s} {us:9.1f} us  {100 * us / total:5.1f}%  {gbps}{extra}")
    if args.json:
        with open(args.json, "w") as f:
            json.dump({"case": case["id"], "full_us": head[0]["us"], "empty_launch_us": head[1]["us"],
                       "sum_alone_us": total, "phases": rows}, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
