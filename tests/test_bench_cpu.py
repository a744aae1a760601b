"""CPU tests of bench.py's host logic and of the NCCL-baseline segment plan (no GPU, no CUDA call)."""

from __future__ import annotations

import time

import bench
from kimi_k3_goalbox_b200 import cases, runtime
from kimi_k3_goalbox_b200.phase_profile import phase_program


def test_both_arms_name_the_same_config():
    class A:
        case = None
        batch = None
        rank_equivalent = False
    for n in (1, 2, 8):
        case = bench.pick_case(A(), n)
        assert bench.config_for(case, n) == bench.config_for(bench.pick_case(A(), n), n)
        assert case["tp"] == n


def test_clock_summary_keeps_only_the_timed_window_and_names_reasons():
    c = bench.ClockSampler(0)
    t = time.time()
    c.samples = [(t - 5, 1000.0, 1965.0, 300.0, 0), (t, 1965.0, 1965.0, 600.0, 0x4), (t + 0.001, 1950.0, 1965.0, 610.0, 0x8)]
    c.t0, c.t1 = t - 0.5, t + 0.5
    s = c.summary()
    assert s["samples"] == 2 and s["sm_mhz"] == 1957.5 and s["reasons"] == ["hw_slowdown", "sw_power_cap"]
    m = bench.merge_clocks([s, dict(s, sm_mhz=1900.0, reasons=[])])
    assert m["sm_mhz"] == 1900.0 and m["samples"] == 4 and m["reasons"] == ["hw_slowdown", "sw_power_cap"]


def test_host_comm_segments_cover_the_program_with_exchanges_in_kernel_order():
    """The NCCL baseline's phase ranges tile the kernel's host-transport program (the peer program plus one split
    of each MoE combine and of the argmax), each exchange right after the phase that writes its partial, with
    parities alternating in program order (the kernel's exchange counter)."""
    for cid, tp in (("kimi-k3-dev-l4-tp1-b8-s8192", 2), ("kimi-k3-syn-l8-tp8-b8-s8192", 8)):
        case = cases.variant(cases.get_case(cid), tp=tp)
        p = case["params"]
        segs = runtime.host_comm_segments(p, tp)
        n_moe = p["layers"] - p["first_dense"]
        total = len(phase_program(p)) + n_moe + 1          # + combine splits + argmax split
        assert segs[0][0] == 0 and segs[-1][1] == -1
        for (a0, b0, _), (a1, _, _) in zip(segs, segs[1:]):
            assert b0 == a1 and a0 < b0 <= total
        parities = [x[2] for _, _, xs in segs for x in xs[:1]]
        assert parities == [i & 1 for i in range(len(parities))]
        # embedding, 2 per layer, argmax
        assert len(parities) == 1 + 2 * p["layers"] + 1
        assert runtime.host_comm_segments(p, 1) == [(0, -1, [])]


def test_clock_poller_process_records_samples_in_the_window(tmp_path, monkeypatch):
    """The NVML poller runs as its own process (a fake pynvml module stands in for the driver here); it must
    record samples while the parent is busy, stop when the sampler exits and hand every sample back."""
    (tmp_path / "pynvml.py").write_text(
        "NVML_CLOCK_SM = 1\n"
        "def nvmlInit(): pass\n"
        "def nvmlDeviceGetHandleByPciBusId(bus): return 0\n"
        "def nvmlDeviceGetHandleByIndex(i): return 0\n"
        "def nvmlDeviceGetMaxClockInfo(h, kind): return 1965\n"
        "def nvmlDeviceGetClockInfo(h, kind): return 1920\n"
        "def nvmlDeviceGetCurrentClocksEventReasons(h): return 0x4\n"
        "def nvmlDeviceGetPowerUsage(h): return 700000\n")
    monkeypatch.setenv("PYTHONPATH", str(tmp_path))
    with bench.ClockSampler(0, bus="00000000:01:00.0") as c:
        time.sleep(0.05)
        c.mark_start()
        busy = time.time() + 0.3
        while time.time() < busy:   # the parent does not read anything while the steps run
            pass
        c.mark_end()
    s = c.summary()
    assert c.source.startswith("nvml"), c.error
    assert s["samples"] >= 10 and s["sm_mhz"] == 1920.0 and s["sm_max_mhz"] == 1965.0, s
    assert s["reasons"] == ["sw_power_cap"] and s["power_w_max"] == 700.0 and s["error"] is None
