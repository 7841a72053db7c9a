"""The roofline arithmetic of bench.py on the CPU: the algorithmic bytes each bench
line divides by the measured time, and the traffic figures it reads from profiles/."""

import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "iree-adreno-genai-tuner_b200"))

import bench  # noqa: E402
import q4b  # noqa: E402


def test_decode_bytes_per_token_3b():
    """int4 weights + fp16 scales of 28 layers and the lm_head, plus KV rows 0..pos read and row pos
    written (2 x 8 KV heads x 128 x 2 bytes per layer per row)."""
    cfg = q4b.SYNTHETIC["3b"]
    weights = 1_656_483_840
    kv_row = 28 * 2 * 8 * 128 * 2
    assert bench.decode_bytes_per_token(cfg, 640) == weights + kv_row * 642
    assert bench.decode_bytes_per_token(cfg, 640, 2) == (weights + kv_row * 642) / 2


def test_gemv_config1_bytes():
    assert bench.GEMV_BYTES == 8_126_464  # qweight + scales + x + y of the 5120 x 3072 GEMV
    assert bench.linear_bytes(5120, 3072, 1) == bench.GEMV_BYTES


def test_profile_traffic_lines():
    """The traffic the bench lines report comes from the committed ncu summaries and is within a
    percent of the algorithmic bytes (no re-reads)."""
    t = bench.profile_traffic("decode_step_3b")
    assert t is not None and abs(t / bench.decode_bytes_per_token(q4b.SYNTHETIC["3b"], 640) - 1) < 0.01
    g = bench.profile_traffic("q4_gemv_mma_5120x3072")
    assert g is not None and abs(g / bench.GEMV_BYTES - 1) < 0.01
    # the decode line: the 1-GPU capture at N = 1, null at N > 1 (no capture of a rank's launch)
    assert bench.decode_traffic(1.73e9, 1) == t
    assert bench.decode_traffic(0.87e9, 2) is None


def test_trace_summary_reads_the_stamp_layout():
    """bench.trace_summary on a synthetic trace (q4b_model_set_trace layout: 15 stamps per layer,
    then lm_head ready / staged / done and the consumers' start): every stage takes 1 us to become
    ready, 1 us to stage and 1 us to run."""
    import numpy as np

    import bench
    L, ctas = 3, 4
    ev = np.zeros((ctas, 15 * L + 4), np.int64)
    for c in range(ctas):
        ev[c, 15 * L + 3] = 1000
        for i in range(15 * L + 3):
            ev[c, i] = 1000 + (i + 1) * 1000
    t = bench.trace_summary(ev, L)
    for stage in bench.TRACE_PHASES:
        assert t[stage]["stage"] == 1.0 and t[stage]["busy"] == 1.0 and t[stage]["wait"] == 1.0
    assert t["layer_us"] == 15.0 and t["ctas"] == ctas


def test_cpu_sweep_baseline_is_bounded():
    import bench
    cb = bench.cpu_sweep_baseline([1], budget_s=0.5)
    assert cb["value"] > 0 and cb["kind"] == "port" and "M=1" in cb["sample"]


def test_clock_sampler_with_a_fake_nvml(monkeypatch):
    """The clock record of a timed region comes from NVML polled on a thread (read-only queries):
    samples at the start, every few ms and at the end; the timing rules' throttle reasons from the
    clocks-event bits; no NVML -> the nvidia-smi form (here: none available, no samples)."""
    import time
    import types

    import bench
    calls = {"n": 0}
    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=1, nvmlInit=lambda: None, nvmlShutdown=lambda: None,
        nvmlDeviceGetHandleByPciBusId=lambda b: "h", nvmlDeviceGetHandleByIndex=lambda i: "h",
        nvmlDeviceGetClockInfo=lambda h, c: 1965 if calls["n"] % 2 else 1900,
        nvmlDeviceGetMaxClockInfo=lambda h, c: 1965)

    def reasons(h):
        calls["n"] += 1
        return 0x4 if calls["n"] == 3 else 0  # sw_power_cap once
    fake.nvmlDeviceGetCurrentClocksEventReasons = reasons
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench.ClockSampler(0) as c:
        time.sleep(0.05)
    s = c.summary()
    assert s["source"] == "nvml" and s["samples"] >= 3 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"] and 1900 <= s["sm_mhz"] <= 1965
    broken = types.SimpleNamespace(nvmlInit=lambda: (_ for _ in ()).throw(RuntimeError("no NVML")))
    monkeypatch.setitem(sys.modules, "pynvml", broken)
    monkeypatch.setattr(bench.subprocess, "Popen", lambda *a, **k: (_ for _ in ()).throw(OSError("no nvidia-smi")))
    with bench.ClockSampler(0) as c:
        pass
    assert c.summary()["samples"] == 0 and c.summary()["source"] == "nvidia-smi"
