"""Benchmark of the int4 Llama hot path on B200 (one process per GPU; torchrun for N > 1).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload decode|gemv|sweep|profile]
                  [--impl ours|reference]

Prints ONE JSON line (rank 0). Workloads:
  decode  (default) BASELINE config 4: Llama-3.2-3B-shape LlamaQ4 (28 layers, hidden 3072, 24 heads,
          8 KV heads, head_dim 128, intermediate 8192, vocab 128256, tied, int4 group 128), seeded
          random init generated on the GPU; 512-token random prompt, chunked prefill (chunk 128),
          then greedy decode with KV buckets {256, ..., 4096} through the native runner (one CUDA
          graph per bucket). One step = one decode token; --steps K times K decode tokens (K + 1
          generated, the first from the prefill) after --warmup W untimed generate calls. At N > 1
          the model is tensor-parallel over N GPUs (strong scaling). value = decode tokens/s. The
          line carries BASELINE config 1 as its `gemv_5120x3072` object (value, roofline, e2e and
          CPU baseline of its own).
  gemv    BASELINE config 1: int4 GEMV y[5120] = dequant(W)[5120, 3072] . x[3072], group 128, fp16 x/y.
          One step = back-to-back calls over 33 distinct weight copies (> 2x the 126 MB L2), each a
          separate kernel launch captured in one CUDA graph (programmatic dependent launch lets a
          call's weight stream start while the previous call finishes). value = weight+scale+x+y
          bytes moved per second, summed over ranks (replicas: the GEMV does not shard).
  sweep   BASELINE config 5: every 3B projection and the lm_head at M in {1, 4, 16, 64} (--shapes,
          --m), each row timed like config 1; value = aggregate GB/s, with one entry per row.
  profile a short fixed launch sequence for profilers (--layers, --prefill, --pos, --bucket).
  gemm    BASELINE config 2: the fp16 GEMM sweep (M in {128, 2048} x the 3B projections, plus the
          M = 1 rows) through q4b_gemm_f16, TFLOP/s against min(tensor peak, AI x HBM).
  ctx     the context-length sweep of scripts/llm/bench.py + summarize.py: ctx 256 .. 4096 (prompt
          = ctx - --new), schedules bucketed and max, --prompts seeded prompts each; one line with
          the per-(schedule, ctx) medians and speed-ups.
--impl reference times the CPU restatement of the reference path (oracle port: whole decode steps with
the int4 GEMVs in C) on the host cores of rank 0; other ranks exit without work.
"""

from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "iree-adreno-genai-tuner_b200"))
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests" / "golden"))

GEMV_N, GEMV_K, GEMV_G = 5120, 3072, 128
GEMV_BYTES = GEMV_N * GEMV_K // 2 + GEMV_N * (GEMV_K // GEMV_G) * 2 + GEMV_K * 2 + GEMV_N * 2  # 8,126,464
GEMV_COPIES = 32
METRIC_GEMV = "int4 GEMV HBM GB/s (5120x3072)"
METRIC_DECODE = "3B-shape int4 batch-1 decode tokens/s"
PROMPT_LEN, CHUNK, BUCKETS = 512, 128, [256, 512, 1024, 2048, 4096]


def decode_bytes_per_token(cfg, pos, tp=1):
    """Algorithmic HBM bytes of one decode token at position pos on one of tp GPUs: int4 weights +
    fp16 scales of every projection and the lm_head shard, KV rows 0..pos read and row pos written."""
    D, H, Hkv, hd = cfg["hidden_size"], cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    I, V, nl, G = cfg["intermediate_size"], cfg["vocab_size"], cfg["num_hidden_layers"], 128

    def q4(n, k):
        return n * k // 2 + n * (k // G) * 2
    layer = q4((H + 2 * Hkv) * hd, D) + q4(D, H * hd) + q4(2 * I, D) + q4(D, I)
    kv_row = nl * 2 * Hkv * hd * 2
    return (nl * layer + q4(V, D) + kv_row * (pos + 1) + kv_row) / tp


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(name, key="traffic_bytes_per_launch"):
    """A figure recorded from an ncu capture in profiles/<name>.txt (a line "<key>: N"): by default the
    dram bytes per launch."""
    p = ROOT / "profiles" / f"{name}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith(key + ":"):
            return float(line.split(":", 1)[1].split()[0])
    return None


def decode_traffic(bytes_tok, world):
    """roofline.traffic of the decode line: the dram bytes per launch of the committed 1-GPU ncu
    capture (profiles/decode_step_3b.txt); null at tp > 1, where no capture of a rank's launch exists
    (a multi-rank command is never run under ncu)."""
    del bytes_tok
    return profile_traffic("decode_step_3b") if world == 1 else None


class ClockSampler:
    """SM clock and throttle reasons during the timed region: NVML polled every 5 ms on a thread
    (read-only queries), else nvidia-smi at its 100 ms minimum; summary = median SM MHz under load,
    max SM MHz, the reasons seen and the sample count."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits (nvml.h): the ones the timing rules name
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}
    PERIOD_S = 0.005

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.nvml = None  # (module, handle) while NVML samples
        self.samples = []  # NVML: (sm_mhz, max_mhz, reason bits)
        self.stop = threading.Event()

    def _nvml_handle(self, nv):
        try:  # the NVML device of this process's CUDA device, by PCI address (CUDA and NVML orders can differ)
            import torch
            p = torch.cuda.get_device_properties(self.gpu)
            return nv.nvmlDeviceGetHandleByPciBusId(f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0")
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.gpu)

    def _nvml_sample(self):
        nv, h = self.nvml
        self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                             nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM),
                             nv.nvmlDeviceGetCurrentClocksEventReasons(h)))

    def _poll(self):
        while not self.stop.wait(self.PERIOD_S):
            try:
                self._nvml_sample()
            except Exception:
                return

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nvml = (nv, self._nvml_handle(nv))
            self._nvml_sample()  # one sample as the region starts
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nvml = None
            self.samples = []
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.nvml:
            self.stop.set()
            self.t.join(timeout=2)
            try:
                self._nvml_sample()  # and one as it ends
                self.nvml[0].nvmlShutdown()
            except Exception:
                pass
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.samples:
            sm = [float(x[0]) for x in self.samples]
            reasons = {nm for _, _, bits in self.samples for nm, bit in self.REASON_BITS.items() if bits & bit}
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(self.samples[-1][1]),
                    "reasons": sorted(reasons), "samples": len(sm), "source": "nvml"}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for nm, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi"}


def dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


def init_dist(world, local):
    import torch
    import torch.distributed as dist
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return dist if world > 1 else None


def max_over_ranks(v, dist_mod):
    import torch
    if dist_mod is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist_mod.all_reduce(t, op=dist_mod.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(v, dist_mod):
    import torch
    if dist_mod is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist_mod.all_reduce(t)
    return float(t.item())


# ---------------------------------------------------------------------------------------------
# CPU baseline (oracle port of the reference's QLinear dequant + linear, scripts/llm/llama_q4.py:72)
# ---------------------------------------------------------------------------------------------

def cpu_gemv_baseline(budget_s=8.0):
    """BASELINE config 1 on the host cores: the C restatement of QLinear._gemv_fused
    (oracle/q4_cpu.c) on the same synthetic 5120 x 3072 inputs, one thread per CPU."""
    import numpy as np

    import golden_inputs as gi
    from oracle import q4_cpu as C
    qw, s, x = gi.gemv_inputs()
    xf = x.astype(np.float32)
    C.gemv(qw, s, GEMV_G, xf)
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 5:
        t0 = time.perf_counter()
        C.gemv(qw, s, GEMV_G, xf)
        times.append(time.perf_counter() - t0)
        if len(times) >= 2000:
            break
    med = statistics.median(times)
    return {"value": GEMV_BYTES / med / 1e9, "unit": "GB/s", "cores": C.threads(), "kind": "port",
            "sample": f"{len(times)} calls of the C restatement of the fused GEMV on 5120x3072 g128 "
                      f"(median {med * 1e3:.3f} ms/call, {C.threads()} threads)"}


# ---------------------------------------------------------------------------------------------
# GPU GEMV workload
# ---------------------------------------------------------------------------------------------

def run_gemv(args, rank, world, local, dist_mod):
    """BASELINE config 1 as its own line: value = weight + scale + x + y bytes per second of the
    chained calls, summed over ranks (replicas: a 5120 x 3072 GEMV is one GPU's work)."""
    import torch
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = json.loads(args.gemv_cfg) if args.gemv_cfg else None
    if dist_mod:
        dist_mod.barrier()
    with ClockSampler(local) as clk:
        per_call, copies, qws, scs, x, ys = chain_measure(dev, GEMV_N, GEMV_K, 1, args.steps, args.warmup, cfg=cfg,
                                                          seed=1234 + rank)
    per_call = max_over_ranks(per_call, dist_mod)
    ms_step = per_call * copies * 1e3
    value = world * GEMV_BYTES / per_call / 1e9
    check = None
    if rank == 0:  # parity spot check of the last pass against the CPU restatement (copy 0)
        from oracle import q4_oracle as O
        ref = O.q4_linear(qws[0].cpu().numpy(), scs[0].cpu().numpy(), GEMV_G, x.float().cpu().numpy())
        check = O.rel_err(ys[0].float().cpu().numpy(), ref)
    e2e_ms = max_over_ranks(gemv_e2e(dev, qws[0], scs[0], x, max(args.steps, 50)), dist_mod)
    if rank != 0:
        return None
    pk = peaks()
    k = kernel_of(1, GEMV_N, GEMV_K, cfg)
    line = {
        "metric": METRIC_GEMV, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int4 weights, fp16 x/y, fp32 accumulate", "data": "synthetic",
        "config": {"workload": "int4 GEMV 5120x3072 group 128 M=1 (BASELINE config 1)",
                   "calls_per_step": copies, "l2": f"inputs larger than L2: {copies} distinct weight "
                   f"copies x {GEMV_BYTES / 1e6:.2f} MB", "parallelism": f"replicas x{world}",
                   "launch": "CUDA graph of separate launches with programmatic dependent launch", "cfg": cfg},
        "roofline": {"bound": "hbm", "achieved": round(GEMV_BYTES / per_call / 1e9, 1), "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": round(GEMV_BYTES / per_call / 1e9 / pk["hbm_gbs"], 4),
                     "traffic": profile_traffic("q4_gemv_ring_5120x3072") if k == 6 else None,
                     "peak_source": pk["source"], "kernel": f"q4_linear kernel {k}",
                     "algorithmic_bytes_per_launch": GEMV_BYTES},
        "e2e": {"value": round(world * GEMV_BYTES / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": GEMV_K * 2, "d2h_bytes_per_step": GEMV_N * 2, "ms_per_call": round(e2e_ms, 4),
                "path": "q4b.QLinear.forward per call with pinned-host x in and y out, synchronised"},
        "gpu_launches": args.steps * copies,
        "clocks": clk.summary(),
        "parity_rel_err": check,
    }
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_gemv_baseline()
    return line


def cpu_decode_baseline(steps=5, warmup=1, pos0=PROMPT_LEN, bucket=1024):
    """The reference's decode step restated on the host cores (oracle/q4_cpu.py): whole 28-layer
    Llama-3.2-3B-shape steps at the bench's positions (pos0, pos0 + 1, ...) and bucket, int4 GEMVs in
    C on one thread per CPU (QLinear._gemv_fused), norm / RoPE / attention / SwiGLU in numpy. The KV
    cache holds random fp16 values instead of the prompt's (the time does not depend on them)."""
    import q4b
    from oracle import q4_cpu as C
    t0 = time.perf_counter()
    m = C.DecodeModel(q4b.SYNTHETIC["3b"], max_ctx=bucket)
    build_s = time.perf_counter() - t0
    tok = 17
    for i in range(warmup):
        tok = m.step(tok, pos0 + i, bucket)
    t0 = time.perf_counter()
    for i in range(steps):
        tok = m.step(tok, pos0 + warmup + i, bucket)
    dt = time.perf_counter() - t0
    return {"value": steps / dt, "unit": "tokens/s", "cores": C.threads(), "kind": "port",
            "sample": f"{steps} whole decode steps (28 layers + lm_head) at positions {pos0 + warmup}.."
                      f"{pos0 + warmup + steps - 1}, bucket {bucket}, after {warmup} warm-up; "
                      f"{dt / steps * 1e3:.0f} ms/token; C int4 GEMVs on {C.threads()} threads + numpy "
                      f"(model build {build_s:.1f} s, KV cache random)",
            "same_config": True}


def run_decode(args, rank, world, local, dist_mod):
    import numpy as np
    import torch

    import q4b
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = q4b.SYNTHETIC["3b"]
    t0 = time.perf_counter()
    model = q4b.LlamaQ4(None, group=128, max_ctx=4096, sd=q4b.SyntheticStateDict(cfg, seed=0, device=dev), cfg=cfg,
                        max_chunk=CHUNK, tp_rank=rank, tp_size=world, device=dev)
    if world > 1:
        model.attach_tp(dist_mod)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    prompt = np.random.default_rng(0).integers(0, cfg["vocab_size"], PROMPT_LEN).tolist()
    n_new = args.steps + 1
    runner = q4b.Runner(model, CHUNK, BUCKETS, "bucketed", graphs=True)
    for _ in range(args.warmup):
        runner.generate(prompt, n_new)
    if dist_mod:
        dist_mod.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        toks, rep = runner.generate(prompt, n_new)
    torch.cuda.synchronize()
    if dist_mod:
        dist_mod.barrier()
    steps = rep["decode_steps"]
    decode_ms = max_over_ranks(rep["decode_ms"], dist_mod)
    value = steps / (decode_ms / 1e3)
    # end to end through the public API with the reference's per-call protocol: each step copies its
    # inputs in and its token out and the host checks stop ids
    rs = q4b.Runner(model, CHUNK, BUCKETS, "bucketed", graphs=True, sync_every_step=True)
    rs.generate(prompt, min(n_new, 17))
    if dist_mod:
        dist_mod.barrier()
    toks_e2e, rep_e2e = rs.generate(prompt, n_new)
    e2e_ms = max_over_ranks(rep_e2e["decode_wall_ms"], dist_mod)
    same = toks_e2e == toks
    gemv = lm = None
    if world == 1 and not args.no_gemv:
        gemv = gemv_measure(dev, steps=50, warmup=5, cpu=not args.no_cpu_baseline)
        lm = lm_head_measure(dev)
    if rank != 0:
        return None
    pk = peaks()
    pos = [PROMPT_LEN + i for i in range(steps)]
    bytes_tok = statistics.mean(decode_bytes_per_token(cfg, p, world) for p in pos)
    achieved = bytes_tok * value / 1e9
    persistent = bool(q4b.lib().q4b_model_decode_path(model.native()))
    # persistent decode: one cooperative kernel per token (plus a 8-byte counter reset); else per layer
    # q|k|v, attention, o, gate|up, down, and embedding + final norm + lm_head (+ TP collectives)
    launches = 1 if persistent else 2 + 5 * cfg["num_hidden_layers"] + (
        0 if world == 1 else 2 * cfg["num_hidden_layers"] + 1)
    # (with tp the persistent step pushes o / down partial sums and argmax keys to the peers' memory
    # inside the kernel: no collective launches)
    line = {
        "metric": METRIC_DECODE, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(decode_ms / steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int4 weights, fp32 activations, fp16 KV cache",
        "data": "synthetic (seeded random init, random prompt ids)",
        "config": {"workload": "Llama-3.2-3B-shape LlamaQ4 batch-1 decode (BASELINE config 4)",
                   "prompt": PROMPT_LEN, "new_tokens": steps + 1, "chunk": CHUNK, "buckets": BUCKETS,
                   "schedule": "bucketed", "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2: 1.66 GB of weights streamed per token",
                   "graphs": "one CUDA graph per (phase, bucket), decode steps back to back on the device",
                   "decode_kernel": "persistent (one cooperative launch per token)" if persistent
                   else "per projection"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": decode_traffic(bytes_tok, world),
                     **({"traffic_note": "null: no ncu capture of a tensor-parallel rank's launch (the "
                                         "1-GPU capture reads 1.007x the algorithmic bytes)"} if world > 1 else {}),
                     "peak_source": pk["source"], "kernel": "decode_step_kernel" if persistent else "decode step (q4_gemv_* dominant)",
                     "algorithmic_bytes_per_token_per_gpu": round(bytes_tok)},
        "e2e": {"value": round(steps / (e2e_ms / 1e3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": 104, "d2h_bytes_per_step": 4,
                "path": "q4b.Runner(sync_every_step=True).generate: per step state H2D, graph, token D2H, sync",
                "tokens_match_async": same},
        "gpu_launches": steps * launches,
        "clocks": clk.summary(),
        "prefill": {"ttft_ms": rep["ttft_ms"], "prefill_tok_s": rep["prefill_tok_s"], "chunks": rep["chunks"]},
        "model_build_s": round(build_s, 1),
        "tokens_head": toks[:8],
    }
    if gemv:
        line["gemv_5120x3072"] = gemv
    if lm:
        line["gemv_lm_head_128256x3072"] = lm
    if not args.no_cpu_baseline and world == 1:  # the host baseline belongs to the N = 1 line
        line["cpu_baseline"] = cpu_decode_baseline(steps=5, warmup=1)
    return line


L2_BYTES = 126 * 2**20
SWEEP_SHAPES = {"qkv": (5120, 3072), "o": (3072, 3072), "gu": (16384, 3072), "down": (3072, 8192),
                "lm": (128256, 3072)}


def linear_bytes(n, k, m, g=128):
    """Algorithmic bytes of one q4_linear call: int4 weights + fp16 scales + fp16 x and y."""
    return n * k // 2 + 2 * n * (k // g) + 2 * m * k + 2 * m * n


def kernel_of(m, n, k, cfg=None, x_f16=True):
    """The kernel number the library's planner picks (include/q4b.h, q4b_q4_linear_kernel)."""
    import ctypes

    import q4b
    from q4b import _lib
    c = _lib.LinearCfg(**cfg) if cfg else None
    return int(q4b.lib().q4b_q4_linear_kernel(m, n, k, 128, 0, 1 if x_f16 else 0, ctypes.byref(c) if c else None))


def chain_measure(dev, n, k, m, steps, warmup, cfg=None, seed=99):
    """Seconds per q4_linear call over distinct weight copies (together more than twice the 126 MB
    L2, so every call streams its weights from HBM), each call a separate launch, all captured in
    one CUDA graph (programmatic dependent launch lets a call's weight stream start while the
    previous call finishes). Returns (seconds per call, copies, weights, scales, x, outputs)."""
    import math

    import torch

    import q4b
    from q4b import ops
    wbytes = n * k // 2 + 2 * n * (k // 128)
    copies = max(1, math.ceil(2 * L2_BYTES / wbytes))
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    # BASELINE config 1's inputs: uniform nibbles packed 8 per int32, |N(0, 0.02)| fp16 scales, fp16 x
    qws = [torch.randint(-2**31, 2**31 - 1, (n, k // 8), dtype=torch.int32, device=dev, generator=g)
           for _ in range(copies)]
    scs = [(torch.randn(n, k // 128, device=dev, generator=g) * 0.02).abs().half() for _ in range(copies)]
    x = torch.randn(m, k, device=dev, generator=g).half()
    ys = [torch.empty(m, n, dtype=torch.float16, device=dev) for _ in range(copies)]
    stream = torch.cuda.Stream(device=dev)

    def one_pass():
        for i in range(copies):
            ops.q4_linear(x, qws[i], scs[i], 128, out=ys[i], cfg=cfg)

    with torch.cuda.stream(stream):
        one_pass()  # allocates the workspace outside the capture
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        graph.capture_begin()
        one_pass()
        graph.capture_end()
        for _ in range(warmup):
            graph.replay()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    if q4b.lib().q4b_device_status(1) != 0:
        raise RuntimeError("q4b: a bounded device wait gave up during the measurement")
    per_call = e0.elapsed_time(e1) / 1e3 / (steps * copies)
    del graph
    return per_call, copies, qws, scs, x, ys


def gemv_e2e(dev, qw, sc, x, steps):
    """Config 1 end to end through the public API: pinned host x -> QLinear.forward -> pinned host
    y, synchronised after every call (ms per call)."""
    import torch

    import q4b
    ql = q4b.QLinear.from_packed(qw, sc, GEMV_G)
    xh = x.cpu().pin_memory()
    yh = torch.empty(1, GEMV_N, dtype=torch.float16).pin_memory()
    for _ in range(5):
        yh.copy_(ql(xh.to(dev, non_blocking=True)), non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        yh.copy_(ql(xh.to(dev, non_blocking=True)), non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / steps


def gemv_measure(dev, steps=50, warmup=5, cpu=True):
    """BASELINE config 1 inside the decode run: its own value, roofline, e2e and CPU baseline."""
    from oracle import q4_oracle as O
    per_call, copies, qws, scs, x, ys = chain_measure(dev, GEMV_N, GEMV_K, 1, steps, warmup)
    ref = O.q4_linear(qws[0].cpu().numpy(), scs[0].cpu().numpy(), GEMV_G, x.float().cpu().numpy())
    err = O.rel_err(ys[0].float().cpu().numpy(), ref)
    e2e_ms = gemv_e2e(dev, qws[0], scs[0], x, max(steps, 50))
    pk = peaks()
    gbs = GEMV_BYTES / per_call / 1e9
    k = kernel_of(1, GEMV_N, GEMV_K)
    out = {"metric": METRIC_GEMV, "value": round(gbs, 1), "unit": "GB/s", "us_per_call": round(per_call * 1e6, 3),
           "kernel": f"q4_linear kernel {k}", "calls": steps * copies,
           "l2": f"{copies} distinct weight copies ({copies * GEMV_BYTES / 1e6:.0f} MB > L2)",
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                        "frac": round(gbs / pk["hbm_gbs"], 4), "peak_source": pk["source"],
                        "traffic": profile_traffic("q4_gemv_ring_5120x3072") if k == 6 else None,
                        "algorithmic_bytes_per_launch": GEMV_BYTES},
           "e2e": {"value": round(GEMV_BYTES / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                   "h2d_bytes_per_step": GEMV_K * 2, "d2h_bytes_per_step": GEMV_N * 2, "ms_per_call": round(e2e_ms, 4),
                   "path": "q4b.QLinear.forward per call with pinned-host x in and y out, synchronised"},
           "parity_rel_err": err}
    if cpu:
        out["cpu_baseline"] = cpu_gemv_baseline()
    return out


def lm_head_measure(dev, steps=20, warmup=3):
    """The 3B lm_head as one GEMV launch (128256 x 3072, 197 MB of int4 + scales, M = 1): GB/s of
    chained launches over two weight copies (> 2x L2) against the HBM roofline."""
    n, k = 128256, 3072
    per_call, copies, *_ = chain_measure(dev, n, k, 1, steps, warmup, seed=7)
    b = linear_bytes(n, k, 1)
    pk = peaks()
    gbs = b / per_call / 1e9
    return {"metric": "int4 GEMV HBM GB/s (128256x3072, one launch)", "value": round(gbs, 1), "unit": "GB/s",
            "us_per_call": round(per_call * 1e6, 2), "kernel": f"q4_linear kernel {kernel_of(1, n, k)}",
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / pk["hbm_gbs"], 4), "peak_source": pk["source"],
                         "traffic": profile_traffic("q4_gemv_ring_lm_head"), "algorithmic_bytes_per_launch": b},
            "calls": steps * copies}


def summarize_ctx(records):
    """scripts/llm/summarize.py:25-44: per (schedule, ctx) medians over the prompts (prefill tok/s,
    TTFT, decode tok/s) and each row's speed-up over the first schedule at the same ctx."""
    groups = {}
    for r in records:
        groups.setdefault((r["schedule"], r["ctx"]), []).append(r)
    order = []
    for r in records:
        if r["schedule"] not in order:
            order.append(r["schedule"])
    rows = []
    for (sched, ctx), rs in sorted(groups.items(), key=lambda kv: (order.index(kv[0][0]), kv[0][1])):
        rows.append(dict(schedule=sched, ctx=ctx, n=len(rs),
                         prefill_tok_s=round(statistics.median(r["prefill_tok_s"] for r in rs), 1),
                         ttft_s=round(statistics.median(r["ttft_ms"] for r in rs) / 1e3, 4),
                         decode_tok_s=round(statistics.median(r["decode_tok_s"] for r in rs), 2)))
    base = {r["ctx"]: r for r in rows if r["schedule"] == order[0]}
    for r in rows:
        b = base.get(r["ctx"])
        r["prefill_x"] = round(r["prefill_tok_s"] / b["prefill_tok_s"], 3) if b else None
        r["decode_x"] = round(r["decode_tok_s"] / b["decode_tok_s"], 3) if b else None
    return rows


def run_ctx(args, rank, world, local, dist_mod):
    """scripts/llm/bench.py:67-104 on the B200: for each context length (prompt = ctx - new tokens,
    then `new` greedy tokens) and schedule, the runner's report on the 3B-shape model; the reference's
    three prompt kinds (tokenised text) become three seeded random-id prompts (no tokenizer or corpus
    here; the ids do not change the work). One JSON line with the summarize.py table."""
    import numpy as np
    import torch

    import q4b
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = q4b.SYNTHETIC["3b"]
    model = q4b.LlamaQ4(None, group=128, max_ctx=max(BUCKETS), sd=q4b.SyntheticStateDict(cfg, seed=0, device=dev),
                        cfg=cfg, max_chunk=CHUNK, tp_rank=rank, tp_size=world, device=dev)
    if world > 1:
        model.attach_tp(dist_mod)
    records = []
    runners = {s: q4b.Runner(model, CHUNK, BUCKETS, s, graphs=True, warmup=1) for s in args.schedules}
    for seed in range(args.prompts):
        for ctx in args.ctx:
            prompt = np.random.default_rng(100 + seed).integers(0, cfg["vocab_size"], ctx - args.new).tolist()
            for sched in args.schedules:
                toks, rep = runners[sched].generate(prompt, args.new)
                records.append(dict(kind=f"seed{seed}", ctx=ctx, schedule=sched, prompt_tokens=rep["prompt_tokens"],
                                    prefill_tok_s=rep["prefill_tok_s"], ttft_ms=rep["ttft_ms"],
                                    decode_tok_s=rep["decode_tok_s"], new_tokens=len(toks)))
    if rank != 0:
        return None
    rows = summarize_ctx(records)
    dec = [r["decode_tok_s"] for r in rows if r["schedule"] == args.schedules[0]]
    if args.out:
        with open(args.out, "a") as f:
            for r in records:
                f.write(json.dumps(dict(r, tag=args.tag)) + "\n")
    return {"metric": "3B-shape decode tokens/s across context lengths (median over prompts)",
            "value": round(statistics.median(dec), 2), "unit": "tokens/s", "n_gpus": world, "steps": args.new,
            "warmup": 1, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4 weights, fp32 activations, fp16 KV cache", "data": "synthetic (seeded random prompt ids)",
            "config": {"workload": "context-length sweep (scripts/llm/bench.py + summarize.py)", "ctx": args.ctx,
                       "new": args.new, "prompts": args.prompts, "schedules": args.schedules, "chunk": CHUNK,
                       "buckets": BUCKETS, "parallelism": f"tp{world}"},
            "rows": rows}


def run_gemm(args, rank, world, local, dist_mod):
    """the fp16 GEMM sweep C = A B (row-major A [M, K], B [K, N], fp32
    accumulate, fp16 C) on the 8 shapes M in {128, 2048} x the 3B projections plus the 4 M = 1 rows,
    through q4b_gemm_f16's default plan. Per shape: mean time of back-to-back calls in a CUDA graph
    over enough (A, B) copies that operands come from HBM (> 2x L2 where one call's bytes are below
    it), TFLOP/s and the attainable roofline min(tensor peak, AI x HBM) (gemm/shapes.py flops and
    min_bytes, BLOG-GEMM.md:109). value = the geometric mean of the 8 shapes' fractions of attainable."""
    import math

    import torch

    from q4b import ops
    from q4b.gemm.shapes import EXTRA, SHAPES
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pk = peaks()
    rows = []
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    gcfg = json.loads(args.gemm_cfg) if args.gemm_cfg else None
    for s in SHAPES + EXTRA:
        # the cfg applies to the tcgen05 shapes; the M = 1 rows keep their default plan
        cfg = gcfg if (gcfg and s.M > 1) else None
        copies = max(1, math.ceil(2 * L2_BYTES / s.min_bytes)) if s.min_bytes < 2 * L2_BYTES else 1
        A = [(torch.rand(s.M, s.K, device=dev, generator=g) * 2 - 1).half() for _ in range(copies)]
        B = [(torch.rand(s.K, s.N, device=dev, generator=g) * 2 - 1).half() for _ in range(copies)]
        C = [torch.empty(s.M, s.N, dtype=torch.float16, device=dev) for _ in range(copies)]
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(stream):
            for i in range(copies):
                ops.gemm_f16(A[i], B[i], out=C[i], cfg=cfg)
            graph = torch.cuda.CUDAGraph()
            graph.capture_begin()
            for i in range(copies):
                ops.gemm_f16(A[i], B[i], out=C[i], cfg=cfg)
            graph.capture_end()
            for _ in range(args.warmup):
                graph.replay()
        stream.synchronize()
        reps = max(1, args.steps)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
        e1.synchronize()
        t = e0.elapsed_time(e1) / 1e3 / (reps * copies)
        ref = A[0].float() @ B[0].float()
        err = float((C[0].float() - ref).abs().max() / ref.abs().max())
        tf = s.flops / t / 1e12
        attainable = min(pk["bf16_tflops"], s.flops / s.min_bytes * pk["hbm_gbs"] / 1e3)
        rows.append({"id": s.id, "shape": s.name, "M": s.M, "N": s.N, "K": s.K, "plan": gemm_plan(s.M, s.N, s.K, cfg),
                     "us": round(t * 1e6, 2),
                     "TFLOP_s": round(tf, 1), "attainable_TFLOP_s": round(attainable, 1),
                     "frac_attainable": round(tf / attainable, 4), "bound": "tensor" if attainable >= pk["bf16_tflops"]
                     else "hbm", "rel_err": err, "copies": copies})
        del graph, A, B, C
        torch.cuda.empty_cache()
    if rank != 0:
        return None
    main = [r for r in rows if r["M"] > 1]
    gm = math.exp(sum(math.log(r["frac_attainable"]) for r in main) / len(main))
    line = {"metric": "fp16 GEMM sweep, fraction of attainable (geomean, 8 shapes)", "value": round(gm, 4),
            "unit": "fraction", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 in/out, fp32 accumulate",
            "data": "synthetic U(-1, 1)",
            "config": {"workload": "fp16 GEMM sweep (BASELINE config 2) + M=1 rows", "layout": "NN", "cfg": gcfg,
                       "parallelism": f"replicas x{world}", "l2": "operand copies > 2x L2 per shape where needed"},
            "roofline": {"bound": "tensor", "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "peak_source": pk["source"],
                         "achieved": max(r["TFLOP_s"] for r in main),
                         "frac": round(max(r["TFLOP_s"] for r in main) / pk["bf16_tflops"], 4), "traffic": None},
            "rows": rows}
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_gemm_baseline()
    return line


def gemm_plan(M, N, K, cfg=None):
    """The schedule q4b_gemm_f16 runs for an NN problem (q4b_gemm_f16_plan), as a candidate string."""
    import ctypes

    from q4b._lib import GemmCfg, lib
    out = GemmCfg()
    cp = ctypes.byref(GemmCfg(**cfg)) if cfg else None
    if lib().q4b_gemm_f16_plan(M, N, K, b"N", b"N", cp, ctypes.byref(out)) != 0:
        return None
    return f"{out.kernel}:bn={out.bn},stages={out.stages},split={out.split}"


def cpu_gemm_baseline(budget_s=10.0):
    """The reference's Cref computation (gemm/shapes.py:62: A.float() @ B.float()) on the host cores
    for the M = 128 x 5120 x 3072 shape, TFLOP/s."""
    import torch
    torch.manual_seed(0)
    M, N, K = 128, 5120, 3072
    a = torch.rand(M, K) * 2 - 1
    b = torch.rand(K, N) * 2 - 1
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        _ = a.half().float() @ b.half().float()
        times.append(time.perf_counter() - t0)
        if len(times) >= 200:
            break
    med = statistics.median(times)
    return {"value": 2 * M * N * K / med / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(times)} x torch CPU fp32 matmul of fp16-rounded U(-1,1) operands, 128x5120x3072 "
                      f"(median {med * 1e3:.1f} ms)"}


def cpu_sweep_baseline(ms, budget_s=12.0):
    """BASELINE config 5 on the host cores, the reference's two QLinear forms on the q|k|v shape
    (5120 x 3072, g128): M = 1 the fused GEMV (the C restatement, one thread per CPU), M > 1
    dequantize_q4 of the whole weight on every call then a float32 matmul (llama_q4.py:72, numpy).
    GB/s = algorithmic bytes of the timed calls / their time (the sweep's metric)."""
    import numpy as np

    from oracle import q4_cpu as C
    from oracle import q4_oracle as O
    n, k = SWEEP_SHAPES["qkv"]
    rng = np.random.default_rng(5)
    qw = rng.integers(-2**31, 2**31 - 1, size=(n, k // 8), dtype=np.int64).astype(np.int32)
    sc = (np.abs(rng.standard_normal((n, k // 128))) * 0.02).astype(np.float16)
    tot_b, tot_s, done = 0, 0.0, []
    per = budget_s / max(1, len(ms))
    for m in ms:
        x = rng.standard_normal((m, k)).astype(np.float32)
        t_end, calls, t = time.perf_counter() + per, 0, 0.0
        while calls < 2 or (time.perf_counter() < t_end and calls < 200):
            t0 = time.perf_counter()
            if m == 1:
                C.gemv(qw, sc, 128, x[0])
            else:
                x @ O.dequantize_q4(qw, sc, 128).T
            t += time.perf_counter() - t0
            calls += 1
        tot_b += calls * linear_bytes(n, k, m)
        tot_s += t
        done.append(f"M={m}: {calls} calls, {t / calls * 1e3:.2f} ms/call")
    return {"value": round(tot_b / tot_s / 1e9, 3), "unit": "GB/s", "cores": C.threads(), "kind": "port",
            "sample": "q|k|v 5120x3072 g128, " + "; ".join(done)}


def run_sweep(args, rank, world, local, dist_mod):
    """every 3B projection (and the lm_head) at M in {1, 4, 16, 64}, each timed as
    a chain over distinct weight copies, against the HBM roofline; one GPU per rank (replicas)."""
    import torch
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pk = peaks()
    rows, tot_b, tot_s = [], 0, 0.0
    shapes = args.shapes or list(SWEEP_SHAPES)
    cfg = json.loads(args.gemv_cfg) if args.gemv_cfg else None
    for name in shapes:
        n, k = SWEEP_SHAPES[name]
        for m in args.m:
            per_call, copies, *_ = chain_measure(dev, n, k, m, args.steps, args.warmup, cfg=cfg)
            b = linear_bytes(n, k, m)
            gbs = b / per_call / 1e9
            rows.append({"shape": name, "N": n, "K": k, "M": m, "bytes": b, "us_per_call": round(per_call * 1e6, 3),
                         "GB_s": round(gbs, 1), "frac": round(gbs / pk["hbm_gbs"], 4), "weight_copies": copies,
                         "kernel": kernel_of(m, n, k, cfg)})
            tot_b += b
            tot_s += per_call
            torch.cuda.empty_cache()
    if rank != 0:
        return None
    value = world * tot_b / tot_s / 1e9
    return {"metric": "int4 projection sweep GB/s (3B shapes x M)", "value": round(value, 1), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, fp16 x/y, fp32 accumulate",
            "data": "synthetic", "config": {"workload": "batched int4 projection sweep (BASELINE config 5)",
                                            "parallelism": f"replicas x{world}", "cfg": cfg,
                                            "l2": "each row: distinct weight copies > 2x L2"},
            "roofline": {"bound": "hbm", "peak": pk["hbm_gbs"], "unit": "GB/s", "peak_source": pk["source"],
                         "achieved": round(tot_b / tot_s / 1e9, 1),
                         "frac": round(tot_b / tot_s / 1e9 / pk["hbm_gbs"], 4), "traffic": None},
            "rows": rows, "gpu_launches": sum(r["weight_copies"] for r in rows) * args.steps,
            **({} if args.no_cpu_baseline or world > 1 else {"cpu_baseline": cpu_sweep_baseline(args.m)})}


def shard_measure(dev, n, k, m, split, rank, world, dist_mod, comm, steps, warmup, seed=99):
    """Seconds per sharded q4_linear call on this rank (the max over ranks is taken by the caller):
    col = this rank's n/t output rows; row = its k/t slice, then an NCCL all-reduce (sum) of the fp32
    partial y. Every rank holds distinct weight copies of its shard (together > 2x L2), all calls of
    one pass captured in one CUDA graph (the all-reduces too). Returns (seconds, copies, max relative
    error of one assembled y against the unsharded call on this GPU)."""
    import math

    import torch

    import q4b
    from q4b import ops
    from q4b.shard import shard_q4, shard_x
    wbytes = (n * k // 2 + 2 * n * (k // 128)) // world
    copies = max(1, math.ceil(2 * L2_BYTES / wbytes))
    g = torch.Generator(device=dev)
    g.manual_seed(seed)  # the same full weights on every rank; each keeps its shard
    x = torch.randn(m, k, device=dev, generator=g).half()
    xr = shard_x(x, rank, world, split)
    qws, scs = [], []
    err = None
    for c in range(copies):
        qw = torch.randint(-2**31, 2**31 - 1, (n, k // 8), dtype=torch.int32, device=dev, generator=g)
        sc = (torch.randn(n, k // 128, device=dev, generator=g) * 0.02).abs().half()
        a, b = shard_q4(qw, sc, 128, rank, world, split)
        qws.append(a)
        scs.append(b)
        if c == 0:  # parity of the assembled result against the unsharded call
            full = ops.q4_linear(x.float(), qw, sc, 128).float()
            part = ops.q4_linear(xr.float(), a, b, 128).float()
            if split == "col":
                parts = [torch.empty_like(part) for _ in range(world)]
                dist_mod.all_gather(parts, part)
                got = torch.cat(parts, 1)
            else:
                dist_mod.all_reduce(part)
                got = part
            err = float((got - full).abs().max() / full.abs().max().clamp_min(1e-30))
        del qw, sc
    ys = [torch.empty(m, qws[0].shape[0], dtype=torch.float16 if split == "col" else torch.float32, device=dev)
          for _ in range(copies)]
    stream = torch.cuda.Stream(device=dev)
    comm = comm if split == "row" else None  # the library's NCCL communicator (capturable)

    def one_pass():
        for i in range(copies):
            ops.q4_linear(xr, qws[i], scs[i], 128, out=ys[i])
            if comm:
                comm.allreduce(ys[i])

    with torch.cuda.stream(stream):
        one_pass()  # workspace and communicator set up outside the capture
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        graph.capture_begin()
        one_pass()
        graph.capture_end()
        for _ in range(warmup):
            graph.replay()
    stream.synchronize()
    dist_mod.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    dist_mod.barrier()
    if q4b.lib().q4b_device_status(1) != 0:
        raise RuntimeError("q4b: a bounded device wait gave up during the measurement")
    per_call = e0.elapsed_time(e1) / 1e3 / (steps * copies)
    del graph  # graphs holding NCCL calls go before the communicator and the process group
    torch.cuda.synchronize()
    return per_call, copies, err


def run_shard(args, rank, world, local, dist_mod):
    """Row e3: the config-5 projections sharded over the N GPUs, column split (no collective) and row
    split (NCCL all-reduce of y), timed per call as the max over ranks; value = every rank's weight
    bytes / that time (aggregate GB/s)."""
    import torch

    from q4b.shard import shard_ok
    from q4b.tp import TpComm
    if world < 2:
        raise SystemExit("--workload shard needs torchrun with 2 or more ranks")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pk = peaks()
    rows, tot_b, tot_s = [], 0, 0.0
    shapes = args.shapes or list(SWEEP_SHAPES)
    comm = TpComm(rank, world, dist_mod) if "row" in args.splits else None
    for name in shapes:
        n, k = SWEEP_SHAPES[name]
        for m in args.m:
            for split in args.splits:
                if not shard_ok(n, k, 128, world, split):
                    continue
                per_call, copies, err = shard_measure(dev, n, k, m, split, rank, world, dist_mod, comm,
                                                      args.steps, args.warmup)
                t = torch.tensor([per_call, err], dtype=torch.float64, device=dev)
                dist_mod.all_reduce(t, op=dist_mod.ReduceOp.MAX)
                per_call, err = float(t[0]), float(t[1])
                b = linear_bytes(n, k, m)
                gbs = b / per_call / 1e9
                rows.append({"shape": name, "N": n, "K": k, "M": m, "split": split, "bytes": b,
                             "us_per_call": round(per_call * 1e6, 3), "GB_s": round(gbs, 1),
                             "frac_of_world_hbm": round(gbs / (world * pk["hbm_gbs"]), 4), "weight_copies": copies,
                             "max_rel_err_vs_unsharded": err})
                tot_b += b
                tot_s += per_call
                torch.cuda.empty_cache()
    if comm:
        comm.close()
    if rank != 0:
        return None
    worst = max(r["max_rel_err_vs_unsharded"] for r in rows)
    return {"metric": "sharded int4 projection sweep GB/s (3B shapes x M, column / row split)",
            "value": round(tot_b / tot_s / 1e9, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4 weights, fp16 x, fp32 accumulate", "data": "synthetic",
            "config": {"workload": "BASELINE config 5 sharded over GPUs (row e3)", "splits": args.splits,
                       "parallelism": f"tp{world}", "l2": "each rank: distinct shard copies > 2x L2",
                       "collective": "row split: NCCL all-reduce (sum) of fp32 y [M, N], inside the timed call"},
            "roofline": {"bound": "hbm", "peak": round(world * pk["hbm_gbs"], 1), "unit": "GB/s",
                         "peak_source": pk["source"] + f" x {world} GPUs",
                         "achieved": round(tot_b / tot_s / 1e9, 1),
                         "frac": round(tot_b / tot_s / 1e9 / (world * pk["hbm_gbs"]), 4), "traffic": None},
            "parity": {"max_rel_err_vs_unsharded": worst, "bar": 1e-3, "ok": worst <= 1e-3},
            "rows": rows, "gpu_launches": sum(r["weight_copies"] for r in rows) * args.steps}


def run_tiny(args, rank, world, local, dist_mod):
    """the tiny LlamaQ4 (4 layers, hidden 256, 8 / 2 heads, head_dim 32, inter 688,
    vocab 1024) with the reference's own quantised weights and greedy stream
    (tests/golden/model_tiny_baseline.npz, written by tests/golden/make_golden.py from the unmodified
    reference): 64-token prompt, chunk 32, KV buckets {128, 256}, 64 new tokens through the runner
    (bucketed schedule, CUDA graphs). value = decode tokens/s (median over --steps generate calls);
    e2e = the same with the per-step host read; the tokens must equal the reference's; cpu_baseline =
    the oracle's step (numpy) on the same request's decode steps."""
    import statistics
    import sys
    import time

    import numpy as np
    import torch

    import q4b
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import golden_inputs as gi
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    spec = gi.MODEL_SPECS["tiny_baseline"]
    z = dict(np.load(ROOT / "tests" / "golden" / "model_tiny_baseline.npz"))
    model = q4b.LlamaQ4.from_packed(spec["cfg"], z, spec["max_ctx"], vocab_chunk=spec["vocab_chunk"],
                                    max_chunk=spec["chunk"], device=dev)
    prompt, want = z["prompt"].tolist(), z["bucketed_tokens"].tolist()
    runner = q4b.Runner(model, spec["chunk"], spec["buckets"], "bucketed", graphs=True)
    for _ in range(args.warmup):
        runner.generate(prompt, spec["max_new"])
    reps = []
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            toks, rep = runner.generate(prompt, spec["max_new"])
            reps.append(rep)
    same = toks == want
    sync = q4b.Runner(model, spec["chunk"], spec["buckets"], "bucketed", graphs=True, sync_every_step=True)
    sync.generate(prompt, spec["max_new"])
    e2e = [sync.generate(prompt, spec["max_new"])[1]["decode_tok_s"] for _ in range(3)]
    value = statistics.median(r["decode_tok_s"] for r in reps)
    line = {"metric": "tiny LlamaQ4 decode tokens/s (BASELINE config 3)", "value": round(value, 1),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, fp32 activations, fp16 KV cache",
            "data": "the reference's own quantised random-init weights (seed 0) and prompt",
            "config": {"workload": "tiny LlamaQ4 (BASELINE config 3)", "prompt": len(prompt),
                       "new_tokens": spec["max_new"], "chunk": spec["chunk"], "buckets": spec["buckets"],
                       "schedule": "bucketed", "graphs": True,
                       "decode_kernel": "per projection (the tiny shape is below the persistent step's)"},
            "tokens_match_reference": same, "ttft_ms": statistics.median(r["ttft_ms"] for r in reps),
            "e2e": {"value": round(statistics.median(e2e), 1), "unit": "tokens/s", "h2d_bytes_per_step": 104,
                    "d2h_bytes_per_step": 4, "path": "q4b.Runner(sync_every_step=True).generate"},
            "clocks": clk.summary(), "gpu_launches": None}
    if not args.no_cpu_baseline and world == 1:
        from oracle import q4_oracle as O
        layers = [dict(wqkv=(z[f"l{i}_wqkv_qweight"], z[f"l{i}_wqkv_scales"], int(z[f"l{i}_wqkv_group"])),
                       wo=(z[f"l{i}_wo_qweight"], z[f"l{i}_wo_scales"], int(z[f"l{i}_wo_group"])),
                       wgu=(z[f"l{i}_wgu_qweight"], z[f"l{i}_wgu_scales"], int(z[f"l{i}_wgu_group"])),
                       wdown=(z[f"l{i}_wdown_qweight"], z[f"l{i}_wdown_scales"], int(z[f"l{i}_wdown_group"])),
                       ln_in=z[f"l{i}_ln_in"], ln_post=z[f"l{i}_ln_post"]) for i in range(spec["cfg"]["num_hidden_layers"])]
        om = O.OracleModel(spec["cfg"], layers, (z["embed_qweight"], z["embed_scales"], int(z["embed_group"])),
                           z["ln_f"], spec["max_ctx"])
        caches = om.new_caches()
        nxt = None
        for s0 in range(0, len(prompt), spec["chunk"]):
            chunk = np.array(prompt[s0:s0 + spec["chunk"]])
            nxt, _ = om.step(chunk, s0, len(chunk) - 1, caches, 128)
        t0, n, pos = time.perf_counter(), 0, len(prompt)
        while n < spec["max_new"] - 1 and time.perf_counter() - t0 < 20.0:
            nxt, _ = om.step(np.array([nxt]), pos, 0, caches, 128 if pos < 128 else 256)
            pos += 1
            n += 1
        line["cpu_baseline"] = {"value": round(n / (time.perf_counter() - t0), 3), "unit": "tokens/s",
                                "cores": os.cpu_count(), "kind": "port",
                                "sample": f"{n} decode steps of the same request (numpy restatement)"}
    return line


def run_profile(args, rank, world, local, dist_mod):
    """A short fixed launch sequence for profilers: a 3B-shaped model with --layers layers, an optional
    --prefill C chunk at position 0, then --steps single-token decode steps at position --pos."""
    import torch

    import q4b
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = dict(q4b.SYNTHETIC["3b"], num_hidden_layers=args.layers)
    model = q4b.LlamaQ4(None, group=128, max_ctx=max(args.bucket, args.pos + args.steps + 1),
                        sd=q4b.SyntheticStateDict(cfg, device=dev), cfg=cfg, max_chunk=max(8, args.prefill),
                        device=dev)
    caches = model.new_caches()
    if args.prefill:
        toks = torch.arange(args.prefill, dtype=torch.int32).reshape(1, -1) * 7 + 3
        model.step(toks, torch.tensor([0]), torch.tensor([args.prefill - 1]), caches, max(args.bucket, args.prefill))
    tok = torch.tensor([[17]], dtype=torch.int32)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        nxt, _ = model.step(tok, torch.tensor([args.pos + i]), torch.tensor([0]), caches, args.bucket)
        tok = nxt.reshape(1, 1)
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    line = {"metric": "profile sequence (3B shape)", "value": round(ms / args.steps, 4), "unit": "ms/step",
            "higher_is_better": False, "n_gpus": 1, "steps": args.steps, "warmup": 0,
            "config": {"workload": "profile", "layers": args.layers, "pos": args.pos, "bucket": args.bucket,
                       "prefill": args.prefill}, "last_token": int(tok)}
    if args.trace:  # one more step with the phase trace on (after the timed ones)
        buf = model.decode_trace(True)
        model.step(tok, torch.tensor([args.pos + args.steps]), torch.tensor([0]), caches, args.bucket)
        torch.cuda.synchronize()
        line["trace"] = trace_summary(buf.cpu().numpy(), args.layers)
        model.decode_trace(False)
    return line


TRACE_PHASES = ("qkv", "attn", "o", "gate_up", "down")


def trace_summary(ev, n_layers):
    """Phase breakdown of one persistent decode step from its trace (q4b_model_set_trace layout),
    in microseconds, averaged over the layers after the first. Per stage: `wait` = median CTA's
    inputs-ready stamp - the last CTA's end of the previous stage (barrier / partial-sum latency),
    `stage` = median (x staged - inputs ready), `busy` = median (done - x staged), `span` = last end -
    first inputs-ready."""
    import numpy as np
    ev = ev.astype(np.int64)
    L = 15 * n_layers
    ev = ev[ev[:, L + 3] > 0]
    t0 = int(ev[:, L + 3].min())
    keys = ("wait", "stage", "busy", "span")
    out = {p: {k: [] for k in keys} for p in TRACE_PHASES}
    for l in range(1, n_layers):
        prev_end = ev[:, 15 * (l - 1) + 14].max()
        for i, p in enumerate(TRACE_PHASES):
            r, x, d = (ev[:, 15 * l + 3 * i + j] for j in range(3))
            out[p]["wait"].append(float(np.median(r) - prev_end))
            out[p]["stage"].append(float(np.median(x - r)))
            out[p]["busy"].append(float(np.median(d - x)))
            out[p]["span"].append(float(d.max() - r.min()))
            prev_end = d.max()
    res = {p: {k: round(float(np.mean(v)) / 1e3, 3) for k, v in d.items()} for p, d in out.items()} if n_layers > 1 else {}
    res["lm_head"] = {"wait": round(float(np.median(ev[:, L]) - ev[:, L - 1].max()) / 1e3, 3),
                      "stage": round(float(np.median(ev[:, L + 1] - ev[:, L])) / 1e3, 3),
                      "busy": round(float(np.median(ev[:, L + 2] - ev[:, L + 1])) / 1e3, 3)}
    res["layer_us"] = round(float(ev[:, L - 1].max() - ev[:, 14].max()) / 1e3 / max(1, n_layers - 1), 3)
    res["step_us"] = round(float(ev[:, L + 2].max() - t0) / 1e3, 3)
    res["ctas"] = int(ev.shape[0])
    return res


def run_reference(args, rank, world):
    """The reference arm: CPU restatement of the reference path on the host cores (rank 0 only)."""
    if rank != 0:
        return None
    if args.workload == "decode":
        cb = cpu_decode_baseline(steps=args.steps, warmup=args.warmup)
        return {"metric": METRIC_DECODE, "value": round(cb["value"], 4), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "int4 weights, fp32 compute", "data": "synthetic", "impl": "reference",
                "config": {"workload": "Llama-3.2-3B-shape LlamaQ4 batch-1 decode (BASELINE config 4)",
                           "prompt": PROMPT_LEN, "chunk": CHUNK, "buckets": BUCKETS, "decode_bucket": 1024},
                "cpu_baseline": cb,
                "e2e": {"value": round(cb["value"], 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
    if args.workload == "gemv":
        cb = cpu_gemv_baseline(budget_s=min(60.0, 3.0 * (args.steps + args.warmup)))
        return {"metric": METRIC_GEMV, "value": round(cb["value"], 4), "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int4 weights, fp32 compute", "data": "synthetic",
                "impl": "reference",
                "config": {"workload": "int4 GEMV 5120x3072 group 128 M=1 (BASELINE config 1)"},
                "cpu_baseline": cb,
                "e2e": {"value": round(cb["value"], 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
    raise SystemExit(f"unknown workload {args.workload}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="decode: tokens (255); gemv: graph replays (200)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "gemv", "sweep", "shard", "tiny", "profile", "ctx", "gemm"])
    ap.add_argument("--splits", nargs="*", default=["col", "row"], help="shard: column and / or row split")
    ap.add_argument("--ctx", type=int, nargs="*", default=[256, 512, 1024, 2048, 4096], help="ctx: context lengths")
    ap.add_argument("--new", type=int, default=64, help="ctx: generated tokens per run")
    ap.add_argument("--prompts", type=int, default=3, help="ctx: prompts per context length")
    ap.add_argument("--schedules", nargs="*", default=["bucketed", "max"], help="ctx: runner schedules")
    ap.add_argument("--out", default=None, help="ctx: append every run's record (JSON lines) here")
    ap.add_argument("--tag", default="run", help="ctx: tag of the records")
    ap.add_argument("--shapes", nargs="*", default=None, help="sweep: subset of " + " ".join(SWEEP_SHAPES))
    ap.add_argument("--m", nargs="*", type=int, default=[1, 4, 16, 64], help="sweep: rows of x")
    ap.add_argument("--layers", type=int, default=1, help="profile: layers of the 3B-shaped model")
    ap.add_argument("--pos", type=int, default=128, help="profile: position of the first decode step")
    ap.add_argument("--bucket", type=int, default=256, help="profile: KV bucket of the decode steps")
    ap.add_argument("--prefill", type=int, default=0, help="profile: rows of one prefill chunk run first")
    ap.add_argument("--trace", action="store_true", help="profile: phase trace of one more decode step")
    ap.add_argument("--no-gemv", action="store_true", help="decode: skip the config-1 GEMV sub-measurement")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--gemv-cfg", default=None, help='JSON q4b_linear_cfg, e.g. {"warps":4,"tiles":2}')
    ap.add_argument("--gemm-cfg", default=None, help='gemm: JSON q4b_gemm_cfg for every shape, e.g. {"kernel":3}')
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3 and args.workload != "profile":
        args.warmup = 3
    if args.steps is None:
        args.steps = {"decode": 255, "gemv": 200, "sweep": 20, "shard": 20, "tiny": 10, "profile": 3, "ctx": 0,
                      "gemm": 20}[args.workload]
    rank, world, local = dist_env()
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line:
            print(json.dumps(line), flush=True)
        return
    dist_mod = init_dist(world, local)
    try:
        run = {"decode": run_decode, "gemv": run_gemv, "sweep": run_sweep, "shard": run_shard, "tiny": run_tiny,
               "profile": run_profile, "ctx": run_ctx, "gemm": run_gemm}[args.workload]
        line = run(args, rank, world, local, dist_mod)
    finally:
        if dist_mod:
            dist_mod.barrier()
            dist_mod.destroy_process_group()
    if line:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
