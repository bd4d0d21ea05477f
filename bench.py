#!/usr/bin/env python
"""Headline benchmark: W8A8 INT8 decode GEMM on B200 (sm_100a).

Workload (the reference's W8A8 configuration): K = N = 8192 int8 weights
(64 MiB, uniform in [-127, 127]) with fp32 per-channel scales |N(0, 0.01)|,
bf16 activations N(0, 1) dynamically quantized per token inside the timed
region, T in {1, 8, 16, 32}, int32 accumulation, bf16 output.

One step = 32 passes over T = 1, 8, 16, 32 (128 GEMMs, each an activation-
quantization launch plus a GEMM launch), captured once in a CUDA graph and
replayed, as the reference times its kernels (10-launch graphs, median of
replays). Weights rotate over 4 copies (256 MiB > the 126 MB L2), so every GEMM
streams its weights from HBM ("L2-flushed" by rotation, as in the reference's
rotated variant).

Reported (one JSON line from rank 0):
  value      us per GEMM for the whole job (all ranks' GEMMs / max-over-ranks time)
  e2e        the same metric through the library's C-ABI call with host buffers
             (cb_exec_w8a8_dynamic_host): pinned activations copied in and fp16
             outputs copied out every GEMM, the copies overlapped with the
             neighbouring GEMMs; beside it the eager Python drop-in
             (w8a8_bmm_full + torch copies) on the same work
  roofline   the GEMM kernel alone: algorithmic bytes per launch / CUDA-event time
  cpu_baseline  the oracle's restatement of the reference's CPU path (rank 0, N = 1)
plus the cuBLAS bf16 comparison (dequantized weights, same rotation), W4A16
group-128 and NVFP4 (block-scaled FP4 tensor cores) measurements of the same shape,
and (the ``tp`` object) the tensor-parallel decode step of a 64-layer dense
decoder's projections at tp = N: us per layer for W8A8, W4A16 and bf16, the
all-reduce's share (NCCL and the one-shot NVLink all-reduce), weight GB/s per
GPU, and the per-GPU projection shards on either side of the capacity gate.
The headline ``value`` stays the per-GPU W8A8 workload at every N (replicas),
so the metric is the same for every N.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--tp on|off]
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cache-barrier_b200"))
sys.path.insert(0, os.path.join(ROOT, "cache-barrier_b200", "dropin"))

METRIC = "µs/GEMM, achieved HBM TB/s and speedup vs cuBLAS bf16 over W×T gate sweep"
UNIT = "us/GEMM"
K_DIM = N_DIM = 8192
TOKENS = (1, 8, 16, 32)
COPIES = 4
CYCLES = 32  # passes over TOKENS per step
W4_COPIES = 8
GROUP = 128
TP_TOKENS = (1, 8, 32, 64)
TP_PRECISIONS = ("w8a8", "w4a16", "bf16")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="cb200", choices=["cb200", "reference"])
    ap.add_argument("--tp", default="on", choices=["on", "off"],
                    help="also time the tensor-parallel dense decode step at tp = N (the 'tp' object)")
    return ap.parse_args()


def _env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML, the library behind nvidia-smi)
# ---------------------------------------------------------------------------
_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    def __init__(self, device_index: int, period_s: float = 0.01):
        self.period = period_s
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.error = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001
            self._nvml = None
            self.error = f"nvml unavailable: {e}"

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception as e:  # noqa: BLE001
                self.error = str(e)
                return
            time.sleep(self.period)

    def start(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
        names = sorted(name for bit, name in _REASONS.items() if self.reasons & bit and name != "gpu_idle")
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
               "reasons": names, "samples": len(self.samples)}
        if self.error:
            out["note"] = self.error
        return out


# ---------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------
def capture(fn):
    import torch
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def time_replays(g, steps, warmup):
    """ms per replay: CUDA events on the current stream, synchronize on both sides."""
    import torch
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / steps


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def committed_traffic(name):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary (profiles/*.json), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def w8a8_bytes(T):
    return K_DIM * N_DIM + 4 * N_DIM + T * K_DIM + 4 * T + 2 * T * N_DIM


def nvfp4_bytes(T):
    """Packed e2m1 weights and activations with their e4m3 scales (one per 16), bf16 out."""
    return K_DIM * N_DIM // 2 + K_DIM * N_DIM // 16 + T * K_DIM // 2 + T * K_DIM // 16 + 2 * T * N_DIM


def w4a16_bytes(T):
    return K_DIM * N_DIM // 2 + (K_DIM // GROUP) * N_DIM * 2 + 2 * T * K_DIM + 2 * T * N_DIM


# ---------------------------------------------------------------------------
# reference arm: the oracle's CPU restatement of the reference's path
# ---------------------------------------------------------------------------
def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle import cpu_baseline as CB
    ctl, cores = CB.blas_threads()
    path = CB.W8A8Cpu(K_DIM, N_DIM, seed=0)
    acts = {T: path.acts(T) for T in TOKENS}
    for _ in range(max(args.warmup, 1)):
        for T in TOKENS:
            path.gemm(acts[T])
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for T in TOKENS:
            path.gemm(acts[T])
    dt = time.perf_counter() - t0
    us = dt * 1e6 / (args.steps * len(TOKENS))
    line = {
        "metric": METRIC, "value": round(us, 2), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 3), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "i8", "data": "synthetic", "impl": "reference",
        "config": {"workload": "W8A8 INT8 GEMM K=N=8192, T in {1,8,16,32}, dynamic per-token act quant, bf16 out",
                   "step": "one pass over T = 1, 8, 16, 32 (4 GEMMs) on the host cores"},
        "cpu_baseline": {"value": round(us, 2), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{args.steps} steps x 4 GEMMs (T=1,8,16,32), K=N=8192, numpy/BLAS fp64 exact "
                                   "int GEMM + per-token quant + fp32 epilogue"},
        "e2e": {"value": round(us, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    del ctl


# ---------------------------------------------------------------------------
# cb200 arm
# ---------------------------------------------------------------------------
def main():
    args = parse_args()
    rank = _env_int("RANK", 0)
    world = _env_int("WORLD_SIZE", 1)
    local = _env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    from cb200 import ops
    import w8a8_bmm  # reference-facing drop-in (e2e path)

    # ---------------- inputs (seeded on the host, resident in HBM) ----------------
    gen = torch.Generator().manual_seed(1234 + rank)
    gdev = torch.Generator(device=dev).manual_seed(4321 + rank)
    w_nk, w_kn_views = [], []
    for _ in range(COPIES):
        wq = torch.randint(-127, 128, (K_DIM, N_DIM), generator=gdev, dtype=torch.int8, device=dev)
        nk = ops.repack_w8_kmajor(wq)
        w_nk.append(nk)
        w_kn_views.append(nk.t())  # the reference's [K, N] view of K-major storage
        del wq
    w_scale = ((torch.randn(N_DIM, generator=gen) * 0.01).abs() + 1e-4).float().to(dev)
    acts = {T: torch.randn(T, K_DIM, generator=gen).to(torch.bfloat16).to(dev) for T in TOKENS}
    qbuf = {T: torch.empty(T, K_DIM, dtype=torch.int8, device=dev) for T in TOKENS}
    sbuf = {T: torch.empty(T, dtype=torch.float32, device=dev) for T in TOKENS}
    obuf = {T: torch.empty(T, N_DIM, dtype=torch.bfloat16, device=dev) for T in TOKENS}

    # A step is CYCLES GEMMs at each token count, grouped by T as a decode step
    # runs them (every layer of one step has the same T; the reference's gate
    # harness likewise times each (W, T) cell as a graph of one shape), with the
    # weights rotating over COPIES copies from one GEMM to the next.
    def step_dynamic():
        for T in TOKENS:
            for c in range(CYCLES):
                ops.w8a8_gemm_dynamic(acts[T], w_nk[c % COPIES], w_scale, q=qbuf[T], s=sbuf[T], out=obuf[T])

    def step_gemm_only():
        for T in TOKENS:
            for c in range(CYCLES):
                ops.w8a8_gemm(qbuf[T], w_nk[c % COPIES], sbuf[T], w_scale, out=obuf[T])

    g_dyn = capture(step_dynamic)
    g_mm = capture(step_gemm_only)
    assert ops.device_status(dev) == 0

    # ---------------- headline: timed steps (max over ranks) ----------------
    for _ in range(args.warmup):
        g_dyn.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record()
    for _ in range(args.steps):
        g_dyn.replay()
    t_end.record()
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    ms_total = t_start.elapsed_time(t_end)
    if world > 1:
        t = torch.tensor([ms_total], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
        dist.barrier()
    torch.cuda.synchronize()
    gemms_per_step = CYCLES * len(TOKENS)
    ms_per_step = ms_total / args.steps
    us_per_gemm_job = ms_total * 1e3 / (args.steps * gemms_per_step * world)
    us_per_gemm_gpu = ms_total * 1e3 / (args.steps * gemms_per_step)

    # ---------------- GEMM kernel alone (roofline) ----------------
    kernel_steps = max(args.steps // 2, 10)
    ms_mm = time_replays(g_mm, kernel_steps, args.warmup)
    us_kernel = ms_mm * 1e3 / gemms_per_step
    alg_bytes = statistics.mean(w8a8_bytes(T) for T in TOKENS)
    achieved_gbs = alg_bytes / (us_kernel * 1e-6) / 1e9
    peaks, peak_src = measured_peaks()
    traffic = committed_traffic("w8a8_gemm_k8192_n8192.json")
    traffic_gemv = committed_traffic("w8a8_gemv_k8192_n8192_t1.json")

    # per-T kernel time (graph of CYCLES launches of one T)
    per_t = {}
    for i, T in enumerate(TOKENS):
        def one_t(T=T, i=i):
            for c in range(CYCLES):
                ops.w8a8_gemm(qbuf[T], w_nk[c % COPIES], sbuf[T], w_scale, out=obuf[T])
        g = capture(one_t)
        per_t[T] = time_replays(g, 10, 2) * 1e3 / CYCLES
        del g

    # ---------------- cuBLAS bf16 on the dequantized weights ----------------
    w_deq = [(wn.float() * w_scale[:, None]).to(torch.bfloat16) for wn in w_nk]  # [N, K], K contiguous
    cub_out = {T: torch.empty(T, N_DIM, dtype=torch.bfloat16, device=dev) for T in TOKENS}

    def cublas_one_t(T):
        def f():
            for c in range(CYCLES):
                torch.mm(acts[T], w_deq[c % COPIES].t(), out=cub_out[T])
        return f

    cub_t = {}
    for T in TOKENS:
        g = capture(cublas_one_t(T))
        cub_t[T] = time_replays(g, 10, 2) * 1e3 / CYCLES
        del g
    cub_mean = statistics.mean(cub_t.values())

    # ---------------- e2e: C-ABI call with host buffers ----------------
    # cb_exec_w8a8_dynamic_host per GEMM: pinned activations copied in, act-quant
    # + GEMM, fp16 result (w8a8_bmm_full's dtype) copied back into pinned host
    # memory; the executor overlaps each call's copies with its neighbours'
    # kernels. Timed with CUDA events on this stream, joined to the executor's.
    host_in = {T: acts[T].cpu().pin_memory() for T in TOKENS}
    host_out = {T: torch.empty(T, N_DIM, dtype=torch.float16).pin_memory() for T in TOKENS}
    ex = ops.HostExecutor(dev)

    def e2e_step():
        for T in TOKENS:
            for c in range(CYCLES):
                ex.w8a8_dynamic_host(host_in[T], w_nk[c % COPIES], w_scale, host_out[T])

    def time_host(step_fn, n_steps, join):
        for _ in range(max(1, args.warmup)):
            step_fn()
        torch.cuda.synchronize()
        if join:
            ex.synchronize()
        if world > 1:
            dist.barrier()
        es = torch.cuda.Event(enable_timing=True)
        ee = torch.cuda.Event(enable_timing=True)
        es.record()
        if join:
            ex.after()
        for _ in range(n_steps):
            step_fn()
        if join:
            ex.before()
        ee.record()
        torch.cuda.synchronize()
        ms = es.elapsed_time(ee)
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms * 1e3 / (n_steps * gemms_per_step * world)

    e2e_steps = max(1, min(args.steps, 50))
    e2e_us = time_host(e2e_step, e2e_steps, join=True)
    assert ex.synchronize() == 0
    # the host-buffer results are the device path's, bit for bit
    for i, T in enumerate(TOKENS):
        ref16 = ops.w8a8_gemm_dynamic(acts[T], w_nk[i % COPIES], w_scale, out_dtype=torch.float16)
        ex.w8a8_dynamic_host(host_in[T], w_nk[i % COPIES], w_scale, host_out[T])
        ex.synchronize()
        assert torch.equal(host_out[T], ref16.cpu()), f"host-buffer path differs at T={T}"
    h2d = sum(T * K_DIM * 2 for T in TOKENS) * CYCLES
    d2h = sum(T * N_DIM * 2 for T in TOKENS) * CYCLES

    # the same work through the eager Python drop-in (w8a8_bmm_full on device
    # tensors, torch copies from / to pinned host memory), for comparison
    dev_in = {T: torch.empty(1, T, K_DIM, dtype=torch.bfloat16, device=dev) for T in TOKENS}
    dev_out = {T: torch.empty(1, T, N_DIM, dtype=torch.float16, device=dev) for T in TOKENS}
    q3 = {T: torch.empty(1, T, K_DIM, dtype=torch.int8, device=dev) for T in TOKENS}
    ws3 = w_scale.view(1, N_DIM)
    wviews = [v.unsqueeze(0) for v in w_kn_views]

    def dropin_step():
        for T in TOKENS:
            for c in range(CYCLES):
                dev_in[T][0].copy_(host_in[T], non_blocking=True)
                w8a8_bmm.w8a8_bmm_full(dev_in[T], wviews[c % COPIES], ws3, bufs=(q3[T], sbuf[T], dev_out[T]))
                host_out[T].copy_(dev_out[T][0], non_blocking=True)

    dropin_us = time_host(dropin_step, e2e_steps, join=False)
    ex.close()

    # ---------------- W4A16 group-128, same shape ----------------
    w4 = None
    try:
        from cb200 import _lib as L
        gen4 = torch.Generator(device=dev).manual_seed(99 + rank)
        natives = []
        for _ in range(W4_COPIES):
            # uniform bytes = two int4 values uniform in [-8, 7], reference layout uint8 [K/2, N]
            packed = torch.randint(0, 256, (K_DIM // 2, N_DIM), generator=gen4, dtype=torch.uint8, device=dev)
            natives.append(ops.repack_w4(packed, L.CB_W4_REF_U8_KN, K_DIM, N_DIM))
            del packed
        s4 = ((torch.randn(K_DIM // GROUP, N_DIM, generator=gen4, device=dev) * 0.02).abs() / 7
              + 1e-4).to(torch.bfloat16)
        o4 = {T: torch.empty(T, N_DIM, dtype=torch.bfloat16, device=dev) for T in TOKENS}
        w4_t = {}
        for T in TOKENS:
            def f(T=T):
                for c in range(CYCLES):
                    ops.w4a16_gemm(acts[T], natives[c % W4_COPIES], s4, N_DIM, GROUP, out=o4[T])
            g = capture(f)
            w4_t[T] = time_replays(g, 10, 2) * 1e3 / CYCLES
            del g
        w4_mean = statistics.mean(w4_t.values())
        w4_bytes = statistics.mean(w4a16_bytes(T) for T in TOKENS)
        w4 = {"us_per_gemm": round(w4_mean, 3), "per_token_us": {str(T): round(v, 3) for T, v in w4_t.items()},
              "achieved_gbs": round(w4_bytes / (w4_mean * 1e-6) / 1e9, 1),
              "frac_of_measured_hbm": round(w4_bytes / (w4_mean * 1e-6) / 1e9 / peaks["hbm_gbs"], 3),
              "speedup_vs_cublas_bf16": round(cub_mean / w4_mean, 3),
              "config": f"K=N=8192 int4 g128 bf16 scales, {W4_COPIES} rotating copies (264 MiB > L2), bf16 acts/out"}
        assert ops.device_status(dev) == 0
    except Exception as e:  # noqa: BLE001
        w4 = {"error": repr(e)}

    # ---------------- NVFP4 W4A4 (e2m1 + e4m3 block scales), same shape ----------------
    fp4 = None
    try:
        gen5 = torch.Generator(device=dev).manual_seed(77 + rank)
        fp4_w = []
        for _ in range(COPIES):
            wb = (torch.randn(N_DIM, K_DIM, generator=gen5, device=dev) / K_DIM ** 0.5).to(torch.bfloat16)
            gw = torch.tensor([448.0 * 6.0 / float(wb.float().abs().max())], device=dev)
            fq, fsf = ops.nvfp4_quantize(wb, gw)
            fp4_w.append((fq, fsf, gw))
            del wb
        fo = {T: torch.empty(T, N_DIM, dtype=torch.bfloat16, device=dev) for T in TOKENS}
        fp4_t, fp4_dyn_t = {}, {}
        for T in TOKENS:
            gx = torch.tensor([448.0 * 6.0 / float(acts[T].float().abs().max())], device=dev)
            qx, sx = ops.nvfp4_quantize(acts[T], gx)
            alphas = [(1.0 / (gx * gw)).float() for (_, _, gw) in fp4_w]

            def f(T=T, qx=qx, sx=sx, alphas=alphas):
                for c in range(CYCLES):
                    ops.nvfp4_gemm(qx, sx, fp4_w[c % COPIES][0], fp4_w[c % COPIES][1], alphas[c % COPIES],
                                   out=fo[T])

            def fd(T=T, qx=qx, sx=sx, alphas=alphas, gx=gx):
                for c in range(CYCLES):
                    ops.nvfp4_quantize(acts[T], gx, q=qx, sf=sx)
                    ops.nvfp4_gemm(qx, sx, fp4_w[c % COPIES][0], fp4_w[c % COPIES][1], alphas[c % COPIES],
                                   out=fo[T])
            for fn, dst in ((f, fp4_t), (fd, fp4_dyn_t)):
                g = capture(fn)
                dst[T] = time_replays(g, 10, 2) * 1e3 / CYCLES
                del g
        fmean = statistics.mean(fp4_t.values())
        fdyn = statistics.mean(fp4_dyn_t.values())
        fbytes = statistics.mean(nvfp4_bytes(T) for T in TOKENS)
        fp4 = {"us_per_gemm": round(fmean, 3), "per_token_us": {str(T): round(v, 3) for T, v in fp4_t.items()},
               "us_per_gemm_with_act_quant": round(fdyn, 3),
               "achieved_gbs": round(fbytes / (fmean * 1e-6) / 1e9, 1),
               "frac_of_measured_hbm": round(fbytes / (fmean * 1e-6) / 1e9 / peaks["hbm_gbs"], 3),
               "speedup_vs_cublas_bf16": round(cub_mean / fmean, 3),
               "speedup_vs_cublas_bf16_with_act_quant": round(cub_mean / fdyn, 3),
               "config": f"K=N=8192 NVFP4 (vLLM formats: e2m1 + e4m3 scales per 16, amax global scales), "
                         f"{COPIES} rotating copies (144 MiB > L2), bf16 acts/out"}
        assert ops.device_status(dev) == 0
    except Exception as e:  # noqa: BLE001
        fp4 = {"error": repr(e)}

    # ---------------- tensor-parallel dense decode at tp = N ----------------
    # 64-layer 27B-class decoder projections (QKV and gate-up column-parallel, O
    # and down row-parallel, each followed by an all-reduce of [T, 5120] bf16),
    # one CUDA graph per decode step, max over ranks; NCCL and the one-shot
    # NVLink all-reduce both measured at N > 1.
    tp = None
    if args.tp == "on":
        try:
            sys.path.insert(0, os.path.join(ROOT, "cache-barrier_b200", "harness"))
            import dense_tp

            del g_dyn, g_mm
            g_dyn = g_mm = None
            torch.cuda.empty_cache()
            logf = (lambda m: print(m, file=sys.stderr, flush=True)) if rank == 0 else (lambda m: None)
            _rows, _prows, summary = dense_tp.measure(world, rank, dev, TP_TOKENS, TP_PRECISIONS,
                                                      ["nccl", "peer"], steps=10, warmup=3, log=logf)
            tp = {"workload": "dense 27B-class decoder projections, 64 layers, hidden 5120, 40 q + 8 kv heads of "
                              "128, FFN 17408; QKV/gate-up column-parallel, O/down row-parallel + all-reduce; "
                              "W8A8 per-channel int8, W4A16 g128 int4, bf16 cuBLAS; random N(0, 0.02) weights",
                  "timing": "one CUDA graph per decode step, 10 replays after 3 warm-up, max over ranks; "
                            "per-projection: a graph of one projection's GEMM in all 64 layers",
                  **summary}
            assert ops.device_status(dev) == 0
        except Exception as e:  # noqa: BLE001
            tp = {"error": repr(e)}

    # ---------------- CPU baseline (rank 0, N = 1) ----------------
    cpu = None
    if world == 1 and rank == 0:
        from oracle import cpu_baseline as CB
        ctl, cores = CB.blas_threads()
        path = CB.W8A8Cpu(K_DIM, N_DIM, seed=0)
        mean_s, per = CB.time_path(path, TOKENS, reps=3, warmup=1)
        cpu = {"value": round(mean_s * 1e6, 1), "unit": UNIT, "cores": cores, "kind": "port",
               "sample": "T=1,8,16,32 x 3 timed reps each (median), K=N=8192: per-token quant, exact int GEMM "
                         "(numpy fp64 BLAS), fp32 epilogue, bf16 cast"}
        # the W4A16 CPU configuration: T=16, K=N=4096, int4 g128 bf16 scales, explicit dequant + matmul
        p4 = CB.W4A16Cpu(4096, 4096, 128, seed=0)
        m4, _ = CB.time_path(p4, [16], reps=5, warmup=1)
        if isinstance(w4, dict) and "error" not in w4:
            w4["cpu_baseline"] = {"value": round(m4 * 1e6, 1), "unit": UNIT, "cores": cores, "kind": "port",
                                  "sample": "T=16, K=N=4096 int4 g128: explicit dequant (part of the timed path) "
                                            "+ fp32 matmul + bf16 cast, median of 5"}
        del ctl

    assert ops.device_status(dev) == 0
    if world > 1:
        dist.barrier()
        del g_dyn, g_mm
        dist.destroy_process_group()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(us_per_gemm_job, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "i8",
            "data": "synthetic",
            "config": {
                "workload": "W8A8 INT8 GEMM K=N=8192, T in {1,8,16,32}, dynamic per-token act quant, int32 acc, "
                            "bf16 out (replicas: each GPU runs the full workload)",
                "step": f"{CYCLES} GEMMs at each of T=1,8,16,32, grouped by T as a decode step runs them, = "
                        f"{gemms_per_step} GEMMs (act-quant + GEMM launches), one CUDA graph replay",
                "l2": f"inputs larger than L2: consecutive GEMMs read different weight copies ({COPIES} copies, "
                      "256 MiB)",
                "parallelism": f"replicas x{world} (headline); tensor parallel tp={world} (the tp object)",
            },
            "us_per_gemm_per_gpu": round(us_per_gemm_gpu, 3),
            "per_token_kernel_us": {str(T): round(v, 3) for T, v in per_t.items()},
            "achieved_hbm_tbs": round(achieved_gbs / 1e3, 3),
            "cublas_bf16_us_per_gemm": round(cub_mean, 3),
            "cublas_bf16_per_token_us": {str(T): round(v, 3) for T, v in cub_t.items()},
            "speedup_vs_cublas_bf16": round(cub_mean / us_per_gemm_gpu, 3),
            "kernel_speedup_vs_cublas_bf16": round(cub_mean / us_kernel, 3),
            "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved_gbs / peaks["hbm_gbs"], 4),
                         "peak_source": f"{peak_src} MEASURED_PEAKS.json hbm_gbs" if peak_src == "measured"
                         else "fallback 6.65 TB/s",
                         "kernel": "w8a8_gemm_kernel (tcgen05 kind::i8) at T = 8/16/32, "
                                   "w8a8_gemv_kernel (dp4a) at T = 1",
                         "alg_bytes_per_launch": int(alg_bytes), "us_per_launch": round(us_kernel, 3),
                         "traffic": (traffic or {}).get("dram_bytes_per_launch"),
                         "traffic_by_kernel": {
                             "w8a8_gemm_kernel (T=16 capture)": (traffic or {}).get("dram_bytes_per_launch"),
                             "w8a8_gemv_kernel (T=1 capture)": (traffic_gemv or {}).get("dram_bytes_per_launch")}},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_us, 3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "cb_exec_w8a8_dynamic_host (C ABI, pinned host activations in and fp16 results out "
                           "per GEMM; copies overlapped with the neighbouring GEMMs on the executor's streams)",
                    "dropin_eager_us_per_gemm": round(dropin_us, 3),
                    "dropin_eager_api": "w8a8_bmm.w8a8_bmm_full + torch copies, eager Python"},
            "gpu_launches": args.steps * gemms_per_step * 2,  # timed region: act-quant + GEMM per GEMM
            "clocks": clock_info,
            "w4a16": w4,
            "nvfp4": fp4,
            "tp": tp,
        }
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
