"""CARM hardware parameters of one B200, measured (no datasheet values).

Port of profiling/portable/measure_params.py (cache-barrier): the same six
parameters, timed the same way (CUDA graphs, median of replays), with the
W4A16 dequant throughput measured on this repository's sm_100a kernel through
the drop-in ``bench_l2_barrier.batched_int4_gemm`` instead of the Triton one.

  t0_graph_us   per-launch fixed cost of a tiny bmm under CUDA graphs (:57-60)
  t0_eager_us   the same launched eagerly (:63-78)
  bw_l2_tbs     L2-resident re-read bandwidth, differential slope of a
                sum-reduce between 0.15 and 0.55 x nominal L2 (:45-55)
  bw_hbm_tbs    DRAM re-read bandwidth, slope between 3 and 6 x nominal L2
  peak_tflops   fp16 tensor-core throughput of cuBLAS on large square GEMMs (:81-91)
  effective_l2_capacity_mb   residency cliff of the warm re-read bandwidth
                between 0.4 and 1.5 x nominal L2 (:94-117)
  r_dequant_tbs packed-int4 bytes/s of the W4A16 GEMM at the decode shape
                H = 128, K = 128, T = 1, differential over N = 256 -> 512 (:120-142)

    python cache-barrier_b200/harness/measure_params.py --out params_b200.json
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from common import ClockSampler, gpu_info, graph_time_us, save_json  # noqa: E402

import torch  # noqa: E402

DEV = "cuda"


def read_bw(mb: float):
    x = torch.randn(int(mb * 2**20 // 4), dtype=torch.float32, device=DEV)
    us = graph_time_us(lambda: x.sum(), inner=12)
    del x
    torch.cuda.empty_cache()
    return mb * 2**20 / (us * 1e-6) / 1e12, us


def diff_bw(mb_small: float, mb_large: float) -> float:
    _, ts = read_bw(mb_small)
    _, tl = read_bw(mb_large)
    return (mb_large - mb_small) * 2**20 / ((tl - ts) * 1e-6) / 1e12


def t0_graph() -> float:
    x = torch.randn(8, 1, 64, dtype=torch.float16, device=DEV)
    w = torch.randn(8, 64, 16, dtype=torch.float16, device=DEV)
    return graph_time_us(lambda: torch.bmm(x, w), inner=20)


def t0_eager() -> float:
    x = torch.randn(8, 1, 64, dtype=torch.float16, device=DEV)
    w = torch.randn(8, 64, 16, dtype=torch.float16, device=DEV)
    for _ in range(50):
        torch.bmm(x, w)
    torch.cuda.synchronize()
    ts = []
    for _ in range(200):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        torch.bmm(x, w)
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e) * 1e3)
    return statistics.median(ts)


def peak_tflops() -> float:
    best = 0.0
    for m, k, n in ((8192, 8192, 8192), (4096, 16384, 8192), (16384, 8192, 8192)):
        a = torch.randn(m, k, dtype=torch.float16, device=DEV)
        b = torch.randn(k, n, dtype=torch.float16, device=DEV)
        c = torch.empty(m, n, dtype=torch.float16, device=DEV)
        us = graph_time_us(lambda: torch.matmul(a, b, out=c), inner=5, reps=20)
        best = max(best, 2.0 * m * k * n / (us * 1e-6) / 1e12)
        del a, b, c
        torch.cuda.empty_cache()
    return best


def c_eff(l2_mb: float):
    lo, hi = 0.4 * l2_mb, 1.5 * l2_mb
    sizes = [lo + i * (hi - lo) / 13 for i in range(14)]
    pts = [(mb, read_bw(mb)[0]) for mb in sizes]
    run_max, m_max, cliff = 0.0, None, None
    for m, b in pts:
        if b > run_max:
            run_max, m_max = b, m
        elif b < 0.95 * run_max:
            cliff = (m_max + m) / 2
            break
    return cliff, [(round(m, 1), round(b, 3)) for m, b in pts]


# One token per batch entry runs the W4A16 dp4a GEMV (exact int4 weights, 15-bit
# fixed-point activations, per-channel scale on the fp32 sum).
R_DEQUANT_KERNEL = "cb200 w4a16_gemv_kernel (dp4a), per-channel scales, T=1"


def r_dequant():
    import bench_l2_barrier as B

    H, K = 128, 128
    times = {}
    for n in (256, 512):
        x = torch.randn(H, 1, K, dtype=torch.float16, device=DEV)
        w = torch.randn(H, K, n, dtype=torch.float16, device=DEV)
        wp, sc = B.quantize_weights_int4(w)
        B.batched_int4_gemm(x, wp, sc, K, BLOCK_M=16)  # repacks once, outside capture
        times[n] = graph_time_us(lambda: B.batched_int4_gemm(x, wp, sc, K, BLOCK_M=16))
        del x, w, wp, sc
        torch.cuda.empty_cache()
    d_packed = H * K * (512 - 256) // 2
    return d_packed / ((times[512] - times[256]) * 1e-6) / 1e12, {str(k): round(v, 3) for k, v in times.items()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=None)
    ap.add_argument("--only", choices=["all", "r_dequant"], default="all",
                    help="r_dequant: re-measure only the dequant rate and update it in --out")
    args = ap.parse_args()
    torch.manual_seed(0)
    info = gpu_info()
    if args.only == "r_dequant":
        p = {}
        if args.out and os.path.exists(args.out):
            with open(args.out) as f:
                p = json.load(f)
        with ClockSampler(0) as clk:
            rd, rd_times = r_dequant()
        p.update({"r_dequant_tbs": round(rd, 4), "r_dequant_times_us": rd_times, "r_dequant_clocks": clk.info,
                  "r_dequant_kernel": R_DEQUANT_KERNEL})
        print(f"  r_dequant_tbs: {p['r_dequant_tbs']}  times {rd_times}", flush=True)
        if args.out:
            save_json(args.out, p)
        return
    l2 = torch.cuda.get_device_properties(0).L2_cache_size / 2**20
    print(info, flush=True)
    with ClockSampler(0) as clk:
        p = {"t0_graph_us": round(t0_graph(), 3), "t0_eager_us": round(t0_eager(), 3)}
        p["bw_l2_tbs"] = round(diff_bw(0.15 * l2, 0.55 * l2), 3)
        p["bw_hbm_tbs"] = round(diff_bw(3 * l2, 6 * l2), 3)
        p["peak_tflops"] = round(peak_tflops(), 1)
        ce, curve = c_eff(l2)
        p["effective_l2_capacity_mb"] = round(ce, 1) if ce else None
        p["c_eff_curve_mb_tbs"] = curve
        rd, rd_times = r_dequant()
        p["r_dequant_tbs"] = round(rd, 4)
        p["r_dequant_times_us"] = rd_times
    p.update({"gpu": info, "nominal_l2_mb": round(l2, 1), "clocks": clk.info,
              "r_dequant_kernel": R_DEQUANT_KERNEL})
    for k, v in p.items():
        if k not in ("c_eff_curve_mb_tbs",):
            print(f"  {k}: {v}", flush=True)
    if args.out:
        save_json(args.out, p)


if __name__ == "__main__":
    main()
