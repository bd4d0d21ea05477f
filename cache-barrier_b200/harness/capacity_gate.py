"""Capacity-gate 2D sweep on one B200: weight working set W x tokens T, three precisions.

Port of profiling/gate/bench_capacity_gate.py (cache-barrier) to the sm_100a
kernels. Two shape families:

  square (default)  K = N with bf16-equivalent weight bytes W = 2*K*N in
                    {8, 16, ..., 1024} MB plus 8 MB steps around the measured
                    effective L2 capacity C_eff; W4A16 with g128 scales
                    (dense_ops.quantize_w4a16 / apply_w4a16_linear), W8A8 with
                    dynamic per-token act quant inside the timed region
                    (ops.w8a8_gemm_dynamic), NVFP4 W4A4 on the block-scaled
                    FP4 tensor cores with the activations quantized per call
                    (ops.nvfp4_quantize + ops.nvfp4_gemm; the reference's
                    matched-precision path, profiling/cuda_validation/
                    bench_moe_nvfp4_native.py), bf16 cuBLAS torch.mm.
  bmm               the reference's batched family H = 128, K = 128,
                    N = 32 * W_MB (bench_capacity_gate.py:80-83), driven
                    through the drop-in names exactly as the reference harness
                    calls them (kernel_batched_w4a16_simple[grid](...),
                    quantize_acts_w8 + w8a8_bmm, torch.bmm).

Each cell is timed L2-hot (the same weights every launch, as the reference's
warm loop) and L2-flushed (launch i reads copy i % R, R >= 2*C_eff/bytes + 1
copies, as profiling/dense_qwen/bench_l2_boundary.py:50). CUDA-graph timing,
10 launches per graph, median of 20 replays. Speedups are bf16 time / quantized
time of the same variant; the gate is the smallest W at which a precision
beats bf16 for that T.

    python cache-barrier_b200/harness/capacity_gate.py --params params_b200.json --out gate.json
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from common import ClockSampler, gpu_info, graph_time_us_indexed, save_json  # noqa: E402

import torch  # noqa: E402

W_MB_SQUARE = [8, 16, 32, 64, 128, 256, 512, 1024]
T_SWEEP = [1, 2, 4, 8, 16, 32, 40, 64, 128, 256, 512]


def square_kn(w_mb: float) -> int:
    """K = N (multiple of 128) whose bf16 weight is closest to w_mb MB."""
    k = math.sqrt(w_mb * 2**20 / 2)
    return max(128, int(round(k / 128)) * 128)


def copies_for(nbytes: int, c_eff_mb: float, flushed: bool) -> int:
    if not flushed:
        return 1
    return max(2, int(2 * c_eff_mb * 2**20 / nbytes) + 1)


# ------------------------------------------------------------------ square family
def square_cell(K: int, T: int, c_eff_mb: float, flushed: bool, reps: int) -> dict:
    from cb200 import ops
    import dense_ops

    N = K
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(K * 131 + T)
    x = torch.randn(T, K, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty(T, N, device=dev, dtype=torch.bfloat16)
    r = {}

    # bf16 cuBLAS
    R = copies_for(2 * K * N, c_eff_mb, flushed)
    wb = [(torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(R)]
    r["bf16_us"] = graph_time_us_indexed(lambda i: (lambda: torch.mm(x, wb[i % R].t(), out=out)), reps=reps)
    r["bf16_copies"] = R

    # W8A8 (dynamic act quant + GEMM)
    R8 = copies_for(K * N, c_eff_mb, flushed)
    w8 = []
    for i in range(R8):
        wf = wb[i % R].float()
        s = torch.clamp(wf.abs().amax(dim=1) / 127.0, min=1e-8)
        w8.append((torch.clamp(torch.round(wf / s[:, None]), -127, 127).to(torch.int8).contiguous(), s))
        del wf
    q = torch.empty(T, K, device=dev, dtype=torch.int8)
    sa = torch.empty(T, device=dev, dtype=torch.float32)
    r["w8a8_us"] = graph_time_us_indexed(
        lambda i: (lambda: ops.w8a8_gemm_dynamic(x, w8[i % R8][0], w8[i % R8][1], q=q, s=sa, out=out)), reps=reps)
    r["w8a8_mm_us"] = graph_time_us_indexed(
        lambda i: (lambda: ops.w8a8_gemm(q, w8[i % R8][0], sa, w8[i % R8][1], out=out)), reps=reps)
    r["w8a8_copies"] = R8
    del w8

    # W4A16 g128
    R4 = copies_for(K * N // 2, c_eff_mb, flushed)
    w4 = [dense_ops.quantize_w4a16(wb[i % R], 128) for i in range(R4)]
    r["w4a16_us"] = graph_time_us_indexed(
        lambda i: (lambda: dense_ops.apply_w4a16_linear(x, w4[i % R4][0], w4[i % R4][1], N, K, out=out)),
        reps=reps)
    r["w4a16_copies"] = R4
    del w4

    # NVFP4 (e2m1 + e4m3 scales per 16; amax global scales as the reference's harness)
    RF = copies_for(K * N // 2 + K * N // 16, c_eff_mb, flushed)
    gx = torch.tensor([448.0 * 6.0 / float(x.float().abs().max())], device=dev)
    qx, sx = ops.nvfp4_quantize(x, gx)
    wf4 = []
    for i in range(RF):
        gw = torch.tensor([448.0 * 6.0 / float(wb[i % R].float().abs().max())], device=dev)
        qw, sw = ops.nvfp4_quantize(wb[i % R], gw)
        wf4.append((qw, sw, (1.0 / (gx * gw)).float()))

    def fp4_dyn(i):
        def f():
            ops.nvfp4_quantize(x, gx, q=qx, sf=sx)
            ops.nvfp4_gemm(qx, sx, wf4[i % RF][0], wf4[i % RF][1], wf4[i % RF][2], out=out)
        return f

    r["nvfp4_us"] = graph_time_us_indexed(fp4_dyn, reps=reps)
    r["nvfp4_mm_us"] = graph_time_us_indexed(
        lambda i: (lambda: ops.nvfp4_gemm(qx, sx, wf4[i % RF][0], wf4[i % RF][1], wf4[i % RF][2], out=out)),
        reps=reps)
    r["nvfp4_copies"] = RF
    del wf4, wb
    torch.cuda.empty_cache()
    return r


# ------------------------------------------------------------------ reference bmm family
def bmm_cell(w_mb: int, T: int, c_eff_mb: float, flushed: bool, reps: int) -> dict:
    import bench_l2_barrier as B
    import w8a8_bmm as W8

    H, K = 128, 128
    N = 32 * w_mb
    dev = torch.device("cuda")
    x = torch.randn(H, T, K, dtype=torch.float16, device=dev) / 4
    c = torch.empty(H, T, N, dtype=torch.float16, device=dev)
    r = {}
    R = copies_for(2 * H * K * N, c_eff_mb, flushed)
    ws = [torch.randn(H, K, N, dtype=torch.float16, device=dev) / 8 for _ in range(R)]
    r["bf16_us"] = graph_time_us_indexed(lambda i: (lambda: torch.bmm(x, ws[i % R], out=c)), reps=reps)

    R4 = copies_for(H * K * N // 2, c_eff_mb, flushed)
    w4 = [B.quantize_weights_int4(ws[i % R]) for i in range(R4)]

    def w4_fn(i):
        wp, wsc = w4[i % R4]
        grid = (H, 1)

        def f():
            B.kernel_batched_w4a16_simple[grid](
                x, wp, wsc, c, T, N, K, x.stride(0), x.stride(1), x.stride(2), wp.stride(0), wp.stride(1),
                wp.stride(2), wsc.stride(0), wsc.stride(1), c.stride(0), c.stride(1), c.stride(2),
                BLOCK_M=16, BLOCK_N=64, BLOCK_K=K)
        return f

    for i in range(R4):  # the first call per weight repacks it (outside capture)
        w4_fn(i)()
    r["w4a16_us"] = graph_time_us_indexed(w4_fn, reps=reps)

    R8 = copies_for(H * K * N, c_eff_mb, flushed)
    w8 = [W8.quantize_weights_w8(ws[i % R]) for i in range(R8)]
    q = torch.empty_like(x, dtype=torch.int8)
    s = torch.empty(H * T, dtype=torch.float32, device=dev)
    o8 = torch.empty(H, T, N, dtype=torch.float16, device=dev)

    def w8_fn(i):
        wq, wsc = w8[i % R8]

        def f():
            W8.quantize_acts_w8(x, q, s)
            W8.w8a8_bmm(q, wq, s, wsc, o8, **W8._pick_config(T))
        return f

    r["w8a8_us"] = graph_time_us_indexed(w8_fn, reps=reps)
    r["copies"] = {"bf16": R, "w4a16": R4, "w8a8": R8}
    del ws, w4, w8
    torch.cuda.empty_cache()
    return r


def gate_of(rows, prec, T, variant):
    """Smallest W (MB) from which ``prec`` stays faster than bf16 at this T."""
    pts = sorted((r["w_mb"], r[f"sp_{prec}"]) for r in rows if r["tokens"] == T and r["variant"] == variant)
    for i, (w, _) in enumerate(pts):
        if all(sp > 1.0 for _, sp in pts[i:]):
            return w
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--params", default=None, help="CARM params JSON (measure_params.py); gives C_eff")
    ap.add_argument("--family", choices=["square", "bmm"], default="square")
    ap.add_argument("--wsweep", default=None, help="comma-separated bf16-equivalent MB")
    ap.add_argument("--tsweep", default=",".join(map(str, T_SWEEP)))
    ap.add_argument("--variants", default="hot,flushed")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()

    c_eff = 100.0
    if args.params:
        with open(args.params) as f:
            c_eff = json.load(f).get("effective_l2_capacity_mb") or c_eff
    if args.wsweep:
        wsweep = [float(w) for w in args.wsweep.split(",")]
    elif args.family == "square":
        # doubling sizes plus 8 MB steps around the gate (bf16 bytes cross C_eff there)
        fine = [round(c_eff + d) for d in (-16, -8, 8, 16)]
        wsweep = sorted(set(W_MB_SQUARE + [w for w in fine if w > 0]))
    else:
        wsweep = [8, 16, 32, 64, 96, 128, 192, 256]
    tsweep = [int(t) for t in args.tsweep.split(",")]

    print(f"{gpu_info()}  family={args.family}  C_eff={c_eff:.1f} MB", flush=True)
    rows = []
    with ClockSampler(0) as clk:
        for variant in args.variants.split(","):
            for T in tsweep:
                for w_mb in wsweep:
                    if args.family == "square":
                        K = square_kn(w_mb)
                        r = square_cell(K, T, c_eff, variant == "flushed", args.reps)
                        r.update({"K": K, "N": K, "w_mb": round(2 * K * K / 2**20, 2)})
                    else:
                        r = bmm_cell(int(w_mb), T, c_eff, variant == "flushed", args.reps)
                        r.update({"H": 128, "K": 128, "N": 32 * int(w_mb), "w_mb": w_mb})
                    r.update({"tokens": T, "variant": variant})
                    r["sp_w8a8"] = round(r["bf16_us"] / r["w8a8_us"], 4)
                    r["sp_w4a16"] = round(r["bf16_us"] / r["w4a16_us"], 4)
                    if "nvfp4_us" in r:
                        r["sp_nvfp4"] = round(r["bf16_us"] / r["nvfp4_us"], 4)
                    rows.append(r)
                    print(f"{variant:7s} T={T:4d} W={r['w_mb']:8.1f} MB  bf16 {r['bf16_us']:8.2f}  "
                          f"w8a8 {r['w8a8_us']:8.2f} ({r['sp_w8a8']:.2f}x)  "
                          f"w4a16 {r['w4a16_us']:8.2f} ({r['sp_w4a16']:.2f}x)"
                          + (f"  nvfp4 {r['nvfp4_us']:8.2f} ({r['sp_nvfp4']:.2f}x)" if "nvfp4_us" in r else ""),
                          flush=True)
    precs = ("w8a8", "w4a16", "nvfp4") if args.family == "square" else ("w8a8", "w4a16")
    gates = {v: {str(T): {p: gate_of(rows, p, T, v) for p in precs} for T in tsweep}
             for v in args.variants.split(",")}
    out = {"experiment": f"capacity_gate_{args.family}", "gpu": gpu_info(), "c_eff_mb": c_eff,
           "timing": "CUDA graphs, 10 launches/graph, median of replays; flushed = rotating weight copies",
           "clocks": clk.info, "gates_mb": gates, "rows": rows}
    if args.out:
        save_json(args.out, out)


if __name__ == "__main__":
    main()
