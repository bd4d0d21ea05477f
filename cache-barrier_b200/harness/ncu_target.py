"""Nsight Compute target for the quantized GEMM kernels.

Counterpart of the reference's NCU targets (profiling/w8a8/ncu_target_w8a8.py:1-33):
warms the kernel up, then runs a few launches between cudaProfilerStart/Stop so
``ncu --profile-from-start off`` (or ``-s/-c``) captures steady-state launches.
Weights rotate over several copies so each captured launch streams its weights
from HBM (working set larger than L2).

    python cache-barrier_b200/harness/ncu_target.py --op w8a8 --tokens 32 --k 8192 --n 8192
    ncu --set full --clock-control none -k regex:w8a8_gemm -s 3 -c 1 -o prof \\
        python cache-barrier_b200/harness/ncu_target.py --op w8a8 --tokens 32
"""

from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import torch  # noqa: E402

from cb200 import _lib as L  # noqa: E402
from cb200 import ops  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", choices=["w8a8", "w8a8_dynamic", "fp8", "w4a16", "nvfp4", "mla"], default="w8a8")
    ap.add_argument("--heads", type=int, default=16, help="mla: batch of heads (latents [heads, tokens, k])")
    ap.add_argument("--batch", type=int, default=1,
                    help="w8a8: batch of GEMMs (the reference's gate shapes: --batch 128 --k 128 --n 32*W)")
    ap.add_argument("--tokens", type=int, default=32)
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--n", type=int, default=8192)
    ap.add_argument("--copies", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--launches", type=int, default=3)
    args = ap.parse_args()

    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    T, K, N = args.tokens, args.k, args.n
    a = torch.randn(T, K, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty(T, N, dtype=torch.bfloat16, device=dev)
    if args.op.startswith("w8a8"):
        Hb = args.batch
        if Hb > 1:
            a = torch.randn(Hb, T, K, generator=g, device=dev).to(torch.bfloat16)
            out = torch.empty(Hb, T, N, dtype=torch.bfloat16, device=dev)
        wshape = (Hb, K, N) if Hb > 1 else (K, N)
        ws_ = ((torch.randn(*wshape[:-2], N, generator=g, device=dev) * 0.01).abs() + 1e-4).float()
        weights = [ops.repack_w8_kmajor(torch.randint(-127, 128, wshape, generator=g, dtype=torch.int8, device=dev))
                   for _ in range(args.copies)]
        q, s = ops.quant_act_i8(a)

        def run(i):
            if args.op == "w8a8":
                ops.w8a8_gemm(q, weights[i % args.copies], s, ws_, out=out)
            else:
                ops.w8a8_gemm_dynamic(a, weights[i % args.copies], ws_, q=q, s=s, out=out)
    elif args.op == "fp8":
        # e4m3 x e4m3 per-token / per-channel (tcgen05.mma.kind::f8f6f4), fp32 accumulators
        ws_ = ((torch.randn(N, generator=g, device=dev) * 0.01).abs() + 1e-4).float()
        weights = []
        for _ in range(args.copies):
            w = (torch.randn(N, K, generator=g, device=dev) * 0.05).to(torch.bfloat16)
            qw, _ = ops.quant_act_fp8(w)
            weights.append(qw)
            del w
        qa, sa = ops.quant_act_fp8(a)

        def run(i):
            ops.fp8_gemm(qa, weights[i % args.copies], sa, ws_, out=out)
    elif args.op == "mla":
        # latent reconstruction: [heads, T, K] bf16 x int4 g128 [heads, K, N] (weight-stationary kernel)
        H = args.heads
        a = torch.randn(H, T, K, generator=g, device=dev).to(torch.bfloat16)
        out = torch.empty(H, T, N, dtype=torch.bfloat16, device=dev)
        sc = ((torch.randn(H, K // 128, N, generator=g, device=dev) * 0.02).abs() / 7 + 1e-4).to(torch.bfloat16)
        weights = [ops.repack_w4(torch.randint(0, 256, (H, K // 2, N), generator=g, dtype=torch.uint8, device=dev),
                                 L.CB_W4_REF_U8_KN, K, N) for _ in range(args.copies)]

        def run(i):
            ops.w4a16_gemm(a, weights[i % args.copies], sc, N, 128, out=out)
    elif args.op == "nvfp4":
        gx = torch.tensor([448.0 * 6.0 / float(a.float().abs().max())], device=dev)
        qa, sa = ops.nvfp4_quantize(a, gx)
        weights = []
        for _ in range(args.copies):
            w = (torch.randn(N, K, generator=g, device=dev) / K ** 0.5).to(torch.bfloat16)
            gw = torch.tensor([448.0 * 6.0 / float(w.float().abs().max())], device=dev)
            qw, sw = ops.nvfp4_quantize(w, gw)
            weights.append((qw, sw, (1.0 / (gx * gw)).float()))
            del w

        def run(i):
            qw, sw, alpha = weights[i % args.copies]
            ops.nvfp4_gemm(qa, sa, qw, sw, alpha, out=out)
    else:
        sc = ((torch.randn(K // 128, N, generator=g, device=dev) * 0.02).abs() / 7 + 1e-4).to(torch.bfloat16)
        weights = [ops.repack_w4(torch.randint(0, 256, (K // 2, N), generator=g, dtype=torch.uint8, device=dev),
                                 L.CB_W4_REF_U8_KN, K, N) for _ in range(args.copies)]

        def run(i):
            ops.w4a16_gemm(a, weights[i % args.copies], sc, N, 128, out=out)

    for i in range(args.warmup):
        run(i)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    for i in range(args.launches):
        run(args.warmup + i)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    assert ops.device_status(dev) == 0
    print("ok", args.op, T, K, N)


if __name__ == "__main__":
    main()
