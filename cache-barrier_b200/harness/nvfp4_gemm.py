"""NVFP4 W4A4 GEMM on B200: the sm_100a kernel vs vLLM's CUTLASS FP4 GEMM, cuBLAS bf16
and the W8A8 kernel, at the decode shape of the W8A8 configuration.

The reference measures native FP4 on B200 through vLLM
(profiling/cuda_validation/bench_moe_nvfp4_native.py: weights quantized with
scaled_fp4_quant and an amax global scale, activations with a neutral global
scale, graph-timed). Here, for K = N = 8192 and T in {1, 8, 16, 32}:
  cb_nvfp4     cb_nvfp4_gemm on vLLM-format operands (weights rotate over 4 copies,
               36 MiB each with scales, so every launch streams from HBM)
  vllm_fp4     vllm._custom_ops.cutlass_scaled_fp4_mm on the same operands (if it loads)
  cb_quant     cb_nvfp4_quantize of the activations (the per-call quantization)
  cublas_bf16  torch.mm on bf16 weights (same rotation)
  cb_w8a8      cb_w8a8_gemm on int8 weights (same rotation)
CUDA graphs of 32 launches, median of replays; NVML clocks sampled meanwhile.

    python cache-barrier_b200/harness/nvfp4_gemm.py --out nvfp4_gemm.json
"""

from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from common import ClockSampler, gpu_info, graph_time_us_indexed, save_json  # noqa: E402

import torch  # noqa: E402

COPIES = 4


def nvfp4_bytes(T: int, K: int, N: int) -> int:
    """Algorithmic bytes of one NVFP4 GEMM: packed weights and their scales,
    packed activations and their scales, bf16 output."""
    return K * N // 2 + K * N // 16 + T * K // 2 + T * K // 16 + 2 * T * N


def main():
    from cb200 import ops

    ap = argparse.ArgumentParser()
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--n", type=int, default=8192)
    ap.add_argument("--tokens", default="1,8,16,32")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    K, N = args.k, args.n
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    try:
        import vllm._custom_ops as vops
        if not hasattr(vops, "cutlass_scaled_fp4_mm"):
            vops = None
    except Exception:  # vLLM absent or its extension does not load here
        vops = None

    fp4_w, bf16_w, i8_w = [], [], []
    ws8 = (torch.rand(N, device=dev) * 0.01 + 1e-4).float()
    for _ in range(COPIES):
        w = (torch.randn(N, K, device=dev, generator=g) / K ** 0.5).to(torch.bfloat16)
        gw = torch.tensor([448.0 * 6.0 / float(w.float().abs().max())], device=dev)
        q, sf = ops.nvfp4_quantize(w, gw)
        fp4_w.append((q, sf, gw))
        bf16_w.append(w)
        i8_w.append(torch.randint(-127, 128, (N, K), device=dev, generator=g, dtype=torch.int8))
    rows = []
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    for T in [int(t) for t in args.tokens.split(",")]:
        x = torch.randn(T, K, device=dev, generator=g).to(torch.bfloat16)
        gx = torch.tensor([448.0 * 6.0 / float(x.float().abs().max())], device=dev)
        qx, sx = ops.nvfp4_quantize(x, gx)
        alphas = [(1.0 / (gx * gw)).float() for (_, _, gw) in fp4_w]
        out = torch.empty(T, N, dtype=torch.bfloat16, device=dev)
        r = {"tokens": T, "K": K, "N": N}
        r["cb_nvfp4_us"] = round(graph_time_us_indexed(
            lambda i: (lambda: ops.nvfp4_gemm(qx, sx, fp4_w[i % COPIES][0], fp4_w[i % COPIES][1],
                                              alphas[i % COPIES], out=out)), inner=32), 3)
        r["cb_quant_us"] = round(graph_time_us_indexed(lambda i: (lambda: ops.nvfp4_quantize(x, gx, q=qx, sf=sx)),
                                                       inner=32), 3)
        if vops is not None:
            sxv = sx.view(torch.float8_e4m3fn)
            wv = [(q, sf.view(torch.float8_e4m3fn)) for (q, sf, _) in fp4_w]
            try:
                r["vllm_fp4_us"] = round(graph_time_us_indexed(
                    lambda i: (lambda: vops.cutlass_scaled_fp4_mm(qx, wv[i % COPIES][0], sxv, wv[i % COPIES][1],
                                                                  alphas[i % COPIES], torch.bfloat16)),
                    inner=32), 3)
            except Exception as e:  # report, do not fail the sweep
                r["vllm_fp4_error"] = str(e)[:200]
        r["cublas_bf16_us"] = round(graph_time_us_indexed(
            lambda i: (lambda: torch.mm(x, bf16_w[i % COPIES].t(), out=out)), inner=32), 3)
        aq, a_s = ops.quant_act_i8(x)
        r["cb_w8a8_us"] = round(graph_time_us_indexed(
            lambda i: (lambda: ops.w8a8_gemm(aq, i8_w[i % COPIES], a_s, ws8, out=out)), inner=32), 3)
        r["cb_nvfp4_tbs"] = round(nvfp4_bytes(T, K, N) / r["cb_nvfp4_us"] / 1e6, 3)
        r["speedup_vs_cublas_bf16"] = round(r["cublas_bf16_us"] / r["cb_nvfp4_us"], 3)
        if "vllm_fp4_us" in r:
            r["speedup_vs_vllm_fp4"] = round(r["vllm_fp4_us"] / r["cb_nvfp4_us"], 3)
        rows.append(r)
        print(r, flush=True)
    clock_info = clocks.stop()
    res = {"experiment": "nvfp4_w4a4_gemm", "gpu": gpu_info(), "clocks": clock_info,
           "method": "CUDA graphs of 32 launches, weights rotating over 4 copies, median of 30 replays",
           "rows": rows}
    if args.out:
        save_json(args.out, res)


if __name__ == "__main__":
    main()
