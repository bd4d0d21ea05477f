"""Dense L2-boundary sweep with the fp8 W8A8 path against vLLM's cutlass fp8 GEMM.

Restates the method of profiling/dense_qwen/bench_l2_boundary.py:49-83 (K = 8192,
M = 16, N chosen so the bf16 weight is 8..320 MB, "warm" = the same weights
replayed, "rotated" = max(2, 2 C_eff / bytes + 1) weight copies advanced per
launch inside the captured graph) and times, on the same box and the same
operands:

  bf16      torch.mm (cuBLAS) on the bf16 weights
  fp8_cb    cb_fp8_gemm (tcgen05 kind::f8f6f4), per-tensor e4m3 weights and
            activations quantized beforehand ("mm-only", as the reference's w8a8_mm)
  fp8_vllm  vllm._custom_ops.cutlass_scaled_mm on vLLM's own scaled_fp8_quant
            operands (the reference's w8a8_mm path), when vLLM's ops load
  int8_cb   cb_w8a8_gemm on per-channel int8 weights (mm-only)
  nvfp4_cb  cb_nvfp4_gemm on NVFP4 weights and activations (mm-only)

    python cache-barrier_b200/harness/l2_boundary.py --out l2_boundary_b200.json
"""

from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import torch  # noqa: E402

from common import ClockSampler, gpu_info, graph_time_us_indexed, save_json  # noqa: E402

K = 8192
M = 16


def one(N: int, rotate: bool, c_eff_mb: float, vops):
    from cb200 import ops

    dev = torch.device("cuda")
    n_cop = 1 if not rotate else max(2, int(2 * c_eff_mb * 1e6 / (K * N * 2)) + 1)
    g = torch.Generator(device=dev).manual_seed(N)
    ws = [(torch.randn(N, K, device=dev, generator=g) / K ** 0.5).to(torch.bfloat16) for _ in range(n_cop)]
    x = (torch.randn(M, K, device=dev, generator=g) / 32).to(torch.bfloat16)
    # fp8, ours: per-tensor e4m3 weights and activations (as vLLM's scaled_fp8_quant)
    fq = [ops.quant_act_fp8(w, "per_tensor") for w in ws]
    xq, xs = ops.quant_act_fp8(x, "per_tensor")
    # int8 per-channel weights (K-major), per-token activations
    i8 = []
    for w in ws:
        wf = w.float()
        s = torch.clamp(wf.abs().amax(dim=1) / 127.0, min=1e-8)
        i8.append((torch.clamp(torch.round(wf / s[:, None]), -127, 127).to(torch.int8).contiguous(), s.contiguous()))
        del wf
    xi, xis = ops.quant_act_i8(x)
    # NVFP4
    gx = torch.tensor([448.0 * 6.0 / float(x.float().abs().max())], device=dev)
    qx4, sx4 = ops.nvfp4_quantize(x, gx)
    f4 = []
    for w in ws:
        gw = torch.tensor([448.0 * 6.0 / float(w.float().abs().max())], device=dev)
        q4, s4 = ops.nvfp4_quantize(w, gw)
        f4.append((q4, s4, (1.0 / (gx * gw)).float()))
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)

    paths = {
        "bf16": lambda i: (lambda: torch.mm(x, ws[i % n_cop].t(), out=out)),
        "fp8_cb": lambda i: (lambda: ops.fp8_gemm(xq, fq[i % n_cop][0], xs, fq[i % n_cop][1], out=out)),
        "int8_cb": lambda i: (lambda: ops.w8a8_gemm(xi, i8[i % n_cop][0], xis, i8[i % n_cop][1], out=out)),
        "nvfp4_cb": lambda i: (lambda: ops.nvfp4_gemm(qx4, sx4, f4[i % n_cop][0], f4[i % n_cop][1], f4[i % n_cop][2],
                                                      out=out)),
    }
    if vops is not None:
        vw = [vops.scaled_fp8_quant(w) for w in ws]
        vxq, vxs = vops.scaled_fp8_quant(x)
        paths["fp8_vllm"] = lambda i: (lambda: vops.cutlass_scaled_mm(vxq, vw[i % n_cop][0].t(), vxs, vw[i % n_cop][1],
                                                                      torch.bfloat16))
    r = {}
    for tag, mk in paths.items():
        r[tag] = round(graph_time_us_indexed(mk, inner=10, reps=30), 2)
    assert ops.device_status(dev) == 0
    del ws, fq, i8, f4
    torch.cuda.empty_cache()
    return r, n_cop


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--c-eff-mb", type=float, default=98.8, help="effective L2 capacity (B200, measure_params.py)")
    ap.add_argument("--t0-us", type=float, default=2.07, help="graph launch floor (B200, measure_params.py)")
    ap.add_argument("--targets-mb", default="8,16,24,32,40,48,64,96,128,160,192,256,320")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    try:
        import vllm._custom_ops as vops
    except Exception as e:  # noqa: BLE001
        print(f"vLLM ops unavailable: {e!r}", flush=True)
        vops = None
    targets = [float(v) for v in args.targets_mb.split(",")]
    rows = []
    with ClockSampler(0) as clk:
        for mode in ("warm", "rotated"):
            for mb in targets:
                N = int(mb * 1e6 / K / 2 / 256) * 256
                wmb = K * N * 2 / 1e6
                r, n_cop = one(N, mode == "rotated", args.c_eff_mb, vops)

                def bw(mbytes, us):
                    return round(mbytes / max(us - args.t0_us, 0.05), 2)

                row = {"mode": mode, "N": N, "wt_mb_bf16": round(wmb, 1), "wt_mb_fp8": round(wmb / 2, 1),
                       "n_copies": n_cop, **r, "bw_bf16": bw(wmb, r["bf16"]), "bw_fp8_cb": bw(wmb / 2, r["fp8_cb"]),
                       "bw_int8_cb": bw(wmb / 2, r["int8_cb"]), "bw_nvfp4_cb": bw(wmb * 9 / 32, r["nvfp4_cb"])}
                if "fp8_vllm" in r:
                    row["bw_fp8_vllm"] = bw(wmb / 2, r["fp8_vllm"])
                    row["fp8_cb_speedup_vs_vllm"] = round(r["fp8_vllm"] / r["fp8_cb"], 3)
                row["fp8_cb_speedup_vs_bf16"] = round(r["bf16"] / r["fp8_cb"], 3)
                rows.append(row)
                print(f"{mode:7s} {wmb:6.1f} MB  bf16 {r['bf16']:7.2f}  fp8_cb {r['fp8_cb']:7.2f}  "
                      f"fp8_vllm {r.get('fp8_vllm', float('nan')):7.2f}  int8_cb {r['int8_cb']:7.2f}  "
                      f"nvfp4_cb {r['nvfp4_cb']:7.2f} us", flush=True)
    out = {"experiment": "l2_boundary_sweep_dense_fp8", "gpu": gpu_info(), "K": K, "M": M,
           "method": "graph_time_us_indexed (10 launches per graph, median of 30 replays); mm-only (activations "
                     "quantized beforehand); BW = weight MB / (t - t0); rotated copies advance per launch",
           "c_eff_mb": args.c_eff_mb, "t0_us": args.t0_us, "clocks": clk.info, "rows": rows}
    if args.out:
        save_json(args.out, out)


if __name__ == "__main__":
    main()
