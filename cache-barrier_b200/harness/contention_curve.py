"""Contention-degree sweep: effective weight bandwidth against the number R of
distinct weight copies cycled through one captured graph.

Port of profiling/dense_qwen/bench_contention_curve.py:30-58 onto these kernels.
Same shapes (kv_proj K = 5120, N = 2048 and q_proj K = 5120, N = 6144, M = 16),
same copy counts R = 1, 2, 3, 4, 6, 8, 12 (launch i of the graph reads copy
i % R), the same bandwidth rule (operand MB / (t - t0), t0 the graph launch
floor) and the lm_head extreme point (K = 5120, N = 248832). Paths, all
mm-only (activations quantized beforehand, as the reference's w8a8 path):

  bf16      torch.mm (cuBLAS)
  int8_cb   cb_w8a8_gemm, per-channel int8 weights, per-token int8 activations
  fp8_cb    cb_fp8_gemm, per-tensor e4m3 weights and activations (the operands
            vLLM's scaled_fp8_quant makes, the reference's w8a8 path)
  fp8_vllm  vllm._custom_ops.cutlass_scaled_mm on the same kind of operands,
            when vLLM's GPU ops load

    python cache-barrier_b200/harness/contention_curve.py --out contention_b200.json
"""

from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import torch  # noqa: E402

from common import ClockSampler, gpu_info, graph_time_us_indexed, save_json  # noqa: E402

M = 16
COPIES = [1, 2, 3, 4, 6, 8, 12]
SHAPES = [("kv_proj", 5120, 2048), ("q_proj", 5120, 6144)]
LM_HEAD = ("lm_head", 5120, 248832)


def operands(K: int, N: int, R: int, vops):
    """R weight copies in every path's format, and one activation tile."""
    from cb200 import ops

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(N + R)
    ws = [(torch.randn(N, K, device=dev, generator=g) / K ** 0.5).to(torch.bfloat16) for _ in range(R)]
    x = (torch.randn(M, K, device=dev, generator=g) / 32).to(torch.bfloat16)
    i8 = []
    for w in ws:
        wf = w.float()
        s = torch.clamp(wf.abs().amax(dim=1) / 127.0, min=1e-8)
        i8.append((torch.clamp(torch.round(wf / s[:, None]), -127, 127).to(torch.int8).contiguous(), s.contiguous()))
        del wf
    f8 = [ops.quant_act_fp8(w, "per_tensor") for w in ws]
    ops_in = {"x": x, "xi": ops.quant_act_i8(x), "xf": ops.quant_act_fp8(x, "per_tensor"), "ws": ws, "i8": i8,
              "f8": f8}
    if vops is not None:
        ops_in["vw"] = [vops.scaled_fp8_quant(w) for w in ws]
        ops_in["vx"] = vops.scaled_fp8_quant(x)
    return ops_in


def time_paths(K: int, N: int, R: int, vops, paths=("bf16", "int8_cb", "fp8_cb", "fp8_vllm")):
    from cb200 import ops

    o = operands(K, N, R, vops)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    x, (xi, xis), (xf, xfs) = o["x"], o["xi"], o["xf"]
    makers = {
        "bf16": lambda i: (lambda: torch.mm(x, o["ws"][i % R].t(), out=out)),
        "int8_cb": lambda i: (lambda: ops.w8a8_gemm(xi, o["i8"][i % R][0], xis, o["i8"][i % R][1], out=out)),
        "fp8_cb": lambda i: (lambda: ops.fp8_gemm(xf, o["f8"][i % R][0], xfs, o["f8"][i % R][1], out=out)),
    }
    if vops is not None:
        vx, vxs = o["vx"]
        makers["fp8_vllm"] = lambda i: (lambda: vops.cutlass_scaled_mm(vx, o["vw"][i % R][0].t(), vxs,
                                                                       o["vw"][i % R][1], torch.bfloat16))
    res = {p: round(graph_time_us_indexed(makers[p], inner=10, reps=30), 2) for p in paths if p in makers}
    assert ops.device_status(torch.device("cuda")) == 0
    del o
    torch.cuda.empty_cache()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--t0-us", type=float, default=2.07, help="graph launch floor (B200, measure_params.py)")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    try:
        import vllm._custom_ops as vops
    except Exception as e:  # noqa: BLE001
        print(f"vLLM ops unavailable: {e!r}", flush=True)
        vops = None
    rows = []

    def bw(mb, us):  # MB / us = TB/s
        return round(mb / max(us - args.t0_us, 0.05), 3)

    with ClockSampler(0) as clk:
        for name, K, N in SHAPES:
            for R in COPIES:
                r = time_paths(K, N, R, vops)
                mb16, mb8 = K * N * 2 / 1e6, K * N / 1e6
                row = {"shape": name, "K": K, "N": N, "R": R, "operand_mb_bf16": round(mb16, 1),
                       "operand_mb_8bit": round(mb8, 1), "total_ws_mb_bf16": round(mb16 * R, 1), **r,
                       "bw_tbs_bf16": bw(mb16, r["bf16"]), "bw_tbs_int8_cb": bw(mb8, r["int8_cb"]),
                       "bw_tbs_fp8_cb": bw(mb8, r["fp8_cb"])}
                if "fp8_vllm" in r:
                    row["bw_tbs_fp8_vllm"] = bw(mb8, r["fp8_vllm"])
                rows.append(row)
                print(f"{name:8s} R={R:2d} WS {mb16 * R:7.1f} MB bf16 | bf16 {r['bf16']:7.2f}  int8_cb "
                      f"{r['int8_cb']:7.2f}  fp8_cb {r['fp8_cb']:7.2f}  fp8_vllm {r.get('fp8_vllm', float('nan')):7.2f} us",
                      flush=True)
        name, K, N = LM_HEAD
        r = time_paths(K, N, 1, vops)
        mb16, mb8 = K * N * 2 / 1e6, K * N / 1e6
        row = {"shape": name, "K": K, "N": N, "R": 1, "operand_mb_bf16": round(mb16, 1),
               "operand_mb_8bit": round(mb8, 1), "total_ws_mb_bf16": round(mb16, 1), **r,
               "bw_tbs_bf16": bw(mb16, r["bf16"]), "bw_tbs_int8_cb": bw(mb8, r["int8_cb"]),
               "bw_tbs_fp8_cb": bw(mb8, r["fp8_cb"])}
        if "fp8_vllm" in r:
            row["bw_tbs_fp8_vllm"] = bw(mb8, r["fp8_vllm"])
        rows.append(row)
        print(f"lm_head {mb16:.0f} MB bf16: " + "  ".join(f"{k} {v:.1f} us" for k, v in r.items()), flush=True)
    out = {"experiment": "contention_degree_sweep", "gpu": gpu_info(), "M": M, "t0_us": args.t0_us,
           "method": "graph_time_us_indexed (10 launches per graph, launch i reads copy i % R, median of 30 "
                     "replays); mm-only; BW = operand MB / (t - t0)",
           "clocks": clk.info, "rows": rows}
    if args.out:
        save_json(args.out, out)


if __name__ == "__main__":
    main()
