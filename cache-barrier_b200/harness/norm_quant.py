"""RMSNorm + int8 act-quant: fused kernel vs separate launches (the act-quant tax).

Counterpart of the reference's fused norm-quant measurement
(profiling/dense_qwen/results_fused_normquant_h100.json, fields M / norm / fused /
sep / fused_tax_us; profiling/mechanisms/RESULTS.md:17) on the sm_100a kernels:
  norm   torch RMSNorm alone (bf16 out)
  sep    torch RMSNorm then cb_quant_act_i8 (two launches)
  fused  cb_rmsnorm_quant_i8 (one launch)
hidden 5120, M in {1, 16, 64, 256, 1024, 2048}, CUDA-graph timing.

    python cache-barrier_b200/harness/norm_quant.py --out norm_quant.json
"""

from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from common import gpu_info, graph_time_us, save_json  # noqa: E402

import torch  # noqa: E402


def main():
    from cb200 import ops

    ap = argparse.ArgumentParser()
    ap.add_argument("--hidden", type=int, default=5120)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    H = args.hidden
    dev = torch.device("cuda")
    w = (1.0 + 0.1 * torch.randn(H, device=dev)).to(torch.bfloat16)
    rows = []
    for M in (1, 16, 64, 256, 1024, 2048):
        x = torch.randn(M, H, device=dev).to(torch.bfloat16)
        y = torch.empty_like(x)
        q = torch.empty(M, H, device=dev, dtype=torch.int8)
        s = torch.empty(M, device=dev, dtype=torch.float32)

        def norm():
            torch.nn.functional.rms_norm(x, (H,), w, 1e-6)

        def sep():
            yy = torch.nn.functional.rms_norm(x, (H,), w, 1e-6)
            ops.quant_act_i8(yy, q, s)

        def fused():
            ops.rmsnorm_quant_i8(x, w, 1e-6, q=q, s=s)

        r = {"M": M, "norm": round(graph_time_us(norm), 2), "sep": round(graph_time_us(sep), 2),
             "fused": round(graph_time_us(fused), 2)}
        r["fused_tax_us"] = round(r["fused"] - r["norm"], 2)
        rows.append(r)
        print(r, flush=True)
    if args.out:
        save_json(args.out, {"experiment": "fused_rmsnorm_int8_quant", "gpu": gpu_info(), "hidden": H, "rows": rows})


if __name__ == "__main__":
    main()
