"""Batched INT4 BMM for MLA latent reconstruction on one B200.

The reference's MLA benches (profiling/int4_batched_gemm.py:272-275,
profiling/mla_l2_stack/bench_mla_l2_stack.py:40-70) time per-head int4
reconstruction BMMs. This harness runs the DeepSeek-style shape: 16 heads,
kv_lora_rank 512, qk_nope = v = 128, per-head int4 g128 W_UK and W_UV
[16, 512, 128] (4 scale groups along K), bf16 latents [16, b*L, 512] ~ N(0, 1)
for L in {512, 4096} and batch b in 1..32. One step is both reconstructions,
K_nope = lat @ W_UK and V = lat @ W_UV, each a batched W4A16 GEMM with
B = 16, M = b*L, K = 512, N = 128. The latents dominate the bytes, so the
roofline is HBM on the activations (about 102 FLOP per byte).

The contention variant runs 4 such steps on 4 CUDA streams at once, each with
its own latents and weights, with the streams' summed working set above the
effective L2 capacity, and compares the wall time of the 4 concurrent steps
with 4 sequential ones.

    python cache-barrier_b200/harness/mla_bmm.py --out mla.json
"""

from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from common import ClockSampler, gpu_info, graph_time_us, save_json  # noqa: E402

import torch  # noqa: E402

HEADS, RANK, DIM = 16, 512, 128
GROUP = 128


def make_weights(seed: int):
    """Per-head int4 g128 W_UK / W_UV: native buffers, bf16 scales [16, 4, 128], bf16 dequantized copies."""
    import dense_ops

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    out = []
    for _ in range(2):
        natives, scales, deq = [], [], []
        for _h in range(HEADS):
            w = (torch.randn(DIM, RANK, generator=g, device=dev) * 0.02).to(torch.bfloat16)  # [N, K]
            nat, sc, dq = dense_ops.quantize_w4a16(w, GROUP, return_dequant=True)
            natives.append(nat)
            scales.append(sc)
            deq.append(dq)  # [K, N] bf16, the values the kernel multiplies
        out.append((torch.cat(natives), torch.stack(scales), torch.stack(deq)))
    return out


class Step:
    def __init__(self, b: int, L: int, seed: int):
        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(seed)
        self.M = b * L
        self.lat = torch.randn(HEADS, self.M, RANK, generator=g, device=dev).to(torch.bfloat16)
        (self.uk, self.uk_s, self.uk_dq), (self.uv, self.uv_s, self.uv_dq) = make_weights(seed + 1)
        self.k_out = torch.empty(HEADS, self.M, DIM, device=dev, dtype=torch.bfloat16)
        self.v_out = torch.empty(HEADS, self.M, DIM, device=dev, dtype=torch.bfloat16)
        # fused reconstruction: W_UK | W_UV as one [16, 512, 256] weight (two 128-column
        # panels per head), output [K_nope | V] = [16, M, 256]; native tiles are per
        # (head, 128-column panel), so the fused weight interleaves the heads' panels
        per = self.uk.numel() // HEADS
        self.ukv = torch.cat([torch.cat([self.uk[h * per:(h + 1) * per], self.uv[h * per:(h + 1) * per]])
                              for h in range(HEADS)])
        self.ukv_s = torch.cat([self.uk_s, self.uv_s], dim=2).contiguous()
        self.ukv_dq = torch.cat([self.uk_dq, self.uv_dq], dim=2).contiguous()
        self.kv_out = torch.empty(HEADS, self.M, 2 * DIM, device=dev, dtype=torch.bfloat16)

    def cb200(self):
        from cb200 import ops

        ops.w4a16_gemm(self.lat, self.uk, self.uk_s, DIM, GROUP, out=self.k_out)
        ops.w4a16_gemm(self.lat, self.uv, self.uv_s, DIM, GROUP, out=self.v_out)

    def cublas(self):
        torch.bmm(self.lat, self.uk_dq, out=self.k_out)
        torch.bmm(self.lat, self.uv_dq, out=self.v_out)

    def cb200_fused(self):
        from cb200 import ops

        ops.w4a16_gemm(self.lat, self.ukv, self.ukv_s, 2 * DIM, GROUP, out=self.kv_out)

    def cublas_fused(self):
        torch.bmm(self.lat, self.ukv_dq, out=self.kv_out)

    def bytes(self) -> int:
        w = 2 * (HEADS * RANK * DIM // 2 + HEADS * (RANK // GROUP) * DIM * 2)
        return 2 * self.lat.numel() * 2 + w + 2 * self.k_out.numel() * 2

    def flops(self) -> int:
        return 2 * 2 * HEADS * self.M * RANK * DIM

    def check(self) -> float:
        self.cb200()
        torch.cuda.synchronize()
        ref = torch.bmm(self.lat.float(), self.uk_dq.float())
        return ((self.k_out.float() - ref).norm() / ref.norm()).item()


def contention(L: int, b: int, streams: int = 4) -> dict:
    steps = [Step(b, L, 1000 + 17 * i) for i in range(streams)]
    for s in steps:
        s.cb200()
    torch.cuda.synchronize()
    seq_us = graph_time_us(lambda: [s.cb200() for s in steps], inner=2, reps=10)
    ss = [torch.cuda.Stream() for _ in range(streams)]

    def concurrent():
        main = torch.cuda.current_stream()  # the capture stream while a graph is being captured
        for st, s in zip(ss, steps):
            st.wait_stream(main)
            with torch.cuda.stream(st):
                s.cb200()
        for st in ss:
            main.wait_stream(st)

    con_us = graph_time_us(concurrent, inner=2, reps=10)
    ws_mb = sum(s.bytes() for s in steps) / 2**20
    return {"L": L, "batch": b, "streams": streams, "working_set_mb": round(ws_mb, 1),
            "sequential_us": round(seq_us, 2), "concurrent_us": round(con_us, 2),
            "concurrent_gbs": round(sum(s.bytes() for s in steps) / (con_us * 1e-6) / 1e9, 1)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--lens", default="512,4096")
    ap.add_argument("--batches", default="1,2,4,8,16,32")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    info = gpu_info()
    print(info, flush=True)
    rows = []
    with ClockSampler(0) as clk:
        for L in [int(x) for x in args.lens.split(",")]:
            for b in [int(x) for x in args.batches.split(",")]:
                st = Step(b, L, 7 * L + b)
                rel = st.check()
                t = graph_time_us(st.cb200, inner=5, reps=15)
                tc = graph_time_us(st.cublas, inner=5, reps=15)
                tf = graph_time_us(st.cb200_fused, inner=5, reps=15)
                tcf = graph_time_us(st.cublas_fused, inner=5, reps=15)
                st.cb200_fused()
                torch.cuda.synchronize()
                ref_f = torch.bmm(st.lat.float(), st.ukv_dq.float())
                rel_f = ((st.kv_out.float() - ref_f).norm() / ref_f.norm()).item()
                del ref_f
                r = {"L": L, "batch": b, "M": st.M, "cb200_us": round(t, 2), "cublas_bf16_us": round(tc, 2),
                     "speedup_vs_cublas": round(tc / t, 3), "rel_err_vs_dequant": round(rel, 5),
                     "fused_cb200_us": round(tf, 2), "fused_cublas_bf16_us": round(tcf, 2),
                     "fused_speedup_vs_cublas": round(tcf / tf, 3), "fused_rel_err": round(rel_f, 5),
                     "bytes": st.bytes(), "achieved_gbs": round(st.bytes() / (t * 1e-6) / 1e9, 1),
                     "tflops": round(st.flops() / (t * 1e-6) / 1e12, 1)}
                rows.append(r)
                print(f"L={L:5d} b={b:3d} M={st.M:7d}: cb200 {t:9.2f} us ({r['achieved_gbs']} GB/s, "
                      f"{r['tflops']} TF/s)  cuBLAS {tc:9.2f} us  x{r['speedup_vs_cublas']}  rel {rel:.2e} | "
                      f"fused UK|UV: cb200 {tf:9.2f} cuBLAS {tcf:9.2f} x{r['fused_speedup_vs_cublas']} rel {rel_f:.2e}",
                      flush=True)
                del st
                torch.cuda.empty_cache()
        cont = [contention(512, 8), contention(4096, 2)]
        for c in cont:
            print(f"contention L={c['L']} b={c['batch']}: 4 streams, {c['working_set_mb']} MB, "
                  f"sequential {c['sequential_us']} us, concurrent {c['concurrent_us']} us", flush=True)
    out = {"experiment": "mla_latent_reconstruction_int4_bmm", "gpu": info, "heads": HEADS, "kv_lora_rank": RANK,
           "head_dim": DIM, "group": GROUP, "clocks": clk.info, "rows": rows, "contention": cont,
           "timing": "CUDA graphs, median of replays"}
    if args.out:
        save_json(args.out, out)


if __name__ == "__main__":
    main()
