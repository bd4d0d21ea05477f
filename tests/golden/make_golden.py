"""Generate the golden vectors in this directory from the reference itself.

Runs the cache-barrier reference's own code on CPU: its PyTorch quantizers, and
its Triton kernels under Triton's interpreter (TRITON_INTERPRET=1), on seeded
inputs, and writes small ``.npz`` fixtures. The fixtures are what the oracle
and the CUDA kernels are pinned against; this script is only needed to
regenerate them and is not imported by anything else.

    python tests/golden/make_golden.py --ref /path/to/cache-barrier

Reference entry points exercised (paths inside the reference repository):
  profiling/bench_l2_barrier.py      quantize_weights_int4, batched_int4_gemm
                                     (kernel_batched_w4a16_simple)
  profiling/int4_batched_gemm.py     batched_int4_gemm (its own simple kernel)
  profiling/int4_batched_gemm_v2.py  batched_int4_gemm (kernel_batched_w4a16_v3)
  profiling/w8a8/w8a8_bmm.py         quantize_weights_w8, quantize_acts_w8, w8a8_bmm
  kernels/triton_gemm.py             triton_gemm_packed_int4 (static-config path)
"""

from __future__ import annotations

import argparse
import importlib
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def _import_reference(ref: str):
    sys.path.insert(0, os.path.join(ref, "profiling"))
    sys.path.insert(0, os.path.join(ref, "profiling", "w8a8"))
    sys.path.insert(0, os.path.join(ref, "kernels"))
    # kernels/triton_gemm.py imports two helpers from an un-vendored package
    # (tiny_gemm.quantization.packed_int4) that only its __main__ demo uses.
    # Register placeholders so the module imports; the kernels do not call them.
    pkg = types.ModuleType("tiny_gemm")
    sub = types.ModuleType("tiny_gemm.quantization")
    leaf = types.ModuleType("tiny_gemm.quantization.packed_int4")

    def _unavailable(*_a, **_k):
        raise RuntimeError("tiny_gemm is not vendored with the reference")

    leaf.pack_int4_signed = _unavailable
    leaf.quantize_per_tensor_int4 = _unavailable
    sys.modules.update({"tiny_gemm": pkg, "tiny_gemm.quantization": sub,
                        "tiny_gemm.quantization.packed_int4": leaf})
    mods = {}
    for name in ("bench_l2_barrier", "int4_batched_gemm", "int4_batched_gemm_v2", "w8a8_bmm", "triton_gemm"):
        mods[name] = importlib.import_module(name)
    return mods


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def gen_w4a16(m, name, H, T, K, N, seed, keep_w=False):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(H, T, K, generator=g) / 4).half()
    w = (torch.randn(H, K, N, generator=g) / 8).half()
    wp, ws = m["bench_l2_barrier"].quantize_weights_int4(w)
    c_simple = m["bench_l2_barrier"].batched_int4_gemm(x, wp, ws, K)
    c_v1 = m["int4_batched_gemm"].batched_int4_gemm(x, wp, ws, K)
    c_v3 = m["int4_batched_gemm_v2"].batched_int4_gemm(x, wp, ws, K)
    extra = {"w": _np(w)} if keep_w else {}
    np.savez_compressed(os.path.join(OUT, name), x=_np(x), packed=_np(wp), scales=_np(ws),
                        c_simple=_np(c_simple), c_v1=_np(c_v1), c_v3=_np(c_v3), **extra)


def gen_w8a8(m, name, H, M, K, N, seed, act_dtype=torch.float16, keep_w=False):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(H, M, K, generator=g) / 4).to(act_dtype)
    w = (torch.randn(H, K, N, generator=g) / 8).half()
    mod = m["w8a8_bmm"]
    wq, wscale = mod.quantize_weights_w8(w)
    q, s = mod.quantize_acts_w8(a)
    out = mod.w8a8_bmm(q, wq, s, wscale)
    a_store = _np(a.view(torch.int16)) if act_dtype == torch.bfloat16 else _np(a)
    extra = {"w": _np(w)} if keep_w else {}
    np.savez_compressed(os.path.join(OUT, name), a=a_store, a_is_bf16_bits=act_dtype == torch.bfloat16,
                        wq=_np(wq), wscale=_np(wscale), q=_np(q), s=_np(s), out=_np(out), **extra)


def gen_act_quant_ties(m, name):
    """Rows built so a/scale lands exactly on .5 boundaries, zero rows, signed zeros."""
    row0 = [127.0, 2.5, -2.5, 0.5, -0.5, 0.0, -0.0, 126.5, -126.5, 1.5, -1.5, 63.5, -63.5, 100.0, -127.0, 3.0]
    row1 = [0.0] * 16
    row2 = [1e-9] * 8 + [-1e-9] * 8
    row3 = [0.25, -0.125, 0.375, 64.0, -0.0625, 31.75, 7.5, -7.5, 0.0, 1.0, -1.0, 2.0, 4.0, 8.0, 16.0, 32.0]
    a = torch.tensor([row0, row1, row2, row3], dtype=torch.float16).unsqueeze(0)
    q, s = m["w8a8_bmm"].quantize_acts_w8(a)
    np.savez_compressed(os.path.join(OUT, name), a=_np(a), q=_np(q), s=_np(s))


def gen_w4a4(m, name, M, K, N, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(0, 256, (M, K // 2), generator=g, dtype=torch.int32).to(torch.uint8)
    b = torch.randint(0, 256, (K // 2, N), generator=g, dtype=torch.int32).to(torch.uint8)
    # triton_gemm_packed_int4 asserts CUDA tensors (kernels/triton_gemm.py:412), so
    # launch its static kernel the way the wrapper does for explicit tile
    # arguments (:452-467): grid = cdiv(M, BM) * cdiv(N, BN) // GROUP_SIZE_M.
    tg = m["triton_gemm"]
    c = torch.empty((M, N), dtype=torch.float32)
    meta = dict(BLOCK_M=16, BLOCK_N=32, BLOCK_K=64, GROUP_SIZE_M=1)
    grid = ((M + 15) // 16 * ((N + 31) // 32) // 1,)
    tg.kernel_gemm_packed_int4_static[grid](a, b, c, M, N, K, a.stride(0), a.stride(1), b.stride(0), b.stride(1),
                                            c.stride(0), c.stride(1), **meta)
    np.savez_compressed(os.path.join(OUT, name), a_packed=_np(a), b_packed=_np(b), c=_np(c))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    args = ap.parse_args()
    m = _import_reference(args.ref)
    # The interpreter runs "device" code on CPU tensors; the reference modules
    # allocate with device=A.device, so CPU inputs keep everything on the host.
    gen_w4a16(m, "w4a16_h2_t3_k256_n192.npz", H=2, T=3, K=256, N=192, seed=0, keep_w=True)
    gen_w4a16(m, "w4a16_h4_t1_k128_n256.npz", H=4, T=1, K=128, N=256, seed=1)
    gen_w4a16(m, "w4a16_h2_t17_k512_n128.npz", H=2, T=17, K=512, N=128, seed=2)
    gen_w8a8(m, "w8a8_h2_m5_k256_n192.npz", H=2, M=5, K=256, N=192, seed=3, keep_w=True)
    gen_w8a8(m, "w8a8_h1_m1_k512_n256.npz", H=1, M=1, K=512, N=256, seed=4)
    gen_w8a8(m, "w8a8_h2_m33_k128_n64_bf16.npz", H=2, M=33, K=128, N=64, seed=5, act_dtype=torch.bfloat16)
    gen_act_quant_ties(m, "act_quant_ties.npz")
    gen_w4a4(m, "w4a4_m5_k256_n96.npz", M=5, K=256, N=96, seed=6)
    print("wrote fixtures to", OUT)


if __name__ == "__main__":
    main()
