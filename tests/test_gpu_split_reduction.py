"""Split-K reduction of cut tiles on the GPU, for every stream-K GEMM of the library
(W8A8 int8, FP8, W4A16, NVFP4).

A tile whose k-blocks are split over several CTAs is reduced either by its first
contributor (which polls, for at most 10 us, until the others have published
their parts) or, when the others are late, by the last contributor to arrive.
Both paths sum the parts in the same order, so:

  - with the poll skipped (cb_debug_force_last_arriver: every cut tile goes
    through the last-arriver path) outputs are bit-identical to the normal run,
    on shapes that cut many tiles over many contributors;
  - a GEMM launched while another stream's long GEMM holds the SMs (so its CTAs
    start in waves, not together) gives the same bits and a clean status word.
"""

import numpy as np
import pytest
import torch

from _gpu_helpers import to_np_f32
from oracle import quant_oracle as O

pytestmark = pytest.mark.gpu


def _w8a8(d, M, N, K, seed):
    from cb200 import ops
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(M, K, generator=g)).to(torch.bfloat16).to(d)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).to(d)
    ws = (torch.rand(N, generator=g) * 1e-2 + 1e-3).to(d)
    aq, as_ = ops.quant_act_i8(a)
    return lambda: ops.w8a8_gemm(aq, w, as_, ws, out_dtype=torch.float32)


def _fp8(d, M, N, K, seed):
    from cb200 import ops
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).to(d)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16).to(d)
    aq, as_ = ops.quant_act_fp8(a, "per_token")
    wq, ws = ops.quant_act_fp8(w, "per_token")
    return lambda: ops.fp8_gemm(aq, wq, as_, ws, out_dtype=torch.float32)


def _w4a16(d, M, N, K, seed):
    from cb200 import _lib as L
    from cb200 import ops
    rng = np.random.default_rng(seed)
    q = rng.integers(-8, 8, size=(1, K, N)).astype(np.int8)
    s = torch.from_numpy((rng.random((1, K // 128, N)) * 0.02 + 0.001).astype(np.float32)).to(torch.bfloat16)
    a = torch.from_numpy(rng.standard_normal((1, M, K)).astype(np.float32)).to(torch.bfloat16)
    native = ops.repack_w4(torch.from_numpy(O.pack_i32_k8n(q)).to(d), L.CB_W4_I32_K8N, K, N)
    a, s = a.to(d), s.to(d)
    return lambda: ops.w4a16_gemm(a, native, s, N, 128, out_dtype=torch.float32)


def _nvfp4(d, M, N, K, seed):
    from cb200 import ops
    rng = np.random.default_rng(seed)
    ap, asf = O.nvfp4_quant(rng.standard_normal((M, K)).astype(np.float32), 3.0)[:2]
    bp, bsf = O.nvfp4_quant(rng.standard_normal((N, K)).astype(np.float32), 5.0)[:2]
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(d)  # noqa: E731
    args = (t(ap), t(O.nvfp4_swizzle(asf)), t(bp), t(O.nvfp4_swizzle(bsf)),
            torch.tensor([1.0 / 15.0], dtype=torch.float32, device=d))
    return lambda: ops.nvfp4_gemm(*args, out_dtype=torch.float32)


MAKERS = {"w8a8": _w8a8, "fp8": _fp8, "w4a16": _w4a16, "nvfp4": _nvfp4}
# (M, N, K): few tiles over a long K (many contributors per tile), and many
# tiles with a short K (one or two contributors per cut tile)
SHAPES = [(16, 1024, 16384), (1, 256, 8192), (48, 4096, 1024), (130, 2048, 2048)]


def _lib():
    from cb200 import _lib as L
    return L.load()


@pytest.mark.parametrize("kind", list(MAKERS))
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_last_arriver_path_bit_identical(cuda_device, kind, M, N, K):
    from cb200 import ops
    run = MAKERS[kind](cuda_device, M, N, K, seed=M + N + K)
    normal = run()
    torch.cuda.synchronize()
    lib = _lib()
    lib.cb_debug_force_last_arriver(1)
    try:
        forced = [run() for _ in range(3)]
        torch.cuda.synchronize()
    finally:
        lib.cb_debug_force_last_arriver(0)
    for f in forced:
        assert torch.equal(f, normal)
    assert ops.device_status(cuda_device) == 0


@pytest.mark.parametrize("kind", list(MAKERS))
def test_cut_tiles_while_another_stream_holds_the_sms(cuda_device, kind):
    from cb200 import ops
    d = cuda_device
    run = MAKERS[kind](d, 16, 2048, 8192, seed=5)
    ref = run()
    torch.cuda.synchronize()
    big = torch.randn(8192, 8192, device=d, dtype=torch.bfloat16)
    side = torch.cuda.Stream(d)
    outs = []
    for _ in range(4):
        with torch.cuda.stream(side):
            torch.mm(big, big)
        outs.append(run())
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, ref)
    assert ops.device_status(d) == 0
    assert np.isfinite(to_np_f32(ref.cpu())).all()
