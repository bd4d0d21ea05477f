"""The vLLM-shaped drop-in of the dense projection harnesses (dropin/dense_ops.py)
on the GPU, through the C ABI.

The reference's dense harnesses call vLLM ops
(profiling/dense_qwen/bench_l2_boundary.py:54-57, 66-71;
profiling/dense_qwen/bench_dense_proj.py:40-43, 113-115); dense_ops keeps those
call shapes for int8 W8A8, int4 W4A16 and NVFP4. Tolerances:
  - cutlass_scaled_mm / scaled_int8_quant: bit-exact against the oracle
    (int32 accumulators, ((acc * scale_a) * scale_b) + bias in fp32, one
    rounding to out_dtype), with per-token and per-tensor scales, column-major
    and row-major b, with and without bias;
  - apply_w4a16_linear: element-wise |got - ref| <= 1e-2 * |ref| + 2^-12 * (|x| @ |w|)
    against x @ dequant(w) in float64, where dequant(w) is the operand the
    quantizer returns (q * s rounded once to the scale dtype, the kernel's own
    operand): only fp32 accumulation separates the two, and the small absolute
    term bounds it for outputs that cancel to near zero;
  - scaled_fp4_quant: bit-exact against the NVFP4 oracle (values and swizzled
    scales); cutlass_scaled_fp4_mm: fp32 output within 1e-5 of the largest
    output magnitude of the exact product.
"""

import numpy as np
import pytest
import torch

from _gpu_helpers import elementwise_close, oracle_dtype, out_bits, to_np_f32
from oracle import quant_oracle as O

pytestmark = pytest.mark.gpu


def _int8_problem(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    wq_kn = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int32).to(torch.int8)
    ws = (torch.randn(N, generator=g) * 0.01).abs().float() + 1e-4
    bias = (torch.randn(N, generator=g) * 0.5).to(torch.bfloat16)
    return a, wq_kn, ws, bias


@pytest.mark.parametrize("M,N,K", [(1, 256, 512), (16, 1024, 4096), (33, 640, 1280), (64, 7168, 5120)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("with_bias", [False, True])
def test_cutlass_scaled_mm_int8_bit_exact(cuda_device, M, N, K, out_dtype, with_bias):
    import dense_ops
    a, wq_kn, ws, bias = _int8_problem(M, N, K, seed=M * 131 + N + K)
    d = cuda_device
    q, s, azp = dense_ops.scaled_int8_quant(a.to(d))
    assert azp is None and s.shape == (M, 1)
    ref_q, ref_s = O.quant_act_i8(to_np_f32(a))
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), ref_q)
    assert np.array_equal(s.cpu().numpy().reshape(-1).view(np.uint32), ref_s.view(np.uint32))
    # b as vLLM's harness builds it: a column-major [K, N] view of a K-major [N, K] weight
    b = wq_kn.t().contiguous().to(d).t()
    assert b.stride(0) == 1
    out = dense_ops.cutlass_scaled_mm(q, b, s, ws.to(d).view(1, N), out_dtype,
                                      bias=bias.to(d) if with_bias else None)
    torch.cuda.synchronize()
    acc = O.gemm_i8_i32(ref_q, wq_kn.numpy())
    ref = O.w8a8_epilogue(acc, ref_s, ws.numpy(), oracle_dtype(out_dtype),
                          bias=to_np_f32(bias) if with_bias else None)
    assert out.dtype == out_dtype and out.shape == (M, N)
    ref_bits = ref if out_dtype == torch.bfloat16 else ref.view(np.uint16)
    assert np.array_equal(out_bits(out), ref_bits)


@pytest.mark.parametrize("M", [8, 2, 1])
def test_cutlass_scaled_mm_per_tensor_scales_row_major_b(cuda_device, M):
    """Per-tensor scale_a / scale_b (one element each), b row-major (copied to K-major), f32 bias."""
    import dense_ops
    N, K = 384, 768
    g = torch.Generator().manual_seed(77)
    aq = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int32).to(torch.int8)
    wq_kn = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int32).to(torch.int8)
    sa = torch.tensor([0.0123], dtype=torch.float32)
    sb = torch.tensor([0.0041], dtype=torch.float32)
    bias = torch.randn(N, generator=g, dtype=torch.float32)
    d = cuda_device
    out = dense_ops.cutlass_scaled_mm(aq.to(d), wq_kn.to(d), sa.to(d), sb.to(d), torch.bfloat16, bias=bias.to(d))
    torch.cuda.synchronize()
    acc = O.gemm_i8_i32(aq.numpy(), wq_kn.numpy())
    ref = O.w8a8_epilogue(acc, np.full(M, sa.item(), np.float32), np.full(N, sb.item(), np.float32), "bf16",
                          bias=bias.numpy())
    assert np.array_equal(out_bits(out), ref)


def test_cutlass_scaled_mm_rejects_bad_bias(cuda_device):
    import dense_ops
    d = cuda_device
    aq = torch.zeros(4, 64, dtype=torch.int8, device=d)
    b = torch.zeros(128, 64, dtype=torch.int8, device=d).t()
    s = torch.ones(4, 1, device=d)
    with pytest.raises(ValueError):
        dense_ops.cutlass_scaled_mm(aq, b, s, torch.ones(1, 128, device=d), torch.bfloat16,
                                    bias=torch.zeros(127, device=d))


@pytest.mark.parametrize("M,N,K", [(1, 7168, 5120), (8, 1024, 2048), (32, 5120, 17408), (65, 384, 640)])
def test_apply_w4a16_linear(cuda_device, M, N, K):
    import dense_ops
    g = torch.Generator().manual_seed(M + N + K)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    d = cuda_device
    native, scales, w_dq = dense_ops.quantize_w4a16(w.to(d), group_size=128, return_dequant=True)
    y = dense_ops.apply_w4a16_linear(x.to(d), native, scales, N, K)
    torch.cuda.synchronize()
    assert y.shape == (M, N) and y.dtype == torch.bfloat16
    # the quantizer: q in [-8, 7]; the returned operand is q * s rounded once to
    # bf16 (what the kernel's packed multiply yields); |w - q*s| <= s/2 (round to
    # nearest, with s = bf16(amax/7) no value needs the clamp)
    q = O.unpack_native(native.cpu().numpy(), 1, K, N)[0]  # [K, N]
    s = to_np_f32(scales)  # [K/128, N]
    qs = O.dequant_w4(q, s, 128)
    assert q.min() >= -8 and q.max() <= 7
    assert np.array_equal(O.bf16_bits_to_f32(O.round_to(qs, "bf16")), to_np_f32(w_dq))  # -0.0 == 0.0
    err = np.abs(to_np_f32(w).T - qs)
    assert np.all(err <= 0.5 * np.repeat(s, 128, axis=0) * (1 + 2.0**-7))
    xf, wf = to_np_f32(x).astype(np.float64), to_np_f32(w_dq).astype(np.float64)
    ref = xf @ wf
    assert elementwise_close(to_np_f32(y), ref, 1e-2, 2.0 ** -12 * (np.abs(xf) @ np.abs(wf)))


def test_scaled_fp4_quant_and_mm(cuda_device):
    import dense_ops
    M, N, K = 16, 1024, 2048
    g = torch.Generator().manual_seed(5)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = torch.randn(N, K, generator=g).to(torch.bfloat16)
    gx = 448.0 * 6.0 / float(x.float().abs().max())
    gw = 448.0 * 6.0 / float(w.float().abs().max())
    d = cuda_device
    f = lambda v: torch.tensor([v], dtype=torch.float32, device=d)  # noqa: E731
    xq, xs = dense_ops.scaled_fp4_quant(x.to(d), f(gx))
    wq, wsf = dense_ops.scaled_fp4_quant(w.to(d), f(gw))
    out = dense_ops.cutlass_scaled_fp4_mm(xq, wq, xs, wsf, f(1.0 / (gx * gw)), torch.float32)
    torch.cuda.synchronize()
    rq, rs, _ = O.nvfp4_quant(to_np_f32(x), gx)
    wrq, wrs, _ = O.nvfp4_quant(to_np_f32(w), gw)
    assert xs.dtype == torch.float8_e4m3fn and xs.shape == (128, K // 16)
    assert np.array_equal(xq.cpu().numpy(), rq)
    assert np.array_equal(xs.view(torch.uint8).cpu().numpy().reshape(-1), O.nvfp4_swizzle(rs))
    assert np.array_equal(wq.cpu().numpy(), wrq)
    ref = O.nvfp4_gemm(rq, rs, wrq, wrs, 1.0 / (gx * gw))
    got = out.cpu().numpy().astype(np.float64)
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()
