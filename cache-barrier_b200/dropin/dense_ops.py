"""Drop-in for the vLLM custom-op calls of the dense_qwen harnesses, backed by libcb200.

The reference's dense projection benches call vLLM kernels
(profiling/dense_qwen/bench_dense_proj.py:40-43, 113-115;
profiling/dense_qwen/bench_l2_boundary.py:54-57, 66-71). This module keeps those
call shapes for the int8 W8A8 and int4 W4A16 paths:

  cutlass_scaled_mm(a, b, scale_a, scale_b, out_dtype, bias=None)
      a: int8 [M, K], K contiguous; b: int8 [K, N] column-major (b.t() is a
      contiguous [N, K] K-major weight); scale_a: fp32 per-token [M, 1] / [M] or
      per-tensor (one element); scale_b: fp32 per-channel [1, N] / [N] or
      per-tensor. out = cvt((a @ b)_int32 * scale_a * scale_b (+ bias)): the
      bias is added in fp32 before the one rounding to out_dtype, as vLLM's
      epilogue does.
  scaled_int8_quant(x, scale=None) -> (q, scale [M, 1], None)
      dynamic per-token symmetric int8, rounding as the cache-barrier act-quant
      kernel (profiling/w8a8/w8a8_bmm.py:35-39: scale = max(amax/127, 1e-8),
      q = trunc(x/scale + 0.5*sign(x))). Static scales are not supported.
  quantize_w4a16(w, group_size=128, return_dequant=False) -> (w_native, scales [K/G, N][, w_dq [K, N]])
      symmetric int4 per (group, output channel) of a [N, K] (torch Linear)
      weight: s = amax/7 (clamped at 1e-8, rounded to the scale dtype),
      q = round_half_even(w/s) clamped to [-8, 7]; packed as the reference's
      uint8 [K/2, N] then repacked on the device into the kernel layout.
  apply_w4a16_linear(x, w_native, scales, N, K, bias=None)
      x [M, K] @ dequant(w)^T -> [M, N] in x's dtype; takes the place of
      apply_fp8_marlin_linear(x, qw, s, workspace, N, K, None).
  scaled_fp8_quant(x, scale=None, use_per_token_if_dynamic=False) -> (q e4m3 [M, K], scale)
      e4m3 activations (per-tensor dynamic, per-token dynamic or static), and
      cutlass_scaled_mm on e4m3 a / b: the fp8 W8A8 path the reference's dense
      harnesses time (profiling/dense_qwen/bench_l2_boundary.py:54-57, 66-68).
  scaled_fp4_quant(x, global_scale) -> (q uint8 [M, K/2], scales e4m3 [pad(M,128), pad(K/16,4)])
  cutlass_scaled_fp4_mm(a, b, block_scale_a, block_scale_b, alpha, out_dtype)
      NVFP4 in vLLM's call shapes and tensor formats (the reference's native-FP4
      path, profiling/cuda_validation/bench_moe_nvfp4_native.py:97-108).
"""

from __future__ import annotations

try:
    from . import _bootstrap  # noqa: F401
except ImportError:
    import _bootstrap  # noqa: F401

import torch

from cb200 import _lib as L
from cb200 import ops
from cb200.weights import kmajor_int8_for


def _per_row(scale: torch.Tensor, n: int, what: str) -> torch.Tensor:
    s = scale.reshape(-1)
    if s.dtype != torch.float32:
        raise ValueError(f"{what} must be fp32")
    if s.numel() == 1:
        return s.expand(n).contiguous()
    if s.numel() != n:
        raise ValueError(f"{what} must have 1 or {n} elements, got {s.numel()}")
    return s.contiguous()


def cutlass_scaled_mm(a: torch.Tensor, b: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor,
                      out_dtype: torch.dtype, bias: torch.Tensor | None = None) -> torch.Tensor:
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("cutlass_scaled_mm expects 2-D a [M, K] and b [K, N]")
    if a.dtype == torch.float8_e4m3fn and b.dtype == torch.float8_e4m3fn:
        return _scaled_mm_fp8(a, b, scale_a, scale_b, out_dtype, bias)
    if a.dtype != torch.int8 or b.dtype != torch.int8:
        raise ValueError("this drop-in implements the int8 and e4m3 paths (a and b both int8 or both e4m3)")
    M, K = a.shape
    Kb, N = b.shape
    if Kb != K:
        raise ValueError(f"shape mismatch: a {tuple(a.shape)} b {tuple(b.shape)}")
    if out_dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("out_dtype must be bfloat16 or float16")
    w_nk = b.t() if b.stride(0) == 1 else kmajor_int8_for(b)  # column-major b is K-major storage
    if bias is not None and (bias.numel() != N or bias.dtype not in (torch.bfloat16, torch.float16, torch.float32)):
        raise ValueError(f"bias must have N={N} elements of a floating dtype")
    # vLLM adds the bias in its fp32 epilogue, before the one rounding to out_dtype; so does the kernel
    return ops.w8a8_gemm(a, w_nk, _per_row(scale_a, M, "scale_a"), _per_row(scale_b, N, "scale_b"),
                         out_dtype=out_dtype, bias=None if bias is None else bias.reshape(N).contiguous())


def _scaled_mm_fp8(a, b, scale_a, scale_b, out_dtype, bias):
    M, K = a.shape
    Kb, N = b.shape
    if Kb != K:
        raise ValueError(f"shape mismatch: a {tuple(a.shape)} b {tuple(b.shape)}")
    if out_dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("out_dtype must be bfloat16 or float16")
    if b.stride(0) != 1:
        raise ValueError("b must be the column-major [K, N] view of a K-major [N, K] e4m3 weight (as vLLM takes it)")
    sa, sb = scale_a.reshape(-1).float().contiguous(), scale_b.reshape(-1).float().contiguous()
    if sa.numel() not in (1, M) or sb.numel() not in (1, N):
        raise ValueError("scale_a must be per-tensor or per-token, scale_b per-tensor or per-channel")
    if bias is not None and (bias.numel() != N or bias.dtype not in (torch.bfloat16, torch.float16, torch.float32)):
        raise ValueError(f"bias must have N={N} elements of a floating dtype")
    return ops.fp8_gemm(a, b.t(), sa, sb, out_dtype=out_dtype,
                        bias=None if bias is None else bias.reshape(N).contiguous())


def scaled_fp8_quant(x: torch.Tensor, scale: torch.Tensor | None = None, num_token_padding=None, scale_ub=None,
                     use_per_token_if_dynamic: bool = False, output=None):
    """vLLM's scaled_fp8_quant: e4m3 values and the fp32 scale ([1] per tensor, [M, 1] per token).
    Dynamic scale = max(amax / 448, 1 / (448 * 512)); q = e4m3(clamp(x / scale, +-448))."""
    if num_token_padding is not None or scale_ub is not None:
        raise NotImplementedError("token padding and scale upper bounds are not provided")
    if x.dim() != 2:
        raise ValueError("x must be [M, K]")
    if scale is not None:
        q, s = ops.quant_act_fp8(x, "static", scale=scale.reshape(1).float().contiguous(), q=output)
        return q, s.view(1)
    if use_per_token_if_dynamic:
        q, s = ops.quant_act_fp8(x, "per_token", q=output)
        return q, s.view(-1, 1)
    q, s = ops.quant_act_fp8(x, "per_tensor", q=output)
    return q, s.view(1)


def scaled_int8_quant(x: torch.Tensor, scale: torch.Tensor | None = None, azp=None, symmetric: bool = True):
    if scale is not None or azp is not None or not symmetric:
        raise NotImplementedError("only dynamic symmetric per-token int8 quantization is provided")
    q, s = ops.quant_act_i8(x)
    return q, s.view(-1, 1), None


def quantize_w4a16(w: torch.Tensor, group_size: int = 128, return_dequant: bool = False):
    if w.dim() != 2:
        raise ValueError("w must be [N, K]")
    N, K = w.shape
    if K % group_size or group_size % 128:
        raise ValueError("K must be a multiple of group_size, and group_size a multiple of 128")
    sdt = w.dtype if w.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16
    wf = w.float().t().reshape(K // group_size, group_size, N)  # [G, g, N]
    # the scale is rounded to its storage dtype first, so q * s is exactly what the kernel multiplies
    s = torch.clamp(wf.abs().amax(dim=1) / 7.0, min=1e-8).to(sdt).float()  # [G, N]
    qf = torch.clamp(torch.round(wf / s[:, None, :]), -8, 7)
    q = qf.to(torch.int16).reshape(K, N)
    packed = ((q[0::2] & 0xF) | ((q[1::2] & 0xF) << 4)).to(torch.uint8).contiguous()  # [K/2, N]
    native = ops.repack_w4(packed, L.CB_W4_REF_U8_KN, K, N)
    scales = s.to(sdt).contiguous()
    if return_dequant:  # [K, N] in the scales' dtype: q * s rounded once, as the kernel's operand
        return native, scales, (qf * s[:, None, :]).reshape(K, N).to(sdt)
    return native, scales


def apply_w4a16_linear(x: torch.Tensor, w_native: torch.Tensor, scales: torch.Tensor, N: int, K: int,
                       bias: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    if x.shape[-1] != K:
        raise ValueError(f"x has K={x.shape[-1]}, expected {K}")
    groups = scales.shape[0] if scales.dim() == 2 else 1
    group_size = K // groups
    x2 = x.reshape(-1, K)
    y = ops.w4a16_gemm(x2, w_native, scales, N, group_size, out=out, out_dtype=x.dtype)
    if bias is not None:
        y += bias.to(y.dtype)
    return y.reshape(*x.shape[:-1], N)


def scaled_fp4_quant(x: torch.Tensor, input_global_scale: torch.Tensor):
    """NVFP4 quantization of ``x`` [M, K] (vLLM ``scaled_fp4_quant``): packed e2m1
    values uint8 [M, K/2] and the swizzled e4m3 scales, viewed as float8_e4m3fn
    [pad(M, 128), pad(K/16, 4)]."""
    q, sf = ops.nvfp4_quantize(x, input_global_scale.reshape(1).to(torch.float32))
    return q, sf.view(torch.float8_e4m3fn)


def cutlass_scaled_fp4_mm(a: torch.Tensor, b: torch.Tensor, block_scale_a: torch.Tensor, block_scale_b: torch.Tensor,
                          alpha: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
    """``alpha * A @ B^T`` for NVFP4 ``a`` [M, K/2] and ``b`` [N, K/2] with their
    swizzled scales (vLLM ``cutlass_scaled_fp4_mm``)."""
    return ops.nvfp4_gemm(a, block_scale_a.view(torch.uint8), b, block_scale_b.view(torch.uint8),
                          alpha.reshape(1).to(torch.float32), out_dtype=out_dtype)
