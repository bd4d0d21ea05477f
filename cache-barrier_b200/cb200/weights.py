"""Quantized weight containers and layout caches.

``Int4Weight`` holds int4 weights in the kernel-native tiled layout plus their
group scales; ``Int8Weight`` holds K-major int8 weights plus per-channel scales.
Both are built on the device from the reference layouts (profiling/bench_l2_barrier.py:92-99
uint8 [.., K/2, N]; an int32 [.., K/8, N] packing; profiling/w8a8/w8a8_bmm.py:84-89
int8 [.., K, N]) by the library's repack kernels.

``native_int4_for`` / ``kmajor_int8_for`` give drop-in callers that hold only a
reference-layout tensor the native copy, repacked once and cached on the tensor
(invalidated when the tensor is modified in place). The first call must happen
outside CUDA-graph capture.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib as L
from . import ops


def _capturing() -> bool:
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


def native_int4_for(packed: torch.Tensor, K: int, N: int, layout: int = L.CB_W4_REF_U8_KN) -> torch.Tensor:
    """Native-layout copy of reference-layout int4 weights, cached on ``packed``."""
    cached = getattr(packed, "_cb_native_w4", None)
    key = (packed.data_ptr(), packed._version, tuple(packed.shape), tuple(packed.stride()), K, N, layout)
    if cached is not None and cached[0] == key:
        return cached[1]
    if _capturing():
        raise RuntimeError("int4 weights must be repacked before CUDA graph capture: call the GEMM once first")
    native = ops.repack_w4(packed, layout, K, N)
    packed._cb_native_w4 = (key, native)
    return native


def kmajor_int8_for(w_kn: torch.Tensor) -> torch.Tensor:
    """[B, N, K] K-major view/copy of int8 weights given as [B, K, N]."""
    w3 = w_kn if w_kn.dim() == 3 else w_kn.unsqueeze(0)
    if w3.stride(1) == 1:  # already K-major storage: [B, K, N] view of [B, N, K]
        v = w3.transpose(1, 2)
        return v if w_kn.dim() == 3 else v[0]
    cached = getattr(w_kn, "_cb_kmajor_w8", None)
    key = (w_kn.data_ptr(), w_kn._version, tuple(w_kn.shape), tuple(w_kn.stride()))
    if cached is not None and cached[0] == key:
        return cached[1]
    if _capturing():
        raise RuntimeError("int8 weights must be repacked before CUDA graph capture: call the GEMM once first")
    nk = ops.repack_w8_kmajor(w_kn)
    w_kn._cb_kmajor_w8 = (key, nk)
    return nk


@dataclass
class Int4Weight:
    """int4 weights [B, K, N] in the native layout with scales [B, K/group, N]."""

    native: torch.Tensor
    scales: torch.Tensor
    K: int
    N: int
    batch: int
    group_size: int

    @classmethod
    def from_packed(cls, packed: torch.Tensor, scales: torch.Tensor, K: int, group_size: int,
                    layout: int = L.CB_W4_REF_U8_KN) -> "Int4Weight":
        p3 = packed if packed.dim() == 3 else packed.unsqueeze(0)
        N = p3.shape[2]
        s3 = scales
        if s3.dim() == 1:
            s3 = s3.view(1, 1, -1)
        elif s3.dim() == 2:
            s3 = s3.unsqueeze(0) if group_size < K else s3.unsqueeze(1)
        native = ops.repack_w4(p3, layout, K, N)
        return cls(native, s3.contiguous(), K, N, p3.shape[0], group_size)

    def matmul(self, x: torch.Tensor, out: torch.Tensor | None = None,
               out_dtype: torch.dtype | None = None) -> torch.Tensor:
        return ops.w4a16_gemm(x, self.native, self.scales, self.N, self.group_size, out=out, out_dtype=out_dtype)

    @property
    def nbytes(self) -> int:
        return self.native.numel() + self.scales.numel() * self.scales.element_size()


@dataclass
class Int8Weight:
    """int8 weights stored K-major [B, N, K] with fp32 per-channel scales [B, N]."""

    w_nk: torch.Tensor
    scales: torch.Tensor

    @classmethod
    def from_kn(cls, q_kn: torch.Tensor, scales: torch.Tensor) -> "Int8Weight":
        return cls(kmajor_int8_for(q_kn).contiguous(), scales.float().contiguous())

    @property
    def K(self) -> int:
        return self.w_nk.shape[-1]

    @property
    def N(self) -> int:
        return self.w_nk.shape[-2]

    def matmul_dynamic(self, x: torch.Tensor, q: torch.Tensor | None = None, s: torch.Tensor | None = None,
                       out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        return ops.w8a8_gemm_dynamic(x, self.w_nk, self.scales, q=q, s=s, out=out, out_dtype=out_dtype)

    @property
    def nbytes(self) -> int:
        return self.w_nk.numel() + self.scales.numel() * 4
