"""Drop-in for profiling/w8a8/w8a8_bmm.py (cache-barrier), backed by libcb200.

Same names and arguments as the reference:
  quantize_weights_w8(w)                 (:84-89)
  quantize_acts_w8(a, q=None, s=None)    (:92-106)   -> libcb200 act-quant kernel
  _pick_config(M)                        (:109-115)  -> this kernel's tiling, as hints
  w8a8_bmm(aq, wq, a_scale, w_scale, out=None, **hints)  (:118-140) -> tcgen05 kind::i8 GEMM
  w8a8_bmm_full(a, wq, w_scale, bufs=None)              (:143-149) -> quant + GEMM, PDL-chained

Weights: ``quantize_weights_w8`` returns the reference's [H, K, N] int8 values as
a view of K-major [H, N, K] storage (the kernel's operand layout), so no repack
is needed later. A weight given as plain N-contiguous [H, K, N] is repacked
once on the device and cached on the tensor (outside CUDA-graph capture).
"""

from __future__ import annotations

try:
    from . import _bootstrap  # noqa: F401
except ImportError:
    import _bootstrap  # noqa: F401

import torch

from cb200 import ops
from cb200.weights import kmajor_int8_for


def quantize_weights_w8(w: torch.Tensor):
    """[H, K, N] -> (int8 [H, K, N] view of K-major storage, fp32 scales [H, N]).

    Per-(H, N) symmetric int8: s = amax_K |w| / 127 (clamped at 1e-8),
    q = round_half_even(w / s) clamped to [-127, 127], in fp32.
    """
    wf = w.float()
    s = torch.clamp(wf.abs().amax(dim=1) / 127.0, min=1e-8)
    q = torch.clamp(torch.round(wf / s.unsqueeze(1)), -127, 127).to(torch.int8)
    if q.is_cuda:
        q = ops.repack_w8_kmajor(q).transpose(1, 2)
    return q, s.contiguous()


def quantize_acts_w8(a: torch.Tensor, q=None, s=None):
    """[H, M, K] -> (int8 [H, M, K], fp32 [H*M]); fills q/s in place when given."""
    return ops.quant_act_i8(a, q, s)


def _pick_config(M):
    """Tile description of the sm_100a kernel for M tokens (keys as the reference's).

    BLOCK_M is the token tile (MMA N), BLOCK_N the 128 weight rows per tile
    (MMA M), BLOCK_K one 128-byte swizzle row of int8. The values are hints;
    w8a8_bmm ignores tile overrides.
    """
    tn = 16 if M <= 16 else 32 if M <= 32 else 64 if M <= 64 else 128 if M <= 128 else 256
    stages = max(2, min(16, (200 * 1024) // (128 * 128 + tn * 128)))
    return dict(BLOCK_M=tn, BLOCK_N=128, BLOCK_K=128, num_warps=6, num_stages=stages)


def w8a8_bmm(aq, wq, a_scale, w_scale, out=None, BLOCK_M=None, BLOCK_N=None, BLOCK_K=None, num_warps=None,
             num_stages=None):
    """``out[h] = (aq[h] @ wq[h])_int32 * a_scale[h*M + m] * w_scale[h, n]`` -> fp16 (reference)."""
    del BLOCK_M, BLOCK_N, BLOCK_K, num_warps, num_stages
    H, M, K = aq.shape
    N = wq.shape[2]
    w_nk = kmajor_int8_for(wq)
    if out is None:
        out = torch.empty(H, M, N, dtype=torch.float16, device=aq.device)
    return ops.w8a8_gemm(aq, w_nk, a_scale, w_scale, out=out)


def w8a8_bmm_full(a, wq, w_scale, bufs=None):
    """Dynamic act quant + INT8 BMM. ``bufs=(q, s, out)`` for graph capture."""
    q = s = out = None
    if bufs is not None:
        q, s, out = bufs
    H, M, K = a.shape
    N = wq.shape[2]
    w_nk = kmajor_int8_for(wq)
    if out is None:
        out = torch.empty(H, M, N, dtype=torch.float16, device=a.device)
    return ops.w8a8_gemm_dynamic(a, w_nk, w_scale, q=q, s=s, out=out)
