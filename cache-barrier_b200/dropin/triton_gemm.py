"""Drop-in for kernels/triton_gemm.py (cache-barrier): the packed W4A4 GEMM
``triton_gemm_packed_int4`` (:395-485), backed by libcb200 (int4 operands
unpacked to 8 bit, then the tcgen05 kind::i8 GEMM with int32 accumulation and an
fp32 store).

Results: by default this module reproduces what the reference kernel computes.
That kernel subtracts 16 from nibbles >= 8 on a uint8 tensor (:164-167), which
wraps to 240..255 instead of giving -8..-1; ``signed=True`` selects the two's
complement reading its docstring (:407-411) and its own check (:492-520) intend,
which is also the default of ``cb200.ops.w4a4_gemm``. No Triton is involved.
"""

from __future__ import annotations

try:
    from . import _bootstrap  # noqa: F401
except ImportError:
    import _bootstrap  # noqa: F401

import torch

from cb200 import ops


def _bucket_m(m: int):
    """M buckets of the reference's static-config table (:273-280)."""
    if m <= 1:
        return "m1"
    if m <= 4:
        return "small"
    if m <= 8:
        return "medium"
    return None


def _shape_family(n: int, k: int) -> str:
    """Shape families of the reference's static-config table (:283-290)."""
    if n > k:
        return "ffn_up"
    if n == k:
        return "q_proj"
    if n <= 1280:
        return "kv_proj"
    return "ffn_down"


def triton_gemm_packed_int4(A_packed: torch.Tensor, B_packed: torch.Tensor, K: int, BLOCK_M=None, BLOCK_N=None,
                            BLOCK_K=None, GROUP_SIZE_M=None, num_warps=None, num_stages=None,
                            use_static_config=True, signed=False) -> torch.Tensor:
    """GEMM with packed INT4 (2 values per byte): A [M, K//2] uint8, B [K//2, N] uint8 -> fp32 [M, N].

    Tile arguments are accepted and ignored (the kernel tiles itself).
    """
    del BLOCK_M, BLOCK_N, BLOCK_K, GROUP_SIZE_M, num_warps, num_stages, use_static_config
    assert A_packed.is_cuda and B_packed.is_cuda, "All tensors must be on GPU"
    assert A_packed.dtype == torch.uint8 and B_packed.dtype == torch.uint8
    assert K % 2 == 0, "K must be even for packed INT4"
    M, Kp = A_packed.shape
    Kb, N = B_packed.shape
    assert Kp == K // 2 and Kb == K // 2
    return ops.w4a4_gemm(A_packed, B_packed, K, reference_wrap=not signed)
