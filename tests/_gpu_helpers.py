"""Shared helpers for the GPU parity tests (torch <-> numpy views, seeded inputs)."""

import numpy as np
import torch

from oracle import quant_oracle as O


def to_np_f32(t: torch.Tensor) -> np.ndarray:
    """Device/CPU tensor (f16/bf16/f32) -> exact fp32 numpy values."""
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return O.bf16_bits_to_f32(t.view(torch.int16).numpy().view(np.uint16))
    return t.float().numpy()


def out_bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy().view(np.uint32)


def oracle_bits(x_f32: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    if dtype == torch.bfloat16:
        return O.round_to(x_f32, "bf16")
    if dtype == torch.float16:
        return O.round_to(x_f32, "f16").view(np.uint16)
    return np.asarray(x_f32, dtype=np.float32).view(np.uint32)


def oracle_dtype(dtype: torch.dtype) -> str:
    return {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[dtype]


def max_rel(got: np.ndarray, ref: np.ndarray) -> float:
    """max |got - ref| / max |ref|: the norm-wise (infinity-norm) maximum relative
    error. Looser than an element-wise bound; see elementwise_close."""
    denom = float(np.abs(ref).max())
    return float(np.abs(got - ref).max()) / (denom if denom > 0 else 1.0)


def rel_l2(got: np.ndarray, ref: np.ndarray) -> float:
    denom = float(np.linalg.norm(ref))
    return float(np.linalg.norm(got - ref)) / (denom if denom > 0 else 1.0)


def elementwise_close(got: np.ndarray, ref: np.ndarray, rtol: float, atol) -> bool:
    """Element-wise relative error bound with an absolute term:
    |got - ref| <= rtol * |ref| + atol for every element (atol a scalar or an
    array shaped like ref).

    A pure element-wise relative error is undefined for outputs that cancel to
    near zero; the W4A16 tests pass atol = u * (|a| @ |w|), the rigorous bound on
    what rounding the dequantized weight operand to the activation dtype (unit
    roundoff u: 2^-8 for bf16, 2^-11 for f16) can change in each output."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return bool(np.all(np.abs(got - ref) <= rtol * np.abs(ref) + atol))


def operand_rounding_bound(a_f32: np.ndarray, w_f32: np.ndarray, dtype) -> np.ndarray:
    """u * (|a| @ |w|): the largest change that rounding each weight operand
    element w to `dtype` (relative error <= u) can make to each output of a @ w."""
    u = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    return u * np.matmul(np.abs(np.asarray(a_f32, np.float64)), np.abs(np.asarray(w_f32, np.float64)))
