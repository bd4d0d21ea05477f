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
    """max |got - ref| / max |ref| (normwise maximum relative error)."""
    denom = float(np.abs(ref).max())
    return float(np.abs(got - ref).max()) / (denom if denom > 0 else 1.0)


def rel_l2(got: np.ndarray, ref: np.ndarray) -> float:
    denom = float(np.linalg.norm(ref))
    return float(np.linalg.norm(got - ref)) / (denom if denom > 0 else 1.0)
