"""CPU baseline timings — TEST/MEASUREMENT INFRASTRUCTURE ONLY.

Times the oracle's restatement of the reference's CPU-runnable path on the host
cores: the W8A8 path (per-token quantization, exact int GEMM through float64
BLAS, fp32 epilogue, bf16 cast; profiling/w8a8/w8a8_bmm.py:35-41, 78) and the
W4A16 explicit dequant + matmul (profiling/gate/bench_capacity_gate.py:235-244,
restated for bf16 and group-size-128 scales). Only bench.py's CPU-baseline leg
and its reference arm call this module.
"""

from __future__ import annotations

import os
import statistics
import time

import numpy as np

from . import quant_oracle as O


def blas_threads(n: int | None = None):
    """Limit BLAS threads to n (default: all cores); returns (controller, n)."""
    n = n or os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits
        ctl = threadpool_limits(limits=n)
    except Exception:  # noqa: BLE001
        ctl = None
    return ctl, n


class W8A8Cpu:
    """Reference W8A8 CPU path on fixed synthetic inputs (weights prepared once)."""

    def __init__(self, K: int, N: int, seed: int = 0):
        rng = np.random.default_rng(seed)
        self.K, self.N = K, N
        wq = rng.integers(-127, 128, size=(K, N), dtype=np.int64)
        self.w64 = wq.astype(np.float64)  # exact carrier for int8 values
        self.w_scale = (np.abs(rng.standard_normal(N)) * 0.01).astype(np.float32) + np.float32(1e-4)
        self.rng = rng

    def acts(self, T: int) -> np.ndarray:
        a = self.rng.standard_normal((T, self.K)).astype(np.float32)
        return O.bf16_bits_to_f32(O.f32_to_bf16_bits(a))  # bf16-valued

    def gemm(self, a: np.ndarray) -> np.ndarray:
        q, s = O.quant_act_i8(a)
        acc = np.matmul(q.astype(np.float64), self.w64)
        f = (acc.astype(np.float32) * s[:, None]).astype(np.float32) * self.w_scale[None, :]
        return O.f32_to_bf16_bits(f)


class W4A16Cpu:
    """Reference explicit-dequant W4A16 CPU path (g128 bf16 scales)."""

    def __init__(self, K: int, N: int, group: int = 128, seed: int = 0):
        rng = np.random.default_rng(seed)
        self.K, self.N, self.group = K, N, group
        self.q = rng.integers(-8, 8, size=(K, N)).astype(np.int8)
        s = (np.abs(rng.standard_normal((K // group, N))) * 0.02 / 7).astype(np.float32)
        self.scales = O.bf16_bits_to_f32(O.f32_to_bf16_bits(s))
        self.rng = rng

    def acts(self, T: int) -> np.ndarray:
        a = self.rng.standard_normal((T, self.K)).astype(np.float32)
        return O.bf16_bits_to_f32(O.f32_to_bf16_bits(a))

    def gemm(self, a: np.ndarray) -> np.ndarray:
        w = O.dequant_w4(self.q, self.scales, self.group)  # dequant is part of the timed path
        return O.f32_to_bf16_bits(np.matmul(a, w))


def time_path(path, tokens, reps: int = 5, warmup: int = 1):
    """Median seconds per GEMM for each T in tokens; returns (mean over T, per-T dict)."""
    per_t = {}
    for T in tokens:
        a = path.acts(T)
        for _ in range(warmup):
            path.gemm(a)
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            path.gemm(a)
            ts.append(time.perf_counter() - t0)
        per_t[T] = statistics.median(ts)
    return sum(per_t.values()) / len(per_t), per_t
