"""The numerical method of the one- and two-token W4A16 GEMV, checked on the
CPU through its restatement in the oracle: the 15-bit fixed-point image of an
activation row, its exact split into two int8 halves, the worst-case rounding
error (half a fixed-point step, at most 2^-14 of the row's amax), and the
result against the exact product with and without a K split."""

import numpy as np
import pytest

from oracle import quant_oracle as O


def _acts(rng, M, K):
    a = rng.standard_normal((M, K)).astype(np.float32)
    a[:, ::7] *= 1e-3          # small values
    a[:, 5] = 0.0              # zeros
    a[0, :] *= 37.0            # a row with a large amax
    return O.bf16_bits_to_f32(O.f32_to_bf16_bits(a))  # bf16 activations


def test_split_is_exact_and_in_range():
    rng = np.random.default_rng(0)
    a = _acts(rng, 3, 1000)
    X, hi, lo, e = O.w4a16_fixed_point_parts(a, 0, 1000)
    assert np.array_equal(256 * hi + lo, X)
    assert lo.min() >= -128 and lo.max() <= 127
    assert np.abs(hi).max() <= 64
    amax_scaled = np.abs(a).max(axis=1) * np.exp2(e.astype(np.float64))
    assert (amax_scaled >= 2.0 ** 13).all() and (amax_scaled < 2.0 ** 14).all()


def test_rounding_error_bound_is_two_to_minus_14_of_amax():
    rng = np.random.default_rng(1)
    worst = 0.0
    for _ in range(20):
        a = _acts(rng, 2, 512)
        X, _, _, e = O.w4a16_fixed_point_parts(a, 0, 512)
        err = np.abs(np.ldexp(X.astype(np.float64), -e[:, None]) - a.astype(np.float64))
        rel = (err / np.abs(a).max(axis=1, keepdims=True)).max()
        worst = max(worst, rel)
    assert worst <= 2.0 ** -14
    # the bound is attained up to a factor < 2: rows whose amax sits just above a
    # power of two see errors beyond 2^-15 of it
    a = np.full((1, 64), 0.3, dtype=np.float32)
    a[0, 0] = 1.0 + 2.0 ** -10  # amax just above 1: 2^e * amax just above 2^13
    X, _, _, e = O.w4a16_fixed_point_parts(a, 0, 64)
    err = np.abs(np.ldexp(X.astype(np.float64), -e[:, None]) - a.astype(np.float64)).max()
    assert err > 2.0 ** -15 * float(np.abs(a).max())


@pytest.mark.parametrize("group", [128, 1 << 30])
@pytest.mark.parametrize("ksplit", [1, 3])
def test_gemv_restatement_matches_exact_product(group, ksplit):
    rng = np.random.default_rng(2 + ksplit)
    M, K, N = 2, 1000, 96
    a = _acts(rng, M, K)
    q = rng.integers(-8, 8, size=(K, N))
    G = -(-K // min(group, K))
    s = (np.abs(rng.standard_normal((G, N))) * 0.02 / 7 + 1e-4).astype(np.float32)
    got = O.w4a16_fixed_point_gemv(a, q, s, group, ksplit=ksplit)
    w = q.astype(np.float64) * np.repeat(s.astype(np.float64), min(group, K), axis=0)[:K]
    ref = a.astype(np.float64) @ w
    assert np.abs(got - ref).max() <= 1e-3 * np.abs(ref).max()
