"""CPU oracle for the quantized-GEMM hot path — TEST INFRASTRUCTURE ONLY.

This module restates the cache-barrier reference arithmetic in numpy. It is the
checker for the CUDA kernels: only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import it. No product code path calls it.

Pinning: every function below is checked in ``tests/test_oracle_golden.py``
against golden vectors produced by the reference's own code (its Triton kernels
run under Triton's CPU interpreter and its PyTorch quantizers), committed in
``tests/golden/`` together with the script that generated them
(``tests/golden/make_golden.py``). The group-size-128 W4A16 extension has no
reference implementation; its restatement follows the reference's explicit
dequant (profiling/gate/bench_capacity_gate.py:235-244) with the scale indexed
per group, and that case alone is "parity unpinned" beyond the per-channel
pinning.

The fixed-point restatement of the one- and two-token W4A16 GEMV
(``w4a16_fixed_point_parts`` / ``w4a16_fixed_point_gemv``) has no counterpart in
the reference: it states this library's own numerical method, and
``tests/test_oracle_fixed_point.py`` checks it against the exact product.

Exactness: integer GEMMs are computed as float64 matmuls of int8-valued arrays,
which is exact while every partial sum stays below 2**53 (|sum| <= 127*127*K for
K < 5e11).
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# bf16 helpers (numpy has no bfloat16): values are carried as uint16 bit patterns.
# ---------------------------------------------------------------------------


def f32_to_bf16_bits(x) -> np.ndarray:
    """Round fp32 to bf16, round-to-nearest-even, NaN kept quiet."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), out)
    return out


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_to(x, dtype: str) -> np.ndarray:
    """fp32 -> output dtype: 'f16' (np.float16), 'bf16' (uint16 bits) or 'f32'."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f16":
        return x.astype(np.float16)
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    if dtype == "f32":
        return x
    raise ValueError(dtype)


def as_f32(x, dtype: str) -> np.ndarray:
    """Inverse view of round_to: stored values -> fp32."""
    if dtype == "bf16":
        return bf16_bits_to_f32(x)
    return np.asarray(x, dtype=np.float32)


# ---------------------------------------------------------------------------
# Weight quantizers
# ---------------------------------------------------------------------------


def quantize_weights_int4(W: np.ndarray):
    """Per-output-channel symmetric int4, restating quantize_weights_int4
    (profiling/bench_l2_barrier.py:92-99) for fp16 W of shape [..., K, N].

    fp16 arithmetic as torch performs it (each op computed in fp32 and rounded to
    fp16): amax over K, clamp(min=1e-8), /7, W/scale, round half to even, clamp
    to [-8, 7]. Returns (q int8 [..., K, N], scale fp16 [..., N]).
    """
    W = np.asarray(W, dtype=np.float16)
    w_max = np.abs(W).max(axis=-2, keepdims=True)
    w_max = np.where(w_max.astype(np.float32) < np.float32(1e-8), np.float16(1e-8), w_max).astype(np.float16)
    scale = (w_max.astype(np.float32) / np.float32(7.0)).astype(np.float16)
    ratio = (W.astype(np.float32) / scale.astype(np.float32)).astype(np.float16)
    q = np.clip(np.rint(ratio.astype(np.float32)), -8, 7).astype(np.int8)
    return q, scale[..., 0, :]


def quantize_weights_w8(w: np.ndarray):
    """Per-(H, N) symmetric int8, restating quantize_weights_w8
    (profiling/w8a8/w8a8_bmm.py:84-89): s = amax_K(|w|)/127 clamped at 1e-8,
    q = round_half_even(w / s) clamped to [-127, 127], all in fp32."""
    wf = np.asarray(w, dtype=np.float32)
    s = (np.abs(wf).max(axis=-2) / np.float32(127.0)).astype(np.float32)
    s = np.maximum(s, np.float32(1e-8))
    q = np.clip(np.rint(wf / s[..., None, :]), -127, 127).astype(np.int8)
    return q, s


# ---------------------------------------------------------------------------
# W8A8
# ---------------------------------------------------------------------------


def quant_act_i8(a_f32: np.ndarray):
    """Per-row symmetric int8 of a [..., K] (fp32 view of f16/bf16 input),
    restating _quant_act_kernel (profiling/w8a8/w8a8_bmm.py:35-41):
    scale = max(amax/127, 1e-8); q = trunc(a/scale + 0.5*sign(a)) with
    sign(0) = +1, IEEE-rounded fp32 division and addition.
    Returns (q int8 [..., K], scale fp32 [...])."""
    a = np.asarray(a_f32, dtype=np.float32)
    amax = np.abs(a).max(axis=-1)
    scale = np.maximum(amax / np.float32(127.0), np.float32(1e-8)).astype(np.float32)
    half = np.where(a >= 0, np.float32(0.5), np.float32(-0.5))
    y = (a / scale[..., None]).astype(np.float32) + half
    q = np.trunc(y.astype(np.float32)).astype(np.int8)
    return q, scale


def gemm_i8_i32(aq: np.ndarray, wq_kn: np.ndarray) -> np.ndarray:
    """Exact int32 accumulators sum_k aq[..., m, k] * wq[..., k, n]."""
    acc = np.matmul(aq.astype(np.float64), wq_kn.astype(np.float64))
    assert np.abs(acc).max(initial=0) < 2.0**31
    return acc.astype(np.int32)


def w8a8_epilogue(acc: np.ndarray, a_scale: np.ndarray, w_scale: np.ndarray, out_dtype: str,
                  bias: np.ndarray | None = None) -> np.ndarray:
    """((float)acc * a_scale[m]) * w_scale[n], then cast (profiling/w8a8/w8a8_bmm.py:78-81).
    acc [B, M, N] int32, a_scale [B, M] fp32, w_scale [B, N] fp32.
    With ``bias`` ([B, N] or [N], values exactly representable in fp32) the bias
    is added in fp32 before the cast, where vLLM's cutlass_scaled_mm adds it (the
    call of profiling/dense_qwen/bench_l2_boundary.py:66-71)."""
    f = acc.astype(np.float32)
    f = (f * a_scale.astype(np.float32)[..., :, None]).astype(np.float32)
    f = (f * w_scale.astype(np.float32)[..., None, :]).astype(np.float32)
    if bias is not None:
        f = (f + np.asarray(bias, dtype=np.float32)[..., None, :]).astype(np.float32)
    return round_to(f, out_dtype)


def w8a8_dynamic(a_f32: np.ndarray, wq_kn: np.ndarray, w_scale: np.ndarray, out_dtype: str):
    """Act quant + int GEMM + epilogue (w8a8_bmm_full, profiling/w8a8/w8a8_bmm.py:143-149).
    Returns (out, q, a_scale, acc)."""
    q, s = quant_act_i8(a_f32)
    acc = gemm_i8_i32(q, wq_kn)
    return w8a8_epilogue(acc, s, w_scale, out_dtype), q, s, acc


# ---------------------------------------------------------------------------
# W4A16
# ---------------------------------------------------------------------------


def dequant_w4(q: np.ndarray, scales: np.ndarray, group_size: int) -> np.ndarray:
    """w[k, n] = q[k, n] * s[k // group_size, n] in fp32 (exact: 4-bit x <=24-bit).
    q [..., K, N] int, scales [..., G, N] float."""
    K = q.shape[-2]
    gidx = np.arange(K) // group_size
    s = np.asarray(scales, dtype=np.float32)[..., gidx, :]
    return q.astype(np.float32) * s


def w4a16_gemm(a_f32: np.ndarray, q: np.ndarray, scales: np.ndarray, group_size: int) -> np.ndarray:
    """fp32 result of a @ dequant(q, scales), accumulated in float64 (then fp32).
    Explicit-dequant restatement of profiling/gate/bench_capacity_gate.py:235-244."""
    w = dequant_w4(q, scales, group_size).astype(np.float64)
    return np.matmul(np.asarray(a_f32, dtype=np.float64), w).astype(np.float32)


def w4a16_per_channel(a_f32: np.ndarray, q: np.ndarray, scale_n: np.ndarray) -> np.ndarray:
    """kernel_batched_w4a16_simple's order: scale applied once to the accumulator
    (profiling/bench_l2_barrier.py:78-82). scale_n [..., N]."""
    acc = np.matmul(np.asarray(a_f32, dtype=np.float64), q.astype(np.float64))
    return (acc.astype(np.float32) * np.asarray(scale_n, dtype=np.float32)[..., None, :]).astype(np.float32)


def w4a16_fixed_point_parts(a_f32: np.ndarray, group_k0: int, group_k1: int):
    """The one- and two-token GEMV's activation image of a[:, k0:k1] (one CTA's
    k-range): exponent e per token from the range's amax (2^13 <= amax * 2^e <
    2^14), X = rint(a * 2^e) and its exact split X = 256 * hi + lo with lo in
    [-128, 127]. Returns (X, hi, lo, e) with X/hi/lo int64 [M, k1 - k0]."""
    a = np.asarray(a_f32, dtype=np.float32)[:, group_k0:group_k1]
    amax = np.abs(a).max(axis=1) if a.shape[1] else np.zeros(a.shape[0], np.float32)
    _, E = np.frexp(amax)
    e = np.where(amax > 0, 14 - E, 0).astype(np.int64)
    X = np.rint(np.ldexp(a.astype(np.float64), e[:, None])).astype(np.int64)  # exact scaling, round half even
    hi = (X + 128) >> 8
    lo = X - 256 * hi
    return X, hi, lo, e


def w4a16_fixed_point_gemv(a_f32: np.ndarray, q: np.ndarray, scales: np.ndarray, group_size: int,
                           ksplit: int = 1) -> np.ndarray:
    """Restatement of the dp4a GEMV's arithmetic (one or two tokens): per K-split
    part, exact integer sums S_j = sum_k q * X over each 128-k block, accumulated
    as acc += s_j * S_j (fp32, per-group scales; a per-channel scale multiplies
    the sum instead), scaled by 2^-e of the part, parts added in order.
    a [M, K] fp32, q [K, N] int in [-8, 7], scales [G, N]. fp32 [M, N]."""
    a = np.asarray(a_f32, dtype=np.float32)
    M, K = a.shape
    N = q.shape[1]
    KB = -(-K // 128)
    per_channel = group_size >= K
    s = np.asarray(scales, dtype=np.float32)
    out = np.zeros((M, N), dtype=np.float32)
    for ks in range(ksplit):
        kb0, kb1 = ks * KB // ksplit, (ks + 1) * KB // ksplit
        X, _, _, e = w4a16_fixed_point_parts(a, kb0 * 128, min(kb1 * 128, K))
        acc = np.zeros((M, N), dtype=np.float32)
        for j in range(kb0, kb1):
            k0, k1 = j * 128, min(j * 128 + 128, K)
            S = X[:, k0 - kb0 * 128:k1 - kb0 * 128] @ q[k0:k1].astype(np.int64)  # exact
            sc = np.float32(1.0) if per_channel else s[(j * 128) // group_size]
            acc = (acc.astype(np.float64) + np.float64(1.0) * sc * S.astype(np.float64)).astype(np.float32)
        if per_channel and ksplit == 1:
            acc = (acc * s[0]).astype(np.float32)
        part = np.ldexp(acc, -e[:, None]).astype(np.float32)
        out = (out + part).astype(np.float32)
    if per_channel and ksplit > 1:
        out = (out * s[0]).astype(np.float32)
    return out


# ---------------------------------------------------------------------------
# W4A4
# ---------------------------------------------------------------------------


def unpack_rows_i4(packed: np.ndarray, wrap: bool = False) -> np.ndarray:
    """uint8 [M, K/2] (k = 2i low nibble, 2i+1 high) -> int16 [M, K]
    (kernels/triton_gemm.py:159-167). Nibbles >= 8 become v - 16 (signed int4), or,
    with ``wrap``, (v - 16) mod 256 = 240..255: the reference kernel subtracts 16
    on a uint8 tensor, which wraps."""
    lo = (packed & 0xF).astype(np.int16)
    hi = (packed >> 4).astype(np.int16)
    off = 240 if wrap else -16
    lo = np.where(lo >= 8, lo + off, lo)
    hi = np.where(hi >= 8, hi + off, hi)
    out = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), dtype=np.int16)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


def w4a4_gemm(a_packed: np.ndarray, b_packed: np.ndarray, wrap: bool = False) -> np.ndarray:
    """fp32 C = A @ B over unpacked nibbles; exact integer sums, rounded once to fp32
    (kernels/triton_gemm.py:159-176). ``wrap`` selects the reference kernel's
    uint8-wrap reading of negative nibbles (see unpack_rows_i4)."""
    a = unpack_rows_i4(a_packed, wrap)
    b = unpack_rows_i4(np.ascontiguousarray(b_packed.T), wrap).T  # B [K/2, N] packs k along rows
    return np.matmul(a.astype(np.float64), b.astype(np.float64)).astype(np.float32)


# ---------------------------------------------------------------------------
# int4 layout codecs
# ---------------------------------------------------------------------------


def pack_u8_kn(q: np.ndarray) -> np.ndarray:
    """int [..., K, N] in [-8, 7] -> uint8 [..., K/2, N], even k in the low nibble
    (profiling/bench_l2_barrier.py:96-98)."""
    q = np.asarray(q).astype(np.int16)
    even = (q[..., 0::2, :] & 0xF).astype(np.uint8)
    odd = (q[..., 1::2, :] & 0xF).astype(np.uint8)
    return (even | (odd << 4)).astype(np.uint8)


def unpack_u8_kn(p: np.ndarray) -> np.ndarray:
    lo = (p & 0xF).astype(np.int16)
    hi = (p >> 4).astype(np.int16)
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    K2 = p.shape[-2]
    out = np.empty(p.shape[:-2] + (2 * K2, p.shape[-1]), dtype=np.int8)
    out[..., 0::2, :] = lo
    out[..., 1::2, :] = hi
    return out


def pack_i32_k8n(q: np.ndarray) -> np.ndarray:
    """int [..., K, N] -> int32 [..., K/8, N]; nibble j of word (k/8, n) = q[8*(k/8)+j]."""
    q = np.asarray(q).astype(np.int64) & 0xF
    K = q.shape[-2]
    w = np.zeros(q.shape[:-2] + (K // 8, q.shape[-1]), dtype=np.uint32)
    for j in range(8):
        w |= (q[..., j::8, :].astype(np.uint32) << np.uint32(4 * j))
    return w.view(np.int32)


def unpack_i32_k8n(w: np.ndarray) -> np.ndarray:
    u = np.asarray(w).view(np.uint32)
    K8 = u.shape[-2]
    out = np.empty(u.shape[:-2] + (K8 * 8, u.shape[-1]), dtype=np.int8)
    for j in range(8):
        v = ((u >> np.uint32(4 * j)) & 0xF).astype(np.int16)
        out[..., j::8, :] = np.where(v >= 8, v - 16, v)
    return out


_NATIVE_POS = np.array([0, 4, 1, 5, 2, 6, 3, 7])  # nibble position of k0..k7 (order k0,k2,k4,k6,k1,k3,k5,k7)


def pack_native(q: np.ndarray) -> np.ndarray:
    """int [B, K, N] -> flat uint8 native tiled layout (include/cb200.h CB_W4_NATIVE)."""
    q = np.asarray(q)
    if q.ndim == 2:
        q = q[None]
    B, K, N = q.shape
    nt, kt = -(-N // 128), -(-K // 128)
    qp = np.zeros((B, kt * 128, nt * 128), dtype=np.int64)
    qp[:, :K, :N] = q
    nib = (qp & 0xF).astype(np.uint32)
    # [B, kt, 128(k), nt, 128(r)] -> [B, nt, kt, r, k]
    t = nib.reshape(B, kt, 128, nt, 128).transpose(0, 3, 1, 4, 2)
    # k = chunk*32 + word*8 + j
    t = t.reshape(B, nt, kt, 128, 4, 4, 8)
    words = np.zeros(t.shape[:-1], dtype=np.uint32)
    for j in range(8):
        words |= t[..., j] << np.uint32(4 * _NATIVE_POS[j])
    # stored chunk position c' = c ^ ((r >> 1) & 3)
    r = np.arange(128)
    out = np.empty_like(words)
    for c in range(4):
        pos = c ^ ((r >> 1) & 3)
        out[:, :, :, r, pos, :] = words[:, :, :, r, c, :]
    return out.reshape(-1).view(np.uint8)


def unpack_native(buf: np.ndarray, B: int, K: int, N: int) -> np.ndarray:
    nt, kt = -(-N // 128), -(-K // 128)
    words = np.asarray(buf).view(np.uint32).reshape(B, nt, kt, 128, 4, 4)
    r = np.arange(128)
    logical = np.empty_like(words)
    for c in range(4):
        pos = c ^ ((r >> 1) & 3)
        logical[:, :, :, r, c, :] = words[:, :, :, r, pos, :]
    vals = np.empty(logical.shape + (8,), dtype=np.int16)
    for j in range(8):
        v = ((logical >> np.uint32(4 * _NATIVE_POS[j])) & 0xF).astype(np.int16)
        vals[..., j] = np.where(v >= 8, v - 16, v)
    # [B, nt, kt, r, chunk, word, j] -> [B, kt*128, nt*128]
    vals = vals.reshape(B, nt, kt, 128, 128).transpose(0, 2, 4, 1, 3).reshape(B, kt * 128, nt * 128)
    return vals[:, :K, :N].astype(np.int8)


def rmsnorm_quant_i8(x_bits_or_f32, weight_f32, eps, dtype="bf16"):
    """Fused RMSNorm + per-token int8 quantization (csrc/rmsnorm_quant.cu):
    r = 1/sqrt(sum x^2 / H + eps) in fp32, y = round_to_dtype(x * r * w), then the
    act-quant rules of quant_act_i8 on y. x is given as float32 values of a
    16-bit tensor [rows, H]. Returns (q int8, scale fp32, y float32 values).
    No reference kernel exists for this fusion (the reference measures it with
    library ops, profiling/mechanisms/RESULTS.md:17); the quantization step is
    the pinned act-quant restatement."""
    x = np.asarray(x_bits_or_f32, dtype=np.float32)
    w = np.asarray(weight_f32, dtype=np.float32)
    H = x.shape[-1]
    ss = np.sum(x * x, axis=-1, dtype=np.float32)
    r = (np.float32(1.0) / np.sqrt(ss / np.float32(H) + np.float32(eps))).astype(np.float32)
    yf = ((x * r[..., None]).astype(np.float32) * w).astype(np.float32)
    y = bf16_bits_to_f32(f32_to_bf16_bits(yf)) if dtype == "bf16" else yf.astype(np.float16).astype(np.float32)
    q, s = quant_act_i8(y)
    return q, s, y


# ---------------------------------------------------------------------------
# NVFP4 (e2m1 values, e4m3 block scales per 16 elements).
# The reference runs this path through vLLM (profiling/cuda_validation/
# bench_moe_nvfp4_native.py:97-108); its arithmetic is vLLM 0.22.0's
# ref_nvfp4_quant / cast_to_fp4 / dequantize_to_dtype
# (vllm/model_executor/layers/quantization/utils/nvfp4_emulation_utils.py:
# 328-453) and the swizzled scale layout of its convert_swizzled_to_linear
# (:348-355). Pinned in tests/test_oracle_golden.py against fixtures made by
# running those vLLM functions on the CPU (tests/golden/make_golden_nvfp4.py).
# ---------------------------------------------------------------------------

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def e4m3_round(x) -> tuple[np.ndarray, np.ndarray]:
    """Non-negative fp32 -> e4m3 (finite, max 448), round to nearest even.
    Returns (bits uint8, value float32)."""
    x = np.minimum(np.asarray(x, dtype=np.float64), 448.0)
    e = np.floor(np.log2(np.maximum(x, 2.0 ** -9)))
    e = np.maximum(e, -6.0)  # subnormals share the exponent of 2^-6
    quantum = np.exp2(e - 3.0)
    v = np.rint(x / quantum) * quantum  # exact: x / quantum and the product are exact in float64
    v = np.minimum(v, 448.0)
    ev = np.floor(np.log2(np.maximum(v, 2.0 ** -9)))
    normal = v >= 2.0 ** -6
    exp_field = np.where(normal, ev + 7.0, 0.0)
    mant = np.where(normal, v / np.exp2(ev) * 8.0 - 8.0, v / 2.0 ** -9)
    bits = np.where(v == 0, 0, exp_field * 8 + mant).astype(np.uint8)
    return bits, v.astype(np.float32)


def fp8_quant(x_f32: np.ndarray, scale=None):
    """e4m3 quantization of activations as vLLM's scaled_fp8_quant (the call of
    profiling/dense_qwen/bench_l2_boundary.py:54-57): per row of x [..., K] when
    ``scale`` is None (scale = max(amax / 448, 1 / (448 * 512)), IEEE fp32
    division), else with the given scale; q = e4m3(clamp(x / scale, +-448)),
    round to nearest even. Returns (bits uint8 like x, values fp32 like x, scale)."""
    x = np.asarray(x_f32, dtype=np.float32)
    if scale is None:
        amax = np.abs(x).max(axis=-1)
        scale = np.maximum((amax / np.float32(448.0)).astype(np.float32), np.float32(1.0 / (448.0 * 512.0)))
        s = scale[..., None]
    else:
        scale = np.asarray(scale, dtype=np.float32)
        s = scale
    y = np.clip((x / s).astype(np.float32), -448.0, 448.0)
    bits, mag = e4m3_round(np.abs(y))
    neg = np.signbit(y)  # the sign survives rounding to zero (-0.0), as the hardware conversion keeps it
    bits = np.where(neg, bits | 0x80, bits).astype(np.uint8)
    vals = np.where(neg, -mag, mag).astype(np.float32)
    return bits, vals, np.asarray(scale, dtype=np.float32)


def fp8_gemm(a_vals: np.ndarray, w_vals_nk: np.ndarray) -> np.ndarray:
    """Exact sum_k a[..., m, k] * w[..., n, k] of e4m3 values (float64: every
    product of two e4m3 values and their sums at these sizes are exact)."""
    return np.matmul(np.asarray(a_vals, np.float64), np.swapaxes(np.asarray(w_vals_nk, np.float64), -1, -2))


def e4m3_bits_to_f32(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    sign = np.where(b & 0x80, -1.0, 1.0)
    exp_field = (b >> 3) & 0xF
    mant = b & 0x7
    v = np.where(exp_field == 0, mant * 2.0 ** -9, (1.0 + mant / 8.0) * np.exp2(exp_field - 7.0))
    return (sign * v).astype(np.float32)


def e2m1_nibbles(y: np.ndarray) -> np.ndarray:
    """fp32 in [-6, 6] -> e2m1 nibble (cast_to_fp4's thresholds, round to nearest
    even; the sign bit follows y's sign, so negative values that round to 0 give 0x8)."""
    y = np.asarray(y, dtype=np.float32)
    a = np.abs(y)
    m = np.select([a <= 0.25, a < 0.75, a <= 1.25, a < 1.75, a <= 2.5, a < 3.5, a <= 5.0], [0, 1, 2, 3, 4, 5, 6], 7)
    sign = np.signbit(y).astype(np.int64) << 3
    return (sign | m).astype(np.uint8)


def e2m1_to_f32(nib: np.ndarray) -> np.ndarray:
    nib = np.asarray(nib, dtype=np.uint8)
    v = E2M1_VALUES[nib & 7]
    return np.where(nib & 8, -v, v).astype(np.float32)


def nvfp4_quant(x_f32: np.ndarray, global_scale: float):
    """ref_nvfp4_quant (nvfp4_emulation_utils.py:439-453) on [rows, K] fp32 inputs
    (exact values of the 16-bit activations). Returns (packed uint8 [rows, K/2],
    scale bits uint8 [rows, K/16] in row-major order, nibbles uint8 [rows, K])."""
    x = np.asarray(x_f32, dtype=np.float32)
    rows, K = x.shape
    gs = np.float32(global_scale)
    blocks = x.reshape(rows, K // 16, 16)
    vmax = np.max(np.abs(blocks), axis=-1).astype(np.float32)
    s = (gs * (vmax * np.float32(1.0 / 6.0)).astype(np.float32)).astype(np.float32)
    s = np.clip(s, -448.0, 448.0).astype(np.float32)
    s_bits, s_val = e4m3_round(s)
    rgs = np.float32(1.0) / (gs + np.float32(1e8) * np.float32(gs == 0))
    t = (s_val * rgs).astype(np.float32)
    o = (np.float32(1.0) / (t + np.float32(1e8) * (t == 0).astype(np.float32))).astype(np.float32)
    y = np.clip((blocks * o[..., None]).astype(np.float32), -6.0, 6.0).reshape(rows, K)
    nib = e2m1_nibbles(y)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    return packed, s_bits, nib


def nvfp4_swizzle(sf_rows_cols: np.ndarray) -> np.ndarray:
    """Row-major scale bytes [rows, C] -> the swizzled atom layout, zero padded to
    [ceil(rows/128)*128, ceil(C/4)*4] (inverse of convert_swizzled_to_linear)."""
    sf = np.asarray(sf_rows_cols, dtype=np.uint8)
    rows, C = sf.shape
    rp, cp = -(-rows // 128) * 128, -(-C // 4) * 4
    full = np.zeros((rp, cp), dtype=np.uint8)
    full[:rows, :C] = sf
    # [m_tiles, 4 (i4), 32 (i3), k_tiles, 4 (i5)] -> [m_tiles, k_tiles, 32, 4, 4]
    t = full.reshape(rp // 128, 4, 32, cp // 4, 4).transpose(0, 3, 2, 1, 4)
    return np.ascontiguousarray(t).reshape(-1)


def nvfp4_unswizzle(buf: np.ndarray, rows: int, K: int) -> np.ndarray:
    C = K // 16
    rp, cp = -(-rows // 128) * 128, -(-C // 4) * 4
    t = np.asarray(buf, dtype=np.uint8)[: rp * cp].reshape(rp // 128, cp // 4, 32, 4, 4).transpose(0, 3, 2, 1, 4)
    return np.ascontiguousarray(t).reshape(rp, cp)[:rows, :C]


def nvfp4_dequant(packed: np.ndarray, sf_bits: np.ndarray) -> np.ndarray:
    """float64 values e2m1 * e4m3 of [rows, K/2] packed values and [rows, K/16]
    row-major scale bits (no global scale)."""
    p = np.asarray(packed, dtype=np.uint8)
    rows = p.shape[0]
    nib = np.empty((rows, p.shape[1] * 2), dtype=np.uint8)
    nib[:, 0::2] = p & 0xF
    nib[:, 1::2] = p >> 4
    v = e2m1_to_f32(nib).astype(np.float64).reshape(rows, -1, 16)
    return (v * e4m3_bits_to_f32(sf_bits).astype(np.float64)[..., None]).reshape(rows, -1)


def nvfp4_gemm(a_packed, a_sf_bits, b_packed, b_sf_bits, alpha: float) -> np.ndarray:
    """out[m, n] = alpha * sum_k A[m, k] B[n, k] in float64 (exact products; the
    kernel accumulates in fp32), returned as float64."""
    A = nvfp4_dequant(a_packed, a_sf_bits)
    B = nvfp4_dequant(b_packed, b_sf_bits)
    return (A @ B.T) * np.float64(np.float32(alpha))
