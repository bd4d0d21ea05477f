"""The oracle against golden vectors made by the reference's own code
(tests/golden/make_golden.py runs its Triton kernels under the interpreter)."""

import numpy as np
import pytest

from oracle import quant_oracle as O

W4A16_FIXTURES = ["w4a16_h2_t3_k256_n192.npz", "w4a16_h4_t1_k128_n256.npz", "w4a16_h2_t17_k512_n128.npz"]
W8A8_FIXTURES = ["w8a8_h2_m5_k256_n192.npz", "w8a8_h1_m1_k512_n256.npz", "w8a8_h2_m33_k128_n64_bf16.npz"]


def _acts(d):
    if bool(d["a_is_bf16_bits"]):
        return O.bf16_bits_to_f32(d["a"].view(np.uint16))
    return d["a"].astype(np.float32)


def test_quantize_weights_int4_bit_exact(golden):
    d = golden("w4a16_h2_t3_k256_n192.npz")
    q, s = O.quantize_weights_int4(d["w"])
    assert np.array_equal(O.pack_u8_kn(q), d["packed"])
    assert np.array_equal(s.view(np.uint16), d["scales"].view(np.uint16))


@pytest.mark.parametrize("name", W4A16_FIXTURES)
@pytest.mark.parametrize("kernel", ["c_simple", "c_v1", "c_v3"])
def test_w4a16_per_channel_matches_reference_kernels(golden, name, kernel):
    d = golden(name)
    q = O.unpack_u8_kn(d["packed"])
    ref = O.w4a16_per_channel(d["x"].astype(np.float32), q, d["scales"].astype(np.float32))
    out = O.round_to(ref, "f16").astype(np.float32)
    got = d[kernel].astype(np.float32)
    # fp32 accumulation order is the only difference: at most 1 fp16 ulp here.
    assert np.abs(out - got).max() <= 2.0 ** -10 * np.abs(got).max()
    assert (out.view(np.uint32) == got.view(np.uint32)).mean() > 0.999


@pytest.mark.parametrize("name", W8A8_FIXTURES)
def test_w8a8_matches_reference_bit_exact(golden, name):
    d = golden(name)
    q, s = O.quant_act_i8(_acts(d))
    assert np.array_equal(q, d["q"])
    assert np.array_equal(s.reshape(-1).view(np.uint32), d["s"].view(np.uint32))
    if "w" in d:
        wq, ws = O.quantize_weights_w8(d["w"])
        assert np.array_equal(wq, d["wq"])
        assert np.array_equal(ws.view(np.uint32), d["wscale"].view(np.uint32))
    acc = O.gemm_i8_i32(d["q"], d["wq"])
    out = O.w8a8_epilogue(acc, d["s"].reshape(acc.shape[0], -1), d["wscale"], "f16")
    assert np.array_equal(out.view(np.uint16), d["out"].view(np.uint16))


def test_act_quant_ties_and_zero_rows(golden):
    d = golden("act_quant_ties.npz")
    q, s = O.quant_act_i8(d["a"].astype(np.float32))
    assert np.array_equal(q, d["q"])
    assert np.array_equal(s.reshape(-1).view(np.uint32), d["s"].view(np.uint32))
    # half away from zero on exact .5 ties
    assert list(q[0, 0, :5]) == [127, 3, -3, 1, -1]


def test_w4a4_reference_wrap_and_signed(golden):
    d = golden("w4a4_m5_k256_n96.npz")
    # the reference kernel's uint8 arithmetic: reproduced bit for bit
    assert np.array_equal(O.w4a4_gemm(d["a_packed"], d["b_packed"], wrap=True), d["c"])
    # the signed reading differs wherever a negative nibble is present
    signed = O.w4a4_gemm(d["a_packed"], d["b_packed"], wrap=False)
    assert not np.array_equal(signed, d["c"])
    assert np.abs(signed).max() <= 64 * 256


@pytest.mark.parametrize("B,K,N", [(1, 128, 128), (2, 256, 192), (1, 384, 130), (3, 136, 72), (1, 8, 8)])
def test_layout_codecs_round_trip(B, K, N):
    rng = np.random.default_rng(K * N + B)
    q = rng.integers(-8, 8, size=(B, K, N)).astype(np.int8)
    assert np.array_equal(O.unpack_u8_kn(O.pack_u8_kn(q)), q)
    assert np.array_equal(O.unpack_i32_k8n(O.pack_i32_k8n(q)), q)
    nat = O.pack_native(q)
    assert nat.nbytes == B * (-(-N // 128)) * (-(-K // 128)) * 8192
    assert np.array_equal(O.unpack_native(nat, B, K, N), q)


def test_native_layout_word_order():
    # one tile, row 0: k = 0..7 -> nibble order k0,k2,k4,k6,k1,k3,k5,k7 in word 0
    q = np.zeros((1, 128, 128), dtype=np.int8)
    q[0, :8, 0] = [1, 2, 3, 4, 5, 6, -7, -8]
    words = O.pack_native(q).view(np.uint32)
    expect = 0
    for pos, k in enumerate([0, 2, 4, 6, 1, 3, 5, 7]):
        expect |= (int(q[0, k, 0]) & 0xF) << (4 * pos)
    assert words[0] == expect
    # row 2 chunk 0 is stored at chunk position (2 >> 1) & 3 = 1
    q2 = np.zeros((1, 128, 128), dtype=np.int8)
    q2[0, 0, 2] = 5
    w2 = O.pack_native(q2).view(np.uint32).reshape(128, 16)
    assert w2[2, 4] == 5 and w2[2, 0] == 0


def test_bf16_rounding_helper():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e38, 1e-30], dtype=np.float32)
    b = O.f32_to_bf16_bits(x)
    assert list(b[:4]) == [0x3F80, 0x3F80, 0x3F81, 0xC020]
    back = O.bf16_bits_to_f32(b)
    assert np.all(np.abs(back - x) <= np.abs(x) * 2.0 ** -8)


@pytest.mark.parametrize("name", ["bf16_r5_k256_amax", "f16_r3_k128_g1", "bf16_r130_k64_g37"])
def test_nvfp4_quant_matches_vllm_reference(golden, name):
    """Values and scales of vLLM's ref_nvfp4_quant (the arithmetic of the reference's
    native-FP4 path), reproduced exactly."""
    d = golden(f"nvfp4_quant_{name}.npz")
    x = O.bf16_bits_to_f32(d["x_bits"]) if bool(d["x_is_bf16"]) else d["x_bits"].view(np.float16).astype(np.float32)
    packed, s_bits, nib = O.nvfp4_quant(x, float(d["gs"]))
    assert np.array_equal(O.e2m1_to_f32(nib), d["q_values"])
    assert np.array_equal(O.e4m3_bits_to_f32(s_bits), d["scales"])
    # the packed bytes hold element 2i in the low nibble
    assert np.array_equal(packed & 0xF, nib[:, 0::2]) and np.array_equal(packed >> 4, nib[:, 1::2])


def test_nvfp4_swizzle_matches_vllm_layout(golden):
    d = golden("nvfp4_swizzle.npz")
    rows, K = int(d["rows"]), int(d["K"])
    assert np.array_equal(O.nvfp4_unswizzle(d["swizzled"], rows, K), d["linear"])
    again = O.nvfp4_unswizzle(O.nvfp4_swizzle(d["linear"]), rows, K)
    assert np.array_equal(again, d["linear"])


def test_e4m3_rounding_matches_torch_float8():
    import torch
    x = np.concatenate([np.linspace(0, 448, 20001, dtype=np.float32),
                        (2.0 ** np.linspace(-12, 8.8, 10001)).astype(np.float32)])
    bits, val = O.e4m3_round(x)
    t = torch.from_numpy(x).to(torch.float8_e4m3fn)
    assert np.array_equal(bits, t.view(torch.uint8).numpy())
    assert np.array_equal(val, t.float().numpy())
    assert np.array_equal(O.e4m3_bits_to_f32(bits), val)


def test_nvfp4_gemm_oracle_is_dequant_matmul():
    rng = np.random.default_rng(3)
    a = rng.standard_normal((3, 128)).astype(np.float32)
    b = rng.standard_normal((5, 128)).astype(np.float32)
    ap, asf, _ = O.nvfp4_quant(a, 2.0)
    bp, bsf, _ = O.nvfp4_quant(b, 3.0)
    out = O.nvfp4_gemm(ap, asf, bp, bsf, 1.0 / 6.0)
    ref = (O.nvfp4_dequant(ap, asf) @ O.nvfp4_dequant(bp, bsf).T) * np.float64(np.float32(1.0 / 6.0))
    assert np.array_equal(out, ref)
    # dequantized values approximate x * gs (fp4 relative error < 1/3 per element, scale rounding aside)
    assert np.abs(O.nvfp4_dequant(ap, asf) - a * 2.0).max() <= 0.5 * np.abs(a * 2.0).max()


def test_fp8_oracle_pinned_to_torch_e4m3():
    """oracle.fp8_quant's e4m3 rounding (round to nearest even, saturate at 448,
    sign kept on values that round to zero) equals torch's float8_e4m3fn
    conversion on the CPU, and the per-token scale is max(amax / 448, 1 / (448 * 512))."""
    import torch
    rng = np.random.default_rng(17)
    x = (rng.standard_normal((7, 513)) * np.exp(rng.uniform(-12, 8, (7, 1)))).astype(np.float32)
    x[0, :8] = [-1e-9, 1e-9, -0.0, 0.0, 1e6, -1e6, 896.0, -3e-5]
    x[1] = 0.0
    bits, vals, scale = O.fp8_quant(x)
    amax = np.abs(x).max(axis=1)
    assert np.array_equal(scale, np.maximum((amax / np.float32(448)).astype(np.float32), np.float32(1 / (448 * 512))))
    y = np.clip((x / scale[:, None]).astype(np.float32), -448, 448)
    t = torch.from_numpy(y).to(torch.float8_e4m3fn)
    assert np.array_equal(t.view(torch.uint8).numpy(), bits)
    assert np.array_equal(t.float().numpy(), vals)
    assert np.array_equal(O.e4m3_bits_to_f32(bits), vals)
