"""Offline weight packer and on-disk format (cb200.wformat), on the CPU."""

import numpy as np
import pytest
import torch

from oracle import quant_oracle as O


@pytest.fixture(scope="module")
def W():
    from cb200 import wformat

    return wformat


@pytest.mark.parametrize("B,K,N", [(1, 256, 128), (2, 384, 200), (3, 128, 5)])
def test_native_int4_matches_oracle(W, B, K, N):
    rng = np.random.default_rng(B * K + N)
    q = rng.integers(-8, 8, size=(B, K, N)).astype(np.int8)
    ref = O.pack_native(q).reshape(-1).view(np.uint8)
    assert np.array_equal(W.native_int4(O.pack_u8_kn(q), W.W4_REF_U8_KN, K, N), ref)
    assert np.array_equal(W.native_int4(O.pack_i32_k8n(q), W.W4_I32_K8N, K, N), ref)
    # and it decodes back to the signed values
    assert np.array_equal(O.unpack_native(W.native_int4(O.pack_u8_kn(q), W.W4_REF_U8_KN, K, N), B, K, N), q)


def test_kmajor_int8(W):
    w = np.random.default_rng(1).integers(-127, 128, size=(2, 64, 48)).astype(np.int8)
    assert np.array_equal(W.kmajor_int8(w), w.transpose(0, 2, 1))
    assert W.kmajor_int8(w[0]).shape == (1, 48, 64)


def test_save_load_round_trip(W, tmp_path):
    rng = np.random.default_rng(7)
    q = rng.integers(-8, 8, size=(2, 256, 192)).astype(np.int8)
    s4 = torch.rand(2, 2, 192).to(torch.bfloat16)
    p4 = W.pack_int4(O.pack_u8_kn(q), W.W4_REF_U8_KN, 256, 192, s4, 128)
    w8 = rng.integers(-127, 128, size=(1, 64, 32)).astype(np.int8)
    p8 = W.pack_int8(w8, np.abs(rng.standard_normal((1, 32))).astype(np.float32))
    raw = np.arange(10, dtype=np.float16)
    path = tmp_path / "w.cbw"
    W.save(str(path), {"layers.0.qkv": p4, "layers.0.o": p8, "norm": raw}, meta={"model": "test"})
    got = W.load(str(path))
    assert np.array_equal(got["layers.0.qkv"].native, p4.native)
    assert (got["layers.0.qkv"].K, got["layers.0.qkv"].N, got["layers.0.qkv"].group_size) == (256, 192, 128)
    assert np.array_equal(got["layers.0.qkv"].scales, s4.view(torch.int16).numpy().view(np.uint16))
    assert np.array_equal(got["layers.0.o"].w_nk, w8.transpose(0, 2, 1))
    assert np.array_equal(got["layers.0.o"].scales, p8.scales)
    assert np.array_equal(got["norm"], raw)
    # torch tensors on a device (CPU here) come back with their dtype, bf16 included
    gt = W.load(str(path), device="cpu")
    assert gt["layers.0.qkv"].scales.dtype == torch.bfloat16 and torch.equal(gt["layers.0.qkv"].scales, s4)


def test_corruption_detected(W, tmp_path):
    path = tmp_path / "w.cbw"
    W.save(str(path), {"x": np.arange(1000, dtype=np.int32)})
    data = bytearray(path.read_bytes())
    data[-10] ^= 0xFF
    path.write_bytes(bytes(data))
    with pytest.raises(ValueError):
        W.load(str(path))
    path.write_bytes(b"XXXX" + bytes(data[4:]))
    with pytest.raises(ValueError):
        W.load(str(path))
