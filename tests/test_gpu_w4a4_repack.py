"""W4A4 and the weight-repack kernels on the GPU, through the C ABI (exact)."""

import numpy as np
import pytest
import torch

from oracle import quant_oracle as O

pytestmark = pytest.mark.gpu


def test_w4a4_reference_outputs_bit_exact(cuda_device, golden):
    import triton_gemm
    d = golden("w4a4_m5_k256_n96.npz")
    a = torch.from_numpy(d["a_packed"]).to(cuda_device)
    b = torch.from_numpy(d["b_packed"]).to(cuda_device)
    c = triton_gemm.triton_gemm_packed_int4(a, b, 256)
    torch.cuda.synchronize()
    assert c.dtype == torch.float32
    assert np.array_equal(c.cpu().numpy(), d["c"])


@pytest.mark.parametrize("M,N,K", [(1, 64, 64), (5, 96, 256), (16, 1024, 4096), (33, 200, 512), (300, 256, 1024)])
def test_w4a4_signed_exact(cuda_device, M, N, K):
    from cb200 import ops
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randint(0, 256, (M, K // 2), generator=g, dtype=torch.int32).to(torch.uint8)
    b = torch.randint(0, 256, (K // 2, N), generator=g, dtype=torch.int32).to(torch.uint8)
    c = ops.w4a4_gemm(a.to(cuda_device), b.to(cuda_device), K)
    wrap = ops.w4a4_gemm(a.to(cuda_device), b.to(cuda_device), K, reference_wrap=True)
    torch.cuda.synchronize()
    assert np.array_equal(c.cpu().numpy(), O.w4a4_gemm(a.numpy(), b.numpy()))
    # exact while the wrapped integer sums stay below 2**24
    if 255 * 255 * K < 2 ** 24:
        assert np.array_equal(wrap.cpu().numpy(), O.w4a4_gemm(a.numpy(), b.numpy(), wrap=True))


@pytest.mark.parametrize("B,K,N", [(1, 128, 128), (2, 256, 192), (1, 384, 130), (3, 136, 72), (1, 8192, 1024)])
def test_repack_w4_matches_native_codec(cuda_device, B, K, N):
    from cb200 import _lib as L
    from cb200 import ops
    rng = np.random.default_rng(K + N)
    q = rng.integers(-8, 8, size=(B, K, N)).astype(np.int8)
    expect = O.pack_native(q)
    got_u8 = ops.repack_w4(torch.from_numpy(O.pack_u8_kn(q)).to(cuda_device), L.CB_W4_REF_U8_KN, K, N)
    assert np.array_equal(got_u8.cpu().numpy(), expect)
    if K % 8 == 0:
        got_i32 = ops.repack_w4(torch.from_numpy(O.pack_i32_k8n(q)).to(cuda_device), L.CB_W4_I32_K8N, K, N)
        assert np.array_equal(got_i32.cpu().numpy(), expect)


@pytest.mark.parametrize("B,K,N", [(1, 64, 96), (3, 100, 33), (1, 8192, 8192)])
def test_repack_w8_kmajor(cuda_device, B, K, N):
    from cb200 import ops
    w = torch.randint(-127, 128, (B, K, N), dtype=torch.int32).to(torch.int8)
    nk = ops.repack_w8_kmajor(w.to(cuda_device))
    assert torch.equal(nk.cpu(), w.transpose(1, 2).contiguous())


def test_quantize_weights_w8_gpu_view_layout(cuda_device, golden):
    """On the GPU torch divides by the scalar 127 through a reciprocal multiply
    (as the reference's own quantizer does when it runs on CUDA), so a scale may
    differ from the CPU golden by one ulp; given the scales, q is exact."""
    import w8a8_bmm
    d = golden("w8a8_h2_m5_k256_n192.npz")
    q, s = w8a8_bmm.quantize_weights_w8(torch.from_numpy(d["w"]).to(cuda_device))
    assert q.shape == d["wq"].shape and q.stride(1) == 1  # K-major storage
    s_np = s.cpu().numpy()
    ulp = np.abs(s_np.view(np.int32).astype(np.int64) - d["wscale"].view(np.int32).astype(np.int64))
    assert ulp.max() <= 1
    expect = np.clip(np.rint(d["w"].astype(np.float32) / s_np[:, None, :]), -127, 127).astype(np.int8)
    assert np.array_equal(q.cpu().numpy(), expect)
    assert (q.cpu().numpy() == d["wq"]).mean() > 0.999


def test_host_packer_matches_device_repack_and_runs(cuda_device, tmp_path):
    """The offline packer (cb200.wformat) writes the bytes cb_repack_w4 produces;
    weights loaded from a file run in the W4A16 GEMM with identical results."""
    from cb200 import _lib as L
    from cb200 import ops, wformat

    rng = np.random.default_rng(3)
    B, K, N, T = 2, 384, 200, 5
    q = rng.integers(-8, 8, size=(B, K, N)).astype(np.int8)
    packed = O.pack_u8_kn(q)
    dev_native = ops.repack_w4(torch.from_numpy(packed).to(cuda_device), L.CB_W4_REF_U8_KN, K, N)
    s = torch.from_numpy((np.abs(rng.standard_normal((B, K // 128, N))) * 0.01 + 1e-3).astype(np.float32)).to(torch.bfloat16)
    p = wformat.pack_int4(packed, wformat.W4_REF_U8_KN, K, N, s, 128)
    assert np.array_equal(p.native, dev_native.cpu().numpy())
    wformat.save(str(tmp_path / "w.cbw"), {"w": p})
    got = wformat.load(str(tmp_path / "w.cbw"), device=cuda_device)["w"]
    a = torch.randn(B, T, K, device=cuda_device).to(torch.bfloat16)
    o1 = ops.w4a16_gemm(a, dev_native, s.to(cuda_device), N, 128)
    o2 = ops.w4a16_gemm(a, got.native, got.scales, N, 128)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
