"""W8A8 parity on the GPU, through the C ABI: activation quantization and the
int32 accumulators are bit-exact against the oracle, and so is the scaled
output (same fp32 multiplication order, one rounding)."""

import numpy as np
import pytest
import torch

from _gpu_helpers import oracle_bits, oracle_dtype, out_bits, to_np_f32
from oracle import quant_oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [  # (B, M, N, K)
    (1, 1, 256, 512),
    (1, 16, 128, 128),
    (1, 17, 192, 256),
    (2, 5, 192, 256),
    (1, 32, 1024, 4096),
    (1, 33, 640, 1280),
    (3, 64, 256, 384),
    (1, 100, 520, 272),
    (1, 256, 256, 1024),
    (1, 300, 384, 512),
    (128, 1, 512, 128),
    (64, 32, 512, 128),    # short K: one k-block per tile, two epilogue groups
    (16, 20, 1024, 256),   # two k-blocks per tile
    (1, 64, 1280, 2560),   # 64-token tiles with scales from the shared-memory ring, cut tiles
    (1, 8, 8192, 8192),
    # one token per batch entry (the dp4a path): every row-blocking branch,
    # K tails inside a k-step, row blocks that cross batch entries
    (3, 1, 37, 48),
    (1, 1, 333, 160),
    (2, 1, 100, 272),
    (2, 1, 130, 784),
    (1, 1, 300, 1552),
    (1, 1, 520, 4112),
    (1, 1, 1000, 8208),
    # two tokens per batch entry (the dp4a path's two-token kernels)
    (3, 2, 37, 48),
    (2, 2, 130, 784),
    (1, 2, 520, 4112),
]


def _inputs(B, M, N, K, seed, act_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(B, M, K, generator=g).to(act_dtype)
    wq = torch.randint(-127, 128, (B, K, N), generator=g, dtype=torch.int32).to(torch.int8)
    ws = (torch.randn(B, N, generator=g) * 0.01).abs().float() + 1e-4
    return a, wq, ws


@pytest.mark.parametrize("B,M,N,K", SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_w8a8_bit_exact(cuda_device, B, M, N, K, out_dtype):
    from cb200 import ops
    a, wq, ws = _inputs(B, M, N, K, seed=B * 1000003 + M * 1009 + N * 7 + K)
    ref_q, ref_s = O.quant_act_i8(to_np_f32(a))
    ref_acc = O.gemm_i8_i32(ref_q, wq.numpy())
    ref_out = O.w8a8_epilogue(ref_acc, ref_s, ws.numpy(), oracle_dtype(out_dtype))

    a_d = a.to(cuda_device)
    q, s = ops.quant_act_i8(a_d)
    w_nk = ops.repack_w8_kmajor(wq.to(cuda_device))
    acc = torch.full((B, M, N), -7, dtype=torch.int32, device=cuda_device)
    out = ops.w8a8_gemm(q, w_nk, s, ws.to(cuda_device), out_dtype=out_dtype, acc_out=acc)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), ref_q)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), ref_s.reshape(-1).view(np.uint32))
    assert np.array_equal(acc.cpu().numpy(), ref_acc)
    ref_bits = ref_out if out_dtype == torch.bfloat16 else ref_out.view(np.uint16)
    assert np.array_equal(out_bits(out), ref_bits)
    assert ops.device_status(cuda_device) == 0


@pytest.mark.parametrize("B,M,N,K", [(1, 1, 8192, 8192), (1, 32, 8192, 8192), (2, 17, 640, 1280),
                                     (1, 2, 1000, 4112), (1, 1, 333, 160), (1, 1, 96, 1024)])
def test_w8a8_dynamic_equals_two_step(cuda_device, B, M, N, K):
    from cb200 import ops
    a, wq, ws = _inputs(B, M, N, K, seed=77 + M)
    a_d, ws_d = a.to(cuda_device), ws.to(cuda_device)
    w_nk = ops.repack_w8_kmajor(wq.to(cuda_device))
    q, s = ops.quant_act_i8(a_d)
    two = ops.w8a8_gemm(q, w_nk, s, ws_d, out_dtype=torch.bfloat16)
    one = ops.w8a8_gemm_dynamic(a_d, w_nk, ws_d, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(one.view(torch.int16), two.view(torch.int16))
    ref_out, _, _, _ = O.w8a8_dynamic(to_np_f32(a), wq.numpy(), ws.numpy(), "bf16")
    assert np.array_equal(out_bits(one), ref_out)


@pytest.mark.parametrize("M,K,act_dtype", [(1, 1024, torch.bfloat16), (1, 256, torch.float16),
                                           (1, 8192, torch.bfloat16), (2, 1040, torch.float16)])
def test_w8a8_dynamic_fused_quant_outputs(cuda_device, M, K, act_dtype):
    """One token of one GEMM with K <= 1024 quantizes inside the GEMV; with it
    and with the separate quantizer (longer rows, two tokens) the q and scale
    buffers the caller passes receive the quantizer's exact values, and a
    second call with new activations overwrites them."""
    from cb200 import ops
    N = 520
    d = cuda_device
    q = torch.full((M, K), 99, dtype=torch.int8, device=d)
    s = torch.full((M,), -1.0, dtype=torch.float32, device=d)
    for seed in (41, 42):
        a, wq, ws = _inputs(1, M, N, K, seed=seed, act_dtype=act_dtype)
        w_nk = ops.repack_w8_kmajor(wq[0].to(d))
        out = ops.w8a8_gemm_dynamic(a[0].to(d), w_nk, ws[0].to(d), q=q, s=s, out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        ref_out, ref_q, ref_s, _ = O.w8a8_dynamic(to_np_f32(a), wq.numpy(), ws.numpy(), "bf16")
        assert np.array_equal(q.cpu().numpy(), ref_q.reshape(M, K))
        assert np.array_equal(s.cpu().numpy().view(np.uint32), ref_s.reshape(-1).view(np.uint32))
        assert np.array_equal(out_bits(out), ref_out.reshape(M, N))
    assert ops.device_status(d) == 0


def test_w8a8_one_token_batched_bias(cuda_device):
    """One token per batch entry with a per-entry bias [B, N] and f32 output."""
    from cb200 import ops
    B, M, N, K = 3, 1, 70, 1040
    a, wq, ws = _inputs(B, M, N, K, seed=31)
    bias = torch.randn(B, N, generator=torch.Generator().manual_seed(32)).to(torch.bfloat16)
    d = cuda_device
    q, s = ops.quant_act_i8(a.to(d))
    w_nk = ops.repack_w8_kmajor(wq.to(d))
    acc = torch.empty(B, M, N, dtype=torch.int32, device=d)
    out = ops.w8a8_gemm(q, w_nk, s, ws.to(d), out_dtype=torch.float32, acc_out=acc, bias=bias.to(d))
    torch.cuda.synchronize()
    ref_q, ref_s = O.quant_act_i8(to_np_f32(a))
    ref_acc = O.gemm_i8_i32(ref_q, wq.numpy())
    assert np.array_equal(acc.cpu().numpy(), ref_acc)
    ref = O.w8a8_epilogue(ref_acc, ref_s, ws.numpy(), "f32", bias=to_np_f32(bias))
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_w8a8_strided_output_and_canary(cuda_device):
    """Output with a padded row stride: the kernel writes only the [M, N] window."""
    from cb200 import ops
    B, M, N, K, pad = 2, 7, 200, 256, 24
    a, wq, ws = _inputs(B, M, N, K, seed=5)
    a_d = a.to(cuda_device)
    q, s = ops.quant_act_i8(a_d)
    w_nk = ops.repack_w8_kmajor(wq.to(cuda_device))
    big = torch.full((B, M + 1, N + pad), 12345.0, dtype=torch.float32, device=cuda_device)
    view = big[:, :M, :N]
    ops.w8a8_gemm(q, w_nk, s, ws.to(cuda_device), out=view)
    torch.cuda.synchronize()
    ref_q, ref_s = O.quant_act_i8(to_np_f32(a))
    ref = O.w8a8_epilogue(O.gemm_i8_i32(ref_q, wq.numpy()), ref_s, ws.numpy(), "f32")
    got = big.cpu().numpy()
    assert np.array_equal(got[:, :M, :N].view(np.uint32), ref.view(np.uint32))
    assert (got[:, :M, N:] == 12345.0).all() and (got[:, M:, :] == 12345.0).all()


def test_w8a8_golden_reference_outputs(cuda_device, golden):
    """The reference kernel's own fp16 outputs (Triton interpreter), reproduced bit for bit."""
    import w8a8_bmm
    for name in ("w8a8_h2_m5_k256_n192.npz", "w8a8_h1_m1_k512_n256.npz", "w8a8_h2_m33_k128_n64_bf16.npz"):
        d = golden(name)
        if bool(d["a_is_bf16_bits"]):
            a = torch.from_numpy(d["a"]).view(torch.bfloat16)
        else:
            a = torch.from_numpy(d["a"])
        a_d = a.to(cuda_device)
        wq = torch.from_numpy(d["wq"]).to(cuda_device)
        wsc = torch.from_numpy(d["wscale"]).to(cuda_device)
        q, s = w8a8_bmm.quantize_acts_w8(a_d)
        out = w8a8_bmm.w8a8_bmm(q, wq, s, wsc)
        full = w8a8_bmm.w8a8_bmm_full(a_d, wq, wsc)
        torch.cuda.synchronize()
        assert np.array_equal(q.cpu().numpy(), d["q"])
        assert np.array_equal(s.cpu().numpy().view(np.uint32), d["s"].view(np.uint32))
        assert out.dtype == torch.float16
        assert np.array_equal(out_bits(out), d["out"].view(np.uint16))
        assert np.array_equal(out_bits(full), d["out"].view(np.uint16))


def test_w8a8_act_quant_ties(cuda_device, golden):
    from cb200 import ops
    d = golden("act_quant_ties.npz")
    q, s = ops.quant_act_i8(torch.from_numpy(d["a"]).to(cuda_device))
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), d["q"])
    assert np.array_equal(s.cpu().numpy().view(np.uint32), d["s"].view(np.uint32))


def test_w8a8_graph_capture_replay(cuda_device):
    """The ops run inside a captured CUDA graph (static buffers, no allocation)."""
    from cb200 import ops
    B, M, N, K = 1, 16, 1024, 2048
    a, wq, ws = _inputs(B, M, N, K, seed=11)
    a_d, ws_d = a.to(cuda_device), ws.to(cuda_device)
    w_nk = ops.repack_w8_kmajor(wq.to(cuda_device))
    q = torch.empty(B, M, K, dtype=torch.int8, device=cuda_device)
    s = torch.empty(B * M, dtype=torch.float32, device=cuda_device)
    out = torch.empty(B, M, N, dtype=torch.bfloat16, device=cuda_device)
    ops.w8a8_gemm_dynamic(a_d, w_nk, ws_d, q=q, s=s, out=out)  # allocates the workspace
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(3):
            ops.w8a8_gemm_dynamic(a_d, w_nk, ws_d, q=q, s=s, out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    ref_out, _, _, _ = O.w8a8_dynamic(to_np_f32(a), wq.numpy(), ws.numpy(), "bf16")
    assert np.array_equal(out_bits(out), ref_out)
    assert ops.device_status(cuda_device) == 0
