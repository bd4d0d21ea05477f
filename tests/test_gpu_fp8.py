"""FP8 (e4m3) W8A8 on the GPU through the C ABI: the activation quantizer and the
tcgen05 kind::f8f6f4 GEMM.

  - quantizer: bit-exact against the oracle (oracle.fp8_quant, whose e4m3
    rounding is pinned to torch's float8_e4m3fn conversion on the CPU in
    tests/test_oracle_golden.py) in the per-token dynamic, per-tensor dynamic and
    static modes, scales included;
  - GEMM: fp32 accumulation on the tensor cores of exact e4m3 products; fp32
    output within 1e-5 of the largest output magnitude of the exact float64
    product, 16-bit outputs additionally within one rounding (2^-8 relative);
    per-channel and per-tensor scales, bias, batches, ragged shapes; repeated
    calls bit-identical (the split-K partials are summed in a fixed order);
  - against vLLM's own scaled_fp8_quant / cutlass_scaled_mm on the same inputs
    when vLLM's GPU ops load (the reference's fp8 path): the same scales, >= 99.9 %
    identical quantized values (vLLM multiplies by the reciprocal scale, this
    quantizer divides), and GEMM outputs within bf16 rounding.
"""

import numpy as np
import pytest
import torch

from _gpu_helpers import to_np_f32
from oracle import quant_oracle as O

pytestmark = pytest.mark.gpu


def _acts(B, M, K, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(B, M, K, generator=g) * 3.0
    if M > 2:
        a[:, 1] = 0.0  # an all-zero token
        a[:, 2] *= 1e-3
    return a.to(dtype)


@pytest.mark.parametrize("B,M,K", [(1, 1, 64), (1, 16, 8192), (2, 33, 1000), (3, 5, 256)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fp8_quant_per_token_bit_exact(cuda_device, B, M, K, dtype):
    from cb200 import ops
    a = _acts(B, M, K, dtype, seed=B * 100 + M + K)
    q, s = ops.quant_act_fp8(a.to(cuda_device), "per_token")
    torch.cuda.synchronize()
    bits, _, ref_s = O.fp8_quant(to_np_f32(a))
    assert np.array_equal(s.cpu().numpy().reshape(B, M).view(np.uint32), ref_s.view(np.uint32))
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), bits)


@pytest.mark.parametrize("mode", ["per_tensor", "static"])
def test_fp8_quant_per_tensor_modes(cuda_device, mode):
    from cb200 import ops
    B, M, K = 2, 24, 640
    a = _acts(B, M, K, torch.bfloat16, seed=7)
    af = to_np_f32(a)
    if mode == "static":
        given = np.array([0.05, 0.002], dtype=np.float32)
        q, s = ops.quant_act_fp8(a.to(cuda_device), "static", scale=torch.from_numpy(given).to(cuda_device))
        ref_s = given
    else:
        q, s = ops.quant_act_fp8(a.to(cuda_device), "per_tensor")
        amax = np.abs(af.reshape(B, -1)).max(axis=1)
        ref_s = np.maximum((amax / np.float32(448.0)).astype(np.float32), np.float32(1.0 / (448.0 * 512.0)))
    torch.cuda.synchronize()
    assert np.array_equal(s.cpu().numpy().view(np.uint32), ref_s.view(np.uint32))
    for b in range(B):
        bits, _, _ = O.fp8_quant(af[b], scale=ref_s[b])
        assert np.array_equal(q[b].view(torch.uint8).cpu().numpy(), bits)


def _fp8_weights(B, N, K, seed):
    """e4m3 weights [B, N, K] from the oracle's quantizer (per-channel scales)."""
    w = np.random.default_rng(seed).standard_normal((B, N, K)).astype(np.float32) * 0.02
    bits, vals, scale = O.fp8_quant(w)  # one scale per output channel (row of [N, K])
    return bits, vals, scale


SHAPES = [(1, 1, 128, 64), (1, 16, 8192, 8192), (1, 32, 1024, 4096), (2, 17, 384, 1280), (1, 100, 520, 256),
          (1, 300, 256, 512), (4, 8, 2048, 2048)]


@pytest.mark.parametrize("B,M,N,K", SHAPES)
def test_fp8_gemm_matches_exact_product(cuda_device, B, M, N, K):
    from cb200 import ops
    d = cuda_device
    a = _acts(B, M, K, torch.bfloat16, seed=M * 3 + N + K)
    abits, avals, ascale = O.fp8_quant(to_np_f32(a))
    wbits, wvals, wscale = _fp8_weights(B, N, K, seed=N + K)
    exact = O.fp8_gemm(avals, wvals)  # [B, M, N]
    ref = exact * ascale[..., :, None].astype(np.float64) * wscale[..., None, :].astype(np.float64)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(d)  # noqa: E731
    aq = t(abits).view(torch.float8_e4m3fn)
    wq = t(wbits).view(torch.float8_e4m3fn)
    out32 = ops.fp8_gemm(aq, wq, t(ascale.reshape(-1)), t(wscale.reshape(-1)), out_dtype=torch.float32)
    out16 = ops.fp8_gemm(aq, wq, t(ascale.reshape(-1)), t(wscale.reshape(-1)), out_dtype=torch.bfloat16)
    again = ops.fp8_gemm(aq, wq, t(ascale.reshape(-1)), t(wscale.reshape(-1)), out_dtype=torch.float32)
    torch.cuda.synchronize()
    scale = np.abs(ref).max()
    got = out32.cpu().numpy().astype(np.float64)
    assert np.abs(got - ref).max() <= 1e-5 * scale
    got16 = to_np_f32(out16).astype(np.float64)
    assert np.abs(got16 - ref).max() <= 2.0 ** -8 * scale + 1e-5 * scale
    assert torch.equal(out32, again)
    assert ops.device_status(d) == 0


def test_fp8_gemm_per_tensor_scales_and_bias(cuda_device):
    from cb200 import ops
    d = cuda_device
    B, M, N, K = 1, 12, 768, 1536
    a = _acts(B, M, K, torch.bfloat16, seed=11)
    q, s = ops.quant_act_fp8(a.to(d), "per_tensor")
    wbits, wvals, _ = _fp8_weights(B, N, K, seed=5)
    ws = torch.tensor([0.0031], device=d)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(d)
    out = ops.fp8_gemm(q, torch.from_numpy(wbits).to(d).view(torch.float8_e4m3fn), s, ws, out_dtype=torch.float32,
                       bias=bias)
    torch.cuda.synchronize()
    avals = O.e4m3_bits_to_f32(q.view(torch.uint8).cpu().numpy())
    ref = O.fp8_gemm(avals, wvals) * float(s.item()) * 0.0031 + to_np_f32(bias.cpu()).astype(np.float64)
    assert np.abs(out.cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max()


def test_dense_ops_fp8_scaled_mm(cuda_device):
    """The vLLM call shapes of the reference harness: scaled_fp8_quant per tensor,
    b as the column-major view of a K-major e4m3 weight, bf16 out."""
    import dense_ops
    d = cuda_device
    M, N, K = 16, 2048, 8192
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(M, K, generator=g) / 32).to(torch.bfloat16).to(d)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16).to(d)
    xq, xs = dense_ops.scaled_fp8_quant(x)
    wq, wsc = dense_ops.scaled_fp8_quant(w)
    out = dense_ops.cutlass_scaled_mm(xq, wq.t(), xs, wsc, torch.bfloat16)
    torch.cuda.synchronize()
    xv = O.e4m3_bits_to_f32(xq.view(torch.uint8).cpu().numpy())
    wv = O.e4m3_bits_to_f32(wq.view(torch.uint8).cpu().numpy())
    ref = (xv.astype(np.float64) @ wv.astype(np.float64).T) * float(xs.item()) * float(wsc.item())
    got = to_np_f32(out).astype(np.float64)
    assert np.abs(got - ref).max() <= 2.0 ** -8 * np.abs(ref).max() + 1e-5 * np.abs(ref).max()


def _vllm_ops():
    try:
        import vllm._custom_ops as vops
        return vops
    except Exception:  # noqa: BLE001
        return None


def test_fp8_against_vllm(cuda_device):
    vops = _vllm_ops()
    if vops is None:
        pytest.skip("vLLM's GPU ops do not load here")
    import dense_ops
    d = cuda_device
    M, N, K = 16, 4096, 4096
    g = torch.Generator().manual_seed(9)
    x = (torch.randn(M, K, generator=g) / 32).to(torch.bfloat16).to(d)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16).to(d)
    try:
        vxq, vxs = vops.scaled_fp8_quant(x)
        vwq, vws = vops.scaled_fp8_quant(w)
        vout = vops.cutlass_scaled_mm(vxq, vwq.t(), vxs, vws, torch.bfloat16)
        torch.cuda.synchronize()
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"vLLM fp8 ops failed to run: {e!r}")
    xq, xs = dense_ops.scaled_fp8_quant(x)
    torch.cuda.synchronize()
    assert torch.equal(xs.reshape(-1).cpu(), vxs.reshape(-1).float().cpu())
    same = (xq.view(torch.uint8) == vxq.view(torch.uint8)).float().mean().item()
    assert same >= 0.999
    # the GEMM on vLLM's own quantized operands
    out = dense_ops.cutlass_scaled_mm(vxq, vwq.t(), vxs, vws, torch.bfloat16)
    torch.cuda.synchronize()
    ref = to_np_f32(vout).astype(np.float64)
    got = to_np_f32(out).astype(np.float64)
    assert np.abs(got - ref).max() <= 2.0 ** -7 * np.abs(ref).max()
