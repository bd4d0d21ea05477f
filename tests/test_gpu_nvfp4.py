"""NVFP4 (e2m1 values, e4m3 scales per 16 elements) on the GPU through the C ABI.

The quantizer is bit-exact against the oracle (vLLM's ref_nvfp4_quant restated,
pinned by tests/golden/nvfp4_*.npz), swizzled scales and their zero padding
included. The GEMM accumulates in fp32 on the tensor cores' block-scaled FP4
path; it is checked against the oracle's exact float64 product with a relative
tolerance of 1e-5 of the output's largest magnitude (fp32 output) and against
vLLM's own cutlass_scaled_fp4_mm and scaled_fp4_quant when vLLM's ops load."""

import numpy as np
import pytest
import torch

from _gpu_helpers import to_np_f32
from oracle import quant_oracle as O

pytestmark = pytest.mark.gpu


def _x(rows, K, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, K, generator=g).to(dtype)
    if rows > 1:
        x[1, :32] = 0
    return x


@pytest.mark.parametrize("rows,K", [(1, 64), (5, 256), (16, 8192), (130, 512), (33, 320)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_nvfp4_quantize_bit_exact(cuda_device, rows, K, dtype):
    from cb200 import ops
    x = _x(rows, K, dtype, seed=rows * 31 + K)
    gs = 448.0 * 6.0 / float(x.float().abs().max())
    q, sf = ops.nvfp4_quantize(x.to(cuda_device), torch.tensor([gs], dtype=torch.float32, device=cuda_device))
    torch.cuda.synchronize()
    ref_q, ref_s, _ = O.nvfp4_quant(to_np_f32(x), gs)
    assert np.array_equal(q.cpu().numpy(), ref_q)
    assert np.array_equal(sf.cpu().numpy().reshape(-1), O.nvfp4_swizzle(ref_s))
    assert ops.device_status(cuda_device) == 0


def _quantized(rows, K, seed, gs):
    x = np.random.default_rng(seed).standard_normal((rows, K)).astype(np.float32)
    return O.nvfp4_quant(x, gs)[:2]


SHAPES = [(1, 128, 64), (1, 256, 256), (16, 384, 320), (32, 8192, 8192), (8, 1000, 1024), (100, 640, 2048),
          (128, 256, 512), (200, 384, 256)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_nvfp4_gemm_matches_oracle(cuda_device, M, N, K):
    from cb200 import ops
    ap, asf = _quantized(M, K, 1 + M, 3.0)
    bp, bsf = _quantized(N, K, 2 + N, 5.0)
    alpha = 1.0 / 15.0
    ref = O.nvfp4_gemm(ap, asf, bp, bsf, alpha)
    d = cuda_device
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(d)  # noqa: E731
    out32 = ops.nvfp4_gemm(t(ap), t(O.nvfp4_swizzle(asf)), t(bp), t(O.nvfp4_swizzle(bsf)),
                           torch.tensor([alpha], dtype=torch.float32, device=d), out_dtype=torch.float32)
    out16 = ops.nvfp4_gemm(t(ap), t(O.nvfp4_swizzle(asf)), t(bp), t(O.nvfp4_swizzle(bsf)),
                           torch.tensor([alpha], dtype=torch.float32, device=d), out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    got = out32.cpu().numpy().astype(np.float64)
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= 1e-5 * scale
    got16 = out16.float().cpu().numpy().astype(np.float64)
    assert np.abs(got16 - ref).max() <= 2.0 ** -8 * np.abs(ref).max() + 1e-5 * scale
    assert ops.device_status(cuda_device) == 0


def test_nvfp4_gemm_deterministic_and_graph(cuda_device):
    from cb200 import ops
    M, N, K = 16, 2048, 4096
    ap, asf = _quantized(M, K, 5, 2.0)
    bp, bsf = _quantized(N, K, 6, 2.0)
    d = cuda_device
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(d)  # noqa: E731
    a, a_sf, b, b_sf = t(ap), t(O.nvfp4_swizzle(asf)), t(bp), t(O.nvfp4_swizzle(bsf))
    alpha = torch.tensor([0.25], dtype=torch.float32, device=d)
    first = ops.nvfp4_gemm(a, a_sf, b, b_sf, alpha, out_dtype=torch.float32)
    out = torch.empty_like(first)
    ops.nvfp4_gemm(a, a_sf, b, b_sf, alpha, out=out)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(3):
            ops.nvfp4_gemm(a, a_sf, b, b_sf, alpha, out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int32), first.view(torch.int32))


def _vllm_ops():
    try:
        import vllm._custom_ops as vops
        if not hasattr(vops, "cutlass_scaled_fp4_mm") or not hasattr(vops, "scaled_fp4_quant"):
            return None
        return vops
    except Exception:  # vLLM absent or its extension does not load on this box
        return None


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (16, 8192, 8192), (32, 1024, 2048)])
def test_nvfp4_against_vllm(cuda_device, M, N, K):
    """The reference's own dependency for this path: vLLM's quantizer and FP4 GEMM."""
    vops = _vllm_ops()
    if vops is None:
        pytest.skip("vLLM's FP4 ops are not available")
    from cb200 import ops
    d = cuda_device
    g = torch.Generator(device=d).manual_seed(M + N)
    x = torch.randn(M, K, device=d, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=d, generator=g) / K ** 0.5).to(torch.bfloat16)
    gx = torch.tensor([448.0 * 6.0 / float(x.float().abs().max())], device=d)
    gw = torch.tensor([448.0 * 6.0 / float(w.float().abs().max())], device=d)
    qx_v, sx_v = vops.scaled_fp4_quant(x, gx)
    qw_v, sw_v = vops.scaled_fp4_quant(w, gw)
    qx, sx = ops.nvfp4_quantize(x, gx)
    qw, sw = ops.nvfp4_quantize(w, gw)
    torch.cuda.synchronize()
    # Scales: identical to vLLM's GPU quantizer.
    sx_u = sx_v.view(torch.uint8).reshape(-1)[: sx.numel()]
    sw_u = sw_v.view(torch.uint8).reshape(-1)[: sw.numel()]
    assert torch.equal(sx.reshape(-1)[: sx_u.numel()], sx_u) and torch.equal(sw.reshape(-1)[: sw_u.numel()], sw_u)
    # Values: ours equal vLLM's CPU reference (ref_nvfp4_quant) exactly; vLLM's
    # GPU kernel departs from that reference for a small fraction of elements.
    try:
        from vllm.model_executor.layers.quantization.utils.nvfp4_emulation_utils import ref_nvfp4_quant
    except Exception:
        ref_nvfp4_quant = None
    if ref_nvfp4_quant is not None:
        ref_vals, _ = ref_nvfp4_quant(x.float().cpu(), gx.cpu(), 16)
        ours_nib = torch.stack(((qx & 0xF), (qx >> 4)), dim=-1).reshape(M, K).cpu().numpy()
        assert np.array_equal(O.e2m1_to_f32(ours_nib), ref_vals.numpy())
        v_nib = torch.stack(((qx_v.view(torch.uint8) & 0xF), (qx_v.view(torch.uint8) >> 4)), dim=-1)
        gpu_vs_ref = float((O.e2m1_to_f32(v_nib.reshape(M, K).cpu().numpy()) != ref_vals.numpy()).mean())
        print(f"vLLM GPU quantizer vs vLLM CPU reference: {gpu_vs_ref:.2e} of values differ")
    diff_q = (qx != qx_v.view(torch.uint8)).float().mean().item() + (qw != qw_v.view(torch.uint8)).float().mean().item()
    assert diff_q < 2e-2
    alpha = (1.0 / (gx * gw)).to(torch.float32)
    # vLLM's FP4 GEMM writes 16-bit outputs only: compare in bf16, where the two
    # fp32 accumulations (different summation orders) may round one ulp apart
    ours = ops.nvfp4_gemm(qx_v.view(torch.uint8), sx_v.view(torch.uint8), qw_v.view(torch.uint8),
                          sw_v.view(torch.uint8), alpha, out_dtype=torch.bfloat16).float()
    theirs = vops.cutlass_scaled_fp4_mm(qx_v, qw_v, sx_v, sw_v, alpha, torch.bfloat16).float()
    torch.cuda.synchronize()
    assert (ours - theirs).abs().max().item() <= 2.0 ** -7 * theirs.abs().max().item()
    assert (ours == theirs).float().mean().item() > 0.95
