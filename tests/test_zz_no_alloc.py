"""The allocation-free W8A8 entry point (cb_w8a8_gemm_noalloc).

It exists for callers that cannot allocate device memory (another component owns
it, or a foreign-language binding has no allocator): they pass only inputs and
outputs, and the split-K scratch comes from a device array inside the library.
Through the C ABI, two calls in a row with different inputs must give exactly the
results of the workspace-based entry point (cb_w8a8_gemm); W8A8 is bit-exact, so
the tolerance is zero. A bounded device-side wait that expires inside such a call
must reach the caller through cb_w8a8_noalloc_status, not vanish with the next
call. This file is collected last so that a run stopping at its first failure has
already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call_noalloc(lib, q, w_nk, s, ws, out, acc):
    B, M, K = q.shape
    N = w_nk.shape[1]
    st = (ctypes.c_int64 * 8)(q.stride(0), q.stride(1), w_nk.stride(0), w_nk.stride(1), out.stride(0),
                              out.stride(1), M, ws.stride(0))
    return lib.cb_w8a8_gemm_noalloc(q.data_ptr(), s.data_ptr(), w_nk.data_ptr(), ws.data_ptr(), out.data_ptr(), 1,
                                    acc.data_ptr(), B, M, N, K, st, torch.cuda.current_stream().cuda_stream)


def _noalloc_status(lib):
    st = ctypes.c_int(0)
    rc = lib.cb_w8a8_noalloc_status(ctypes.byref(st), torch.cuda.current_stream().cuda_stream)
    return rc, st.value


def test_noalloc_matches_workspace_entry_point_on_two_calls(cuda_device):
    from cb200 import _lib as L
    from cb200 import ops
    lib = L.load()
    B, M, N, K = 1, 16, 2048, 4096  # 512 k-blocks over 148 CTAs: split-K slots and counters in use
    g = torch.Generator().manual_seed(2024)
    wq = torch.randint(-127, 128, (B, K, N), generator=g, dtype=torch.int32).to(torch.int8)
    w_nk = ops.repack_w8_kmajor(wq.to(cuda_device))
    w_scale = ((torch.randn(B, N, generator=g) * 0.01).abs() + 1e-4).to(cuda_device)
    for call in range(2):
        a = torch.randn(B, M, K, generator=g).to(torch.bfloat16).to(cuda_device)
        q, s = ops.quant_act_i8(a)
        acc_ref = torch.empty(B, M, N, dtype=torch.int32, device=cuda_device)
        ref = ops.w8a8_gemm(q, w_nk, s, w_scale, out_dtype=torch.bfloat16, acc_out=acc_ref)
        out = torch.full((B, M, N), -1.0, dtype=torch.bfloat16, device=cuda_device)
        acc = torch.full((B, M, N), -9, dtype=torch.int32, device=cuda_device)
        rc = _call_noalloc(lib, q, w_nk, s, w_scale, out, acc)
        assert rc == L.CB_OK, L.status_str(rc)
        torch.cuda.synchronize()
        assert torch.equal(acc, acc_ref), f"call {call}: int32 accumulators differ"
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"call {call}: outputs differ"
    assert _noalloc_status(lib) == (L.CB_OK, 0)
    assert ops.device_status(cuda_device) == 0


def test_noalloc_reports_an_expired_wait(cuda_device):
    """A call whose bounded wait runs out (forced by the library's test hook: one
    thread per CTA waits 2 ms on a word nothing sets) is reported by
    cb_w8a8_noalloc_status even after a later successful call, and the scratch is
    clean for the calls after the read."""
    from cb200 import _lib as L
    from cb200 import ops
    lib = L.load()
    B, M, N, K = 1, 16, 2048, 4096
    g = torch.Generator().manual_seed(7)
    wq = torch.randint(-127, 128, (B, K, N), generator=g, dtype=torch.int32).to(torch.int8)
    w_nk = ops.repack_w8_kmajor(wq.to(cuda_device))
    w_scale = ((torch.randn(B, N, generator=g) * 0.01).abs() + 1e-4).to(cuda_device)
    a = torch.randn(B, M, K, generator=g).to(torch.bfloat16).to(cuda_device)
    q, s = ops.quant_act_i8(a)
    acc_ref = torch.empty(B, M, N, dtype=torch.int32, device=cuda_device)
    ref = ops.w8a8_gemm(q, w_nk, s, w_scale, out_dtype=torch.bfloat16, acc_out=acc_ref)
    out = torch.empty(B, M, N, dtype=torch.bfloat16, device=cuda_device)
    acc = torch.empty(B, M, N, dtype=torch.int32, device=cuda_device)
    assert _noalloc_status(lib) == (L.CB_OK, 0)
    lib.cb_debug_force_wait_timeout(2_000_000)
    try:
        assert _call_noalloc(lib, q, w_nk, s, w_scale, out, acc) == L.CB_OK  # launched; the wait expires on the GPU
        torch.cuda.synchronize()
    finally:
        lib.cb_debug_force_wait_timeout(0)
    # a later good call does not erase the record
    assert _call_noalloc(lib, q, w_nk, s, w_scale, out, acc) == L.CB_OK
    rc, word = _noalloc_status(lib)
    assert rc == L.CB_ERR_DEVICE_TIMEOUT and word != 0
    assert _noalloc_status(lib) == (L.CB_OK, 0)
    for _ in range(2):
        out.fill_(-1.0)
        acc.fill_(-9)
        assert _call_noalloc(lib, q, w_nk, s, w_scale, out, acc) == L.CB_OK
        torch.cuda.synchronize()
        assert torch.equal(acc, acc_ref)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    assert _noalloc_status(lib) == (L.CB_OK, 0)
    assert ops.device_status(cuda_device) == 0


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    from cb200 import _lib as L
    from cb200 import ops
    lib = L.load()
    B, M, N, K = 1, 200, 256, 256  # 256-token tile: slots larger than the 8 MiB scratch
    q = torch.zeros(B, M, K, dtype=torch.int8, device=cuda_device)
    s = torch.ones(B * M, device=cuda_device)
    w_nk = torch.zeros(B, N, K, dtype=torch.int8, device=cuda_device)
    ws = torch.ones(B, N, device=cuda_device)
    out = torch.zeros(B, M, N, dtype=torch.bfloat16, device=cuda_device)
    acc = torch.zeros(B, M, N, dtype=torch.int32, device=cuda_device)
    assert _call_noalloc(lib, q, w_nk, s, ws, out, acc) == L.CB_ERR_TOO_LARGE
    assert np.all(out.cpu().float().numpy() == 0.0)
    assert ops.workspace_bytes(L.CB_OP_W8A8, B, M, N, K) > 8 << 20
