"""Failure detection on the GPU without a GPU fault.

Every device-side wait in the kernels is bounded; a wait that runs out records
CB_DEVERR_TIMEOUT in the call's status word, and every role of the CTA leaves
its loop, drains the copies and MMAs it issued and frees its tensor memory, so
the context stays usable. These tests make a wait run out on purpose through
the library's test hook (cb_debug_force_wait_timeout: one thread per CTA waits,
with a 2 ms limit, on a workspace word that nothing sets) and check that the
caller is told (cb_workspace_status -> CB_ERR_DEVICE_TIMEOUT) and that the next
call on the same workspace is bit-exact again.
"""

import ctypes

import numpy as np
import pytest
import torch

from _gpu_helpers import to_np_f32
from oracle import quant_oracle as O

pytestmark = pytest.mark.gpu

HOOK_NS = 2_000_000  # 2 ms


def _problem(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(1, M, K, generator=g).to(torch.bfloat16)
    wq = torch.randint(-127, 128, (1, K, N), generator=g, dtype=torch.int32).to(torch.int8)
    ws = (torch.randn(1, N, generator=g) * 0.01).abs().float() + 1e-4
    return a, wq, ws


@pytest.mark.parametrize("M,N,K", [(16, 2048, 4096), (1, 8192, 8192), (40, 512, 256)])
def test_forced_wait_timeout_is_reported_and_recovers(cuda_device, M, N, K):
    from cb200 import _lib as L
    from cb200 import ops
    lib = L.load()
    a, wq, ws = _problem(M, N, K, seed=M + N + K)
    d = cuda_device
    w_nk = ops.repack_w8_kmajor(wq.to(d))
    q, s = ops.quant_act_i8(a.to(d))
    assert ops.device_status(d) == 0
    lib.cb_debug_force_wait_timeout(HOOK_NS)
    try:
        ops.w8a8_gemm(q, w_nk, s, ws.to(d), out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
    finally:
        lib.cb_debug_force_wait_timeout(0)
    # the expired wait is reported (and cleared, counters included) by the status read
    st = ctypes.c_int(0)
    buf = ops.POOL.get(ops.workspace_bytes(L.CB_OP_W8A8, 1, M, N, K), d)
    rc = lib.cb_workspace_status(buf.data_ptr(), ctypes.byref(st), torch.cuda.current_stream(d).cuda_stream)
    assert rc == L.CB_ERR_DEVICE_TIMEOUT and st.value != 0
    assert ops.device_status(d) == 0
    # the context is usable and the same workspace gives exact results again
    acc = torch.empty(1, M, N, dtype=torch.int32, device=d)
    out = ops.w8a8_gemm(q, w_nk, s, ws.to(d), out_dtype=torch.bfloat16, acc_out=acc)
    torch.cuda.synchronize()
    ref_q, ref_s = O.quant_act_i8(to_np_f32(a))
    ref_acc = O.gemm_i8_i32(ref_q, wq.numpy())
    assert np.array_equal(acc.cpu().numpy(), ref_acc)
    ref = O.w8a8_epilogue(ref_acc, ref_s, ws.numpy(), "bf16")
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), ref)
    assert ops.device_status(d) == 0


def test_forced_timeout_on_the_dynamic_chain(cuda_device):
    """The two-launch (act-quant + GEMM, PDL-chained) entry point reports it too."""
    from cb200 import _lib as L
    from cb200 import ops
    lib = L.load()
    M, N, K = 8, 4096, 4096
    a, wq, ws = _problem(M, N, K, seed=9)
    d = cuda_device
    w_nk = ops.repack_w8_kmajor(wq.to(d))
    lib.cb_debug_force_wait_timeout(HOOK_NS)
    try:
        ops.w8a8_gemm_dynamic(a.to(d), w_nk, ws.to(d), out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
    finally:
        lib.cb_debug_force_wait_timeout(0)
    assert ops.device_status(d) & 1
    assert ops.device_status(d) == 0
    out = ops.w8a8_gemm_dynamic(a.to(d), w_nk, ws.to(d), out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    ref, _, _, _ = O.w8a8_dynamic(to_np_f32(a), wq.numpy(), ws.numpy(), "bf16")
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), ref)
