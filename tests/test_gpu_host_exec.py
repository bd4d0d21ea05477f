"""The host-buffer executor (cb_exec_*) on the GPU: activations and results in
pinned host memory, one C call per GEMM, copies overlapped across calls.

  - every result equals the device-buffer path (cb_w8a8_gemm_dynamic) on the
    same inputs bit for bit, for batched and ragged shapes and every output
    dtype, including a sequence of calls of growing size (the executor grows its
    buffers) and calls issued back to back before one synchronize;
  - before(stream) orders later work on a torch stream after the executor's
    copies back: a device-side read of the results on that stream sees them.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _problem(B, M, N, K, seed, dev):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(B, M, K, generator=g) * 2).to(torch.bfloat16)
    w = torch.randint(-127, 128, (B, N, K), generator=g, dtype=torch.int8).to(dev)
    ws = (torch.rand(B, N, generator=g) * 1e-2 + 1e-4).to(dev)
    return a, w, ws


SHAPES = [(1, 1, 256, 128), (1, 16, 8192, 8192), (2, 33, 384, 1280), (3, 5, 1024, 512), (1, 130, 2048, 2048)]


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_host_exec_matches_device_path(cuda_device, out_dtype):
    from cb200 import ops
    d = cuda_device
    ex = ops.HostExecutor(d)
    cases = []
    for i, (B, M, N, K) in enumerate(SHAPES):
        a, w, ws = _problem(B, M, N, K, seed=i, dev=d)
        ref = ops.w8a8_gemm_dynamic(a.to(d), w, ws, out_dtype=out_dtype)
        hin = a.pin_memory()
        hout = torch.empty(B, M, N, dtype=out_dtype).pin_memory()
        cases.append((hin, w, ws, hout, ref))
    # back to back, one synchronize at the end
    for hin, w, ws, hout, _ in cases:
        ex.w8a8_dynamic_host(hin, w, ws, hout)
    assert ex.synchronize() == 0
    torch.cuda.synchronize()
    for _, _, _, hout, ref in cases:
        assert torch.equal(hout, ref.cpu())
    # repeated calls into the same host buffers (the ring of device slots wraps)
    for _ in range(3):
        for hin, w, ws, hout, ref in cases:
            hout.zero_()
            ex.w8a8_dynamic_host(hin, w, ws, hout)
            ex.synchronize()
            assert torch.equal(hout, ref.cpu())
    ex.close()


def test_host_exec_before_orders_a_stream(cuda_device):
    from cb200 import ops
    d = cuda_device
    B, M, N, K = 1, 16, 4096, 4096
    a, w, ws = _problem(B, M, N, K, seed=42, dev=d)
    ref = ops.w8a8_gemm_dynamic(a.to(d), w, ws, out_dtype=torch.float16)
    hin = a.pin_memory()
    hout = torch.zeros(B, M, N, dtype=torch.float16).pin_memory()
    ex = ops.HostExecutor(d)
    ex.after()
    ex.w8a8_dynamic_host(hin, w, ws, hout)
    ex.before()  # the current stream now waits for the copy back
    back = hout.to(d, non_blocking=True)  # enqueued on the current stream
    torch.cuda.synchronize()
    assert torch.equal(back, ref)
    assert ex.synchronize() == 0
    ex.close()


def test_host_exec_rejects_device_tensors(cuda_device):
    from cb200 import ops
    d = cuda_device
    a, w, ws = _problem(1, 4, 256, 128, seed=1, dev=d)
    ex = ops.HostExecutor(d)
    with pytest.raises(ValueError):
        ex.w8a8_dynamic_host(a.to(d), w, ws, torch.empty(1, 4, 256, dtype=torch.float16))
    ex.close()
