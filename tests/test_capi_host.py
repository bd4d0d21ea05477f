"""The C-ABI library on a machine without a GPU: it loads, exports every symbol
include/cb200.h declares, and rejects invalid arguments with status codes (no
compute call is made here)."""

import ctypes
import os
import re

import pytest

from conftest import ROOT


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "cb200.h")).read()
    return sorted(set(re.findall(r"CB_API\s+[\w\s\*]+?\b(cb_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from cb200 import _lib
    return _lib.load()


def test_header_declares_the_abi():
    syms = _declared_symbols()
    for name in ("cb_w8a8_gemm", "cb_w8a8_gemm_dynamic", "cb_quant_act_i8", "cb_w4a16_gemm", "cb_w4a4_gemm",
                 "cb_repack_w4", "cb_repack_w8_kmajor", "cb_workspace_bytes", "cb_status_str"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    from cb200 import _lib
    for name in _declared_symbols():
        assert hasattr(lib, name), f"libcb200.so does not export {name}"
        assert name in _lib.SIGNATURES, f"ctypes binding lacks {name}"


def test_status_strings(lib):
    from cb200 import _lib as L
    assert L.status_str(L.CB_OK) == "ok"
    assert "workspace" in L.status_str(L.CB_ERR_WORKSPACE)
    assert L.status_str(12345) == "unknown status"
    assert lib.cb_version() >= 100


def test_workspace_sizes(lib):
    from cb200 import _lib as L
    small = lib.cb_workspace_bytes(L.CB_OP_W8A8, 1, 1, 8192, 8192)
    big = lib.cb_workspace_bytes(L.CB_OP_W8A8, 1, 512, 8192, 8192)
    assert 0 < small < big
    assert lib.cb_workspace_bytes(L.CB_OP_W4A4, 1, 16, 256, 256) >= 16 * 256 + 256 * 256
    assert lib.cb_workspace_bytes(99, 1, 1, 1, 1) == 0
    assert lib.cb_workspace_bytes(L.CB_OP_W8A8, -1, 1, 1, 1) == 0
    assert lib.cb_w4_native_bytes(2, 256, 130) == 2 * 2 * 2 * 8192


def _st(*v):
    return (ctypes.c_int64 * len(v))(*v)


def test_w8a8_argument_validation_without_device(lib):
    from cb200 import _lib as L
    st = _st(0, 256, 0, 256, 0, 64, 0, 0)
    # empty problem is a no-op
    assert lib.cb_w8a8_gemm(None, None, None, None, None, L.CB_DTYPE_BF16, None, 1, 0, 64, 256, st, None, 0,
                            None) == L.CB_OK
    # null operands
    assert lib.cb_w8a8_gemm(None, None, None, None, None, L.CB_DTYPE_BF16, None, 1, 4, 64, 256, st, None, 0,
                            None) == L.CB_ERR_INVALID_ARG
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: validation fails first
    # K not a multiple of 16
    assert lib.cb_w8a8_gemm(fake, fake, fake, fake, fake, L.CB_DTYPE_BF16, None, 1, 4, 64, 250,
                            _st(0, 256, 0, 256, 0, 64, 0, 0), None, 0, None) == L.CB_ERR_SHAPE
    # bad out dtype
    assert lib.cb_w8a8_gemm(fake, fake, fake, fake, fake, L.CB_DTYPE_I8, None, 1, 4, 64, 256, st, None, 0,
                            None) == L.CB_ERR_DTYPE
    # misaligned operand
    assert lib.cb_w8a8_gemm(ctypes.c_void_p(0x1001), fake, fake, fake, fake, L.CB_DTYPE_BF16, None, 1, 4, 64,
                            256, st, None, 0, None) == L.CB_ERR_ALIGNMENT
    # row stride shorter than K
    assert lib.cb_w8a8_gemm(fake, fake, fake, fake, fake, L.CB_DTYPE_BF16, None, 1, 4, 64, 256,
                            _st(0, 128, 0, 256, 0, 64, 0, 0), None, 0, None) == L.CB_ERR_STRIDE
    # negative size
    assert lib.cb_w8a8_gemm(fake, fake, fake, fake, fake, L.CB_DTYPE_BF16, None, 1, -4, 64, 256, st, None, 0,
                            None) == L.CB_ERR_INVALID_ARG


def test_w4a16_and_w4a4_validation_without_device(lib):
    from cb200 import _lib as L
    fake = ctypes.c_void_p(0x1000)
    st = _st(0, 256, 0, 192, 0, 192)
    # group size must be a multiple of 128 below K
    assert lib.cb_w4a16_gemm(fake, L.CB_DTYPE_BF16, fake, fake, L.CB_DTYPE_BF16, 64, fake, L.CB_DTYPE_BF16, 1, 3,
                             192, 256, st, None, 0, None) == L.CB_ERR_SHAPE
    # activation dtype must be f16/bf16
    assert lib.cb_w4a16_gemm(fake, L.CB_DTYPE_F32, fake, fake, L.CB_DTYPE_BF16, 128, fake, L.CB_DTYPE_BF16, 1, 3,
                             192, 256, st, None, 0, None) == L.CB_ERR_DTYPE
    # W4A4: K multiple of 32, valid nibble mode
    assert lib.cb_w4a4_gemm(fake, fake, fake, 4, 64, 48, 24, 64, 64, 0, None, 0, None) == L.CB_ERR_SHAPE
    assert lib.cb_w4a4_gemm(fake, fake, fake, 4, 64, 64, 32, 64, 64, 7, None, 0, None) == L.CB_ERR_INVALID_ARG
    # W4A4 workspace is required
    assert lib.cb_w4a4_gemm(fake, fake, fake, 4, 64, 64, 32, 64, 64, 0, None, 0, None) == L.CB_ERR_WORKSPACE
    # repack: unknown layout
    assert lib.cb_repack_w4(fake, 5, fake, 1, 128, 128, None) == L.CB_ERR_UNSUPPORTED


def test_python_check_maps_status_to_exceptions():
    from cb200 import _lib as L
    with pytest.raises(ValueError):
        L.check("cb_w8a8_gemm", L.CB_ERR_SHAPE)
    with pytest.raises(L.CbError):
        L.check("cb_w8a8_gemm", L.CB_ERR_DEVICE_TIMEOUT)
    L.check("cb_w8a8_gemm", L.CB_OK)


def test_ops_refuse_cpu_tensors():
    import torch
    from cb200 import ops
    a = torch.zeros(4, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.quant_act_i8(a)
    with pytest.raises(ValueError, match="CUDA"):
        ops.w8a8_gemm(torch.zeros(4, 256, dtype=torch.int8), torch.zeros(64, 256, dtype=torch.int8),
                      torch.zeros(4), torch.zeros(64))
