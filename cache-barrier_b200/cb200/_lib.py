"""ctypes binding of ``libcb200.so`` (the C ABI of ``include/cb200.h``).

The library is the only compute path: if it is missing or fails to load, every
op raises ``RuntimeError``; there is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

# status codes (include/cb200.h)
CB_OK = 0
CB_ERR_INVALID_ARG = 1
CB_ERR_SHAPE = 2
CB_ERR_DTYPE = 3
CB_ERR_ALIGNMENT = 4
CB_ERR_STRIDE = 5
CB_ERR_WORKSPACE = 6
CB_ERR_CUDA = 7
CB_ERR_DEVICE_TIMEOUT = 8
CB_ERR_UNSUPPORTED = 9
CB_ERR_TOO_LARGE = 10

# dtype codes
CB_DTYPE_F16 = 0
CB_DTYPE_BF16 = 1
CB_DTYPE_F32 = 2
CB_DTYPE_I8 = 3
CB_DTYPE_U8 = 4
CB_DTYPE_I32 = 5

# ops
CB_OP_W8A8 = 0
CB_OP_W4A16 = 1
CB_OP_W4A4 = 2
CB_OP_NVFP4 = 3

# fp8 activation quantization modes
CB_FP8_PER_TOKEN = 0
CB_FP8_PER_TENSOR_DYNAMIC = 1
CB_FP8_STATIC = 2

# W4A4 nibble modes
CB_W4A4_SIGNED = 0
CB_W4A4_REF_UINT8_WRAP = 1

# int4 layouts
CB_W4_REF_U8_KN = 0
CB_W4_I32_K8N = 1
CB_W4_NATIVE = 2

_i64 = ctypes.c_int64
_int = ctypes.c_int
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "cb_status_str": (ctypes.c_char_p, [_int]),
    "cb_version": (_int, []),
    "cb_device_sm_count": (_int, []),
    "cb_workspace_bytes": (_sz, [_int, _i64, _i64, _i64, _i64]),
    "cb_workspace_status": (_int, [_vp, ctypes.POINTER(_int), _vp]),
    "cb_quant_act_i8": (_int, [_vp, _int, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp]),
    "cb_w8a8_gemm": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _sz, _vp]),
    "cb_w8a8_gemm_bias": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _i64, _vp, _int, _vp, _i64, _i64, _i64, _i64, _vp,
                                 _vp, _sz, _vp]),
    "cb_quant_act_fp8": (_int, [_vp, _int, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _int, _vp]),
    "cb_fp8_gemm": (_int, [_vp, _vp, _int, _vp, _vp, _int, _vp, _int, _vp, _int, _i64, _i64, _i64, _i64, _vp, _vp, _sz,
                           _vp]),
    "cb_w8a8_gemm_noalloc": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "cb_w8a8_noalloc_status": (_int, [ctypes.POINTER(_int), _vp]),
    "cb_exec_create": (_int, [_int, ctypes.POINTER(_vp)]),
    "cb_exec_destroy": (None, [_vp]),
    "cb_exec_after": (_int, [_vp, _vp]),
    "cb_exec_before": (_int, [_vp, _vp]),
    "cb_exec_synchronize": (_int, [_vp, ctypes.POINTER(_int)]),
    "cb_exec_w8a8_dynamic_host": (_int, [_vp, _vp, _int, _vp, _vp, _i64, _i64, _i64, _vp, _int, _i64, _i64, _i64,
                                         _i64]),
    "cb_debug_force_wait_timeout": (None, [ctypes.c_uint64]),
    "cb_debug_force_last_arriver": (None, [ctypes.c_int]),
    "cb_w8a8_gemm_dynamic": (_int, [_vp, _int, _vp, _vp, _vp, _vp, _vp, _int, _i64, _i64, _i64, _i64, _vp, _vp,
                                    _sz, _vp]),
    "cb_w4a16_gemm": (_int, [_vp, _int, _vp, _vp, _int, _i64, _vp, _int, _i64, _i64, _i64, _i64, _vp, _vp, _sz,
                             _vp]),
    "cb_w4a4_gemm": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _int, _vp, _sz, _vp]),
    "cb_nvfp4_quantize": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _vp]),
    "cb_nvfp4_gemm": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _int, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _sz,
                             _vp]),
    "cb_repack_w4": (_int, [_vp, _int, _vp, _i64, _i64, _i64, _vp]),
    "cb_w4_native_bytes": (_sz, [_i64, _i64, _i64]),
    "cb_repack_w8_kmajor": (_int, [_vp, _vp, _i64, _i64, _i64, _vp]),
    "cb_rmsnorm_quant_i8": (_int, [_vp, _int, _vp, _int, ctypes.c_float, _i64, _i64, _i64, _vp, _i64, _vp, _vp,
                                   _i64, _vp]),
    "cb_symm_bytes": (_sz, [_int, _i64]),
    "cb_symm_alloc": (_int, [_sz, ctypes.POINTER(_vp)]),
    "cb_symm_free": (_int, [_vp]),
    "cb_ipc_get_handle": (_int, [_vp, _vp]),
    "cb_ipc_open_handle": (_int, [_vp, ctypes.POINTER(_vp)]),
    "cb_ipc_close_handle": (_int, [_vp]),
    "cb_peer_allreduce": (_int, [_vp, _vp, _i64, _int, _vp, _int, _int, _i64, _vp, _vp]),
}

_lock = threading.Lock()
_lib = None


def lib_path() -> str:
    return os.environ.get("CB200_LIB", LIB_PATH)


def load() -> ctypes.CDLL:
    """Load (once) and return the library, with argtypes declared."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"libcb200.so not found at {path}; build it with cb200.build.build() "
                    "(the quantized GEMMs have no fallback implementation)")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def status_str(code: int) -> str:
    return load().cb_status_str(code).decode()


class CbError(RuntimeError):
    """A C-ABI call returned a non-zero cb_status."""

    def __init__(self, fn: str, code: int):
        self.code = code
        super().__init__(f"{fn} failed: {status_str(code)} (cb_status {code})")


def check(fn: str, code: int) -> None:
    if code != CB_OK:
        if code in (CB_ERR_INVALID_ARG, CB_ERR_SHAPE, CB_ERR_DTYPE, CB_ERR_ALIGNMENT, CB_ERR_STRIDE,
                    CB_ERR_TOO_LARGE):
            raise ValueError(f"{fn} failed: {status_str(code)} (cb_status {code})")
        raise CbError(fn, code)
