"""Torch-facing wrappers over the C ABI.

Every function here validates shapes/dtypes, takes raw device pointers from the
tensors, and calls into ``libcb200.so`` on the current CUDA stream. Nothing is
computed in PyTorch; tensors are only used as device memory.

Shapes: 2-D operands are a batch of one; 3-D operands are ``[batch, rows, cols]``
as in the reference's batched kernels (profiling/bench_l2_barrier.py:102-125,
profiling/w8a8/w8a8_bmm.py:118-140).
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib as L

_DTYPE_CODE = {torch.float16: L.CB_DTYPE_F16, torch.bfloat16: L.CB_DTYPE_BF16, torch.float32: L.CB_DTYPE_F32}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}") from None


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _strides(*vals):
    arr = (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])
    return arr


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("all tensors must be CUDA tensors (the quantized GEMMs run only on the GPU)")


def _as3d(t: torch.Tensor) -> torch.Tensor:
    if t.dim() == 2:
        return t.unsqueeze(0)
    if t.dim() != 3:
        raise ValueError(f"expected a 2-D or 3-D tensor, got shape {tuple(t.shape)}")
    return t


# ---------------------------------------------------------------------------
# Workspace pool: one zero-initialised scratch buffer per (device, stream).
# ---------------------------------------------------------------------------
class WorkspacePool:
    """Caller-owned split-K scratch for the C ABI.

    Buffers are zero-filled at allocation and left zeroed by the kernels. One
    buffer per (device, stream) so concurrent streams never share scratch. A
    buffer first needed while a CUDA graph is being captured (torch captures on
    its own stream) is allocated from the graph's memory pool; its zero-fill is
    captured with it and re-runs on every replay, which keeps it valid.
    """

    def __init__(self):
        self._bufs = {}
        self._lock = threading.Lock()

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        key = (device.index, _stream(device))
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 20)
                if buf is not None:
                    size = max(size, 2 * buf.numel())
                buf = torch.zeros(size, dtype=torch.uint8, device=device)
                self._bufs[key] = buf
            return buf

    def check_status(self, device: torch.device | None = None) -> int:
        """Synchronising read of the device status word of every buffer on device."""
        worst = 0
        for (idx, stream), buf in list(self._bufs.items()):
            if device is not None and idx != device.index:
                continue
            st = ctypes.c_int(0)
            code = L.load().cb_workspace_status(buf.data_ptr(), ctypes.byref(st), stream)
            if code not in (L.CB_OK, L.CB_ERR_DEVICE_TIMEOUT):
                L.check("cb_workspace_status", code)
            worst |= st.value
        return worst


POOL = WorkspacePool()


def workspace_bytes(op: int, batch: int, M: int, N: int, K: int) -> int:
    return int(L.load().cb_workspace_bytes(op, batch, M, N, K))


# ---------------------------------------------------------------------------
# activation quantization
# ---------------------------------------------------------------------------
def quant_act_i8(a: torch.Tensor, q: torch.Tensor | None = None, s: torch.Tensor | None = None):
    """Per-(batch, row) int8 quantization of ``a`` ([M, K] or [B, M, K], f16/bf16).

    Returns ``(q, s)``: int8 with a's shape and fp32 scales of ``B*M`` elements
    (the reference's flat ``[H*M]`` layout). ``q``/``s`` are filled in place
    when given (graph-capture friendly, as profiling/w8a8/w8a8_bmm.py:92-106).
    """
    _require_cuda(a)
    a3 = _as3d(a)
    B, M, K = a3.shape
    if a3.stride(2) != 1:
        raise ValueError("activations must be contiguous along K")
    if q is None:
        q = torch.empty(a.shape, dtype=torch.int8, device=a.device)
    if s is None:
        s = torch.empty(B * M, dtype=torch.float32, device=a.device)
    q3 = _as3d(q)
    if q3.shape != a3.shape or q.dtype != torch.int8 or q3.stride(2) != 1:
        raise ValueError("q must be an int8 tensor shaped like a, contiguous along K")
    if s.dtype != torch.float32 or s.numel() < B * M or not s.is_contiguous():
        raise ValueError("s must be a contiguous fp32 tensor of at least B*M elements")
    code = L.load().cb_quant_act_i8(a3.data_ptr(), dtype_code(a.dtype), B, M, K, a3.stride(0), a3.stride(1),
                                    q3.data_ptr(), q3.stride(0), q3.stride(1), s.data_ptr(), M, _stream(a.device))
    L.check("cb_quant_act_i8", code)
    return q, s


def rmsnorm_quant_i8(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, q: torch.Tensor | None = None,
                     s: torch.Tensor | None = None, y: torch.Tensor | None = None):
    """Fused RMSNorm + per-token int8 quantization of ``x`` ([rows, H], f16/bf16).

    Returns ``(q, s)`` (int8 like x, fp32 ``[rows]``) exactly as ``quant_act_i8``
    applied to the RMSNorm output ``cvt(x * rsqrt(mean(x^2) + eps) * weight)``;
    ``y`` (optional, like x) receives that output.
    """
    _require_cuda(x, weight, q, s, y)
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be [rows, H], contiguous along H")
    rows, H = x.shape
    if weight.numel() != H or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous [H] tensor")
    if q is None:
        q = torch.empty(rows, H, dtype=torch.int8, device=x.device)
    if s is None:
        s = torch.empty(rows, dtype=torch.float32, device=x.device)
    if q.shape != (rows, H) or q.dtype != torch.int8 or q.stride(1) != 1:
        raise ValueError("q must be int8 [rows, H], contiguous along H")
    if s.dtype != torch.float32 or s.numel() < rows or not s.is_contiguous():
        raise ValueError("s must be a contiguous fp32 tensor of at least rows elements")
    if y is not None and (y.shape != (rows, H) or y.dtype != x.dtype or y.stride(1) != 1):
        raise ValueError("y must be like x")
    code = L.load().cb_rmsnorm_quant_i8(x.data_ptr(), dtype_code(x.dtype), weight.data_ptr(), dtype_code(weight.dtype),
                                        float(eps), rows, H, x.stride(0), q.data_ptr(), q.stride(0), s.data_ptr(),
                                        _ptr(y), y.stride(0) if y is not None else 0, _stream(x.device))
    L.check("cb_rmsnorm_quant_i8", code)
    return q, s


# ---------------------------------------------------------------------------
# W8A8
# ---------------------------------------------------------------------------
def w8a8_gemm(aq: torch.Tensor, w_nk: torch.Tensor, a_scale: torch.Tensor, w_scale: torch.Tensor,
              out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
              acc_out: torch.Tensor | None = None, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``out = (aq @ w_nk^T)_int32 * a_scale[m] * w_scale[n] (+ bias[n])``.

    aq: int8 [M, K] / [B, M, K]; w_nk: int8 [N, K] / [B, N, K] (K contiguous);
    a_scale: fp32 with B*M elements; w_scale: fp32 [N] / [B, N]; bias (optional):
    f16/bf16/f32 [N] / [B, N], added in fp32 before the output rounding.
    """
    _require_cuda(aq, w_nk, a_scale, w_scale, out, acc_out, bias)
    a3, w3 = _as3d(aq), _as3d(w_nk)
    B, M, K = a3.shape
    Bw, N, Kw = w3.shape
    if aq.dtype != torch.int8 or w_nk.dtype != torch.int8:
        raise ValueError("w8a8_gemm expects int8 operands")
    if Kw != K or Bw != B:
        raise ValueError(f"shape mismatch: aq {tuple(a3.shape)} vs w {tuple(w3.shape)}")
    if a3.stride(2) != 1 or w3.stride(2) != 1:
        raise ValueError("operands must be contiguous along K (weights K-major [N, K])")
    if a_scale.dtype != torch.float32 or w_scale.dtype != torch.float32:
        raise ValueError("scales must be fp32")
    if not a_scale.is_contiguous() or a_scale.numel() < B * M:
        raise ValueError("a_scale must be contiguous with B*M elements")
    ws2 = w_scale.reshape(B, N) if w_scale.dim() == 1 else w_scale
    if ws2.stride(-1) != 1:
        raise ValueError("w_scale must be contiguous along N")
    if out is None:
        out = torch.empty((B, M, N) if aq.dim() == 3 else (M, N), dtype=out_dtype, device=aq.device)
    o3 = _as3d(out)
    if o3.shape != (B, M, N) or o3.stride(2) != 1:
        raise ValueError("out must be [B, M, N] contiguous along N")
    acc3 = None
    if acc_out is not None:
        acc3 = _as3d(acc_out)
        if acc_out.dtype != torch.int32 or acc3.shape != o3.shape or acc3.stride() != o3.stride():
            raise ValueError("acc_out must be int32 with out's shape and strides")
    b2, b_sb = None, 0
    if bias is not None:
        b2 = bias.reshape(1, N) if bias.dim() == 1 else bias
        if b2.shape[-1] != N or b2.stride(-1) != 1 or b2.shape[0] not in (1, B):
            raise ValueError("bias must be [N] or [B, N], contiguous along N")
        b_sb = b2.stride(0) if b2.shape[0] == B and B > 1 else 0
        dtype_code(bias.dtype)
    nbytes = workspace_bytes(L.CB_OP_W8A8, B, M, N, K)
    ws = POOL.get(nbytes, aq.device)
    st = _strides(a3.stride(0), a3.stride(1), w3.stride(0), w3.stride(1), o3.stride(0), o3.stride(1), M,
                  ws2.stride(0) if ws2.dim() == 2 else 0)
    if b2 is None:
        code = L.load().cb_w8a8_gemm(a3.data_ptr(), a_scale.data_ptr(), w3.data_ptr(), ws2.data_ptr(), o3.data_ptr(),
                                     dtype_code(out.dtype), _ptr(acc3), B, M, N, K, st, ws.data_ptr(), ws.numel(),
                                     _stream(aq.device))
        L.check("cb_w8a8_gemm", code)
        return out
    code = L.load().cb_w8a8_gemm_bias(a3.data_ptr(), a_scale.data_ptr(), w3.data_ptr(), ws2.data_ptr(), b2.data_ptr(),
                                      dtype_code(b2.dtype), b_sb, o3.data_ptr(), dtype_code(out.dtype), _ptr(acc3), B,
                                      M, N, K, st, ws.data_ptr(), ws.numel(), _stream(aq.device))
    L.check("cb_w8a8_gemm_bias", code)
    return out


def w8a8_gemm_dynamic(a: torch.Tensor, w_nk: torch.Tensor, w_scale: torch.Tensor,
                      q: torch.Tensor | None = None, s: torch.Tensor | None = None,
                      out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Dynamic per-token int8 quantization of ``a`` then the W8A8 GEMM (two launches, PDL-chained)."""
    _require_cuda(a, w_nk, w_scale, q, s, out)
    a3, w3 = _as3d(a), _as3d(w_nk)
    B, M, K = a3.shape
    Bw, N, Kw = w3.shape
    if w_nk.dtype != torch.int8 or Kw != K or Bw != B:
        raise ValueError("w_nk must be int8 [B, N, K] matching a")
    if a3.stride(2) != 1 or w3.stride(2) != 1:
        raise ValueError("operands must be contiguous along K")
    if q is None:
        q = torch.empty((B, M, K), dtype=torch.int8, device=a.device)
    if s is None:
        s = torch.empty(B * M, dtype=torch.float32, device=a.device)
    if q.dtype != torch.int8 or q.numel() != B * M * K or not q.is_contiguous():
        raise ValueError("q buffer must be contiguous int8 with B*M*K elements")
    if s.dtype != torch.float32 or s.numel() < B * M or not s.is_contiguous():
        raise ValueError("s buffer must be contiguous fp32 with B*M elements")
    ws2 = w_scale.reshape(B, N) if w_scale.dim() == 1 else w_scale
    if out is None:
        out = torch.empty((B, M, N) if a.dim() == 3 else (M, N), dtype=out_dtype or a.dtype, device=a.device)
    o3 = _as3d(out)
    if o3.shape != (B, M, N) or o3.stride(2) != 1:
        raise ValueError("out must be [B, M, N] contiguous along N")
    nbytes = workspace_bytes(L.CB_OP_W8A8, B, M, N, K)
    ws = POOL.get(nbytes, a.device)
    st = _strides(a3.stride(0), a3.stride(1), w3.stride(0), w3.stride(1), o3.stride(0), o3.stride(1),
                  ws2.stride(0) if ws2.dim() == 2 else 0)
    code = L.load().cb_w8a8_gemm_dynamic(a3.data_ptr(), dtype_code(a.dtype), q.data_ptr(), s.data_ptr(),
                                         w3.data_ptr(), ws2.data_ptr(), o3.data_ptr(), dtype_code(out.dtype), B, M,
                                         N, K, st, ws.data_ptr(), ws.numel(), _stream(a.device))
    L.check("cb_w8a8_gemm_dynamic", code)
    return out


# ---------------------------------------------------------------------------
# FP8 (e4m3) W8A8
# ---------------------------------------------------------------------------
_FP8_MODES = {"per_token": L.CB_FP8_PER_TOKEN, "per_tensor": L.CB_FP8_PER_TENSOR_DYNAMIC, "static": L.CB_FP8_STATIC}


def quant_act_fp8(a: torch.Tensor, mode: str = "per_token", scale: torch.Tensor | None = None,
                  q: torch.Tensor | None = None):
    """e4m3 quantization of ``a`` ([M, K] or [B, M, K], f16/bf16).

    mode "per_token": one dynamic scale per row (fp32, B*M); "per_tensor": one
    dynamic scale per batch entry (B); "static": ``scale`` (B elements) given.
    Returns ``(q float8_e4m3fn like a, scale)``.
    """
    _require_cuda(a, scale, q)
    a3 = _as3d(a)
    B, M, K = a3.shape
    if a3.stride(2) != 1:
        raise ValueError("activations must be contiguous along K")
    code_mode = _FP8_MODES.get(mode)
    if code_mode is None:
        raise ValueError(f"mode must be one of {sorted(_FP8_MODES)}")
    if mode == "static":
        if scale is None or scale.numel() < B or scale.dtype != torch.float32 or not scale.is_contiguous():
            raise ValueError("static mode needs a contiguous fp32 scale with one value per batch entry")
    elif scale is None:
        scale = torch.empty(B * M if mode == "per_token" else B, dtype=torch.float32, device=a.device)
    if q is None:
        q = torch.empty(a.shape, dtype=torch.float8_e4m3fn, device=a.device)
    q3 = _as3d(q)
    if q3.shape != a3.shape or q.element_size() != 1 or q3.stride(2) != 1:
        raise ValueError("q must be a 1-byte tensor shaped like a, contiguous along K")
    code = L.load().cb_quant_act_fp8(a3.data_ptr(), dtype_code(a.dtype), B, M, K, a3.stride(0), a3.stride(1),
                                     q3.data_ptr(), q3.stride(0), q3.stride(1), scale.data_ptr(),
                                     M if mode == "per_token" else 1, code_mode, _stream(a.device))
    L.check("cb_quant_act_fp8", code)
    return q, scale


def fp8_gemm(aq: torch.Tensor, w_nk: torch.Tensor, a_scale: torch.Tensor, w_scale: torch.Tensor,
             out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
             bias: torch.Tensor | None = None) -> torch.Tensor:
    """``out = ((aq @ w_nk^T) * a_scale) * w_scale (+ bias)`` on e4m3 operands, fp32 accumulation.

    aq: e4m3 [M, K] / [B, M, K]; w_nk: e4m3 [N, K] / [B, N, K] (K contiguous).
    a_scale: B*M values (per token) or B (per tensor); w_scale: B*N (per channel)
    or B (per tensor); bias: optional [N] added in fp32 before the rounding.
    """
    _require_cuda(aq, w_nk, a_scale, w_scale, out, bias)
    a3, w3 = _as3d(aq), _as3d(w_nk)
    B, M, K = a3.shape
    Bw, N, Kw = w3.shape
    if aq.element_size() != 1 or w_nk.element_size() != 1:
        raise ValueError("fp8_gemm expects 1-byte e4m3 operands")
    if Kw != K or Bw != B:
        raise ValueError(f"shape mismatch: aq {tuple(a3.shape)} vs w {tuple(w3.shape)}")
    if a3.stride(2) != 1 or w3.stride(2) != 1:
        raise ValueError("operands must be contiguous along K (weights K-major [N, K])")
    for t, nm in ((a_scale, "a_scale"), (w_scale, "w_scale")):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError(f"{nm} must be contiguous fp32")
    if a_scale.numel() not in (B, B * M):
        raise ValueError("a_scale must have B*M (per token) or B (per tensor) elements")
    if w_scale.numel() not in (B, B * N):
        raise ValueError("w_scale must have B*N (per channel) or B (per tensor) elements")
    a_pt = a_scale.numel() == B and B * M != B
    w_pt = w_scale.numel() == B and B * N != B
    if bias is not None and (bias.numel() != N or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous [N] tensor")
    if out is None:
        out = torch.empty((B, M, N) if aq.dim() == 3 else (M, N), dtype=out_dtype, device=aq.device)
    o3 = _as3d(out)
    if o3.shape != (B, M, N) or o3.stride(2) != 1:
        raise ValueError("out must be [B, M, N] contiguous along N")
    nbytes = workspace_bytes(L.CB_OP_W8A8, B, M, N, K)
    ws = POOL.get(nbytes, aq.device)
    st = _strides(a3.stride(0), a3.stride(1), w3.stride(0), w3.stride(1), o3.stride(0), o3.stride(1),
                  1 if a_pt else M, 1 if w_pt else N)
    code = L.load().cb_fp8_gemm(a3.data_ptr(), a_scale.data_ptr(), int(a_pt), w3.data_ptr(), w_scale.data_ptr(),
                                int(w_pt), _ptr(bias), dtype_code(bias.dtype) if bias is not None else 0,
                                o3.data_ptr(), dtype_code(out.dtype), B, M, N, K, st, ws.data_ptr(), ws.numel(),
                                _stream(aq.device))
    L.check("cb_fp8_gemm", code)
    return out


def repack_w8_kmajor(w_kn: torch.Tensor) -> torch.Tensor:
    """int8 [B, K, N] / [K, N] (N contiguous) -> contiguous [B, N, K] / [N, K]."""
    _require_cuda(w_kn)
    w3 = _as3d(w_kn).contiguous()
    B, K, N = w3.shape
    dst = torch.empty((B, N, K), dtype=torch.int8, device=w_kn.device)
    code = L.load().cb_repack_w8_kmajor(w3.data_ptr(), dst.data_ptr(), B, K, N, _stream(w_kn.device))
    L.check("cb_repack_w8_kmajor", code)
    return dst if w_kn.dim() == 3 else dst[0]


# ---------------------------------------------------------------------------
# W4A16
# ---------------------------------------------------------------------------
def w4_native_bytes(batch: int, K: int, N: int) -> int:
    return int(L.load().cb_w4_native_bytes(batch, K, N))


def repack_w4(src: torch.Tensor, layout: int, K: int, N: int) -> torch.Tensor:
    """Repack int4 weights (reference u8 [B, K/2, N] or int32 [B, K/8, N]) into the native tiled layout."""
    _require_cuda(src)
    s3 = _as3d(src).contiguous()
    B = s3.shape[0]
    if layout == L.CB_W4_REF_U8_KN:
        if src.dtype != torch.uint8 or s3.shape[1:] != (K // 2, N):
            raise ValueError("reference int4 layout is uint8 [B, K/2, N]")
    elif layout == L.CB_W4_I32_K8N:
        if src.dtype != torch.int32 or s3.shape[1:] != (K // 8, N):
            raise ValueError("int32 int4 layout is int32 [B, K/8, N]")
    else:
        raise ValueError(f"unknown source layout {layout}")
    dst = torch.empty(w4_native_bytes(B, K, N), dtype=torch.uint8, device=src.device)
    code = L.load().cb_repack_w4(s3.data_ptr(), layout, dst.data_ptr(), B, K, N, _stream(src.device))
    L.check("cb_repack_w4", code)
    return dst


def w4a16_gemm(a: torch.Tensor, w_native: torch.Tensor, scales: torch.Tensor, N: int, group_size: int,
               out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
               scale_strides: tuple[int, int] | None = None) -> torch.Tensor:
    """``out[b, m, n] = sum_k a[b, m, k] * q[b, k, n] * scales[b, k // group_size, n]``.

    a: f16/bf16 [M, K] / [B, M, K]; w_native: uint8 from ``repack_w4``;
    scales: [G, N] / [B, G, N] (f16/bf16/f32), N contiguous, or [B, N] for the
    per-channel case (group_size >= K). ``scale_strides`` overrides the
    (batch, group) element strides of ``scales``.
    """
    _require_cuda(a, w_native, scales, out)
    a3 = _as3d(a)
    B, M, K = a3.shape
    if a3.stride(2) != 1:
        raise ValueError("activations must be contiguous along K")
    if w_native.dtype != torch.uint8 or w_native.numel() < w4_native_bytes(B, K, N):
        raise ValueError("w_native must be a uint8 native-layout buffer for [B, K, N]")
    if scales.stride(-1) != 1:
        raise ValueError("scales must be contiguous along N")
    if scale_strides is not None:
        s_sb, s_sg = scale_strides
    elif scales.dim() == 3:
        s_sb, s_sg = scales.stride(0), scales.stride(1)
    elif scales.dim() == 2:
        if group_size >= K:  # per-(batch, channel) scales [B, N], the reference layout
            s_sb, s_sg = scales.stride(0), 0
        else:  # [G, N] for a batch of one
            s_sb, s_sg = 0, scales.stride(0)
    else:
        s_sb, s_sg = 0, 0
    if out is None:
        out = torch.empty((B, M, N) if a.dim() == 3 else (M, N), dtype=out_dtype or a.dtype, device=a.device)
    o3 = _as3d(out)
    if o3.shape != (B, M, N) or o3.stride(2) != 1:
        raise ValueError("out must be [B, M, N] contiguous along N")
    nbytes = workspace_bytes(L.CB_OP_W4A16, B, M, N, K)
    ws = POOL.get(nbytes, a.device)
    st = _strides(a3.stride(0), a3.stride(1), s_sb, s_sg, o3.stride(0), o3.stride(1))
    code = L.load().cb_w4a16_gemm(a3.data_ptr(), dtype_code(a.dtype), w_native.data_ptr(), scales.data_ptr(),
                                  dtype_code(scales.dtype), group_size, o3.data_ptr(), dtype_code(out.dtype), B, M,
                                  N, K, st, ws.data_ptr(), ws.numel(), _stream(a.device))
    L.check("cb_w4a16_gemm", code)
    return out


# ---------------------------------------------------------------------------
# W4A4
# ---------------------------------------------------------------------------
def w4a4_gemm(a_packed: torch.Tensor, b_packed: torch.Tensor, K: int, out: torch.Tensor | None = None,
              reference_wrap: bool = False):
    """fp32 ``C = int4(A) @ int4(B)``; A uint8 [M, K/2], B uint8 [K/2, N].

    Nibbles are two's complement int4 unless ``reference_wrap``, which reproduces
    the reference kernel's uint8 arithmetic (negative nibbles enter as 240..255,
    kernels/triton_gemm.py:164-167)."""
    _require_cuda(a_packed, b_packed, out)
    M = a_packed.shape[0]
    N = b_packed.shape[1]
    if a_packed.stride(1) != 1 or b_packed.stride(1) != 1:
        raise ValueError("packed operands must be row-contiguous")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=a_packed.device)
    nbytes = workspace_bytes(L.CB_OP_W4A4, 1, M, N, K)
    ws = POOL.get(nbytes, a_packed.device)
    code = L.load().cb_w4a4_gemm(a_packed.data_ptr(), b_packed.data_ptr(), out.data_ptr(), M, N, K,
                                 a_packed.stride(0), b_packed.stride(0), out.stride(0),
                                 L.CB_W4A4_REF_UINT8_WRAP if reference_wrap else L.CB_W4A4_SIGNED,
                                 ws.data_ptr(), ws.numel(),
                                 _stream(a_packed.device))
    L.check("cb_w4a4_gemm", code)
    return out


# ---------------------------------------------------------------------------
# NVFP4 (e2m1 values, e4m3 scales per 16 elements; vLLM's tensor formats)
# ---------------------------------------------------------------------------
def nvfp4_scale_shape(rows: int, K: int) -> tuple[int, int]:
    """Shape of the swizzled scale tensor: rows padded to 128, K/16 to 4."""
    return (-(-rows // 128) * 128, -(-(K // 16) // 4) * 4)


def nvfp4_quantize(x: torch.Tensor, global_scale: torch.Tensor, q: torch.Tensor | None = None,
                   sf: torch.Tensor | None = None):
    """``x`` [rows, K] f16/bf16 -> (packed e2m1 uint8 [rows, K/2], swizzled e4m3
    scales uint8 ``nvfp4_scale_shape(rows, K)``), with ``global_scale`` one fp32
    on the device (vLLM's ``scaled_fp4_quant(x, global_scale)``)."""
    _require_cuda(x, global_scale, q, sf)
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be [rows, K] with contiguous rows")
    rows, K = x.shape
    if global_scale.dtype != torch.float32 or global_scale.numel() != 1:
        raise ValueError("global_scale must be one fp32 value")
    if q is None:
        q = torch.empty((rows, K // 2), dtype=torch.uint8, device=x.device)
    if sf is None:
        sf = torch.empty(nvfp4_scale_shape(rows, K), dtype=torch.uint8, device=x.device)
    if q.dtype != torch.uint8 or sf.dtype != torch.uint8 or not sf.is_contiguous():
        raise ValueError("q and sf must be uint8, sf contiguous")
    if sf.numel() < nvfp4_scale_shape(rows, K)[0] * nvfp4_scale_shape(rows, K)[1]:
        raise ValueError("sf is too small")
    code = L.load().cb_nvfp4_quantize(x.data_ptr(), dtype_code(x.dtype), rows, K, x.stride(0),
                                      global_scale.data_ptr(), q.data_ptr(), q.stride(0), sf.data_ptr(),
                                      _stream(x.device))
    L.check("cb_nvfp4_quantize", code)
    return q, sf


def nvfp4_gemm(a: torch.Tensor, a_sf: torch.Tensor, b: torch.Tensor, b_sf: torch.Tensor, alpha: torch.Tensor,
               out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
    """``out[m, n] = alpha * A[m] . B[n]`` for packed NVFP4 activations ``a``
    [M, K/2] and weights ``b`` [N, K/2] with their swizzled scales (vLLM's
    ``cutlass_scaled_fp4_mm(a, b, a_sf, b_sf, alpha, out_dtype)``)."""
    _require_cuda(a, a_sf, b, b_sf, alpha, out)
    if a.dtype != torch.uint8 or b.dtype != torch.uint8 or a.dim() != 2 or b.dim() != 2:
        raise ValueError("a and b must be packed uint8 [rows, K/2]")
    M, K = a.shape[0], a.shape[1] * 2
    N = b.shape[0]
    if b.shape[1] * 2 != K:
        raise ValueError("a and b disagree on K")
    if a.stride(1) != 1 or b.stride(1) != 1 or not a_sf.is_contiguous() or not b_sf.is_contiguous():
        raise ValueError("operands must have contiguous rows and contiguous scales")
    if alpha.dtype != torch.float32 or alpha.numel() != 1:
        raise ValueError("alpha must be one fp32 value")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    if out.shape != (M, N) or out.stride(1) != 1:
        raise ValueError("out must be [M, N] contiguous along N")
    nbytes = workspace_bytes(L.CB_OP_NVFP4, 1, M, N, K)
    ws = POOL.get(nbytes, a.device)
    code = L.load().cb_nvfp4_gemm(a.data_ptr(), a_sf.data_ptr(), b.data_ptr(), b_sf.data_ptr(), alpha.data_ptr(),
                                  out.data_ptr(), dtype_code(out.dtype), M, N, K, a.stride(0), b.stride(0),
                                  out.stride(0), ws.data_ptr(), ws.numel(), _stream(a.device))
    L.check("cb_nvfp4_gemm", code)
    return out


def device_status(device: torch.device | None = None) -> int:
    """Synchronising check of the kernels' device-side status words (0 = no timeout)."""
    return POOL.check_status(device)


# ---------------------------------------------------------------------------
# Host-buffer executor (cb_exec_*)
# ---------------------------------------------------------------------------
class HostExecutor:
    """W8A8 dynamic-quant GEMM on host (pinned) activations and outputs.

    Each call enqueues the copy in, the PDL-chained quantizer + GEMM and the
    copy out on the executor's own streams and returns; consecutive calls
    overlap one call's copies with the neighbouring calls' kernels. Outputs are
    valid after ``synchronize()`` (or after work ordered by ``before(stream)``).
    """

    def __init__(self, device: torch.device | int | None = None):
        if device is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        elif isinstance(device, int):
            dev = torch.device("cuda", device)
        else:
            dev = device
        self.device = dev
        self._lib = L.load()
        h = ctypes.c_void_p()
        L.check("cb_exec_create", self._lib.cb_exec_create(dev.index, ctypes.byref(h)))
        self._h = h
        self._call = self._lib.cb_exec_w8a8_dynamic_host

    def close(self):
        if self._h is not None and self._h.value:
            self._lib.cb_exec_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001  (interpreter shutdown)
            pass

    def after(self, stream: torch.cuda.Stream | None = None):
        """Later executor work waits for the work already on ``stream``."""
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        L.check("cb_exec_after", self._lib.cb_exec_after(self._h, s.cuda_stream))

    def before(self, stream: torch.cuda.Stream | None = None):
        """Later work on ``stream`` waits for all executor work enqueued so far."""
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        L.check("cb_exec_before", self._lib.cb_exec_before(self._h, s.cuda_stream))

    def synchronize(self) -> int:
        """Waits for all executor work; returns the device status word (0 = no timeout)."""
        st = ctypes.c_int(0)
        code = self._lib.cb_exec_synchronize(self._h, ctypes.byref(st))
        if code not in (L.CB_OK, L.CB_ERR_DEVICE_TIMEOUT):
            L.check("cb_exec_synchronize", code)
        return st.value

    def w8a8_dynamic_host(self, a_host: torch.Tensor, w_nk: torch.Tensor, w_scale: torch.Tensor,
                          out_host: torch.Tensor) -> torch.Tensor:
        """``out_host = w8a8_bmm_full(a_host, w)`` with ``a_host`` f16/bf16 [M, K] / [B, M, K] and
        ``out_host`` f16/bf16/f32 [M, N] / [B, M, N] contiguous host tensors (pinned for overlap);
        ``w_nk`` int8 [N, K] / [B, N, K] (K contiguous) and ``w_scale`` fp32 [N] / [B, N] on this device."""
        if a_host.is_cuda or out_host.is_cuda or not a_host.is_contiguous() or not out_host.is_contiguous():
            raise ValueError("a_host and out_host must be contiguous host tensors")
        if not w_nk.is_cuda or w_nk.dtype != torch.int8 or w_nk.stride(-1) != 1 or not w_scale.is_cuda:
            raise ValueError("w_nk must be an int8 CUDA tensor contiguous along K, w_scale a CUDA tensor")
        if w_scale.dtype != torch.float32:
            raise ValueError("w_scale must be fp32")
        K = a_host.shape[-1]
        M = a_host.shape[-2]
        B = a_host.shape[0] if a_host.dim() == 3 else 1
        N = w_nk.shape[-2]
        if w_nk.shape[-1] != K or out_host.shape[-1] != N or out_host.numel() != B * M * N:
            raise ValueError("shape mismatch between a_host, w_nk and out_host")
        wsb = w_nk.stride(0) if w_nk.dim() == 3 else 0
        ssb = w_scale.stride(0) if w_scale.dim() == 2 else 0
        code = self._call(self._h, a_host.data_ptr(), _DTYPE_CODE[a_host.dtype], w_nk.data_ptr(), w_scale.data_ptr(),
                          wsb, w_nk.stride(-2), ssb, out_host.data_ptr(), _DTYPE_CODE[out_host.dtype], B, M, N, K)
        if code:
            L.check("cb_exec_w8a8_dynamic_host", code)
        return out_host
