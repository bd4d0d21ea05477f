"""Offline weight packer and on-disk format for the sm_100a kernels.

The reference keeps int4 weights as ``uint8 [B, K/2, N]`` (even k in the low
nibble, profiling/bench_l2_barrier.py:92-99) or ``int32 [B, K/8, N]`` and int8
weights as ``[B, K, N]`` (profiling/w8a8/w8a8_bmm.py:84-89); the kernels read
the native tiled int4 layout (include/cb200.h ``CB_W4_NATIVE``) and K-major int8.
This module converts on the host (no GPU needed, so weights can be prepared
once, offline) and stores the kernel-ready bytes with their scales:

  file  = b"CBW1" | u32 header length | JSON header | zero padding to 64 |
          tensor blobs, each starting on a 64-byte boundary
  header = {"version": 1, "meta": {...},
            "tensors": [{"name", "kind", "dtype", "shape", "offset", "nbytes",
                         "crc32", and per kind "batch", "K", "N", "group_size"}]}

``kind`` is ``w4_native`` (uint8 bytes of the native layout), ``w8_kmajor``
(int8 [B, N, K]) or ``scales`` / ``raw`` (any numpy dtype). ``load`` checks
every CRC and returns numpy arrays, or torch tensors on ``device``.
"""

from __future__ import annotations

import json
import struct
import zlib
from dataclasses import dataclass, field

import numpy as np

MAGIC = b"CBW1"
VERSION = 1
ALIGN = 64

# stored position of nibble k0..k7 inside a native 32-bit word (order k0,k2,k4,k6,k1,k3,k5,k7)
_POS = np.array([0, 4, 1, 5, 2, 6, 3, 7], dtype=np.uint32)

W4_REF_U8_KN = 0
W4_I32_K8N = 1


def _nibbles(src: np.ndarray, layout: int, K: int, N: int) -> np.ndarray:
    """Unsigned nibbles uint8 [B, K, N] of a reference-layout int4 tensor."""
    s = np.asarray(src)
    if layout == W4_REF_U8_KN:
        s = s.reshape(-1, K // 2, N).astype(np.uint8)
        out = np.empty((s.shape[0], K, N), dtype=np.uint8)
        out[:, 0::2, :] = s & 0xF
        out[:, 1::2, :] = s >> 4
        return out
    if layout == W4_I32_K8N:
        u = s.reshape(-1, K // 8, N).view(np.uint32) if s.dtype == np.int32 else s.reshape(-1, K // 8, N).astype(np.uint32)
        out = np.empty((u.shape[0], K, N), dtype=np.uint8)
        for j in range(8):
            out[:, j::8, :] = (u >> np.uint32(4 * j)) & 0xF
        return out
    raise ValueError(f"unknown int4 layout {layout}")


def native_int4(src: np.ndarray, layout: int, K: int, N: int) -> np.ndarray:
    """Reference-layout int4 weights -> flat uint8 bytes of the native tiled layout:
    per (batch, 128-row n-tile, 128-k k-tile) one 8 KiB tile; row r of a tile is
    four 16-byte chunks (32 k each) stored at chunk ^ ((r >> 1) & 3); a chunk's
    four words hold 8 consecutive k each, nibble positions _POS."""
    nib = _nibbles(src, layout, K, N)
    B = nib.shape[0]
    nt, kt = -(-N // 128), -(-K // 128)
    full = np.zeros((B, kt * 128, nt * 128), dtype=np.uint32)
    full[:, :K, :N] = nib
    # [B, kt, k128, nt, r128] -> [B, nt, kt, r, chunk, word, j]
    t = full.reshape(B, kt, 128, nt, 128).transpose(0, 3, 1, 4, 2).reshape(B, nt, kt, 128, 4, 4, 8)
    words = (t << (np.uint32(4) * _POS)).sum(axis=-1, dtype=np.uint32)  # nibbles occupy disjoint bits
    rows = np.arange(128)
    stored = np.empty_like(words)
    for c in range(4):
        stored[:, :, :, rows, c ^ ((rows >> 1) & 3), :] = words[:, :, :, rows, c, :]
    return np.ascontiguousarray(stored).view(np.uint8).reshape(-1)


def kmajor_int8(w_kn: np.ndarray) -> np.ndarray:
    """int8 [B, K, N] (or [K, N]) -> contiguous [B, N, K]."""
    w = np.asarray(w_kn, dtype=np.int8)
    if w.ndim == 2:
        w = w[None]
    return np.ascontiguousarray(w.transpose(0, 2, 1))


@dataclass
class PackedInt4:
    native: np.ndarray  # uint8, native layout
    scales: np.ndarray  # [B, K/group, N] or per-channel [B, N]
    batch: int
    K: int
    N: int
    group_size: int


@dataclass
class PackedInt8:
    w_nk: np.ndarray  # int8 [B, N, K]
    scales: np.ndarray  # fp32 [B, N]


def pack_int4(src, layout: int, K: int, N: int, scales, group_size: int) -> PackedInt4:
    """``scales`` may be a numpy array or a torch tensor (bf16 kept as bf16)."""
    src = _to_numpy(src)
    native = native_int4(src, layout, K, N)
    B = np.asarray(src).reshape(-1, *np.asarray(src).shape[-2:]).shape[0]
    return PackedInt4(native, _to_numpy(scales), B, K, N, group_size)


def pack_int8(w_kn, scales) -> PackedInt8:
    return PackedInt8(kmajor_int8(_to_numpy(w_kn)), np.ascontiguousarray(_to_numpy(scales), dtype=np.float32))


class _Bf16(np.ndarray):
    """uint16 bit patterns of a bfloat16 tensor (stored with dtype name 'bfloat16')."""

    def __new__(cls, a):
        return np.asarray(a, dtype=np.uint16).view(cls)


@dataclass
class _Entry:
    name: str
    kind: str
    array: np.ndarray
    extra: dict = field(default_factory=dict)


def _entry(name: str, kind: str, a, extra: dict) -> _Entry:
    if isinstance(a, _Bf16):
        return _Entry(name, kind, np.asarray(a).view(np.uint16), {**extra, "_dtype": "bfloat16"})
    return _Entry(name, kind, a, extra)


def _entries(tensors: dict) -> list[_Entry]:
    out = []
    for name, t in tensors.items():
        if isinstance(t, PackedInt4):
            info = {"batch": t.batch, "K": t.K, "N": t.N, "group_size": t.group_size}
            out.append(_Entry(name, "w4_native", np.asarray(t.native, dtype=np.uint8), info))
            out.append(_entry(name + ".scales", "scales", t.scales, {}))
        elif isinstance(t, PackedInt8):
            B, N, K = t.w_nk.shape
            out.append(_Entry(name, "w8_kmajor", t.w_nk, {"batch": B, "K": K, "N": N}))
            out.append(_entry(name + ".scales", "scales", t.scales, {}))
        else:
            out.append(_entry(name, "raw", t, {}))
    return out


def save(path: str, tensors: dict, meta: dict | None = None) -> None:
    """Writes packed weights (PackedInt4 / PackedInt8) and raw arrays. torch tensors
    are accepted and stored by dtype name (bfloat16 as its 16-bit pattern)."""
    ents = _entries({k: _to_numpy(v) for k, v in tensors.items()})
    descs, blobs, offset = [], [], 0
    for e in ents:
        a = np.ascontiguousarray(e.array)
        raw = a.view(np.uint8).reshape(-1).tobytes() if a.size else b""
        dname = e.extra.pop("_dtype", None) or a.dtype.name
        d = {"name": e.name, "kind": e.kind, "dtype": dname, "shape": list(a.shape), "offset": offset,
             "nbytes": len(raw), "crc32": zlib.crc32(raw) & 0xFFFFFFFF, **e.extra}
        descs.append(d)
        blobs.append(raw)
        offset += len(raw)
        offset += (-offset) % ALIGN
    header = json.dumps({"version": VERSION, "meta": meta or {}, "tensors": descs}).encode()
    head = MAGIC + struct.pack("<I", len(header)) + header
    head += b"\0" * ((-len(head)) % ALIGN)
    with open(path, "wb") as f:
        f.write(head)
        pos = 0
        for d, raw in zip(descs, blobs):
            f.write(b"\0" * (d["offset"] - pos))
            f.write(raw)
            pos = d["offset"] + len(raw)


def _to_numpy(v):
    try:
        import torch
    except ImportError:  # pragma: no cover
        torch = None
    if torch is not None and isinstance(v, torch.Tensor):
        t = v.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            return _Bf16(t.view(torch.int16).numpy().view(np.uint16))
        return t.numpy()
    if isinstance(v, PackedInt4):
        return PackedInt4(_to_numpy(v.native), _to_numpy(v.scales), v.batch, v.K, v.N, v.group_size)
    if isinstance(v, PackedInt8):
        return PackedInt8(_to_numpy(v.w_nk), _to_numpy(v.scales))
    return v


def load(path: str, device=None) -> dict:
    """Reads a file written by ``save``. Returns {name: PackedInt4 | PackedInt8 | array};
    with ``device`` the arrays are torch tensors on it (bf16 restored)."""
    with open(path, "rb") as f:
        data = f.read()
    if data[:4] != MAGIC:
        raise ValueError("not a CBW1 weight file")
    (hlen,) = struct.unpack("<I", data[4:8])
    header = json.loads(data[8:8 + hlen])
    if header.get("version") != VERSION:
        raise ValueError(f"unsupported version {header.get('version')}")
    base = 8 + hlen + ((-(8 + hlen)) % ALIGN)
    arrays = {}
    for d in header["tensors"]:
        raw = data[base + d["offset"]: base + d["offset"] + d["nbytes"]]
        if len(raw) != d["nbytes"] or (zlib.crc32(raw) & 0xFFFFFFFF) != d["crc32"]:
            raise ValueError(f"tensor {d['name']}: size or checksum mismatch")
        dt = np.uint16 if d["dtype"] == "bfloat16" else np.dtype(d["dtype"])
        a = np.frombuffer(raw, dtype=dt).reshape(d["shape"]).copy()
        arrays[d["name"]] = (d, a)
    out = {}
    for name, (d, a) in arrays.items():
        if d["kind"] == "scales":
            continue
        sc = arrays.get(name + ".scales")
        if d["kind"] == "w4_native":
            out[name] = PackedInt4(_dev(a, "uint8", device), _dev(sc[1], sc[0]["dtype"], device), d["batch"], d["K"],
                                   d["N"], d["group_size"])
        elif d["kind"] == "w8_kmajor":
            out[name] = PackedInt8(_dev(a, "int8", device), _dev(sc[1], sc[0]["dtype"], device))
        else:
            out[name] = _dev(a, d["dtype"], device)
    return out


def _dev(a: np.ndarray, dtype_name: str, device):
    if device is None:
        return a
    import torch

    if dtype_name == "bfloat16":
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(a).to(device)
