"""GGML block types and host-side repacking -- the `jevons-formats` items the matmul path uses.

Mirrors crates/jevons-formats/src/gguf.rs:109-145 (`TensorType`, `block()`) and
crates/jevons-formats/src/quant.rs:13-193 (`q4k_scale_min`, `dequantize`, `Packed`, `packed_words`,
`pack`).
All work happens in libjk.so; this module only marshals arguments.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass

import numpy as np

from ._lib import check, load


class TensorType(enum.IntEnum):
    """GGML storage type ids (gguf.rs:110-132). Unknown ids are rejected by `block()`."""

    F32 = 0
    F16 = 1
    Q5_0 = 6
    Q8_0 = 8
    Q4K = 12
    Q6K = 14

    def block(self):
        """(elements per block, bytes per block) -- TensorType::block (gguf.rs:134-145)."""
        return block(int(self))


def block(type_id: int):
    e, b = ctypes.c_uint64(), ctypes.c_uint64()
    st = load().jk_tensor_type_block(int(type_id), ctypes.byref(e), ctypes.byref(b))
    if st != 0:
        return None
    return e.value, b.value


def q4k_scale_min(j: int, scales) -> tuple:
    """quant.rs:14-23: the 6-bit (scale, min) pair j of a Q4_K super-block's 12 scale bytes."""
    buf = (ctypes.c_uint8 * 12).from_buffer_copy(bytes(scales)[:12])
    sc, mn = ctypes.c_uint8(), ctypes.c_uint8()
    check(load().jk_q4k_scale_min(int(j), buf, ctypes.byref(sc), ctypes.byref(mn)))
    return sc.value, mn.value


def packed_words(kind) -> tuple:
    """quant.rs:128-136: words per block of the (q, h, s, d) regions."""
    w = (ctypes.c_size_t * 4)()
    check(load().jk_packed_words(int(kind), w))
    return tuple(w)


@dataclass
class Packed:
    """quant.rs:111-117: structure-of-arrays regions (u32 words, d as f32)."""

    q: np.ndarray
    h: np.ndarray
    s: np.ndarray
    d: np.ndarray


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p) if a.size else None


def pack(kind, raw) -> Packed:
    """quant.rs:156-193: repacks whole GGML blocks into the SoA regions (values unchanged)."""
    raw = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray))
                               else np.asarray(raw).view(np.uint8).reshape(-1))
    bk = block(int(kind))
    size = bk[1] if bk else 1
    blocks = raw.size // size if size else 0
    wq, wh, ws, wd = packed_words(kind)
    q = np.zeros(blocks * wq, np.uint32)
    h = np.zeros(blocks * wh, np.uint32)
    s = np.zeros(blocks * ws, np.uint32)
    d = np.zeros(blocks * wd, np.float32)
    check(load().jk_pack(int(kind), raw.ctypes.data_as(ctypes.c_void_p), raw.size, _ptr(q), q.size, _ptr(h),
                         h.size, _ptr(s), s.size, _ptr(d), d.size))
    return Packed(q, h, s, d)


def dequantize(kind, raw) -> np.ndarray:
    """quant.rs:83-101 on the host (jk_dequantize): whole blocks of `kind` -> f32, bit-exact."""
    raw = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray))
                               else np.asarray(raw).view(np.uint8).reshape(-1))
    bk = block(int(kind))
    if bk is None:  # raises JK_ERR_UNSUPPORTED "unsupported tensor type"
        check(load().jk_dequantize(int(kind), None, 0, None, 0))
    elems, size = bk
    out = np.empty(raw.size // size * elems if raw.size % size == 0 else 0, np.float32)
    check(load().jk_dequantize(int(kind), _ptr(raw), raw.size, _ptr(out), out.size))
    return out
