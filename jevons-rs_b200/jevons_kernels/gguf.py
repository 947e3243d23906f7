"""GGUF reader and weight loader over libjk.so -- jevons-formats' `Gguf`.

Mirrors crates/jevons-formats/src/gguf.rs: `Gguf.open` (:234-324), `get` / `u64` / `f32`
(:326-343), `tensor` (:345-350), `read` / `read_range` / `read_f32` (:352-391), and `TensorInfo`
(:148-162). Parsing and validation run in the library's native reader; errors raise JkError with
the reference's messages. `load_qmatrix` is the load path GGUF -> raw blocks -> QMatrix.upload.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from ._lib import GgufTensorInfo, JkError, check, load
from .formats import TensorType

# GGUF metadata value kinds (gguf.rs:195-231)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_INTS = (U8, I8, U16, I16, U32, I32, U64, I64)


@dataclass
class TensorInfo:
    name: str
    dims: list[int]   # GGML order: dims[0] is the contiguous row length
    kind: int          # GGML type id
    offset: int        # absolute byte offset in the file
    bytes: int

    def elements(self) -> int:
        return int(np.prod(self.dims, dtype=object))


class Gguf:
    """An open GGUF file: metadata and tensor table validated, tensor data read on demand."""

    def __init__(self, handle):
        self._h = handle

    @staticmethod
    def open(path: str) -> "Gguf":
        h = ctypes.c_void_p()
        check(load().jk_gguf_open(str(path).encode(), ctypes.byref(h)))
        return Gguf(h)

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            load().jk_gguf_close(self._h)
            self._h = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def handle(self):
        return self._h

    # ---- tensors ----------------------------------------------------------------------------
    @staticmethod
    def _info(ti: GgufTensorInfo) -> TensorInfo:
        return TensorInfo(ti.name.decode(), [int(ti.dims[d]) for d in range(ti.n_dims)], int(ti.type), int(ti.offset),
                          int(ti.bytes))

    @property
    def tensors(self) -> dict[str, TensorInfo]:
        out = {}
        for i in range(load().jk_gguf_tensor_count(self._h)):
            ti = GgufTensorInfo()
            check(load().jk_gguf_tensor_at(self._h, i, ctypes.byref(ti)))
            info = self._info(ti)
            out[info.name] = info
        return out

    def tensor(self, name: str) -> TensorInfo:
        ti = GgufTensorInfo()
        check(load().jk_gguf_tensor(self._h, name.encode(), ctypes.byref(ti)))
        return self._info(ti)

    def read_range(self, info: TensorInfo, start: int, length: int) -> bytes:
        buf = ctypes.create_string_buffer(max(int(length), 1))
        check(load().jk_gguf_read(self._h, info.name.encode(), int(start), int(length), buf))
        return buf.raw[: int(length)]

    def read(self, info: TensorInfo) -> bytes:
        return self.read_range(info, 0, info.bytes)

    def read_f32(self, name: str) -> np.ndarray:
        info = self.tensor(name)
        out = np.empty(max(info.bytes // 4, 1), np.float32)
        check(load().jk_gguf_read_f32(self._h, name.encode(), out.ctypes.data_as(ctypes.c_void_p), out.size))
        return out[: info.bytes // 4]

    # ---- metadata ---------------------------------------------------------------------------
    def _kind(self, key: str):
        kind, elem, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
        check(load().jk_gguf_value_kind(self._h, key.encode(), ctypes.byref(kind), ctypes.byref(elem), ctypes.byref(n)))
        return kind.value, elem.value, n.value

    def _scalar(self, key: str, kind: int, index: int):
        lib, k = load(), key.encode()
        if kind == STRING:
            s, n = ctypes.c_char_p(), ctypes.c_size_t()
            check(lib.jk_gguf_str(self._h, k, index, ctypes.byref(s), ctypes.byref(n)))
            return ctypes.string_at(s, n.value).decode("utf-8")
        if kind == BOOL:
            b = ctypes.c_int()
            check(lib.jk_gguf_bool(self._h, k, index, ctypes.byref(b)))
            return bool(b.value)
        if kind in (F32, F64):  # as f32, as Gguf::f32 reads floats
            f = ctypes.c_float()
            check(lib.jk_gguf_f32(self._h, k, index, ctypes.byref(f)))
            return float(f.value)
        if kind in _INTS:
            v = ctypes.c_int64()
            st = lib.jk_gguf_i64(self._h, k, index, ctypes.byref(v))
            if st == 0:
                return int(v.value)
            u = ctypes.c_uint64()
            check(lib.jk_gguf_u64(self._h, k, index, ctypes.byref(u)))
            return int(u.value)
        raise JkError(1, f"metadata kind {kind} of {key} has no scalar reader")

    def get(self, key: str):
        """The metadata value (Gguf::get): int, float (as f32), bool, str or a list of them."""
        kind, elem, n = self._kind(key)
        if kind == ARRAY:
            return [self._scalar(key, elem, i) for i in range(n)]
        return self._scalar(key, kind, -1)

    def u64(self, key: str) -> int:
        """Gguf::u64 (gguf.rs:332-336)."""
        v = ctypes.c_uint64()
        check(load().jk_gguf_u64(self._h, key.encode(), -1, ctypes.byref(v)))
        return int(v.value)

    def f32(self, key: str) -> float:
        """Gguf::f32 (gguf.rs:338-343)."""
        v = ctypes.c_float()
        check(load().jk_gguf_f32(self._h, key.encode(), -1, ctypes.byref(v)))
        return float(v.value)


def load_qmatrix(gpu, g: Gguf, name: str):
    """One weight tensor -> device QMatrix [experts * n, k] (k = dims[0], n = dims[1])."""
    from .gemm import QMatrix
    out = ctypes.c_void_p()
    check(load().jk_qmatrix_from_gguf(gpu.device, g.handle, name.encode(), ctypes.byref(out)))
    return QMatrix(out.value)


__all__ = ["Gguf", "TensorInfo", "TensorType", "load_qmatrix"]
