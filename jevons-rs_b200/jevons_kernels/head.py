"""Q6_K embedding-table ("head") operators over libjk.so.

Mirrors the host launchers of crates/jevons-gemma4-diffusion/src/gpu/ops.rs:

  * `embed`               ops.rs:921-954   (kernel embed_q6k, :223-291)
  * `pick`                ops.rs:1133-1157 (kernel pick_logits, :590-635)
  * `q6k_transposed_f16`  ops.rs:732-749   (kernel q6k_transpose, :672-715)
  * `softcap_logits`      ops.rs:1159-1168 (kernel softcap, :751-760)

The reference's `Q6kTable` (ops.rs:912-919) is the packed regions of the Q6_K embedding
`QMatrix` (model.rs:181-184); here the operators take that `QMatrix` itself. Buffers are `Buf`s
(torch tensors); every call is asynchronous on the current torch stream and runs in libjk.so.
Token ids and pairs are int32 tensors holding the reference's u32 values.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import JkError, check, load
from .formats import TensorType
from .gemm import Buf, Gpu, QMatrix, _stream


def _need(buf: Buf, count: int, dtype, what: str) -> None:
    if buf.tensor.dtype != dtype:
        raise JkError(1, f"{what} must be {dtype}")
    if buf.len() < count:
        raise JkError(1, f"{what} holds {buf.len()} values, needs {count}")


def _table(table: QMatrix, d: int, what: str) -> None:
    if table.kind != TensorType.Q6K:
        raise JkError(2, f"{what}: the table must be Q6_K")
    if table.k != d:
        raise JkError(3, f"{what}: table rows hold {table.k} values, d = {d}")


def embed(gpu: Gpu, tokens: Buf, table: QMatrix, w_attn: Buf, sc: Buf | None, out: Buf, x_attn: Buf, rows: int,
          first_canvas: int, d: int, eps: float) -> None:
    """Embedding rows `out[t] = E[tokens[t]] * sqrt(d)`; rows t >= first_canvas add `sc` (the
    self-conditioning rows, when given) and are RMS-normalised without weight; `x_attn[t]` =
    f16(norm(out[t]) * w_attn) (ops::embed, ops.rs:921-954)."""
    _table(table, d, "embed")
    _need(tokens, rows, torch.int32, "tokens")
    _need(w_attn, d, torch.float32, "w_attn")
    _need(out, rows * d, torch.float32, "out")
    _need(x_attn, rows * d, torch.float16, "x_attn")
    if sc is not None:
        _need(sc, max(rows - first_canvas, 0) * d, torch.float32, "sc")
    check(load().jk_embed_q6k(table.handle, tokens.ptr(), rows, w_attn.ptr(), sc.ptr() if sc is not None else None,
                              first_canvas, ctypes.c_float(eps), out.ptr(), x_attn.ptr(), _stream()))


def pick(gpu: Gpu, x: Buf, pairs: Buf, count: int, table: QMatrix, out: Buf, cap: float, d: int) -> None:
    """Logits `out[p] = cap * tanh(x[row] . E[token] / cap)` for the (row, token) pairs
    `pairs[2p], pairs[2p+1]`; x is f16 [rows, d] (ops::pick, ops.rs:1133-1157)."""
    _table(table, d, "pick")
    _need(pairs, 2 * count, torch.int32, "pairs")
    _need(out, count, torch.float32, "out")
    if x.tensor.dtype != torch.float16:
        raise JkError(1, "pick: x must be f16")
    check(load().jk_pick_logits(table.handle, x.ptr(), x.len() // d, pairs.ptr(), count, ctypes.c_float(cap),
                                out.ptr(), _stream()))


def q6k_transposed_f16(gpu: Gpu, table: QMatrix, rows: int, d: int, out: Buf | None = None) -> Buf:
    """Dequantized, transposed FP16 copy [d, rows] of the table (ops.rs:732-749), in a new
    buffer or in `out` (f16, rows * d values) when given."""
    _table(table, d, "q6k_transposed_f16")
    if rows != table.experts * table.n:
        raise JkError(3, f"q6k_transposed_f16: the table has {table.experts * table.n} rows, not {rows}")
    if out is None:
        out = gpu.empty(rows * d, torch.float16)
    else:
        _need(out, rows * d, torch.float16, "out")
    check(load().jk_q6k_transpose_f16(table.handle, out.ptr(), rows * d, _stream()))
    return out


def softcap_logits(gpu: Gpu, x: Buf, len_: int, cap: float) -> None:
    """In-place `x = cap * tanh(x / cap)` over the first len_ f32 values (ops.rs:1159-1168)."""
    _need(x, len_, torch.float32, "x")
    check(load().jk_softcap(x.ptr(), len_, ctypes.c_float(cap), _stream()))
