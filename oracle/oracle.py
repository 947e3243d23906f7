"""TEST INFRASTRUCTURE ONLY: numpy / ctypes front end of the CPU oracle.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may import this module. The product library never calls it.

Two restatements of the reference's GGML block decoding live here, and the tests require
them to agree bit for bit:

* ``dequantize`` -- the C library ``libjk_oracle.so`` built from ``jk_oracle.c``, which follows
  the reference's CPU code ``crates/jevons-formats/src/quant.rs:14-101`` statement by statement;
* ``dequantize_words`` -- a vectorised numpy decode that follows the reference's GPU decode
  from packed 32-bit words (``crates/jevons-kernels/src/gemm.rs:286-384``, ``unpack_slot``), an
  independent formulation of the same format inside the reference itself.

``matmul_f64`` is the f64 product of the reference's GPU tests
(``crates/jevons-gemma4-diffusion/src/gpu/tests.rs:445-452``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libjk_oracle.so")

# GGML type ids (crates/jevons-formats/src/gguf.rs:123-131)
F32, F16, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 6, 8, 12, 14
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_K: (256, 144), Q5_0: (32, 22), Q6_K: (256, 210), Q8_0: (32, 34)}

_lib = None


def build(force: bool = False) -> str:
    """Compiles libjk_oracle.so from jk_oracle.c (gcc, OpenMP, no FP contraction)."""
    src = os.path.join(HERE, "jk_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call([
            "gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared",
            src, "-o", LIB_PATH, "-lm",
        ])
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        P, S = ctypes.c_void_p, ctypes.c_size_t
        L.jko_block.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]
        L.jko_half_to_float.argtypes = [ctypes.c_uint16]
        L.jko_half_to_float.restype = ctypes.c_float
        L.jko_q4k_scale_min.argtypes = [ctypes.c_int, P, P, P]
        L.jko_dequantize.argtypes = [ctypes.c_int, P, S, P, S]
        L.jko_packed_words.argtypes = [ctypes.c_int, P]
        L.jko_pack.argtypes = [ctypes.c_int, P, S, P, P, P, P]
        L.jko_matmul_f64.argtypes = [P, S, S, P, S, P]
        L.jko_row_norms.argtypes = [P, S, S, P]
        L.jko_gemv_fused.argtypes = [ctypes.c_int, P, S, S, P, S, P, ctypes.c_int]
        L.jko_max_threads.restype = ctypes.c_int
        L.jko_quantize_act_q8.argtypes = [P, S, S, P, P, S]
        L.jko_matmul_q8_int8.argtypes = [P, S, S, P, P, S, S, P, P]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def block(kind: int):
    e, b = ctypes.c_uint64(), ctypes.c_uint64()
    if not lib().jko_block(kind, ctypes.byref(e), ctypes.byref(b)):
        return None
    return e.value, b.value


def half_to_float(h: int) -> float:
    return lib().jko_half_to_float(h)


def q4k_scale_min(j: int, q: bytes):
    buf = np.frombuffer(bytes(q), dtype=np.uint8).copy()
    sc, m = ctypes.c_uint8(), ctypes.c_uint8()
    lib().jko_q4k_scale_min(j, _ptr(buf), ctypes.byref(sc), ctypes.byref(m))
    return sc.value, m.value


class OracleError(ValueError):
    pass


def dequantize(kind: int, raw, out_len: int | None = None) -> np.ndarray:
    """quant.rs:83-101: whole rows of ``kind`` to f32. Raises on unsupported type / bad sizes."""
    raw = np.ascontiguousarray(np.frombuffer(bytes(raw), dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw.view(np.uint8).reshape(-1))
    bk = block(kind)
    if bk is None:
        raise OracleError("unsupported tensor type")
    if out_len is None:
        out_len = raw.size // bk[1] * bk[0]
    out = np.empty(out_len, dtype=np.float32)
    rc = lib().jko_dequantize(kind, _ptr(raw), raw.size, _ptr(out), out.size)
    if rc == 1:
        raise OracleError("unsupported tensor type")
    if rc == 2:
        raise OracleError("dequantization size mismatch")
    return out


def packed_words(kind: int):
    w = np.zeros(4, dtype=np.uint64)
    lib().jko_packed_words(kind, _ptr(w))
    return tuple(int(v) for v in w)


def pack(kind: int, raw):
    """quant.rs:156-193: returns (q, h, s, d) numpy arrays (u32, u32, u32, f32)."""
    raw = np.ascontiguousarray(np.frombuffer(bytes(raw), dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw.view(np.uint8).reshape(-1))
    bk = block(kind)
    if bk is None or kind not in (Q4_K, Q6_K, Q5_0, Q8_0):
        raise OracleError(f"{kind} has no GPU block layout")
    if raw.size % bk[1]:
        raise OracleError("tensor is not a whole number of blocks")
    blocks = raw.size // bk[1]
    wq, wh, ws, wd = packed_words(kind)
    q = np.zeros(blocks * wq, np.uint32)
    h = np.zeros(blocks * wh, np.uint32)
    s = np.zeros(blocks * ws, np.uint32)
    d = np.zeros(blocks * wd, np.float32)
    rc = lib().jko_pack(kind, _ptr(raw), raw.size, _ptr(q), _ptr(h), _ptr(s), _ptr(d))
    if rc:
        raise OracleError("pack failed")
    return q, h, s, d


def matmul_f64(x: np.ndarray, w_dense: np.ndarray) -> np.ndarray:
    """tests.rs:445-452: out[r, c] = sum_j f64(x[r, j]) * f64(w[c, j]); x already rounded."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w_dense = np.ascontiguousarray(w_dense, dtype=np.float32)
    m, k = x.shape
    n = w_dense.shape[0]
    assert w_dense.shape[1] == k
    out = np.empty((m, n), dtype=np.float64)
    lib().jko_matmul_f64(_ptr(x), m, k, _ptr(w_dense), n, _ptr(out))
    return out


def row_norms(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape[0], dtype=np.float64)
    lib().jko_row_norms(_ptr(a), a.shape[0], a.shape[1], _ptr(out))
    return out


def gemv_fused(kind: int, raw: np.ndarray, n: int, k: int, x: np.ndarray, threads: int = 0) -> np.ndarray:
    """CPU baseline: fused dequant-dot over raw GGML rows (f32 accumulate, OpenMP)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m = x.shape[0]
    out = np.empty((m, n), dtype=np.float32)
    raw = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
    rc = lib().jko_gemv_fused(kind, _ptr(raw), n, k, _ptr(x), m, _ptr(out), threads)
    if rc:
        raise OracleError("gemv_fused: bad arguments")
    return out


def max_threads() -> int:
    return lib().jko_max_threads()


# ---------------------------------------------------------------------------------------------
# Second restatement: decode from packed words, following the reference's GPU unpacking
# (crates/jevons-kernels/src/gemm.rs:32-68 helpers, :286-384 unpack_slot), vectorised.
# ---------------------------------------------------------------------------------------------

def _f16(u16):
    return u16.astype(np.uint16).view(np.float16).astype(np.float32)


def dequantize_words(kind: int, raw) -> np.ndarray:
    with np.errstate(all="ignore"):  # NaN/inf scales decode like the reference, silently
        return _dequantize_words(kind, raw)


def _dequantize_words(kind: int, raw) -> np.ndarray:
    raw = np.ascontiguousarray(np.frombuffer(bytes(raw), dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw.view(np.uint8).reshape(-1))
    if kind == Q4_K:
        blk = raw.reshape(-1, 144)
        words = blk.view("<u4")  # [B, 36]
        head = words[:, :4]
        d = _f16(head[:, 0] & 0xFFFF)
        dmin = _f16(head[:, 0] >> 16)
        s = [head[:, 1], head[:, 2], head[:, 3]]

        def byte3(i):
            return (s[i // 4] >> np.uint32(8 * (i % 4))) & 0xFF

        out = np.empty((blk.shape[0], 256), np.float32)
        for step in range(4):  # gemm.rs:171-199 / :311-336 (pair = step % 4)
            for hh in range(2):
                j = 2 * step + hh
                lo = j < 4
                jj = j if lo else j - 4
                a, b, c = byte3(jj), byte3(jj + 4), byte3(jj + 8)
                sc = (a & 63) if lo else ((c & 15) | ((a >> 6) << 4))
                mn = (b & 63) if lo else ((c >> 4) | ((b >> 6) << 4))
                dd = (d * sc.astype(np.float32)).astype(np.float32)
                mm = (dmin * mn.astype(np.float32)).astype(np.float32)
                qw = words[:, 4 + 8 * step: 4 + 8 * step + 8]  # 32 bytes of qs
                qb = qw.view(np.uint8).reshape(-1, 32)
                q = ((qb >> (4 * hh)) & 15).astype(np.float32)
                out[:, 64 * step + 32 * hh: 64 * step + 32 * hh + 32] = (dd[:, None] * q).astype(np.float32) - mm[:, None]
        return out.reshape(-1)
    if kind == Q6_K:
        blk = raw.reshape(-1, 210)
        ql = blk[:, :128]
        qh = blk[:, 128:192]
        sc = blk[:, 192:208].view(np.int8).astype(np.float32)
        d = _f16(blk[:, 208].astype(np.uint16) | (blk[:, 209].astype(np.uint16) << 8))
        out = np.empty((blk.shape[0], 256), np.float32)
        for c in range(4):  # gemm.rs:364-383: chunk c of 64 values, sub jj = 2*(c%2)+hh
            nh = c // 2
            for hh in range(2):
                jj = 2 * (c % 2) + hh
                nib = 4 * (jj // 2)
                hshift = 2 * jj
                qlb = ql[:, 64 * nh + 32 * (jj % 2): 64 * nh + 32 * (jj % 2) + 32]
                qhb = qh[:, 32 * nh: 32 * nh + 32]
                q = ((qlb >> nib) & 15) | (((qhb >> hshift) & 3) << 4)
                s_lo = (d * sc[:, 8 * nh + 2 * jj]).astype(np.float32)
                s_hi = (d * sc[:, 8 * nh + 2 * jj + 1]).astype(np.float32)
                qf = q.astype(np.float32) - np.float32(32.0)
                base = 128 * nh + 32 * jj
                out[:, base: base + 16] = s_lo[:, None] * qf[:, :16]
                out[:, base + 16: base + 32] = s_hi[:, None] * qf[:, 16:]
        return out.reshape(-1)
    if kind == Q8_0:
        blk = raw.reshape(-1, 34)
        d = _f16(blk[:, 0].astype(np.uint16) | (blk[:, 1].astype(np.uint16) << 8))
        q = blk[:, 2:].view(np.int8).astype(np.float32)
        return (d[:, None] * q).astype(np.float32).reshape(-1)
    if kind == Q5_0:
        blk = raw.reshape(-1, 22)
        d = _f16(blk[:, 0].astype(np.uint16) | (blk[:, 1].astype(np.uint16) << 8))
        qh = blk[:, 2:6].copy().view("<u4")[:, 0]
        qs = blk[:, 6:22]
        out = np.empty((blk.shape[0], 32), np.float32)
        for j in range(32):  # gemm.rs:352-363
            byte = j % 16
            nib = (j // 16) * 4
            qv = ((qs[:, byte].astype(np.uint32) >> nib) & 15) | (((qh >> j) & 1) << 4)
            out[:, j] = d * (qv.astype(np.float32) - np.float32(16.0))
        return out.reshape(-1)
    raise OracleError("unsupported tensor type")


# ---------------------------------------------------------------------------------------------
# Expert grouping and grouped products
# ---------------------------------------------------------------------------------------------

def group_routes(ids, experts: int, bm: int):
    """Restates the reference's `group` kernel (crates/jevons-gemma4-diffusion/src/gpu/ops.rs:523-585)
    on the CPU: thread e counts the ids equal to e (:545-552), thread 0 prefix-sums the counts and
    the bm-row tile counts (:554-567), offsets[e] = start (:569-572), the ids of expert e go to
    consecutive positions in ascending assignment order (:573-579), and expert e's jobs are
    (e, start + t * bm) at job_starts[e] + t (:580-584). Ids >= experts belong to no expert.
    Returns (sorted [assignments] u32 -- positions past offsets[experts] stay 0 --,
    offsets [experts + 1] u32, jobs [1 + 2 * njobs] u32)."""
    ids = np.asarray(ids, dtype=np.int64).reshape(-1)
    counts = np.array([int(np.count_nonzero(ids == e)) for e in range(experts)], dtype=np.int64)
    starts = np.zeros(experts + 1, dtype=np.int64)
    starts[1:] = np.cumsum(counts)
    tiles = (counts + bm - 1) // bm
    job_starts = np.zeros(experts + 1, dtype=np.int64)
    job_starts[1:] = np.cumsum(tiles)
    sorted_ = np.zeros(ids.size, dtype=np.uint32)
    jobs = np.zeros(1 + 2 * int(job_starts[experts]), dtype=np.uint32)
    jobs[0] = job_starts[experts]
    for e in range(experts):
        members = np.nonzero(ids == e)[0]
        sorted_[starts[e]:starts[e] + members.size] = members
        for t in range(int(tiles[e])):
            j = int(job_starts[e]) + t
            jobs[1 + 2 * j] = e
            jobs[2 + 2 * j] = starts[e] + t * bm
    return sorted_, starts.astype(np.uint32), jobs


def matmul_grouped_f64(x: np.ndarray, w_dense: np.ndarray, n: int, ids, in_div: int) -> np.ndarray:
    """The grouped product's definition (gemm.rs:9-11, the expected values of the reference test
    crates/jevons-gemma4-diffusion/src/gpu/tests.rs:381-390): output row a = x[a // in_div] . W_e^T
    with e = ids[a] and W_e = rows [e * n, (e + 1) * n) of the dequantized matrix; f64 sums."""
    ids = np.asarray(ids, dtype=np.int64).reshape(-1)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros((ids.size, n), dtype=np.float64)
    for e in np.unique(ids):
        rows = np.nonzero(ids == e)[0]
        out[rows] = matmul_f64(x[rows // in_div], w_dense[e * n:(e + 1) * n])
    return out


# ---- Q6_K embedding-table ("head") operators ----------------------------------------------------
# Definitions of crates/jevons-gemma4-diffusion/src/gpu/ops.rs (embed_q6k :223-291, pick_logits
# :590-635, q6k_transpose :672-715, softcap :751-760), evaluated as the reference's own test does
# (crates/jevons-gemma4-diffusion/src/gpu/tests.rs:556-648): the table is quant::dequantize of the
# Q6_K bytes, sums and norms in f64.

def embed_rows_f32(table: np.ndarray, tokens) -> np.ndarray:
    """embed_q6k before any normalisation: `dq*s*(q-32)*sqrt(d)` in f32 (ops.rs:249-270); the
    decoded weight is exact, so this is one f32 rounding of table[token] * f32(sqrt(d))."""
    d = table.shape[1]
    return table[np.asarray(tokens, dtype=np.int64)] * np.float32(np.sqrt(np.float32(d)))


def _rms_norm_f64(x: np.ndarray, eps: float) -> np.ndarray:
    r = 1.0 / np.sqrt((x * x).sum(axis=-1, keepdims=True) / x.shape[-1] + np.float64(np.float32(eps)))
    return x * r


def embed_q6k_f64(table: np.ndarray, tokens, w_attn: np.ndarray, cond, first_canvas: int, eps: float):
    """(out, x_attn) of embed_q6k (ops.rs:223-291) in f64, as tests.rs:591-619 evaluates them:
    row = E[token] * sqrt(d); canvas rows (index >= first_canvas) add cond[index - first_canvas]
    when given and are RMS-normalised; x_attn = norm(row) * w_attn."""
    d = table.shape[1]
    rows = table[np.asarray(tokens, dtype=np.int64)].astype(np.float64) * np.sqrt(np.float64(d))
    for i in range(first_canvas, rows.shape[0]):
        if cond is not None:
            rows[i] += np.asarray(cond, np.float64).reshape(-1, d)[i - first_canvas]
        rows[i] = _rms_norm_f64(rows[i], eps)
    return rows, _rms_norm_f64(rows, eps) * np.asarray(w_attn, np.float64)


def pick_logits_f64(table: np.ndarray, x_f16: np.ndarray, pairs, cap: float) -> np.ndarray:
    """pick_logits (ops.rs:590-635) as tests.rs:636-646 evaluates it: cap * tanh(x[row].E[token] / cap)."""
    pr = np.asarray(pairs, dtype=np.int64).reshape(-1, 2)
    x64 = np.asarray(x_f16, np.float32).astype(np.float64)
    dots = np.einsum("pd,pd->p", x64[pr[:, 0]], table[pr[:, 1]].astype(np.float64))
    return np.float64(cap) * np.tanh(dots / np.float64(cap))


def q6k_transpose_f16(table: np.ndarray) -> np.ndarray:
    """q6k_transpose (ops.rs:672-715): f16 (round to nearest even) of the table, transposed to [d, rows]."""
    return np.ascontiguousarray(table.astype(np.float16).T)


def softcap_f64(x: np.ndarray, cap: float) -> np.ndarray:
    """softcap (ops.rs:751-760): cap * tanh(x / cap)."""
    return np.float64(cap) * np.tanh(np.asarray(x, np.float64) / np.float64(cap))


# ---------------------------------------------------------------------------------------------
# The Q8_0 int8 path (the build's own definition; the reference only plans it,
# docs/cubecl-int8-plan.md:48-60): per-32 activation quantization and the product of exact int32
# block dots scaled in f32. Restated in jk_oracle.c.
# ---------------------------------------------------------------------------------------------

def q8_m_pad(m: int) -> int:
    return (m + 3) // 4 * 4


def quantize_act_q8(x: np.ndarray):
    """x f32 [m, k] -> (xq int8 [m, k], xd f32 [k / 32, m_pad]) as jk_quantize_act_q8 defines them."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    mp = q8_m_pad(m)
    xq = np.empty((m, k), np.int8)
    xd = np.zeros((k // 32, mp), np.float32)
    lib().jko_quantize_act_q8(_ptr(x), m, k, _ptr(xq), _ptr(xd), mp)
    return xq, xd


def matmul_q8_int8(raw: np.ndarray, n: int, k: int, xq: np.ndarray, xd: np.ndarray, with_dots: bool = False):
    """The int8 product over raw Q8_0 rows (exact int32 block dots, f32 scaling in block order)."""
    raw = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    xd = np.ascontiguousarray(xd, dtype=np.float32)
    m = xq.shape[0]
    out = np.empty((m, n), np.float32)
    dots = np.empty((m, n, k // 32), np.int32) if with_dots else None
    lib().jko_matmul_q8_int8(_ptr(raw), n, k, _ptr(xq), _ptr(xd), m, xd.shape[1], _ptr(out),
                             _ptr(dots) if with_dots else None)
    return (out, dots) if with_dots else out
