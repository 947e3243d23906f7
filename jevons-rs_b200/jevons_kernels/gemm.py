"""Quantized-weight matrix products -- the `jevons-kernels` API over libjk.so.

Mirrors crates/jevons-kernels/src/lib.rs:17-303 (`Gpu`, `Buf`) and
crates/jevons-kernels/src/gemm.rs:817-1321 (`QMatrix`, `Plan`, `SplitScratch`, `matmul`,
`matmul_plan`, `matvec`, `matmul_tiled`, `GEMV_ROWS`) plus
crates/jevons-burn/src/kernels.rs:99-129 (`f16_linear`, `f16_linear_scaled`):

    out[r, c] = sum_k x[r, k] * W[c, k]     x: [m, k] (f16 / bf16 / f32), W: [experts * n, k], out f32 [m, n]

Device memory and streams come from PyTorch (plumbing only); every product runs in the CUDA
kernels of libjk.so, launched asynchronously on the current torch stream. Errors raise JkError
with the library's message (the reference returns Err(String) or panics).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from ._lib import Groups as _Groups
from ._lib import JkError, Plan, check, load
from .formats import Packed, TensorType, block, pack

GEMV_ROWS = 16  # gemm.rs:1019

_DTYPE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class Gpu:
    """One CUDA device (Gpu::new, lib.rs:181-191): checks it is a B200 (sm_100) and selects it."""

    def __init__(self, device: int = 0):
        check(load().jk_gpu_init(int(device)))
        self.device = int(device)
        torch.cuda.set_device(self.device)

    @staticmethod
    def new(device: int = 0) -> "Gpu":
        return Gpu(device)

    def sync(self) -> None:
        """Blocks until all queued work of the current stream has completed (lib.rs:300-302)."""
        check(load().jk_gpu_sync(_stream()))

    def torch_device(self) -> torch.device:
        return torch.device("cuda", self.device)

    def device_error(self) -> int:
        """Reads and clears the device-side error word (0 = clean)."""
        code = ctypes.c_uint32()
        check(load().jk_device_error(self.device, ctypes.byref(code)))
        return code.value

    # uploads / reads (lib.rs:198-289), in terms of torch tensors
    def upload_f32(self, data) -> "Buf":
        return Buf(torch.as_tensor(np.asarray(data, np.float32)).to(self.torch_device()))

    def upload_f16(self, data) -> "Buf":
        return Buf(torch.as_tensor(np.asarray(data, np.float32)).to(self.torch_device()).half())

    def upload_bf16(self, data) -> "Buf":
        return Buf(torch.as_tensor(np.asarray(data, np.float32)).to(self.torch_device()).bfloat16())

    def zeros(self, len_: int, dtype=torch.float32) -> "Buf":
        return Buf(torch.zeros(max(int(len_), 1), dtype=dtype, device=self.torch_device()), int(len_))

    def empty(self, len_: int, dtype=torch.float32) -> "Buf":
        return Buf(torch.empty(max(int(len_), 1), dtype=dtype, device=self.torch_device()), int(len_))

    def read_f32(self, buf: "Buf") -> np.ndarray:
        return buf.tensor[: buf.len()].float().cpu().numpy()


class Buf:
    """A device allocation with a logical element count (Buf, lib.rs:75-124): a torch tensor."""

    def __init__(self, tensor: torch.Tensor, len_: int | None = None):
        if not tensor.is_cuda:
            raise JkError(1, "Buf must live on a CUDA device")
        self.tensor = tensor.contiguous().view(-1) if not tensor.is_contiguous() else tensor.view(-1)
        self._len = self.tensor.numel() if len_ is None else int(len_)

    @staticmethod
    def from_tensor(t: torch.Tensor) -> "Buf":
        return Buf(t)

    def len(self) -> int:
        return self._len

    def is_empty(self) -> bool:
        return self._len == 0

    def with_len(self, len_: int) -> "Buf":
        return Buf(self.tensor, len_)

    def ptr(self):
        return ctypes.c_void_p(self.tensor.data_ptr())

    def dtype_code(self) -> int:
        try:
            return _DTYPE[self.tensor.dtype]
        except KeyError:
            raise JkError(1, f"unsupported activation dtype {self.tensor.dtype}") from None


class QMatrix:
    """Quantized weights [experts * n, k] resident on the device (gemm.rs:817-953)."""

    def __init__(self, handle, keepalive=None):
        self._h = ctypes.c_void_p(handle)
        self._keep = keepalive
        t, n, k, e, b = ctypes.c_int(), ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        check(load().jk_qmatrix_info(self._h, ctypes.byref(t), ctypes.byref(n), ctypes.byref(k), ctypes.byref(e),
                                     ctypes.byref(b)))
        self.kind = TensorType(t.value)
        self.n, self.k, self.experts, self._bytes = n.value, k.value, e.value, b.value

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                load().jk_qmatrix_destroy(h)
            except Exception:
                pass
            self._h = ctypes.c_void_p(0)

    @property
    def handle(self):
        return self._h

    @staticmethod
    def upload(gpu: Gpu, kind, n: int, k: int, experts: int, raw) -> "QMatrix":
        """QMatrix::upload (gemm.rs:832-854): raw GGML bytes -> device, validated and repacked."""
        arr = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray))
                                   else np.asarray(raw).view(np.uint8).reshape(-1))
        out = ctypes.c_void_p()
        check(load().jk_qmatrix_upload(gpu.device, int(kind), n, k, experts, arr.ctypes.data_as(ctypes.c_void_p),
                                       arr.size, ctypes.byref(out)))
        return QMatrix(out.value)

    @staticmethod
    def from_packed(gpu: Gpu, kind, n: int, k: int, experts: int, p: Packed) -> "QMatrix":
        """QMatrix::from_packed (gemm.rs:856-899)."""
        def ptr(a):
            return a.ctypes.data_as(ctypes.c_void_p) if a.size else None
        q, h, s = (np.ascontiguousarray(a, np.uint32) for a in (p.q, p.h, p.s))
        d = np.ascontiguousarray(p.d, np.float32)
        out = ctypes.c_void_p()
        check(load().jk_qmatrix_from_packed(gpu.device, int(kind), n, k, experts, ptr(q), q.size, ptr(h), h.size,
                                            ptr(s), s.size, ptr(d), d.size, ctypes.byref(out)))
        return QMatrix(out.value)

    @staticmethod
    def f16_view(gpu: Gpu, n: int, k: int, weights: torch.Tensor) -> "QMatrix":
        """QMatrix::f16_view (gemm.rs:906-929): row-major FP16 weights [n, k], not copied."""
        if weights.dtype != torch.float16 or not weights.is_cuda or not weights.is_contiguous():
            raise JkError(1, "f16_view needs a contiguous FP16 CUDA tensor")
        if weights.numel() != n * k:
            raise JkError(3, f"F16 [{n}, {k}] has an unsupported shape")
        out = ctypes.c_void_p()
        check(load().jk_qmatrix_f16_view(gpu.device, n, k, ctypes.c_void_p(weights.data_ptr()), ctypes.byref(out)))
        return QMatrix(out.value, keepalive=weights)

    def bytes(self) -> int:
        """Device bytes held (QMatrix::bytes, gemm.rs:950-952)."""
        return self._bytes

    def dequantize(self, out: Buf | None = None) -> torch.Tensor:
        """Device dequantization to f32 [experts * n, k] (bit-exact with quant::dequantize)."""
        total = self.experts * self.n * self.k
        if out is None:
            dev = torch.device("cuda", torch.cuda.current_device())
            t = torch.empty(total, dtype=torch.float32, device=dev)
        else:
            t = out.tensor
            if t.dtype != torch.float32:
                raise JkError(1, "dequantize output must be f32")
        check(load().jk_qmatrix_dequantize(self._h, ctypes.c_void_p(t.data_ptr()), total if out is None else out.len(),
                                           _stream()))
        return t[:total].view(self.experts * self.n, self.k)


class SplitScratch:
    """Device scratch for split-K partial sums, grown on demand (gemm.rs:1040-1065)."""

    def __init__(self, gpu: Gpu | None = None):
        dev = gpu.device if gpu is not None else torch.cuda.current_device()
        h = ctypes.c_void_p()
        check(load().jk_split_scratch_create(dev, ctypes.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                load().jk_split_scratch_destroy(h)
            except Exception:
                pass
            self._h = ctypes.c_void_p(0)

    @property
    def handle(self):
        return self._h


def tile_n(n: int) -> int:
    """Weight-row tile of the tensor-core kernel (the reference's default column tile, gemm.rs:968-971)."""
    return 128


def _plan_heuristic(w: QMatrix, m: int, row_invariant: bool, groups_target: int = 0) -> Plan:
    p = Plan()
    check(load().jk_plan_heuristic(w.handle, m, 1 if row_invariant else 0, int(groups_target), ctypes.byref(p)))
    return p


def _plan_valid_for(self: Plan, w: QMatrix, m: int) -> bool:
    return bool(load().jk_plan_valid_for(ctypes.byref(self), w.handle, m))


Plan.heuristic = staticmethod(_plan_heuristic)
Plan.valid_for = _plan_valid_for
Plan.ROW_TILES = (32, 64, 96, 128, 256)
Plan.COL_TILES = (128, 256)  # 256: a CTA pair per tile (block-quantized weights, bm >= 128)


def _args(x: Buf, out: Buf):
    return x.ptr(), x.dtype_code(), x.len(), out.ptr(), out.len()


def matmul_plan(gpu: Gpu, x: Buf, m: int, w: QMatrix, out: Buf, dummy=None, scratch: SplitScratch | None = None,
                plan: Plan | None = None) -> None:
    """matmul_plan (gemm.rs:1092-1119). `dummy` is accepted for signature parity and unused."""
    xp, xt, xl, op, ol = _args(x, out)
    check(load().jk_matmul_plan(w.handle, xp, xt, xl, m, op, ol, scratch.handle if scratch else None, plan,
                                _stream()))


def matmul(gpu: Gpu, x: Buf, m: int, w: QMatrix, out: Buf, dummy=None, scratch: SplitScratch | None = None) -> None:
    """matmul (gemm.rs:1069-1088): the heuristic plan for this device."""
    xp, xt, xl, op, ol = _args(x, out)
    check(load().jk_matmul(w.handle, xp, xt, xl, m, op, ol, scratch.handle if scratch else None, _stream()))


def matmul_tiled(gpu: Gpu, x: Buf, m: int, w: QMatrix, out: Buf, dummy=None, bm: int = 128, bn: int = 128) -> None:
    """matmul_tiled (gemm.rs:1121-1133)."""
    xp, xt, xl, op, ol = _args(x, out)
    check(load().jk_matmul_tiled(w.handle, xp, xt, xl, m, op, ol, bm, bn, _stream()))


def set_max_ctas(gpu: Gpu, max_sms: int) -> None:
    """Caps the SMs the products on gpu's device may occupy (0 = all). A multi-GPU caller leaves
    SMs free for its communication kernels with this (jk_set_max_ctas)."""
    check(load().jk_set_max_ctas(gpu.device, int(max_sms)))


def get_max_ctas(gpu: Gpu) -> tuple[int, int]:
    """(cap, SM count) of gpu's device; cap 0 = no cap."""
    cap, total = ctypes.c_int(), ctypes.c_int()
    check(load().jk_get_max_ctas(gpu.device, ctypes.byref(cap), ctypes.byref(total)))
    return cap.value, total.value


def matvec(gpu: Gpu, x: Buf, m: int, w: QMatrix, out: Buf, dummy=None) -> None:
    """matvec (gemm.rs:1135-1168): m <= GEMV_ROWS."""
    xp, xt, xl, op, ol = _args(x, out)
    check(load().jk_matvec(w.handle, xp, xt, xl, m, op, ol, _stream()))


def matmul_splitk_noalloc(gpu: Gpu, x: Buf, m: int, w: QMatrix, out: Buf, bm: int = 256) -> None:
    """Split-K (stream-K) product whose scratch is a fixed buffer inside the library, for callers
    that cannot allocate device memory while the product runs (no cudaMalloc / cudaFree is made).
    bf16 or f16 activations; calls on one device must not overlap on the GPU (they share the buffer)."""
    xp, xt, xl, op, ol = _args(x, out)
    check(load().jk_matmul_splitk_noalloc(w.handle, xp, xt, xl, m, op, ol, int(bm), _stream()))


def q8_scales_len(m: int, k: int) -> int:
    """Length of the block-major activation scales jk_quantize_act_q8 writes: k / 32 rows of m
    rounded up to a multiple of 4."""
    return k // 32 * ((m + 3) // 4 * 4)


def quantize_act_q8(gpu: Gpu, x: Buf, m: int, k: int, xq: Buf, xd: Buf) -> None:
    """Per-32 activation quantization for the Q8_0 int8 path (jk_quantize_act_q8): xq int8 [m, k],
    xd f32 [k / 32, m_pad] block-major scales."""
    if xq.tensor.dtype != torch.int8 or xd.tensor.dtype != torch.float32:
        raise JkError(1, "quantize_act_q8 writes int8 quants and f32 scales")
    check(load().jk_quantize_act_q8(x.ptr(), x.dtype_code(), int(m), int(k), xq.ptr(), xq.len(), xd.ptr(), xd.len(),
                                    _stream()))


def matmul_q8_int8(gpu: Gpu, w: QMatrix, xq: Buf, xd: Buf, m: int, out: Buf) -> None:
    """The Q8_0 product on int8 tensor cores (jk_matmul_q8_int8): exact int32 block dots, scaled
    in f32 in block order."""
    check(load().jk_matmul_q8_int8(w.handle, xq.ptr(), xq.len(), xd.ptr(), xd.len(), int(m), out.ptr(), out.len(),
                                   _stream()))


class Groups:
    """Expert grouping on the device (gemm.rs:955-966): `ids` = sorted assignment indices,
    `offsets` [experts + 1], `jobs` [1 + 2 * max_jobs]; input row = id // in_div; `rows` output
    rows (assignments)."""

    def __init__(self, ids: Buf, offsets: Buf, jobs: Buf, max_jobs: int, in_div: int, rows: int):
        self.ids, self.offsets, self.jobs = ids, offsets, jobs
        self.max_jobs, self.in_div, self.rows = int(max_jobs), int(in_div), int(rows)

    def _c(self) -> _Groups:
        for b in (self.ids, self.offsets, self.jobs):
            if b.tensor.dtype not in (torch.int32, torch.uint32) or b.tensor.device.type != "cuda":
                raise JkError(1, "groups buffers must be 32-bit integer device buffers")
        if self.jobs.len() < 1 + 2 * self.max_jobs or self.ids.len() < self.rows:
            raise JkError(1, "groups buffers shorter than max_jobs / rows")
        return _Groups(self.ids.ptr(), self.offsets.ptr(), self.jobs.ptr(), self.max_jobs, self.in_div, self.rows)


def group_max_jobs(assignments: int, experts: int, bm: int) -> int:
    """Job-count bound jk_group_experts needs room for: ceil(a / bm) + min(experts, a)."""
    return int(load().jk_group_max_jobs(assignments, experts, bm))


def group_routes(gpu: Gpu, ids: Buf, sorted_: Buf, offsets: Buf, jobs: Buf, assignments: int, experts: int,
                 bm: int) -> None:
    """ops::group_routes (crates/jevons-gemma4-diffusion/src/gpu/ops.rs:1100-1128): deterministic
    grouping of `assignments` expert ids into sorted ids, offsets and jobs of `bm`-row tiles."""
    for b in (ids, sorted_, offsets, jobs):
        if b.tensor.dtype not in (torch.int32, torch.uint32):
            raise JkError(1, "grouping buffers must be 32-bit integers")
    if ids.len() < assignments or sorted_.len() < assignments or offsets.len() < experts + 1:
        raise JkError(1, "grouping buffers too short")
    check(load().jk_group_experts(gpu.device, ids.ptr(), assignments, experts, int(bm), sorted_.ptr(), offsets.ptr(),
                                  jobs.ptr(), jobs.len(), _stream()))


def matmul_grouped(gpu: Gpu, x: Buf, w: QMatrix, g: Groups, out: Buf, bm: int, bn: int = 128, splits: int = 1,
                   scratch: SplitScratch | None = None) -> None:
    """matmul_grouped (gemm.rs:1271-1321): each assignment row times its expert's weights on the
    tensor cores; the jobs must have been built with tiles of `bm` rows. A scratch is required
    (the sorted activation rows are gathered into it); one is created if none is given."""
    if scratch is None:
        scratch = SplitScratch(gpu)
    gc = g._c()
    check(load().jk_matmul_grouped(w.handle, x.ptr(), x.dtype_code(), x.len(), ctypes.byref(gc), out.ptr(),
                                   out.len(), int(bm), int(bn), int(splits), scratch.handle, _stream()))


def matvec_grouped(gpu: Gpu, x: Buf, w: QMatrix, g: Groups, out: Buf, mr: int) -> None:
    """matvec_grouped (gemm.rs:1170-1200): the grouped product on the small-row kernel, jobs of
    `mr` <= GEMV_ROWS rows."""
    gc = g._c()
    check(load().jk_matvec_grouped(w.handle, x.ptr(), x.dtype_code(), x.len(), ctypes.byref(gc), out.ptr(),
                                   out.len(), int(mr), _stream()))


def f16_linear(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """jevons_burn::kernels::f16_linear (kernels.rs:107-114): f32 x @ weight^T with FP16 weight [N, K].

    x is cast to FP16 first, so its magnitudes must stay within the FP16 range."""
    if weight.dtype != torch.float16:
        raise JkError(1, "f16 matmul needs FP16 operands")
    x16 = x.to(torch.float16).contiguous()
    w = weight.contiguous()
    m, k = x16.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise JkError(1, "f16 matmul needs dense row-major [M, K] x [N, K]")
    out = torch.empty(m, n, dtype=torch.float32, device=x16.device)
    check(load().jk_f16_linear(ctypes.c_void_p(x16.data_ptr()), m, k, ctypes.c_void_p(w.data_ptr()), n,
                               ctypes.c_void_p(out.data_ptr()), _stream()))
    return out


F16_ROW_LIMIT = 16384.0  # kernels.rs:105
_SCALED_SCRATCH: dict = {}


def f16_linear_scaled(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """kernels.rs:116-129 (jk_f16_linear_scaled): rows with max |x| > 16384 are divided down by
    max / 16384 before the FP16 cast and their outputs multiplied back; other rows use exactly 1."""
    if weight.dtype != torch.float16:
        raise JkError(1, "f16 matmul needs FP16 operands")
    x32 = x.float().contiguous()
    w = weight.contiguous()
    m, k = x32.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise JkError(1, "f16 matmul needs dense row-major [M, K] x [N, K]")
    dev = x32.device.index if x32.device.index is not None else torch.cuda.current_device()
    if dev not in _SCALED_SCRATCH:
        _SCALED_SCRATCH[dev] = SplitScratch(Gpu(dev))
    out = torch.empty(m, n, dtype=torch.float32, device=x32.device)
    check(load().jk_f16_linear_scaled(ctypes.c_void_p(x32.data_ptr()), m, k, ctypes.c_void_p(w.data_ptr()), n,
                                      ctypes.c_void_p(out.data_ptr()), _SCALED_SCRATCH[dev].handle, _stream()))
    return out


__all__ = ["GEMV_ROWS", "Gpu", "Buf", "QMatrix", "Plan", "SplitScratch", "matmul", "matmul_plan", "matmul_tiled",
           "matvec", "matmul_splitk_noalloc", "q8_scales_len", "quantize_act_q8", "matmul_q8_int8", "Groups", "group_max_jobs", "group_routes", "matmul_grouped",
           "matvec_grouped", "f16_linear", "f16_linear_scaled", "tile_n", "TensorType", "block", "pack", "JkError"]
