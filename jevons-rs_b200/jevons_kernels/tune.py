"""Measured launch plans for the dense and grouped products -- the reference's Tuner over libjk.so.

Mirrors crates/jevons-gemma4-diffusion/src/gpu/tune.rs: `bucket` (:74-76), `pick` (:548-562),
`Tuner.new` / `dense` / `grouped` / `tune_dense` / `tune_grouped` / `save` (:139-192, 231-346,
412-446). Candidate plans are timed on the device with CUDA events; row-invariant requests only
consider plans without split-K, so tuning never changes a result a caller relies on being exact.
"""
from __future__ import annotations

import ctypes

from ._lib import Plan, check, load
from .gemm import Buf, Gpu, QMatrix, SplitScratch, _stream


def bucket(m: int) -> int:
    """Row-count bucket: plans measured at m = bucket serve every m in (bucket/2, bucket]."""
    return int(load().jk_tune_bucket(int(m)))


def pick(times, plans, baseline: Plan) -> Plan | None:
    """The fastest plan unless it beats the heuristic baseline by less than 5%."""
    if not plans:
        return None
    n = len(plans)
    t = (ctypes.c_double * n)(*times)
    p = (Plan * n)(*plans)
    out = Plan()
    check(load().jk_tune_pick(t, p, n, baseline, ctypes.byref(out)))
    return out


class Tuner:
    """Plan table for one device, optionally stored in `path` (Tuner::new, tune.rs:139-155)."""

    def __init__(self, gpu: Gpu, path: str | None = None, load_stored: bool = True):
        h = ctypes.c_void_p()
        check(load().jk_tuner_create(gpu.device, path.encode() if path else None, int(load_stored), ctypes.byref(h)))
        self._h = h
        self.gpu = gpu

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                load().jk_tuner_destroy(h)
            except Exception:
                pass
            self._h = ctypes.c_void_p(0)

    def __len__(self) -> int:
        return int(load().jk_tuner_size(self._h))

    def dense(self, w: QMatrix, m: int, row_invariant: bool) -> Plan:
        """The stored plan for w's shape and bucket(m), else Plan::heuristic (tune.rs:162-175)."""
        out = Plan()
        check(load().jk_tuner_plan(self._h, w.handle, int(m), int(bool(row_invariant)), ctypes.byref(out)))
        return out

    def tune_dense(self, ws: list[QMatrix], m: int, row_invariant: bool, x: Buf, out: Buf,
                   scratch: SplitScratch | None = None) -> Plan:
        """Times the candidates over `ws` (same shape) at bucket(m) rows and stores the pick."""
        arr = (ctypes.c_void_p * len(ws))(*[w.handle.value for w in ws])
        chosen = Plan()
        check(load().jk_tuner_tune(self._h, arr, len(ws), int(m), int(bool(row_invariant)), x.ptr(), x.dtype_code(),
                                   x.len(), out.ptr(), out.len(), scratch.handle if scratch else None, _stream(),
                                   ctypes.byref(chosen)))
        return chosen

    def grouped(self, w: QMatrix, rows: int) -> Plan:
        """The grouped tile {bm, bn, 1} for w and bucket(rows), else {32, 128} (tune.rs:177-192)."""
        out = Plan()
        check(load().jk_tuner_group_plan(self._h, w.handle, int(rows), ctypes.byref(out)))
        return out

    def tune_grouped(self, ws: list[QMatrix], m: int, top_k: int, x: Buf, out: Buf,
                     scratch: SplitScratch | None = None, ids: Buf | None = None) -> Plan:
        """Times the grouped tiles for m tokens routed top_k ways (tune.rs:271-346). Without `ids`
        the reference's synthetic balanced routing is used: route i goes to expert
        ((i // top_k) * 7 + (i % top_k) * 13) % experts."""
        import torch
        experts = ws[0].experts
        a = bucket(m) * top_k
        dev = x.tensor.device
        if ids is None:
            i = torch.arange(a, device=dev, dtype=torch.int64)
            ids = Buf((((i // top_k) * 7 + (i % top_k) * 13) % experts).to(torch.int32))
        mj = int(load().jk_group_max_jobs(a, experts, 32))
        sorted_ = torch.empty(max(a, 1), dtype=torch.int32, device=dev)
        offsets = torch.empty(experts + 1, dtype=torch.int32, device=dev)
        jobs = torch.empty(1 + 2 * mj, dtype=torch.int32, device=dev)
        arr = (ctypes.c_void_p * len(ws))(*[w.handle.value for w in ws])
        chosen = Plan()
        check(load().jk_tuner_tune_grouped(self._h, arr, len(ws), int(m), int(top_k), ids.ptr(), ids.len(), x.ptr(),
                                           x.dtype_code(), x.len(), out.ptr(), out.len(),
                                           ctypes.c_void_p(sorted_.data_ptr()), ctypes.c_void_p(offsets.data_ptr()),
                                           ctypes.c_void_p(jobs.data_ptr()), jobs.numel(),
                                           scratch.handle if scratch else None, _stream(), ctypes.byref(chosen)))
        return chosen

    def save(self) -> None:
        check(load().jk_tuner_save(self._h))
