"""Measured launch plans for the dense products -- the reference's Tuner over libjk.so.

Mirrors crates/jevons-gemma4-diffusion/src/gpu/tune.rs: `bucket` (:74-76), `pick` (:548-562),
`Tuner.new` / `dense` / `tune_dense` / `save` (:139-175, 231-269, 412-446). Candidate plans are
timed on the device with CUDA events; row-invariant requests only consider plans without
split-K, so tuning never changes a result a caller relies on being exact.
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

    def save(self) -> None:
        check(load().jk_tuner_save(self._h))
