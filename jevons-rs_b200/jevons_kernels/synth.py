"""Seeded synthetic GGML weights and activations with the benchmark configurations' shapes.

No model checkpoints are available, so weights are drawn from the distributions each benchmark
configuration names, then encoded into GGML block bytes (the inverse of the decode in
crates/jevons-formats/src/quant.rs). Generator: numpy PCG64 (`np.random.default_rng(seed)`).

    Q8_0  d = f16(|N(0, 0.02)| / 127), q ~ U{-127..127}                  (config 0, 3)
    Q4_K  d, dmin = f16(|N(0, 0.01)|), 6-bit scales/mins ~ U{0..63}, q ~ U{0..15}  (config 1, 4)
    Q6_K  d = f16(|N(0, 0.002)|), int8 sub-scales ~ U{-64..63}, q ~ U{0..63}     (config 2)
    Q5_0  d = f16(|N(0, 0.02)| / 16), q ~ U{0..31}
Activations: f32 N(0, sigma), optionally rounded to bf16 / f16.
"""
from __future__ import annotations

import numpy as np

Q8_0, Q4_K, Q6_K, Q5_0 = 8, 12, 14, 6


def _f16_bits(a: np.ndarray) -> np.ndarray:
    return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)


def q8_0_blocks(rng: np.random.Generator, rows: int, k: int, d_sigma: float = 0.02) -> np.ndarray:
    nb = rows * k // 32
    d = _f16_bits(np.abs(rng.normal(0.0, d_sigma, nb)) / 127.0)
    q = rng.integers(-127, 128, size=(nb, 32), dtype=np.int16).astype(np.int8)
    out = np.empty((nb, 34), np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def q4k_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Packs 8 six-bit scales and mins per block into the 12 scale bytes (inverse of
    q4k_scale_min, quant.rs:14-23)."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.empty((sc.shape[0], 12), np.uint8)
    out[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    return out


def q4k_blocks(rng: np.random.Generator, rows: int, k: int, d_sigma: float = 0.01) -> np.ndarray:
    nb = rows * k // 256
    out = np.empty((nb, 144), np.uint8)
    out[:, 0:2] = _f16_bits(np.abs(rng.normal(0.0, d_sigma, nb))).view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = _f16_bits(np.abs(rng.normal(0.0, d_sigma, nb))).view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = q4k_scales(rng.integers(0, 64, (nb, 8)), rng.integers(0, 64, (nb, 8)))
    q = rng.integers(0, 16, size=(nb, 4, 2, 32), dtype=np.uint8)  # [pair][lo/hi][l]
    out[:, 16:] = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(nb, 128)
    return out.reshape(-1)


def q6k_blocks(rng: np.random.Generator, rows: int, k: int, d_sigma: float = 0.002) -> np.ndarray:
    nb = rows * k // 256
    q = rng.integers(0, 64, size=(nb, 2, 4, 32), dtype=np.uint8)  # [nh][i][l]
    out = np.empty((nb, 210), np.uint8)
    ql = np.empty((nb, 2, 2, 32), np.uint8)
    ql[:, :, 0, :] = (q[:, :, 0, :] & 15) | ((q[:, :, 2, :] & 15) << 4)
    ql[:, :, 1, :] = (q[:, :, 1, :] & 15) | ((q[:, :, 3, :] & 15) << 4)
    qh = (q[:, :, 0, :] >> 4) | ((q[:, :, 1, :] >> 4) << 2) | ((q[:, :, 2, :] >> 4) << 4) | ((q[:, :, 3, :] >> 4) << 6)
    out[:, 0:128] = ql.reshape(nb, 128)
    out[:, 128:192] = qh.reshape(nb, 64)
    out[:, 192:208] = rng.integers(-64, 64, size=(nb, 16), dtype=np.int16).astype(np.int8).view(np.uint8)
    out[:, 208:210] = _f16_bits(np.abs(rng.normal(0.0, d_sigma, nb))).view(np.uint8).reshape(nb, 2)
    return out.reshape(-1)


def q5_0_blocks(rng: np.random.Generator, rows: int, k: int, d_sigma: float = 0.02) -> np.ndarray:
    nb = rows * k // 32
    q = rng.integers(0, 32, size=(nb, 32), dtype=np.uint32)
    out = np.empty((nb, 22), np.uint8)
    out[:, 0:2] = _f16_bits(np.abs(rng.normal(0.0, d_sigma, nb)) / 16.0).view(np.uint8).reshape(nb, 2)
    qh = np.zeros(nb, np.uint32)
    for e in range(32):
        qh |= (q[:, e] >> 4) << e
    out[:, 2:6] = qh.astype("<u4").view(np.uint8).reshape(nb, 4)
    out[:, 6:22] = ((q[:, :16] & 15) | ((q[:, 16:] & 15) << 4)).astype(np.uint8)
    return out.reshape(-1)


def weights(kind: int, rng: np.random.Generator, rows: int, k: int) -> np.ndarray:
    if kind == Q8_0:
        return q8_0_blocks(rng, rows, k)
    if kind == Q4_K:
        return q4k_blocks(rng, rows, k)
    if kind == Q6_K:
        return q6k_blocks(rng, rows, k)
    if kind == Q5_0:
        return q5_0_blocks(rng, rows, k)
    raise ValueError(f"no generator for type {kind}")


def activations(rng: np.random.Generator, m: int, k: int, sigma: float = 1.0, round_to: str | None = None) -> np.ndarray:
    """f32 N(0, sigma) activations [m, k]; round_to 'bf16' / 'f16' rounds each value (kept as f32)."""
    x = rng.normal(0.0, sigma, size=(m, k)).astype(np.float32)
    if round_to == "f16":
        x = x.astype(np.float16).astype(np.float32)
    elif round_to == "bf16":
        x = bf16_round(x)
    return x


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round f32 to the nearest bf16 (ties to even), returned as f32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)
