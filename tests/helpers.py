"""Helpers shared by the GPU parity tests: seeded weights through the product API, the f64
oracle product, and the output tolerance.

Tolerance (stated once, used everywhere): for every output element
    |got[r, c] - want[r, c]| <= TOL * |x_r| * |w_c|      with TOL = 1e-3,
where want is the f64 product over the oracle's dequantized weights and the activations already
rounded to the dtype the kernel reads, |x_r| and |w_c| are Euclidean norms of the activation
row and the dequantized weight row (the tolerance BASELINE.json's north star states for bf16/f32
accumulation).

For FP16 activations -- the reference's own configuration, where both the reference and this
build round dequantized weights to FP16 -- the reference's GPU-test rule must hold as well:
    max |got - want| <= 2e-3 * max(|want|, 1e-6)        (crates/jevons-gemma4-diffusion/src/gpu/tests.rs:37-47)
With bf16 activations the weights are rounded to bf16 (8 significant bits instead of FP16's 11),
so only the per-element bound applies there. For Q4_K with bf16 activations the tensor-core
operand is computed in packed bf16 arithmetic, q * bf16(d*sc) - bf16(dmin*m) with one rounding,
whose per-weight error is at most 2^-8 * (q*|d*sc| + |dmin*m|) (not 2^-9 * |w|); the per-element
bound above covers it with a wide margin, as the full-size tests of the bench workload show.
"""
import numpy as np

from oracle import oracle
from jevons_kernels import synth

TOL = 1e-3
REF_TOL = 2e-3
KINDS = {"Q4_K": oracle.Q4_K, "Q6_K": oracle.Q6_K, "Q8_0": oracle.Q8_0, "Q5_0": oracle.Q5_0}


def make_weights(gpu, kind, n, k, experts=1, seed=0):
    from jevons_kernels.gemm import QMatrix
    rng = np.random.default_rng(seed)
    raw = synth.weights(kind, rng, experts * n, k)
    w = QMatrix.upload(gpu, kind, n, k, experts, raw)
    dense = oracle.dequantize(kind, raw).reshape(experts * n, k)
    return w, raw, dense


def activations(m, k, dtype, seed=1, sigma=1.0):
    """Returns (torch tensor on cuda of `dtype`, f32 numpy array of the exact values it holds)."""
    import torch
    rng = np.random.default_rng(seed)
    x = synth.activations(rng, m, k, sigma)
    t = torch.from_numpy(x).cuda().to(dtype)
    return t, t.float().cpu().numpy()


def assert_close(name, got, x_exact, dense, want=None, ref_rule=False):
    """got: [m, n] f32 numpy; x_exact: [m, k] f32 values the kernel read; dense: [n, k] f32.
    ref_rule: also apply the reference's normalized 2e-3 rule (FP16 operands)."""
    if want is None:
        want = oracle.matmul_f64(x_exact, dense)
    err = np.abs(got.astype(np.float64) - want)
    bound = TOL * np.outer(oracle.row_norms(x_exact), oracle.row_norms(dense))
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert np.all(err <= bound), (
        f"{name}: |err| {err[worst]:.3e} > {bound[worst]:.3e} at {worst} (got {got[worst]}, want {want[worst]})")
    if ref_rule:
        scale = max(np.abs(want).max(), 1e-6)
        assert err.max() / scale <= REF_TOL, f"{name}: normalized error {err.max() / scale:.2e}"
    return want
