"""GPU: the Q8_0 int8 tensor-core path (jk_quantize_act_q8 + jk_matmul_q8_int8) through the C ABI.

The reference plans this path (docs/cubecl-int8-plan.md:48-60: per-32 activation quantization,
integer block dots, block scales applied in f32) but has no implementation, so its parity is
pinned to the CPU restatement in oracle/jk_oracle.c:
  * the quantized activations and their scales are bit-exact with jko_quantize_act_q8;
  * the product is bit-exact with jko_matmul_q8_int8 (same int32 block dots, same f32 operations
    in the same block order);
  * the int32 block dots are exact: with unit scales the product is the integer sum of the dots;
  * against the f64 product over the unquantized activations, every element is within the
    activation-quantization bound  sum_b (d_x[r, b] / 2) * sum_j |w[c, 32b + j]|  (plus 1e-5 of
    the f32 sum of magnitudes for the accumulation).
Shapes include BASELINE config 3 (Parakeet encoder linears, M=750, f32 activations ~N(0, 1)).
"""
import numpy as np
import pytest
import torch

from helpers import KINDS, make_weights
from oracle import oracle
from jevons_kernels import synth

pytestmark = pytest.mark.gpu


def quantize(gpu, x, m, k):
    from jevons_kernels.gemm import Buf, q8_scales_len, quantize_act_q8
    xq = torch.empty(m * k, dtype=torch.int8, device="cuda")
    xd = torch.full((q8_scales_len(m, k),), float("nan"), device="cuda")
    quantize_act_q8(gpu, Buf(x), m, k, Buf(xq), Buf(xd))
    return xq, xd


def product(gpu, w, xq, xd, m, n):
    from jevons_kernels.gemm import Buf, matmul_q8_int8
    out = torch.full((m, n), float("nan"), device="cuda")
    matmul_q8_int8(gpu, w, Buf(xq), Buf(xd), m, Buf(out))
    return out.cpu().numpy()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,k", [(1, 64), (5, 1024), (130, 4096)])
def test_quantizer_is_bit_exact(gpu, dtype, m, k):
    rng = np.random.default_rng(m + k)
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32) * 3).cuda().to(dtype)
    x[0, :32] = 0  # an all-zero block: d = 0, q = 0
    xq, xd = quantize(gpu, x, m, k)
    want_q, want_d = oracle.quantize_act_q8(x.float().cpu().numpy())
    assert np.array_equal(xq.cpu().numpy().reshape(m, k), want_q)
    assert np.array_equal(xd.cpu().numpy().reshape(k // 32, -1).view(np.uint32), want_d.view(np.uint32))
    assert gpu.device_error() == 0


@pytest.mark.parametrize("n,k,m", [(256, 1024, 37), (320, 192, 130), (128, 4096, 256), (640, 2560, 300)])
def test_product_is_bit_exact_with_the_restatement(gpu, n, k, m):
    """Partial weight tiles (n % 128), a half stage (k % 128 == 64), partial activation tiles."""
    w, raw, _ = make_weights(gpu, KINDS["Q8_0"], n, k, seed=n + k)
    x = torch.from_numpy(np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)).cuda()
    xq, xd = quantize(gpu, x, m, k)
    got = product(gpu, w, xq, xd, m, n)
    want = oracle.matmul_q8_int8(raw, n, k, xq.cpu().numpy().reshape(m, k), xd.cpu().numpy().reshape(k // 32, -1))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), np.abs(got - want).max()
    assert gpu.device_error() == 0


def test_block_dots_are_exact_int32(gpu):
    """Unit weight and activation scales: every output is the integer sum of its block dots, exact
    in f32 (|sum| < 2^24), so any inexact int32 dot would show."""
    from jevons_kernels.gemm import QMatrix
    n, k, m = 256, 512, 130
    rng = np.random.default_rng(9)
    nb = n * k // 32
    raw = np.empty((nb, 34), np.uint8)
    raw[:, 0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    raw[:, 2:] = rng.integers(-127, 128, size=(nb, 32)).astype(np.int8).view(np.uint8)
    w = QMatrix.upload(gpu, oracle.Q8_0, n, k, 1, raw.reshape(-1))
    xi = rng.integers(-127, 128, size=(m, k)).astype(np.float32)
    xi.reshape(m, k // 32, 32)[:, :, 0] = 127  # amax = 127 in every block: d = 1, q = x
    xq, xd = quantize(gpu, torch.from_numpy(xi).cuda(), m, k)
    assert np.array_equal(xq.cpu().numpy().reshape(m, k), xi.astype(np.int8))
    got = product(gpu, w, xq, xd, m, n)
    qw = raw[:, 2:].view(np.int8).reshape(n, k).astype(np.int64)
    want = xi.astype(np.int64) @ qw.T
    assert np.array_equal(got.astype(np.int64), want) and np.all(got == np.round(got))
    assert gpu.device_error() == 0


def quantization_bound(x, dense, xd, m):
    """sum_b (d_x[r, b] / 2) * ||w[c, block b]||_1 + 1e-5 * sum_j |x_rj w_cj|."""
    n, k = dense.shape
    wabs = np.abs(dense.astype(np.float64)).reshape(n, k // 32, 32).sum(axis=2)  # [n, nblk]
    dx = xd.reshape(k // 32, -1)[:, :m].astype(np.float64)                       # [nblk, m]
    return 0.5 * dx.T @ wabs.T + 1e-5 * (np.abs(x.astype(np.float64)) @ np.abs(dense.astype(np.float64)).T)


# BASELINE config 3 (crates/jevons-parakeet/src/config.rs:183-186, encoder.rs:53-61).
@pytest.mark.parametrize("name,n,k", [("ffn_up", 4096, 1024), ("ffn_down", 1024, 4096), ("attn_qkvo", 1024, 1024)])
def test_config3_parakeet_on_int8_tensor_cores(gpu, name, n, k):
    m = 750
    w, raw, dense = make_weights(gpu, KINDS["Q8_0"], n, k, seed=300 + n + k)
    x = synth.activations(np.random.default_rng(3), m, k)
    xq, xd = quantize(gpu, torch.from_numpy(x).cuda(), m, k)
    got = product(gpu, w, xq, xd, m, n)
    xq_h, xd_h = xq.cpu().numpy().reshape(m, k), xd.cpu().numpy()
    want = oracle.matmul_q8_int8(raw, n, k, xq_h, xd_h.reshape(k // 32, -1))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"cfg3 {name}: not bit-exact"
    exact = oracle.matmul_f64(x, dense)
    err = np.abs(got.astype(np.float64) - exact)
    bound = quantization_bound(x, dense, xd_h, m)
    assert np.all(err <= bound), f"cfg3 {name}: {err.max():.3e} beyond the quantization bound"
    assert gpu.device_error() == 0


def test_int8_product_rejects_other_weights_and_small_buffers(gpu):
    from jevons_kernels.gemm import Buf, JkError, matmul_q8_int8
    w4, _, _ = make_weights(gpu, KINDS["Q4_K"], 128, 256)
    xq = torch.zeros(4 * 256, dtype=torch.int8, device="cuda")
    xd = torch.zeros(8 * 4, device="cuda")
    out = torch.zeros(4 * 128, device="cuda")
    with pytest.raises(JkError, match="Q8_0"):
        matmul_q8_int8(gpu, w4, Buf(xq), Buf(xd), 4, Buf(out))
    w8, _, _ = make_weights(gpu, KINDS["Q8_0"], 128, 256)
    with pytest.raises(JkError, match="too small"):
        matmul_q8_int8(gpu, w8, Buf(xq), Buf(xd), 5, Buf(out))
