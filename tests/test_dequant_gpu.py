"""GPU: device dequantization is bit-exact with the oracle (quant.rs:83-101) for every type,
through both upload paths, for dense and multi-expert matrices."""
import numpy as np
import pytest

from helpers import KINDS
from oracle import oracle
from jevons_kernels import formats, synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", list(KINDS))
@pytest.mark.parametrize("n,k,experts", [(64, 256, 1), (192, 1024, 1), (128, 512, 3)])
def test_device_dequant_is_bit_exact(gpu, name, n, k, experts):
    from jevons_kernels.gemm import QMatrix
    kind = KINDS[name]
    raw = synth.weights(kind, np.random.default_rng(n + k + experts), experts * n, k)
    w = QMatrix.upload(gpu, kind, n, k, experts, raw)
    got = w.dequantize().cpu().numpy().reshape(-1)
    want = oracle.dequantize(kind, raw)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert gpu.device_error() == 0


def assert_bits_equal(got, want):
    """Bit-exact, except that any NaN equals any NaN: GPU arithmetic returns the canonical NaN
    (0x7FFFFFFF) where x86 propagates the input's payload; both are NaN in the reference's terms."""
    g, w = got.view(np.uint32), want.view(np.uint32)
    nan_w, nan_g = np.isnan(want), np.isnan(got)
    assert np.array_equal(nan_w, nan_g), f"NaN positions differ at {np.flatnonzero(nan_w != nan_g)[:8]}"
    bad = np.flatnonzero((g != w) & ~nan_w)
    assert bad.size == 0, f"{bad.size} values differ, first at {bad[:4]}: got {got[bad[:4]]} want {want[bad[:4]]}"


@pytest.mark.parametrize("name", list(KINDS))
def test_device_dequant_bit_exact_on_arbitrary_bytes(gpu, name):
    """Any block bytes (NaN/inf/subnormal scales included) decode exactly like the reference."""
    from jevons_kernels.gemm import QMatrix
    kind = KINDS[name]
    n, k = 64, 512
    size = oracle.block(kind)[1]
    per = oracle.block(kind)[0]
    raw = np.random.default_rng(5).integers(0, 256, size=n * k // per * size, dtype=np.uint8)
    w = QMatrix.upload(gpu, kind, n, k, 1, raw)
    got = w.dequantize().cpu().numpy().reshape(-1)
    want = oracle.dequantize(kind, raw)
    assert np.isnan(want).any()  # the case exercises NaN scales
    assert_bits_equal(got, want)


@pytest.mark.parametrize("name", list(KINDS))
def test_from_packed_equals_upload(gpu, name):
    from jevons_kernels.gemm import QMatrix
    kind = KINDS[name]
    n, k = 128, 512
    raw = synth.weights(kind, np.random.default_rng(9), n, k)
    a = QMatrix.upload(gpu, kind, n, k, 1, raw)
    b = QMatrix.from_packed(gpu, kind, n, k, 1, formats.pack(kind, raw))
    assert a.bytes() == b.bytes() == len(raw)
    assert np.array_equal(a.dequantize().cpu().numpy(), b.dequantize().cpu().numpy())


def test_full_size_q4k_dequant_checksum(gpu):
    """Config 4's vocab-head matrix (N=262144, K=2560): device decode == oracle decode, compared as
    a checksum of per-row checksums (both exact)."""
    from jevons_kernels.gemm import QMatrix
    n, k = 262144, 2560
    raw = synth.q4k_blocks(np.random.default_rng(4), n, k)
    w = QMatrix.upload(gpu, oracle.Q4_K, n, k, 1, raw)
    got = w.dequantize()
    bits = got.view(dtype=__import__("torch").int32).to(__import__("torch").int64)
    dev_sum = int((bits.sum(dim=1) * (1 + __import__("torch").arange(n, device=bits.device))).sum().item())
    want = oracle.dequantize(oracle.Q4_K, raw).reshape(n, k).view(np.int32).astype(np.int64)
    host_sum = int((want.sum(axis=1) * (1 + np.arange(n, dtype=np.int64))).sum())
    assert dev_sum == host_sum
