"""GPU: the Q6_K embedding-table operators against the oracle.

Follows the reference's own test of these kernels
(crates/jevons-gemma4-diffusion/src/gpu/tests.rs:556-648,
`q6k_embedding_rows_and_candidate_logits_match_dequantized_table`): the table is
quant::dequantize of the Q6_K bytes, the expected values are f64 sums, and errors are normalised
by the largest expected magnitude (tests.rs:37-47) with the reference's tolerances -- 1e-5 for
the f32 embedding rows, 2e-3 for the f16 attention input, 1e-4 for candidate logits. Decoded
values are exact, so the embedding rows before any normalisation and the transposed f16 table
are compared bit for bit. The table is a Q6_K QMatrix, as the model's embedding is
(model.rs:174-184), so its rows are a multiple of 64; the reference test's 40-row table becomes a
64-row one with the same tokens, pairs, d, eps and cap.
"""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


def q6k_table(rng, rows, d):
    """Q6_K bytes with the reference test's value ranges (tests.rs:546-554): random ql/qh bytes,
    scales in (-100, 100), d in [0.001, 0.011)."""
    nb = rows * d // 256
    raw = np.empty((nb, 210), np.uint8)
    raw[:, :192] = rng.integers(0, 256, size=(nb, 192), dtype=np.uint8)
    raw[:, 192:208] = rng.integers(-99, 100, size=(nb, 16)).astype(np.int8).view(np.uint8)
    raw[:, 208:210] = (0.001 + rng.random(nb) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return raw.reshape(-1)


def normalized_error(got, want):
    scale = max(1e-6, float(np.abs(want).max()))
    return float(np.abs(np.asarray(got, np.float64) - want).max()) / scale


def table_of(gpu, rng, vocab, d):
    from jevons_kernels.gemm import QMatrix
    raw = q6k_table(rng, vocab, d)
    return QMatrix.upload(gpu, oracle.Q6_K, vocab, d, 1, raw), oracle.dequantize(oracle.Q6_K, raw).reshape(vocab, d)


def i32(gpu, values):
    from jevons_kernels.gemm import Buf
    return Buf(torch.tensor(np.asarray(values, np.int64).astype(np.int32), device=gpu.torch_device()))


def run_embed(gpu, table, tokens, w, cond, first_canvas, d, eps):
    from jevons_kernels import head
    rows = len(tokens)
    out, xn = gpu.zeros(rows * d), gpu.zeros(rows * d, torch.float16)
    head.embed(gpu, i32(gpu, tokens), table, gpu.upload_f32(w), None if cond is None else gpu.upload_f32(cond),
               out, xn, rows, first_canvas, d, eps)
    torch.cuda.synchronize()
    return gpu.read_f32(out).reshape(rows, d), gpu.read_f32(xn).reshape(rows, d)


@pytest.mark.parametrize("vocab,d,tokens,first_canvas,with_cond", [
    (64, 512, [3, 39, 0, 17], 2, False),          # the reference test's case (on a 64-row table)
    (64, 2560, [5, 63, 0, 1, 7, 7], 1, True),     # the bench model dimension, self-conditioning rows
    (64, 8448, [9, 2, 60], 1, True),              # d / 8 > 1024: two octets per thread
    (64, 256, [1, 2, 3], 0, False),               # every row a canvas row
    (64, 1024, [1, 2, 3], 5, False),              # no canvas rows
])
def test_embed_rows_match_dequantized_table(gpu, vocab, d, tokens, first_canvas, with_cond):
    rng = np.random.default_rng(vocab + d)
    eps = 1e-6
    table, dense = table_of(gpu, rng, vocab, d)
    w = rng.uniform(-1.0, 1.0, d).astype(np.float32)
    canvas = max(len(tokens) - first_canvas, 0)
    cond = rng.uniform(-1.0, 1.0, canvas * d).astype(np.float32) if with_cond else None
    out, xn = run_embed(gpu, table, tokens, w, cond, first_canvas, d, eps)
    want, want_x = oracle.embed_q6k_f64(dense, tokens, w, cond, first_canvas, eps)
    assert normalized_error(out, want) <= 1e-5
    assert normalized_error(xn, want_x) <= 2e-3
    plain = min(first_canvas, len(tokens))
    exact = oracle.embed_rows_f32(dense, tokens[:plain])
    assert np.array_equal(out[:plain].view(np.uint32), exact.view(np.uint32)), "pre-norm rows are not bit-exact"
    assert gpu.device_error() == 0


def test_embed_of_zero_rows_is_a_no_op(gpu):
    from jevons_kernels import head
    rng = np.random.default_rng(3)
    table, _ = table_of(gpu, rng, 64, 512)
    out, xn = gpu.zeros(0), gpu.zeros(0, torch.float16)
    head.embed(gpu, i32(gpu, [0]).with_len(0), table, gpu.upload_f32(np.ones(512)), None, out, xn, 0, 0, 512, 1e-6)
    torch.cuda.synchronize()
    assert gpu.device_error() == 0


def test_embed_flags_token_outside_table_and_keeps_other_rows(gpu):
    rng = np.random.default_rng(4)
    vocab, d, eps = 64, 512, 1e-6
    table, dense = table_of(gpu, rng, vocab, d)
    w = rng.uniform(-1.0, 1.0, d).astype(np.float32)
    tokens = [3, vocab + 5, 7]
    out, xn = run_embed(gpu, table, tokens, w, None, 3, d, eps)
    assert gpu.device_error() == 2
    want, want_x = oracle.embed_q6k_f64(dense, [3, 7], w, None, 2, eps)
    assert normalized_error(out[[0, 2]], want) <= 1e-5
    assert normalized_error(xn[[0, 2]], want_x) <= 2e-3
    assert np.all(out[1] == 0.0)


def run_pick(gpu, table, x16, pairs, cap, d):
    from jevons_kernels import head
    from jevons_kernels.gemm import Buf
    count = len(pairs) // 2
    logits = gpu.zeros(count)
    head.pick(gpu, Buf(torch.from_numpy(x16).to(gpu.torch_device())), i32(gpu, pairs), count, table, logits, cap, d)
    torch.cuda.synchronize()
    return gpu.read_f32(logits)


def test_pick_logits_reference_case(gpu):
    rng = np.random.default_rng(5)
    vocab, d, cap = 64, 512, 30.0
    table, dense = table_of(gpu, rng, vocab, d)
    x16 = rng.uniform(-1.0, 1.0, 2 * d).astype(np.float16).reshape(2, d)
    pairs = [0, 5, 1, 39, 1, 0]
    got = run_pick(gpu, table, x16, pairs, cap, d)
    assert normalized_error(got, oracle.pick_logits_f64(dense, x16, pairs, cap)) <= 1e-4
    assert gpu.device_error() == 0


@pytest.mark.parametrize("vocab,d,rows,count,cap", [(1024, 2560, 16, 1000, 30.0), (128, 256, 3, 13, 5.0),
                                                    (64, 8448, 2, 9, 30.0)])
def test_pick_logits_many_pairs(gpu, vocab, d, rows, count, cap):
    rng = np.random.default_rng(vocab + count)
    table, dense = table_of(gpu, rng, vocab, d)
    x16 = rng.uniform(-1.0, 1.0, rows * d).astype(np.float16).reshape(rows, d)
    pairs = np.stack([rng.integers(0, rows, count), rng.integers(0, vocab, count)], axis=1).reshape(-1)
    got = run_pick(gpu, table, x16, pairs, cap, d)
    assert normalized_error(got, oracle.pick_logits_f64(dense, x16, pairs, cap)) <= 1e-4
    assert gpu.device_error() == 0


def test_pick_logits_flags_pairs_outside_x_or_table(gpu):
    rng = np.random.default_rng(6)
    vocab, d, cap = 64, 512, 30.0
    table, dense = table_of(gpu, rng, vocab, d)
    x16 = rng.uniform(-1.0, 1.0, 2 * d).astype(np.float16).reshape(2, d)
    pairs = [0, 1, 2, 1, 1, vocab, 1, 3]
    got = run_pick(gpu, table, x16, pairs, cap, d)
    assert gpu.device_error() == 2
    assert np.isnan(got[1]) and np.isnan(got[2])
    want = oracle.pick_logits_f64(dense, x16, [0, 1, 1, 3], cap)
    assert normalized_error(got[[0, 3]], want) <= 1e-4


@pytest.mark.parametrize("vocab,d", [(64, 256), (128, 512), (4096, 2560), (192, 8448)])
def test_q6k_transpose_is_bit_exact(gpu, vocab, d):
    from jevons_kernels import head
    rng = np.random.default_rng(vocab * 7 + d)
    table, dense = table_of(gpu, rng, vocab, d)
    got = head.q6k_transposed_f16(gpu, table, vocab, d).tensor[: vocab * d].cpu().numpy().reshape(d, vocab)
    want = oracle.q6k_transpose_f16(dense)
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))
    assert gpu.device_error() == 0


def test_q6k_transpose_rejects_a_table_of_another_type(gpu):
    from jevons_kernels import head, synth
    from jevons_kernels._lib import JkError
    from jevons_kernels.gemm import QMatrix
    w = QMatrix.upload(gpu, oracle.Q4_K, 64, 256, 1, synth.q4k_blocks(np.random.default_rng(0), 64, 256))
    with pytest.raises(JkError, match="Q6_K"):
        head.q6k_transposed_f16(gpu, w, 64, 256)


@pytest.mark.parametrize("n", [1, 3, 4, 1003, 1 << 20])
def test_softcap_in_place(gpu, n):
    from jevons_kernels import head
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 40.0).astype(np.float32)
    buf = gpu.upload_f32(x)
    head.softcap_logits(gpu, buf, n, 30.0)
    torch.cuda.synchronize()
    assert normalized_error(gpu.read_f32(buf), oracle.softcap_f64(x, 30.0)) <= 1e-6


def test_full_vocabulary_head_is_matmul_then_softcap(gpu):
    """model.rs:1192-1205: logits = softcap(x . E^T) over the whole table with the matmul path."""
    from jevons_kernels import head
    from jevons_kernels.gemm import Buf, SplitScratch, matmul
    rng = np.random.default_rng(8)
    vocab, d, rows, cap = 2048, 2560, 5, 30.0
    table, dense = table_of(gpu, rng, vocab, d)
    x16 = rng.uniform(-1.0, 1.0, rows * d).astype(np.float16).reshape(rows, d)
    out = gpu.zeros(rows * vocab)
    matmul(gpu, Buf(torch.from_numpy(x16).to(gpu.torch_device())), rows, table, out, scratch=SplitScratch(gpu))
    head.softcap_logits(gpu, out, rows * vocab, cap)
    torch.cuda.synchronize()
    # The product rounds decoded weights to the activation type (f16) for the tensor cores, so the
    # product path's bound applies: |err| <= 1e-3 |x_r| |w_c| before capping, and capping
    # (cap * tanh(v / cap), slope <= 1) keeps it.
    xe = x16.astype(np.float32)
    want = oracle.softcap_f64(oracle.matmul_f64(xe, dense), cap)
    bound = 1e-3 * np.outer(oracle.row_norms(xe), oracle.row_norms(dense))
    assert np.all(np.abs(gpu.read_f32(out).reshape(rows, vocab) - want) <= bound)
    assert gpu.device_error() == 0
