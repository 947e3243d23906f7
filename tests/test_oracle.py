"""CPU tests: the oracle is pinned to the reference's known answers and to a second restatement,
and the product's host-side format functions agree with it. No GPU needed."""
import json
import os

import numpy as np
import pytest

from oracle import oracle
from jevons_kernels import formats, synth

HERE = os.path.dirname(os.path.abspath(__file__))
KAT = json.load(open(os.path.join(HERE, "golden", "quant_kat.json")))
TYPES = [("q4k", oracle.Q4_K, 512), ("q6k", oracle.Q6_K, 512), ("q8_0", oracle.Q8_0, 128), ("q5_0", oracle.Q5_0, 128)]


# --- known answers from crates/jevons-formats/src/quant.rs:199-237 --------------------------------

@pytest.mark.parametrize("impl", ["oracle", "product"])
def test_q4k_decodes_scale_high_bits_for_upper_groups(impl):
    case = KAT["q4k_scale_min"]
    fn = oracle.q4k_scale_min if impl == "oracle" else formats.q4k_scale_min
    for j, want in case["expect"].items():
        assert fn(int(j), bytes(case["scales"])) == tuple(want)


def test_q8_0_and_q5_0_dequantize_signed_values():
    for name in ("q8_0", "q5_0"):
        case = KAT[name]
        out = oracle.dequantize(case["type"], bytes(case["bytes"]))
        for i, want in case["expect"].items():
            assert out[int(i)] == want, (name, i, out[int(i)], want)


@pytest.mark.parametrize("impl", ["oracle", "product"])
def test_packing_splits_quants_and_scales_without_changing_values(impl):
    case = KAT["pack_q8_0"]
    raw = bytes(case["bytes"])
    if impl == "oracle":
        q, h, s, d = oracle.pack(case["type"], raw)
        with pytest.raises(oracle.OracleError):
            oracle.pack(case["type"], raw[: case["bad_len"]])
    else:
        p = formats.pack(case["type"], raw)
        q, d = p.q, p.d
        from jevons_kernels._lib import JkError
        with pytest.raises(JkError):
            formats.pack(case["type"], raw[: case["bad_len"]])
    assert len(q) == case["q_len"] and list(d) == case["d"]
    assert int(q[0]) == case["q0"]


def test_dequantize_rejects_bad_sizes_and_types():
    with pytest.raises(oracle.OracleError):
        oracle.dequantize(oracle.Q8_0, bytes(33))
    with pytest.raises(oracle.OracleError):
        oracle.dequantize(oracle.Q8_0, bytes(34), out_len=31)
    with pytest.raises(oracle.OracleError):
        oracle.dequantize(99, bytes(34))


def test_block_sizes_match_gguf():
    # TensorType::block (gguf.rs:134-145)
    want = {0: (1, 4), 1: (1, 2), 12: (256, 144), 6: (32, 22), 14: (256, 210), 8: (32, 34)}
    for t, wb in want.items():
        assert oracle.block(t) == wb
        assert formats.block(t) == wb
    assert oracle.block(2) is None and formats.block(2) is None


# --- the oracle against a second restatement (the reference's GPU word decode) --------------------

@pytest.mark.parametrize("name,kind,k", TYPES)
def test_oracle_matches_word_level_decode_bit_exact(name, kind, k):
    rng = np.random.default_rng(7)
    raw = synth.weights(kind, rng, 64, k)
    a = oracle.dequantize(kind, raw)
    b = oracle.dequantize_words(kind, raw)
    assert a.view(np.uint32).tolist() == b.view(np.uint32).tolist()


@pytest.mark.parametrize("name,kind,k", TYPES)
def test_oracle_matches_word_level_decode_on_random_bytes(name, kind, k):
    # Arbitrary bytes (any scale, NaN/inf halves included) must decode identically too.
    rng = np.random.default_rng(11)
    size = oracle.block(kind)[1]
    raw = rng.integers(0, 256, size=size * 97, dtype=np.uint8)
    a = oracle.dequantize(kind, raw)
    b = oracle.dequantize_words(kind, raw)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_oracle_regression_vectors():
    v = np.load(os.path.join(HERE, "golden", "oracle_vectors.npz"))
    for name, kind, _ in TYPES:
        got = oracle.dequantize(kind, v[f"{name}_raw"])
        assert np.array_equal(got.view(np.uint32), v[f"{name}_f32"].view(np.uint32)), name


def test_half_conversion_is_exact():
    bits = np.arange(0, 1 << 16, 97, dtype=np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle.half_to_float(int(b)) for b in bits], np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))
    assert np.all(np.isnan(got[~finite]) == np.isnan(want[~finite]))


# --- product host repacking == oracle pack ---------------------------------------------------------

@pytest.mark.parametrize("name,kind,k", TYPES)
def test_product_pack_equals_oracle_pack(name, kind, k):
    rng = np.random.default_rng(3)
    raw = synth.weights(kind, rng, 8, k)
    q, h, s, d = oracle.pack(kind, raw)
    p = formats.pack(kind, raw)
    assert np.array_equal(q, p.q) and np.array_equal(h, p.h) and np.array_equal(s, p.s)
    assert np.array_equal(d.view(np.uint32), p.d.view(np.uint32))
    assert formats.packed_words(kind) == oracle.packed_words(kind)


# --- synthetic generators --------------------------------------------------------------------------

def test_q4k_generator_ranges():
    rng = np.random.default_rng(0)
    raw = synth.q4k_blocks(rng, 4, 1024).reshape(-1, 144)
    for blk in raw[:8]:
        for j in range(8):
            sc, mn = oracle.q4k_scale_min(j, bytes(blk[4:16]))
            assert 0 <= sc < 64 and 0 <= mn < 64


def test_q4k_scale_packing_roundtrip():
    rng = np.random.default_rng(1)
    sc = rng.integers(0, 64, (50, 8))
    mn = rng.integers(0, 64, (50, 8))
    packed = synth.q4k_scales(sc, mn)
    for b in range(50):
        for j in range(8):
            assert oracle.q4k_scale_min(j, bytes(packed[b])) == (sc[b, j], mn[b, j])


def test_bf16_round_matches_torch():
    torch = pytest.importorskip("torch")
    x = np.random.default_rng(2).normal(0, 3, 4096).astype(np.float32)
    want = torch.from_numpy(x).bfloat16().float().numpy()
    assert np.array_equal(synth.bf16_round(x), want)


# ---- expert grouping (crates/jevons-gemma4-diffusion/src/gpu/ops.rs:523-585) -----------------

def test_group_oracle_known_answer():
    # ids of 5 assignments over 3 experts: counts [2, 1, 2], starts [0, 2, 3, 5]
    s, o, j = oracle.group_routes([2, 0, 2, 1, 0], 3, 1)
    assert o.tolist() == [0, 2, 3, 5]
    assert s.tolist() == [1, 4, 3, 0, 2]  # ascending assignment index within each expert
    assert j.tolist() == [5, 0, 0, 0, 1, 1, 2, 2, 3, 2, 4]
    s, o, j = oracle.group_routes([2, 0, 2, 1, 0], 3, 2)
    assert j.tolist() == [3, 0, 0, 1, 2, 2, 3]
    s, o, j = oracle.group_routes([], 4, 32)
    assert o.tolist() == [0] * 5 and j.tolist() == [0] and s.size == 0


@pytest.mark.parametrize("a,experts,bm", [(42, 4, 32), (300, 16, 8), (1000, 128, 1), (64, 1, 64)])
def test_group_oracle_reference_invariants(a, experts, bm):
    """The grouping assertions of the reference test tests.rs:338-357 hold for the oracle."""
    ids = np.random.default_rng(a).integers(0, experts, a)
    s, o, j = oracle.group_routes(ids, experts, bm)
    seen = np.zeros(a, bool)
    for e in range(experts):
        for p in range(o[e], o[e + 1]):
            assert ids[s[p]] == e and not seen[s[p]]
            seen[s[p]] = True
    assert seen.all()
    covered = 0
    for q in range(j[0]):
        e, start = j[1 + 2 * q], j[2 + 2 * q]
        assert o[e] <= start < o[e + 1]
        covered += min(o[e + 1] - start, bm)
    assert covered == a


def test_group_max_jobs_bounds_every_grouping():
    """jk_group_max_jobs (host-only, no GPU) is never below the job count of a grouping, and never
    above the reference callers' ceil(a / bm) + experts."""
    from jevons_kernels._lib import load
    rng = np.random.default_rng(5)
    for _ in range(200):
        experts = int(rng.integers(1, 300))
        a = int(rng.integers(0, 3000))
        bm = int(rng.choice([1, 2, 3, 8, 16, 32, 64, 128, 256]))
        ids = rng.integers(0, experts, a) if rng.random() < 0.5 else np.minimum(rng.geometric(0.2, a) - 1, experts - 1)
        _, _, j = oracle.group_routes(ids, experts, bm)
        bound = load().jk_group_max_jobs(a, experts, bm)
        assert j[0] <= bound <= -(-a // bm) + experts
    assert load().jk_group_max_jobs(10, 4, 0) == 0


def test_grouped_product_definition():
    """matmul_grouped_f64 is row a = x[a // in_div] . W_{ids[a]}^T, checked against a plain loop."""
    rng = np.random.default_rng(9)
    experts, n, k, tokens, top_k = 3, 5, 7, 4, 2
    w = rng.standard_normal((experts * n, k)).astype(np.float32)
    x = rng.standard_normal((tokens, k)).astype(np.float32)
    ids = rng.integers(0, experts, tokens * top_k)
    got = oracle.matmul_grouped_f64(x, w, n, ids, top_k)
    for a in range(tokens * top_k):
        e = ids[a]
        for c in range(n):
            want = sum(float(x[a // top_k, i]) * float(w[e * n + c, i]) for i in range(k))
            assert abs(got[a, c] - want) <= 1e-12 * max(1.0, abs(want))


def test_head_oracle_follows_the_reference_test_definitions():
    """The head operators' oracle (ops.rs:223-291, 590-635, 672-715 as tests.rs:556-648 checks
    them): plain rows are table rows times sqrt(d), canvas rows have unit RMS, the transposed table
    is the f16 of the dequantized table, pick is a capped dot product."""
    rng = np.random.default_rng(11)
    vocab, d, eps = 64, 512, 1e-6
    raw = synth.q6k_blocks(rng, vocab, d)
    dense = oracle.dequantize(oracle.Q6_K, raw).reshape(vocab, d)
    tokens = [3, 9, 63, 0]
    w = np.ones(d, np.float32)
    out, xn = oracle.embed_q6k_f64(dense, tokens, w, None, 2, eps)
    exact = oracle.embed_rows_f32(dense, tokens)
    assert np.allclose(out[:2], exact[:2], rtol=1e-7, atol=0)
    assert np.allclose(np.sqrt((out[2:] ** 2).mean(axis=1)), 1.0, rtol=1e-5)
    assert np.allclose(xn, out / np.sqrt((out ** 2).mean(axis=1, keepdims=True) + eps), rtol=1e-12)
    t = oracle.q6k_transpose_f16(dense)
    assert t.shape == (d, vocab) and t.dtype == np.float16 and t[5, 7] == np.float16(dense[7, 5])
    x = rng.standard_normal((2, d)).astype(np.float16)
    got = oracle.pick_logits_f64(dense, x, [1, 4, 0, 60], 30.0)
    dot = float(np.dot(x[1].astype(np.float64), dense[4].astype(np.float64)))
    assert got[0] == pytest.approx(30.0 * np.tanh(dot / 30.0), rel=1e-12)


# --- the Q8_0 int8 path's restatement (the build's definition; no reference implementation) -------

def test_q8_activation_quantizer_restatement():
    rng = np.random.default_rng(12)
    x = (rng.standard_normal((7, 96)) * 2).astype(np.float32)
    x[3, 32:64] = 0
    xq, xd = oracle.quantize_act_q8(x)
    assert xd.shape == (3, 8) and np.all(xd[:, 7] == 0)  # m_pad = 8: padding rows stay zero
    assert np.all(xd[1, 3] == 0) and np.all(xq[3, 32:64] == 0)
    d = np.repeat(xd[:, :7].T, 32, axis=1)                 # [m, k] scale of each element
    assert np.all(np.abs(xq.astype(np.float32) * d - x) <= d / 2 * (1 + 1e-6))
    assert np.abs(xq).max() == 127
    amax = np.abs(x.reshape(7, 3, 32)).max(axis=2)
    assert np.array_equal(xd[:, :7].T, (amax / np.float32(127)).astype(np.float32))


def test_q8_int8_restatement_dots_and_order():
    from jevons_kernels import synth
    rng = np.random.default_rng(13)
    n, k, m = 64, 128, 5
    raw = synth.q8_0_blocks(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    xq, xd = oracle.quantize_act_q8(x)
    out, dots = oracle.matmul_q8_int8(raw, n, k, xq, xd, with_dots=True)
    qw = raw.reshape(n * k // 32, 34)[:, 2:].view(np.int8).reshape(n, k // 32, 32).astype(np.int64)
    want_dots = np.einsum("rbj,cbj->rcb", xq.reshape(m, k // 32, 32).astype(np.int64), qw)
    assert np.array_equal(dots, want_dots)
    dw = raw.reshape(n * k // 32, 34)[:, :2].copy().view(np.float16).astype(np.float32).reshape(n, k // 32)
    acc = np.zeros((m, n), np.float32)
    for b in range(k // 32):  # fma in block order == f64 product rounded once per block
        s = (dw[None, :, b] * xd[b, :m][:, None]).astype(np.float32)
        acc = (dots[:, :, b].astype(np.float64) * s.astype(np.float64) + acc.astype(np.float64)).astype(np.float32)
    assert np.array_equal(out, acc)
