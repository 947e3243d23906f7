"""GPU: the tcgen05 tensor-core product (matmul_plan / matmul / matmul_tiled, gemm.rs:1067-1257)
against the f64 oracle, every valid plan, bitwise row invariance, edge shapes and the BASELINE
configurations. Mirrors crates/jevons-gemma4-diffusion/src/gpu/tests.rs:427-480."""
import numpy as np
import pytest
import torch

from helpers import KINDS, activations, assert_close, make_weights
from oracle import oracle
from jevons_kernels import synth

pytestmark = pytest.mark.gpu

M_CASES = [3, 16, 70, 150, 300]


def all_plans(w, m):
    from jevons_kernels.gemm import Plan
    plans = [Plan(0, 128, 1)]
    for bm in Plan.ROW_TILES:
        for bn in Plan.COL_TILES:
            for splits in (1, 2, 8):
                plans.append(Plan(bm, bn, splits))
    return [p for p in plans if p.valid_for(w, m)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("name,k", [("Q8_0", 512), ("Q4_K", 512), ("Q6_K", 512), ("Q5_0", 512)])
def test_every_plan_matches_oracle_and_tiles_are_row_invariant(gpu, name, k, dtype):
    from jevons_kernels.gemm import Buf, SplitScratch, matmul_plan
    n = 256
    w, raw, dense = make_weights(gpu, KINDS[name], n, k, seed=11)
    scratch = SplitScratch(gpu)
    for m in M_CASES:
        x, x_exact = activations(m, k, dtype, seed=m)
        want = oracle.matmul_f64(x_exact, dense)
        reference = None
        for plan in all_plans(w, m):
            out = torch.full((m, n), float("nan"), device="cuda")
            matmul_plan(gpu, Buf(x), m, w, Buf(out), None, scratch, plan)
            got = out.cpu().numpy()
            assert_close(f"{name} m={m} {plan} {dtype}", got, x_exact, dense, want, ref_rule=dtype == torch.float16)
            if plan.bm > 0 and plan.splits == 1:
                # Tile shape must not change any row's accumulation order (tests.rs:470-477).
                if reference is None:
                    reference = got
                else:
                    assert np.array_equal(reference.view(np.uint32), got.view(np.uint32)), f"{name} m={m} {plan}"
    assert gpu.device_error() == 0


@pytest.mark.parametrize("name", ["Q4_K", "Q8_0"])
def test_rows_are_invariant_across_m(gpu, name):
    """Row-invariant plans give every row the same bits whatever m is (prefix reuse, gemm.rs:1090)."""
    from jevons_kernels.gemm import Buf, Plan, matmul_plan
    n, k = 384, 1024
    w, _, _ = make_weights(gpu, KINDS[name], n, k, seed=2)
    x, _ = activations(300, k, torch.bfloat16, seed=4)
    full = torch.empty(300, n, device="cuda")
    matmul_plan(gpu, Buf(x), 300, w, Buf(full), None, None, Plan(256, 128, 1))
    for m in (1, 5, 33, 129):
        part = torch.empty(m, n, device="cuda")
        matmul_plan(gpu, Buf(x[:m].contiguous()), m, w, Buf(part), None, None, Plan(64, 128, 1))
        assert torch.equal(part, full[:m]), m


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("name", ["Q4_K", "Q6_K", "Q8_0"])
def test_activation_dtypes(gpu, name, dtype):
    from jevons_kernels.gemm import Buf, Plan, SplitScratch, matmul_plan
    n, k, m = 256, 512, 96
    w, _, dense = make_weights(gpu, KINDS[name], n, k, seed=5)
    x, x_exact = activations(m, k, dtype, seed=6)
    if dtype == torch.float32:
        x_exact = synth.bf16_round(x_exact)  # f32 activations are rounded to bf16 for the MMA
    out = torch.empty(m, n, device="cuda")
    matmul_plan(gpu, Buf(x), m, w, Buf(out), None, SplitScratch(gpu), Plan(128, 128, 2))
    assert_close(f"{name} {dtype}", out.cpu().numpy(), x_exact, dense)


@pytest.mark.parametrize("name,n,k", [("Q8_0", 64, 64), ("Q8_0", 192, 320), ("Q4_K", 64, 256), ("Q6_K", 320, 768),
                                      ("Q5_0", 64, 128), ("Q4_K", 192, 2560)])
@pytest.mark.parametrize("m", [1, 31, 33, 257])
def test_ragged_shapes(gpu, name, n, k, m):
    """Partial weight tiles (n % 128 != 0), partial row tiles, partial super-block stages."""
    from jevons_kernels.gemm import Buf, Plan, matmul_plan
    w, _, dense = make_weights(gpu, KINDS[name], n, k, seed=n + k)
    x, x_exact = activations(m, k, torch.bfloat16, seed=m)
    for bm in (32, 256):
        # one spare row after the output must stay untouched
        out = torch.full((m + 1, n), float("nan"), device="cuda")
        matmul_plan(gpu, Buf(x), m, w, Buf(out), None, None, Plan(bm, 128, 1))
        assert_close(f"{name} {n}x{k} m={m} bm={bm}", out[:m].cpu().numpy(), x_exact, dense)
        assert torch.isnan(out[m]).all()


def test_multi_expert_matrix_dense_product_uses_expert_zero(gpu):
    from jevons_kernels.gemm import Buf, Plan, matmul_plan
    n, k, e, m = 128, 512, 3, 40
    w, _, dense = make_weights(gpu, KINDS["Q4_K"], n, k, experts=e, seed=8)
    x, x_exact = activations(m, k, torch.bfloat16, seed=9)
    out = torch.empty(m, n, device="cuda")
    matmul_plan(gpu, Buf(x), m, w, Buf(out), None, None, Plan(64, 128, 1))
    assert_close("expert 0", out.cpu().numpy(), x_exact, dense[:n])


def test_heuristic_plans_and_matmul(gpu):
    from jevons_kernels.gemm import Buf, Plan, SplitScratch, matmul
    w, _, dense = make_weights(gpu, KINDS["Q4_K"], 10240, 2560, seed=1)
    # row tiles stop at 128 for block-quantized weights (tensor-memory weight stages); the cost
    # model picks the tile that fills the waves best: m=256 on 148 SMs -> 96-row tiles (240 tiles,
    # 2 waves of the faster 96-row main loop beat 160 tiles of 128 rows)
    for m, want in ((1, 0), (2, 0), (32, 32), (100, 128), (192, 64), (256, 96), (512, 128)):
        p = Plan.heuristic(w, m, False, 148)
        assert (p.bm, p.splits) == (want, 1) and p.valid_for(w, m), (m, p)
        assert Plan.heuristic(w, m, True).splits == 1 and Plan.heuristic(w, m, True).bm > 0
    # with 400 SMs, 64-row tiles (320) fit in one wave
    p400 = Plan.heuristic(w, 256, False, 400)
    assert (p400.bm, p400.splits) == (64, 1)
    # few long tiles (N=2560, K=10240: 40 tiles of 160 k-blocks): K is split (stream-K)
    w_long, _, _ = make_weights(gpu, KINDS["Q4_K"], 2560, 10240, seed=3)
    assert Plan.heuristic(w_long, 256, False, 148).splits > 1
    x, x_exact = activations(32, 2560, torch.bfloat16, seed=1)
    out = torch.empty(32, 10240, device="cuda")
    matmul(gpu, Buf(x), 32, w, Buf(out), None, SplitScratch(gpu))
    assert_close("cfg1 heuristic", out.cpu().numpy(), x_exact, dense)


def test_plan_validation(gpu):
    from jevons_kernels.gemm import Buf, JkError, Plan, matmul_plan
    w, _, _ = make_weights(gpu, KINDS["Q8_0"], 128, 256)
    assert not Plan(48, 128, 1).valid_for(w, 4)
    assert not Plan(64, 64, 1).valid_for(w, 4)
    assert not Plan(64, 128, 8).valid_for(w, 4)  # k/64 = 4 < 8 splits
    assert not Plan(0, 128, 1).valid_for(w, 17)
    assert Plan(128, 256, 1).valid_for(w, 4) and not Plan(64, 256, 1).valid_for(w, 4)  # pair tiles: bm >= 128
    x = torch.zeros(4, 256, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(JkError, match="not valid"):
        matmul_plan(gpu, Buf(x), 4, w, Buf(torch.zeros(4, 128, device="cuda")), None, None, Plan(48, 128, 1))
    with pytest.raises(JkError, match="scratch"):
        matmul_plan(gpu, Buf(x), 4, w, Buf(torch.zeros(4, 128, device="cuda")), None, None, Plan(64, 128, 2))


# --- FP16 weights: the Burn-facing f16_linear (crates/jevons-burn/src/kernels.rs:131-309) ---------

@pytest.mark.parametrize("m,n,k", [(32, 64, 256), (32, 4160, 512), (64, 256, 1024), (512, 384, 512),
                                   (32, 6144, 4096), (128, 4096, 4096), (32, 131136, 4096)])
def test_f16_linear_matches_f32_matmul(gpu, m, n, k):
    from jevons_kernels.gemm import f16_linear
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n)
    x = (torch.rand(m, k, device="cuda", generator=g) * 2 - 1).half()
    w = ((torch.rand(n, k, device="cuda", generator=g) * 2 - 1) * 0.1).half()
    want = x.float() @ w.float().t()
    got = f16_linear(x, w)
    worst = (want - got).abs().max().item()
    scale = want.abs().max().item()
    assert worst <= 2e-3 * max(scale, 1.0), (m, n, k, worst)


def test_f16_outputs_beyond_the_fp16_range_stay_exact(gpu):
    from jevons_kernels.gemm import f16_linear
    m, n, k = 128, 256, 4096
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.rand(m, k, device="cuda", generator=g) * 2 + 29
    w = (torch.rand(n, k, device="cuda", generator=g) * 0.2 + 0.9).half()
    want = x.half().float() @ w.float().t()
    got = f16_linear(x, w)
    worst = (want - got).abs().max().item()
    assert worst <= want[0, 0].abs().item() * 1e-3


def test_f16_linear_scaled_handles_huge_rows(gpu):
    """jk_f16_linear_scaled (kernels.rs:116-129): a row far beyond the FP16 range is scaled down and
    back; rows within it give exactly the f16_linear product of the FP16-cast row."""
    from jevons_kernels.gemm import f16_linear, f16_linear_scaled
    m, n, k = 32, 128, 256
    x = torch.randn(m, k, device="cuda")
    x[3] *= 1e6
    x[7] *= 3e4  # just above the 16384 limit
    w = (torch.randn(n, k, device="cuda") * 0.05).half()
    want = x.double() @ w.double().t()
    got = f16_linear_scaled(x, w)
    rel = ((want - got.double()).abs().max(dim=1).values / want.abs().max(dim=1).values).max().item()
    assert rel < 2e-3
    plain = [r for r in range(m) if r not in (3, 7)]
    ref = f16_linear(x[plain].contiguous(), w)
    assert torch.equal(got[plain], ref)


# --- BASELINE configurations -------------------------------------------------------------------

def test_config1_q4k_m32(gpu):
    """Q4_K M=32, K=2560 -> N=10240, bf16 activations, full size vs oracle."""
    from jevons_kernels.gemm import Buf, Plan, matmul_plan
    w, _, dense = make_weights(gpu, KINDS["Q4_K"], 10240, 2560, seed=1)
    x, x_exact = activations(32, 2560, torch.bfloat16, seed=1)
    out = torch.empty(32, 10240, device="cuda")
    matmul_plan(gpu, Buf(x), 32, w, Buf(out), None, None, Plan(32, 128, 1))
    assert_close("cfg1", out.cpu().numpy(), x_exact, dense)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_bench_headline_q4k_m256_full_size(gpu, dtype):
    """The bench's timed workload exactly (Q4_K M=256, K=2560 -> N=10240, the bench's seeds) through
    the public entry points: the whole-tile plan {128, 128, 1}, the CTA-pair plan {256, 256, 1} and
    the heuristic plan, every output element against the f64 oracle."""
    from jevons_kernels.gemm import Buf, Plan, QMatrix, SplitScratch, matmul, matmul_plan
    n, k, m = 10240, 2560, 256
    raw = synth.q4k_blocks(np.random.default_rng(1), n, k)
    w = QMatrix.upload(gpu, oracle.Q4_K, n, k, 1, raw)
    dense = oracle.dequantize(oracle.Q4_K, raw).reshape(n, k)
    x = torch.from_numpy(synth.activations(np.random.default_rng(2), m, k)).cuda().to(dtype)
    x_exact = x.float().cpu().numpy()
    want = oracle.matmul_f64(x_exact, dense)
    scratch = SplitScratch(gpu)
    for plan in (Plan(128, 128, 1), Plan(256, 256, 1), Plan.heuristic(w, m, False), None):
        out = torch.full((m, n), float("nan"), device="cuda")
        if plan is None:
            matmul(gpu, Buf(x), m, w, Buf(out), None, scratch)
        else:
            matmul_plan(gpu, Buf(x), m, w, Buf(out), None, scratch, plan)
        assert_close(f"bench headline {plan} {dtype}", out.cpu().numpy(), x_exact, dense, want,
                     ref_rule=dtype == torch.float16)
    assert gpu.device_error() == 0


# FastConformer (Parakeet) encoder linears, Q8_0 weights, M=750 frames of f32
# activations ~N(0, 1): FFN 1024 -> 4096 -> 1024 and four 1024 -> 1024 attention projections
# (crates/jevons-parakeet/src/config.rs:183-186, encoder.rs:53-61).
CONFIG3_SHAPES = [("ffn_up", 4096, 1024), ("ffn_down", 1024, 4096), ("attn_qkvo", 1024, 1024)]


@pytest.mark.parametrize("name,n,k", CONFIG3_SHAPES)
def test_config3_parakeet_q8_0_m750(gpu, name, n, k):
    """Config 3 through jk_matmul (f32 activations are rounded to bf16 for the tensor cores, so the
    oracle product uses the bf16-rounded rows) against the f64 oracle."""
    from jevons_kernels.gemm import Buf, SplitScratch, matmul
    m = 750
    w, _, dense = make_weights(gpu, KINDS["Q8_0"], n, k, seed=300 + n + k)
    x, x_exact = activations(m, k, torch.float32, seed=3)
    x_exact = synth.bf16_round(x_exact)
    out = torch.full((m, n), float("nan"), device="cuda")
    matmul(gpu, Buf(x), m, w, Buf(out), None, SplitScratch(gpu))
    assert_close(f"cfg3 {name}", out.cpu().numpy(), x_exact, dense)
    assert gpu.device_error() == 0


def test_config2_q6k_m256(gpu):
    """Q6_K M=256, K=10240 -> N=2560, bf16 activations ~N(0, 0.5)."""
    from jevons_kernels.gemm import Buf, Plan, SplitScratch, matmul_plan
    w, _, dense = make_weights(gpu, KINDS["Q6_K"], 2560, 10240, seed=2)
    x, x_exact = activations(256, 10240, torch.bfloat16, seed=2, sigma=0.5)
    out = torch.empty(256, 2560, device="cuda")
    for plan in (Plan(256, 128, 1), Plan.heuristic(w, 256, False)):
        matmul_plan(gpu, Buf(x), 256, w, Buf(out), None, SplitScratch(gpu), plan)
        assert_close(f"cfg2 {plan}", out.cpu().numpy(), x_exact, dense)


def test_config4_vocab_head_sampled_and_linear(gpu):
    """Q4_K vocab head M=2048, K=2560 -> N=262144: a sampled block of outputs
    against the oracle, and linearity out(a + b) == out(a) + out(b) within tolerance."""
    from jevons_kernels.gemm import Buf, Plan, matmul_plan
    n, k, m = 262144, 2560, 2048
    rng = np.random.default_rng(4)
    raw = synth.q4k_blocks(rng, n, k)
    from jevons_kernels.gemm import QMatrix
    w = QMatrix.upload(gpu, oracle.Q4_K, n, k, 1, raw)
    x, x_exact = activations(m, k, torch.bfloat16, seed=4)
    out = torch.empty(m, n, device="cuda")
    matmul_plan(gpu, Buf(x), m, w, Buf(out), None, None, Plan(256, 128, 1))
    cols = np.sort(rng.choice(n, 300, replace=False))
    rows = np.sort(rng.choice(m, 40, replace=False))
    dense_cols = oracle.dequantize(oracle.Q4_K, raw.reshape(n, -1)[cols]).reshape(len(cols), k)
    got = out[torch.from_numpy(rows).cuda()][:, torch.from_numpy(cols).cuda()].cpu().numpy()
    assert_close("cfg4 sample", got, x_exact[rows], dense_cols)
    # linearity on exact-in-bf16 halves: a = x, b = x (so a + b = 2x exactly) -> out(2x) == 2 out(x)
    out2 = torch.empty_like(out)
    matmul_plan(gpu, Buf((x * 2).contiguous()), m, w, Buf(out2), None, None, Plan(256, 128, 1))
    assert torch.equal(out2, out * 2)


@pytest.mark.parametrize("name,n,k", [("Q4_K", 192, 2560), ("Q8_0", 192, 320), ("Q4_K", 128, 10240), ("Q6_K", 64, 2560)])
@pytest.mark.parametrize("m", [31, 257])
@pytest.mark.parametrize("bn", [128, 256])
def test_stream_k_fixup_shapes(gpu, name, n, k, m, bn):
    """Stream-K fix-up: partial weight tiles (n % 128 != 0), partial row tiles, tiles split over
    many CTAs (k = 10240 on one weight tile), and output rows that are not 16-byte aligned (the
    per-element store path). A spare element after the output must stay untouched."""
    from jevons_kernels.gemm import Buf, Plan, SplitScratch, matmul_plan
    w, _, dense = make_weights(gpu, KINDS[name], n, k, seed=n + k + m)
    x, x_exact = activations(m, k, torch.bfloat16, seed=m + 1)
    want = oracle.matmul_f64(x_exact, dense)
    scratch = SplitScratch(gpu)
    for bm in (32, 256) if bn == 128 else (128, 256):
        for splits in (2, 4):
            assert Plan(bm, bn, splits).valid_for(w, m)
            for shift in (0, 1):
                big = torch.full((m * n + 2,), float("nan"), device="cuda")
                out = big[shift:shift + m * n].view(m, n)
                matmul_plan(gpu, Buf(x), m, w, Buf(out), None, scratch,
                            Plan(bm, bn, splits))
                assert_close(f"{name} {n}x{k} m={m} bm={bm} s={splits} shift={shift}", out.cpu().numpy(), x_exact,
                             dense, want)
                assert torch.isnan(big[shift + m * n]).item()
                if shift:
                    assert torch.isnan(big[0]).item()
    assert gpu.device_error() == 0


@pytest.mark.parametrize("name", ["Q4_K", "Q6_K", "Q8_0", "Q5_0"])
def test_long_k_wraps_every_stage_ring(gpu, name):
    """k = 10240 (160 k-blocks) wraps the weight-stage rings many times for every row tile, with
    whole tiles and with stream-K: the tensor-memory stage rings of 32..128-row tiles hold only
    2 or 3 stages, so any phase-tracking slip between the dequantizer groups shows up here."""
    from jevons_kernels.gemm import Buf, Plan, SplitScratch, matmul_plan
    n, k, m = 256, 10240, 200
    w, _, dense = make_weights(gpu, KINDS[name], n, k, seed=31)
    x, x_exact = activations(m, k, torch.bfloat16, seed=32, sigma=0.5)
    want = oracle.matmul_f64(x_exact, dense)
    scratch = SplitScratch(gpu)
    for bm in (32, 64, 128, 256):
        for splits in (1, 2):
            out = torch.full((m, n), float("nan"), device="cuda")
            matmul_plan(gpu, Buf(x), m, w, Buf(out), None, scratch, Plan(bm, 128, splits))
            assert_close(f"{name} k={k} bm={bm} s={splits}", out.cpu().numpy(), x_exact, dense, want)
    assert gpu.device_error() == 0


def test_sm_cap_keeps_products_correct(gpu):
    """jk_set_max_ctas: products launched under a cap (stream-K, whole tiles, small-row kernel)
    stay within tolerance; the cap is per device and 0 lifts it."""
    from jevons_kernels.gemm import Buf, Plan, SplitScratch, get_max_ctas, matmul_plan, matvec, set_max_ctas
    w, _, dense = make_weights(gpu, KINDS["Q4_K"], 2560, 2560, seed=3)
    scratch = SplitScratch(gpu)
    try:
        for cap in (37, 132, 0):
            set_max_ctas(gpu, cap)
            assert get_max_ctas(gpu)[0] == cap
            for m, plan in ((256, Plan(256, 128, 2)), (96, Plan(128, 128, 1))):
                x, x_exact = activations(m, 2560, torch.bfloat16, seed=m + cap)
                out = torch.full((m, 2560), float("nan"), device="cuda")
                matmul_plan(gpu, Buf(x), m, w, Buf(out), None, scratch, plan)
                assert_close(f"cap {cap} m={m} {plan}", out.cpu().numpy(), x_exact, dense)
            x, x_exact = activations(1, 2560, torch.bfloat16, seed=cap)
            out = torch.full((1, 2560), float("nan"), device="cuda")
            matvec(gpu, Buf(x), 1, w, Buf(out))
            assert_close(f"cap {cap} gemv", out.cpu().numpy(), x_exact, dense)
    finally:
        set_max_ctas(gpu, 0)
    assert gpu.device_error() == 0
