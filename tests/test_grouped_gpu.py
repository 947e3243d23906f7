"""GPU: expert grouping (jk_group_experts) and the grouped products (jk_matmul_grouped,
jk_matvec_grouped) through the C ABI, against the CPU oracle.

Follows the reference's own tests of this path:
  * crates/jevons-gemma4-diffusion/src/gpu/tests.rs:330-357 -- the grouping covers every
    assignment exactly once inside its expert's range, and the jobs cover every position once;
  * tests.rs:360-420 -- grouped products use each assignment's expert weights, for every row tile,
    column tile and split count, and with splits == 1 the tile shape changes no output bit.
The device grouping must equal the oracle's restatement of the reference kernel bit for bit
(it is integer work); products are held to the library tolerance of helpers.assert_close.
"""
import numpy as np
import pytest
import torch

from helpers import KINDS, activations, assert_close, make_weights
from oracle import oracle

pytestmark = pytest.mark.gpu


def u32(a):
    return torch.from_numpy(np.asarray(a, dtype=np.uint32).view(np.int32)).cuda()


def device_groups(gpu, ids, experts, bm, max_jobs=None):
    """Runs jk_group_experts; returns (sorted, offsets, jobs) numpy u32 and the device buffers."""
    from jevons_kernels.gemm import Buf, group_max_jobs, group_routes
    a = len(ids)
    if max_jobs is None:
        max_jobs = -(-a // bm) + experts  # the reference callers' bound (model.rs:593)
    ids_t = u32(ids) if a else torch.zeros(1, dtype=torch.int32, device="cuda")
    bufs = (torch.full((max(a, 1),), -1, dtype=torch.int32, device="cuda"),
            torch.full((experts + 1,), -1, dtype=torch.int32, device="cuda"),
            torch.full((1 + 2 * max_jobs,), -1, dtype=torch.int32, device="cuda"))
    assert group_max_jobs(a, experts, bm) <= max_jobs
    group_routes(gpu, Buf(ids_t, a), Buf(bufs[0], a), Buf(bufs[1]), Buf(bufs[2]), a, experts, bm)
    torch.cuda.synchronize()
    sorted_, offsets, jobs = (b.cpu().numpy().view(np.uint32) for b in bufs)
    return sorted_[:a], offsets, jobs, bufs, max_jobs


def check_reference_invariants(ids, experts, bm, sorted_, offsets, jobs):
    """The assertions of the reference test tests.rs:338-357."""
    a = len(ids)
    seen = np.zeros(a, bool)
    for e in range(experts):
        for s in range(offsets[e], offsets[e + 1]):
            asg = sorted_[s]
            assert ids[asg] == e
            assert not seen[asg]
            seen[asg] = True
    assert seen.all()
    covered = 0
    for j in range(jobs[0]):
        e, start = jobs[1 + 2 * j], jobs[2 + 2 * j]
        assert offsets[e] <= start < offsets[e + 1]
        covered += min(offsets[e + 1] - start, bm)
    assert covered == a


@pytest.mark.parametrize("a,experts,bm,dist", [
    (0, 4, 32, "uniform"), (1, 4, 32, "uniform"), (42, 4, 32, "uniform"), (42, 4, 1, "uniform"),
    (256, 128, 8, "uniform"), (1000, 8, 64, "skewed"), (4096, 256, 128, "uniform"), (5000, 1, 256, "one"),
    (33, 1024, 16, "uniform"), (40000, 64, 256, "skewed"), (777, 60, 3, "uniform"),
])
def test_grouping_matches_oracle_bit_for_bit(gpu, a, experts, bm, dist):
    rng = np.random.default_rng(a * 31 + experts)
    if dist == "uniform":
        ids = rng.integers(0, experts, a)
    elif dist == "skewed":
        ids = np.minimum(rng.geometric(0.3, a) - 1, experts - 1)
    else:
        ids = np.zeros(a, np.int64)
    sorted_, offsets, jobs, _, _ = device_groups(gpu, ids, experts, bm)
    ws, wo, wj = oracle.group_routes(ids, experts, bm)
    np.testing.assert_array_equal(offsets, wo)
    np.testing.assert_array_equal(sorted_, ws)
    np.testing.assert_array_equal(jobs[:wj.size], wj)
    check_reference_invariants(ids, experts, bm, sorted_, offsets, jobs)
    assert gpu.device_error() == 0


def test_grouping_reference_routes(gpu):
    """The route pattern of the reference's grouped-product test (tests.rs:375-377)."""
    tokens, top_k, experts = 21, 2, 4
    ids = np.array([(a * 7 + a // top_k) % experts for a in range(tokens * top_k)])
    for bm in (32, 64, 128, 256):
        sorted_, offsets, jobs, _, _ = device_groups(gpu, ids, experts, bm)
        ws, wo, wj = oracle.group_routes(ids, experts, bm)
        assert (sorted_ == ws).all() and (offsets == wo).all() and (jobs[:wj.size] == wj).all()
        check_reference_invariants(ids, experts, bm, sorted_, offsets, jobs)


def test_grouping_rejects_bad_arguments(gpu):
    from jevons_kernels._lib import JkError
    from jevons_kernels.gemm import Buf, group_routes
    ids = u32([0, 1, 2])
    s, o = torch.zeros(3, dtype=torch.int32, device="cuda"), torch.zeros(5, dtype=torch.int32, device="cuda")
    with pytest.raises(JkError, match="jobs buffer"):
        group_routes(gpu, Buf(ids), Buf(s), Buf(o), Buf(torch.zeros(3, dtype=torch.int32, device="cuda")), 3, 4, 1)
    big = torch.zeros(2000, dtype=torch.int32, device="cuda")
    with pytest.raises(JkError, match="1..1024 experts"):
        group_routes(gpu, Buf(ids), Buf(s), Buf(big), Buf(big), 3, 1025, 1)


def test_out_of_range_ids_are_left_out_and_reported(gpu):
    ids = np.array([0, 5, 1, 1, 9, 0])  # experts = 4: ids 5 and 9 are invalid
    sorted_, offsets, jobs, _, _ = device_groups(gpu, ids, 4, 2)
    assert offsets[4] == 4
    assert sorted(sorted_[:4].tolist()) == [0, 2, 3, 5]
    assert gpu.device_error() == 2  # ERR_BAD_LAUNCH, cleared by the read
    assert gpu.device_error() == 0


def grouped_case(gpu, kind, n, k, experts, tokens, top_k, seed, dtype=torch.float16, pattern="reference"):
    w, raw, dense = make_weights(gpu, kind, n, k, experts=experts, seed=seed)
    x, x_exact = activations(tokens, k, dtype, seed=seed + 1)
    a = tokens * top_k
    if pattern == "reference":
        ids = np.array([(i * 7 + i // top_k) % experts for i in range(a)])
    else:
        rng = np.random.default_rng(seed + 2)
        ids = np.stack([rng.permutation(experts)[:top_k] for _ in range(tokens)]).reshape(-1)
    return w, dense, x, x_exact, ids


def run_grouped(gpu, w, x, ids, experts, in_div, bm, bn=128, splits=1, scratch=None, mr=None):
    from jevons_kernels.gemm import Buf, Groups, matmul_grouped, matvec_grouped
    tile = mr if mr is not None else bm
    a = len(ids)
    _, _, _, bufs, max_jobs = device_groups(gpu, ids, experts, tile)
    g = Groups(Buf(bufs[0], a), Buf(bufs[1]), Buf(bufs[2]), max_jobs, in_div, a)
    out = torch.full((a, w.n), float("nan"), device="cuda")
    if mr is not None:
        matvec_grouped(gpu, Buf(x), w, g, Buf(out), mr)
    else:
        matmul_grouped(gpu, Buf(x), w, g, Buf(out), bm, bn, splits, scratch)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def check_grouped(name, got, x_exact, dense, n, ids, in_div, ref_rule=False):
    want = oracle.matmul_grouped_f64(x_exact, dense, n, ids, in_div)
    # per-element bound with each row's own expert rows: check expert by expert
    for e in np.unique(ids):
        rows = np.nonzero(ids == e)[0]
        assert_close(f"{name} expert {e}", got[rows], x_exact[rows // in_div], dense[e * n:(e + 1) * n],
                     want=want[rows], ref_rule=ref_rule)


@pytest.mark.parametrize("name", ["Q8_0", "Q4_K", "Q6_K", "Q5_0"])
def test_grouped_products_use_each_assignments_expert_weights(gpu, name):
    """tests.rs:360-420 with the reference's shapes: 21 tokens, top_k 2, 4 experts, n 128, k 256;
    every row tile, column tile and split count; row invariance across tiles at splits == 1."""
    from jevons_kernels.gemm import Plan, SplitScratch
    tokens, top_k, experts, n, k = 21, 2, 4, 128, 256
    w, dense, x, x_exact, ids = grouped_case(gpu, KINDS[name], n, k, experts, tokens, top_k, seed=3)
    scratch = SplitScratch(gpu)
    reference = None
    for bm in Plan.ROW_TILES:
        for bn in Plan.COL_TILES:
            if bn == 256 and bm < 128:
                continue
            for splits in (1, 2):
                got = run_grouped(gpu, w, x, ids, experts, top_k, bm, bn, splits, scratch)
                check_grouped(f"{name} grouped {bm}x{bn}/{splits}", got, x_exact, dense, n, ids, top_k,
                              ref_rule=True)
                if splits == 1:
                    if reference is None:
                        reference = got
                    else:
                        assert np.array_equal(reference, got), f"grouped {bm}x{bn}: tile shape changed the result"
    assert gpu.device_error() == 0


@pytest.mark.parametrize("name,mr", [("Q4_K", 1), ("Q6_K", 2), ("Q8_0", 4), ("Q5_0", 8), ("Q4_K", 16)])
def test_matvec_grouped_decode_routes(gpu, name, mr):
    """Decode-sized routing: a few tokens, top_k 8 of 64 experts, jobs of mr rows."""
    tokens, top_k, experts, n, k = 3, 8, 64, 256, 512
    w, dense, x, x_exact, ids = grouped_case(gpu, KINDS[name], n, k, experts, tokens, top_k, seed=mr + 10,
                                             dtype=torch.bfloat16, pattern="topk")
    got = run_grouped(gpu, w, x, ids, experts, top_k, bm=0, mr=mr)
    check_grouped(f"{name} matvec_grouped mr={mr}", got, x_exact, dense, n, ids, top_k)
    assert gpu.device_error() == 0


def test_matvec_grouped_shared_experts_rows_beyond_tile(gpu):
    """Several rows per expert (more than mr): an expert's rows span several jobs."""
    tokens, top_k, experts, n, k = 24, 2, 4, 128, 512
    w, dense, x, x_exact, ids = grouped_case(gpu, oracle.Q4_K, n, k, experts, tokens, top_k, seed=5)
    for mr in (1, 3, 8, 16):
        got = run_grouped(gpu, w, x, ids, experts, top_k, bm=0, mr=mr)
        check_grouped(f"matvec_grouped mr={mr}", got, x_exact, dense, n, ids, top_k)


def test_down_projection_in_div_1_f32_and_bf16(gpu):
    """The down projection reads one activation row per assignment (in_div = 1), here in f32 and
    bf16, through both grouped products."""
    experts, n, k, a = 8, 256, 1024, 50
    w, _, dense = make_weights(gpu, oracle.Q6_K, n, k, experts=experts, seed=77)
    rng = np.random.default_rng(78)
    ids = rng.integers(0, experts, a)
    for dtype in (torch.float32, torch.bfloat16):
        x, x_exact = activations(a, k, dtype, seed=79)
        got = run_grouped(gpu, w, x, ids, experts, 1, bm=64)
        # f32 activations are rounded to bf16 by the gather, as the dense product does
        xr = torch.from_numpy(x_exact).bfloat16().float().numpy()
        check_grouped(f"matmul_grouped {dtype}", got, xr, dense, n, ids, 1)
        got = run_grouped(gpu, w, x, ids, experts, 1, bm=0, mr=4)
        check_grouped(f"matvec_grouped {dtype}", got, x_exact, dense, n, ids, 1)


def test_grouped_f16_weights(gpu):
    """FP16 weights exist only as single-expert views (gemm.rs:908-925, experts = 1): a grouping
    with one expert runs the F16 tensor-core path; bf16 activations are refused for it."""
    from jevons_kernels.gemm import Buf, Groups, QMatrix, SplitScratch, matmul_grouped
    from jevons_kernels._lib import JkError
    n, k, tokens, top_k = 256, 512, 10, 3
    rng = np.random.default_rng(12)
    wt = torch.from_numpy((rng.standard_normal((n, k)) * 0.05).astype(np.float16)).cuda()
    w = QMatrix.f16_view(gpu, n, k, wt)
    dense = wt.float().cpu().numpy()
    x, x_exact = activations(tokens, k, torch.float16, seed=13)
    ids = np.zeros(tokens * top_k, np.int64)
    for bm in (32, 128):
        got = run_grouped(gpu, w, x, ids, 1, top_k, bm=bm)
        check_grouped(f"F16 grouped bm={bm}", got, x_exact, dense, n, ids, top_k, ref_rule=True)
    got = run_grouped(gpu, w, x, ids, 1, top_k, bm=0, mr=8)
    check_grouped("F16 matvec_grouped", got, x_exact, dense, n, ids, top_k)
    xb = x.bfloat16()
    _, _, _, bufs, mj = device_groups(gpu, ids, 1, 32)
    g = Groups(Buf(bufs[0], len(ids)), Buf(bufs[1]), Buf(bufs[2]), mj, top_k, len(ids))
    out = torch.zeros(len(ids), n, device="cuda")
    with pytest.raises(JkError, match="FP16 weights need FP16"):
        matmul_grouped(gpu, Buf(xb), w, g, Buf(out), 32, 128, 1, SplitScratch(gpu))


@pytest.mark.slow
def test_grouped_moe_layer_shapes(gpu):
    """A MoE-sized layer: 128 experts of Q4_K [704, 2816], 300 tokens x top 8 (2400 rows), bm 128
    on single CTAs and CTA pairs; then the same routes through the small-row kernel."""
    experts, n, k, tokens, top_k = 128, 704, 2816, 300, 8
    w, dense, x, x_exact, ids = grouped_case(gpu, oracle.Q4_K, n, k, experts, tokens, top_k, seed=21,
                                             dtype=torch.bfloat16, pattern="topk")
    from jevons_kernels.gemm import SplitScratch
    scratch = SplitScratch(gpu)
    a = got128 = run_grouped(gpu, w, x, ids, experts, top_k, bm=128, bn=128, scratch=scratch)
    check_grouped("moe 128x128", a, x_exact, dense, n, ids, top_k)
    got256 = run_grouped(gpu, w, x, ids, experts, top_k, bm=128, bn=256, scratch=scratch)
    assert np.array_equal(got128, got256)
    got_mv = run_grouped(gpu, w, x[:2], ids[:16], experts, top_k, bm=0, mr=1)
    check_grouped("moe matvec", got_mv, x_exact[:2], dense, n, ids[:16], top_k)
    assert gpu.device_error() == 0


def test_grouped_scratch_keeps_stream_k_flags_zero(gpu):
    """A grouped product and a stream-K dense product share one scratch: the gathered rows must not
    land on the stream-K flag words."""
    from jevons_kernels.gemm import Buf, Plan, SplitScratch, matmul_plan
    experts, n, k = 4, 256, 1024
    w, _, dense = make_weights(gpu, oracle.Q8_0, n, k, experts=experts, seed=31)
    scratch = SplitScratch(gpu)
    ids = np.arange(400) % experts
    x, x_exact = activations(200, k, torch.bfloat16, seed=32)
    got = run_grouped(gpu, w, x, ids, experts, 2, bm=128, scratch=scratch)
    check_grouped("grouped", got, x_exact, dense, n, ids, 2)
    xd, xd_exact = activations(96, k, torch.bfloat16, seed=33)
    out = torch.zeros(96, n, device="cuda")
    matmul_plan(gpu, Buf(xd), 96, w, Buf(out), scratch=scratch, plan=Plan(64, 128, 4))
    torch.cuda.synchronize()
    assert_close("stream-K after grouped", out.cpu().numpy(), xd_exact, dense[:n])
    assert gpu.device_error() == 0


def test_grouped_argument_errors(gpu):
    from jevons_kernels.gemm import Buf, Groups, SplitScratch, matmul_grouped, matvec_grouped
    from jevons_kernels._lib import JkError
    experts, n, k = 2, 128, 256
    w, _, _ = make_weights(gpu, oracle.Q8_0, n, k, experts=experts, seed=41)
    ids = np.array([0, 1, 1, 0])
    _, _, _, bufs, mj = device_groups(gpu, ids, experts, 32)
    g = Groups(Buf(bufs[0], 4), Buf(bufs[1]), Buf(bufs[2]), mj, 2, 4)
    x = torch.zeros(2, k, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(4, n, device="cuda")
    with pytest.raises(JkError, match="not valid"):
        matmul_grouped(gpu, Buf(x), w, g, Buf(out), 48, 128, 1, SplitScratch(gpu))
    with pytest.raises(JkError, match="too small"):
        matmul_grouped(gpu, Buf(x, k), w, g, Buf(out), 32, 128, 1, SplitScratch(gpu))
    with pytest.raises(JkError, match="1..16"):
        matvec_grouped(gpu, Buf(x), w, g, Buf(out), 17)
