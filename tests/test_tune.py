"""The plan tuner (crates/jevons-gemma4-diffusion/src/gpu/tune.rs).

CPU: the reference's own unit tests of `bucket` and `pick` (tune.rs:590-611), through the C ABI.
GPU: tuning picks valid plans (no split-K when row invariance is asked for), the tuned plan
computes the same product, lookups fall back to the heuristic, and the stored table loads back
only on the device profile it was measured on.
"""
import os

import numpy as np
import pytest

from jevons_kernels._lib import Plan
from jevons_kernels import tune


def test_row_buckets_cover_each_power_of_two_range():
    assert tune.bucket(1) == 4
    assert tune.bucket(12) == 16
    assert tune.bucket(16) == 16
    assert tune.bucket(17) == 32
    assert tune.bucket(300) == 512


def test_heuristic_plan_is_kept_unless_clearly_slower():
    h, a, b = Plan(128, 128, 1), Plan(64, 128, 1), Plan(32, 128, 2)
    assert tune.pick([1.00, 0.97], [h, a], h) == h
    assert tune.pick([1.00, 0.90], [h, a], h) == a
    assert tune.pick([0.80, 0.90], [a, b], h) == a
    assert tune.pick([], [], h) is None


def _setup(gpu, m, copies=4, n=10240, k=2560):
    import torch
    from jevons_kernels import synth
    from jevons_kernels.gemm import Buf, QMatrix
    from oracle import oracle
    raw = synth.q4k_blocks(np.random.default_rng(5), n, k)
    ws = [QMatrix.upload(gpu, oracle.Q4_K, n, k, 1, raw) for _ in range(copies)]
    b = tune.bucket(m)
    x = torch.from_numpy(synth.activations(np.random.default_rng(6), b, k)).cuda().bfloat16()
    out = torch.empty(b * n, device="cuda")
    return raw, ws, Buf(x), Buf(out)


@pytest.mark.gpu
@pytest.mark.parametrize("m,row_invariant", [(256, True), (200, False), (8, False)])
def test_tuned_plan_is_valid_and_computes_the_same_product(gpu, m, row_invariant):
    import torch
    from jevons_kernels.gemm import Buf, SplitScratch, matmul_plan  # noqa: F401 (attaches Plan.heuristic)
    raw, ws, xb, ob = _setup(gpu, m)
    sc = SplitScratch(gpu)
    t = tune.Tuner(gpu)
    chosen = t.tune_dense(ws, m, row_invariant, xb, ob, sc)
    assert len(t) == 1
    assert t.dense(ws[0], m, row_invariant) == chosen
    if row_invariant:
        assert chosen.bm > 0 and chosen.splits == 1
    x = xb.tensor[: m * ws[0].k].view(m, ws[0].k)
    a = torch.empty(m, ws[0].n, device="cuda")
    b = torch.empty(m, ws[0].n, device="cuda")
    heur = Plan.heuristic(ws[0], m, row_invariant)
    matmul_plan(gpu, Buf(x), m, ws[0], Buf(a), scratch=sc, plan=chosen)
    matmul_plan(gpu, Buf(x), m, ws[0], Buf(b), scratch=sc, plan=heur)
    torch.cuda.synchronize()
    if row_invariant:
        assert torch.equal(a, b), "row-invariant plans must agree bit for bit"
    else:
        from helpers import assert_close
        from oracle import oracle
        dense = oracle.dequantize(oracle.Q4_K, raw).reshape(ws[0].n, ws[0].k)
        assert_close("tuned", a.cpu().numpy(), x.float().cpu().numpy(), dense)
    assert gpu.device_error() == 0


@pytest.mark.gpu
def test_lookup_falls_back_to_the_heuristic_and_table_round_trips(gpu, tmp_path):
    from jevons_kernels import gemm  # noqa: F401 (attaches Plan.heuristic)
    path = str(tmp_path / "autotune.txt")
    raw, ws, xb, ob = _setup(gpu, 64, copies=2)
    t = tune.Tuner(gpu, path)
    assert t.dense(ws[0], 64, True) == Plan.heuristic(ws[0], 64, True)
    chosen = t.tune_dense(ws, 64, True, xb, ob)
    t.save()
    lines = open(path).read().splitlines()
    assert lines[1] == f"dense 12 {ws[0].n} {ws[0].k} 64 1 {chosen.bm} {chosen.bn} {chosen.splits}"
    again = tune.Tuner(gpu, path)
    assert len(again) == 1 and again.dense(ws[0], 40, True) == chosen
    assert len(tune.Tuner(gpu, path, load_stored=False)) == 0
    with open(path, "w") as f:  # another profile line: the stored plans are ignored
        f.write("v0 another device\n" + "\n".join(lines[1:]) + "\n")
    assert len(tune.Tuner(gpu, path)) == 0
    os.remove(path)


@pytest.mark.gpu
def test_grouped_tuning_picks_a_tile_that_computes_the_grouped_product(gpu, tmp_path):
    import torch
    from jevons_kernels import synth
    from jevons_kernels.gemm import (Buf, Groups, QMatrix, SplitScratch, group_max_jobs, group_routes,
                                     matmul_grouped)
    from oracle import oracle
    experts, n, k, m, top_k = 16, 256, 512, 48, 4
    raw = synth.q4k_blocks(np.random.default_rng(12), experts * n, k)
    ws = [QMatrix.upload(gpu, oracle.Q4_K, n, k, experts, raw) for _ in range(2)]
    a = tune.bucket(m) * top_k
    x = torch.from_numpy(synth.activations(np.random.default_rng(13), a, k)).cuda().bfloat16()
    out = torch.empty(a * n, device="cuda")
    path = str(tmp_path / "autotune.txt")
    t = tune.Tuner(gpu, path)
    assert t.grouped(ws[0], m) == Plan(32, 128, 1)
    chosen = t.tune_grouped(ws, m, top_k, Buf(x), Buf(out), SplitScratch(gpu))
    assert t.grouped(ws[0], m) == chosen and chosen.splits == 1 and n % chosen.bn == 0
    t.save()
    assert f"grouped 12 {n} {k} {experts} {tune.bucket(m)} {chosen.bm} {chosen.bn}" in open(path).read()
    assert tune.Tuner(gpu, path).grouped(ws[0], m) == chosen
    # the chosen tile computes the grouped product of the reference's synthetic routes
    ids = (np.arange(a) // top_k * 7 + np.arange(a) % top_k * 13) % experts
    ids_t = torch.from_numpy(ids.astype(np.int32)).cuda()
    mj = group_max_jobs(a, experts, chosen.bm)
    sorted_ = torch.empty(a, dtype=torch.int32, device="cuda")
    offsets = torch.empty(experts + 1, dtype=torch.int32, device="cuda")
    jobs = torch.empty(1 + 2 * mj, dtype=torch.int32, device="cuda")
    group_routes(gpu, Buf(ids_t), Buf(sorted_), Buf(offsets), Buf(jobs), a, experts, chosen.bm)
    g = Groups(Buf(sorted_), Buf(offsets), Buf(jobs), mj, 1, a)
    res = torch.empty(a, n, device="cuda")
    matmul_grouped(gpu, Buf(x), ws[0], g, Buf(res), chosen.bm, chosen.bn, 1, SplitScratch(gpu))
    torch.cuda.synchronize()
    dense = oracle.dequantize(oracle.Q4_K, raw).reshape(experts * n, k)
    xe = x.float().cpu().numpy()
    want = oracle.matmul_grouped_f64(xe, dense, n, ids, 1)
    # the product bound of every GPU test, per route with its own expert's rows:
    # |err[r, c]| <= 1e-3 |x_r| |W_ids[r], c|
    wn = oracle.row_norms(dense).reshape(experts, n)
    bound = 1e-3 * oracle.row_norms(xe)[:, None] * wn[ids]
    assert np.all(np.abs(res.cpu().numpy() - want) <= bound)
    assert gpu.device_error() == 0
