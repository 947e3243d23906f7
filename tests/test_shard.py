"""CPU: the multi-GPU host logic (column shards, per-rank weight slices, the rank-major all-gather)
run as world-size-2 gloo process groups, checked against the single-process oracle product."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _paths():
    for p in (os.path.join(ROOT, "jevons-rs_b200"), ROOT, HERE):
        if p not in sys.path:
            sys.path.insert(0, p)


_paths()
from jevons_kernels.shard import SHARD_ALIGN, column_shard, shard_rows  # noqa: E402
from oracle import oracle  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("n,world", [(10240, 2), (10240, 8), (262144, 8), (192, 3), (640, 4), (64, 1)])
def test_column_shards_tile_the_rows(n, world):
    spans = [column_shard(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (lo, hi), (lo2, _) in zip(spans, spans[1:]):
        assert hi == lo2
    sizes = [hi - lo for lo, hi in spans]
    assert all(s % SHARD_ALIGN == 0 and s > 0 for s in sizes)
    assert max(sizes) - min(sizes) <= SHARD_ALIGN


def test_column_shard_rejects_bad_shapes():
    with pytest.raises(ValueError):
        column_shard(100, 2, 0)
    with pytest.raises(ValueError):
        column_shard(64, 2, 0)
    with pytest.raises(ValueError):
        column_shard(128, 2, 2)


def test_shard_rows_slices_whole_rows():
    from jevons_kernels import synth
    raw = synth.weights(oracle.Q6_K, np.random.default_rng(0), 256, 512)
    full = oracle.dequantize(oracle.Q6_K, raw).reshape(256, 512)
    part = np.frombuffer(shard_rows(raw, oracle.Q6_K, 256, 512, 64, 192), np.uint8)
    assert np.array_equal(oracle.dequantize(oracle.Q6_K, part).reshape(128, 512), full[64:192])
    with pytest.raises(ValueError):
        shard_rows(raw[:-1], oracle.Q6_K, 256, 512, 0, 64)


def _worker(rank, world, port, kind, n, k, m, fail_rank):
    _paths()
    import torch
    import torch.distributed as dist
    from jevons_kernels import synth
    from jevons_kernels.shard import column_shard, gather_shards, logical_columns, shard_rows
    from oracle import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        raw = synth.weights(kind, np.random.default_rng(11), n, k)      # every rank holds the file
        x = synth.activations(np.random.default_rng(12), m, k, round_to="bf16")
        lo, hi = column_shard(n, world, rank)
        part = np.frombuffer(shard_rows(raw, kind, n, k, lo, hi), np.uint8)
        w = oracle.dequantize(kind, part).reshape(hi - lo, k)
        local = torch.from_numpy(oracle.matmul_f64(x, w).astype(np.float32))
        if rank == fail_rank:
            raise RuntimeError("planted failure before the all-gather")
        gathered, _ = gather_shards(local)
        full = logical_columns(gathered).reshape(m, -1).numpy()
        want = oracle.matmul_f64(x, oracle.dequantize(kind, raw).reshape(n, k)).astype(np.float32)
        assert full.shape == (m, n)
        assert np.array_equal(full, want), "gathered columns differ from the single-process product"
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind,n,k,m", [(oracle.Q4_K, 1024, 512, 5), (oracle.Q8_0, 512, 256, 3)])
def test_two_rank_gather_matches_single_process_product(kind, n, k, m):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port(), kind, n, k, m, -1), nprocs=2, join=True)


def test_a_rank_that_fails_surfaces_as_an_error():
    """Rank 1 raises before the collective: the spawn reports its exception (rank 0's collective
    ends by the process group timeout or the peer's exit) instead of hanging."""
    import torch.multiprocessing as mp
    with pytest.raises(Exception):
        mp.spawn(_worker, args=(2, _free_port(), oracle.Q4_K, 256, 256, 2, 1), nprocs=2, join=True)
