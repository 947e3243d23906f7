"""GPU, 2 devices: jk_sharded_matmul_allgather -- the column-sharded product whose output shards
the copy engines push into every peer over NVLink -- run as two processes (one per GPU), against
the f64 oracle product of the whole matrix; and a peer that never signals, which must end the
other rank's bounded wait with an error instead of a hang. Skipped with fewer than 2 GPUs."""
import os
import socket
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, case, q):
    try:
        for p in (os.path.join(ROOT, "jevons-rs_b200"), ROOT, HERE):
            sys.path.insert(0, p)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from helpers import TOL
        from oracle import oracle
        from jevons_kernels import synth
        from jevons_kernels.gemm import Gpu, QMatrix, SplitScratch
        from jevons_kernels.shard import PeerGather, column_shard, shard_rows
        gpu = Gpu(rank)
        n_total, k, m = 2048, 1024, 200
        raw = synth.q4k_blocks(np.random.default_rng(5), n_total, k)
        lo, hi = column_shard(n_total, world, rank)
        w = QMatrix.upload(gpu, oracle.Q4_K, hi - lo, k, 1, np.frombuffer(shard_rows(raw, oracle.Q4_K, n_total, k, lo, hi), np.uint8))
        x = torch.from_numpy(synth.activations(np.random.default_rng(6), m, k)).cuda().bfloat16()
        pg = PeerGather(gpu, m, hi - lo, buffers=2)
        scratch = SplitScratch(gpu)
        if case == "product":
            for call in range(4):  # waiting per call, two calls per wait, and SM-pushed chunks
                buf = call % 2
                if call < 2:
                    pg.run(w, x, i=call % 2, wait=True, chunks=3, scratch=scratch)
                elif call == 3:
                    pg.run(w, x, i=0, wait=False, chunks=2, scratch=scratch)
                    pg.run(w, x, i=1, wait=False, chunks=1, scratch=scratch)
                    pg.wait()
                else:
                    # 8 chunks (7 row chunks at m=200): the last one reaches the peers through the
                    # SMs' copy kernel; the buffer is cleared first so that stale rows cannot pass
                    pg.output(0).zero_()
                    torch.cuda.synchronize()
                    dist.barrier()
                    pg.run(w, x, i=0, wait=True, chunks=8, scratch=scratch)
                    buf = 0
                torch.cuda.synchronize()
                got = pg.output(buf).permute(1, 0, 2).reshape(m, n_total).cpu().numpy()
                dense = oracle.dequantize(oracle.Q4_K, raw).reshape(n_total, k)
                xe = x.float().cpu().numpy()
                want = oracle.matmul_f64(xe, dense)
                bound = TOL * np.outer(oracle.row_norms(xe), oracle.row_norms(dense))
                err = np.abs(got - want)
                assert np.all(err <= bound), f"rank {rank} call {call}: {err.max()}"
            assert gpu.device_error() == 0
        else:  # rank 1 never calls: rank 0's bounded wait must end with the timeout bit
            if rank == 0:
                pg.run(w, x, i=0, wait=True, chunks=1, scratch=scratch)
                torch.cuda.synchronize()
                assert gpu.device_error() & 1 == 1
        dist.barrier()
        pg.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent
        import traceback
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("case", ["product", "silent_peer"])
def test_sharded_allgather_two_gpus(case):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, case, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r, msg = q.get(timeout=240)
        results[r] = msg
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
