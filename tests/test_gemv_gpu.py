"""GPU: the small-row kernel (matvec, m <= 16; gemm.rs:1135-1168) against the f64 oracle."""
import numpy as np
import pytest
import torch

from helpers import KINDS, activations, assert_close, make_weights

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", list(KINDS))
@pytest.mark.parametrize("m", [1, 2, 3, 16])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_matvec_matches_oracle(gpu, name, m, dtype):
    from jevons_kernels.gemm import Buf, matvec
    n, k = 320, 1024
    w, raw, dense = make_weights(gpu, KINDS[name], n, k, seed=m)
    x, x_exact = activations(m, k, dtype, seed=m + 10)
    out = torch.full((m, n), float("nan"), device="cuda")
    matvec(gpu, Buf(x), m, w, Buf(out))
    assert_close(f"{name} m={m} {dtype}", out.cpu().numpy(), x_exact, dense)


@pytest.mark.parametrize("name", list(KINDS))
@pytest.mark.parametrize("n,k", [(64, 256), (4096, 4096), (2560, 10240)])
def test_matvec_shapes(gpu, name, n, k):
    from jevons_kernels.gemm import Buf, matvec
    w, raw, dense = make_weights(gpu, KINDS[name], n, k, seed=n)
    x, x_exact = activations(1, k, torch.float32, seed=3)
    out = torch.empty((1, n), device="cuda")
    matvec(gpu, Buf(x), 1, w, Buf(out))
    assert_close(f"{name} {n}x{k}", out.cpu().numpy(), x_exact, dense)


def test_matvec_config0_q8_0(gpu):
    """Q8_0 4096x4096, f32 activations, M=1, seed 0."""
    from jevons_kernels.gemm import Buf, matvec
    w, raw, dense = make_weights(gpu, KINDS["Q8_0"], 4096, 4096, seed=0)
    x, x_exact = activations(1, 4096, torch.float32, seed=0)
    out = torch.empty((1, 4096), device="cuda")
    matvec(gpu, Buf(x), 1, w, Buf(out))
    assert_close("cfg0", out.cpu().numpy(), x_exact, dense)


def test_matvec_rejects_too_many_rows(gpu):
    from jevons_kernels.gemm import Buf, JkError, matvec
    w, _, _ = make_weights(gpu, KINDS["Q8_0"], 64, 64)
    x = torch.zeros(17, 64, device="cuda")
    with pytest.raises(JkError):
        matvec(gpu, Buf(x), 17, w, Buf(torch.zeros(17, 64, device="cuda")))


def test_matvec_zero_rows_is_a_no_op(gpu):
    from jevons_kernels.gemm import Buf, matvec
    w, _, _ = make_weights(gpu, KINDS["Q4_K"], 64, 256)
    out = torch.full((1, 64), 7.0, device="cuda")
    matvec(gpu, Buf(torch.zeros(1, 256, device="cuda")), 0, w, Buf(out))
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)


def test_matvec_buffer_size_checks(gpu):
    from jevons_kernels.gemm import Buf, JkError, matvec
    w, _, _ = make_weights(gpu, KINDS["Q4_K"], 64, 256)
    with pytest.raises(JkError, match="too small"):
        matvec(gpu, Buf(torch.zeros(2, 256, device="cuda")), 2, w, Buf(torch.zeros(64, device="cuda")))


@pytest.mark.parametrize("name", list(KINDS))
@pytest.mark.parametrize("m", [1, 2])
def test_matvec_many_row_groups(gpu, name, m):
    """More 8-row groups than resident warps: every warp walks several groups."""
    from jevons_kernels.gemm import Buf, matvec
    n, k = 40960, 256
    w, raw, dense = make_weights(gpu, KINDS[name], n, k, seed=5)
    x, x_exact = activations(m, k, torch.bfloat16, seed=6)
    out = torch.full((m, n), float("nan"), device="cuda")
    matvec(gpu, Buf(x), m, w, Buf(out))
    assert_close(f"{name} {n}x{k} m={m}", out.cpu().numpy(), x_exact, dense)


@pytest.mark.parametrize("name", ["Q8_0", "Q5_0"])
@pytest.mark.parametrize("k", [64, 320, 2368])
def test_matvec_partial_last_step(gpu, name, k):
    """K not a multiple of 256 (32-weight block formats): the last 256-step is partial."""
    from jevons_kernels.gemm import Buf, matvec
    n = 192
    w, raw, dense = make_weights(gpu, KINDS[name], n, k, seed=k)
    x, x_exact = activations(2, k, torch.float32, seed=k + 1)
    out = torch.full((2, n), float("nan"), device="cuda")
    matvec(gpu, Buf(x), 2, w, Buf(out))
    assert_close(f"{name} k={k}", out.cpu().numpy(), x_exact, dense)


@pytest.mark.parametrize("name", list(KINDS))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_matvec_unaligned_activations(gpu, name, dtype):
    """Activations that do not start on a 16-byte boundary take the scalar staging loads."""
    from jevons_kernels.gemm import Buf, matvec
    n, k = 256, 512
    w, raw, dense = make_weights(gpu, KINDS[name], n, k, seed=9)
    x, x_exact = activations(1, k + 1, dtype, seed=10)
    xs = x.view(-1)[1:]
    assert xs.data_ptr() % 16 != 0
    out = torch.full((1, n), float("nan"), device="cuda")
    matvec(gpu, Buf(xs), 1, w, Buf(out))
    assert_close(f"{name} unaligned", out.cpu().numpy(), x_exact.reshape(-1)[1:].reshape(1, k), dense)


@pytest.mark.parametrize("m", [1, 3])
def test_matvec_f16_view(gpu, m):
    """FP16 weights through a view of a caller-owned tensor."""
    from jevons_kernels.gemm import Buf, QMatrix, matvec
    n, k = 512, 1536
    rng = np.random.default_rng(4)
    wt = torch.from_numpy(rng.normal(0, 0.05, (n, k)).astype(np.float32)).cuda().half()
    w = QMatrix.f16_view(gpu, n, k, wt)
    x, x_exact = activations(m, k, torch.bfloat16, seed=12)
    out = torch.full((m, n), float("nan"), device="cuda")
    matvec(gpu, Buf(x), m, w, Buf(out))
    assert_close(f"F16 m={m}", out.cpu().numpy(), x_exact, wt.float().cpu().numpy())


def test_matvec_chain_orders_reads_and_writes(gpu):
    """Back-to-back products on one stream: the second reads the first's output (read after
    write) and overwrites the first's input (write after read). Run once with a device sync
    after every product and once back to back: the kernels are deterministic, so both runs
    must agree bit for bit, and the synchronised run is checked against the oracle."""
    from jevons_kernels.gemm import Buf, matvec
    k = 2048
    mats = [make_weights(gpu, KINDS[nm], k, k, seed=20 + i) for i, nm in enumerate(["Q4_K", "Q6_K", "Q8_0"])]
    a0, a_exact = activations(1, k, torch.float32, seed=30)

    def run(sync):
        a = a0.clone()
        b = torch.full((1, k), float("nan"), device="cuda")
        seen = []
        for i, (src, dst) in enumerate([(a, b), (b, a), (a, b)]):
            matvec(gpu, Buf(src), 1, mats[i][0], Buf(dst))
            if sync:
                seen.append(dst.cpu().numpy())
        torch.cuda.synchronize()
        return b.cpu().numpy(), seen

    for _ in range(3):
        back_to_back, _ = run(False)
        stepwise, seen = run(True)
        assert np.array_equal(back_to_back, stepwise)
    inputs = [a_exact, seen[0], seen[1]]
    for i in range(3):
        assert_close(f"chain {i}", seen[i], inputs[i], mats[i][2])
