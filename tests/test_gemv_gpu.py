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
