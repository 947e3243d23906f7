"""GPU: the allocation-free split-K product (jk_matmul_splitk_noalloc), through the C ABI, against
the f64 oracle and against the existing split-K entry point (jk_matmul_plan with a growable
jk_split_scratch).

The allocation-free variant exists for callers that cannot allocate device memory while a product
runs (a framework owning every device allocation, latency paths that cannot afford cudaMalloc's
device synchronisation): its scratch is a fixed buffer inside libjk.so. It must give the same
products, within the library tolerance, call after call -- the buffer keeps the previous call's
contents, so two calls in a row check that nothing stale leaks.

This file is named to be collected last, so a run that stops at the first failure has already
run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import KINDS, activations, assert_close, make_weights
from jevons_kernels._lib import JkError, Plan, check, load

pytestmark = pytest.mark.gpu


def noalloc(w, x, m, out, bm):
    xt = {torch.bfloat16: 2, torch.float16: 1, torch.float32: 0}[x.dtype]
    return load().jk_matmul_splitk_noalloc(w.handle, ctypes.c_void_p(x.data_ptr()), xt, x.numel(), m,
                                           ctypes.c_void_p(out.data_ptr()), out.numel(), bm,
                                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("name,n,k,m,bm", [("Q4_K", 10240, 2560, 256, 256), ("Q6_K", 2560, 10240, 96, 128),
                                           ("Q8_0", 1024, 1024, 37, 64)])
def test_noalloc_matches_scratch_product_twice(gpu, name, n, k, m, bm):
    from jevons_kernels.gemm import SplitScratch
    w, _, dense = make_weights(gpu, KINDS[name], n, k, seed=n + m)
    x, x_exact = activations(m, k, torch.bfloat16, seed=m)
    ref = torch.empty(m, n, device="cuda")
    scratch = SplitScratch(gpu)
    check(load().jk_matmul_plan(w.handle, ctypes.c_void_p(x.data_ptr()), 2, x.numel(), m,
                                ctypes.c_void_p(ref.data_ptr()), ref.numel(), scratch.handle, Plan(bm, 128, 2),
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    ref_np = ref.cpu().numpy().astype(np.float64)
    for call in range(2):  # the second call runs on the buffer the first one left behind
        out = torch.full((m, n), float("nan"), device="cuda")
        check(noalloc(w, x, m, out, bm))
        got = out.cpu().numpy()
        assert_close(f"{name} noalloc call {call} vs oracle", got, x_exact, dense)
        assert_close(f"{name} noalloc call {call} vs jk_matmul_plan", got, x_exact, dense, want=ref_np)
    assert gpu.device_error() == 0


def test_noalloc_rejects_f32_activations_and_bad_tiles(gpu):
    w, _, _ = make_weights(gpu, KINDS["Q4_K"], 256, 512)
    x = torch.zeros(8, 512, device="cuda")
    out = torch.zeros(8, 256, device="cuda")
    assert noalloc(w, x, 8, out, 64) == 2  # JK_ERR_UNSUPPORTED: f32 would need a conversion buffer
    assert "bf16 or f16" in load().jk_last_error().decode()
    xb = x.bfloat16()
    assert noalloc(w, xb, 8, out, 48) == 1
    with pytest.raises(JkError):
        check(noalloc(w, xb, 9, out, 64))  # buffers too small for m=9
