"""CPU tests of the C ABI boundary: libjk.so loads, exports every symbol include/jk.h declares,
and its host-side validation answers like the reference (no GPU calls)."""
import ctypes
import os
import re

import numpy as np
import pytest

from jevons_kernels import _lib
from jevons_kernels._lib import JkError, check, load

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "jk.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(jk_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_expected_entry_points():
    syms = declared_symbols()
    for name in ("jk_qmatrix_upload", "jk_matmul_plan", "jk_matvec", "jk_f16_linear", "jk_pack",
                 "jk_plan_heuristic", "jk_qmatrix_dequantize", "jk_last_error"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"libjk.so lacks {missing}"


def test_python_binding_covers_every_declared_symbol():
    assert set(declared_symbols()) <= set(_lib.SIGNATURES), set(declared_symbols()) - set(_lib.SIGNATURES)


def test_abi_version():
    assert load().jk_abi_version() == 1


def upload(kind, n, k, experts, raw):
    out = ctypes.c_void_p()
    arr = np.frombuffer(bytes(raw), np.uint8) if len(raw) else np.zeros(1, np.uint8)
    st = load().jk_qmatrix_upload(0, kind, n, k, experts, arr.ctypes.data_as(ctypes.c_void_p), len(raw),
                                  ctypes.byref(out))
    return st, load().jk_last_error().decode()


def test_upload_rejects_wrong_byte_count_with_reference_message():
    # gemm.rs:841-845: "{kind:?} [{experts}x{n}, {k}] has the wrong byte count"
    st, msg = upload(12, 64, 256, 1, bytes(144 * 64 - 1))
    assert st == 3 and msg == "Q4K [1x64, 256] has the wrong byte count"


def test_upload_rejects_unsupported_shape_with_reference_message():
    # gemm.rs:875-885: n % 64 and k % 64 -> "... has an unsupported shape"
    st, msg = upload(8, 32, 64, 1, bytes(34 * 2 * 32))
    assert st == 3 and msg == "Q8_0 [1x32, 64] has an unsupported shape"
    st, msg = upload(8, 64, 96, 1, bytes(34 * 3 * 64))
    assert st == 3 and msg == "Q8_0 [1x64, 96] has an unsupported shape"


def test_upload_rejects_types_without_gpu_layout():
    st, msg = upload(0, 64, 64, 1, bytes(4 * 64 * 64))
    assert st == 2 and "not supported" in msg
    st, msg = upload(2, 64, 64, 1, bytes(16))
    assert st == 2


def test_errors_are_thread_local_messages():
    import threading
    seen = {}

    def worker():
        seen["msg"] = upload(12, 64, 256, 1, bytes(10))[1]
    upload(8, 32, 64, 1, bytes(34 * 2 * 32))
    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert "Q4K" in seen["msg"]
    assert load().jk_last_error().decode().startswith("Q8_0")


def test_check_raises_jkerror():
    st, _ = upload(12, 64, 256, 1, bytes(1))
    with pytest.raises(JkError) as e:
        check(st)
    assert e.value.status == 3 and "wrong byte count" in str(e.value)


def test_q4k_scale_min_rejects_out_of_range_j():
    sc, mn = ctypes.c_uint8(), ctypes.c_uint8()
    buf = (ctypes.c_uint8 * 12)()
    assert load().jk_q4k_scale_min(8, buf, ctypes.byref(sc), ctypes.byref(mn)) == 1


def test_pack_rejects_small_regions():
    raw = np.zeros(34, np.uint8)
    q = np.zeros(7, np.uint32)
    d = np.zeros(1, np.float32)
    st = load().jk_pack(8, raw.ctypes.data_as(ctypes.c_void_p), 34, q.ctypes.data_as(ctypes.c_void_p), 7, None, 0,
                        None, 0, d.ctypes.data_as(ctypes.c_void_p), 1)
    assert st == 1


def test_head_operators_reject_null_arguments_without_a_device():
    lib = load()
    null = ctypes.c_void_p(0)
    assert lib.jk_embed_q6k(null, null, 1, null, null, 0, ctypes.c_float(1e-6), null, null, null) == 1
    assert lib.jk_last_error().decode() == "embed_q6k: null table"
    assert lib.jk_pick_logits(null, null, 1, null, 1, ctypes.c_float(30.0), null, null) == 1
    assert lib.jk_last_error().decode() == "pick_logits: null table"
    assert lib.jk_q6k_transpose_f16(null, null, 0, null) == 1
    assert lib.jk_softcap(null, 4, ctypes.c_float(30.0), null) == 1
    assert "softcap" in lib.jk_last_error().decode()
    assert lib.jk_softcap(null, 0, ctypes.c_float(30.0), null) == 0  # nothing to do


# --- host dequantization: quant::dequantize (crates/jevons-formats/src/quant.rs:83-101) -------------

def host_dequantize(kind, raw, out_len=None):
    raw = np.ascontiguousarray(np.frombuffer(bytes(raw), np.uint8)) if not isinstance(raw, np.ndarray) else raw
    if out_len is None:
        elems, size = {0: (1, 4), 1: (1, 2), 12: (256, 144), 14: (256, 210), 6: (32, 22), 8: (32, 34)}[kind]
        out_len = len(raw) // size * elems
    out = np.full(max(out_len, 1), np.nan, np.float32)
    st = load().jk_dequantize(kind, raw.ctypes.data_as(ctypes.c_void_p) if len(raw) else None, len(raw),
                              out.ctypes.data_as(ctypes.c_void_p), out_len)
    return st, out[:out_len]


@pytest.mark.parametrize("name", ["Q4_K", "Q6_K", "Q8_0", "Q5_0"])
def test_host_dequantize_is_bit_exact_with_the_oracle(name):
    from oracle import oracle
    from jevons_kernels import synth
    kind = {"Q4_K": oracle.Q4_K, "Q6_K": oracle.Q6_K, "Q8_0": oracle.Q8_0, "Q5_0": oracle.Q5_0}[name]
    raw = synth.weights(kind, np.random.default_rng(5), 320, 1024)
    st, got = host_dequantize(kind, raw)
    assert st == 0
    want = oracle.dequantize(kind, raw)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # arbitrary bytes: NaN / inf / subnormal scales and every quant pattern
    junk = np.random.default_rng(6).integers(0, 256, size=len(raw), dtype=np.uint8)
    st, got = host_dequantize(kind, junk)
    want = oracle.dequantize(kind, junk)
    assert st == 0
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert same.all()


def test_host_dequantize_reference_known_answers():
    """The reference's own dequantization KATs (quant.rs:210-225), kept in tests/golden."""
    import json
    kat = json.load(open(os.path.join(REPO, "tests", "golden", "quant_kat.json")))
    for case in ("q8_0", "q5_0"):
        st, out = host_dequantize(kat[case]["type"], bytes(kat[case]["bytes"]))
        assert st == 0
        for i, v in kat[case]["expect"].items():
            assert out[int(i)] == v, (case, i)


def test_host_dequantize_errors_follow_the_reference():
    st, _ = host_dequantize(8, bytes(33), 32)
    assert st == 3 and load().jk_last_error().decode() == "dequantization size mismatch"
    st, _ = host_dequantize(8, bytes(34), 31)
    assert st == 3
    st, _ = host_dequantize(2, bytes(18), 32)
    assert st == 2 and load().jk_last_error().decode() == "unsupported tensor type"
    st, out = host_dequantize(1, np.float16([1.5, -2.0]).view(np.uint8).copy())
    assert st == 0 and list(out) == [1.5, -2.0]
    st, out = host_dequantize(0, np.float32([3.25]).view(np.uint8).copy())
    assert st == 0 and out[0] == 3.25
