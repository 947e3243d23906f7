"""ctypes binding of libjk.so (the C ABI declared in include/jk.h).

The library is the product: there is no CPU or PyTorch fallback. If libjk.so is missing or
fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libjk.so")

# Every symbol include/jk.h declares, with (restype, argtypes).
P, S, I, U32, U64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64


class Plan(ctypes.Structure):
    """Plan (crates/jevons-kernels/src/gemm.rs:973-979): bm == 0 selects the small-row kernel."""

    _fields_ = [("bm", ctypes.c_int32), ("bn", ctypes.c_int32), ("splits", ctypes.c_int32)]

    def __repr__(self):
        return f"Plan(bm={self.bm}, bn={self.bn}, splits={self.splits})"

    def __eq__(self, other):
        return isinstance(other, Plan) and (self.bm, self.bn, self.splits) == (other.bm, other.bn, other.splits)

    def __hash__(self):
        return hash((self.bm, self.bn, self.splits))


class Groups(ctypes.Structure):
    """jk_groups: Groups (crates/jevons-kernels/src/gemm.rs:955-966) as device pointers."""

    _fields_ = [("sorted", ctypes.c_void_p), ("offsets", ctypes.c_void_p), ("jobs", ctypes.c_void_p),
                ("max_jobs", ctypes.c_size_t), ("in_div", ctypes.c_uint32), ("rows", ctypes.c_size_t)]


class GgufTensorInfo(ctypes.Structure):
    """jk_gguf_tensor_info: TensorInfo (crates/jevons-formats/src/gguf.rs:148-156)."""

    _fields_ = [("name", ctypes.c_char_p), ("n_dims", ctypes.c_uint32), ("dims", ctypes.c_uint64 * 4),
                ("type", ctypes.c_int32), ("offset", ctypes.c_uint64), ("bytes", ctypes.c_uint64)]


SIGNATURES = {
    "jk_last_error": (ctypes.c_char_p, []),
    "jk_abi_version": (I, []),
    "jk_tensor_type_block": (I, [I, ctypes.POINTER(U64), ctypes.POINTER(U64)]),
    "jk_q4k_scale_min": (I, [I, P, ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(ctypes.c_uint8)]),
    "jk_packed_words": (I, [I, P]),
    "jk_pack": (I, [I, P, S, P, S, P, S, P, S, P, S]),
    "jk_gpu_init": (I, [I]),
    "jk_gpu_sync": (I, [P]),
    "jk_device_error": (I, [I, ctypes.POINTER(U32)]),
    "jk_qmatrix_upload": (I, [I, I, S, S, S, P, S, ctypes.POINTER(P)]),
    "jk_qmatrix_from_packed": (I, [I, I, S, S, S, P, S, P, S, P, S, P, S, ctypes.POINTER(P)]),
    "jk_qmatrix_f16_view": (I, [I, S, S, P, ctypes.POINTER(P)]),
    "jk_qmatrix_destroy": (None, [P]),
    "jk_qmatrix_info": (I, [P, ctypes.POINTER(I), ctypes.POINTER(S), ctypes.POINTER(S), ctypes.POINTER(S),
                            ctypes.POINTER(S)]),
    "jk_qmatrix_dequantize": (I, [P, P, S, P]),
    "jk_plan_heuristic": (I, [P, S, I, I, ctypes.POINTER(Plan)]),
    "jk_plan_valid_for": (I, [ctypes.POINTER(Plan), P, S]),
    "jk_split_scratch_create": (I, [I, ctypes.POINTER(P)]),
    "jk_split_scratch_destroy": (None, [P]),
    "jk_matmul_plan": (I, [P, P, I, S, S, P, S, P, Plan, P]),
    "jk_matmul": (I, [P, P, I, S, S, P, S, P, P]),
    "jk_matvec": (I, [P, P, I, S, S, P, S, P]),
    "jk_matmul_tiled": (I, [P, P, I, S, S, P, S, I, I, P]),
    "jk_f16_linear": (I, [P, S, S, P, S, P, P]),
    "jk_f16_linear_scaled": (I, [P, S, S, P, S, P, P, P]),
    "jk_dequantize": (I, [I, P, S, P, S]),
    "jk_quantize_act_q8": (I, [P, I, S, S, P, S, P, S, P]),
    "jk_matmul_q8_int8": (I, [P, P, S, P, S, S, P, S, P]),
    "jk_ipc_alloc": (I, [I, S, ctypes.POINTER(P), P]),
    "jk_ipc_free": (I, [I, P]),
    "jk_ipc_open": (I, [I, P, ctypes.POINTER(P)]),
    "jk_ipc_close": (I, [I, P]),
    "jk_sharded_matmul_allgather": (I, [P, P, I, S, S, I, I, P, P, I, I, P, P]),
    "jk_allgather_wait": (I, [I, P, I, I, P]),
    "jk_matmul_splitk_noalloc": (I, [P, P, I, S, S, P, S, I, P]),
    "jk_set_max_ctas": (I, [I, I]),
    "jk_get_max_ctas": (I, [I, ctypes.POINTER(I), ctypes.POINTER(I)]),
    "jk_group_max_jobs": (S, [S, S, I]),
    "jk_group_experts": (I, [I, P, S, S, I, P, P, P, S, P]),
    "jk_matmul_grouped": (I, [P, P, I, S, ctypes.POINTER(Groups), P, S, I, I, I, P, P]),
    "jk_matvec_grouped": (I, [P, P, I, S, ctypes.POINTER(Groups), P, S, I, P]),
    "jk_embed_q6k": (I, [P, P, S, P, P, S, ctypes.c_float, P, P, P]),
    "jk_pick_logits": (I, [P, P, S, P, S, ctypes.c_float, P, P]),
    "jk_q6k_transpose_f16": (I, [P, P, S, P]),
    "jk_softcap": (I, [P, S, ctypes.c_float, P]),
    "jk_gguf_open": (I, [ctypes.c_char_p, ctypes.POINTER(P)]),
    "jk_gguf_close": (None, [P]),
    "jk_gguf_tensor_count": (S, [P]),
    "jk_gguf_metadata_count": (S, [P]),
    "jk_gguf_tensor_at": (I, [P, S, ctypes.POINTER(GgufTensorInfo)]),
    "jk_gguf_tensor": (I, [P, ctypes.c_char_p, ctypes.POINTER(GgufTensorInfo)]),
    "jk_gguf_read": (I, [P, ctypes.c_char_p, U64, U64, P]),
    "jk_gguf_read_f32": (I, [P, ctypes.c_char_p, P, S]),
    "jk_gguf_value_kind": (I, [P, ctypes.c_char_p, ctypes.POINTER(I), ctypes.POINTER(I), ctypes.POINTER(S)]),
    "jk_gguf_u64": (I, [P, ctypes.c_char_p, ctypes.c_int64, ctypes.POINTER(U64)]),
    "jk_gguf_i64": (I, [P, ctypes.c_char_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_int64)]),
    "jk_gguf_f32": (I, [P, ctypes.c_char_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_float)]),
    "jk_gguf_bool": (I, [P, ctypes.c_char_p, ctypes.c_int64, ctypes.POINTER(I)]),
    "jk_gguf_str": (I, [P, ctypes.c_char_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(S)]),
    "jk_qmatrix_from_gguf": (I, [I, P, ctypes.c_char_p, ctypes.POINTER(P)]),
    "jk_tune_bucket": (S, [S]),
    "jk_tune_pick": (I, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(Plan), S, Plan, ctypes.POINTER(Plan)]),
    "jk_tuner_create": (I, [I, ctypes.c_char_p, I, ctypes.POINTER(P)]),
    "jk_tuner_destroy": (None, [P]),
    "jk_tuner_size": (S, [P]),
    "jk_tuner_plan": (I, [P, P, S, I, ctypes.POINTER(Plan)]),
    "jk_tuner_tune": (I, [P, ctypes.POINTER(P), S, S, I, P, I, S, P, S, P, P, ctypes.POINTER(Plan)]),
    "jk_tuner_save": (I, [P]),
    "jk_tuner_group_plan": (I, [P, P, S, ctypes.POINTER(Plan)]),
    "jk_tuner_tune_grouped": (I, [P, ctypes.POINTER(P), S, S, S, P, S, P, I, S, P, S, P, P, P, S, P, P,
                                  ctypes.POINTER(Plan)]),
}

STATUS = {0: "JK_OK", 1: "JK_ERR_INVALID", 2: "JK_ERR_UNSUPPORTED", 3: "JK_ERR_SHAPE", 4: "JK_ERR_CUDA",
          5: "JK_ERR_NCCL", 6: "JK_ERR_TIMEOUT"}


class JkError(RuntimeError):
    """A failing jk_* call: `status` is the jk_status code, the message is jk_last_error()."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status
        self.message = message


_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libjk.so is not built ({LIB_PATH}); run jevons-rs_b200/build.py")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status: int) -> None:
    if status != 0:
        raise JkError(status, load().jk_last_error().decode("utf-8", "replace"))
