"""ctypes binding of ``libmolten_cuda.so`` (the C ABI in include/molten_cuda.h).

The library is the product: there is no Python or CPU fallback. Importing this
module without the built library raises, and every C call that returns an
error raises :class:`McError` with the library's message.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmolten_cuda.so"

MC_OK = 0
MC_EINVAL = -1
MC_ECUDA = -2
MC_EUNSUPPORTED = -3
MC_ENCCL = -4
MC_ETIMEOUT = -5

TEST_SKIP_LOGIT_PUBLISH = 1
TEST_SKIP_BARRIER_ARRIVE = 2

ROUTE_SOFTMAX_RENORM = 0
ROUTE_SIGMOID_BIAS = 1
DTYPE_BF16 = 0
DTYPE_F32 = 1


class McError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"molten_cuda error {code}: {msg}")
        self.code = code


class Sampling(C.Structure):
    """mc_sampling."""

    _fields_ = [
        ("temperature", C.c_float),
        ("top_k", C.c_uint32),
        ("top_p", C.c_float),
        ("repetition_penalty", C.c_float),
        ("seed", C.c_uint64),
    ]


class QW(C.Structure):
    """mc_qweights."""

    _fields_ = [
        ("codes", C.c_void_p),
        ("scales", C.c_void_p),
        ("biases", C.c_void_p),
        ("out_features", C.c_int32),
        ("in_features", C.c_int32),
        ("group_size", C.c_int32),
        ("bits", C.c_int32),
    ]


P = C.c_void_p
I = C.c_int
F = C.c_float
QP = C.POINTER(QW)

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "mc_create": (I, [I, P, C.POINTER(P)]),
    "mc_destroy": (I, [P]),
    "mc_set_stream": (I, [P, P]),
    "mc_sync": (I, [P]),
    "mc_last_error": (C.c_char_p, []),
    "mc_version": (C.c_char_p, []),
    "mc_check_quant": (I, [QP]),
    "mc_gemv_quant": (I, [P, QP, P, P, I]),
    "mc_gemv_head_argmax": (I, [P, QP, P, P, I]),
    "mc_token_tail": (I, [P, P, P, P, I, P, P, P, I, F, I]),
    "mc_argmax_bf16": (I, [P, P, I, P, I]),
    "mc_add_rmsnorm": (I, [P, P, P, P, P, P, I, F, I]),
    "mc_router_addnorm_route": (I, [P, P, P, P, P, P, P, I, P, I, P, P, P, P, I, I, F, F, I]),
    "mc_gemv_router": (I, [P, P, I, P, P, I, I, I]),
    "mc_route_token": (I, [P, P, I, I, P, F, P, P, I]),
    "mc_gemv_gather_act": (I, [P, QP, QP, P, P, P, I, I]),
    "mc_gemv_gather_down_combine4": (I, [P, QP, P, P, P, P, I, I]),
    "mc_moe_decode_layer": (I, [P, P, P, P, P, P, P, I, P, I, P, P, P, QP, QP, QP, I, P, P,
                                C.c_size_t, F, F]),
    "mc_moe_decode_workspace_words": (C.c_size_t, [I]),
    "mc_map_ids": (I, [P, P, C.c_size_t, P, I, P]),
    "mc_ep_alloc": (I, [P, C.c_size_t, C.POINTER(C.c_void_p)]),
    "mc_ep_free": (I, [P, P]),
    "mc_ipc_handle": (I, [P, P, P]),
    "mc_ipc_open": (I, [P, P, C.POINTER(C.c_void_p)]),
    "mc_ipc_close": (I, [P, P]),
    "mc_ep_dispatch": (I, [P, P, I, I, P, P, I, I, I, P, C.c_size_t, P]),
    "mc_ep_tiles": (I, [P, P, I, I, I, I, P, P, P, I]),
    "mc_ep_unique_id": (I, [P]),
    "mc_ep_init": (I, [P, I, I, P, I]),
    "mc_ep_reserve": (I, [P, I, I, I, I, I]),
    "mc_ep_place": (I, [P, I, I, I, P, P]),
    "mc_ep_moe_prefill": (I, [P, P, P, I, QP, QP, QP, P, I, P, P]),
    "mc_ep_status": (I, [P, P]),
    "mc_ep_counts": (I, [P, P, C.c_size_t]),
    "mc_ep_finalize": (I, [P]),
    "mc_ep_set_profile": (I, [P, I]),
    "mc_ep_phase_ms": (I, [P, P]),
    "mc_ep_return": (I, [P, P, C.c_size_t, I, P, I, I, I, P, C.c_size_t, P]),
    "mc_moe_decode_layer_noalloc": (I, [P, P, P, P, P, P, P, I, P, I, P, P, P, QP, QP, QP, I, P,
                                        P, F, F]),
    "mc_moe_decode_proj_workspace_words": (C.c_size_t, [I]),
    "mc_moe_decode_layer_proj": (I, [P, P, QP, P, P, P, P, P, I, P, I, P, P, P, QP, QP, QP, I, P,
                                     P, C.c_size_t, F, F]),
    "mc_proj3_gemv_scatter": (I, [P, QP, QP, QP, P, P, P, P, I, I]),
    "mc_conv3_gemv": (I, [P, QP, P, P, P, P, P, I]),
    "mc_gemv_gu_act": (I, [P, QP, QP, P, P, I]),
    "mc_sample_workspace_bytes": (C.c_size_t, [I]),
    "mc_sample_draw": (I, [P, P, I, P, C.POINTER(Sampling), C.c_uint32, P, P, P, C.c_size_t]),
    "mc_sample_mark": (I, [P, P, P, I, P]),
    "mc_moe_route_batch": (I, [P, P, I, I, I, P, F, P, P]),
    "mc_moe_sort_map": (I, [P, P, I, I, I, P, P, P, P, P, P, I]),
    "mc_gather_rows_bf16": (I, [P, P, P, I, I, P]),
    "mc_gemm_q4_grouped": (I, [P, P, I, QP, I, P, P, P, I, P]),
    "mc_gemm_q4_grouped_gu": (I, [P, P, I, QP, QP, I, P, P, P, I, P]),
    "mc_moe_prefill_workspace_size": (C.c_size_t, [I, I, I, I]),
    "mc_moe_prefill": (I, [P, P, P, I, QP, QP, QP, I, I, P, P, C.c_size_t, P]),
    "mc_silu_mul_bf16": (I, [P, P, P, P, C.c_size_t]),
    "mc_moe_combine_rows": (I, [P, P, P, P, P, I, I, I]),
    "mc_eval_math": (I, [P, I, P, P, I]),
    "mc_set_trace": (I, [P, P, I]),
    "mc_set_l2_prefetch": (I, [P, P, C.c_size_t, P, C.c_size_t]),
    "mc_set_wait_limit": (I, [P, C.c_ulonglong]),
    "mc_set_test_flags": (I, [P, I]),
    "mc_copy_async": (I, [P, P, P, C.c_size_t]),
    "mc_gemm_q4_workspace_words": (C.c_size_t, [I]),
    "mc_gemm_q4": (I, [P, P, I, QP, P, P, C.c_size_t, P]),
}

_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Loads the library once (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m molten_b200.build` "
                "(the CUDA library is required; there is no fallback)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != MC_OK:
        raise McError(rc, lib().mc_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
