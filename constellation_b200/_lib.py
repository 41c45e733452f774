"""ctypes binding of ``libconstellation_b200.so`` (the C ABI in ``include/constellation_b200.h``).

The library is built in-tree by ``constellation_b200.build``.  There is no fallback: if
the shared library is missing or fails to load, importing this module raises, and
every product entry point fails with that error.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libconstellation_b200.so"

CST_OK = 0
CST_ERR_UNKNOWN_EXPERT = 1
CST_ERR_NOT_RESIDENT = 2
CST_ERR_INVALID_ARG = 3
CST_ERR_BACKEND = 4
CST_ERR_CUDA = 5
CST_ERR_PEER = 6
CST_ERR_DEVICE_TIMEOUT = 7

CST_DTYPE_FP16 = 1
CST_DTYPE_BF16 = 2
CST_DTYPE_FP32 = 3

CST_FLAG_ADD_SHARED = 1

#: every symbol the header declares (tests check the library exports all of them)
EXPORTED = (
    "cst_create", "cst_destroy", "cst_upload_expert", "cst_free_expert", "cst_find_slot",
    "cst_set_shared_slot", "cst_route", "cst_moe_routed", "cst_moe_layer", "cst_grouped_ffn",
    "cst_expert_forward", "cst_device_error", "cst_ctx_info", "cst_last_error", "cst_abi_version",
    "cst_profile_enable", "cst_profile_read", "cst_shared_combine", "cst_combine_rows", "cst_dequant_fp8",
    "cst_route_noalloc", "cst_moe_routed_range", "cst_set_gemm_mode", "cst_rmsnorm",
    "cst_ipc_alloc", "cst_ipc_open", "cst_ipc_close", "cst_ipc_free", "cst_moe_routed_push", "cst_reduce_pushed",
    "cst_encode_infer_request", "cst_decode_infer_request", "cst_encode_infer_response", "cst_decode_infer_response",
    "cst_serve_infer_request", "cst_gather_rows", "cst_set_expert_own_tokens_only",
)
CST_INFER_REQUEST_FIXED_BYTES = 24
CST_INFER_RESPONSE_FIXED_BYTES = 20
CST_MAX_PEERS = 8
CST_GEMM_AUTO, CST_GEMM_DECODE, CST_GEMM_PREFILL = 0, 1, 2
CST_N_STAGES = 7
STAGE_NAMES = ("router", "route_pack", "pack_x", "grouped_up_gate", "pack_h", "grouped_down", "combine")


class CstConfig(ctypes.Structure):
    _fields_ = [
        ("hidden_dim", ctypes.c_int32),
        ("inter_dim", ctypes.c_int32),
        ("n_routed_experts", ctypes.c_int32),
        ("n_group", ctypes.c_int32),
        ("topk_group", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("norm_topk_prob", ctypes.c_int32),
        ("routed_scaling_factor", ctypes.c_float),
        ("block_size", ctypes.c_int32),
        ("n_slots", ctypes.c_int32),
        ("max_tokens", ctypes.c_int32),
        ("max_rows", ctypes.c_int32),
    ]


class CstExpertWeights(ctypes.Structure):
    _fields_ = [
        ("w_up", ctypes.c_void_p),
        ("w_up_scale", ctypes.c_void_p),
        ("w_gate", ctypes.c_void_p),
        ("w_gate_scale", ctypes.c_void_p),
        ("w_down", ctypes.c_void_p),
        ("w_down_scale", ctypes.c_void_p),
        ("rows", ctypes.c_int32),
        ("cols", ctypes.c_int32),
        ("row_block", ctypes.c_int32),
        ("col_block", ctypes.c_int32),
    ]


class CstError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[cst status {code}] {msg}")
        self.code = code


class CstIpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_uint8 * 64)]


class CstPeerSet(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("tl", ctypes.c_int32),
                ("tl_cap", ctypes.c_int32), ("recv", ctypes.c_void_p * CST_MAX_PEERS),
                ("flags", ctypes.c_void_p * CST_MAX_PEERS), ("epoch", ctypes.c_void_p), ("done", ctypes.c_void_p),
                ("x_offset", ctypes.c_int64), ("gather_epoch", ctypes.c_void_p),
                ("presence_offset", ctypes.c_int64)]


class CstInferRequest(ctypes.Structure):
    _fields_ = [("expert_id", ctypes.c_int32), ("batch_size", ctypes.c_int32), ("hidden_dim", ctypes.c_int32),
                ("input_dtype", ctypes.c_uint32), ("output_dtype", ctypes.c_uint32),
                ("activation_bytes", ctypes.c_uint32), ("activation", ctypes.c_void_p)]


class CstInferResponse(ctypes.Structure):
    _fields_ = [("status_code", ctypes.c_int32), ("batch_size", ctypes.c_int32), ("hidden_dim", ctypes.c_int32),
                ("output_dtype", ctypes.c_uint32), ("output_bytes", ctypes.c_uint32), ("output", ctypes.c_void_p)]


def _load() -> ctypes.CDLL:
    if not LIB_PATH.is_file():
        raise ImportError(
            f"{LIB_PATH.name} is not built; run `python -m constellation_b200.build` "
            "(nvcc, sm_100a). The MoE path has no CPU fallback.")
    lib = ctypes.CDLL(str(LIB_PATH))
    P, I32, U32, F, I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint32, ctypes.c_float, ctypes.c_int64
    sig = {
        "cst_create": (ctypes.c_int, [I32, ctypes.POINTER(CstConfig), ctypes.POINTER(P)]),
        "cst_destroy": (None, [P]),
        "cst_upload_expert": (ctypes.c_int, [P, I32, I32, ctypes.POINTER(CstExpertWeights), P]),
        "cst_free_expert": (ctypes.c_int, [P, I32]),
        "cst_find_slot": (I32, [P, I32]),
        "cst_set_expert_own_tokens_only": (ctypes.c_int, [P, I32, I32]),
        "cst_set_shared_slot": (ctypes.c_int, [P, I32]),
        "cst_set_gemm_mode": (ctypes.c_int, [P, I32]),
        "cst_rmsnorm": (ctypes.c_int, [P, I32, I32, I32, P, ctypes.c_float, P, I32, P]),
        "cst_route": (ctypes.c_int, [P, P, I32, I32, P, P, P, I32, P, P, P, P, P]),
        "cst_moe_routed": (ctypes.c_int, [P, P, I32, I32, P, P, I32, U32, P, I32, P]),
        "cst_moe_routed_range": (ctypes.c_int, [P, P, I32, I32, P, P, I32, I32, I32, P, I32, P]),
        "cst_moe_layer": (ctypes.c_int, [P, P, I32, I32, P, P, P, I32, U32, P, P, I32, P, P, P]),
        "cst_grouped_ffn": (ctypes.c_int, [P, P, I32, I32, P, P, P, I32, P]),
        "cst_expert_forward": (ctypes.c_int, [P, I32, P, I32, I32, P, I32, P]),
        "cst_device_error": (ctypes.c_int, [P]),
        "cst_ctx_info": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int64), I32]),
        "cst_last_error": (ctypes.c_char_p, []),
        "cst_shared_combine": (ctypes.c_int, [P, P, I32, I32, P, P, P, I32, P]),
        "cst_dequant_fp8": (ctypes.c_int, [P, P, I32, I32, I32, P, P]),
        "cst_route_noalloc": (ctypes.c_int, [P, I32, I32, I32, P, P, P, I32, I32, I32, I32, I32, F, P, P, P]),
        "cst_combine_rows": (ctypes.c_int, [P, P, ctypes.c_int64, P, I32, I32, P, P, I32, P, I32, P]),
        "cst_profile_enable": (ctypes.c_int, [P, I32]),
        "cst_profile_read": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_float), I32]),
        "cst_abi_version": (I32, []),
        "cst_ipc_alloc": (ctypes.c_int, [ctypes.c_int64, ctypes.POINTER(P), ctypes.POINTER(CstIpcHandle)]),
        "cst_ipc_open": (ctypes.c_int, [ctypes.POINTER(CstIpcHandle), ctypes.POINTER(P)]),
        "cst_ipc_close": (ctypes.c_int, [P]),
        "cst_ipc_free": (ctypes.c_int, [P]),
        "cst_moe_routed_push": (ctypes.c_int, [P, P, I32, P, P, I32, ctypes.POINTER(CstPeerSet), P]),
        "cst_reduce_pushed": (ctypes.c_int, [P, ctypes.POINTER(CstPeerSet), P, I32, P, I32, P]),
        "cst_gather_rows": (ctypes.c_int, [P, ctypes.POINTER(CstPeerSet), P, I32, P]),
        "cst_encode_infer_request": (ctypes.c_int, [ctypes.POINTER(CstInferRequest), P, I64, ctypes.POINTER(I64)]),
        "cst_decode_infer_request": (ctypes.c_int, [P, I64, ctypes.POINTER(CstInferRequest)]),
        "cst_encode_infer_response": (ctypes.c_int, [ctypes.POINTER(CstInferResponse), P, I64, ctypes.POINTER(I64)]),
        "cst_decode_infer_response": (ctypes.c_int, [P, I64, ctypes.POINTER(CstInferResponse)]),
        "cst_serve_infer_request": (ctypes.c_int, [ctypes.POINTER(P), I32, I32, P, I64, P, I64, ctypes.POINTER(I64),
                                                   P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    del F
    return lib


lib = _load()


def last_error() -> str:
    return lib.cst_last_error().decode(errors="replace")


def check(rc: int) -> None:
    if rc != CST_OK:
        raise CstError(rc, last_error())
