"""ctypes binding of libefmoe.so (the C ABI in include/efmoe.h).

The library is loaded from the package directory.  There is no fallback: if
it is missing, every op raises ``EfmoeUnavailable``.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libefmoe.so")

EF_OK = 0
STATUS = {
    -1: "EF_ERR_INVALID",
    -2: "EF_ERR_UNSUPPORTED",
    -3: "EF_ERR_CUDA",
    -4: "EF_ERR_WORKSPACE",
    -5: "EF_ERR_TIMEOUT",
    -6: "EF_ERR_SLOT_MISS",
    -7: "EF_ERR_RANGE",
    -8: "EF_ERR_NOT_READY",
    -9: "EF_ERR_IO",
}
EF_DT_BF16, EF_DT_F16, EF_DT_F32 = 0, 1, 2
EF_ROUTER_SOFTMAX, EF_ROUTER_SIGMOID_GROUP = 0, 1
EF_PATH_AUTO, EF_PATH_GEMV, EF_PATH_GEMM, EF_PATH_GEMM_PAIR = 0, 1, 2, 3


class EfmoeUnavailable(RuntimeError):
    pass


class EfmoeError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


class QWeight(ctypes.Structure):
    _fields_ = [("w", ctypes.c_void_p), ("scales", ctypes.c_void_p), ("biases", ctypes.c_void_p)]


class MoECfg(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int),
        ("inter", ctypes.c_int),
        ("n_experts", ctypes.c_int),
        ("top_k", ctypes.c_int),
        ("bits", ctypes.c_int),
        ("group_size", ctypes.c_int),
        ("router_mode", ctypes.c_int),
        ("norm_topk", ctypes.c_int),
        ("n_group", ctypes.c_int),
        ("topk_group", ctypes.c_int),
        ("routed_scaling", ctypes.c_float),
        ("n_shared", ctypes.c_int),
        ("shared_inter", ctypes.c_int),
        ("act_dtype", ctypes.c_int),
        ("gate_dtype", ctypes.c_int),
        ("path", ctypes.c_int),
        ("out_f32", ctypes.c_int),
    ]


class PoolCfg(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("budget", ctypes.c_int), ("headroom", ctypes.c_int),
                ("policy", ctypes.c_int), ("decay", ctypes.c_double)]


class PoolStats(ctypes.Structure):
    _fields_ = [("accesses", ctypes.c_longlong), ("hits", ctypes.c_longlong), ("misses", ctypes.c_longlong),
                ("copies_sync", ctypes.c_longlong), ("copies_prefetch", ctypes.c_longlong),
                ("prefetch_used", ctypes.c_longlong), ("evictions", ctypes.c_longlong),
                ("tokens", ctypes.c_longlong), ("h2d_bytes", ctypes.c_double), ("copy_ms", ctypes.c_double),
                ("host_hits", ctypes.c_longlong), ("host_reads", ctypes.c_longlong),
                ("host_reads_ahead", ctypes.c_longlong), ("host_evictions", ctypes.c_longlong),
                ("read_wait_ms", ctypes.c_double), ("copy_wait_ms", ctypes.c_double),
                ("route_wait_ms", ctypes.c_double), ("host_ms", ctypes.c_double)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


EF_POLICY_FREQ, EF_POLICY_LRU, EF_POLICY_BELADY = 0, 1, 2


class FileArray(ctypes.Structure):
    _fields_ = [("file", ctypes.c_int), ("bf16", ctypes.c_int), ("offset", ctypes.c_longlong),
                ("stride", ctypes.c_longlong)]


class StoreInfo(ctypes.Structure):
    _fields_ = [("blob_bytes", ctypes.c_size_t), ("offsets", ctypes.c_size_t * 10), ("n_layers", ctypes.c_int),
                ("n_readers", ctypes.c_int), ("direct", ctypes.c_int), ("reads", ctypes.c_longlong),
                ("file_bytes", ctypes.c_double)]

class KQWeight(ctypes.Structure):
    _fields_ = [("blocks", ctypes.c_void_p), ("type", ctypes.c_int), ("expert_stride", ctypes.c_longlong)]


_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_QW = QWeight
_QWP = ctypes.POINTER(QWeight)
_CFGP = ctypes.POINTER(MoECfg)

# name -> (restype, argtypes); every function declared in include/efmoe.h
SIGNATURES = {
    "ef_version": (ctypes.c_char_p, []),
    "ef_status_string": (ctypes.c_char_p, [_I]),
    "ef_last_error_message": (ctypes.c_char_p, []),
    "ef_get_device_error": (_I, [_P, ctypes.POINTER(_I)]),
    "ef_trace_enable": (_I, [_I]),
    "ef_trace_read": (_I, [_P, _I]),
    "ef_moe_workspace_size": (_SZ, [_CFGP, _I]),
    "ef_moe_forward": (_I, [_CFGP, _P, _I, _P, _P, _QW, _QW, _QW, _QWP, _QWP, _QWP, _P, _P, _P, _P, _SZ, _P]),
    "ef_moe_forward_noalloc": (_I, [_CFGP, _P, _I, _P, _P, _QW, _QW, _QW, _QWP, _QWP, _QWP, _P, _P, _P, _P]),
    "ef_router_workspace_size": (_SZ, [_CFGP, _I]),
    "ef_router_topk": (_I, [_CFGP, _P, _I, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "ef_permute_workspace_size": (_SZ, [_I, _I, _I, _I]),
    "ef_permute": (_I, [_P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _SZ, _P]),
    "ef_combine": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _I, _P]),
    "ef_experts_workspace_size": (_SZ, [_CFGP, _I]),
    "ef_moe_experts_forward": (_I, [_CFGP, _P, _I, _P, _QW, _QW, _QW, _QWP, _QWP, _QWP, _P, _P, _SZ, _P]),
    "ef_quantized_matmul_workspace_size": (_SZ, [_I, _I, _I]),
    "ef_quantized_matmul": (_I, [_P, _I, _I, _P, _P, _P, _I, _I, _I, _I, _P, _P, _SZ, _P]),
    "ef_dequantize": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _I, _P]),
    "ef_gather_qmm_workspace_size": (_SZ, [_I, _I, _I, _I, _I]),
    "ef_gather_qmm": (_I, [_P, _I, _I, _P, _I, _QW, _I, _I, _I, _I, _I, _P, _P, _SZ, _P]),
    "ef_ep_dispatch_workspace_size": (_SZ, [_CFGP, _I]),
    "ef_ep_dispatch": (_I, [_CFGP, _I, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "ef_ep_combine": (_I, [_CFGP, _P, _P, _P, _I, _I, _P, _P]),
    "ef_ep_group_create": (_I, [_CFGP, _I, _I, _I, _I, _P]),
    "ef_ep_group_handle": (_I, [_P, _P]),
    "ef_ep_group_open": (_I, [_P, _P]),
    "ef_ep_workspace_size": (_SZ, [_P, _I]),
    "ef_ep_forward": (_I, [_P, _P, _I, _P, _P, _QW, _QW, _QW, _QWP, _QWP, _QWP, _P, _I, _P, _P, _P, _SZ, _P]),
    "ef_ep_group_destroy": (_I, [_P]),
    "ef_kquant_moe_workspace_size": (_SZ, [_CFGP, _I]),
    "ef_kquant_moe_forward": (_I, [_CFGP, _P, _I, _P, _P, KQWeight, KQWeight, KQWeight, ctypes.POINTER(KQWeight),
                                   ctypes.POINTER(KQWeight), ctypes.POINTER(KQWeight), _P, _P, _P, _P, _SZ, _P]),
    "ef_policy_create": (_I, [_I, _I, ctypes.c_double, _P]),
    "ef_policy_get": (_I, [_P, ctypes.c_longlong]),
    "ef_policy_put": (None, [_P, ctypes.c_longlong]),
    "ef_policy_trim": (_I, [_P, _P, _I]),
    "ef_policy_size": (_I, [_P]),
    "ef_policy_keys": (_I, [_P, _P, _I]),
    "ef_policy_score": (ctypes.c_double, [_P, ctypes.c_longlong]),
    "ef_policy_destroy": (None, [_P]),
    "ef_policy_end_token": (None, [_P]),
    "ef_policy_set_predictor": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _I]),
    "ef_pool_set_predictor": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _I]),
    "ef_pool_create": (_I, [_CFGP, ctypes.POINTER(PoolCfg), _QWP, _QWP, _QWP, _P]),
    "ef_pool_workspace_size": (_SZ, [_P, _I]),
    "ef_pool_moe_forward": (_I, [_P, _I, _P, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _SZ, _P]),
    "ef_pool_end_token": (_I, [_P]),
    "ef_pool_decode_workspace_size": (_SZ, [_P, _I]),
    "ef_pool_decode_step": (_I, [_P, _P, _I, _P, _P, _I, ctypes.c_float, _P, _SZ, _P]),
    "ef_pool_resident": (_I, [_P, _I, _P, _I, ctypes.POINTER(_I)]),
    "ef_pool_record_routing": (_I, [_P, _I]),
    "ef_pool_routing_trace": (_I, [_P, _P, ctypes.c_longlong, _P, _P, ctypes.c_longlong, _P]),
    "ef_pool_get_stats": (_I, [_P, ctypes.POINTER(PoolStats)]),
    "ef_pool_reset_stats": (_I, [_P]),
    "ef_pool_destroy": (_I, [_P]),
    "ef_kquant_dequantize": (_I, [_I, _P, ctypes.c_longlong, _P, _P]),
    "ef_kquant_matmul_workspace_size": (_SZ, [_I, _I]),
    "ef_kquant_matmul": (_I, [_P, _I, _I, _P, _I, _I, _I, _P, _P, _SZ, _P]),
    "ef_store_open": (_I, [_CFGP, _I, _P, _I, ctypes.POINTER(FileArray), _I, _I, _P]),
    "ef_store_get_info": (_I, [_P, ctypes.POINTER(StoreInfo)]),
    "ef_store_read": (_I, [_P, _I, _P, _P, _P]),
    "ef_store_close": (_I, [_P]),
    "ef_pool_create_from_store": (_I, [_CFGP, ctypes.POINTER(PoolCfg), _P, _I, _P]),
}

_lib = None


def lib():
    """Load libefmoe.so (raises EfmoeUnavailable when it is not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise EfmoeUnavailable(f"{LIB_PATH} is not built (run python -m expertflow_b200.build)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != EF_OK:
        msg = lib().ef_last_error_message()
        raise EfmoeError(status, msg.decode() if msg else "")


def version() -> str:
    return lib().ef_version().decode()


class TraceRec(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("ms", ctypes.c_float)]


def trace_enable(on: bool) -> None:
    lib().ef_trace_enable(int(on))


def trace_read(max_recs: int = 1 << 16) -> list:
    """[(kernel name, milliseconds)] for every launch since the last read."""
    buf = (TraceRec * max_recs)()
    n = lib().ef_trace_read(ctypes.cast(buf, ctypes.c_void_p), max_recs)
    return [(buf[i].name.decode(), float(buf[i].ms)) for i in range(n)]
