"""ctypes binding of liblq.so (include/lq.h). There is no fallback: if the library cannot be loaded,
or a call returns an error code, the caller gets an exception."""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblq.so")

LQ_OK, LQ_E_ARG, LQ_E_SHAPE, LQ_E_ALIGN, LQ_E_UNSUPPORTED, LQ_E_CUDA, LQ_E_DEVICE, LQ_E_SCRATCH = range(8)
F16, BF16, F32 = 0, 1, 2
FAM_AUTO, FAM_QMV, FAM_TC, FAM_TCV, FAM_QMVG, FAM_QMVQ = 0, 1, 2, 3, 4, 5

# every function the header declares, with its argument types (checked by tests on CPU)
_vp, _i, _u32p = ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p


class Cfg(ctypes.Structure):
    _fields_ = [("family", ctypes.c_int), ("p", ctypes.c_int * 7)]


SIGNATURES = {
    "lq_qmm": ([_vp, _u32p, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, ctypes.POINTER(Cfg), _vp], _i),
    "lq_qmm_split": ([_vp, _u32p, _vp, _vp, _i, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_int), _i, _i,
                      _i, _i, _i, _i, ctypes.POINTER(Cfg), _vp], _i),
    "lq_qmm_glu": ([_vp, _u32p, _vp, _vp, _u32p, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, ctypes.POINTER(Cfg), _vp], _i),
    "lq_quantize": ([_vp, _i, _i, _i, _i, _i, _u32p, _vp, _vp, _i, _vp], _i),
    "lq_dequantize": ([_u32p, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp], _i),
    "lq_router_logits": ([_vp, _i, _vp, _i, _vp, _i, _i, _i, _vp], _i),
    "lq_route_topk": ([_vp, _i, _i, _i, _i, _vp, _vp, _vp], _i),
    "lq_moe_group": ([_vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp], _i),
    "lq_moe_gather": ([_vp, _vp, _i, _i, _i, _vp, _vp], _i),
    "lq_moe_experts": ([_vp, _vp, _vp, _vp, _i, _i, _i, _u32p, _vp, _vp, _u32p, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i,
                        _vp, _i, _vp], _i),
    "lq_moe_route": ([_vp, _i, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp], _i),
    "lq_moe_combine": ([_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp], _i),
    "lq_moe_down_combine": ([_vp, _vp, _vp, _vp, _u32p, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp], _i),
    "lq_moe_decode_workspace": ([_i, _i, _i, _i], ctypes.c_size_t),
    "lq_peer_sync_bytes": ([], ctypes.c_size_t),
    "lq_peer_scatter_rows": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, ctypes.POINTER(ctypes.c_void_p), _i, _i,
                              ctypes.POINTER(ctypes.c_void_p), _vp], _i),
    "lq_moe_group_range": ([_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp], _i),
    "lq_peer_gather_cols": ([_vp, _i, _i, _i, _i, _i, ctypes.POINTER(ctypes.c_void_p), _i, _i,
                             ctypes.POINTER(ctypes.c_void_p), _vp], _i),
    "lq_moe_decode": ([_vp, _vp, _i, _i, _i, _i, _u32p, _vp, _vp, _u32p, _vp, _vp, _u32p, _vp, _vp, _i, _i, _i, _i, _i,
                       _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp], _i),
    "lq_add_rms_norm": ([_vp, _vp, _vp, _vp, _vp, _i, _i, ctypes.c_float, _i, _vp], _i),
    "lq_moe_combine_norm": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, ctypes.c_float, _i, _vp], _i),
    "lq_scatter_rows": ([_vp, _vp, _i, _i, _vp, _i, _i, _vp], _i),
    "lq_kv_attend": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, ctypes.c_float, _i, _i, _i, _i, _i, _i, _vp,
                      ctypes.c_size_t, _vp, _vp], _i),
    "lq_kv_attend_workspace": ([_i, _i, _i, _i], ctypes.c_size_t),
    "lq_qmm_dense": ([_vp, _u32p, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, ctypes.c_size_t, ctypes.POINTER(Cfg), _vp],
                     _i),
    "lq_qmm_dense_workspace": ([_i, _i], ctypes.c_size_t),
    "lq_qmm_dense_gather": ([_vp, _u32p, _vp, _vp, ctypes.POINTER(ctypes.c_void_p), _i, _i, _i, _i, _i, _i, _i, _i, _i,
                             _vp, ctypes.c_size_t, ctypes.POINTER(Cfg), _vp], _i),
    "lq_ipc_export": ([_vp, _vp, ctypes.POINTER(ctypes.c_size_t)], _i),
    "lq_ipc_import": ([_vp, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)], _i),
    "lq_ipc_close": ([_vp, ctypes.c_size_t], _i),
    "lq_kv_attend_noalloc": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, ctypes.c_float, _i, _i, _i, _i, _i, _i,
                              _vp, _vp], _i),
    "lq_supported": ([_i, _i, _i, _i, _i, _i, _i], _i),
    "lq_list_configs": ([_i, _i, _i, _i, _i, _i, ctypes.POINTER(Cfg), _i], _i),
    "lq_device_status": ([_i], ctypes.c_uint),
    "lq_last_cuda_error": ([], ctypes.c_char_p),
    "lq_strerror": ([_i], ctypes.c_char_p),
    "lq_version": ([], _i),
}

_lib = None
_lock = threading.Lock()


class LQError(RuntimeError):
    def __init__(self, fn: str, code: int):
        lib = _lib
        msg = lib.lq_strerror(code).decode() if lib else str(code)
        extra = ""
        if code == LQ_E_CUDA and lib:
            extra = ": " + lib.lq_last_cuda_error().decode()
        super().__init__(f"{fn} failed with {msg} ({code}){extra}")
        self.code = code


def lib():
    """The loaded liblq.so (built in-tree by locals_b200.build / __graft_entry__.build())."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(f"liblq.so is missing at {LIB_PATH}: run `python -m locals_b200.build`")
                L = ctypes.CDLL(LIB_PATH)
                for name, (args, res) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.argtypes = args
                    fn.restype = res
                _lib = L
    return _lib


def call(name: str, *args) -> None:
    rc = getattr(lib(), name)(*args)
    if rc != LQ_OK:
        raise LQError(name, rc)


def cfg(family: int = FAM_AUTO, *params: int):
    c = Cfg()
    c.family = family
    for i, v in enumerate(params[:7]):
        c.p[i] = int(v)
    return ctypes.byref(c)


def device_status(clear: bool = True) -> int:
    return int(lib().lq_device_status(1 if clear else 0))
