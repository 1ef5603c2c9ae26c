"""ctypes binding of the C ABI in ``include/qv_gpu.h`` (the library ``libquiver_b200.so``).

This is the Python side of the drop-in boundary: every call goes straight to the CUDA library.
There is no CPU fallback; importing this module fails loudly when the library cannot be loaded.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# QUIVER_B200_LIB selects another build of the library (e.g. an instrumented one).
LIB_PATH = os.environ.get("QUIVER_B200_LIB") or os.path.join(HERE, "libquiver_b200.so")

QV_OK, QV_ERR_INVALID, QV_ERR_CUDA, QV_ERR_OOM, QV_ERR_IO, QV_ERR_STATE, QV_ERR_UNSUPPORTED, \
    QV_ERR_DEVICE = range(8)
QV_FILTER_LABEL_SET, QV_FILTER_LABEL_BITMAP, QV_FILTER_POSITION_BITMAP = 1, 2, 3
METRIC_CODES = {"l2": 0, "euclidean": 0, "ip": 1, "inner_product": 1, "dot": 1, "cosine": 2,
                "cos": 2, "angular": 2}
METRIC_NAMES = {0: "l2", 1: "ip", 2: "cosine"}
STORAGE_CODES = {"float32": 0, "sq8": 1}
STORAGE_NAMES = {0: "float32", 1: "sq8"}


class qv_filter(C.Structure):
    _fields_ = [("kind", C.c_uint32), ("data", C.c_void_p), ("size", C.c_uint64)]


class qv_ivfpq_params(C.Structure):
    _fields_ = [("dim", C.c_size_t), ("metric", C.c_uint32), ("nlist", C.c_size_t),
                ("m", C.c_size_t), ("train_iterations", C.c_size_t), ("store_vectors", C.c_int),
                ("seed", C.c_uint64)]


class qv_search_stats(C.Structure):
    _fields_ = [("kernel_launches", C.c_uint64), ("rescanned_queries", C.c_uint64),
                ("dominant_kernel_ms", C.c_double), ("dominant_kernel_work", C.c_double),
                ("dominant_work_is_bytes", C.c_uint32), ("dominant_kernel", C.c_char * 64)]


# (name, restype, argtypes); every function returns qv_status unless stated.
_vp, _sz, _u32, _u64, _int = C.c_void_p, C.c_size_t, C.c_uint32, C.c_uint64, C.c_int
_PP = C.POINTER(C.c_void_p)
_SIGNATURES = {
    "qv_last_error": (C.c_char_p, []),
    "qv_version": (C.c_char_p, []),
    "qv_device_count": (_int, [C.POINTER(_int)]),
    "qv_last_search_stats": (_int, [C.POINTER(qv_search_stats)]),
    "qv_set_timing": (_int, [_int]),
    "qv_device_free": (_int, [_int, _vp]),
    "qv_flat_create": (_int, [_int, _sz, _u32, _PP]),
    "qv_flat_destroy": (_int, [_vp]),
    "qv_flat_add": (_int, [_vp, _vp, _sz, _vp]),
    "qv_flat_reserve": (_int, [_vp, _sz]),
    "qv_flat_add_device": (_int, [_vp, _vp, _sz, _vp, _vp]),
    "qv_flat_search": (_int, [_vp, _vp, _sz, _sz, _vp, _vp, _vp]),
    "qv_flat_search_device": (_int, [_vp, _vp, _sz, _sz, _vp, _vp, _vp, _vp, _vp]),
    "qv_flat_set_row_offset": (_int, [_vp, _u64]),
    "qv_flat_search_device_noalloc": (_int, [_vp, _vp, _sz, _sz, _vp, _vp, _vp, _vp, _vp]),
    "qv_flat_noalloc_max_bytes": (_sz, []),
    "qv_flat_info": (_int, [_vp, C.POINTER(_sz), C.POINTER(_sz), C.POINTER(_u32)]),
    "qv_flat_rows": (_int, [_vp, _sz, _sz, _vp, _vp]),
    "qv_flat_save": (_int, [_vp, C.c_char_p]),
    "qv_flat_load": (_int, [_int, C.c_char_p, _int, _PP]),
    "qv_flat_filter_bitmap": (_int, [_vp, _vp, _PP]),
    "qv_ivfpq_create": (_int, [_int, C.POINTER(qv_ivfpq_params), _PP]),
    "qv_ivfpq_destroy": (_int, [_vp]),
    "qv_ivfpq_train": (_int, [_vp, _vp, _sz]),
    "qv_ivfpq_set_trained": (_int, [_vp, _vp, _vp]),
    "qv_ivfpq_is_trained": (_int, [_vp, C.POINTER(_int)]),
    "qv_ivfpq_add": (_int, [_vp, _vp, _sz, _vp]),
    "qv_ivfpq_encode": (_int, [_vp, _vp, _sz, _vp, _vp]),
    "qv_ivfpq_search": (_int, [_vp, _vp, _sz, _sz, _sz, _sz, _vp, _vp, _vp]),
    "qv_ivfpq_search_device": (_int, [_vp, _vp, _sz, _sz, _sz, _sz, _vp, _vp, _vp, _vp]),
    "qv_ivfpq_candidates_device": (_int, [_vp, _vp, _sz, _sz, _sz, _vp, _vp, _vp, _vp, _vp]),
    "qv_ivfpq_refine_device": (_int, [_vp, _vp, _sz, _sz, _vp, _vp, _vp]),
    "qv_ivfpq_filter_bitmap": (_int, [_vp, _vp, _PP]),
    "qv_ivfpq_info": (_int, [_vp, C.POINTER(qv_ivfpq_params), C.POINTER(_sz), C.POINTER(_sz)]),
    "qv_ivfpq_list_sizes": (_int, [_vp, _vp]),
    "qv_ivfpq_labels": (_int, [_vp, _vp]),
    "qv_ivfpq_save": (_int, [_vp, C.c_char_p]),
    "qv_ivfpq_load": (_int, [_int, C.c_char_p, _int, _PP]),
    "qv_ivfpq_load_shard": (_int, [_int, C.c_char_p, _int, _u64, _u64, _PP]),
    "qv_ivfpq_set_list_base": (_int, [_vp, _vp]),
    "qv_hnsw_store_create": (_int, [_int, _sz, _u32, _u32, _PP]),
    "qv_hnsw_store_destroy": (_int, [_vp]),
    "qv_hnsw_store_train": (_int, [_vp, _vp, _sz]),
    "qv_hnsw_store_is_trained": (_int, [_vp, C.POINTER(_int)]),
    "qv_hnsw_store_add": (_int, [_vp, _vp, _sz, _vp]),
    "qv_hnsw_store_remove": (_int, [_vp, _u64, C.POINTER(_int)]),
    "qv_hnsw_store_info": (_int, [_vp, C.POINTER(_sz), C.POINTER(_sz), C.POINTER(_sz),
                                  C.POINTER(_u32), C.POINTER(_u32)]),
    "qv_hnsw_store_vector": (_int, [_vp, _u64, _vp]),
    "qv_hnsw_store_codes": (_int, [_vp, _sz, _sz, _vp]),
    "qv_hnsw_store_sq8_params": (_int, [_vp, _vp, _vp]),
    "qv_hnsw_store_search": (_int, [_vp, _vp, _sz, _sz, _vp, _vp, _vp]),
    "qv_hnsw_store_search_device": (_int, [_vp, _vp, _sz, _sz, _vp, _vp, _vp, _vp, _vp]),
    "qv_merge_topk_device": (_int, [_int, _sz, _sz, _sz, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "qv_select_topk_device": (_int, [_int, _sz, _sz, _sz, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
}
EXPORTED = tuple(_SIGNATURES)

_lib = None
_lock = threading.Lock()


def _load():
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            try:
                from . import build as _build
                _build.build()
            except Exception as e:  # the CUDA path is the product: no fallback
                raise ImportError(f"quiver_b200: {LIB_PATH} is missing and could not be built "
                                  f"({e}); run `python -m quiver_b200.build`") from e
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _lib = lib
        return lib


def lib():
    return _load()


class QuiverError(ValueError):
    """Raised for failures the reference reports as quiver::Error (surfaced as ValueError)."""


def check(status: int) -> None:
    if status == QV_OK:
        return
    msg = lib().qv_last_error().decode(errors="replace")
    if status in (QV_ERR_INVALID, QV_ERR_IO, QV_ERR_STATE):
        raise QuiverError(msg)
    if status == QV_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if status == QV_ERR_OOM:
        raise MemoryError(msg)
    raise RuntimeError(f"quiver_b200 CUDA failure ({status}): {msg}")


def ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def last_search_stats() -> dict:
    s = qv_search_stats()
    check(lib().qv_last_search_stats(C.byref(s)))
    return {"kernel_launches": int(s.kernel_launches), "rescanned_queries": int(s.rescanned_queries),
            "dominant_kernel_ms": float(s.dominant_kernel_ms),
            "dominant_kernel_work": float(s.dominant_kernel_work),
            "dominant_work_is_bytes": bool(s.dominant_work_is_bytes),
            "dominant_kernel": s.dominant_kernel.decode(errors="replace")}


def set_timing(enable: bool) -> None:
    check(lib().qv_set_timing(int(bool(enable))))


def device_count() -> int:
    n = C.c_int(0)
    check(lib().qv_device_count(C.byref(n)))
    return int(n.value)


def make_filter(allowed: np.ndarray | None):
    """qv_filter for a uint64 array of allowed labels, choosing a dense label bitmap or a label set
    with the reference binding's rule (python/quiver_ext.cc:40-51). Returns (struct, keepalive)."""
    if allowed is None:
        return None, None
    a = np.ascontiguousarray(allowed, dtype=np.uint64).reshape(-1)
    n = a.size
    max_label = int(a.max()) if n else 0
    if max_label < (1 << 32) and max_label // 64 <= 16 * n + 1024:
        universe = max_label + 1 if n else 0
        words = np.zeros(max(1, (universe + 63) // 64), dtype=np.uint64)
        if n:
            np.bitwise_or.at(words, (a >> np.uint64(6)).astype(np.int64),
                             np.left_shift(np.uint64(1), a & np.uint64(63)))
        f = qv_filter(QV_FILTER_LABEL_BITMAP, words.ctypes.data, universe)
        return f, words
    f = qv_filter(QV_FILTER_LABEL_SET, a.ctypes.data, n)
    return f, a
