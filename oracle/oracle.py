"""Test infrastructure only: ctypes access to the two CPU checkers built by ``oracle/Makefile``.

* :class:`Oracle` wraps ``_build/libqv_oracle.so``, our plain-C restatement of the reference hot
  path (``qv_oracle.c``; every function there cites the reference file:line it follows).
* :class:`Reference` wraps ``_ref/libquiver_ref.so``: the reference Quiver library compiled from
  its own sources plus the ``ref_shim.cc`` C shim. It exists only where the reference sources were
  present at build time.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs use this module,
always as the checker or the timed CPU baseline, never as part of the product path.
"""
from __future__ import annotations

import ctypes as C
import os
import struct
import subprocess
import zlib
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libqv_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libquiver_ref.so")

METRICS = {"l2": 0, "ip": 1, "cosine": 2}
ORDER_SCALAR, ORDER_AVX2 = 0, 2
INVALID = np.uint64(2**64 - 1)

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_sz = C.c_size_t


def build(ref_root: Optional[str] = None) -> None:
    """Builds the C restatement, and the reference library when its sources are present."""
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)
    # The reference checkout: QUIVER_REFERENCE when set, else a "reference" directory beside
    # this repository.
    ref_root = ref_root or os.environ.get(
        "QUIVER_REFERENCE", os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
    if os.path.isdir(os.path.join(ref_root, "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref_root}"], check=True)


def metric_code(metric) -> int:
    return METRICS[metric] if isinstance(metric, str) else int(metric)


def bitmap_from_labels(allowed) -> tuple[Optional[np.ndarray], int]:
    """Dense BitsetFilter words for a set of allowed labels (include/quiver/filter.h:39-71)."""
    if allowed is None:
        return None, 0
    a = np.asarray(list(allowed) if not isinstance(allowed, np.ndarray) else allowed,
                   dtype=np.uint64).reshape(-1)
    universe = int(a.max()) + 1 if a.size else 0
    words = np.zeros(max(1, (universe + 63) // 64), dtype=np.uint64)
    if a.size:
        np.bitwise_or.at(words, (a >> np.uint64(6)).astype(np.int64),
                         np.left_shift(np.uint64(1), a & np.uint64(63)))
    return words, universe


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


class Oracle:
    """Our C restatement of the reference hot path."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        L = self.lib = C.CDLL(path)
        L.qvo_dot.restype = C.c_float
        L.qvo_dot.argtypes = [_f32p, _f32p, _sz, C.c_int]
        L.qvo_l2sqr.restype = C.c_float
        L.qvo_l2sqr.argtypes = [_f32p, _f32p, _sz, C.c_int]
        L.qvo_normalize_rows.argtypes = [_f32p, _sz, _sz, C.c_int]
        L.qvo_flat_search.argtypes = [_f32p, _u64p, _sz, _sz, C.c_int, C.c_int, _f32p, _sz, _sz,
                                      C.c_void_p, C.c_uint64, _u64p, _f32p]
        L.qvo_coarse_assign.argtypes = [_f32p, _sz, _sz, _f32p, _sz, C.c_int, _u32p]
        L.qvo_pq_encode.argtypes = [_f32p, _sz, _sz, _f32p, _sz, _u8p]
        L.qvo_ivf_encode.argtypes = [_f32p, _sz, _f32p, _sz, _sz, C.c_int, C.c_int, _f32p, _sz,
                                     _u32p, _u8p]
        L.qvo_precompute.argtypes = [_f32p, _sz, _f32p, _sz, _sz, _f32p]
        L.qvo_ip_table.argtypes = [_f32p, _sz, _sz, _f32p, _f32p]
        L.qvo_l2_table.argtypes = [_f32p, _sz, _sz, _f32p, _f32p]
        L.qvo_ivf_search.argtypes = [C.c_void_p, _f32p, _sz, _sz, _sz, _sz, C.c_void_p,
                                     C.c_uint64, C.c_int, _u64p, _f32p]
        for fn in (L.qvo_l2sqr_sq8, L.qvo_dot_sq8):
            fn.restype = C.c_float
            fn.argtypes = [_f32p, _u8p, _f32p, _f32p, _sz]
        L.qvo_sq8_train.argtypes = [_f32p, _sz, _sz, _f32p, _f32p]
        L.qvo_sq8_encode.argtypes = [_f32p, _f32p, _sz, _f32p, _sz, _u8p]
        L.qvo_exact_scan.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, _sz, C.c_int,
                                     _u32p, _sz, _f32p, _sz, _sz, _u32p, _f32p]

    def dot(self, a, b, order=ORDER_AVX2) -> float:
        a, b = _f32(a), _f32(b)
        return float(self.lib.qvo_dot(a, b, a.size, order))

    def l2sqr(self, a, b, order=ORDER_AVX2) -> float:
        a, b = _f32(a), _f32(b)
        return float(self.lib.qvo_l2sqr(a, b, a.size, order))

    def normalize_rows(self, x, order=ORDER_AVX2) -> np.ndarray:
        x = _f32(x).copy()
        self.lib.qvo_normalize_rows(x, x.shape[0], x.shape[1], order)
        return x

    def flat_search(self, stored, labels, metric, queries, k, allowed=None, order=ORDER_AVX2):
        """``stored`` holds rows as the index stores them (normalized already for cosine)."""
        stored, queries = _f32(stored), _f32(queries)
        labels = np.ascontiguousarray(labels, dtype=np.uint64)
        nq = queries.shape[0]
        out_l = np.empty((nq, k), np.uint64)
        out_d = np.empty((nq, k), np.float32)
        bm, universe = bitmap_from_labels(allowed)
        rc = self.lib.qvo_flat_search(stored, labels, stored.shape[0], stored.shape[1],
                                      metric_code(metric), order, queries, nq, k,
                                      None if bm is None else bm.ctypes.data, universe, out_l, out_d)
        assert rc == 0
        return out_l, out_d

    def l2sqr_sq8(self, q, code, vmin, vscale) -> float:
        q, code = _f32(q), np.ascontiguousarray(code, dtype=np.uint8)
        return float(self.lib.qvo_l2sqr_sq8(q, code, _f32(vmin), _f32(vscale), q.size))

    def dot_sq8(self, q, code, vmin, vscale) -> float:
        q, code = _f32(q), np.ascontiguousarray(code, dtype=np.uint8)
        return float(self.lib.qvo_dot_sq8(q, code, _f32(vmin), _f32(vscale), q.size))

    def sq8_train(self, x):
        x = _f32(x)
        vmin = np.empty(x.shape[1], np.float32)
        vscale = np.empty(x.shape[1], np.float32)
        assert self.lib.qvo_sq8_train(x, x.shape[0], x.shape[1], vmin, vscale) == 0
        return vmin, vscale

    def sq8_encode(self, vmin, vscale, x) -> np.ndarray:
        x = _f32(x)
        out = np.empty(x.shape, np.uint8)
        self.lib.qvo_sq8_encode(_f32(vmin), _f32(vscale), x.shape[1], x, x.shape[0], out)
        return out

    def exact_scan(self, metric, queries, k, ids, rows=None, codes=None, vmin=None, vscale=None):
        """HNSW's filtered exact scan over the listed node ids, on float32 rows or SQ8 codes
        (stored as the index holds them: prepared for cosine). Returns (node ids, distances)."""
        queries = _f32(queries)
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        nq = queries.shape[0]
        out_i = np.empty((nq, k), np.uint32)
        out_d = np.empty((nq, k), np.float32)
        if codes is None:
            data, storage = _f32(rows), 0
            vmin = vscale = None
            ptrs = (None, None)
        else:
            data, storage = np.ascontiguousarray(codes, dtype=np.uint8), 1
            vmin, vscale = _f32(vmin), _f32(vscale)
            ptrs = (vmin.ctypes.data, vscale.ctypes.data)
        rc = self.lib.qvo_exact_scan(storage, data.ctypes.data, ptrs[0], ptrs[1], data.shape[1],
                                     metric_code(metric), ids, ids.size, queries, nq, k, out_i,
                                     out_d)
        assert rc == 0
        return out_i, out_d

    def coarse_assign(self, cents, x, by_ip=False) -> np.ndarray:
        cents, x = _f32(cents), _f32(x)
        out = np.empty(x.shape[0], np.uint32)
        self.lib.qvo_coarse_assign(cents, cents.shape[0], cents.shape[1], x, x.shape[0],
                                   int(by_ip), out)
        return out

    def pq_encode(self, codebooks, m, x) -> np.ndarray:
        codebooks, x = _f32(codebooks), _f32(x)
        out = np.empty((x.shape[0], m), np.uint8)
        self.lib.qvo_pq_encode(codebooks, m, x.shape[1] // m, x, x.shape[0], out)
        return out

    def ivf_encode(self, cents, codebooks, m, metric, x, order=ORDER_AVX2):
        cents, codebooks, x = _f32(cents), _f32(codebooks), _f32(x)
        n, d = x.shape
        assign = np.empty(n, np.uint32)
        codes = np.empty((n, m), np.uint8)
        self.lib.qvo_ivf_encode(cents, cents.shape[0], codebooks, m, d, metric_code(metric), order,
                                x, n, assign, codes)
        return assign, codes

    def precompute(self, cents, codebooks, m) -> np.ndarray:
        cents, codebooks = _f32(cents), _f32(codebooks)
        nlist, d = cents.shape
        out = np.empty((nlist, m, 256), np.float32)
        self.lib.qvo_precompute(cents, nlist, codebooks, m, d // m, out)
        return out

    def ip_table(self, codebooks, m, q) -> np.ndarray:
        q = _f32(q)
        out = np.empty((m, 256), np.float32)
        self.lib.qvo_ip_table(_f32(codebooks), m, q.size // m, q, out)
        return out

    def l2_table(self, codebooks, m, q) -> np.ndarray:
        q = _f32(q)
        out = np.empty((m, 256), np.float32)
        self.lib.qvo_l2_table(_f32(codebooks), m, q.size // m, q, out)
        return out

    def ivf_search(self, qvr: "QvrIvf", queries, k, nprobe, refine_factor=0, allowed=None,
                   order=ORDER_AVX2):
        queries = _f32(queries)
        nq = queries.shape[0]
        pre = None
        if qvr.metric == 0 and qvr.nlist * qvr.m * 256 * 4 <= (256 << 20):
            pre = self.precompute(qvr.centroids, qvr.codebooks, qvr.m)
        keep = [qvr.centroids, qvr.codebooks, qvr.offsets, qvr.codes, qvr.labels, qvr.vectors, pre]

        class _Ix(C.Structure):
            _fields_ = [("dim", _sz), ("nlist", _sz), ("m", _sz), ("metric", C.c_int),
                        ("centroids", C.c_void_p), ("codebooks", C.c_void_p),
                        ("offsets", C.c_void_p), ("codes", C.c_void_p), ("labels", C.c_void_p),
                        ("vectors", C.c_void_p), ("precomputed", C.c_void_p)]

        def ptr(a):
            return None if a is None else a.ctypes.data

        ix = _Ix(qvr.dim, qvr.nlist, qvr.m, qvr.metric, ptr(keep[0]), ptr(keep[1]), ptr(keep[2]),
                 ptr(keep[3]), ptr(keep[4]), ptr(keep[5]), ptr(keep[6]))
        out_l = np.empty((nq, k), np.uint64)
        out_d = np.empty((nq, k), np.float32)
        bm, universe = bitmap_from_labels(allowed)
        rc = self.lib.qvo_ivf_search(C.addressof(ix), queries, nq, k, nprobe, refine_factor,
                                     None if bm is None else bm.ctypes.data, universe, order,
                                     out_l, out_d)
        assert rc == 0
        del keep
        return out_l, out_d


class ReferenceError_(RuntimeError):
    pass


class Reference:
    """The reference library itself (compiled from its own sources) through ref_shim.cc."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = self.lib = C.CDLL(path)
        L.qvref_last_error.restype = C.c_char_p
        L.qvref_simd_isa.restype = C.c_char_p
        L.qvref_hardware_threads.restype = C.c_uint
        L.qvref_dot.restype = C.c_float
        L.qvref_dot.argtypes = [_f32p, _f32p, _sz]
        L.qvref_l2sqr.restype = C.c_float
        L.qvref_l2sqr.argtypes = [_f32p, _f32p, _sz]
        L.qvref_normalize_rows.argtypes = [_f32p, _sz, _sz]
        vp = C.POINTER(C.c_void_p)
        L.qvref_flat_new.argtypes = [_sz, C.c_uint32, vp]
        L.qvref_flat_free.argtypes = [C.c_void_p]
        L.qvref_flat_add.argtypes = [C.c_void_p, _f32p, _sz, C.c_void_p]
        L.qvref_flat_search.argtypes = [C.c_void_p, _f32p, _sz, _sz, C.c_void_p, _sz, C.c_int,
                                        C.c_int, _u64p, _f32p]
        L.qvref_flat_vectors.argtypes = [C.c_void_p, _f32p]
        L.qvref_flat_save.argtypes = [C.c_void_p, C.c_char_p]
        L.qvref_ivf_new.argtypes = [_sz, C.c_uint32, _sz, _sz, C.c_int, _sz, C.c_uint64, vp]
        L.qvref_ivf_free.argtypes = [C.c_void_p]
        L.qvref_ivf_train.argtypes = [C.c_void_p, _f32p, _sz, C.c_int]
        L.qvref_ivf_add.argtypes = [C.c_void_p, _f32p, _sz, C.c_void_p, C.c_int]
        L.qvref_ivf_save.argtypes = [C.c_void_p, C.c_char_p]
        L.qvref_ivf_load.argtypes = [C.c_char_p, vp]
        L.qvref_ivf_size.restype = _sz
        L.qvref_ivf_size.argtypes = [C.c_void_p]
        L.qvref_ivf_search.argtypes = [C.c_void_p, _f32p, _sz, _sz, _sz, _sz, C.c_void_p, _sz,
                                       C.c_int, C.c_int, _u64p, _f32p]
        L.qvref_nearest_batch.argtypes = [_f32p, _sz, _sz, _f32p, _sz, C.c_int, _u32p]
        L.qvref_pq_encode.argtypes = [_f32p, _sz, _sz, _f32p, _sz, _u8p]
        L.qvref_pq_tables.argtypes = [_f32p, _sz, _sz, _f32p, _f32p, _f32p]
        for fn in (L.qvref_l2sqr_sq8, L.qvref_dot_sq8):
            fn.restype = C.c_float
            fn.argtypes = [_f32p, _u8p, _f32p, _f32p, _sz]
        L.qvref_sq8_train.argtypes = [_f32p, _sz, _sz, _f32p, _f32p]
        L.qvref_sq8_encode.argtypes = [_f32p, _f32p, _sz, _f32p, _sz, _u8p]
        L.qvref_hnsw_new.argtypes = [_sz, C.c_uint32, C.c_uint32, _sz, _sz, C.c_uint64, vp]
        L.qvref_hnsw_free.argtypes = [C.c_void_p]
        L.qvref_hnsw_train.argtypes = [C.c_void_p, _f32p, _sz]
        L.qvref_hnsw_add.argtypes = [C.c_void_p, _f32p, _sz, C.c_void_p, C.c_int]
        L.qvref_hnsw_remove.argtypes = [C.c_void_p, C.c_uint64]
        L.qvref_hnsw_vector.argtypes = [C.c_void_p, C.c_uint64, _f32p]
        L.qvref_hnsw_search.argtypes = [C.c_void_p, _f32p, _sz, _sz, _sz, C.c_void_p, _sz,
                                        C.c_int, C.c_double, C.c_int, _u64p, _f32p]

    def _check(self, rc: int) -> None:
        if rc != 0:
            raise ReferenceError_(self.lib.qvref_last_error().decode())

    @property
    def isa(self) -> str:
        return self.lib.qvref_simd_isa().decode()

    @property
    def threads(self) -> int:
        return int(self.lib.qvref_hardware_threads())

    def dot(self, a, b) -> float:
        a, b = _f32(a), _f32(b)
        return float(self.lib.qvref_dot(a, b, a.size))

    def l2sqr(self, a, b) -> float:
        a, b = _f32(a), _f32(b)
        return float(self.lib.qvref_l2sqr(a, b, a.size))

    def normalize_rows(self, x) -> np.ndarray:
        x = _f32(x).copy()
        self.lib.qvref_normalize_rows(x, x.shape[0], x.shape[1])
        return x

    def nearest_batch(self, cents, x, by_ip=False) -> np.ndarray:
        cents, x = _f32(cents), _f32(x)
        out = np.empty(x.shape[0], np.uint32)
        self._check(self.lib.qvref_nearest_batch(cents, cents.shape[0], cents.shape[1], x,
                                                 x.shape[0], int(by_ip), out))
        return out

    def pq_encode(self, codebooks, m, x) -> np.ndarray:
        codebooks, x = _f32(codebooks), _f32(x)
        out = np.empty((x.shape[0], m), np.uint8)
        self._check(self.lib.qvref_pq_encode(codebooks, x.shape[1], m, x, x.shape[0], out))
        return out

    def pq_tables(self, codebooks, m, q):
        q = _f32(q)
        ip = np.empty((m, 256), np.float32)
        l2 = np.empty((m, 256), np.float32)
        self._check(self.lib.qvref_pq_tables(_f32(codebooks), q.size, m, q, ip, l2))
        return ip, l2

    def l2sqr_sq8(self, q, code, vmin, vscale) -> float:
        q, code = _f32(q), np.ascontiguousarray(code, dtype=np.uint8)
        return float(self.lib.qvref_l2sqr_sq8(q, code, _f32(vmin), _f32(vscale), q.size))

    def dot_sq8(self, q, code, vmin, vscale) -> float:
        q, code = _f32(q), np.ascontiguousarray(code, dtype=np.uint8)
        return float(self.lib.qvref_dot_sq8(q, code, _f32(vmin), _f32(vscale), q.size))

    def sq8_train(self, x):
        x = _f32(x)
        vmin = np.empty(x.shape[1], np.float32)
        vscale = np.empty(x.shape[1], np.float32)
        self._check(self.lib.qvref_sq8_train(x, x.shape[0], x.shape[1], vmin, vscale))
        return vmin, vscale

    def sq8_encode(self, vmin, vscale, x) -> np.ndarray:
        x = _f32(x)
        out = np.empty(x.shape, np.uint8)
        self._check(self.lib.qvref_sq8_encode(_f32(vmin), _f32(vscale), x.shape[1], x,
                                              x.shape[0], out))
        return out

    def hnsw(self, dim, metric, storage="float32", M=16, ef_construction=200, seed=0x5eed):
        return RefHnsw(self, dim, metric, storage, M, ef_construction, seed)

    def flat(self, dim, metric):
        return RefFlat(self, dim, metric)

    def ivf(self, dim, metric, nlist, m, store_vectors=False, train_iterations=20, seed=1234):
        return RefIvf(self, dim, metric, nlist, m, store_vectors, train_iterations, seed)

    def ivf_load(self, path):
        h = C.c_void_p()
        self._check(self.lib.qvref_ivf_load(str(path).encode(), C.byref(h)))
        return RefIvf(self, handle=h)


def _label_args(labels, n):
    if labels is None:
        return None, None
    la = np.ascontiguousarray(labels, dtype=np.uint64)
    assert la.shape[0] == n
    return la, la.ctypes.data


def _filter_args(allowed):
    if allowed is None:
        return None, None, 0, 0
    a = np.ascontiguousarray(np.asarray(list(allowed) if not isinstance(allowed, np.ndarray)
                                        else allowed, dtype=np.uint64).reshape(-1))
    return a, (a.ctypes.data if a.size else None), a.size, 1


class RefFlat:
    def __init__(self, ref: Reference, dim: int, metric):
        self.ref, self.dim = ref, dim
        self.h = C.c_void_p()
        ref._check(ref.lib.qvref_flat_new(dim, metric_code(metric), C.byref(self.h)))
        self.n = 0

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.qvref_flat_free(self.h)
            self.h = None

    def add(self, x, labels=None):
        x = _f32(x)
        la, lp = _label_args(labels, x.shape[0])
        self.ref._check(self.ref.lib.qvref_flat_add(self.h, x, x.shape[0], lp))
        self.n += x.shape[0]

    def stored(self) -> np.ndarray:
        out = np.empty((self.n, self.dim), np.float32)
        self.ref._check(self.ref.lib.qvref_flat_vectors(self.h, out))
        return out

    def search(self, q, k, allowed=None, threads=0):
        q = _f32(q)
        nq = q.shape[0]
        out_l = np.empty((nq, k), np.uint64)
        out_d = np.empty((nq, k), np.float32)
        a, ap, na, has = _filter_args(allowed)
        self.ref._check(self.ref.lib.qvref_flat_search(self.h, q, nq, k, ap, na, has, threads,
                                                       out_l, out_d))
        return out_l, out_d

    def save(self, path):
        self.ref._check(self.ref.lib.qvref_flat_save(self.h, str(path).encode()))


class RefHnsw:
    """The reference HnswIndex; used for its filtered exact scan (exact_scan_threshold)."""

    def __init__(self, ref: Reference, dim, metric, storage, M, ef_construction, seed):
        self.ref, self.dim = ref, dim
        self.h = C.c_void_p()
        st = {"float32": 0, "sq8": 1}[storage]
        ref._check(ref.lib.qvref_hnsw_new(dim, metric_code(metric), st, M, ef_construction, seed,
                                          C.byref(self.h)))

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.qvref_hnsw_free(self.h)
            self.h = None

    def train(self, x):
        x = _f32(x)
        self.ref._check(self.ref.lib.qvref_hnsw_train(self.h, x, x.shape[0]))

    def add(self, x, labels=None, threads=0):
        x = _f32(x)
        la, lp = _label_args(labels, x.shape[0])
        self.ref._check(self.ref.lib.qvref_hnsw_add(self.h, x, x.shape[0], lp, threads))

    def remove(self, label) -> bool:
        return bool(self.ref.lib.qvref_hnsw_remove(self.h, int(label)))

    def vector(self, label) -> np.ndarray:
        out = np.empty(self.dim, np.float32)
        self.ref._check(self.ref.lib.qvref_hnsw_vector(self.h, int(label), out))
        return out

    def search(self, q, k, allowed=None, ef=64, exact_scan_threshold=0.02, threads=0):
        q = _f32(q)
        nq = q.shape[0]
        out_l = np.empty((nq, k), np.uint64)
        out_d = np.empty((nq, k), np.float32)
        a, ap, na, has = _filter_args(allowed)
        self.ref._check(self.ref.lib.qvref_hnsw_search(self.h, q, nq, k, ef, ap, na, has,
                                                       exact_scan_threshold, threads, out_l,
                                                       out_d))
        return out_l, out_d


class RefIvf:
    def __init__(self, ref: Reference, dim=0, metric=0, nlist=0, m=0, store_vectors=False,
                 train_iterations=20, seed=1234, handle=None):
        self.ref = ref
        if handle is not None:
            self.h = handle
        else:
            self.h = C.c_void_p()
            ref._check(ref.lib.qvref_ivf_new(dim, metric_code(metric), nlist, m, int(store_vectors),
                                             train_iterations, seed, C.byref(self.h)))

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.qvref_ivf_free(self.h)
            self.h = None

    def __len__(self):
        return int(self.ref.lib.qvref_ivf_size(self.h))

    def train(self, x, threads=0):
        x = _f32(x)
        self.ref._check(self.ref.lib.qvref_ivf_train(self.h, x, x.shape[0], threads))

    def add(self, x, labels=None, threads=0):
        x = _f32(x)
        la, lp = _label_args(labels, x.shape[0])
        self.ref._check(self.ref.lib.qvref_ivf_add(self.h, x, x.shape[0], lp, threads))

    def save(self, path):
        self.ref._check(self.ref.lib.qvref_ivf_save(self.h, str(path).encode()))

    def search(self, q, k, nprobe, refine_factor=0, allowed=None, threads=0):
        q = _f32(q)
        nq = q.shape[0]
        out_l = np.empty((nq, k), np.uint64)
        out_d = np.empty((nq, k), np.float32)
        a, ap, na, has = _filter_args(allowed)
        self.ref._check(self.ref.lib.qvref_ivf_search(self.h, q, nq, k, nprobe, refine_factor, ap,
                                                      na, has, threads, out_l, out_d))
        return out_l, out_d


# ---- .qvr reader (test side): restates src/internal/file_format.cc:200-287 -------------------------

def _crc32c(data: bytes) -> int:
    """CRC-32C (Castagnoli, reflected polynomial 0x82F63B78), bitwise; slow but only for tests."""
    table = _crc32c.table
    if table is None:
        table = []
        for i in range(256):
            c = i
            for _ in range(8):
                c = (c >> 1) ^ 0x82F63B78 if c & 1 else c >> 1
            table.append(c)
        _crc32c.table = table = np.array(table, dtype=np.uint32)
    crc = 0xFFFFFFFF
    for b in data:
        crc = int(table[(crc ^ b) & 0xFF]) ^ (crc >> 8)
    return crc ^ 0xFFFFFFFF


_crc32c.table = None


class QvrIvf:
    """Sections of an IVF-PQ ``.qvr`` (src/ivfpq_index.cc:24-43, :465-505)."""

    def __init__(self, path: str, verify_header: bool = True):
        raw = open(path, "rb").read()
        assert raw[:8] == b"QUIVERDB", "bad magic"
        version, kind, endian, nsec, fsize, tcrc, hcrc = struct.unpack_from("<IIIIQII", raw, 8)
        assert kind == 3 and endian == 0x01020304 and fsize == len(raw)
        if verify_header:
            assert hcrc == _crc32c(raw[:36])
        sections = {}
        for i in range(nsec):
            tag, crc, off, size = struct.unpack_from("<IIQQ", raw, 64 + 24 * i)
            sections[struct.pack("<I", tag).decode()] = raw[off:off + size]
        meta = struct.unpack_from("<QQQQQQIIII", sections["META"])
        (self.dim, self.nlist, self.m, self.count, self.train_iterations, self.seed, self.metric,
         store, trained, _) = meta
        self.store_vectors, self.trained = bool(store), bool(trained)
        self.centroids = np.frombuffer(sections["CENT"], np.float32).reshape(self.nlist, self.dim)
        self.codebooks = np.frombuffer(sections["PQCB"], np.float32).reshape(self.m, 256,
                                                                            self.dim // self.m)
        self.offsets = np.frombuffer(sections["LOFF"], np.uint64).copy()
        self.codes = np.frombuffer(sections["CODE"], np.uint8).reshape(self.count, self.m)
        self.labels = np.frombuffer(sections["LABL"], np.uint64).copy()
        self.vectors = (np.frombuffer(sections["VECT"], np.float32).reshape(self.count, self.dim)
                        if "VECT" in sections else None)

    def assignments(self) -> np.ndarray:
        """Cell of each stored entry, list-major order."""
        sizes = np.diff(self.offsets).astype(np.int64)
        return np.repeat(np.arange(self.nlist, dtype=np.uint32), sizes)


def crc32c(data: bytes) -> int:
    return _crc32c(data)


def zlib_crc(data: bytes) -> int:  # convenience for fixture manifests
    return zlib.crc32(data) & 0xFFFFFFFF
