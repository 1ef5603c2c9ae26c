"""quiver_b200: Quiver's exact Flat and IVF-PQ nearest-neighbour search on NVIDIA B200 (sm_100a).

A drop-in for the ``quiver.FlatIndex`` / ``quiver.IvfPqIndex`` Python surface of the reference
(python/quiver/__init__.py:166-251): same constructors, methods, argument meaning, result layout
and errors. Every call runs through the C ABI (include/qv_gpu.h) on the GPU; there is no CPU path.

    >>> import numpy as np, quiver_b200 as quiver
    >>> index = quiver.FlatIndex(dim=128, metric="cosine")
    >>> index.add(np.random.rand(10_000, 128))
    >>> labels, distances = index.search(np.random.rand(5, 128), k=10)

Distances are "smaller is closer": squared L2 for ``"l2"``, ``1 - <q, x>`` for ``"ip"``, and
``1 - cos(q, x)`` for ``"cosine"``. Missing results come back as label ``-1`` and distance ``inf``.
GPU-specific additions are keyword-only: ``device=`` selects the CUDA device.
"""
from __future__ import annotations

import ctypes as C
from typing import Iterable, Optional, Tuple, Union

import numpy as np

from . import _native
from ._native import QuiverError, check, device_count, last_search_stats, lib, make_filter, ptr

__all__ = ["FlatIndex", "IvfPqIndex", "HnswStore", "QuiverError", "device_count",
           "last_search_stats"]
__version__ = "0.1.0"

ArrayLike = Union[np.ndarray, Iterable]
_MAX_LABEL = 2**63 - 1  # results are int64 with -1 for empty slots


def _metric_code(metric: str) -> int:
    try:
        return _native.METRIC_CODES[metric]
    except KeyError:
        raise ValueError(f"unknown metric '{metric}' (expected l2, ip, or cosine)") from None


def _as_matrix(x: ArrayLike, dim: int) -> np.ndarray:
    a = np.ascontiguousarray(x, dtype=np.float32)
    if a.ndim == 1:
        a = a.reshape(1, -1)
    if a.ndim != 2:
        raise ValueError(f"expected a 1-D or 2-D array, got shape {a.shape}")
    if a.shape[1] != dim:
        raise ValueError(f"expected dimension {dim}, got {a.shape[1]}")
    return a


def _as_labels(labels: Optional[ArrayLike], n: Optional[int] = None) -> Optional[np.ndarray]:
    """Integers in [0, 2**63) from an array or any iterable, as contiguous uint64."""
    if labels is None:
        return None
    if isinstance(labels, np.ndarray) and labels.dtype != object:
        a = labels.reshape(-1)
        if a.size and not np.issubdtype(a.dtype, np.integer):
            raise TypeError("labels must be integers")
        if a.size and np.issubdtype(a.dtype, np.signedinteger) and a.min() < 0:
            raise ValueError("labels must be non-negative")
        if a.size and int(a.max()) > _MAX_LABEL:
            raise ValueError("labels must be below 2**63")
        out = np.ascontiguousarray(a, dtype=np.uint64)
    else:
        items = labels.reshape(-1).tolist() if isinstance(labels, np.ndarray) else (
            [labels] if isinstance(labels, (int, np.integer)) else list(labels))
        vals = []
        for v in items:  # checked as Python ints so numpy never rounds 2**63 through float64
            if isinstance(v, bool) or not isinstance(v, (int, np.integer)):
                raise TypeError("labels must be integers")
            if v < 0:
                raise ValueError("labels must be non-negative")
            if v > _MAX_LABEL:
                raise ValueError("labels must be below 2**63")
            vals.append(int(v))
        out = np.array(vals, dtype=np.uint64)
    if n is not None and out.shape[0] != n:
        raise ValueError(f"got {out.shape[0]} labels for {n} vectors")
    return out


def _results(labels: np.ndarray, dists: np.ndarray):
    return labels.view(np.int64), dists  # 2**64-1 reads back as -1


def _result_arrays(nq: int, k: int):
    total = nq * k
    if total > (1 << 40):
        raise ValueError("nq * k is too large")
    return np.empty((nq, k), np.uint64), np.empty((nq, k), np.float32)


class FlatIndex:
    """Exact brute-force index on one GPU (reference: include/quiver/flat_index.h)."""

    def __init__(self, dim: int, metric: str = "l2", *, device: int = 0, _native_handle=None):
        self._h = C.c_void_p()
        if _native_handle is not None:
            self._h = _native_handle
        else:
            check(lib().qv_flat_create(int(device), int(dim), _metric_code(metric),
                                       C.byref(self._h)))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._h = None
            try:
                lib().qv_flat_destroy(h)
            except (TypeError, AttributeError):  # interpreter shutdown: module globals are gone
                pass

    def _info(self):
        n, d, m = C.c_size_t(), C.c_size_t(), C.c_uint32()
        check(lib().qv_flat_info(self._h, C.byref(n), C.byref(d), C.byref(m)))
        return n.value, d.value, m.value

    def add(self, vectors: ArrayLike, labels: Optional[ArrayLike] = None) -> None:
        x = _as_matrix(vectors, self.dim)
        la = _as_labels(labels, x.shape[0])
        check(lib().qv_flat_add(self._h, ptr(x), x.shape[0], ptr(la)))

    def reserve(self, n: int) -> None:
        """Sizes the GPU row storage for n rows at once (no counterpart in the reference)."""
        check(lib().qv_flat_reserve(self._h, int(n)))

    def add_device(self, vectors, labels=None, stream=None) -> None:
        """Appends rows already in GPU memory: ``vectors`` a contiguous float32 CUDA tensor
        [n, dim] on this index's device, ``labels`` None or a contiguous int64 CUDA tensor [n];
        the same checks and results as :meth:`add` (no counterpart in the reference)."""
        if vectors.dim() != 2 or vectors.shape[1] != self.dim or not vectors.is_contiguous():
            raise ValueError(f"expected a contiguous [n, {self.dim}] tensor")
        n = int(vectors.shape[0])
        lp = None
        if labels is not None:
            if labels.numel() != n or not labels.is_contiguous():
                raise ValueError("labels must be a contiguous tensor of n entries")
            lp = labels.data_ptr()
        check(lib().qv_flat_add_device(self._h, vectors.data_ptr(), n, lp,
                                       C.c_void_p(stream) if stream else None))

    def search(self, queries: ArrayLike, k: int = 10, filter: Optional[ArrayLike] = None,
               num_threads: int = 0) -> Tuple[np.ndarray, np.ndarray]:
        """k-NN search. Returns (labels int64 [nq, k], distances float32 [nq, k]).
        ``num_threads`` is accepted for compatibility; the GPU decides its own parallelism."""
        q = _as_matrix(queries, self.dim)
        if k <= 0:
            raise ValueError("k must be positive")
        allowed = _as_labels(filter) if filter is not None else None
        f, keep = make_filter(allowed)
        labels, dists = _result_arrays(q.shape[0], int(k))
        check(lib().qv_flat_search(self._h, ptr(q), q.shape[0], int(k),
                                   C.byref(f) if f is not None else None, ptr(labels), ptr(dists)))
        del keep
        return _results(labels, dists)

    def rows(self, first: int = 0, count: Optional[int] = None):
        """Stored vectors (normalized for cosine) and labels of rows [first, first + count)."""
        n = len(self)
        count = n - first if count is None else count
        v = np.empty((count, self.dim), np.float32)
        la = np.empty(count, np.uint64)
        check(lib().qv_flat_rows(self._h, first, count, ptr(v), ptr(la)))
        return v, la

    def save(self, path: str) -> None:
        check(lib().qv_flat_save(self._h, str(path).encode()))

    @classmethod
    def load(cls, path: str, verify_checksums: bool = True, *, device: int = 0) -> "FlatIndex":
        h = C.c_void_p()
        check(lib().qv_flat_load(int(device), str(path).encode(), int(verify_checksums),
                                 C.byref(h)))
        return cls(0, _native_handle=h)

    def __len__(self) -> int:
        return self._info()[0]

    @property
    def dim(self) -> int:
        return self._info()[1]

    @property
    def metric(self) -> str:
        return _native.METRIC_NAMES[self._info()[2]]

    @property
    def handle(self):
        return self._h

    def __repr__(self) -> str:
        return f"FlatIndex(dim={self.dim}, metric={self.metric!r}, size={len(self)})"


class IvfPqIndex:
    """Inverted-file index over product-quantized residuals (reference:
    include/quiver/ivfpq_index.h). :meth:`train` gives the reference's centroids and codebooks
    bit for bit (its k-means assignment steps run on the GPU); trained state can also come from
    :meth:`load` (a ``.qvr`` written by the reference or by :meth:`save`) or :meth:`set_trained`."""

    def __init__(self, dim: int, metric: str = "l2", nlist: int = 1024, m: int = 16,
                 store_vectors: bool = False, train_iterations: int = 20, seed: int = 1234,
                 *, device: int = 0, _native_handle=None):
        self._h = C.c_void_p()
        if _native_handle is not None:
            self._h = _native_handle
        else:
            p = _native.qv_ivfpq_params(int(dim), _metric_code(metric), int(nlist), int(m),
                                        int(train_iterations), int(bool(store_vectors)), int(seed))
            check(lib().qv_ivfpq_create(int(device), C.byref(p), C.byref(self._h)))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._h = None
            try:
                lib().qv_ivfpq_destroy(h)
            except (TypeError, AttributeError):  # interpreter shutdown: module globals are gone
                pass

    def _info(self):
        p = _native.qv_ivfpq_params()
        n, mem = C.c_size_t(), C.c_size_t()
        check(lib().qv_ivfpq_info(self._h, C.byref(p), C.byref(n), C.byref(mem)))
        return p, n.value, mem.value

    def train(self, vectors: ArrayLike, num_threads: int = 0) -> None:
        """IvfPqIndex::train; ``num_threads`` is accepted for compatibility."""
        x = _as_matrix(vectors, self.dim)
        check(lib().qv_ivfpq_train(self._h, ptr(x), x.shape[0]))

    def set_trained(self, centroids: ArrayLike, codebooks: ArrayLike) -> None:
        """Installs trained state: centroids [nlist, dim], codebooks [m, 256, dim // m]."""
        p = self._info()[0]
        c = np.ascontiguousarray(centroids, dtype=np.float32).reshape(p.nlist, p.dim)
        cb = np.ascontiguousarray(codebooks, dtype=np.float32).reshape(p.m, 256, p.dim // p.m)
        check(lib().qv_ivfpq_set_trained(self._h, ptr(c), ptr(cb)))

    def add(self, vectors: ArrayLike, labels: Optional[ArrayLike] = None,
            num_threads: int = 0) -> None:
        x = _as_matrix(vectors, self.dim)
        la = _as_labels(labels, x.shape[0])
        check(lib().qv_ivfpq_add(self._h, ptr(x), x.shape[0], ptr(la)))

    def encode(self, vectors: ArrayLike) -> Tuple[np.ndarray, np.ndarray]:
        """(cell uint32 [n], codes uint8 [n, m]) exactly as add() computes them."""
        x = _as_matrix(vectors, self.dim)
        a = np.empty(x.shape[0], np.uint32)
        c = np.empty((x.shape[0], self.m), np.uint8)
        check(lib().qv_ivfpq_encode(self._h, ptr(x), x.shape[0], ptr(a), ptr(c)))
        return a, c

    def search(self, queries: ArrayLike, k: int = 10, nprobe: int = 16, refine_factor: int = 0,
               filter: Optional[ArrayLike] = None,
               num_threads: int = 0) -> Tuple[np.ndarray, np.ndarray]:
        q = _as_matrix(queries, self.dim)
        if k <= 0:
            raise ValueError("k must be positive")
        allowed = _as_labels(filter) if filter is not None else None
        f, keep = make_filter(allowed)
        labels, dists = _result_arrays(q.shape[0], int(k))
        check(lib().qv_ivfpq_search(self._h, ptr(q), q.shape[0], int(k), int(nprobe),
                                    int(refine_factor), C.byref(f) if f is not None else None,
                                    ptr(labels), ptr(dists)))
        del keep
        return _results(labels, dists)

    def save(self, path: str) -> None:
        check(lib().qv_ivfpq_save(self._h, str(path).encode()))

    @classmethod
    def load(cls, path: str, verify_checksums: bool = True, *, device: int = 0,
             label_range: Optional[Tuple[int, int]] = None) -> "IvfPqIndex":
        """Loads a .qvr; ``label_range=(begin, end)`` keeps one id-range shard of it."""
        h = C.c_void_p()
        if label_range is None:
            check(lib().qv_ivfpq_load(int(device), str(path).encode(), int(verify_checksums),
                                      C.byref(h)))
        else:
            check(lib().qv_ivfpq_load_shard(int(device), str(path).encode(),
                                            int(verify_checksums), int(label_range[0]),
                                            int(label_range[1]), C.byref(h)))
        return cls(0, _native_handle=h)

    def list_sizes(self) -> list:
        sizes = np.empty(self.nlist, np.uint64)
        check(lib().qv_ivfpq_list_sizes(self._h, ptr(sizes)))
        return [int(s) for s in sizes]

    def stored_labels(self) -> np.ndarray:
        """Labels in storage (list-major) order."""
        out = np.empty(len(self), np.uint64)
        check(lib().qv_ivfpq_labels(self._h, ptr(out)))
        return out

    def __len__(self) -> int:
        return self._info()[1]

    @property
    def dim(self) -> int:
        return self._info()[0].dim

    @property
    def nlist(self) -> int:
        return self._info()[0].nlist

    @property
    def m(self) -> int:
        return self._info()[0].m

    @property
    def metric(self) -> str:
        return _native.METRIC_NAMES[self._info()[0].metric]

    @property
    def is_trained(self) -> bool:
        t = C.c_int()
        check(lib().qv_ivfpq_is_trained(self._h, C.byref(t)))
        return bool(t.value)

    @property
    def memory_bytes(self) -> int:
        return self._info()[2]

    @property
    def handle(self):
        return self._h

    def __repr__(self) -> str:
        return f"IvfPqIndex(dim={self.dim}, nlist={self.nlist}, m={self.m}, size={len(self)})"


class HnswStore:
    """The vector storage of an HNSW index on one GPU and the exact scan ``HnswIndex.search``
    falls back to when a filter admits few vectors (reference: include/quiver/hnsw_index.h:25-121,
    src/hnsw_index.cc:723-760). ``storage`` is ``"float32"`` or ``"sq8"`` (8-bit scalar
    quantization, trained once on prepared vectors). Nodes are numbered in insertion order.
    :meth:`search` returns what the reference's filtered search returns when it takes the exact
    scan, bit for bit."""

    def __init__(self, dim: int, metric: str = "l2", storage: str = "float32", *,
                 device: int = 0):
        if storage not in _native.STORAGE_CODES:
            raise ValueError(f"unknown storage '{storage}' (expected float32 or sq8)")
        self._h = C.c_void_p()
        check(lib().qv_hnsw_store_create(int(device), int(dim), _metric_code(metric),
                                         _native.STORAGE_CODES[storage], C.byref(self._h)))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._h = None
            try:
                lib().qv_hnsw_store_destroy(h)
            except (TypeError, AttributeError):
                pass

    def _info(self):
        live, nodes, d = C.c_size_t(), C.c_size_t(), C.c_size_t()
        m, st = C.c_uint32(), C.c_uint32()
        check(lib().qv_hnsw_store_info(self._h, C.byref(live), C.byref(nodes), C.byref(d),
                                       C.byref(m), C.byref(st)))
        return live.value, nodes.value, d.value, m.value, st.value

    def train(self, vectors: ArrayLike) -> None:
        x = _as_matrix(vectors, self.dim)
        check(lib().qv_hnsw_store_train(self._h, ptr(x), x.shape[0]))

    @property
    def is_trained(self) -> bool:
        t = C.c_int()
        check(lib().qv_hnsw_store_is_trained(self._h, C.byref(t)))
        return bool(t.value)

    def add(self, vectors: ArrayLike, labels: Optional[ArrayLike] = None) -> None:
        x = _as_matrix(vectors, self.dim)
        la = _as_labels(labels, x.shape[0])
        check(lib().qv_hnsw_store_add(self._h, ptr(x), x.shape[0], ptr(la)))

    def remove(self, label: int) -> bool:
        r = C.c_int()
        check(lib().qv_hnsw_store_remove(self._h, int(label), C.byref(r)))
        return bool(r.value)

    def get_vector(self, label: int) -> np.ndarray:
        """The stored vector (decoded for SQ8, normalized for cosine)."""
        out = np.empty(self.dim, np.float32)
        check(lib().qv_hnsw_store_vector(self._h, int(label), ptr(out)))
        return out

    def codes(self, first: int = 0, count: Optional[int] = None) -> np.ndarray:
        """SQ8 codes of nodes [first, first + count)."""
        n = self.num_nodes
        count = n - first if count is None else count
        out = np.empty((count, self.dim), np.uint8)
        check(lib().qv_hnsw_store_codes(self._h, int(first), int(count), ptr(out)))
        return out

    def sq8_params(self) -> Tuple[np.ndarray, np.ndarray]:
        vmin = np.empty(self.dim, np.float32)
        vscale = np.empty(self.dim, np.float32)
        check(lib().qv_hnsw_store_sq8_params(self._h, ptr(vmin), ptr(vscale)))
        return vmin, vscale

    def search(self, queries: ArrayLike, k: int = 10, filter: Optional[ArrayLike] = None
               ) -> Tuple[np.ndarray, np.ndarray]:
        """Exact scan over the live vectors whose label ``filter`` admits (every live vector when
        None). Returns (labels int64 [nq, k], distances float32 [nq, k])."""
        q = _as_matrix(queries, self.dim)
        if k <= 0:
            raise ValueError("k must be positive")
        allowed = _as_labels(filter) if filter is not None else None
        f, keep = make_filter(allowed)
        labels, dists = _result_arrays(q.shape[0], int(k))
        check(lib().qv_hnsw_store_search(self._h, ptr(q), q.shape[0], int(k),
                                         C.byref(f) if f is not None else None, ptr(labels),
                                         ptr(dists)))
        del keep
        return _results(labels, dists)

    def __len__(self) -> int:
        return self._info()[0]

    @property
    def num_nodes(self) -> int:
        return self._info()[1]

    @property
    def dim(self) -> int:
        return self._info()[2]

    @property
    def metric(self) -> str:
        return _native.METRIC_NAMES[self._info()[3]]

    @property
    def storage(self) -> str:
        return _native.STORAGE_NAMES[self._info()[4]]

    def __repr__(self) -> str:
        return (f"HnswStore(dim={self.dim}, metric={self.metric!r}, storage={self.storage!r}, "
                f"size={len(self)})")
