"""Multi-GPU search: the database is sharded by id range, one process per GPU.

Every rank holds one contiguous id range of the collection on its own GPU and receives the whole
query batch. Each rank computes its local top-k (Flat) or top-``keep`` ADC candidates (IVF-PQ) with
the CUDA library, the per-rank (distance, key, label) triples are packed into one buffer and
exchanged with one NCCL all-gather over NVLink (``torch.distributed`` is only the transport), and a device k-way merge
(``qv_merge_topk_device``) produces the global result. Keys are global row ids (Flat) or
``list << 32 | offset-in-full-list`` (IVF-PQ), so ties break exactly as on one GPU.

IVF-PQ with exact re-ranking needs a second exchange for parity with the reference, which
re-ranks the global best ``k * refine_factor`` ADC candidates (src/ivfpq_index.cc:303-373): after
the merge, every rank computes exact distances for the merged candidates it stores (+inf for the
rest), a MIN all-reduce combines them, and the top k are selected on the device.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

from . import FlatIndex, IvfPqIndex, _as_labels, _as_matrix
from ._native import check, lib

_INVALID = np.uint64(2**64 - 1)


def _world(group):
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def _stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def _all_gather(t: torch.Tensor, world: int, group) -> torch.Tensor:
    if world == 1:
        return t.unsqueeze(0)
    t = t.contiguous()
    # Concatenated along dim 0 (the form every backend accepts), then viewed per rank.
    out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, t, group=group)
    return out.view((world,) + tuple(t.shape))


def _all_gather_triples(d: torch.Tensor, key: torch.Tensor, lab: torch.Tensor, world: int,
                        group):
    """All-gathers per-rank (distance float32, key int64, label int64) arrays of one shape with ONE
    collective: the three are packed bit for bit into a single int32 buffer (5 words per entry),
    exchanged, and unpacked per rank as contiguous [world, ...] arrays."""
    if world == 1:
        return d.unsqueeze(0), key.unsqueeze(0), lab.unsqueeze(0)
    n = d.numel()
    buf = torch.empty(5 * n, dtype=torch.int32, device=d.device)
    buf[:n] = d.contiguous().view(torch.int32).reshape(-1)
    buf[n:3 * n] = key.contiguous().view(torch.int32).reshape(-1)
    buf[3 * n:] = lab.contiguous().view(torch.int32).reshape(-1)
    out = _all_gather(buf, world, group)  # [world, 5n]
    shape = (world,) + tuple(d.shape)
    gd = out[:, :n].contiguous().view(torch.float32).view(shape)
    gk = out[:, n:3 * n].contiguous().view(torch.int64).view(shape)
    gl = out[:, 3 * n:].contiguous().view(torch.int64).view(shape)
    return gd, gk, gl


def shard_range(n: int, rank: int, world: int):
    """Rank `rank`'s id range [lo, hi) of n rows split over `world` ranks."""
    return rank * n // world, (rank + 1) * n // world


def list_bases(sizes: torch.Tensor, rank: int, world: int, group=None) -> torch.Tensor:
    """Per IVF list, the number of entries held by the ranks below `rank` (an exclusive prefix
    over ranks of every rank's list sizes, exchanged with one all-gather)."""
    if world == 1:
        return torch.zeros_like(sizes)
    every = _all_gather(sizes, world, group)
    return every[:rank].sum(dim=0)


def _merge(parts_d, parts_k, parts_l, k, device):
    world, nq, kk = parts_d.shape
    od = torch.empty((nq, k), dtype=torch.float32, device=parts_d.device)
    ok = torch.empty((nq, k), dtype=torch.int64, device=parts_d.device)
    ol = torch.empty((nq, k), dtype=torch.int64, device=parts_d.device)
    check(lib().qv_merge_topk_device(device, world, nq, kk, parts_d.data_ptr(),
                                     parts_k.data_ptr(), parts_l.data_ptr(), od.data_ptr(),
                                     ok.data_ptr(), ol.data_ptr(), C.c_void_p(_stream_ptr())))
    return od, ok, ol


class ShardedFlatIndex:
    """Exact Flat search over an id-range-sharded collection (one shard per rank)."""

    def __init__(self, dim: int, metric: str = "l2", *, device: Optional[int] = None, group=None):
        self.rank, self.world = _world(group)
        self.group = group
        self.device = torch.cuda.current_device() if device is None else int(device)
        self.local = FlatIndex(dim, metric, device=self.device)
        self.ntotal = 0
        self._gid = torch.empty(0, dtype=torch.int64, device=f"cuda:{self.device}")
        self._range = None  # [first, end) when rows were added by add_range_device

    @property
    def dim(self) -> int:
        return self.local.dim

    def add(self, vectors, labels=None) -> None:
        """Every rank passes the same batch; rank r keeps rows [r*n/W, (r+1)*n/W) of it."""
        x = _as_matrix(vectors, self.dim)
        n = x.shape[0]
        la = _as_labels(labels, n)
        lo, hi = shard_range(n, self.rank, self.world)
        gids = np.arange(self.ntotal + lo, self.ntotal + hi, dtype=np.int64)
        mine = la[lo:hi] if la is not None else gids.astype(np.uint64)
        self.add_shard(x[lo:hi], mine, gids)
        self.ntotal += n

    def add_range_device(self, vectors: torch.Tensor, first_id: int) -> None:
        """Appends rows already on this rank's GPU whose global ids, and labels, are first_id,
        first_id + 1, ...: consecutive calls extend one contiguous id range (this rank's shard).
        The index then reports global row ids as its keys itself (no per-row id table), so a
        shard of tens of millions of rows needs no host copy."""
        n = int(vectors.shape[0])
        if self._range is None:
            if len(self.local) != 0:
                raise ValueError("add_range_device cannot follow add_shard")
            check(lib().qv_flat_set_row_offset(self.local.handle, int(first_id)))
            self._range = [int(first_id), int(first_id)]
        if int(first_id) != self._range[1]:
            raise ValueError(f"rows must extend the id range [{self._range[0]}, {self._range[1]})")
        ids = torch.arange(first_id, first_id + n, dtype=torch.int64, device=vectors.device)
        self.local.add_device(vectors, ids)
        self._range[1] += n

    def add_shard(self, vectors, labels, global_ids) -> None:
        """Appends this rank's rows directly (labels and global row ids given per row)."""
        if self._range is not None:
            raise ValueError("add_shard cannot follow add_range_device")
        self.local.add(vectors, labels)
        g = torch.as_tensor(np.ascontiguousarray(global_ids, dtype=np.int64),
                            device=self._gid.device)
        self._gid = torch.cat([self._gid, g])

    def search_device(self, queries: torch.Tensor, k: int):
        """Queries on this rank's GPU (float32 [nq, dim]); returns device (dists, labels) after
        the cross-rank merge, identical on every rank."""
        nq = queries.shape[0]
        d = torch.empty((nq, k), dtype=torch.float32, device=queries.device)
        lab = torch.empty((nq, k), dtype=torch.int64, device=queries.device)
        key = torch.empty((nq, k), dtype=torch.int64, device=queries.device)
        check(lib().qv_flat_search_device(self.local.handle, queries.data_ptr(), nq, k, None,
                                          lab.data_ptr(), d.data_ptr(), key.data_ptr(),
                                          C.c_void_p(_stream_ptr())))
        if self.world == 1:
            return d, lab
        if self._range is not None:
            gkey = key  # the index's row offset already made the keys global ids
        else:
            valid = key >= 0  # unfilled slots carry key 2^64-1 (-1 as int64)
            gkey = torch.where(valid, self._gid[key.clamp(min=0)], key)
        od, _, ol = _merge(*_all_gather_triples(d, gkey, lab, self.world, self.group), k,
                           self.device)
        return od, ol

    def search(self, queries, k: int = 10):
        q = _as_matrix(queries, self.dim)
        dq = torch.from_numpy(q).to(f"cuda:{self.device}", non_blocking=True)
        d, lab = self.search_device(dq, int(k))
        return lab.cpu().numpy(), d.cpu().numpy()


class ReplicatedFlatIndex:
    """Exact Flat search with the collection replicated on every rank and each query batch split
    by rank: rank r answers queries [r*nq/W, (r+1)*nq/W) of every batch from its own full copy.
    No exchange on the search path; the answers are the single-index answers (every rank holds
    every row in the same order). Memory per GPU is the whole collection (C1: 0.74 GB)."""

    def __init__(self, dim: int, metric: str = "l2", *, device: Optional[int] = None, group=None):
        self.rank, self.world = _world(group)
        self.group = group
        self.device = torch.cuda.current_device() if device is None else int(device)
        self.local = FlatIndex(dim, metric, device=self.device)

    @property
    def dim(self) -> int:
        return self.local.dim

    def add(self, vectors, labels=None) -> None:
        """Every rank passes the same batch and keeps all of it."""
        self.local.add(vectors, labels)

    def query_range(self, nq: int):
        return shard_range(nq, self.rank, self.world)

    def search_device(self, queries: torch.Tensor, k: int):
        """Queries of the whole batch on this rank's GPU (float32 [nq, dim]); returns device
        (dists, labels) of this rank's slice of the batch (rows query_range(nq))."""
        lo, hi = self.query_range(queries.shape[0])
        mine = queries[lo:hi]
        d = torch.empty((hi - lo, k), dtype=torch.float32, device=queries.device)
        lab = torch.empty((hi - lo, k), dtype=torch.int64, device=queries.device)
        if hi > lo:
            check(lib().qv_flat_search_device(self.local.handle, mine.data_ptr(), hi - lo, k,
                                              None, lab.data_ptr(), d.data_ptr(), None,
                                              C.c_void_p(_stream_ptr())))
        return d, lab

    def search(self, queries, k: int = 10, gather: bool = False):
        """Host API: this rank answers its slice of the batch (labels, distances as numpy); with
        gather=True the slices are all-gathered so every rank returns the whole batch's answers."""
        q = _as_matrix(queries, self.dim)
        lo, hi = self.query_range(q.shape[0])
        lab, d = self.local.search(q[lo:hi], int(k))
        if not gather or self.world == 1:
            return lab, d
        dev = torch.device(f"cuda:{self.device}")
        return gather_query_slices(torch.from_numpy(d).to(dev), torch.from_numpy(lab).to(dev),
                                   q.shape[0], self.world, self.group)


def gather_query_slices(d: torch.Tensor, lab: torch.Tensor, nq: int, world: int, group=None):
    """All-gathers every rank's (distances, labels) answers for its query slice shard_range(nq,
    rank, world) and returns the whole batch's answers in query order (numpy labels, distances).
    Slices differ in length by at most one row; each is padded to the longest for the exchange."""
    k = d.shape[1]
    parts = [shard_range(nq, r, world) for r in range(world)]
    width = max(hi - lo for lo, hi in parts)
    pd = torch.full((width, k), float("inf"), dtype=torch.float32, device=d.device)
    pl = torch.full((width, k), -1, dtype=torch.int64, device=d.device)
    pd[:d.shape[0]] = d
    pl[:lab.shape[0]] = lab
    gd = _all_gather(pd, world, group).cpu().numpy()
    gl = _all_gather(pl, world, group).cpu().numpy()
    out_d = np.concatenate([gd[r, :hi - lo] for r, (lo, hi) in enumerate(parts)])
    out_l = np.concatenate([gl[r, :hi - lo] for r, (lo, hi) in enumerate(parts)])
    return out_l, out_d


class ShardedIvfPqIndex:
    """IVF-PQ search over an id-range-sharded index (one shard per rank).

    Built either from a populated .qvr (each rank keeps the entries whose label lies in its id
    range) or, with :meth:`from_trained`, from a trained .qvr plus each rank's own rows added on
    its GPU."""

    def __init__(self, path: Optional[str] = None, *, total: int, device: Optional[int] = None,
                 group=None, local: Optional[IvfPqIndex] = None):
        self.rank, self.world = _world(group)
        self.group = group
        self.device = torch.cuda.current_device() if device is None else int(device)
        if local is None:
            lo, hi = shard_range(total, self.rank, self.world)
            local = IvfPqIndex.load(path, device=self.device,
                                    label_range=None if self.world == 1 else (lo, hi))
        self.local = local
        self.total = total

    @classmethod
    def from_trained(cls, trained, vectors, labels, *, total: int,
                     device: Optional[int] = None, group=None) -> "ShardedIvfPqIndex":
        """Starts every rank from trained, empty state (a .qvr path, or an IvfPqIndex already
        trained on this rank's device) and adds this rank's rows (``labels`` = their global ids,
        in id order). Each list's entries of lower ranks are counted so that candidate keys
        (list << 32 | offset in the full list) equal those of one index holding every row in id
        order."""
        rank, world = _world(group)
        dev = torch.cuda.current_device() if device is None else int(device)
        local = IvfPqIndex.load(trained, device=dev) if isinstance(trained, str) else trained
        local.add(vectors, labels)
        if world > 1:
            sizes = torch.tensor(local.list_sizes(), dtype=torch.int64, device=f"cuda:{dev}")
            base = list_bases(sizes, rank, world, group).cpu().numpy().astype(np.uint32)
            check(lib().qv_ivfpq_set_list_base(local.handle, base.ctypes.data))
        return cls(total=total, device=dev, group=group, local=local)

    def filter_bitmap(self, allowed) -> Optional[torch.Tensor]:
        """Device position bitmap of this shard (bit i of word i >> 6 = stored entry i is
        admitted) for a set of allowed labels, None for no filter. Built once on the host from
        the shard's stored labels; pass it to :meth:`search_device` to keep it resident."""
        if allowed is None:
            return None
        mask = np.isin(self.local.stored_labels(), _as_labels(allowed))
        packed = np.packbits(mask, bitorder="little")
        words = np.zeros(max(1, (mask.size + 63) // 64) * 8, np.uint8)
        words[:packed.size] = packed
        return torch.from_numpy(words.view(np.int64)).to(f"cuda:{self.device}")

    def search_device(self, queries: torch.Tensor, k: int, nprobe: int = 16,
                      refine_factor: int = 0, bitmap: Optional[torch.Tensor] = None):
        nq = queries.shape[0]
        dev = queries.device
        sp = C.c_void_p(_stream_ptr())
        bm = bitmap.data_ptr() if bitmap is not None else None
        if self.world == 1:
            od = torch.empty((nq, k), dtype=torch.float32, device=dev)
            ol = torch.empty((nq, k), dtype=torch.int64, device=dev)
            check(lib().qv_ivfpq_search_device(self.local.handle, queries.data_ptr(), nq, k,
                                               nprobe, refine_factor, bm, ol.data_ptr(),
                                               od.data_ptr(), sp))
            return od, ol
        refine = refine_factor > 0 and bool(self._store_vectors())
        factor = refine_factor if refine else 1
        keep = min(self.total, self.total if factor > self.total // max(k, 1) else k * factor)
        d = torch.empty((nq, keep), dtype=torch.float32, device=dev)
        key = torch.empty((nq, keep), dtype=torch.int64, device=dev)
        lab = torch.empty((nq, keep), dtype=torch.int64, device=dev)
        check(lib().qv_ivfpq_candidates_device(self.local.handle, queries.data_ptr(), nq, keep,
                                               nprobe, bm, d.data_ptr(), key.data_ptr(),
                                               lab.data_ptr(), sp))
        d, key, lab = _merge(*_all_gather_triples(d, key, lab, self.world, self.group), keep,
                             self.device)
        if not refine:
            return d[:, :k].contiguous(), lab[:, :k].contiguous()
        exact = torch.empty((nq, keep), dtype=torch.float32, device=dev)
        check(lib().qv_ivfpq_refine_device(self.local.handle, queries.data_ptr(), nq, keep,
                                           key.data_ptr(), exact.data_ptr(), sp))
        dist.all_reduce(exact, op=dist.ReduceOp.MIN, group=self.group)
        od = torch.empty((nq, k), dtype=torch.float32, device=dev)
        ok = torch.empty((nq, k), dtype=torch.int64, device=dev)
        ol = torch.empty((nq, k), dtype=torch.int64, device=dev)
        check(lib().qv_select_topk_device(self.device, nq, keep, k, exact.data_ptr(),
                                          key.data_ptr(), lab.data_ptr(), od.data_ptr(),
                                          ok.data_ptr(), ol.data_ptr(), sp))
        return od, ol

    def _store_vectors(self) -> int:
        return self.local._info()[0].store_vectors

    def search(self, queries, k: int = 10, nprobe: int = 16, refine_factor: int = 0,
               filter=None):
        q = _as_matrix(queries, self.local.dim)
        dq = torch.from_numpy(q).to(f"cuda:{self.device}", non_blocking=True)
        d, lab = self.search_device(dq, int(k), int(nprobe), int(refine_factor),
                                    self.filter_bitmap(filter))
        return lab.cpu().numpy(), d.cpu().numpy()
