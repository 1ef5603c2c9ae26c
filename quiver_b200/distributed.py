"""Multi-GPU search: the database is sharded by id range, one process per GPU.

Every rank holds one contiguous id range of the collection on its own GPU and receives the whole
query batch. Each rank computes its local top-k (Flat) or top-``keep`` ADC candidates (IVF-PQ) with
the CUDA library, the per-rank (distance, key, label) triples are exchanged with one NCCL
all-gather over NVLink (``torch.distributed`` is only the transport), and a device k-way merge
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
    out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    return out


def _merge(parts_d, parts_k, parts_l, k, device):
    world, nq, kk = parts_d.shape
    od = torch.empty((nq, k), dtype=torch.float32, device=parts_d.device)
    ok = torch.empty((nq, k), dtype=torch.int64, device=parts_d.device)
    ol = torch.empty((nq, k), dtype=torch.int64, device=parts_d.device)
    check(lib().qv_merge_topk_device(device, world, nq, kk, parts_d.data_ptr(),
                                     parts_k.data_ptr(), parts_l.data_ptr(), od.data_ptr(),
                                     ok.data_ptr(), ol.data_ptr(), C.c_void_p(_stream_ptr())))
    if k < kk:
        pass
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

    @property
    def dim(self) -> int:
        return self.local.dim

    def add(self, vectors, labels=None) -> None:
        """Every rank passes the same batch; rank r keeps rows [r*n/W, (r+1)*n/W) of it."""
        x = _as_matrix(vectors, self.dim)
        n = x.shape[0]
        la = _as_labels(labels, n)
        lo, hi = self.rank * n // self.world, (self.rank + 1) * n // self.world
        gids = np.arange(self.ntotal + lo, self.ntotal + hi, dtype=np.int64)
        mine = la[lo:hi] if la is not None else gids.astype(np.uint64)
        self.add_shard(x[lo:hi], mine, gids)
        self.ntotal += n

    def add_shard(self, vectors, labels, global_ids) -> None:
        """Appends this rank's rows directly (labels and global row ids given per row)."""
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
        valid = key >= 0  # unfilled slots carry key 2^64-1 (-1 as int64)
        gkey = torch.where(valid, self._gid[key.clamp(min=0)], key)
        if self.world == 1:
            return d, lab
        od, _, ol = _merge(_all_gather(d, self.world, self.group),
                           _all_gather(gkey, self.world, self.group),
                           _all_gather(lab, self.world, self.group), k, self.device)
        return od, ol

    def search(self, queries, k: int = 10):
        q = _as_matrix(queries, self.dim)
        dq = torch.from_numpy(q).to(f"cuda:{self.device}", non_blocking=True)
        d, lab = self.search_device(dq, int(k))
        return lab.cpu().numpy(), d.cpu().numpy()


class ShardedIvfPqIndex:
    """IVF-PQ search over an id-range-sharded .qvr (one shard per rank)."""

    def __init__(self, path: str, *, total: int, device: Optional[int] = None, group=None):
        self.rank, self.world = _world(group)
        self.group = group
        self.device = torch.cuda.current_device() if device is None else int(device)
        lo, hi = self.rank * total // self.world, (self.rank + 1) * total // self.world
        self.local = IvfPqIndex.load(path, device=self.device,
                                     label_range=None if self.world == 1 else (lo, hi))
        self.total = total

    def search_device(self, queries: torch.Tensor, k: int, nprobe: int = 16,
                      refine_factor: int = 0):
        nq = queries.shape[0]
        refine = refine_factor > 0 and bool(self._store_vectors())
        factor = refine_factor if refine else 1
        keep = min(self.total, self.total if factor > self.total // max(k, 1) else k * factor)
        dev = queries.device
        d = torch.empty((nq, keep), dtype=torch.float32, device=dev)
        key = torch.empty((nq, keep), dtype=torch.int64, device=dev)
        lab = torch.empty((nq, keep), dtype=torch.int64, device=dev)
        sp = C.c_void_p(_stream_ptr())
        check(lib().qv_ivfpq_candidates_device(self.local.handle, queries.data_ptr(), nq, keep,
                                               nprobe, None, d.data_ptr(), key.data_ptr(),
                                               lab.data_ptr(), sp))
        if self.world > 1:
            d, key, lab = _merge(_all_gather(d, self.world, self.group),
                                 _all_gather(key, self.world, self.group),
                                 _all_gather(lab, self.world, self.group), keep, self.device)
        if not refine:
            return d[:, :k].contiguous(), lab[:, :k].contiguous()
        exact = torch.empty((nq, keep), dtype=torch.float32, device=dev)
        check(lib().qv_ivfpq_refine_device(self.local.handle, queries.data_ptr(), nq, keep,
                                           key.data_ptr(), exact.data_ptr(), sp))
        if self.world > 1:
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

    def search(self, queries, k: int = 10, nprobe: int = 16, refine_factor: int = 0):
        q = _as_matrix(queries, self.local.dim)
        dq = torch.from_numpy(q).to(f"cuda:{self.device}", non_blocking=True)
        d, lab = self.search_device(dq, int(k), int(nprobe), int(refine_factor))
        return lab.cpu().numpy(), d.cpu().numpy()
