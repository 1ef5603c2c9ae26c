"""Sharded search on two GPUs (NCCL), one process per GPU: the id-range-sharded FlatIndex and
IVF-PQ index return exactly what one index holding every row returns (distances, labels, and
tie order through the global keys). Skipped where fewer than two GPUs are visible.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

from conftest import GOLDEN, golden_ivf_inputs

pytestmark = pytest.mark.gpu
WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _flat_worker(rank, world, port, out_q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        import quiver_b200 as qv
        from quiver_b200.distributed import ReplicatedFlatIndex, ShardedFlatIndex
        from quiver_b200.synthetic import mixture
        out = {}
        for metric in ("cosine", "l2", "ip"):
            db = mixture(40000, 100, 300, 0.35, 1.0, centre_seed=3, seed=4)
            q = mixture(300, 100, 300, 0.35, 1.0, centre_seed=3, seed=5)
            sharded = ShardedFlatIndex(100, metric, device=rank)
            sharded.add(db)
            d, lab = sharded.search_device(torch.from_numpy(q).cuda(), 10)
            full = qv.FlatIndex(100, metric, device=rank)
            full.add(db)
            fl, fd = full.search(q, 10)
            out[metric] = (d.cpu().numpy(), lab.cpu().numpy(), fd, fl)
            # Rows replicated, queries split by rank: each rank's slice, and the gathered batch.
            rep = ReplicatedFlatIndex(100, metric, device=rank)
            rep.add(db)
            sd, sl = rep.search_device(torch.from_numpy(q).cuda(), 10)
            gl, gd = rep.search(q, 10, gather=True)
            lo, hi = rep.query_range(len(q))
            out[metric + "/slice"] = (sd.cpu().numpy(), sl.cpu().numpy(), fd[lo:hi], fl[lo:hi])
            out[metric + "/gathered"] = (gd, gl, fd, fl)
        out_q.put((rank, out, None))
    except Exception as e:  # noqa: BLE001
        out_q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def _ivf_worker(rank, world, port, out_q, case):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        import quiver_b200 as qv
        from oracle.oracle import QvrIvf
        from quiver_b200.distributed import ShardedIvfPqIndex, shard_range
        path = os.path.join(GOLDEN, case["name"] + ".qvr")
        ref = QvrIvf(path)
        base, q = golden_ivf_inputs(case)
        trained = qv.IvfPqIndex(case["dim"], case["metric"], case["nlist"], case["m"],
                                store_vectors=True, device=rank)
        trained.set_trained(ref.centroids, ref.codebooks)
        lo, hi = shard_range(len(base), rank, world)
        sharded = ShardedIvfPqIndex.from_trained(trained, base[lo:hi],
                                                 np.arange(lo, hi, dtype=np.uint64),
                                                 total=len(base), device=rank)
        full = qv.IvfPqIndex.load(path, device=rank)
        out = {}
        dq = torch.from_numpy(q).cuda()
        for nprobe, rf in ((4, 0), (16, 2), (3, 3)):
            d, lab = sharded.search_device(dq, 10, nprobe, rf)
            fl, fd = full.search(q, 10, nprobe=nprobe, refine_factor=rf)
            out[(nprobe, rf)] = (d.cpu().numpy(), lab.cpu().numpy(), fd, fl)
        allowed = np.arange(0, len(base), 7, dtype=np.uint64)
        lab, d = sharded.search(q, 10, nprobe=8, filter=allowed)
        fl, fd = full.search(q, 10, nprobe=8, filter=allowed)
        out["filtered"] = (d, lab, fd, fl)
        out_q.put((rank, out, None))
    except Exception as e:  # noqa: BLE001
        out_q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def _wide_worker(rank, world, port, out_q):
    """Config 4's layout at test size: 768-dim inner product, k=100, each rank's id range added
    from device memory (add_range_device), the wide tensor-core screen, one packed all-gather and
    the device merge."""
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        import quiver_b200 as qv
        from quiver_b200.distributed import ShardedFlatIndex, shard_range
        from quiver_b200.synthetic import config4_chunk
        db = config4_chunk(60000, 1)
        q = config4_chunk(200, 62)
        lo, hi = shard_range(len(db), rank, world)
        sharded = ShardedFlatIndex(768, "ip", device=rank)
        sharded.add_range_device(torch.from_numpy(db[lo:hi]).cuda(), lo)
        d, lab = sharded.search_device(torch.from_numpy(q).cuda(), 100)
        full = qv.FlatIndex(768, "ip", device=rank)
        full.add(db)
        fl, fd = full.search(q, 100)
        out_q.put((rank, {"wide": (d.cpu().numpy(), lab.cpu().numpy(), fd, fl)}, None))
    except Exception as e:  # noqa: BLE001
        out_q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def _spawn(target, *extra):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, WORLD, port, q) + extra) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            rank, value, err = q.get(timeout=300)
            assert err is None, f"rank {rank}: {err}"
            res[rank] = value
    finally:
        for p in procs:
            p.join(timeout=120)
    return res


def _same(got_d, got_l, want_d, want_l, what):
    bad = np.argwhere((got_d != want_d) | (got_l.astype(np.int64) != want_l.astype(np.int64)))
    if bad.size:
        i = bad[0][0]
        raise AssertionError(f"{what}: {len(np.unique(bad[:, 0]))} queries differ; query {i}: "
                             f"got {got_d[i].tolist()} {got_l[i].tolist()} want "
                             f"{want_d[i].tolist()} {want_l[i].tolist()}")


def test_sharded_flat_equals_one_index():
    res = _spawn(_flat_worker)
    for rank in range(WORLD):
        for metric, (d, lab, fd, fl) in res[rank].items():
            _same(d, lab, fd, fl, f"rank {rank} {metric}")


@pytest.mark.parametrize("idx", range(3))
def test_sharded_ivf_equals_one_index(manifest, idx):
    res = _spawn(_ivf_worker, manifest["ivf"][idx])
    for rank in range(WORLD):
        for key, (d, lab, fd, fl) in res[rank].items():
            _same(d, lab, fd, fl, f"rank {rank} {key}")


def test_sharded_wide_flat_equals_one_index():
    res = _spawn(_wide_worker)
    for rank in range(WORLD):
        for key, (d, lab, fd, fl) in res[rank].items():
            _same(d, lab, fd, fl, f"rank {rank} {key}")
