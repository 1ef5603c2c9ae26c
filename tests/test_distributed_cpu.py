"""The multi-GPU plumbing on CPU: world_size-2 gloo process groups.

The sharded search (quiver_b200/distributed.py) splits the collection into id ranges, searches
each range on its own GPU, all-gathers every rank's (distance, key, label) lists and merges them
by (distance, key). These tests run that host-side logic with the gloo backend in two processes:
the id-range split, the all-gather helper, the IVF list-base exchange that makes shard-local
candidate keys equal the unsharded index's keys, and an end-to-end check that per-shard exact
top-k lists merged by (distance, key) reproduce the single-index top-k, including ties. The
device merge kernel itself is covered by the GPU tests.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn_name, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        out_q.put((rank, globals()[fn_name](rank, world), None))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        out_q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def _run(fn_name):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(r, WORLD, port, fn_name, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(WORLD):
        rank, value, err = q.get(timeout=120)
        assert err is None, f"rank {rank}: {err}"
        results[rank] = value
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return results


# ---- rank functions (module level so that spawn can import them) -------------------------------

def _gather_in_rank_order(rank, world):
    from quiver_b200.distributed import _all_gather
    t = torch.arange(6, dtype=torch.int64).reshape(2, 3) + 100 * rank
    return _all_gather(t, world, None).numpy()


def _list_bases(rank, world):
    from quiver_b200.distributed import list_bases
    sizes = torch.as_tensor(np.random.default_rng(rank).integers(0, 50, 16), dtype=torch.int64)
    return sizes.numpy(), list_bases(sizes, rank, world).numpy()


def _sharded_exact_topk(rank, world):
    """Each rank: exact L2 top-k over its id range with global ids as keys; all-gather; merge by
    (distance, key). Integer data makes ties frequent, so the key order is what is tested."""
    from quiver_b200.distributed import _all_gather_triples, shard_range
    rng = np.random.default_rng(5)
    n, nq, dim, k = 1001, 7, 6, 12
    db = rng.integers(0, 3, (n, dim)).astype(np.float32)
    q = rng.integers(0, 3, (nq, dim)).astype(np.float32)
    lo, hi = shard_range(n, rank, world)
    d = ((q[:, None, :] - db[None, lo:hi, :]) ** 2).sum(-1)
    keys = np.arange(lo, hi)
    order = np.lexsort((np.broadcast_to(keys, d.shape), d), axis=1)[:, :k]
    ld = np.take_along_axis(d, order, 1).astype(np.float32)
    lk = keys[order].astype(np.int64)
    gd, gk, gl = _all_gather_triples(torch.from_numpy(ld), torch.from_numpy(lk),
                                     torch.from_numpy(lk * 3 + 1), world, None)
    gd, gk = gd.numpy(), gk.numpy()
    assert np.array_equal(gl.numpy(), gk * 3 + 1)  # labels travel with their entries
    # merge by (distance, key) across ranks
    cd = np.concatenate(list(gd), axis=1)
    ck = np.concatenate(list(gk), axis=1)
    m = np.lexsort((ck, cd), axis=1)[:, :k]
    merged_d, merged_k = np.take_along_axis(cd, m, 1), np.take_along_axis(ck, m, 1)
    full = ((q[:, None, :] - db[None, :, :]) ** 2).sum(-1)
    fo = np.lexsort((np.broadcast_to(np.arange(n), full.shape), full), axis=1)[:, :k]
    return (merged_d, merged_k, np.take_along_axis(full, fo, 1).astype(np.float32), fo)


def _ivf_keys_match_unsharded(rank, world):
    """IVF keys: list << 32 | (entries of that list on lower ranks + offset in this shard's list)
    equal the offsets one index holding all rows in id order would give."""
    from quiver_b200.distributed import list_bases, shard_range
    rng = np.random.default_rng(9)
    n, nlist = 500, 8
    assign = rng.integers(0, nlist, n)
    lo, hi = shard_range(n, rank, world)
    mine = assign[lo:hi]
    sizes = torch.as_tensor(np.bincount(mine, minlength=nlist), dtype=torch.int64)
    base = list_bases(sizes, rank, world).numpy()
    seen = np.zeros(nlist, np.int64)
    keys = []
    for row, l in zip(range(lo, hi), mine):
        keys.append((row, (int(l) << 32) | int(base[l] + seen[l])))
        seen[l] += 1
    full_seen = np.zeros(nlist, np.int64)
    want = {}
    for row, l in enumerate(assign):
        want[row] = (int(l) << 32) | int(full_seen[l])
        full_seen[l] += 1
    return all(want[row] == key for row, key in keys)


def _query_slices_gathered(rank, world):
    """Rows replicated, queries split by rank: each rank answers its slice of an odd-sized batch
    (slices differ in length); the gathered answers come back in query order on every rank."""
    from quiver_b200.distributed import gather_query_slices, shard_range
    nq, k = 7, 3
    lo, hi = shard_range(nq, rank, world)
    rows = np.arange(lo, hi)
    d = torch.from_numpy((rows[:, None] * 10 + np.arange(k)[None, :]).astype(np.float32))
    lab = torch.from_numpy((rows[:, None] * 100 + np.arange(k)[None, :]).astype(np.int64))
    return gather_query_slices(d, lab, nq, world, None)


def _triples_bit_exact(rank, world):
    """The packed exchange keeps every bit: signed zeros, infinities, NaN payloads, keys and
    labels near 2^63 and the -1 padding."""
    from quiver_b200.distributed import _all_gather_triples
    d = torch.tensor([[0.5 + rank, float("inf"), -0.0], [float("nan"), -1e-38, 3.0]])
    key = torch.tensor([[2**62 + rank, -1, 5], [0, 2**63 - 1, -2]], dtype=torch.int64)
    lab = torch.tensor([[7, -1, 2**63 - 1 - rank], [1, 2, 3 + rank]], dtype=torch.int64)
    gd, gk, gl = _all_gather_triples(d, key, lab, world, None)
    return gd.view(torch.int32).numpy(), gk.numpy(), gl.numpy(), d.view(torch.int32).numpy()


def _collective_timeout_entry(rank, world, port, out_q):
    """Rank 1 never joins the collective; rank 0 must get an error from its group's short timeout
    instead of waiting for ever. The rendezvous itself has a long timeout (a spawned rank can take
    a while to import torch on a loaded host); the collective runs on a subgroup with a 2 s one."""
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=180))
        short = dist.new_group(list(range(world)), timeout=timedelta(seconds=2), backend="gloo")
    except Exception as e:  # noqa: BLE001 - reported to the test instead of a silent exit
        out_q.put((rank, "setup failed: " + repr(e), -1.0))
        os._exit(1)
    if rank == 1:
        time.sleep(8)  # absent from the collective until rank 0 has given up
        os._exit(0)
    t0 = time.time()
    try:
        from quiver_b200.distributed import _all_gather
        _all_gather(torch.zeros(4), world, short)
        out_q.put((rank, "no error", time.time() - t0))
    except Exception as e:  # noqa: BLE001 - the failure being tested
        out_q.put((rank, repr(e), time.time() - t0))
    os._exit(0)


# ---- tests ---------------------------------------------------------------------------------------

def test_shard_ranges_partition_the_ids():
    from quiver_b200.distributed import shard_range
    for n in (0, 1, 7, 1000, 1_183_514):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1


def test_all_gather_returns_ranks_in_order():
    res = _run("_gather_in_rank_order")
    for rank in range(WORLD):
        got = res[rank]
        assert got.shape == (WORLD, 2, 3)
        for r in range(WORLD):
            assert np.array_equal(got[r], np.arange(6).reshape(2, 3) + 100 * r)


def test_list_bases_are_exclusive_prefixes():
    res = _run("_list_bases")
    sizes = [res[r][0] for r in range(WORLD)]
    for r in range(WORLD):
        assert np.array_equal(res[r][1], sum((sizes[i] for i in range(r)), np.zeros(16, np.int64)))


def test_sharded_topk_merge_equals_single_index():
    res = _run("_sharded_exact_topk")
    for r in range(WORLD):
        md, mk, fd, fk = res[r]
        assert np.array_equal(md, fd)
        assert np.array_equal(mk, fk)


def test_ivf_shard_keys_equal_unsharded_keys():
    res = _run("_ivf_keys_match_unsharded")
    assert all(res[r] for r in range(WORLD))


def test_query_slices_gather_in_query_order():
    res = _run("_query_slices_gathered")
    want_d = (np.arange(7)[:, None] * 10 + np.arange(3)[None, :]).astype(np.float32)
    want_l = (np.arange(7)[:, None] * 100 + np.arange(3)[None, :]).astype(np.int64)
    for rank in range(WORLD):
        lab, d = res[rank]
        assert np.array_equal(d, want_d) and np.array_equal(lab, want_l)


def test_packed_triples_exchange_is_bit_exact():
    res = _run("_triples_bit_exact")
    for rank in range(WORLD):
        gd, gk, gl, _ = res[rank]
        for r in range(WORLD):
            assert np.array_equal(gd[r], res[r][3])
            assert gk[r, 0, 0] == 2**62 + r and gk[r, 0, 1] == -1 and gk[r, 1, 1] == 2**63 - 1
            assert gl[r, 0, 2] == 2**63 - 1 - r and gl[r, 1, 2] == 3 + r


def test_a_rank_missing_from_a_collective_is_detected_by_timeout():
    """Failure detection on the host: a rank that never arrives makes the other rank's collective
    fail after the process group's short timeout (no GPU involved)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_collective_timeout_entry, args=(r, WORLD, port, q))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    # Generous: the spawned ranks first import torch, slow on a loaded host; the failure latency
    # itself is measured inside the rank (`waited`).
    rank, err, waited = q.get(timeout=240)
    assert not err.startswith("setup failed"), err
    assert rank == 0 and err != "no error", "the collective returned without its peer"
    assert waited < 30, f"the failure took {waited:.1f} s to surface"
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
