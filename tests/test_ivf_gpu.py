"""IvfPqIndex on the GPU through the C ABI: bit-exact assignments and PQ codes against the
reference-trained .qvr fixtures, and search parity (nprobe sweep, refine, filter) against the
reference's golden outputs and the oracle."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden_ivf_inputs
from parity import assert_sorted, assert_topk_parity

pytestmark = pytest.mark.gpu


def _qvr(case):
    return os.path.join(GOLDEN, case["name"] + ".qvr")


@pytest.mark.parametrize("idx", range(3))
def test_encode_bit_exact_against_reference_qvr(gpu, manifest, idx):
    from oracle.oracle import QvrIvf
    case = manifest["ivf"][idx]
    base, _ = golden_ivf_inputs(case)
    qv = QvrIvf(_qvr(case))
    ix = gpu.IvfPqIndex.load(_qvr(case))
    assign, codes = ix.encode(base)
    order = np.argsort(qv.labels)
    assert np.array_equal(qv.assignments()[order], assign)
    assert np.array_equal(qv.codes[order], codes)
    # add() through the GPU reproduces the reference's lists exactly (order, codes, labels)
    fresh = gpu.IvfPqIndex(case["dim"], case["metric"], case["nlist"], case["m"],
                           store_vectors=True)
    fresh.set_trained(qv.centroids, qv.codebooks)
    fresh.add(base[:700])
    fresh.add(base[700:])
    assert fresh.list_sizes() == [int(x) for x in np.diff(qv.offsets)]
    assert np.array_equal(fresh.stored_labels(), qv.labels)


@pytest.mark.parametrize("idx", range(3))
@pytest.mark.parametrize("store_vectors", [True, False])
def test_streamed_add_equals_reference(gpu, manifest, tmp_path, monkeypatch, idx, store_vectors):
    """add() streams its rows in chunks (here 333 rows, so the last chunk is ragged and both pinned
    staging halves are reused); the lists, codes, labels and stored vectors equal the reference's
    .qvr exactly, with and without stored vectors (src/ivfpq_index.cc:208-271)."""
    from oracle.oracle import QvrIvf
    case = manifest["ivf"][idx]
    base, q = golden_ivf_inputs(case)
    qv = QvrIvf(_qvr(case))
    monkeypatch.setenv("QV_IVF_ADD_CHUNK_ROWS", "333")
    ix = gpu.IvfPqIndex(case["dim"], case["metric"], case["nlist"], case["m"],
                        store_vectors=store_vectors)
    ix.set_trained(qv.centroids, qv.codebooks)
    ix.add(base[:1500])
    ix.add(base[1500:])
    ix.save(tmp_path / "streamed.qvr")
    got = QvrIvf(tmp_path / "streamed.qvr")
    assert np.array_equal(got.offsets, qv.offsets)
    assert np.array_equal(got.labels, qv.labels)
    assert np.array_equal(got.codes, qv.codes)
    if store_vectors:
        assert np.array_equal(got.vectors, qv.vectors)
    assign, codes = ix.encode(base)  # encode() streams the same way
    order = np.argsort(qv.labels)
    assert np.array_equal(qv.assignments()[order], assign)
    assert np.array_equal(qv.codes[order], codes)


@pytest.mark.parametrize("idx", range(3))
def test_search_matches_reference_golden(gpu, manifest, idx):
    case = manifest["ivf"][idx]
    _, q = golden_ivf_inputs(case)
    g = np.load(os.path.join(GOLDEN, case["name"] + "_search.npz"))
    ix = gpu.IvfPqIndex.load(_qvr(case))
    for nprobe, rf in case["searches"]:
        l, d = ix.search(q, 10, nprobe=nprobe, refine_factor=rf)
        assert_sorted(d)
        assert_topk_parity(l, d, g[f"labels_{nprobe}_{rf}"], g[f"dists_{nprobe}_{rf}"],
                           exact=True, what=f"{case['name']} nprobe={nprobe} rf={rf}")
    l, d = ix.search(q, 10, nprobe=case["filter_nprobe"], filter=g["filt_allowed"])
    assert_topk_parity(l, d, g["filt_labels"], g["filt_dists"], exact=True, what="filtered")
    assert np.isin(l[l >= 0], g["filt_allowed"].astype(np.int64)).all()
    l, d = ix.search(q[:5], 10, nprobe=case["nlist"], refine_factor=1 << 62)
    assert_topk_parity(l, d, g["sat_labels"], g["sat_dists"], exact=True, what="saturated keep")


@pytest.mark.parametrize("metric", ["l2", "ip", "cosine"])
def test_search_matches_oracle_larger(gpu, oracle, reference, tmp_path, metric):
    from oracle.oracle import QvrIvf
    from quiver_b200.synthetic import clustered
    base = clustered(20000, 64, 30, 5)
    q = clustered(200, 64, 30, 6)
    r = reference.ivf(64, metric, 128, 16, store_vectors=True, train_iterations=6)
    r.train(base[:8000])
    r.add(base)
    path = tmp_path / "ix.qvr"
    r.save(path)
    qv = QvrIvf(path)
    ix = gpu.IvfPqIndex.load(path)
    for nprobe, rf in [(1, 0), (8, 0), (32, 4), (128, 1)]:
        l, d = ix.search(q, 10, nprobe=nprobe, refine_factor=rf)
        wl, wd = oracle.ivf_search(qv, q, 10, nprobe, rf)
        assert_topk_parity(l, d, wl, wd, exact=True, what=f"{metric} {nprobe} {rf}")
        rl, rd = r.search(q, 10, nprobe, rf)
        assert_topk_parity(l, d, rl, rd, exact=True, what=f"ref {metric} {nprobe} {rf}")


def test_errors_and_roundtrip(gpu, tmp_path, manifest):
    case = manifest["ivf"][0]
    base, q = golden_ivf_inputs(case)
    ix = gpu.IvfPqIndex(case["dim"], "l2", nlist=case["nlist"], m=case["m"], store_vectors=True)
    assert not ix.is_trained
    with pytest.raises(ValueError, match="trained"):
        ix.add(base[:3])
    with pytest.raises(ValueError, match="max\\(nlist, 256\\)"):
        ix.train(base[:100])  # too few rows (src/ivfpq_index.cc:145)
    with pytest.raises(ValueError):
        gpu.IvfPqIndex(10, m=3)
    l, d = ix.search(q[:2], 4)
    assert (l == -1).all() and np.isinf(d).all()
    loaded = gpu.IvfPqIndex.load(_qvr(case))
    loaded.save(tmp_path / "again.qvr")
    again = gpu.IvfPqIndex.load(tmp_path / "again.qvr")
    assert again.list_sizes() == loaded.list_sizes() and len(again) == len(loaded)
    a = again.search(q, 5, nprobe=8, refine_factor=2)
    b = loaded.search(q, 5, nprobe=8, refine_factor=2)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    l, _ = loaded.search(base[5], 1, nprobe=case["nlist"], refine_factor=2)
    assert l[0, 0] == 5  # self-match (tests/test_quantizer.cc:258)
    # Non-finite queries are rejected (src/ivfpq_index.cc:428) by a trained, filled index and by
    # an untrained one; the index stays usable.
    for bad in (np.nan, np.inf):
        qb = q[:6].copy()
        qb[3, 1] = bad
        with pytest.raises(ValueError, match="NaN"):
            loaded.search(qb, 5, nprobe=8, refine_factor=2)
        with pytest.raises(ValueError, match="NaN"):
            ix.search(qb, 5)
    c = loaded.search(q, 5, nprobe=8, refine_factor=2)
    assert np.array_equal(c[0], b[0]) and np.array_equal(c[1], b[1])
    assert loaded.memory_bytes > 0


def test_sharded_load_merges_to_unsharded(gpu, manifest):
    """Two id-range shards of one .qvr, candidates merged, equal the unsharded search."""
    import ctypes as C
    import torch
    case = manifest["ivf"][2]
    _, q = golden_ivf_inputs(case)
    whole = gpu.IvfPqIndex.load(_qvr(case))
    n = len(whole)
    shards = [gpu.IvfPqIndex.load(_qvr(case), label_range=(0, n // 2)),
              gpu.IvfPqIndex.load(_qvr(case), label_range=(n // 2, n))]
    assert len(shards[0]) + len(shards[1]) == n
    lib = gpu.lib()
    keep, nq = 10, q.shape[0]
    dq = torch.from_numpy(q).cuda()
    parts_d = torch.empty((2, nq, keep), dtype=torch.float32, device="cuda")
    parts_k = torch.empty((2, nq, keep), dtype=torch.int64, device="cuda")
    parts_l = torch.empty((2, nq, keep), dtype=torch.int64, device="cuda")
    for i, s in enumerate(shards):
        gpu._native.check(lib.qv_ivfpq_candidates_device(
            s.handle, dq.data_ptr(), nq, keep, 8, None, parts_d[i].data_ptr(),
            parts_k[i].data_ptr(), parts_l[i].data_ptr(), None))
    od = torch.empty((nq, keep), dtype=torch.float32, device="cuda")
    ol = torch.empty((nq, keep), dtype=torch.int64, device="cuda")
    ok = torch.empty((nq, keep), dtype=torch.int64, device="cuda")
    gpu._native.check(lib.qv_merge_topk_device(0, 2, nq, keep, parts_d.data_ptr(),
                                               parts_k.data_ptr(), parts_l.data_ptr(),
                                               od.data_ptr(), ok.data_ptr(), ol.data_ptr(), None))
    torch.cuda.synchronize()
    wl, wd = whole.search(q, keep, nprobe=8)
    assert_topk_parity(ol.cpu().numpy(), od.cpu().numpy(), wl, wd, exact=True, what="sharded")


def test_many_lists_probe_selection(gpu, oracle, tmp_path):
    """nlist = 40,000: the probe selection reads its composites from global memory (too many
    lists for shared memory); results equal the oracle's on the saved index."""
    from oracle.oracle import QvrIvf
    rng = np.random.default_rng(17)
    dim, nlist, m = 16, 40_000, 4
    cents = rng.standard_normal((nlist, dim)).astype(np.float32)
    books = rng.standard_normal((m, 256, dim // m)).astype(np.float32) * np.float32(0.3)
    base = (cents[rng.integers(0, nlist, 60_000)] +
            rng.standard_normal((60_000, dim)).astype(np.float32) * np.float32(0.2))
    q = cents[rng.integers(0, nlist, 64)] + rng.standard_normal((64, dim)).astype(np.float32) * 0.2
    q = q.astype(np.float32)
    ix = gpu.IvfPqIndex(dim, "l2", nlist, m, store_vectors=True)
    ix.set_trained(cents, books)
    ix.add(base)
    path = tmp_path / "many.qvr"
    ix.save(path)
    qv = QvrIvf(path)
    for nprobe, rf in [(1, 0), (16, 0), (40, 2)]:
        l, d = ix.search(q, 10, nprobe=nprobe, refine_factor=rf)
        wl, wd = oracle.ivf_search(qv, q, 10, nprobe, rf)
        assert_topk_parity(l, d, wl, wd, exact=True, what=f"nlist {nlist} nprobe {nprobe} {rf}")


@pytest.mark.parametrize("metric,n,nlist,m,iters", [("l2", 20000, 128, 16, 6),
                                                    ("cosine", 9000, 16, 8, 5),
                                                    ("ip", 70000, 64, 4, 3)])
def test_train_bit_exact_against_reference(gpu, reference, tmp_path, metric, n, nlist, m, iters):
    """IvfPqIndex::train with the assignments on the GPU gives the reference's coarse centroids
    and PQ codebooks bit for bit (src/ivfpq_index.cc:144-206, src/product_quantizer.cc:29-153):
    empty clusters split (nlist 128 over 30 clusters), the k * 256 subsample (nlist 16 and 64),
    cosine normalization, and the 65,536-row PQ subsample with inner-product cells (n = 70,000).
    The trained index then adds and searches like the reference's."""
    from oracle.oracle import QvrIvf
    from quiver_b200.synthetic import clustered
    base = clustered(n, 64, 30, 5)
    q = clustered(64, 64, 30, 6)
    ix = gpu.IvfPqIndex(64, metric, nlist, m, store_vectors=True, train_iterations=iters, seed=77)
    ix.train(base)
    assert ix.is_trained
    with pytest.raises(ValueError, match="already trained"):
        ix.train(base)
    r = reference.ivf(64, metric, nlist, m, store_vectors=True, train_iterations=iters, seed=77)
    r.train(base)
    ix.save(tmp_path / "gpu.qvr")
    r.save(tmp_path / "ref.qvr")
    g, w = QvrIvf(tmp_path / "gpu.qvr"), QvrIvf(tmp_path / "ref.qvr")
    assert np.array_equal(g.centroids, w.centroids), "coarse centroids differ"
    assert np.array_equal(g.codebooks, w.codebooks), "PQ codebooks differ"
    ix.add(base[:5000])
    r.add(base[:5000])
    l, d = ix.search(q, 10, nprobe=8, refine_factor=2)
    rl, rd = r.search(q, 10, 8, 2)
    assert_topk_parity(l, d, rl, rd, exact=True, what=f"trained {metric}")


@pytest.mark.parametrize("metric", ["l2", "ip", "cosine"])
def test_coarse_probe_paths_agree_with_ties(gpu, oracle, tmp_path, monkeypatch, metric):
    """The coarse probe's two paths (the centroid table searched as an exact Flat index on the
    tensor cores, and the float32 distance table with the radix selection, QV_IVF_COARSE=simt)
    pick the same lists with the same distances, including among exactly tied centroids (each
    centroid row appears four times, and some queries sit on a centroid): ties go to the lower
    list id, as CentroidTable's stable selection does (src/ivfpq_index.cc:285-297). Both equal
    the oracle."""
    from oracle.oracle import QvrIvf
    rng = np.random.default_rng(41)
    dim, nlist, m = 32, 256, 8
    distinct = rng.standard_normal((nlist // 4, dim)).astype(np.float32)
    cents = distinct[rng.permutation(np.repeat(np.arange(nlist // 4), 4))]
    books = rng.standard_normal((m, 256, dim // m)).astype(np.float32) * 0.3
    base = (cents[rng.integers(0, nlist, 6000)] +
            rng.standard_normal((6000, dim)).astype(np.float32) * 0.2)
    q = np.concatenate([cents[rng.integers(0, nlist, 40)],
                        rng.standard_normal((160, dim)).astype(np.float32)])
    if metric == "cosine":  # centroids of a cosine index are trained on normalized rows
        cents = cents / np.linalg.norm(cents, axis=1, keepdims=True)
    ix = gpu.IvfPqIndex(dim, metric, nlist, m, store_vectors=True)
    ix.set_trained(cents, books)
    ix.add(base)
    ix.save(tmp_path / "ties.qvr")
    qv = QvrIvf(tmp_path / "ties.qvr")
    for nprobe, rf in [(1, 0), (3, 0), (8, 2), (24, 0)]:
        monkeypatch.delenv("QV_IVF_COARSE", raising=False)
        tl, td = ix.search(q, 10, nprobe=nprobe, refine_factor=rf)
        monkeypatch.setenv("QV_IVF_COARSE", "simt")
        sl, sd = ix.search(q, 10, nprobe=nprobe, refine_factor=rf)
        what = f"{metric} nprobe {nprobe} rf {rf}"
        assert np.array_equal(tl, sl), what
        assert np.array_equal(td.view(np.uint32), sd.view(np.uint32)), what
        wl, wd = oracle.ivf_search(qv, q, 10, nprobe, rf)
        assert_topk_parity(tl, td, wl, wd, exact=True, what="oracle " + what)
    # add()'s assignment takes the same two paths (CentroidTable::nearest_batch: ||c||^2 - 2<x,c>,
    # or -<x,c> for the inner-product metric); rows sitting on a centroid tie with its copies.
    rows = np.concatenate([cents[rng.integers(0, nlist, 300)], base[:700]])
    monkeypatch.delenv("QV_IVF_COARSE", raising=False)
    ta, tc_codes = ix.encode(rows)
    monkeypatch.setenv("QV_IVF_COARSE", "simt")
    sa, s_codes = ix.encode(rows)
    assert np.array_equal(ta, sa) and np.array_equal(tc_codes, s_codes)
    # the index's lists (filled by add() on the default path) hold the same cells
    assert np.array_equal(qv.assignments()[np.argsort(qv.labels)][:700], sa[300:])
