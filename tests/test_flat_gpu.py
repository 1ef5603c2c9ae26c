"""FlatIndex on the GPU through the C ABI, against the reference's golden outputs and the oracle.

Distances must be bit-identical to the reference's (the GPU re-ranks in the reference's own float
summation order) and labels identical except among tied distances."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden_flat_inputs
from parity import assert_sorted, assert_topk_parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("idx", range(6))
def test_flat_matches_reference_golden(gpu, manifest, idx):
    case = manifest["flat"][idx]
    base, q, labels = golden_flat_inputs(case)
    g = np.load(os.path.join(GOLDEN, case["name"] + ".npz"))
    ix = gpu.FlatIndex(case["dim"], case["metric"])
    ix.add(base, labels)
    l, d = ix.search(q, case["k"])
    assert_sorted(d)
    assert_topk_parity(l, d, g["labels"], g["dists"], exact=True, what=case["name"])
    l, d = ix.search(q, case["k"], filter=g["filt_allowed"])
    assert_topk_parity(l, d, g["filt_labels"], g["filt_dists"], exact=True, what="filtered")
    l, d = ix.search(q[:3], case["n"] + 5) if case["n"] + 5 <= 1024 else (None, None)
    if l is not None:
        assert_topk_parity(l, d, g["all_labels"], g["all_dists"], exact=True, what="k>n")


@pytest.mark.parametrize("metric", ["l2", "ip", "cosine"])
@pytest.mark.parametrize("dim", [1, 13, 100, 128, 129, 768])
def test_flat_matches_oracle_shapes(gpu, oracle, metric, dim):
    rng = np.random.default_rng(dim * 7 + len(metric))
    n = 777 if dim < 700 else 300
    base = rng.standard_normal((n, dim)).astype(np.float32)
    q = rng.standard_normal((19, dim)).astype(np.float32)
    labels = rng.permutation(n).astype(np.uint64) * 5
    ix = gpu.FlatIndex(dim, metric)
    ix.add(base[: n // 2], labels[: n // 2])
    ix.add(base[n // 2:], labels[n // 2:])  # two adds: appends keep row order
    stored = oracle.normalize_rows(base) if metric == "cosine" else base
    v, la = ix.rows()
    assert np.array_equal(v, stored) and np.array_equal(la, labels)
    for k in (1, 10, 64):
        l, d = ix.search(q, k)
        wl, wd = oracle.flat_search(stored, labels, metric, q, k)
        assert_topk_parity(l, d, wl, wd, exact=True, what=f"{metric} d={dim} k={k}")


def test_known_answer(gpu):
    # tests/test_flat.cc:37-52 of the reference.
    base = np.array([[1, 0, 0, 0], [0, 2, 0, 0], [1, 1, 0, 0]], np.float32)
    q = np.array([3, 0.1, 0, 0], np.float32)
    cos = gpu.FlatIndex(4, "cosine")
    cos.add(base)
    l, d = cos.search(q, 3)
    assert l[0, 0] == 0 and abs(d[0, 0] - (1 - 3 / np.sqrt(9.01))) < 1e-5
    ip = gpu.FlatIndex(4, "ip")
    ip.add(base)
    l, d = ip.search(q, 3)
    assert l[0, 0] == 2 and abs(d[0, 0] - (1 - 3.1)) < 1e-5


def test_fewer_than_k_and_filters(gpu):
    # tests/test_flat.cc:54-72 of the reference.
    x = np.random.default_rng(3).standard_normal((10, 8)).astype(np.float32)
    ix = gpu.FlatIndex(8)
    ix.add(x, labels=np.arange(100, 110))
    l, d = ix.search(x[:1], 50)
    assert (l[0] >= 0).sum() == 10 and np.isinf(d[0, 10:]).all()
    l, d = ix.search(x[:1], 5, filter={103, 107})
    assert set(l[0, :2].tolist()) <= {103, 107} and l[0, 2] == -1 and np.isinf(d[0, 4])
    l, _ = ix.search(x[:2], 3, filter=[])
    assert (l == -1).all()
    l, _ = ix.search(x[:1], 3, filter=[2**62])  # sparse labels take the label-set path
    assert (l == -1).all()


def test_empty_index_and_errors(gpu, monkeypatch):
    ix = gpu.FlatIndex(4)
    l, d = ix.search(np.ones((2, 4)), 3)
    assert (l == -1).all() and np.isinf(d).all()
    with pytest.raises(ValueError, match="NaN"):
        ix.add(np.array([[1, np.nan, 0, 0]], np.float32))
    with pytest.raises(ValueError, match="NaN"):
        ix.search(np.array([[1, np.inf, 0, 0]], np.float32), 1)
    # With rows stored the device search itself detects the non-finite query (and copies no
    # results out); both the tensor-core and the SIMT screen paths.
    full = gpu.FlatIndex(4)
    full.add(np.random.default_rng(1).standard_normal((300, 4)).astype(np.float32))
    for screen in ("", "simt"):
        monkeypatch.setenv("QV_FLAT_SCREEN", screen)
        for bad in (np.nan, np.inf, -np.inf):
            q = np.ones((20, 4), np.float32)
            q[7, 2] = bad
            with pytest.raises(ValueError, match="NaN"):
                full.search(q, 3)
        l, _ = full.search(np.ones((20, 4), np.float32), 3)  # the index stays usable
        assert (l >= 0).all()
    monkeypatch.delenv("QV_FLAT_SCREEN")
    with pytest.raises(ValueError, match="2\\*\\*63"):
        ix.add(np.zeros((1, 4)), labels=[2**63])
    with pytest.raises(ValueError, match="dimension"):
        ix.add(np.zeros((1, 5)))
    with pytest.raises(ValueError):
        gpu.FlatIndex(0)
    with pytest.raises(ValueError):
        gpu.FlatIndex(4, metric="hamming")


def test_uncertified_queries_take_the_exact_rescan(gpu, oracle, monkeypatch):
    """Integer data has exact distance ties; with a candidate budget of k the certificate cannot
    separate the boundary, so those queries must be answered by the exact rescan."""
    from quiver_b200.synthetic import skewed_ints
    base = skewed_ints(4000, 16, 3)
    base[:, 8:] = 0  # many equal distances
    q = skewed_ints(25, 16, 4)
    q[:, 8:] = 0
    labels = np.arange(4000, dtype=np.uint64)
    ix = gpu.FlatIndex(16)
    ix.add(base)
    monkeypatch.setenv("QV_FLAT_KK", "10")
    l, d = ix.search(q, 10)
    stats = gpu.last_search_stats()
    assert stats["rescanned_queries"] > 0
    wl, wd = oracle.flat_search(base, labels, "l2", q, 10)
    assert_topk_parity(l, d, wl, wd, exact=True, what="rescan")


@pytest.mark.parametrize("k,filtered", [(10, False), (10, True), (300, False)])
def test_rescan_split_over_row_slices(gpu, oracle, monkeypatch, k, filtered):
    """Uncertified queries over 60,000 rows: each is rescanned by several blocks over row slices
    (per-slice k best, then a merge), with exact ties at the boundary, a label filter and a large
    k (fewer slices); the results equal the oracle's."""
    from quiver_b200.synthetic import skewed_ints
    base = skewed_ints(60000, 16, 13)
    base[:, 6:] = 0  # many equal distances
    q = skewed_ints(40, 16, 14)
    q[:, 6:] = 0
    labels = np.arange(60000, dtype=np.uint64)
    allowed = np.random.default_rng(15).choice(60000, 20000, replace=False).astype(np.uint64) \
        if filtered else None
    ix = gpu.FlatIndex(16)
    ix.add(base)
    monkeypatch.setenv("QV_FLAT_KK", str(k))
    gpu._native.set_timing(True)
    l, d = ix.search(q, k, filter=allowed)
    stats = gpu.last_search_stats()
    gpu._native.set_timing(False)
    assert stats["rescanned_queries"] > 0
    wl, wd = oracle.flat_search(base, labels, "l2", q, k, allowed=allowed)
    assert_topk_parity(l, d, wl, wd, exact=True, what=f"sliced rescan k={k}")


def test_save_load_roundtrip_and_reference_format(gpu, tmp_path, reference):
    x = np.random.default_rng(4).standard_normal((100, 16)).astype(np.float32)
    ix = gpu.FlatIndex(16, "cosine")
    ix.add(x)
    ix.save(tmp_path / "flat.qvr")
    back = gpu.FlatIndex.load(tmp_path / "flat.qvr")
    assert len(back) == 100 and back.metric == "cosine"
    assert np.array_equal(back.search(x, 5)[0], ix.search(x, 5)[0])
    # a file written by the reference library loads and searches identically
    rf = reference.flat(16, "cosine")
    rf.add(x)
    rf.save(tmp_path / "ref.qvr")
    from_ref = gpu.FlatIndex.load(tmp_path / "ref.qvr")
    rl, rd = rf.search(x, 5)
    l, d = from_ref.search(x, 5)
    assert_topk_parity(l, d, rl, rd, exact=True, what="reference .qvr")


def test_config0_full_size_against_reference(gpu, reference):
    """Benchmark config 0 at its full size (100k x 128 skewed ints, 1,000 queries, k=10)."""
    from quiver_b200.synthetic import config0
    base, q = config0()
    ix = gpu.FlatIndex(128, "l2")
    ix.add(base)
    l, d = ix.search(q, 10)
    rf = reference.flat(128, "l2")
    rf.add(base)
    rl, rd = rf.search(q, 10)
    assert_topk_parity(l, d, rl, rd, exact=True, what="config0")


# The MMAs take ceil(dim / 16) K-steps of 16: dims 20, 40 and 50 take 2, 3 and 4 in one
# 64-column atom; 72, 96, 100 and 128 take 5, 6, 7 and 8 in two.
@pytest.mark.parametrize("metric,dim,pair", [
    ("l2", 100, "0"), ("ip", 100, "0"), ("cosine", 100, "0"), ("l2", 50, "0"), ("ip", 72, "0"),
    ("cosine", 96, "0"), ("l2", 128, "0"), ("ip", 40, "0"), ("cosine", 20, "0"),
    ("cosine", 100, "1"), ("l2", 128, "1"), ("ip", 40, "1")])
def test_tensor_core_screen_equals_simt_screen(gpu, oracle, monkeypatch, metric, dim, pair):
    """The tcgen05 fp16 screen (in single CTAs, and in CTA pairs with QV_TC_PAIR=1) and the
    float32 SIMT screen must produce identical final results (both are re-ranked exactly and
    certified)."""
    monkeypatch.setenv("QV_TC_PAIR", pair)
    from quiver_b200.synthetic import mixture
    base = mixture(20000, dim, 50, 0.35, 1.0, centre_seed=3, seed=4)
    if metric != "cosine":
        base = base * np.float32(3.0)
    q = mixture(300, dim, 50, 0.35, 1.0, centre_seed=3, seed=5)
    ix = gpu.FlatIndex(dim, metric)
    ix.add(base)
    stored = oracle.normalize_rows(base) if metric == "cosine" else base
    for k in (10, 20):  # best lists of 24 and of 32 groups
        monkeypatch.delenv("QV_FLAT_SCREEN", raising=False)
        gpu._native.set_timing(True)
        l1, d1 = ix.search(q, k)
        st = gpu.last_search_stats()
        gpu._native.set_timing(False)
        assert st["dominant_kernel"] == "flat_screen_tc_kernel"
        monkeypatch.setenv("QV_FLAT_SCREEN", "simt")
        l2_, d2 = ix.search(q, k)
        assert np.array_equal(d1, d2) and np.array_equal(l1, l2_)
        wl, wd = oracle.flat_search(stored, np.arange(20000, dtype=np.uint64), metric, q, k)
        assert_topk_parity(l1, d1, wl, wd, exact=True, what=f"tc {metric} k={k}")


def test_device_searches_are_asynchronous_and_ordered(gpu, oracle):
    """qv_flat_search_device only enqueues: two searches queued back to back on one stream (and
    a third on the CUDA default stream, NULL) all return correct results after one
    synchronization; a query holding NaN gets no results (QV_INVALID_LABEL, NaN distance) and the
    other queries of its batch are answered."""
    import ctypes as C
    import torch
    from quiver_b200.synthetic import mixture
    base = mixture(50_000, 100, 80, 0.35, 1.0, centre_seed=9, seed=10)
    ix = gpu.FlatIndex(100, "cosine")
    ix.add(base)
    lib = gpu.lib()
    stream = torch.cuda.Stream()
    batches = [mixture(nq, 100, 80, 0.35, 1.0, centre_seed=9, seed=s)
               for nq, s in [(700, 11), (333, 12), (64, 13)]]
    batches[1][5, 7] = np.nan
    outs = []
    for i, q in enumerate(batches):
        dq = torch.from_numpy(q).cuda()
        lab = torch.empty((len(q), 10), dtype=torch.int64, device="cuda")
        dst = torch.empty((len(q), 10), dtype=torch.float32, device="cuda")
        s = C.c_void_p(stream.cuda_stream) if i < 2 else None
        if i < 2:
            stream.wait_stream(torch.cuda.current_stream())
        gpu._native.check(lib.qv_flat_search_device(ix.handle, dq.data_ptr(), len(q), 10, None,
                                                    lab.data_ptr(), dst.data_ptr(), None, s))
        outs.append((dq, lab, dst))
    torch.cuda.synchronize()
    stored = oracle.normalize_rows(base)
    ids = np.arange(len(base), dtype=np.uint64)
    for i, (q, (_, lab, dst)) in enumerate(zip(batches, outs)):
        l, d = lab.cpu().numpy(), dst.cpu().numpy()
        good = np.isfinite(q).all(axis=1)
        wl, wd = oracle.flat_search(stored, ids, "cosine", q[good], 10)
        assert_topk_parity(l[good], d[good], wl, wd, exact=True, what=f"async batch {i}")
        assert (l[~good] == -1).all() and np.isnan(d[~good]).all()


def test_add_from_device_memory_equals_host_add(gpu):
    """reserve + add_device (rows already on the GPU, added in chunks) store exactly what add()
    stores, search identically, and reject NaN values and the reserved label as add() does."""
    import torch
    rng = np.random.default_rng(21)
    x = rng.standard_normal((5000, 72)).astype(np.float32)
    labels = rng.permutation(5000).astype(np.uint64) * 3
    host = gpu.FlatIndex(72, "cosine")
    host.add(x, labels)
    dev = gpu.FlatIndex(72, "cosine")
    dev.reserve(5000)
    dx = torch.from_numpy(x).cuda()
    dl = torch.from_numpy(labels.astype(np.int64)).cuda()
    dev.add_device(dx[:1234], dl[:1234])
    dev.add_device(dx[1234:], dl[1234:])
    hv, hl = host.rows()
    dv, dlab = dev.rows()
    assert np.array_equal(hv, dv) and np.array_equal(hl, dlab)
    q = rng.standard_normal((50, 72)).astype(np.float32)
    a, b = host.search(q, 10), dev.search(q, 10)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    seq = gpu.FlatIndex(72, "l2")
    seq.add_device(dx[:10])  # no labels: size() + i
    assert np.array_equal(seq.rows()[1], np.arange(10, dtype=np.uint64))
    bad = dx[:4].clone()
    bad[2, 3] = float("nan")
    with pytest.raises(ValueError, match="NaN"):
        dev.add_device(bad)
    with pytest.raises(ValueError, match="2\\^64-1"):
        dev.add_device(dx[:2], torch.tensor([1, -1], dtype=torch.int64, device="cuda"))
    assert len(dev) == 5000  # a rejected add leaves the index unchanged


@pytest.mark.parametrize("dim", [100, 256])  # the narrow and the wide tensor-core screens
def test_screen_barrier_timeout_is_reported_and_the_index_stays_usable(gpu, oracle, monkeypatch,
                                                                        dim):
    """Failure detection without a GPU fault: the test hook makes CTA 0's TMA producer skip one
    ring fill, so the MMA issuer's bounded barrier wait (shortened to 2 ms) runs out. The kernel
    must raise its error word, drain its work in flight, free TMEM and exit; the search reports
    QV_ERR_DEVICE (its queries were answered by the exact rescan), and the next search on the
    same index and context is exact."""
    from quiver_b200.synthetic import mixture
    base = mixture(20000, dim, 50, 0.35, 1.0, centre_seed=3, seed=4)
    q = mixture(300, dim, 50, 0.35, 1.0, centre_seed=3, seed=5)
    ix = gpu.FlatIndex(dim, "cosine")
    ix.add(base)
    monkeypatch.setenv("QV_TC_WAIT_LIMIT_US", "2000")
    monkeypatch.setenv("QV_TC_TEST_SKIP_FILL", "2")
    with pytest.raises(RuntimeError, match="timed out"):
        ix.search(q, 10)
    monkeypatch.delenv("QV_TC_TEST_SKIP_FILL")
    monkeypatch.delenv("QV_TC_WAIT_LIMIT_US")
    gpu._native.set_timing(True)
    l, d = ix.search(q, 10)
    st = gpu.last_search_stats()
    gpu._native.set_timing(False)
    assert st["dominant_kernel"].startswith("flat_screen_tc")
    wl, wd = oracle.flat_search(oracle.normalize_rows(base), np.arange(20000, dtype=np.uint64),
                                "cosine", q, 10)
    assert_topk_parity(l, d, wl, wd, exact=True, what="after a screen timeout")


@pytest.mark.parametrize("pair", ["0", "1"])
@pytest.mark.parametrize("metric,dim,k", [("ip", 768, 100), ("l2", 256, 10), ("cosine", 520, 40)])
def test_wide_screen_equals_simt_screen(gpu, oracle, monkeypatch, pair, metric, dim, k):
    """The wide tensor-core screen (dim > 128 or k > 24), in single CTAs and in CTA pairs
    (tcgen05 cta_group::2), gives the SIMT screen's exact results. (Queries its certificate
    cannot prove complete, when distances near rank k are packed within the screen's error
    bound, are answered by the exact rescan: the results are exact either way.)"""
    from quiver_b200.synthetic import mixture
    base = mixture(30000, dim, 40, 0.35, 1.0, centre_seed=5, seed=6)
    if metric == "l2":
        base = base * np.float32(2.0)
    q = mixture(257, dim, 40, 0.35, 1.0, centre_seed=5, seed=7)
    ix = gpu.FlatIndex(dim, metric)
    ix.add(base)
    monkeypatch.setenv("QV_TC_WIDE_PAIR", pair)
    gpu._native.set_timing(True)
    l1, d1 = ix.search(q, k)
    st = gpu.last_search_stats()
    gpu._native.set_timing(False)
    assert st["dominant_kernel"] == "flat_screen_tc_wide_kernel"
    assert st["rescanned_queries"] < len(q) // 4
    monkeypatch.setenv("QV_FLAT_SCREEN", "simt")
    l2_, d2 = ix.search(q, k)
    assert np.array_equal(d1, d2) and np.array_equal(l1, l2_)
