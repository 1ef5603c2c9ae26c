"""Parity at the benchmarked sizes: every workload bench.py measures is built here exactly as the
bench builds it and compared with the reference library itself (oracle/_ref, the reference's own
sources compiled on this host), on a query subset where the reference would take minutes.

* Benchmark config 1 (Flat cosine, 1,183,514 x 100 mixture, k=10): the whole 10k batch on the
  tensor-core screen equals the float32 SIMT screen bit for bit; 512 queries equal the reference.
* Config 2 (IVF-PQ L2, nlist 2048, m 32) and config 3 (cosine, m 25, refine 8): the reference-trained
  empty index, the full database added on the GPU; stored lists, codes and vectors equal the
  reference's own add() of the same rows byte for byte (compared in the .qvr files both write, and
  the GPU-written file is loaded and searched by the reference library); searches equal the
  reference's at every nprobe the bench sweeps, with refine 8 and the 1 % id filter for config 3.
* Flat k=100 at dim 768 (config 4's shape), inner product.

Distances are compared bit for bit; labels may differ only among exactly tied distances
(tests/parity.py). These tests reproduce src/flat_index.cc:69-140 and src/ivfpq_index.cc:208-381
of the reference on its own outputs."""
import os

import numpy as np
import pytest

from conftest import GOLDEN
from parity import assert_sorted, assert_topk_parity

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def c1():
    from quiver_b200.synthetic import config1
    return config1()


def test_config1_full_size(gpu, reference, c1, monkeypatch):
    db, q = c1
    ix = gpu.FlatIndex(100, "cosine")
    ix.add(db)
    monkeypatch.delenv("QV_FLAT_SCREEN", raising=False)
    gpu._native.set_timing(True)
    l_tc, d_tc = ix.search(q, 10)
    st = gpu.last_search_stats()
    gpu._native.set_timing(False)
    assert st["dominant_kernel"] == "flat_screen_tc_kernel"
    assert st["rescanned_queries"] >= 0
    assert_sorted(d_tc)
    monkeypatch.setenv("QV_FLAT_SCREEN", "simt")
    l_simt, d_simt = ix.search(q, 10)
    monkeypatch.delenv("QV_FLAT_SCREEN")
    assert np.array_equal(d_tc, d_simt), "tensor-core and SIMT screens differ in distances"
    assert np.array_equal(l_tc, l_simt), "tensor-core and SIMT screens differ in labels"
    rf = reference.flat(100, "cosine")
    rf.add(db)
    sub = np.random.default_rng(5).choice(len(q), 512, replace=False)
    rl, rd = rf.search(q[sub], 10)
    assert_topk_parity(l_tc[sub], d_tc[sub], rl, rd, exact=True, what="config 1 vs reference")


def _ivf_both(gpu, reference, name, db, tmp_path):
    """The reference-trained empty index with db added by the GPU and by the reference."""
    trained = os.path.join(GOLDEN, name)
    ix = gpu.IvfPqIndex.load(trained)
    labels = np.arange(len(db), dtype=np.uint64)
    half = len(db) // 2  # two add() calls: appends keep every list's input order
    ix.add(db[:half], labels[:half])
    ix.add(db[half:], labels[half:])
    ref = reference.ivf_load(trained)
    ref.add(db, labels)
    return ix, ref


def _same_lists(gpu_ix, ref_ix, tmp_path):
    """Both indexes saved: lists, codes, labels (and vectors) equal byte for byte; the GPU-written
    file loads in the reference library."""
    from oracle.oracle import QvrIvf
    gp, rp = tmp_path / "gpu.qvr", tmp_path / "ref.qvr"
    gpu_ix.save(gp)
    ref_ix.save(rp)
    g, r = QvrIvf(gp), QvrIvf(rp)
    assert (g.dim, g.nlist, g.m, g.count, g.metric) == (r.dim, r.nlist, r.m, r.count, r.metric)
    assert np.array_equal(g.centroids, r.centroids) and np.array_equal(g.codebooks, r.codebooks)
    assert np.array_equal(g.offsets, r.offsets), "list sizes differ"
    assert np.array_equal(g.labels, r.labels), "stored label order differs"
    assert np.array_equal(g.codes, r.codes), "PQ codes differ"
    if r.vectors is not None:
        assert np.array_equal(g.vectors, r.vectors), "stored vectors differ"
    return gp


def test_config2_full_size(gpu, reference, tmp_path):
    from quiver_b200.synthetic import config2
    db, q = config2()
    ix, ref = _ivf_both(gpu, reference, "ivf_c2_trained.qvr", db, tmp_path)
    gpu_file = _same_lists(ix, ref, tmp_path)
    from_gpu = reference.ivf_load(gpu_file)  # the reference reads what the GPU wrote
    sub = q[np.random.default_rng(6).choice(len(q), 256, replace=False)]
    for nprobe in (1, 4, 8, 16, 32, 64):
        l, d = ix.search(sub, 10, nprobe=nprobe)
        assert_sorted(d)
        rl, rd = ref.search(sub, 10, nprobe)
        assert_topk_parity(l, d, rl, rd, exact=True, what=f"config 2 nprobe {nprobe}")
        if nprobe in (1, 64):
            fl, fd = from_gpu.search(sub, 10, nprobe)
            assert_topk_parity(fl, fd, rl, rd, exact=True, what=f"reference on GPU file {nprobe}")


def test_config3_full_size(gpu, reference, tmp_path, c1):
    db, q = c1  # config 3 uses config 1's rows and queries
    ix, ref = _ivf_both(gpu, reference, "ivf_c3_trained.qvr", db, tmp_path)
    _same_lists(ix, ref, tmp_path)
    sub = q[np.random.default_rng(7).choice(len(q), 256, replace=False)]
    rng = np.random.default_rng(7)  # the bench's filter: a seeded random 1 % of the ids
    allowed = np.sort(rng.choice(len(db), len(db) // 100, replace=False)).astype(np.uint64)
    for nprobe, rf, filt in [(64, 8, None), (64, 8, allowed), (16, 0, None), (64, 0, allowed)]:
        l, d = ix.search(sub, 10, nprobe=nprobe, refine_factor=rf, filter=filt)
        assert_sorted(d)
        rl, rd = ref.search(sub, 10, nprobe, rf, filt)
        assert_topk_parity(l, d, rl, rd, exact=True,
                           what=f"config 3 nprobe {nprobe} refine {rf} filter {filt is not None}")
        if filt is not None:
            assert np.isin(l[l >= 0].astype(np.uint64), allowed).all()


def test_flat_k100_dim768(gpu, reference):
    """Config 4's shape (768-dim inner product over an L2-normalized mixture, k=100) at a size the
    reference answers in seconds."""
    from quiver_b200.synthetic import config4_chunk
    db = config4_chunk(200_000, 0)
    q = config4_chunk(300, 63)
    ix = gpu.FlatIndex(768, "ip")
    ix.add(db)
    l, d = ix.search(q, 100)
    assert_sorted(d)
    rf = reference.flat(768, "ip")
    rf.add(db)
    rl, rd = rf.search(q, 100)
    assert_topk_parity(l, d, rl, rd, exact=True, what="dim 768 k 100")
