"""The GPU HNSW vector store and its filtered exact scan against the reference's HnswIndex
(src/hnsw_index.cc:723-760, its exact_scan_threshold fallback): SQ8 training and codes equal the
reference's ScalarQuantizer on the prepared rows, and searches return the reference's results
bit for bit (labels may differ only among exactly tied distances, tests/parity.py), through both
the gathered scan (selective filters) and the in-place scan (broad ones)."""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from parity import assert_sorted, assert_topk_parity

pytestmark = pytest.mark.gpu

with open(os.path.join(GOLDEN, "hnsw_manifest.json")) as fh:
    MANIFEST = json.load(fh)


def _golden_inputs(case):
    import sys
    sys.path.insert(0, GOLDEN)
    from make_hnsw_golden import hnsw_inputs
    return hnsw_inputs((case["storage"], case["metric"], case["n"], case["dim"], case["seed"]))


def _decoded(codes, vmin, vscale):
    # vmin + code * vscale rounded once: the product of an 8-bit and a 24-bit significand and
    # the sum are exact in float64 here, so one rounding to float32 gives the FMA's result.
    return (codes.astype(np.float64) * vscale.astype(np.float64)
            + vmin.astype(np.float64)).astype(np.float32)


@pytest.mark.parametrize("case", MANIFEST["hnsw"], ids=lambda c: c["name"])
def test_store_matches_reference_goldens(gpu, case):
    base, queries, allowed = _golden_inputs(case)
    g = np.load(os.path.join(GOLDEN, case["name"] + ".npz"))
    st = gpu.HnswStore(case["dim"], case["metric"], case["storage"])
    st.add(base)
    assert len(st) == case["n"] and st.num_nodes == case["n"]
    if case["storage"] == "sq8":
        vmin, vscale = st.sq8_params()
        assert np.array_equal(vmin, g["vmin"]) and np.array_equal(vscale, g["vscale"])
        codes = st.codes()
        assert np.array_equal(codes[:256], g["codes_head"])
        assert hashlib.sha256(codes.tobytes()).digest() == g["codes_sha256"].tobytes()
        want = _decoded(codes[:5], vmin, vscale)
        for i in range(5):
            assert np.array_equal(st.get_vector(i), want[i])
    for s in case["selectivities"]:
        tag = f"{int(s * 1000)}"
        l, d = st.search(queries, case["k"], filter=allowed[s])
        assert_sorted(d)
        assert_topk_parity(l, d, g[f"labels_{tag}"], g[f"dists_{tag}"], exact=True,
                           what=f"{case['name']} selectivity {s}")


@pytest.mark.parametrize("storage", ["float32", "sq8"])
@pytest.mark.parametrize("metric", ["l2", "ip", "cosine"])
def test_large_store_gathered_and_in_place_scans(gpu, oracle, reference, storage, metric):
    """200,000 x 128: a 1 % filter takes the gathered scan, a 40 % filter the in-place scan;
    both equal the oracle's restatement, and the 1 % case equals the reference's HnswIndex."""
    from quiver_b200.synthetic import clustered
    n, dim = 200_000, 128
    x = clustered(n, dim, 64, 77)
    q = clustered(64, dim, 64, 78)
    st = gpu.HnswStore(dim, metric, storage)
    st.add(x[: n // 2])
    st.add(x[n // 2:])
    prepared = oracle.normalize_rows(x) if metric == "cosine" else x
    kw = {"rows": prepared}
    if storage == "sq8":
        vmin, vscale = st.sq8_params()
        kw = {"codes": st.codes(), "vmin": vmin, "vscale": vscale}
    rng = np.random.default_rng(5)
    for share in (0.01, 0.4):
        allowed = np.sort(rng.choice(n, int(n * share), replace=False)).astype(np.uint64)
        sub = q[:16] if share > 0.1 else q
        l, d = st.search(sub, 10, filter=allowed)
        oi, od = oracle.exact_scan(metric, sub, 10, allowed.astype(np.uint32), **kw)
        assert_topk_parity(l, d, oi.astype(np.uint64), od, exact=True,
                           what=f"{storage} {metric} share {share}")
        assert np.isin(l[l >= 0].astype(np.uint64), allowed).all()
    if storage == "float32" and metric == "l2":
        h = reference.hnsw(dim, metric, storage, M=8, ef_construction=32)
        h.add(x[:20_000])
        small = gpu.HnswStore(dim, metric, storage)
        small.add(x[:20_000])
        allowed = np.sort(rng.choice(20_000, 200, replace=False)).astype(np.uint64)
        rl, rd = h.search(q, 10, allowed=allowed, exact_scan_threshold=1.0)
        l, d = small.search(q, 10, filter=allowed)
        assert_topk_parity(l, d, rl, rd, exact=True, what="reference HnswIndex")


@pytest.mark.parametrize("storage", ["float32", "sq8"])
def test_removed_nodes_and_label_rules(gpu, oracle, reference, storage):
    """Soft deletes leave the scan (src/hnsw_index.cc:711-714); a removed label may be added
    again, a live one may not (src/hnsw_index.cc:588-596)."""
    from quiver_b200.synthetic import clustered
    n, dim = 3000, 24
    x = clustered(n, dim, 8, 91)
    q = clustered(20, dim, 8, 92)
    labels = np.arange(n, dtype=np.uint64) * 5 + 3
    st = gpu.HnswStore(dim, "l2", storage)
    h = reference.hnsw(dim, "l2", storage, M=8, ef_construction=40)
    st.add(x, labels)
    h.add(x, labels)
    allowed = np.sort(np.random.default_rng(1).choice(labels, 60, replace=False))
    gone = allowed[::3]
    for lab in gone:
        assert st.remove(int(lab)) and h.remove(int(lab))
    assert not st.remove(int(gone[0]))  # already removed
    assert not st.remove(10**12)  # never present
    assert len(st) == n - len(gone) and st.num_nodes == n
    l, d = st.search(q, 10, filter=allowed)
    rl, rd = h.search(q, 10, allowed=allowed, exact_scan_threshold=1.0)
    assert_topk_parity(l, d, rl, rd, exact=True, what=f"{storage} after removals")
    assert not np.isin(l.astype(np.uint64), gone).any()
    # No filter: every live node.
    l, d = st.search(q[:3], 5)
    assert not np.isin(l.astype(np.uint64), gone).any()
    with pytest.raises(ValueError, match="already in the index"):
        st.add(x[:1], labels[1:2])
    st.add(x[:1] * 0.5, gone[:1])  # the removed label comes back as a new node
    assert len(st) == n - len(gone) + 1 and st.num_nodes == n + 1
    with pytest.raises(ValueError, match="duplicate labels"):
        st.add(x[:2], np.array([7, 7], np.uint64))
    with pytest.raises(ValueError, match="NaN or infinity"):
        st.search(np.full((1, dim), np.nan, np.float32), 3)


def test_sq8_training_rules(gpu):
    x = np.random.default_rng(0).standard_normal((300, 16)).astype(np.float32)
    st = gpu.HnswStore(16, "l2", "sq8")
    assert not st.is_trained
    with pytest.raises(ValueError, match="untrained"):
        st.add(x[:100])
    st.train(x[:10])  # explicit training on any sample
    assert st.is_trained
    with pytest.raises(ValueError, match="already trained"):
        st.train(x)
    st.add(x[:100])
    f32 = gpu.HnswStore(16, "l2", "float32")
    with pytest.raises(ValueError, match="only applies to SQ8"):
        f32.train(x)
    assert f32.is_trained
    empty = gpu.HnswStore(16, "cosine", "float32")
    l, d = empty.search(x[:2], 4, filter=[1, 2])
    assert (l == -1).all() and np.isinf(d).all()
