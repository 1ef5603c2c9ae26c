"""The oracle's restatement of HNSW's SQ8 storage and filtered exact scan, pinned against the
reference library's own outputs (tests/golden/make_hnsw_golden.py): the AVX2 SQ8 kernels
(src/simd/kernels_avx2.cc:85-129), ScalarQuantizer train / encode (src/scalar_quantizer.cc), and
HnswIndex::search's exact-scan fallback (src/hnsw_index.cc:723-760). No GPU needed."""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from parity import assert_topk_parity

with open(os.path.join(GOLDEN, "hnsw_manifest.json")) as fh:
    MANIFEST = json.load(fh)


def _golden_inputs(case):
    import sys
    sys.path.insert(0, GOLDEN)
    from make_hnsw_golden import hnsw_inputs  # the generator's own seeded inputs
    return hnsw_inputs((case["storage"], case["metric"], case["n"], case["dim"], case["seed"]))


def test_sq8_kernels_match_reference_goldens(oracle):
    import sys
    sys.path.insert(0, GOLDEN)
    from make_hnsw_golden import sq8_inputs
    g = np.load(os.path.join(GOLDEN, "sq8_kernels.npz"))
    for i, dim in enumerate(g["dims"]):
        x = sq8_inputs(int(dim))
        assert np.float32(oracle.l2sqr_sq8(*x)) == g["l2sqr_sq8"][i], f"l2sqr_sq8 dim {dim}"
        assert np.float32(oracle.dot_sq8(*x)) == g["dot_sq8"][i], f"dot_sq8 dim {dim}"
        # The reference's own test of these kernels (tests/test_distance.cc:42-64): within 1e-5
        # of the exact sum.
        q, code, vmin, vscale = (np.asarray(v, np.float64) for v in x)
        dec = code * vscale + vmin
        for got, want in ((oracle.l2sqr_sq8(*x), np.sum((q - dec) ** 2)),
                          (oracle.dot_sq8(*x), np.sum(q * dec))):
            assert abs(got - want) <= 1e-5 * max(1.0, abs(want)) + 1e-4, (dim, got, want)


@pytest.mark.parametrize("case", [c for c in MANIFEST["hnsw"] if c["storage"] == "sq8"],
                         ids=lambda c: c["name"])
def test_sq8_train_and_encode_match_reference_goldens(oracle, case):
    base, _, _ = _golden_inputs(case)
    g = np.load(os.path.join(GOLDEN, case["name"] + ".npz"))
    prepared = oracle.normalize_rows(base) if case["metric"] == "cosine" else base
    vmin, vscale = oracle.sq8_train(prepared)
    assert np.array_equal(vmin, g["vmin"]) and np.array_equal(vscale, g["vscale"])
    codes = oracle.sq8_encode(vmin, vscale, prepared)
    assert np.array_equal(codes[:256], g["codes_head"])
    assert hashlib.sha256(codes.tobytes()).digest() == g["codes_sha256"].tobytes()


@pytest.mark.parametrize("case", MANIFEST["hnsw"], ids=lambda c: c["name"])
def test_exact_scan_matches_reference_hnsw_goldens(oracle, case):
    base, queries, allowed = _golden_inputs(case)
    g = np.load(os.path.join(GOLDEN, case["name"] + ".npz"))
    prepared = oracle.normalize_rows(base) if case["metric"] == "cosine" else base
    store = {"rows": prepared}
    if case["storage"] == "sq8":
        store = {"codes": oracle.sq8_encode(g["vmin"], g["vscale"], prepared),
                 "vmin": g["vmin"], "vscale": g["vscale"]}
    for s in case["selectivities"]:
        tag = f"{int(s * 1000)}"
        ids = allowed[s].astype(np.uint32)  # default labels: label == node id
        oi, od = oracle.exact_scan(case["metric"], queries, case["k"], ids, **store)
        ol = np.where(oi == np.uint32(2**32 - 1), np.uint64(2**64 - 1), oi.astype(np.uint64))
        assert_topk_parity(ol, od, g[f"labels_{tag}"], g[f"dists_{tag}"], exact=True,
                           what=f"{case['name']} selectivity {s}")


def test_exact_scan_matches_compiled_reference_randomized(oracle, reference):
    """Random stores, filters, removals of nothing; every storage and metric, dims with every
    tail length of the SQ8 and float32 kernels."""
    rng = np.random.default_rng(42)
    for storage in ("float32", "sq8"):
        for metric in ("l2", "ip", "cosine"):
            for dim in (5, 24, 37, 64):
                n = 600
                x = rng.standard_normal((n, dim)).astype(np.float32)
                h = reference.hnsw(dim, metric, storage, M=8, ef_construction=40)
                h.add(x)
                prepared = oracle.normalize_rows(x) if metric == "cosine" else x
                allowed = np.sort(rng.choice(n, 40, replace=False)).astype(np.uint64)
                q = rng.standard_normal((12, dim)).astype(np.float32)
                rl, rd = h.search(q, 7, allowed=allowed, exact_scan_threshold=1.0)
                if storage == "float32":
                    oi, od = oracle.exact_scan(metric, q, 7, allowed.astype(np.uint32),
                                               rows=prepared)
                else:
                    vmin, vscale = oracle.sq8_train(prepared)
                    codes = oracle.sq8_encode(vmin, vscale, prepared)
                    oi, od = oracle.exact_scan(metric, q, 7, allowed.astype(np.uint32),
                                               codes=codes, vmin=vmin, vscale=vscale)
                assert_topk_parity(oi.astype(np.uint64), od, rl, rd, exact=True,
                                   what=f"{storage} {metric} dim {dim}")
