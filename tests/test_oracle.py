"""The CPU oracle (our C restatement, oracle/qv_oracle.c) pinned against the reference's outputs:
the golden fixtures written by tests/golden/make_golden.py from the reference library itself, and,
where the reference library is built in this checkout, fresh randomized comparisons."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden_flat_inputs, golden_ivf_inputs
from parity import assert_topk_parity


def test_reduction_kernels_match_reference_bits(oracle):
    g = np.load(os.path.join(GOLDEN, "kernels.npz"))
    from quiver_b200.synthetic import gaussian
    off = 0
    for i, d in enumerate(g["dims"]):
        a = gaussian(1, int(d), 1000 + int(d))[0] * 3
        b = gaussian(1, int(d), 2000 + int(d))[0]
        assert np.float32(oracle.dot(a, b)) == g["dot"][i], d
        assert np.float32(oracle.l2sqr(a, b)) == g["l2sqr"][i], d
        n = oracle.normalize_rows(a[None])[0]
        assert np.array_equal(n, g["normalized"][off:off + d]), d
        off += int(d)


def test_known_answer_cosine_and_inner_product(oracle):
    # tests/test_flat.cc:37-52 of the reference.
    base = np.array([[1, 0, 0, 0], [0, 2, 0, 0], [1, 1, 0, 0]], np.float32)
    q = np.array([[3, 0.1, 0, 0]], np.float32)
    lab = np.arange(3, dtype=np.uint64)
    l, d = oracle.flat_search(oracle.normalize_rows(base), lab, "cosine", q, 3)
    assert l[0, 0] == 0 and abs(d[0, 0] - (1 - 3 / np.sqrt(9.01))) < 1e-5
    l, d = oracle.flat_search(base, lab, "ip", q, 3)
    assert l[0, 0] == 2 and abs(d[0, 0] - (1 - 3.1)) < 1e-5


@pytest.mark.parametrize("idx", range(6))
def test_flat_matches_golden(oracle, manifest, idx):
    case = manifest["flat"][idx]
    base, q, labels = golden_flat_inputs(case)
    g = np.load(os.path.join(GOLDEN, case["name"] + ".npz"))
    stored = oracle.normalize_rows(base) if case["metric"] == "cosine" else base
    l, d = oracle.flat_search(stored, labels, case["metric"], q, case["k"])
    assert_topk_parity(l, d, g["labels"], g["dists"], exact=True, what=case["name"])
    l, d = oracle.flat_search(stored, labels, case["metric"], q, case["k"],
                              allowed=g["filt_allowed"])
    assert_topk_parity(l, d, g["filt_labels"], g["filt_dists"], exact=True, what="filtered")
    l, d = oracle.flat_search(stored, labels, case["metric"], q[:3], case["n"] + 5)
    assert_topk_parity(l, d, g["all_labels"], g["all_dists"], exact=True, what="k>n")


@pytest.mark.parametrize("idx", range(3))
def test_ivf_encode_matches_reference_qvr(oracle, manifest, idx):
    from oracle.oracle import QvrIvf
    case = manifest["ivf"][idx]
    base, _ = golden_ivf_inputs(case)
    qv = QvrIvf(os.path.join(GOLDEN, case["name"] + ".qvr"))
    assign, codes = oracle.ivf_encode(qv.centroids, qv.codebooks, qv.m, case["metric"], base)
    order = np.argsort(qv.labels)  # default labels are the input row ids
    assert np.array_equal(qv.labels[order], np.arange(case["n"]))
    assert np.array_equal(qv.assignments()[order], assign)
    assert np.array_equal(qv.codes[order], codes)


@pytest.mark.parametrize("idx", range(3))
def test_ivf_search_matches_golden(oracle, manifest, idx):
    from oracle.oracle import QvrIvf
    case = manifest["ivf"][idx]
    _, q = golden_ivf_inputs(case)
    qv = QvrIvf(os.path.join(GOLDEN, case["name"] + ".qvr"))
    g = np.load(os.path.join(GOLDEN, case["name"] + "_search.npz"))
    for nprobe, rf in case["searches"]:
        l, d = oracle.ivf_search(qv, q, 10, nprobe, rf)
        assert_topk_parity(l, d, g[f"labels_{nprobe}_{rf}"], g[f"dists_{nprobe}_{rf}"],
                           exact=True, what=f"{case['name']} nprobe={nprobe} rf={rf}")
    l, d = oracle.ivf_search(qv, q, 10, case["filter_nprobe"], 0, allowed=g["filt_allowed"])
    assert_topk_parity(l, d, g["filt_labels"], g["filt_dists"], exact=True, what="filtered")
    l, d = oracle.ivf_search(qv, q[:5], 10, case["nlist"], 1 << 62)
    assert_topk_parity(l, d, g["sat_labels"], g["sat_dists"], exact=True, what="saturated keep")


def test_oracle_matches_compiled_reference_randomized(oracle, reference):
    rng = np.random.default_rng(7)
    for d in (1, 7, 12, 36, 100, 131):
        a = rng.standard_normal((4, d)).astype(np.float32) * rng.uniform(0.01, 50)
        b = rng.standard_normal((4, d)).astype(np.float32)
        for x, y in zip(a, b):
            assert oracle.dot(x, y) == reference.dot(x, y)
            assert oracle.l2sqr(x, y) == reference.l2sqr(x, y)
        assert np.array_equal(oracle.normalize_rows(a), reference.normalize_rows(a))
    cents = rng.standard_normal((37, 24)).astype(np.float32)
    x = rng.standard_normal((500, 24)).astype(np.float32)
    for by_ip in (False, True):
        assert np.array_equal(oracle.coarse_assign(cents, x, by_ip),
                              reference.nearest_batch(cents, x, by_ip))
    cb = rng.standard_normal((6, 256, 4)).astype(np.float32)
    assert np.array_equal(oracle.pq_encode(cb, 6, x), reference.pq_encode(cb, 6, x))
    ip, l2 = reference.pq_tables(cb, 6, x[0])
    assert np.array_equal(oracle.ip_table(cb, 6, x[0]), ip)
    assert np.array_equal(oracle.l2_table(cb, 6, x[0]), l2)


def test_oracle_plants_are_caught(oracle, manifest):
    """A mistake planted in the oracle's output (on the CPU) must fail the comparator."""
    case = manifest["flat"][1]
    base, q, labels = golden_flat_inputs(case)
    g = np.load(os.path.join(GOLDEN, case["name"] + ".npz"))
    l, d = oracle.flat_search(base, labels, case["metric"], q, case["k"])
    d2 = d.copy()
    d2[3, 4] = np.nextafter(d2[3, 4], np.float32(np.inf))
    with pytest.raises(AssertionError):
        assert_topk_parity(l, d2, g["labels"], g["dists"], exact=True)
    l2 = l.copy()
    l2[5, 0] = 123456789
    with pytest.raises(AssertionError):
        assert_topk_parity(l2, d, g["labels"], g["dists"], exact=True)
