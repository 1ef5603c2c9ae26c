"""The parity comparator shared by the tests.

* Distances, rank by rank: bit-identical when ``exact``; otherwise
  ``|got - want| / max(1, |want|) <= rtol`` (the reference's own idiom, tests/test_distance.cc:21-23).
* Labels, per query: identical sets after leaving out labels whose distance ties the k-th (boundary)
  distance within the tolerance: the reference's bounded heaps leave the choice among equal
  distances unspecified (src/flat_index.cc:89-95, src/ivfpq_index.cc:348-358), and the order among
  equal distances is free.
"""
from __future__ import annotations

import numpy as np

INVALID = np.uint64(2**64 - 1)


def _close(g, w, rtol):
    both_inf = np.isinf(g) & np.isinf(w) & (np.sign(g) == np.sign(w))
    with np.errstate(invalid="ignore"):
        ok = np.abs(g - w) / np.maximum(1.0, np.abs(w)) <= rtol
    return both_inf | ok


def assert_topk_parity(got_labels, got_dists, want_labels, want_dists, exact=True, rtol=1e-5,
                       what=""):
    gl = np.asarray(got_labels).astype(np.uint64)
    wl = np.asarray(want_labels).astype(np.uint64)
    gd = np.asarray(got_dists, dtype=np.float32)
    wd = np.asarray(want_dists, dtype=np.float32)
    assert gl.shape == wl.shape and gd.shape == wd.shape, (gl.shape, wl.shape)
    tol = 0.0 if exact else rtol
    if exact:
        same = (gd == wd) | (np.isnan(gd) & np.isnan(wd))
    else:
        same = _close(gd.astype(np.float64), wd.astype(np.float64), rtol)
    bad = np.argwhere(~same)
    assert bad.size == 0, (f"{what}: {bad.shape[0]} distance mismatches, first at {bad[0]}: "
                           f"got {gd[tuple(bad[0])]!r} want {wd[tuple(bad[0])]!r}")
    for q in range(gl.shape[0]):
        k = gl.shape[1]
        boundary = wd[q, k - 1]
        if np.isinf(boundary):
            g = set(gl[q][gd[q] != np.inf].tolist())
            w = set(wl[q][wd[q] != np.inf].tolist())
            assert g == w, f"{what}: query {q} label sets differ: {sorted(g ^ w)[:10]}"
            assert np.all((gl[q] == INVALID) == (wl[q] == INVALID)), f"{what}: query {q} padding"
            continue
        margin = tol * max(1.0, abs(float(boundary)))
        inner_g = set(gl[q][gd[q].astype(np.float64) < float(boundary) - margin].tolist())
        inner_w = set(wl[q][wd[q].astype(np.float64) < float(boundary) - margin].tolist())
        assert inner_g == inner_w, (f"{what}: query {q} labels differ away from ties: "
                                    f"{sorted(inner_g ^ inner_w)[:10]}")
        assert len(set(gl[q].tolist())) == k or INVALID in gl[q], f"{what}: duplicate labels q={q}"


def assert_sorted(dists):
    d = np.asarray(dists, dtype=np.float64)
    fin = np.where(np.isinf(d), 3.0e38, d)
    assert np.all(np.diff(fin, axis=1) >= 0), "results are not sorted closest-first"
