"""Generates the HNSW-storage golden fixtures in this directory by running the reference library.

The reference is compiled from its own sources by ``oracle/Makefile`` into
``oracle/_ref/libquiver_ref.so`` (needs the reference checkout, so run this where it exists):

    make -C oracle ref REF=<reference checkout> && python tests/golden/make_hnsw_golden.py

Outputs, all from the reference's public API on seeded synthetic inputs:

* ``sq8_kernels.npz``: simd::active().l2sqr_sq8 / dot_sq8 (the AVX2 kernels) per dimension;
* ``hnsw_<storage>_<metric>.npz``: an HnswIndex (float32 or SQ8 storage) built from seeded rows,
  the SQ8 parameters and codes ScalarQuantizer produces for its prepared rows (the first 256
  nodes' codes in full, a SHA-256 of all of them; checked here
  against the vectors the index reports), and HnswIndex::search_batch with a label filter and
  exact_scan_threshold 1.0, which takes the exact scan (src/hnsw_index.cc:743-760), at two
  selectivities (0.5 % and 5 % of the labels).

Inputs are regenerated from the seeds recorded in ``hnsw_manifest.json``.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import Reference  # noqa: E402
from quiver_b200.synthetic import clustered, gaussian  # noqa: E402

SQ8_DIMS = [1, 3, 7, 8, 9, 15, 16, 17, 24, 31, 32, 33, 40, 63, 64, 100, 128, 129, 200, 768]
HNSW_CASES = [
    # (storage, metric, n, dim, seed)
    ("float32", "l2", 4000, 40, 21),
    ("float32", "ip", 4000, 40, 22),
    ("float32", "cosine", 4000, 100, 23),
    ("sq8", "l2", 4000, 40, 24),
    ("sq8", "ip", 4000, 100, 25),
    ("sq8", "cosine", 4000, 100, 26),
]
SELECTIVITIES = (0.005, 0.05)
NQ, K = 40, 10


def sq8_inputs(dim: int):
    rng = np.random.default_rng(3000 + dim)
    q = rng.standard_normal(dim).astype(np.float32) * 2
    code = rng.integers(0, 256, dim).astype(np.uint8)
    vmin = (-rng.random(dim) * 1.5).astype(np.float32)
    vscale = (0.01 + (np.arange(dim) % 7) * 0.003).astype(np.float32)
    return q, code, vmin, vscale


def hnsw_inputs(case):
    storage, metric, n, dim, seed = case
    base = clustered(n, dim, 16, seed)
    queries = gaussian(NQ, dim, seed + 100)
    allowed = {s: np.sort(np.random.default_rng(seed + int(s * 1000)).choice(
        n, max(1, int(n * s)), replace=False)).astype(np.uint64) for s in SELECTIVITIES}
    return base, queries, allowed


def main() -> None:
    ref = Reference()
    ins = [sq8_inputs(d) for d in SQ8_DIMS]
    np.savez_compressed(
        os.path.join(HERE, "sq8_kernels.npz"), dims=np.array(SQ8_DIMS),
        l2sqr_sq8=np.array([ref.l2sqr_sq8(*x) for x in ins], np.float32),
        dot_sq8=np.array([ref.dot_sq8(*x) for x in ins], np.float32))
    manifest = {"reference_isa": ref.isa, "sq8_dims": SQ8_DIMS, "hnsw": []}
    for case in HNSW_CASES:
        storage, metric, n, dim, seed = case
        base, queries, allowed = hnsw_inputs(case)
        h = ref.hnsw(dim, metric, storage, M=12, ef_construction=80, seed=seed)
        h.add(base)
        out = {}
        prepared = ref.normalize_rows(base) if metric == "cosine" else base
        if storage == "sq8":
            vmin, vscale = ref.sq8_train(prepared)  # the index trained on its first batch
            codes = ref.sq8_encode(vmin, vscale, prepared)
            decoded = np.array([h.vector(i) for i in range(50)])
            want = (codes[:50].astype(np.float32) * vscale + vmin).astype(np.float32)
            assert np.allclose(decoded, want, rtol=0, atol=1e-6), "SQ8 state differs"
            # The codes: the first 256 nodes in full, all of them through a digest (keeps the
            # fixture small).
            out.update(vmin=vmin, vscale=vscale, codes_head=codes[:256],
                       codes_sha256=np.frombuffer(hashlib.sha256(codes.tobytes()).digest(),
                                                  np.uint8))
        else:
            stored = np.array([h.vector(i) for i in range(n)])
            assert np.array_equal(stored, prepared), "stored rows differ from the prepared rows"
        for s in SELECTIVITIES:
            rl, rd = h.search(queries, K, allowed=allowed[s], exact_scan_threshold=1.0)
            tag = f"{int(s * 1000)}"
            out[f"labels_{tag}"], out[f"dists_{tag}"] = rl, rd
        name = f"hnsw_{storage}_{metric}"
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
        manifest["hnsw"].append(dict(name=name, storage=storage, metric=metric, n=n, dim=dim,
                                     seed=seed, clusters=16, query_seed=seed + 100, nq=NQ, k=K,
                                     selectivities=list(SELECTIVITIES), M=12,
                                     ef_construction=80))
    with open(os.path.join(HERE, "hnsw_manifest.json"), "w") as fh:
        json.dump(manifest, fh, indent=1)
    print("wrote HNSW goldens; reference ISA:", ref.isa)


if __name__ == "__main__":
    main()
