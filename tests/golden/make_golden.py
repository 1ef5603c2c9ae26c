"""Generates the golden fixtures in this directory by running the reference Quiver library itself.

The reference is compiled from its own sources by ``oracle/Makefile`` into
``oracle/_ref/libquiver_ref.so`` (needs the reference checkout, so run this where it exists):

    make -C oracle ref REF=<reference checkout> && python tests/golden/make_golden.py

Every output below is produced by the reference's public API (FlatIndex / IvfPqIndex /
ProductQuantizer / CentroidTable / simd kernels) on seeded synthetic inputs; the tests compare both
our C restatement (oracle/) and the GPU library against these files. Inputs are regenerated from
the seeds recorded in each file, so only outputs and trained state are stored.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import Reference  # noqa: E402
from quiver_b200.synthetic import clustered, gaussian, skewed_ints  # noqa: E402

FLAT_CASES = [
    # (name, metric, n, dim, nq, k, generator, seed)
    ("flat_l2_d13", "l2", 300, 13, 20, 7, "gaussian", 1),
    ("flat_l2_d100", "l2", 2000, 100, 40, 10, "clustered", 2),
    ("flat_ip_d33", "ip", 1500, 33, 30, 10, "gaussian", 3),
    ("flat_cos_d100", "cosine", 2000, 100, 40, 10, "clustered", 4),
    ("flat_cos_d129", "cosine", 1000, 129, 20, 25, "gaussian", 5),
    ("flat_l2_ints", "l2", 3000, 128, 30, 10, "skewed", 6),
]

IVF_CASES = [
    # (name, metric, n, dim, nlist, m, seed)
    ("ivf_l2", "l2", 2000, 40, 16, 10, 11),
    ("ivf_ip", "ip", 2000, 40, 16, 10, 12),
    ("ivf_cos", "cosine", 2000, 40, 16, 10, 13),
]
IVF_SEARCHES = [(1, 0), (4, 0), (16, 0), (4, 3), (16, 2)]  # (nprobe, refine_factor)


def gen(kind: str, n: int, dim: int, seed: int) -> np.ndarray:
    if kind == "gaussian":
        return gaussian(n, dim, seed)
    if kind == "clustered":
        return clustered(n, dim, 20, seed)
    return skewed_ints(n, dim, seed)


def main() -> None:
    ref = Reference()
    manifest = {"reference_isa": ref.isa, "flat": [], "ivf": []}
    rng_dims = [1, 2, 3, 4, 5, 7, 8, 9, 12, 15, 16, 17, 31, 32, 33, 36, 63, 64, 65, 96, 100, 127,
                128, 129, 256, 384, 768, 1000]
    a = [gaussian(1, d, 1000 + d)[0] * 3 for d in rng_dims]
    b = [gaussian(1, d, 2000 + d)[0] for d in rng_dims]
    np.savez_compressed(
        os.path.join(HERE, "kernels.npz"), dims=np.array(rng_dims),
        dot=np.array([ref.dot(x, y) for x, y in zip(a, b)], np.float32),
        l2sqr=np.array([ref.l2sqr(x, y) for x, y in zip(a, b)], np.float32),
        normalized=np.concatenate([ref.normalize_rows(x[None])[0] for x in a]).astype(np.float32))

    for name, metric, n, dim, nq, k, kind, seed in FLAT_CASES:
        base = gen(kind, n, dim, seed)
        q = gen(kind, nq, dim, seed + 100)
        labels = np.arange(n, dtype=np.uint64) * 3 + 7
        f = ref.flat(dim, metric)
        f.add(base, labels)
        rl, rd = f.search(q, k)
        allowed = np.sort(np.random.default_rng(seed).choice(labels, n // 5, replace=False))
        fl, fd = f.search(q, k, allowed=allowed)
        big_l, big_d = f.search(q[:3], n + 5)  # k > n: padded
        np.savez_compressed(os.path.join(HERE, name + ".npz"), labels=rl, dists=rd,
                            filt_allowed=allowed, filt_labels=fl, filt_dists=fd, all_labels=big_l,
                            all_dists=big_d)
        manifest["flat"].append(dict(name=name, metric=metric, n=n, dim=dim, nq=nq, k=k,
                                     generator=kind, seed=seed, query_seed=seed + 100,
                                     label_rule="3*i+7", filter_seed=seed))

    for name, metric, n, dim, nlist, m, seed in IVF_CASES:
        base = clustered(n, dim, 12, seed)
        q = clustered(50, dim, 12, seed + 100)
        ix = ref.ivf(dim, metric, nlist, m, store_vectors=True, train_iterations=8, seed=seed)
        ix.train(base)
        ix.add(base)
        path = os.path.join(HERE, name + ".qvr")
        ix.save(path)
        out = {}
        for nprobe, rf in IVF_SEARCHES:
            rl, rd = ix.search(q, 10, nprobe, rf)
            out[f"labels_{nprobe}_{rf}"] = rl
            out[f"dists_{nprobe}_{rf}"] = rd
        allowed = np.sort(np.random.default_rng(seed).choice(n, n // 10, replace=False)).astype(
            np.uint64)
        rl, rd = ix.search(q, 10, 8, 0, allowed=allowed)
        out["filt_allowed"], out["filt_labels"], out["filt_dists"] = allowed, rl, rd
        rl, rd = ix.search(q[:5], 10, nlist, 1 << 62)  # saturated keep: exact over everything
        out["sat_labels"], out["sat_dists"] = rl, rd
        np.savez_compressed(os.path.join(HERE, name + "_search.npz"), **out)
        manifest["ivf"].append(dict(name=name, metric=metric, n=n, dim=dim, nlist=nlist, m=m,
                                    seed=seed, query_seed=seed + 100, clusters=12,
                                    train_iterations=8, searches=IVF_SEARCHES, filter_nprobe=8))
    with open(os.path.join(HERE, "manifest.json"), "w") as fh:
        json.dump(manifest, fh, indent=1)
    print("wrote goldens; reference ISA:", ref.isa)


if __name__ == "__main__":
    main()
