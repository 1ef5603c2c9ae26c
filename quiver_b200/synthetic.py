"""Seeded synthetic workloads for the benchmark configurations and the tests.

The reference measured on ann-benchmarks SIFT1M / GloVe-1.2M, which are not available here; these
generators stand in for them with the shapes, sizes and value distributions the benchmark
configurations specify:

* ``skewed_ints``: every component min(G - 1, 255) with G ~ Geometric(p=0.03), i.e. P(v) is
  proportional to 0.97^v clipped to 0..255, cast to float32 (SIFT-like integer descriptors).
* ``mixture``: a C-component Gaussian mixture (centres N(0, s_c^2), per-component sigma, equal
  weights), L2-normalized in float32 (GloVe-like angular data).
* ``gaussian`` / ``clustered``: small test distributions (standard normal; blobs around 2*N(0,1)
  centres with unit noise).

All use numpy's PCG64 (``np.random.default_rng``), so a seed fixes the data on every machine.
"""
from __future__ import annotations

import numpy as np


def skewed_ints(n: int, dim: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.minimum(rng.geometric(0.03, (n, dim)) - 1, 255).astype(np.float32)


def mixture(n: int, dim: int, components: int, sigma: float, centre_scale: float, centre_seed: int,
            seed: int, sigma_from_centre_norm: bool = False, chunk: int = 1 << 20) -> np.ndarray:
    """L2-normalized mixture samples. ``sigma_from_centre_norm``: per-component sigma is
    ``sigma * ||centre||`` instead of ``sigma``."""
    rc = np.random.default_rng(centre_seed)
    centres = (rc.standard_normal((components, dim)) * centre_scale).astype(np.float32)
    sig = (sigma * np.linalg.norm(centres, axis=1) if sigma_from_centre_norm
           else np.full(components, sigma)).astype(np.float32)
    rng = np.random.default_rng(seed)
    out = np.empty((n, dim), np.float32)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        a = rng.integers(0, components, e - s)
        x = centres[a] + sig[a, None] * rng.standard_normal((e - s, dim), dtype=np.float32)
        x /= np.linalg.norm(x, axis=1, keepdims=True).astype(np.float32)
        out[s:e] = x
    return out


def gaussian(n: int, dim: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((n, dim), dtype=np.float32)


def clustered(n: int, dim: int, clusters: int, seed: int) -> np.ndarray:
    centres = 2.0 * np.random.default_rng(clusters * 1000003 + dim).standard_normal(
        (clusters, dim), dtype=np.float32)
    rng = np.random.default_rng(seed)
    a = rng.integers(0, clusters, n)
    return (centres[a] + rng.standard_normal((n, dim), dtype=np.float32)).astype(np.float32)


# ---- benchmark configurations 0..4 ------------------------------------------------------------------

def config0(seed_db: int = 0, seed_q: int = 1):
    """FlatIndex L2, k=10: 100,000 x 128 skewed ints, 1,000 queries."""
    return skewed_ints(100_000, 128, seed_db), skewed_ints(1_000, 128, seed_q)


def config1(n: int = 1_183_514, nq: int = 10_000):
    """FlatIndex cosine, k=10: 1,183,514 x 100 from a 1,000-component mixture (sigma 0.35)."""
    db = mixture(n, 100, 1000, 0.35, 1.0, centre_seed=42, seed=0)
    q = mixture(nq, 100, 1000, 0.35, 1.0, centre_seed=42, seed=1)
    return db, q


def config2(n: int = 1_000_000, nq: int = 10_000):
    """IvfPqIndex L2 (nlist 2048, m 32): 1,000,000 x 128 skewed ints like config 0, 10,000 queries;
    the first 100,000 rows are the training sample."""
    return skewed_ints(n, 128, 2), skewed_ints(nq, 128, 3)


def config3(n: int = 1_183_514, nq: int = 10_000):
    """IvfPqIndex cosine (nlist 2048, m 25, refine 8): config 1's rows and queries; the first
    100,000 rows are the training sample."""
    return config1(n, nq)


def config4_chunk(rows: int, chunk_index: int, dim: int = 768):
    """One chunk of config 4 (40M x 768 inner product, 4,096-component mixture, sigma 0.5*||c||)."""
    seed = np.random.SeedSequence(4).spawn(64)[chunk_index]
    return mixture(rows, dim, 4096, 0.5, 1.0 / np.sqrt(dim), centre_seed=44,
                   seed=int(seed.generate_state(1)[0]), sigma_from_centre_norm=True)


C4_ROWS, C4_DIM, C4_COMPONENTS = 40_000_000, 768, 4096
C4_CHUNK = 1_000_000  # rows per generation chunk; shard boundaries of 1/2/4/8 ranks fall on them


def config4_centres(dim: int = C4_DIM):
    """Config 4's mixture centres N(0, 1/dim) and per-component sigma 0.5 * ||centre|| (numpy)."""
    rc = np.random.default_rng(44)
    centres = (rc.standard_normal((C4_COMPONENTS, dim)) / np.sqrt(dim)).astype(np.float32)
    return centres, (0.5 * np.linalg.norm(centres, axis=1)).astype(np.float32)


def config4_device(first: int, end: int, device, queries: bool = False):
    """Config 4 rows [first, end) generated on a CUDA device in chunks of C4_CHUNK rows, yielded
    as (first id, float32 tensor [rows, 768]), L2-normalized. Each chunk's values depend only on
    its global position (a generator seeded per chunk), so every sharding of the 40M rows sees
    the same collection. ``queries``: the query stream instead (another seed family)."""
    import torch
    centres, sig = config4_centres()
    c = torch.from_numpy(centres).to(device)
    s = torch.from_numpy(sig).to(device)
    pos = first
    while pos < end:
        chunk = pos // C4_CHUNK
        stop = min(end, (chunk + 1) * C4_CHUNK)
        g = torch.Generator(device=device)
        g.manual_seed((9_000_000 if queries else 4_000_000) + chunk)
        # Draw the whole chunk, then keep the part in [pos, stop): the values of a row do not
        # depend on which part of its chunk is requested.
        full = C4_CHUNK
        a = torch.randint(0, C4_COMPONENTS, (full,), generator=g, device=device)
        x = torch.randn((full, C4_DIM), generator=g, device=device)
        lo, hi = pos - chunk * C4_CHUNK, stop - chunk * C4_CHUNK
        a, x = a[lo:hi], x[lo:hi]
        x.mul_(s[a, None]).add_(c[a])
        x.div_(torch.linalg.vector_norm(x, dim=1, keepdim=True))
        yield pos, x.contiguous()
        pos = stop
