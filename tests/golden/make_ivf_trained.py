"""Trains the IVF-PQ indexes of configs 2 and 3 with the reference Quiver library and saves them.

Configs 2 and 3 load "centroids and codebooks trained by the reference on a 100,000-vector sample
from its saved file". This script does that training with the reference's own
IvfPqIndex::train (compiled from its sources into oracle/_ref/libquiver_ref.so by oracle/Makefile)
and writes the trained, still empty indexes:

    make -C oracle ref REF=<reference checkout> && python tests/golden/make_ivf_trained.py

  ivf_c2_trained.qvr  L2, dim 128, nlist 2048, m 32, trained on rows [0, 100000) of config 2
  ivf_c3_trained.qvr  cosine, dim 100, nlist 2048, m 25, store_vectors, trained on rows
                      [0, 100000) of config 3

The bench and the tests load these files and add the full databases on the GPU.
"""
from __future__ import annotations

import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import Reference  # noqa: E402
from quiver_b200.synthetic import config2, config3  # noqa: E402

SAMPLE = 100_000


def main() -> None:
    ref = Reference()
    jobs = [("ivf_c2_trained.qvr", "l2", 128, 32, False, lambda: config2(SAMPLE, 1)[0]),
            ("ivf_c3_trained.qvr", "cosine", 100, 25, True, lambda: config3()[0][:SAMPLE])]
    for name, metric, dim, m, store, sample in jobs:
        x = sample()
        assert x.shape == (SAMPLE, dim)
        ix = ref.ivf(dim, metric, 2048, m, store_vectors=store)
        t0 = time.time()
        ix.train(x)
        ix.save(os.path.join(HERE, name))
        print(f"{name}: trained in {time.time() - t0:.1f} s", flush=True)


if __name__ == "__main__":
    main()
