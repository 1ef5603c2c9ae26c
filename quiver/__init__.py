"""`import quiver` for the GPU build: the reference's Python package name bound to quiver_b200.

Code written against the reference's Python surface (python/quiver/__init__.py:166-251 of the
reference: ``quiver.FlatIndex``, ``quiver.IvfPqIndex`` with the same constructors, ``add``,
``search``, ``save``/``load``) runs unchanged on the GPU when this directory is on the import path
instead of the reference's package. Only the hot path is provided: of the reference's
``HnswIndex``, the GPU build holds the vector storage and the filtered exact scan
(``quiver.HnswStore``); the graph walk is not part of this build.
"""
from quiver_b200 import (FlatIndex, HnswStore, IvfPqIndex, QuiverError, device_count,
                         last_search_stats)

__all__ = ["FlatIndex", "IvfPqIndex", "HnswStore", "QuiverError", "device_count",
           "last_search_stats"]


def __getattr__(name):
    raise AttributeError(f"quiver.{name} is not part of the GPU build of the hot path "
                         f"(FlatIndex, IvfPqIndex and HnswStore only)")
