"""The C-ABI library loads and exports every entry point include/qv_gpu.h declares, and the
Python layer's host-side argument handling matches the reference binding (no GPU needed)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def _declared():
    text = open(os.path.join(ROOT, "include", "qv_gpu.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qv_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from quiver_b200 import _native
    lib = C.CDLL(_native.LIB_PATH)
    declared = _declared()
    assert len(declared) > 30
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_native.EXPORTED) == set(declared)


def test_label_validation_matches_reference_binding():
    from quiver_b200 import _as_labels
    assert _as_labels([1, 2, 2**63 - 1]).dtype == np.uint64
    with pytest.raises(ValueError, match="2\\*\\*63"):
        _as_labels([2**63])
    with pytest.raises(ValueError, match="2\\*\\*63"):
        _as_labels(np.array([0, 2**64 - 1], dtype=np.uint64))
    with pytest.raises(ValueError, match="non-negative"):
        _as_labels([-1])
    with pytest.raises(TypeError):
        _as_labels([1.5])
    with pytest.raises(TypeError):
        _as_labels([True])
    assert _as_labels(set()).size == 0
    assert _as_labels(i for i in [3, 4]).tolist() == [3, 4]
    assert _as_labels(range(3)).tolist() == [0, 1, 2]
    with pytest.raises(ValueError, match="labels for"):
        _as_labels([1, 2], n=3)


def test_filter_kind_follows_make_filter_rule():
    from quiver_b200._native import QV_FILTER_LABEL_BITMAP, QV_FILTER_LABEL_SET, make_filter
    f, words = make_filter(np.array([1, 5, 64], dtype=np.uint64))
    assert f.kind == QV_FILTER_LABEL_BITMAP and f.size == 65
    assert int(words[0]) == (1 << 1) | (1 << 5) and int(words[1]) == 1
    f, _ = make_filter(np.array([2**40], dtype=np.uint64))
    assert f.kind == QV_FILTER_LABEL_SET
    f, _ = make_filter(np.array([], dtype=np.uint64))
    assert f.kind == QV_FILTER_LABEL_BITMAP and f.size == 0


def test_matrix_coercion():
    from quiver_b200 import _as_matrix
    assert _as_matrix([1.0, 2.0], 2).shape == (1, 2)
    with pytest.raises(ValueError, match="dimension"):
        _as_matrix(np.zeros((2, 3)), 4)
    with pytest.raises(ValueError):
        _as_matrix(np.zeros((2, 3, 4)), 3)


def test_quiver_alias_package_is_the_gpu_build():
    """`import quiver` resolves to this build's classes (the reference's package name)."""
    import quiver
    import quiver_b200
    assert quiver.FlatIndex is quiver_b200.FlatIndex
    assert quiver.IvfPqIndex is quiver_b200.IvfPqIndex
    import pytest
    with pytest.raises(AttributeError, match="not part of the GPU build"):
        quiver.HnswIndex  # noqa: B018
