"""The quiver C++ API (include/quiver/*.h, built as quiver_b200/libquiver.so over the C ABI).

tests/cpp/api_test.cc is compiled against the installed headers and the in-tree libraries. The CPU
test runs its host-only cases (thread pool, filters, metric names, and, on a machine without a GPU,
that constructing an index fails loudly). The GPU tests run its device cases (restatements of the
reference's FlatIndex / IvfPqIndex / regression tests) and use its dump modes to check that
FlatIndex::search_batch and IvfPqIndex::search_batch, called from C++ with each Filter class,
return the reference's golden results.
"""
import os
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, ROOT, golden_flat_inputs, golden_ivf_inputs
from parity import assert_sorted, assert_topk_parity

PKG = os.path.join(ROOT, "quiver_b200")
SRC = os.path.join(ROOT, "tests", "cpp", "api_test.cc")


@pytest.fixture(scope="module")
def api_test(tmp_path_factory):
    from quiver_b200 import build as qb
    if not os.path.exists(qb.LIB):
        pytest.fail("quiver_b200/libquiver_b200.so is not built (python -m quiver_b200.build)")
    if not os.path.exists(qb.CPP_LIB):
        qb.build_cpp()
    exe = str(tmp_path_factory.mktemp("cpp") / "api_test")
    cmd = [qb._cxx(), "-std=c++20", "-O1", "-Wall", "-Wextra", "-I", os.path.join(ROOT, "include"),
           SRC, "-o", exe, "-L", PKG, "-lquiver", "-lquiver_b200", f"-Wl,-rpath,{PKG}",
           "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "warning" not in r.stderr, r.stderr
    return exe


def _run(exe, *args, timeout=300):
    r = subprocess.run([exe, *args], capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, f"api_test {' '.join(args)} failed:\n{r.stdout}\n{r.stderr}"
    return r.stdout


def test_cpp_api_host_cases(api_test):
    out = _run(api_test, "cpu")
    assert "0 failure(s)" in out and "FAILED" not in out


@pytest.mark.gpu
def test_cpp_api_device_cases(api_test, gpu, tmp_path):
    out = _run(api_test, "gpu", os.path.join(GOLDEN, "ivf_l2.qvr"), str(tmp_path))
    assert "0 failure(s)" in out and "FAILED" not in out, out


def _dump_flat(exe, d, case, base, labels, q, kind, allowed):
    spec = f"{case['metric']} {case['dim']} {case['n']} {q.shape[0]} {case['k']} {kind} {len(allowed)}"
    (d / "spec.txt").write_text(spec)
    base.astype(np.float32).tofile(d / "base.bin")
    labels.astype(np.uint64).tofile(d / "labels.bin")
    q.astype(np.float32).tofile(d / "queries.bin")
    np.asarray(allowed, dtype=np.uint64).tofile(d / "allowed.bin")
    _run(exe, "flat", str(d))
    k = case["k"]
    return (np.fromfile(d / "out_labels.bin", dtype=np.uint64).reshape(-1, k),
            np.fromfile(d / "out_dists.bin", dtype=np.float32).reshape(-1, k))


@pytest.mark.gpu
@pytest.mark.parametrize("idx", range(6))
def test_cpp_flat_search_batch_matches_reference_golden(api_test, gpu, manifest, tmp_path, idx):
    case = manifest["flat"][idx]
    base, q, labels = golden_flat_inputs(case)
    g = np.load(os.path.join(GOLDEN, case["name"] + ".npz"))
    l, d = _dump_flat(api_test, tmp_path, case, base, labels, q, 0, [])
    assert_sorted(d)
    assert_topk_parity(l, d, g["labels"], g["dists"], exact=True, what=case["name"])
    for kind, name in ((1, "LabelSetFilter"), (2, "BitsetFilter"), (3, "PredicateFilter")):
        l, d = _dump_flat(api_test, tmp_path, case, base, labels, q, kind, g["filt_allowed"])
        assert_topk_parity(l, d, g["filt_labels"], g["filt_dists"], exact=True,
                           what=f"{case['name']} {name}")


@pytest.mark.gpu
@pytest.mark.parametrize("idx", range(3))
def test_cpp_ivf_search_batch_matches_reference_golden(api_test, gpu, manifest, tmp_path, idx):
    case = manifest["ivf"][idx]
    _, q = golden_ivf_inputs(case)
    g = np.load(os.path.join(GOLDEN, case["name"] + "_search.npz"))
    qvr = os.path.join(GOLDEN, case["name"] + ".qvr")
    q.astype(np.float32).tofile(tmp_path / "queries.bin")

    def search(nprobe, rf, kind=0, allowed=()):
        (tmp_path / "spec.txt").write_text(
            f"{qvr} {q.shape[0]} 10 {nprobe} {rf} {kind} {len(allowed)}")
        np.asarray(allowed, dtype=np.uint64).tofile(tmp_path / "allowed.bin")
        _run(api_test, "ivf", str(tmp_path))
        return (np.fromfile(tmp_path / "out_labels.bin", dtype=np.uint64).reshape(-1, 10),
                np.fromfile(tmp_path / "out_dists.bin", dtype=np.float32).reshape(-1, 10))

    for nprobe, rf in case["searches"]:
        l, d = search(nprobe, rf)
        assert_topk_parity(l, d, g[f"labels_{nprobe}_{rf}"], g[f"dists_{nprobe}_{rf}"],
                           exact=True, what=f"{case['name']} nprobe={nprobe} rf={rf}")
    for kind in (1, 2, 3):
        l, d = search(case["filter_nprobe"], 0, kind, g["filt_allowed"])
        assert_topk_parity(l, d, g["filt_labels"], g["filt_dists"], exact=True,
                           what=f"{case['name']} filter kind {kind}")
