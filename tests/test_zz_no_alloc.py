"""The allocation-free Flat search entry point, qv_flat_search_device_noalloc.

It serves callers that must not allocate device memory while they search (a serving loop with a
fixed device-memory budget, or code running where cudaMalloc/cudaFree are not allowed): all its
temporaries live in one fixed device array inside the library. These tests call it through the C
ABI and check that it returns exactly what the allocating entry point qv_flat_search_device
returns for the same inputs, on two calls in a row (the shared scratch keeps the previous call's
contents, so the second call checks that it is reset properly), and that a request too large for
the fixed scratch is refused with a clear error. This file is collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _search(gpu, fn, index, dq, k, bitmap=None):
    import torch
    nq = dq.shape[0]
    labels = torch.full((nq, k), -7, dtype=torch.int64, device=dq.device)
    dists = torch.full((nq, k), -7.0, dtype=torch.float32, device=dq.device)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    bm = None if bitmap is None else bitmap.data_ptr()
    gpu._native.check(fn(index.handle, dq.data_ptr(), nq, k, bm, labels.data_ptr(),
                         dists.data_ptr(), None, stream))
    torch.cuda.synchronize()
    return labels.cpu().numpy(), dists.cpu().numpy()


def _position_bitmap(n, seed):
    """Device words with a random half of the n stored rows admitted."""
    import torch
    keep = np.random.default_rng(seed).random(n) < 0.5
    packed = np.packbits(keep, bitorder="little")
    words = np.zeros(((n + 63) // 64) * 8, np.uint8)
    words[:packed.size] = packed
    return torch.from_numpy(words.view(np.int64)).cuda(), keep


def _same(got, want, what):
    gl, gd = got
    wl, wd = want
    assert np.array_equal(gd, wd, equal_nan=True), f"{what}: distances differ"
    assert np.array_equal(gl, wl), f"{what}: labels differ"


@pytest.mark.parametrize("metric", ["cosine", "l2", "ip"])
@pytest.mark.parametrize("filtered", [False, True])
def test_noalloc_equals_allocating_entry_point_twice(gpu, metric, filtered):
    import torch
    from quiver_b200.synthetic import mixture
    base = mixture(30000, 100, 60, 0.35, 1.0, centre_seed=7, seed=8)
    ix = gpu.FlatIndex(100, metric)
    ix.add(base)
    lib = gpu.lib()
    bitmap, keep = _position_bitmap(30000, 11) if filtered else (None, None)
    for call, (nq, k, seed) in enumerate([(300, 10, 9), (129, 25, 10)]):
        q = mixture(nq, 100, 60, 0.35, 1.0, centre_seed=7, seed=seed)
        dq = torch.from_numpy(q).cuda()
        want = _search(gpu, lib.qv_flat_search_device, ix, dq, k, bitmap)
        got = _search(gpu, lib.qv_flat_search_device_noalloc, ix, dq, k, bitmap)
        _same(got, want, f"{metric} filtered={filtered} call {call}")
        assert (got[0] >= 0).all()
        if filtered:
            assert keep[got[0]].all(), "a row the bitmap rejects was returned"


def test_noalloc_nonfinite_queries_and_empty_index(gpu):
    """A query holding NaN or infinity gets no results from both entry points (QV_INVALID_LABEL,
    NaN distance) while the others are answered; an empty index fills every slot as unfilled."""
    import torch
    lib = gpu.lib()
    rng = np.random.default_rng(12)
    ix = gpu.FlatIndex(64, "l2")
    ix.add(rng.standard_normal((4000, 64)).astype(np.float32))
    q = rng.standard_normal((40, 64)).astype(np.float32)
    q[3, 5] = np.nan
    q[17, 0] = np.inf
    dq = torch.from_numpy(q).cuda()
    for call in range(2):
        want = _search(gpu, lib.qv_flat_search_device, ix, dq, 10)
        got = _search(gpu, lib.qv_flat_search_device_noalloc, ix, dq, 10)
        _same(got, want, f"non-finite call {call}")
        for bad in (3, 17):
            assert (got[0][bad] == -1).all() and np.isnan(got[1][bad]).all()
        good = np.setdiff1d(np.arange(40), [3, 17])
        assert (got[0][good] >= 0).all() and np.isfinite(got[1][good]).all()
    empty = gpu.FlatIndex(64, "ip")
    ok = torch.from_numpy(rng.standard_normal((5, 64)).astype(np.float32)).cuda()
    for fn in (lib.qv_flat_search_device, lib.qv_flat_search_device_noalloc):
        l, d = _search(gpu, fn, empty, ok, 7)
        assert (l == -1).all() and np.isinf(d).all() and (d > 0).all()


def test_noalloc_refuses_requests_beyond_its_scratch(gpu):
    import torch
    ix = gpu.FlatIndex(64, "ip")
    ix.add(np.random.default_rng(1).standard_normal((5000, 64)).astype(np.float32))
    limit = gpu.lib().qv_flat_noalloc_max_bytes()
    assert limit == 64 << 20
    nq = 200000  # about 200k * 64 * 4 bytes of query copies alone: more than the scratch holds
    dq = torch.zeros((nq, 64), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError, match="scratch"):
        _search(gpu, gpu.lib().qv_flat_search_device_noalloc, ix, dq, 10)
