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


def _search(gpu, fn, index, dq, k):
    import torch
    nq = dq.shape[0]
    labels = torch.full((nq, k), -7, dtype=torch.int64, device=dq.device)
    dists = torch.full((nq, k), -7.0, dtype=torch.float32, device=dq.device)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    gpu._native.check(fn(index.handle, dq.data_ptr(), nq, k, None, labels.data_ptr(),
                         dists.data_ptr(), None, stream))
    torch.cuda.synchronize()
    return labels.cpu().numpy(), dists.cpu().numpy()


@pytest.mark.parametrize("metric", ["cosine", "l2"])
def test_noalloc_equals_allocating_entry_point_twice(gpu, metric):
    import torch
    from quiver_b200.synthetic import mixture
    base = mixture(30000, 100, 60, 0.35, 1.0, centre_seed=7, seed=8)
    ix = gpu.FlatIndex(100, metric)
    ix.add(base)
    lib = gpu.lib()
    for call, (nq, k, seed) in enumerate([(300, 10, 9), (129, 25, 10)]):
        q = mixture(nq, 100, 60, 0.35, 1.0, centre_seed=7, seed=seed)
        dq = torch.from_numpy(q).cuda()
        want_l, want_d = _search(gpu, lib.qv_flat_search_device, ix, dq, k)
        got_l, got_d = _search(gpu, lib.qv_flat_search_device_noalloc, ix, dq, k)
        assert np.array_equal(got_d, want_d), f"call {call}: distances differ"
        assert np.array_equal(got_l, want_l), f"call {call}: labels differ"
        assert (got_l >= 0).all()


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
