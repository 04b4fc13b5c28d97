"""The allocation-free scatter entry point (mtl_scatter_add_noalloc).

It exists for callers that may not allocate GPU memory on the scatter path —
code living inside another runtime's memory budget, or a frame loop where an
allocation could stall or fail mid-frame. It takes its scratch from a fixed
array compiled into the library, shared by every call on the device.

Checked here through the C ABI against the regular entry point (mtl_launch of
`scatter_add` with caller-provided scratch) and against the oracle, on two
calls in a row so that the second call runs over the leftovers of the first,
and with unaligned caller pointers at small sizes. Tolerance as for every
scatter test: bit-exact counts, 1e-5 relative (and 1e-5 absolute) sums.

This file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest

import mantle_cuda as M
from mantle_cuda import _lib as L

pytestmark = pytest.mark.gpu


def _noalloc(acc, hist, v, idx, n, nbins, accumulate, stream):
    ptr = lambda b: C.c_void_p(b.ptr) if b is not None else None  # noqa: E731
    L.check(L.lib().mtl_scatter_add_noalloc(ptr(acc), ptr(hist), ptr(v), ptr(idx), n, nbins, accumulate,
                                            C.c_void_p(stream)))


def _regular(acc, hist, v, idx, n, nbins, accumulate, dev):
    args = (acc, hist, v, idx, nbins, accumulate)
    ws = M.Buffer(dev, np.uint8, max(M.workspace_bytes(M.kernels.scatter_add, args, n), 16))
    M.launch(M.kernels.scatter_add, args, n, stream=dev.stream, workspace=ws)
    dev.synchronize()


@pytest.mark.parametrize("nbins", [1 << 16, 1000])
def test_noalloc_matches_regular_entry_point_twice(dev, nbins):
    rng = np.random.default_rng(11)
    for call in range(2):
        n = (1 << 22) + 3 * call
        v = M.Buffer(dev, rng.random(n, dtype=np.float32))
        idx = M.Buffer(dev, rng.integers(-5, nbins + 5, n, dtype=np.int32))
        a1, h1 = M.Buffer(dev, np.float32, nbins), M.Buffer(dev, np.int32, nbins)
        a2, h2 = M.Buffer(dev, np.float32, nbins), M.Buffer(dev, np.int32, nbins)
        _regular(a1, h1, v, idx, n, nbins, 0, dev)
        _noalloc(a2, h2, v, idx, n, nbins, 0, dev.stream)
        dev.synchronize()
        assert np.array_equal(h1.array(), h2.array())
        np.testing.assert_allclose(a2.array(), a1.array(), rtol=1e-5, atol=1e-5)
        # the histogram alone, accumulating onto what the call above left
        _noalloc(None, h2, None, idx, n, nbins, 1, dev.stream)
        dev.synchronize()
        assert np.array_equal(h2.array(), 2 * h1.array())


def test_noalloc_matches_oracle_twice(dev):
    # Against the oracle directly (float64 sums, exact counts), two calls in a
    # row over the same shared scratch.
    from mantle_cuda.workloads import seeded_integers, seeded_uniform
    from oracle import oracle as O
    nbins = 1 << 16
    for call in range(2):
        n = (1 << 20) + 7 * call
        vh = seeded_uniform(40 + call, n, 0, 1, 0)
        ih = seeded_integers(40 + call, n, nbins, 1)
        acc, hist = M.Buffer(dev, np.float32, nbins), M.Buffer(dev, np.int32, nbins)
        _noalloc(acc, hist, M.Buffer(dev, vh), M.Buffer(dev, ih), n, nbins, 0, dev.stream)
        dev.synchronize()
        want_a, want_h = O.scatter_f64(vh, ih, nbins)
        assert np.array_equal(hist.array().view(np.uint32), want_h)
        np.testing.assert_allclose(acc.array(), want_a, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("n", [5, 7, 4 * 74 + 3, 1001])
def test_noalloc_unaligned_small_inputs(dev, n):
    # Caller pointers one element past an allocation's start take the
    # plain-load path; every element must land, whatever n is.
    import torch
    from oracle import oracle as O
    nbins = 1 << 16
    rng = np.random.default_rng(n)
    vh = rng.random(n + 1, dtype=np.float32)
    ih = rng.integers(0, nbins, n + 1, dtype=np.int32)
    vt, it = torch.from_numpy(vh).cuda(), torch.from_numpy(ih).cuda()
    acc = torch.zeros(nbins, device="cuda")
    hist = torch.zeros(nbins, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    L.check(L.lib().mtl_scatter_add_noalloc(C.c_void_p(acc.data_ptr()), C.c_void_p(hist.data_ptr()),
                                            C.c_void_p(vt[1:].data_ptr()), C.c_void_p(it[1:].data_ptr()), n,
                                            nbins, 0, C.c_void_p(dev.stream)))
    dev.synchronize()
    want_a, want_h = O.scatter_f64(vh[1:], ih[1:], nbins)
    assert np.array_equal(hist.cpu().numpy().view(np.uint32), want_h)
    np.testing.assert_allclose(acc.cpu().numpy(), want_a, rtol=1e-5, atol=1e-5)


def test_noalloc_large_bins_and_bad_arguments(dev):
    # 2^20 bins fit no cluster's shared memory: the kernel takes the L2-atomic
    # route, which needs no scratch at all.
    nbins = 1 << 20
    acc = M.Buffer(dev, np.float32, nbins)
    v = M.Buffer(dev, np.ones(16, np.float32))
    idx = M.Buffer(dev, np.arange(16, dtype=np.int32) * 4096)
    _noalloc(acc, None, v, idx, 16, nbins, 0, dev.stream)
    dev.synchronize()
    got = acc.array()
    assert got.sum() == 16.0 and np.all(got[np.arange(16) * 4096] == 1.0)
    with pytest.raises(M.ArgumentError):
        _noalloc(acc, None, v, idx, -1, nbins, 0, dev.stream)
    with pytest.raises(M.ArgumentError):
        _noalloc(acc, None, v, idx, 16, 0, 0, dev.stream)
