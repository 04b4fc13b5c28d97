"""The reference's small elementwise and 2-D kernels on the GPU against the
oracle: stir! and the independent-chains graph of bench/independent.jl,
touch4! (bench/stress.jl), sched_write!/sched_accum! in the RPS memory_saving
graph (test/test_window.jl:727-771), transpose_scale! and frombytes!
(test/test_window.jl:30-33, 84-87).

Tolerances: bit-exact for everything but sin; stir! goes through the GPU's
sinf, which may differ from the C library's in the last place, and six stages
of x*k + sin(x) can double such a difference each stage: 2e-5 relative."""
import numpy as np
import pytest

import mantle_cuda as M
from mantle_cuda.workloads import build_independent, seeded_integers, seeded_uniform
from oracle import oracle as O

STIR_RTOL = 2e-5


def test_oracle_stir_transpose_frombytes_match_numpy():
    x = seeded_uniform(1, 1000, -4, 4, 0)
    np.testing.assert_allclose(O.stir(x, 1.001), x * np.float32(1.001) + np.sin(x), rtol=1e-6, atol=1e-6)
    w, h = 7, 5
    src = seeded_uniform(1, w * h, -1, 1, 1)
    want = np.array([np.float32(2.0) * src[y * w + x] for x in range(w) for y in range(h)], np.float32)
    assert np.array_equal(O.transpose_scale(src, w, h, 2.0), want)
    b = np.array([0, 1, 255, 256, 0x1234, 0xFFFFFFFF], np.uint32)
    assert np.array_equal(O.frombytes(b), (b & 0xFF).astype(np.float32))
    a, c, d, e = (seeded_uniform(2, 64, -1, 1, k) for k in range(4))
    assert np.array_equal(O.touch4(a, c, d, e), ((a * np.float32(1.0001) + c) + d) + e)


@pytest.mark.gpu
def test_stir_kernel_matches_oracle(dev):
    n = (1 << 20) + 3
    x = seeded_uniform(3, n, -3, 3, 0)
    src, dst = M.Buffer(dev, x), M.Buffer(dev, np.float32, n)
    M.launch(M.kernels.stir, (dst, src, 1.001), n, stream=dev.stream)
    dev.synchronize()
    np.testing.assert_allclose(dst.array(), O.stir(x, 1.001), rtol=1e-6, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("barriers", ["derived", "backend", "both"])
def test_independent_chains_match_oracle(dev, barriers):
    # bench/independent.jl's graph at its size: 8 chains x 6 stages of stir!
    # over 1 << 20 floats, interleaved declaration.
    w = build_independent(dev)
    M.run(w.plan, barriers=barriers)
    M.run(w.plan, barriers=barriers)
    dev.synchronize()
    for c in range(w.chains):
        want = w.inputs["sources"][c]
        for _ in range(w.stages):
            want = O.stir(want, w.k)
        np.testing.assert_allclose(w.outputs[c].array(), want, rtol=STIR_RTOL, atol=1e-5)
    # :backend chains every pass
    assert w.plan.nedges("backend") == w.chains * w.stages - 1
    # transients alias: two intermediates per chain at most are alive at once,
    # and the handovers between chains that share bytes add edges
    assert M.peakbytes(w.plan) <= 2 * w.chains * 4 * w.n
    # without aliasing the derived edges are each chain's stages in order and
    # nothing between the chains
    w2 = build_independent(dev, alias=False)
    assert w2.plan.nedges("derived") == w2.chains * (w2.stages - 1)
    assert w.plan.nedges("derived") >= w2.plan.nedges("derived")


@pytest.mark.gpu
def test_touch4_is_bit_exact(dev):
    n = (1 << 18) + 1
    a, b, c, d = (seeded_uniform(5, n, -1, 1, k) for k in range(4))
    bufs = [M.Buffer(dev, v) for v in (a, b, c, d)]
    g = M.Graph(dev)
    M.compute(g, "touch4", lambda p: M.dispatch(p, M.kernels.touch4, (
        M.use(p, bufs[0], read=True, write=True), M.use(p, bufs[1], read=True), M.use(p, bufs[2], read=True),
        M.use(p, bufs[3], read=True)), n))
    M.run(M.Plan(g))
    dev.synchronize()
    assert np.array_equal(bufs[0].array(), O.touch4(a, b, c, d))


@pytest.mark.gpu
@pytest.mark.parametrize("policy", ["overlap", "compact"])
def test_rps_memory_saving_graph_runs(dev, policy):
    # test/test_window.jl:736-771: six sched_write! into six transients, six
    # sched_accum! into one output. Both policies give out = 1 + ... + 6.
    n = 256
    g = M.Graph(dev)
    out = M.Buffer(dev, np.zeros(n, np.float32))
    ts = [M.Transient.Buffer(g, np.float32, n) for _ in range(6)]
    for i in range(6):
        M.compute(g, f"draw{i}", lambda p, i=i: M.dispatch(p, M.kernels.sched_write, (
            M.use(p, ts[i], write=True), float(i + 1)), n))
    for i in range(6):
        M.compute(g, f"blt{i}", lambda p, i=i: M.dispatch(p, M.kernels.sched_accum, (
            M.use(p, out, read=True, write=True), M.use(p, ts[i], read=True)), n))
    plan = M.Plan(g, policy=M.Compact() if policy == "compact" else M.Overlap())
    M.run(plan)
    dev.synchronize()
    assert np.all(out.array() == 21.0)
    M.run(plan)
    dev.synchronize()
    assert np.all(out.array() == 42.0)


@pytest.mark.gpu
@pytest.mark.parametrize("w,h", [(256, 128), (100, 37), (1, 1), (33, 1000)])
def test_transpose_scale_matches_oracle(dev, w, h):
    src_h = seeded_uniform(7, w * h, -1, 1, 0)
    src, out = M.Buffer(dev, src_h), M.Buffer(dev, np.zeros(w * h, np.float32))
    g = M.Graph(dev)
    M.compute(g, "transpose", lambda p: M.dispatch(p, M.kernels.transpose_scale, (
        M.use(p, out, write=True), M.use(p, src, read=True), w, h, 2.0), (w, h)))
    M.run(M.Plan(g))
    dev.synchronize()
    assert np.array_equal(out.array(), O.transpose_scale(src_h, w, h, 2.0))
    with pytest.raises(M.ArgumentError):
        M.launch(M.kernels.transpose_scale, (out, src, w, h, 2.0), (w + 1, h), stream=dev.stream)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 7, (1 << 16) + 3])
@pytest.mark.parametrize("offset", [0, 1])
def test_frombytes_matches_oracle(dev, n, offset):
    import torch
    raw = seeded_integers(8, n + offset, 1 << 30, 0).astype(np.uint32) * np.uint32(3)
    src = torch.from_numpy(raw.view(np.int32)).cuda()
    dst = torch.zeros(n + offset, device="cuda")
    M.launch(M.kernels.frombytes, (dst[offset:], src[offset:]), n, stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(dst[offset:].cpu().numpy(), O.frombytes(raw[offset:]))
