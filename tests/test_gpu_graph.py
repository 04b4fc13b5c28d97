"""GPU parity of the graph path: every result read back through the C ABI and
compared with the oracle on the same seeded inputs.

Tolerances: bit-exact for integer counts, the elementwise chain and the
in-place updates (same operation order and rounding on both sides); 1e-5
relative (plus 1e-5 absolute for near-empty bins) for float scatter sums,
whose order of addition is not fixed.
"""
import numpy as np
import pytest

import mantle_cuda as M
from mantle_cuda.workloads import build_chain, build_scatter, seeded_integers, seeded_uniform
from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def test_chain_unfused_matches_oracle_bit_exact(dev):
    for n in (1 << 20, (1 << 16) + 3, 5):
        w = build_chain(dev, n=n, seed=3)
        M.run(w.plan)
        want = O.chain8(w.inputs["x"], w.inputs["y"], w.inputs["z"])
        assert np.array_equal(w.out.array(), want)
        assert w.plan.nkernels() >= 8


def test_chain_single_kernel_and_passes_agree(dev):
    n = (1 << 18) + 1
    w = build_chain(dev, n=n, seed=4, single_kernel=True)
    M.run(w.plan)
    I = w.inputs
    assert np.array_equal(w.out.array(), O.chain8(I["x"], I["y"], I["z"]))
    assert np.array_equal(O.chain8_passes(I["x"], I["y"], I["z"]), O.chain8(I["x"], I["y"], I["z"]))


def test_chain_fused_is_one_kernel_and_bit_exact(dev):
    for n in (1 << 22, (1 << 16) + 3, 5):
        w = build_chain(dev, n=n, seed=5, fuse=True)
        M.run(w.plan)
        I = w.inputs
        assert np.array_equal(w.out.array(), O.chain8(I["x"], I["y"], I["z"]))
        assert w.plan.nkernels() == 1
        assert M.peakbytes(w.plan) == 0
        # replaying is idempotent: the chain only reads x, y, z
        M.run(w.plan)
        M.run(w.plan, barriers="backend")
        assert np.array_equal(w.out.array(), O.chain8(I["x"], I["y"], I["z"]))


def test_fused_run_stores_a_transient_read_later(dev):
    from test_phases import _chain_graph
    n = (1 << 18) + 1
    g, b = _chain_graph(dev, n, keep_t3=True)
    x, y, z = (seeded_uniform(6, n, -1, 1, k) for k in range(3))
    for name, h in (("x", x), ("y", y), ("z", z)):
        b[name].update(h)
    plan = M.Plan(g, fuse=True)
    M.run(plan)
    # the oracle's pass-by-pass run keeps every intermediate; t4 is the fourth
    out = np.empty_like(x)
    tmp = np.empty(7 * n, np.float32)
    f = lambda a: a.ctypes.data_as(O.C.POINTER(O.C.c_float))  # noqa: E731
    O.lib().oracle_chain8_passes(f(x), f(y), f(z), f(out), f(tmp), n, 0)
    assert np.array_equal(b["side"].array(), tmp[3 * n:4 * n])
    assert np.array_equal(b["out"].array(), O.chain8(x, y, z))
    assert plan.nkernels() == 1


def test_chain_transients_are_placed_in_two_slots(dev):
    # Stage k reads t[k] and writes t[k+1]: only adjacent transients are ever
    # live together, so the slab holds two, not seven (bench/chain.jl:1-10).
    w = build_chain(dev, n=1 << 20)
    assert M.peakbytes(w.plan) == 2 * 4 * (1 << 20)
    assert M.naivebytes(w.plan) == 7 * 4 * (1 << 20)


@pytest.mark.parametrize("nbins", [1, 7, 4096, 1 << 16, 1 << 17, 1 << 18])
def test_scatter_matches_oracle(dev, nbins):
    n = (1 << 20) + 5
    v = seeded_uniform(1, n, 0, 1, 0)
    idx = seeded_integers(1, n, nbins, 1)
    acc, hist = M.Buffer(dev, np.float32, nbins), M.Buffer(dev, np.int32, nbins)
    vb, ib = M.Buffer(dev, v), M.Buffer(dev, idx)
    g = M.Graph(dev)
    M.compute(g, "s", lambda p: M.dispatch(p, M.kernels.scatter_add, (
        M.use(p, acc, write=True), M.use(p, hist, write=True), M.use(p, vb, read=True),
        M.use(p, ib, read=True), nbins, 0), n))
    plan = M.Plan(g)
    M.run(plan)
    M.run(plan)  # overwrite semantics: a second replay gives the same bins
    want_a, want_h = O.scatter_f64(v, idx, nbins)
    assert np.array_equal(hist.array().view(np.uint32), want_h)
    np.testing.assert_allclose(acc.array(), want_a, rtol=RTOL, atol=1e-5)


@pytest.mark.parametrize("offset", [0, 1, 3])  # elements: 0 streams tiles by bulk copy, else direct loads
@pytest.mark.parametrize("with_acc", [True, False])
def test_scatter_alignment_and_histogram_only(dev, offset, with_acc):
    import torch
    n, nbins = (1 << 19) + 3, 1 << 16
    v = seeded_uniform(2, n + offset, 0, 1, 0)
    idx = seeded_integers(2, n + offset, nbins, 1)
    vt, it = torch.from_numpy(v).cuda(), torch.from_numpy(idx).cuda()
    acc = torch.zeros(nbins, device="cuda") if with_acc else None
    hist = torch.zeros(nbins, dtype=torch.int32, device="cuda")
    args = (acc, hist, vt[offset:], it[offset:], nbins, 0)
    ws = torch.empty(M.workspace_bytes(M.kernels.scatter_add, args, n), dtype=torch.uint8, device="cuda")
    M.launch(M.kernels.scatter_add, args, n, stream=torch.cuda.current_stream().cuda_stream, workspace=ws)
    torch.cuda.synchronize()
    want_a, want_h = O.scatter_f64(v[offset:], idx[offset:], nbins)
    assert np.array_equal(hist.cpu().numpy().view(np.uint32), want_h)
    if with_acc:
        np.testing.assert_allclose(acc.cpu().numpy(), want_a, rtol=RTOL, atol=1e-5)


@pytest.mark.parametrize("n", [1, 5, 7, 4 * 74 + 3, 4 * 148 + 3, 1001, 20011])
@pytest.mark.parametrize("nbins", [1 << 16, 1000])
def test_scatter_unaligned_small_inputs_lose_no_element(dev, n, nbins):
    # Unaligned values and indices take the plain-load path, whose per-cluster
    # element ranges must cover every element for sizes far below the grid's
    # cluster count too (n = 5 over 74 clusters, ragged tails).
    import torch
    v = seeded_uniform(17, n + 1, 0, 1, 0)
    idx = seeded_integers(17, n + 1, nbins, 1)
    vt, it = torch.from_numpy(v).cuda(), torch.from_numpy(idx).cuda()
    acc = torch.zeros(nbins, device="cuda")
    hist = torch.zeros(nbins, dtype=torch.int32, device="cuda")
    args = (acc, hist, vt[1:], it[1:], nbins, 0)
    ws = torch.empty(max(M.workspace_bytes(M.kernels.scatter_add, args, n), 16), dtype=torch.uint8, device="cuda")
    M.launch(M.kernels.scatter_add, args, n, stream=torch.cuda.current_stream().cuda_stream, workspace=ws)
    torch.cuda.synchronize()
    want_a, want_h = O.scatter_f64(v[1:], idx[1:], nbins)
    assert np.array_equal(hist.cpu().numpy().view(np.uint32), want_h)
    np.testing.assert_allclose(acc.cpu().numpy(), want_a, rtol=RTOL, atol=1e-5)


def skewed_indices(seed, n, nbins, hot=64, frac=0.9):
    """Indices where `frac` of the elements fall in `hot` bins (spread over the
    bin range) and the rest uniformly: the shape of additive splats, many
    points on the same pixels (bench/two_scatters.jl:20-26)."""
    rng = np.random.Generator(np.random.PCG64([seed, 9]))
    hot_bins = rng.choice(nbins, hot, replace=False).astype(np.int32)
    idx = rng.integers(0, nbins, n, dtype=np.int32)
    pick = rng.uniform(size=n) < frac
    idx[pick] = hot_bins[rng.integers(0, hot, int(pick.sum()))]
    return idx


@pytest.mark.parametrize("family", ["scatter_add", "scatter_add_dense"])
@pytest.mark.parametrize("shape", ["uniform", "skewed", "one bin", "sorted", "eight bins"])
def test_scatter_repeated_bins_both_families(dev, family, shape):
    # scatter_add_dense: warps whose bins pile up sum in the warp first (one
    # atomic per bin per warp), the others take the plain form; scatter_add is
    # plain throughout. The result is the oracle's whichever form ran.
    import torch
    n, nbins = (1 << 20) + 4, 1 << 16
    v = seeded_uniform(31, n, 0, 1, 0)
    if shape == "uniform":
        idx = seeded_integers(31, n, nbins, 1)
    elif shape == "skewed":
        idx = skewed_indices(31, n, nbins)
    elif shape == "one bin":
        idx = np.full(n, 40000, np.int32)
    elif shape == "eight bins":
        idx = (seeded_integers(31, n, 8, 1) * 8191).astype(np.int32)
    else:
        idx = np.sort(seeded_integers(31, n, nbins, 1))
    kernel = getattr(M.kernels, family)
    acc = torch.zeros(nbins, device="cuda")
    hist = torch.zeros(nbins, dtype=torch.int32, device="cuda")
    args = (acc, hist, torch.from_numpy(v).cuda(), torch.from_numpy(idx).cuda(), nbins, 0)
    ws = torch.empty(M.workspace_bytes(kernel, args, n), dtype=torch.uint8, device="cuda")
    M.launch(kernel, args, n, stream=torch.cuda.current_stream().cuda_stream, workspace=ws)
    torch.cuda.synchronize()
    want_a, want_h = O.scatter_f64(v, idx, nbins)
    assert np.array_equal(hist.cpu().numpy().view(np.uint32), want_h)
    np.testing.assert_allclose(acc.cpu().numpy(), want_a, rtol=RTOL, atol=1e-5)


@pytest.mark.parametrize("out_offset", [0, 1])  # 0: four bins a thread in the final sum; 1: one
def test_scatter_accumulates_into_aligned_and_unaligned_tables(dev, out_offset):
    import torch
    n, nbins = (1 << 18) + 1, 1 << 16
    v = seeded_uniform(3, n, 0, 1, 0)
    idx = seeded_integers(3, n, nbins, 1)
    base_a = seeded_uniform(3, nbins, -1, 1, 2)
    base_h = seeded_integers(3, nbins, 1000, 3)
    acc = torch.zeros(nbins + out_offset, device="cuda")[out_offset:]
    hist = torch.zeros(nbins + out_offset, dtype=torch.int32, device="cuda")[out_offset:]
    acc.copy_(torch.from_numpy(base_a))
    hist.copy_(torch.from_numpy(base_h))
    args = (acc, hist, torch.from_numpy(v).cuda(), torch.from_numpy(idx).cuda(), nbins, 1)
    ws = torch.empty(M.workspace_bytes(M.kernels.scatter_add, args, n), dtype=torch.uint8, device="cuda")
    M.launch(M.kernels.scatter_add, args, n, stream=torch.cuda.current_stream().cuda_stream, workspace=ws)
    torch.cuda.synchronize()
    want_a, want_h = O.scatter_f64(v, idx, nbins)
    assert np.array_equal(hist.cpu().numpy().view(np.uint32), want_h + base_h.astype(np.uint32))
    np.testing.assert_allclose(acc.cpu().numpy(), want_a + base_a, rtol=RTOL, atol=1e-5)


def test_scatter_edge_cases(dev):
    nbins = 1000
    # out-of-range indices (negative and >= nbins) are skipped, never written
    idx = np.array([-1, 0, 999, 1000, 5, 5, 5, 2**31 - 1, -2**31], np.int32)
    v = np.arange(1, idx.size + 1, dtype=np.float32)
    acc, hist = M.Buffer(dev, np.float32, nbins), M.Buffer(dev, np.int32, nbins)
    M.launch(M.kernels.scatter_add, (acc, hist, M.Buffer(dev, v), M.Buffer(dev, idx), nbins, 0), idx.size,
             stream=dev.stream, workspace=M.Buffer(dev, np.uint8, M.workspace_bytes(
                 M.kernels.scatter_add, (acc, hist, M.Buffer(dev, v), M.Buffer(dev, idx), nbins, 0), idx.size)))
    dev.synchronize()
    want_a, want_h = O.scatter_f64(v, idx, nbins)
    assert np.array_equal(hist.array().view(np.uint32), want_h)
    np.testing.assert_allclose(acc.array(), want_a, rtol=RTOL)


def test_scatter_empty_input_and_accumulate(dev):
    nbins = 64
    acc, hist = M.Buffer(dev, np.float32, nbins), M.Buffer(dev, np.int32, nbins)
    acc.update(np.full(nbins, 2.0, np.float32))
    hist.update(np.full(nbins, 3, np.int32))
    v, idx = M.Buffer(dev, np.float32, 4), M.Buffer(dev, np.int32, 4)
    args = (acc, hist, v, idx, nbins, 1)
    ws = M.Buffer(dev, np.uint8, max(M.workspace_bytes(M.kernels.scatter_add, args, 0), 16))
    M.launch(M.kernels.scatter_add, args, 0, stream=dev.stream, workspace=ws)  # n = 0, accumulate
    dev.synchronize()
    assert np.all(acc.array() == 2.0) and np.all(hist.array() == 3)
    args = (acc, hist, v, idx, nbins, 0)
    M.launch(M.kernels.scatter_add, args, 0, stream=dev.stream, workspace=ws)  # n = 0, overwrite
    dev.synchronize()
    assert np.all(acc.array() == 0.0) and np.all(hist.array() == 0)
    # accumulate adds this call's sums to what is there
    vv = np.ones(100, np.float32)
    ii = (np.arange(100) % nbins).astype(np.int32)
    args = (acc, hist, M.Buffer(dev, vv), M.Buffer(dev, ii), nbins, 1)
    ws = M.Buffer(dev, np.uint8, M.workspace_bytes(M.kernels.scatter_add, args, 100))
    M.launch(M.kernels.scatter_add, args, 100, stream=dev.stream, workspace=ws)
    M.launch(M.kernels.scatter_add, args, 100, stream=dev.stream, workspace=ws)
    dev.synchronize()
    want = 2 * np.bincount(ii, minlength=nbins)
    assert np.array_equal(hist.array(), want.astype(np.int32))
    assert np.array_equal(acc.array(), want.astype(np.float32))


def test_scatter_launch_refuses_short_buffers(dev):
    acc = M.Buffer(dev, np.float32, 10)
    idx = M.Buffer(dev, np.int32, 100)
    v = M.Buffer(dev, np.float32, 100)
    with pytest.raises(M.ArgumentError):
        M.launch(M.kernels.scatter_add, (acc, None, v, idx, 11, 0), 100, stream=dev.stream,
                 workspace=M.Buffer(dev, np.uint8, 1 << 20))
    with pytest.raises(M.ArgumentError):
        M.launch(M.kernels.scatter_add, (acc, None, v, idx, 10, 0), 101, stream=dev.stream,
                 workspace=M.Buffer(dev, np.uint8, 1 << 20))


def test_scatter_workload_graph_replays(dev):
    n, nbins, nupd = (1 << 20) + 7, 1 << 16, (1 << 16) + 1
    w = build_scatter(dev, n=n, nbins=nbins, nupd=nupd, seed=5)
    reps = 3
    for _ in range(reps):
        M.run(w.plan)
    I = w.inputs
    acc_a, hist = O.scatter_f64(I["va"], I["ia"], nbins)
    acc_b, _ = O.scatter_f64(I["vb"], I["ib"], nbins, hist=False)
    b = I["b"]
    for _ in range(reps):
        b = O.touch3(b, I["c"], I["d"])
    assert np.array_equal(w.bufs["hist"].array().view(np.uint32), hist)
    np.testing.assert_allclose(w.bufs["acc_a"].array(), acc_a, rtol=RTOL, atol=1e-5)
    np.testing.assert_allclose(w.bufs["acc_b"].array(), acc_b, rtol=RTOL, atol=1e-5)
    assert np.array_equal(w.bufs["b"].array(), b)
    # The three updates are a read-after-write chain. The scatters touch
    # nothing in common, but each has a scratch transient; with aliasing the
    # placer gives both the same bytes, which orders the second scatter after
    # the first (the handover), and without aliasing they are independent.
    pos = {p.name: k for k, p in enumerate(w.plan.passes)}
    assert w.plan.edges(pos["scatter a"]) == []
    assert w.plan.edges(pos["scatter b"]) == [pos["scatter a"]]
    assert w.plan.edges(pos["update 1"]) == []
    assert w.plan.edges(pos["update 2"]) == [pos["update 1"]]
    assert w.plan.edges(pos["update 3"]) == [pos["update 2"]]
    w2 = build_scatter(dev, n=n, nbins=nbins, nupd=nupd, seed=5, alias=False)
    pos = {p.name: k for k, p in enumerate(w2.plan.passes)}
    assert w2.plan.edges(pos["scatter b"]) == []
    # aliased: the two scratch buffers share bytes; not aliased: both are held
    assert M.peakbytes(w2.plan) == M.naivebytes(w2.plan)
    assert M.peakbytes(w.plan) < M.naivebytes(w.plan)


def test_backend_and_both_modes_agree(dev):
    n, nbins, nupd = 1 << 18, 1 << 10, 1 << 12
    results = []
    for mode in ("derived", "backend", "both"):
        w = build_scatter(dev, n=n, nbins=nbins, nupd=nupd, seed=9)
        M.run(w.plan, barriers=mode)
        results.append((w.bufs["hist"].array(), w.bufs["b"].array()))
    for h, b in results[1:]:
        assert np.array_equal(h, results[0][0]) and np.array_equal(b, results[0][1])
    with pytest.raises(M.ArgumentError):
        M.run(w.plan, barriers="global")


def random_mix_graph(dev, seed, n=4096, passes=12, policy=M.Overlap, alias=True):
    """bench/fuzz.jl:42-65 with this repository's seeded generator: pass i writes
    transient i and reads two earlier results; `out` copies the last."""
    rng = np.random.default_rng(seed)
    g = M.Graph(dev)
    src = M.Buffer(dev, np.ones(n, np.float32))
    out = M.Buffer(dev, np.zeros(n, np.float32))
    bufs = [M.Transient.Buffer(g, np.float32, n) for _ in range(passes)]
    sources = [src]
    choices = []
    for i in range(passes):
        a, b = int(rng.integers(0, len(sources))), int(rng.integers(0, len(sources)))
        choices.append((a, b))
        A, Bx, dst = sources[a], sources[b], bufs[i]
        M.compute(g, f"p{i + 1}", lambda p, A=A, Bx=Bx, dst=dst, i=i: M.dispatch(p, M.kernels.mix, (
            M.use(p, dst, write=True), M.use(p, A, read=True), M.use(p, Bx, read=True), float(i + 1)), n))
        sources.append(dst)
    M.compute(g, "out", lambda p: M.dispatch(p, M.kernels.keep, (
        M.use(p, out, write=True), M.use(p, bufs[-1], read=True)), n))
    return g, out, M.Plan(g, policy=policy, alias=alias), O.fuzz_expected(choices, passes)


@pytest.mark.parametrize("policy", [M.Overlap, M.Compact])
def test_random_dags_match_cpu_replay(dev, policy):
    """bench/fuzz.jl: derived and backend barriers agree, and both equal the
    CPU replay exactly, on random DAGs whose transients alias."""
    wrong = disagree = 0
    for seed in range(12):
        g, out, plan, want = random_mix_graph(dev, seed, policy=policy)
        M.run(plan, barriers="backend")
        ref = out.array()
        out.update(np.zeros(out.n, np.float32))
        M.run(plan, barriers="derived")
        got = out.array()
        disagree += not np.array_equal(got, ref)
        wrong += not (np.all(got == want) and np.all(ref == want))
    assert wrong == 0 and disagree == 0


def test_update_routes(dev):
    n = 1 << 16
    buf = M.Buffer(dev, np.zeros(n, np.float32))
    out = M.Buffer(dev, np.float32, n)
    g = M.Graph(dev)
    ref = M.Update(g, buf)
    part = M.Update(g, buf, range=(1, 100))
    M.compute(g, "copy", lambda p: M.dispatch(p, M.kernels.bump, (
        M.use(p, out, write=True), M.use(p, buf, read=True), 1.0), n))
    plan = M.Plan(g)
    assert plan.names[0] == "updates"
    M.run(plan)  # clean frame: nothing written
    assert np.all(out.array() == 1.0)
    host = np.arange(n, dtype=np.float32)
    ref(host)  # pageable host memory: staged
    M.run(plan)
    assert np.array_equal(out.array(), host + 1)
    dsrc = M.Buffer(dev, np.full(n, 7.0, np.float32))
    ref(dsrc)  # device source: device to device
    M.run(plan)
    assert np.all(out.array() == 8.0)
    part(np.full(100, 9.0, np.float32))  # partial, in place
    M.run(plan)
    got = out.array()
    assert np.all(got[:100] == 10.0) and np.all(got[100:] == 8.0)
    with pytest.raises(M.ArgumentError):
        part(np.zeros(99, np.float32))
        M.run(plan)


def test_custom_pass_orders_its_own_launches(dev):
    """test/test_window.jl:1613-1687: two dependent launches inside one custom
    pass; n small so unordered launches would visibly race."""
    n = 1 << 14
    g = M.Graph(dev)
    src = M.Buffer(dev, np.ones(n, np.float32))
    mid = M.Transient.Buffer(g, np.float32, n)
    out = M.Buffer(dev, np.zeros(n, np.float32))

    def body(p):
        a = M.use(p, mid, read=True, write=True)
        b = M.use(p, src, read=True)
        c = M.use(p, out, write=True)

        def work(ctx):
            M.launch(M.kernels.bump, (ctx.storage(a), ctx.storage(b), 1.0), n, stream=ctx.stream)
            M.launch(M.kernels.bump, (ctx.storage(c), ctx.storage(a), 10.0), n, stream=ctx.stream)
        return work

    M.custom(g, "dependent launches", body)
    plan = M.Plan(g)
    assert len(plan.passes) == 1
    for mode in ("derived", "backend", "both"):
        for _ in range(3):
            out.update(np.zeros(n, np.float32))
            M.run(plan, barriers=mode)
            assert np.all(out.array() == 12.0)
    # a body that returns nothing callable is refused at declaration
    g2 = M.Graph(dev)
    with pytest.raises(M.ArgumentError):
        M.custom(g2, "bad", lambda p: None)


def test_profiled_plan_times_every_pass(dev):
    n, nbins, nupd = 1 << 18, 1 << 10, 1 << 12
    w = build_scatter(dev, n=n, nbins=nbins, nupd=nupd, profile=True)
    with pytest.raises(M.ArgumentError):
        M.timings(build_scatter(dev, n=n, nbins=nbins, nupd=nupd).plan)
    for _ in range(30):
        M.run(w.plan)
        dev.synchronize()
    ts = M.timings(w.plan)
    assert [t.name for t in ts] == w.plan.names
    for t in ts:
        assert 0 < t.samples <= M.NSAMPLES
        assert 0 < t.gpu_ms < 100


def test_copy_pass(dev):
    n = 1000
    a = M.Buffer(dev, np.arange(n, dtype=np.float32))
    b = M.Buffer(dev, np.float32, n)
    c = M.Buffer(dev, np.float32, n)
    g = M.Graph(dev)
    M.copy(g, "copy", b, a)
    M.compute(g, "scale", lambda p: M.dispatch(p, M.kernels.scaleby, (
        M.use(p, c, write=True), M.use(p, b, read=True), 3.0), n))
    plan = M.Plan(g)
    M.run(plan)
    assert np.array_equal(c.array(), np.arange(n, dtype=np.float32) * 3)


def test_set_arg_reaches_the_next_run(dev):
    """Plan.set_arg changes a scalar for the next run!, both for a plan that is
    a single kernel (launched without its graph) and for a fused run."""
    n = 4096 + 3
    a_h = seeded_uniform(5, n, -1, 1, 0)
    b_h = seeded_uniform(5, n, -1, 1, 1)
    a, b = M.Buffer(dev, a_h), M.Buffer(dev, b_h)
    c = M.Buffer(dev, np.float32, n)
    g = M.Graph(dev)
    p = M.compute(g, "scale", lambda p: M.dispatch(p, M.kernels.scaleby, (
        M.use(p, c, write=True), M.use(p, a, read=True), 3.0), n))
    plan = M.Plan(g)
    M.run(plan)
    assert np.array_equal(c.array(), a_h * np.float32(3))
    plan.set_arg(p, 0, 2, -0.5)
    M.run(plan)
    assert np.array_equal(c.array(), a_h * np.float32(-0.5))

    t, d = M.Buffer(dev, np.float32, n), M.Buffer(dev, np.float32, n)
    g2 = M.Graph(dev)
    q = M.compute(g2, "scale", lambda p: M.dispatch(p, M.kernels.scaleby, (
        M.use(p, t, write=True), M.use(p, a, read=True), 2.0), n))
    M.compute(g2, "add", lambda p: M.dispatch(p, M.kernels.add, (
        M.use(p, d, write=True), M.use(p, t, read=True), M.use(p, b, read=True)), n))
    plan2 = M.Plan(g2, fuse=True)
    M.run(plan2)
    assert plan2.nkernels() == 1
    np.testing.assert_allclose(d.array(), a_h * 2 + b_h, rtol=1e-6, atol=1e-7)
    plan2.set_arg(q, 0, 2, 4.0)
    M.run(plan2)
    np.testing.assert_allclose(d.array(), a_h * 4 + b_h, rtol=1e-6, atol=1e-7)

    # the same two passes unfused: two compiled kernels, one graph node each;
    # the scalar is compiled into the first kernel, so set_arg replaces that
    # node's kernel in both barrier modes' graphs
    plan3 = M.Plan(g2)
    for barriers in ("derived", "backend"):
        d.update(np.zeros(n, np.float32))
        M.run(plan3, barriers=barriers)
        assert plan3.nkernels(barriers) == 2
        np.testing.assert_allclose(d.array(), a_h * 4 + b_h, rtol=1e-6, atol=1e-7)
    plan3.set_arg(q, 0, 2, -3.0)
    for barriers in ("derived", "backend"):
        d.update(np.zeros(n, np.float32))
        M.run(plan3, barriers=barriers)
        np.testing.assert_allclose(d.array(), a_h * -3 + b_h, rtol=1e-6, atol=1e-7)


def test_disjoint_slices_both_land(dev):
    """test/test_window.jl:391-420: two writes into disjoint halves of one buffer
    are not ordered against each other, and both land."""
    n = 256
    b = M.Buffer(dev, np.zeros(n, np.float32))
    g = M.Graph(dev)
    M.compute(g, "lower", lambda p: M.dispatch(p, M.kernels.fill_span, (
        M.use(p, b, write=True, range=(1, 128)), 0, 1.0), 128))
    M.compute(g, "upper", lambda p: M.dispatch(p, M.kernels.fill_span, (
        M.use(p, b, write=True, range=(129, 256)), 128, 2.0), 128))
    plan = M.Plan(g)
    assert plan.edges(1) == []
    M.run(plan)
    got = b.array()
    assert np.all(got[:128] == 1.0) and np.all(got[128:] == 2.0)
    # a span past the end is refused before anything is launched
    g2 = M.Graph(dev)
    with pytest.raises(M.ArgumentError):
        M.compute(g2, "past", lambda p: M.dispatch(p, M.kernels.fill_span, (
            M.use(p, b, write=True), 200, 1.0), 128))
        M.Plan(g2)


def test_counters_restart_every_frame(dev):
    """test/test_window.jl:343-384: clear then 512 atomic increments per frame;
    the tally counts frames."""
    g = M.Graph(dev)
    cnt = M.Buffer(dev, np.zeros(1, np.uint32))
    tally = M.Buffer(dev, np.zeros(1, np.uint32))
    M.compute(g, "clear", lambda p: M.dispatch(p, M.kernels.clear_and_tally, (
        M.use(p, cnt, write=True), M.use(p, tally, read=True, write=True)), 1))
    M.compute(g, "accumulate", lambda p: M.dispatch(p, M.kernels.bump_counter, (
        M.use(p, cnt, read=True, write=True),), 512))
    plan = M.Plan(g)
    for _ in range(40):
        M.run(plan)
    assert int(tally.array()[0]) == 40
    assert int(cnt.array()[0]) == 512
