"""The product's compile phases (C++, through the C ABI, no GPU) against the
reference's known answers and against the oracle on random corpora: schedule
order, transitions per pass, offsets, peak, and the edge lowering."""
import json
from pathlib import Path

import numpy as np
import pytest

import mantle_cuda as M
from graphspec import (USAGE, build_oracle, build_product, oracle_transitions, product_key,
                       product_transitions, random_chain_spec, random_usage_spec)
from oracle import oracle as O

G = json.loads((Path(__file__).parent / "golden" / "reference_expectations.json").read_text())


def test_usage_rules_match_the_oracle_exhaustively():
    codes = [USAGE[k] for k in USAGE]
    codes += [c | O.UNORDERED for c in codes if O.base(c) == O.STORAGE]
    for u in codes:
        assert M.reads(u) == O.reads(u) and M.writes(u) == O.writes(u)
        for v in codes:
            assert M.needs_transition(u, v) == O.needs_transition(u, v), (hex(u), hex(v))
    rng = np.random.default_rng(0)
    for _ in range(300):
        seq = [int(x) for x in rng.choice(codes, size=int(rng.integers(1, 9)))]
        init = int(rng.choice([0] + codes))
        got = M.transitions(seq, initial=init)
        want = O.transitions(seq, initial=init or None)
        assert [(t.from_, list(t.waits), t.to) for t in got] == [(t.from_, t.waits, t.to) for t in want]


def test_hazard_rules_golden():
    for names, count in G["hazard_rules"]["cases"]:
        assert len(M.transitions([USAGE[n] for n in names])) == count
    assert len(M.transitions([USAGE[n] for n in G["webgpu"]["usages"]], backend=1)) == 0


def _items(rows):
    out = []
    for r in rows:
        if len(r) == 4 and isinstance(r[3], list):
            out.append(M.Item(r[0], tuple(r[1]), r[2], 1, [(tuple(d), tuple(w) if w else None) for d, w in r[3]]))
        else:
            out.append(M.Item(r[0], tuple(r[1]), r[2], r[3], None, r[4]))
    return out


def test_placement_golden():
    offs, _ = M.place(_items(G["pinned"]["items"]))
    assert offs["a"] == G["pinned"]["want_offset_a"]
    offs, _ = M.place(_items(G["alignment"]["items"]))
    assert offs["b"] % G["alignment"]["align_of_b"] == 0
    assert M.place(_items(G["gaps_height"]["items"]))[1] == G["gaps_height"]["height"]


def test_placement_matches_oracle_on_random_problems():
    rng = np.random.default_rng(1)
    for case in range(200):
        n = int(rng.integers(1, 40))
        rows = []
        for i in range(n):
            lo = int(rng.integers(0, 50))
            hi = lo + int(rng.integers(0, 20))
            size = int(rng.integers(0, 5000))
            align = int(rng.choice([1, 8, 256]))
            gaps = []
            if rng.random() < 0.2 and hi - lo > 4:
                a = lo + int(rng.integers(0, (hi - lo) // 2))
                gaps = [((a, a + 2), (0, max(1, size // 2)) if rng.random() < 0.5 else None)]
            rows.append((str(i), (lo, hi), size, align, gaps))
        for strategy in ("lowest", "best"):
            mi = [M.Item(r[0], r[1], r[2], r[3], r[4]) for r in rows]
            oi = [O.Item(r[0], r[1], r[2], r[3], list(r[4])) for r in rows]
            (mo, mh), (oo, oh) = M.place(mi, strategy), O.place(oi, strategy)
            assert mo == oo and mh == oh, (case, strategy)
        assert M.maxload(mi) == O.maxload(oi)


def test_hand_derived_ten_transitions():
    h = G["hand_set"]
    g, plan, names = build_product(h["graph"], alias=h["alias"])
    want = {(p, (b, None), USAGE[f], USAGE[t], frozenset(USAGE[x] for x in w)) for p, b, f, t, w in h["transitions"]}
    assert product_transitions(g, plan, names) == want
    # Each chain is its own CUDA-graph branch: stage k waits on stage k-1 of the
    # same chain only.
    pos = {p.name: k for k, p in enumerate(plan.passes)}
    for c in (1, 2):
        assert plan.edges(pos[f"c{c} s1"]) == []
        assert plan.edges(pos[f"c{c} s2"]) == [pos[f"c{c} s1"]]
        assert plan.edges(pos[f"c{c} s3"]) == [pos[f"c{c} s2"]]


def test_rps_orders_and_peak():
    e = G["rps_memory_saving"]
    _, fast, _ = build_product(e["graph"], policy=M.Overlap)
    _, small, _ = build_product(e["graph"], policy=M.Compact)
    assert fast.names == e["overlap_order"]
    assert small.names == e["compact_order"]
    assert M.peakbytes(small) * e["peak_ratio"] == M.peakbytes(fast)


def test_program_order_cost_and_six_chains_and_aliasing():
    def cost(spec):
        _, pl, _ = build_product(spec)
        pre = [pl.pre(k) for k in range(len(pl.order))]
        return (sum(1 for x in pre if x), sum(len(x) for x in pre), M.peakbytes(pl))
    e = G["program_order"]
    assert cost(e["declared"]) == cost(e["hoisted"])
    s = G["six_chains"]
    _, loose, _ = build_product(s["graph"], policy=M.Overlap)
    _, tight, _ = build_product(s["graph"], policy=M.Compact)
    assert M.peakbytes(tight) < M.peakbytes(loose)
    assert loose.names[:2] == s["loose_first_two"] and tight.names[:2] == s["tight_first_two"]
    a = G["aliasing_trade"]["graph"]
    _, on, _ = build_product(a, alias=True)
    _, off, _ = build_product(a, alias=False)
    assert M.peakbytes(on) < M.peakbytes(off)


def test_slices_golden():
    s = G["slices"]
    gr = s["graphs"]

    def touched(key):
        g, pl, names = build_product(gr[key])
        return pl, {t.resource for k in range(len(pl.order)) for t in pl.pre(k)}

    assert len(touched("whole")[1]) == s["whole_resources"]
    assert len(touched("sliced")[1]) == s["sliced_resources"]
    assert len(touched("identical")[1]) == s["identical_resources"]
    assert len(touched("reader_whole")[0].pre(1)) == s["reader_whole_waits"]
    assert len(touched("reader_sliced")[0].pre(1)) == s["reader_sliced_waits"]
    pl, _ = touched("partial")
    segs = [{t.resource for t in pl.pre(k)} for k in range(3)]
    assert pl.pre(1) and segs[0] & segs[1] and not segs[0] & segs[2]
    assert pl.edges(1) == [0] and pl.edges(2) == []  # mid waits on low; tail waits on nothing
    pl, _ = touched("parts_then_whole")
    assert len(pl.pre(4)) == s["whole_after_parts_transitions"]
    assert pl.edges(4) == [0, 1, 2, 3] and all(pl.edges(k) == [] for k in range(4))
    pl, _ = touched("sliced_transient")
    assert any(t.resource == 0 for k in range(len(pl.order)) for t in pl.pre(k))
    g = M.Graph(None)
    b = M.VirtualBuffer(np.float32, 256)
    with pytest.raises(M.ArgumentError):
        M.compute(g, "past the end", lambda p: M.use(p, b, write=True, range=(200, 400)))


def test_never_used_transient_is_named():
    g = M.Graph(None)
    used = M.Transient.Buffer(g, np.float32, 1 << 10)
    M.Transient.Buffer(g, np.float32, 1 << 9)
    src = M.VirtualBuffer(np.float32, 1 << 10)
    M.compute(g, "c", lambda p: (M.use(p, used, write=True), M.use(p, src, read=True)))
    with pytest.raises(M.ArgumentError, match=G["never_used"]["message"]):
        M.Plan(g)


def test_update_pass_is_declared_first():
    g = M.Graph(None)
    pos = M.VirtualBuffer(np.float32, 100)
    out = M.VirtualBuffer(np.float32, 100)
    M.compute(g, "plot", lambda p: (M.use(p, pos, read=True), M.use(p, out, write=True)))
    M.Update(g, pos)
    plan = M.Plan(g)
    assert plan.names == ["updates", "plot"]
    assert plan.edges(1) == [0]


def _compare(spec, **kw):
    g, plan, names = build_product(spec, **kw)
    og = build_oracle(spec)
    res = O.compile_graph(og, alias=kw.get("alias", True),
                          policy="compact" if kw.get("policy") is M.Compact else "overlap")
    assert plan.names == [og.passes[i]["name"] for i in res["order"]]
    assert product_transitions(g, plan, names) == oracle_transitions(og, res)
    assert M.peakbytes(plan) == res["peak"] and M.naivebytes(plan) == res["naive"]
    return g, plan, og, res


@pytest.mark.parametrize("slicing", [0.0, 0.5])
@pytest.mark.parametrize("policy", [M.Overlap, M.Compact])
def test_random_usage_graphs_match_the_oracle(slicing, policy):
    """bench/stress.jl over this repository's generator: the product's walk is
    the local hazard set, and equals the oracle's."""
    for seed in range(20):
        spec = random_usage_spec(np.random.default_rng(seed), slicing=slicing, unordered=0.15)
        g, plan, og, res = _compare(spec, policy=policy)
        name = {v: k for k, v in og.ids.items()}
        local = set()
        for p, (pid, span), f, t, w in O.local_hazards(og, res):
            local.add((p, (name[pid], tuple(span) if span else None), f, t, w))
        assert oracle_transitions(og, res) == local


@pytest.mark.parametrize("alias", [True, False])
def test_random_chain_graphs_match_the_oracle(alias):
    for seed in range(25):
        spec = random_chain_spec(np.random.default_rng(100 + seed))
        g, plan, og, res = _compare(spec, alias=alias)
        ntrans = len(spec["transients"])
        for t in range(ntrans):
            assert plan.offset(g.transients[t]) == res["offsets"][t]


def test_edges_order_every_conflicting_pair():
    """The lowering's promise: two passes that touch overlapping bytes, at least
    one writing, not both unordered, are ordered by a path of edges; passes
    that do not conflict are never ordered unless a chain through others does."""
    for seed in range(40):
        spec = random_usage_spec(np.random.default_rng(500 + seed), slicing=0.5, unordered=0.2)
        g, plan, names = build_product(spec)
        n = len(plan.order)
        reach = [set() for _ in range(n)]
        for k in range(n):
            for q in plan.edges(k):
                assert q < k
                reach[k] |= reach[q] | {q}
        by = {p["name"]: p for p in spec["passes"]}
        ps = [by[p.name] for p in plan.passes]

        def overlap(a, b):
            (ra, ua, xa), (rb, ub, xb) = a, b
            if ra != rb:
                return False
            if xa is None or xb is None:
                return True
            return max(xa[0], xb[0]) <= min(xa[1], xb[1])

        for j in range(n):
            for i in range(j):
                conflict = any(
                    overlap(a, b) and (O.writes(USAGE[a[1]]) or O.writes(USAGE[b[1]]))
                    and not (a[1].startswith("u") and b[1].startswith("u"))
                    for a in ps[i]["usages"] for b in ps[j]["usages"])
                if conflict:
                    assert i in reach[j], (seed, i, j)


def _chain_graph(dev, n, keep_t3=False):
    """The eight-op chain over transients; with keep_t3 a copy pass reads the
    fourth intermediate after the chain, so that value must reach memory."""
    from mantle_cuda import kernels as K
    g = M.Graph(dev)
    mk = (lambda: M.VirtualBuffer(np.float32, n)) if dev is None else (lambda: M.Buffer(dev, np.float32, n))
    x, y, z, out, side = mk(), mk(), mk(), mk(), mk()
    t = [M.Transient.Buffer(g, np.float32, n) for _ in range(7)]
    W = lambda p, b: M.use(p, b, write=True)  # noqa: E731
    R = lambda p, b: M.use(p, b, read=True)  # noqa: E731
    M.compute(g, "axpy", lambda p: M.dispatch(p, K.axpy, (W(p, t[0]), R(p, x), R(p, y), 0.5), n))
    M.compute(g, "mul", lambda p: M.dispatch(p, K.mul, (W(p, t[1]), R(p, t[0]), R(p, z)), n))
    M.compute(g, "add", lambda p: M.dispatch(p, K.add, (W(p, t[2]), R(p, t[1]), R(p, y)), n))
    M.compute(g, "fma", lambda p: M.dispatch(p, K.fma, (W(p, t[3]), R(p, t[2]), R(p, x), R(p, z)), n))
    M.compute(g, "abs", lambda p: M.dispatch(p, K.abs, (W(p, t[4]), R(p, t[3])), n))
    M.compute(g, "sqrt", lambda p: M.dispatch(p, K.sqrt_abs, (W(p, t[5]), R(p, t[4])), n))
    M.compute(g, "scale", lambda p: M.dispatch(p, K.scale, (W(p, t[6]), R(p, t[5]), 2.0), n))
    M.compute(g, "sub", lambda p: M.dispatch(p, K.sub, (W(p, out), R(p, t[6]), R(p, x)), n))
    if keep_t3:
        M.copy(g, "keep t4", side, t[3])
    return g, dict(x=x, y=y, z=z, out=out, side=side)


def test_fusion_merges_the_chain_and_elides_its_transients():
    n = 1 << 20
    g, _ = _chain_graph(None, n)
    unfused = M.Plan(g)
    assert [p.name for p in unfused.passes] == ["axpy", "mul", "add", "fma", "abs", "sqrt", "scale", "sub"]
    assert M.peakbytes(unfused) == 2 * 4 * n
    fused = M.Plan(g, fuse=True)
    assert len(fused.passes) == 1 and fused.passes[0].name == "axpy"
    assert M.peakbytes(fused) == 0  # every intermediate lives in registers
    assert M.naivebytes(fused) == 7 * 4 * n


def test_fusion_keeps_a_transient_read_outside_the_run():
    n = 1 << 16
    g, _ = _chain_graph(None, n, keep_t3=True)
    fused = M.Plan(g, fuse=True)
    # the run ends before the copy; t4 is stored, the other six are not
    assert [p.name for p in fused.passes] == ["axpy", "keep t4"]
    assert M.peakbytes(fused) == 4 * n
    # the copy waits for the fused run
    assert fused.edges(1) == [0]
