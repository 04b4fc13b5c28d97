"""The oracle against the reference's own known answers (tests/golden), before
anything is compared with it. CPU only."""
import json
from pathlib import Path

import pytest

from graphspec import USAGE, build_oracle, oracle_key, oracle_transitions
from oracle import oracle as O

G = json.loads((Path(__file__).parent / "golden" / "reference_expectations.json").read_text())
U = lambda names: [USAGE[n] for n in names]  # noqa: E731


def test_spans_are_half_open():
    s = G["spans"]
    assert O.overlaps((0, 3), (2, 5)) == s["overlap_0_3__2_5"]
    assert O.overlaps((0, 3), (3, 5)) == s["overlap_0_3__3_5"]
    assert (9 - 3) == s["length_3_9"]


def test_csv_end_column_trap_and_gaps():
    c = G["csv_end_trap"]
    assert list(O.readproblem(c["upper_file"], 10)[0][0].live) == c["upper_live"]
    assert list(O.readproblem(c["end_file"], 10)[0][0].live) == c["end_live"]
    g = G["csv_gaps"]
    gaps = O.readproblem(g["file"], 10)[0][0].gaps
    assert [[list(d), list(w) if w else None] for d, w in gaps] == g["gaps"]


def test_segments_apply_gaps():
    for case in G["segments"]["cases"]:
        name, live, size, gaps = case["item"]
        it = O.Item(name, tuple(live), size, 1, [(tuple(d), tuple(w) if w else None) for d, w in gaps])
        assert [[list(s), h] for s, h in O.segments(it)] == case["want"]


def _items(rows):
    out = []
    for r in rows:
        name, live, size = r[0], tuple(r[1]), r[2]
        if len(r) == 4 and isinstance(r[3], list):
            out.append(O.Item(name, live, size, 1, [(tuple(d), tuple(w) if w else None) for d, w in r[3]]))
        else:
            out.append(O.Item(name, live, size, r[3], [], r[4]))
    return out


def valid(items, offsets):
    for a in items:
        for b in items:
            if a.id < b.id and O.conflicts(a, b):
                oa, ob = offsets[a.id], offsets[b.id]
                if oa < ob + b.size and ob < oa + a.size:
                    return False
    return True


def test_pinned_alignment_and_gaps():
    items = _items(G["pinned"]["items"])
    offs, _ = O.place(items)
    assert offs["a"] == G["pinned"]["want_offset_a"] and valid(items, offs)
    items = _items(G["alignment"]["items"])
    offs, _ = O.place(items)
    assert offs["b"] % G["alignment"]["align_of_b"] == 0 and valid(items, offs)
    items = _items(G["gaps_height"]["items"])
    assert O.place(items)[1] == G["gaps_height"]["height"]
    for strategy in ("lowest", "best"):
        offs, h = O.place(items, strategy)
        assert h >= O.maxload(items) and valid(items, offs)


def test_hazard_rules():
    for usages, count in G["hazard_rules"]["cases"]:
        assert len(O.transitions(U(usages))) == count
    assert O.needs_transition(O.SAMPLED, O.COPY_SRC) == G["buffers_have_no_layouts"]["needs_transition_buffer_sampled_copysrc"]
    w = G["write_waits_on_readers"]
    last = O.transitions(U(w["usages"]))[-1]
    assert set(last.waits) == set(U(w["last_waits"]))
    assert len(O.transitions(U(G["webgpu"]["usages"]), webgpu=True)) == G["webgpu"]["count"]
    for name in ("ColorClear", "ColorKeep", "DepthClear", "DepthKeep"):
        u = USAGE[name]
        assert [O.discards(u), O.reads(u), O.writes(u)] == G["discards"][name]


def _hand(entry, key_of):
    return {(p, (b, None), USAGE[f], USAGE[t], frozenset(USAGE[x] for x in w))
            for p, b, f, t, w in entry["transitions"]}


def test_hand_derived_ten_transitions():
    h = G["hand_set"]
    g = build_oracle(h["graph"])
    r = O.compile_graph(g, alias=h["alias"])
    assert oracle_transitions(g, r) == _hand(h, None)
    assert sorted(len(x) for x in r["prepass"]) == sorted(h["per_pass_counts"])
    name = {v: k for k, v in g.ids.items()}
    local = {(p, (name[pid], span), f, t, w) for p, (pid, span), f, t, w in O.local_hazards(g, r)}
    assert local == oracle_transitions(g, r)


def test_rps_schedule_orders_and_peak():
    e = G["rps_memory_saving"]
    for policy, want in (("overlap", e["overlap_order"]), ("compact", e["compact_order"])):
        g = build_oracle(e["graph"])
        r = O.compile_graph(g, policy=policy)
        assert [g.passes[i]["name"] for i in r["order"]] == want
    fast = O.compile_graph(build_oracle(e["graph"]), policy="overlap")["peak"]
    small = O.compile_graph(build_oracle(e["graph"]), policy="compact")["peak"]
    assert small * e["peak_ratio"] == fast


def _cost(spec):
    g = build_oracle(spec)
    r = O.compile_graph(g)
    return (sum(1 for x in r["prepass"] if x), sum(len(x) for x in r["prepass"]), r["peak"]), g, r


def test_program_order_costs_the_same_and_is_a_linear_extension():
    e = G["program_order"]
    forced, _, _ = _cost(e["hoisted"])
    ours, g, r = _cost(e["declared"])
    assert ours == forced
    pos = {g.passes[i]["name"]: k for k, i in enumerate(r["order"])}
    ps = g.passes
    for j in range(len(ps)):
        for i in range(j):
            dep = any(a == b and (O.writes(Ua) or O.writes(Ub)) for a, Ua in ps[i]["usages"] for b, Ub in ps[j]["usages"])
            assert not dep or pos[ps[i]["name"]] < pos[ps[j]["name"]]


def test_compact_policy_cuts_peak_and_aliasing_trade():
    e = G["six_chains"]
    gl, gt = build_oracle(e["graph"]), build_oracle(e["graph"])
    loose, tight = O.compile_graph(gl, policy="overlap"), O.compile_graph(gt, policy="compact")
    assert tight["peak"] < loose["peak"]
    assert [gl.passes[i]["name"] for i in loose["order"]][:2] == e["loose_first_two"]
    assert [gt.passes[i]["name"] for i in tight["order"]][:2] == e["tight_first_two"]
    a = G["aliasing_trade"]["graph"]
    on, off = O.compile_graph(build_oracle(a), alias=True), O.compile_graph(build_oracle(a), alias=False)
    assert on["peak"] < off["peak"]
    assert sum(1 for x in on["prepass"] if x) >= sum(1 for x in off["prepass"] if x)


def test_slices():
    s = G["slices"]
    gr = s["graphs"]

    def touched(spec):
        g = build_oracle(spec)
        r = O.compile_graph(g)
        return g, r, {t.resource for x in r["prepass"] for t in x}

    assert len(touched(gr["whole"])[2]) == s["whole_resources"]
    assert len(touched(gr["sliced"])[2]) == s["sliced_resources"]
    assert len(touched(gr["identical"])[2]) == s["identical_resources"]
    for key, want in (("reader_whole", s["reader_whole_waits"]), ("reader_sliced", s["reader_sliced_waits"])):
        g, r, _ = touched(gr[key])
        assert len(r["prepass"][1]) == want
    g, r, _ = touched(gr["partial"])
    segs = [{t.resource for t in r["prepass"][k]} for k in range(3)]
    assert r["prepass"][1] and segs[0] & segs[1] and not segs[0] & segs[2]
    g, r, _ = touched(gr["parts_then_whole"])
    assert len(r["prepass"][4]) == s["whole_after_parts_transitions"]
    g, r, _ = touched(gr["sliced_transient"])
    assert any(t.resource == 0 for x in r["prepass"] for t in x)
    with pytest.raises(ValueError):
        g = O.OGraph()
        g.buffer("b", 256)
        g.use(g.add_pass("past the end"), "b", O.SW, (200, 400))


def test_transient_nothing_uses_is_an_error():
    g = O.OGraph()
    g.transient("used", 1024)
    g.transient("unused", 512)
    g.buffer("src", 1024)
    p = g.add_pass("c")
    g.use(p, "used", O.SW)
    g.use(p, "src", O.SR)
    with pytest.raises(ValueError, match="never used"):
        O.compile_graph(g)
