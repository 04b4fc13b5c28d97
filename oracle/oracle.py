"""CPU oracle for the Mantle.jl hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs import this module, and only as the checker (or as the timed CPU
baseline). The product (mantle.jl_b200) never imports it.

Two halves:

* A pure-Python restatement of the reference's portable algorithms — the usage
  vocabulary (src/sync/usage.jl), the hazard walk (src/sync/transition.jl), the
  placer and its bound (src/memory/*.jl), and the compile phases of the Lava
  backend (ext/MantleLavaExt.jl:1329-1822): Dag, Schedule, Liveness, Place,
  Aliasing, Barriers. Each function cites what it follows. Independent of the
  product's C++ so the two can be compared.
* ctypes access to mantle_oracle.c for the numeric work (elementwise chain,
  in-place updates, scatter-add/histogram), built by oracle/build.py.

Parity pins: the known answers of the reference's own tests, transcribed with
their file:line into tests/golden/reference_expectations.json, are checked
against this module by tests/test_oracle_golden.py. The reference cannot run
here (Julia and its Vulkan stack are absent), so there are no generated
fixtures; the numeric oracle for the scatter-add, the eight-op chain, the FFT,
GEMM and convolution has no reference implementation to pin against ("parity
unpinned" for those: the workload statement is the definition).

One deliberate deviation, also made by the product: Liveness counts a pass that
names only a slice of a transient as touching it. The reference looks the
transient up by its own id only (ext/MantleLavaExt.jl:1484-1490), so a
slice-only use does not extend the interval, and the placer may give those
bytes to another transient live at that pass.
"""
from __future__ import annotations

import ctypes as C
import itertools
import os
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# ── usage vocabulary (src/sync/usage.jl) ────────────────────────────────────
# The same 32-bit codes the C ABI uses, so results compare without a mapping.
STORAGE, COPY_SRC, COPY_DST, INDIRECT, UNIFORM, VERTICES, INDICES = 1, 2, 3, 4, 5, 6, 7
SAMPLED, PRESENT, TRACE_READ, TRACE_BUILD, COLOR, DEPTH, UNDEFINED = 8, 9, 10, 11, 12, 13, 14
RD, WR, SRD, SWR, DISCARD, IMAGE, UNORDERED = 1 << 5, 1 << 6, 1 << 7, 1 << 8, 1 << 9, 1 << 10, 1 << 11
BASE = 0x1F

SR = STORAGE | RD          # Storage{BufferKind,ReadOnly}
SW = STORAGE | WR          # Storage{BufferKind,WriteOnly}
SRW = STORAGE | RD | WR    # Storage{BufferKind,ReadWrite}


def base(u: int) -> int:
    return u & BASE


def inner(u: int) -> int:
    """inner(Unordered{U}) = U, usage.jl:163-164."""
    return u & ~UNORDERED


def unordered(u: int) -> bool:
    return bool(u & UNORDERED)


def reads(u: int) -> bool:
    """usage.jl:120-126."""
    b = base(u)
    if b in (UNDEFINED, COPY_DST, TRACE_BUILD):
        return False
    if b == STORAGE:
        return bool(u & RD)
    if b == COLOR:
        return not (u & DISCARD)
    if b == DEPTH:
        return not (u & DISCARD) and bool(u & (RD | SRD))
    return True


def writes(u: int) -> bool:
    """usage.jl:128-133."""
    b = base(u)
    if b in (COPY_DST, TRACE_BUILD, COLOR):
        return True
    if b == STORAGE:
        return bool(u & WR)
    if b == DEPTH:
        return bool(u & (WR | SWR))
    return False


def discards(u: int) -> bool:
    """usage.jl:142-144."""
    return base(u) in (COLOR, DEPTH) and bool(u & DISCARD)


def needs_transition(before: int, after: int, webgpu: bool = False) -> bool:
    """The portable rule, src/sync/transition.jl:56-66; WebGPU: never (backend.jl:22)."""
    if webgpu:
        return False
    both_unordered = unordered(before) and unordered(after)
    b, a = inner(before), inner(after)
    if not writes(b) and not writes(a):
        return False
    if both_unordered:
        return False
    return b != a or writes(b)


@dataclass
class Transition:
    resource: int
    from_: int
    waits: list
    to: int


@dataclass
class ResourceState:
    current: int | None = None
    pending: list = field(default_factory=list)


def transition_step(out: list, resource, st: ResourceState, nxt: int, webgpu: bool = False) -> None:
    """transition!(out, backend, resource, state, next), transition.jl:79-92."""
    frm = st.current
    if frm is not None and needs_transition(frm, nxt, webgpu):
        if writes(nxt):
            waits = []
            for u in [frm] + st.pending:
                if u not in waits:
                    waits.append(u)
        else:
            waits = [frm]
        out.append(Transition(resource, frm, waits, nxt))
        st.current = nxt
    elif frm is None:
        st.current = nxt
    if writes(nxt):
        st.pending = []
    else:
        st.pending.append(nxt)


def transitions(usages, initial=None, webgpu=False) -> list[Transition]:
    """transitions(backend, kind, usages; initial), transition.jl:103-111."""
    st = ResourceState(initial, [])
    out: list[Transition] = []
    for u in usages:
        transition_step(out, 1, st, u, webgpu)
    return out


# ── memory (src/memory/*.jl) ────────────────────────────────────────────────
@dataclass
class Item:
    """model.jl:39-49. live = (lower, upper), half-open."""
    id: str
    live: tuple
    size: int
    alignment: int = 1
    gaps: list = field(default_factory=list)   # [((lo, hi), window or None)]
    offset: int | None = None


def overlaps(a, b) -> bool:
    """interval.jl:26: half-open spans share a point."""
    return a[0] < b[1] and b[0] < a[1]


def segments(i: Item):
    """model.jl:54-65."""
    if not i.gaps:
        return [(i.live, i.size)]
    out = []
    t = i.live[0]
    for during, window in sorted(i.gaps, key=lambda g: g[0][0]):
        if t < during[0]:
            out.append(((t, during[0]), i.size))
        if window is not None:
            out.append((during, window[1] - window[0]))
        t = during[1]
    if t < i.live[1]:
        out.append(((t, i.live[1]), i.size))
    return out


def conflicts(a: Item, b: Item) -> bool:
    """placement.jl:7-14."""
    if not overlaps(a.live, b.live):
        return False
    if not a.gaps and not b.gaps:
        return True
    return any(overlaps(sa, sb) for sa, _ in segments(a) for sb, _ in segments(b))


def alignup(x: int, a: int) -> int:
    return ((x + a - 1) // a) * a


def _priority(i: Item):
    """placement.jl:37: (-size, -length(live), id)."""
    return (-i.size, -(i.live[1] - i.live[0]), i.id)


def place(items: list[Item], strategy: str = "lowest"):
    """placement.jl:46-99 -> ({id: offset}, height)."""
    order = sorted([k for k, it in enumerate(items) if it.offset is not None], key=lambda k: _priority(items[k])) + \
        sorted([k for k, it in enumerate(items) if it.offset is None], key=lambda k: _priority(items[k]))
    offsets: dict[str, int] = {}
    settled: list[int] = []
    height = 0
    for idx in order:
        item = items[idx]
        blocked = sorted((offsets[items[j].id], offsets[items[j].id] + items[j].size)
                         for j in settled if conflicts(item, items[j]))
        if item.offset is not None:
            off = item.offset
        elif strategy == "best":
            best, waste, cursor = 0, None, 0
            for lo, hi in blocked:
                if cursor + item.size <= lo and (waste is None or (lo - cursor) - item.size < waste):
                    best, waste = cursor, (lo - cursor) - item.size
                cursor = max(cursor, alignup(hi, item.alignment))
            off = cursor if waste is None else best
        else:
            off = 0
            for lo, hi in blocked:
                if off + item.size <= lo:
                    break
                off = max(off, alignup(hi, item.alignment))
        for lo, hi in blocked:
            if off < hi and lo < off + item.size:
                raise ValueError(f"item {item.id} at {off} collides with [{lo}, {hi})")
        offsets[item.id] = off
        settled.append(idx)
        height = max(height, off + item.size)
    return offsets, height


def maxload(items: list[Item]) -> int:
    """bound.jl:14-28."""
    ev = []
    for it in items:
        for span, h in segments(it):
            if span[0] == span[1]:
                continue
            ev += [(span[0], h), (span[1], -h)]
    if not ev:
        return 0
    ev.sort()
    best = cur = 0
    for _, d in ev:
        cur += d
        best = max(best, cur)
    return best


def fragmentation(items: list[Item], height: int):
    """bound.jl:41-44."""
    L = maxload(items)
    return (1.0, 0.0) if L == 0 else (height / L, max((i.size for i in items), default=0) / L)


def parsegap(s: str, addend: int):
    """csv.jl:10-22: `lo-hi` or `lo-hi@wlo:whi`; `end`-style files add 1 to hi."""
    at = s.split("@")
    span = at[0].split("-")
    if len(span) != 2:
        raise ValueError(f"improperly formed gap: {s}")
    during = (int(span[0]), int(span[1]) + addend)
    window = None
    if len(at) > 1:
        w = at[1].split(":")
        if len(w) != 2:
            raise ValueError(f"improperly formed gap: {s}")
        window = (int(w[0]), int(w[1]))
    return (during, window)


def readproblem(text: str, capacity: int):
    """csv.jl:24-56 over the file's text: a column named `end` is an inclusive last
    time and adds 1 to every upper bound, gaps included; `upper` is exclusive."""
    lines = [ln for ln in text.splitlines() if ln.strip()]
    addend = 0
    cols = {}
    for i, raw in enumerate(x.strip() for x in lines[0].split(",")):
        key = {"buffer": "id", "buffer_id": "id", "begin": "lower", "start": "lower"}.get(raw, raw)
        if key == "end":
            key, addend = "upper", 1
        if key in cols:
            raise ValueError(f"duplicate column: {key}")
        cols[key] = i
    for req in ("id", "lower", "upper", "size"):
        if req not in cols:
            raise ValueError(f"missing required column: {req}")
    items = []
    for line in lines[1:]:
        f = line.split(",")
        if len(f) != len(cols):
            raise ValueError(f"row has {len(f)} fields, header has {len(cols)}")
        at = lambda k: f[cols[k]]  # noqa: E731
        gaps = [parsegap(g, addend) for g in at("gaps").split(" ") if g] if "gaps" in cols else []
        items.append(Item(at("id"), (int(at("lower")), int(at("upper")) + addend), int(at("size")),
                          int(at("alignment")) if "alignment" in cols else 1, gaps,
                          int(at("offset")) if "offset" in cols else None))
    return items, capacity


# ── graph model and compile phases (ext/MantleLavaExt.jl) ──────────────────
@dataclass
class Res:
    kind: str            # "persistent" | "transient" | "view"
    n: int
    elem: int = 4
    parent: int = 0
    rng: tuple | None = None  # (first, last), 1-based inclusive
    tindex: int = -1


class OGraph:
    """The recorded graph: resource ids handed out on first use (resourceid,
    :526-530), slices interned by (parent, range) (:700-710), the shared update
    pass declared first (:785-792)."""

    def __init__(self):
        self.res: dict[int, Res] = {}
        self.ids: dict[object, int] = {}
        self.views: dict[tuple, int] = {}
        self.transients: list[object] = []   # keys, in creation order
        self.tsize: dict[object, int] = {}
        self.passes: list[dict] = []

    def _rid(self, key, make) -> int:
        if key not in self.ids:
            rid = len(self.ids) + 1
            self.ids[key] = rid
            self.res[rid] = make()
        return self.ids[key]

    def buffer(self, key, n, elem=4):
        self._persist = getattr(self, "_persist", {})
        self._persist[key] = (n, elem)
        return key

    def transient(self, key, n, elem=4):
        self.transients.append(key)
        self.tsize[key] = (n, elem)
        return key

    def rid_of(self, key) -> int:
        if key in self.tsize:
            n, e = self.tsize[key]
            return self._rid(key, lambda: Res("transient", n, e, tindex=self.transients.index(key)))
        n, e = self._persist[key]
        return self._rid(key, lambda: Res("persistent", n, e))

    def view(self, pid: int, rng) -> int:
        k = (pid, tuple(rng))
        if k not in self.views:
            parent = self.res[pid]
            vid = len(self.ids) + 1
            self.ids[("view", k)] = vid
            self.res[vid] = Res("view", rng[1] - rng[0] + 1, parent.elem, pid, tuple(rng))
            self.views[k] = vid
        return self.views[k]

    def add_pass(self, name, kind="compute") -> dict:
        p = {"name": name, "kind": kind, "usages": []}
        self.passes.append(p)
        return p

    def use(self, p, key, usage, rng=None) -> int:
        pid = self.rid_of(key)
        if rng is not None:
            n = self.res[pid].n
            if not (rng[0] >= 1 and rng[1] <= n):
                raise ValueError(f"use(): range {rng} is outside the buffer's 1:{n}.")
            rid = self.view(pid, rng)
        else:
            rid = pid
        p["usages"].append((rid, usage))
        return rid

    def update(self, key):
        up = next((p for p in self.passes if p["kind"] == "update"), None)
        if up is None:
            up = {"name": "updates", "kind": "update", "usages": []}
            self.passes.insert(0, up)
        rid = self.rid_of(key)
        if not any(u[0] == rid for u in up["usages"]):
            up["usages"].append((rid, COPY_DST))

    def overlapping(self, a: int, b: int) -> bool:
        """:1329-1345."""
        if a == b:
            return True
        ra, rb = self.res.get(a), self.res.get(b)
        if ra is None or rb is None:
            return False
        if ra.kind != "view" and rb.kind != "view":
            return False
        pa = ra.parent if ra.kind == "view" else a
        pb = rb.parent if rb.kind == "view" else b
        if pa != pb:
            return False
        if not (ra.kind == "view" and rb.kind == "view"):
            return True
        return max(ra.rng[0], rb.rng[0]) <= min(ra.rng[1], rb.rng[1])

    def transient_of(self, rid: int) -> int:
        r = self.res[rid]
        if r.kind == "view":
            r = self.res[r.parent]
        return r.tindex if r.kind == "transient" else -1


SCORE_MAX = 0x1FFF


def compile_graph(g: OGraph, alias=True, policy="overlap"):
    """Dag, Schedule, Liveness, Place, Aliasing, Barriers (src/phases.jl:90)."""
    ps = g.passes
    n = len(ps)
    # Dag, :1353-1368
    deps = [[] for _ in ps]
    for j in range(n):
        for i in range(j):
            if any(g.overlapping(idi, idj) and (writes(Ui) or writes(Uj))
                   for idj, Uj in ps[j]["usages"] for idi, Ui in ps[i]["usages"]):
                deps[j].append(i)
    # Schedule, :1385-1466
    order = []
    if n:
        remaining = [len(d) for d in deps]
        dependents = [[] for _ in range(n)]
        for j in range(n):
            for i in deps[j]:
                dependents[i].append(j)

        def ids(p):
            out = []
            for rid, _ in p["usages"]:
                if rid not in out:
                    out.append(rid)
            return out

        touches: dict[int, int] = {}
        for p in ps:
            for rid in ids(p):
                touches[rid] = touches.get(rid, 0) + 1
        seen: dict[int, int] = {}

        def bytesof(rid):
            r = g.res.get(rid)
            return r.n * r.elem if r is not None and r.kind == "transient" else 0

        maxalloc = max(1, max((sum(bytesof(r) for r in ids(p)) for p in ps), default=0))
        mshift, oshift = (16, 0) if policy == "compact" else (0, 16)
        ready = [i for i in range(n) if remaining[i] == 0]
        while ready:
            best, bestscore = 0, -1
            for k, i in enumerate(ready):
                alloc = freed = 0
                for rid in ids(ps[i]):
                    b = bytesof(rid)
                    if b == 0:
                        continue
                    s = seen.get(rid, 0)
                    if s == 0:
                        alloc += b
                    if s + 1 == touches[rid]:
                        freed += b
                mem = min(max((SCORE_MAX * (maxalloc - alloc)) // maxalloc, 0), SCORE_MAX) + \
                    min(max((SCORE_MAX * freed) // maxalloc, 0), SCORE_MAX)
                ordv = min(max(n - (i + 1), 0), 0xFFFF)
                score = (mem << mshift) | (ordv << oshift)
                if score > bestscore:
                    best, bestscore = k, score
            i = ready.pop(best)
            order.append(i)
            for rid in ids(ps[i]):
                seen[rid] = seen.get(rid, 0) + 1
            for j in dependents[i]:
                remaining[j] -= 1
                if remaining[j] == 0:
                    ready.append(j)
        if len(order) != n:
            raise ValueError("cycle in the DAG")
    # Liveness, :1478-1507 (slice uses count for their transient; see module doc)
    T = len(g.transients)
    first, last = [None] * T, [0] * T
    for pos, i in enumerate(order, start=1):
        for rid, _ in ps[i]["usages"]:
            t = g.transient_of(rid)
            if t < 0:
                continue
            first[t] = pos if first[t] is None else min(first[t], pos)
            last[t] = max(last[t], pos)
    for t in range(T):
        if last[t] == 0:
            raise ValueError(f"transient {t + 1} is never used by any pass")
    lastpass = max(last, default=0) + 1
    nbytes = [g.tsize[k][0] * g.tsize[k][1] for k in g.transients]
    items = [Item(str(t + 1), (first[t], last[t] + 1) if alias else (0, lastpass), nbytes[t], 256)
             for t in range(T)]
    # Place, :1549-1568
    offsets_by_id, peak = place(items) if items else ({}, 0)
    offsets = [offsets_by_id.get(str(t + 1), 0) for t in range(T)]
    # Aliasing, :1582-1593
    alias_begins: dict[int, list] = {}
    for i in range(T):
        for j in range(T):
            if i == j or not (last[j] < first[i]):
                continue
            if offsets[i] < offsets[j] + nbytes[j] and offsets[j] < offsets[i] + nbytes[i]:
                alias_begins.setdefault(first[i], []).append((i, j))
    # Barriers, :1650-1822
    byparent: dict[int, list] = {}
    slices: dict[int, list] = {}
    for (pid, rng), vid in list(g.views.items()):
        byparent.setdefault(pid, []).append(rng)
        slices.setdefault(pid, []).append(vid)
    segs: dict[int, list] = {}
    for pid, ranges in byparent.items():
        nel = g.res[pid].n
        cuts = sorted(set([1, nel + 1] + [r[0] for r in ranges] + [r[1] + 1 for r in ranges]))
        spans = [(cuts[k], cuts[k + 1] - 1) for k in range(len(cuts) - 1) if cuts[k + 1] - 1 >= cuts[k]]
        sids = [g.view(pid, s) for s in spans]
        segs[pid] = sids
        for r in ranges:
            segs[g.views[(pid, r)]] = [sids[k] for k, s in enumerate(spans) if s[0] >= r[0] and s[1] <= r[1]]

    def segments_of(rid):
        return segs.get(rid, [rid])

    final: dict[int, int] = {}
    for i in order:
        for rid, U in ps[i]["usages"]:
            for sid in segments_of(rid):
                final[sid] = U
    states: dict[int, ResourceState] = {}

    def state(sid):
        if sid not in states:
            states[sid] = ResourceState(final.get(sid), [])
        return states[sid]

    prepass = []
    trid = [g.rid_of(k) for k in g.transients]
    for pos, i in enumerate(order, start=1):
        p = ps[i]
        pre: list[Transition] = []
        for rid, U in p["usages"]:
            for sid in segments_of(rid):
                transition_step(pre, sid, state(sid), U)
        needed = list(pre)
        handovers = alias_begins.get(pos, [])
        for newi in dict.fromkeys(h[0] for h in handovers):
            to = next((U for rid, U in p["usages"] if g.overlapping(rid, trid[newi])), None)
            if to is None:
                continue
            waits = []
            for a, o in handovers:
                if a != newi:
                    continue
                keys = [trid[o]] + slices.get(trid[o], []) + segments_of(trid[o])
                for k in keys:
                    st = states.get(k)
                    if st is not None and st.current is not None and st.current not in waits:
                        waits.append(st.current)
            if not waits:
                continue
            needed.append(Transition(0, waits[0], waits, to))
        prepass.append(needed)
    return {"order": order, "deps": deps, "prepass": prepass, "peak": peak, "naive": sum(nbytes),
            "offsets": offsets, "alias_begins": alias_begins, "items": items}


def local_hazards(g: OGraph, result) -> set:
    """The local barrier set from the declared usages alone (bench/stress.jl:151-196):
    atomic partition derived here, state seeded from each piece's last use."""
    ps = [g.passes[i] for i in result["order"]]
    ranges: dict[int, list] = {}

    def normal(rid):
        r = g.res[rid]
        return (r.parent, r.rng) if r.kind == "view" else (rid, None)

    for p in ps:
        for rid, _ in p["usages"]:
            pid, span = normal(rid)
            if span is not None:
                ranges.setdefault(pid, []).append(span)
    spansof = {}
    for pid, rs in ranges.items():
        nel = g.res[pid].n
        cuts = sorted(set([1, nel + 1] + [r[0] for r in rs] + [r[1] + 1 for r in rs]))
        spansof[pid] = [(cuts[k], cuts[k + 1] - 1) for k in range(len(cuts) - 1) if cuts[k + 1] - 1 >= cuts[k]]

    def pieces(rid):
        pid, span = normal(rid)
        if pid not in spansof:
            return [(pid, span)]
        return [(pid, s) for s in spansof[pid] if span is None or (s[0] >= span[0] and s[1] <= span[1])]

    final = {}
    for p in ps:
        for rid, U in p["usages"]:
            for key in pieces(rid):
                final[key] = U
    cur, pend, req = {}, {}, set()
    for p in ps:
        for rid, U in p["usages"]:
            for key in pieces(rid):
                if key not in cur:
                    cur[key] = final.get(key)
                    pend[key] = []
                frm = cur[key]
                if frm is not None and needs_transition(frm, U):
                    w = list(dict.fromkeys([frm] + pend[key])) if writes(U) else [frm]
                    req.add((p["name"], key, frm, U, frozenset(w)))
                    cur[key] = U
                if writes(U):
                    pend[key] = []
                else:
                    pend[key].append(U)
    return req


def fuzz_expected(choices, passes: int) -> float:
    """What the random mix! DAG computes, replayed on the CPU (bench/fuzz.jl:75-83):
    every buffer starts at 1 and each pass collapses to one Float32.
    `choices[i] = (a, b)` are the source indices pass i+1 drew."""
    vals = [np.float32(1.0)]
    for i in range(1, passes + 1):
        a, b = choices[i - 1]
        va, vb = vals[a], vals[b]
        vals.append(np.float32(np.float32(np.float32(va * np.float32(0.5)) + np.float32(vb * np.float32(0.25))) + np.float32(i)))
    return vals[-1]


# ── numeric oracle (mantle_oracle.c) ────────────────────────────────────────
_lib = None
LIB = HERE / "liboracle.so"


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            from oracle.build import build  # noqa: WPS433
            build()
        h = C.CDLL(str(LIB))
        f32p, i32p, u32p, f64p = (C.POINTER(C.c_float), C.POINTER(C.c_int32), C.POINTER(C.c_uint32),
                                  C.POINTER(C.c_double))
        h.oracle_chain8.argtypes = [f32p, f32p, f32p, f32p, C.c_int64, C.c_int]
        h.oracle_chain8_passes.argtypes = [f32p, f32p, f32p, f32p, f32p, C.c_int64, C.c_int]
        h.oracle_touch3.argtypes = [f32p, f32p, f32p, C.c_int64, C.c_int]
        h.oracle_scatter_f64.argtypes = [f32p, i32p, C.c_int64, C.c_int32, f64p, u32p, C.c_int]
        h.oracle_scatter_f32.argtypes = [f32p, i32p, C.c_int64, C.c_int32, f32p, u32p, f32p, u32p, C.c_int]
        h.oracle_mix.argtypes = [f32p, f32p, f32p, C.c_float, C.c_int64]
        h.oracle_stir.argtypes = [f32p, f32p, C.c_float, C.c_int64]
        h.oracle_touch4.argtypes = [f32p, f32p, f32p, f32p, C.c_int64]
        h.oracle_transpose_scale.argtypes = [f32p, f32p, C.c_int32, C.c_int32, C.c_float, C.c_int64, C.c_int64]
        h.oracle_frombytes.argtypes = [f32p, u32p, C.c_int64]
        h.oracle_fft_f64.argtypes = [f32p, f64p, C.c_int64, C.c_int, C.c_int, C.c_int]
        h.oracle_fft_f32.argtypes = [f32p, f32p, C.c_int64, C.c_int, C.c_int, C.c_int]
        u16p = C.POINTER(C.c_uint16)
        h.oracle_gemm_bf16.argtypes = [u16p, u16p, f64p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                       C.c_int64, C.c_int]
        h.oracle_conv_bf16.argtypes = [u16p, u16p, f64p, u16p] + [C.c_int] * 10
        h.oracle_gap_fc.argtypes = [u16p, f32p, f64p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        u8p = C.POINTER(C.c_uint8)
        h.oracle_advect.argtypes = [f32p, f32p, C.c_float, C.c_float, C.c_int64]
        h.oracle_splat.argtypes = [f64p, f32p, f32p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int64]
        h.oracle_pack_bgra8.argtypes = [u8p, f32p, C.c_int64]
        h.oracle_unpack_bgra8.argtypes = [f32p, u8p, C.c_int, C.c_int]
        h.oracle_blur3x3.argtypes = [f32p, f32p, C.c_int, C.c_int]
        I = C.c_int  # noqa: E741
        h.oracle_sc_move_lights.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, I, I]
        h.oracle_sc_cull.argtypes = [u8p, f32p, f32p, I]
        h.oracle_raster_instances.restype = C.c_int64
        h.oracle_raster_instances.argtypes = [f32p, u32p, u32p, u32p, f32p, f32p, u32p, C.c_uint32, f32p, f32p, f32p,
                                              f32p, f32p, I, I, I, I, I]
        h.oracle_sc_tile_lights.argtypes = [u32p, u32p, f32p, f32p, f32p, I, I, I, I, I]
        h.oracle_sc_shade.argtypes = [f32p, u32p, u32p, u32p, f32p, f32p, f32p, u32p, u32p, f32p, f32p, f32p,
                                      I, I, I, I, I]
        h.oracle_sc_ssao.argtypes = [f32p, f32p, u32p, f32p, I, I, I]
        h.oracle_sc_ao_blur.argtypes = [f32p, f32p, f32p, I, I]
        h.oracle_sc_bright.argtypes = [f32p, f32p, f32p, I, I, I]
        h.oracle_sc_blur.argtypes = [f32p, f32p, I, I, I, I]
        h.oracle_sc_composite.argtypes = [f32p, f32p, f32p, f32p, I, I, I, I, I]
        h.oracle_max_threads.restype = C.c_int
        _lib = h
    return _lib


def _p(a, t):
    return a.ctypes.data_as(C.POINTER(t)) if a is not None else None


def chain8(x, y, z, threads=0):
    out = np.empty_like(x)
    lib().oracle_chain8(_p(x, C.c_float), _p(y, C.c_float), _p(z, C.c_float), _p(out, C.c_float), x.size, threads)
    return out


def chain8_passes(x, y, z, threads=0):
    out = np.empty_like(x)
    tmp = np.empty(7 * x.size, np.float32)
    lib().oracle_chain8_passes(_p(x, C.c_float), _p(y, C.c_float), _p(z, C.c_float), _p(out, C.c_float),
                               _p(tmp, C.c_float), x.size, threads)
    return out


def stir(src, k):
    """stir!(dst, src, k): dst = src*k + sin(src) (bench/independent.jl:37-40)."""
    src = np.ascontiguousarray(src, np.float32)
    out = np.empty_like(src)
    lib().oracle_stir(_p(out, C.c_float), _p(src, C.c_float), float(k), src.size)
    return out


def touch4(a, b, c, d):
    """touch4!(a, b, c, d): a*1.0001 + b + c + d (bench/stress.jl:42-45)."""
    a = np.array(a, np.float32)
    lib().oracle_touch4(_p(a, C.c_float), _p(b, C.c_float), _p(c, C.c_float), _p(d, C.c_float), a.size)
    return a


def transpose_scale(src, w, h, a, nx=None, ny=None):
    """transpose_scale!(dst, src, w, h, a) over the ndrange (nx, ny), default
    (w, h) (test/test_window.jl:30-33); dst has w*h elements, zero where the
    ndrange does not reach."""
    src = np.ascontiguousarray(src, np.float32)
    nx = w if nx is None else nx
    ny = h if ny is None else ny
    out = np.zeros(w * h, np.float32)
    lib().oracle_transpose_scale(_p(out, C.c_float), _p(src, C.c_float), w, h, float(a), nx, ny)
    return out


def frombytes(src):
    """frombytes!(dst, src): Float32(src & 0xff) (test/test_window.jl:84-87)."""
    src = np.ascontiguousarray(src, np.uint32)
    out = np.empty(src.size, np.float32)
    lib().oracle_frombytes(_p(out, C.c_float), _p(src, C.c_uint32), src.size)
    return out


def touch3(b, c, d, threads=0):
    b = b.copy()
    lib().oracle_touch3(_p(b, C.c_float), _p(c, C.c_float), _p(d, C.c_float), b.size, threads)
    return b


def scatter_f64(v, idx, nbins, acc=True, hist=True, threads=0):
    a = np.zeros(nbins, np.float64) if acc else None
    h = np.zeros(nbins, np.uint32) if hist else None
    lib().oracle_scatter_f64(_p(v, C.c_float), _p(idx, C.c_int32), idx.size, nbins, _p(a, C.c_double),
                             _p(h, C.c_uint32), threads)
    return a, h


def fft(x, inverse=False, threads=0, f32=False):
    """Batched DFT along the last axis of a complex64 array (batch, n):
    complex128 from the double checker, or complex64 from the float variant."""
    x = np.ascontiguousarray(x, dtype=np.complex64)
    batch, n = (1, x.shape[0]) if x.ndim == 1 else x.shape
    xv = x.view(np.float32)
    if f32:
        out = np.empty(x.shape, np.complex64)
        lib().oracle_fft_f32(_p(xv, C.c_float), _p(out.view(np.float32), C.c_float), batch, n, int(inverse), threads)
    else:
        out = np.empty(x.shape, np.complex128)
        lib().oracle_fft_f64(_p(xv, C.c_float), _p(out.view(np.float64), C.c_double), batch, n, int(inverse),
                             threads)
    return out


def bf16_bits(x) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (uint16), rounding to nearest, ties to even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_to_f32(h) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def gemm_bf16(A, B, M, N, K, batch=1, row0=0, rows=None, threads=0):
    """C = A.B for bfloat16 bit-pattern inputs (batch, M, K) and (batch, K, N), in
    double; only rows [row0, row0+rows) of each batch."""
    rows = M - row0 if rows is None else rows
    A = np.ascontiguousarray(A, dtype=np.uint16)
    B = np.ascontiguousarray(B, dtype=np.uint16)
    out = np.empty((batch, rows, N), np.float64)
    lib().oracle_gemm_bf16(_p(A, C.c_uint16), _p(B, C.c_uint16), _p(out, C.c_double), M, N, K, batch, row0, rows,
                           threads)
    return out


def conv_bf16(x, w, stride, pad, relu=True, threads=0):
    """NHWC conv of bfloat16 bit patterns x (n, h, w, cin) with HWIO weights w
    (k, k, cin, cout): (double result, bfloat16 result), both (n, ho, wo, cout)."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    w = np.ascontiguousarray(w, dtype=np.uint16)
    n, h, wd, cin = x.shape
    k, _, _, cout = w.shape
    ho, wo = (h + 2 * pad - k) // stride + 1, (wd + 2 * pad - k) // stride + 1
    od = np.empty((n, ho, wo, cout), np.float64)
    oh = np.empty((n, ho, wo, cout), np.uint16)
    lib().oracle_conv_bf16(_p(x, C.c_uint16), _p(w, C.c_uint16), _p(od, C.c_double), _p(oh, C.c_uint16), n, h, wd,
                           cin, cout, k, stride, pad, int(relu), threads)
    return od, oh


def gap_fc(act, w, threads=0):
    """act: (n, h, w, c) bfloat16 bits; w: (c, classes) float32 -> (n, classes) double."""
    act = np.ascontiguousarray(act, dtype=np.uint16)
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, h, wd, c = act.shape
    classes = w.shape[1]
    out = np.empty((n, classes), np.float64)
    lib().oracle_gap_fc(_p(act, C.c_uint16), _p(w, C.c_float), _p(out, C.c_double), n, h * wd, c, classes, threads)
    return out


def nchw_to_nhwc(x, cpad):
    """bfloat16 bits (n, c, h, w) -> (n, h, w, cpad) with zero channels appended."""
    n, c, h, w = x.shape
    out = np.zeros((n, h, w, cpad), np.uint16)
    out[..., :c] = np.transpose(x, (0, 2, 3, 1))
    return out


def cnn_forward(x_nchw_bits, ws, fc, layers, cpad, threads=0):
    """A CNN forward pass on the CPU: NCHW->NHWC (channels padded to cpad), then
    for each (name, k, cin, cout, stride) a conv (padding k//2) in double with
    ReLU, rounded to bfloat16 like stored activations; GAP+FC in double."""
    a = nchw_to_nhwc(x_nchw_bits, cpad)
    for name, k, _, cout, s in layers:
        _, a = conv_bf16(a, ws[name], s, k // 2, relu=True, threads=threads)
    return gap_fc(a, fc, threads=threads)


def advect(pos, vel, dt, radius):
    """advect! on copies of pos, vel (n, 3) float32; returns (pos, vel)."""
    pos = np.ascontiguousarray(pos, np.float32).copy()
    vel = np.ascontiguousarray(vel, np.float32).copy()
    lib().oracle_advect(_p(pos, C.c_float), _p(vel, C.c_float), dt, radius, pos.shape[0])
    return pos, vel


def splat(fb, pos, col, size, mvp, w, h, col_stride, size_stride):
    """Additive splat into fb ((h, w, 4) float64, modified and returned)."""
    pos = np.ascontiguousarray(pos, np.float32)
    col = np.ascontiguousarray(col, np.float32)
    size = np.ascontiguousarray(size, np.float32)
    mvp = np.ascontiguousarray(mvp, np.float32)
    lib().oracle_splat(_p(fb, C.c_double), _p(pos, C.c_float), _p(col, C.c_float), _p(size, C.c_float),
                       _p(mvp, C.c_float), w, h, col_stride, size_stride, pos.shape[0])
    return fb


def pack_bgra8(src):
    src = np.ascontiguousarray(src, np.float32)
    out = np.empty(src.shape[:-1] + (4,), np.uint8)
    lib().oracle_pack_bgra8(_p(out, C.c_uint8), _p(src, C.c_float), src.size // 4)
    return out


def unpack_bgra8(src, w, h):
    src = np.ascontiguousarray(src, np.uint8)
    out = np.empty((w, h, 4), np.float32)
    lib().oracle_unpack_bgra8(_p(out, C.c_float), _p(src, C.c_uint8), w, h)
    return out


def blur3x3(src, w, h):
    src = np.ascontiguousarray(src, np.float32)
    out = np.empty((w, h, 4), np.float32)
    lib().oracle_blur3x3(_p(out, C.c_float), _p(src, C.c_float), w, h)
    return out


def max_threads() -> int:
    return lib().oracle_max_threads()


# ── seeded inputs (the workloads' synthetic data) ──────────────────────────
def uniform(seed: int, n: int, lo: float, hi: float, stream: int = 0) -> np.ndarray:
    """float32 uniform[lo, hi) from numpy's PCG64 (seed, stream)."""
    rng = np.random.Generator(np.random.PCG64([seed, stream]))
    return rng.uniform(lo, hi, n).astype(np.float32)


def integers(seed: int, n: int, hi: int, stream: int = 0) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64([seed, stream]))
    return rng.integers(0, hi, n, dtype=np.int32)


# ── the showcase's compute passes (showcase_oracle.c) ───────────────────────
# Arrays: images [H][W] (float4 images as (H, W, 4) float32), packed RGBA8
# g-buffer channels uint32, lights and instances (n, 4) float32, P the scene
# constants (float32[80], offsets as in showcase_oracle.c).
def _f(a):
    return _p(np.ascontiguousarray(a, np.float32), C.c_float)


def _u(a):
    return _p(np.ascontiguousarray(a, np.uint32), C.c_uint32)


def sc_move_lights(centers, params, home, lcol, P, first):
    """-> (pos, centers', params') after moving the lights (showcase.jl:214-229)."""
    n = home.shape[0]
    pos = np.zeros((n, 4), np.float32)
    c = np.array(centers, np.float32, copy=True)
    q = np.array(params, np.float32, copy=True)
    lib().oracle_sc_move_lights(_p(pos, C.c_float), _p(c, C.c_float), _p(q, C.c_float), _f(home), _f(lcol), _f(P),
                                first, n)
    return pos, c, q


def raster_instances(ppos, pnrm, visible, count, centers, sizes, colors, params, M, mode, w, h):
    """The triangle rasteriser of oracle/raster_oracle.c: draw instances
    visible[:count] (1-based) of the prototype. Returns (depth (h, w) float32,
    [out0, out1, out2] (h, w) uint32 or None per mode, pieces drawn)."""
    f = lambda a: None if a is None else np.ascontiguousarray(a, np.float32)  # noqa: E731
    dep = np.zeros((h, w), np.float32)
    outs = [np.zeros((h, w), np.uint32) if (mode == 0 or (mode == 2 and k < 2)) else None for k in range(3)]
    vis = np.ascontiguousarray(visible, np.uint32)
    n = lib().oracle_raster_instances(
        _p(dep, C.c_float), *[_p(o, C.c_uint32) for o in outs], _p(f(ppos), C.c_float), _p(f(pnrm), C.c_float),
        _p(vis, C.c_uint32), int(count), _p(f(centers), C.c_float), _p(f(sizes), C.c_float), _p(f(colors), C.c_float),
        _p(f(params), C.c_float), _p(f(M), C.c_float), mode, w, h, int(np.asarray(ppos).shape[0]),
        int(np.asarray(centers).shape[0]))
    return dep, outs, n


def sc_cull(centers, M):
    """Boolean mask of the instances inside the frustum of the 16-float column-major M."""
    keep = np.zeros(centers.shape[0], np.uint8)
    lib().oracle_sc_cull(_p(keep, C.c_uint8), _f(centers), _f(M), centers.shape[0])
    return keep.astype(bool)


def sc_tile_lights(dep, lpos, P, tile, pertile):
    h, w = dep.shape
    ntx, nty = -(-w // tile), -(-h // tile)
    tl = np.zeros(ntx * nty * pertile, np.uint32)
    tc = np.zeros(ntx * nty, np.uint32)
    lib().oracle_sc_tile_lights(_p(tl, C.c_uint32), _p(tc, C.c_uint32), _f(dep), _f(lpos), _f(P), w, h, tile,
                                lpos.shape[0], pertile)
    return tl, tc


def sc_ssao(dep, nrm, P, nsample):
    h, w = dep.shape
    ao = np.zeros((-(-h // 2), -(-w // 2), 2), np.float32)
    lib().oracle_sc_ssao(_p(ao, C.c_float), _f(dep), _u(nrm), _f(P), w, h, nsample)
    return ao


def sc_ao_blur(src, P):
    aoh, aow = src.shape[:2]
    dst = np.zeros((aoh, aow), np.float32)
    lib().oracle_sc_ao_blur(_p(dst, C.c_float), _f(src), _f(P), aow, aoh)
    return dst


def sc_shade(alb, mat, nrm, dep, lpos, lcol, tl, tc, smap, aomap, P, tile, pertile):
    h, w = dep.shape
    hdr = np.zeros((h, w, 4), np.float32)
    lib().oracle_sc_shade(_p(hdr, C.c_float), _u(alb), _u(mat), _u(nrm), _f(dep), _f(lpos), _f(lcol), _u(tl), _u(tc),
                          _f(smap), _f(aomap), _f(P), w, h, tile, pertile, smap.shape[0])
    return hdr


def sc_bright(hdr, P, shift):
    h, w = hdr.shape[:2]
    dst = np.zeros((-(-h // shift), -(-w // shift), 4), np.float32)
    lib().oracle_sc_bright(_p(dst, C.c_float), _f(hdr), _f(P), w, h, shift)
    return dst


def sc_blur(src, dx, dy):
    bh, bw = src.shape[:2]
    dst = np.zeros_like(src, dtype=np.float32)
    lib().oracle_sc_blur(_p(dst, C.c_float), _f(src), bw, bh, dx, dy)
    return dst


def sc_composite(hdr, bloom, P, shift):
    h, w = hdr.shape[:2]
    bh, bw = bloom.shape[:2]
    out = np.zeros((h, w, 4), np.float32)
    lib().oracle_sc_composite(_p(out, C.c_float), _f(hdr), _f(bloom), _f(P), w, h, bw, bh, shift)
    return out
