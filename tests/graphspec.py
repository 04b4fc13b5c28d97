"""One graph description, two builders: the product (the C++ phases through the
C ABI) and the oracle (the Python restatement). Results are compared keyed by
what a resource *means* — (name, range) — never by the ids either side handed
out.

spec = {"persistent": [[name, n], ...], "transients": [[name, n], ...],
        "passes": [{"name": ..., "usages": [[resource, usage, range or None], ...]}],
        "updates": [name, ...]}
usage strings: R, W, RW, uR, uW, uRW (Unordered), CopySrc, CopyDst.
"""
import numpy as np

import mantle_cuda as M
from oracle import oracle as O

USAGE = {"R": O.SR, "W": O.SW, "RW": O.SRW, "uR": O.SR | O.UNORDERED, "uW": O.SW | O.UNORDERED,
         "uRW": O.SRW | O.UNORDERED, "CopySrc": O.COPY_SRC, "CopyDst": O.COPY_DST,
         "Sampled": O.SAMPLED, "ColorClear": O.COLOR | O.DISCARD, "ColorKeep": O.COLOR,
         "DepthClear": O.DEPTH | O.RD | O.WR | O.DISCARD, "DepthKeep": O.DEPTH | O.RD | O.WR,
         "ImageW": O.STORAGE | O.WR | O.IMAGE}
NAME = {v: k for k, v in USAGE.items() if k in ("R", "W", "RW", "uR", "uW", "uRW", "CopySrc", "CopyDst")}


def build_product(spec, dev=None, **plan_kw):
    g = M.Graph(dev)
    objs = {}
    for name, n in spec.get("transients", []):
        objs[name] = M.Transient.Buffer(g, np.float32, n)
    for name, n in spec.get("persistent", []):
        objs[name] = M.VirtualBuffer(np.float32, n) if dev is None else M.Buffer(dev, np.float32, n)
    for name in spec.get("updates", []):
        M.Update(g, objs[name])
    for p in spec["passes"]:
        ph = M.compute(g, p["name"]).__enter__()
        for res, u, rng in p["usages"]:
            M.use(ph, objs[res], usage=USAGE[u], range=tuple(rng) if rng else None)
    plan = M.Plan(g, **plan_kw)
    names = {g.rid(o): k for k, o in objs.items()}
    return g, plan, names


def product_key(g, names, rid):
    if rid == 0:
        return ("handover", None)
    parent, rng = g.normal_id(rid)
    return (names[parent], tuple(rng) if rng else None)


def product_transitions(g, plan, names):
    out = set()
    for pos, p in enumerate(plan.passes):
        for t in plan.pre(pos):
            out.add((p.name, product_key(g, names, t.resource), t.from_, t.to, frozenset(t.waits)))
    return out


def build_oracle(spec):
    g = O.OGraph()
    for name, n in spec.get("transients", []):
        g.transient(name, n)
    for name, n in spec.get("persistent", []):
        g.buffer(name, n)
    for name in spec.get("updates", []):
        g.update(name)
    for p in spec["passes"]:
        op = g.add_pass(p["name"])
        for res, u, rng in p["usages"]:
            g.use(op, res, USAGE[u], tuple(rng) if rng else None)
    return g


def oracle_key(g, rid):
    if rid == 0:
        return ("handover", None)
    r = g.res[rid]
    if r.kind == "view":
        pk = next(k for k, v in g.ids.items() if v == r.parent)
        return (pk, tuple(r.rng))
    return (next(k for k, v in g.ids.items() if v == rid), None)


def oracle_transitions(g, res):
    out = set()
    for pos, i in enumerate(res["order"]):
        for t in res["prepass"][pos]:
            out.add((g.passes[i]["name"], oracle_key(g, t.resource), t.from_, t.to, frozenset(t.waits)))
    return out


def random_usage_spec(rng, nbufs=5, npasses=12, n=256, slicing=0.0, unordered=0.0):
    """usage_graph (bench/stress.jl:56-96) with this repository's generator: random
    read/write/readwrite usages on persistent buffers, ranges drawn from a small
    set of cut points so identical, disjoint and overlapping slices all occur."""
    cuts = [1, n // 4, n // 3, n // 2, (3 * n) // 4, n]
    spec = {"persistent": [[f"b{i}", n] for i in range(1, nbufs + 1)], "passes": []}
    for i in range(1, npasses + 1):
        k = int(rng.integers(1, min(4, nbufs) + 1))
        picks = rng.permutation(nbufs)[:k]
        us = []
        for j in picks:
            r, w = bool(rng.integers(0, 2)), bool(rng.integers(0, 2))
            if not (r or w):
                r = True
            u = "RW" if (r and w) else ("R" if r else "W")
            if rng.random() < unordered:
                u = "u" + u
            rg = None
            if rng.random() < slicing:
                a, b = sorted((int(rng.choice(cuts)), int(rng.choice(cuts))))
                rg = [a, max(a, b)]
            us.append([f"b{j + 1}", u, rg])
        spec["passes"].append({"name": f"p{i}", "usages": us})
    return spec


def random_chain_spec(rng, npasses=12, n=256):
    """chain_graph (bench/stress.jl:98-122): write-then-read over transients, so
    the placer aliases them and the handover appears."""
    spec = {"persistent": [["seed", n], ["out", n]], "transients": [[f"t{i}", n] for i in range(1, npasses + 1)],
            "passes": []}
    sources = ["seed"]
    for i in range(1, npasses + 1):
        a, b = sources[int(rng.integers(0, len(sources)))], sources[int(rng.integers(0, len(sources)))]
        us = [[f"t{i}", "W", None], [a, "R", None]]
        if b != a:
            us.append([b, "R", None])
        spec["passes"].append({"name": f"p{i}", "usages": us})
        sources.append(f"t{i}")
    spec["passes"].append({"name": "out", "usages": [["out", "W", None], [f"t{npasses}", "R", None]]})
    return spec
