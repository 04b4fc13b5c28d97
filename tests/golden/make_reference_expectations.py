"""Writes reference_expectations.json: the known answers the reference's own
test suite asserts for the graph path, transcribed with the file:line they come
from. The reference is Julia on Vulkan and cannot run here, so these values are
copied from its assertions, not computed; every graph below is written in the
graph-spec format of tests/graphspec.py.

    python tests/golden/make_reference_expectations.py
"""
import json
from pathlib import Path

OUT = Path(__file__).resolve().parent / "reference_expectations.json"


def interleaved(chains, stages, n=1024):
    """build_interleaved (bench/independent.jl:43-54): chain c stage s reads
    b{c}_{s} and writes b{c}_{s+1}; stages interleaved across chains."""
    return {
        "transients": [[f"b{c}_{k}", n] for c in range(1, chains + 1) for k in range(1, stages + 2)],
        "passes": [{"name": f"c{c} s{s}", "usages": [[f"b{c}_{s}", "R", None], [f"b{c}_{s + 1}", "W", None]]}
                   for s in range(1, stages + 1) for c in range(1, chains + 1)],
    }


def rps(n=256):
    """memory_saving (test/test_window.jl:752-769): draw i writes t_i, blt i
    accumulates t_i into `out`."""
    return {
        "persistent": [["out", n]],
        "transients": [[f"t{i}", n] for i in range(6)],
        "passes": [{"name": f"draw{i}", "usages": [[f"t{i}", "W", None]]} for i in range(6)]
        + [{"name": f"blt{i}", "usages": [["out", "RW", None], [f"t{i}", "R", None]]} for i in range(6)],
    }


def program_order(hoist, n=256):
    """program_order (test/test_window.jl:793-812)."""
    ps = [{"name": str(i - 1), "usages": [[f"t{i}", "W", None]]} for i in range(1, 7)]
    ps += [{"name": str(i + 5), "usages": [["out", "RW", None], [f"t{i}", "R", None]]} for i in range(1, 7)]
    dr = lambda i: {"name": str(10 + 2 * i), "usages": [[f"t{i}", "W", None]]}  # noqa: E731
    bl = lambda i: {"name": str(11 + 2 * i), "usages": [["out", "RW", None], [f"t{i}", "R", None]]}  # noqa: E731
    if hoist:
        ps += [dr(i) for i in range(1, 7)] + [bl(i) for i in range(1, 7)]
    else:
        for i in range(1, 7):
            ps += [dr(i), bl(i)]
    return {"persistent": [["out", n]], "transients": [[f"t{i}", n] for i in range(1, 7)], "passes": ps}


def six_chains(n=4096):
    """scheduling reorders passes (test/test_window.jl:834-848): six chains of
    four stages over five transients each, declared interleaved."""
    return {
        "transients": [[f"c{c}_{k}", n] for c in range(1, 7) for k in range(1, 6)],
        "passes": [{"name": f"c{c} s{s}", "usages": [[f"c{c}_{s + 1}", "W", None], [f"c{c}_{s}", "R", None]]}
                   for s in range(1, 5) for c in range(1, 7)],
    }


def alias_chain(n=4096):
    """aliasing trades memory against barriers (test/test_window.jl:870-884)."""
    return {
        "transients": [[f"t{i}", n] for i in range(1, 13)],
        "passes": [{"name": f"p{i}", "usages": [[f"t{i}", "W", None], [f"t{i - 1}", "R", None]]}
                   for i in range(2, 13)],
    }


def slices(kind):
    """disjoint slices of one buffer (test/test_window.jl:391-564)."""
    n = 256
    if kind in ("whole", "sliced"):
        r1 = None if kind == "whole" else [1, 128]
        r2 = None if kind == "whole" else [129, 256]
        return {"persistent": [["b", n]], "passes": [
            {"name": "lower", "usages": [["b", "W", r1]]}, {"name": "upper", "usages": [["b", "W", r2]]}]}
    if kind in ("reader_whole", "reader_sliced"):
        r1 = None if kind == "reader_whole" else [1, 128]
        r2 = None if kind == "reader_whole" else [129, 256]
        return {"persistent": [["b", n]], "passes": [
            {"name": "write low", "usages": [["b", "W", r1]]}, {"name": "read high", "usages": [["b", "R", r2]]}]}
    if kind == "identical":
        return {"persistent": [["b", n]], "passes": [
            {"name": "first", "usages": [["b", "W", [1, 128]]]}, {"name": "second", "usages": [["b", "W", [1, 128]]]}]}
    if kind == "partial":
        return {"persistent": [["b", n]], "passes": [
            {"name": "low", "usages": [["b", "W", [1, 128]]]}, {"name": "mid", "usages": [["b", "W", [64, 200]]]},
            {"name": "tail", "usages": [["b", "W", [201, 256]]]}]}
    if kind == "parts_then_whole":
        parts = [[1, 64], [65, 128], [129, 192], [193, 256]]
        return {"persistent": [["b", n]], "passes": [
            {"name": f"part {k + 1}", "usages": [["b", "W", r]]} for k, r in enumerate(parts)]
            + [{"name": "whole", "usages": [["b", "RW", None]]}]}
    if kind == "sliced_transient":
        return {"persistent": [["out", n]], "transients": [["a", n], ["b", n]], "passes": [
            {"name": "fill a", "usages": [["a", "W", None]]}, {"name": "read a", "usages": [["a", "R", None]]},
            {"name": "slice of b", "usages": [["b", "W", [1, 128]]]},
            {"name": "drain", "usages": [["out", "W", None], ["b", "R", None]]}]}
    raise KeyError(kind)


def main():
    hand = []  # the 10-transition hand set, test/test_window.jl:607-612
    for c in (1, 2):
        for k in (1, 2, 3):
            if k > 1:
                hand.append([f"c{c} s{k}", f"b{c}_{k}", "W", "R", ["W"]])
            frm = "W" if k == 3 else "R"
            hand.append([f"c{c} s{k}", f"b{c}_{k + 1}", frm, "W", [frm]])
    g = {
        "generated_by": "tests/golden/make_reference_expectations.py",
        "spans": {"source": "test/runtests.jl:8-18",
                  "length_3_9": 6, "empty_4_4": True, "overlap_0_3__2_5": True, "overlap_0_3__3_5": False,
                  "from_closed_0_2": [0, 3]},
        "csv_end_trap": {"source": "test/runtests.jl:20-26",
                         "upper_file": "id,lower,upper,size\nb,0,3,4\n", "upper_live": [0, 3],
                         "end_file": "id,lower,end,size\nb,0,3,4\n", "end_live": [0, 4]},
        "csv_gaps": {"source": "test/runtests.jl:28-37",
                     "file": "id,lower,upper,size,gaps\nb,0,20,4,9-11 12-14@2:13\n",
                     "gaps": [[[9, 11], None], [[12, 14], [2, 13]]]},
        "segments": {"source": "test/runtests.jl:39-44",
                     "cases": [{"item": ["x", [0, 10], 4, [[[4, 6], None]]], "want": [[[0, 4], 4], [[6, 10], 4]]},
                               {"item": ["y", [0, 10], 4, [[[4, 6], [0, 1]]]],
                                "want": [[[0, 4], 4], [[4, 6], 1], [[6, 10], 4]]}]},
        "pinned": {"source": "test/runtests.jl:115-122",
                   "items": [["a", [0, 10], 4, 1, 16], ["b", [0, 10], 4, 1, None], ["c", [0, 10], 4, 1, None]],
                   "want_offset_a": 16},
        "alignment": {"source": "test/runtests.jl:124-130",
                      "items": [["a", [0, 10], 3, 1, None], ["b", [0, 10], 3, 256, None]], "align_of_b": 256},
        "gaps_height": {"source": "test/runtests.jl:146-151",
                        "items": [["a", [0, 10], 2, [[[0, 5], [0, 1]]]], ["b", [0, 10], 2, [[[5, 10], [1, 2]]]]],
                        "height": 4, "broken_optimal_height": 3},
        "hazard_rules": {"source": "test/runtests.jl:225-235",
                         "cases": [[["R", "R"], 0], [["W", "W"], 1], [["uW", "uW"], 0], [["uW", "W"], 1]]},
        "buffers_have_no_layouts": {"source": "test/runtests.jl:237-241",
                                    "needs_transition_buffer_sampled_copysrc": False},
        "write_waits_on_readers": {"source": "test/runtests.jl:250-256",
                                   "usages": ["ColorClear", "Sampled", "CopySrc", "ImageW"],
                                   "last_waits": ["CopySrc", "Sampled"]},
        "webgpu": {"source": "test/runtests.jl:277-279", "usages": ["ColorClear", "Sampled", "CopySrc"], "count": 0},
        "discards": {"source": "test/runtests.jl:293-296,209-220",
                     "ColorClear": [True, False, True], "ColorKeep": [False, True, True],
                     "DepthClear": [True, False, True], "DepthKeep": [False, True, True]},
        "hand_set": {"source": "test/test_window.jl:566-623", "graph": interleaved(2, 3), "alias": False,
                     "transitions": hand, "per_pass_counts": [1, 1, 2, 2, 2, 2]},
        "rps_memory_saving": {"source": "test/test_window.jl:736-780", "graph": rps(),
                              "overlap_order": [f"draw{i}" for i in range(6)] + [f"blt{i}" for i in range(6)],
                              "compact_order": [x for i in range(6) for x in (f"draw{i}", f"blt{i}")],
                              "peak_ratio": 6},
        "program_order": {"source": "test/test_window.jl:782-832", "hoisted": program_order(True),
                          "declared": program_order(False)},
        "six_chains": {"source": "test/test_window.jl:834-854", "graph": six_chains(),
                       "loose_first_two": ["c1 s1", "c2 s1"], "tight_first_two": ["c1 s1", "c1 s2"]},
        "aliasing_trade": {"source": "test/test_window.jl:870-890", "graph": alias_chain()},
        "slices": {"source": "test/test_window.jl:391-564",
                   "whole_resources": 1, "sliced_resources": 2, "reader_whole_waits": 1, "reader_sliced_waits": 0,
                   "identical_resources": 1, "whole_after_parts_transitions": 4,
                   "graphs": {k: slices(k) for k in ("whole", "sliced", "reader_whole", "reader_sliced",
                                                     "identical", "partial", "parts_then_whole",
                                                     "sliced_transient")}},
        "never_used": {"source": "test/test_window.jl:1595-1611", "message": "is never used by any pass"},
    }
    OUT.write_text(json.dumps(g, indent=1))
    print(OUT)


if __name__ == "__main__":
    main()
