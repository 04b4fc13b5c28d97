"""Headless triangle rasterisation (the raster_instances kernel family): the
g-buffer and shadow passes of bench/showcase.jl and the g-buffer of
bench/deferred.jl.

CPU: the oracle (oracle/raster_oracle.c) against hand-computed coverage —
pixel centres inside a quad, the shared diagonal covered once with no gap,
back faces culled, the near plane clipping a quad that crosses it — and the
crystal scene's plausibility.

GPU: the kernels against the oracle on the same inputs. Coverage is decided
with integer edge functions on snapped vertices and both sides do the same
float operations in the same order (no FMA contraction on either), so depth
and the packed g-buffer channels are compared bit for bit; then the whole
showcase frame with its two raster passes, against the oracle's frame.
"""
import numpy as np
import pytest

import mantle_cuda as M
from mantle_cuda.workloads import SC_OFF, crystal_scene, shard_geometry
from oracle import oracle as O


def ortho(w, h):
    """World (x, y) in pixels -> NDC, z as is, w = 1 (column-major)."""
    m = np.array([[2.0 / w, 0, 0, -1], [0, 2.0 / h, 0, -1], [0, 0, 1, 0], [0, 0, 0, 1]], np.float32)
    return m.T.reshape(-1).copy()


def quad(x0, y0, x1, y1, z, front=True):
    """Two triangles covering [x0, x1] x [y0, y1] at depth z, wound so they
    face the viewer (kept by back-face culling) or away from it."""
    a, b, c, d = (x0, y0), (x1, y0), (x1, y1), (x0, y1)
    tris = [(a, d, c), (a, c, b)] if front else [(a, b, c), (a, c, d)]
    pos = np.array([[p[0], p[1], z, 1.0] for t in tris for p in t], np.float32)
    nrm = np.tile(np.array([0, 0, -1, 0], np.float32), (6, 1))
    return pos, nrm


def one_instance(n=1):
    c = np.zeros((n, 4), np.float32)
    s = np.tile(np.array([1, 1, 1, 0], np.float32), (n, 1))  # unit scale, no yaw
    col = np.tile(np.array([0.2, 0.4, 0.6, 0.8], np.float32), (n, 1))
    return c, s, col


def test_oracle_quad_covers_exactly_the_pixel_centres_inside():
    w, h = 40, 30
    pos, nrm = quad(5.25, 3.75, 31.25, 21.25, 0.5)
    c, s, col = one_instance()
    dep, outs, n = O.raster_instances(pos, nrm, [1], 1, c, s, col, None, ortho(w, h), 2, w, h)
    xs, ys = np.arange(w) + 0.5, np.arange(h) + 0.5
    want = (ys[:, None] > 3.75) & (ys[:, None] < 21.25) & (xs[None] > 5.25) & (xs[None] < 31.25)
    assert np.array_equal(dep < 1, want) and n == 2
    assert np.abs(dep[want] - 0.5).max() <= 1e-6  # the plane's depth, up to the barycentric weights' rounding
    # the diagonal is shared: every pixel along it is covered (no gap), and
    # the flat colour and normal are the same whichever triangle won
    assert np.all(outs[0][want] == outs[0][want][0])
    assert outs[0][want][0] == (51 | 102 << 8 | 153 << 16 | 204 << 24)
    assert np.all(outs[1][want] == (128 | 128 << 8 | 0 << 16 | 255 << 24))
    assert np.all(outs[0][~want] == 0xFF000000)


def test_oracle_back_faces_are_culled_and_edges_on_samples_tie_once():
    w, h = 16, 16
    pos, nrm = quad(2.5, 2.5, 12.5, 10.5, 0.25, front=False)
    c, s, col = one_instance()
    dep, _, n = O.raster_instances(pos, nrm, [1], 1, c, s, col, None, ortho(w, h), 2, w, h)
    assert n == 0 and np.all(dep == 1.0)
    # two quads sharing the vertical edge x = 8.5, which runs through pixel
    # centres: each centre on it belongs to exactly one of them
    p1, n1 = quad(2.5, 2.5, 8.5, 12.5, 0.25)
    p2, _ = quad(8.5, 2.5, 14.5, 12.5, 0.75)
    pos = np.concatenate([p1, p2])
    nrm = np.concatenate([n1, n1])
    dep, _, n = O.raster_instances(pos, nrm, [1], 1, c, s, col, None, ortho(w, h), 2, w, h)
    assert n == 4
    near = lambda a, v: np.abs(a - v) <= 1e-6  # noqa: E731
    col8 = dep[3:12, 8]
    assert np.all(near(col8, 0.25) | near(col8, 0.75))
    assert np.all(near(dep[3:12, 3:8], 0.25)) and np.all(near(dep[3:12, 9:14], 0.75))
    # the nearer surface wins where two overlap, whatever their order
    p3, _ = quad(0.5, 0.5, 15.5, 15.5, 0.5)
    for order in ((p1, p3), (p3, p1)):
        dep, _, _ = O.raster_instances(np.concatenate(order), np.concatenate([n1, n1]), [1], 1, c, s, col, None,
                                       ortho(w, h), 2, w, h)
        assert np.all(near(dep[3:12, 3:8], 0.25)) and near(dep[14, 14], 0.5)


def test_oracle_near_plane_clips_a_quad_that_crosses_it():
    # a perspective camera looking down -z at a floor quad running from in
    # front of the near plane to far behind it: only the part with z_view <= -near
    # is drawn, with depths in [0, 1)
    w, h = 64, 48
    from mantle_cuda.workloads import showcase_camera
    vp, _ = showcase_camera(0.0, 30.0, 2.0, w, h)
    m = np.asarray(vp, np.float32).T.reshape(-1).copy()
    big = 400.0
    pos = np.array([[-big, 0, -big, 1], [-big, 0, big, 1], [big, 0, big, 1],
                    [-big, 0, -big, 1], [big, 0, big, 1], [big, 0, -big, 1]], np.float32)
    nrm = np.tile(np.array([0, 1, 0, 0], np.float32), (6, 1))
    c, s, col = one_instance()
    dep, outs, n = O.raster_instances(pos, nrm, [1], 1, c, s, col, None, m, 2, w, h)
    cov = dep < 1
    assert n >= 2 and 0.02 < cov.mean() < 0.9  # the ground below the horizon (the camera looks up at y = 13)
    assert dep[cov].min() >= 0 and dep[cov].max() < 1
    assert cov[-1].all() and not cov[0].any()  # ground at the bottom, sky at the top
    assert np.all(outs[1][cov] == (128 | 255 << 8 | 128 << 16 | 255 << 24))  # the up normal


def test_crystal_scene_is_plausible():
    ppos, pnrm = shard_geometry()
    assert ppos.shape == (72, 4) and np.allclose(np.linalg.norm(pnrm[:, :3], axis=1), 1)
    # the side and top faces (three of every four triangles) face outwards;
    # the base cap is wound the other way in the reference's own geometry
    # (its normal is +y, showcase.jl:65), which nothing sees from below
    mid = ppos[:, :3].reshape(24, 3, 3).mean(1)
    out = np.einsum("ij,ij->i", mid, pnrm[::3, :3]).reshape(6, 4)
    assert (out[:, :3] > 0).all() and np.allclose(pnrm[::3, :3].reshape(6, 4, 3)[:, 3], [0, 1, 0])
    sc = crystal_scene(320, 184, smap_res=256)
    assert sc.centers.shape == (5044, 4) and sc.sizes.shape == (5044, 4) and sc.rasterised


# ── GPU ──────────────────────────────────────────────────────────────────────
def _dev(a):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).cuda()
    return torch.from_numpy(a).cuda()


def _launch_raster(ppos, pnrm, visible, count, centers, sizes, colors, params, P, off, mode, w, h):
    import torch
    depth = torch.zeros(h * w, device="cuda")
    outs = [torch.zeros(h * w, dtype=torch.int32, device="cuda") if (mode == 0 or (mode == 2 and k < 2)) else None
            for k in range(3)]
    opt = lambda a: None if a is None else _dev(a)  # noqa: E731
    vis = np.zeros(max(centers.shape[0], len(visible)), np.uint32)  # the cull's list has a slot per instance
    vis[:len(visible)] = visible
    args = (depth, *outs, _dev(ppos), opt(pnrm), _dev(vis),
            _dev(np.array([count], np.uint32)), _dev(centers), _dev(sizes), opt(colors), opt(params), _dev(P), off,
            mode, w, h, ppos.shape[0])
    n = centers.shape[0]
    ws = torch.empty(M.workspace_bytes(M.kernels.raster_instances, args, n), dtype=torch.uint8, device="cuda")
    M.launch(M.kernels.raster_instances, args, n, stream=torch.cuda.current_stream().cuda_stream, workspace=ws)
    torch.cuda.synchronize()
    return (depth.cpu().numpy().reshape(h, w),
            [None if o is None else o.cpu().numpy().view(np.uint32).reshape(h, w) for o in outs])


@pytest.fixture(scope="module")
def crystals():
    sc = crystal_scene(1600, 900, smap_res=2048)
    lpos, centers, params = O.sc_move_lights(sc.centers, sc.params, sc.home, sc.lcol, sc.P, sc.first)
    return sc, centers, params


@pytest.mark.gpu
def test_gbuffer_matches_oracle_bit_for_bit(dev, crystals):
    sc, centers, params = crystals
    keep = O.sc_cull(centers, sc.P[0:16])
    vis = (np.nonzero(keep)[0] + 1).astype(np.uint32)
    rng = np.random.default_rng(5)
    vis = vis[rng.permutation(vis.size)]  # the cull's list order is not fixed: it must not matter
    want_d, want_o, _ = O.raster_instances(sc.ppos, sc.pnrm, vis, vis.size, centers, sc.sizes, sc.colors, params,
                                           sc.P[0:16], 0, sc.w, sc.h)
    got_d, got_o = _launch_raster(sc.ppos, sc.pnrm, vis, vis.size, centers, sc.sizes, sc.colors, params, sc.P, 0, 0,
                                  sc.w, sc.h)
    assert 0.5 < (want_d < 1).mean() < 1.0
    assert np.array_equal(got_d, want_d)
    for k in range(3):
        assert np.array_equal(got_o[k], want_o[k]), f"out{k}: {(got_o[k] != want_o[k]).sum()} pixels differ"


@pytest.mark.gpu
def test_shadow_map_matches_oracle_bit_for_bit(dev, crystals):
    sc, centers, _ = crystals
    keep = O.sc_cull(centers, sc.P[32:48])
    vis = (np.nonzero(keep)[0] + 1).astype(np.uint32)
    res = sc.smap_res
    want_d, _, _ = O.raster_instances(sc.ppos, None, vis, vis.size, centers, sc.sizes, None, None, sc.P[32:48], 1,
                                      res, res)
    got_d, _ = _launch_raster(sc.ppos, None, vis, vis.size, centers, sc.sizes, None, None, sc.P, SC_OFF["sunvp"], 1,
                              res, res)
    assert 0.05 < (want_d < 1).mean()
    assert np.array_equal(got_d, want_d)


@pytest.mark.gpu
def test_deferred_boxes_and_edge_cases_match_oracle(dev):
    # bench/deferred.jl's g-buffer: unit cubes scaled per instance (no yaw),
    # normals as given; a list with entries that name no instance, and a count
    # beyond the list (both skipped, never read past the instances)
    rng = np.random.default_rng(11)
    faces = []
    for axis in range(3):
        for sgn in (1.0, -1.0):
            nvec = np.zeros(3)
            nvec[axis] = sgn
            u = np.zeros(3)
            u[(axis + 1) % 3] = 1
            v = np.zeros(3)
            v[(axis + 2) % 3] = 1
            if sgn < 0:
                u, v = v, u
            q = (nvec - u - v, nvec + u - v, nvec + u + v, nvec - u + v)
            for k in (0, 1, 2, 0, 2, 3):
                faces.append((q[k], nvec))
    ppos = np.array([[*p, 1.0] for p, _ in faces], np.float32)
    pnrm = np.array([[*n_, 0.0] for _, n_ in faces], np.float32)
    ninst = 400
    centers = np.c_[rng.uniform(-40, 40, ninst), rng.uniform(0, 8, ninst), rng.uniform(-40, 40, ninst),
                    np.full(ninst, 9.0)].astype(np.float32)
    sizes = np.c_[rng.uniform(0.5, 3, (ninst, 3)), np.zeros(ninst)].astype(np.float32)
    colors = rng.uniform(0, 1, (ninst, 4)).astype(np.float32)
    from mantle_cuda.workloads import showcase_camera
    w, h = 640, 400
    vp, _ = showcase_camera(1.0, 46.0, 13.0, w, h)
    P = np.zeros(32, np.float32)
    P[16:32] = np.asarray(vp, np.float32).T.reshape(-1)
    vis = np.arange(1, ninst + 1, dtype=np.uint32)
    vis[::37] = 0          # names no instance
    vis[5] = ninst + 7     # past the instances
    want_d, want_o, _ = O.raster_instances(ppos, pnrm, vis, ninst + 50, centers, sizes, colors, None, P[16:32], 2, w,
                                           h)
    got_d, got_o = _launch_raster(ppos, pnrm, vis, ninst + 50, centers, sizes, colors, None, P, 16, 2, w, h)
    assert 0.05 < (want_d < 1).mean() < 0.95
    assert np.array_equal(got_d, want_d)
    assert np.array_equal(got_o[0], want_o[0]) and np.array_equal(got_o[1], want_o[1])


@pytest.mark.gpu
def test_raster_refuses_bad_shapes(dev):
    import torch
    d = torch.zeros(64, device="cuda")
    pp = torch.zeros(8, 4, device="cuda")
    one = torch.ones(4, device="cuda")
    u = torch.zeros(4, dtype=torch.int32, device="cuda")
    base = [d, None, None, None, pp, None, u, u, one, one, None, None, torch.zeros(16, device="cuda"), 0, 1, 8, 8, 6]
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for k, v in ((17, 7), (14, 3), (15, 0), (13, 4)):  # vertices not in threes; mode; width; matrix past the buffer
        args = list(base)
        args[k] = v
        with pytest.raises(M.ArgumentError):
            M.launch(M.kernels.raster_instances, tuple(args), 1, stream=s, workspace=ws)


@pytest.mark.gpu
def test_showcase_frame_with_raster_passes_matches_oracle(dev, crystals):
    """The frame of bench/showcase.jl with its g-buffer and shadow passes
    rasterised inside the graph (15 passes), against the oracle's frame:
    raster outputs bit for bit, the shaded output within the showcase
    tolerance."""
    from mantle_cuda.workloads import build_showcase
    sc, centers, params = crystals
    w = build_showcase(dev, sc)
    assert "gbuffer" in w.plan.names and "shadow" in w.plan.names
    M.run(w.plan)
    M.run(w.plan)
    dev.synchronize()
    B = w.bufs
    vis = (np.nonzero(O.sc_cull(centers, sc.P[0:16]))[0] + 1).astype(np.uint32)
    svis = (np.nonzero(O.sc_cull(centers, sc.P[32:48]))[0] + 1).astype(np.uint32)
    dep, (alb, mat, nrm), _ = O.raster_instances(sc.ppos, sc.pnrm, vis, vis.size, centers, sc.sizes, sc.colors,
                                                 params, sc.P[0:16], 0, sc.w, sc.h)
    smap, _, _ = O.raster_instances(sc.ppos, None, svis, svis.size, centers, sc.sizes, None, None, sc.P[32:48], 1,
                                    sc.smap_res, sc.smap_res)
    assert np.array_equal(B["dep"].array().reshape(sc.h, sc.w), dep)
    assert np.array_equal(B["alb"].array().view(np.uint32).reshape(sc.h, sc.w), alb)
    assert np.array_equal(B["nrm"].array().view(np.uint32).reshape(sc.h, sc.w), nrm)
    assert np.array_equal(B["smap"].array().reshape(sc.smap_res, sc.smap_res), smap)
    lpos, _, _ = O.sc_move_lights(sc.centers, sc.params, sc.home, sc.lcol, sc.P, sc.first)
    tl, tc = O.sc_tile_lights(dep, lpos, sc.P, sc.tile, sc.pertile)
    aomap = O.sc_ao_blur(O.sc_ssao(dep, nrm, sc.P, sc.nsample), sc.P)
    hdr = O.sc_shade(alb, mat, nrm, dep, lpos, sc.lcol, tl, tc, smap, aomap, sc.P, sc.tile, sc.pertile)
    bloom = O.sc_blur(O.sc_blur(O.sc_bright(hdr, sc.P, sc.shift), 1, 0), 0, 1)
    want = O.sc_composite(hdr, bloom, sc.P, sc.shift)
    got = B["out"].array().reshape(sc.h, sc.w, 4)
    ok = np.abs(got.astype(np.float64) - want) <= 1e-6 + 1e-5 * np.abs(want)
    assert ok.mean() >= 0.995, f"{(~ok).sum()} of {ok.size} outside tolerance"
