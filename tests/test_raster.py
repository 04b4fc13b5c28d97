"""Point clouds and the image chain (bench/two_scatters.jl, bench/chain.jl) as
CUDA kernels: advect, clear, additive point splat, BGRA8 readback, unpack and
3x3 blur, against the oracle.

Tolerances: advect, coverage, unpack and blur are bit-exact (same operation
order and rounding on both sides). The splat's framebuffer sums depend on the
order points land in: <= 1e-5 relative (plus 1e-6 absolute) against the
double-precision oracle; its BGRA8 bytes are then exact when packed from the
same floats, and within one step of the oracle's own bytes.
"""
import numpy as np
import pytest

import mantle_cuda as M
from mantle_cuda.workloads import RASTER_H, RASTER_W, build_raster, camera, point_cloud
from oracle import oracle as O


def test_oracle_image_known_answers():
    w, h = 3, 2
    raw = np.zeros((h, w, 4), np.uint8)
    raw[1, 2] = (10, 20, 30, 255)  # B, G, R, A at pixel i=2, j=1
    img = O.unpack_bgra8(raw, w, h)
    assert np.array_equal(img[2, 1], np.float32([30, 20, 10, 255]) / np.float32(255))
    assert np.all(img[..., 3] == 1.0)
    # a constant image blurs to itself; bytes survive unpack -> pack
    const = np.full((w, h, 4), 0.25, np.float32)
    assert np.array_equal(O.blur3x3(const, w, h), const)
    rng = np.random.default_rng(0)
    raw = rng.integers(0, 256, (h, w, 4), dtype=np.uint8)
    raw[..., 3] = 255
    back = O.pack_bgra8(np.transpose(O.unpack_bgra8(raw, w, h), (1, 0, 2)))
    assert np.array_equal(back, raw)


def test_oracle_splat_coverage():
    # a point at the centre of a 4x4 target with size 2 covers the 2x2 middle
    mvp = np.eye(4, dtype=np.float32).reshape(-1)
    fb = np.zeros((4, 4, 4))
    O.splat(fb, np.zeros((1, 3), np.float32), np.ones((1, 4), np.float32), np.float32([2.0]), mvp, 4, 4, 1, 0)
    assert np.array_equal(fb[..., 0] > 0, np.array([[0, 0, 0, 0], [0, 1, 1, 0], [0, 1, 1, 0], [0, 0, 0, 0]], bool))
    # behind the camera (z < 0) or outside x/y: clipped
    fb[:] = 0
    O.splat(fb, np.float32([[0, 0, -0.5], [1.5, 0, 0.5]]), np.ones((1, 4), np.float32), np.float32([2.0]), mvp, 4, 4,
            0, 0)
    assert not fb.any()


@pytest.mark.gpu
def test_advect_bit_exact(dev):
    pos, vel = point_cloud(3, 50_001)
    pos *= 1.7  # most points start outside the radius: the reflection branch runs
    P, V = M.Buffer(dev, pos.reshape(-1)), M.Buffer(dev, vel.reshape(-1))
    M.launch(M.kernels.advect_points, (P, V, 1.0 / 60, 1.6), pos.shape[0], stream=dev.stream)
    dev.synchronize()
    wp, wv = O.advect(pos, vel, np.float32(1.0 / 60), np.float32(1.6))
    assert np.array_equal(P.array().reshape(-1, 3), wp)
    assert np.array_equal(V.array().reshape(-1, 3), wv)


@pytest.mark.gpu
def test_splat_edge_cases(dev):
    w, h = 37, 23
    mvp = camera(0.7, w, h)
    pos, _ = point_cloud(4, 3000)
    pos[:10] = np.nan                      # NaN positions are dropped
    pos[10:20] *= 50                       # far outside: clipped
    size = np.random.default_rng(5).uniform(-1, 9, pos.shape[0]).astype(np.float32)
    size[20] = 1e9                         # one huge point covers the whole target
    col = np.random.default_rng(6).uniform(0, 0.01, (pos.shape[0], 4)).astype(np.float32)
    fb = M.Buffer(dev, np.zeros(4 * w * h, np.float32))
    args = (fb, M.Buffer(dev, pos.reshape(-1)), M.Buffer(dev, col.reshape(-1)), M.Buffer(dev, size),
            M.Buffer(dev, mvp), w, h, 1, 1)
    M.launch(M.kernels.splat_points, args, pos.shape[0], stream=dev.stream)
    dev.synchronize()
    want = O.splat(np.zeros((h, w, 4)), pos, col, size, mvp, w, h, 1, 1)
    got = fb.array().reshape(h, w, 4)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    with pytest.raises(M.ArgumentError, match="strides"):
        M.launch(M.kernels.splat_points, args[:7] + (2, 0), pos.shape[0], stream=dev.stream)


@pytest.mark.gpu
def test_two_scatters_and_chain_graph(dev):
    w, h = RASTER_W, RASTER_H
    r = build_raster(dev, na=20_000, nb=10_000, seed=7)
    M.run(r.plan)
    I, B = r.inputs, r.bufs
    pa, va = O.advect(I["pos_a"], I["vel_a"], np.float32(1.0 / 60), np.float32(1.6))
    pb, vb = O.advect(I["pos_b"], I["vel_b"], np.float32(1.0 / 60), np.float32(1.6))
    assert np.array_equal(B["pos_a"].array().reshape(-1, 3), pa)
    assert np.array_equal(B["vel_b"].array().reshape(-1, 3), vb)
    fb = np.zeros((h, w, 4))
    fb[:] = (0.02, 0.02, 0.04, 1.0)
    fb[:] = fb.astype(np.float32)
    O.splat(fb, pa, I["col_a"], I["size_a"], I["mvp"], w, h, 1, 0)
    O.splat(fb, pb, I["col_b"], I["size_b"], I["mvp"], w, h, 0, 1)
    got_fb = B["fb"].array().reshape(h, w, 4)
    np.testing.assert_allclose(got_fb, fb, rtol=1e-5, atol=1e-6)
    assert (got_fb[..., 0] > 0.021).sum() > 1000  # the clouds are on screen
    raw = B["raw"].array().reshape(h, w, 4)
    assert np.array_equal(raw, O.pack_bgra8(got_fb))
    assert np.abs(raw.astype(int) - O.pack_bgra8(fb.astype(np.float32)).astype(int)).max() <= 1
    img = O.unpack_bgra8(raw, w, h)
    for _ in range(3):
        img = O.blur3x3(img, w, h)
    assert np.array_equal(B["out"].array().reshape(w, h, 4), img)
    # the chain's transients: only adjacent stages are live together
    assert M.peakbytes(r.plan) == 2 * 16 * w * h
