"""Implicit-GEMM convolution and the CNN forward pass: the oracle against torch
on the CPU, each CUDA kernel against the oracle on the GPU.

Tolerances. A conv layer's stored output is its fp32 sum rounded once to
bfloat16: against the oracle's double result the error is at most half a
bfloat16 ulp (2^-9 relative) plus the fp32 accumulation error, so the layer
tests hold |got - ref| <= 2^-8 |ref| + 1e-3 max|ref|. Logits of the whole
network (nine bf16 roundings deep) are held to the workload's 1e-2: max|got -
ref| <= 1e-2 max|ref|.
"""
import numpy as np
import pytest

import mantle_cuda as M
from mantle_cuda.workloads import CNN_CLASSES, CNN_LAYERS, STEM_CPAD, build_cnn
from oracle import oracle as O


def close_layer(got_bits, ref):
    got = O.bf16_to_f32(got_bits).astype(np.float64)
    assert got.shape == ref.shape
    tol = 2.0 ** -8 * np.abs(ref) + 1e-3 * np.abs(ref).max()
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance, worst {np.abs(got - ref).max()}"


def test_oracle_conv_matches_torch():
    import torch
    rng = np.random.default_rng(1)
    for (n, h, w, cin, cout, k, s, p) in [(2, 9, 11, 8, 16, 3, 2, 1), (1, 16, 16, 3, 8, 7, 2, 3), (1, 5, 5, 4, 4, 3, 1, 1)]:
        x = O.bf16_bits(rng.standard_normal((n, h, w, cin)).astype(np.float32))
        wt = O.bf16_bits(rng.standard_normal((k, k, cin, cout)).astype(np.float32))
        od, oh = O.conv_bf16(x, wt, s, p, relu=True)
        xt = torch.tensor(O.bf16_to_f32(x), dtype=torch.float64).permute(0, 3, 1, 2)
        wtt = torch.tensor(O.bf16_to_f32(wt), dtype=torch.float64).permute(3, 2, 0, 1)
        ref = torch.relu(torch.nn.functional.conv2d(xt, wtt, stride=s, padding=p)).permute(0, 2, 3, 1).numpy()
        assert np.abs(od - ref).max() <= 1e-12 * max(1.0, np.abs(ref).max())
        assert np.array_equal(oh, O.bf16_bits(od.astype(np.float32)))


def test_oracle_gap_fc_and_layout():
    rng = np.random.default_rng(2)
    act = O.bf16_bits(rng.random((3, 2, 3, 16)).astype(np.float32))
    w = rng.standard_normal((16, 5)).astype(np.float32)
    want = O.bf16_to_f32(act).astype(np.float64).mean(axis=(1, 2)) @ w.astype(np.float64)
    assert np.allclose(O.gap_fc(act, w), want, rtol=1e-13, atol=1e-13)
    x = np.arange(2 * 3 * 4 * 5, dtype=np.uint16).reshape(2, 3, 4, 5)
    y = O.nchw_to_nhwc(x, 8)
    assert y.shape == (2, 4, 5, 8) and np.array_equal(y[..., :3], np.transpose(x, (0, 2, 3, 1))) and not y[..., 3:].any()


def test_cnn_flop_count():
    from mantle_cuda.workloads import cnn_macs_per_image
    assert cnn_macs_per_image() == 869961728


def _rand_bits(rng, shape, scale=1.0, nonneg=False):
    x = rng.standard_normal(shape).astype(np.float32) * scale
    return O.bf16_bits(np.abs(x) if nonneg else x)


# Inputs under 128 KiB take the cp.async gather path. Larger ones with Cin a
# multiple of 64 take rectangular tiles (one tiled TMA box per filter tap) when
# a rectangle keeps at least 85 % of the 128 MMA rows busy, flat im2col runs
# otherwise; with Cin = 8 the 8-channel im2col path.
@pytest.mark.gpu
@pytest.mark.parametrize("n,h,w,cin,cout,k,s,relu", [
    (2, 14, 14, 64, 64, 3, 1, 1),     # gather; BN = 64, stride 1
    (3, 15, 13, 64, 128, 3, 2, 1),    # gather; BN = 128, stride 2, odd sizes
    (2, 7, 7, 256, 512, 3, 1, 0),     # gather; BN = 256, two column tiles, no ReLU
    (2, 30, 22, 8, 64, 7, 2, 1),      # gather; 8 channels, 7x7, K not a multiple of 64
    (1, 9, 9, 128, 256, 3, 2, 1),     # gather; fewer pixels than one tile
    (4, 28, 28, 64, 64, 3, 1, 1),     # rectangles 4 x 28; BN = 64
    (2, 56, 56, 64, 128, 3, 2, 1),    # rectangles 4 x 28; stride 2, BN = 128
    (2, 56, 56, 64, 64, 3, 1, 1),     # rectangles 2 x 56, two CTAs per SM
    (8, 13, 35, 64, 64, 3, 1, 1),     # rectangles 7 x 18, ragged in both directions
    (4, 26, 104, 128, 256, 3, 2, 1),  # rectangles 7 x 18 of a 13 x 52 output, stride 2, BN = 256
    (5, 15, 17, 128, 256, 3, 1, 1),   # im2col; tiles span rows and images, ragged last tile
    (6, 14, 14, 256, 512, 3, 2, 1),   # im2col; 7x7 outputs, BN = 256
    (3, 7, 7, 512, 512, 3, 1, 0),     # im2col; 7x7 in and out, no ReLU
    (100, 14, 14, 128, 512, 3, 1, 1),  # im2col; 154 M tiles, two column tiles each, several per CTA
    (195, 7, 7, 512, 512, 3, 1, 1),   # im2col, two 128-pixel runs per CTA (150 one-run tiles > 148 SMs);
                                      # the last tile's second run past the end
    (2, 112, 96, 8, 64, 7, 2, 1),     # 8-channel im2col (the stem's shape)
    (3, 61, 45, 8, 128, 7, 2, 1),     # 8-channel im2col; odd sizes
])
def test_conv_matches_oracle(dev, n, h, w, cin, cout, k, s, relu):
    import torch
    rng = np.random.default_rng(7)
    x = _rand_bits(rng, (n, h, w, cin), nonneg=True)
    wt = _rand_bits(rng, (k, k, cin, cout), scale=float(np.sqrt(2.0 / (k * k * cin))))
    pad = k // 2
    ho, wo = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
    xt = torch.from_numpy(x.view(np.int16)).cuda()
    wtt = torch.from_numpy(wt.view(np.int16)).cuda()
    out = torch.full((n, ho, wo, cout), -1, dtype=torch.int16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    M.launch(M.kernels.conv2d_bf16, (out, xt, wtt, h, w, cin, cout, k, s, pad, relu, 0, 0), n, stream=st)
    torch.cuda.synchronize()
    ref, _ = O.conv_bf16(x, wt, s, pad, relu=bool(relu))
    close_layer(out.cpu().numpy().view(np.uint16), ref)


# An input stored with its padding columns: with 4 channels at stride 2 and
# output rows up to 128 pixels, the raw-row path (each stage one bulk copy of
# input rows, the stride-2 windows read in place by the descriptor); otherwise
# the window paths when the stored margin equals the padding (and the input is
# at least 128 KiB) — 8 channels (128-byte windows) or 4 (64-byte windows, two
# filter rows per K block) — the im2col or gather paths otherwise.
@pytest.mark.gpu
@pytest.mark.parametrize("cin,n,h,w,cout,k,s,pad,wpad", [
    (8, 2, 112, 96, 64, 7, 2, 3, 3),     # window: the stem's geometry
    (8, 3, 57, 122, 128, 7, 2, 3, 3),    # window; odd height, BN = 128
    (8, 6, 40, 40, 64, 5, 1, 2, 2),      # im2col-chunk: the 8-wide window would leave the stored row
    (8, 1, 20, 18, 64, 7, 2, 3, 3),      # gather (small input) with a margin
    (8, 2, 112, 96, 64, 7, 2, 3, 4),     # im2col-chunk path: margin wider than the padding
    (4, 3, 112, 96, 64, 7, 2, 3, 3),     # 4 channels, raw input rows: the stem's geometry
    (4, 6, 61, 46, 128, 7, 2, 3, 3),     # raw rows, odd height (last stage partial), two column blocks
    (4, 12, 31, 40, 64, 7, 2, 3, 3),     # raw rows, one stage per image
    (4, 2, 40, 300, 64, 7, 2, 3, 3),     # 4-channel window rectangles 4 x 30: output rows wider than 128
    (4, 11, 6, 258, 64, 7, 2, 3, 3),     # 4-channel window, flat runs (3 x 129 outputs: no rectangle fills 85 %)
])
@pytest.mark.parametrize("stem_pair", ["1", "0"])
def test_conv_with_stored_margin(dev, monkeypatch, stem_pair, cin, n, h, w, cout, k, s, pad, wpad):
    import torch
    monkeypatch.setenv("MTL_CONV_STEM_PAIR", stem_pair)
    rng = np.random.default_rng(11)
    x = _rand_bits(rng, (n, h, w, cin), nonneg=True)
    x[..., 3:] = 0  # padded channels, as the network stores them
    wt = _rand_bits(rng, (k, k, cin, cout), scale=float(np.sqrt(2.0 / (k * k * 3))))
    stored = np.zeros((n, h, w + 2 * wpad, cin), np.uint16)
    stored[:, :, wpad:wpad + w] = x
    ho, wo = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
    xt = torch.from_numpy(stored.view(np.int16)).cuda()
    wtt = torch.from_numpy(wt.view(np.int16)).cuda()
    out = torch.full((n, ho, wo, cout), -1, dtype=torch.int16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    M.launch(M.kernels.conv2d_bf16, (out, xt, wtt, h, w, cin, cout, k, s, pad, 1, wpad, 0), n, stream=st)
    torch.cuda.synchronize()
    ref, _ = O.conv_bf16(x, wt, s, pad, relu=True)
    close_layer(out.cpu().numpy().view(np.uint16), ref)


# Stored margins on both sides: the input rows carry `wpad` zero columns and the
# output rows `owp`, which the kernel writes as zeros. Stride-1 layers whose
# input margin equals the padding take the flat-halo path (one TMA load per
# channel block, taps as shifted views, weights resident in shared memory)
# when the halo fits one box and wastes under 15 % of the MMA rows.
@pytest.mark.gpu
@pytest.mark.parametrize("n,h,w,cin,cout,k,s,pad,wpad,owp", [
    (4, 56, 56, 64, 64, 3, 1, 1, 1, 1),     # halo, BN = 64: the first stage's second conv
    (3, 56, 56, 64, 64, 3, 1, 1, 1, 0),     # halo, output without margins
    (4, 28, 28, 128, 128, 3, 1, 1, 1, 1),   # halo, two 64-wide column blocks (weights 2 x 144 KiB)
    (48, 28, 28, 128, 128, 3, 1, 1, 1, 1),  # halo, several tiles per CTA on three stages
    (2, 40, 40, 64, 128, 3, 1, 1, 1, 1),    # halo, BN = 128, three stages
    (3, 37, 45, 64, 64, 3, 1, 1, 1, 1),     # halo, odd sizes, tiles end past the image
    (2, 30, 30, 64, 64, 5, 1, 2, 2, 2),     # 5x5: the halo exceeds one box -> rectangles, 2-pixel margins
    (2, 112, 112, 64, 64, 3, 2, 1, 0, 1),   # stride-2 halo writing margins (the first stage's stride-2 conv)
    (2, 112, 112, 64, 64, 3, 2, 1, 1, 1),   # the same over an input with stored margins: rectangles
    (4, 28, 28, 128, 256, 3, 2, 1, 1, 1),   # flat im2col runs, margins in and out
    (1, 9, 9, 64, 64, 3, 1, 1, 0, 1),       # gather (small input) writing margins
])
def test_conv_margins_and_halo(dev, n, h, w, cin, cout, k, s, pad, wpad, owp):
    import torch
    rng = np.random.default_rng(17)
    x = _rand_bits(rng, (n, h, w, cin), nonneg=True)
    wt = _rand_bits(rng, (k, k, cin, cout), scale=float(np.sqrt(2.0 / (k * k * cin))))
    stored = np.zeros((n, h, w + 2 * wpad, cin), np.uint16)
    stored[:, :, wpad:wpad + w] = x
    ho, wo = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
    xt = torch.from_numpy(stored.view(np.int16)).cuda()
    wtt = torch.from_numpy(wt.view(np.int16)).cuda()
    out = torch.full((n, ho, wo + 2 * owp, cout), -1, dtype=torch.int16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    M.launch(M.kernels.conv2d_bf16, (out, xt, wtt, h, w, cin, cout, k, s, pad, 1, wpad, owp), n, stream=st)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    ref, _ = O.conv_bf16(x, wt, s, pad, relu=True)
    close_layer(got[:, :, owp:owp + wo], ref)
    assert not got[:, :, :owp].any() and not got[:, :, owp + wo:].any()


# A one-run layer with fewer tiles than SMs (a small batch, such as one GPU's
# share of a batch split over eight) splits each tile's K blocks into parts:
# fp32 planes in the launch's scratch, added in part order by a second
# kernel. The same layer given the scratch (split) and not (whole), both
# against the oracle, margins included.
@pytest.mark.gpu
@pytest.mark.parametrize("n,h,w,cin,cout,s,owp", [
    (8, 7, 7, 512, 512, 1, 0),     # flat im2col runs: 8 tiles, 72 K blocks
    (8, 14, 14, 256, 512, 2, 1),   # flat runs, stride 2, margins out
    (6, 14, 14, 256, 256, 1, 1),   # rectangles, margins out
    (3, 28, 28, 256, 256, 2, 0),   # stride 2, 14 x 14 outputs
])
def test_conv_split_k(dev, n, h, w, cin, cout, s, owp):
    import torch
    rng = np.random.default_rng(29)
    k, pad = 3, 1
    x = _rand_bits(rng, (n, h, w, cin), nonneg=True)
    wt = _rand_bits(rng, (k, k, cin, cout), scale=float(np.sqrt(2.0 / (k * k * cin))))
    ho, wo = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
    xt = torch.from_numpy(x.view(np.int16)).cuda()
    wtt = torch.from_numpy(wt.view(np.int16)).cuda()
    ref, _ = O.conv_bf16(x, wt, s, pad, relu=True)
    st = torch.cuda.current_stream().cuda_stream
    plane = n * ho * wo * cout * 4
    for split in (True, False):
        out = torch.full((n, ho, wo + 2 * owp, cout), -1, dtype=torch.int16, device="cuda")
        args = (out, xt, wtt, h, w, cin, cout, k, s, pad, 1, 0, owp)
        need = M.workspace_bytes(M.kernels.conv2d_bf16, args, n)
        assert need >= 2 * plane and need % plane == 0, need
        ws = torch.full((need // 4,), float("nan"), dtype=torch.float32, device="cuda") if split else None
        M.launch(M.kernels.conv2d_bf16, args, n, stream=st, workspace=ws)
        torch.cuda.synchronize()
        got = out.cpu().numpy().view(np.uint16)
        close_layer(got[:, :, owp:owp + wo], ref)
        assert not got[:, :, :owp].any() and not got[:, :, owp + wo:].any()


# Stride-2 halo: a 3x3 stride-2 conv (padding 1) over plain NHWC rows reads
# the input as four parity planes (tensor maps with pixel and row stride 2).
# A tile is T output rows; per plane one load brings the frame of plane rows
# y0 - 1 .. y0 + T and columns -1 .. Wo - 1 (pq = Wo + 1 positions a row), and
# tap (r, c) of MMA row m reads frame position m + (r != 0) * pq + (c != 0).
def stride2_taps(p):
    """Filter taps (r, c) read from parity plane p = 2 * row parity + column parity."""
    rows = [1] if p >> 1 == 0 else [0, 2]
    cols = [1] if p & 1 == 0 else [0, 2]
    return [(r, c) for r in rows for c in cols]


@pytest.mark.parametrize("h,w", [(10, 14), (9, 13), (12, 7)])
def test_stride2_frame_addressing_matches_oracle(h, w):
    """The stride-2 halo kernel's frames and shifted reads, restated in numpy,
    against the oracle's direct convolution (even and odd sizes)."""
    rng = np.random.default_rng(23)
    n, cin, cout = 2, 8, 16
    x = _rand_bits(rng, (n, h, w, cin), nonneg=True)
    wt = _rand_bits(rng, (3, 3, cin, cout), scale=0.3)
    ref, _ = O.conv_bf16(x, wt, 2, 1, relu=False)
    ho, wo = ref.shape[1:3]
    xf = O.bf16_to_f32(x).astype(np.float64)
    wf = O.bf16_to_f32(wt).astype(np.float64)
    pq = wo + 1
    T = min(128 // pq, ho)
    got = np.zeros((n, ho, wo, cout))
    for img in range(n):
        for y0 in range(0, ho, T):
            acc = np.zeros((128, cout))
            for p in range(4):
                pr, pc = p >> 1, p & 1
                # past the frame: stale shared memory, never read for an output pixel
                frame = np.full((128 + pq + 1, cin), np.nan)
                frame[:(T + 1) * pq] = 0.0
                for R in range(T + 1):
                    for J in range(-1, wo):
                        iy, ix = 2 * (y0 - 1 + R) + pr, 2 * J + pc
                        if 0 <= iy < h and 0 <= ix < w:
                            frame[R * pq + J + 1] = xf[img, iy, ix]
                for (r, c) in stride2_taps(p):
                    off = (pq if r else 0) + (1 if c else 0)
                    acc += frame[off:off + 128] @ wf[r, c]
            for m in range(128):
                y, xo = y0 + m // pq, m % pq
                if m // pq < T and y < ho and xo < wo:
                    got[img, y, xo] = acc[m]
    assert np.allclose(got, ref, rtol=1e-12, atol=1e-12)


@pytest.mark.gpu
@pytest.mark.parametrize("n,h,w,cin,cout,owp", [
    (4, 112, 112, 64, 64, 0),    # the first stage's stride-2 conv (BN = 64, two rows a tile, six stages)
    (4, 56, 56, 64, 128, 0),     # the second stage's (BN = 128, four stages: one tile in flight)
    (3, 24, 40, 128, 256, 1),    # two channel blocks, four column blocks, output margins
    (3, 37, 45, 64, 64, 1),      # odd sizes: a short last tile, odd planes one row / column shorter
    (48, 56, 56, 64, 128, 0),    # several tiles per CTA: both issuers wait on the same four stages
    (24, 112, 112, 64, 64, 1),   # several tiles per CTA over six stages, output margins
])
def test_conv_stride2_halo(dev, n, h, w, cin, cout, owp):
    import torch
    rng = np.random.default_rng(29)
    x = _rand_bits(rng, (n, h, w, cin), nonneg=True)
    wt = _rand_bits(rng, (3, 3, cin, cout), scale=float(np.sqrt(2.0 / (9 * cin))))
    ref, _ = O.conv_bf16(x, wt, 2, 1, relu=True)
    ho, wo = ref.shape[1:3]
    xt = torch.from_numpy(x.view(np.int16)).cuda()
    wtt = torch.from_numpy(wt.view(np.int16)).cuda()
    out = torch.full((n, ho, wo + 2 * owp, cout), -1, dtype=torch.int16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    M.launch(M.kernels.conv2d_bf16, (out, xt, wtt, h, w, cin, cout, 3, 2, 1, 1, 0, owp), n, stream=st)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    close_layer(got[:, :, owp:owp + wo], ref)
    assert not got[:, :, :owp].any() and not got[:, :, owp + wo:].any()


# The stem straight from an NCHW input: each stage's channel-plane rows are
# bulk-copied to shared memory and converted there to padded NHWC rows. With
# 64 output channels the weights-in-tensor-memory kernel (two output rows per
# MMA chain) runs, unless MTL_CONV_STEM_PAIR=0 selects the pixel-row kernel.
@pytest.mark.gpu
@pytest.mark.parametrize("n,c,h,w,cout,owp,k,pad", [
    (2, 3, 224, 224, 64, 0, 7, 3),   # the network's stem
    (3, 3, 61, 96, 128, 1, 7, 3),    # odd height (a partial last stage), two column blocks, output margins
    (3, 3, 61, 96, 64, 1, 7, 3),     # odd output height: the last row pair has one row; output margins
    (2, 3, 30, 200, 64, 2, 7, 3),    # 100 output columns: the MMA's N (112) runs past the row
    (5, 1, 40, 48, 64, 0, 7, 3),     # one channel
    (4, 4, 33, 64, 64, 0, 7, 3),     # four channels (no padding channel)
    (3, 3, 42, 64, 64, 1, 7, 2),     # even padding: the converter's aligned-word path
])
@pytest.mark.parametrize("stem_pair", ["1", "0"])
def test_conv_nchw_matches_oracle(dev, monkeypatch, stem_pair, n, c, h, w, cout, owp, k, pad):
    import torch
    monkeypatch.setenv("MTL_CONV_STEM_PAIR", stem_pair)
    rng = np.random.default_rng(19)
    s = 2
    x = _rand_bits(rng, (n, c, h, w), nonneg=True)
    wt = _rand_bits(rng, (k, k, 4, cout), scale=float(np.sqrt(2.0 / (k * k * c))))
    wt[:, :, c:] = 0
    ho, wo = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
    xt = torch.from_numpy(x.view(np.int16)).cuda()
    wtt = torch.from_numpy(wt.view(np.int16)).cuda()
    out = torch.full((n, ho, wo + 2 * owp, cout), -1, dtype=torch.int16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    M.launch(M.kernels.conv2d_nchw_bf16, (out, xt, wtt, h, w, c, cout, k, s, pad, 1, owp), n, stream=st)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    ref, _ = O.conv_bf16(O.nchw_to_nhwc(x, 4), wt, s, pad, relu=True)
    close_layer(got[:, :, owp:owp + wo], ref)
    assert not got[:, :, :owp].any() and not got[:, :, owp + wo:].any()


@pytest.mark.gpu
def test_conv_nchw_refusals(dev):
    import torch
    t = torch.zeros(1 << 20, dtype=torch.int16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    with pytest.raises(M.MantleError, match="W a multiple of 8"):
        M.launch(M.kernels.conv2d_nchw_bf16, (t, t, t, 16, 20, 3, 64, 7, 2, 3, 1, 0), 1, stream=st)
    with pytest.raises(M.MantleError, match="C <= 4"):
        M.launch(M.kernels.conv2d_nchw_bf16, (t, t, t, 16, 16, 5, 64, 7, 2, 3, 1, 0), 1, stream=st)


@pytest.mark.gpu
@pytest.mark.parametrize("w", [23, 24])  # scalar path, vector path (W a multiple of 8)
@pytest.mark.parametrize("cp", [4, 8])
def test_nchw_to_nhwc_with_margin(dev, w, cp):
    import torch
    rng = np.random.default_rng(12)
    x = _rand_bits(rng, (3, 3, 17, w))
    xt = torch.from_numpy(x.view(np.int16)).cuda()
    out = torch.full((3, 17, w + 6, cp), -1, dtype=torch.int16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    M.launch(M.kernels.nchw_to_nhwc_bf16, (out, xt, 3, 17, w, cp, 3), 3, stream=st)
    torch.cuda.synchronize()
    want = np.zeros((3, 17, w + 6, cp), np.uint16)
    want[:, :, 3:3 + w] = O.nchw_to_nhwc(x, cp)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want)


@pytest.mark.gpu
def test_conv_refusals(dev):
    import torch
    t = torch.zeros(1 << 20, dtype=torch.int16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    with pytest.raises(M.MantleError, match="Cin must be a multiple of 8"):
        M.launch(M.kernels.conv2d_bf16, (t, t, t, 8, 8, 3, 64, 3, 1, 1, 1, 0, 0), 1, stream=st)
    with pytest.raises(M.MantleError, match="Cout must be a multiple of 64"):
        M.launch(M.kernels.conv2d_bf16, (t, t, t, 8, 8, 8, 32, 3, 1, 1, 1, 0, 0), 1, stream=st)
    with pytest.raises(M.MantleError, match="bytes"):
        M.launch(M.kernels.conv2d_bf16, (t, t, t, 64, 64, 64, 64, 3, 1, 1, 1, 0, 0), 8, stream=st)


@pytest.mark.gpu
def test_cnn_small_batch_matches_oracle(dev):
    w = build_cnn(dev, batch=2)
    M.run(w.plan)
    x, ws, fc = w.host_params()
    want = O.cnn_forward(x, ws, fc, CNN_LAYERS, STEM_CPAD)
    got = w.logits.array().reshape(2, CNN_CLASSES)
    assert np.abs(got - want).max() <= 1e-2 * np.abs(want).max()
    assert np.corrcoef(got.ravel(), want.ravel())[0, 1] > 0.9999
    # the activations are transients: the placer aliases them
    assert M.peakbytes(w.plan) < M.naivebytes(w.plan)


@pytest.mark.gpu
def test_cnn_one_gpus_share_of_eight_matches_oracle(dev):
    # Batch 32, one GPU's share of the batch-256 network on eight: the late
    # layers split their K blocks; images at both ends and inside, against the
    # oracle.
    w = build_cnn(dev, batch=32)
    M.run(w.plan)
    x, ws, fc = w.host_params()
    got = w.logits.array().reshape(32, CNN_CLASSES)
    images = [0, 13, 31]
    want = O.cnn_forward(x[images], ws, fc, CNN_LAYERS, STEM_CPAD)
    for j, i in enumerate(images):
        assert np.abs(got[i] - want[j]).max() <= 1e-2 * np.abs(want[j]).max(), f"image {i}"


@pytest.mark.gpu
def test_cnn_full_batch_sampled_images(dev):
    # The benchmark shape (batch 256), checked against the oracle at both ends
    # of every 32-image shard an 8-GPU run gives a rank (0, 31, 32, 63, ...,
    # 255), and one image inside a shard.
    w = build_cnn(dev)
    M.run(w.plan)
    x, ws, fc = w.host_params()
    got = w.logits.array().reshape(256, CNN_CLASSES)
    images = sorted({k for r in range(8) for k in (32 * r, 32 * r + 31)} | {201})
    want = O.cnn_forward(x[images], ws, fc, CNN_LAYERS, STEM_CPAD)
    for j, i in enumerate(images):
        assert np.abs(got[i] - want[j]).max() <= 1e-2 * np.abs(want[j]).max(), f"image {i}"


@pytest.mark.gpu
@pytest.mark.parametrize("n,hw,c,classes", [
    (37, 49, 512, 1000),  # 16-byte loads in both kernels, ragged image tile
    (3, 5, 64, 10),       # fewer pixels than pixel groups; scalar FC loads
    (2, 3, 6, 12),        # 4-byte GAP loads (C not a multiple of 8)
    (4, 9, 1536, 8),      # the widest C: one pixel group, threads loop over the channel units
    (5, 49, 96, 1000),    # pooled in the FC kernel with 16-channel slices: two CTAs of each cluster idle
])
@pytest.mark.parametrize("fused", ["0", "1"])  # two kernels; pooling inside the FC kernel
def test_gap_fc_matches_oracle(dev, monkeypatch, fused, n, hw, c, classes):
    import torch
    monkeypatch.setenv("MTL_GAPFC_FUSED", fused)
    rng = np.random.default_rng(13)
    act = _rand_bits(rng, (n, hw, 1, c), nonneg=True)
    w = (rng.standard_normal((c, classes)) * np.sqrt(2.0 / c)).astype(np.float32)
    at = torch.from_numpy(act.view(np.int16)).cuda()
    wt = torch.from_numpy(w).cuda()
    logits = torch.full((n, classes), float("nan"), device="cuda")
    args = (logits, at, wt, hw, c, classes)
    scratch = torch.empty(M.workspace_bytes(M.kernels.gap_fc, args, n), dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    M.launch(M.kernels.gap_fc, args, n, stream=st, workspace=scratch)
    torch.cuda.synchronize()
    want = O.gap_fc(act, w)
    got = logits.cpu().numpy()
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()
