"""Batched complex FFT (lengths 16, 256, 4096): the oracle against numpy.fft on
the CPU, and the CUDA kernel against the oracle on the GPU.

Tolerance (fp32 FFT): relative L2 error <= 1e-5 per transform batch against the
double-precision oracle, for the forward output and for the forward-inverse
round trip against the input.
"""
import numpy as np
import pytest

import mantle_cuda as M
from mantle_cuda.workloads import build_fft, seeded_complex
from oracle import oracle as O

RTOL = 1e-5


def rel(a, b):
    return float(np.linalg.norm((a - b).ravel()) / np.linalg.norm(np.asarray(b).ravel()))


@pytest.mark.parametrize("n", [16, 256, 4096])
def test_oracle_fft_matches_numpy(n):
    x = seeded_complex(9, (7, n))
    assert rel(O.fft(x), np.fft.fft(x.astype(np.complex128), axis=1)) < 1e-14
    assert rel(O.fft(x, inverse=True), np.fft.ifft(x.astype(np.complex128), axis=1)) < 1e-14


def test_oracle_fft_known_answers():
    # a unit impulse at 0 transforms to all ones; a pure tone e^{2 pi i 3 j / n}
    # to n at bin 3 and zero elsewhere
    n = 256
    imp = np.zeros((1, n), np.complex64)
    imp[0, 0] = 1
    assert np.allclose(O.fft(imp), 1.0, atol=1e-15)
    j = np.arange(n)
    tone = np.exp(2j * np.pi * 3 * j / n).astype(np.complex64)[None]
    want = np.zeros(n)
    want[3] = n
    assert np.abs(O.fft(tone)[0] - want).max() < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("n,batch", [(16, 1000), (256, 333), (4096, 65), (4096, 1)])
def test_fft_matches_oracle(dev, n, batch):
    w = build_fft(dev, batch=batch, n=n, seed=11)
    M.run(w.plan)
    x = w.inputs["x"]
    want = O.fft(x)
    got = w.spectrum.array().reshape(batch, n)
    assert rel(got, want) < RTOL
    back = w.back.array().reshape(batch, n)
    assert rel(back, x) < RTOL
    assert rel(back, O.fft(want.astype(np.complex64), inverse=True)) < RTOL


@pytest.mark.gpu
def test_fft_in_place_and_direct_launch(dev):
    import torch
    n, batch = 4096, 40
    x = seeded_complex(12, (batch, n))
    t = torch.from_numpy(x.copy()).to("cuda")
    s = torch.cuda.current_stream().cuda_stream
    M.launch(M.kernels.fft_c2c, (t, t, n, 0), batch, stream=s)
    torch.cuda.synchronize()
    assert rel(t.cpu().numpy(), O.fft(x)) < RTOL
    M.launch(M.kernels.fft_c2c, (t, t, n, 1), batch, stream=s)
    torch.cuda.synchronize()
    assert rel(t.cpu().numpy(), x) < RTOL


@pytest.mark.gpu
def test_fft_refuses_bad_launches(dev):
    import torch
    t = torch.zeros(4096 * 2, dtype=torch.complex64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    with pytest.raises(M.MantleError, match="not supported"):
        M.launch(M.kernels.fft_c2c, (t, t, 512, 0), 2, stream=s)
    with pytest.raises(M.MantleError, match="bytes"):
        M.launch(M.kernels.fft_c2c, (t, t, 4096, 0), 3, stream=s)
    with pytest.raises(M.MantleError, match="overlap"):
        M.launch(M.kernels.fft_c2c, (t[1:], t[:-1], 16, 0), 10, stream=s)
    M.launch(M.kernels.fft_c2c, (t, t, 4096, 0), 0, stream=s)  # empty batch: nothing to do


@pytest.mark.gpu
def test_fft_full_size_round_trip(dev):
    # The benchmark shape: 16384 transforms of 4096. Forward checked against the
    # oracle on a sample of transforms; the round trip on all of them.
    w = build_fft(dev)
    M.run(w.plan)
    x = w.inputs["x"]
    # every 997th transform, and both ends of every 2048-transform shard an
    # 8-GPU run gives a rank
    rows = np.unique(np.concatenate([np.arange(0, w.batch, 997), np.arange(0, w.batch, 2048),
                                     np.arange(2047, w.batch, 2048)]))
    spec = w.spectrum.array().reshape(w.batch, w.n)
    assert rel(spec[rows], O.fft(x[rows])) < RTOL
    assert rel(w.back.array().reshape(w.batch, w.n), x) < RTOL
