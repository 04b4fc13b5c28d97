"""Batched bf16 GEMM with fp32 accumulation (tcgen05 tensor cores): the oracle
on the CPU, and the CUDA kernel against the oracle on the GPU.

Tolerance: the workload allows 1e-2 relative error for bf16-in/fp32-accumulate
GEMM. The tests hold the kernel to |C - C_ref| <= 1e-2 * max|C_ref| elementwise
and, tighter, to a relative Frobenius error <= 1e-5 against the double-precision
oracle (fp32 accumulation over K <= 8192 of products that are exact).
"""
import os

import numpy as np
import pytest

import mantle_cuda as M
from mantle_cuda.workloads import build_gemm
from oracle import oracle as O

RTOL_MAX = 1e-2
RTOL_FRO = 1e-5


def check(got, want):
    got = np.asarray(got, np.float64)
    scale = np.abs(want).max()
    assert np.abs(got - want).max() <= RTOL_MAX * scale
    assert np.linalg.norm((got - want).ravel()) <= RTOL_FRO * np.linalg.norm(want.ravel())


def test_oracle_gemm_matches_numpy():
    rng = np.random.default_rng(3)
    b, m, n, k = 3, 37, 24, 56
    A = O.bf16_bits(rng.standard_normal((b, m, k)).astype(np.float32))
    B = O.bf16_bits(rng.standard_normal((b, k, n)).astype(np.float32))
    want = np.matmul(O.bf16_to_f32(A).astype(np.float64), O.bf16_to_f32(B).astype(np.float64))
    assert np.array_equal(O.gemm_bf16(A, B, m, n, k, b), want)
    assert np.array_equal(O.gemm_bf16(A, B, m, n, k, b, row0=10, rows=5), want[:, 10:15])


def test_bf16_rounding_is_nearest_even():
    # the bfloat16 ulp at 1 is 2^-7: halfway cases go to the even mantissa
    x = np.array([1.0, 1 + 2 ** -8, 1 + 3 * 2 ** -8, 1 + 2 ** -7 + 2 ** -9, -0.0], np.float32)
    want = [1.0, 1.0, 1 + 2 ** -6, 1 + 2 ** -7, -0.0]
    got = O.bf16_to_f32(O.bf16_bits(x))
    assert list(got) == want and np.signbit(got[-1])


@pytest.mark.gpu
@pytest.mark.parametrize("batch,m,n,k", [
    (1, 128, 256, 64),      # one tile, one k-block
    (2, 256, 512, 1024),    # several tiles and k-blocks
    (3, 200, 264, 72),      # ragged M, N and K
    (1, 1000, 1000, 1000),  # ragged everywhere, N and K multiples of 8 only
    (1, 64, 8, 8),          # smaller than a tile
    (1, 384, 264, 136),     # a last row tile half past M, a last column tile mostly past N
    (2, 512, 768, 512),     # several tiles a CTA
    (40, 96, 2048, 128),    # M within one run: 128 x 256 tiles, several a CTA (both accumulators)
])
def test_gemm_matches_oracle(dev, batch, m, n, k):
    w = build_gemm(dev, batch=batch, M=m, N=n, K=k, seed=5)
    M.run(w.plan)
    A, B = w.host_operands()
    want = O.gemm_bf16(A, B, m, n, k, batch)
    check(w.C.array().reshape(batch, m, n), want)


@pytest.mark.gpu
def test_gemm_direct_launch_and_refusals(dev):
    import torch
    from mantle_cuda.workloads import gemm_operands
    A, B = gemm_operands(2, 384, 512, 256, seed=9)
    C = torch.full((2, 384, 512), float("nan"), device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    M.launch(M.kernels.gemm_bf16, (C, A, B, 384, 512, 256), 2, stream=s)
    torch.cuda.synchronize()
    want = torch.matmul(A.double(), B.double()).cpu().numpy()
    check(C.cpu().numpy(), want)
    with pytest.raises(M.MantleError, match="multiples of 8"):
        M.launch(M.kernels.gemm_bf16, (C, A, B, 384, 510, 256), 1, stream=s)
    with pytest.raises(M.MantleError, match="bytes"):
        M.launch(M.kernels.gemm_bf16, (C, A, B, 384, 512, 256), 3, stream=s)
    # K = 0: C is the empty sum
    M.launch(M.kernels.gemm_bf16, (C, A, B, 384, 512, 0), 2, stream=s)
    torch.cuda.synchronize()
    assert float(C.abs().max()) == 0.0


@pytest.mark.gpu
def test_gemm_full_size_sampled_rows(dev):
    # The benchmark shape: 8 GEMMs of 8192^3. Every batch is checked on 8 rows
    # spread over the tiles (both halves of a TMEM accumulator, every lane quarter).
    w = build_gemm(dev)
    M.run(w.plan)
    A, B = w.host_operands()
    C = w.C.array().reshape(w.batch, w.M, w.N)
    for r0 in (0, 95, 130, 4133, 8191):
        want = O.gemm_bf16(A, B, w.M, w.N, w.K, w.batch, row0=r0, rows=1)
        check(C[:, r0:r0 + 1], want)


@pytest.mark.gpu
def test_stalled_producer_wait_runs_out_and_the_context_stays_usable(dev):
    # The failure path of the bounded waits, made to run in milliseconds: the
    # limit is shortened to 20 ms and CTA 0's producer of the next launch
    # loads nothing, so its MMA issuer's wait on the first stage runs out. The
    # launch must return, the timeout must be counted, the other CTAs' tiles
    # must be right, and the next normal launch on the same context must be
    # right everywhere.
    import time

    import torch
    from mantle_cuda.workloads import gemm_operands
    A, B = gemm_operands(1, 512, 512, 512, seed=13)
    want = torch.matmul(A.double(), B.double()).cpu().numpy()
    C = torch.full((1, 512, 512), float("nan"), device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    M.kernel_timeouts(reset=True)
    try:
        M.set_wait_limit(20_000_000)
        M.inject_stall("gemm_bf16", 1)
        t0 = time.perf_counter()
        M.launch(M.kernels.gemm_bf16, (C, A, B, 512, 512, 512), 1, stream=s)
        torch.cuda.synchronize()
        took = time.perf_counter() - t0
    finally:
        M.inject_stall("gemm_bf16", 0)
        M.set_wait_limit(0)
    ran_out = M.kernel_timeouts()
    assert ran_out == 1, ran_out  # one CTA gave up, whichever of its threads' waits ran out first
    assert took < 1.0
    got = C.cpu().numpy()
    # tile 0 (columns 0..255 of rows 0..255: two 128-row runs, or of rows
    # 0..127 with MTL_GEMM_RUNS=1) belonged to the stalled CTA; the rest was
    # computed
    tm = 128 if os.environ.get("MTL_GEMM_RUNS") == "1" else 256
    assert np.isnan(got[0, :tm, :256]).all()
    check(got[0, tm:, :], want[0, tm:, :])
    check(got[0, :tm, 256:], want[0, :tm, 256:])
    # the same context, the default limit, no stall: every tile, no new timeout
    C.fill_(float("nan"))
    M.launch(M.kernels.gemm_bf16, (C, A, B, 512, 512, 512), 1, stream=s)
    torch.cuda.synchronize()
    check(C.cpu().numpy(), want)
    assert M.kernel_timeouts(reset=True) == ran_out
    with pytest.raises(M.ArgumentError):
        M.set_wait_limit(1000)
    with pytest.raises(M.MantleError):
        M.inject_stall("fft_c2c", 1)
