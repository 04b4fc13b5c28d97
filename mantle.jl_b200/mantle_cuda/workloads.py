"""The graphs of the benchmark workloads, recorded through the public API the
way the reference's bench/*.jl scripts record theirs.

* elementwise chain: three Float32 vectors, eight dependent kernels
  (axpy a=0.5, mul, add, fma, abs, sqrt(abs), scale 2, sub) over transients —
  the multi-pass shape of bench/chain.jl with the op list of the workload.
* two scatters + three updates: two scatter-adds of Float32 values by Int32
  index into separate accumulators, one Int32 histogram fused into the first,
  and three in-place updates (touch1!/touch2!/touch3!, bench/stress.jl:30-45)
  on one buffer, ordered read-after-write by the derived hazards — the shape of
  bench/two_scatters.jl and bench/three_updates.jl.

Inputs are synthetic and seeded (numpy PCG64); nothing is read from disk.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import Buffer, Graph, Plan, Transient, Update, compute, dispatch, kernels, use


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """The contiguous slice [lo, hi) of `total` independent units (images,
    GEMMs of a batch, transforms) that rank `rank` of `world` runs. The units
    split evenly: a total that `world` does not divide is refused, so every
    rank does the same work and the slices, gathered in rank order, are the
    whole batch."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if total % world:
        raise ValueError(f"{total} units do not split evenly over {world} ranks")
    per = total // world
    return rank * per, (rank + 1) * per


def seeded_uniform(seed: int, n: int, lo: float, hi: float, stream: int = 0) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64([seed, stream]))
    return rng.uniform(lo, hi, n).astype(np.float32)


def seeded_integers(seed: int, n: int, hi: int, stream: int = 0) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64([seed, stream]))
    return rng.integers(0, hi, n, dtype=np.int32)


# ── elementwise chain ───────────────────────────────────────────────────────
@dataclass
class ChainWorkload:
    n: int
    x: Buffer
    y: Buffer
    z: Buffer
    out: Buffer
    graph: Graph
    plan: Plan
    inputs: dict = field(default_factory=dict)

    # compulsory bytes of one replay: read x, y, z, write out
    @property
    def bytes_compulsory(self) -> int:
        return 16 * self.n

    # bytes the eight unfused passes move: 12+12+12+16+8+8+8+12 per element
    @property
    def bytes_unfused(self) -> int:
        return 88 * self.n


def build_chain(dev, n: int = 1 << 22, seed: int = 0, fuse: bool = False, single_kernel: bool = False,
                **plan_kw) -> ChainWorkload:
    x_h = seeded_uniform(seed, n, -1, 1, 0)
    y_h = seeded_uniform(seed, n, -1, 1, 1)
    z_h = seeded_uniform(seed, n, -1, 1, 2)
    x, y, z = Buffer(dev, x_h), Buffer(dev, y_h), Buffer(dev, z_h)
    out = Buffer(dev, np.float32, n)
    g = Graph(dev)
    if single_kernel:
        compute(g, "chain8", lambda p: dispatch(p, kernels.chain8, (
            use(p, out, write=True), use(p, x, read=True), use(p, y, read=True), use(p, z, read=True)), n))
    else:
        t = [Transient.Buffer(g, np.float32, n) for _ in range(7)]
        W = lambda p, b: use(p, b, write=True)  # noqa: E731
        R = lambda p, b: use(p, b, read=True)  # noqa: E731
        compute(g, "axpy", lambda p: dispatch(p, kernels.axpy, (W(p, t[0]), R(p, x), R(p, y), 0.5), n))
        compute(g, "mul", lambda p: dispatch(p, kernels.mul, (W(p, t[1]), R(p, t[0]), R(p, z)), n))
        compute(g, "add", lambda p: dispatch(p, kernels.add, (W(p, t[2]), R(p, t[1]), R(p, y)), n))
        compute(g, "fma", lambda p: dispatch(p, kernels.fma, (W(p, t[3]), R(p, t[2]), R(p, x), R(p, z)), n))
        compute(g, "abs", lambda p: dispatch(p, kernels.abs, (W(p, t[4]), R(p, t[3])), n))
        compute(g, "sqrt", lambda p: dispatch(p, kernels.sqrt_abs, (W(p, t[5]), R(p, t[4])), n))
        compute(g, "scale", lambda p: dispatch(p, kernels.scale, (W(p, t[6]), R(p, t[5]), 2.0), n))
        compute(g, "sub", lambda p: dispatch(p, kernels.sub, (W(p, out), R(p, t[6]), R(p, x)), n))
    plan = Plan(g, fuse=fuse, **plan_kw)
    return ChainWorkload(n, x, y, z, out, g, plan, {"x": x_h, "y": y_h, "z": z_h})


# ── independent chains (bench/independent.jl) ───────────────────────────────
@dataclass
class IndependentWorkload:
    n: int
    chains: int
    stages: int
    k: float
    sources: list
    outputs: list
    graph: Graph
    plan: Plan
    inputs: dict

    @property
    def bytes_step(self) -> int:
        """Each stir stage reads and writes n Float32."""
        return 8 * self.n * self.chains * self.stages


def build_independent(dev, n: int = 1 << 20, chains: int = 8, stages: int = 6, k: float = 1.001, seed: int = 6,
                      **plan_kw) -> IndependentWorkload:
    """bench/independent.jl:43-56: `chains` independent chains of `stages`
    stir! passes each, declared interleaved stage by stage (c1 s1, c2 s1, ...),
    every intermediate a transient. The reference's first buffer of a chain is
    a transient nothing writes; here it is a persistent buffer of seeded data,
    and the last is a persistent output, so the result can be checked."""
    src_h = [seeded_uniform(seed, n, -2, 2, c) for c in range(chains)]
    sources = [Buffer(dev, x) for x in src_h]
    outputs = [Buffer(dev, np.float32, n) for _ in range(chains)]
    g = Graph(dev)
    bufs = [[sources[c]] + [Transient.Buffer(g, np.float32, n) for _ in range(stages - 1)] + [outputs[c]]
            for c in range(chains)]
    for s_ in range(stages):
        for c in range(chains):
            compute(g, f"c{c + 1} s{s_ + 1}", lambda p, c=c, s_=s_: dispatch(p, kernels.stir, (
                use(p, bufs[c][s_ + 1], write=True), use(p, bufs[c][s_], read=True), k), n))
    plan = Plan(g, **plan_kw)
    return IndependentWorkload(n, chains, stages, k, sources, outputs, g, plan, {"sources": src_h})


# ── two scatters + histogram + three updates ────────────────────────────────
@dataclass
class ScatterWorkload:
    n: int
    nbins: int
    nupd: int
    bufs: dict
    graph: Graph
    plan: Plan
    inputs: dict
    refs: dict

    @property
    def bytes_scatter(self) -> int:
        """Algorithmic bytes of the two scatters: value + index per element each."""
        return 16 * self.n

    @property
    def bytes_updates(self) -> int:
        """The three updates: 8 + 12 + 16 bytes per element."""
        return 36 * self.nupd

    @property
    def bytes_step(self) -> int:
        return self.bytes_scatter + self.bytes_updates


def build_scatter(dev, n: int = 1 << 24, nbins: int = 1 << 16, nupd: int = 1 << 20, seed: int = 0,
                  rank: int = 0, with_updates_from_host: bool = False, **plan_kw) -> ScatterWorkload:
    """`rank` offsets the seed streams so every GPU of a multi-GPU run has its
    own independent graph and data."""
    s = 10 * rank
    inputs = {
        "va": seeded_uniform(seed, n, 0, 1, s + 0),
        "ia": seeded_integers(seed, n, nbins, s + 1),
        "vb": seeded_uniform(seed, n, 0, 1, s + 2),
        "ib": seeded_integers(seed, n, nbins, s + 3),
        "b": seeded_uniform(seed, nupd, -1, 1, s + 4),
        "c": seeded_uniform(seed, nupd, -1, 1, s + 5),
        "d": seeded_uniform(seed, nupd, -1, 1, s + 6),
    }
    bufs = {k: Buffer(dev, v) for k, v in inputs.items()}
    bufs["acc_a"] = Buffer(dev, np.float32, nbins)
    bufs["acc_b"] = Buffer(dev, np.float32, nbins)
    bufs["hist"] = Buffer(dev, np.int32, nbins)
    B = bufs
    g = Graph(dev)
    refs = {}
    if with_updates_from_host:
        for k in ("va", "ia", "vb", "ib"):
            refs[k] = Update(g, B[k])

    compute(g, "scatter a", lambda p: dispatch(p, kernels.scatter_add, (
        use(p, B["acc_a"], write=True), use(p, B["hist"], write=True),
        use(p, B["va"], read=True), use(p, B["ia"], read=True), nbins, 0), n))
    compute(g, "scatter b", lambda p: dispatch(p, kernels.scatter_add, (
        use(p, B["acc_b"], write=True), None,
        use(p, B["vb"], read=True), use(p, B["ib"], read=True), nbins, 0), n))
    compute(g, "update 1", lambda p: dispatch(p, kernels.touch1, (use(p, B["b"], read=True, write=True),), nupd))
    compute(g, "update 2", lambda p: dispatch(p, kernels.touch2, (
        use(p, B["b"], read=True, write=True), use(p, B["c"], read=True)), nupd))
    compute(g, "update 3", lambda p: dispatch(p, kernels.touch3, (
        use(p, B["b"], read=True, write=True), use(p, B["c"], read=True), use(p, B["d"], read=True)), nupd))
    plan = Plan(g, **plan_kw)
    return ScatterWorkload(n, nbins, nupd, bufs, g, plan, inputs, refs)


# ── batched FFT, forward then inverse ───────────────────────────────────────
@dataclass
class FftWorkload:
    batch: int
    n: int
    x: Buffer
    spectrum: Buffer
    back: Buffer
    graph: Graph
    plan: Plan
    inputs: dict

    @property
    def bytes_step(self) -> int:
        """Read and write 8 B per ComplexF32 point, once per direction."""
        return 2 * 2 * 8 * self.batch * self.n


def seeded_complex(seed: int, shape: tuple, stream: int = 0) -> np.ndarray:
    """ComplexF32, real and imaginary parts uniform[-1, 1] (independent streams)."""
    size = int(np.prod(shape))
    re = seeded_uniform(seed, size, -1, 1, 2 * stream)
    im = seeded_uniform(seed, size, -1, 1, 2 * stream + 1)
    return (re + 1j * im).astype(np.complex64).reshape(shape)


def build_fft(dev, batch: int = 16384, n: int = 4096, seed: int = 2, rank: int = 0, world: int = 1,
              **plan_kw) -> FftWorkload:
    """Two passes: the forward transform of x into the spectrum, then the
    inverse of the spectrum back into x's shape. With world > 1 this rank
    transforms its shard_range of the `batch` transforms (the same input rows
    whatever the world size); `FftWorkload.batch` is the shard's size."""
    lo, hi = shard_range(batch, rank, world)
    x_h = seeded_complex(seed, (batch, n), stream=0)
    if (lo, hi) != (0, batch):
        x_h = np.ascontiguousarray(x_h[lo:hi])
    batch = hi - lo
    x = Buffer(dev, x_h.reshape(-1))
    spectrum = Buffer(dev, np.complex64, batch * n)
    back = Buffer(dev, np.complex64, batch * n)
    g = Graph(dev)
    compute(g, "fft forward", lambda p: dispatch(p, kernels.fft_c2c, (
        use(p, spectrum, write=True), use(p, x, read=True), n, 0), batch))
    compute(g, "fft inverse", lambda p: dispatch(p, kernels.fft_c2c, (
        use(p, back, write=True), use(p, spectrum, read=True), n, 1), batch))
    plan = Plan(g, **plan_kw)
    return FftWorkload(batch, n, x, spectrum, back, g, plan, {"x": x_h})


# ── batched dense GEMM ──────────────────────────────────────────────────────
@dataclass
class GemmWorkload:
    batch: int
    M: int
    N: int
    K: int
    A: Buffer
    B: Buffer
    C: Buffer
    graph: Graph
    plan: Plan
    tensors: dict

    @property
    def flops_step(self) -> int:
        return 2 * self.batch * self.M * self.N * self.K

    def host_operands(self):
        """A and B as bfloat16 bit patterns (uint16) on the host, (batch, M, K) and (batch, K, N)."""
        import torch
        a = self.tensors["A"].view(torch.int16).cpu().numpy().view(np.uint16)
        b = self.tensors["B"].view(torch.int16).cpu().numpy().view(np.uint16)
        return a.reshape(self.batch, self.M, self.K), b.reshape(self.batch, self.K, self.N)


def gemm_operands(batch: int, M: int, N: int, K: int, seed: int = 1, device: str = "cuda"):
    """A, B ~ normal(0, 1)/sqrt(K), rounded to bfloat16, drawn on the device by
    torch's Philox generator (seed `seed`): A first, then B."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    scale = 1.0 / float(np.sqrt(K))
    A = (torch.randn((batch, M, K), generator=g, device=device) * scale).to(torch.bfloat16)
    B = (torch.randn((batch, K, N), generator=g, device=device) * scale).to(torch.bfloat16)
    return A, B


def build_gemm(dev, batch: int = 8, M: int = 8192, N: int = 8192, K: int = 8192, seed: int = 1, rank: int = 0,
               world: int = 1, **plan_kw) -> GemmWorkload:
    """One pass: C[b] = A[b]·B[b] over the batch (bf16 in, fp32 out). With
    world > 1 this rank runs its shard_range of the batch (the same operands
    whatever the world size); `GemmWorkload.batch` is the shard's size."""
    lo, hi = shard_range(batch, rank, world)
    A_t, B_t = gemm_operands(batch, M, N, K, seed=seed, device=f"cuda:{dev.ordinal}")
    if (lo, hi) != (0, batch):
        A_t, B_t = A_t[lo:hi].contiguous(), B_t[lo:hi].contiguous()
    batch = hi - lo
    A = Buffer.wrap(dev, A_t, dtype=np.uint16)
    B = Buffer.wrap(dev, B_t, dtype=np.uint16)
    C = Buffer(dev, np.float32, batch * M * N)
    g = Graph(dev)
    compute(g, "gemm", lambda p: dispatch(p, kernels.gemm_bf16, (
        use(p, C, write=True), use(p, A, read=True), use(p, B, read=True), M, N, K), batch))
    plan = Plan(g, **plan_kw)
    return GemmWorkload(batch, M, N, K, A, B, C, g, plan, {"A": A_t, "B": B_t})


# ── CNN inference ───────────────────────────────────────────────────────────
# (name, kernel, cin, cout, stride): a 7x7 stride-2 stem to 64 channels, then
# four stages of two 3x3 convolutions (64/128/256/512 channels, stride 2 at
# each stage start), every one followed by ReLU; global average pool; 512->1000.
CNN_LAYERS = [("stem", 7, 3, 64, 2),
              ("s1c1", 3, 64, 64, 2), ("s1c2", 3, 64, 64, 1),
              ("s2c1", 3, 64, 128, 2), ("s2c2", 3, 128, 128, 1),
              ("s3c1", 3, 128, 256, 2), ("s3c2", 3, 256, 256, 1),
              ("s4c1", 3, 256, 512, 2), ("s4c2", 3, 512, 512, 1)]
CNN_CLASSES = 1000
STEM_CPAD = 4  # the stem's weights cover 4 input channels (the 4th zero): 8-byte pixels


def cnn_macs_per_image(h: int = 224, w: int = 224) -> int:
    macs = 0
    for _, k, cin, cout, s in CNN_LAYERS:
        p = k // 2
        h, w = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
        macs += h * w * cout * k * k * cin
    return macs + CNN_LAYERS[-1][3] * CNN_CLASSES


@dataclass
class CnnWorkload:
    batch: int
    x: Buffer
    logits: Buffer
    weights: dict
    graph: Graph
    plan: Plan
    tensors: dict

    @property
    def flops_step(self) -> int:
        return 2 * cnn_macs_per_image() * self.batch

    def host_params(self):
        """Input (NCHW) and conv weights (HWIO, channels as stored) as bfloat16
        bits, FC weights as float32, all on the host."""
        import torch
        bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
        x = bits(self.tensors["x"])
        ws = {name: bits(self.tensors[name]) for name, *_ in CNN_LAYERS}
        return x, ws, self.tensors["fc"].cpu().numpy()


def cnn_parameters(seed: int = 3, device: str = "cuda"):
    """He-normal weights (std sqrt(2 / fan_in), fan_in = k*k*Cin) in bfloat16,
    HWIO layout, drawn in layer order from torch's Philox generator seeded
    `seed`; the stem's padding channels are zero. FC weights float32
    (512 x classes, inputs by outputs), drawn last."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = {}
    for name, k, cin, cout, _ in CNN_LAYERS:
        std = float(np.sqrt(2.0 / (k * k * cin)))
        w = torch.randn((k, k, cin, cout), generator=g, device=device) * std
        if name == "stem":
            pad = torch.zeros((k, k, STEM_CPAD, cout), device=device)
            pad[:, :, :cin] = w
            w = pad
        out[name] = w.to(torch.bfloat16).contiguous()
    c = CNN_LAYERS[-1][3]
    out["fc"] = (torch.randn((c, CNN_CLASSES), generator=g, device=device) * float(np.sqrt(2.0 / c))).contiguous()
    return out


def cnn_input(batch_total: int, seed: int = 3, device: str = "cuda"):
    """NCHW bfloat16 input, uniform[0, 1), from a generator seeded seed + 1."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed + 1)
    return torch.rand((batch_total, 3, 224, 224), generator=g, device=device).to(torch.bfloat16)


def build_cnn(dev, batch: int = 256, seed: int = 3, rank: int = 0, world: int = 1, **plan_kw) -> CnnWorkload:
    """The forward pass as one graph: nine conv+ReLU passes over transients
    (aliased by the placer; the stem reads the NCHW input and converts it to
    padded NHWC rows in shared memory; the input of each stride-1 conv is
    stored with its padding columns), then GAP+FC into the logits. With
    world > 1 this rank runs images [rank*batch/world, (rank+1)*batch/world)."""
    import torch
    device = f"cuda:{dev.ordinal}"
    lo, hi = shard_range(batch, rank, world)
    per = hi - lo
    x_all = cnn_input(batch, seed, device)
    x_t = x_all[lo:hi].contiguous()
    del x_all
    params = cnn_parameters(seed, device)
    x = Buffer.wrap(dev, x_t, dtype=np.uint16)
    W = {name: Buffer.wrap(dev, params[name], dtype=np.uint16) for name, *_ in CNN_LAYERS}
    fc = Buffer.wrap(dev, params["fc"], dtype=np.float32)
    logits = Buffer(dev, np.float32, per * CNN_CLASSES)
    g = Graph(dev)
    h = w = 224
    cur, cin, wpad = x, 3, 0
    for i, (name, k, _, cout, s) in enumerate(CNN_LAYERS):
        pad = k // 2
        ho, wo = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
        # ahead of a stride-1 conv, store its padding columns (zeros, written by
        # this conv's epilogue), which lets that conv read every filter tap as
        # one shifted run of stored pixels
        nxt_layer = CNN_LAYERS[i + 1] if i + 1 < len(CNN_LAYERS) else None
        owp = nxt_layer[1] // 2 if nxt_layer is not None and nxt_layer[4] == 1 else 0
        nxt = Transient.Buffer(g, np.uint16, per * ho * (wo + 2 * owp) * cout)
        if i == 0:  # the stem reads the NCHW input itself (converted in shared memory)
            compute(g, name, lambda p, src=cur, dst=nxt, wt=W[name], h=h, w=w, cout=cout, k=k, s=s, pad=pad,
                    owp=owp: dispatch(p, kernels.conv2d_nchw_bf16, (
                        use(p, dst, write=True), use(p, src, read=True), use(p, wt, read=True),
                        h, w, 3, cout, k, s, pad, 1, owp), per))
        else:
            compute(g, name, lambda p, src=cur, dst=nxt, wt=W[name], h=h, w=w, cin=cin, cout=cout, k=k, s=s, pad=pad,
                    wpad=wpad, owp=owp: dispatch(p, kernels.conv2d_bf16, (
                        use(p, dst, write=True), use(p, src, read=True), use(p, wt, read=True),
                        h, w, cin, cout, k, s, pad, 1, wpad, owp), per))
        cur, h, w, cin, wpad = nxt, ho, wo, cout, owp
    compute(g, "gap_fc", lambda p: dispatch(p, kernels.gap_fc, (
        use(p, logits, write=True), use(p, cur, read=True), use(p, fc, read=True), h * w, cin, CNN_CLASSES), per))
    plan = Plan(g, **plan_kw)
    tensors = dict(params)
    tensors["x"] = x_t
    return CnnWorkload(per, x, logits, W, g, plan, tensors)


# ── point clouds and the image chain (bench/two_scatters.jl, bench/chain.jl) ─
RASTER_W, RASTER_H = 1000, 750


def camera(angle: float, w: int = RASTER_W, h: int = RASTER_H) -> np.ndarray:
    """The reference's orbit camera (bench/two_scatters.jl:28-40): proj * view
    as 16 float32, column-major."""
    eye = np.array([3.2 * np.cos(angle), 1.2, 3.2 * np.sin(angle)])
    f = -eye / np.linalg.norm(eye)
    r = np.cross(f, [0.0, 1.0, 0.0])
    r /= np.linalg.norm(r)
    u = np.cross(r, f)
    view = np.array([[r[0], r[1], r[2], -r @ eye], [u[0], u[1], u[2], -u @ eye],
                     [-f[0], -f[1], -f[2], f @ eye], [0, 0, 0, 1.0]])
    tn = np.tan(60.0 * np.pi / 360.0)
    near, far = 0.1, 100.0
    proj = np.array([[1 / ((w / h) * tn), 0, 0, 0], [0, -1 / tn, 0, 0],
                     [0, 0, far / (near - far), near * far / (near - far)], [0, 0, -1, 0]])
    return (proj @ view).astype(np.float32).T.reshape(-1).copy()  # column-major


def point_cloud(seed: int, n: int, stream: int = 0):
    """Positions on a noisy unit sphere, the reference's `cloud` (unit normal
    direction times 1 + 0.05 N(0,1)), and a drift velocity 0.35 N(0,1)."""
    rng = np.random.Generator(np.random.PCG64([seed, stream]))
    d = rng.standard_normal((n, 3)).astype(np.float32)
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    pos = (d * (1.0 + 0.05 * rng.standard_normal((n, 1)))).astype(np.float32)
    vel = (0.35 * rng.standard_normal((n, 3))).astype(np.float32)
    return pos, vel


def tint(pos: np.ndarray) -> np.ndarray:
    """The reference's colour ramp: 0.06 * (0.45 + 0.55 y, 0.55, 1 - 0.35 y, 1)."""
    y = pos[:, 1]
    c = np.stack([0.45 + 0.55 * y, np.full_like(y, 0.55), 1.0 - 0.35 * y, np.ones_like(y)], axis=1)
    return (np.float32(0.06) * c.astype(np.float32)).astype(np.float32)


@dataclass
class RasterWorkload:
    bufs: dict
    graph: Graph
    plan: Plan
    inputs: dict


def build_raster(dev, na: int = 200_000, nb: int = 100_000, seed: int = 0, stages: int = 3, dt: float = 1.0 / 60,
                 angle: float = 0.0, **plan_kw) -> RasterWorkload:
    """bench/two_scatters.jl + bench/chain.jl as one graph: advect both clouds,
    clear the framebuffer, splat cloud A (per-point colour, size 2) and cloud B
    (one colour, per-point sizes 1 + 3 U[0,1)) additively, read the
    framebuffer as BGRA8, unpack it and blur it `stages` times."""
    w, h = RASTER_W, RASTER_H
    pa, va = point_cloud(seed, na, 0)
    pb, vb = point_cloud(seed, nb, 1)
    rng = np.random.Generator(np.random.PCG64([seed, 2]))
    inputs = {"pos_a": pa, "vel_a": va, "col_a": tint(pa), "size_a": np.array([2.0], np.float32),
              "pos_b": pb, "vel_b": vb, "col_b": np.array([[0.10, 0.04, 0.01, 1.0]], np.float32),
              "size_b": (1.0 + 3.0 * rng.random(nb)).astype(np.float32), "mvp": camera(angle)}
    B = {k: Buffer(dev, v.reshape(-1)) for k, v in inputs.items()}
    B["fb"] = Buffer(dev, np.float32, 4 * w * h)
    B["raw"] = Buffer(dev, np.uint8, 4 * w * h)
    B["out"] = Buffer(dev, np.float32, 4 * w * h)
    g = Graph(dev)
    stage = [Transient.Buffer(g, np.float32, 4 * w * h) for _ in range(stages)]

    def advect(p):
        for x, v, n in (("pos_a", "vel_a", na), ("pos_b", "vel_b", nb)):
            dispatch(p, kernels.advect_points, (use(p, B[x], read=True, write=True),
                                                use(p, B[v], read=True, write=True), dt, 1.6), n)
    compute(g, "advect", advect)
    compute(g, "clear", lambda p: dispatch(p, kernels.clear_rgba, (use(p, B["fb"], write=True), 0.02, 0.02, 0.04, 1.0),
                                           w * h))

    def scatters(p):
        fb = use(p, B["fb"], read=True, write=True)
        for s, n, cs, ss in (("a", na, 1, 0), ("b", nb, 0, 1)):
            dispatch(p, kernels.splat_points, (fb, use(p, B["pos_" + s], read=True), use(p, B["col_" + s], read=True),
                                               use(p, B["size_" + s], read=True), use(p, B["mvp"], read=True),
                                               w, h, cs, ss), n)
    compute(g, "scatters", scatters)
    compute(g, "copy", lambda p: dispatch(p, kernels.pack_bgra8, (use(p, B["raw"], write=True),
                                                                  use(p, B["fb"], read=True)), w * h))
    compute(g, "unpack", lambda p: dispatch(p, kernels.unpack_bgra8, (use(p, stage[0], write=True),
                                                                      use(p, B["raw"], read=True), w, h), (w, h)))
    src = stage[0]
    for k in range(stages):
        dst = B["out"] if k == stages - 1 else stage[k + 1]
        compute(g, f"blur {k + 1}", lambda p, s=src, d=dst: dispatch(p, kernels.blur3x3, (
            use(p, d, write=True), use(p, s, read=True), w, h), (w, h)))
        src = dst
    plan = Plan(g, **plan_kw)
    return RasterWorkload(B, g, plan, inputs)


# ── the showcase's compute passes (bench/showcase.jl), headless ─────────────
# The reference fills its g-buffer and shadow map with raster passes (a graphics
# stack this backend does not have). Here a seeded analytic scene — the floor
# plane and spheres standing in for the crystals — is ray-cast on the host into
# the same buffers: packed RGBA8 albedo+roughness, metal+emission, normal, and
# depth in [0, 1] (1 = sky) as the reference's projection writes it.
SC_PARAMS = 80
SC_OFF = dict(vp=0, invvp=16, sunvp=32, eye=48, sun=52, suncol=56, fog=60, emit=61, stexel=62, sbias=63, aoamb=64,
              aodirect=65, aoradius=66, aobias=67, threshold=68, exposure=69, bloom=70, aosharp=71, time=72)


def _look(eye, f, r, u):
    """The reference's view matrix (row-major here): rows r, u, -f with translation."""
    v = np.eye(4)
    v[0, :3], v[1, :3], v[2, :3] = r, u, -f
    v[0, 3], v[1, 3], v[2, 3] = -r @ eye, -u @ eye, f @ eye
    return v


def showcase_camera(t: float, radius: float, height: float, w: int, h: int):
    """camera (bench/showcase.jl:115-127): orbit around (0, 13, 0); Vulkan
    clip (y down, depth 0..1); returns (vp row-major float64, eye)."""
    eye = np.array([radius * np.cos(0.11 * t), height + 4.0 * np.sin(0.17 * t), radius * np.sin(0.11 * t)])
    f = np.array([0.0, 13.0, 0.0]) - eye
    f /= np.linalg.norm(f)
    r = np.cross(f, [0.0, 1.0, 0.0])
    r /= np.linalg.norm(r)
    u = np.cross(r, f)
    tn = np.tan(50.0 * np.pi / 360.0)
    near, far = 0.5, 400.0
    proj = np.zeros((4, 4))
    proj[0, 0], proj[1, 1] = 1.0 / ((w / h) * tn), -1.0 / tn
    proj[2, 2], proj[2, 3], proj[3, 2] = far / (near - far), near * far / (near - far), -1.0
    return proj @ _look(eye, f, r, u), eye


def showcase_sunmatrix(sundir, extent: float, depth: float):
    """sunmatrix (bench/showcase.jl:132-144): orthographic box down the sun."""
    sundir = np.asarray(sundir, np.float64)
    f = -sundir / np.linalg.norm(sundir)
    up = np.array([1.0, 0.0, 0.0]) if abs(f[1]) > 0.95 else np.array([0.0, 1.0, 0.0])
    r = np.cross(f, up)
    r /= np.linalg.norm(r)
    u = np.cross(r, f)
    eye = sundir / np.linalg.norm(sundir) * (0.5 * depth)
    near, far = 1.0, depth
    proj = np.eye(4)
    proj[0, 0], proj[1, 1] = 1.0 / extent, -1.0 / extent
    proj[2, 2], proj[2, 3] = -1.0 / (far - near), -near / (far - near)
    return proj @ _look(eye, f, r, u)


def _colmajor(m):
    return np.asarray(m, np.float32).T.reshape(-1)


def _raycast(origin, dirs, spheres):
    """Nearest hit of rays (n, 3) against the plane y = 0 and spheres (m, 4):
    (t, index) with index -1 for the floor, -2 for a miss. float64, in chunks,
    on the GPU when there is one."""
    import torch
    dv = "cuda" if torch.cuda.is_available() else "cpu"
    sp = torch.as_tensor(np.asarray(spheres, np.float64), device=dv)
    o_all = torch.as_tensor(np.broadcast_to(origin, dirs.shape).copy(), device=dv)
    d_all = torch.as_tensor(dirs, device=dv)
    t_out = np.empty(dirs.shape[0])
    i_out = np.empty(dirs.shape[0], np.int64)
    for a in range(0, dirs.shape[0], 1 << 18):
        o, d = o_all[a:a + (1 << 18)], d_all[a:a + (1 << 18)]
        tf = -o[:, 1] / d[:, 1]
        floor = (d[:, 1] < 0) & (tf > 0)
        t = torch.where(floor, tf, torch.full_like(tf, float("inf")))
        idx = torch.where(floor, torch.full_like(tf, -1, dtype=torch.int64), torch.full_like(tf, -2, dtype=torch.int64))
        oc = o[:, None, :] - sp[None, :, :3]                       # (n, m, 3)
        b = (oc * d[:, None, :]).sum(-1)
        disc = b * b - ((oc * oc).sum(-1) - sp[None, :, 3] ** 2)
        ts = torch.where(disc > 0, -b - torch.sqrt(disc.clamp(min=0)), torch.full_like(b, float("inf")))
        ts = torch.where(ts > 1e-3, ts, torch.full_like(ts, float("inf")))
        tmin, k = ts.min(1)
        better = tmin < t
        t = torch.where(better, tmin, t)
        idx = torch.where(better, k, idx)
        t_out[a:a + len(d)] = t.cpu().numpy()
        i_out[a:a + len(d)] = idx.cpu().numpy()
    return t_out, i_out


@dataclass
class ShowcaseScene:
    w: int
    h: int
    tile: int
    pertile: int
    nsample: int
    shift: int
    P: np.ndarray        # float32[80] scene constants
    alb: np.ndarray      # (h, w) uint32
    mat: np.ndarray
    nrm: np.ndarray
    dep: np.ndarray      # (h, w) float32
    smap: np.ndarray     # (res, res) float32
    home: np.ndarray     # (nlight, 4) light orbit centres and reach (sc_move_lights moves them)
    lcol: np.ndarray     # (nlight, 4) colour and intensity
    centers: np.ndarray  # (ninst, 4) instance bounding spheres; the last nlight stand for the lights
    params: np.ndarray   # (ninst, 4) instance surface parameters
    # for a scene whose g-buffer and shadow map are rasterised in the frame
    # (crystal_scene): the prototype triangle list and the instances' scale and
    # yaw and colour; alb/mat/nrm/dep/smap are then None
    ppos: np.ndarray | None = None   # (V, 4) prototype positions
    pnrm: np.ndarray | None = None   # (V, 4) prototype normals
    sizes: np.ndarray | None = None  # (ninst, 4) scale xyz, yaw
    colors: np.ndarray | None = None  # (ninst, 4) albedo rgb, roughness
    smap_res: int = 0

    @property
    def first(self) -> int:
        return self.centers.shape[0] - self.home.shape[0]

    @property
    def rasterised(self) -> bool:
        return self.ppos is not None


def shard_geometry():
    """The crystal prototype of bench/showcase.jl:47-67: a six-sided base ring
    (radius 1 at y = -1), a narrower ring (0.72 at y = 0.45), an apex and a
    base point; 24 triangles wound counter-clockwise seen from outside, each
    vertex carrying its face normal. Returns (positions, normals), (72, 4)
    float32 each (w = 1 for positions, 0 for normals)."""
    n = 6
    ring = lambda y, r: [np.array([r * np.cos(2 * np.pi * i / n), y, r * np.sin(2 * np.pi * i / n)])  # noqa: E731
                         for i in range(n)]
    bot, top = ring(-1.0, 1.0), ring(0.45, 0.72)
    apex, base = np.array([0.0, 1.0, 0.0]), np.array([0.0, -1.0, 0.0])
    pos, nrm = [], []

    def tri(a, b, c):
        fn = np.cross(b - a, c - a)
        fn /= np.linalg.norm(fn)
        for q in (a, b, c):
            pos.append([*q, 1.0])
            nrm.append([*fn, 0.0])

    for i in range(n):
        j = (i + 1) % n
        tri(bot[i], top[j], bot[j])
        tri(bot[i], top[i], top[j])
        tri(top[i], apex, top[j])
        tri(base, bot[j], bot[i])
    return np.asarray(pos, np.float32), np.asarray(nrm, np.float32)


def crystal_field(rng, n: int, clearing: float = 46.0, nhero: int = 26, nseed: int = 34, spread: float = 24.0,
                  extent: float = 230.0, hmax: float = 13.0, fat: float = 0.30):
    """The instances of bench/showcase.jl:72-110 (crystals): a wide dark floor
    shard, a ring of `nhero` tall crystals around an open plaza, and clustered
    smaller ones beyond it, drawn from `rng` (numpy's PCG64 here, so the
    stream is not the reference's, the distributions are). Returns centers
    (x, y, z, bounding radius), sizes (scale xyz, yaw), colors (rgb,
    roughness), params (metalness, emission, 0, 0), each (n, 4) float32."""
    centers = [[0.0, -0.02, 0.0, 900.0]]
    sizes = [[900.0, 0.02, 900.0, 0.0]]
    colors = [[0.045, 0.047, 0.056, 0.13]]
    params = [[0.30, 0.0, 0.0, 0.0]]

    def one(x, z, hgt, rad):
        centers.append([x, hgt, z, np.sqrt(rad * rad + hgt * hgt) * 1.05])
        sizes.append([rad, hgt, rad, 2 * np.pi * rng.uniform()])
        t = rng.uniform()
        c = ([0.26 + 0.16 * t, 0.32 + 0.14 * t, 0.46 + 0.12 * t] if t < 0.80
             else list(np.array([0.62, 0.44, 0.30]) * (0.7 + 0.5 * rng.uniform())))
        colors.append([*c, 0.08 + 0.42 * rng.uniform() ** 2])
        params.append([0.9 if rng.uniform() < 0.4 else 0.05, 0.0, 0.0, 0.0])

    for _ in range(nhero):
        a = 2 * np.pi * rng.uniform()
        r = clearing + 18 * rng.uniform()
        hgt = 20 + 22 * rng.uniform()
        one(r * np.cos(a), r * np.sin(a), hgt, 0.20 * hgt * (0.7 + 0.5 * rng.uniform()))
    cand = [(extent * (rng.uniform() - 0.5), extent * (rng.uniform() - 0.5)) for _ in range(3 * nseed)]
    seeds = [q for q in cand if np.hypot(*q) > clearing + 12][:nseed]
    while len(centers) < n:
        sx, sz = seeds[rng.integers(0, len(seeds))]
        x = sx + spread * rng.standard_normal()
        z = sz + spread * rng.standard_normal()
        if np.hypot(x, z) < clearing:
            continue
        hgt = 1.5 + hmax * rng.uniform() ** 2.2
        one(x, z, hgt, fat * hgt * (0.55 + 0.9 * rng.uniform()))
    f = lambda a: np.asarray(a, np.float32)  # noqa: E731
    return f(centers), f(sizes), f(colors), f(params)


def showcase_scene(w: int = 1600, h: int = 900, seed: int = 9, smap_res: int = 2048, nlight: int = 44,
                   nspheres: int = 90, ninst: int = 5044, t: float = 3.0) -> ShowcaseScene:
    """A seeded scene at the reference's settings (bench/showcase.jl:28-45,
    647-676): 16-pixel tiles with up to 32 lights, 12 occlusion samples, bloom
    at a quarter of each axis, the sun at normalize(-0.62, 0.22, 0.35)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    vp, eye = showcase_camera(t, 62.0, 14.0, w, h)
    inv = np.linalg.inv(vp)
    sun = np.array([-0.62, 0.22, 0.35])
    sun /= np.linalg.norm(sun)
    extent, sdepth = 150.0, 520.0
    sunvp = showcase_sunmatrix(np.array([-0.62, 0.045, 0.35]), extent, sdepth)
    # spheres: a ring of large ones around a plaza and smaller ones beyond
    ang = rng.uniform(0, 2 * np.pi, nspheres)
    dist = np.where(np.arange(nspheres) < 26, rng.uniform(46, 64, nspheres), rng.uniform(60, 140, nspheres))
    rad = np.where(np.arange(nspheres) < 26, rng.uniform(4, 9, nspheres), rng.uniform(1, 4, nspheres))
    spheres = np.stack([dist * np.cos(ang), rad * rng.uniform(0.3, 1.0, nspheres), dist * np.sin(ang), rad], 1)
    col = rng.uniform(0.2, 0.7, (nspheres, 3))
    rough = rng.uniform(0.08, 0.5, nspheres) ** 2 + 0.04
    metal = np.where(rng.uniform(size=nspheres) < 0.4, 0.9, 0.05)
    emit = np.where(rng.uniform(size=nspheres) < 0.1, rng.uniform(0.3, 1.0, nspheres), 0.0)

    # primary rays through pixel centres
    py, px = np.mgrid[0:h, 0:w].astype(np.float64)
    nx, ny = 2 * (px + 0.5) / w - 1, 2 * (py + 0.5) / h - 1
    pts = np.stack([nx, ny], -1).reshape(-1, 2)
    near = np.c_[pts, np.zeros(len(pts)), np.ones(len(pts))] @ inv.T
    far = np.c_[pts, np.ones(len(pts)), np.ones(len(pts))] @ inv.T
    near, far = near[:, :3] / near[:, 3:], far[:, :3] / far[:, 3:]
    dirs = far - near
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    tt, idx = _raycast(near, dirs, spheres)
    world = near + dirs * np.where(np.isfinite(tt), tt, 0)[:, None]
    clip = np.c_[world, np.ones(len(world))] @ vp.T
    dep = np.where(idx > -2, clip[:, 2] / clip[:, 3], 1.0).astype(np.float32)
    dep = np.where(dep < 1.0, dep, np.float32(1.0)).astype(np.float32)
    n = np.zeros_like(world)
    n[idx == -1] = [0.0, 1.0, 0.0]
    sp = idx >= 0
    n[sp] = (world[sp] - spheres[idx[sp], :3]) / spheres[idx[sp], 3:4]
    q8 = lambda x: np.clip(np.rint(np.asarray(x) * 255.0), 0, 255).astype(np.uint32)  # noqa: E731
    alb_rgb = np.where(sp[:, None], col[np.maximum(idx, 0)], [0.045, 0.047, 0.056])
    alb_r = np.where(sp, rough[np.maximum(idx, 0)], 0.13)
    met = np.where(sp, metal[np.maximum(idx, 0)], 0.30)
    emi = np.where(sp, emit[np.maximum(idx, 0)], 0.0)
    alb = q8(alb_rgb[:, 0]) | q8(alb_rgb[:, 1]) << 8 | q8(alb_rgb[:, 2]) << 16 | q8(alb_r) << 24
    mat = q8(met) | q8(emi) << 8 | np.uint32(255) << 24
    nrm = q8(0.5 * n[:, 0] + 0.5) | q8(0.5 * n[:, 1] + 0.5) << 8 | q8(0.5 * n[:, 2] + 0.5) << 16 | np.uint32(255) << 24

    # the shadow map: depth (the sun's clip z) of the nearest surface per texel
    ty, tx = np.mgrid[0:smap_res, 0:smap_res].astype(np.float64)
    sx, sy = 2 * (tx + 0.5) / smap_res - 1, 2 * (ty + 0.5) / smap_res - 1
    sinv = np.linalg.inv(sunvp)
    spts = np.stack([sx, sy], -1).reshape(-1, 2)
    o = np.c_[spts, np.zeros(len(spts)), np.ones(len(spts))] @ sinv.T
    e = np.c_[spts, np.ones(len(spts)), np.ones(len(spts))] @ sinv.T
    o, e = o[:, :3] / o[:, 3:], e[:, :3] / e[:, 3:]
    sd = e - o
    sl = np.linalg.norm(sd, axis=1, keepdims=True)
    st, sidx = _raycast(o, sd / sl, spheres)
    sw = o + sd / sl * np.where(np.isfinite(st), st, 0)[:, None]
    sz = (np.c_[sw, np.ones(len(sw))] @ sunvp.T)[:, 2]
    smap = np.where(sidx > -2, sz, 1.0).astype(np.float32).reshape(smap_res, smap_res)

    # lights (bench/showcase.jl:659-664) and instances
    a = rng.uniform(0, 2 * np.pi, nlight)
    r = 12 + 62 * rng.uniform(size=nlight)
    home = np.stack([r * np.cos(a), 2 + 17 * rng.uniform(size=nlight) ** 1.6, r * np.sin(a),
                     24 + 22 * rng.uniform(size=nlight)], 1).astype(np.float32)
    hue = 6 * rng.uniform(size=nlight)
    i6, fr = np.floor(hue).astype(int), hue - np.floor(hue)
    tints = np.array([[1, f, 0] if i == 0 else [1 - f, 1, 0] if i == 1 else [0, 1, f] if i == 2 else
                      [0, 1 - f, 1] if i == 3 else [f, 0, 1] if i == 4 else [1, 0, 1 - f] for i, f in zip(i6, fr)])
    lcol = np.c_[0.1 + 0.9 * tints, np.full(nlight, 5.5)].astype(np.float32)
    centers = np.c_[rng.uniform(-230, 230, ninst), rng.uniform(0, 40, ninst), rng.uniform(-230, 230, ninst),
                    rng.uniform(1, 20, ninst)].astype(np.float32)
    params = np.zeros((ninst, 4), np.float32)

    P = np.zeros(SC_PARAMS, np.float32)
    P[0:16], P[16:32], P[32:48] = _colmajor(vp), _colmajor(inv), _colmajor(sunvp)
    P[48:51], P[52:55] = eye, sun
    P[56:60] = [1.0, 0.55, 0.28, 6.5]
    smap_texel = 2 * extent / smap_res
    for k, v in dict(fog=0.0035, emit=9.0, stexel=smap_texel, sbias=0.004, aoamb=2.6, aodirect=0.6, aoradius=4.5,
                     aobias=0.05, threshold=1.6, exposure=0.85, bloom=0.30, aosharp=900.0, time=t).items():
        P[SC_OFF[k]] = v
    return ShowcaseScene(w, h, 16, 32, 12, 4, P, alb.reshape(h, w), mat.reshape(h, w), nrm.reshape(h, w),
                         dep.reshape(h, w), smap, home, lcol, centers, params)


@dataclass
class ShowcaseWorkload:
    scene: ShowcaseScene
    bufs: dict
    graph: Graph
    plan: Plan

    @property
    def nlight(self) -> int:
        return self.scene.home.shape[0]


def crystal_scene(w: int = 1600, h: int = 900, seed: int = 9, smap_res: int = 2048, nshard: int = 5000,
                  nlight: int = 44, t: float = 3.0) -> ShowcaseScene:
    """The showcase's own scene (bench/showcase.jl:620-676): `nshard` crystal
    instances of the 24-triangle prototype plus one small crystal riding on
    each of the `nlight` lights, seen by the orbit camera at time t and the
    sun's orthographic box; settings as showcase_scene. The g-buffer and the
    shadow map are rasterised by the frame itself (build_showcase adds the
    two raster passes), so they are None here."""
    rng = np.random.Generator(np.random.PCG64(seed))
    ppos, pnrm = shard_geometry()
    centers, sizes, colors, params = crystal_field(rng, nshard)
    base = showcase_scene(w=16, h=16, seed=seed, smap_res=16, nlight=nlight, ninst=nshard + nlight, t=t)
    home, lcol = base.home, base.lcol
    lc, ls, lk, lp = [], [], [], []
    for i in range(nlight):  # the sources ride along as instances (bench/showcase.jl:623-629)
        r = 0.4 + 0.7 * rng.uniform()
        lc.append([0.0, 0.0, 0.0, 2 * r])
        ls.append([r, r * 1.6, r, 2 * np.pi * rng.uniform()])
        lk.append([*lcol[i, :3], 0.5])
        lp.append([0.0, 1.0, 0.0, 0.0])
    f = lambda a: np.asarray(a, np.float32)  # noqa: E731
    centers = np.concatenate([centers, f(lc)])
    sizes = np.concatenate([sizes, f(ls)])
    colors = np.concatenate([colors, f(lk)])
    params = np.concatenate([params, f(lp)])
    vp, _ = showcase_camera(t, 62.0, 14.0, w, h)
    P = base.P.copy()
    P[0:16], P[16:32] = _colmajor(vp), _colmajor(np.linalg.inv(vp))
    _, eye = showcase_camera(t, 62.0, 14.0, w, h)
    P[48:51] = eye
    P[SC_OFF["stexel"]] = 2 * 150.0 / smap_res
    return ShowcaseScene(w, h, 16, 32, 12, 4, P, None, None, None, None, None, home, lcol, centers, params,
                         ppos=ppos, pnrm=pnrm, sizes=sizes, colors=colors, smap_res=smap_res)


def build_showcase(dev, scene: ShowcaseScene, **plan_kw) -> ShowcaseWorkload:
    """The showcase's compute passes as one graph, in the reference's order
    (bench/showcase.jl:700-790): clear the two counters, move the lights, cull
    against the camera and the sun, write both draw commands, then tiles, SSAO,
    the AO blur, lighting, bright pass, the separable bloom blur and the
    composite. For a rasterised scene (crystal_scene) the shadow map and the
    g-buffer are drawn by two raster passes after the draw counts, from the
    culled lists, as bench/showcase.jl:727-745 draws them; otherwise they are
    persistent inputs. Either way they are persistent buffers (readable after
    the frame); the tile lists, occlusion, HDR and bloom images are transients,
    placed and aliased by the planner. Scene constants live in the persistent
    buffer `P` (update it per frame)."""
    s = scene
    w, h, tile, pertile, shift = s.w, s.h, s.tile, s.pertile, s.shift
    ntx, nty = -(-w // tile), -(-h // tile)
    aow, aoh = -(-w // 2), -(-h // 2)
    bw, bh = -(-w // shift), -(-h // shift)
    ninst, nlight = s.centers.shape[0], s.home.shape[0]
    res = s.smap_res if s.rasterised else s.smap.shape[0]
    inputs = dict(P=s.P, home=s.home.reshape(-1), lcol=s.lcol.reshape(-1), centers=s.centers.reshape(-1),
                  params=s.params.reshape(-1))
    if s.rasterised:
        inputs.update(ppos=s.ppos.reshape(-1), pnrm=s.pnrm.reshape(-1), sizes=s.sizes.reshape(-1),
                      colors=s.colors.reshape(-1))
    else:
        inputs.update(alb=s.alb.reshape(-1), mat=s.mat.reshape(-1), nrm=s.nrm.reshape(-1), dep=s.dep.reshape(-1),
                      smap=s.smap.reshape(-1))
    B = {k: Buffer(dev, np.ascontiguousarray(v)) for k, v in inputs.items()}
    if s.rasterised:
        for k in ("alb", "mat", "nrm"):
            B[k] = Buffer(dev, np.uint32, w * h)
        B["dep"] = Buffer(dev, np.float32, w * h)
        B["smap"] = Buffer(dev, np.float32, res * res)
    B["lpos"] = Buffer(dev, np.float32, 4 * nlight)
    for k in ("visible", "sunvisible"):
        B[k] = Buffer(dev, np.ones(ninst, np.uint32))
    for k in ("counter", "suncounter"):
        B[k] = Buffer(dev, np.zeros(1, np.uint32))
    for k in ("drawcmd", "sundrawcmd"):
        B[k] = Buffer(dev, np.zeros(4, np.uint32))
    B["out"] = Buffer(dev, np.float32, 4 * w * h)
    g = Graph(dev)
    tl = Transient.Buffer(g, np.uint32, ntx * nty * pertile)
    tc = Transient.Buffer(g, np.uint32, ntx * nty)
    aoraw = Transient.Buffer(g, np.float32, 2 * aow * aoh)
    aomap = Transient.Buffer(g, np.float32, aow * aoh)
    hdr = Transient.Buffer(g, np.float32, 4 * w * h)
    bloom_a = Transient.Buffer(g, np.float32, 4 * bw * bh)
    bloom_b = Transient.Buffer(g, np.float32, 4 * bw * bh)
    R = lambda p, b: use(p, b, read=True)  # noqa: E731
    W = lambda p, b: use(p, b, write=True)  # noqa: E731
    RW = lambda p, b: use(p, b, read=True, write=True)  # noqa: E731

    def clear(p):
        dispatch(p, kernels.fill_span, (W(p, B["counter"]), 0, 0.0), 1)
        dispatch(p, kernels.fill_span, (W(p, B["suncounter"]), 0, 0.0), 1)

    def draw_count(p):
        dispatch(p, kernels.sc_write_draw, (W(p, B["drawcmd"]), R(p, B["counter"]), 72), 1)
        dispatch(p, kernels.sc_write_draw, (W(p, B["sundrawcmd"]), R(p, B["suncounter"]), 72), 1)

    compute(g, "clear count", clear)
    compute(g, "lights", lambda p: dispatch(p, kernels.sc_move_lights, (
        W(p, B["lpos"]), RW(p, B["centers"]), RW(p, B["params"]), R(p, B["home"]), R(p, B["lcol"]), R(p, B["P"]),
        ninst - nlight), nlight))
    compute(g, "cull", lambda p: dispatch(p, kernels.sc_cull, (
        W(p, B["visible"]), RW(p, B["counter"]), R(p, B["centers"]), R(p, B["P"]), 0), ninst))
    compute(g, "sun cull", lambda p: dispatch(p, kernels.sc_cull, (
        W(p, B["sunvisible"]), RW(p, B["suncounter"]), R(p, B["centers"]), R(p, B["P"]), 32), ninst))
    compute(g, "draw count", draw_count)
    if s.rasterised:
        nv = s.ppos.shape[0]
        compute(g, "shadow", lambda p: dispatch(p, kernels.raster_instances, (
            W(p, B["smap"]), None, None, None, R(p, B["ppos"]), None, R(p, B["sunvisible"]), R(p, B["suncounter"]),
            R(p, B["centers"]), R(p, B["sizes"]), None, None, R(p, B["P"]), SC_OFF["sunvp"], 1, res, res, nv),
            ninst))
        compute(g, "gbuffer", lambda p: dispatch(p, kernels.raster_instances, (
            W(p, B["dep"]), W(p, B["alb"]), W(p, B["mat"]), W(p, B["nrm"]), R(p, B["ppos"]), R(p, B["pnrm"]),
            R(p, B["visible"]), R(p, B["counter"]), R(p, B["centers"]), R(p, B["sizes"]), R(p, B["colors"]),
            R(p, B["params"]), R(p, B["P"]), SC_OFF["vp"], 0, w, h, nv), ninst))
    compute(g, "tiles", lambda p: dispatch(p, kernels.sc_tile_lights, (
        W(p, tl), W(p, tc), R(p, B["dep"]), R(p, B["lpos"]), R(p, B["P"]), w, h, tile, nlight, pertile),
        (ntx, nty)))
    compute(g, "ssao", lambda p: dispatch(p, kernels.sc_ssao, (
        W(p, aoraw), R(p, B["dep"]), R(p, B["nrm"]), R(p, B["P"]), w, h, s.nsample), (aow, aoh)))
    compute(g, "ao blur", lambda p: dispatch(p, kernels.sc_ao_blur, (W(p, aomap), R(p, aoraw), R(p, B["P"])),
                                             (aow, aoh)))
    compute(g, "light", lambda p: dispatch(p, kernels.sc_shade, (
        W(p, hdr), R(p, B["alb"]), R(p, B["mat"]), R(p, B["nrm"]), R(p, B["dep"]), R(p, B["lpos"]),
        R(p, B["lcol"]), R(p, tl), R(p, tc), R(p, B["smap"]), R(p, aomap), R(p, B["P"]), tile, pertile,
        res), (w, h)))
    compute(g, "bright", lambda p: dispatch(p, kernels.sc_bright, (W(p, bloom_a), R(p, hdr), R(p, B["P"]), w, h,
                                                                   shift), (bw, bh)))
    compute(g, "blur x", lambda p: dispatch(p, kernels.sc_blur, (W(p, bloom_b), R(p, bloom_a), 1, 0), (bw, bh)))
    compute(g, "blur y", lambda p: dispatch(p, kernels.sc_blur, (W(p, bloom_a), R(p, bloom_b), 0, 1), (bw, bh)))
    compute(g, "composite", lambda p: dispatch(p, kernels.sc_composite, (
        W(p, B["out"]), R(p, hdr), R(p, bloom_a), R(p, B["P"]), bw, bh, shift), (w, h)))
    return ShowcaseWorkload(scene, B, g, Plan(g, **plan_kw))
