"""mantle_cuda — Mantle.jl's runtime API, backed by the B200 CUDA shim.

Names follow the reference's API (src/Mantle.jl:34-73, src/runtime/api.jl,
ext/MantleLavaExt.jl), with Julia's `!` dropped:

    import mantle_cuda as M
    dev = M.Device()
    x = M.Buffer(dev, np.ones(n, np.float32))
    g = M.Graph(dev)
    t = M.Transient.Buffer(g, np.float32, n)

    @M.compute(g, "scale")                 # compute!(g, "scale") do p ... end
    def _(p):
        M.dispatch(p, M.kernels.scaleby, (M.use(p, t, write=True),
                                          M.use(p, x, read=True), 2.0), n)

    plan = M.Plan(g)                       # Plan(g; coalesce, alias, profile, policy)
    M.run(plan)                            # run!(plan; barriers = :derived)

Ranges passed to `use(..., range=...)` and `Update(..., range=...)` are Julia's
`first:last` — a (first, last) tuple, 1-based and inclusive — or a Python
`range` object (0-based, half-open), converted once at the boundary.

Every call checks the status the library returns and raises `ArgumentError`
for mistakes in the call (the reference's ArgumentError) and `MantleError` for
everything else. Nothing here falls back to a CPU path.
"""
from __future__ import annotations

import ctypes as C
import math
import threading
from collections import deque
from dataclasses import dataclass
from typing import Any, Callable, Sequence

import numpy as np

from . import _lib as L
from ._lib import ArgumentError, MantleError, check, lib

__all__ = [
    "Device", "Buffer", "Scalar", "Graph", "Transient", "compute", "custom", "use", "dispatch",
    "copy", "Update", "Plan", "run", "timings", "peakbytes", "naivebytes", "storage", "update",
    "backend", "kernels", "PassTiming", "NSAMPLES", "Overlap", "Compact", "ArgumentError",
    "MantleError", "Storage", "CopySrc", "CopyDst", "Indirect", "Unordered", "transitions", "Comm",
    "needs_transition", "reads", "writes", "npipelines", "Array",
]

NSAMPLES = 120  # src/runtime/api.jl:246


# ── policies (src/phases.jl:41-58) ──────────────────────────────────────────
class Policy:
    code = L.POLICY_OVERLAP


class Overlap(Policy):
    """Prefer declaration order and leave lifetimes long (RPS's default)."""
    code = L.POLICY_OVERLAP


class Compact(Policy):
    """Prefer passes that free more bytes than they allocate."""
    code = L.POLICY_COMPACT


# ── usages (src/sync/usage.jl) ───────────────────────────────────────────────
def Storage(read: bool = False, write: bool = False, image: bool = False) -> int:
    return L.U_STORAGE | (L.U_READ if read else 0) | (L.U_WRITE if write else 0) | (L.U_IMAGE if image else 0)


CopySrc = L.U_COPY_SRC
CopyDst = L.U_COPY_DST
Indirect = L.U_INDIRECT
Uniform = L.U_UNIFORM
Sampled = L.U_SAMPLED
Undefined = L.U_UNDEFINED


def Unordered(u: int) -> int:
    return u | L.U_UNORDERED


def reads(u: int) -> bool:
    return bool(lib().mtl_usage_reads(u))


def writes(u: int) -> bool:
    return bool(lib().mtl_usage_writes(u))


def needs_transition(before: int, after: int, kind: int = L.KIND_BUFFER, backend: int = L.BACKEND_CUDA) -> bool:
    return bool(lib().mtl_needs_transition(backend, kind, before, after))


@dataclass(frozen=True)
class TransitionT:
    """Transition(resource, from, waits, to), src/sync/transition.jl:16-21."""
    resource: int
    from_: int
    waits: tuple
    to: int


def _transitions_from(buf, n) -> list[TransitionT]:
    return [TransitionT(t.resource, t.from_, tuple(t.waits[: t.nwaits]), t.to) for t in buf[:n]]


def transitions(usages: Sequence[int], kind: int = L.KIND_BUFFER, initial: int = 0,
                backend: int = L.BACKEND_CUDA) -> list[TransitionT]:
    """transitions(backend, kind, usages; initial), src/sync/transition.jl:103-111."""
    arr = (C.c_uint32 * max(len(usages), 1))(*usages)
    cap = len(usages) + 1
    out = (L.Transition * cap)()
    n = C.c_int32()
    check(lib().mtl_transitions(backend, kind, arr, len(usages), initial, out, cap, C.byref(n)))
    return _transitions_from(out, n.value)


# ── device ──────────────────────────────────────────────────────────────────
class Device:
    """Mantle.Device(): one CUDA device and its stream (ext/MantleLavaExt.jl:16-25)."""

    def __init__(self, ordinal: int = 0, pool_cap: int = 0):
        h = C.c_void_p()
        check(lib().mtl_device_open(ordinal, pool_cap, C.byref(h)))
        self.handle = h
        self.ordinal = ordinal
        sm, l2, hbm, ma, mi = C.c_int32(), C.c_int64(), C.c_int64(), C.c_int32(), C.c_int32()
        check(lib().mtl_device_info(h, C.byref(sm), C.byref(l2), C.byref(hbm), C.byref(ma), C.byref(mi)))
        self.sm_count, self.l2_bytes, self.hbm_bytes = sm.value, l2.value, hbm.value
        self.compute_capability = (ma.value, mi.value)

    @property
    def stream(self) -> int:
        s = C.c_void_p()
        check(lib().mtl_device_stream(self.handle, C.byref(s)))
        return s.value or 0

    def synchronize(self) -> None:
        check(lib().mtl_device_synchronize(self.handle))

    def close(self) -> None:
        if self.handle:
            check(lib().mtl_device_close(self.handle))
            self.handle = None


def backend(dev: Device) -> int:
    """The stream kernels launched outside a graph go on (src/runtime/api.jl:37-49)."""
    return dev.stream


# ── persistent buffers ──────────────────────────────────────────────────────
_DTYPES = {np.dtype(np.float32), np.dtype(np.int32), np.dtype(np.uint32), np.dtype(np.uint8),
           np.dtype(np.float64), np.dtype(np.int64), np.dtype(np.uint16), np.dtype(np.float16),
           np.dtype(np.complex64)}


class Buffer:
    """A persistent buffer, owned by its handle and never freed by hand.

    Buffer(dev, data; capacity) and Buffer(dev, T, n), ext/MantleLavaExt.jl:77-88.
    Length and capacity are separate so a count that changes never reallocates.
    """

    def __init__(self, dev: Device, data_or_dtype: Any, n: int | None = None, *, capacity: int | None = None):
        self.dev = dev
        if n is None:
            data = np.ascontiguousarray(data_or_dtype)
            self.dtype = data.dtype
            self.n = data.shape[0] if data.ndim else 1
            self.shape = data.shape
        else:
            self.dtype = np.dtype(data_or_dtype)
            self.n = int(n)
            self.shape = (self.n,)
            data = None
        if self.dtype not in _DTYPES and self.dtype.kind != "V":
            raise ArgumentError(L.ERR_ARGUMENT, f"Buffer: unsupported element type {self.dtype}")
        self.elems = int(np.prod(self.shape)) if self.shape else 1
        self.capacity = max(int(capacity or self.elems), self.elems)
        self.nbytes = self.capacity * self.dtype.itemsize
        h = C.c_void_p()
        check(lib().mtl_buffer_alloc(dev.handle, self.nbytes, C.byref(h)))
        self.handle = h
        p = C.c_void_p()
        check(lib().mtl_buffer_device_ptr(h, C.byref(p)))
        self.ptr = p.value or 0
        if data is not None:
            self.update(data)

    def __len__(self) -> int:
        return self.n

    @classmethod
    def wrap(cls, dev: Device, owner, dtype=None, n: int | None = None) -> "Buffer":
        """A persistent buffer over device memory someone else owns (a torch
        tensor or any object with __cuda_array_interface__); `owner` is kept
        alive as long as the buffer. dtype/n default to the owner's.

        The library runs on its own stream, which is not ordered after the
        owner's: wrapping a torch tensor synchronises its device, so writes
        still pending on torch's streams land before any plan reads it. Later
        writes through the owner need the same care (or the library's stream)."""
        if hasattr(owner, "data_ptr"):
            import torch
            if owner.is_cuda:
                torch.cuda.synchronize(owner.device)
            ptr, nbytes = owner.data_ptr(), owner.numel() * owner.element_size()
            dt = np.dtype(dtype) if dtype is not None else np.dtype(str(owner.dtype).replace("torch.", ""))
        else:
            cai = owner.__cuda_array_interface__
            ptr = cai["data"][0]
            dt = np.dtype(dtype) if dtype is not None else np.dtype(cai["typestr"])
            nbytes = int(np.prod(cai["shape"])) * np.dtype(cai["typestr"]).itemsize
        self = cls.__new__(cls)
        self.dev = dev
        self.dtype = dt
        self.n = int(n) if n is not None else nbytes // dt.itemsize
        self.shape = (self.n,)
        self.elems = self.n
        self.capacity = self.n
        self.nbytes = nbytes
        h = C.c_void_p()
        check(lib().mtl_buffer_wrap(dev.handle, C.c_void_p(ptr), nbytes, C.byref(h)))
        self.handle = h
        self.ptr = ptr
        self._owner = owner
        return self

    @property
    def stride(self) -> int:
        return 1

    def update(self, data, range: tuple[int, int] | None = None) -> "Buffer":
        """update!(buf, r, data), ext/MantleLavaExt.jl:103-112 (synchronous)."""
        arr = np.ascontiguousarray(data, dtype=self.dtype)
        first = 1 if range is None else _first_last(range)[0]
        off = (first - 1) * self.dtype.itemsize
        if off + arr.nbytes > self.nbytes:
            raise ArgumentError(L.ERR_ARGUMENT, f"update!: {arr.size} elements at {first} exceed capacity {self.capacity}")
        check(lib().mtl_buffer_upload(self.handle, arr.ctypes.data_as(C.c_void_p), off, arr.nbytes))
        return self

    def array(self) -> np.ndarray:
        """Array(buf), ext/MantleLavaExt.jl:122 (synchronises)."""
        out = np.empty(self.shape, dtype=self.dtype)
        check(lib().mtl_buffer_download(self.handle, out.ctypes.data_as(C.c_void_p), 0, out.nbytes))
        return out

    @property
    def __cuda_array_interface__(self):
        return {"shape": self.shape, "typestr": self.dtype.str, "data": (self.ptr, False), "version": 3}

    def release(self) -> None:
        if getattr(self, "handle", None):
            lib().mtl_buffer_release(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class Scalar(Buffer):
    """One value shared by every element (stride 0), ext/MantleLavaExt.jl:90-96."""

    def __init__(self, dev: Device, x, dtype=np.float32):
        super().__init__(dev, np.array([x], dtype=dtype))

    @property
    def stride(self) -> int:
        return 0


def update(buf: Buffer, data, range=None) -> Buffer:
    return buf.update(data, range)


def Array(x) -> np.ndarray:
    return x.array()


# ── graph recording ─────────────────────────────────────────────────────────
def _first_last(r) -> tuple[int, int]:
    if isinstance(r, range):
        if r.step != 1:
            raise ArgumentError(L.ERR_ARGUMENT, "use(): ranges must be contiguous")
        return r.start + 1, r.stop
    a, b = r
    return int(a), int(b)


class TransientBuffer:
    """Transient.Buffer(g, T, n): storage is the plan's (ext/MantleLavaExt.jl:388-392)."""

    def __init__(self, g: "Graph", dtype, n: int):
        self.graph = g
        self.dtype = np.dtype(dtype)
        self.n = int(n)
        rid = C.c_int32()
        check(lib().mtl_graph_transient(g.handle, self.n, self.dtype.itemsize, C.byref(rid)))
        self.rid = rid.value
        self.index = len(g.transients)
        g.transients.append(self)

    def __len__(self) -> int:
        return self.n

    def __repr__(self) -> str:
        return f"Transient.Buffer({self.dtype}, {self.n})"


class Transient:
    Buffer = TransientBuffer


class Graph:
    """Graph(dev): passes recorded once, compiled by Plan, replayed by run."""

    def __init__(self, dev: Device | None = None):
        self.dev = dev
        h = C.c_void_p()
        check(lib().mtl_graph_create(dev.handle if dev else None, C.byref(h)))
        self.handle = h
        self.transients: list[TransientBuffer] = []
        self.passes: list[PassHandle] = []
        self.updates: list[UpdateRef] = []
        self._persistent: dict[int, int] = {}
        self._keep: list[Any] = []  # buffers and callbacks the graph must keep alive

    def rid(self, x) -> int:
        if isinstance(x, UseHandle):
            return x.resource_rid
        if isinstance(x, TransientBuffer):
            if x.graph is not self:
                raise ArgumentError(L.ERR_ARGUMENT, "transient belongs to another graph")
            return x.rid
        if isinstance(x, Buffer):
            key = id(x)
            if key not in self._persistent:
                rid = C.c_int32()
                check(lib().mtl_graph_persistent(self.handle, x.handle, x.capacity, x.dtype.itemsize, C.byref(rid)))
                self._persistent[key] = rid.value
                self._keep.append(x)
            return self._persistent[key]
        if isinstance(x, VirtualBuffer):
            key = id(x)
            if key not in self._persistent:
                rid = C.c_int32()
                check(lib().mtl_graph_persistent(self.handle, None, x.n, x.dtype.itemsize, C.byref(rid)))
                self._persistent[key] = rid.value
                self._keep.append(x)
            return self._persistent[key]
        raise ArgumentError(L.ERR_ARGUMENT, f"not a resource of this graph: {x!r}")

    def resource(self, rid: int) -> dict:
        k, parent, first, last, elems = C.c_int32(), C.c_int32(), C.c_int64(), C.c_int64(), C.c_uint64()
        check(lib().mtl_graph_resource(self.handle, rid, C.byref(k), C.byref(parent), C.byref(first),
                                       C.byref(last), C.byref(elems)))
        return {"kind": k.value, "parent": parent.value, "first": first.value, "last": last.value,
                "elems": elems.value}

    def normal_id(self, rid: int):
        """(parent, range) for a slice, (rid, None) otherwise — what a resource means."""
        r = self.resource(rid)
        return (r["parent"], (r["first"], r["last"])) if r["kind"] == 2 else (rid, None)

    def __del__(self):
        try:
            if self.handle:
                lib().mtl_graph_release(self.handle)
                self.handle = None
        except Exception:
            pass


class VirtualBuffer:
    """A persistent buffer without storage, for compiling graphs on a machine
    without a GPU (the phases only)."""

    def __init__(self, dtype, n: int):
        self.dtype = np.dtype(dtype)
        self.n = int(n)

    def __len__(self) -> int:
        return self.n


@dataclass
class UseHandle:
    """What `use` returns: the binding a kernel argument takes. A slice binds
    its whole buffer; the range only scopes the hazards."""
    resource: Any
    resource_rid: int
    tracked_rid: int


class PassHandle:
    def __init__(self, graph: Graph, index: int, name: str, kind: int):
        self.graph = graph
        self.index = index
        self.name = name
        self.kind = kind
        self.ndispatch = 0


def _pass(g: Graph, name: str, kind: int) -> PassHandle:
    idx = C.c_int32()
    check(lib().mtl_graph_pass(g.handle, name.encode(), kind, C.byref(idx)))
    p = PassHandle(g, idx.value, name, kind)
    g.passes.append(p)
    return p


class _PassCtx:
    def __init__(self, g, name, kind):
        self.g, self.name, self.kind = g, name, kind

    def __enter__(self) -> PassHandle:
        self.p = _pass(self.g, self.name, self.kind)
        return self.p

    def __exit__(self, *exc):
        return False

    def __call__(self, body: Callable[[PassHandle], Any]):
        p = _pass(self.g, self.name, self.kind)
        r = body(p)
        if self.kind == L.PASS_CUSTOM:
            _set_custom(p, r)
        return p


def compute(g: Graph, name: str, body: Callable[[PassHandle], Any] | None = None):
    """compute!(f, g, name), ext/MantleLavaExt.jl:744-749.

    `compute(g, name, body)` runs body(p) now; `compute(g, name)` is a decorator
    or a context manager."""
    ctx = _PassCtx(g, name, L.PASS_COMPUTE)
    return ctx(body) if body is not None else ctx


def custom(g: Graph, name: str, body: Callable[[PassHandle], Any] | None = None):
    """custom!(f, g, name), ext/MantleLavaExt.jl:757-766: body(p) declares the
    uses and returns a callable `work(ctx)` that launches whatever it likes on
    `ctx.stream`; `ctx.storage(x)` is the device address of a declared resource.
    The work is captured into the plan's CUDA graph when the plan is built."""
    ctx = _PassCtx(g, name, L.PASS_CUSTOM)
    return ctx(body) if body is not None else ctx


def _set_custom(p: PassHandle, work) -> None:
    if not callable(work):
        check_msg = ("custom!: the block has to return a zero-argument callable — it is what runs "
                     "at record time. Declare the uses, then return the work.")
        raise ArgumentError(L.ERR_ARGUMENT, check_msg)

    g = p.graph

    def trampoline(_user, stream, plan_handle):
        try:
            work(CustomContext(g, stream or 0, plan_handle))
            return 0
        except Exception as e:  # reported as a failed capture
            trampoline.error = e
            return 1

    trampoline.error = None
    cb = L.CUSTOM_FN(trampoline)
    p.graph._keep.extend([cb, work, trampoline])
    p._trampoline = trampoline
    check(lib().mtl_graph_custom(p.graph.handle, p.index, cb, None))


class CustomContext:
    """What a custom! body's work receives: the capture stream, and the storage
    of the resources the pass declared, resolved in the plan being built."""

    def __init__(self, g: Graph, stream: int, plan_handle):
        self.graph, self.stream, self._plan = g, stream, plan_handle

    def storage(self, x) -> "DevicePtr":
        if isinstance(x, UseHandle):
            x = x.resource
        p = C.c_void_p()
        check(lib().mtl_plan_resource_ptr(self._plan, self.graph.rid(x), C.byref(p)))
        n = x.n * x.dtype.itemsize if hasattr(x, "dtype") else 0
        return DevicePtr(p.value or 0, n)


def use(p: PassHandle, x, read: bool = False, write: bool = False, range=None, usage: int | None = None) -> UseHandle:
    """use(p, x; read, write, range), ext/MantleLavaExt.jl:722-730."""
    if usage is None:
        if not (read or write):
            raise ArgumentError(L.ERR_ARGUMENT, "use() needs read, write, or both")
        usage = Storage(read, write)
    g = p.graph
    rid = g.rid(x)
    first, last = (0, 0) if range is None else _first_last(range)
    out = C.c_int32()
    check(lib().mtl_graph_use(g.handle, p.index, rid, usage, first, last, C.byref(out)))
    return UseHandle(x.resource if isinstance(x, UseHandle) else x, rid, out.value)


class Kernel:
    def __init__(self, name: str):
        k = C.c_int32()
        check(lib().mtl_kernel_lookup(name.encode(), C.byref(k)))
        self.id = k.value
        self.name = name
        nm, sig = C.c_char_p(), C.c_char_p()
        check(lib().mtl_kernel_info(self.id, C.byref(nm), C.byref(sig)))
        self.signature = sig.value.decode()

    def __repr__(self) -> str:
        return f"Kernel({self.name}: {self.signature})"


class _Kernels:
    """The built-in sm_100a kernel families, by name: M.kernels.mix, ..."""

    def __getattr__(self, name: str) -> Kernel:
        if name.startswith("_"):
            raise AttributeError(name)
        k = Kernel(name)
        setattr(self, name, k)
        return k

    def names(self) -> list[str]:
        out = []
        for i in range(lib().mtl_kernel_count()):
            nm, sig = C.c_char_p(), C.c_char_p()
            check(lib().mtl_kernel_info(i, C.byref(nm), C.byref(sig)))
            out.append(nm.value.decode())
        return out


kernels = _Kernels()


def _arg(g: Graph | None, x, sig: str) -> L.Arg:
    a = L.Arg()
    if x is None:
        a.kind = L.ARG_NULL
    elif g is not None and isinstance(x, (UseHandle, TransientBuffer, Buffer, VirtualBuffer)):
        a.kind = L.ARG_RESOURCE
        a.rid = g.rid(x)
    elif isinstance(x, (Buffer,)):
        a.kind = L.ARG_PTR
        a.v.ptr = x.ptr
        a.bytes = x.nbytes
    elif hasattr(x, "data_ptr") and hasattr(x, "element_size"):  # a torch tensor
        a.kind = L.ARG_PTR
        a.v.ptr = x.data_ptr()
        a.bytes = x.numel() * x.element_size()
    elif isinstance(x, DevicePtr):
        a.kind = L.ARG_PTR
        a.v.ptr = x.ptr
        a.bytes = x.nbytes
    elif sig == "f":
        a.kind, a.v.f32 = L.ARG_F32, float(x)
    elif sig == "i":
        a.kind, a.v.i32 = L.ARG_I32, int(x)
    elif sig == "I":
        a.kind, a.v.i64 = L.ARG_I64, int(x)
    elif sig == "d":
        a.kind, a.v.f64 = L.ARG_F64, float(x)
    else:
        raise ArgumentError(L.ERR_ARGUMENT, f"cannot pass {x!r} where the kernel takes '{sig}'")
    return a


@dataclass
class DevicePtr:
    ptr: int
    nbytes: int = 0


def _kernel(kernel) -> Kernel:
    return kernel if isinstance(kernel, Kernel) else Kernel(str(kernel))


def _nd(ndrange) -> tuple[int, ...]:
    return tuple(int(v) for v in ndrange) if isinstance(ndrange, (tuple, list)) else (int(ndrange),)


def dispatch(p: PassHandle, kernel, args: Sequence, ndrange, group=None) -> None:
    """dispatch!(p, kernel, args, ndrange; group), ext/MantleLavaExt.jl:751-752."""
    k = _kernel(kernel)
    if len(args) != len(k.signature):
        raise ArgumentError(L.ERR_ARGUMENT, f"dispatch!: {k.name} takes {len(k.signature)} arguments ({k.signature}), got {len(args)}")
    arr = (L.Arg * max(len(args), 1))(*[_arg(p.graph, x, s) for x, s in zip(args, k.signature)])
    nd = _nd(ndrange)
    nda = (C.c_int64 * 3)(*nd, *([1] * (3 - len(nd))))
    grp = None
    if group is not None:
        gg = _nd(group)
        grp = (C.c_int32 * 3)(*gg, *([0] * (3 - len(gg))))
    check(lib().mtl_graph_dispatch(p.graph.handle, p.index, k.id, arr, len(args), nda, len(nd), grp))
    p.ndispatch += 1


def launch(kernel, args: Sequence, ndrange, stream: int = 0, workspace=None) -> None:
    """Launch a built-in kernel outside any graph on `stream` (pointer args:
    Buffers, torch tensors or DevicePtr)."""
    k = _kernel(kernel)
    arr = (L.Arg * max(len(args), 1))(*[_arg(None, x, s) for x, s in zip(args, k.signature)])
    nd = _nd(ndrange)
    nda = (C.c_int64 * 3)(*nd, *([1] * (3 - len(nd))))
    wptr, wbytes = (0, 0)
    if workspace is not None:
        wa = _arg(None, workspace, "B")
        wptr, wbytes = wa.v.ptr, wa.bytes
    check(lib().mtl_launch(k.id, arr, len(args), nda, len(nd), C.c_void_p(wptr), wbytes, C.c_void_p(stream)))


def workspace_bytes(kernel, args: Sequence, ndrange) -> int:
    k = _kernel(kernel)
    arr = (L.Arg * max(len(args), 1))(*[_arg(None, x, s) for x, s in zip(args, k.signature)])
    nd = _nd(ndrange)
    nda = (C.c_int64 * 3)(*nd, *([1] * (3 - len(nd))))
    out = C.c_uint64()
    check(lib().mtl_kernel_workspace(k.id, arr, len(args), nda, len(nd), C.byref(out)))
    return out.value


def copy(g: Graph, name: str, dst, src) -> PassHandle:
    """copy!(g, name, dst, src), ext/MantleLavaExt.jl:934-943."""
    idx = C.c_int32()
    check(lib().mtl_graph_copy(g.handle, name.encode(), g.rid(dst), g.rid(src), C.byref(idx)))
    p = PassHandle(g, idx.value, name, L.PASS_COPY)
    g.passes.append(p)
    return p


class UpdateRef:
    """What Update returns (ext/MantleLavaExt.jl:776-782). Calling it stores a
    reference — any thread, any moment; nothing is copied until run."""

    def __init__(self, g: Graph, buf, index: int, first: int, last: int):
        self.graph, self.buffer, self.index, self.first, self.last = g, buf, index, first, last
        self._lock = threading.Lock()
        self._pending = None

    def __call__(self, data) -> None:
        with self._lock:
            self._pending = data

    def take(self):
        with self._lock:
            d, self._pending = self._pending, None
            return d


def Update(g: Graph, buf, range=None) -> UpdateRef:
    """Update(g, buf; range), ext/MantleLavaExt.jl:794-802."""
    first, last = (0, 0) if range is None else _first_last(range)
    idx = C.c_int32()
    check(lib().mtl_graph_update(g.handle, g.rid(buf), first, last, C.byref(idx)))
    r = UpdateRef(g, buf, idx.value, first, last)
    g.updates.append(r)
    return r


# ── plans ───────────────────────────────────────────────────────────────────
@dataclass(frozen=True)
class PassTiming:
    """src/runtime/api.jl:186-207."""
    name: str
    kind: str
    host_ms: float
    gpu_ms: float
    samples: int


_KIND = {L.PASS_COMPUTE: "compute", L.PASS_CUSTOM: "custom", L.PASS_UPDATE: "update", L.PASS_COPY: "copy"}
_BARRIERS = {"derived": L.BARRIERS_DERIVED, "backend": L.BARRIERS_BACKEND, "both": L.BARRIERS_BOTH}


class Plan:
    """Plan(g; coalesce, alias, profile, policy), ext/MantleLavaExt.jl:1936-1942."""

    def __init__(self, g: Graph, coalesce: bool = True, alias: bool = True, profile: bool = False,
                 policy: type[Policy] | Policy = Overlap, fuse: bool = False):
        self.graph = g
        self.profile = profile
        code = policy.code
        opts = L.PlanOpts(int(coalesce), int(alias), int(profile), code, int(fuse))
        h = C.c_void_p()
        check(lib().mtl_plan_compile(g.handle, C.byref(opts), C.byref(h)))
        self.handle = h
        self._inflight: deque = deque(maxlen=4)
        n = C.c_int32()
        check(lib().mtl_plan_npasses(h, C.byref(n)))
        order = (C.c_int32 * max(n.value, 1))()
        check(lib().mtl_plan_order(h, order, n.value))
        self.order = list(order[: n.value])

    # The analysis, in scheduled order.
    @property
    def passes(self) -> list[PassHandle]:
        by = {p.index: p for p in self.graph.passes}
        out = []
        for i in self.order:
            if i not in by:  # the shared update pass
                nm = C.c_char_p()
                check(lib().mtl_graph_pass_name(self.graph.handle, i, C.byref(nm)))
                by[i] = PassHandle(self.graph, i, nm.value.decode(), L.PASS_UPDATE)
            out.append(by[i])
        return out

    @property
    def names(self) -> list[str]:
        return [p.name for p in self.passes]

    def pre(self, position: int) -> list[TransitionT]:
        """The transitions the pass at `position` needs before it runs (PassPlan.pre)."""
        cap = 256
        out = (L.Transition * cap)()
        n = C.c_int32()
        check(lib().mtl_plan_transitions(self.handle, position, out, cap, C.byref(n)))
        if n.value > cap:
            out = (L.Transition * n.value)()
            check(lib().mtl_plan_transitions(self.handle, position, out, n.value, C.byref(n)))
        return _transitions_from(out, n.value)

    def edges(self, position: int) -> list[int]:
        """Positions whose completion the pass at `position` waits on (CUDA graph edges)."""
        cap = len(self.order) + 1
        out = (C.c_int32 * cap)()
        n = C.c_int32()
        check(lib().mtl_plan_edges(self.handle, position, out, cap, C.byref(n)))
        return list(out[: n.value])

    def deps(self, pass_index: int) -> list[int]:
        cap = len(self.order) + 1
        out = (C.c_int32 * cap)()
        n = C.c_int32()
        check(lib().mtl_plan_deps(self.handle, pass_index, out, cap, C.byref(n)))
        return list(out[: n.value])

    def offset(self, t: TransientBuffer) -> int:
        o = C.c_int64()
        check(lib().mtl_plan_offset(self.handle, t.index, C.byref(o)))
        return o.value

    def ptr(self, x) -> int:
        p = C.c_void_p()
        check(lib().mtl_plan_resource_ptr(self.handle, self.graph.rid(x), C.byref(p)))
        return p.value or 0

    def nkernels(self, barriers: str = "derived") -> int:
        n = C.c_int32()
        check(lib().mtl_plan_nkernels(self.handle, _BARRIERS[barriers], C.byref(n)))
        return n.value

    def nedges(self, barriers: str = "derived") -> int:
        n = C.c_int32()
        check(lib().mtl_plan_nedges(self.handle, _BARRIERS[barriers], C.byref(n)))
        return n.value

    def set_arg(self, p: PassHandle, dispatch_index: int, arg_index: int, value) -> None:
        """Change a scalar argument of a dispatch (a per-frame value such as dt)."""
        import ctypes
        nm, sig = C.c_char_p(), C.c_char_p()
        a = L.Arg()
        a.kind, a.v.f32 = L.ARG_F32, float(value)
        if isinstance(value, (int, np.integer)) and not isinstance(value, bool):
            a.kind, a.v.i32 = L.ARG_I32, int(value)
        check(lib().mtl_plan_set_arg(self.handle, p.index, dispatch_index, arg_index, ctypes.byref(a)))

    def release(self) -> None:
        if getattr(self, "handle", None):
            lib().mtl_plan_release(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


def run(plan: Plan, barriers: str = "derived") -> None:
    """run!(plan; barriers = :derived | :backend | :both), ext/MantleLavaExt.jl:2076-2128."""
    if barriers not in _BARRIERS:
        raise ArgumentError(L.ERR_ARGUMENT, f"barriers must be :derived, :backend or :both, got {barriers}")
    keep = []
    for ref in plan.graph.updates:
        data = ref.take()
        if data is None:
            continue
        if isinstance(data, Buffer):
            ptr, nbytes, on_dev = data.ptr, data.elems * data.dtype.itemsize, 1
        elif hasattr(data, "data_ptr") and getattr(data, "is_cuda", False):
            ptr, nbytes, on_dev = data.data_ptr(), data.numel() * data.element_size(), 1
        elif hasattr(data, "data_ptr"):  # a host torch tensor
            t = data.contiguous()
            ptr, nbytes, on_dev = t.data_ptr(), t.numel() * t.element_size(), 0
            data = t
        else:
            arr = np.ascontiguousarray(data, dtype=getattr(ref.buffer, "dtype", None))
            ptr, nbytes, on_dev = arr.ctypes.data, arr.nbytes, 0
            data = arr
        keep.append(data)
        check(lib().mtl_plan_update(plan.handle, ref.index, C.c_void_p(ptr), nbytes, on_dev))
    check(lib().mtl_plan_run(plan.handle, _BARRIERS[barriers]))
    plan._inflight.append(keep)


def timings(plan: Plan) -> list[PassTiming]:
    """timings(plan), src/runtime/api.jl:209-241: per pass in scheduled order."""
    n = len(plan.order)
    out = (L.Timing * max(n, 1))()
    cnt = C.c_int32()
    check(lib().mtl_plan_timings(plan.handle, out, n, C.byref(cnt)))
    return [PassTiming(t.name.decode(), _KIND.get(t.kind, "?"), t.host_ms, t.gpu_ms, t.samples)
            for t in out[: cnt.value]]


def peakbytes(plan: Plan) -> int:
    v = C.c_int64()
    check(lib().mtl_plan_peakbytes(plan.handle, C.byref(v)))
    return v.value


def naivebytes(plan: Plan) -> int:
    v = C.c_int64()
    check(lib().mtl_plan_naivebytes(plan.handle, C.byref(v)))
    return v.value


def npipelines(plan: Plan) -> int:
    """Distinct kernel families the plan launches (the analogue of pipelines)."""
    return plan.nkernels()


def storage(x, plan: Plan | None = None) -> int:
    """The device address behind a resource (ext/MantleLavaExt.jl:1190-1194)."""
    if isinstance(x, Buffer):
        return x.ptr
    if isinstance(x, UseHandle):
        x = x.resource
    if plan is None:
        raise ArgumentError(L.ERR_ARGUMENT, "storage(): a transient has storage only inside a plan")
    return plan.ptr(x)


# ── placement (src/memory) ─────────────────────────────────────────────────
@dataclass
class Item:
    """Item(id, live, size; alignment, gaps, offset), src/memory/model.jl:39-49."""
    id: str
    live: tuple[int, int]
    size: int
    alignment: int = 1
    gaps: list = None
    offset: int | None = None


def _items(items: Sequence[Item]):
    arr = (L.ItemT * max(len(items), 1))()
    keep = []
    for i, it in enumerate(items):
        gaps = it.gaps or []
        g = (L.GapT * max(len(gaps), 1))()
        for k, (during, window) in enumerate(gaps):
            g[k].lower, g[k].upper = during
            g[k].window_lower, g[k].window_upper = window if window is not None else (-1, -1)
        idb = str(it.id).encode()
        keep += [g, idb]
        arr[i].lower, arr[i].upper = it.live
        arr[i].size, arr[i].alignment = it.size, it.alignment
        arr[i].offset = -1 if it.offset is None else it.offset
        arr[i].ngaps, arr[i].gaps, arr[i].id = len(gaps), g, idb
    return arr, keep


def place(items: Sequence[Item], strategy: str = "lowest") -> tuple[dict, int]:
    """place(problem, strategy) -> (offsets by id, height), src/memory/placement.jl:46-76."""
    arr, keep = _items(items)
    offs = (C.c_int64 * max(len(items), 1))()
    h = C.c_int64()
    check(lib().mtl_place(arr, len(items), L.BEST_FIT if strategy == "best" else L.LOWEST_FIT, offs, C.byref(h)))
    return {it.id: offs[i] for i, it in enumerate(items)}, h.value


def maxload(items: Sequence[Item]) -> int:
    arr, keep = _items(items)
    v = C.c_int64()
    check(lib().mtl_maxload(arr, len(items), C.byref(v)))
    return v.value


def kernel_timeouts(reset: bool = False) -> int:
    """How many bounded waits inside the library's kernels ran out on the
    current device (0 in a healthy run); reset clears the count."""
    v = C.c_int64()
    check(lib().mtl_kernel_timeouts(int(reset), C.byref(v)))
    return v.value


def inject_failure(entry_point: str, count: int = 1) -> None:
    """Make the next `count` calls of an entry point fail (host-side fault injection)."""
    check(lib().mtl_inject_failure(entry_point.encode(), count))


def set_wait_limit(ns: int = 0) -> None:
    """The wall-clock limit of the kernels' bounded waits on the current
    device (0 restores the default 2 s; at least 1 ms)."""
    check(lib().mtl_set_wait_limit(int(ns)))


def inject_stall(kernel: str, launches: int = 1) -> None:
    """In the next `launches` launches of `kernel` ("gemm_bf16"), CTA 0's
    producer loads nothing, so that CTA's waits run out (a test of the
    bounded-wait path); 0 clears."""
    check(lib().mtl_inject_stall(kernel.encode(), launches))


class Comm:
    """An NCCL communicator over the GPUs of one node (one per process/GPU),
    for the final all-gather of a sharded run. `unique_id` is NCCL's 128-byte
    id, made by one rank with Comm.unique_id() and shared over any host channel."""

    @staticmethod
    def unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        check(lib().mtl_comm_unique_id(buf))
        return buf.raw

    @staticmethod
    def set_timeout(seconds: float) -> None:
        """How long set-up and each all-gather may wait for the other ranks
        before failing with a timeout (the communicator is then aborted);
        60 s unless set, for the whole process."""
        check(lib().mtl_comm_set_timeout(float(seconds)))

    def __init__(self, dev: Device, nranks: int, rank: int, unique_id: bytes):
        if len(unique_id) != 128:
            raise ArgumentError(L.ERR_ARGUMENT, "Comm: the NCCL unique id is 128 bytes")
        h = C.c_void_p()
        idb = C.create_string_buffer(bytes(unique_id), 128)
        check(lib().mtl_comm_init(dev.handle, nranks, rank, idb, C.byref(h)))
        self.handle, self.dev, self.nranks, self.rank = h, dev, nranks, rank

    def allgather(self, send: Buffer, recv: Buffer, nbytes: int | None = None) -> None:
        """recv = the concatenation of every rank's `send` (nbytes each), on the
        device's stream."""
        nbytes = send.nbytes if nbytes is None else int(nbytes)
        if recv.nbytes < nbytes * self.nranks:
            raise ArgumentError(L.ERR_ARGUMENT, f"allgather: recv holds {recv.nbytes} bytes, needs {nbytes * self.nranks}")
        check(lib().mtl_allgather(self.handle, C.c_void_p(send.ptr), C.c_void_p(recv.ptr), nbytes))

    def release(self) -> None:
        if getattr(self, "handle", None):
            lib().mtl_comm_release(self.handle)
            self.handle = None

    def abort(self) -> None:
        if getattr(self, "handle", None):
            lib().mtl_comm_abort(self.handle)
            self.handle = None
