"""The C entry points in the order the Julia extension (INTEGRATION.md,
`ext/MantleCUDAExt.jl`) calls them, driven here through raw ctypes with no help
from the Python mirror: Device, Buffer(dev, data), Buffer(dev, T, n), Graph,
Transient.Buffer, compute! + use + dispatch!, custom! (a C callback that
resolves storage() and launches on the capture stream), copy!, Update, Plan
(profiled), run! with a pending update, timings, peakbytes, Array.

The frame: x (updated from the host each frame) -> stir! -> a transient ->
custom! scaleby! x2 -> y -> copy! -> z. Checked against the oracle."""
import ctypes as C

import numpy as np
import pytest

from mantle_cuda import _lib as L
from mantle_cuda.workloads import seeded_uniform
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def ok(st):
    assert st == L.OK, L.lib().mtl_last_error().decode()


def test_julia_binding_sequence_over_the_c_abi():
    lib = L.lib()
    n = 4096
    # Device(Val(:cuda)); backend(dev)
    dev = C.c_void_p()
    ok(lib.mtl_device_open(0, 0, C.byref(dev)))
    stream = C.c_void_p()
    ok(lib.mtl_device_stream(dev, C.byref(stream)))

    def buffer(nbytes, data=None):  # Buffer(dev, T, n) / Buffer(dev, data) + update!
        h = C.c_void_p()
        ok(lib.mtl_buffer_alloc(dev, nbytes, C.byref(h)))
        if data is not None:
            ok(lib.mtl_buffer_upload(h, data.ctypes.data, 0, data.nbytes))
        return h

    x0 = seeded_uniform(20, n, -2, 2, 0)
    x1 = seeded_uniform(20, n, -2, 2, 1)
    x, y, z = buffer(4 * n, x0), buffer(4 * n), buffer(4 * n)

    g = C.c_void_p()  # Graph(dev)
    ok(lib.mtl_graph_create(dev, C.byref(g)))
    t = C.c_int32()  # Transient.Buffer(g, Float32, n)
    ok(lib.mtl_graph_transient(g, n, 4, C.byref(t)))

    def rid(h):  # resourceid(g, buf)
        r = C.c_int32()
        ok(lib.mtl_graph_persistent(g, h, n, 4, C.byref(r)))
        return r.value

    rx, ry, rz = rid(x), rid(y), rid(z)

    def newpass(name, kind):
        p = C.c_int32()
        ok(lib.mtl_graph_pass(g, name, kind, C.byref(p)))
        return p.value

    def use(p, r, usage):
        out = C.c_int32()
        ok(lib.mtl_graph_use(g, p, r, L.U_STORAGE | usage, 0, 0, C.byref(out)))

    def lookup(name):  # family(kernel): nameof(stir!) -> "stir"
        k = C.c_int32()
        ok(lib.mtl_kernel_lookup(name, C.byref(k)))
        return k.value

    # compute!(g, "stir") do p; dispatch!(p, stir!, (use(t; write), use(x; read), 1.001f0), n)
    p1 = newpass(b"stir", L.PASS_COMPUTE)
    use(p1, t.value, L.U_WRITE)
    use(p1, rx, L.U_READ)
    args = (L.Arg * 3)()
    args[0].kind, args[0].rid = L.ARG_RESOURCE, t.value
    args[1].kind, args[1].rid = L.ARG_RESOURCE, rx
    args[2].kind = L.ARG_F32
    args[2].v.f32 = 1.001
    nd = (C.c_int64 * 1)(n)
    ok(lib.mtl_graph_dispatch(g, p1, lookup(b"stir"), args, 3, nd, 1, None))

    # custom!(g, "scale") do p; use(t; read); use(y; write); () -> scaleby! on the capture stream
    p2 = newpass(b"scale", L.PASS_CUSTOM)
    use(p2, t.value, L.U_READ)
    use(p2, ry, L.U_WRITE)
    scaleby = lookup(b"scaleby")
    calls = []

    def body(_user, cap_stream, plan):
        def storage(r):
            ptr = C.c_void_p()
            if lib.mtl_plan_resource_ptr(plan, r, C.byref(ptr)) != L.OK:
                return None
            return ptr.value

        dst, src = storage(ry), storage(t.value)
        if not dst or not src:
            return 1
        la = (L.Arg * 3)()
        la[0].kind, la[0].v.ptr, la[0].bytes = L.ARG_PTR, dst, 4 * n
        la[1].kind, la[1].v.ptr, la[1].bytes = L.ARG_PTR, src, 4 * n
        la[2].kind = L.ARG_F32
        la[2].v.f32 = 2.0
        calls.append(1)
        return lib.mtl_launch(scaleby, la, 3, (C.c_int64 * 1)(n), 1, None, 0, cap_stream)

    cb = L.CUSTOM_FN(body)
    ok(lib.mtl_graph_custom(g, p2, cb, None))

    # copy!(g, "copy", z, y)
    p3 = C.c_int32()
    ok(lib.mtl_graph_copy(g, b"copy", rz, ry, C.byref(p3)))

    # ref = Update(g, x)
    u = C.c_int32()
    ok(lib.mtl_graph_update(g, rx, 0, 0, C.byref(u)))

    # Plan(g; profile = true)
    opts = L.PlanOpts(1, 1, 1, L.POLICY_OVERLAP, 0)
    plan = C.c_void_p()
    ok(lib.mtl_plan_compile(g, C.byref(opts), C.byref(plan)))
    assert calls == [1]  # the custom! work ran once, at instantiation

    host = np.empty(n, np.float32)
    for frame, data in enumerate((x0, x1, x1)):
        # ref(data); run!(plan): mtl_plan_update for the pending data, then the replay
        if frame > 0:
            ok(lib.mtl_plan_update(plan, u.value, data.ctypes.data, data.nbytes, 0))
        ok(lib.mtl_plan_run(plan, L.BARRIERS_DERIVED))
        ok(lib.mtl_buffer_download(z, host.ctypes.data, 0, host.nbytes))  # Array(z)
        want = O.stir(data, 1.001) * np.float32(2.0)
        np.testing.assert_allclose(host, want, rtol=1e-6, atol=1e-6)

    # timings(plan)
    npass = C.c_int32()
    ok(lib.mtl_plan_npasses(plan, C.byref(npass)))
    tim = (L.Timing * npass.value)()
    got = C.c_int32()
    ok(lib.mtl_plan_timings(plan, tim, npass.value, C.byref(got)))
    names = [tim[i].name.decode() for i in range(got.value)]
    assert {"stir", "scale", "copy"} <= set(names)
    # peakbytes(plan): the one transient
    peak = C.c_int64()
    ok(lib.mtl_plan_peakbytes(plan, C.byref(peak)))
    assert peak.value >= 4 * n

    # finalizers, in any order
    ok(lib.mtl_graph_release(g))
    ok(lib.mtl_plan_release(plan))
    for h in (x, y, z):
        ok(lib.mtl_buffer_release(h))
    ok(lib.mtl_device_close(dev))
