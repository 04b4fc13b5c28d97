"""ctypes binding of libmantle_cuda.so (declarations: include/mantle_cuda.h).

The library is built in-tree (mantle.jl_b200/build.py). There is no fallback:
if the shared library is missing or does not export the ABI this module
expects, importing fails with an error that says so.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmantle_cuda.so"

# status codes
OK, ERR_ARGUMENT, ERR_CUDA, ERR_STATE, ERR_OOM, ERR_UNSUPPORTED, ERR_TIMEOUT, ERR_NCCL, ERR_INJECTED = range(9)

# usage codes
U_STORAGE, U_COPY_SRC, U_COPY_DST, U_INDIRECT, U_UNIFORM, U_VERTICES, U_INDICES = 1, 2, 3, 4, 5, 6, 7
U_SAMPLED, U_PRESENT, U_TRACE_READ, U_TRACE_BUILD, U_COLOR, U_DEPTH, U_UNDEFINED = 8, 9, 10, 11, 12, 13, 14
U_READ, U_WRITE, U_STENCIL_READ, U_STENCIL_WRITE = 1 << 5, 1 << 6, 1 << 7, 1 << 8
U_DISCARD, U_IMAGE, U_UNORDERED = 1 << 9, 1 << 10, 1 << 11

KIND_BUFFER, KIND_IMAGE, KIND_ACCEL = 0, 1, 2
BACKEND_CUDA, BACKEND_WEBGPU = 0, 1
PASS_COMPUTE, PASS_CUSTOM, PASS_UPDATE, PASS_COPY = 0, 1, 2, 3
ARG_RESOURCE, ARG_PTR, ARG_F32, ARG_I32, ARG_I64, ARG_F64, ARG_NULL = range(7)
POLICY_OVERLAP, POLICY_COMPACT = 0, 1
BARRIERS_DERIVED, BARRIERS_BACKEND, BARRIERS_BOTH = 0, 1, 2
LOWEST_FIT, BEST_FIT = 0, 1
MAX_WAITS = 16


class ArgValue(C.Union):
    _fields_ = [("f32", C.c_float), ("i32", C.c_int32), ("i64", C.c_int64), ("f64", C.c_double),
                ("ptr", C.c_uint64)]


class Arg(C.Structure):
    _fields_ = [("kind", C.c_int32), ("rid", C.c_int32), ("v", ArgValue), ("bytes", C.c_uint64)]


class Transition(C.Structure):
    _fields_ = [("resource", C.c_int32), ("from_", C.c_uint32), ("to", C.c_uint32),
                ("nwaits", C.c_int32), ("waits", C.c_uint32 * MAX_WAITS)]


class GapT(C.Structure):
    _fields_ = [("lower", C.c_int64), ("upper", C.c_int64), ("window_lower", C.c_int64),
                ("window_upper", C.c_int64)]


class ItemT(C.Structure):
    _fields_ = [("lower", C.c_int64), ("upper", C.c_int64), ("size", C.c_int64),
                ("alignment", C.c_int64), ("offset", C.c_int64), ("ngaps", C.c_int32),
                ("gaps", C.POINTER(GapT)), ("id", C.c_char_p)]


class PlanOpts(C.Structure):
    _fields_ = [("coalesce", C.c_int32), ("alias", C.c_int32), ("profile", C.c_int32),
                ("policy", C.c_int32), ("fuse", C.c_int32)]


class Timing(C.Structure):
    _fields_ = [("name", C.c_char * 64), ("kind", C.c_int32), ("samples", C.c_int32),
                ("host_ms", C.c_double), ("gpu_ms", C.c_double)]


CUSTOM_FN = C.CFUNCTYPE(C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p)

P = C.c_void_p
I32, U32, I64, U64 = C.c_int32, C.c_uint32, C.c_int64, C.c_uint64
PI32, PI64, PU64, PP = C.POINTER(I32), C.POINTER(I64), C.POINTER(U64), C.POINTER(P)

# name: (restype, argtypes)
PROTOTYPES = {
    "mtl_last_error": (C.c_char_p, []),
    "mtl_abi_version": (I32, []),
    "mtl_inject_failure": (I32, [C.c_char_p, I32]),
    "mtl_usage_reads": (I32, [U32]),
    "mtl_usage_writes": (I32, [U32]),
    "mtl_usage_discards": (I32, [U32]),
    "mtl_needs_transition": (I32, [I32, I32, U32, U32]),
    "mtl_transitions": (I32, [I32, I32, C.POINTER(U32), I32, U32, C.POINTER(Transition), I32, PI32]),
    "mtl_place": (I32, [C.POINTER(ItemT), I32, I32, PI64, PI64]),
    "mtl_maxload": (I32, [C.POINTER(ItemT), I32, PI64]),
    "mtl_device_open": (I32, [I32, U64, PP]),
    "mtl_device_close": (I32, [P]),
    "mtl_device_synchronize": (I32, [P]),
    "mtl_device_stream": (I32, [P, PP]),
    "mtl_device_info": (I32, [P, PI32, PI64, PI64, PI32, PI32]),
    "mtl_buffer_alloc": (I32, [P, U64, PP]),
    "mtl_buffer_wrap": (I32, [P, P, U64, PP]),
    "mtl_buffer_upload": (I32, [P, P, U64, U64]),
    "mtl_buffer_download": (I32, [P, P, U64, U64]),
    "mtl_buffer_device_ptr": (I32, [P, PP]),
    "mtl_buffer_release": (I32, [P]),
    "mtl_graph_create": (I32, [P, PP]),
    "mtl_graph_release": (I32, [P]),
    "mtl_graph_persistent": (I32, [P, P, U64, U32, PI32]),
    "mtl_graph_transient": (I32, [P, U64, U32, PI32]),
    "mtl_graph_pass": (I32, [P, C.c_char_p, I32, PI32]),
    "mtl_graph_use": (I32, [P, I32, I32, U32, I64, I64, PI32]),
    "mtl_kernel_lookup": (I32, [C.c_char_p, PI32]),
    "mtl_kernel_info": (I32, [I32, C.POINTER(C.c_char_p), C.POINTER(C.c_char_p)]),
    "mtl_kernel_count": (I32, []),
    "mtl_graph_dispatch": (I32, [P, I32, I32, C.POINTER(Arg), I32, PI64, I32, PI32]),
    "mtl_graph_custom": (I32, [P, I32, CUSTOM_FN, P]),
    "mtl_graph_copy": (I32, [P, C.c_char_p, I32, I32, PI32]),
    "mtl_graph_update": (I32, [P, I32, I64, I64, PI32]),
    "mtl_plan_compile": (I32, [P, C.POINTER(PlanOpts), PP]),
    "mtl_plan_release": (I32, [P]),
    "mtl_plan_run": (I32, [P, I32]),
    "mtl_plan_update": (I32, [P, I32, P, U64, I32]),
    "mtl_plan_set_arg": (I32, [P, I32, I32, I32, C.POINTER(Arg)]),
    "mtl_plan_npasses": (I32, [P, PI32]),
    "mtl_plan_order": (I32, [P, PI32, I32]),
    "mtl_plan_transitions": (I32, [P, I32, C.POINTER(Transition), I32, PI32]),
    "mtl_plan_edges": (I32, [P, I32, PI32, I32, PI32]),
    "mtl_plan_deps": (I32, [P, I32, PI32, I32, PI32]),
    "mtl_plan_peakbytes": (I32, [P, PI64]),
    "mtl_plan_naivebytes": (I32, [P, PI64]),
    "mtl_plan_offset": (I32, [P, I32, PI64]),
    "mtl_plan_ntransients": (I32, [P, PI32]),
    "mtl_plan_resource_ptr": (I32, [P, I32, PP]),
    "mtl_plan_nkernels": (I32, [P, I32, PI32]),
    "mtl_plan_nedges": (I32, [P, I32, PI32]),
    "mtl_plan_timings": (I32, [P, C.POINTER(Timing), I32, PI32]),
    "mtl_graph_resource": (I32, [P, I32, PI32, PI32, PI64, PI64, PU64]),
    "mtl_graph_npasses": (I32, [P, PI32]),
    "mtl_graph_pass_name": (I32, [P, I32, C.POINTER(C.c_char_p)]),
    "mtl_kernel_workspace": (I32, [I32, C.POINTER(Arg), I32, PI64, I32, PU64]),
    "mtl_launch": (I32, [I32, C.POINTER(Arg), I32, PI64, I32, P, U64, P]),
    "mtl_scatter_add_noalloc": (I32, [P, P, P, P, I64, I32, I32, P]),
    "mtl_kernel_timeouts": (I32, [I32, C.POINTER(C.c_int64)]),
    "mtl_set_wait_limit": (I32, [C.c_uint64]),
    "mtl_inject_stall": (I32, [C.c_char_p, I32]),
    "mtl_comm_unique_id": (I32, [P]),
    "mtl_comm_init": (I32, [P, I32, I32, P, PP]),
    "mtl_comm_release": (I32, [P]),
    "mtl_comm_abort": (I32, [P]),
    "mtl_allgather": (I32, [P, P, P, U64]),
    "mtl_comm_set_timeout": (I32, [C.c_double]),
}


class MantleError(RuntimeError):
    """An entry point returned a non-zero status; the message is the library's."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class ArgumentError(MantleError, ValueError):
    """The reference's ArgumentError: a mistake in the call, caught before any work."""


_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python mantle.jl_b200/build.py` "
            "(there is no CPU fallback for the CUDA path)")
    h = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | getattr(os, "RTLD_LOCAL", 0))
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(h, name)  # AttributeError = the library lacks an entry point
        fn.restype = res
        fn.argtypes = args
    if h.mtl_abi_version() != 1:
        raise ImportError(f"{LIB_PATH} has ABI {h.mtl_abi_version()}, expected 1")
    _lib = h
    return h


def check(status: int) -> None:
    if status == OK:
        return
    msg = lib().mtl_last_error().decode(errors="replace")
    if status == ERR_ARGUMENT:
        raise ArgumentError(status, msg)
    raise MantleError(status, msg)
