"""The C-ABI library loads without a GPU and exports every symbol that
include/mantle_cuda.h declares; host-only entry points answer; calls that need
a device fail with a status, never a crash."""
import ctypes as C
import re
from pathlib import Path

import pytest

import mantle_cuda as M
from mantle_cuda import _lib as L

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(mtl_[a-z0-9_]+)\s*\(", text))
    return names


def test_every_declared_symbol_is_exported():
    lib = C.CDLL(str(L.LIB_PATH))
    missing = [s for s in sorted(declared_symbols()) if not hasattr(lib, s)]
    assert not missing, f"declared in include/ but not exported: {missing}"
    assert len(declared_symbols()) >= 60


def test_prototypes_cover_the_header():
    assert declared_symbols() <= set(L.PROTOTYPES), sorted(declared_symbols() - set(L.PROTOTYPES))


def test_abi_version_and_kernel_table():
    assert L.lib().mtl_abi_version() == 1
    names = M.kernels.names()
    for k in ("mix", "keep", "touch1", "touch2", "touch3", "touch4", "stir", "chain8", "scatter_add"):
        assert k in names
    assert M.kernels.scatter_add.signature == "bbbBii"
    with pytest.raises(M.ArgumentError):
        M.kernels.no_such_kernel


def test_device_calls_fail_with_a_status_without_a_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(M.MantleError):
        M.Device(0)


def test_injected_failure_is_reported_then_cleared():
    M.inject_failure("mtl_graph_create", 1)
    with pytest.raises(M.MantleError) as e:
        M.Graph(None)
    assert e.value.status == L.ERR_INJECTED
    M.Graph(None)  # the injection was one-shot
