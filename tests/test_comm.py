"""The NCCL communicator of the backend (mtl_comm_init / mtl_allgather /
mtl_comm_abort), on one GPU.

* A one-rank communicator's all-gather is a device copy: checked against the
  host data it was filled from.
* A communicator whose second rank never joins must fail on the host with
  MTL_ERR_TIMEOUT after the set timeout, abort itself, and leave the process
  able to make a working communicator afterwards. Nothing waits on the GPU in
  this case (NCCL's set-up waits for the peer over its host bootstrap), and it
  runs in a child process under a host timeout of its own.
"""
import os
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest

import mantle_cuda as M
from mantle_cuda import _lib as L

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def test_one_rank_allgather_is_a_copy(dev):
    comm = M.Comm(dev, 1, 0, M.Comm.unique_id())
    try:
        data = np.arange(1000, dtype=np.float32) * 0.5 - 7.0
        send = M.Buffer(dev, data)
        recv = M.Buffer(dev, np.float32, 1000)
        comm.allgather(send, recv)
        dev.synchronize()
        assert np.array_equal(recv.array(), data)
        with pytest.raises(M.ArgumentError):
            comm.allgather(send, M.Buffer(dev, np.float32, 999))
    finally:
        comm.release()


def test_missing_rank_times_out_then_a_new_communicator_works():
    script = textwrap.dedent(f"""
        import sys
        sys.path.insert(0, {str(ROOT / "mantle.jl_b200")!r})
        import numpy as np
        import mantle_cuda as M
        from mantle_cuda import _lib as L
        dev = M.Device(0)
        M.Comm.set_timeout(3.0)
        try:
            M.Comm(dev, 2, 0, M.Comm.unique_id())  # rank 1 never joins
            print("joined")
        except M.MantleError as e:
            print("status", e.status, "timeout" if e.status == L.ERR_TIMEOUT else "other", str(e))
        M.Comm.set_timeout(60.0)
        c = M.Comm(dev, 1, 0, M.Comm.unique_id())
        x = M.Buffer(dev, np.arange(16, dtype=np.int32))
        y = M.Buffer(dev, np.int32, 16)
        c.allgather(x, y)
        dev.synchronize()
        print("after", bool(np.array_equal(y.array(), np.arange(16))))
        c.release()
    """)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True, timeout=120, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "timeout" in r.stdout, r.stdout + r.stderr[-2000:]
    assert "after True" in r.stdout, r.stdout


def test_comm_refuses_bad_arguments(dev):
    with pytest.raises(M.ArgumentError):
        M.Comm(dev, 2, 2, M.Comm.unique_id())
    with pytest.raises(M.ArgumentError):
        M.Comm(dev, 1, 0, b"short")
    with pytest.raises(M.ArgumentError):
        M.Comm.set_timeout(0.0)
