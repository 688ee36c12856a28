"""Failure detection of the multi-GPU exchange, in forms that fault no GPU.

* A bounded device wait that runs out: a world-2 peer all-gather on one GPU
  whose second "rank" is a local buffer standing in for a peer that never
  publishes its epoch.  With a 1 ms limit the kernel gives up, records bit 1
  (wait timeout) in the device status word and returns; the context stays
  usable.  The epochs are then out of step (this rank advanced, the peer
  did not); ``mote_cuda_peer_flags_reset`` zeroes the flag array, and a
  gather whose peer has published (the test writes the peer's epoch, as the
  peer's kernel would) completes with status 0.
* An NCCL communicator whose second rank never joins: rank 0 alone creates
  a world-2 communicator with a 2 s deadline (``mote_cuda_comm_init_timeout``,
  nonblocking NCCL init, polled, then aborted) and gets status 10001 instead
  of blocking its host thread.  It runs in a child process with its own
  limit; nothing is launched on the GPU.
"""
from __future__ import annotations

import ctypes
import subprocess
import sys
import textwrap
import time
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from mote_b200 import comm  # noqa: E402
from mote_b200._native import lib  # noqa: E402

ROOT = Path(__file__).resolve().parents[1]
WAIT_TIMEOUT_BIT = 1
COUNT = 64  # f16 elements per rank


def _status() -> int:
    st = ctypes.c_uint(0)
    assert lib().mote_cuda_device_status(ctypes.byref(st), 1) == 0
    return st.value


def _table(ptrs) -> torch.Tensor:
    return torch.tensor(list(ptrs), dtype=torch.int64, device="cuda")


def _read_u32(ptr: int, n: int) -> list[int]:
    out = np.zeros(n, np.uint32)
    assert lib().mote_cuda_memcpy_device_to_host(out.ctypes.data, ptr, out.nbytes) == 0
    return out.tolist()


def test_peer_wait_expires_and_flags_resync():
    torch.cuda.set_device(0)
    s = torch.cuda.Stream()
    stream = s.cuda_stream
    world = 2
    # this rank's receive buffer and flags, and a stand-in for rank 1's
    recv = [torch.zeros(world * COUNT, dtype=torch.float16, device="cuda") for _ in range(2)]
    flags = [torch.zeros(world + 2, dtype=torch.int32, device="cuda") for _ in range(2)]
    recv_table = _table(t.data_ptr() for t in recv)
    flag_table = _table(t.data_ptr() for t in flags)
    own = flags[0].data_ptr()
    send = torch.arange(COUNT, device="cuda", dtype=torch.float32).half()
    assert _status() == 0

    # rank 1 never publishes: the 1 ms wait runs out
    t0 = time.perf_counter()
    st = lib().mote_cuda_all_gather_p2p_f16_timeout(
        send.data_ptr(), recv_table.data_ptr(), flag_table.data_ptr(), own, COUNT, 0, world,
        1_000_000, stream)
    assert st == 0
    s.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert _status() & WAIT_TIMEOUT_BIT
    assert _status() == 0  # read-and-clear
    # the slice reached both buffers; this rank is at epoch 1, the peer at 0
    for t in recv:
        assert torch.equal(t[:COUNT], send)
    assert _read_u32(own, world + 2) == [1, 0, 0, 1]
    assert _read_u32(flags[1].data_ptr(), world + 2) == [1, 0, 0, 0]

    # the context is still usable: an ordinary launch succeeds
    x = torch.ones(4, device="cuda")
    assert float((x + 1).sum()) == 8.0

    # resync: zero the flag arrays (every rank does its own)
    for f in flags:
        assert lib().mote_cuda_peer_flags_reset(f.data_ptr(), world, stream) == 0
    s.synchronize()
    assert _read_u32(own, world + 2) == [0, 0, 0, 0]

    # the peer publishes epoch 1 (what its gather's last CTA stores), then
    # this rank's gather finds it and completes without a timeout
    flags[0][1] = 1
    torch.cuda.synchronize()
    send2 = send * 2
    st = lib().mote_cuda_all_gather_p2p_f16_timeout(
        send2.data_ptr(), recv_table.data_ptr(), flag_table.data_ptr(), own, COUNT, 0, world,
        1_000_000, stream)
    assert st == 0
    s.synchronize()
    assert _status() == 0
    assert _read_u32(own, world + 2) == [1, 1, 0, 1]
    for t in recv:
        assert torch.equal(t[:COUNT], send2)

    # argument checks of the bounded entry and the reset
    assert lib().mote_cuda_all_gather_p2p_f16_timeout(
        send.data_ptr(), recv_table.data_ptr(), flag_table.data_ptr(), own, COUNT, 0, world, 0,
        stream) == 1
    assert lib().mote_cuda_peer_flags_reset(None, world, stream) == 1


_NEVER_JOINS = textwrap.dedent("""
    import ctypes, sys, time
    sys.path.insert(0, sys.argv[1])
    from mote_b200._native import lib
    assert lib().mote_cuda_set_device(0) == 0
    uid = ctypes.create_string_buffer(128)
    assert lib().mote_cuda_comm_unique_id(uid) == 0
    comm = ctypes.c_void_p(12345)
    t0 = time.perf_counter()
    st = lib().mote_cuda_comm_init_timeout(ctypes.byref(comm), 2, uid, 0, 2000)
    dt = time.perf_counter() - t0
    print(st, comm.value, round(dt, 2), flush=True)
""")


def test_nccl_init_deadline_when_a_rank_never_joins():
    env = {"NCCL_NVLS_ENABLE": "0"}
    import os

    env = {**os.environ, **env}
    proc = subprocess.run([sys.executable, "-c", _NEVER_JOINS, str(ROOT)], capture_output=True,
                          text=True, timeout=120, env=env)
    assert proc.returncode == 0, proc.stderr[-2000:]
    status, handle, seconds = proc.stdout.split()[-3:]
    assert int(status) == comm.COMM_TIMEOUT
    assert handle == "None"
    assert 1.5 <= float(seconds) < 60.0
