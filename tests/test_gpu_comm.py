"""Multi-GPU exchange (NCCL and peer stores) for the column-sharded linear.

World size 1 runs on any single GPU (the gather is then a copy, the fused
linear + all-gather equals the plain GEMV bit for bit, and CUDA graphs
replaying the peer kernels check that the device-side epoch advances); the
two-rank test needs two GPUs and runs each rank as a spawned process: both
ranks compute their shard of a Q4_0 linear with the GEMV kernel, gather it
with NCCL and with peer stores and also run the fused linear + all-gather
(on the tcgen05 GEMM for 40 tokens, rank 1 with a ragged 488-row shard);
rank 0 compares the logits with the CPU oracle (reference tolerance abs 0.01
/ rel 0.002 on the f16 outputs) and the two gather transports with each
other (bit-identical).
"""
from __future__ import annotations

import ctypes
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from mote_b200 import comm  # noqa: E402
from mote_b200._native import lib  # noqa: E402


def _one(obj):
    return [obj]


@pytest.fixture(scope="module")
def stream():
    torch.cuda.set_device(0)
    s = torch.cuda.Stream()
    torch.cuda.set_stream(s)
    return s


def test_nccl_world1_is_a_copy(stream):
    g = comm.NcclAllGather(1, 0, _one)
    try:
        send = torch.randn(64, device="cuda").half()
        recv = torch.zeros(64, device="cuda", dtype=torch.float16)
        g.all_gather(send.data_ptr(), recv.data_ptr(), 64, stream.cuda_stream)
        torch.cuda.synchronize()
        assert torch.equal(send, recv)
    finally:
        g.close()


def test_peer_world1_graph_replays(stream):
    g = comm.PeerAllGather(1, 0, 64, _one)
    try:
        send = torch.zeros(64, device="cuda", dtype=torch.float16)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            g.all_gather(send.data_ptr(), 0, stream.cuda_stream)
        recv = torch.empty(0)
        for i in range(3):
            send.copy_(torch.full((64,), float(i + 1), device="cuda").half())
            graph.replay()
            torch.cuda.synchronize()
            recv = torch.frombuffer(bytearray(128), dtype=torch.float16)
            st = lib().mote_cuda_memcpy_device_to_host(recv.data_ptr(), g.recv[0], 128)
            assert st == 0
            assert torch.all(recv == float(i + 1))
        flags = np.zeros(3, np.uint32)
        assert lib().mote_cuda_memcpy_device_to_host(flags.ctypes.data, g.flags, 12) == 0
        assert flags.tolist() == [3, 0, 3]  # published epoch, counter reset, own epoch
        status = ctypes.c_uint(0)
        assert lib().mote_cuda_device_status(ctypes.byref(status), 1) == 0 and status.value == 0
        del graph
    finally:
        g.close()


# 1-16 tokens: the GEMV with the peer epilogue; more (N % 16 == 0): the
# tcgen05 GEMM with the peer epilogue against the plain tcgen05 GEMM
@pytest.mark.parametrize("m,n,k", [(1, 1000, 512), (5, 2048, 2048), (16, 296, 4096),
                                   (40, 1024, 512), (300, 2048, 1024)])
def test_fused_world1_equals_plain_gemv(stream, oracle_lib, m, n, k):
    from tests import _fixtures as fx

    w = torch.from_numpy(fx.q4_0_weights(oracle_lib, n, k, seed=m + n)).cuda()
    x = torch.randn(m, k, device="cuda").half()
    plain = torch.empty(m, n, device="cuda", dtype=torch.float16)
    assert lib().mote_cuda_quantized_linear_q4_0_f16(x.data_ptr(), w.data_ptr(),
                                                     plain.data_ptr(), m, n, k,
                                                     stream.cuda_stream) == 0
    op = comm.ShardedLinearQ4_0(1, 0, m, n, k, _one)
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            op(x.data_ptr(), w.data_ptr(), 1, stream.cuda_stream)
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        got = np.empty(m * n, np.float16)
        assert lib().mote_cuda_memcpy_device_to_host(got.ctypes.data, op.outputs[1], got.nbytes) == 0
        # a shard of 1 covers all rows: same tiles, same split, same sums
        assert np.array_equal(got.reshape(m, n), plain.cpu().numpy())
        status = ctypes.c_uint(0)
        assert lib().mote_cuda_device_status(ctypes.byref(status), 1) == 0 and status.value == 0
        del graph
    finally:
        op.close()


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, m: int, n: int, k: int, out_dir: str):
    import datetime

    import torch
    import torch.distributed as dist

    from mote_b200 import comm as c
    from mote_b200._native import lib as L
    from oracle import ref

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    s = torch.cuda.Stream()
    torch.cuda.set_stream(s)

    def exchange(obj):
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    rng = np.random.default_rng(5)
    w = ref.q4_0_quantize(rng.normal(0, 0.02, (n, k)).astype(np.float32), n, k)
    x = rng.normal(0, 1, (m, k)).astype(np.float16)
    sh = c.shard_rows(n, world, rank)
    lo, hi = sh.weight_bytes(k)
    pitch = (k // 32) * 18
    w_local = np.zeros(sh.rows * pitch, np.uint8)
    w_local[: hi - lo] = w[lo:hi]
    wt = torch.from_numpy(w_local).cuda()
    xt = torch.from_numpy(x).cuda()
    y = torch.empty((m, sh.rows), dtype=torch.float16, device="cuda")
    assert L().mote_cuda_quantized_linear_q4_0_f16(xt.data_ptr(), wt.data_ptr(), y.data_ptr(), m,
                                                   sh.rows, k, s.cuda_stream) == 0
    count = m * sh.rows
    nccl = c.NcclAllGather(world, rank, exchange)
    peer = c.PeerAllGather(world, rank, count, exchange)
    try:
        recv = torch.empty(world * count, dtype=torch.float16, device="cuda")
        nccl.all_gather(y.data_ptr(), recv.data_ptr(), count, s.cuda_stream)
        outs = []
        for b in (0, 1, 0):  # alternate the two buffers, reuse the first
            p = peer.all_gather(y.data_ptr(), b, s.cuda_stream)
            torch.cuda.synchronize()
            host = np.empty(world * count, np.float16)
            assert L().mote_cuda_memcpy_device_to_host(host.ctypes.data, p, host.nbytes) == 0
            outs.append(host)
        torch.cuda.synchronize()
        status = ctypes.c_uint(0)
        assert L().mote_cuda_device_status(ctypes.byref(status), 1) == 0
        nccl_host = recv.cpu().numpy()
        logits = c.gathered_to_rows(nccl_host.astype(np.float32), m, sh)
        fused = c.ShardedLinearQ4_0(world, rank, m, n, k, exchange)
        w_real = torch.from_numpy(np.ascontiguousarray(w[lo:hi])).cuda()
        fused_out = []
        for b in (0, 1, 0):
            ptr = fused(xt.data_ptr(), w_real.data_ptr(), b, s.cuda_stream)
            torch.cuda.synchronize()
            host = np.empty(m * n, np.float16)
            assert L().mote_cuda_memcpy_device_to_host(host.ctypes.data, ptr, host.nbytes) == 0
            fused_out.append(host.reshape(m, n).astype(np.float32))
        assert L().mote_cuda_device_status(ctypes.byref(status), 1) == 0
        if rank == 0:
            want = ref.quantized_linear_f32(x.astype(np.float32), w, ref.Q4_0, m, n, k).reshape(m, n)
            want = want.astype(np.float16).astype(np.float32)
            tol = np.maximum(0.01, 0.002 * np.abs(want))
            np.save(os.path.join(out_dir, "result.npy"), np.array([
                float(np.all(np.abs(logits - want) <= tol)
                      and all(np.all(np.abs(f - want) <= tol) for f in fused_out)),
                float(all(np.array_equal(o, nccl_host) for o in outs)),
                float(status.value == 0)]))
        dist.barrier()
        fused.close(barrier=lambda: dist.barrier())
    finally:
        peer.close(barrier=lambda: dist.barrier())
        nccl.close()
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("m", [1, 4, 40])
def test_two_rank_sharded_linear(tmp_path, m):
    import torch.multiprocessing as mp

    mp.start_processes(_rank_main, args=(2, _port(), m, 1000, 512, str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    ok_values, same, status_ok = np.load(tmp_path / "result.npy")
    assert ok_values == 1.0 and same == 1.0 and status_ok == 1.0
