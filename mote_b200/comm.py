"""Column-sharded Q4_0 linears across GPUs: shard geometry and the exchange.

A linear with N output features (lm_head: N = 128256) is split by weight
rows: rank g owns rows ``[g * shard, g * shard + shard)`` (the last rank's
tail past N is padding), computes ``y_g = x @ W_g^T`` with the single-GPU
kernel, and an all-gather delivers every ``y_g`` to every rank.  Q4_0 rows
are contiguous ``K/32*18``-byte records, so a shard is one contiguous byte
range of the full weight tensor.

The gathered buffer is rank-major ``[G][M][shard]``; :func:`gathered_to_rows`
gives the ``[M, N]`` view (a copy only for M > 1).

Transports (``libmote_cuda.so``): :class:`NcclAllGather` wraps the NCCL
entry points; :class:`PeerAllGather` maps the other ranks' receive buffers
through CUDA IPC and stores into them directly.  Bootstrap (exchanging the
NCCL id or the IPC handles) goes through a caller-supplied ``exchange``
function -- e.g. ``torch.distributed.all_gather_object`` -- so this module
has no process-group dependency of its own.

The reference backend is single-device (crates/mote-backend-hip/src/
context.rs:13-80); this module has no reference counterpart.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, Sequence

from . import errors
from ._native import lib

TILE_ROWS = 16  # the GEMV's row tile: shards stay tile-aligned


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    n: int          # total output features
    rows: int       # padded rows per rank (identical on every rank)
    start: int      # first global row of this rank

    @property
    def stop(self) -> int:
        """One past the last real (non-padding) row of this rank."""
        return min(self.n, self.start + self.rows)

    @property
    def real_rows(self) -> int:
        return max(0, self.stop - self.start)

    def weight_bytes(self, k: int) -> tuple[int, int]:
        """Byte range of this shard's real rows in the full Q4_0 tensor."""
        pitch = (k // 32) * 18
        return self.start * pitch, self.stop * pitch


def shard_rows(n: int, world: int, rank: int, align: int = TILE_ROWS) -> Shard:
    """Equal, ``align``-row shards covering ``n`` rows (the tail is padding)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if n < 0 or align < 1:
        raise ValueError("n must be >= 0 and align >= 1")
    per = -(-n // world)
    rows = -(-per // align) * align
    return Shard(rank=rank, world=world, n=n, rows=rows, start=rank * rows)


def gathered_to_rows(gathered, m: int, shard: Shard):
    """``[G][M][rows]`` (flat or shaped, numpy or torch) -> ``[M, N]``."""
    g = gathered.reshape(shard.world, m, shard.rows)
    full = g.permute(1, 0, 2) if hasattr(g, "permute") else g.transpose(1, 0, 2)
    return full.reshape(m, shard.world * shard.rows)[:, : shard.n]


Exchange = Callable[[object], Sequence[object]]


COMM_TIMEOUT = 10001  # status: NCCL deadline passed, communicator aborted


class NcclAllGather:
    """``ncclAllGather`` of f16 through ``mote_cuda_comm_*``.

    With ``timeout_s`` the communicator is created nonblocking with that
    deadline (``mote_cuda_comm_init_timeout``): if not every rank joins in
    time the init is aborted and :class:`errors.Runtime` raised with status
    ``COMM_TIMEOUT`` instead of blocking the host."""

    def __init__(self, world: int, rank: int, exchange: Exchange,
                 timeout_s: float | None = None):
        uid = ctypes.create_string_buffer(128)
        if rank == 0:
            errors.check(lib().mote_cuda_comm_unique_id(uid), "NCCL unique id")
        ids = exchange(bytes(uid.raw) if rank == 0 else None)
        uid = ctypes.create_string_buffer(bytes(ids[0]), 128)
        self.comm = None
        comm = ctypes.c_void_p()
        if timeout_s is None:
            st = lib().mote_cuda_comm_init(ctypes.byref(comm), world, uid, rank)
        else:
            st = lib().mote_cuda_comm_init_timeout(ctypes.byref(comm), world, uid, rank,
                                                   max(1, int(timeout_s * 1000)))
        errors.check(st, "NCCL init")
        self.comm = comm.value
        self.world, self.rank = world, rank

    def all_gather(self, send_ptr: int, recv_ptr: int, count: int, stream: int) -> None:
        errors.check(lib().mote_cuda_comm_all_gather_f16(self.comm, send_ptr, recv_ptr, count,
                                                         stream), "NCCL all-gather")

    def close(self) -> None:
        if self.comm:
            comm, self.comm = self.comm, None
            errors.check(lib().mote_cuda_comm_destroy(comm), "NCCL destroy")

    def abort(self) -> None:
        """Ends the communicator without a barrier with the other ranks."""
        if self.comm:
            comm, self.comm = self.comm, None
            errors.check(lib().mote_cuda_comm_abort(comm), "NCCL abort")


class PeerBuffers:
    """``buffers`` device buffers of ``nbytes`` on every rank plus one flag
    array (``world + 2`` zeroed words), exported as CUDA IPC handles and
    mapped on every other rank.  ``tables[b]`` is the device array of the
    ranks' pointers to buffer ``b`` and ``flag_table`` that of their flag
    arrays -- the arguments the peer-store kernels take.  Built on every
    rank with the same arguments and this rank's device current."""

    def __init__(self, world: int, rank: int, nbytes: int, exchange: Exchange,
                 buffers: int = 2):
        self.world, self.rank, self.nbytes = world, rank, nbytes
        L = lib()
        self._owned: list[int] = []
        self._opened: list[int] = []

        def alloc(n: int) -> int:
            p = ctypes.c_void_p()
            errors.check(L.mote_cuda_malloc(ctypes.byref(p), max(n, 1)), "allocate")
            self._owned.append(p.value)
            return p.value

        flag_words = world + 2
        self.local = [alloc(nbytes) for _ in range(buffers)]
        self.flags = alloc(flag_words * 4)
        zero = (ctypes.c_uint32 * flag_words)()
        errors.check(L.mote_cuda_memcpy_host_to_device(self.flags, zero, flag_words * 4),
                     "zero flags")

        def handle(ptr: int) -> bytes:
            h = ctypes.create_string_buffer(64)
            errors.check(L.mote_cuda_ipc_get_handle(ptr, h), "IPC handle")
            return bytes(h.raw)

        everyone = exchange([handle(p) for p in self.local] + [handle(self.flags)])

        def peer(r: int, i: int) -> int:
            if r == rank:
                return [*self.local, self.flags][i]
            p = ctypes.c_void_p()
            h = ctypes.create_string_buffer(bytes(everyone[r][i]), 64)
            errors.check(L.mote_cuda_ipc_open_handle(h, ctypes.byref(p)), "open IPC handle")
            self._opened.append(p.value)
            return p.value

        ptrs = [[peer(r, i) for i in range(buffers + 1)] for r in range(world)]

        def table(values: list[int]) -> int:
            host = (ctypes.c_uint64 * world)(*values)
            dev = alloc(8 * world)
            errors.check(L.mote_cuda_memcpy_host_to_device(dev, host, 8 * world), "peer table")
            return dev

        self.tables = [table([ptrs[r][b] for r in range(world)]) for b in range(buffers)]
        self.flag_table = table([ptrs[r][buffers] for r in range(world)])

    def reset_flags(self, stream: int, barrier: Callable[[], None]) -> None:
        """Resynchronises the epochs after a flag wait expired (device status
        bit 1): with no exchange in flight on any rank, every rank zeroes its
        own flag array between two barriers, and the epochs restart
        together."""
        barrier()
        errors.check(lib().mote_cuda_peer_flags_reset(self.flags, self.world, stream),
                     "reset peer flags")
        errors.check(lib().mote_cuda_stream_synchronize(stream), "synchronize")
        barrier()

    def close(self, barrier: Callable[[], None] | None = None) -> None:
        """Unmaps the peers' buffers, waits at ``barrier`` (every rank must
        have unmapped this rank's buffers before they are freed), frees."""
        L = lib()
        for p in self._opened:
            L.mote_cuda_ipc_close_handle(p)
        self._opened = []
        if barrier is not None:
            barrier()
        for p in self._owned:
            L.mote_cuda_free(p)
        self._owned = []


class PeerAllGather(PeerBuffers):
    """All-gather by direct stores into the peers' receive buffers
    (``world * count`` f16 each; alternate the two buffers so a rank never
    overwrites a gather a slower peer is still reading)."""

    def __init__(self, world: int, rank: int, count: int, exchange: Exchange,
                 buffers: int = 2):
        if count % 8:
            raise ValueError("count must be a multiple of 8 (16-byte stores)")
        self.count = count
        super().__init__(world, rank, world * count * 2, exchange, buffers)
        self.recv = self.local

    def all_gather(self, send_ptr: int, buffer: int, stream: int,
                   wait_ns: int | None = None) -> int:
        """Gathers into receive buffer ``buffer``; returns its pointer.  The
        wait for the other ranks is bounded by ``wait_ns`` (default 1 s); on
        expiry the device status records it."""
        if wait_ns is None:
            st = lib().mote_cuda_all_gather_p2p_f16(
                send_ptr, self.tables[buffer], self.flag_table, self.flags, self.count,
                self.rank, self.world, stream)
        else:
            st = lib().mote_cuda_all_gather_p2p_f16_timeout(
                send_ptr, self.tables[buffer], self.flag_table, self.flags, self.count,
                self.rank, self.world, int(wait_ns), stream)
        errors.check(st, "peer all-gather")
        return self.local[buffer]


class ShardedLinearQ4_0(PeerBuffers):
    """Column-sharded Q4_0 linear whose epilogue stores every rank's slice
    into all ranks' full ``[rows, n]`` f16 output buffers (two, alternated)
    and synchronises the ranks at the end of the kernel."""

    def __init__(self, world: int, rank: int, rows: int, n: int, k: int, exchange: Exchange,
                 buffers: int = 2):
        self.shard = shard_rows(n, world, rank)
        self.rows, self.n, self.k = rows, n, k
        super().__init__(world, rank, rows * n * 2, exchange, buffers)
        self.outputs = self.local

    def __call__(self, x_ptr: int, w_shard_ptr: int, buffer: int, stream: int) -> int:
        """``out[buffer] = x @ W^T`` (all columns, on every rank); returns it."""
        errors.check(lib().mote_cuda_quantized_linear_q4_0_f16_allgather(
            x_ptr, w_shard_ptr, self.tables[buffer], self.flag_table, self.flags, self.rows,
            self.shard.rows, self.k, self.n, self.rank, self.world, stream),
            "sharded linear + all-gather")
        return self.local[buffer]
