"""Host logic of the column-sharded linear (no GPU).

Shard geometry, the rank-major -> [M, N] reassembly, and a world-size-2
``gloo`` run in which each rank computes its shard of a Q4_0 linear with the
CPU oracle and the shards are all-gathered: the reassembled logits must equal
the unsharded oracle result bit for bit (row-sharding never changes a dot
product).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from mote_b200.comm import TILE_ROWS, gathered_to_rows, shard_rows


@pytest.mark.parametrize("n,world", [(128256, 1), (128256, 2), (128256, 4), (128256, 8),
                                     (14336, 8), (1000, 3), (16, 4), (0, 2)])
def test_shards_are_equal_aligned_and_cover_n(n, world):
    shards = [shard_rows(n, world, r) for r in range(world)]
    rows = {s.rows for s in shards}
    assert len(rows) == 1 and shards[0].rows % TILE_ROWS == 0
    covered = [i for s in shards for i in range(s.start, s.stop)]
    assert covered == list(range(n))
    assert shards[-1].start + shards[-1].rows >= n
    if n % (world * TILE_ROWS) == 0:
        assert all(s.real_rows == n // world for s in shards)


def test_lm_head_shard_sizes():
    assert shard_rows(128256, 8, 0).rows == 16032
    assert shard_rows(14336, 8, 7).start == 12544
    k = 4096
    lo, hi = shard_rows(128256, 2, 1).weight_bytes(k)
    assert (lo, hi) == (64128 * 2304, 128256 * 2304)


def test_invalid_ranks():
    with pytest.raises(ValueError):
        shard_rows(100, 2, 2)
    with pytest.raises(ValueError):
        shard_rows(100, 0, 0)


@pytest.mark.parametrize("m", [1, 3])
def test_gathered_to_rows(m):
    n, world = 100, 3
    sh = shard_rows(n, world, 0)
    full = np.arange(m * n, dtype=np.float32).reshape(m, n)
    gathered = np.zeros((world, m, sh.rows), np.float32)
    for r in range(world):
        s = shard_rows(n, world, r)
        gathered[r, :, : s.real_rows] = full[:, s.start:s.stop]
    assert np.array_equal(gathered_to_rows(gathered.reshape(-1), m, sh), full)
    torch = pytest.importorskip("torch")
    assert np.array_equal(gathered_to_rows(torch.from_numpy(gathered), m, sh).numpy(), full)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank: int, world: int, port: int, m: int, n: int, k: int, out_dir: str):
    import torch
    import torch.distributed as dist

    from oracle import ref

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(21)
        w = ref.q4_0_quantize(rng.normal(0, 0.02, (n, k)).astype(np.float32), n, k)
        x = rng.normal(0, 1, (m, k)).astype(np.float16).astype(np.float32)
        sh = shard_rows(n, world, rank)
        lo, hi = sh.weight_bytes(k)
        y = np.zeros((m, sh.rows), np.float32)
        if sh.real_rows:
            y[:, : sh.real_rows] = ref.quantized_linear_f32(
                x, w[lo:hi], ref.Q4_0, m, sh.real_rows, k).reshape(m, sh.real_rows)
        # the bootstrap path the GPU transports use
        ids = [None] * world
        dist.all_gather_object(ids, f"rank{rank}")
        assert ids == [f"rank{r}" for r in range(world)]
        gathered = torch.empty(world * m * sh.rows, dtype=torch.float32)
        dist.all_gather_into_tensor(gathered, torch.from_numpy(y.reshape(-1)))
        logits = gathered_to_rows(gathered, m, sh).numpy()
        if rank == 0:
            full = ref.quantized_linear_f32(x, w, ref.Q4_0, m, n, k).reshape(m, n)
            np.save(os.path.join(out_dir, "ok.npy"), np.array([np.array_equal(logits, full)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("m", [1, 2])
def test_gloo_world2_sharded_linear_matches_unsharded(tmp_path, oracle_lib, m):
    torch = pytest.importorskip("torch")
    import torch.multiprocessing as mp

    n, k, world = 200, 256, 2
    mp.start_processes(_gloo_rank, args=(world, _free_port(), m, n, k, str(tmp_path)),
                       nprocs=world, start_method="spawn", join=True)
    assert bool(np.load(tmp_path / "ok.npy")[0])
