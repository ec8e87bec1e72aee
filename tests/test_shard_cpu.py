"""Row sharding's host logic on CPU: the shard boundaries, and that gathering
every rank's shard of a matmul (two gloo ranks, the oracle as each rank's
matmul) reproduces the unsharded result bit for bit -- rows are independent,
as the reference's rayon row split assumes (rce-op-qmm/src/lib.rs:502, 654,
742)."""
import os
import socket

import numpy as np
import pytest

import oracle as O
from rce_b200.shard import TILE_ROWS, row_shards


@pytest.mark.parametrize("n,world", [(4096, 2), (14336, 8), (1024, 4), (700, 3), (16, 2), (48, 8)])
def test_row_shards_cover_in_tiles(n, world):
    sh = row_shards(n, world)
    assert sh[0][0] == 0 and sh[-1][1] == n
    for (a0, a1), (b0, b1) in zip(sh, sh[1:]):
        assert a1 == b0
    for a0, a1 in sh:
        assert a0 % TILE_ROWS == 0 and a0 <= a1
    sizes = [a1 - a0 for a0, a1 in sh]
    assert max(sizes) - min(sizes) <= TILE_ROWS or n < TILE_ROWS * world


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    import torch.distributed as dist

    from rce_b200.shard import torch_exchange

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, k = 700, 512
        from rce_b200 import synth
        w = synth.weights(O.GGUF_Q4_K, n, k, np.random.default_rng(5))
        x = synth.activations(3, k, np.random.default_rng(6))
        row_bytes = k // 256 * 144
        r0, r1 = row_shards(n, world)[rank]
        mine = O.mm_batched(x, 3, w[r0 * row_bytes:r1 * row_bytes], O.GGUF_Q4_K, r1 - r0, k)
        parts = torch_exchange()(mine)
        full = np.concatenate(parts, axis=1)
        want = O.mm_batched(x, 3, w, O.GGUF_Q4_K, n, k)
        q.put((rank, bool(np.array_equal(full, want))))
    finally:
        dist.destroy_process_group()


def test_gathered_shards_equal_the_whole_on_two_gloo_ranks():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
