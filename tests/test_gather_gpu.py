"""The row-sharded matmul with its all-gather fused over peer memory
(rce_qmm_mm_batched_device_multi_gather + rce_qmm_peer_unpack), on two GPUs:
one process per GPU, gloo only to exchange the peer buffers' IPC handles.
Every rank's gathered output must equal, bit for bit, the concatenation of
each shard's own matmul (same shapes, same kernels); a second matmul reading
the first's gathered output, the tensor-core GEMM route (20 tokens: the bulk
mode, plain values and one release flag per peer,
rce_qmm_mm_batched_device_multi_gather_bulk + rce_qmm_peer_unpack_bulk), and
a second round through the same buffers (new epochs), likewise; and two
shards sharing x gathered from one grouped
launch (rce_qmm_mm_batched_device_multi_gather) against each rank's grouped
device call, at 1, 3 and 20 tokens.  Skipped with fewer than two GPUs.
On one GPU: an unpack whose words never arrive ends its bounded wait with
the timeout in the context's error word, and the context stays usable."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist

    import oracle as O
    import rce_b200 as R
    from rce_b200 import synth
    from rce_b200.shard import PeerGroup, row_shards, torch_exchange

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    res = {}
    pg = None
    try:
        torch.cuda.set_device(rank)
        ctx = R.Context(rank)
        dt = O.GGUF_Q4_K
        n1, n2, k = 1024, 512, 2048
        w1 = synth.weights(dt, n1, k, np.random.default_rng(1))
        w2 = synth.weights(dt, n2, n1, np.random.default_rng(2))

        def shards(wb, n, kk):
            rb = kk // 256 * 144
            return [(r0, R.QuantWeight.from_owned_bytes(wb[r0 * rb:r1 * rb], dt, r1 - r0, kk, ctx=ctx))
                    for r0, r1 in row_shards(n, world)]

        s1, s2 = shards(w1, n1, k), shards(w2, n2, n1)
        pg = PeerGroup(ctx, world, rank, torch_exchange())
        for t_rows, tag in ((3, "gemv"), (20, "gemm")):
            pg.output(f"y1{tag}", t_rows, n1)
            pg.output(f"y2{tag}", t_rows, n2)
            ok = []
            for rnd in range(2):  # the second round reuses the buffers with new epochs
                x = torch.from_numpy(synth.activations(t_rows, k, np.random.default_rng(3 + t_rows + rnd))).cuda()
                pg.mm(x, s1[rank][1], f"y1{tag}", s1[rank][0])
                y1 = pg.gather(f"y1{tag}")
                pg.mm(y1, s2[rank][1], f"y2{tag}", s2[rank][0])
                y2 = pg.gather(f"y2{tag}")
                torch.cuda.synchronize()
                got1, got2 = y1.cpu().numpy(), y2.cpu().numpy()
                want1 = torch.cat([R.mm_batched_device(x, w) for _, w in s1], dim=1)
                want2 = torch.cat([R.mm_batched_device(want1, w) for _, w in s2], dim=1)
                torch.cuda.synchronize()
                ok.append(bool(np.array_equal(got1, want1.cpu().numpy())) and
                          bool(np.array_equal(got2, want2.cpu().numpy())))
                dist.barrier()  # a peer may not overwrite y2's words before this rank has read them
            res[tag] = tuple(ok)
        # grouped: two shards sharing x in one launch (q/k/v-style), two rounds
        w3 = synth.weights(dt, 512, k, np.random.default_rng(7))
        s3 = shards(w3, 512, k)
        okg = []
        for t_rows in (1, 3, 20):
            pg.output(f"ga{t_rows}", t_rows, n1)
            pg.output(f"gb{t_rows}", t_rows, 512)
            for rnd in range(2):
                x = torch.from_numpy(synth.activations(t_rows, k, np.random.default_rng(50 + t_rows + rnd))).cuda()
                pg.mm_multi(x, [s1[rank][1], s3[rank][1]], [f"ga{t_rows}", f"gb{t_rows}"], [s1[rank][0], s3[rank][0]])
                ya, yb = pg.gather(f"ga{t_rows}"), pg.gather(f"gb{t_rows}")
                torch.cuda.synchronize()
                got_a, got_b = ya.cpu().numpy(), yb.cpu().numpy()
                per = [R.mm_multi_device(x, [s1[r][1], s3[r][1]]) for r in range(world)]
                want_a = torch.cat([p_[0] for p_ in per], dim=1).cpu().numpy()
                want_b = torch.cat([p_[1] for p_ in per], dim=1).cpu().numpy()
                okg.append(bool(np.array_equal(got_a, want_a)) and bool(np.array_equal(got_b, want_b)))
                dist.barrier()
        res["group"] = tuple(okg)
        res["device_error"] = ctx.device_error()
        dist.barrier()
    except Exception as e:  # reported to the parent, never a hang
        res["error"] = repr(e)
    finally:
        if pg is not None:
            try:
                dist.barrier()
            except Exception:
                pass
            pg.close()
        dist.destroy_process_group()
    q.put((rank, res))


def test_fused_gather_two_gpus():
    import multiprocessing as mp

    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert "error" not in res[r], res[r]
        assert res[r]["gemv"] == (True, True), res
        assert res[r]["gemm"] == (True, True), res
        assert res[r]["group"] == (True,) * 6, res
        assert res[r]["device_error"] == 0


def test_unpack_wait_expires_and_is_reported(ctx):
    # Failure detection without a GPU fault: a receive buffer that no peer
    # ever writes (one GPU, nothing else running).  The unpack kernel's
    # bounded wait runs out after about a second, records the timeout in the
    # context's error word and returns; the context stays usable.
    import ctypes
    import time

    import torch

    import oracle as O
    import rce_b200 as R
    import refcases
    from rce_b200 import _lib

    L = _lib.lib()
    t_rows, n, own0, own1 = 2, 64, 0, 32
    ll = torch.zeros((t_rows, n), dtype=torch.int64, device="cuda:0")  # every word at epoch 0
    y = torch.zeros((t_rows, n), device="cuda:0")
    stream = torch.cuda.current_stream()
    assert ctx.device_error() == 0
    t0 = time.time()
    rc = L.rce_qmm_peer_unpack(ctx.handle, ctypes.c_void_p(ll.data_ptr()), ctypes.c_void_p(y.data_ptr()), n, t_rows,
                               n, own0, own1, 7, None, ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, L.rce_qmm_last_error()
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert ctx.device_error() == 1  # kKernelErrWaitTimeout, cleared by the read
    assert 0.5 < waited < 30, waited
    assert torch.count_nonzero(y) == 0  # nothing copied for the words that never arrived
    # the context and the device still work
    n2, k2 = 256, 1024
    w, _, _, _, x = refcases.seeded_case(O.GGUF_Q4_K, n2, k2, 1, 3)
    qw = R.QuantWeight.from_owned_bytes(w, O.GGUF_Q4_K, n2, k2, ctx=ctx)
    got = R.mm_batched(x, 1, qw)
    want = O.mm_batched(x, 1, w, O.GGUF_Q4_K, n2, k2)
    assert float(np.abs(got - want).max() / np.abs(want).max()) <= 1e-3
    assert ctx.device_error() == 0
