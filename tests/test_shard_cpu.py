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


# ---- PeerGroup's protocol bookkeeping over host memory, two gloo ranks ------
#
# HostTransport stands in for librce_qmm.so's peer entry points: receive
# buffers are host shared-memory segments laid out as the kernels lay them out
# ({value, epoch} words at [t][ldy] + row, epoch in the high 32 bits; bulk
# values at the same places and slot `rank` of the u32 flags at flag_off), and
# each rank's matmul is a float matrix product.  PeerGroup's own logic --
# epochs (absolute, and relative to a device counter advanced by begin_step),
# this rank's own range, flag offsets, the alternation of the two bulk
# buffers -- runs unchanged.

class _Ctx:
    handle = None
    device = 0
    prefill_min_tokens = 16


class HostTransport:
    def __init__(self):
        self.mem = {}       # address -> (SharedMemory, uint8 view)
        self.tensors = {}   # data_ptr -> torch tensor (outputs, counters, inputs)
        self.weights = {}   # handle -> float32 [rows, k]
        self.owned = []

    # memory
    def _register(self, shm):
        view = np.ndarray((shm.size,), dtype=np.uint8, buffer=shm.buf)
        addr = view.ctypes.data
        self.mem[addr] = (shm, view)
        return addr

    def rce_qmm_peer_alloc(self, ctx, nbytes, ptr_ref, handle_buf):
        from multiprocessing import shared_memory

        shm = shared_memory.SharedMemory(create=True, size=max(int(nbytes), 8))
        shm.buf[:] = b"\0" * shm.size
        self.owned.append(shm)
        ptr_ref._obj.value = self._register(shm)
        name = shm.name.encode()
        ctypes_buf = handle_buf
        ctypes_buf.raw = name + b"\0" * (64 - len(name))
        return 0

    def rce_qmm_peer_open(self, ctx, handle_buf, ptr_ref):
        from multiprocessing import shared_memory

        shm = shared_memory.SharedMemory(name=handle_buf.raw.rstrip(b"\0").decode())
        ptr_ref._obj.value = self._register(shm)
        return 0

    def rce_qmm_peer_close(self, ctx, p):
        return 0

    def rce_qmm_peer_free(self, ctx, p):
        return 0

    def zeros(self, shape, dtype, device):
        import torch

        t = torch.zeros(shape, dtype=dtype)
        self.tensors[t.data_ptr()] = t
        return t

    def stream(self, stream, device):
        return None

    def _view(self, addr, dtype):
        return self.mem[int(addr)][1].view(dtype)

    def _epoch(self, rel, base):
        return (int(rel) + (int(self.tensors[base.value][0]) if base is not None and base.value else 0)) & 0xFFFFFFFF

    def rce_qmm_peer_epoch_advance(self, ctx, base, delta, s):
        self.tensors[base.value][0] += int(delta)
        return 0

    # the gathered matmul: rows to the own output and to every peer
    def _mm(self, x_ptr, t_rows, hs, n, world, rank, offs, ys, lds):
        x = self.tensors[int(x_ptr.value)][:t_rows].numpy()
        for i in range(n):
            yv = x @ self.weights[hs[i]].T
            y = self.tensors[ys[i]]
            y[:t_rows, offs[i]:offs[i] + yv.shape[1]] = torch_from(yv)
            yield i, yv

    def rce_qmm_mm_batched_device_multi_gather(self, ctx, x, ldx, t_rows, hs, n, world, rank, offs, ys, lds, lls,
                                               epoch, base, s):
        e = self._epoch(epoch, base)
        for i, yv in self._mm(x, t_rows, hs, n, world, rank, offs, ys, lds):
            words = (np.uint64(e) << np.uint64(32)) | yv.astype(np.float32).view(np.uint32).astype(np.uint64)
            for r in range(world):
                if r != rank:
                    ll = self._view(lls[i * world + r], np.uint64).reshape(-1, lds[i])
                    ll[:t_rows, offs[i]:offs[i] + yv.shape[1]] = words
        return 0

    def rce_qmm_mm_batched_device_multi_gather_bulk(self, ctx, x, ldx, t_rows, hs, n, world, rank, offs, ys, lds,
                                                    bufs, flag_offs, epoch, base, s):
        e = self._epoch(epoch, base)
        for i, yv in self._mm(x, t_rows, hs, n, world, rank, offs, ys, lds):
            for r in range(world):
                if r != rank:
                    b = self._view(bufs[i * world + r], np.uint8)
                    vals = b[:flag_offs[i]].view(np.float32)[:t_rows * lds[i]].reshape(t_rows, lds[i])
                    vals[:, offs[i]:offs[i] + yv.shape[1]] = yv
                    b[flag_offs[i]:flag_offs[i] + 64].view(np.uint32)[rank] = e
        return 0

    @staticmethod
    def _wait(cond, what):
        import time

        t0 = time.time()
        while not cond():
            if time.time() - t0 > 30:
                raise TimeoutError(what)
            time.sleep(0.001)

    def rce_qmm_peer_unpack(self, ctx, ll_ptr, y_ptr, ldy, t_rows, n, own0, own1, epoch, base, s):
        e = self._epoch(epoch, base)
        ll = self._view(ll_ptr.value, np.uint64).reshape(-1, ldy)[:t_rows, :n]
        others = np.ones(n, bool)
        others[own0:own1] = False

        def arrived():
            ep = (ll[:, others] >> np.uint64(32)).astype(np.int64)
            return bool(np.all(((ep - e) & 0xFFFFFFFF) < (1 << 31)))  # this epoch or a later one

        self._wait(arrived, f"words of epoch {e}")
        y = self.tensors[y_ptr.value]
        y[:t_rows, :n][:, torch_from(others)] = torch_from((ll[:, others] & np.uint64(0xFFFFFFFF))
                                                           .astype(np.uint32).view(np.float32))
        return 0

    def rce_qmm_peer_unpack_bulk(self, ctx, buf_ptr, flag_off, y_ptr, ldy, t_rows, n, own0, own1, world, rank,
                                 epoch, base, s):
        e = self._epoch(epoch, base)
        b = self._view(buf_ptr.value, np.uint8)
        flags = b[flag_off:flag_off + 64].view(np.uint32)
        peers = [r for r in range(world) if r != rank]
        self._wait(lambda: all(((int(flags[r]) - e) & 0xFFFFFFFF) < (1 << 31) for r in peers),
                   f"flags of epoch {e}")
        if any(int(flags[r]) != e for r in peers):
            raise RuntimeError("bulk buffer overrun")  # the kernel reports kKernelErrOverrun
        vals = b[:flag_off].view(np.float32)[:t_rows * ldy].reshape(t_rows, ldy)
        y = self.tensors[y_ptr.value]
        keep = np.ones(n, bool)
        keep[own0:own1] = False
        y[:t_rows, :n][:, torch_from(keep)] = torch_from(vals[:, :n][:, keep].copy())
        return 0

    def close(self):
        for shm in self.owned:
            shm.close()
            shm.unlink()


def torch_from(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a))


def _peer_rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from rce_b200.qmm import QuantWeight
    from rce_b200.shard import PeerGroup, torch_exchange

    class HostWeight(QuantWeight):
        def close(self):
            pass

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    tr = HostTransport()
    try:
        rng = np.random.default_rng(30)
        k = 32
        full = {"a": rng.standard_normal((64, k)).astype(np.float32),   # word-mode output (3 tokens)
                "b": rng.standard_normal((48, k)).astype(np.float32)}   # bulk-mode output (20 tokens)
        pg = PeerGroup(_Ctx(), world, rank, torch_exchange(), transport=tr)
        pg.output("a", 3, 64)
        pg.output("b", 20, 48)
        shards = {}
        for h, (name, W) in enumerate(full.items()):
            r0, r1 = row_shards(W.shape[0], world)[rank]
            tr.weights[h + 1] = W[r0:r1]
            shards[name] = (HostWeight(h + 1, O.GGUF_Q4_K, r1 - r0, k, _Ctx()), r0)
        bad = []

        def expect(cond, what):
            if not cond:
                bad.append(what)

        def x_of(t, seed):
            x = torch.from_numpy(np.random.default_rng(seed).standard_normal((t, k)).astype(np.float32))
            tr.tensors[x.data_ptr()] = x
            return x

        def check_out(name, x, what):
            got = pg.view(name).numpy()[:x.shape[0]]
            expect(np.allclose(got, x.numpy() @ full[name].T, rtol=1e-5, atol=1e-5), what)

        # absolute epochs, calls gathered one by one
        for it in range(3):
            xa, xb = x_of(3, 100 + it), x_of(20, 200 + it)
            w, r0 = shards["a"]
            pg.mm(xa, w, "a", r0)
            pg.gather("a")
            check_out("a", xa, f"word-mode output, call {it}")
            w, r0 = shards["b"]
            pg.mm(xb, w, "b", r0)
            o = pg.outputs["b"]
            expect(o.bulk_mode and o.bulk_sel == it % 2, f"bulk buffers alternate, call {it}")
            pg.gather("b")
            check_out("b", xb, f"bulk-mode output, call {it}")
        # steps: epochs relative to the counter begin_step advances
        for it in range(3):
            xa, xb = x_of(3, 300 + it), x_of(20, 400 + it)
            pg.begin_step(2)
            ea = pg.mm(xa, shards["a"][0], "a", shards["a"][1])
            eb = pg.mm(xb, shards["b"][0], "b", shards["b"][1])
            expect((ea, eb) == (1, 2), f"relative epochs {ea, eb}")
            pg.gather("a")
            pg.gather("b")
            pg.end_step()
            check_out("a", xa, f"word-mode output, step {it}")
            check_out("b", xb, f"bulk-mode output, step {it}")
            # the counter continues above the 6 absolute epochs of the calls
            # before: begin_step raises it, end_step carries it back
            expect(int(pg._base[0]) == 6 + 2 + 4 * it, f"epoch counter {int(pg._base[0])}")
            expect(pg.epoch == 6 + 4 + 4 * it, f"absolute epoch {pg.epoch}")
            # no rank starts the next call into an output before every peer
            # has gathered this one (the calls of a step come before its
            # gathers)
            dist.barrier()
        # this rank's own rows come from its own matmul, never from the buffer
        r0, r1 = row_shards(64, world)[rank]
        expect((pg.outputs["a"].own0, pg.outputs["a"].own1) == (r0, r1), "own range")
        dist.barrier()
        q.put((rank, bad))
    except Exception as e:  # report, then fail the test on the host
        q.put((rank, repr(e)))
    finally:
        dist.barrier()
        tr.close()
        dist.destroy_process_group()


def test_peer_group_protocol_on_two_gloo_ranks():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: [], 1: []}, res
