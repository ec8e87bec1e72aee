"""Row sharding of the quantized matmul over the GPUs of one node, with the
output all-gather fused into the matmul (NVLink stores of {value, epoch}
words into peer-mapped receive buffers, or for prefill batches plain values
and one release flag per peer; librce_qmm.so's
rce_qmm_mm_batched_device_multi_gather[_bulk] and rce_qmm_peer_unpack[_bulk]).

Rows of a GGUF weight are independent -- the reference splits them over host
threads with rayon (rce-op-qmm/src/lib.rs:502, 654, 742) -- so a row shard
per GPU gives, row for row, the single-GPU result.  One process per GPU;
torch.distributed (any backend) only exchanges the buffers' IPC handles.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Tuple

from ._lib import check, lib
from .qmm import Context, QuantWeight, _check_weight, _stream_handle

TILE_ROWS = 16  # shards start on a 16-row tile of the device layout


def row_shards(n_rows: int, world: int) -> List[Tuple[int, int]]:
    """[row0, row1) of each rank: whole 16-row tiles, as even as possible,
    rank order, covering [0, n_rows)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    tiles = (n_rows + TILE_ROWS - 1) // TILE_ROWS
    out = []
    for r in range(world):
        t0 = tiles * r // world
        t1 = tiles * (r + 1) // world
        out.append((min(n_rows, t0 * TILE_ROWS), min(n_rows, t1 * TILE_ROWS)))
    return out


BULK_MIN_TOKENS = 16  # outputs this tall also get a bulk buffer (plain values, one flag per peer)


class _Output:
    """One gathered output: this rank's full y, the peers' receive buffers
    of {value, epoch} words, optionally the bulk buffers, and what the last
    matmul into it was (its epoch, this rank's rows, the mode)."""

    def __init__(self, y, ll, t_rows, n_rows, bulk=None, flag_off=0):
        self.y, self.ll, self.t_rows, self.n_rows = y, ll, t_rows, n_rows
        self.bulk, self.flag_off = bulk, flag_off  # bulk: two buffer sets, alternated per bulk call
        self.own0 = self.own1 = 0
        self.epoch = None
        self.bulk_mode = False
        self.bulk_calls = 0  # bulk calls made into this output
        self.bulk_sel = 0    # the buffer set of the latest one


class PeerGroup:
    """The buffers one rank shares with the others for gathered outputs: per
    output name, this rank's full output (a torch tensor), a receive buffer
    of 8-byte {value, epoch} words that the other ranks write over NVLink
    (decode-sized calls), and for outputs of BULK_MIN_TOKENS or more tokens
    a bulk buffer of plain values plus one release flag per peer (prefill
    calls; half the NVLink bytes).  `exchange` is a callable (obj -> list of
    every rank's obj, in rank order), e.g. torch_exchange().

    Run-ahead: bulk values carry no epoch, so consecutive bulk calls into an
    output alternate between two bulk buffers: a rank may start the next
    call into an output while its peers still unpack the previous one, but
    not the one after (every rank gathers an output before its second next
    call into it, as the step pattern mm... then gather... does).  A buffer
    overwritten by a later call before its unpack is reported as an error,
    never mixed.  Word-mode outputs carry the epoch in every word and a
    gather accepts a later call's words, which replace the earlier ones: a
    rank must not start the next call into a word-mode output before every
    peer has gathered the previous one whenever the values differ (a
    barrier between steps, or each output's gather before its next call).
    In a CUDA graph, capture an even number of bulk calls per output, so
    that every replay alternates the same way."""

    def __init__(self, ctx: Context, world: int, rank: int, exchange, transport=None):
        if not 2 <= world <= 8:
            raise ValueError("world must be 2..8")
        self.ctx, self.world, self.rank, self._exchange = ctx, world, rank, exchange
        # the library entry points, device tensors and stream handles this
        # group uses (librce_qmm.so and CUDA unless a test supplies another)
        self._t = transport if transport is not None else _LibTransport()
        self.epoch = 0
        self._own: List[int] = []          # own allocations (device pointers)
        self._opened: List[int] = []       # peers' allocations mapped here
        self.outputs: Dict[str, _Output] = {}
        # step mode: epochs relative to a device counter that begin_step
        # advances, so calls captured in a CUDA graph use fresh epochs on
        # every replay
        self._base = None
        self._rel = None
        self._step_calls = 0

    def _shared(self, nbytes: int) -> List[int]:
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        check(self._t.rce_qmm_peer_alloc(self.ctx.handle, nbytes, ctypes.byref(ptr), handle))
        self._own.append(ptr.value)
        handles = self._exchange(handle.raw)
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(ptr.value)
                continue
            p = ctypes.c_void_p()
            check(self._t.rce_qmm_peer_open(self.ctx.handle, ctypes.create_string_buffer(h, 64), ctypes.byref(p)))
            self._opened.append(p.value)
            ptrs.append(p.value)
        return ptrs

    def output(self, name: str, t_rows: int, n_rows: int):
        """Create the gathered output `name` ([t_rows, n_rows] f32; collective:
        every rank creates the same names in the same order)."""
        import torch

        if name not in self.outputs:
            ll = self._shared(8 * t_rows * n_rows)
            bulk, flag_off = None, 0
            if t_rows >= BULK_MIN_TOKENS:
                flag_off = (4 * t_rows * n_rows + 63) // 64 * 64
                bulk = [(ctypes.c_void_p * self.world)(*self._shared(flag_off + 64)) for _ in range(2)]
            y = self._t.zeros((t_rows, n_rows), torch.float32, self.ctx.device)
            self.outputs[name] = _Output(y, (ctypes.c_void_p * self.world)(*ll), t_rows, n_rows, bulk, flag_off)
        return self.outputs[name].y

    def view(self, name: str):
        """This rank's full output `name` (complete after gather(name))."""
        return self.outputs[name].y

    def _next_epoch(self):
        if self._rel is not None:
            self._rel += 1
            return self._rel, ctypes.c_void_p(self._base.data_ptr())
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF or 1
        return self.epoch, None

    def _bulk_call(self, x, outs) -> bool:
        pmt = self.ctx.prefill_min_tokens
        return pmt > 0 and x.shape[0] >= pmt and all(o.bulk is not None for o in outs)

    def mm(self, x, w: QuantWeight, name: str, row_offset: int, stream=None) -> int:
        """x [T, K] (CUDA f32) times this rank's row shard w (rows
        [row_offset, row_offset + w.n_rows) of the full weight): this rank's
        rows of output `name`, sent to every rank.  Returns the epoch to
        pass to gather()."""
        return self.mm_multi(x, [w], [name], [row_offset], stream=stream)

    def mm_multi(self, x, weights, names, row_offsets, stream=None) -> int:
        """mm() for 1-4 row shards that read the same x (weights of one dtype
        and K, e.g. attention q, k, v), in one launch
        (rce_qmm_mm_batched_device_multi_gather; batches of
        ctx.prefill_min_tokens or more tokens into outputs with a bulk buffer:
        rce_qmm_mm_batched_device_multi_gather_bulk).  Shard i goes into
        output names[i] at row_offsets[i].  One epoch for all the outputs
        (returned; gather() each name as usual)."""
        weights, names, row_offsets = list(weights), list(names), [int(r) for r in row_offsets]
        if not (1 <= len(weights) <= 4 and len(names) == len(weights) == len(row_offsets)):
            raise ValueError("mm_multi takes 1 to 4 weights, one output name and row offset each")
        outs = []
        for w, name, r0 in zip(weights, names, row_offsets):
            _check_weight(w)
            o = self.outputs[name]
            if x.shape[0] > o.t_rows or x.shape[1] != w.n_cols or r0 + w.n_rows > o.n_rows:
                raise ValueError(f"shape mismatch with the gathered output {name}")
            outs.append(o)
        epoch, base = self._next_epoch()
        n = len(weights)
        hs = (ctypes.c_void_p * n)(*[w.handle for w in weights])
        offs = (ctypes.c_int64 * n)(*row_offsets)
        ys = (ctypes.c_void_p * n)(*[o.y.data_ptr() for o in outs])
        lds = (ctypes.c_size_t * n)(*[o.n_rows for o in outs])
        bulk = self._bulk_call(x, outs)
        s = self._t.stream(stream, x.device)
        if bulk:
            sel = [o.bulk_calls % 2 for o in outs]
            bufs = (ctypes.c_void_p * (n * self.world))(*[o.bulk[s_][r] for o, s_ in zip(outs, sel)
                                                          for r in range(self.world)])
            flags = (ctypes.c_size_t * n)(*[o.flag_off for o in outs])
            check(self._t.rce_qmm_mm_batched_device_multi_gather_bulk(
                self.ctx.handle, ctypes.c_void_p(x.data_ptr()), x.stride(0), x.shape[0], hs, n, self.world,
                self.rank, offs, ys, lds, bufs, flags, epoch, base, s))
        else:
            lls = (ctypes.c_void_p * (n * self.world))(*[o.ll[r] for o in outs for r in range(self.world)])
            check(self._t.rce_qmm_mm_batched_device_multi_gather(
                self.ctx.handle, ctypes.c_void_p(x.data_ptr()), x.stride(0), x.shape[0], hs, n, self.world,
                self.rank, offs, ys, lds, lls, epoch, base, s))
        for i, (o, w, r0) in enumerate(zip(outs, weights, row_offsets)):
            o.own0, o.own1, o.epoch, o.bulk_mode = r0, r0 + w.n_rows, epoch, bulk
            if bulk:
                o.bulk_sel = sel[i]
                o.bulk_calls += 1
        return epoch

    def gather(self, name: str, epoch: Optional[int] = None, t_rows: Optional[int] = None, stream=None):
        """Complete output `name` on this rank: wait (on `stream`, bounded)
        for the other ranks' rows of the call with `epoch` (default: the
        latest mm into `name`) and copy them in.  Returns the tensor."""
        o = self.outputs[name]
        epoch = o.epoch if epoch is None else epoch
        base = ctypes.c_void_p(self._base.data_ptr()) if self._rel is not None else None
        rows = o.t_rows if t_rows is None else t_rows
        s = self._t.stream(stream, o.y.device)
        if o.bulk_mode:
            check(self._t.rce_qmm_peer_unpack_bulk(self.ctx.handle, ctypes.c_void_p(o.bulk[o.bulk_sel][self.rank]),
                                                 o.flag_off,
                                                 ctypes.c_void_p(o.y.data_ptr()), o.n_rows, rows, o.n_rows,
                                                 int(o.own0), int(o.own1), self.world, self.rank, int(epoch), base, s))
        else:
            check(self._t.rce_qmm_peer_unpack(self.ctx.handle, ctypes.c_void_p(o.ll[self.rank]),
                                            ctypes.c_void_p(o.y.data_ptr()), o.n_rows, rows, o.n_rows, int(o.own0),
                                            int(o.own1), int(epoch), base, s))
        return o.y

    def begin_step(self, calls: int, stream=None) -> None:
        """Start a step of at most `calls` mm calls whose epochs are relative
        to a device counter advanced here by `calls` -- capture begin_step,
        the calls and the gathers in one CUDA graph and every replay uses
        new epochs.  Every rank must use the same `calls` and call sequence.
        The counter starts at (and, coming from absolute epochs, is raised
        to) the last absolute epoch, so epochs only grow across both modes:
        make the first begin_step after absolute calls outside a capture."""
        import torch

        if self._base is None:
            self._base = self._t.zeros((1,), torch.int32, self.ctx.device)
            self._base.fill_(self.epoch)
        elif self._rel is None and self.epoch > 0:
            self._base.clamp_(min=self.epoch)
        self._rel = 0
        self._step_calls = int(calls)
        check(self._t.rce_qmm_peer_epoch_advance(self.ctx.handle, ctypes.c_void_p(self._base.data_ptr()), int(calls),
                                               self._t.stream(stream, self._base.device)))

    def end_step(self) -> None:
        """Leave step mode: later calls use absolute epochs again, above
        every epoch the steps used (the counter is read back: this
        synchronises with the device, so call it outside a capture)."""
        if self._rel is not None and self._base is not None:
            self.epoch = max(self.epoch, int(self._base.cpu()[0]) + self._step_calls) & 0xFFFFFFFF
        self._rel = None

    def close(self) -> None:
        for p in self._opened:
            self._t.rce_qmm_peer_close(self.ctx.handle, ctypes.c_void_p(p))
        for p in self._own:
            self._t.rce_qmm_peer_free(self.ctx.handle, ctypes.c_void_p(p))
        self._opened, self._own, self.outputs = [], [], {}


class _LibTransport:
    """librce_qmm.so's entry points, CUDA tensors and stream handles."""

    def __getattr__(self, name):
        return getattr(lib(), name)

    @staticmethod
    def zeros(shape, dtype, device: int):
        import torch

        return torch.zeros(shape, dtype=dtype, device=f"cuda:{device}")

    @staticmethod
    def stream(stream, device):
        return _stream_handle(stream, device)


def _wrap_device(ptr: int, shape, device: int):
    """A torch view of device memory owned elsewhere (kept alive by the
    PeerGroup)."""
    import torch

    class _Mem:
        def __init__(self, p, n):
            self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (p, False), "version": 3}

    n = 1
    for d in shape:
        n *= d
    with torch.cuda.device(device):
        return torch.as_tensor(_Mem(ptr, n), device=f"cuda:{device}").view(*shape)


def torch_exchange(group=None):
    """An `exchange` for PeerGroup over torch.distributed."""
    import torch.distributed as dist

    def ex(obj):
        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, obj, group=group)
        return out

    return ex
