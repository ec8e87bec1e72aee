"""Benchmark of the B200 GGUF quantized-matmul path.

Workload: the Llama-3-8B-shaped Q4_K decode matmul
stack -- 32 layers x {q 4096x4096, k 1024x4096, v 1024x4096, o 4096x4096,
gate 14336x4096, up 14336x4096, down 4096x14336}, 3,925,868,544 weight bytes,
batch 1 (``--batch 16`` for the batch-16 variant), seeded synthetic weights
with the configuration's distributions and N(0,1) activations.  One step =
one decode token through all 224 matmuls in layer order, replayed from a
CUDA graph; on one GPU the matrices that read the same activation share a
launch (q, k, v and gate, up through rce_qmm_mm_batched_device_multi: 4
launches per layer; ``--no-group`` for one launch per matrix).  With N GPUs every matrix is row-sharded N ways
and each output is all-gathered by the matmul itself: its kernel stores the
rows, as {value, epoch} words, into every other GPU's receive buffer over
NVLink; the step ends with each GPU unpacking the seven outputs (waiting
for every word of the step's last epochs) -- strong scaling: the model is
fixed, value counts its bytes once.

value  = weight bytes of the whole model x steps / device time (max over ranks)
e2e    = the same through the public API with host buffers, copies in and out
         on every call, timed by the wall clock around the synchronous calls:
         the host C-ABI call rce_qmm_mm_batched on one GPU; with N GPUs each
         rank's row-shard matmul with its fused gather (PeerGroup), its input
         copied in from pinned memory and the whole gathered output copied back
roofline = the dominant kernel (the 14336x4096 / 4096x14336 Q4_K GEMVs) timed
         launch by launch with CUDA events, algorithmic bytes / duration
cpu_baseline = the C restatement of the reference's CPU path (oracle/) on one
         layer of the same stack, all host threads
prefill  = BASELINE configs[2]: Q4_K 14336x4096 weight (row-sharded N ways),
         M = 1, 16, 128, 512 f32 activations through mm_batched_device (the
         tcgen05 GEMM from ctx.prefill_min_tokens = 16 tokens on, the GEMV
         below); four distinct weights per pass (132 MB > L2) replayed from a
         CUDA graph, CUDA events; TFLOP/s = 2 M N K / time, against the
         measured bf16 dense peak
formats_gemv = one GPU: the decode GEMV of every supported format (Q4_K, Q5_K,
         Q6_K, Q8_0, Q4_0) at 14336x4096 and 4096x14336, 8 distinct weights
         per shape in a CUDA graph, CUDA events
stack_batch16 = one GPU: the same stack at batch 16 (configs[3]'s second batch
         size), every matmul through mm_batched's routing (the tcgen05 GEMM),
         replayed from a CUDA graph; GB/s of weights and tokens/s
baseline_configs_gemv = one GPU: configs[0] (Q8_0 4096x4096, seed 0) and
         configs[1] (Q4_0 11008x4096 / 4096x11008, seed 1) at their own shapes
prefill.e2e_m512 = configs[2] at M = 512 through the host C-ABI
         (rce_qmm_mm_batched), wall clock
cpu_baseline.one_thread = the same CPU sample on one host thread
The weights (3.9 GB) are far larger than L2 (126 MB), so no L2 flush is
needed between steps.

``--impl reference`` times the reference's CPU path (the oracle port; the Rust
crate cannot be built here) on the same metric: each step is one layer's
seven matmuls (122,683,392 weight bytes), all host threads.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "quant GEMV weight GB/s vs HBM peak; prefill GEMM TFLOP/s; 1/2/4/8 GPU"
Q4_K = 12
D_MODEL, D_FF, D_KV = 4096, 14336, 1024
# (name, n_rows, n_cols)
LAYER = [("q", D_MODEL, D_MODEL), ("k", D_KV, D_MODEL), ("v", D_KV, D_MODEL), ("o", D_MODEL, D_MODEL),
         ("gate", D_FF, D_MODEL), ("up", D_FF, D_MODEL), ("down", D_MODEL, D_FF)]
# matrices that read the same activation run as one launch on one GPU
# (rce_qmm_mm_batched_device_multi): attention q, k, v and FFN gate, up
GROUPS = [("q", "k", "v"), ("o",), ("gate", "up"), ("down",)]


def q4k_bytes(n, k):
    return n * k // 256 * 144


def layer_bytes():
    return sum(q4k_bytes(n, k) for _, n, k in LAYER)


def load_peaks():
    for p in (os.path.join(ROOT, "MEASURED_PEAKS.json"),):
        if os.path.exists(p):
            d = json.load(open(p))
            return d.get("hbm_gbs"), d.get("bf16_tflops"), "measured"
    return 6650.0, 1590.0, "fallback"


# ---- clocks -------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.path = tempfile.mktemp(prefix="clocks_", suffix=".csv")
        self.proc = None
        self.windows = []
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def mark(self):
        return time.time()

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self, t0, t1):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as f:
            lines = f.read().strip().splitlines()
        # nvidia-smi -lms has no timestamps: spread the samples evenly over the
        # sampling lifetime and keep the ones inside [t0, t1] (widened to one
        # interval each side so short regions still get samples)
        mine = [ln.split(", ") for ln in lines if self.uuid and self.uuid in ln]
        if not mine:
            mine = [ln.split(", ") for ln in lines]
        if not mine:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        for r in mine:
            try:
                rows.append((float(r[1]), float(r[2]), r[4:8]))
            except (ValueError, IndexError):
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unparsed samples"]}
        n = len(rows)
        start, end = self.t_start, self.t_end
        span = max(end - start, 1e-3)
        sel = [rows[i] for i in range(n) if t0 - 0.15 <= start + span * (i + 0.5) / n <= t1 + 0.15]
        if not sel:
            sel = rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in sel for j, v in enumerate(r[2]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(r[0] for r in sel), "sm_max_mhz": max(r[1] for r in sel),
                "reasons": reasons, "samples": len(sel)}


# ---- the reference arm ------------------------------------------------------------

def cpu_layer_sample(seed=3):
    from rce_b200 import synth

    rng = np.random.default_rng(seed)
    mats = [(name, n, k, synth.q4_k(n, k, rng)) for name, n, k in LAYER]
    xs = {D_MODEL: synth.activations(1, D_MODEL, rng)[0], D_FF: synth.activations(1, D_FF, rng)[0]}
    return mats, xs


def time_cpu_layer(mats, xs, threads, reps=None, budget_s=10.0):
    import oracle as O

    times = []
    t_total = 0.0
    r = 0
    while True:
        t0 = time.perf_counter()
        for name, n, k, w in mats:
            O.mm_1d(xs[k], w, Q4_K, n, k, nthreads=threads)
        dt = time.perf_counter() - t0
        times.append(dt)
        t_total += dt
        r += 1
        if reps is not None and r >= reps:
            break
        if reps is None and (t_total >= budget_s or r >= 200):
            break
    return times


def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    mats, xs = cpu_layer_sample()
    time_cpu_layer(mats, xs, threads, reps=max(1, args.warmup))
    times = time_cpu_layer(mats, xs, threads, reps=args.steps)
    lb = layer_bytes()
    tot = sum(times)
    value = lb * len(times) / tot / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * tot / len(times), 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, configuration distributions)",
        "config": config_dict(args, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "one layer of the stack per step (7 Q4_K matmuls, 122,683,392 weight bytes), "
                                   "oracle/qmm_oracle.c restating rce-op-qmm mm_1d_q4_k, rows over all host threads"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference crate is Rust and no Rust toolchain exists here; its CPU path is timed through the "
                "bit-exact C restatement",
    }
    print(json.dumps(line), flush=True)


def config_dict(args, world):
    return {"workload": "llama3-8b-shaped Q4_K decode matmul stack (configs[3])", "layers": args.layers,
            "batch": args.batch, "matmuls_per_step": 7 * args.layers,
            "launches_per_layer": (len(GROUPS) if not args.no_group else 7), "weight_bytes": layer_bytes() * args.layers,
            "parallelism": f"row-shard x{world} + all-gather" if world > 1 else "single GPU",
            "l2": "no flush: weights 3.9 GB >> 126 MB L2" if args.layers >= 8 else "small stack (profiling)"}


# ---- prefill GEMM ---------------------------------------------------------

PREFILL_N, PREFILL_K, PREFILL_MS = D_FF, D_MODEL, (1, 16, 128, 512)


def prefill_section(args, rank, world, dev, stream, ctx, pg=None):
    import torch
    import torch.distributed as dist

    import rce_b200 as R
    from rce_b200 import synth

    ns = PREFILL_N // world
    ws = []
    for i in range(4):
        g = torch.Generator(device=dev)
        g.manual_seed(2_000_000 + 97 * i + rank)
        raw = synth.device_weights(Q4_K, ns, PREFILL_K, g, dev)
        ws.append(R.QuantWeight.from_device_bytes(raw, Q4_K, ns, PREFILL_K, ctx=ctx))
        del raw
    out = {}
    for m in PREFILL_MS:
        g = torch.Generator(device=dev)
        g.manual_seed(2)
        x = torch.randn((m, PREFILL_K), device=dev, generator=g)
        y = torch.empty((m, ns), device=dev)
        names = [f"prefill{m}_{i}" for i in range(len(ws))]
        if world > 1:
            for nm in names:
                pg.output(nm, m, PREFILL_N)

        def one():
            if world > 1:
                # every shard's matmul first, then the gathers: weight i's
                # outputs cross NVLink while weight i + 1's GEMM runs
                pg.begin_step(len(ws), stream=stream)
                for w, nm in zip(ws, names):
                    pg.mm(x, w, nm, rank * ns, stream=stream)
                for nm in names:
                    pg.gather(nm, stream=stream)
            else:
                for w in ws:
                    R.mm_batched_device(x, w, y, stream=stream)

        with torch.cuda.stream(stream):
            for _ in range(3):
                one()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        # two passes per graph: a bulk-gathered output alternates between two
        # receive buffers per call, so every replay must make an even number
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            one()
            one()
        reps = 10
        with torch.cuda.stream(stream):
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize(dev)
            if world > 1:
                dist.barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / (reps * 2 * len(ws))
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        flops = 2.0 * m * PREFILL_N * PREFILL_K
        out[f"m{m}"] = {"us": round(ms * 1e3, 2), "tflops": round(flops / (ms / 1e3) / 1e12, 1),
                        "path": "tcgen05 GEMM" if m >= ctx.prefill_min_tokens else "GEMV"}
        del graph
    if pg is not None:
        pg.end_step()
    if world == 1:
        # end to end through the host C-ABI (rce_qmm_mm_batched: host
        # activations in, host outputs out, synchronous), M = 512
        m = 512
        g = torch.Generator(device=dev)
        g.manual_seed(2)
        xh = torch.randn((m, PREFILL_K), device=dev, generator=g).cpu().numpy()
        yh = np.empty(m * ns, np.float32)
        R.mm_batched(xh, m, ws[0], yh)
        calls = 10
        t0 = time.perf_counter()
        for i in range(calls):
            R.mm_batched(xh, m, ws[i % len(ws)], yh)
        dt = (time.perf_counter() - t0) / calls
        out["e2e_m512"] = {"us": round(dt * 1e6, 1), "tflops": round(2.0 * m * ns * PREFILL_K / dt / 1e12, 1),
                           "h2d_bytes": m * PREFILL_K * 4, "d2h_bytes": m * ns * 4,
                           "timing": "wall clock around synchronous rce_qmm_mm_batched calls (host buffers)"}
    return out


# ---- MoE FFN ------------------------------------------------------------

MOE_E, MOE_K, MOE_T = 8, 2, 256


def formats_section(args, dev, stream, ctx):
    """Decode GEMV (one token) of every supported format at the stack's two
    large shapes: 8 distinct weights per shape (more bytes than L2) launched
    back to back in a CUDA graph, CUDA events; GB/s of algorithmic bytes."""
    import torch

    import rce_b200 as R
    from rce_b200 import synth
    from rce_b200.gguf import GgufDtype, tensor_byte_size

    out = {}
    for fmt in (GgufDtype.Q4K, GgufDtype.Q5K, GgufDtype.Q6K, GgufDtype.Q8_0, GgufDtype.Q4_0):
        res = {}
        for n, k in ((D_FF, D_MODEL), (D_MODEL, D_FF)):
            ws = []
            for i in range(8):
                g = torch.Generator(device=dev)
                g.manual_seed(5_000_000 + 31 * i + int(fmt))
                raw = synth.device_weights(fmt, n, k, g, dev)
                ws.append(R.QuantWeight.from_device_bytes(raw, fmt, n, k, ctx=ctx))
                del raw
            x = torch.randn((1, k), device=dev)
            y = torch.empty((1, n), device=dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                for w in ws:
                    R.mm_batched_device(x, w, y, stream=stream)
            stream.synchronize()
            with torch.cuda.graph(graph, stream=stream):
                for w in ws:
                    R.mm_batched_device(x, w, y, stream=stream)
            with torch.cuda.stream(stream):
                for _ in range(3):
                    graph.replay()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                reps = 20
                e0.record(stream)
                for _ in range(reps):
                    graph.replay()
                e1.record(stream)
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * len(ws))
            alg = tensor_byte_size(fmt, n * k) + 4 * k + 4 * n
            res[f"{n}x{k}"] = {"us": round(us, 2), "gbs": round(alg / (us / 1e6) / 1e9, 1)}
            del graph, ws
        out[fmt.name] = res
    return out


def baseline_configs_section(args, dev, stream, ctx, hbm):
    """configs[0] (Q8_0 4096x4096, seed 0) and configs[1] (Q4_0 11008x4096 and
    4096x11008, seed 1) at their own shapes: the one-token decode GEMV, 8
    distinct weights per shape (more bytes than L2) back to back in a CUDA
    graph, CUDA events; GB/s of algorithmic bytes and the fraction of HBM."""
    import torch

    import rce_b200 as R
    from rce_b200 import synth
    from rce_b200.gguf import GgufDtype, tensor_byte_size

    out = {}
    for name, fmt, n, k, seed in (("configs[0] Q8_0 4096x4096", GgufDtype.Q8_0, 4096, 4096, 0),
                                  ("configs[1] Q4_0 11008x4096", GgufDtype.Q4_0, 11008, 4096, 1),
                                  ("configs[1] Q4_0 4096x11008", GgufDtype.Q4_0, 4096, 11008, 1)):
        ws = []
        for i in range(8):
            g = torch.Generator(device=dev)
            g.manual_seed(seed * 1_000_003 + i)
            raw = synth.device_weights(fmt, n, k, g, dev)
            ws.append(R.QuantWeight.from_device_bytes(raw, fmt, n, k, ctx=ctx))
            del raw
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        x = torch.randn((1, k), device=dev, generator=g)
        y = torch.empty((1, n), device=dev)
        with torch.cuda.stream(stream):
            for w in ws:
                R.mm_batched_device(x, w, y, stream=stream)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for w in ws:
                R.mm_batched_device(x, w, y, stream=stream)
        with torch.cuda.stream(stream):
            for _ in range(3):
                graph.replay()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            reps = 20
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * len(ws))
        alg = tensor_byte_size(fmt, n * k) + 4 * k + 4 * n
        gbs = alg / (us / 1e6) / 1e9
        out[name] = {"us": round(us, 2), "gbs": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 4),
                     "alg_bytes": alg}
        del graph, ws
    return out


def moe_section(args, rank, world, dev, stream, ctx, calls=0):
    """Mixtral-shaped MoE FFN: 8 experts of Q4_K gate/up 14336x4096 and down
    4096x14336, 256 tokens, top-2 from softmax of N(0,1) router logits.
    Experts are placed world-ways (8/world per GPU); every GPU routes all
    tokens, runs its experts' rows, and the outputs are summed over NCCL."""
    import torch
    import torch.distributed as dist

    import rce_b200 as R
    from rce_b200 import synth

    if MOE_E % world:
        return None
    per = MOE_E // world
    lo, hi = rank * per, (rank + 1) * per
    gate, up, down = [None] * MOE_E, [None] * MOE_E, [None] * MOE_E
    for e in range(lo, hi):
        for lst, (n, k), salt in ((gate, (D_FF, D_MODEL), 1), (up, (D_FF, D_MODEL), 2), (down, (D_MODEL, D_FF), 3)):
            g = torch.Generator(device=dev)
            g.manual_seed(4_000_000 + 1009 * e + salt)
            raw = synth.device_weights(Q4_K, n, k, g, dev)
            lst[e] = R.QuantWeight.from_device_bytes(raw, Q4_K, n, k, ctx=ctx)
            del raw
    g = torch.Generator(device=dev)
    g.manual_seed(4)
    x = torch.randn((MOE_T, D_MODEL), device=dev, generator=g)
    logits = torch.randn((MOE_T, MOE_E), device=dev, generator=g)
    out = torch.empty((MOE_T, D_MODEL), device=dev)

    def one():
        R.moe_ffn_device(x, logits, MOE_K, gate, up, down, expert_range=(lo, hi), out=out, stream=stream)
        if world > 1:
            dist.all_reduce(out)

    if calls:  # profiling: the calls only, no timing
        with torch.cuda.stream(stream):
            for _ in range(calls):
                one()
        stream.synchronize()
        return None
    with torch.cuda.stream(stream):
        for _ in range(3):
            one()
    stream.synchronize()
    reps = 10
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            one()
        e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    flops = 2.0 * MOE_T * MOE_K * 3 * D_FF * D_MODEL
    wbytes = MOE_E * (2 * q4k_bytes(D_FF, D_MODEL) + q4k_bytes(D_MODEL, D_FF))
    return {"workload": "configs[4]: Mixtral-shaped MoE FFN, 8 experts x Q4_K gate/up 14336x4096 + down 4096x14336, "
                        "256 tokens, top-2 of softmax(N(0,1) logits), renormalised",
            "placement": f"{per} experts per GPU" + (", outputs summed with NCCL all-reduce" if world > 1 else ""),
            "ms": round(ms, 4), "tokens_per_s": round(MOE_T / (ms / 1e3), 1),
            "tflops": round(flops / (ms / 1e3) / 1e12, 1), "weight_gbs": round(wbytes / (ms / 1e3) / 1e9, 1),
            "path": "expert-grouped tensor-core launches (gate+up of all local experts in one, down in one), "
                    "row counts read on the device",
            "timing": "CUDA events around 10 back-to-back calls (no host synchronisation inside a call)"}


# ---- our arm -------------------------------------------------------------------------

def build_stack(args, rank, world, dev):
    import torch

    import rce_b200 as R
    from rce_b200 import synth

    ctx = R.default_context(dev.index)
    layers = []
    for li in range(args.layers):
        mats = []
        for mi, (name, n, k) in enumerate(LAYER):
            ns = n // world
            g = torch.Generator(device=dev)
            g.manual_seed(3_000_000 + 7919 * li + 131 * mi + rank)
            raw = synth.device_weights(Q4_K, ns, k, g, dev)
            w = R.QuantWeight.from_device_bytes(raw, Q4_K, ns, k, ctx=ctx)
            del raw
            mats.append((name, ns, k, w))
        layers.append(mats)
    torch.cuda.synchronize(dev)
    return ctx, layers


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-group", action="store_true",
                    help="one launch per matrix (no grouped q/k/v and gate/up launches)")
    ap.add_argument("--profile", action="store_true", help="short run for ncu: warm-up + steps only")
    ap.add_argument("--profile-moe", action="store_true",
                    help="for ncu: only the configs[4] MoE FFN on one GPU, warm-up + steps calls (five launches each)")
    ap.add_argument("--profile-prefill", type=int, default=0, metavar="M",
                    help="for ncu: only the configs[2] prefill matmul at M tokens, warm-up + steps launches")
    ap.add_argument("--profile-gemv", default="", metavar="FORMAT",
                    help="for ncu: only the one-token decode GEMV of a 14336x4096 weight in FORMAT "
                         "(Q4K, Q5K, Q6K, Q8_0, Q4_0), warm-up + steps launches")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if world > 1:
            import torch.distributed as dist

            dist.init_process_group("gloo", init_method="env://")
        run_reference(args, rank, world)
        if world > 1:
            dist.destroy_process_group()
        return

    import datetime

    import torch
    import torch.distributed as dist

    import rce_b200 as R

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.profile_gemv:
        from rce_b200 import synth
        from rce_b200.gguf import GgufDtype

        fmt = GgufDtype[args.profile_gemv]
        ctx = R.default_context(dev.index)
        g = torch.Generator(device=dev)
        g.manual_seed(5)
        raw = synth.device_weights(fmt, D_FF, D_MODEL, g, dev)
        w = R.QuantWeight.from_device_bytes(raw, fmt, D_FF, D_MODEL, ctx=ctx)
        x = torch.randn((1, D_MODEL), device=dev, generator=g)
        y = torch.empty((1, D_FF), device=dev)
        for _ in range(args.warmup + args.steps):
            R.mm_batched_device(x, w, y)
        torch.cuda.synchronize(dev)
        print(json.dumps({"profile_gemv": args.profile_gemv, "launches": args.warmup + args.steps}))
        return
    if args.profile_moe:
        stream = torch.cuda.Stream(dev)
        moe_section(args, 0, 1, dev, stream, R.default_context(dev.index), calls=args.warmup + args.steps)
        print(json.dumps({"profile_moe": True, "calls": args.warmup + args.steps}))
        return
    if args.profile_prefill:
        from rce_b200 import synth

        ctx = R.default_context(dev.index)
        g = torch.Generator(device=dev)
        g.manual_seed(2)
        raw = synth.device_weights(Q4_K, PREFILL_N, PREFILL_K, g, dev)
        w = R.QuantWeight.from_device_bytes(raw, Q4_K, PREFILL_N, PREFILL_K, ctx=ctx)
        x = torch.randn((args.profile_prefill, PREFILL_K), device=dev, generator=g)
        y = torch.empty((args.profile_prefill, PREFILL_N), device=dev)
        for _ in range(args.warmup + args.steps):
            R.mm_batched_device(x, w, y)
        torch.cuda.synchronize(dev)
        print(json.dumps({"profile_prefill": args.profile_prefill, "launches": args.warmup + args.steps}))
        return
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    ctx, layers = build_stack(args, rank, world, dev)
    pg = None
    if world > 1:
        from rce_b200.shard import PeerGroup, torch_exchange

        pg = PeerGroup(ctx, world, rank, torch_exchange())
    m = args.batch
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    xs = {D_MODEL: torch.randn((m, D_MODEL), device=dev, generator=gen),
          D_FF: torch.randn((m, D_FF), device=dev, generator=gen)}
    ys = {name: torch.empty((m, n // world), device=dev) for name, n, _ in LAYER}
    if world > 1:
        for name, n, _ in LAYER:
            pg.output(name, m, n)
    stream = torch.cuda.Stream(dev)
    grouped = not args.no_group
    per_layer = len(GROUPS) if grouped else 7
    launches_per_step = per_layer * args.layers + (8 if world > 1 else 0)

    def step():
        if world > 1:
            pg.begin_step(per_layer * args.layers, stream=stream)
        for mats in layers:
            if grouped:
                by = {name: (ns, k, w) for name, ns, k, w in mats}
                for grp in GROUPS:
                    k = by[grp[0]][1]
                    if world > 1:
                        pg.mm_multi(xs[k], [by[nm][2] for nm in grp], list(grp), [rank * by[nm][0] for nm in grp],
                                    stream=stream)
                    elif len(grp) == 1:
                        R.mm_batched_device(xs[k], by[grp[0]][2], ys[grp[0]], stream=stream)
                    else:
                        R.mm_multi_device(xs[k], [by[nm][2] for nm in grp], [ys[nm] for nm in grp], stream=stream)
                continue
            for name, ns, k, w in mats:
                if world > 1:
                    pg.mm(xs[k], w, name, rank * ns, stream=stream)
                else:
                    R.mm_batched_device(xs[k], w, ys[name], stream=stream)
        if world > 1:
            for name, _, _ in LAYER:
                pg.gather(name, stream=stream)

    graph = None
    with torch.cuda.stream(stream):
        for _ in range(2):
            step()  # eager warm-up: allocates per-stream workspaces before capture
    stream.synchronize()
    if world > 1:
        dist.barrier()
    # the whole step (at N > 1 with its gathers and the final wait) as one CUDA graph
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()

    def run(n):
        with torch.cuda.stream(stream):
            for _ in range(n):
                if graph is not None:
                    graph.replay()
                else:
                    step()

    run(args.warmup)
    stream.synchronize()
    uuid = ""
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid) if rank == 0 else None
    if clocks:
        clocks.t_start = time.time()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    ev0.record(stream)
    run(args.steps)
    ev1.record(stream)
    ev1.synchronize()
    t_wall1 = time.time()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    total_bytes = layer_bytes() * args.layers
    value = total_bytes * args.steps / (ms / 1e3) / 1e9

    if args.profile:
        if clocks:
            clocks.t_end = time.time()
            clocks.stop()
        if rank == 0:
            print(json.dumps({"profile_run": True, "ms_per_step": ms / args.steps, "value": value}))
        del graph
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
            pg.close()
            dist.barrier()
            dist.destroy_process_group()
        return
    del graph
    torch.cuda.synchronize(dev)

    # ---- roofline: per kernel type, the 32 layers' launches back to back in a
    # CUDA graph, timed with CUDA events on the launching stream ----------------
    kern = {}
    for name, n, k in LAYER:
        g_t = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_t, stream=stream):
            for mats in layers:
                for nm, ns, kk, w in mats:
                    if nm == name:
                        R.mm_batched_device(xs[kk], w, ys[nm], stream=stream)
        with torch.cuda.stream(stream):
            for _ in range(3):
                g_t.replay()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            reps = 10
            e0.record(stream)
            for _ in range(reps):
                g_t.replay()
            e1.record(stream)
        e1.synchronize()
        avg_ms = e0.elapsed_time(e1) / (reps * args.layers)
        ns = n // world
        alg = q4k_bytes(ns, k) + 4 * m * k + 4 * m * ns
        kern[name] = {"avg_us": avg_ms * 1e3, "alg_bytes": alg, "gbs": alg / (avg_ms / 1e3) / 1e9,
                      "total_ms": avg_ms * args.layers}
        del g_t
    # the grouped launches of the step, timed the same way
    groups = {}
    if grouped:
        for grp in GROUPS:
            if len(grp) == 1:
                continue
            g_t = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_t, stream=stream):
                for mats in layers:
                    by = {nm: (ns, kk, w) for nm, ns, kk, w in mats}
                    R.mm_multi_device(xs[by[grp[0]][1]], [by[nm][2] for nm in grp], [ys[nm] for nm in grp],
                                      stream=stream)
            with torch.cuda.stream(stream):
                for _ in range(3):
                    g_t.replay()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                reps = 10
                e0.record(stream)
                for _ in range(reps):
                    g_t.replay()
                e1.record(stream)
            e1.synchronize()
            avg_ms = e0.elapsed_time(e1) / (reps * args.layers)
            dims = {nm: (n // world, k) for nm, n, k in LAYER}  # this GPU's shards
            alg = sum(q4k_bytes(dims[nm][0], dims[nm][1]) + 4 * m * dims[nm][0] for nm in grp) + 4 * m * dims[grp[0]][1]
            groups["+".join(grp)] = {"avg_us": round(avg_ms * 1e3, 2), "gbs": round(alg / (avg_ms / 1e3) / 1e9, 1)}
            del g_t
    if clocks:
        clocks.t_end = time.time()
        clocks.stop()
    dom = max(kern, key=lambda nm: kern[nm]["total_ms"])
    hbm, bf16, peak_kind = load_peaks()
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "gemv_q4k_traffic.json")
    if os.path.exists(tpath):
        try:
            tj = json.load(open(tpath))
            key = f"{D_FF if dom in ('gate', 'up') else D_MODEL}x{D_MODEL if dom != 'down' else D_FF}_m{m}_w{world}"
            traffic = tj.get(key)
        except Exception:
            traffic = None

    if pg is not None:
        pg.end_step()  # absolute epochs for the eager legs below
    # ---- the batch-16 decode stack (configs[3] at batch 16), one GPU: the
    # same 32 layers, each matmul through mm_batched's routing (the tensor-core
    # GEMM from 16 tokens), grouped as the step above ---------------------------
    stack16 = None
    if world == 1 and m == 1:
        x16 = {D_MODEL: torch.randn((16, D_MODEL), device=dev, generator=gen),
               D_FF: torch.randn((16, D_FF), device=dev, generator=gen)}
        y16 = {name: torch.empty((16, n), device=dev) for name, n, _ in LAYER}

        def step16():
            for mats in layers:
                by = {name: (ns, k, w) for name, ns, k, w in mats}
                for grp in GROUPS:
                    k = by[grp[0]][1]
                    if len(grp) == 1:
                        R.mm_batched_device(x16[k], by[grp[0]][2], y16[grp[0]], stream=stream)
                    else:
                        R.mm_multi_device(x16[k], [by[nm][2] for nm in grp], [y16[nm] for nm in grp],
                                          stream=stream)

        with torch.cuda.stream(stream):
            for _ in range(2):
                step16()
        stream.synchronize()
        g16 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g16, stream=stream):
            step16()
        with torch.cuda.stream(stream):
            for _ in range(3):
                g16.replay()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            reps = 20
            e0.record(stream)
            for _ in range(reps):
                g16.replay()
            e1.record(stream)
        e1.synchronize()
        ms16 = e0.elapsed_time(e1) / reps
        v16 = layer_bytes() * args.layers / (ms16 / 1e3) / 1e9
        stack16 = {"batch": 16, "ms_per_step": round(ms16, 4), "value": round(v16, 1), "unit": "GB/s",
                   "frac_of_hbm": round(v16 / load_peaks()[0], 4),
                   "tokens_per_s": round(16 / (ms16 / 1e3), 1),
                   "path": "tcgen05 GEMM per matmul (two-term activations), grouped q+k+v and gate+up"}
        del g16
    prefill = prefill_section(args, rank, world, dev, stream, ctx, pg)
    moe = moe_section(args, rank, world, dev, stream, ctx)
    formats = formats_section(args, dev, stream, ctx) if world == 1 else None
    base_cfgs = baseline_configs_section(args, dev, stream, ctx, load_peaks()[0]) if world == 1 else None

    # ---- e2e through the public API with host buffers -----------------------------
    # N = 1: the C-ABI call rce_qmm_mm_batched (host in, host out; it stages
    # through pinned memory and synchronises).  N > 1: per matmul the host
    # activations are staged into pinned memory and copied in, the row shard's
    # matmul runs with its fused NVLink gather (PeerGroup.mm + gather), and the
    # whole gathered output is copied back to the host, synchronously.
    e2e = None
    hx = {k: v.cpu().numpy() for k, v in xs.items()}
    hy = {name: np.empty((m, n // world), np.float32) for name, n, _ in LAYER}
    h2d = d2h = 0
    for name, n, k in LAYER:
        h2d += 4 * m * k * args.layers
        d2h += 4 * m * (n // world if world == 1 else n) * args.layers
    if world > 1:
        px = {k: torch.empty((m, k), dtype=torch.float32, pin_memory=True) for k in xs}
        dx = {k: torch.empty((m, k), dtype=torch.float32, device=dev) for k in xs}
        py = {name: torch.empty((m, n), dtype=torch.float32, pin_memory=True) for name, n, _ in LAYER}
        hyf = {name: np.empty((m, n), np.float32) for name, n, _ in LAYER}

    def e2e_step():
        for mats in layers:
            for name, ns, k, w in mats:
                if world == 1:
                    R.mm_batched(hx[k], m, w, hy[name].reshape(-1))
                    continue
                with torch.cuda.stream(stream):
                    px[k].numpy()[...] = hx[k]
                    dx[k].copy_(px[k], non_blocking=True)
                    pg.mm(dx[k], w, name, rank * ns, stream=stream)
                    py[name].copy_(pg.gather(name, stream=stream), non_blocking=True)
                stream.synchronize()
                hyf[name][...] = py[name].numpy()

    e2e_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        e2e_step()
    t1 = time.perf_counter()
    e2e_s = t1 - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = {"value": round(total_bytes * args.e2e_steps / e2e_s / 1e9, 3), "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": args.e2e_steps,
           "timing": ("wall clock around the synchronous host C-ABI calls (rce_qmm_mm_batched)" if world == 1 else
                      "wall clock around synchronous per-matmul calls: pinned host copy in, row-shard matmul with "
                      "its fused NVLink gather (PeerGroup.mm + gather), full output copied back; max over ranks")}

    # ---- CPU baseline (rank 0, N = 1) ---------------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        mats_h, xs_h = cpu_layer_sample()
        times = time_cpu_layer(mats_h, xs_h, threads, budget_s=10.0)
        t1 = time_cpu_layer(mats_h, xs_h, 1, reps=2)
        cpu = {"value": round(layer_bytes() * len(times) / sum(times) / 1e9, 3), "unit": "GB/s", "cores": threads,
               "kind": "port",
               "one_thread": {"value": round(layer_bytes() * len(t1) / sum(t1) / 1e9, 3), "unit": "GB/s", "cores": 1,
                              "sample": "2 passes over the same layer, one host thread"},
               "sample": f"{len(times)} passes over one layer of the stack (7 Q4_K matmuls, 122,683,392 weight bytes), "
                         "batch 1, oracle/qmm_oracle.c (bit-exact restatement of rce-op-qmm mm_1d_q4_k), rows split "
                         "over all host threads as rayon does"}

    if rank == 0:
        clk = clocks.summary(t_wall0, t_wall1) if clocks else {}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "q4_k x f32 (f32 accumulate)",
            "data": "synthetic (seeded, configuration distributions; random weights)",
            "config": config_dict(args, world),
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "hbm", "kernel": f"gemv_kernel<Q4_K> ({dom})",
                         "timing": "32 launches of this matrix back to back in a CUDA graph, CUDA events",
                         "achieved": round(kern[dom]["gbs"], 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(kern[dom]["gbs"] / hbm, 4), "peak_kind": peak_kind,
                         "traffic": traffic,
                         "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum of this kernel from an ncu "
                                           "capture of the same launch (profiles/gemv_q4k_traffic.json), not this run",
                         "alg_bytes_per_launch": kern[dom]["alg_bytes"],
                         "avg_launch_us": round(kern[dom]["avg_us"], 2)},
            "kernels": {nm: {"avg_us": round(v["avg_us"], 2), "gbs": round(v["gbs"], 1)} for nm, v in kern.items()},
            "grouped_launches": groups,
            "stack_frac_of_hbm": round(value / world / hbm, 4),
            "stack_batch16": stack16,
            "prefill_gemm": {
                "workload": f"configs[2]: Q4_K {PREFILL_N}x{PREFILL_K} weight, M f32 activations, fp16 operands, "
                            "f32 accumulation in tensor memory",
                "per_m": prefill,
                "roofline": {"bound": "tensor", "m": 512, "achieved": prefill["m512"]["tflops"], "peak": bf16,
                             "unit": "TFLOP/s", "frac": round(prefill["m512"]["tflops"] / bf16 / max(world, 1), 4),
                             "peak_kind": f"{peak_kind} bf16 dense (burst)"},
            },
            "moe_ffn": moe,
            "formats_gemv": formats,
            "baseline_configs_gemv": base_cfgs,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize(dev)
        dist.barrier()
        pg.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
