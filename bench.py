"""Benchmark of the gated-GQA attention hot path (BASELINE.json metric:
decode attention µs/layer at 32K context and prefill attention TFLOP/s, as a
fraction of the HBM / tensor-core roofline).

Default workload (one "step"): one token of M=1 decode through the 16
full-attention layers of the hybrid decoder, every layer with its own bf16 KV
cache of 32768 positions (the 32K-context decode of the metric; 16 x 134 MB of
KV, larger than the 126 MB L2, so no flush is needed). value = µs per layer.
The same run measures config 2 (4096-token prefill in 8 chunks of 512) and
reports it under "prefill".

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload decode32k|batched|longctx]

N > 1 runs under torchrun, one rank per GPU. The headline decode32k gives
every rank its own sequence (weak scaling, no collective) and reports the
per-GPU µs per layer call of the slowest rank. The same line carries, at every
N, the two multi-GPU splits of the path as nested blocks: "batched" (config 3,
64 sequences sharded over the GPUs, strong scaling) and "longctx" /
"longctx_m3" (config 4, one 262144-position sequence whose KV is split over
the GPUs, partials exchanged through peer memory, strong scaling), each with
its roofline against N x the measured HBM bandwidth.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for sub in ("lisa-rs_b200", "oracle"):
    sys.path.insert(0, os.path.join(ROOT, sub))

METRIC = "decode attn µs/layer @32K ctx & prefill attn TFLOP/s, % of HBM/TC roofline"
UNIT = "µs/layer"
QH, KVH, HD = 24, 4, 256
QROW, KROW, OROW = QH * 512, KVH * HD, QH * HD
LAYERS = 16
CTX = 32768
PREFILL_TOKENS, PREFILL_CHUNK = 4096, 512
PREFILL_FLOP = 4 * QH * HD * sum(range(1, PREFILL_TOKENS + 1))  # causal-exact QK^T + PV
DEEP_BASE = 16384  # the deep-chunk line: one 512-row chunk at this base
DEEP_FLOP = 4 * QH * HD * sum(range(DEEP_BASE + 1, DEEP_BASE + PREFILL_CHUNK + 1))
# DRAM bytes of one decode layer call at ctx 32768 (split kernel read 134.30 MB
# + write 3.46 MB, combine read 2.49 MB), from an ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum) of both kernels.
DECODE_TRAFFIC_32K = 140.24e6
DECODE_TRAFFIC_SOURCE = "ncu capture of both kernels at commit e1fb7d8 (kernels unchanged since in their data path)"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def decode_bytes(ctx: int, rows: int) -> int:
    """Algorithmic HBM bytes of one decode layer: the K and V cache read
    (4 heads x ctx x 256 x 2 B x 2 = 4096 B/token), the q/gate, k, v f32 inputs
    read, the gated bf16 output written and the appended K/V rows written."""
    return 4096 * ctx + rows * (QROW * 4 + 2 * KROW * 4 + OROW * 2 + 2 * KROW * 2)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def _fields(self):
        """The driver names the reasons clocks_event_reasons.* or, on older
        drivers, clocks_throttle_reasons.*; use whichever it accepts."""
        for f in (self.FIELDS, self.FIELDS.replace("clocks_event_reasons", "clocks_throttle_reasons")):
            try:
                r = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={f}", "--format=csv,noheader"],
                                   capture_output=True, text=True, timeout=20)
                if r.returncode == 0:
                    return f
            except Exception:
                pass
        return None

    def __enter__(self):
        try:
            fields = self._fields()
            if fields is None:
                return self
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
def dist_setup():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed(fn, steps, warmup, world, stream):
    """W untimed steps, then K steps bracketed by barrier + synchronize, timed
    with CUDA events on the launching stream; returns max-over-ranks ms."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1), world)


def make_weights(gen, n):
    import torch

    import lisa_attn

    ws = []
    for _ in range(n):
        qn = (1 + 0.02 * torch.randn(HD, generator=gen, device="cuda")).to(torch.bfloat16)
        kn = (1 + 0.02 * torch.randn(HD, generator=gen, device="cuda")).to(torch.bfloat16)
        ws.append(lisa_attn.AttentionWeights(qn, kn))
    return ws


def fill_caches(runner, gen, layers, filled):
    import torch

    for layer in range(layers):
        kc, vc = runner.kv_cache(layer)
        for c in (kc, vc):
            for h in range(KVH):
                c[h, :filled].copy_(torch.randn((filled, HD), generator=gen, device="cuda").to(torch.bfloat16))
    torch.cuda.synchronize()


def bench_decode32k(args, rank, world, local):
    import torch

    import lisa_attn

    stream = torch.cuda.current_stream()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0x5EED + 3 + rank)
    runner = lisa_attn.AttnRunner(LAYERS, CTX)
    fill_caches(runner, gen, LAYERS, CTX - 1)
    ws = make_weights(gen, LAYERS)
    base = CTX - 1
    qs = [torch.randn((1, QROW), generator=gen, device="cuda") for _ in range(LAYERS)]
    ks = [torch.randn((1, KROW), generator=gen, device="cuda") for _ in range(LAYERS)]
    vs = [torch.randn((1, KROW), generator=gen, device="cuda") for _ in range(LAYERS)]
    outs = [torch.empty((1, OROW), dtype=torch.bfloat16, device="cuda") for _ in range(LAYERS)]

    def step_eager():
        for layer in range(LAYERS):
            runner.decode_layer(layer, base, 1, qs[layer], ks[layer], vs[layer], ws[layer], outs[layer], stream)

    # The 16 layer calls of a step are replayed as one CUDA graph so the timed
    # region measures the GPU path rather than Python call overhead (the same
    # kernels and launch parameters; e2e below stays eager).
    step_eager()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            for layer in range(LAYERS):
                runner.decode_layer(layer, base, 1, qs[layer], ks[layer], vs[layer], ws[layer], outs[layer], cap)
    torch.cuda.synchronize()

    def step():
        graph.replay()

    with ClockSampler(local) as clk:
        # keep the GPU under this load long enough for nvidia-smi to sample it
        # (one step is under a millisecond), then the timed region itself
        t_end = time.perf_counter() + 1.5
        while time.perf_counter() < t_end:
            for _ in range(20):
                step()
            torch.cuda.synchronize()
        ms = timed(step, args.steps, args.warmup, world, stream)
    # per-launch duration of the layer call (split-KV kernel + its combine)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(LAYERS)]
    per_layer = []
    for _ in range(max(1, args.steps // 2)):
        for layer in range(LAYERS):
            evs[layer][0].record(stream)
            runner.decode_layer(layer, base, 1, qs[layer], ks[layer], vs[layer], ws[layer], outs[layer], stream)
            evs[layer][1].record(stream)
        torch.cuda.synchronize()
        per_layer += [a.elapsed_time(b) for a, b in evs]
    layer_ms = max_over_ranks(statistics.mean(per_layer), world)

    # end to end through the public API with pinned host buffers: every step
    # copies the 16 layers' f32 inputs (q_gate, k, v) host->device in one
    # transfer from a pinned buffer, makes the 16 layer calls on views of the
    # device copy, and reads the 16 gated outputs back in one transfer
    width = QROW + 2 * KROW
    hin = torch.empty((LAYERS, width), dtype=torch.float32).pin_memory()
    for layer in range(LAYERS):
        hin[layer, :QROW].copy_(qs[layer].view(-1).cpu())
        hin[layer, QROW:QROW + KROW].copy_(ks[layer].view(-1).cpu())
        hin[layer, QROW + KROW:].copy_(vs[layer].view(-1).cpu())
    din = torch.empty((LAYERS, width), dtype=torch.float32, device="cuda")
    dq = [din[layer, :QROW].view(1, QROW) for layer in range(LAYERS)]
    dk = [din[layer, QROW:QROW + KROW].view(1, KROW) for layer in range(LAYERS)]
    dv = [din[layer, QROW + KROW:].view(1, KROW) for layer in range(LAYERS)]
    dout = torch.empty((LAYERS, OROW), dtype=torch.bfloat16, device="cuda")
    douts = [dout[layer].view(1, OROW) for layer in range(LAYERS)]
    hout = torch.empty((LAYERS, OROW), dtype=torch.bfloat16).pin_memory()

    def step_e2e():
        din.copy_(hin, non_blocking=True)
        for layer in range(LAYERS):
            runner.decode_layer(layer, base, 1, dq[layer], dk[layer], dv[layer], ws[layer], douts[layer], stream)
        hout.copy_(dout, non_blocking=True)

    ms_e2e = timed(step_e2e, args.steps, args.warmup, world, stream)
    runner.check_device_error()
    return {"ms": ms, "layer_ms": layer_ms, "ms_e2e": ms_e2e, "clocks": clk.summary(),
            "h2d": LAYERS * (QROW + 2 * KROW) * 4, "d2h": LAYERS * OROW * 2}


def bench_prefill(args, world):
    import torch

    import lisa_attn

    stream = torch.cuda.current_stream()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0x5EED + 2)
    runner = lisa_attn.AttnRunner(1, PREFILL_TOKENS)
    w = make_weights(gen, 1)[0]
    q = torch.randn((PREFILL_TOKENS, QROW), generator=gen, device="cuda").to(torch.bfloat16)
    k = torch.randn((PREFILL_TOKENS, KROW), generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn((PREFILL_TOKENS, KROW), generator=gen, device="cuda").to(torch.bfloat16)
    out = torch.empty((PREFILL_TOKENS, OROW), dtype=torch.bfloat16, device="cuda")
    chunks = [(c * PREFILL_CHUNK, PREFILL_CHUNK) for c in range(PREFILL_TOKENS // PREFILL_CHUNK)]

    def step_eager():
        for b, m in chunks:
            runner.prefill_layer(0, b, m, q[b:b + m], k[b:b + m], v[b:b + m], w, out[b:b + m], stream)

    # The 8 chunk calls are replayed as one CUDA graph (the same kernels and
    # launch parameters) so the timed region measures the GPU path; the eager
    # sequence of library calls is timed as well.
    step_eager()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            for b, m in chunks:
                runner.prefill_layer(0, b, m, q[b:b + m], k[b:b + m], v[b:b + m], w, out[b:b + m], cap)
    torch.cuda.synchronize()

    ms = timed(graph.replay, args.steps, args.warmup, world, stream)
    ms_eager = timed(step_eager, args.steps, args.warmup, world, stream)
    runner.check_device_error()

    # One 512-row chunk deep into the context (base 16384 over a filled
    # cache), captured once with the planner's grid (which splits its units
    # into two key ranges) and once with splitting off.
    deep = lisa_attn.AttnRunner(1, DEEP_BASE + PREFILL_CHUNK)
    kc, vc = deep.kv_cache(0)
    kc.copy_(torch.randn(kc.shape, generator=gen, device="cuda").to(torch.bfloat16))
    vc.copy_(torch.randn(vc.shape, generator=gen, device="cuda").to(torch.bfloat16))
    lib = lisa_attn.load_library()
    deep_ms = {}
    for name, mode in (("auto", 0), ("never", 1)):
        prev = lib.lisa_attn_debug_prefill_split(mode)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap):
            with torch.cuda.graph(g, stream=cap):
                deep.prefill_layer(0, DEEP_BASE, PREFILL_CHUNK, q[:PREFILL_CHUNK], k[:PREFILL_CHUNK],
                                   v[:PREFILL_CHUNK], w, out[:PREFILL_CHUNK], cap)
        lib.lisa_attn_debug_prefill_split(prev)
        torch.cuda.synchronize()
        deep_ms[name] = timed(g.replay, args.steps, args.warmup, world, stream) / args.steps
    deep.check_device_error()
    return ms, ms_eager, deep_ms


def cpu_baseline_decode(seconds: float = 8.0, threads: int | None = None):
    """The oracle (CPU restatement of the reference shaders) on one decode layer
    at ctx 32768, all host threads; returns (µs/layer, threads, reps)."""
    import numpy as np

    import oracle as O

    if threads:
        O.set_num_threads(threads)
    rng = np.random.default_rng(0x5EED)
    qn = O.f32_to_bf16((1 + 0.02 * rng.standard_normal(HD)).astype(np.float32))
    kn = O.f32_to_bf16((1 + 0.02 * rng.standard_normal(HD)).astype(np.float32))
    kc = O.f32_to_bf16(rng.standard_normal((KVH, CTX, HD)).astype(np.float32))
    vc = O.f32_to_bf16(rng.standard_normal((KVH, CTX, HD)).astype(np.float32))
    q = rng.standard_normal((1, QROW)).astype(np.float32)
    k = rng.standard_normal((1, KROW)).astype(np.float32)
    v = rng.standard_normal((1, KROW)).astype(np.float32)
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        O.attention_layer(q, k, v, CTX - 1, qn, kn, kc, vc, sliced=True)
        times.append(time.perf_counter() - t0)
    return statistics.median(times) * 1e6, O.num_threads(), len(times)


def fill_random(t, gen):
    """Seeded N(0,1) bf16 into a large cache tensor without materialising it
    twice: a 64 MB random pool copied with shifting offsets."""
    import torch

    flat = t.view(-1)
    pool = torch.randn(32 << 20, generator=gen, device=t.device).to(torch.bfloat16)
    off, k = 0, 0
    while off < flat.numel():
        n = min(pool.numel() - (k * 4097) % 4096, flat.numel() - off)
        start = (k * 4097) % 4096
        flat[off:off + n].copy_(pool[start:start + n])
        off += n
        k += 1


def bench_longctx(args, rank, world, local, rows=1):
    """one sequence of 262144 positions, one layer, M=1
    (new row at 262143) or the M=3 verify variant (rows at 262141..262143);
    the KV is split into one window per rank (lisa_split.plan_windows) and the
    window partials are exchanged through peer memory inside the step
    (lisa_attn_xchg_decode: split kernel, publishing combine, bounded-wait
    merge). The step is captured in a CUDA graph. Strong scaling: the job is
    one decode step whatever the number of GPUs."""
    import torch

    import lisa_split

    cap = 262144
    base = cap - rows
    stream = torch.cuda.current_stream()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0x5EED + 4 + rank)
    win = lisa_split.plan_windows(cap, world)[rank]
    dec = lisa_split.SplitKVDecoder(win, max_rows=3)
    fill_random(dec.k, gen)
    fill_random(dec.v, gen)
    w = make_weights(gen, 1)[0]
    g0 = torch.Generator(device="cuda")
    g0.manual_seed(0x5EED + rows)  # identical inputs on every rank
    q = torch.randn((rows, QROW), generator=g0, device="cuda")
    k = torch.randn((rows, KROW), generator=g0, device="cuda")
    v = torch.randn((rows, KROW), generator=g0, device="cuda")
    out = torch.empty((rows, OROW), dtype=torch.bfloat16, device="cuda")
    # warm up eagerly, then capture one step (every rank does the same count
    # of steps: each one is an exchange all ranks take part in)
    for _ in range(3):
        dec.decode(base, q, k, v, w, out, stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream()
    with torch.cuda.stream(cs):
        with torch.cuda.graph(graph, stream=cs):
            dec.decode(base, q, k, v, w, out, cs)
    torch.cuda.synchronize()
    barrier(world)
    with ClockSampler(local) as clk:
        for _ in range(200):  # a fixed count, identical on every rank
            graph.replay()
        torch.cuda.synchronize()
        ms = timed(graph.replay, args.steps, args.warmup, world, stream)
    dec.check_device_error()
    return {"ms": ms, "clocks": clk.summary(), "bytes": 4096 * cap + rows * (QROW * 4 + 2 * KROW * 4 + OROW * 2),
            "per_gpu_bytes_max": 4096 * max(w_.rows for w_ in lisa_split.plan_windows(cap, world))}


def bench_batched(args, rank, world, local):
    """64 sequences, contexts U[1024, 32768] (seeded), 16
    attention layers each, M=1; sequences sharded over ranks (lisa_split
    plan_sequences), no collective. Per layer, this rank's sequences go
    through one lisa_attn_decode_batch call (3 launches); the 16 layer calls
    of a step are one CUDA graph. value = µs per layer step (all 64 sequences
    through one layer)."""
    import numpy as np
    import torch

    import lisa_attn
    import lisa_split

    rng = np.random.default_rng(0x5EED + 3)
    ctx = rng.integers(1024, 32769, size=64).tolist()
    mine = lisa_split.plan_sequences(ctx, world)[rank]
    stream = torch.cuda.current_stream()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0x5EED + 30 + rank)
    runners = []
    for i in mine:
        r = lisa_attn.AttnRunner(LAYERS, ctx[i])
        for layer in range(LAYERS):
            kc, vc = r.kv_cache(layer)
            fill_random(kc, gen)
            fill_random(vc, gen)
        runners.append(r)
    bases = [ctx[i] - 1 for i in mine]
    n = len(runners)
    bd = lisa_attn.BatchDecoder(n, sum(ctx[i] for i in mine))
    ws = make_weights(gen, LAYERS)
    q = torch.randn((LAYERS, n, QROW), generator=gen, device="cuda")
    k = torch.randn((LAYERS, n, KROW), generator=gen, device="cuda")
    v = torch.randn((LAYERS, n, KROW), generator=gen, device="cuda")
    out = torch.empty((LAYERS, n, OROW), dtype=torch.bfloat16, device="cuda")

    def step_on(st):
        for layer in range(LAYERS):
            bd.decode(runners, layer, bases, q[layer], k[layer], v[layer], ws[layer], out[layer], st)

    step_on(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap_stream = torch.cuda.Stream()
    with torch.cuda.stream(cap_stream):
        with torch.cuda.graph(graph, stream=cap_stream):
            step_on(cap_stream)
    torch.cuda.synchronize()

    with ClockSampler(local) as clk:
        for _ in range(10):
            graph.replay()
        torch.cuda.synchronize()
        ms = timed(graph.replay, args.steps, args.warmup, world, stream)
    bd.check_device_error()
    total_ctx = sum(ctx)
    return {"ms": ms, "clocks": clk.summary(), "bytes": 4096 * total_ctx * LAYERS, "ctx_sum": total_ctx,
            "launches": 3 * LAYERS}


def bench_qmv(args, world):
    """The fused q/k/v affine-u4 QMV of a decode step (lisa_attn_qmv_u4, M=1,
    hidden 5120 -> 12288 + 1024 + 1024 rows): four layers' weight sets are
    cycled (4 x 41 MB, larger than L2) so every launch streams its weights
    from HBM; one CUDA graph of 16 launches per step."""
    import torch

    import lisa_attn

    k = 5120
    ns = (QROW, KROW, KROW)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0x5EED + 11)
    sets = []
    for _ in range(4):
        projs = []
        for n in ns:
            pk = torch.randint(-2 ** 31, 2 ** 31 - 1, (n, k // 8), generator=gen, device="cuda", dtype=torch.int32)
            sc = (0.01 + 0.01 * torch.rand((n, k // 64), generator=gen, device="cuda")).to(torch.bfloat16)
            bi = (-0.08 * torch.rand((n, k // 64), generator=gen, device="cuda")).to(torch.bfloat16)
            projs.append((pk, sc, bi))
        sets.append(projs)
    x = torch.randn((1, k), generator=gen, device="cuda").to(torch.bfloat16)
    outs = [torch.empty((1, n), dtype=torch.float32, device="cuda") for n in ns]
    stream = torch.cuda.current_stream()
    for i in range(4):
        lisa_attn.qmv_u4(x, sets[i], outs, stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream()
    with torch.cuda.stream(cs):
        with torch.cuda.graph(graph, stream=cs):
            for i in range(16):
                lisa_attn.qmv_u4(x, sets[i % 4], outs, cs)
    torch.cuda.synchronize()
    ms = timed(graph.replay, args.steps, args.warmup, world, stream)
    us = ms * 1000.0 / args.steps / 16
    nbytes = sum(n * (k // 2 + (k // 64) * 4) for n in ns) + k * 2 + sum(ns) * 4
    return us, nbytes


def bench_gdn(args, world):
    """The Gated DeltaNet recurrence of one decode token (lisa_attn_gdn_recurrence,
    M=1, 48 value heads x 128 x 128 f32 state) for the 48 linear-attention
    layers of a step, each with its own state (48 x 3 MB, larger than L2);
    one CUDA graph per step. Returns (µs per layer call, algorithmic bytes)."""
    import torch

    import lisa_attn

    vh, kh, d, layers = 48, 16, 128, 48
    conv_dim = 2 * kh * d + vh * d
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0x5EED + 12)
    states = [0.1 * torch.randn((vh, d, d), generator=gen, device="cuda") for _ in range(layers)]
    conv = torch.randn((1, conv_dim), generator=gen, device="cuda")
    q = torch.randn((1, kh * d), generator=gen, device="cuda") / d
    k = torch.randn((1, kh * d), generator=gen, device="cuda") / d ** 0.5
    beta = torch.sigmoid(torch.randn((1, vh), generator=gen, device="cuda"))
    decay = torch.full((1, vh), 0.95, device="cuda")
    y = torch.empty((1, vh * d), device="cuda")
    stream = torch.cuda.current_stream()
    lisa_attn.gdn_recurrence(conv, q, k, beta, decay, states[0], y, vh, vh // kh, stream=stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream()
    with torch.cuda.stream(cs):
        with torch.cuda.graph(graph, stream=cs):
            for st in states:
                lisa_attn.gdn_recurrence(conv, q, k, beta, decay, st, y, vh, vh // kh, stream=cs)
    torch.cuda.synchronize()
    ms = timed(graph.replay, args.steps, args.warmup, world, stream)
    us = ms * 1000.0 / args.steps / layers
    nbytes = 2 * vh * d * d * 4 + (conv_dim + 2 * kh * d + 2 * vh + vh * d) * 4
    return us, nbytes


def emit(line: dict) -> None:
    print(json.dumps(line), flush=True)


def run_reference(args, rank, world):
    """--impl reference: the reference's attention math on the host cores (the
    oracle port: lisa-rs is Metal-only and its Rust cannot be built here), one
    32K decode layer per step, on rank 0 only."""
    if rank != 0:
        return
    import oracle as O

    threads = os.cpu_count() or 1
    O.set_num_threads(threads)
    us, nthr, _ = cpu_baseline_decode(seconds=0.1, threads=threads)  # warm-up (page in, OpenMP pool)
    samples = []
    for _ in range(max(0, args.warmup - 1)):
        cpu_baseline_decode(seconds=0.0, threads=threads)
    for _ in range(args.steps):
        us, nthr, _ = cpu_baseline_decode(seconds=0.0, threads=threads)
        samples.append(us)
    value = statistics.mean(samples)
    sample = f"one M=1 decode layer at ctx {CTX} per step (1/16 of a decode32k step), oracle port, {nthr} threads"
    emit({"impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": args.gpus,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(value / 1000, 3),
          "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
          "config": {"workload": "decode32k", "ctx": CTX, "rows": 1, "layers_per_step": 1},
          "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": nthr, "kind": "port", "sample": sample},
          "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode32k", choices=["decode32k", "batched", "longctx", "qmv", "gdn"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decode-only", action="store_true", help="skip the batched / longctx blocks")
    ap.add_argument("--rows", type=int, default=1, choices=[1, 3], help="rows of --workload longctx")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        run_reference(args, rank, world)
        return

    import torch

    rank, world, local = dist_setup()
    pk = peaks()
    hbm_job = pk["hbm_gbs"] * world

    def split_block(r, kind):
        """Nested line of a multi-GPU split (config 3 or 4): whole-job time,
        roofline against world x measured HBM."""
        step_us = r["ms"] * 1000.0 / args.steps
        gbs = r["bytes"] / (step_us * 1e-6) / 1e9
        blk = {"ms_per_step": round(step_us / 1000, 4), "higher_is_better": False, "scaling": "strong",
               "n_gpus": world, "clocks": r["clocks"],
               "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": round(hbm_job, 1), "unit": "GB/s",
                            "frac": round(gbs / hbm_job, 4), "traffic": None, "peak_source": pk["source"],
                            "note": f"whole job: algorithmic bytes / step time, peak = {world} x measured HBM"}}
        if kind == "batched":
            blk.update({"workload": "config 3: 64 sequences, ctx U[1024,32768] seeded (sum %d), 16 attention "
                                    "layers, M=1; sequences sharded over the GPUs, no collective; one CUDA graph "
                                    "per step" % r["ctx_sum"],
                        "value": round(step_us / LAYERS, 3), "unit": "µs/layer (all 64 sequences)",
                        "launches_per_step": r["launches"]})
        else:
            blk.update({"workload": "config 4: one sequence, ctx 262144, rows %d; KV split into one window per "
                                    "GPU, window partials exchanged by peer stores + bounded-wait merge inside the "
                                    "step (no collective library call); one CUDA graph per step" % r["rows"],
                        "value": round(step_us, 3), "unit": "µs/step (one layer)",
                        "per_gpu_kv_bytes": r["per_gpu_bytes_max"]})
        return blk

    if args.workload in ("qmv", "gdn"):
        us, nbytes = (bench_qmv if args.workload == "qmv" else bench_gdn)(args, world)
        gbs = nbytes / (us * 1e-6) / 1e9
        if rank == 0:
            emit({"metric": METRIC, "value": round(us, 3), "unit": "µs/launch", "n_gpus": world, "steps": args.steps,
                  "warmup": args.warmup, "higher_is_better": False, "dtype": "f32", "data": "synthetic",
                  "config": {"workload": args.workload},
                  "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                               "frac": round(gbs / pk["hbm_gbs"], 4), "algorithmic_bytes": nbytes}})
        return
    if args.workload in ("batched", "longctx"):
        r = bench_batched(args, rank, world, local) if args.workload == "batched" else \
            bench_longctx(args, rank, world, local, rows=args.rows)
        if args.workload == "longctx":
            r["rows"] = args.rows
        if rank == 0:
            blk = split_block(r, args.workload)
            emit({"metric": METRIC, "value": blk["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
                  "warmup": args.warmup, "ms_per_step": blk["ms_per_step"], "higher_is_better": False,
                  "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                  "config": {"workload": blk["workload"], "parallelism": f"{world} ranks"},
                  "roofline": blk["roofline"], "clocks": blk["clocks"]})
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    r = bench_decode32k(args, rank, world, local)
    torch.cuda.empty_cache()
    pf_ms, pf_ms_eager, deep_ms = bench_prefill(args, world)
    torch.cuda.empty_cache()
    qmv_us, qmv_bytes = bench_qmv(args, world)
    gdn_us, gdn_bytes = bench_gdn(args, world)
    torch.cuda.empty_cache()
    blocks = {}
    if not args.decode_only:
        rb = bench_batched(args, rank, world, local)
        blocks["batched"] = split_block(rb, "batched")
        torch.cuda.empty_cache()
        for rows in (1, 3):
            rl = bench_longctx(args, rank, world, local, rows=rows)
            rl["rows"] = rows
            blocks["longctx" if rows == 1 else "longctx_m3"] = split_block(rl, "longctx")
            torch.cuda.empty_cache()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        us, nthr, reps = cpu_baseline_decode(seconds=10.0)
        cpu = {"value": round(us, 2), "unit": UNIT, "cores": nthr, "kind": "port",
               "sample": f"{reps} oracle runs of one M=1 decode layer at ctx {CTX} (median)"}
    if rank != 0:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    # per-GPU figures: every rank decodes its own 32K sequence (weak scaling),
    # the slowest rank's time is reported
    value = r["ms"] * 1000.0 / args.steps / LAYERS  # µs per layer call on one GPU
    e2e = r["ms_e2e"] * 1000.0 / args.steps / LAYERS
    layer_bytes = decode_bytes(CTX, 1)
    # average duration of one layer call (split + combine) over the timed
    # region: K steps x 16 back-to-back calls, CUDA events on the stream
    achieved = layer_bytes / (value * 1e-6) / 1e9
    pf_tflops = PREFILL_FLOP / (pf_ms / args.steps * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(r["ms"] / args.steps, 4), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "decode32k: M=1 decode, ctx 32768, 16 stacked attention layers per step, "
                               "one sequence per GPU (value = per-GPU µs per layer call, slowest rank), "
                               "step replayed as a CUDA graph", "ctx": CTX, "rows": 1, "layers": LAYERS,
                   "sequences": world, "parallelism": f"sequences sharded, dp{world}, no collective",
                   "l2": "inputs larger than L2 (16 x 134 MB KV per step)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": DECODE_TRAFFIC_32K,
                     "traffic_source": DECODE_TRAFFIC_SOURCE, "peak_source": pk["source"],
                     "kernel": "decode_split_kernel<1> + decode_combine_kernel (one layer call, one GPU)",
                     "algorithmic_bytes": layer_bytes, "layer_us_timed": round(value, 3),
                     "layer_us_isolated": round(r["layer_ms"] * 1000, 3)},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e, 3), "unit": UNIT, "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]},
        "gpu_launches": 2 * LAYERS * args.steps,
        "clocks": r["clocks"],
        "prefill": {"workload": "config 2: 4096 tokens, 8 chunks of 512, one layer; the 8 chunk calls replayed "
                                "as a CUDA graph", "ms": round(pf_ms / args.steps, 4),
                    "ms_eager_calls": round(pf_ms_eager / args.steps, 4),
                    "tflops": round(pf_tflops, 2), "flop": PREFILL_FLOP,
                    "frac_burst": round(pf_tflops / pk["bf16_tflops"], 4),
                    "frac_sustained": round(pf_tflops / pk["bf16_tflops_sustained"], 4),
                    "roofline": {"bound": "tensor", "achieved": round(pf_tflops, 2), "peak": pk["bf16_tflops"],
                                 "unit": "TFLOP/s", "frac": round(pf_tflops / pk["bf16_tflops"], 4), "traffic": None,
                                 "kernel": "prefill_prologue_kernel + prefill_attn_kernel, 8 chunk calls"},
                    "gpu_launches_per_step": 2 * (PREFILL_TOKENS // PREFILL_CHUNK),
                    "deep_chunk": {"workload": f"one 512-row chunk at base {DEEP_BASE} over a filled cache, "
                                               "CUDA graph; grid as planned (key ranges split) and unsplit",
                                   "ms": round(deep_ms["auto"], 4), "ms_unsplit": round(deep_ms["never"], 4),
                                   "tflops": round(DEEP_FLOP / (deep_ms["auto"] * 1e-3) / 1e12, 2),
                                   "tflops_unsplit": round(DEEP_FLOP / (deep_ms["never"] * 1e-3) / 1e12, 2),
                                   "frac_burst": round(DEEP_FLOP / (deep_ms["auto"] * 1e-3) / 1e12
                                                       / pk["bf16_tflops"], 4)}},
    }
    qmv_gbs = qmv_bytes / (qmv_us * 1e-6) / 1e9
    line["qmv"] = {"workload": "fused q/k/v affine-u4 QMV of one decode step (lisa_attn_qmv_u4, M=1, 5120 -> "
                               "12288+1024+1024), 4 weight sets cycled (164 MB > L2), 16 launches per CUDA graph",
                   "us_per_launch": round(qmv_us, 3), "algorithmic_bytes": qmv_bytes,
                   "roofline": {"bound": "hbm", "achieved": round(qmv_gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                                "frac": round(qmv_gbs / pk["hbm_gbs"], 4), "traffic": None}}
    gdn_gbs = gdn_bytes / (gdn_us * 1e-6) / 1e9
    line["gdn"] = {"workload": "Gated DeltaNet recurrence of one decode token for 48 layers, each its own 3 MB f32 "
                               "state (144 MB > L2), 48 launches per CUDA graph (lisa_attn_gdn_recurrence)",
                   "us_per_layer": round(gdn_us, 3), "algorithmic_bytes": gdn_bytes,
                   "roofline": {"bound": "hbm", "achieved": round(gdn_gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                                "frac": round(gdn_gbs / pk["hbm_gbs"], 4), "traffic": None}}
    line.update(blocks)
    emit(line)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
