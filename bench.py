"""Benchmark of the paged decode-attention path on B200 (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c1|c3|c4|c4p|c5|s2|c2d|c3d] [--driver]

Default workload: BASELINE config 2 (Qwen2.5-0.5B shape batched ragged decode:
64 sequences per GPU, 14 q heads / 2 KV heads, head_dim 64, context lengths
U[256, 4096], 16-token pages from a shuffled shared pool, 512-token split-K
partitions, 24 layers). One step = one decode step of all 24 layers: per layer
ONE launch, lc_rope_append_decode, which adds the biases to the new token's
q/k/v, rotates q and k, appends k and v to the paged cache and runs the paged
attention over the cache (the two-launch form, lc_rope_append then
lc_paged_decode, is `--unfused`). Multi-GPU: weak scaling, the global batch of
64*N sequences is sharded by sequence (longest-first bin packing,
lc_shard_sequences); no collective on the data path.

`value` is decode-attention KV GB/s summed over ranks (each unique KV byte
counted once per layer), inputs resident in HBM, timed with CUDA events over K
replays of a CUDA graph of the step, max over ranks. `e2e` is the same metric
through the C ABI with the step's inputs copied from pinned host memory and its
outputs copied back inside the timed region. The 24 per-layer caches total
~1.7 GB per GPU (> 126 MB L2), so no L2 flush is needed between steps.

`--impl reference` runs the reference's own kernels (compiled unchanged from
its sources into oracle/_ref) the way the reference launches them: per
sequence, rope -> update_kv_cache -> flash_decoding, one launch each. It loads
only oracle/_ref (its RoPE tables come from that library's host code) and, on
N ranks, rank 0 runs the whole global batch on its GPU.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "lucciola-rs_b200"), str(ROOT / "tests")]

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "decode-attn KV GB/s & % HBM peak; tokens/s at batch 64, 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0

CONFIGS = {
    # name: (workload label, batch per rank, Hq, Hkv, hd, layers, ctx spec, partition tokens)
    "c2": ("qwen2.5-0.5b batched ragged decode (BASELINE config 2)", 64, 14, 2, 64, 24,
           ("uniform", 256, 4096), 512),
    "c1": ("qwen2.5-0.5b single-sequence decode (BASELINE config 1)", 1, 14, 2, 64, 24,
           ("fixed", 1024), 0),
    "c3": ("qwen2.5-7b batched decode (BASELINE config 3)", 32, 28, 4, 128, 28,
           ("fixed", 8192), 512),
}


# ------------------------------------------------------------------ helpers --

def host_link_gbs(device, nbytes=16 << 20, reps=5):
    """This box's pinned host <-> device copy bandwidth (median of `reps`
    copies of `nbytes` each way, CUDA events), reported beside `e2e`: the
    end-to-end number moves with it from box to box."""
    import torch
    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(nbytes, dtype=torch.uint8, device=device)
    res = {}
    for name, fn in (("h2d_gbs", lambda: d.copy_(h, non_blocking=True)),
                     ("d2h_gbs", lambda: h.copy_(d, non_blocking=True))):
        fn()
        torch.cuda.synchronize(device)
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        res[name] = round(nbytes / (sorted(ts)[reps // 2] * 1e-3) / 1e9, 2)
    res["bytes_per_copy"] = nbytes
    return res


def env_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the GPU is loaded."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(device_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for line in out.splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), max=float(parts[2]), power=float(parts[3]),
                                 hw=parts[5], hwt=parts[6], swt=parts[7], pcap=parts[8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = set()
        for r in rows:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in rows),
                "sm_max_mhz": max(r["max"] for r in rows), "reasons": sorted(reasons),
                "samples": len(rows), "power_w_max": max(r["power"] for r in rows)}


# ----------------------------------------------------------------- workload --

class Workload:
    """Synthetic paged decode batch for one rank, resident on the GPU."""

    def __init__(self, cfg_name: str, rank: int, world: int, device, seed: int = 1234,
                 layers: int | None = None, rope_table=None, shard: bool = True):
        """`rope_table(max_pos, head_dim, base) -> (cos, sin)` builds the RoPE
        tables (the product library's by default). With shard=False this
        process takes the whole global batch of batch_per_rank * world
        sequences (the reference arm, which runs on one GPU)."""
        (self.label, self.batch_per_rank, self.hq, self.hkv, self.hd, self.layers, ctx_spec,
         self.ptok) = CONFIGS[cfg_name]
        if layers:
            self.layers = layers
        self.cfg_name = cfg_name
        rng = np.random.default_rng(seed)
        global_batch = self.batch_per_rank * world
        if ctx_spec[0] == "fixed":
            ctx_all = np.full(global_batch, ctx_spec[1], np.int32)
        else:
            ctx_all = rng.integers(ctx_spec[1], ctx_spec[2] + 1, global_batch).astype(np.int32)
        if world > 1 and shard:
            import lucciola as L
            owner = np.array(L.shard_sequences(ctx_all.tolist(), world))
        else:
            owner = np.zeros(global_batch, np.int64)
            rank = 0
        self.global_batch = global_batch
        self.global_kv_tokens = int(ctx_all.sum() + global_batch)
        self.ctx = ctx_all[owner == rank].astype(np.int32)  # cached tokens before this step
        self.batch = len(self.ctx)
        self.device = device
        hd, hq, hkv, L_ = self.hd, self.hq, self.hkv, self.layers
        gen = torch.Generator(device=device)
        gen.manual_seed(seed + 7919 * rank)
        # Pages: room for the context plus the token appended this step.
        pages = (self.ctx + 1 + 15) // 16
        self.num_blocks = int(pages.sum()) + 1
        perm = torch.randperm(self.num_blocks, generator=gen, device=device).to(torch.int32).cpu().numpy()
        self.max_pages = int(pages.max())
        tables = np.full((self.batch, self.max_pages), -1, np.int32)
        off = 0
        for b, n in enumerate(pages):
            tables[b, :n] = perm[off:off + n]
            off += n
        self.tables_np = tables
        self.tables = torch.from_numpy(tables).to(device)
        self.positions_np = self.ctx.copy()  # the new token's position
        self.positions = torch.from_numpy(self.positions_np).to(device)
        self.max_ctx = int(self.ctx.max()) + 1
        shape = (self.num_blocks, L_, hkv, 16, hd)
        self.k_pool = torch.empty(shape, dtype=torch.bfloat16, device=device)
        self.v_pool = torch.empty(shape, dtype=torch.bfloat16, device=device)
        for t in (self.k_pool, self.v_pool):
            flat = t.view(-1)
            step = 1 << 28
            for i in range(0, flat.numel(), step):
                chunk = flat[i:i + step]
                chunk.copy_(torch.randn(chunk.numel(), generator=gen, device=device,
                                        dtype=torch.float32).to(torch.bfloat16))
        self.row = (hq + 2 * hkv) * hd
        self.qkv = torch.randn((L_, self.batch, self.row), generator=gen, device=device).to(torch.bfloat16)
        bias = torch.randn((L_, self.row), generator=gen, device=device) * 0.01
        self.q_bias = bias[:, :hq * hd].to(torch.bfloat16).contiguous()
        self.k_bias = bias[:, hq * hd:(hq + hkv) * hd].to(torch.bfloat16).contiguous()
        self.v_bias = bias[:, (hq + hkv) * hd:].to(torch.bfloat16).contiguous()
        self.out = torch.empty((L_, self.batch, hq * hd), dtype=torch.bfloat16, device=device)
        if rope_table is None:
            import lucciola as L
            rope_table = L.rope_table_host
        cos, sin = rope_table(32768, hd, 1e6)
        self.cos = torch.from_numpy(cos).to(device)
        self.sin = torch.from_numpy(sin).to(device)
        # bytes: each unique KV byte of the attended context, once per layer
        self.kv_bytes_per_layer = int((self.ctx.astype(np.int64) + 1).sum()) * hkv * hd * 2 * 2
        self.kv_bytes_per_step = self.kv_bytes_per_layer * L_
        self.h2d_bytes = self.qkv.numel() * 2 + self.positions.numel() * 4
        self.d2h_bytes = self.out.numel() * 2


def workload_config(w: Workload, world: int) -> dict:
    """The `config` object of both arms' JSON lines (the workload, not the
    implementation; each line's `step` key says how it was run)."""
    return {"workload": w.label, "batch_per_gpu": w.batch_per_rank,
            "global_batch": w.global_batch, "q_heads": w.hq, "kv_heads": w.hkv,
            "head_dim": w.hd, "layers": w.layers, "page_tokens": 16,
            "partition_tokens": w.ptok or "auto",
            "kv_tokens_per_layer": w.global_kv_tokens,
            "parallelism": f"sequence-sharded x{world}",
            "l2": "no flush: %d per-layer caches, ~%.1f GB per GPU > 126 MB L2" %
                  (w.layers, w.global_kv_tokens * w.hkv * w.hd * 4 * w.layers / world / 1e9)}


# ------------------------------------------------------------------ our arm --

class OursStep:
    """One decode step: per layer the fused bias+RoPE+append+attention launch
    (lc_rope_append_decode), or with fused=False the two-launch form
    (lc_rope_append, then lc_paged_decode)."""

    def __init__(self, w: Workload, fused: bool = True):
        import lucciola as L
        self.L = L
        self.w = w
        self.fused = fused
        self.ws = L.alloc_decode_workspace(w.batch, w.hq, w.hkv, w.hd, device=w.device)

    def layer(self, l, decode_events=None, out=None, gate=None):
        w, L = self.w, self.L
        out = w.out[l] if out is None else out
        if not self.fused:
            L.rope_append(w.qkv[l], w.positions, w.q_bias[l], w.k_bias[l], w.v_bias[l], w.cos,
                          w.sin, w.k_pool, w.v_pool, w.num_blocks, w.layers, l, w.hq, w.hkv,
                          w.hd, w.tables)
        if decode_events is not None:
            decode_events[0].record()
        if self.fused:
            L.rope_append_decode(out, w.qkv[l], w.positions, w.q_bias[l], w.k_bias[l],
                                 w.v_bias[l], w.cos, w.sin, w.k_pool, w.v_pool, w.num_blocks,
                                 w.layers, l, w.hq, w.hkv, w.hd, w.tables, w.max_ctx,
                                 partition_tokens=w.ptok, workspace=self.ws, gate=gate)
        else:
            L.paged_decode(out, w.qkv[l], w.k_pool, w.v_pool, w.num_blocks, w.layers, l,
                           w.hq, w.hkv, w.hd, w.tables, w.positions, w.max_ctx, len_offset=1,
                           partition_tokens=w.ptok, workspace=self.ws)
        if decode_events is not None:
            decode_events[1].record()

    def step(self):
        for l in range(self.w.layers):
            self.layer(l)

    launches_per_step = property(lambda self: (1 if self.fused else 2) * self.w.layers)


def time_graph(graph, steps, warmup, stream):
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def decode_kernel_time(runner, reps):
    """Average duration of one lc_paged_decode launch: CUDA events around each
    launch, launches queued behind a sleep so host latency is not timed."""
    w = runner.w
    pairs = []
    torch.cuda.synchronize()
    torch.cuda._sleep(50_000_000)
    for _ in range(reps):
        for l in range(w.layers):
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            runner.layer(l, decode_events=ev)
            pairs.append(ev)
    torch.cuda.synchronize()
    times = [a.elapsed_time(b) for a, b in pairs]
    return sum(times) / len(times)


def cpu_baseline(w: Workload, budget_s: float = 12.0):
    """The CPU oracle (restatement of the reference algorithm) on a bounded
    sample of the same workload: all sequences of this rank, one layer per
    repetition, all host cores."""
    import oracle.oracle as O
    from workloads import randn_bf16
    rng = np.random.default_rng(99)
    hq, hkv, hd = w.hq, w.hkv, w.hd
    pages = (w.ctx + 1 + 15) // 16
    nb = int(pages.sum()) + 1
    tables = np.full((w.batch, int(pages.max())), -1, np.int32)
    perm = rng.permutation(nb).astype(np.int32)
    off = 0
    for b, n in enumerate(pages):
        tables[b, :n] = perm[off:off + n]
        off += n
    k_pool = randn_bf16(rng, (nb, 1, hkv, 16, hd))
    v_pool = randn_bf16(rng, (nb, 1, hkv, 16, hd))
    qkv = randn_bf16(rng, (w.batch, w.row))
    qb, kb, vb = (randn_bf16(rng, (n * hd,)) for n in (hq, hkv, hkv))
    cos, sin = O.rope_table(int(w.ctx.max()) + 2, hd, 1e6)
    threads = os.cpu_count() or 1

    def timed(nthreads, budget):
        reps, t0 = 0, time.perf_counter()
        while True:
            x = qkv.copy()
            O.rope_append(x, w.positions_np, qb, kb, vb, cos, sin, k_pool, v_pool, 1, 0, hq, hkv,
                          hd, tables)
            O.paged_decode(x, k_pool, v_pool, 0, hq, hkv, hd, tables, w.positions_np, 1,
                           len_offset=1, threads=nthreads)
            reps += 1
            if time.perf_counter() - t0 >= budget or reps >= 64:
                break
        return reps, time.perf_counter() - t0

    reps, dt = timed(threads, budget_s)
    reps1, dt1 = timed(1, budget_s / 3)  # the scalar restatement on one core
    return {"value": round(w.kv_bytes_per_layer * reps / dt / 1e9, 3), "unit": "GB/s",
            "cores": threads, "kind": "port",
            "single_core_value": round(w.kv_bytes_per_layer * reps1 / dt1 / 1e9, 3),
            "sample": f"{reps} x one layer of the rank-0 batch ({w.batch} sequences, "
                      f"{int(w.ctx.sum() + w.batch)} KV tokens) through the CPU oracle "
                      f"(oracle/lc_oracle.c: rope+append, then decode attention split by "
                      f"(sequence, head) over {threads} threads), {dt:.1f} s; single core: "
                      f"{reps1} x in {dt1:.1f} s"}


def run_ours(args, rank, world, local):
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
    import lucciola as L
    L.set_dependent_launch(args.pdl)
    w = Workload(args.config, rank, world, device, layers=args.layers)
    if args.partition is not None:
        w.ptok = args.partition
    runner = OursStep(w, fused=not args.unfused)
    if args.mode == "kernel":
        # Plain eager launches, nothing else: the command profiled by ncu.
        for _ in range(args.warmup + args.steps):
            runner.step()
        torch.cuda.synchronize()
        if rank == 0:
            print(json.dumps({"mode": "kernel", "config": args.config, "steps": args.steps,
                              "warmup": args.warmup, "launches_per_step": runner.launches_per_step}))
        if dist:
            dist.destroy_process_group()
        return
    # eager warm-up: caches tensor maps and kernel attributes before capture
    for _ in range(2):
        runner.step()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        runner.step()
    torch.cuda.synchronize()

    # settle clocks under this load and keep sampling through the timed region
    sampler = ClockSampler(local) if rank == 0 else None
    t_end = time.perf_counter() + 1.0
    while time.perf_counter() < t_end:
        for _ in range(20):
            graph.replay()
        torch.cuda.synchronize()

    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ms_total = time_graph(graph, args.steps, args.warmup, torch.cuda.current_stream())
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms_step = ms_total / args.steps

    # e2e: the step's inputs come from pinned host memory and its outputs go
    # back, through the same C-ABI calls, inside the timed region. The whole
    # step, transfers included, is one CUDA graph. Inputs go in groups of 1, 2,
    # 4, 8, ... layers (the first layer starts after one layer's copy).
    qkv_host = w.qkv.cpu().pin_memory()
    pos_host = w.positions.cpu().pin_memory()
    comp_s, copy_s = torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)
    groups, g0, size = [], 0, 1
    while g0 < w.layers:
        groups.append((g0, min(g0 + size, w.layers)))
        g0, size = g0 + size, size * 2
    host_out = None
    g_e2e = torch.cuda.CUDAGraph()
    if runner.fused:
        # Fused step: each group's copy is followed on the copy stream by a
        # 4-byte copy that sets the group's gate; each layer's launch waits for
        # its gate on the device before it reads its rows, so the compute stream
        # holds decode launches only and keeps their programmatic overlap. The
        # launches write their outputs straight into mapped pinned host memory.
        from cuda.bindings import runtime as cudart
        nbytes = w.out.numel() * 2
        err, hptr = cudart.cudaHostAlloc(nbytes, cudart.cudaHostAllocMapped)
        assert int(err) == 0, err
        err, dptr = cudart.cudaHostGetDevicePointer(hptr, 0)
        assert int(err) == 0 and int(dptr) == int(hptr), (err, dptr, hptr)
        import ctypes
        host_out = hptr
        out_host = torch.frombuffer((ctypes.c_uint8 * nbytes).from_address(int(hptr)),
                                    dtype=torch.bfloat16).view(w.out.shape)
        gates = torch.zeros(len(groups), dtype=torch.int32, device=device)
        one_host = torch.ones(1, dtype=torch.int32).pin_memory()
        group_of = {l: gi for gi, (a, b) in enumerate(groups) for l in range(a, b)}
        with torch.cuda.graph(g_e2e, stream=comp_s):
            copy_s.wait_stream(comp_s)
            w.positions.copy_(pos_host, non_blocking=True)  # read by the launches' set-up
            with torch.cuda.stream(copy_s):
                for gi, (a, b) in enumerate(groups):
                    w.qkv[a:b].copy_(qkv_host[a:b], non_blocking=True)
                    gates[gi:gi + 1].copy_(one_host, non_blocking=True)
            for l in range(w.layers):
                runner.layer(l, out=out_host[l], gate=gates[group_of[l]:group_of[l] + 1])
            comp_s.wait_stream(copy_s)
            gates.zero_()  # closed again for the next step
        e2e_how = ("pinned host qkv/positions in (qkv in groups of 1, 2, 4, ... layers on a copy "
                   "stream, each group opening a device gate the layer's launch waits on); the "
                   "launches write their outputs into mapped pinned host memory; one CUDA graph")
    else:
        # Two-launch step: cross-stream waits on the copies; outputs go back in
        # the mirrored groups (..., 4, 2, 1 layers), each as soon as its last
        # layer is done.
        out_host = torch.empty(w.out.shape, dtype=w.out.dtype).pin_memory()
        out_groups, g1 = [], w.layers
        for a, b in groups:
            out_groups.append((g1 - (b - a), g1))
            g1 -= b - a
        out_end = {b - 1: (a, b) for a, b in out_groups}
        with torch.cuda.graph(g_e2e, stream=comp_s):
            copy_s.wait_stream(comp_s)
            ev_in = {}
            with torch.cuda.stream(copy_s):
                w.positions.copy_(pos_host, non_blocking=True)
                for a, b in groups:
                    w.qkv[a:b].copy_(qkv_host[a:b], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(copy_s)
                    ev_in[a] = ev
            for l in range(w.layers):
                if l in ev_in:
                    comp_s.wait_event(ev_in[l])
                runner.layer(l)
                if l in out_end:
                    a, b = out_end[l]
                    ev = torch.cuda.Event()
                    ev.record(comp_s)
                    copy_s.wait_event(ev)
                    with torch.cuda.stream(copy_s):
                        out_host[a:b].copy_(w.out[a:b], non_blocking=True)
            comp_s.wait_stream(copy_s)
        e2e_how = ("pinned host qkv/positions in (groups of 1, 2, 4, ... layers), outputs out "
                   "(mirrored groups), on a copy stream overlapped with the compute stream; one "
                   "CUDA graph")
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e2e_ms_step = time_graph(g_e2e, args.steps, args.warmup, torch.cuda.current_stream()) / args.steps

    # per-launch duration of the dominant kernel (roofline)
    dec_ms = decode_kernel_time(runner, max(2, min(args.steps, 8)))

    vals = torch.tensor([ms_step, e2e_ms_step, dec_ms, float(w.kv_bytes_per_step)],
                        dtype=torch.float64, device=device)
    if dist:
        mx = vals[:3].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = vals[3:].clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        ms_step, e2e_ms_step, dec_ms = mx.tolist()
        kv_bytes_all = tot.item()
    else:
        kv_bytes_all = float(w.kv_bytes_per_step)

    if rank == 0:
        peak, peak_kind = measured_peak()
        link = host_link_gbs(device)  # after the timed regions
        value = kv_bytes_all / (ms_step * 1e-3) / 1e9
        e2e_value = kv_bytes_all / (e2e_ms_step * 1e-3) / 1e9
        # Dominant kernel's average launch duration over the timed region: the
        # fused step's graph holds nothing but its `layers` decode launches.
        # The unfused step also holds lc_rope_append launches, so there the
        # isolated single-launch duration stands in.
        launch_ms = ms_step / w.layers if runner.fused else dec_ms
        achieved = w.kv_bytes_per_layer / (launch_ms * 1e-3) / 1e9
        isolated = w.kv_bytes_per_layer / (dec_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded bf16 ~N(0,1) K/V/Q, uniform context lengths)",
            "config": workload_config(w, world),
            "step": ("per layer: lc_rope_append + lc_paged_decode" if args.unfused else
                     "per layer: lc_rope_append_decode (fused bias+RoPE+append+attention)") +
                    "; CUDA graph" +
                    (f"; programmatic dependent launch mode {args.pdl}" if args.pdl else ""),
            "tokens_per_s": round(w.global_batch / (ms_step * 1e-3), 1),
            "pct_hbm": round(100 * value / world / peak, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": TRAFFIC.get(args.config),
                         "kernel": "paged_decode_kernel<%d,%s>" % (w.hd, "fused" if runner.fused else "plain"),
                         "peak_kind": f"{peak_kind} (burst copy)",
                         "launch_ms": round(launch_ms, 5),
                         "launch_timing": ("CUDA events over the timed region / decode launches "
                                           "in it (the graph holds only this kernel)"
                                           if runner.fused else
                                           "CUDA events around single launches"),
                         "isolated_launch_ms": round(dec_ms, 5),
                         "isolated_achieved": round(isolated, 1),
                         "isolated_frac": round(isolated / peak, 4),
                         "isolated_timing": "CUDA events around single launches queued behind "
                                            "a GPU sleep (no overlap with neighbouring layers)"},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": int(w.h2d_bytes), "d2h_bytes_per_step": int(w.d2h_bytes),
                    "ms_per_step": round(e2e_ms_step, 5),
                    "how": e2e_how, "host_link": link},
            "gpu_launches": runner.launches_per_step * args.steps,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(w)
        else:
            line["cpu_baseline"] = None
        print(json.dumps(line), flush=True)
    del graph, g_e2e
    if host_out is not None:
        torch.cuda.synchronize()
        from cuda.bindings import runtime as cudart
        cudart.cudaFreeHost(host_out)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_driver(args, rank, world, local):
    """The decode workload through the batched token-step driver (lc_kv_pool):
    the pool hands out the pages (all sequences grown together, so each
    sequence's pages interleave with the others'), and every step is the token
    loop a server runs: lc_kv_pool_prepare_step on the host (page reservation,
    table and position upload), then one replay of a CUDA graph holding the
    layers' lc_kv_pool_decode_layer launches. Positions advance by one token per
    step, so the context grows and new pages are taken as sequences cross page
    boundaries. Timed with CUDA events around K steps, host work included."""
    import lucciola as L
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
    L.set_dependent_launch(args.pdl)
    w = Workload(args.config, rank, world, device)
    settle_steps = 400
    total_steps = 2 + settle_steps + args.warmup + args.steps
    B, ctx = w.batch, w.ctx.astype(np.int64)
    max_seq_len = int(ctx.max()) + total_steps + 16
    num_blocks = int(((ctx + total_steps + 15) // 16).sum()) + B
    del w.k_pool, w.v_pool
    torch.cuda.empty_cache()
    pool = L.KVPool(w.layers, w.hq, w.hkv, w.hd, B, max_seq_len, num_blocks)
    slots = [pool.add_sequence() for _ in range(B)]
    # reserve the cached context a page round at a time across all sequences
    for k in range(1, (int(ctx.max()) + 15) // 16 + 1):
        pos = np.minimum(ctx, 16 * k) - 1
        pool.prepare_step(slots, pos.tolist())
    kp, vp = pool.pools()
    gen = torch.Generator(device=device)
    gen.manual_seed(4242 + rank)
    for t in (kp, vp):
        flat = t.view(-1)
        for i in range(0, flat.numel(), 1 << 28):
            chunk = flat[i:i + (1 << 28)]
            chunk.copy_(torch.randn(chunk.numel(), generator=gen, device=device,
                                    dtype=torch.float32).to(torch.bfloat16))
    positions = ctx.copy()

    def prepare():
        pool.prepare_step(slots, positions.tolist())
        positions[:] += 1

    def layers():
        for l in range(w.layers):
            pool.decode_layer(l, w.out[l], w.qkv[l], w.q_bias[l], w.k_bias[l], w.v_bias[l],
                              w.cos, w.sin)

    for _ in range(2):  # eager: kernel attributes and tensor maps cached before capture
        prepare()
        layers()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        layers()
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 else None
    for _ in range(settle_steps):
        prepare()
        graph.replay()
    for _ in range(args.warmup):
        prepare()
        graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    kv_tokens = 0
    cur = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(args.steps):
        kv_tokens += int(positions.sum()) + B  # context + the new token, per kv head
        prepare()
        graph.replay()
    e1.record(cur)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms_step = e0.elapsed_time(e1) / args.steps
    kv_bytes = float(kv_tokens) * w.hkv * w.hd * 2 * 2 * w.layers  # over the K steps
    vals = torch.tensor([ms_step, kv_bytes], dtype=torch.float64, device=device)
    if dist:
        mx = vals[:1].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = vals[1:].clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        ms_step, kv_bytes = mx.item(), tot.item()
    if rank == 0:
        peak, peak_kind = measured_peak()
        value = kv_bytes / args.steps / (ms_step * 1e-3) / 1e9
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded bf16 ~N(0,1) K/V/Q, uniform context lengths)",
            "config": {"workload": w.label + ", through the token-step driver (lc_kv_pool)",
                       "batch_per_gpu": w.batch_per_rank, "global_batch": w.global_batch,
                       "q_heads": w.hq, "kv_heads": w.hkv, "head_dim": w.hd,
                       "layers": w.layers, "page_tokens": 16,
                       "parallelism": f"sequence-sharded x{world}",
                       "l2": "no flush: %.1f GB of pools per GPU > 126 MB L2" %
                             (2 * kp.numel() * 2 / 1e9),
                       "step": "lc_kv_pool_prepare_step (host: pages, table + position "
                               "upload) then one CUDA graph replay of the layers' "
                               "lc_kv_pool_decode_layer launches; positions advance one "
                               "token per step" +
                               (f"; programmatic dependent launch mode {args.pdl}"
                                if args.pdl else "")},
            "tokens_per_s": round(w.global_batch / (ms_step * 1e-3), 1),
            "pct_hbm": round(100 * value / world / peak, 2),
            "peak_kind": f"{peak_kind} (burst copy)",
            "gpu_launches": w.layers * args.steps,
            "clocks": clocks,
            "free_blocks_after": pool.num_free_blocks,
        }
        print(json.dumps(line), flush=True)
    del graph
    pool.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# dram__bytes_read.sum + dram__bytes_write.sum of one launch of each config's
# dominant kernel, from the ncu captures summarised in profiles/ (same
# per-launch work as the bench's launches): the fused decode (c2, c3), the
# prefill (c4, reported in MB to one decimal there), the fused QKV projection
# (c4p) and the top-k filter (s2).
TRAFFIC: dict = {"c2": 75958016, "c3": 543651840, "c4": 77800000, "c4p": 101494272,
                 "s2": 19465984}


# ------------------------------------------------------------ reference arm --

def run_reference(args, rank, world, local):
    if rank != 0:
        return  # rank 0 alone runs the reference arm
    import ctypes as C
    import oracle.oracle as O
    try:
        R = O.ref_lib()
    except Exception as e:  # pragma: no cover - only when the build is missing
        print(json.dumps({"impl": "reference", "unavailable": f"reference kernels not built: {e}"}))
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    # The reference has one GPU path: rank 0 runs the whole global batch (the
    # same sequences the repo arm shards over `world` ranks). Its RoPE tables
    # come from the reference library's host restatement of RopeCache::new, so
    # this process loads nothing of the product.
    w = Workload(args.config, 0, world, device, layers=args.layers, rope_table=O.ref_rope_table,
                 shard=False)
    host_pos = (C.c_int * w.batch)(*w.positions_np.tolist())
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731

    def step():
        s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        for l in range(w.layers):
            rc = R.ref_rope_append(P(w.qkv[l]), w.row, w.batch, 1, P(w.positions), P(w.q_bias[l]),
                                   P(w.k_bias[l]), P(w.v_bias[l]), P(w.cos), P(w.sin),
                                   P(w.k_pool), P(w.v_pool), w.layers, l, w.hq, w.hkv, w.hd,
                                   P(w.tables), w.max_pages, 32768, s)
            rc |= R.ref_paged_decode(P(w.out[l]), w.hq * w.hd, P(w.qkv[l]), w.row, P(w.k_pool),
                                     P(w.v_pool), w.layers, l, w.hq, w.hkv, w.hd, P(w.tables),
                                     w.max_pages, P(w.positions), host_pos, w.batch, 32768, s)
            if rc:
                raise RuntimeError(f"reference launch failed ({rc})")

    step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms_step = e0.elapsed_time(e1) / args.steps
    clocks = sampler.stop()

    qkv_host = w.qkv.cpu().pin_memory()
    pos_host = w.positions.cpu().pin_memory()
    out_host = torch.empty(w.out.shape, dtype=w.out.dtype).pin_memory()
    e0.record()
    for _ in range(args.steps):
        w.qkv.copy_(qkv_host, non_blocking=True)
        w.positions.copy_(pos_host, non_blocking=True)
        step()
        out_host.copy_(w.out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    value = w.kv_bytes_per_step / (ms_step * 1e-3) / 1e9
    e2e_value = w.kv_bytes_per_step / (e2e_ms * 1e-3) / 1e9
    peak, _ = measured_peak()
    cfg = workload_config(w, world)
    if world > 1:
        cfg["parallelism"] = (f"none: the reference has no multi-GPU path; one GPU ran the "
                              f"global batch that the repo arm shards over {world}")
    line = {
        "impl": "reference",
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded bf16 ~N(0,1) K/V/Q, uniform context lengths)",
        "config": cfg,
        "step": "per layer and sequence: the reference kernels rope -> update_kv_cache_kernel "
                "-> flash_decoding_kernel (rope.cu/kv_cache.cu/attention.cu compiled unchanged "
                "for sm_100a), launched as src/kernels.rs and src/layers/kv_cache.rs do",
        "tokens_per_s": round(w.batch / (ms_step * 1e-3), 1),
        "pct_hbm": round(100 * value / peak, 3),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": 1,
                         "kind": "reference",
                         "sample": "the reference's implementation of this path is CUDA only; "
                                   "this arm runs its kernels on one B200 from one host thread, "
                                   "full workload"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "e2e_with_copies": {"value": round(e2e_value, 3), "unit": "GB/s",
                            "h2d_bytes_per_step": int(w.h2d_bytes),
                            "d2h_bytes_per_step": int(w.d2h_bytes), "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": w.layers * w.batch * 3 * args.steps,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------- head-sharded decode (c5) --

HEAD_SHARDED = {"c5": ("qwen2.5-72b decode sharded by kv head (BASELINE config 5)", 128, 64, 8,
                       128, 80, ("uniform", 1024, 32768))}


def run_head_sharded(args, rank, world, local):
    """KV-head sharding: rank r owns kv heads [r*8/N, (r+1)*8/N) of every layer
    (identical block tables everywhere), runs the fused decode on its heads, and
    [B][Hq][hd] is assembled on every rank either by an NCCL all-gather plus a
    permute (--gather nccl) or by the decode itself, which stores each row into
    every rank's exchange region, followed by a device-side wait for the peers
    (--gather peer). Two physical layers alternate; tokens/s is extrapolated to
    the model's 80 layers (attention only)."""
    import lucciola as L
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
    L.set_dependent_launch(args.pdl)
    label, B, hq, hkv, hd, model_layers, spec = HEAD_SHARDED[args.config]
    first, nloc = L.shard_kv_heads(hq, hkv, world, rank)
    hq_loc = nloc * (hq // hkv)
    rng = np.random.default_rng(5150)            # identical lengths and tables on every rank
    ctx = rng.integers(spec[1], spec[2] + 1, B).astype(np.int32)
    pages = (ctx + 1 + 15) // 16
    nb = int(pages.sum()) + 1
    perm = rng.permutation(nb).astype(np.int32)
    tables_np = np.full((B, int(pages.max())), -1, np.int32)
    off = 0
    for b, n in enumerate(pages):
        tables_np[b, :n] = perm[off:off + n]
        off += n
    tables = torch.from_numpy(tables_np).to(device)
    positions = torch.from_numpy(ctx).to(device)
    layers = 2
    gen = torch.Generator(device=device)
    gen.manual_seed(77 + rank)
    shape = (nb, layers, nloc, 16, hd)
    k_pool = torch.empty(shape, dtype=torch.bfloat16, device=device)
    v_pool = torch.empty(shape, dtype=torch.bfloat16, device=device)
    for t in (k_pool, v_pool):
        flat = t.view(-1)
        for i in range(0, flat.numel(), 1 << 28):
            chunk = flat[i:i + (1 << 28)]
            chunk.copy_(torch.randn(chunk.numel(), generator=gen, device=device).to(torch.bfloat16))
    row = (hq_loc + 2 * nloc) * hd
    qkv = torch.randn((layers, B, row), generator=gen, device=device).to(torch.bfloat16)
    bias = (torch.randn((layers, row), generator=gen, device=device) * 0.01).to(torch.bfloat16)
    qb = bias[:, :hq_loc * hd].contiguous()
    kb = bias[:, hq_loc * hd:(hq_loc + nloc) * hd].contiguous()
    vb = bias[:, (hq_loc + nloc) * hd:].contiguous()
    cos, sin = (torch.from_numpy(x).to(device) for x in L.rope_table_host(32768 + 16, hd, 1e6))
    ws = L.alloc_decode_workspace(B, hq_loc, nloc, hd, device=device)
    max_ctx = int(ctx.max()) + 1
    status = torch.zeros(1, dtype=torch.int32, device=device)
    peer = args.gather == "peer"
    region = group = None
    if peer:
        # One exchange region per rank: signal words, then the layers' [B][Hq][hd]
        # outputs at the same offsets everywhere; this rank's heads start at
        # column first * (hq / hkv) * hd.
        region = L.PeerRegion(L.PEER_SIGNAL_BYTES + layers * B * hq * hd * 2)
        handles = [region.handle]
        if dist:
            handles = [None] * world
            dist.all_gather_object(handles, region.handle)
        group = L.PeerGroup.open(rank, world, region, handles) if world > 1 else \
            L.PeerGroup.local(0, 1, [region])
        full = region.view(L.PEER_SIGNAL_BYTES, (layers, B, hq * hd), torch.bfloat16)
        col0 = first * (hq // hkv) * hd
    else:
        out_loc = torch.empty((layers, B, hq_loc * hd), dtype=torch.bfloat16, device=device)
        gathered = torch.empty((layers, world * B, hq_loc * hd), dtype=torch.bfloat16,
                               device=device)
        full = torch.empty((layers, B, hq * hd), dtype=torch.bfloat16, device=device)

    def step():
        for l in range(layers):
            if peer:
                L.rope_append_decode(full[l][:, col0:col0 + hq_loc * hd], qkv[l], positions,
                                     qb[l], kb[l], vb[l], cos, sin, k_pool, v_pool, nb, layers, l,
                                     hq_loc, nloc, hd, tables, max_ctx, workspace=ws,
                                     dev_status=status, peer_group=group)
                group.wait(dev_status=status)
                continue
            L.rope_append_decode(out_loc[l], qkv[l], positions, qb[l], kb[l], vb[l], cos, sin,
                                 k_pool, v_pool, nb, layers, l, hq_loc, nloc, hd, tables, max_ctx,
                                 workspace=ws, dev_status=status)
            if dist:
                dist.all_gather_into_tensor(gathered[l], out_loc[l])
                full[l].copy_(L.assemble_head_shards(gathered[l], world))
            else:
                full[l].copy_(out_loc[l])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # Clocks settle under this load for about a second, sampled meanwhile. Every
    # rank runs the same number of steps (each holds a collective): the count
    # comes from the slowest rank's step time.
    t0 = time.perf_counter()
    step()
    torch.cuda.synchronize()
    t_one = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=device)
    if dist:
        dist.all_reduce(t_one, op=dist.ReduceOp.MAX)
    n_settle = max(1, min(2000, int(1.0 / max(t_one.item(), 1e-4))))
    sampler = ClockSampler(local) if rank == 0 else None
    for _ in range(n_settle):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms_step = e0.elapsed_time(e1) / args.steps
    if dist:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    kv_bytes_rank = float((ctx.astype(np.int64) + 1).sum()) * nloc * hd * 2 * 2 * layers
    dev_word = torch.tensor([int(status.item())], dtype=torch.int32, device=device)
    if dist:
        dist.all_reduce(dev_word, op=dist.ReduceOp.MAX)
    dev_word = int(dev_word.item())
    vals = torch.tensor([ms_step, kv_bytes_rank], dtype=torch.float64, device=device)
    if dist:
        mx = vals[:1].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = vals[1:].clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        ms_step, kv_bytes_all = mx.item(), tot.item()
    else:
        kv_bytes_all = kv_bytes_rank
    if rank == 0:
        peak, kind = measured_peak()
        t_layer = ms_step / layers
        value = kv_bytes_all / (ms_step * 1e-3) / 1e9
        print(json.dumps({
            "metric": "decode-attn KV GB/s (KV-head sharded) and tokens/s, attention-only, "
                      "80-layer extrapolated",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded bf16 ~N(0,1), uniform context lengths)",
            "config": {"workload": label, "batch": B, "q_heads": hq, "kv_heads": hkv,
                       "head_dim": hd, "kv_heads_per_gpu": nloc, "physical_layers": layers,
                       "kv_tokens": int(ctx.sum() + B),
                       "parallelism": f"kv-head sharded x{world}, " + (
                           "outputs stored into every rank by the decode (NVLink peer stores)"
                           if peer else "NCCL all-gather of outputs"),
                       "step": "per layer: lc_rope_append_decode_peer on local heads writing "
                               "[B][Hq][hd] on every rank, lc_peer_wait" if peer else
                               "per layer: lc_rope_append_decode on local heads, "
                               "all_gather_into_tensor, permute to [B][Hq][hd]"},
            "ms_per_layer": round(t_layer, 4),
            "tokens_per_s_80_layers": round(B / (model_layers * t_layer * 1e-3), 1),
            "pct_hbm_per_gpu": round(100 * value / world / peak, 2),
            "device_status": dev_word,
            "clocks": clocks,
        }), flush=True)
    if group is not None:
        torch.cuda.synchronize()
        if dist:
            dist.barrier()  # every rank is done with the peers' regions
        group.close()
        if dist:
            dist.barrier()
        region.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------- decode-step projections (c2d/c3d) --

DECODE_PROJ = {
    "c2d": ("qwen2.5-0.5b decode-step projections at batch 64 (BASELINE config 2 shape): QKV "
            "with bias + RoPE + paged append fused, then o_proj with the residual", 64, 14, 2, 64,
            896),
    "c3d": ("qwen2.5-7b decode-step projections at batch 32 (BASELINE config 3 shape): QKV with "
            "bias + RoPE + paged append fused, then o_proj with the residual", 32, 28, 4, 128,
            3584),
}


def run_decode_proj_bench(args, rank, world, local):
    """One decode step's projections per layer at M = batch token rows (the
    weight-streaming kernel of proj_decode.cu): lc_qkv_proj_rope_append (the
    new token of every sequence: bias, RoPE, paged append) then lc_proj_gemm
    for o_proj with the residual in place. Weight sets rotate over enough
    layers to exceed L2 twice over. The bound is reading the weights: the
    metric is weight bytes per second. Beside it, the reference's sequence:
    cublasGemmEx (torch.matmul, bf16 in, fp32 compute) then lc_rope_append, and
    torch.matmul plus the residual add for o_proj."""
    import lucciola as L
    label, B, hq, hkv, hd, hidden = DECODE_PROJ[args.config]
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    # a launch's first weight loads overlap the preceding launch's tail
    L.set_dependent_launch(args.pdl)
    gen = torch.Generator(device=device)
    gen.manual_seed(919)
    N, K, No = (hq + 2 * hkv) * hd, hidden, hidden
    wbytes = (N * K + No * hq * hd) * 2  # per layer
    layers = max(4, -(-2 * 126 * 2 ** 20 // wbytes))
    wq = [(torch.randn(N, K, generator=gen, device=device) * K ** -0.5).to(torch.bfloat16)
          for _ in range(layers)]
    wo = [(torch.randn(No, hq * hd, generator=gen, device=device) * (hq * hd) ** -0.5)
          .to(torch.bfloat16) for _ in range(layers)]
    x = torch.randn(B, K, generator=gen, device=device).to(torch.bfloat16)
    attn = torch.randn(B, hq * hd, generator=gen, device=device).to(torch.bfloat16)
    hidden_st = torch.randn(B, No, generator=gen, device=device).to(torch.bfloat16)
    qkv = torch.empty(B, N, dtype=torch.bfloat16, device=device)
    rng = np.random.default_rng(5)
    ctx = rng.integers(256, 4096, B).astype(np.int32)
    pages = (ctx + 1 + 15) // 16
    nb = int(pages.sum()) + 1
    perm = rng.permutation(nb).astype(np.int32)
    tables_np = np.full((B, int(pages.max())), -1, np.int32)
    off = 0
    for b, n in enumerate(pages):
        tables_np[b, :n] = perm[off:off + n]
        off += n
    tables = torch.from_numpy(tables_np).to(device)
    positions = torch.from_numpy(ctx).to(device)
    k_pool = torch.zeros((nb, 1, hkv, 16, hd), dtype=torch.bfloat16, device=device)
    v_pool = torch.zeros_like(k_pool)
    bias = (torch.randn(N, generator=gen, device=device) * 0.01).to(torch.bfloat16)
    qb, kb, vb = (bias[:hq * hd].contiguous(), bias[hq * hd:(hq + hkv) * hd].contiguous(),
                  bias[(hq + hkv) * hd:].contiguous())
    cos, sin = (torch.from_numpy(t).to(device) for t in L.rope_table_host(4096 + 16, hd, 1e6))

    def ours(l):
        L.qkv_proj_rope_append(qkv, x, wq[l], positions, qb, kb, vb, cos, sin, k_pool, v_pool, nb,
                               1, 0, hq, hkv, hd, tables, tokens_per_seq=1)
        L.proj_gemm(hidden_st, attn, wo[l], residual=hidden_st)

    def library(l):
        torch.matmul(x, wq[l].t(), out=qkv)
        L.rope_append(qkv, positions, qb, kb, vb, cos, sin, k_pool, v_pool, nb, 1, 0, hq, hkv, hd,
                      tables)
        hidden_st.add_(torch.matmul(attn, wo[l].t()))

    if args.mode == "kernel":
        for i in range(args.warmup + args.steps):
            ours(i % layers)
        torch.cuda.synchronize()
        print(json.dumps({"mode": "kernel", "config": args.config,
                          "launches": 2 * (args.warmup + args.steps)}))
        return

    def timed(fn, steps):
        # One CUDA graph over all rotated layers, replayed: the launches run
        # back to back on the device, with no host-side launch cost between
        # them (the same for both arms).
        for i in range(max(args.warmup, 3) * layers):
            fn(i % layers)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for l in range(layers):
                fn(l)
        for _ in range(max(args.warmup, 3)):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / (steps * layers)

    sampler = ClockSampler(local)
    t_end = time.perf_counter() + 1.0
    while time.perf_counter() < t_end:
        for l in range(layers):
            ours(l)
    torch.cuda.synchronize()
    ms = timed(ours, args.steps)
    ms_lib = timed(library, args.steps)
    clocks = sampler.stop()
    # the two launches separately (CUDA events around each, back to back)
    qkv_only = timed(lambda l: L.qkv_proj_rope_append(qkv, x, wq[l], positions, qb, kb, vb, cos,
                                                      sin, k_pool, v_pool, nb, 1, 0, hq, hkv, hd,
                                                      tables, tokens_per_seq=1), args.steps)
    lib_gemm_only = timed(lambda l: torch.matmul(x, wq[l].t(), out=qkv), args.steps)
    peak, peak_kind = measured_peak()
    value = wbytes / (ms * 1e-3) / 1e9
    q_bytes = N * K * 2
    q_gbs = q_bytes / (qkv_only * 1e-3) / 1e9
    print(json.dumps({
        "metric": "decode-step projection weight GB/s (QKV fused with bias + RoPE + append, "
                  "o_proj with residual)",
        "value": round(value, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded bf16 x ~N(0,1), w ~N(0,1/hidden))",
        "config": {"workload": label, "batch": B, "qkv_n": N, "hidden": K,
                   "layers_rotated": layers, "programmatic_dependent_launch": args.pdl,
                   "plan_qkv": dict(zip(("split", "ctas", "clusters_that_fit", "ctas_per_sm"),
                                        L.proj_decode_plan(N, K))),
                   "plan_o": dict(zip(("split", "ctas", "clusters_that_fit", "ctas_per_sm"),
                                      L.proj_decode_plan(No, hq * hd))),
                   "l2": "no flush: %d distinct weight sets, %.0f MB > 2 x 126 MB L2" %
                         (layers, layers * wbytes / 1e6),
                   "timing": "both arms: one CUDA graph over the rotated layers, replayed "
                             "--steps times"},
        "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(value / peak, 4), "peak_kind": f"{peak_kind} (burst copy)",
                     "qkv_launch_ms": round(qkv_only, 5), "qkv_achieved": round(q_gbs, 1),
                     "qkv_frac": round(q_gbs / peak, 4)},
        "library_path": {"ms_per_layer": round(ms_lib, 5),
                         "qkv_gemm_ms": round(lib_gemm_only, 5),
                         "qkv_gemm_gbs": round(q_bytes / (lib_gemm_only * 1e-3) / 1e9, 1),
                         "how": "torch.matmul (cublasGemmEx) + lc_rope_append; torch.matmul + "
                                "residual add for o_proj"},
        "speedup_vs_library": round(ms_lib / ms, 3),
        "gpu_launches": 2 * args.steps * layers,
        "clocks": clocks,
    }), flush=True)


# ------------------------------------------------------------ prefill (c4) --

PREFILL = {"c4": ("qwen2.5-1.5b causal prefill into the paged cache (BASELINE config 4)",
                  4, 12, 2, 128, 28, 4096)}


def causal_flops(batch, tokens, hq, hd, start=0):
    """4*hd flops per (query, visible key, q head): QK^T and PV."""
    keys = sum(start + i + 1 for i in range(tokens))
    return 4.0 * batch * keys * hq * hd


def run_prefill_bench(args, rank, world, local):
    import lucciola as L
    label, B, hq, hkv, hd, layers, T = PREFILL[args.config]
    if args.layers:  # fewer layers for profiling captures; per-layer work unchanged
        layers = args.layers
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(4321)
    pages = (T + 15) // 16
    nb = B * pages + 1
    perm = torch.randperm(nb, generator=gen, device=device).to(torch.int32)
    tables = perm[:B * pages].reshape(B, pages).contiguous()
    shape = (nb, layers, hkv, 16, hd)
    k_pool = torch.randn(shape, generator=gen, device=device).to(torch.bfloat16)
    v_pool = torch.randn(shape, generator=gen, device=device).to(torch.bfloat16)
    row = (hq + 2 * hkv) * hd
    qkv = torch.randn((layers, B * T, row), generator=gen, device=device).to(torch.bfloat16)
    bias = (torch.randn((layers, row), generator=gen, device=device) * 0.01).to(torch.bfloat16)
    qb, kb, vb = (bias[:, :hq * hd].contiguous(), bias[:, hq * hd:(hq + hkv) * hd].contiguous(),
                  bias[:, (hq + hkv) * hd:].contiguous())
    cos, sin = (torch.from_numpy(x).to(device) for x in L.rope_table_host(T + 16, hd, 1e6))
    positions = torch.arange(T, dtype=torch.int32, device=device).repeat(B)
    start = torch.zeros(B, dtype=torch.int32, device=device)
    out = torch.empty((layers, B * T, hq * hd), dtype=torch.bfloat16, device=device)

    def layer(l, ev=None):
        L.rope_append(qkv[l], positions, qb[l], kb[l], vb[l], cos, sin, k_pool, v_pool, nb, layers,
                      l, hq, hkv, hd, tables, tokens_per_seq=T)
        if ev is not None:
            ev[0].record()
        L.paged_prefill(out[l], qkv[l], k_pool, v_pool, nb, layers, l, hq, hkv, hd, tables, start,
                        T, 0)
        if ev is not None:
            ev[1].record()

    def step():
        for l in range(layers):
            layer(l)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=device)):
        step()
    sampler = ClockSampler(local)
    t_end = time.perf_counter() + 1.0
    while time.perf_counter() < t_end:
        graph.replay()
        torch.cuda.synchronize()
    ms_step = time_graph(graph, args.steps, args.warmup, torch.cuda.current_stream()) / args.steps
    clocks = sampler.stop()
    # per-launch duration of the prefill kernel (events around each launch)
    pairs = []
    torch.cuda._sleep(50_000_000)
    for l in range(min(layers, 8)):
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        layer(l, ev)
        pairs.append(ev)
    torch.cuda.synchronize()
    launch_ms = sum(a.elapsed_time(b) for a, b in pairs) / len(pairs)
    flops = causal_flops(B, T, hq, hd)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak_burst = float(peaks.get("bf16_tflops", 1590.0))
    peak_sust = float(peaks.get("bf16_tflops_sustained", 1400.0))
    kind = "measured" if peaks else "fallback"
    achieved = flops / (launch_ms * 1e-3) / 1e12
    step_tflops = flops * layers / (ms_step * 1e-3) / 1e12
    line = {
        "metric": "causal prefill attention TFLOP/s (4 x 4096 tokens, per layer)",
        "value": round(step_tflops, 1), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded bf16 ~N(0,1) Q/K/V, RoPE theta 1e6)",
        "config": {"workload": label, "sequences": B, "tokens": T, "q_heads": hq,
                   "kv_heads": hkv, "head_dim": hd, "layers": layers,
                   "flops_per_layer": flops,
                   "step": "per layer: lc_rope_append (prompt rows) + lc_paged_prefill; CUDA graph"},
        "ms_per_layer": round(ms_step / layers, 4),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak_sust,
                     "unit": "TFLOP/s", "frac": round(achieved / peak_sust, 4),
                     "traffic": TRAFFIC.get(args.config),
                     "kernel": f"paged_prefill_kernel<{hd}>",
                     "peak_kind": f"{kind} (sustained bf16 GEMM; burst {peak_burst})",
                     "launch_ms": round(launch_ms, 4)},
        "gpu_launches": 2 * layers * args.steps,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    del graph


PROJ = {"c4p": ("qwen2.5-1.5b QKV projection of a 4 x 4096-token prompt with bias + RoPE + "
                 "paged KV append fused into the GEMM epilogue (BASELINE config 4 shape)",
                 4, 12, 2, 128, 1536, 4096)}


def run_proj_bench(args, rank, world, local):
    """lc_qkv_proj_rope_append: qkv = x . w_qkv^T on the tensor cores (CTA pairs)
    with bias + RoPE + the paged K/V append in its epilogue, one launch per layer.
    Beside it, the same work as the reference runs it: cublasGemmEx (through
    torch.matmul, bf16 in, fp32 compute, bf16 out) then lc_rope_append."""
    import lucciola as L
    label, B, hq, hkv, hd, hidden, T = PROJ[args.config]
    layers = 4  # distinct x / w per layer: 4 x 56 MB > 126 MB L2, no flush needed
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(777)
    M, N, K = B * T, (hq + 2 * hkv) * hd, hidden
    xs = [torch.randn(M, K, generator=gen, device=device).to(torch.bfloat16) for _ in range(layers)]
    ws = [(torch.randn(N, K, generator=gen, device=device) * K ** -0.5).to(torch.bfloat16)
          for _ in range(layers)]
    qkv = torch.empty(M, N, dtype=torch.bfloat16, device=device)
    pages = (T + 15) // 16
    nb = B * pages + 1
    perm = torch.randperm(nb, generator=gen, device=device).to(torch.int32)
    tables = perm[:B * pages].reshape(B, pages).contiguous()
    k_pool = torch.zeros((nb, layers, hkv, 16, hd), dtype=torch.bfloat16, device=device)
    v_pool = torch.zeros_like(k_pool)
    bias = (torch.randn((layers, N), generator=gen, device=device) * 0.01).to(torch.bfloat16)
    qb, kb, vb = (bias[:, :hq * hd].contiguous(), bias[:, hq * hd:(hq + hkv) * hd].contiguous(),
                  bias[:, (hq + hkv) * hd:].contiguous())
    cos, sin = (torch.from_numpy(x).to(device) for x in L.rope_table_host(T + 16, hd, 1e6))
    positions = torch.arange(T, dtype=torch.int32, device=device).repeat(B)

    def fused(l):
        L.qkv_proj_rope_append(qkv, xs[l], ws[l], positions, qb[l], kb[l], vb[l], cos, sin,
                               k_pool, v_pool, nb, layers, l, hq, hkv, hd, tables,
                               tokens_per_seq=T)

    def library(l):
        torch.matmul(xs[l], ws[l].t(), out=qkv)
        L.rope_append(qkv, positions, qb[l], kb[l], vb[l], cos, sin, k_pool, v_pool, nb, layers,
                      l, hq, hkv, hd, tables, tokens_per_seq=T)

    if args.mode == "kernel":  # eager launches only, for profilers
        for i in range(args.warmup + args.steps):
            fused(i % layers)
        torch.cuda.synchronize()
        print(json.dumps({"mode": "kernel", "config": args.config, "launches":
                          args.warmup + args.steps}))
        return

    def timed(fn):
        for i in range(args.warmup):
            fn(i % layers)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            fn(i % layers)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    sampler = ClockSampler(local)
    t_end = time.perf_counter() + 1.0
    while time.perf_counter() < t_end:
        fused(0)
    torch.cuda.synchronize()
    ms = timed(fused)
    ms_lib = timed(library)
    clocks = sampler.stop()
    flops = 2.0 * M * N * K
    peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get("bf16_tflops_sustained") \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 1400.0
    value = flops / (ms * 1e-3) / 1e12
    print(json.dumps({
        "metric": "prefill QKV projection TFLOP/s (bias + RoPE + paged KV append fused)",
        "value": round(value, 1), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded bf16 ~N(0,1) x, w ~N(0,1/hidden))",
        "config": {"workload": label, "tokens": M, "n": N, "k": K, "layers_rotated": layers,
                   "l2": "no flush: 4 distinct x/w of 56 MB each > 126 MB L2"},
        "roofline": {"bound": "tensor", "achieved": round(value, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(value / peak, 4),
                     "traffic": TRAFFIC.get(args.config),
                     "kernel": "proj_gemm2_kernel<qkv rope>",
                     "peak_kind": "measured (sustained cuBLAS bf16)"},
        "library_path": {"ms": round(ms_lib, 5),
                         "tflops": round(flops / (ms_lib * 1e-3) / 1e12, 1),
                         "how": "torch.matmul (cublasGemmEx, bf16, fp32 compute) then "
                                "lc_rope_append, as the reference sequences them"},
        "gpu_launches": args.steps, "clocks": clocks}), flush=True)


SAMPLING = {"s2": ("top-k / top-p token sampling over the Qwen2 vocabulary for config 2's batch "
                   "(64 rows x 151936 logits, top_k 64, top_p 0.9)", 64, 151936, 64, 0.9)}


def run_sampling_bench(args, rank, world, local):
    """lc_sample_top_p on a batch of logits rows (one launch of the 32-partition
    top-k filter for all rows, one of the sort-and-draw). --impl reference runs
    the reference's kernels (oracle/_ref) one row at a time, as
    CudaFunctions::apply_sort_and_sample launches them."""
    label, B, V, top_k, top_p = SAMPLING[args.config]
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(99)
    nbuf = 8  # 8 x 19.4 MB of logits > 126 MB L2: no flush needed
    logits = [(torch.randn(B, V, generator=gen, device=device) * 3).to(torch.bfloat16)
              for _ in range(nbuf)]
    rand = torch.rand(B, generator=gen, device=device)
    tp = torch.full((B,), top_p, dtype=torch.float32, device=device)
    out = torch.zeros(B, dtype=torch.int32, device=device)
    if args.impl == "reference":
        import ctypes as C
        import oracle.oracle as O
        R = O.ref_lib()
        cand = torch.zeros(2 * 32 * (top_k // 32), dtype=torch.int32, device=device)
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        rv = rand.cpu().tolist()

        def step(i):
            x = logits[i % nbuf]
            for r in range(B):
                R.ref_sample_top_p(C.c_void_p(x[r].data_ptr()), V, top_k, top_p, rv[r],
                                   C.c_void_p(cand.data_ptr()), C.c_void_p(out[r:].data_ptr()),
                                   stream)
        launches = 2 * B
    else:
        import lucciola as L
        ws = L.alloc_sample_workspace(B, top_k, device=device)

        def step(i):
            L.sample_top_p(out, logits[i % nbuf], top_k, tp, rand, ws)
        launches = 2
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    peak, peak_kind = measured_peak()
    gbs = B * V * 2 / (ms * 1e-3) / 1e9
    line = {"metric": "token sampling rows/s (top-k 64, top-p 0.9, Qwen2 vocabulary)",
            "value": round(B / (ms * 1e-3), 1), "unit": "rows/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded bf16 logits ~N(0, 9), uniform draws)",
            "config": {"workload": label, "rows": B, "vocab": V, "top_k": top_k,
                       "top_p": top_p, "l2": "8 rotating logits batches of 19.4 MB > L2"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "traffic": TRAFFIC.get(args.config),
                         "kernel": "topk_filter_kernel + sort_sample_kernel",
                         "peak_kind": f"{peak_kind} (burst copy)",
                         "algorithmic_bytes": B * V * 2},
            "gpu_launches": launches * args.steps, "clocks": clocks}
    if args.impl == "reference":
        line["impl"] = "reference"
        line["cpu_baseline"] = {"value": line["value"], "unit": "rows/s", "cores": 0,
                                "kind": "reference",
                                "sample": "the reference's CUDA kernels (oracle/_ref), one row "
                                          "per launch pair; its path has no CPU implementation"}
        line["e2e"] = {"value": line["value"], "unit": "rows/s", "h2d_bytes_per_step": 0,
                       "d2h_bytes_per_step": 0}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS) + sorted(PREFILL) + sorted(HEAD_SHARDED) +
                    sorted(PROJ) + sorted(SAMPLING) + sorted(DECODE_PROJ),
                    default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mode", choices=["bench", "kernel"], default="bench",
                    help="kernel: eager launches only (for profilers), no JSON metrics")
    ap.add_argument("--pdl", type=int, default=2, choices=[0, 1, 2],
                    help="programmatic dependent launch mode (lc_set_dependent_launch); the "
                         "step satisfies mode 2's contract: between layers nothing writes the "
                         "context lengths, tables or the next layer's cached pages")
    ap.add_argument("--layers", type=int, default=None,
                    help="kernel mode and the prefill config only: fewer layers (smaller "
                         "pools) for profiler captures")
    ap.add_argument("--unfused", action="store_true",
                    help="two launches per layer (lc_rope_append, lc_paged_decode)")
    ap.add_argument("--driver", action="store_true",
                    help="decode configs: run the workload through the batched token-step "
                         "driver (lc_kv_pool) with positions advancing every step")
    ap.add_argument("--partition", type=int, default=None,
                    help="override the split-K partition size in tokens (0 = auto)")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="config 5: assemble all heads by peer stores from the decode "
                         "(lc_rope_append_decode_peer + lc_peer_wait; the default: level "
                         "with the all-gather at 2 GPUs, 2 %% ahead at 4) or by an NCCL "
                         "all-gather after it")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.layers is not None and args.mode != "kernel" and args.config not in PREFILL:
        ap.error("--layers changes the workload; it is for --mode kernel and the prefill "
                 "config (profiling) only")
    rank, world, local = env_dist()
    if args.config in HEAD_SHARDED:
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference is "
                                  "single-GPU; its arm is run on the decode headline (config 2)"}))
            return 0
        run_head_sharded(args, rank, world, local)
        return 0
    if args.config in SAMPLING:
        if rank == 0:
            run_sampling_bench(args, rank, world, local)
        return 0
    if args.config in DECODE_PROJ:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm is run on "
                              "the decode headline (config 2); its projections are cuBLAS, timed "
                              "beside ours in this config's library_path"}))
            return 0
        if rank == 0:
            run_decode_proj_bench(args, rank, world, local)
        return 0
    if args.config in PROJ:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm is run on "
                              "the decode headline (config 2); its projection is cuBLAS, timed "
                              "beside ours in this config's library_path"}))
            return 0
        if rank == 0:
            run_proj_bench(args, rank, world, local)
        return 0
    if args.config in PREFILL:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm is run on "
                              "the decode headline (config 2); its prefill is T sequential "
                              "decode launches per layer"}))
            return 0
        if rank == 0:
            run_prefill_bench(args, rank, world, local)
        return 0
    if args.impl == "reference":
        run_reference(args, rank, world, local)
    elif args.driver:
        run_driver(args, rank, world, local)
    else:
        run_ours(args, rank, world, local)
    return 0


if __name__ == "__main__":
    sys.exit(main())
