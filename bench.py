"""Benchmark of the B200 LCSA hot path (block selection + block-sparse attention), one JSON line on rank 0.

Metric: block-sparse attention effective TFLOP/s — 4·128³ FLOP per kept (query block, key block,
head) triple, over the whole path's device time (pooling + selection + attention) — plus ms per 30-layer chunk.
Workload (default, every N): config 3 (1920×1152 chunk: 12 heads, 135 × 405 blocks, R = 11, keep 30 %) as one
steady-state streamed chunk: a step = 30 DiT layers, each with its window cache of 2 earlier slices and fresh seeded
q / k_new / v_new resident in HBM (per layer 159 MB of chunk data + 212 MB of cache read, larger than L2, so no flush
is needed). N > 1 (torchrun, one process per GPU): the same chunk split by query blocks, each rank pooling its shard,
NCCL all-gathers of the pooled rows and of the current slice's K/V inside the timed region; strong scaling, time =
max over ranks. --fresh: 30 independent layer calls on fresh full Q/K/V. --shard: one config's (head, query block)
items split across the ranks with no data-path collective; --replicas: one independent chunk per GPU (weak scaling).

--impl reference: the CPU baseline arm — the reference's Swift/MLX path cannot run off Apple hardware, so this times
the CPU oracle (a C/OpenMP restatement of the reference's selection and block-masked attention) on all host threads,
on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))


def load_pkg():
    from __graft_entry__ import _load_package
    pkg = _load_package()
    pkg.build()
    import importlib
    return pkg, importlib.import_module("fvsr_b200.configs")


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    return 1590.0, 6650.0, "fallback"


def profiled_traffic():
    """Per-launch DRAM bytes of the attention kernel from the committed ncu summary, if one exists."""
    p = ROOT / "profiles" / "attn_bf16_config3_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            return None
    return None


# ---------------------------------------------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------------------------------------------
class Clocks:
    """nvidia-smi samples (every 50 ms) of SM clock and throttle reasons; only the samples taken inside the timed
    region count. The sampler is started, and its first sample awaited, before the region begins."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_uuid: str | None):
        self.proc = None
        self.uuid = device_uuid
        self.first = ""
        self.window = None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"]
        if self.uuid:
            cmd += ["-i", self.uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            import select
            if select.select([self.proc.stdout], [], [], 5.0)[0]:  # running once it has printed a line
                self.first = self.proc.stdout.readline()
        except Exception:
            self.proc = None

    def mark(self, t0: float, t1: float):
        self.window = (t0, t1)

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.06)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        import datetime
        rows = []
        for line in (self.first + out).strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                t = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((t, float(f[2]), float(f[3]), f[6:10]))
            except ValueError:
                continue
        inside = [r for r in rows if self.window and self.window[0] <= r[0] <= self.window[1]]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = {n for r in inside for n, v in zip(names, r[3]) if v.lower().startswith("active")}
        sms = [r[1] for r in inside]
        return {"sm_mhz": statistics.median(sms) if sms else None,
                "sm_max_mhz": max(r[2] for r in rows) if rows else None, "reasons": sorted(reasons),
                "samples": len(sms), "sample_interval_ms": 50}


# ---------------------------------------------------------------------------------------------------------------
# CPU baseline (oracle port, all host threads, bounded sample)
# ---------------------------------------------------------------------------------------------------------------
def cpu_baseline(cfg_id: int = 3, heads_sample: int = 12, seed: int = 3000):
    import numpy as np
    from oracle import oracle as orc
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import detrand
    pkg, cfgs = load_pkg()
    cfg = cfgs.CONFIGS[cfg_id]
    g = cfg.geometry()
    threads = os.cpu_count() or 1
    orc.set_num_threads(threads)
    c = g.channels
    q = detrand.normal(seed, (g.nq * 128, c))
    k = detrand.normal(seed + 1, (g.nk * 128, c))
    v = detrand.normal(seed + 2, (g.nk * 128, c))
    loc = orc.local_block_mask(g.bh, g.bw, g.local_range)
    t0 = time.perf_counter()
    pq, pk = orc.pool(q), orc.pool(k)
    probs, mask, kidx, kcnt = orc.select(pq, pk, g.heads, g.q_slices, g.s, loc, g.topk)
    t_sel = time.perf_counter() - t0
    items = np.arange(heads_sample * g.nq, dtype=np.int32)           # every query block of the first heads
    t0 = time.perf_counter()
    orc.attention(q, k, v, kidx, kcnt, g.heads, items=items, fast=True)
    t_att = time.perf_counter() - t0
    kept = int(kcnt[:heads_sample].sum())
    frac = heads_sample / g.heads
    secs = t_sel * frac + t_att                                        # selection prorated to the sampled heads
    flops = 4.0 * 128 ** 3 * kept
    return {"value": flops / secs / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"config {cfg_id}, one layer: full pooling + selection (prorated to {heads_sample}/{g.heads} "
                      f"heads) + fp32 attention over all query blocks of {heads_sample} head(s) ({kept} kept triples); "
                      f"{secs:.2f} s", "seconds": secs, "kept_triples": kept}


def run_reference(args):
    """The reference arm: the reference's path is Swift/MLX on Apple GPUs (unavailable on this box), so its CPU
    restatement (the oracle: selection + fp32 attention, all host threads) runs one layer of the same workload per
    step — a bounded sample — on the same metric and config as the GPU arm."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    _, cfgs = load_pkg()
    cfg = cfgs.CONFIGS[args.config]
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(args.config, seed=3000 + i)
        if i >= args.warmup:
            vals.append(r)
    v = statistics.median(x["value"] for x in vals)
    ms = statistics.median(x["seconds"] for x in vals) * 1e3
    line = {
        "impl": "reference",
        "metric": f"block-sparse attn effective TFLOP/s (+ ms per 30-layer chunk), config {args.config}", "value": v,
        "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "ms_per_chunk_projected": ms * args.layers, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded normal, window order)",
        "config": {"workload": f"config {args.config}: {cfg.name}", "sample": vals[-1]["sample"]},
        "cpu_baseline": {k: vals[-1][k] for k in ("kind", "cores", "sample")} | {"value": v, "unit": "TFLOP/s"},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's own path is Swift/MLX on Apple GPUs (unavailable on this box); this arm is the CPU "
                "oracle restating it, one layer of the workload per step",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------------------------------
def run_ours(args):
    import torch

    pkg, cfgs = load_pkg()
    import importlib
    ranks = importlib.import_module("fvsr_b200.ranks")
    info = ranks.rank_info()
    world, rank, local = info.world, info.rank, info.local
    torch.cuda.set_device(local)
    ranks.init(info, "nccl", timeout_s=120, device=torch.device("cuda", local))
    cfg = cfgs.CONFIGS[args.config]
    g = cfg.geometry()
    layers = args.layers
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    shard = args.shard if args.shard is not None else args.config == 5

    if shard:
        # the config's (head, query block) items split across ranks (strong scaling, no data-path collective: LCSA
        # heads are independent, so each rank holds the Q/K/V of the heads its items touch, as a tensor-parallel
        # QKV projection leaves them); inputs are seeded per head, so the ranks together solve the one-GPU problem
        sh_world, sh_rank = (world, rank) if not args.as_rank else (int(args.as_rank.split("/")[1]),
                                                                    int(args.as_rank.split("/")[0]))
        sh = pkg.shard_items(g.heads, g.nq, sh_world, sh_rank)
        g_loc = pkg.Geometry(**{**g.__dict__, "heads": max(sh.heads, 1)})
        item_begin, item_count = sh.local_range(g.nq) if sh.heads > 0 else (0, 0)

        def make_inputs(l):
            parts = [cfgs.synth_qkv(cfg, pkg.Geometry(**{**g.__dict__, "heads": 1}),
                                    cfgs.seed_of(args.config, 0, l) * 64 + h, device=dev)
                     for h in range(sh.head_lo, max(sh.head_hi, sh.head_lo) + 1)]
            return tuple(torch.cat([pt[i] for pt in parts], dim=1).contiguous() for i in range(3))
    else:
        g_loc = g
        item_begin, item_count = 0, g.heads * g.nq

        def make_inputs(l):
            return cfgs.synth_qkv(cfg, g, cfgs.seed_of(args.config, rank, l), device=dev)

    # inputs: one fresh seeded (q, k, v) per layer, resident in HBM
    inputs = [make_inputs(l) for l in range(layers)]
    ws = pkg.make_workspace(g_loc, dev)
    kidx = torch.empty((g_loc.heads, g_loc.nq, g_loc.nk), dtype=torch.int32, device=dev)
    kcnt = torch.empty((g_loc.heads, g_loc.nq), dtype=torch.int32, device=dev)
    outs = [torch.empty_like(inputs[0][0]) for _ in range(2)]
    kept = []

    import ctypes
    L = pkg.lib()
    p = g_loc.params()

    def select_call(q, k):
        pkg._check(L.fvsr_lcsa_select(ctypes.byref(p), pkg._ptr(q), pkg._ptr(k), None, pkg._ptr(kidx), pkg._ptr(kcnt),
                                      None, None, pkg._ptr(ws), ws.numel(), pkg._stream()))

    order = torch.empty(max(item_count, 1), dtype=torch.int32, device=dev)
    use_split = shard and not args.no_split
    persistent = use_split and pkg.schedule_is_persistent(
        g_loc, item_begin, item_count, torch.cuda.get_device_properties(dev).multi_processor_count)
    sched = torch.empty(pkg.schedule_size(g_loc, item_count) if use_split else 1, dtype=torch.uint8, device=dev)

    def order_call():
        """The work order of the rank's items: the balanced unit schedule when sharded (long key lists split,
        partials merged), else the longest-first item order."""
        if use_split:
            pkg._check(L.fvsr_lcsa_schedule(ctypes.byref(p), pkg._ptr(kcnt), item_begin, item_count, pkg._ptr(sched),
                                            sched.numel(), pkg._stream()))
        else:
            pkg._check(L.fvsr_lcsa_item_order(ctypes.byref(p), pkg._ptr(kcnt), item_begin, item_count,
                                              pkg._ptr(order), pkg._stream()))

    def attention_only(q, k, v, out):
        if use_split:
            pkg._check(L.fvsr_lcsa_attention_scheduled(ctypes.byref(p), pkg._ptr(q), pkg._ptr(k), pkg._ptr(v),
                                                       pkg._ptr(kidx), pkg._ptr(kcnt), pkg._ptr(out), item_begin,
                                                       item_count, pkg._ptr(sched), sched.numel(), pkg._stream()))
            return
        pkg._check(L.fvsr_lcsa_attention_range(ctypes.byref(p), pkg._ptr(q), pkg._ptr(k), pkg._ptr(v),
                                               pkg._ptr(kidx), pkg._ptr(kcnt), pkg._ptr(out), item_begin, item_count,
                                               pkg._ptr(order), pkg._stream()))

    def attention_call(q, k, v, out):
        order_call()
        attention_only(q, k, v, out)

    def layer_call(l, out):
        """One layer through the C ABI. Unsharded: fvsr_lcsa_layer (pooling, the one-launch selection that also
        orders the items, the attention). Sharded: fvsr_lcsa_select, then the attention over this rank's items."""
        q, k, v = inputs[l]
        if not shard:
            pkg._check(L.fvsr_lcsa_layer(ctypes.byref(p), pkg._ptr(q), pkg._ptr(k), pkg._ptr(v), pkg._ptr(out),
                                         pkg._ptr(kidx), pkg._ptr(kcnt), pkg._ptr(ws), ws.numel(), pkg._stream()))
            return
        select_call(q, k)
        attention_call(q, k, v, out)

    def step():
        for l in range(layers):
            layer_call(l, outs[l & 1])

    # kept triples per layer of this rank's items (deterministic given the inputs; read once, outside the timed region)
    for l in range(layers):
        layer_call(l, outs[0])
        kept.append(int(kcnt.view(-1)[item_begin:item_begin + item_count].sum().item()))
    flops_per_step = 4.0 * 128 ** 3 * sum(kept)
    total_kept = sum(kept)
    total_kept = int(round(ranks.sum_over_ranks(total_kept, dev)))
    flops_all_ranks = 4.0 * 128 ** 3 * total_kept

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    run_step = step
    if not args.no_graph:
        # the 30 layer calls of a step (3 kernels each unsharded) replayed as one CUDA graph: the C ABI calls make no
        # host synchronisation and no allocation, so they capture as they are
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        graph.replay()
        torch.cuda.synchronize()
        run_step = graph.replay
    ranks.barrier()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    clocks = Clocks(uuid)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t_begin = time.time()
    e0.record(stream)
    for _ in range(args.steps):
        run_step()
    e1.record(stream)
    torch.cuda.synchronize()
    clocks.mark(t_begin, time.time())
    clk = clocks.stop()
    ms = ranks.max_over_ranks(e0.elapsed_time(e1) / args.steps, dev)
    pkg.device_check()

    # dominant kernel: the bf16 attention alone, CUDA events on the launching stream, over all layers
    att_ms = []
    for l in range(layers):
        q, k, v = inputs[l]
        select_call(q, k)
        order_call()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        attention_only(q, k, v, outs[0])
        a1.record(stream)
        a1.synchronize()
        att_ms.append(a0.elapsed_time(a1))
    att_avg = sum(att_ms) / len(att_ms)
    att_tflops = 4.0 * 128 ** 3 * (sum(kept) / layers) / (att_avg * 1e-3) / 1e12
    sel_ms = ms / layers - att_avg

    # end to end through the C ABI with host buffers.
    # Unsharded runs stream as the reference does (DiT.swift:504-538): every layer keeps its window K/V cache on the
    # device (kv_slices − q_slices slices), and a step (one chunk) uploads only the chunk's q, k_new and v_new from
    # pinned host memory, runs fvsr_lcsa_forward (append, select over cache ⊕ current, attention, trim) and reads the
    # output back. Sharded runs upload each layer's q, k and v whole (their ranks hold head slices, not caches).
    # Copies run on their own streams: H2D of layer l+1 and D2H of layer l−1 overlap the compute of layer l.
    e2e = None
    e2e_kind = None
    if args.e2e_steps > 0 and not shard and g.kv_slices > g.q_slices:
        e2e_kind = "streaming layer call (fvsr_lcsa_forward with a device-resident window K/V cache per layer)"
        new_sl, kv_len = g.q_slices, g.kv_slices - g.q_slices
        srows = g.s * 128                     # token rows of one slice
        nbuf = 3
        nrot = g.kv_slices                    # distinct K/V slices per layer, uploaded in rotation
        host = []                             # per buffer set: q, then K and V of each of the nrot slices
        for l in range(nbuf):
            q, k, v = inputs[l]
            host.append((q.cpu().pin_memory(),
                         [k[i * srows:(i + new_sl) * srows].cpu().pin_memory() for i in range(nrot)],
                         [v[i * srows:(i + new_sl) * srows].cpu().pin_memory() for i in range(nrot)]))
        caches = []
        for l in range(layers):               # steady state: the cache holds slices 1 .. kv_len of the rotation
            c = pkg.KVCache(g, kv_len, new_sl)
            k, v = inputs[l % nbuf][1], inputs[l % nbuf][2]  # the data the layer's uploads rotate through
            for i in range(1, 1 + kv_len):
                c.append(k[i * srows:(i + new_sl) * srows], v[i * srows:(i + new_sl) * srows], new_sl)
            caches.append(c)
        wsf = pkg.make_workspace(g, dev)
        dq = [torch.empty_like(host[0][0], device=dev) for _ in range(2)]
        dk = [torch.empty_like(host[0][1][0], device=dev) for _ in range(2)]
        dv = [torch.empty_like(host[0][2][0], device=dev) for _ in range(2)]
        hout = [torch.empty(inputs[0][0].shape, dtype=inputs[0][0].dtype, pin_memory=True) for _ in range(2)]
        kcnt_f = torch.empty((layers, g.heads, g.nq), dtype=torch.int32, device=dev)
        up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        ready = [torch.cuda.Event() for _ in range(2)]
        free = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        read = [torch.cuda.Event() for _ in range(2)]
        for ev in free + read:
            ev.record(stream)
        h2d = sum(t.numel() * t.element_size() for t in (host[0][0], host[0][1][0], host[0][2][0])) * layers
        d2h = outs[0].numel() * outs[0].element_size() * layers
        pf = g.params()

        def e2e_step(t):
            for l in range(layers):
                b = l & 1
                hq, hk, hv = host[l % nbuf]
                with torch.cuda.stream(up):
                    up.wait_event(free[b])
                    dq[b].copy_(hq, non_blocking=True)
                    dk[b].copy_(hk[t % nrot], non_blocking=True)
                    dv[b].copy_(hv[t % nrot], non_blocking=True)
                    ready[b].record(up)
                stream.wait_event(ready[b])
                stream.wait_event(read[b])    # outs[b] was read back
                pkg._check(L.fvsr_lcsa_forward(ctypes.byref(pf), pkg._ptr(dq[b]), pkg._ptr(dk[b]), pkg._ptr(dv[b]),
                                               caches[l].handle, pkg._ptr(outs[b]), None, pkg._ptr(kcnt_f[l]),
                                               pkg._ptr(wsf), wsf.numel(), pkg._stream()))
                free[b].record(stream)
                done[b].record(stream)
                with torch.cuda.stream(down):
                    down.wait_event(done[b])
                    hout[b].copy_(outs[b], non_blocking=True)
                    read[b].record(down)
            stream.wait_stream(down)

        # kept triples of each rotation phase (deterministic), read outside the timed region
        kept_phase = []
        for t in range(nrot):
            e2e_step(t)
            torch.cuda.synchronize()
            kept_phase.append(int(kcnt_f.sum().item()))
        ranks.barrier()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for t in range(args.e2e_steps):
            e2e_step(t)
        f1.record(stream)
        torch.cuda.synchronize()
        pkg.device_check()
        e2e_ms = f0.elapsed_time(f1) / args.e2e_steps
        e2e_flops = 4.0 * 128 ** 3 * sum(kept_phase[t % nrot] for t in range(args.e2e_steps)) / args.e2e_steps
        e2e_ms = ranks.max_over_ranks(e2e_ms, dev)
        e2e_flops = ranks.sum_over_ranks(e2e_flops, dev)
        for c in caches:
            c.close()
        e2e = {"value": e2e_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "kind": e2e_kind}
    elif args.e2e_steps > 0:
        e2e_kind = "per layer H2D of q, k and v whole, select + attention, D2H of the output"
        nbuf = 3
        host = [tuple(t.cpu().pin_memory() for t in inputs[l]) for l in range(nbuf)]
        dbuf = [tuple(torch.empty_like(t) for t in inputs[0]) for _ in range(2)]
        hout = [torch.empty(inputs[0][0].shape, dtype=inputs[0][0].dtype, pin_memory=True) for _ in range(2)]
        cp = torch.cuda.Stream(device=dev)
        ready = [torch.cuda.Event() for _ in range(2)]
        free = [torch.cuda.Event() for _ in range(2)]
        h2d = sum(t.numel() * t.element_size() for t in host[0]) * layers
        d2h = outs[0].numel() * outs[0].element_size() * layers

        def e2e_step():
            for l in range(layers):
                b = l & 1
                with torch.cuda.stream(cp):
                    cp.wait_event(free[b])
                    for dst, src in zip(dbuf[b], host[l % nbuf]):
                        dst.copy_(src, non_blocking=True)
                    ready[b].record(cp)
                stream.wait_event(ready[b])
                q, k, v = dbuf[b]
                select_call(q, k)
                attention_call(q, k, v, outs[b])
                free[b].record(stream)
                hout[b].copy_(outs[b], non_blocking=True)
            torch.cuda.current_stream().synchronize()

        e2e_step()
        ranks.barrier()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        f1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = ranks.max_over_ranks(f0.elapsed_time(f1) / args.e2e_steps, dev)
        e2e = {"value": flops_all_ranks / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "kind": e2e_kind}

    if rank == 0:
        peak, hbm, peak_kind = peaks()
        # the committed ncu figure is one config-3 launch over all items; other workloads have no capture behind them
        tr = profiled_traffic() if args.config == 3 and not shard else None
        value = flops_all_ranks / (ms * 1e-3) / 1e12
        line = {
            "metric": f"block-sparse attn effective TFLOP/s (+ ms per 30-layer chunk), config {args.config}",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong" if shard else "weak",
            "vs_baseline": None, "dtype": "bf16" if cfg.dtype == "bf16" else "f32",
            "data": "synthetic (seeded normal Q/K/V per layer, window order, resident in HBM)",
            "config": {"workload": f"config {args.config}: {cfg.name}", "layers_per_step": layers,
                       "heads": g.heads, "q_blocks": g.nq, "k_blocks": g.nk, "topk": g.topk,
                       "kept_triples_per_layer": total_kept / layers, "l2": "inputs > L2 (371 MB per layer), no flush",
                       "launch": "eager" if args.no_graph else "CUDA graph of one step",
                       "parallelism": (f"{world} GPUs, (head, query block) items sharded, no collective" if shard
                                       else (f"{world} independent streams" if world > 1 else "1 GPU")),
                       **({"emulated_rank": args.as_rank} if shard and args.as_rank else {}),
                       **({"schedule": "persistent equal shares" if persistent else "longest-first items"}
                          if shard else {})},
            "ms_per_layer": ms / layers,
            # "rest" = step time per layer minus the attention kernel timed alone: pooling, selection and the
            # dependency gaps between the kernels of the graph
            "breakdown_ms_per_layer": {"attention": att_avg, "rest (pool, select, gaps)": sel_ms},
            "roofline": {"kernel": "attn_bf16_sm100_kernel", "bound": "tensor", "achieved": att_tflops, "peak": peak,
                         "unit": "TFLOP/s", "frac": att_tflops / peak, "peak_kind": f"{peak_kind} bf16 burst",
                         "traffic": (tr or {}).get("bytes_per_launch"),
                         "traffic_source": (tr or {}).get("source")},
            "clocks": clk,
            # per layer, unsharded: pool, selection (which orders the items), attention; sharded: pool, selection,
            # order (or schedule), attention, and the combine step when the range runs the persistent kernel
            "gpu_launches": (3 if not shard else (5 if persistent else 4)) * layers * args.steps,
            "e2e": e2e,
        }
        if not args.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_baseline(args.config)
                line["cpu_baseline"].pop("seconds", None)
            except Exception as exc:  # the baseline is reported, never required
                line["cpu_baseline"] = {"error": str(exc)}
        print(json.dumps(line), flush=True)
    ranks.barrier()
    ranks.shutdown()


def run_chunk(args):
    """The metric's workload as the reference streams it: one steady-state chunk of config `--config` (default 3, the
    1920×1152 chunk) = 30 DiT layers, each layer holding its window cache of kvLen = kv_slices − 1 slices and
    receiving the chunk's q, k_new and v_new (fresh seeded data per layer, resident in HBM). At N = 1 a layer is one
    fvsr_lcsa_forward call. At N > 1 the chunk's query blocks are split across the ranks (shard.py): each rank holds
    only its shard of q / k_new / v_new, pools it, all-gathers the pooled rows and the slice's K/V over NVLink (NCCL,
    inside the timed region), computes the full selection and attends for its own query blocks. Strong scaling: the
    chunk is the same at every N; time = max over ranks."""
    import torch
    pkg, cfgs = load_pkg()
    import importlib
    ranks = importlib.import_module("fvsr_b200.ranks")
    shard_mod = importlib.import_module("fvsr_b200.shard")
    info = ranks.rank_info()
    world, rank, local = info.world, info.rank, info.local
    if world > 1 and args.spare_sms > 0:  # NCCL's kernels must fit in the SMs the selection leaves to the gather
        os.environ.setdefault("NCCL_MAX_CTAS", str(args.spare_sms))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ranks.init(info, "nccl", timeout_s=120, device=dev)
    cfg = cfgs.CONFIGS[args.config]
    g_full = cfg.geometry()                       # q_slices = 1, kv_slices = 3: the steady chunk
    if g_full.q_slices != 1:
        raise SystemExit(f"config {args.config} has {g_full.q_slices} query slices; the chunk mode takes one")
    g = pkg.Geometry(**{**g_full.__dict__})
    kv_len, layers = g.kv_slices - g.q_slices, args.layers
    srows = g.s * 128
    comm = None
    if world > 1:
        nccl = importlib.import_module("fvsr_b200.nccl")
        comm = nccl.Comm(rank, world, dev)
    sc = shard_mod.ShardedChunk(pkg, g, kv_len, layers, rank, world, comm, dev, spare_sms=args.spare_sms)
    sh = sc.shard
    stream = torch.cuda.current_stream()
    # per layer: the seeded full tensors of the one-GPU problem (q of the chunk, K/V of cache ⊕ current), of which
    # this rank keeps its query shard, padded K/V shards of the current slice, and the cache prefill
    qs, ks, vs, full = [], [], [], []
    for l in range(layers):
        q, k, v = cfgs.synth_qkv(cfg, g_full, cfgs.seed_of(args.config, 0, l), device=dev)
        sc.prefill(l, [k[i * srows:(i + 1) * srows] for i in range(kv_len)],
                   [v[i * srows:(i + 1) * srows] for i in range(kv_len)])
        qs.append(q[sh.begin * 128:sh.end * 128].clone())
        kp = torch.zeros((sc.shard_rows(), g.channels), dtype=q.dtype, device=dev)
        vp = torch.zeros_like(kp)
        kp[:sh.blocks * 128] = k[kv_len * srows + sh.begin * 128:kv_len * srows + sh.end * 128]
        vp[:sh.blocks * 128] = v[kv_len * srows + sh.begin * 128:kv_len * srows + sh.end * 128]
        ks.append(kp)
        vs.append(vp)
        if l < args.roofline_layers:
            full.append((q, k, v))
        del q, k, v
    outs = [torch.empty((sh.blocks * 128, g.channels), dtype=qs[0].dtype, device=dev) for _ in range(2)]
    kcnt = torch.zeros((layers, g.heads, g.nq), dtype=torch.int32, device=dev)

    def step():
        st = torch.cuda.current_stream()          # the capture stream inside torch.cuda.graph
        for l in range(layers):
            sc.layer(l, qs[l], ks[l], vs[l], outs[l & 1], kcnt=kcnt[l], stream=st)

    if comm is not None:                          # set NCCL's connections up before any capture
        comm.group_start()
        comm.all_gather(sc.pq_send, sc.pq_full, stream)
        comm.group_end()
        comm.group_start()
        comm.all_gather(ks[0], torch.empty((world * ks[0].shape[0], g.channels), dtype=ks[0].dtype, device=dev),
                        sc.comm_stream)
        comm.group_end()
        torch.cuda.synchronize()
    launch = "CUDA graph of one step (page choices fixed at capture)"
    run_step = None
    if not args.no_graph:
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            run_step = graph.replay
        except Exception as exc:  # a capture the stack refuses: time the same calls eagerly
            launch = f"eager (graph capture failed: {type(exc).__name__})"
            run_step = None
            for c in sc.caches:   # the failed capture left the page tables mid-step: start the caches over
                c.reset()
            for l in range(layers):
                q, k, v = cfgs.synth_qkv(cfg, g_full, cfgs.seed_of(args.config, 0, l), device=dev)
                sc.prefill(l, [k[i * srows:(i + 1) * srows] for i in range(kv_len)],
                           [v[i * srows:(i + 1) * srows] for i in range(kv_len)])
    if run_step is None:
        if args.no_graph:
            launch = "eager"
        run_step = step
    for _ in range(max(args.warmup, 3)):
        run_step()
    torch.cuda.synchronize()
    kept = int(kcnt.sum().item())                 # the chunk's kept triples (every rank selects the same)
    ranks.barrier()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    clocks = Clocks(uuid)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t_begin = time.time()
    e0.record(stream)
    for _ in range(args.steps):
        run_step()
    e1.record(stream)
    torch.cuda.synchronize()
    clocks.mark(t_begin, time.time())
    clk = clocks.stop()
    ms = ranks.max_over_ranks(e0.elapsed_time(e1) / args.steps, dev)
    pkg.device_check()
    if comm is not None:
        comm.check()
    if run_step is not step:
        run_step = None                           # the bound replay holds the graph (and its NCCL work) alive
        graph.reset()
        del graph
    torch.cuda.synchronize()
    flops = 4.0 * 128 ** 3 * kept

    # the collective this partition adds, alone: the two K/V all-gathers of one layer (the slice's shards into a
    # page-sized buffer) on the communication stream, back to back, CUDA events on that stream, max over ranks
    gather_ms = None
    if comm is not None:
        kdst = torch.empty((world * ks[0].shape[0], g.channels), dtype=ks[0].dtype, device=dev)
        vdst = torch.empty_like(kdst)
        cs = sc.comm_stream

        def kv_gather_once():
            comm.group_start()
            comm.all_gather(ks[0], kdst, cs)
            comm.all_gather(vs[0], vdst, cs)
            comm.group_end()

        for _ in range(3):
            kv_gather_once()
        torch.cuda.synchronize()
        ranks.barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(cs)
        for _ in range(20):
            kv_gather_once()
        c1.record(cs)
        torch.cuda.synchronize()
        gather_ms = ranks.max_over_ranks(c0.elapsed_time(c1) / 20, dev)
        del kdst, vdst

    # the dominant kernel alone: the attention of whole fresh layers (one GPU's problem), CUDA events on its stream;
    # then the same launches back to back from a graph (the power-capped rate the step sees)
    L = pkg.lib()
    ws = pkg.make_workspace(g_full, dev)
    nroof = len(full)
    kidx1 = [torch.empty((g.heads, g.nq, g.nk), dtype=torch.int32, device=dev) for _ in range(nroof)]
    kcnt1 = [torch.empty((g.heads, g.nq), dtype=torch.int32, device=dev) for _ in range(nroof)]
    order = [torch.empty(g.heads * g.nq, dtype=torch.int32, device=dev) for _ in range(nroof)]
    out1 = torch.empty((g.nq * 128, g.channels), dtype=qs[0].dtype, device=dev)
    p1 = g_full.params()
    att_ms, att_kept = [], []

    def attention(i):
        q, k, v = full[i]
        pkg._check(L.fvsr_lcsa_attention_range(ctypes.byref(p1), pkg._ptr(q), pkg._ptr(k), pkg._ptr(v),
                                               pkg._ptr(kidx1[i]), pkg._ptr(kcnt1[i]), pkg._ptr(out1), 0,
                                               g.heads * g.nq, pkg._ptr(order[i]), pkg._stream()))

    for i, (q, k, v) in enumerate(full):
        pkg._check(L.fvsr_lcsa_select(ctypes.byref(p1), pkg._ptr(q), pkg._ptr(k), None, pkg._ptr(kidx1[i]),
                                      pkg._ptr(kcnt1[i]), None, None, pkg._ptr(ws), ws.numel(), pkg._stream()))
        pkg._check(L.fvsr_lcsa_item_order(ctypes.byref(p1), pkg._ptr(kcnt1[i]), 0, g.heads * g.nq,
                                          pkg._ptr(order[i]), pkg._stream()))
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        attention(i)
        a1.record(stream)
        a1.synchronize()
        att_ms.append(a0.elapsed_time(a1))
        att_kept.append(int(kcnt1[i].sum().item()))
    att_b2b = None
    if nroof and not args.no_graph:
        ag = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ag):
            for _ in range(max(1, 30 // nroof)):
                for i in range(nroof):
                    attention(i)
        for _ in range(2):
            ag.replay()
        torch.cuda.synchronize()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record(stream)
        for _ in range(3):
            ag.replay()
        b1.record(stream)
        torch.cuda.synchronize()
        att_b2b = b0.elapsed_time(b1) / (3 * max(1, 30 // nroof) * nroof)
        ag.reset()
        del ag
    del full
    att_avg = sum(att_ms) / len(att_ms)
    att_tflops = 4.0 * 128 ** 3 * (sum(att_kept) / len(att_kept)) / (att_avg * 1e-3) / 1e12
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count

    # end to end through the public API with host buffers: per layer the rank's q, k_new and v_new shards uploaded
    # from pinned memory (beside the previous layer's compute) and its output rows read back
    e2e = None
    if args.e2e_steps > 0:
        hq = [qs[l % 3].cpu().pin_memory() for l in range(3)]
        hk = [ks[l % 3].cpu().pin_memory() for l in range(3)]
        hv = [vs[l % 3].cpu().pin_memory() for l in range(3)]
        dq = [torch.empty_like(qs[0]) for _ in range(2)]
        dk = [torch.empty_like(ks[0]) for _ in range(2)]
        dv = [torch.empty_like(vs[0]) for _ in range(2)]
        hout = [torch.empty(outs[0].shape, dtype=outs[0].dtype, pin_memory=True) for _ in range(2)]
        up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        ready = [torch.cuda.Event() for _ in range(2)]
        free = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        read = [torch.cuda.Event() for _ in range(2)]
        for ev in free + read:
            ev.record(stream)
        kc2 = torch.zeros_like(kcnt)

        def e2e_step():
            for l in range(layers):
                b = l & 1
                with torch.cuda.stream(up):
                    up.wait_event(free[b])
                    dq[b].copy_(hq[l % 3], non_blocking=True)
                    dk[b].copy_(hk[l % 3], non_blocking=True)
                    dv[b].copy_(hv[l % 3], non_blocking=True)
                    ready[b].record(up)
                stream.wait_event(ready[b])
                stream.wait_event(read[b])
                sc.layer(l, dq[b], dk[b], dv[b], outs[b], kcnt=kc2[l], stream=stream)
                free[b].record(stream)
                done[b].record(stream)
                with torch.cuda.stream(down):
                    down.wait_event(done[b])
                    hout[b].copy_(outs[b], non_blocking=True)
                    read[b].record(down)
            stream.wait_stream(down)

        for _ in range(3):                        # the caches reach their steady state (every slice the same data)
            e2e_step()
        torch.cuda.synchronize()
        kept_e2e = int(kc2.sum().item())
        ranks.barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        f1.record(stream)
        torch.cuda.synchronize()
        pkg.device_check()
        e2e_ms = ranks.max_over_ranks(f0.elapsed_time(f1) / args.e2e_steps, dev)
        h2d = sum(t.numel() * t.element_size() for t in (hq[0], hk[0], hv[0])) * layers
        d2h = outs[0].numel() * outs[0].element_size() * layers
        e2e = {"value": 4.0 * 128 ** 3 * kept_e2e / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
               "kind": "per layer: this rank's q / k_new / v_new shards from pinned host memory, the layer call "
                       "(collectives included), its output rows back to the host"}

    if rank == 0:
        peak, hbm, peak_kind = peaks()
        sustained = None
        try:
            sustained = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops_sustained"])
        except Exception:
            pass
        tr = profiled_traffic() if args.config == 3 else None
        value = flops / (ms * 1e-3) / 1e12
        par = "1 GPU" if world == 1 else (f"{world} GPUs: query blocks split ({sh.width} per rank), pooled rows and "
                                          f"the slice's K/V all-gathered by NCCL inside the step")
        line = {
            "metric": f"block-sparse attn effective TFLOP/s (+ ms per 30-layer chunk), config {args.config}",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16" if cfg.dtype == "bf16" else "f32",
            "data": "synthetic (seeded normal Q/K/V per layer, window order, resident in HBM)",
            "config": {"workload": f"config {args.config}: {cfg.name}, one steady-state streamed chunk",
                       "layers_per_step": layers, "heads": g.heads, "q_blocks": g.nq, "k_blocks": g.nk,
                       "kv_len": kv_len, "topk": g.topk, "kept_triples_per_layer": kept / layers,
                       "l2": f"per layer {3 * g.nq * 128 * g.channels * 2 / 1e6:.0f} MB of chunk data + "
                             f"{2 * kv_len * srows * g.channels * 2 / 1e6:.0f} MB of cache read (> L2), no flush",
                       "launch": launch, "parallelism": par},
            "ms_per_layer": ms / layers,
            # N = 1: the attention of a layer back to back in a graph (as in the step, under the power cap) and the
            # rest. N > 1: the rank's layer (max over ranks), the K/V all-gather alone, and the one-GPU references
            "breakdown_ms_per_layer": (
                ({"attention back to back": att_b2b, "rest (append, pooling, selection, gaps)": ms / layers - att_b2b}
                 if world == 1 else
                 {"layer (max over ranks)": ms / layers,
                  "kv_all_gather_alone": gather_ms,
                  "kv_all_gather_bytes_received_per_rank": 2 * (world - 1) * ks[0].numel() * ks[0].element_size(),
                  "one_gpu_attention_of_the_whole_layer_back_to_back": att_b2b,
                  "ideal_layer (one-GPU attention / N)": att_b2b / world})
                if att_b2b else None),
            "chunk_frac_of_sustained_peak": (value / world / sustained) if sustained and cfg.dtype == "bf16" else None,
            "roofline": (
                {"kernel": "attn_bf16_sm100_kernel", "bound": "tensor", "achieved": att_tflops, "peak": peak,
                 "unit": "TFLOP/s", "frac": att_tflops / peak, "peak_kind": f"{peak_kind} bf16 burst",
                 "ms_alone_per_layer": att_avg, "traffic": (tr or {}).get("bytes_per_launch"),
                 "traffic_source": (tr or {}).get("source"),
                 "timed": f"the attention of {len(att_ms)} whole fresh layers alone, CUDA events"}
                if cfg.dtype == "bf16" else
                {"kernel": "attn_f32_kernel", "bound": "fp32 FMA", "achieved": att_tflops,
                 "peak": nsm * 128 * 2 * (clk.get("sm_mhz") or 1965.0) * 1e6 / 1e12, "unit": "TFLOP/s",
                 "frac": att_tflops / (nsm * 128 * 2 * (clk.get("sm_mhz") or 1965.0) * 1e6 / 1e12),
                 "peak_kind": f"FFMA: {nsm} SMs x 128 lanes x 2 FLOP x the sampled SM clock",
                 "ms_alone_per_layer": att_avg, "traffic": None,
                 "timed": f"the attention of {len(att_ms)} whole fresh layers alone, CUDA events"}),
            "clocks": clk,
            # per layer: N = 1 key pooling (the append), query pooling, selection, attention; N > 1 two pooling
            # launches, selection, attention (two launches when split around the gather; NCCL's kernels not counted)
            "gpu_launches": (4 if world == 1 or sc.partial is None else 5) * layers * args.steps,
            "e2e": e2e,
        }
        if not args.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_baseline(args.config)
                line["cpu_baseline"].pop("seconds", None)
            except Exception as exc:  # the baseline is reported, never required
                line["cpu_baseline"] = {"error": str(exc)}
        print(json.dumps(line), flush=True)
    ranks.barrier()
    torch.cuda.synchronize()
    sc.close()
    if comm is not None:                          # no graph holds NCCL work any more: the teardown cannot wait
        comm.destroy()
    ranks.shutdown()


def run_stream4(args):
    """Config 4 as BASELINE.json states it: a streamed sequence of 10 chunks at the 1280×768 output (12 heads, 6×10
    spatial blocks): chunk 0 carries 3 temporal slices, every later chunk one; kvLen 2 (the window attends to the
    current slice plus two cached ones); 30 DiT layers per chunk, each with its own window cache appended in place and
    trimmed (DiT.swift:504-538, fvsr_lcsa_forward); Q/K/V seeded per (chunk, layer) and resident in HBM before the
    timed region. One step = the whole 10-chunk sequence (the caches start empty). Prints one JSON line."""
    import torch
    pkg, cfgs = load_pkg()
    cfg = cfgs.CONFIGS[4]
    layers, chunks, kv_len = args.layers, 10, 2
    g0 = cfg.geometry(q_slices=3)
    srows = g0.s * 128
    data = []                                   # per chunk, per layer: (q, k_new, v_new, geometry)
    for c in range(chunks):
        qs_ = 3 if c == 0 else 1
        row = []
        for l in range(layers):
            have = 0 if c == 0 else min(kv_len, 3 + c - 1)
            g = cfg.geometry(q_slices=qs_, kv_slices=have + qs_)
            q, k, v = cfgs.synth_qkv(cfg, g, cfgs.seed_of(4, c, l), kv_rows=qs_ * srows)
            row.append((q, k, v, g))
        data.append(row)
    caches = [pkg.KVCache(g0, kv_len, 3) for _ in range(layers)]
    wsg = pkg.Geometry(**{**g0.__dict__, "kv_slices": kv_len + 3})
    ws = pkg.make_workspace(wsg)
    out = [torch.empty((3 * srows, g0.channels), dtype=torch.bfloat16, device="cuda")]
    kcnt = [torch.zeros((layers, g0.heads, (3 if c == 0 else 1) * g0.s), dtype=torch.int32, device="cuda")
            for c in range(chunks)]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(chunks + 1)]

    def sequence(timed=False):
        for c in caches:
            c.reset()
        if timed:
            ev[0].record()
        for c in range(chunks):
            for l in range(layers):
                q, k, v, g = data[c][l]
                pkg.lcsa_forward(q, k, v, caches[l], g, out=out[0][: q.shape[0]], kcnt=kcnt[c][l], workspace=ws)
            if timed:
                ev[c + 1].record()

    for _ in range(max(args.warmup, 3)):
        sequence()
    torch.cuda.synchronize()
    per_chunk = []
    for _ in range(max(args.steps, 1)):
        sequence(timed=True)
        torch.cuda.synchronize()
        per_chunk.append([ev[c].elapsed_time(ev[c + 1]) for c in range(chunks)])
    pkg.device_check()
    kept = [int(kcnt[c].sum().item()) for c in range(chunks)]
    import statistics
    ms = [statistics.median(x[c] for x in per_chunk) for c in range(chunks)]
    total_ms = sum(ms)
    fl = 4.0 * 128 ** 3
    for c in caches:
        c.close()
    print(json.dumps({
        "metric": "config 4 streamed sequence: effective TFLOP/s over 10 chunks (+ ms per 30-layer chunk)",
        "value": fl * sum(kept) / (total_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_sequence": total_ms,
        "ms_per_chunk": {"chunk0 (3 slices)": ms[0], "steady (median of chunks 1-9)": statistics.median(ms[1:])},
        "tflops_per_chunk": [fl * kept[c] / (ms[c] * 1e-3) / 1e12 for c in range(chunks)],
        "kept_triples_per_chunk": kept, "steps": args.steps, "warmup": args.warmup, "gpu_launches_per_layer": 4,
        "launch": "host C-ABI calls (fvsr_lcsa_forward per layer), CUDA events per chunk",
        "config": {"workload": "config 4: 1280x768, 12 heads, 6x10 blocks, chunk 0 = 3 slices then 1, kvLen 2, "
                               "30 layers per chunk, R=11, keep 60%", "dtype": "bf16"}}), flush=True)


def run_linear(args):
    """The DiT block's linear layers at the config's chunk (M = the chunk's tokens; FlashVSR dim 1536, FFN 8960) on
    the tcgen05 GEMM (fvsr_linear / fvsr_linear_qkv): the q/k/v projection, the output projection, the FFN's first
    layer with GELU(tanh) and its second with the gated residual (DiT.swift:496-499, 539-547). Each shape: 10 calls
    from a CUDA graph after warm-up, CUDA events; TFLOP/s = 2·M·N·K per call ÷ time, against the measured bf16 burst
    peak; torch.matmul (cuBLAS) on the same shapes beside it. Prints one JSON line."""
    import torch
    pkg, cfgs = load_pkg()
    cfg = cfgs.CONFIGS[args.config]
    g = cfg.geometry()
    m = g.nq * 128
    d, f = 1536, 8960
    gen = torch.Generator(device="cuda").manual_seed(9)

    def rnd(*shape, scale=1.0):
        return (scale * torch.randn(shape, generator=gen, device="cuda")).to(torch.bfloat16)

    x = rnd(m, d)
    h = rnd(m, f)
    w_qkv, b_qkv = rnd(3 * d, d, scale=d ** -0.5), rnd(3 * d, scale=0.1)
    w_o, b_o = rnd(d, d, scale=d ** -0.5), rnd(d, scale=0.1)
    w_1, b_1 = rnd(f, d, scale=d ** -0.5), rnd(f, scale=0.1)
    w_2, b_2 = rnd(d, f, scale=f ** -0.5), rnd(d, scale=0.1)
    gate = rnd(d, scale=0.5)
    tok = rnd(m, d)
    outs = [torch.empty((m, d), dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    hid = torch.empty((m, f), dtype=torch.bfloat16, device="cuda")
    shapes = {
        "qkv": (3 * d, d, lambda: pkg.linear_qkv(x, w_qkv, b_qkv, outs=outs),
                lambda: torch.matmul(x, w_qkv.t())),
        "o": (d, d, lambda: pkg.linear(x, w_o, b_o, out=outs[0]), lambda: torch.matmul(x, w_o.t())),
        "ffn1_gelu": (f, d, lambda: pkg.linear(x, w_1, b_1, epilogue=pkg.FVSR_LINEAR_GELU, out=hid),
                      lambda: torch.matmul(x, w_1.t())),
        "ffn2_gated_residual": (d, f, lambda: pkg.linear(h, w_2, b_2, epilogue=pkg.FVSR_LINEAR_GATED_RESIDUAL,
                                                         gate=gate, resid=tok, out=outs[1]),
                                lambda: torch.matmul(h, w_2.t())),
    }
    peak, _, kind = peaks()
    res = {}
    total_flop, total_ms = 0.0, 0.0
    for name, (n, k, ours, lib_fn) in shapes.items():
        flop = 2.0 * m * n * k
        t_ours = graph_time_us(ours, 10, max(args.warmup, 3)) / 1e3
        t_lib = graph_time_us(lib_fn, 10, max(args.warmup, 3)) / 1e3
        res[name] = {"m": m, "n": n, "k": k, "ms": t_ours, "tflops": flop / (t_ours * 1e-3) / 1e12,
                     "frac_of_peak": flop / (t_ours * 1e-3) / 1e12 / peak,
                     "torch_matmul_ms": t_lib, "torch_matmul_tflops": flop / (t_lib * 1e-3) / 1e12}
        total_flop += flop
        total_ms += t_ours
    # the block's row normalisations at the same M (bytes moved = read + write of (M, d) bf16)
    vecs = [rnd(d, scale=0.3) for _ in range(4)]
    nout = torch.empty_like(x)
    norm_calls = {"layernorm_modulated": lambda: pkg.layernorm(x, shift=vecs[0], scale=vecs[1], out=nout),
                  "layernorm_affine": lambda: pkg.layernorm(x, weight=vecs[2], bias=vecs[3], out=nout),
                  "rmsnorm": lambda: pkg.rmsnorm(x, vecs[2], out=nout),
                  "copy_same_bytes": lambda: nout.copy_(x)}
    norms = {}
    for name, fn in norm_calls.items():
        us = graph_time_us(fn, 20, max(args.warmup, 3))
        norms[name] = {"us": us, "gbs": 2 * m * d * 2 / (us * 1e-6) / 1e9}
    pkg.device_check()
    print(json.dumps({"metric": f"DiT block linear layers on tcgen05, config {args.config} chunk (M = {m})",
                      "value": total_flop / (total_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_block": total_ms,
                      "peak": peak, "peak_kind": f"{kind} bf16 burst", "frac": total_flop / (total_ms * 1e-3) / 1e12 / peak,
                      "layers": res, "norms": norms, "gpu_launches_per_block": 4, "launch": "CUDA graph of 10 calls per shape",
                      "note": "torch_matmul is cuBLAS on the same shapes without the bias / epilogue, for reference"}),
          flush=True)


def run_block(args):
    """Whole DiT blocks (blockForward, DiT.swift:486-549) on the library's kernels (dit.block_forward): one steady
    streamed chunk of config `--config` (default 3: 1920×1152, 17,280 tokens, dim 1536, 12 heads, FFN 8960) through
    `--layers` blocks chained as in the model (block l's output is block l+1's input), each block with its own
    random-initialised weights, cached context K/V (512 text tokens) and window K/V cache of kvLen 2 slices (prefilled).
    A step = the chunk through all blocks; CUDA events; then one more step with an event after each stage for the
    breakdown. TFLOP/s = the algorithmic FLOPs of every linear layer, the LCSA over its kept triples and the
    cross-attention ÷ time. Prints one JSON line."""
    import torch
    pkg, cfgs = load_pkg()
    import importlib
    dit = importlib.import_module("fvsr_b200.dit")
    cfg = cfgs.CONFIGS[args.config]
    g = cfg.geometry()
    if g.q_slices != 1 or cfg.dtype != "bf16":
        raise SystemExit(f"config {args.config}: the block mode takes a bf16 one-slice chunk")
    c, ffn, lc, kv_len, layers = g.channels, 8960, 512, g.kv_slices - g.q_slices, args.layers
    rows, srows = g.nq * 128, g.s * 128
    gen = torch.Generator(device="cuda").manual_seed(4242)
    weights, caches, mods = [], [], []
    for l in range(layers):
        weights.append(dit.BlockWeights.random(c=c, f=ffn, lc=lc, seed=100 + l))
        cache = pkg.KVCache(g, kv_len=kv_len, max_new_slices=1)
        for _ in range(kv_len):
            ks = torch.randn((srows, c), generator=gen, device="cuda").to(torch.bfloat16)
            cache.append(ks, torch.randn((srows, c), generator=gen, device="cuda").to(torch.bfloat16), 1)
        caches.append(cache)
        mods.append([(s * torch.randn((c,), generator=gen, device="cuda")).to(torch.bfloat16)
                     for s in (0.2, 0.2, 0.5, 0.2, 0.2, 0.5)])
    tok0 = torch.randn((rows, c), generator=gen, device="cuda").to(torch.bfloat16)
    tok = torch.empty_like(tok0)
    rope = pkg.rope_tables(2, 8 * g.bh, 8 * g.bw, t0=4 + 2 * 3)
    buf = dit.BlockBuffers(rows, c, ffn)
    ws = pkg.make_workspace(g)
    kcnt = torch.zeros((layers, g.heads, g.nq), dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()

    def step(timeline=None):
        tok.copy_(tok0)
        for l in range(layers):
            dit.block_forward(weights[l], tok, mods[l], caches[l], g, rope, buf, ws, kcnt=kcnt[l], stream=stream,
                              timeline=timeline)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    kept = [int(x) for x in kcnt.sum(dim=(1, 2)).tolist()]
    flops = sum(dit.block_flops(rows, c, ffn, lc, k) for k in kept)
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(0).uuid)
    except Exception:
        pass
    clocks = Clocks(uuid)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t_begin = time.time()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    clocks.mark(t_begin, time.time())
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    timeline = []
    step(timeline)
    torch.cuda.synchronize()
    pkg.device_check()
    stages = {}
    for (_, a), (name, b) in zip(timeline, timeline[1:]):
        if name != "begin":
            stages[name] = stages.get(name, 0.0) + a.elapsed_time(b)
    total = sum(stages.values())
    lin_flop = 2.0 * rows * c * (6 * c + 2 * ffn) * layers
    lcsa_flop = sum(4.0 * 128 ** 3 * k for k in kept)
    stage_flop = {"qkv": 2.0 * rows * c * 3 * c, "lcsa": lcsa_flop / layers, "o": 2.0 * rows * c * c,
                  "ca.q": 2.0 * rows * c * c, "ca.attention": 4.0 * rows * lc * c, "ca.o": 2.0 * rows * c * c,
                  "ffn1 (GELU)": 2.0 * rows * c * ffn, "ffn2": 2.0 * rows * ffn * c}
    peak, _, kind = peaks()
    for cch in caches:
        cch.close()
    value = flops / (ms * 1e-3) / 1e12
    print(json.dumps({
        "metric": f"DiT block stack effective TFLOP/s, config {args.config} streamed chunk", "value": value,
        "unit": "TFLOP/s", "ms_per_step": ms, "ms_per_block": ms / layers, "steps": args.steps,
        "warmup": args.warmup, "layers": layers, "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic (random-init block weights, seeded tokens, prefilled caches)",
        "frac_of_peak": value / peak, "peak": peak, "peak_kind": f"{kind} bf16 burst",
        "flop_per_step": {"linear": lin_flop, "lcsa": lcsa_flop, "cross_attention": 4.0 * rows * lc * c * layers},
        "kept_triples_per_block": sum(kept) / layers,
        "breakdown_ms_per_block": {k: v / layers for k, v in stages.items()},
        "breakdown_share": {k: v / total for k, v in stages.items()},
        "stage_tflops": {k: fl * layers / (stages[k] * 1e-3) / 1e12 for k, fl in stage_flop.items()},
        "norm_gbs": {k: 4.0 * rows * c * layers / (stages[k] * 1e-3) / 1e9 for k in ("norm1", "norm3", "ca.norm_q",
                                                                                    "norm2")},
        "clocks": clk,
        "config": {"workload": f"config {args.config}: {cfg.name}, one steady chunk ({rows} tokens) through "
                               f"{layers} blocks", "dim": c, "ffn": ffn, "context_tokens": lc, "heads": g.heads,
                   "kv_len": kv_len, "topk": g.topk, "launch": "host C-ABI calls, no graph", "l2": "inputs > L2"}}),
        flush=True)


def run_kv_append(args):
    """The window cache's in-place append (fvsr_kv_cache_append + trim, DiT.swift:507-511, 532-538) as HBM traffic:
    per chunk the chunk's q_slices new slices of K and V are read and written into their cache pages and the K slices
    are pooled. Prints one JSON line: achieved GB/s of those algorithmic bytes against the measured copy bandwidth."""
    import torch
    pkg, cfgs = load_pkg()
    cfg = cfgs.CONFIGS[args.config]
    g = cfg.geometry()
    kv_len = g.kv_slices - g.q_slices
    rows = g.q_slices * g.s * 128
    elt = 2 if cfg.dtype == "bf16" else 4
    # enough distinct source chunks that successive appends read more than the 126 MB L2 holds
    nbuf = max(2, -(-3 * 126_000_000 // (2 * rows * g.channels * elt)))
    srcs = [cfgs.synth_qkv(cfg, g, 777 + i, kv_rows=rows)[1:] for i in range(nbuf)]
    cache = pkg.KVCache(g, kv_len, g.q_slices)
    while cache.slices < kv_len:
        cache.append(srcs[0][0][: g.s * 128], srcs[0][1][: g.s * 128], 1)
    # K and V new rows read once and written once; the pooled K vectors (fp32, one per block and head) written once.
    bytes_per = 2 * 2 * rows * g.channels * elt + g.q_slices * g.s * g.channels * 4
    n = max(args.steps, 1) * 20
    it = [0]

    def one():
        k, v = srcs[it[0] % nbuf]
        it[0] += 1
        cache.append(k, v, g.q_slices)
        cache.trim()

    for _ in range(max(args.warmup, 3)):
        one()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # host-launched: one C-ABI append + trim per chunk, as a caller issues them
    e0.record()
    for _ in range(n):
        one()
    e1.record()
    torch.cuda.synchronize()
    eager_us = e0.elapsed_time(e1) * 1e3 / n
    # device rate: the same n appends captured once in a CUDA graph (pages chosen at capture) and replayed
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(n):
            one()
    reps = 5
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    pkg.device_check()
    us = e0.elapsed_time(e1) * 1e3 / (reps * n)
    del graph
    _, hbm, kind = peaks()
    gbs = bytes_per / (us * 1e-6) / 1e9
    cache.close()
    print(json.dumps({"metric": f"KV-cache append GB/s, config {args.config} chunk", "value": gbs, "unit": "GB/s",
                      "us_per_chunk": us, "bytes_per_chunk": bytes_per, "chunks": reps * n, "gpu_launches": reps * n,
                      "launch": "CUDA graph of the appends",
                      "eager": {"us_per_chunk": eager_us, "value": bytes_per / (eager_us * 1e-6) / 1e9,
                                "note": "one host call of fvsr_kv_cache_append + trim per chunk (host-paced)"},
                      "l2": f"{nbuf} source chunks rotated ({nbuf * 2 * rows * g.channels * elt / 1e6:.0f} MB > L2)",
                      "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                                   "peak_kind": kind},
                      "config": {"workload": f"config {args.config}: {cfg.name}", "new_slices": g.q_slices,
                                 "slice_blocks": g.s, "heads": g.heads, "dtype": cfg.dtype}}), flush=True)


def run_prepare(args):
    """The q/k/v side of one layer (fvsr_lcsa_prepare: WanRMSNorm + ropeApply of q and k, windowPartition of q, k, v,
    pooled q and k; DiT.swift:34-47, 100-107, 113-118, 161-162) as HBM traffic, and the whole token-order layer
    (fvsr_lcsa_forward_tokens) beside the window-order one (fvsr_lcsa_forward). Prints one JSON line."""
    import torch
    pkg, cfgs = load_pkg()
    cfg = cfgs.CONFIGS[args.config]
    g = cfg.geometry()
    L, C = g.nq * 128, g.channels
    dt = torch.bfloat16 if cfg.dtype == "bf16" else torch.float32
    elt = 2 if cfg.dtype == "bf16" else 4
    # enough distinct (q, k, v) sets that successive calls read more than the 126 MB L2 holds
    nbuf = max(2, -(-3 * 126_000_000 // (3 * L * C * elt)))
    gen = torch.Generator(device="cuda").manual_seed(4321)
    srcs = [[torch.randn((L, C), generator=gen, device="cuda").to(dt) for _ in range(3)] for _ in range(nbuf)]
    wq, wk = ((1.0 + 0.1 * torch.randn((C,), generator=gen, device="cuda")).to(dt) for _ in range(2))
    tabs = pkg.rope_tables(2 * g.q_slices, 8 * g.bh, 8 * g.bw, t0=4)
    outs = {n: torch.empty((L, C), dtype=dt, device="cuda") for n in ("q", "k", "v")}
    pooled = [torch.empty((g.nq, C), dtype=torch.float32, device="cuda") for _ in range(2)]
    lib, p = pkg.lib(), g.params()
    it = [0]

    def one():
        q, k, v = srcs[it[0] % nbuf]
        it[0] += 1
        pkg._check(lib.fvsr_lcsa_prepare(ctypes.byref(p), q.data_ptr(), k.data_ptr(), v.data_ptr(), wq.data_ptr(),
                                         wk.data_ptr(), 1e-6, tabs[0].data_ptr(), tabs[1].data_ptr(),
                                         outs["q"].data_ptr(), outs["k"].data_ptr(), outs["v"].data_ptr(),
                                         pooled[0].data_ptr(), pooled[1].data_ptr(),
                                         torch.cuda.current_stream().cuda_stream))

    n = max(args.steps, 1) * 20
    us = graph_time_us(one, n, max(args.warmup, 3))
    # algorithmic bytes: q, k, v read and written once; the rotation tables read once; pooled q and k written
    bytes_per = 2 * 3 * L * C * elt + 2 * L * 64 * 4 + 2 * g.nq * C * 4
    _, hbm, kind = peaks()
    gbs = bytes_per / (us * 1e-6) / 1e9

    # whole layer: token-order (prepare into the cache, select, attend, token-order output) vs window-order
    kv_len = g.kv_slices - g.q_slices
    layer = {}
    for mode in ("tokens", "window"):
        cache = pkg.KVCache(g, kv_len, g.q_slices)
        while cache.slices < kv_len:
            cache.append(outs["k"][: g.s * 128], outs["v"][: g.s * 128], 1)
        full = pkg.Geometry(**{**g.__dict__, "kv_slices": g.kv_slices})
        ws = pkg.make_workspace(full)
        out = torch.empty((L, C), dtype=dt, device="cuda")
        qwin = torch.empty_like(out)
        it[0] = 0

        def layer_call():
            q, k, v = srcs[it[0] % nbuf]
            it[0] += 1
            if mode == "tokens":
                pkg.lcsa_forward_tokens(q, k, v, cache, g, norm_q=wq, norm_k=wk, eps=1e-6, rope=tabs, q_win=qwin,
                                        out=out, workspace=ws)
            else:
                pkg.lcsa_forward(q, k, v, cache, g, out=out, workspace=ws)

        layer[mode] = graph_time_us(layer_call, max(args.steps, 1) * 5, max(args.warmup, 3)) / 1e3
        cache.close()
    pkg.device_check()
    print(json.dumps({"metric": f"prepare GB/s (RMSNorm + RoPE + window partition + pooling), config {args.config}",
                      "value": gbs, "unit": "GB/s", "us_per_call": us, "bytes_per_call": bytes_per,
                      "gpu_launches": n, "launch": "CUDA graph of the calls",
                      "l2": f"{nbuf} source sets rotated ({nbuf * 3 * L * C * elt / 1e6:.0f} MB > L2)",
                      "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                                   "peak_kind": kind},
                      "layer_ms": {"forward_tokens (linear outputs in, token order out)": layer["tokens"],
                                   "forward (window order in and out, no norm or rotation)": layer["window"]},
                      "config": {"workload": f"config {args.config}: {cfg.name}", "tokens": L, "channels": C,
                                 "dtype": cfg.dtype}}), flush=True)


def run_stream(args):
    """Whole chunks through the streaming driver (fvsr_stream_*): the reference's chunk loop for `layers` DiT blocks at
    the config's output size with the reference's defaults (top-k ratio 2·768·1280/(H·W), kvRatio 3, range 11) —
    each layer from its linear outputs (token order) to the attention output (token order). Synthetic linear outputs
    per layer (three rotated sets); chunk 0 (3 slices) and then steady chunks (1 slice against kvLen + 1)."""
    import torch
    pkg, cfgs = load_pkg()
    cfg = cfgs.CONFIGS[args.config]
    out_h, out_w = cfg.bh * 128, cfg.bw * 128
    layers = args.layers or cfg.layers
    st = pkg.Stream(cfg.heads, out_h, out_w, layers, pkg.FVSR_BF16 if cfg.dtype == "bf16" else pkg.FVSR_F32)
    st.begin()
    dt = torch.bfloat16 if cfg.dtype == "bf16" else torch.float32
    gen = torch.Generator(device="cuda").manual_seed(2468)
    C = cfg.heads * 128
    sets = []
    for chunk_kind in (0, 1):
        g = st.geometry(chunk_kind)[0]
        L = g.nq * 128
        sets.append([[torch.randn((L, C), generator=gen, device="cuda").to(dt) for _ in range(3)] for _ in range(3)])
    norms = [[(1.0 + 0.1 * torch.randn((C,), generator=gen, device="cuda")).to(dt) for _ in range(2)]
             for _ in range(layers)]
    outs = [torch.empty((st.geometry(k)[0].nq * 128, C), dtype=dt, device="cuda") for k in (0, 1)]
    qwin = [torch.empty_like(o) for o in outs]
    kcnts = [torch.zeros((layers, cfg.heads, st.geometry(k)[0].nq), dtype=torch.int32, device="cuda") for k in (0, 1)]
    kept = {}

    def chunk(k):
        kind = 0 if k == 0 else 1
        g = st.geometry(k)[0]
        st.start_chunk(k)
        for i in range(layers):
            q, kk, v = sets[kind][i % 3]
            st.layer(i, q, kk, v, norm_q=norms[i][0], norm_k=norms[i][1], eps=1e-6, q_win=qwin[kind],
                     out=outs[kind], kcnt=kcnts[kind][i])
        return g

    e = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    torch.cuda.synchronize()
    e[0].record()
    g0 = chunk(0)
    e[1].record()
    torch.cuda.synchronize()
    ms0 = e[0].elapsed_time(e[1])
    kept[0] = int(kcnts[0].sum().item())
    k = 1
    for _ in range(max(args.warmup, 3)):
        chunk(k)
        k += 1
    n = max(args.steps, 1)
    torch.cuda.synchronize()
    e[0].record()
    for _ in range(n):
        g1 = chunk(k)
        k += 1
    e[1].record()
    torch.cuda.synchronize()
    pkg.device_check()
    ms1 = e[0].elapsed_time(e[1]) / n
    kept[1] = int(kcnts[1].sum().item())
    st.close()
    fl = cfgs.kept_flops
    print(json.dumps({"metric": f"streaming chunk through the driver, config {args.config} output size, reference "
                                "defaults", "value": fl(kept[1]) / (ms1 * 1e-3) / 1e12, "unit": "TFLOP/s",
                      "ms_per_chunk": ms1, "chunks_timed": n, "layers": layers,
                      "chunk0": {"ms": ms0, "q_slices": g0.q_slices, "kept_triples": kept[0],
                                 "tflops": fl(kept[0]) / (ms0 * 1e-3) / 1e12},
                      "steady": {"q_slices": g1.q_slices, "kv_slices": "kvLen 3 + the current slice", "topk": g1.topk,
                                 "kept_triples_per_chunk": kept[1]},
                      "launch": "host C-ABI calls per layer (fvsr_stream_layer), no graph",
                      "config": {"workload": f"{out_w}x{out_h} output, {cfg.heads} heads, topk ratio default",
                                 "dtype": cfg.dtype}}), flush=True)


def graph_time_us(fn, n, warmup):
    """Device µs per call of fn (which launches on the current stream): n calls captured once in a CUDA graph, the
    graph replayed after warm-up, CUDA events around the replays."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(n):
            fn()
    reps = 5
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) * 1e3 / (reps * n)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1, help="GPUs of the run (one process per GPU under torchrun)")
    ap.add_argument("--steps", type=int, default=20,
                    help="timed steps (one step = one 30-layer chunk; 20 keep the clock sampler inside the region "
                         "for about ten samples)")
    ap.add_argument("--warmup", type=int, default=3, help="untimed warm-up steps (at least 3)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"],
                    help="ours: the CUDA path; reference: the CPU arm (the oracle port on the host cores)")
    ap.add_argument("--config", type=int, default=3, help="workload 1-5 (configs.py); 3 = the metric's chunk")
    ap.add_argument("--layers", type=int, default=30, help="layer calls per step")
    ap.add_argument("--e2e-steps", type=int, default=2,
                    help="steps of the end-to-end measurement through the C ABI with host buffers (0 = skip)")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip timing the CPU oracle on a sample")
    ap.add_argument("--as-rank", default=None, metavar="R/N",
                    help="development: one GPU times rank R's share of an N-way sharded run (no process group)")
    ap.add_argument("--no-split", action="store_true",
                    help="sharded runs: longest-first item order without splitting long key lists")
    ap.add_argument("--no-graph", action="store_true", help="launch the step's kernels one by one instead of a CUDA graph")
    ap.add_argument("--shard", dest="shard", action="store_true", default=None,
                    help="split the config's (head, query block) items across the ranks (default for config 5)")
    ap.add_argument("--replicas", dest="shard", action="store_false",
                    help="one independent copy of the config per rank (default except for config 5)")
    ap.add_argument("--chunk", action="store_true",
                    help="the streamed-chunk step (query blocks split across ranks at N > 1) for any config, 5 included")
    ap.add_argument("--spare-sms", type=int, default=32,
                    help="chunk mode, N > 1: SMs the selection leaves to the K/V gather started before it (0: the gather "
                         "starts after the selection)")
    ap.add_argument("--fresh", action="store_true",
                    help="30 independent layer calls on fresh full Q/K/V (no cache) instead of a streamed chunk")
    ap.add_argument("--roofline-layers", type=int, default=8,
                    help="chunk mode: fresh layers whose attention is timed alone for the roofline")
    ap.add_argument("--kv-append", action="store_true",
                    help="measure the window cache's in-place append (HBM GB/s) instead of the layer step")
    ap.add_argument("--prepare", action="store_true",
                    help="measure the token-order q/k/v pass (HBM GB/s) and the token-order layer")
    ap.add_argument("--linear", action="store_true",
                    help="the DiT block's linear layers at the config's chunk on the tcgen05 GEMM (vs cuBLAS)")
    ap.add_argument("--stream4", action="store_true",
                    help="config 4 as a streamed sequence: 10 chunks of 1280x768, chunk 0 of 3 slices, kvLen 2")
    ap.add_argument("--stream", action="store_true",
                    help="run whole chunks through the streaming driver (reference chunk loop and defaults)")
    ap.add_argument("--block", action="store_true",
                    help="whole DiT blocks (norms, linear layers, LCSA, cross-attention, FFN) on a streamed chunk")
    args = ap.parse_args()
    if args.block:
        run_block(args)
        return
    if args.stream:
        run_stream(args)
        return
    if args.stream4:
        run_stream4(args)
        return
    if args.linear:
        run_linear(args)
        return
    if args.kv_append:
        run_kv_append(args)
        return
    if args.prepare:
        run_prepare(args)
        return
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif not args.chunk and (args.fresh or args.shard is not None or args.as_rank or args.config == 5):
        run_ours(args)
    else:
        run_chunk(args)


if __name__ == "__main__":
    main()
