#!/usr/bin/env python
"""Benchmark of the flat HTRC operator on B200: milliseconds per attention layer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg3|cfg2]

Workload (default cfg3: the benchmark's full-resolution configuration): one layer = 24 heads of a 32x48x84 video latent
(129,024 tokens), d=128, bf16 Q/K/V from the seeded smooth-field generator (htrc_b200.synth), leaf 64,
tile 64, fast mode (256 exact leaves), INT8 store.  A step is one whole layer: every head runs the full
operator (key pack, tile prep, leaf stats, row-max selection, routing, far+near attention).  Under
torchrun the 24 heads are split across the N ranks and the bf16 outputs are all-gathered over NCCL on a
side stream, overlapped with the next head.

Printed JSON line (rank 0): value = ms per layer, device-resident inputs, max over ranks; e2e = the same
through the public API (htrc_b200.forward_into) with pinned host inputs and outputs, host<->device copies
inside the timed region; roofline of the dominant kernel from live CUDA events; cpu_baseline = the
oracle port timed on a bounded tile sample on this host (rank 0, N=1).

--impl reference times the reference's algorithm on the host CPU (the NumPy oracle port of
h3/htrc_flat.py's production path, all host threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "flat-HTRC ms per 129k-token 24-head d128 layer @1/8 B200; mean |ΔlogZ|"
WORKLOADS = {
    "cfg3": dict(grid=(32, 48, 84), heads=24, exact_leaves=256,
                 name="cfg3: 129,024-token 32x48x84 latent layer, 24 heads, d128, leaf 64, tile 64, fast (E=256), INT8"),
    "cfg2": dict(grid=(16, 32, 32), heads=24, exact_leaves=256,
                 name="cfg2: 16,384-token 16x32x32 latent layer, 24 heads, d128, leaf 64, tile 64, fast (E=256), INT8"),
    # profiling-sized case: one head, half of cfg3's frames (leaf state ~400 MB > L2, < 1 GB on the device)
    "prof": dict(grid=(16, 48, 84), heads=1, exact_leaves=256,
                 name="prof: one 64,512-token 16x48x84 head, d128, leaf 64, tile 64, fast (E=256), INT8"),
}
LAUNCHES_PER_HEAD = 6      # key pack, tile prep, leaf stats, row-max, route, tile attention


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg3", choices=list(WORKLOADS))
    ap.add_argument("--cpu-tiles", type=int, default=4, help="tiles of the CPU-baseline sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-modes", action="store_true", help="skip the per-mode head timings")
    ap.add_argument("--store", default="int8", choices=["int8", "fp8"],
                    help="far-field state: int8 (the production path, the headline) or fp8 (e4m3 state, store='fp8'; "
                         "no oracle sample)")
    ap.add_argument("--streams", type=int, default=2, choices=[1, 2],
                    help="heads of a layer alternate over this many streams, each with its own workspace (2, the "
                         "default: one head's small kernels and the tile kernel's last partial wave overlap the "
                         "next head; the per-stage events then include that overlap)")
    return ap.parse_args()


# ------------------------------------------------------------------------------------------ helpers
def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.proc = None
        self.th = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.th = threading.Thread(target=self._read, daemon=True)
        self.th.start()
        # the first query initialises NVML, which can stall the GPU for a while: let it finish before the
        # caller's timed region starts
        t0 = time.time()
        while not self.rows and time.time() - t0 < 10.0 and self.proc.poll() is None:
            time.sleep(0.05)
        self.rows.clear()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.th:
            self.th.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def oracle_sample(q, k, v, exact_leaves, tiles, threads):
    """CPU oracle on a tile sample of one head: (per-head seconds, per-sample seconds, out rows, lse rows)."""
    from threadpoolctl import threadpool_limits

    from oracle import flat_oracle as O
    with threadpool_limits(limits=threads):
        t0 = time.perf_counter()
        prep = O.prepare_head(q, k, v)
        t1 = time.perf_counter()
        out, lse = O.attention_tiles(prep, tiles, exact_leaves=exact_leaves)
        t2 = time.perf_counter()
    return t1 - t0, t2 - t1, out, lse


# ------------------------------------------------------------------------------------------ reference arm
def run_reference(a, wl, rank):
    if rank != 0:
        return
    import numpy as np

    from htrc_b200 import synth
    threads = host_threads()
    q, k, v = synth.head_inputs(wl["grid"], 128, head=0)
    qn, kn, vn = q.float().numpy(), k.float().numpy(), v.float().numpy()
    n = qn.shape[0]
    nt = -(-n // 64)
    rng = np.random.default_rng(0)
    preps, times = [], []
    for step in range(a.warmup + a.steps):
        tiles = np.sort(rng.choice(nt, size=a.cpu_tiles, replace=False))
        dp, dt, _, _ = oracle_sample(qn, kn, vn, wl["exact_leaves"], tiles, threads)
        if step >= a.warmup:
            preps.append(dp)
            times.append(dt)
    per_tile = statistics.mean(times) / a.cpu_tiles
    ms_layer = (statistics.mean(preps) + per_tile * nt) * wl["heads"] * 1e3
    line = {"metric": METRIC, "impl": "reference", "value": ms_layer, "unit": "ms/layer", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_layer, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8+bf16 (restated in f32/f64 on CPU)",
            "data": "synthetic: seeded smooth-field Q/K, N(0,1) V (cfg generator), bf16",
            "config": {"workload": wl["name"], "tokens": n, "heads": wl["heads"], "dim": 128, "leaf": 64,
                       "tile": 64, "exact_leaves": wl["exact_leaves"]},
            "cpu_baseline": {"value": ms_layer, "unit": "ms/layer", "cores": threads, "kind": "port",
                             "sample": f"per step: the per-head preparation (bf16 K/V, key pack, tile centres) of "
                                       f"head 0 plus {a.cpu_tiles} random query tiles (of {nt}); layer = "
                                       f"{wl['heads']} x (prep + {nt} x per-tile), oracle/flat_oracle.py"},
            "e2e": {"value": ms_layer, "unit": "ms/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------ our arm
def run_ours(a, wl, rank, world, local_rank):
    import numpy as np
    import torch

    import htrc_b200
    from htrc_b200 import flat as F
    from htrc_b200 import shard, synth

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
    H = wl["heads"]
    try:
        my_heads = list(shard.heads_of_rank(H, rank, world))
    except ValueError as e:
        raise SystemExit(str(e))
    E = wl["exact_leaves"]

    # ---- inputs: pinned host copies (for e2e) and device-resident copies (for the device timing)
    host = {}
    for h in my_heads:
        q, k, v = synth.head_inputs(wl["grid"], 128, head=h)
        host[h] = tuple(t.pin_memory() for t in (q, k, v))
    n, m = host[my_heads[0]][0].shape[0], host[my_heads[0]][1].shape[0]
    nt, nb = -(-n // 64), m // 64
    kx = min(E, nb)
    dq = {h: tuple(t.to(dev, non_blocking=True) for t in host[h]) for h in my_heads}
    out = {h: torch.empty((n, 128), dtype=torch.float32, device=dev) for h in my_heads}
    lse = {h: torch.empty((n,), dtype=torch.float32, device=dev) for h in my_heads}
    from htrc_b200 import _lib as _L
    store = _L.STORES[a.store]
    fp8 = store == _L.STORE_FP8
    wsb = F.workspace_bytes(n, m, E, 0, 0, 0, store=store)
    ws = F.new_workspace(wsb, dev)
    comp = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)
    # heads alternate over `streams` streams with a workspace each: one head's small kernels and the last
    # partial wave of its tile kernel overlap the next head's work
    head_streams = [comp] + [torch.cuda.Stream(dev) for _ in range(a.streams - 1)]
    head_ws = [ws] + [F.new_workspace(wsb, dev) for _ in range(a.streams - 1)]
    gathered = None
    obf = None
    if world > 1:
        obf = {h: torch.empty((n, 128), dtype=torch.bfloat16, device=dev) for h in my_heads}
        gathered = [torch.empty((world, n, 128), dtype=torch.bfloat16, device=dev) for _ in my_heads]
    ev_done = [torch.cuda.Event() for _ in my_heads]
    nev = 6

    def layer(stage_events=None, gather=True, nstreams=None):
        streams = head_streams[:nstreams] if nstreams else head_streams
        for s_ in streams[1:]:
            s_.wait_stream(comp)
        for i, h in enumerate(my_heads):
            evs = stage_events[i] if stage_events is not None else None
            hs = streams[i % len(streams)]
            with torch.cuda.stream(hs):
                F.forward_into(*dq[h], None, None, exact_leaves=E, out=out[h], lse=lse[h],
                               workspace=head_ws[i % len(head_ws)], stage_events=evs, stream=hs, store=store)
                if world > 1 and gather:
                    obf[h].copy_(out[h])
                    ev_done[i].record(hs)
            if world > 1 and gather:
                side.wait_event(ev_done[i])
                with torch.cuda.stream(side):
                    shard.gather_slot(obf[h], out=gathered[i])
        for s_ in streams[1:]:
            comp.wait_stream(s_)
        if world > 1 and gather:
            comp.wait_stream(side)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    torch.cuda.synchronize(dev)
    for _ in range(a.warmup):
        layer()
    barrier()
    for w in head_ws:
        F.device_status(w)

    # ---- device-resident timed region, with per-stage events of every head
    stage_evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(nev)] for _ in my_heads] for _ in range(a.steps)]
    clocks = ClockSampler(dev.index if world == 1 else int(os.environ.get("LOCAL_RANK", 0)))
    clocks.start()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(comp)
    for s in range(a.steps):
        # with one head stream the stage events are taken here; with two they would include the overlap
        # of the two streams' kernels, so they come from a separate pass below
        layer(stage_evs[s] if a.streams == 1 else None)
    t1.record(comp)
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(t0.elapsed_time(t1) / a.steps)
    gather_info = None
    if world > 1:
        # the same layer without the output gathers: the gathers' exposed (not overlapped) time
        barrier()
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        g0.record(comp)
        for _ in range(a.steps):
            layer(gather=False)
        g1.record(comp)
        barrier()
        ms_nog = max_over_ranks(g0.elapsed_time(g1) / a.steps)
        gather_info = {"compute_only_ms": ms_nog, "exposed_ms": ms - ms_nog,
                       "bytes_per_rank_per_step": len(my_heads) * world * n * 128 * 2,
                       "how": "bf16 outputs all-gathered (NCCL) per local head on a side stream, overlapped with the "
                              "next head; exposed = layer time - the same layer without the gathers"}
    stage_timing = "CUDA events around each stage of every head in the timed region (heads on one stream)"
    if a.streams > 1:
        barrier()
        for s in range(a.steps):
            layer(stage_evs[s], gather=False, nstreams=1)
        barrier()
        stage_timing = ("CUDA events around each stage of every head in a separate pass of the same layers with the "
                        "heads on one stream (the timed region's two streams overlap consecutive heads)")
    for w in head_ws:
        F.device_status(w)
    stage_names = ["prep", "stats", "rowmax", "route", "tile"]
    stage_ms = {nm: statistics.mean(stage_evs[s][i][j].elapsed_time(stage_evs[s][i][j + 1])
                                    for s in range(a.steps) for i in range(len(my_heads)))
                for j, nm in enumerate(stage_names)}

    # ---- parity at full size on a tile sample of head 0 (rank 0): mean |dlogZ| vs the oracle
    parity = {}
    cpu = None
    if rank == 0 and not a.no_cpu and not fp8:
        h0 = my_heads[0]
        qn, kn, vn = (t.float().numpy() for t in host[h0])
        rng = np.random.default_rng(1)
        tiles = np.sort(rng.choice(nt, size=a.cpu_tiles, replace=False))
        threads = host_threads()
        dp, dt, ro, rl = oracle_sample(qn, kn, vn, E, tiles, threads)
        rows = (tiles[:, None] * 64 + np.arange(64)[None, :]).reshape(-1)
        valid = rows < n
        lse_d = lse[h0].cpu().numpy()[rows[valid]]
        out_d = out[h0].cpu().numpy()[rows[valid]]
        parity = {"logz_mae": float(np.abs(lse_d - rl[valid]).mean()),
                  "out_maxabs": float(np.abs(out_d - ro[valid]).max()),
                  "sample": f"{len(tiles)} random tiles of head {h0} vs oracle/flat_oracle.py"}
        # error of the operator against exact softmax attention on the same rows
        qs = dq[h0][0][torch.as_tensor(rows[valid], device=dev)].float()
        kk, vv = dq[h0][1].float(), dq[h0][2].float()
        s_ = (qs @ kk.T) / math.sqrt(128)
        ex = torch.softmax(s_, -1) @ vv
        od = out[h0][torch.as_tensor(rows[valid], device=dev)]
        parity["rel_l2_vs_exact"] = float((od - ex).norm() / ex.norm())
        del s_
        if world == 1:
            per_tile = dt / len(tiles)
            cpu_ms = (dp + per_tile * nt) * H * 1e3
            cpu = {"value": cpu_ms, "unit": "ms/layer", "cores": threads, "kind": "port",
                   "sample": f"head {h0}: per-head preparation + {len(tiles)} query tiles ({len(tiles) * 64} rows of "
                             f"{n}) through oracle/flat_oracle.py; layer = {H} x (prep + {nt} x per-tile)"}

    # ---- end to end through the public API with pinned host buffers
    e2e = None
    if not a.no_e2e:
        qb = [torch.empty_like(dq[my_heads[0]][j]) for j in range(3) for _ in range(2)]
        stage_in = [(qb[0], qb[2], qb[4]), (qb[1], qb[3], qb[5])]
        stage_out = [(torch.empty((n, 128), dtype=torch.float32, device=dev),
                      torch.empty((n,), dtype=torch.float32, device=dev)) for _ in range(2)]
        host_out = {h: (torch.empty((n, 128), dtype=torch.float32).pin_memory(),
                        torch.empty((n,), dtype=torch.float32).pin_memory()) for h in my_heads}
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        in_done = [torch.cuda.Event() for _ in range(2)]
        comp_done = [torch.cuda.Event() for _ in range(2)]
        out_done = [torch.cuda.Event() for _ in range(2)]

        def e2e_layer():
            for s_ in head_streams[1:]:
                s_.wait_stream(comp)
            for i, h in enumerate(my_heads):
                b = i % 2
                hs = head_streams[i % len(head_streams)]
                # staging buffer b is free once the head that last used it (two heads back, in this layer or
                # the previous one) finished computing; an event not recorded yet is a no-op
                s_in.wait_event(comp_done[b])
                with torch.cuda.stream(s_in):
                    for dst, src in zip(stage_in[b], host[h]):
                        dst.copy_(src, non_blocking=True)
                    in_done[b].record(s_in)
                hs.wait_event(in_done[b])
                # staging output b is free once the copy-out of the head that last wrote it (two heads back,
                # in this layer or the previous one) finished; an event not recorded yet is a no-op
                hs.wait_event(out_done[b])
                with torch.cuda.stream(hs):
                    htrc_b200.forward_into(*stage_in[b], None, None, exact_leaves=E, store=store, out=stage_out[b][0],
                                           lse=stage_out[b][1], workspace=head_ws[i % len(head_ws)], stream=hs)
                comp_done[b].record(hs)
                s_out.wait_event(comp_done[b])
                with torch.cuda.stream(s_out):
                    host_out[h][0].copy_(stage_out[b][0], non_blocking=True)
                    host_out[h][1].copy_(stage_out[b][1], non_blocking=True)
                    out_done[b].record(s_out)
            for s_ in head_streams[1:]:
                comp.wait_stream(s_)

        def join_copies():
            # the copy streams run across layer boundaries (layer L's last copies-out overlap layer L + 1's
            # compute); the timed region ends only after every copy of every timed layer
            comp.wait_stream(s_in)
            comp.wait_stream(s_out)

        for _ in range(a.warmup):
            e2e_layer()
        join_copies()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        for _ in range(a.steps):
            e2e_layer()
        join_copies()
        e1.record(comp)
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
        h2d = sum(sum(t.numel() * t.element_size() for t in host[h]) for h in my_heads) * world
        d2h = sum(sum(t.numel() * t.element_size() for t in host_out[h]) for h in my_heads) * world
        same = all(bool(torch.equal(host_out[h][0].to(dev), out[h])) for h in (my_heads[0], my_heads[-1]))
        e2e = {"value": e2e_ms, "unit": "ms/layer", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "htrc_b200.forward_into, pinned host q/k/v in and out/lse back, copies overlapped on "
                      f"2 copy streams (also across layers), heads on {a.streams} compute stream(s)",
               "matches_device_run": same}

    # ---- the reference runner's modes on head 0 (rank 0, one GPU): ms per head through FlatRunner's
    # CUDA graph (static-buffer copies included), and the k-means ordering alone
    modes = None
    if rank == 0 and world == 1 and not a.no_modes:
        from htrc_b200 import runner as R
        h0 = my_heads[0]
        modes = {}
        for mode in list(R.MODES) + ["fast+iso", "fast+fp8"]:
            extra = {"fast+iso": dict(backend="cuda", curvature="iso"), "fast+fp8": dict(store="fp8")}.get(mode, {})
            r = R.FlatRunner(n, m, mode=mode.split("+")[0], device=dev, **extra)
            if r.graph is None:
                modes[mode] = f"graph capture failed: {r.graph_error}"
                continue
            for _ in range(2):
                r.head(*dq[h0])
            torch.cuda.synchronize(dev)
            m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            m0.record(comp)
            for _ in range(3):
                r.head(*dq[h0])
            m1.record(comp)
            torch.cuda.synchronize(dev)
            r.check_status()
            modes[mode] = m0.elapsed_time(m1) / 3
            r.close()
            del r
        import ctypes

        from htrc_b200 import _lib
        kb = ctypes.c_size_t()
        _lib.check(_lib.lib().htrc_kmeans_scratch_size(n, kb), "kmeans scratch")
        kscr = torch.empty(int(kb.value), dtype=torch.uint8, device=dev)
        perm = torch.empty((n,), dtype=torch.int32, device=dev)

        def km():
            _lib.check(_lib.lib().htrc_kmeans_order(_lib.ptr(dq[h0][0]), _lib.DTYPE_BF16, n, 128, _lib.ptr(perm),
                                                    _lib.ptr(kscr), int(kb.value), _lib.stream_ptr()), "kmeans")
        km()
        torch.cuda.synchronize(dev)
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record(comp)
        for _ in range(5):
            km()
        k1.record(comp)
        torch.cuda.synchronize(dev)
        modes = {"ms_per_head": modes, "kmeans_order_ms": k0.elapsed_time(k1) / 5,
                 "note": "head 0 of the workload through FlatRunner (CUDA graph) per mode of "
                         "h3/htrc_flat_runner.py:48-53: fast E=256, balanced E=512, accurate E=1024 + k-means, "
                         "max E=1024 + k-means + 32-row tiles; fast+iso: fast with the isotropic curvature term; "
                         "fast+fp8: fast with the e4m3 far-field state (store='fp8')"}

    # ---- roofline of the dominant kernel (tile attention) from the live events
    peaks, peak_src = measured_peaks()
    npad = nt * 64
    near = 2.0 * npad * (kx * 64) * 128
    far = 2.0 * npad * (nb - kx) * 128 if kx < nb else 0.0
    # INT8: bf16 PV + int8 QK at half cost; fp8: fp16 / bf16 QK and PV at full cost
    flops_bf16_equiv = 2.0 * (near + far) if fp8 else (near + far) + 0.5 * (near + far)
    tile_ms = stage_ms["tile"]
    achieved = flops_bf16_equiv / (tile_ms * 1e-3) / 1e12
    peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    traffic = None
    tp = ROOT / "profiles" / "tile_attention_traffic.json"
    if tp.exists() and not fp8:
        traffic = json.loads(tp.read_text()).get("bytes_per_launch", {}).get(a.workload)
    roof = {"kernel": "tile_fp8_kernel (far + near passes)" if fp8 else "tile_attention_kernel", "bound": "tensor",
            "achieved": achieved, "peak": peak,
            "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
            "peak_source": f"{peak_src} bf16_tflops_sustained", "flop_per_launch": flops_bf16_equiv,
            "flop_count": ("fp16/bf16 QK + PV flops" if fp8 else "bf16 PV flops + int8 QK ops/2") +
                          " over the routed tokens and non-routed leaves, one head",
            "ms_per_launch": tile_ms}

    # ---- every stage against its binding roofline (algorithmic bytes or flop per head / stage time)
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    pitch = -(-nb // 16) * 16
    stage_bytes = {
        "prep": m * (2 * 128 + 128 + 4) + n * 2 * 128 + npad * (2 * 128 + 8),   # k pack + q codes (bf16 q)
        "stats": nt * nb * (128 + 256) + 2 * nt * pitch * 4,                    # g8 + vbar + sg/lz written
        "rowmax": nt * nb * 128 + 2 * nt * pitch * 4 + nt * pitch * 4,          # g8 + sg/lz read, sel written
        "route": nt * pitch * 4 + nt * (pitch + kx * 4),                        # sel read, excl/idx written
    }
    if fp8:
        stage_bytes["prep"] = n * 2 * 128 + npad * 2 * 2 * 128                  # bf16 q read; bf16 + fp16 rows
        stage_bytes["stats"] = nt * nb * (128 + 128) + 3 * nt * pitch * 4       # g + vbar codes, sg/sv/lz
    stage_roof = {nm: {"bound": "hbm", "bytes": b_, "achieved_gbs": b_ / (stage_ms[nm] * 1e-3) / 1e9,
                       "frac": b_ / (stage_ms[nm] * 1e-3) / 1e9 / hbm}
                  for nm, b_ in stage_bytes.items()}
    stage_roof["stats"]["tensor_frac"] = (6.0 * nt * m * 128 / (stage_ms["stats"] * 1e-3) / 1e12) / peak
    stage_roof["tile"] = {"bound": "tensor", "frac": roof["frac"]}

    if rank == 0:
        line = {"metric": METRIC, "value": ms, "unit": "ms/layer", "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": False, "scaling": "strong",
                "vs_baseline": None,
                "dtype": ("fp8 (e4m3) state; fp16 far / bf16 near QK and PV, f32 softmax" if fp8 else
                          "int8 QK + bf16 PV, f32 softmax"),
                "data": "synthetic: seeded smooth-field Q/K (4x8x8 grid trilinear + 0.5 noise, RMS 3), N(0,1) V, bf16",
                "config": {"workload": wl["name"].replace("INT8", "fp8 (e4m3) state") if fp8 else wl["name"],
                           "tokens": n, "heads": H,
                           "dim": 128, "leaf": 64, "tile": 64, "store": a.store,
                           "exact_leaves": E, "heads_per_gpu": len(my_heads), "head_streams": a.streams,
                           "l2": "inputs larger than L2: 2.4 GB of distinct q/k/v per layer, "
                                 + ("1.0" if fp8 else "1.6") + " GB leaf state per head",
                           "parallelism": f"heads/{world}" + (" + bf16 output all_gather (NCCL)" if world > 1 else "")},
                "stage_ms_per_head": stage_ms, "stage_timing": stage_timing, "stage_roofline": stage_roof,
                "gather": gather_info, "modes": modes,
                **parity,
                "roofline": roof, "cpu_baseline": cpu,
                "e2e": e2e,
                "gpu_launches": a.steps * len(my_heads) * LAUNCHES_PER_HEAD, "clocks": clk}
        print(json.dumps(line), flush=True)


def main():
    a = parse()
    wl = WORKLOADS[a.workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        run_reference(a, wl, rank)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(a, wl, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
