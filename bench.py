#!/usr/bin/env python
"""Benchmark of the flat HTRC operator on B200: milliseconds per attention layer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg3|cfg2|cfg4|cfg5]

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

--workload cfg5 times the hierarchical operator (htrc_b200.tree, the NumPy law of src/htrc_reference/model.py on the
GPU) on the 243-frame configuration instead; its cpu_baseline times the float64 tree oracle on a sample, and its
reference arm the reference's own NumPy model (build_forest + evaluate) on a sample, both extrapolated.

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
    # the denoise-step workload: a step is one transformer block = CFG batch 2 x 24 heads (48 (batch, head)
    # pairs), fresh seeded inputs per block (two distinct blocks resident, alternated); value = block time / 2
    "cfg4": dict(grid=(32, 48, 84), heads=24, batch=2, blocks=2, exact_leaves=256,
                 name="cfg4: per step one denoise-step block: CFG batch 2 x 24 heads of 129,024 tokens (48 (batch, "
                      "head) pairs, fresh seeded Q/K/V per block, 2 distinct blocks resident and alternated), d128, "
                      "leaf 64, tile 64, fast (E=256), INT8; value = ms per 24-head layer = block time / 2"),
    # the hierarchical operator (htrc_b200.tree): a step is one 24-head layer at 243 frames; heads split over ranks
    "cfg5": dict(grid=(61, 48, 84), heads=24, tree=True, leaf=64, fanout=16, threshold=0.02,
                 name="cfg5: hierarchical HTRC, 245,952-token 61x48x84 latent layer, 24 heads, d128, leaf 64, fanout "
                      "16, threshold 0.02, 32 k-means query centres, second-order log-mass + value dipole"),
    # profiling-sized hierarchical case: one 64,512-token head (forest 0.3 GB, records ~1.7 GB)
    "tree_prof": dict(grid=(16, 48, 84), heads=1, tree=True, leaf=64, fanout=16, threshold=0.02,
                      name="tree_prof: hierarchical HTRC, one 64,512-token 16x48x84 head, d128, leaf 64, fanout 16, "
                           "threshold 0.02, 32 k-means query centres"),
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
    ap.add_argument("--workload", default="auto", choices=["auto"] + list(WORKLOADS),
                    help="auto (default): cfg3 (one full-resolution layer) on one GPU, cfg4 (one CFG-batch block "
                         "of the denoise step, pairs sharded over the ranks) under torchrun")
    ap.add_argument("--cpu-tiles", type=int, default=4, help="tiles of the CPU-baseline sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-modes", action="store_true", help="skip the per-mode head timings")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="skip timing the reference's own Triton operator on this GPU (installed under baseline/_ref)")
    ap.add_argument("--ref-steps", type=int, default=3, help="layers timed for the reference's GPU operator")
    ap.add_argument("--no-ref-cpu", action="store_true",
                    help="skip timing the reference's own CPU implementations (torch backend, NumPy model)")
    ap.add_argument("--store", default="int8", choices=["int8", "fp8", "bf16"],
                    help="far-field state: int8 (the production path, the headline), fp8 (e4m3 state, store='fp8') "
                         "or bf16 (store='bf16'); the last two without the oracle sample")
    ap.add_argument("--precision", default="tf32", choices=["tf32", "fp32"],
                    help="leaf-statistics dots: tf32 operands (PROD's setting, the reference's production path; the "
                         "default) or float32-accurate")
    ap.add_argument("--division", default="ieee", choices=["ieee", "triton"],
                    help="division forming the query/offset/slope codes in the timed layers: IEEE (the reference's "
                         "formula as written, the library's default) or the reference's GPU division (div.full.f32); "
                         "the comparison with the reference's own operator uses a Triton-division run of head 0, the "
                         "comparison with the oracle an IEEE one")
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


def oracle_sample(q, k, v, exact_leaves, tiles, threads, precision="fp32"):
    """CPU oracle on a tile sample of one head: (per-head seconds, per-sample seconds, out rows, lse rows,
    the prepared head)."""
    from threadpoolctl import threadpool_limits

    from oracle import flat_oracle as O
    with threadpool_limits(limits=threads):
        t0 = time.perf_counter()
        prep = O.prepare_head(q, k, v)
        t1 = time.perf_counter()
        out, lse = O.attention_tiles(prep, tiles, exact_leaves=exact_leaves, precision=precision)
        t2 = time.perf_counter()
    return t1 - t0, t2 - t1, out, lse, prep


def oracle_routing(prep, tiles, exact_leaves, threads, precision="fp32"):
    """The oracle's routing masks (bool [len(tiles), nb]) of sampled tiles: its own float64 leaf statistics,
    INT8 state, row-max selection and top-E (parity check; not timed)."""
    from threadpoolctl import threadpool_limits

    from oracle import flat_oracle as O
    with threadpool_limits(limits=threads):
        mu, qt = prep["mu"][tiles], prep["qt"][tiles]
        g, lz, vbf = O.leaf_stats(mu, prep["k"], prep["v"], prep["leaf"], 1.0 / math.sqrt(prep["k"].shape[1]),
                                  precision)
        g8, sg, _ = O.state_int8(g, vbf)
        _, _, dq8, sdq = O.query_codes(qt, mu)
        _, excl = O.route(O.rowmax_select(dq8, sdq, g8, sg, lz), exact_leaves)
    return excl != 0


def full_size_codes(F, head, prep, exact_leaves, threads):
    """Bit-exactness of the INT8 codes at the full size of one head (parity check; not timed): key codes and
    scales (k8, ks), tile centres, query and offset codes and scales (q8, sq, dq8, sdq) of every row, from
    the device's stage-by-stage run against the oracle."""
    import numpy as np
    from threadpoolctl import threadpool_limits

    from oracle import flat_oracle as O
    st = F.run_stages(*head, exact_leaves=exact_leaves)
    with threadpool_limits(limits=threads):
        q8, sq, dq8, sdq = O.query_codes(prep["qt"], prep["mu"])
    nt = prep["qt"].shape[0]
    dev = {k_: st[k_].cpu().numpy() for k_ in ("k8", "ks", "mu", "q8", "sq", "dq8", "sdq")}
    res = {"k8": bool(np.array_equal(dev["k8"], prep["k8"])), "ks": bool(np.array_equal(dev["ks"], prep["ks"])),
           "mu": bool(np.array_equal(dev["mu"], prep["mu"])),
           "q8": bool(np.array_equal(dev["q8"].reshape(nt, 64, -1), q8)),
           "sq": bool(np.array_equal(dev["sq"].reshape(nt, 64), sq)),
           "dq8": bool(np.array_equal(dev["dq8"].reshape(nt, 64, -1), dq8)),
           "sdq": bool(np.array_equal(dev["sdq"].reshape(nt, 64), sdq)),
           "rows": prep["n"], "keys": int(prep["k8"].shape[0])}
    del st
    return res


# ------------------------------------------------------------------------------------------ installed reference
def load_installed_reference():
    """The unmodified reference, installed under baseline/_ref by baseline/install_ref.sh (or the directory
    $HTRC_REFERENCE names): h3/htrc_flat.py with its Triton kernels (h3/htrc_flat_triton.py),
    h3/htrc_flat_runner.py and the NumPy package htrc_reference.  Returns {"flat", "runner", "model", "root"};
    raises when it is absent."""
    import importlib.util
    roots = [os.environ.get("HTRC_REFERENCE"), str(ROOT / "baseline" / "_ref")]
    root = next((Path(r) for r in roots if r and (Path(r) / "h3" / "htrc_flat.py").exists()), None)
    if root is None:
        raise FileNotFoundError("reference not installed: no h3/htrc_flat.py under baseline/_ref or $HTRC_REFERENCE")

    def load(name, path):
        if name not in sys.modules:
            spec = importlib.util.spec_from_file_location(name, path)
            mod = importlib.util.module_from_spec(spec)
            sys.modules[name] = mod
            spec.loader.exec_module(mod)
        return sys.modules[name]

    # the runner loads htrc_flat.py under this module name (h3/htrc_flat_runner.py:38-45, :90): one copy
    flat = load("_apl_htrc_flat", root / "h3" / "htrc_flat.py")
    runner = load("_ref_htrc_flat_runner", root / "h3" / "htrc_flat_runner.py")
    model = None
    for cand in (root, root / "src"):
        if (cand / "htrc_reference" / "model.py").exists():
            model = load("_ref_htrc_reference_model", cand / "htrc_reference" / "model.py")
            break
    return {"flat": flat, "runner": runner, "model": model, "root": str(root)}


def reference_gpu_leg(wl, dev, heads, dq, ours, steps, oracle_rows=None):
    """The reference's own flat operator on this GPU, on the same inputs: ``flat_attention(**PROD, leaf=64)``
    (h3/htrc_flat.py:391-399 -> _flat_triton :181-276, Triton kernels h3/htrc_flat_triton.py) eager with a
    reused workspace dict, and through its CUDA-graph ``FlatRunner(mode="fast", leaf=64)``
    (h3/htrc_flat_runner.py:85-177) with the chunk planned from free memory.  Head 0 once more in one chunk
    (``tile_chunk >= tiles``) to read its routing mask ``ws["excl"]`` and split partials ``ws["pm"]``/``ws["pl"]``
    (log-Z = logsumexp over the splits of pm + log pl), compared with this library's outputs ``ours``
    ({"out", "lse", "mask"} of head 0) and, on ``oracle_rows`` = (rows, oracle out, oracle lse), with the CPU
    oracle: how far each GPU operator sits from the float64 restatement on the same rows."""
    import torch
    try:
        ref = load_installed_reference()
        import triton  # noqa: F401
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    flat, runner = ref["flat"], ref["runner"]
    comp = torch.cuda.current_stream(dev)
    cfg = {**flat.PROD, **runner.MODES["fast"], "leaf": 64, "exact_leaves": wl["exact_leaves"]}
    res = {"impl": "h3/htrc_flat.py flat_attention(**PROD, **MODES['fast'], leaf=64), Triton backend, unmodified, "
                   "from " + ("baseline/_ref" if "baseline" in ref["root"] else "$HTRC_REFERENCE"),
           "config": {k: (v if not isinstance(v, dict) else dict(v)) for k, v in cfg.items()}}
    n, m = int(dq[heads[0]][0].shape[0]), int(dq[heads[0]][1].shape[0])
    nt, nb = -(-n // 64), m // 64
    t_c = time.time()
    try:
        ws = {}
        for h in heads:                                     # warm-up layer: compiles the Triton kernels
            flat.flat_attention(*dq[h], ws=ws, **cfg)
        torch.cuda.synchronize(dev)
        res["compile_and_first_layer_s"] = time.time() - t_c

        def timed(fn, k):
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(comp)
            for _ in range(k):
                fn()
            e1.record(comp)
            torch.cuda.synchronize(dev)
            return e0.elapsed_time(e1) / k

        clocks = ClockSampler(dev.index)
        clocks.start()
        res["eager_ms_per_layer"] = timed(lambda: [flat.flat_attention(*dq[h], ws=ws, **cfg) for h in heads], steps)
        res["eager_clocks"] = clocks.stop()
        del ws
        torch.cuda.empty_cache()
        free = torch.cuda.mem_get_info(dev)[0]
        r = runner.FlatRunner(n, m, free_bytes=free, mode="fast", leaf=64, device=dev)
        res["runner"] = {"tile_chunk": r.cfg["tile_chunk"], "graph": r.graph is not None, "graph_error": r.graph_error}
        for h in heads[:2]:
            r.head(*dq[h])
        clocks = ClockSampler(dev.index)
        clocks.start()
        res["runner_ms_per_layer"] = timed(lambda: [r.head(*dq[h]) for h in heads], steps)
        res["runner_clocks"] = clocks.stop()
        r.close()
        del r
        torch.cuda.empty_cache()
        res["ms_per_layer"] = min(res["eager_ms_per_layer"], res["runner_ms_per_layer"])
        res["heads_timed"] = len(heads)
        res["steps"] = steps
        # head 0 in one chunk: routing mask and log-Z of the reference against ours
        ws0 = {}
        out_r = flat.flat_attention(*dq[heads[0]], ws=ws0, **{**cfg, "tile_chunk": nt}).float()
        excl_r = ws0["excl"][:nt].ne(0)
        pm, pl = ws0["pm"][:nt].float(), ws0["pl"][:nt].float()
        mm = pm.amax(1, keepdim=True)
        mm = torch.where(torch.isinf(mm), torch.zeros_like(mm), mm)
        lse_r = (mm[:, 0] + torch.log((pl * torch.exp(pm - mm)).sum(1))).reshape(-1)[:n]
        mask = ours["mask"][:nt, :nb].ne(0)
        tiles_agree = (mask == excl_r).all(1)
        rows_agree = tiles_agree.repeat_interleave(64)[:n]
        d_out = (ours["out"] - out_r).abs().amax(1)
        d_lse = (ours["lse"] - lse_r).abs()
        p = {"routing_agreement": (mask == excl_r).float().mean().item(),
             "tiles_all_agree": tiles_agree.float().mean().item(),
             "out_maxabs_all_rows": d_out.max().item(),
             "out_maxabs_agreeing_tiles": d_out[rows_agree].max().item() if bool(rows_agree.any()) else None,
             "rows_over_2e-2": int((d_out > 2e-2).sum().item()),
             "lse_mae": d_lse.mean().item(), "lse_maxabs": d_lse.max().item(),
             "precision": cfg["precision"], "division": ours["division"],
             "how": "this library's route_mask / out / lse of head 0 (the same precision setting) against the "
                    "reference's ws['excl'], output and logsumexp of its split partials ws['pm'], ws['pl'] (one "
                    "chunk), same inputs, same B200"}
        if oracle_rows is not None:
            rows, o_out, o_lse = oracle_rows
            ri = torch.as_tensor(rows, device=dev)
            oo, ol = torch.as_tensor(o_out, device=dev), torch.as_tensor(o_lse, device=dev)
            p["vs_oracle_sample"] = {
                "rows": int(len(rows)),
                "ref_out_maxabs": (out_r[ri] - oo).abs().max().item(), "ref_lse_mae": (lse_r[ri] - ol).abs().mean().item(),
                "ours_out_maxabs": (ours["out_ieee"][ri] - oo).abs().max().item(),
                "ours_lse_mae": (ours["lse_ieee"][ri] - ol).abs().mean().item(),
                "how": "both GPU operators against the CPU oracle (the float64 restatement at the same precision "
                       "setting, IEEE division) on its sampled tiles; this library's row from its IEEE-division "
                       "run"}
        g = torch.Generator().manual_seed(5)
        rows = torch.randperm(n, generator=g)[:256].to(dev)
        qs = dq[heads[0]][0][rows].float()
        s_ = (qs @ dq[heads[0]][1].float().T) / math.sqrt(128)
        ex = torch.softmax(s_, -1) @ dq[heads[0]][2].float()
        p["rel_l2_vs_exact_ref"] = float((out_r[rows] - ex).norm() / ex.norm())
        p["rel_l2_vs_exact_ours"] = float((ours["out"][rows] - ex).norm() / ex.norm())
        res["parity_head0"] = p
        del ws0, out_r, s_
        torch.cuda.empty_cache()
    except Exception as e:  # noqa: BLE001
        res["error"] = f"{type(e).__name__}: {e}"[:400]
    return res


def reference_cpu_legs(threads, budget_tiles=64, budget_s=20.0):
    """The reference's own CPU implementations, timed on this host with ``threads`` threads: its float32 torch
    backend ``flat_attention(backend="torch")`` (h3/htrc_flat.py:279-388) on configuration 1 (one head,
    N = M = 4096, d 64), on the 24 configuration-2 heads (as many as fit in ``budget_s``, the rest
    extrapolated) and on a ``budget_tiles``-tile sample of one configuration-3 head (x tiles x 24:
    extrapolated); and the NumPy hierarchical model ``build_forest`` + ``evaluate``
    (src/htrc_reference/model.py:68-137) on all 4096 configuration-1 queries (leaf 64, opening threshold
    0.02, one expansion centre: the mean query)."""
    import numpy as np
    import torch

    from htrc_b200 import synth
    try:
        ref = load_installed_reference()
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    flat, model = ref["flat"], ref["model"]
    old = torch.get_num_threads()
    torch.set_num_threads(threads)
    res = {"kind": "reference-torch", "cores": threads}
    try:
        q1, k1, v1 = synth.cluster_inputs(4096, 64, seed=0)
        tq, tk, tv = (torch.from_numpy(x) for x in (q1, k1, v1))
        kw = dict(backend="torch", tile=64, leaf=64, exact_leaves=16, tile_chunk=32, precision="fp32")
        flat.flat_attention(tq, tk, tv, **kw)
        t0 = time.perf_counter()
        for _ in range(3):
            flat.flat_attention(tq, tk, tv, **kw)
        res["cfg1_torch_flat_ms_per_head"] = (time.perf_counter() - t0) / 3 * 1e3
        res["cfg1_torch_flat_config"] = "N = M = 4096, d 64, leaf 64, tile 64, exact_leaves 16, fp32"
        if model is not None:
            scale = 1.0 / math.sqrt(64)
            qd, kd, vd = q1.astype(np.float64), k1.astype(np.float64), v1.astype(np.float64)
            centre = qd.mean(0) * scale
            t0 = time.perf_counter()
            forest = model.build_forest(kd, vd, centre, leaf_size=64)
            t1 = time.perf_counter()
            for i in range(qd.shape[0]):
                model.evaluate(kd, vd, qd[i] * scale, centre, forest, opening_threshold=0.02)
            t2 = time.perf_counter()
            res["cfg1_numpy_hierarchical"] = {"build_forest_ms": (t1 - t0) * 1e3, "evaluate_s_all_queries": t2 - t1,
                                              "queries": int(qd.shape[0]), "threads": 1,
                                              "note": "single-threaded Python/NumPy; one expansion centre (the mean "
                                                      "query; the model takes one centre)"}
        kw = dict(backend="torch", tile=64, leaf=64, exact_leaves=256, tile_chunk=32, precision="fp32")
        t_all, done = 0.0, 0
        for h in range(24):
            q, k, v = synth.head_inputs(synth.GRID_SMALL, 128, head=h)
            t0 = time.perf_counter()
            flat.flat_attention(q.float(), k.float(), v.float(), **kw)
            t_all += time.perf_counter() - t0
            done += 1
            if t_all > budget_s:
                break
        res["cfg2_torch_flat"] = {"ms_per_layer": t_all / done * 24 * 1e3, "heads_timed": done,
                                  "extrapolated": done < 24, "timed_s": t_all,
                                  "sample": f"{done} whole heads of 16,384 tokens" + (f", x24/{done}" if done < 24 else "")}
        q, k, v = synth.head_inputs(synth.GRID_FULL, 128, head=0)
        n = q.shape[0]
        nt = -(-n // 64)
        t0 = time.perf_counter()
        flat.flat_attention(q[:budget_tiles * 64].float(), k.float(), v.float(), **kw)
        dt = time.perf_counter() - t0
        res["cfg3_torch_flat"] = {"ms_per_layer": dt / budget_tiles * nt * 24 * 1e3, "extrapolated": True,
                                  "timed_s": dt, "sample": f"{budget_tiles} of {nt} query tiles of head 0, "
                                                          f"x{nt}/{budget_tiles} x24"}
    except Exception as e:  # noqa: BLE001
        res["error"] = f"{type(e).__name__}: {e}"[:300]
    finally:
        torch.set_num_threads(old)
    return res


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
        dp, dt, _, _, _ = oracle_sample(qn, kn, vn, wl["exact_leaves"], tiles, threads)
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
    batch, nblocks = wl.get("batch", 1), wl.get("blocks", 1)
    layers_per_step = batch                     # a step is `batch` layers of H heads
    try:
        my_pairs = list(shard.heads_of_rank(H * batch, rank, world))   # (batch, head) pair p = batch * H + head
    except ValueError as e:
        raise SystemExit(str(e))
    E = wl["exact_leaves"]
    # the jobs of step s: block s % nblocks, this rank's pairs, keyed (block, batch, head); slot i = i-th pair
    step_jobs = [[(b, p // H, p % H) for p in my_pairs] for b in range(nblocks)]
    all_jobs = [j for js in step_jobs for j in js]
    nslots = len(my_pairs)

    # ---- inputs: pinned host copies (for e2e) and device-resident copies (for the device timing)
    host = {}
    for j in all_jobs:
        q, k, v = synth.head_inputs(wl["grid"], 128, block=j[0], batch=j[1], head=j[2])
        host[j] = tuple(t.pin_memory() for t in (q, k, v))
    n, m = host[all_jobs[0]][0].shape[0], host[all_jobs[0]][1].shape[0]
    nt, nb = -(-n // 64), m // 64
    kx = min(E, nb)
    dq = {j: tuple(t.to(dev, non_blocking=True) for t in host[j]) for j in all_jobs}
    out = [torch.empty((n, 128), dtype=torch.float32, device=dev) for _ in range(nslots)]
    lse = [torch.empty((n,), dtype=torch.float32, device=dev) for _ in range(nslots)]
    from htrc_b200 import _lib as _L
    store = _L.STORES[a.store]
    fp8 = store != _L.STORE_INT8           # the operand-form state paths (fp8 or bf16)
    bf16_state = store == _L.STORE_BF16
    prec = F.precision_code(a.precision, a.division)
    prec_ieee = F.precision_code(a.precision, "ieee")
    prec_ref = F.precision_code(a.precision, "triton")
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
        obf = [torch.empty((n, 128), dtype=torch.bfloat16, device=dev) for _ in range(nslots)]
        gathered = [torch.empty((world, n, 128), dtype=torch.bfloat16, device=dev) for _ in range(nslots)]
    ev_done = [torch.cuda.Event() for _ in range(nslots)]
    nev = 6

    def layer(step, stage_events=None, gather=True, nstreams=None):
        streams = head_streams[:nstreams] if nstreams else head_streams
        for s_ in streams[1:]:
            s_.wait_stream(comp)
        for i, h in enumerate(step_jobs[step % nblocks]):
            evs = stage_events[i] if stage_events is not None else None
            hs = streams[i % len(streams)]
            with torch.cuda.stream(hs):
                F.forward_into(*dq[h], None, None, exact_leaves=E, out=out[i], lse=lse[i],
                               workspace=head_ws[i % len(head_ws)], stage_events=evs, stream=hs, store=store,
                               precision=prec)
                if world > 1 and gather:
                    obf[i].copy_(out[i])
                    ev_done[i].record(hs)
            if world > 1 and gather:
                side.wait_event(ev_done[i])
                with torch.cuda.stream(side):
                    shard.gather_slot(obf[i], out=gathered[i])
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
    for s in range(a.warmup):
        layer(s)
    barrier()
    for w in head_ws:
        F.device_status(w)

    # ---- device-resident timed region, with per-stage events of every head
    stage_evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(nev)] for _ in range(nslots)]
                 for _ in range(a.steps)]
    clocks = ClockSampler(dev.index if world == 1 else int(os.environ.get("LOCAL_RANK", 0)))
    clocks.start()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(comp)
    for s in range(a.steps):
        # with one head stream the stage events are taken here; with two they would include the overlap
        # of the two streams' kernels, so they come from a separate pass below
        layer(s, stage_evs[s] if a.streams == 1 else None)
    t1.record(comp)
    barrier()
    clk = clocks.stop()
    ms_step = max_over_ranks(t0.elapsed_time(t1) / a.steps)
    ms = ms_step / layers_per_step
    gather_info = None
    if world > 1:
        # the same layer without the output gathers: the gathers' exposed (not overlapped) time
        barrier()
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        g0.record(comp)
        for s in range(a.steps):
            layer(s, gather=False)
        g1.record(comp)
        barrier()
        ms_nog = max_over_ranks(g0.elapsed_time(g1) / a.steps)
        gather_info = {"compute_only_ms_per_step": ms_nog, "exposed_ms_per_step": ms_step - ms_nog,
                       "exposed_ms_per_layer": (ms_step - ms_nog) / layers_per_step,
                       "bytes_per_rank_per_step": nslots * world * n * 128 * 2,
                       "how": "bf16 outputs all-gathered (NCCL) per local head on a side stream, overlapped with the "
                              "next head; exposed = layer time - the same layer without the gathers"}
    stage_timing = "CUDA events around each stage of every head in the timed region (heads on one stream)"
    if a.streams > 1:
        barrier()
        for s in range(a.steps):
            layer(s, stage_evs[s], gather=False, nstreams=1)
        barrier()
        stage_timing = ("CUDA events around each stage of every head in a separate pass of the same layers with the "
                        "heads on one stream (the timed region's two streams overlap consecutive heads)")
    for w in head_ws:
        F.device_status(w)
    stage_names = ["prep", "stats", "rowmax", "route", "tile"]
    stage_ms = {nm: statistics.mean(stage_evs[s][i][j].elapsed_time(stage_evs[s][i][j + 1])
                                    for s in range(a.steps) for i in range(nslots))
                for j, nm in enumerate(stage_names)}

    # ---- parity at full size on a tile sample of head 0 (rank 0): mean |dlogZ| vs the oracle
    parity = {}
    cpu = None
    ref_gpu = None
    oracle_rows = None
    h0 = all_jobs[0]
    mask0 = out0 = lse0 = None
    if rank == 0:
        # the first job once more with its routing mask exported
        mask0 = torch.zeros((nt, F.leaf_pitch(nb)), dtype=torch.uint8, device=dev)
        out0 = torch.empty((n, 128), dtype=torch.float32, device=dev)
        lse0 = torch.empty((n,), dtype=torch.float32, device=dev)
        # with the reference's GPU arithmetic (its Triton division), for the comparison with its operator
        F.forward_into(*dq[h0], None, None, exact_leaves=E, out=out0, lse=lse0, workspace=ws, store=store,
                       route_mask=mask0, precision=prec_ref)
        # and with IEEE code division, the oracle's arithmetic
        mask0i, out0i, lse0i = torch.zeros_like(mask0), torch.empty_like(out0), torch.empty_like(lse0)
        F.forward_into(*dq[h0], None, None, exact_leaves=E, out=out0i, lse=lse0i, workspace=ws, store=store,
                       route_mask=mask0i, precision=prec_ieee)
        torch.cuda.synchronize(dev)
        F.device_status(ws)
    if rank == 0 and not a.no_cpu and not fp8:
        qn, kn, vn = (t.float().numpy() for t in host[h0])
        rng = np.random.default_rng(1)
        tiles = np.sort(rng.choice(nt, size=a.cpu_tiles, replace=False))
        threads = host_threads()
        dp, dt, ro, rl, prep = oracle_sample(qn, kn, vn, E, tiles, threads, a.precision)
        rows = (tiles[:, None] * 64 + np.arange(64)[None, :]).reshape(-1)
        valid = rows < n
        oracle_rows = (rows[valid], ro[valid], rl[valid])
        lse_d = lse0i.cpu().numpy()[rows[valid]]
        out_d = out0i.cpu().numpy()[rows[valid]]
        excl_o = oracle_routing(prep, tiles, E, threads, a.precision)
        excl_d = mask0i[torch.as_tensor(tiles, device=dev)][:, :nb].cpu().numpy()
        parity = {"logz_mae": float(np.abs(lse_d - rl[valid]).mean()),
                  "out_maxabs": float(np.abs(out_d - ro[valid]).max()),
                  "routing_agreement_sample": float((excl_o == (excl_d != 0)).mean()),
                  "sample": f"{len(tiles)} random tiles of head {h0} vs oracle/flat_oracle.py at precision "
                            f"{a.precision}, IEEE code division (the oracle computes its own float64 leaf "
                            f"statistics, selection and routing for them)"}
        parity["codes_full_size"] = full_size_codes(F, dq[h0], prep, E, threads)
        # error of the operator against exact softmax attention on the same rows
        qs = dq[h0][0][torch.as_tensor(rows[valid], device=dev)].float()
        kk, vv = dq[h0][1].float(), dq[h0][2].float()
        s_ = (qs @ kk.T) / math.sqrt(128)
        ex = torch.softmax(s_, -1) @ vv
        od = out0i[torch.as_tensor(rows[valid], device=dev)]
        parity["rel_l2_vs_exact"] = float((od - ex).norm() / ex.norm())
        del s_
        if world == 1:
            per_tile = dt / len(tiles)
            cpu_ms = (dp + per_tile * nt) * H * 1e3
            cpu = {"value": cpu_ms, "unit": "ms/layer", "cores": threads, "kind": "port",
                   "sample": f"head {h0}: per-head preparation + {len(tiles)} query tiles ({len(tiles) * 64} rows of "
                             f"{n}) through oracle/flat_oracle.py; layer = {H} x (prep + {nt} x per-tile)"}
            if not a.no_ref_cpu:
                cpu["reference_torch"] = reference_cpu_legs(threads)
    if rank == 0 and world == 1 and not a.no_ref_gpu and not fp8:
        ref_gpu = reference_gpu_leg(wl, dev, step_jobs[0][:H], dq, {"out": out0, "lse": lse0, "mask": mask0,
                                                                    "out_ieee": out0i, "lse_ieee": lse0i,
                                                                    "division": "triton"},
                                    max(1, min(a.steps, a.ref_steps)), oracle_rows)
        if "ms_per_layer" in ref_gpu:
            ref_gpu["ours_over_ref"] = ms / ref_gpu["ms_per_layer"]

    # ---- end to end through the public API with pinned host buffers
    e2e = None
    if not a.no_e2e:
        qb = [torch.empty_like(dq[h0][j]) for j in range(3) for _ in range(2)]
        stage_in = [(qb[0], qb[2], qb[4]), (qb[1], qb[3], qb[5])]
        stage_out = [(torch.empty((n, 128), dtype=torch.float32, device=dev),
                      torch.empty((n,), dtype=torch.float32, device=dev)) for _ in range(2)]
        host_out = [(torch.empty((n, 128), dtype=torch.float32).pin_memory(),
                        torch.empty((n,), dtype=torch.float32).pin_memory()) for _ in range(nslots)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        in_done = [torch.cuda.Event() for _ in range(2)]
        comp_done = [torch.cuda.Event() for _ in range(2)]
        out_done = [torch.cuda.Event() for _ in range(2)]

        def e2e_layer(step):
            for s_ in head_streams[1:]:
                s_.wait_stream(comp)
            for i, h in enumerate(step_jobs[step % nblocks]):
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
                                           lse=stage_out[b][1], workspace=head_ws[i % len(head_ws)], stream=hs,
                                           precision=prec)
                comp_done[b].record(hs)
                s_out.wait_event(comp_done[b])
                with torch.cuda.stream(s_out):
                    host_out[i][0].copy_(stage_out[b][0], non_blocking=True)
                    host_out[i][1].copy_(stage_out[b][1], non_blocking=True)
                    out_done[b].record(s_out)
            for s_ in head_streams[1:]:
                comp.wait_stream(s_)

        def join_copies():
            # the copy streams run across layer boundaries (layer L's last copies-out overlap layer L + 1's
            # compute); the timed region ends only after every copy of every timed layer
            comp.wait_stream(s_in)
            comp.wait_stream(s_out)

        for s in range(a.warmup):
            e2e_layer(s)
        join_copies()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        for s in range(a.steps):
            e2e_layer(s)
        join_copies()
        e1.record(comp)
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / a.steps) / layers_per_step
        h2d = sum(sum(t.numel() * t.element_size() for t in host[h]) for h in step_jobs[0]) * world
        d2h = sum(sum(t.numel() * t.element_size() for t in o) for o in host_out) * world
        # the last timed e2e step and the last device pass computed the same block: identical outputs
        torch.cuda.synchronize(dev)
        same = all(bool(torch.equal(host_out[i][0].to(dev), out[i])) for i in (0, nslots - 1))
        e2e = {"value": e2e_ms, "unit": "ms/layer", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "htrc_b200.forward_into, pinned host q/k/v in and out/lse back, copies overlapped on "
                      f"2 copy streams (also across layers), heads on {a.streams} compute stream(s)",
               "matches_device_run": same}

    # ---- the reference runner's modes on head 0 (rank 0, one GPU): ms per head through FlatRunner's
    # CUDA graph (static-buffer copies included), and the k-means ordering alone
    modes = None
    if rank == 0 and world == 1 and not a.no_modes:
        from htrc_b200 import runner as R
        modes = {}
        for mode in list(R.MODES) + ["fast+iso", "fast+fp8", "fast+bf16", "fast+leaf32", "fast+leaf16"]:
            extra = {"fast+iso": dict(backend="cuda", curvature="iso"), "fast+fp8": dict(store="fp8"),
                     "fast+bf16": dict(store="bf16"), "fast+leaf32": dict(leaf=32),
                     "fast+leaf16": dict(leaf=16)}.get(mode, {})
            r = R.FlatRunner(n, m, mode=mode.split("+")[0], device=dev, **{"leaf": 64, **extra})
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
                         "fast+fp8: fast with the e4m3 far-field state (store='fp8'); fast+bf16: with the bf16 "
                         "far-field state (store='bf16'); fast+leaf32 / fast+leaf16: "
                         "fast with leaves of 32 / 16 keys (E=256 leaves, so 8,192 / 4,096 exact keys per tile; leaf "
                         "16 is the default of the reference's runner); the others leaf 64"}

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
        stage_bytes["rowmax"] = nt * nb * 128 + 2 * nt * pitch * 4 + nt * pitch * 4
    if bf16_state:
        stage_bytes["stats"] = nt * nb * (256 + 256) + nt * pitch * 4           # bf16 g + vbar, lz
        stage_bytes["rowmax"] = nt * nb * 256 + nt * pitch * 4 + nt * pitch * 4  # bf16 g + lz read, sel written
    stage_roof = {nm: {"bound": "hbm", "bytes": b_, "achieved_gbs": b_ / (stage_ms[nm] * 1e-3) / 1e9,
                       "frac": b_ / (stage_ms[nm] * 1e-3) / 1e9 / hbm}
                  for nm, b_ in stage_bytes.items()}
    stage_roof["stats"]["tensor_frac"] = (6.0 * nt * m * 128 / (stage_ms["stats"] * 1e-3) / 1e12) / peak
    stage_roof["tile"] = {"bound": "tensor", "frac": roof["frac"]}

    if rank == 0:
        line = {"metric": METRIC, "value": ms, "unit": "ms/layer", "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": False, "scaling": "strong",
                "vs_baseline": None,
                "dtype": ("bf16 state; bf16 QK and PV, f32 softmax" if bf16_state else
                          "fp8 (e4m3) state; fp16 far / bf16 near QK and PV, f32 softmax" if fp8 else
                          "int8 QK + bf16 PV, f32 softmax"),
                "data": "synthetic: seeded smooth-field Q/K (4x8x8 grid trilinear + 0.5 noise, RMS 3), N(0,1) V, bf16",
                "config": {"workload": (wl["name"].replace("INT8", "bf16 state") if bf16_state else
                                        wl["name"].replace("INT8", "fp8 (e4m3) state") if fp8 else wl["name"]),
                           "tokens": n, "heads": H, "cfg_batch": batch, "blocks_resident": nblocks,
                           "dim": 128, "leaf": 64, "tile": 64, "store": a.store,
                           "exact_leaves": E, "precision": a.precision, "division": a.division, "pairs_per_gpu": nslots,
                           "layers_per_step": layers_per_step,
                           "head_streams": a.streams,
                           "l2": "inputs larger than L2: 2.4 GB of distinct q/k/v per layer, "
                                 + ("2.1" if bf16_state else "1.0" if fp8 else "1.6") + " GB leaf state per head",
                           "parallelism": f"(batch, head) pairs/{world}" +
                                          (" + bf16 output all_gather (NCCL)" if world > 1 else "")},
                "stage_ms_per_head": stage_ms, "stage_timing": stage_timing, "stage_roofline": stage_roof,
                "gather": gather_info, "modes": modes,
                **parity,
                "roofline": roof, "cpu_baseline": cpu, "reference_gpu": ref_gpu,
                "e2e": e2e,
                "gpu_launches": a.steps * nslots * LAUNCHES_PER_HEAD, "clocks": clk}
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------------
# the hierarchical operator (workload cfg5)

def tree_launches(levels):
    """Kernels one head launches through htrc_b200.tree.tree_attention with a forest of `levels` levels: the
    k-means (8 x 2 + 3) and the centre conversion, the build (leaves, level 1 from the keys, one merge per higher
    level), the walk (2 grouping, one per internal level, count, scan) and the values (one per internal level,
    the leaf blocks, the final merge)."""
    internal = max(0, levels - 1)
    return 20 + (1 + (1 if levels >= 2 else 0) + max(0, levels - 2)) + (2 + internal + 2) + (internal + 2)


def tree_oracle_sample(k, v, q, centres, assign, rows_per_centre=6, ncentres=2, wl=None, out=None, lse=None,
                       cnt=None):
    """The float64 tree oracle on a bounded sample of one head: the forests of `ncentres` centres and
    `rows_per_centre` of their queries.  Returns (timing dict, parity dict or None)."""
    import numpy as np
    from oracle import tree_oracle as T
    kn, vn = k.float().cpu().numpy(), v.float().cpu().numpy()
    qn = q.float().cpu().numpy()
    cen = centres.float().cpu().numpy().astype(np.float64)
    asg = assign.cpu().numpy().astype(np.int64)
    sc = 1.0 / math.sqrt(128)
    t_forest, t_eval, nq = 0.0, 0.0, 0
    errs, lerr, agree, total = [], [], 0, 0
    for c in np.unique(asg)[:ncentres]:
        rows = np.nonzero(asg == c)[0]
        rows = rows[np.linspace(0, rows.size - 1, min(rows_per_centre, rows.size)).round().astype(int)]
        t0 = time.perf_counter()
        lv = T.forest(kn, vn, cen[c], leaf_size=wl["leaf"], fanout=wl["fanout"])
        t1 = time.perf_counter()
        ref, ref_lse, info = T.evaluate(kn, vn, qn[rows].astype(np.float64) * sc, cen[c], lv,
                                        opening_threshold=wl["threshold"])
        t2 = time.perf_counter()
        t_forest += t1 - t0
        t_eval += t2 - t1
        nq += rows.size
        if out is not None:
            errs.append(np.abs(out[rows] - ref).max())
            lerr.append(np.abs(lse[rows] - ref_lse))
            rc = np.stack([info[x] for x in ("visited_nodes", "accepted_nodes", "exact_leaves")], 1)
            agree += int((cnt[rows] == rc).all(1).sum())
            total += rows.size
    timing = {"forest_s_per_centre": t_forest / ncentres, "evaluate_s_per_query": t_eval / nq, "queries": nq,
              "centres": ncentres}
    parity = None
    if out is not None:
        parity = {"rows": total, "centres": ncentres, "out_maxabs": float(max(errs)),
                  "logz_mae": float(np.concatenate(lerr).mean()), "counters_agree": agree / total,
                  "oracle": "oracle/tree_oracle.py (float64 restatement of src/htrc_reference/model.py)"}
    return timing, parity


def run_tree(a, wl, rank, world, local_rank):
    import numpy as np
    import torch

    from htrc_b200 import shard, synth, tree

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
    H = wl["heads"]
    try:
        mine = list(shard.heads_of_rank(H, rank, world))
    except ValueError as e:
        raise SystemExit(str(e))
    kw = dict(leaf_size=wl["leaf"], fanout=wl["fanout"], opening_threshold=wl["threshold"])
    host = {h: tuple(t.pin_memory() for t in synth.head_inputs(wl["grid"], 128, head=h)) for h in mine}
    dq = {h: tuple(t.to(dev, non_blocking=True) for t in host[h]) for h in mine}
    n = host[mine[0]][0].shape[0]
    out_host = {h: torch.empty((n, 128), dtype=torch.float32).pin_memory() for h in mine}
    lse_host = {h: torch.empty((n,), dtype=torch.float32).pin_memory() for h in mine}

    def layer():
        for h in mine:
            tree.tree_attention(*dq[h], **kw)

    def layer_e2e():
        for h in mine:
            q, k, v = (t.to(dev, non_blocking=True) for t in host[h])
            o, l_ = tree.tree_attention(q, k, v, return_lse=True, **kw)
            out_host[h].copy_(o, non_blocking=True)
            lse_host[h].copy_(l_, non_blocking=True)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(a.warmup):
        layer()
    barrier()
    clk_s = ClockSampler(local_rank)
    clk_s.start()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        layer()
    e1.record()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    clk = clk_s.stop()
    e2e = None
    if not a.no_e2e:
        layer_e2e()
        barrier()
        e0.record()
        for _ in range(a.steps):
            layer_e2e()
        e1.record()
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
        per_head_in = sum(t.numel() * t.element_size() for t in host[mine[0]])
        e2e = {"value": e2e_ms, "unit": "ms/layer", "h2d_bytes_per_step": per_head_in * len(mine) * world,
               "d2h_bytes_per_step": (n * 128 * 4 + n * 4) * len(mine) * world,
               "api": "htrc_b200.tree.tree_attention with pinned host q/k/v copied in and out / lse copied back"}
    # stage times of one head (its own pass, events between the stages)
    marks = []
    h0 = mine[0]
    out, lse, info = tree.tree_attention(*dq[h0], return_lse=True, return_info=True, marks=marks, **kw)
    torch.cuda.synchronize()
    stage_ms = {marks[i][0]: marks[i - 1][1].elapsed_time(marks[i][1]) for i in range(1, len(marks))}
    stage_ms["start"] = stage_ms.pop("start", 0.0)          # build -> walk gap (host allocation): reported as is
    leaves = int(info["leaves"].sum().item())
    levels = info["forest"].levels
    peaks, src = measured_peaks()
    peak = peaks["bf16_tflops"]
    flop = leaves * 2 * (2 * 64 * 128)                       # S = q.k and P.v per (query, visited leaf) of 64 keys
    achieved = flop / (stage_ms["leaves"] * 1e-3) / 1e12
    roof = {"kernel": "tree_leafblock_tc_kernel", "bound": "tensor", "achieved": achieved, "peak": peak,
            "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
            "peak_source": f"{src} bf16_tflops (burst: the stage is timed alone)",
            "flop_per_launch": flop, "note": "bf16-equivalent flop of the law's leaf work: 2 x 2*64*128 per (query, "
            "visited leaf); the kernel issues the PV product twice (bf16 hi + lo parts of P)"}
    counters = {x: float(info[x].float().mean().item()) for x in ("visited_nodes", "accepted_nodes", "exact_leaves",
                                                                   "leaves")}
    cpu, parity = None, None
    if rank == 0 and world == 1 and not a.no_cpu:
        q0, k0, v0 = dq[h0]
        cnt = torch.stack([info["visited_nodes"], info["accepted_nodes"], info["exact_leaves"]], 1).cpu().numpy()
        timing, parity = tree_oracle_sample(k0, v0, q0, info["centres"], info["assign"], wl=wl,
                                            out=out.float().cpu().numpy(), lse=lse.float().cpu().numpy(), cnt=cnt)
        ncen = int(info["centres"].shape[0])
        layer_s = (timing["forest_s_per_centre"] * ncen + timing["evaluate_s_per_query"] * n) * H
        cpu = {"value": layer_s * 1e3, "unit": "ms/layer", "cores": 1, "kind": "port",
               "sample": f"oracle/tree_oracle.py (float64 NumPy) on head 0: the forests of {timing['centres']} "
                         f"centres and {timing['queries']} of their queries, extrapolated to {ncen} centres x {n} "
                         f"queries x {H} heads", **timing}
    if rank == 0:
        line = {"metric": f"hierarchical-HTRC ms per {n:,}-token {H}-head d128 layer", "value": ms, "unit": "ms/layer",
                "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": False,
                "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16 q.k and P.v on tcgen05 (P as bf16 hi + lo), f32 node predictions and decisions",
                "data": "synthetic: seeded smooth-field Q/K (4x8x8 grid trilinear + 0.5 noise, RMS 3), N(0,1) V, bf16",
                "config": {"workload": wl["name"], "tokens": n, "heads": H, "dim": 128, "leaf": wl["leaf"],
                           "fanout": wl["fanout"], "threshold": wl["threshold"], "levels": levels,
                           "nodes_per_level": info["forest"].nodes, "heads_per_gpu": len(mine),
                           "l2": "inputs larger than L2: 189 MB of q/k/v and 1.1 GB of forest per head",
                           "parallelism": f"heads/{world}, no collective (outputs stay on their rank)"},
                "stage_ms_head0": stage_ms, "counters_mean_head0": counters,
                "roofline": roof, "cpu_baseline": cpu, "parity_head0": parity, "e2e": e2e,
                "gpu_launches": a.steps * len(mine) * tree_launches(levels), "clocks": clk}
        print(json.dumps(line), flush=True)


def run_tree_reference(a, wl, rank):
    """The reference's own NumPy hierarchical model (src/htrc_reference: build_forest + evaluate, one query at a
    time) on a bounded sample of the cfg5 workload, extrapolated to the layer; rank 0 only."""
    if rank != 0:
        return
    import numpy as np
    from htrc_b200 import synth
    model = None
    ref_dir = ROOT / "baseline" / "_ref"
    if (ref_dir / "htrc_reference" / "model.py").exists():
        sys.path.insert(0, str(ref_dir))
        from htrc_reference import model                        # noqa: F401
    if model is None:
        print(json.dumps({"impl": "reference", "unavailable": "the reference package is not installed under "
                          "baseline/_ref (baseline/install_ref.sh)"}), flush=True)
        return
    q, k, v = (t.float().numpy().astype(np.float64) for t in synth.head_inputs(wl["grid"], 128, head=0))
    sc = 1.0 / math.sqrt(128)
    centre = (q[::64] * sc).mean(0)
    times = []
    for step in range(a.warmup + a.steps):
        t0 = time.perf_counter()
        forest = model.build_forest(k, v, centre, leaf_size=wl["leaf"], fanout=wl["fanout"])
        t1 = time.perf_counter()
        for i in range(2):
            model.evaluate(k, v, q[(1000 * step + 977 * i) % q.shape[0]] * sc, centre, forest,
                           opening_threshold=wl["threshold"])
        t2 = time.perf_counter()
        times.append(((t1 - t0) * 32 + (t2 - t1) / 2 * q.shape[0]) * wl["heads"] * 1e3)
    val = statistics.median(times[a.warmup:])
    print(json.dumps({"impl": "reference", "metric": "hierarchical-HTRC ms per 245,952-token 24-head d128 layer",
                      "value": val, "unit": "ms/layer", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
                      "higher_is_better": False, "config": {"workload": wl["name"]},
                      "cpu_baseline": {"value": val, "unit": "ms/layer", "cores": 1, "kind": "reference",
                                       "sample": "src/htrc_reference build_forest at one centre + evaluate of 2 "
                                                 "queries per step on head 0, extrapolated to 32 centres x 245,952 "
                                                 "queries x 24 heads"},
                      "e2e": {"value": val, "unit": "ms/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


def main():
    a = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if a.workload == "auto":
        a.workload = "cfg3" if world == 1 else "cfg4"
    wl = WORKLOADS[a.workload]
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        if wl.get("tree"):
            run_tree_reference(a, wl, rank)
        else:
            run_reference(a, wl, rank)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if wl.get("tree"):
            run_tree(a, wl, rank, world, local_rank)
        else:
            run_ours(a, wl, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
