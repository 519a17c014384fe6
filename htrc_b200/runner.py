"""Production entry point of the flat HTRC operator on B200: CUDA-graph head runner.

Same call shape as the reference's h3/htrc_flat_runner.py (``FlatRunner``, ``MODES``, ``CHUNKS``,
``predicted_peak_mib``, ``plan_chunk``):

    runner = FlatRunner(queries, keys, free_bytes=free_vram, mode="fast", leaf=64)   # leaf default: 16
    outputs = runner.run([(head, q, k, v), ...])          # q [Q,128], k/v [K,128] on CUDA
    runner.run(jobs, sink=lambda i, out: block_out[i].copy_(out))

One head is a single ``htrc_flat_forward`` launch sequence with no host synchronisation and no
allocation, so it is captured once into a CUDA graph (static q/k/v/out/lse buffers) and replayed per
head; if capture fails the runner falls back to eager launches and records ``graph_error``.
As in the reference, the configuration is PROD updated by the mode and the caller's overrides, so without a
``leaf=`` override the leaf is ``flat_attention``'s default of 16 keys (pass ``leaf=64`` for the production
benchmark's leaf).
Differences from the reference: ``head()`` and ``run()`` without a sink always return fresh tensors
(the reference's eager path returns views of one reused workspace buffer, h3/htrc_flat.py:234 with
h3/htrc_flat_triton.py:302-312); ``lse=True`` also returns the per-query log-partition.
"""
from __future__ import annotations

import torch

from . import _lib
from . import flat as _flat

MODES = {
    "fast": dict(exact_leaves=256, order="seq", tile=64),
    "balanced": dict(exact_leaves=512, order="seq", tile=64),
    "accurate": dict(exact_leaves=1024, order="kmeans", tile=64),
    "max": dict(exact_leaves=1024, order="kmeans", tile=32),
}
"""Routing budgets of the reference's modes (h3/htrc_flat_runner.py:48-53)."""
CHUNKS = (1024, 512, 256, 128, 64, 32, 16)

STATIC_MIB = 0.0      # graph runner's static q (fp32) / k / v (bf16) copies, added per call below
KMEANS_MIB = 0.0      # the k-means ordering's scratch is part of the library workspace (order="kmeans")


def predicted_peak_mib(keys: int, tile: int, tile_chunk: int, splits: int = 8, leaf: int = 16,
                       dim: int = 128, order: str = "seq", graph: bool = True, queries: int = 0,
                       exact_leaves: int = 256, group: int = 1) -> float:
    """Device memory of one head above the caller's q/k/v, in MiB: this library's workspace
    (htrc_flat_workspace_size: codes, per-chunk state, k-means scratch) for the chunk size, plus the
    static graph copies.  Same signature as the reference's model (h3/htrc_flat_runner.py:61-68);
    ``splits`` is accepted and unused."""
    q = int(queries) if queries else int(tile) * max(1, int(tile_chunk))
    ws = _flat.workspace_bytes(q, int(keys), int(exact_leaves), 0, int(tile_chunk), 0, int(group),
                               _flat.order_code(order), int(tile), leaf=int(leaf))
    static = (q * dim * 4 + 2 * keys * dim * 2 + q * (dim + 1) * 4) if graph else 0
    kmeans = KMEANS_MIB if order == "kmeans" else 0.0
    return (ws + static) / 2 ** 20 + kmeans


def plan_chunk(free_bytes: int, keys: int, tile: int, splits: int = 8, order: str = "seq",
               graph: bool = True, queries: int = 0, leaf: int = 16, exact_leaves: int = 256,
               group: int = 1) -> int:
    """Largest tile chunk whose predicted peak fits in ``free_bytes`` (h3/htrc_flat_runner.py:71-84);
    raises MemoryError when even the smallest chunk does not fit."""
    nt = -(-int(queries) // int(tile)) if queries else 0
    # the whole sequence in one chunk first: one launch per stage, and the tile kernel's grid covers every
    # SM (a chunk of 128 tiles is 64 CTAs on 148 SMs)
    cands = ((nt,) if nt > CHUNKS[0] else ()) + CHUNKS
    for c in cands:
        eff = min(c, nt) if nt else c
        if predicted_peak_mib(keys, tile, eff, splits, leaf, order=order, graph=graph, queries=queries,
                              exact_leaves=exact_leaves, group=group) * 2 ** 20 <= free_bytes:
            return c
    need = predicted_peak_mib(keys, tile, CHUNKS[-1], splits, leaf, order=order, graph=graph, queries=queries,
                              exact_leaves=exact_leaves, group=group)
    raise MemoryError(f"flat HTRC needs ~{need:.0f} MiB at the smallest chunk, {int(free_bytes) >> 20} MiB free")


class FlatRunner:
    """Runs heads of one (queries, keys) shape; see the module docstring."""

    def __init__(self, queries: int, keys: int, *, free_bytes: int | None = None,
                 mode: str = "balanced", tile_chunk: int | None = None, use_graph: bool = True,
                 device="cuda", dim: int = 128, sink_leaves: int = 0, tail_rows: int = 0,
                 lse: bool = False, **overrides):
        if mode not in MODES:
            raise ValueError(f"mode must be one of {list(MODES)}")
        self.mode = mode
        self.device = torch.device(device)
        base = dict(_flat.PROD)
        base.update(MODES[mode])
        overrides = dict(overrides)
        if "kern" in overrides:                          # a caller's kern dict updates PROD's launch knobs key by key
            base["kern"] = {**base.get("kern", {}), **overrides.pop("kern")}
        base.update(overrides)
        base["sink_leaves"] = int(sink_leaves)
        base["leaf"] = int(base.get("leaf", 16))        # flat_attention's default leaf (h3/htrc_flat.py:100)
        self.leaf = base["leaf"]
        self.tail_rows = int(tail_rows)
        self.want_lse = bool(lse)
        self.queries, self.keys, self.dim = int(queries), int(keys), int(dim)
        self.group = _flat.group_of(base.get("kern"))
        self.order = _flat.order_code(base["order"])
        self.curvature = _flat.curvature_code(base.get("curvature", "lin"))
        self.store = _lib.STORES.get(base.get("store", "int8"), _lib.STORE_INT8)
        self.qk_scale_block = int(base.get("qk_scale_block") or 0)
        if tile_chunk is None:
            if free_bytes is None and self.device.type == "cuda" and torch.cuda.is_available():
                # plan from the device's free memory (the reference falls back to PROD's 128-tile chunk,
                # sized for a 16 GB card; the chunk size changes no result)
                free_bytes = int(torch.cuda.mem_get_info(self.device)[0] * 0.8)
            if free_bytes is not None:
                tile_chunk = plan_chunk(free_bytes, keys, base["tile"], base.get("splits", 8), base["order"],
                                        use_graph, queries=int(queries), leaf=self.leaf,
                                        exact_leaves=base["exact_leaves"], group=self.group)
            else:
                tile_chunk = base["tile_chunk"]
        base["tile_chunk"] = int(tile_chunk)
        self.cfg = base
        self.predicted_mib = predicted_peak_mib(keys, base["tile"], base["tile_chunk"], base.get("splits", 8),
                                                self.leaf, order=base["order"], graph=use_graph, queries=int(queries),
                                                exact_leaves=base["exact_leaves"], group=self.group)
        self.ws = {}
        self.graph = None
        self.graph_error = None
        self._capturing = False
        self._sq = self._sk = self._sv = self._so = self._sl = self._tk = self._tv = self._w = None
        # validate the configuration once (raises NotImplementedError / ValueError like the operator)
        probe_q = torch.empty((1, dim), device="meta")
        probe_k = torch.empty((base["leaf"], dim), device="meta")
        try:
            _flat._check_args(probe_q, probe_k, probe_k, base["tile"], base["exact_leaves"], base["order"],
                              base.get("curvature", "lin"), base["leaf"], base.get("select", "max"),
                              base["backend"], base["store"], base["dot"], base.get("sel_stride", 1),
                              base.get("quant"), base["sink_leaves"], None)
        except ValueError as exc:
            if "CUDA tensors" not in str(exc):
                raise
        _flat._check_scale_block(base.get("qk_scale_block"), base["store"], self.leaf)
        if use_graph:
            self._capture()

    # -- eager path
    def _call(self, q, k, v, tail=None):
        if tail is None and self._tk is not None:
            tail = (self._tk, self._tv)
        c = {k_: v_ for k_, v_ in self.cfg.items()}
        return _flat.flat_attention(q, k, v, tail=tail, ws=self.ws, return_lse=self.want_lse, **c)

    # -- graph path
    def _capture(self):
        dev = self.device
        c = self.cfg
        with torch.cuda.device(dev):
            self._sq = torch.zeros((self.queries, self.dim), device=dev, dtype=torch.float32)
            self._sk = torch.zeros((self.keys, self.dim), device=dev, dtype=torch.bfloat16)
            self._sv = torch.zeros_like(self._sk)
            self._sq.normal_()
            self._sk.normal_()
            self._sv.normal_()
            if self.tail_rows:
                self._tk = torch.randn((self.tail_rows, self.dim), device=dev, dtype=torch.float32)
                self._tv = torch.randn_like(self._tk)
            self._so = torch.empty((self.queries, self.dim), device=dev, dtype=torch.float32)
            self._sl = torch.empty((self.queries,), device=dev, dtype=torch.float32)
            nbytes = _flat.workspace_bytes(self.queries, self.keys, c["exact_leaves"], c["sink_leaves"],
                                           c["tile_chunk"], self.tail_rows, self.group, self.order, c["tile"],
                                           self.curvature, self.store, self.leaf)
            self._w = _flat.new_workspace(nbytes, dev)
            kw = dict(exact_leaves=c["exact_leaves"], sink_leaves=c["sink_leaves"], tile_chunk=c["tile_chunk"],
                      scale=c.get("scale"), out=self._so, lse=self._sl, workspace=self._w, group=self.group,
                      order=self.order, tile=c["tile"], curvature=self.curvature, store=self.store,
                      qk_scale_block=self.qk_scale_block, precision=_flat.precision_code(c.get("precision", "fp32"),
                                                                               c.get("division", "ieee")),
                      leaf=self.leaf)
            self._capturing = True
            try:
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side), torch.inference_mode():
                    for _ in range(2):
                        _flat.forward_into(self._sq, self._sk, self._sv, self._tk, self._tv, **kw)
                torch.cuda.current_stream().wait_stream(side)
                torch.cuda.synchronize()
                _flat.device_status(self._w)
                g = torch.cuda.CUDAGraph()
                with torch.inference_mode(), torch.cuda.graph(g, capture_error_mode="thread_local"):
                    _flat.forward_into(self._sq, self._sk, self._sv, self._tk, self._tv, **kw)
                torch.cuda.synchronize()
                self.graph = g
            except Exception as exc:  # noqa: BLE001  (fall back to eager launching, as the reference does)
                self.graph = None
                self.graph_error = f"{type(exc).__name__}: {exc}"[:300]
                self._sq = self._sk = self._sv = self._so = self._sl = self._w = None
                torch.cuda.empty_cache()
            finally:
                self._capturing = False

    def _set_tail(self, tail):
        if self.tail_rows and self.graph is not None and tail is not None:
            self._tk.copy_(tail[0])
            self._tv.copy_(tail[1])

    def _replay(self, q, k, v, tail):
        self._set_tail(tail)
        self._sq.copy_(q)
        self._sk.copy_(k)
        self._sv.copy_(v)
        self.graph.replay()

    def head(self, q, k, v, tail=None):
        """One head; returns a fresh fp32 [Q, D] tensor (and lse [Q] if the runner was built with
        lse=True).  tail=(tk, tv) [tail_rows, D]."""
        if self.graph is None:
            with torch.inference_mode():
                return self._call(q, k, v, tail=tail)
        self._replay(q, k, v, tail)
        if self.want_lse:
            return self._so.clone(), self._sl.clone()
        return self._so.clone()

    def run(self, jobs, sink=None):
        """jobs: list of (head_index, q, k, v[, (tail_k, tail_v)]).  Outputs in job order, or via
        sink(i, output) (graph path: the static output buffer itself, no copy)."""
        results = [None] * len(jobs)
        for i, job in enumerate(jobs):
            q, k, v = job[1], job[2], job[3]
            tail = job[4] if len(job) > 4 else None
            if self.graph is None or sink is None:
                out = self.head(q, k, v, tail=tail)
                if sink is None:
                    results[i] = out
                else:
                    sink(i, out)
            else:
                self._replay(q, k, v, tail)
                sink(i, (self._so, self._sl) if self.want_lse else self._so)
        return results if sink is None else None

    def check_status(self):
        """Raise if a kernel reported a device-side failure since the last check."""
        w = self._w if self._w is not None else self.ws.get("workspace")
        if w is not None:
            _flat.device_status(w)

    def close(self):
        self.graph = None
        self._sq = self._sk = self._sv = self._so = self._sl = self._w = None
