"""Hierarchical HTRC on B200: the law of the reference's NumPy teaching model (src/htrc_reference/model.py)
for many queries and several query centres, on the CUDA kernels of ``csrc/tree.cu`` (C ABI
``include/htrc_tree.h``).

Reference surface kept (model.py):
  build_forest(keys, values, center, *, leaf_size=16, fanout=4)              model.py:68-86
  evaluate(keys, values, query, center, forest, *, opening_threshold=0.01)   model.py:98-137
    -> (output, {"visited_nodes", "accepted_nodes", "exact_leaves"})
with the reference's ValueErrors (exact_stats / merge_stats are the forest's node statistics,
``Forest.level_stats``).  Extensions: `center` may hold several centres ([C, D]) with
`assign=` naming each query's centre; `query` may hold many rows ([N, D]); `return_lse=True` adds the
log-sum-exp of the accepted log-masses.  ``tree_attention(q, k, v)`` is the whole operator of the
hierarchical benchmark configuration (k-means query centres, leaf 64, fanout 16, threshold 0.02).

Arithmetic is float32 on the GPU (the reference's model is float64): keys, values and queries are
read as given (float32 or bfloat16; other float types are converted to float32), rows narrower than
128 are zero-padded, which changes no dot product.  There is no CPU path: without the built library or
a GPU every call raises.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

D_MAX = 128


def _dims(m, n, ncen, leaf, fanout, kv_dtype, q_dtype, scale, thr):
    d = _lib.HtrcTreeDims()
    d.n_keys, d.n_queries, d.n_centres = int(m), int(n), int(ncen)
    d.leaf_size, d.fanout = int(leaf), int(fanout)
    d.kv_dtype, d.q_dtype = kv_dtype, q_dtype
    d.scale, d.threshold = float(scale), float(thr)
    return d


def _rows(x, name, device, dtype=None):
    """x as a contiguous [rows, 128] device tensor (float32, or bfloat16 kept), zero-padded columns."""
    t = torch.as_tensor(x)
    if t.ndim != 2 or t.shape[0] == 0:
        raise ValueError("keys/values must be matching nonempty matrices")
    if t.shape[1] > D_MAX:
        raise NotImplementedError(f"{name}: rows wider than {D_MAX} are not supported")
    if dtype is None:
        dtype = torch.bfloat16 if t.dtype == torch.bfloat16 else torch.float32
    t = t.to(device=device, dtype=dtype)
    if t.shape[1] < D_MAX:
        t = torch.nn.functional.pad(t, (0, D_MAX - t.shape[1]))
    return t.contiguous()


def _code(t):
    return _lib.DTYPE_BF16 if t.dtype == torch.bfloat16 else _lib.DTYPE_F32


def _device(device):
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.type != "cuda":
        raise RuntimeError("htrc_b200.tree runs on a CUDA device only (no CPU fallback)")
    return dev


def _buffer(nbytes, device):
    return torch.empty(max(int(nbytes), 256) + 256, dtype=torch.uint8, device=device)


def _aligned(buf):
    off = (-buf.data_ptr()) % 256
    return buf.data_ptr() + off, buf.numel() - off


class Forest:
    """One forest per centre on the device (model.py:68-86): leaf log-masses and key logits, and per
    level >= 1 the node log-mass L, mean key g, mean value u, Hessian H and value Jacobian J."""

    def __init__(self, keys, values, centres, leaf_size, fanout, width, vwidth, device):
        self.keys, self.values, self.centres = keys, values, centres
        self.leaf_size, self.fanout, self.width, self.vwidth, self.device = leaf_size, fanout, width, vwidth, device
        dims = self.dims(0, 1.0, 0.0)
        nl = _lib._i32()
        nodes = (_lib._i32 * _lib.TREE_MAX_LEVELS)()
        _lib.check(_lib.lib().htrc_tree_levels(ctypes.byref(dims), ctypes.byref(nl), nodes), "tree levels")
        self.nodes = [int(nodes[i]) for i in range(nl.value)]
        need = ctypes.c_size_t()
        _lib.check(_lib.lib().htrc_tree_forest_size(ctypes.byref(dims), ctypes.byref(need)), "tree forest size")
        self._buf = _buffer(need.value, device)
        self._ptr, nbytes = _aligned(self._buf)
        _lib.check(_lib.lib().htrc_tree_build(ctypes.byref(dims), _lib.ptr(keys), _lib.ptr(values), _lib.ptr(centres),
                                              self._ptr, nbytes, _lib.stream_ptr()), "tree build")

    @property
    def n_centres(self):
        return int(self.centres.shape[0])

    @property
    def levels(self):
        return len(self.nodes)

    def dims(self, n_queries, scale, thr, q_dtype=None):
        kv = _code(self.keys)
        return _dims(self.keys.shape[0], n_queries, self.n_centres, self.leaf_size, self.fanout, kv,
                     kv if q_dtype is None else q_dtype, scale, thr)

    def level_stats(self, level, centre=0):
        """Float32 views of one centre's level: L [n] (level 0: leaf log-masses), and for level >= 1 g [n, D],
        u [n, Dv], H [n, D, D], J [n, Dv, D]; level 0 also gives the key logits a [n_keys]."""
        dims = self.dims(0, 1.0, 0.0)
        outs = [ctypes.c_void_p() for _ in range(6)]
        _lib.check(_lib.lib().htrc_tree_forest_view(ctypes.byref(dims), self._ptr, int(level),
                                                    *[ctypes.byref(o) for o in outs]), "tree forest view")
        n, c, D, Dv = self.nodes[level], int(centre), self.width, self.vwidth

        fl = self._buf[: (self._buf.numel() // 4) * 4].view(torch.float32)

        def at(p, count):
            return fl[(p - self._buf.data_ptr()) // 4:][:count]

        out = {"L": at(outs[1].value, self.n_centres * n).view(self.n_centres, n)[c]}
        if level == 0:
            m = self.keys.shape[0]
            out["a"] = at(outs[0].value, self.n_centres * m).view(self.n_centres, m)[c]
            return out
        out["g"] = at(outs[2].value, self.n_centres * n * D_MAX).view(self.n_centres, n, D_MAX)[c, :, :D]
        out["u"] = at(outs[3].value, self.n_centres * n * D_MAX).view(self.n_centres, n, D_MAX)[c, :, :Dv]
        big = self.n_centres * n * D_MAX * D_MAX
        out["H"] = at(outs[4].value, big).view(self.n_centres, n, D_MAX, D_MAX)[c, :, :D, :D]
        out["J"] = at(outs[5].value, big).view(self.n_centres, n, D_MAX, D_MAX)[c].transpose(1, 2)[:, :Dv, :D]
        return out


def build_forest(keys, values, center, *, leaf_size=16, fanout=4, device=None):
    """Forest of the keys/values at one centre [D] or several [C, D] (scaled query space), model.py:68-86."""
    if leaf_size < 1 or fanout < 2:
        raise ValueError("leaf_size must be positive and fanout >= 2")
    if leaf_size > 64 or fanout > 64:
        raise NotImplementedError("leaf_size and fanout above 64 are not supported")
    dev = _device(device)
    kt = torch.as_tensor(keys)
    vt = torch.as_tensor(values)
    if kt.ndim != 2 or vt.ndim != 2 or kt.shape[0] != vt.shape[0] or kt.shape[0] == 0:
        raise ValueError("keys/values must be matching nonempty matrices")
    ct = torch.as_tensor(center, dtype=torch.float64 if not torch.is_tensor(center) else None)
    ct = ct.reshape(1, -1) if ct.ndim == 1 else ct
    if ct.ndim != 2 or ct.shape[1] != kt.shape[1]:
        raise ValueError("scaled query dimension mismatch")
    if ct.shape[0] > _lib.TREE_MAX_CENTRES:
        raise NotImplementedError(f"more than {_lib.TREE_MAX_CENTRES} centres")
    kd = _rows(kt, "keys", dev)
    vd = _rows(vt, "values", dev, kd.dtype)
    cd = _rows(ct, "center", dev, torch.float32)
    return Forest(kd, vd, cd, int(leaf_size), int(fanout), int(kt.shape[1]), int(vt.shape[1]), dev)


def _run(forest, qd, assign, scale, thr, stream=None, marks=None):
    """Walk + values for device queries qd [N, 128] (forest's dtype) -> out [N, 128], lse [N] and counters
    [4, N] int32 (visited_nodes, accepted_nodes, exact_leaves, leaves visited).  marks: None, or a list that
    receives (name, CUDA event) after each stage (walk, accept, leaves, final) for stage timing."""
    n = qd.shape[0]
    dev = forest.device
    L = _lib.lib()
    dims = forest.dims(n, scale, thr, _code(qd))
    out = torch.empty((n, D_MAX), dtype=torch.float32, device=dev)
    lse = torch.empty((n,), dtype=torch.float32, device=dev)
    cnt = torch.zeros((4, n), dtype=torch.int32, device=dev)
    if n == 0:
        return out, lse, cnt
    need = ctypes.c_size_t()
    _lib.check(L.htrc_tree_walk_size(ctypes.byref(dims), ctypes.byref(need)), "tree walk size")
    wbuf = _buffer(need.value, dev)
    wptr, wbytes = _aligned(wbuf)
    s = _lib.stream_ptr(stream)

    def mark(name):
        if marks is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record(torch.cuda.current_stream() if stream is None else stream)
            marks.append((name, e))

    mark("start")
    nrec = _lib._i64()
    _lib.check(L.htrc_tree_walk(ctypes.byref(dims), _lib.ptr(qd), _lib.ptr(assign), _lib.ptr(forest.centres),
                                forest._ptr, wptr, wbytes, _lib.ptr(cnt[0]), _lib.ptr(cnt[1]), _lib.ptr(cnt[3]),
                                ctypes.byref(nrec), s), "tree walk")
    mark("walk")
    _lib.check(L.htrc_tree_records_size(nrec.value, ctypes.byref(need)), "tree records size")
    rbuf = _buffer(need.value, dev)
    rptr, rbytes = _aligned(rbuf)
    stages = [(_lib.TREE_STAGE_ALL, None)] if marks is None else \
        [(_lib.TREE_STAGE_ACCEPT, "accept"), (_lib.TREE_STAGE_LEAVES, "leaves"), (_lib.TREE_STAGE_FINAL, "final")]
    for bits, name in stages:
        _lib.check(L.htrc_tree_values(ctypes.byref(dims), _lib.ptr(forest.keys), _lib.ptr(forest.values),
                                      _lib.ptr(qd), _lib.ptr(forest.centres), forest._ptr, wptr, rptr, nrec.value,
                                      rbytes, _lib.ptr(out), _lib.ptr(lse), _lib.ptr(cnt[2]), bits, s), "tree values")
        if name:
            mark(name)
    return out, lse, cnt


def evaluate(keys, values, query, center, forest, *, opening_threshold=0.01, assign=None, return_lse=False):
    """Approximate attention of already-scaled queries through the forest (model.py:98-137).

    query [D] (the reference's form: returns out [Dv] and integer counters) or [N, D] (out [N, Dv] and
    counter tensors).  With several centres, `assign` [N] names each query's centre.  The keys and
    values must be the ones the forest was built from (the leaves' exact attention reads them)."""
    if opening_threshold < 0:
        raise ValueError("opening_threshold must be nonnegative")
    if not isinstance(forest, Forest):
        raise TypeError("forest must come from htrc_b200.tree.build_forest")
    qt = torch.as_tensor(query)
    single = qt.ndim == 1
    qt = qt.reshape(1, -1) if single else qt
    if qt.ndim != 2 or qt.shape[1] != forest.width:
        raise ValueError("scaled query dimension mismatch")
    kt = torch.as_tensor(keys)
    if kt.shape[0] != forest.keys.shape[0]:
        raise ValueError("keys differ from the forest's keys")
    ct = torch.as_tensor(center)
    if ct.reshape(-1, forest.width).shape[0] != forest.n_centres:
        raise ValueError("center differs from the forest's centres")
    n = qt.shape[0]
    if assign is None:
        if forest.n_centres != 1:
            raise ValueError("assign= is required with several centres")
        assign = torch.zeros(n, dtype=torch.int32, device=forest.device)
    assign = torch.as_tensor(assign).to(device=forest.device, dtype=torch.int32).contiguous()
    if assign.shape != (n,):
        raise ValueError("assign must hold one centre index per query")
    qd = _rows(qt, "query", forest.device, forest.keys.dtype) if n else torch.empty(
        (0, D_MAX), dtype=forest.keys.dtype, device=forest.device)
    out, lse, cnt = _run(forest, qd, assign, 1.0, opening_threshold)
    out = out[:, :forest.vwidth]
    info = {"visited_nodes": cnt[0], "accepted_nodes": cnt[1], "exact_leaves": cnt[2]}
    if single:
        out = out[0]
        lse = lse[0]
        info = {k: int(v[0]) for k, v in info.items()}
    return (out, info, lse) if return_lse else (out, info)


def queries_centres(q, scale, device=None):
    """The operator's query centres: the accurate mode's k-means (32 clusters, Lloyd x 8 on an even sample of
    at most 4096 rows) in the scaled space, and each row's nearest centre: (centres [32, 128], assign [N])."""
    qd = q if q.is_cuda else q.to(_device(device))
    n = qd.shape[0]
    L = _lib.lib()
    need = ctypes.c_size_t()
    _lib.check(L.htrc_tree_centres_scratch_size(n, ctypes.byref(need)), "tree centres scratch")
    buf = _buffer(need.value, qd.device)
    p, nbytes = _aligned(buf)
    centres = torch.empty((_lib.TREE_KMEANS_CENTRES, D_MAX), dtype=torch.float32, device=qd.device)
    assign = torch.empty((n,), dtype=torch.int32, device=qd.device)
    _lib.check(L.htrc_tree_centres(_lib.ptr(qd), _code(qd), n, float(scale), _lib.ptr(centres), _lib.ptr(assign), p,
                                   nbytes, _lib.stream_ptr()), "tree centres")
    return centres, assign


def tree_attention(q, k, v, *, leaf_size=64, fanout=16, opening_threshold=0.02, scale=None, return_lse=False,
                   return_info=False, centres=None, assign=None, marks=None):
    """The hierarchical operator on one head: q [N, 128], k / v [M, 128] (bfloat16 or float32, on the
    GPU).  Query centres: the k-means of `queries_centres` unless `centres` [C, 128] (scaled space) and
    `assign` [N] are given.  Returns out [N, 128] float32 (+ lse [N], + counters dict)."""
    if opening_threshold < 0:
        raise ValueError("opening_threshold must be nonnegative")
    if q.ndim != 2 or k.ndim != 2 or v.ndim != 2 or q.shape[1] != D_MAX or k.shape[1] != D_MAX or \
            v.shape[1] != D_MAX or k.shape[0] != v.shape[0] or k.shape[0] == 0:
        raise ValueError("q [N, 128], k and v [M, 128] expected")
    sc = 1.0 / math.sqrt(q.shape[1]) if scale is None else float(scale)
    dev = q.device
    kv_dtype = torch.bfloat16 if k.dtype == torch.bfloat16 else torch.float32
    qd, kd, vd = (x.to(dtype=kv_dtype).contiguous() for x in (q, k, v))
    if marks is not None:
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        marks.append(("begin", e))
    if centres is None:
        centres, assign = queries_centres(qd, sc)
    elif assign is None:
        raise ValueError("assign= is required with explicit centres")
    if marks is not None:
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        marks.append(("centres", e))
    forest = Forest(kd, vd, centres.to(device=dev, dtype=torch.float32).contiguous(), int(leaf_size), int(fanout),
                    D_MAX, D_MAX, dev)
    if marks is not None:
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        marks.append(("build", e))
    out, lse, cnt = _run(forest, qd, assign.to(device=dev, dtype=torch.int32).contiguous(), sc, opening_threshold,
                         marks=marks)
    res = [out]
    if return_lse:
        res.append(lse)
    if return_info:
        res.append({"visited_nodes": cnt[0], "accepted_nodes": cnt[1], "exact_leaves": cnt[2], "leaves": cnt[3],
                    "centres": centres, "assign": assign, "forest": forest})
    return res[0] if len(res) == 1 else tuple(res)
