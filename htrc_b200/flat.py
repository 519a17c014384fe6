"""Flat (tree-free) HTRC attention on B200: the host side of the operator.

Mirrors the call surface of the reference's h3/htrc_flat.py (``flat_attention``, ``PROD``,
``flat_attention_prod``) for its production path -- ``backend="triton", store="int8", dot="bf16",
select="max", curvature="lin"`` (htrc_flat.py:99-139, :181-276, :391-399) -- and runs it through the
C-ABI library libhtrc_flat.so (hand-written sm_100a kernels).  There is no other backend and no CPU
fallback: configurations the kernels do not implement raise ``NotImplementedError`` and argument
errors raise the reference's ``ValueError``s.

State format: ``store="int8"`` (the production path) or ``store="fp8"``: the reference's e4m3 far-field
state with per-(centre, leaf) row scales, fp16 far-field dots and a bf16 near field
(h3/htrc_flat_triton.py FP8=1), on its own sm_100a kernels.

Curvature: ``curvature="iso"`` with ``backend="cuda"`` (or "b200") adds the isotropic second-order far-field
term of the reference's torch backend (h3/htrc_flat.py:331-333) to the INT8 production path; the
reference's triton backend rejects it, and so does ``backend="triton"`` here.

Query order and groups: ``order="kmeans"`` (the accurate/max modes) reorders the queries on the device
by the reference's k-means permutation before tiling and writes the output back in the caller's order
(h3/htrc_flat.py:47-65, :146-147, :159-165); ``kern={"group": G}`` lets G consecutive tiles share one
expansion centre, far-field state and routing (:223-231).

Precision: ``precision="tf32"`` (PROD's setting) runs the leaf-statistics dots on tf32 operand values, the
float32 centre and softmax weights with their low 13 mantissa bits cleared, which is how the reference's
tensor-core dots read them on sm_100 (h3/htrc_flat_triton.py:57, :62-63); any other value runs them
float32-accurate (the reference's "ieee").  ``division="triton"`` (an addition; default "ieee") forms the query
and offset codes and the slope scaling with PTX div.full.f32, the instruction the reference's Triton kernels
use for their float32 ``/`` on the GPU: with PROD's precision the codes then match the reference's GPU
operator, while "ieee" matches its formula as written (and its CPU-recorded fixtures).

Additions over the reference: ``return_lse=True`` also returns the log-partition per query
(logit units, scale * q.k), ``backend`` accepts "cuda"/"b200" as names of the same path, and
``qk_scale_block=64`` gives the INT8 keys one scale per 64-key leaf and the query rows one per tile
(one absmax scale per 64-token block; the reference's are per key and per row, the default).
"""
from __future__ import annotations

import ctypes
import math
import time

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_ptr

DIM, TILE, LEAF = 128, 64, 64
LEAVES = (64, 32, 16)       # leaf sizes with kernels (32 and 16: INT8 state, linear far field)
TILES = (64, 32)          # query tile rows the kernels take (32: the "max" mode, held as 64 rows)

PROD = dict(tile=64, exact_leaves=256, tile_chunk=128, backend="triton", precision="tf32",
            store="int8", dot="bf16", splits=4, kern=dict(tile_warps=4, tile_bn=64, tile_stages=2))
"""The reference's production configuration (h3/htrc_flat.py:391-392).  The launch knobs in ``kern``
and ``splits`` are accepted and ignored: the kernels here have their own fixed shapes."""

_BACKENDS = ("triton", "cuda", "b200")


def leaf_pitch(nb: int) -> int:
    return int(lib().htrc_leaf_pitch(int(nb)))


class _Tick:
    """Stage timer with the reference's semantics (h3/htrc_flat.py:32-44): when ``prof`` is a dict,
    synchronise and accumulate milliseconds per stage name."""

    def __init__(self, prof):
        self.prof = prof
        if prof is not None:
            torch.cuda.synchronize()
            self.t = time.perf_counter()

    def __call__(self, name):
        if self.prof is not None:
            torch.cuda.synchronize()
            t = time.perf_counter()
            self.prof[name] = self.prof.get(name, 0.0) + 1e3 * (t - self.t)
            self.t = t


def _check_args(q, k, v, tile, exact_leaves, order, curvature, leaf, select, backend, store, dot,
                sel_stride, quant, sink_leaves, tail):
    """The reference's argument errors (h3/htrc_flat.py:118-132, :187-212), then what this library
    implements."""
    if backend not in _BACKENDS and backend != "torch":
        raise ValueError(f"unknown backend {backend}")
    if backend == "torch":
        if sink_leaves or tail is not None:
            raise ValueError("sink_leaves / tail are supported by the triton backend only")
        if select not in ("max", "bound"):
            raise ValueError("select must be max or bound")
        if order not in ("seq", "kmeans"):
            raise ValueError("order must be seq or kmeans")
        if curvature not in ("lin", "iso"):
            raise ValueError("curvature must be lin or iso")
        raise NotImplementedError("backend='torch' is the reference's float32 CPU specification; this library runs "
                                  "the sm_100a INT8 production path (pass **PROD, or backend='triton', store='int8', "
                                  "dot='bf16')")
    if curvature != "lin" and (backend == "triton" or curvature != "iso"):
        raise ValueError("triton backend needs curvature='lin'" if backend == "triton" else
                         "curvature must be lin or iso")
    m = int(k.shape[0])
    if m % leaf:
        raise ValueError("triton backend: key count must be a multiple of the leaf size")
    if dot == "bf16" and store not in ("bf16", "fp8", "int8"):
        raise ValueError("dot='bf16' needs store='bf16', 'fp8' or 'int8'")
    if store in ("fp8", "int8") and (dot != "bf16" or select == "bound" or (quant or {}).get("state")):
        raise ValueError("store='fp8' needs dot='bf16', select='max' and no state fake-quant")
    if store not in _lib.STORES or dot != "bf16":
        raise NotImplementedError("only the dot='bf16' paths with store='int8' (production), 'fp8' or 'bf16' are "
                                  "implemented")
    if store in ("fp8", "bf16") and curvature != "lin":
        raise NotImplementedError("curvature='iso' is implemented on the INT8 path only")
    if int(tile) not in TILES or int(leaf) not in LEAVES:
        raise NotImplementedError(f"the kernels implement tile=64 or 32 and leaf=64, 32 or 16 (got tile={tile}, "
                                  f"leaf={leaf})")
    if int(leaf) != LEAF and (store != "int8" or curvature != "lin"):
        raise NotImplementedError(f"leaf={leaf} is implemented for store='int8' with curvature='lin' (the fp8 "
                                  f"state and the iso term take leaf={LEAF})")
    if int(sel_stride) != 1:
        raise NotImplementedError("sel_stride != 1 is not implemented")
    for key in ("kv", "q"):
        if (quant or {}).get(key) and quant[key] not in _lib.FQ_FORMATS:
            raise ValueError(f"unknown quant format {quant[key]}")
    if q.dim() != 2 or k.dim() != 2 or v.dim() != 2 or int(q.shape[1]) != DIM or k.shape != v.shape or \
            int(k.shape[1]) != DIM:
        raise ValueError(f"q [N, {DIM}], k/v [M, {DIM}] expected")
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("q, k, v must be CUDA tensors (there is no CPU path)")


def _check_scale_block(qk_scale_block, store, leaf=LEAF):
    """qk_scale_block: None/0 (the reference's per-key and per-row INT8 scales) or 64 (one per leaf / tile)."""
    b = int(qk_scale_block or 0)
    if b not in (0, 64):
        raise ValueError("qk_scale_block must be None, 0 or 64")
    if b and store != "int8":
        raise NotImplementedError("qk_scale_block applies to the INT8 query and key codes (store='int8')")
    if b and int(leaf) != LEAF:
        raise NotImplementedError(f"qk_scale_block=64 gives one key scale per 64-key leaf (leaf={LEAF})")
    return b


def fake_quant(x, fmt, group=0, out_dtype=torch.float32):
    """Round-trip x [..., 128] (CUDA, f32 or bf16) through a low-bit format with symmetric per-group
    scales (group 0: one scale per row; fp4: 16) -- h3/htrc_flat.py:68-97, on the device.  fmt: int8,
    int4, fp8 (e4m3), fp4 (e2m1).  Returns float32 like the reference (or ``out_dtype``)."""
    if fmt not in _lib.FQ_FORMATS:
        raise ValueError(f"unknown quant format {fmt}")
    d = int(x.shape[-1])
    gsz = int(group) if group else (16 if fmt == "fp4" else d)
    if d % gsz:
        raise ValueError("quant group must divide the feature size")
    if not x.is_cuda:
        raise ValueError("fake_quant runs on the device (there is no CPU path)")
    xs = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
    xs = xs.reshape(-1, d).contiguous()
    out = torch.empty(xs.shape, dtype=out_dtype, device=x.device)
    dt = lambda t: _lib.DTYPE_BF16 if t == torch.bfloat16 else _lib.DTYPE_F32  # noqa: E731
    check(lib().htrc_fake_quant(ptr(xs), dt(xs.dtype), int(xs.shape[0]), d, _lib.FQ_FORMATS[fmt], int(group), ptr(out),
                                dt(out_dtype), stream_ptr()), "htrc_fake_quant")
    return out.reshape(x.shape)


def dequant_rows(x8, scale, out):
    """out[r, :] = x8[r, :] * scale[r] (fp8 e4m3 codes -> bf16), h3/htrc_flat_triton.py:287-294; x8 [rows, 128]
    and scale [rows] may be strided views, out [rows, 128] bf16 contiguous."""
    rows, d = int(x8.shape[0]), int(x8.shape[1])
    if x8.element_size() != 1 or x8.stride(1) != 1 or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("dequant_rows: x8 [rows, D] one-byte codes with unit column stride, out bf16 contiguous")
    sc = scale if scale.dtype == torch.float32 else scale.float()
    check(lib().htrc_dequant_rows(ptr(x8), int(x8.stride(0)), ptr(sc), int(sc.stride(0)), rows, d, ptr(out),
                                  stream_ptr()), "htrc_dequant_rows")
    return out


def _prep_inputs(q, k, v, tail, quant=None):
    """Device inputs of the kernels: q f32/bf16, k/v bf16.  With ``quant`` (kv / q formats and a group,
    h3/htrc_flat.py:190-195) k, v and q are fake-quantised first; the near field then sees the
    quantised keys rounded to bf16, as the reference's bf16 path does (its leaf statistics see them
    unrounded)."""
    quant = quant or {}
    qg = int(quant.get("group", 0))
    if quant.get("kv"):
        k = fake_quant(k, quant["kv"], qg, out_dtype=torch.bfloat16)
        v = fake_quant(v, quant["kv"], qg, out_dtype=torch.bfloat16)
    if quant.get("q"):
        q = fake_quant(q, quant["q"], qg)
    qd = q if q.dtype in (torch.float32, torch.bfloat16) else q.float()
    qd = qd.contiguous()
    kb = k.to(torch.bfloat16).contiguous()
    vb = v.to(torch.bfloat16).contiguous()
    tk = tv = None
    if tail is not None and tail[0] is not None and int(tail[0].shape[0]) > 0:
        tk = tail[0].float().contiguous()
        tv = tail[1].float().contiguous()
    return qd, kb, vb, tk, tv


def group_of(kern) -> int:
    """G consecutive tiles per centre: the reference's ``max(1, int(kern.get("group", 1)))``
    (h3/htrc_flat.py:223)."""
    return max(1, int((kern or {}).get("group", 1)))


def order_code(order) -> int:
    """The triton path permutes for order == "kmeans" and keeps the sequence otherwise
    (h3/htrc_flat.py:146)."""
    return _lib.ORDER_KMEANS if order == "kmeans" else _lib.ORDER_SEQ


def precision_code(precision, division="ieee") -> int:
    """The arithmetic flags of the C ABI: the reference maps precision == "tf32" to tf32 dots and anything else
    to IEEE float32 (h3/htrc_flat.py:126-130); division "triton" adds the reference's GPU division of the
    codes."""
    if division not in _lib.DIVISIONS:
        raise ValueError("division must be 'ieee' or 'triton'")
    return (_lib.PREC_TF32 if precision == "tf32" else _lib.PREC_FP32) | _lib.DIVISIONS[division]


def curvature_code(curvature) -> int:
    return _lib.CURV_ISO if curvature == "iso" else _lib.CURV_LIN


def _args(qd, kb, vb, tk, tv, exact_leaves, sink_leaves, tile_chunk, scale, out=None, lse=None, ws=None,
          stage_events=None, group=1, order=_lib.ORDER_SEQ, tile=TILE, curvature=_lib.CURV_LIN,
          store=_lib.STORE_INT8, qk_scale_block=0, route_mask=None, precision=_lib.PREC_TF32, leaf=LEAF):
    a = _lib.HtrcFlatArgs()
    a.q = ptr(qd)
    a.q_dtype = _lib.DTYPE_BF16 if qd.dtype == torch.bfloat16 else _lib.DTYPE_F32
    a.k, a.v = ptr(kb), ptr(vb)
    a.n_queries, a.n_keys = int(qd.shape[0]), int(kb.shape[0])
    a.dim, a.tile, a.leaf = DIM, int(tile), int(leaf)
    a.exact_leaves, a.sink_leaves = int(exact_leaves), int(sink_leaves)
    a.tile_chunk = int(tile_chunk) if tile_chunk else 0
    a.scale = float(scale) if scale is not None else 0.0
    a.tail_k, a.tail_v = ptr(tk), ptr(tv)
    a.n_tail = int(tk.shape[0]) if tk is not None else 0
    a.out, a.lse = ptr(out), ptr(lse)
    a.group, a.order, a.curvature, a.store = int(group), int(order), int(curvature), int(store)
    a.qk_scale_block = int(qk_scale_block or 0)
    a.route_mask = ptr(route_mask)
    a.precision = int(precision)
    if ws is not None:
        a.workspace, a.workspace_bytes = ptr(ws), int(ws.numel())
    if stage_events:
        handles = []
        for ev in stage_events:
            if ev.cuda_event == 0:          # torch creates CUDA events lazily: create it now
                ev.record()
            handles.append(ev.cuda_event)
        arr = (ctypes.c_void_p * len(handles))(*handles)
        a.stage_events = ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p))
        a.n_stage_events = len(handles)
        a._keep = arr
    return a


def workspace_bytes(n_queries, n_keys, exact_leaves, sink_leaves=0, tile_chunk=0, n_tail=0, group=1,
                    order=_lib.ORDER_SEQ, tile=TILE, curvature=_lib.CURV_LIN, store=_lib.STORE_INT8, leaf=LEAF) -> int:
    """Device workspace one forward call needs."""
    a = _lib.HtrcFlatArgs()
    a.n_queries, a.n_keys, a.dim, a.tile, a.leaf = int(n_queries), int(n_keys), DIM, int(tile), int(leaf)
    a.q_dtype = _lib.DTYPE_F32
    a.exact_leaves, a.sink_leaves = int(exact_leaves), int(sink_leaves)
    a.tile_chunk, a.n_tail = int(tile_chunk or 0), int(n_tail)
    a.group, a.order, a.curvature, a.store = int(group), int(order), int(curvature), int(store)
    nbytes = ctypes.c_size_t()
    check(lib().htrc_flat_workspace_size(a, nbytes), "workspace size")
    return int(nbytes.value)


def new_workspace(nbytes, device):
    """A device workspace of nbytes for ``forward_into``: its device status word (the first 256 bytes)
    starts at zero; the rest needs no initialisation."""
    w = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
    w[:256].zero_()
    return w


def _workspace(ws, nbytes, device):
    """A uint8 device buffer of at least nbytes, reused through the ``ws`` dict like the reference's
    workspace (h3/htrc_flat_triton.py:302-312)."""
    if ws is None:
        return new_workspace(nbytes, device)
    b = ws.get("workspace")
    if b is None or b.numel() < nbytes or b.device != device:
        b = new_workspace(nbytes, device)
        ws["workspace"] = b
    return b


def _check_buffers(qd, kb, vb, tk, tv, out, lse, workspace, route_mask, tile, group, leaf=LEAF):
    """Shapes, dtypes, contiguity and device of every buffer the C ABI will read or write, checked on the
    host before any launch (the library trusts its pointers and sizes)."""
    def need(t, name, shape, dtypes):
        if not isinstance(t, torch.Tensor) or tuple(t.shape) != tuple(shape) or t.dtype not in dtypes \
                or not t.is_contiguous():
            got = "None" if not isinstance(t, torch.Tensor) else \
                f"{tuple(t.shape)} {t.dtype}" + ("" if t.is_contiguous() else " non-contiguous")
            raise ValueError(f"{name}: a contiguous {'/'.join(str(d).split('.')[-1] for d in dtypes)} tensor "
                             f"{list(shape)} expected, got {got}")

    if qd is None or qd.dim() != 2:
        raise ValueError("qd: [N, 128] expected")
    n, m = int(qd.shape[0]), int(kb.shape[0]) if kb is not None and kb.dim() == 2 else -1
    need(qd, "qd", (n, DIM), (torch.float32, torch.bfloat16))
    need(kb, "kb", (m, DIM), (torch.bfloat16,))
    need(vb, "vb", (m, DIM), (torch.bfloat16,))
    need(out, "out", (n, DIM), (torch.float32,))
    if lse is not None:
        need(lse, "lse", (n,), (torch.float32,))
    if tk is not None or tv is not None:
        nt_ = int(tk.shape[0]) if tk is not None and tk.dim() == 2 else -1
        need(tk, "tk", (nt_, DIM), (torch.float32,))
        need(tv, "tv", (nt_, DIM), (torch.float32,))
    if workspace is None or workspace.dtype != torch.uint8 or not workspace.is_contiguous():
        raise ValueError("workspace: a contiguous uint8 tensor expected")
    if route_mask is not None:
        if route_mask.dtype != torch.uint8 or not route_mask.is_contiguous():
            raise ValueError("route_mask: a contiguous uint8 tensor [groups, leaf_pitch(nb)]")
        rows = -(-(-(-n // int(tile))) // max(1, int(group)))
        pitch = -(-(m // int(leaf)) // 16) * 16   # htrc_leaf_pitch: leaves rounded up to 16 (host-side)
        if route_mask.numel() < rows * pitch:
            raise ValueError(f"route_mask: at least {rows} x {pitch} bytes expected ([ceil(tiles / group), "
                             f"leaf_pitch(nb)]), got {route_mask.numel()}")
    devs = {t.device for t in (qd, kb, vb, out, lse, tk, tv, workspace, route_mask) if t is not None}
    if len(devs) != 1 or next(iter(devs)).type != "cuda":
        raise ValueError(f"every buffer must be on one CUDA device, got {sorted(str(d) for d in devs)}")


def forward_into(qd, kb, vb, tk, tv, *, exact_leaves, sink_leaves=0, tile_chunk=0, scale=None, out, lse=None,
                 workspace, stream=None, stage_events=None, group=1, order=_lib.ORDER_SEQ, tile=TILE,
                 curvature=_lib.CURV_LIN, store=_lib.STORE_INT8, qk_scale_block=0, route_mask=None,
                 precision=_lib.PREC_TF32, leaf=LEAF):
    """One head through ``htrc_flat_forward`` into caller-provided buffers (no allocation; CUDA-graph
    capturable).  qd [N, 128] f32/bf16, kb/vb [M, 128] bf16, out [N, 128] f32, lse [N] f32 or None;
    stage_events: optional list of torch.cuda.Event recorded between the stages (see
    include/htrc_flat.h); group / order: ``group_of(kern)`` / ``order_code(order)``; tile: 64 or 32;
    store: ``_lib.STORES[store]``; qk_scale_block: 0 or 64; route_mask: optional uint8
    [ceil(nt / group), leaf_pitch(nb)] device tensor that receives the routing masks (1 = leaf exact);
    precision: ``_lib.PREC_TF32`` (the production setting of PROD, the default) or ``_lib.PREC_FP32``;
    leaf: 64, 32 or 16 keys (32 and 16 with the INT8 state and the linear far field)."""
    _check_buffers(qd, kb, vb, tk, tv, out, lse, workspace, route_mask, tile, group, leaf)
    a = _args(qd, kb, vb, tk, tv, exact_leaves, sink_leaves, tile_chunk, scale, out, lse, workspace, stage_events,
              group, order, tile, curvature, store, qk_scale_block, route_mask, precision, leaf)
    check(lib().htrc_flat_forward(a, stream_ptr(stream)), "htrc_flat_forward")


def device_status(workspace, stream=None) -> int:
    """Read and clear the device status word; raises if any failure bit is set."""
    st = ctypes.c_int32(0)
    check(lib().htrc_flat_status(ptr(workspace), st, stream_ptr(stream)), "htrc_flat_status")
    if st.value:
        bits = [name for b, name in _lib.STATUS_BITS.items() if st.value & b]
        other = st.value & ~sum(_lib.STATUS_BITS)
        if other:
            bits.append(f"unknown bits {other:#x} (a workspace whose status word was not zeroed?)")
        raise _lib.HtrcError("device status: " + ", ".join(bits))
    return 0


@torch.inference_mode()
def flat_attention(q, k, v, *, tile=64, exact_leaves=64, order="seq", curvature="lin",
                   tile_chunk=32, precision="fp32", leaf=16, scale=None, prof=None,
                   select="max", backend="torch", store="fp32", splits=8, dot="tf32",
                   sel_stride=1, kern=None, quant=None, sink_leaves=0, tail=None, ws=None,
                   return_lse=False, qk_scale_block=None, division="ieee"):
    """q [N, 128], k/v [M, 128] on a CUDA device -> out [N, 128] float32 (and lse [N] with
    return_lse).  Signature and defaults of the reference (h3/htrc_flat.py:99-103); see PROD."""
    _check_args(q, k, v, tile, exact_leaves, order, curvature, leaf, select, backend, store, dot,
                sel_stride, quant, sink_leaves, tail)
    qsb = _check_scale_block(qk_scale_block, store, leaf)
    qd, kb, vb, tk, tv = _prep_inputs(q, k, v, tail, quant)
    grp, oc, cc, sc = group_of(kern), order_code(order), curvature_code(curvature), _lib.STORES[store]
    pc = precision_code(precision, division)
    if prof is not None:
        st = run_stages(qd, kb, vb, tk, tv, exact_leaves=exact_leaves, sink_leaves=sink_leaves,
                        tile_chunk=tile_chunk, scale=scale, prof=prof, group=grp, order=oc, tile=tile, curvature=cc,
                        store=sc, qk_scale_block=qsb, precision=pc, leaf=leaf)
        return (st["out"], st["lse"]) if return_lse else st["out"]
    n = int(qd.shape[0])
    out = torch.empty((n, DIM), dtype=torch.float32, device=q.device)
    lse = torch.empty((n,), dtype=torch.float32, device=q.device) if return_lse else None
    nbytes = workspace_bytes(n, int(kb.shape[0]), exact_leaves, sink_leaves, tile_chunk,
                             int(tk.shape[0]) if tk is not None else 0, grp, oc, tile, cc, sc, leaf)
    w = _workspace(ws, nbytes, q.device)
    forward_into(qd, kb, vb, tk, tv, exact_leaves=exact_leaves, sink_leaves=sink_leaves,
                 tile_chunk=tile_chunk, scale=scale, out=out, lse=lse, workspace=w, group=grp, order=oc, tile=tile,
                 curvature=cc, store=sc, qk_scale_block=qsb, precision=pc, leaf=leaf)
    return (out, lse) if return_lse else out


def flat_attention_prod(q, k, v, **over):
    """Production configuration of the flat operator (h3/htrc_flat.py:397-399)."""
    return flat_attention(q, k, v, **{**PROD, **over})


@torch.inference_mode()
def flat_attention_heads(q, k, v, *, return_lse=False, ws=None, **cfg):
    """Head-batched entry (an addition): q [H, N, 128], k/v [H, M, 128] -> out [H, N, 128] float32 (and lse
    [H, N] with return_lse), every head with ``flat_attention(**cfg)`` semantics (the same defaults), on one
    device workspace, launched back to back on the current stream."""
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3 or q.shape[0] != k.shape[0] or k.shape != v.shape:
        raise ValueError("q [H, N, D], k/v [H, M, D] expected")
    h, n = int(q.shape[0]), int(q.shape[1])
    c = {**dict(tile=64, exact_leaves=64, order="seq", curvature="lin", tile_chunk=32, leaf=16, select="max",
                backend="torch", store="fp32", dot="tf32", sel_stride=1, kern=None, quant=None, sink_leaves=0,
                tail=None, scale=None, qk_scale_block=None, precision="fp32", division="ieee"), **cfg}
    _check_args(q[0], k[0], v[0], c["tile"], c["exact_leaves"], c["order"], c["curvature"], c["leaf"], c["select"],
                c["backend"], c["store"], c["dot"], c["sel_stride"], c["quant"], c["sink_leaves"], c["tail"])
    qsb = _check_scale_block(c["qk_scale_block"], c["store"], c["leaf"])
    out = torch.empty((h, n, DIM), dtype=torch.float32, device=q.device)
    lse = torch.empty((h, n), dtype=torch.float32, device=q.device) if return_lse else None
    grp, oc, cc = group_of(c["kern"]), order_code(c["order"]), curvature_code(c["curvature"])
    sc = _lib.STORES[c["store"]]
    w = None
    for i in range(h):
        qd, kb, vb, tk, tv = _prep_inputs(q[i], k[i], v[i], c["tail"], c["quant"])
        if w is None:
            nbytes = workspace_bytes(n, int(kb.shape[0]), c["exact_leaves"], c["sink_leaves"], c["tile_chunk"],
                                     int(tk.shape[0]) if tk is not None else 0, grp, oc, c["tile"], cc, sc,
                                     c["leaf"])
            w = _workspace(ws, nbytes, q.device)
        forward_into(qd, kb, vb, tk, tv, exact_leaves=c["exact_leaves"], sink_leaves=c["sink_leaves"],
                     tile_chunk=c["tile_chunk"], scale=c["scale"], out=out[i], lse=lse[i] if return_lse else None,
                     workspace=w, group=grp, order=oc, tile=c["tile"], curvature=cc, store=sc, qk_scale_block=qsb,
                     precision=precision_code(c["precision"], c["division"]), leaf=c["leaf"])
    return (out, lse) if return_lse else out


@torch.inference_mode()
def run_stages(qd, kb, vb, tk=None, tv=None, *, exact_leaves, sink_leaves=0, tile_chunk=0, scale=None,
               prof=None, stream=None, group=1, order=_lib.ORDER_SEQ, tile=TILE, curvature=_lib.CURV_LIN,
               store=_lib.STORE_INT8, qk_scale_block=0, precision=_lib.PREC_TF32, leaf=LEAF):
    """The same operator launched stage by stage through the C ABI's stage entry points, returning
    every intermediate (perm, k8, ks, mu, q8, sq, dq8, sdq, g8, sg, lz, vb, sel, idx, excl, out, lse; with
    store=STORE_FP8: perm, mu, qb, dqh, g8 / vb8 e4m3 codes, sg, sv, lz, sel, idx, excl, out, lse).
    Used for stage timing (``prof``, the reference's stage names prep/stats/select/tile/finish) and
    for per-stage parity tests.  The state of all centre rows is kept (tile_chunk only sets the launch
    granularity of the state stages, in groups of ``group`` tiles)."""
    L = lib()
    dev = qd.device
    s = stream_ptr(stream)
    tick = _Tick(prof)
    n, m = int(qd.shape[0]), int(kb.shape[0])
    tile = int(tile)
    nt, nb = -(-n // tile), m // int(leaf)
    grp = max(1, int(group))
    ng = -(-nt // grp)
    pitch = leaf_pitch(nb)
    sink = max(0, min(int(sink_leaves), nb))
    kx = min(int(exact_leaves) + sink, nb)
    sc = 1.0 / math.sqrt(DIM) if scale is None else float(scale)
    qdt = _lib.DTYPE_BF16 if qd.dtype == torch.bfloat16 else _lib.DTYPE_F32
    e = lambda *shape, dt=torch.float32: torch.empty(shape, dtype=dt, device=dev)  # noqa: E731
    if int(leaf) not in LEAVES or (int(leaf) != LEAF and (store != _lib.STORE_INT8 or curvature != _lib.CURV_LIN
                                                            or qk_scale_block)):
        raise NotImplementedError(f"leaf={leaf}: leaves of 64, or 32 / 16 with the INT8 state and the linear far field")
    if store in (_lib.STORE_FP8, _lib.STORE_BF16):
        if curvature != _lib.CURV_LIN:
            raise NotImplementedError("curvature='iso' is implemented on the INT8 path only")
        return _run_stages_fp8(qd, kb, vb, tk, tv, n=n, m=m, nt=nt, nb=nb, ng=ng, grp=grp, pitch=pitch, sink=sink,
                               kx=kx, sc=sc, qdt=qdt, tile=tile, tile_chunk=tile_chunk, exact_leaves=exact_leaves,
                               order=order, s=s, tick=tick, e=e, precision=int(precision),
                               bf16=store == _lib.STORE_BF16)
    r = dict(k8=e(m, DIM, dt=torch.int8), ks=e(m), mu=e(ng, DIM), mu_hi=e(ng, DIM, dt=torch.bfloat16),
             mu_lo=e(ng, DIM, dt=torch.bfloat16), q8=e(nt * TILE, DIM, dt=torch.int8), sq=e(nt * TILE),
             dq8=e(nt * TILE, DIM, dt=torch.int8), sdq=e(nt * TILE), g8=e(ng, nb, DIM, dt=torch.int8),
             sg=e(ng, pitch), lz=e(ng, pitch), vb=e(ng, nb, DIM, dt=torch.bfloat16), sel=torch.zeros((nt, pitch),
             dtype=torch.float32, device=dev), idx=e(ng, max(kx, 1), dt=torch.int32),
             excl=e(ng, pitch, dt=torch.uint8), out=e(n, DIM), lse=e(n),
             status=torch.zeros((1,), dtype=torch.int32, device=dev), perm=None)
    iso = curvature == _lib.CURV_ISO
    r.update(kn2=e(m) if iso else None, dd=e(nt * TILE) if iso else None, cv=e(ng, pitch) if iso else None)
    stp = ptr(r["status"])
    if qk_scale_block:
        check(L.htrc_pack_int8_blocks(ptr(kb), _lib.DTYPE_BF16, m, DIM, _lib.ROUND_HALF_EVEN, int(qk_scale_block),
                                      ptr(r["k8"]), ptr(r["ks"]), ptr(r["kn2"]), s), "htrc_pack_int8_blocks")
    else:
        check(L.htrc_pack_int8(ptr(kb), _lib.DTYPE_BF16, m, DIM, _lib.ROUND_HALF_EVEN, ptr(r["k8"]), ptr(r["ks"]),
                               ptr(r["kn2"]), s), "htrc_pack_int8")
    if order == _lib.ORDER_KMEANS:
        r["perm"] = e(n, dt=torch.int32)
        nbytes = ctypes.c_size_t()
        check(L.htrc_kmeans_scratch_size(n, nbytes), "htrc_kmeans_scratch_size")
        scratch = torch.empty(int(nbytes.value), dtype=torch.uint8, device=dev)
        check(L.htrc_kmeans_order(ptr(qd), qdt, n, DIM, ptr(r["perm"]), ptr(scratch), int(nbytes.value), s),
              "htrc_kmeans_order")
    perm = ptr(r["perm"])
    check(L.htrc_tile_prep_ex(ptr(qd), qdt, n, DIM, tile, perm, grp, ptr(r["mu"]), ptr(r["mu_hi"]), ptr(r["mu_lo"]),
                              ptr(r["q8"]), ptr(r["sq"]), ptr(r["dq8"]), ptr(r["sdq"]), ptr(r["dd"]),
                              int(qk_scale_block or 0), int(precision), s), "htrc_tile_prep_ex")
    tail_part = None
    if tk is not None:
        tail_part = e(n, DIM + 2)
        check(L.htrc_tail_partial(ptr(qd), qdt, n, DIM, ptr(tk), ptr(tv), int(tk.shape[0]), sc, ptr(tail_part), s),
              "htrc_tail_partial")
    tick("prep")
    gstep = ng if not tile_chunk or tile_chunk <= 0 else min(max(1, int(tile_chunk) // grp), ng)
    far = kx < nb
    if far:
        for g0 in range(0, ng, gstep):
            gc = min(gstep, ng - g0)
            check(L.htrc_leaf_stats(ptr(r["mu_hi"]), ptr(r["mu_lo"]), ng, g0, gc, ptr(kb), ptr(vb), m, DIM, int(leaf), sc,
                                    ptr(r["g8"][g0]), ptr(r["sg"][g0]), ptr(r["lz"][g0]), ptr(r["vb"][g0]),
                                    ptr(r["kn2"]), ptr(r["cv"][g0]) if iso else None, int(precision), stp, s),
                  "htrc_leaf_stats")
    tick("stats")
    if far and kx > 0:
        check(L.htrc_rowmax_select(ptr(r["dq8"]), ptr(r["sdq"]), ptr(r["dd"]), 0, nt, grp, ptr(r["g8"]), ptr(r["sg"]),
                                   ptr(r["lz"]), ptr(r["cv"]), nb, DIM, ptr(r["sel"]), stp, s), "htrc_rowmax_select")
    check(L.htrc_route(ptr(r["sel"]), nt, nb, int(exact_leaves), sink, grp, ptr(r["idx"]), ptr(r["excl"]), s),
          "htrc_route")
    tick("select")
    check(L.htrc_tile_attention(ptr(r["q8"]), ptr(r["sq"]), ptr(r["dq8"]), ptr(r["sdq"]), n, tile, 0, nt, grp,
                                ptr(r["g8"]),
                                ptr(r["sg"]), ptr(r["lz"]), ptr(r["vb"]), ptr(r["excl"]), ptr(r["idx"]), kx, nb,
                                ptr(r["k8"]), ptr(r["ks"]), ptr(vb), m, DIM, int(leaf), sc, ptr(tail_part), perm,
                                ptr(r["cv"]), ptr(r["dd"]), ptr(r["out"]), ptr(r["lse"]), stp, s), "htrc_tile_attention")
    tick("tile")
    tick("finish")
    r["kx"], r["nb"], r["pitch"], r["group"], r["tile"], r["leaf"] = kx, nb, pitch, grp, tile, int(leaf)
    return r


def _run_stages_fp8(qd, kb, vb, tk, tv, *, n, m, nt, nb, ng, grp, pitch, sink, kx, sc, qdt, tile, tile_chunk,
                    exact_leaves, order, s, tick, e, precision, bf16=False):
    """run_stages for the fp8 state (store="fp8"): tile prep with bf16 rows and fp16 offsets, e4m3 leaf
    statistics, fp8 row-max selection, routing and the fp8 tile kernel.  bf16=True: the bf16 state
    (store="bf16"): bf16 offsets (key "dqh" holds bf16 then), bf16 g / vbar values in "g8" / "vb8" (uint16
    bit patterns viewed as bfloat16), no scales."""
    if bf16:
        return _run_stages_bf16(qd, kb, vb, tk, tv, n=n, m=m, nt=nt, nb=nb, ng=ng, grp=grp, pitch=pitch, sink=sink,
                                kx=kx, sc=sc, qdt=qdt, tile=tile, tile_chunk=tile_chunk, exact_leaves=exact_leaves,
                                order=order, s=s, tick=tick, e=e, precision=precision)
    L = lib()
    dev = qd.device
    r = dict(mu=e(ng, DIM), mu_hi=e(ng, DIM, dt=torch.bfloat16), mu_lo=e(ng, DIM, dt=torch.bfloat16),
             qb=e(nt * TILE, DIM, dt=torch.bfloat16), dqh=e(nt * TILE, DIM, dt=torch.float16),
             g8=e(ng, nb, DIM, dt=torch.uint8), vb8=e(ng, nb, DIM, dt=torch.uint8), sg=e(ng, pitch), sv=e(ng, pitch),
             lz=e(ng, pitch), sel=torch.zeros((nt, pitch), dtype=torch.float32, device=dev),
             idx=e(ng, max(kx, 1), dt=torch.int32), excl=e(ng, pitch, dt=torch.uint8), out=e(n, DIM), lse=e(n),
             status=torch.zeros((1,), dtype=torch.int32, device=dev), perm=None)
    stp = ptr(r["status"])
    if order == _lib.ORDER_KMEANS:
        r["perm"] = e(n, dt=torch.int32)
        nbytes = ctypes.c_size_t()
        check(L.htrc_kmeans_scratch_size(n, nbytes), "htrc_kmeans_scratch_size")
        scratch = torch.empty(int(nbytes.value), dtype=torch.uint8, device=dev)
        check(L.htrc_kmeans_order(ptr(qd), qdt, n, DIM, ptr(r["perm"]), ptr(scratch), int(nbytes.value), s),
              "htrc_kmeans_order")
    perm = ptr(r["perm"])
    check(L.htrc_tile_prep_fp8(ptr(qd), qdt, n, DIM, tile, perm, grp, ptr(r["mu"]), ptr(r["mu_hi"]), ptr(r["mu_lo"]),
                               ptr(r["qb"]), ptr(r["dqh"]), precision, s), "htrc_tile_prep_fp8")
    tail_part = None
    if tk is not None:
        tail_part = e(n, DIM + 2)
        check(L.htrc_tail_partial(ptr(qd), qdt, n, DIM, ptr(tk), ptr(tv), int(tk.shape[0]), sc, ptr(tail_part), s),
              "htrc_tail_partial")
    tick("prep")
    gstep = ng if not tile_chunk or tile_chunk <= 0 else min(max(1, int(tile_chunk) // grp), ng)
    far = kx < nb
    if far:
        for g0 in range(0, ng, gstep):
            gc = min(gstep, ng - g0)
            check(L.htrc_leaf_stats_fp8(ptr(r["mu_hi"]), ptr(r["mu_lo"]), ng, g0, gc, ptr(kb), ptr(vb), m, DIM, LEAF,
                                        sc, ptr(r["g8"][g0]), ptr(r["sg"][g0]), ptr(r["lz"][g0]), ptr(r["vb8"][g0]),
                                        ptr(r["sv"][g0]), precision, stp, s), "htrc_leaf_stats_fp8")
    tick("stats")
    if far and kx > 0:
        check(L.htrc_rowmax_select_fp8(ptr(r["dqh"]), 0, nt, grp, ptr(r["g8"]), ptr(r["sg"]), ptr(r["lz"]), nb, DIM,
                                       ptr(r["sel"]), stp, s), "htrc_rowmax_select_fp8")
    check(L.htrc_route(ptr(r["sel"]), nt, nb, int(exact_leaves), sink, grp, ptr(r["idx"]), ptr(r["excl"]), s),
          "htrc_route")
    tick("select")
    r["far_part"] = e(n, DIM + 2) if far else None
    check(L.htrc_tile_attention_fp8(ptr(r["qb"]), ptr(r["dqh"]), n, tile, 0, nt, grp, ptr(r["g8"]), ptr(r["sg"]),
                                    ptr(r["lz"]), ptr(r["vb8"]), ptr(r["sv"]), ptr(r["excl"]), ptr(r["idx"]), kx, nb,
                                    ptr(kb), ptr(vb), m, DIM, LEAF, sc, ptr(tail_part), perm, ptr(r["far_part"]),
                                    ptr(r["out"]), ptr(r["lse"]), stp, s), "htrc_tile_attention_fp8")
    tick("tile")
    tick("finish")
    r["kx"], r["nb"], r["pitch"], r["group"], r["tile"], r["leaf"] = kx, nb, pitch, grp, tile, LEAF
    return r


def _run_stages_bf16(qd, kb, vb, tk, tv, *, n, m, nt, nb, ng, grp, pitch, sink, kx, sc, qdt, tile, tile_chunk,
                     exact_leaves, order, s, tick, e, precision):
    """run_stages for the bf16 state (store="bf16"): tile prep with bf16 rows and bf16 offsets, bf16 leaf
    statistics (no scales), bf16 row-max selection, routing and the bf16-state tile kernel.  Keys: qb, dqb, gb,
    vbb (bfloat16), lz, sel, idx, excl, out, lse."""
    L = lib()
    dev = qd.device
    r = dict(mu=e(ng, DIM), mu_hi=e(ng, DIM, dt=torch.bfloat16), mu_lo=e(ng, DIM, dt=torch.bfloat16),
             qb=e(nt * TILE, DIM, dt=torch.bfloat16), dqb=e(nt * TILE, DIM, dt=torch.bfloat16),
             gb=e(ng, nb, DIM, dt=torch.bfloat16), vbb=e(ng, nb, DIM, dt=torch.bfloat16),
             lz=e(ng, pitch), sel=torch.zeros((nt, pitch), dtype=torch.float32, device=dev),
             idx=e(ng, max(kx, 1), dt=torch.int32), excl=e(ng, pitch, dt=torch.uint8), out=e(n, DIM), lse=e(n),
             status=torch.zeros((1,), dtype=torch.int32, device=dev), perm=None)
    stp = ptr(r["status"])
    if order == _lib.ORDER_KMEANS:
        r["perm"] = e(n, dt=torch.int32)
        nbytes = ctypes.c_size_t()
        check(L.htrc_kmeans_scratch_size(n, nbytes), "htrc_kmeans_scratch_size")
        scratch = torch.empty(int(nbytes.value), dtype=torch.uint8, device=dev)
        check(L.htrc_kmeans_order(ptr(qd), qdt, n, DIM, ptr(r["perm"]), ptr(scratch), int(nbytes.value), s),
              "htrc_kmeans_order")
    perm = ptr(r["perm"])
    check(L.htrc_tile_prep_bf16(ptr(qd), qdt, n, DIM, tile, perm, grp, ptr(r["mu"]), ptr(r["mu_hi"]), ptr(r["mu_lo"]),
                                ptr(r["qb"]), ptr(r["dqb"]), precision, s), "htrc_tile_prep_bf16")
    tail_part = None
    if tk is not None:
        tail_part = e(n, DIM + 2)
        check(L.htrc_tail_partial(ptr(qd), qdt, n, DIM, ptr(tk), ptr(tv), int(tk.shape[0]), sc, ptr(tail_part), s),
              "htrc_tail_partial")
    tick("prep")
    gstep = ng if not tile_chunk or tile_chunk <= 0 else min(max(1, int(tile_chunk) // grp), ng)
    far = kx < nb
    if far:
        for g0 in range(0, ng, gstep):
            gc = min(gstep, ng - g0)
            check(L.htrc_leaf_stats_bf16(ptr(r["mu_hi"]), ptr(r["mu_lo"]), ng, g0, gc, ptr(kb), ptr(vb), m, DIM, LEAF,
                                         sc, ptr(r["gb"][g0]), ptr(r["lz"][g0]), ptr(r["vbb"][g0]), precision, stp, s),
                  "htrc_leaf_stats_bf16")
    tick("stats")
    if far and kx > 0:
        check(L.htrc_rowmax_select_bf16(ptr(r["dqb"]), 0, nt, grp, ptr(r["gb"]), ptr(r["lz"]), nb, DIM,
                                        ptr(r["sel"]), stp, s), "htrc_rowmax_select_bf16")
    check(L.htrc_route(ptr(r["sel"]), nt, nb, int(exact_leaves), sink, grp, ptr(r["idx"]), ptr(r["excl"]), s),
          "htrc_route")
    tick("select")
    r["far_part"] = e(n, DIM + 2) if far else None
    check(L.htrc_tile_attention_bf16(ptr(r["qb"]), ptr(r["dqb"]), n, tile, 0, nt, grp, ptr(r["gb"]), ptr(r["lz"]),
                                     ptr(r["vbb"]), ptr(r["excl"]), ptr(r["idx"]), kx, nb, ptr(kb), ptr(vb), m, DIM,
                                     LEAF, sc, ptr(tail_part), perm, ptr(r["far_part"]), ptr(r["out"]), ptr(r["lse"]),
                                     stp, s), "htrc_tile_attention_bf16")
    tick("tile")
    tick("finish")
    r["kx"], r["nb"], r["pitch"], r["group"], r["tile"], r["leaf"] = kx, nb, pitch, grp, tile, LEAF
    return r
