"""Generate the golden fixtures of the flat HTRC production path by running the REFERENCE itself.

Run once, in a container that has the reference checkout, naming its directory with ``HTRC_REFERENCE``
or ``--reference``:

    TRITON_INTERPRET=1 python tests/golden/make_golden.py --reference <checkout> [case ...]

It imports the reference's ``h3/htrc_flat.py`` unmodified and calls
``flat_attention(q, k, v, **PROD, leaf=L, exact_leaves=E, ...)`` on CPU tensors with Triton's
interpreter, recording every stage the reference passes between its kernels (the INT8 keys, the
leaf state g8/sg/lz/vbar, the row-max selection, the exclusion mask, the split partials and the
output).  The fixtures are written as ``tests/golden/<case>.npz`` and are the only thing the tests
read; the reference is never needed at test time.

Triton 3.6's interpreter has two defects on this path, fixed here by a harness-side shim (the
reference is not modified):
  1. ``create_dot`` multiplies bfloat16 operands as their raw uint16 bit patterns -> the shim widens
     bfloat16 operands to float32 before the product;
  2. float32 -> bfloat16, float16 and float8 (e4m3) casts truncate -> the shim rounds to nearest even
     (float8 saturating at +-448), as the GPU does.
The interpreter also evaluates ``tl.dot(..., input_precision="tf32")`` in float32 and ``/`` as
IEEE division; the fixtures therefore pin the reference's arithmetic at float32 precision.
"""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from htrc_b200 import synth  # noqa: E402


def _shim():
    from triton.runtime import interpreter as itp
    import triton.language as tl

    B = itp.InterpreterBuilder
    orig_dot = B.create_dot
    orig_cast = B.cast_impl
    orig_fp2fp = B.create_fp_to_fp

    def widen(h):
        if h.dtype.scalar == tl.bfloat16:
            data = (h.data.astype(np.uint32) << 16).view(np.float32)
            return itp.TensorHandle(data, tl.float32)
        return h

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        return orig_dot(self, widen(a), widen(b), d, input_precision, max_num_imprecise_acc)

    def to_bf16(src, dst_type):
        x = np.ascontiguousarray(src.data, dtype=np.float32).view(np.uint32).astype(np.uint64)
        bits = ((x + 0x7FFF + ((x >> 16) & 1)) >> 16).astype(np.uint16)
        return itp.TensorHandle(bits, dst_type.scalar)

    def to_f16(src, dst_type):
        x = np.ascontiguousarray(src.data, dtype=np.float32)
        return itp.TensorHandle(x.astype(np.float16), dst_type.scalar)      # numpy rounds to nearest even

    def to_e4m3(src, dst_type):
        # nearest-even e4m3fn with saturation at +-448 (the GPU's cvt.rn.satfinite), as code bytes
        x = np.ascontiguousarray(src.data, dtype=np.float32).astype(np.float64)
        a = np.minimum(np.abs(x), 448.0)
        e = np.floor(np.log2(np.maximum(a, 2.0 ** -9)))
        quantum = np.where(a < 2.0 ** -6, 2.0 ** -9, 2.0 ** (e - 3))
        r = np.minimum(np.rint(a / quantum) * quantum, 448.0)
        sub = r < 2.0 ** -6
        er = np.floor(np.log2(np.maximum(r, 2.0 ** -6)))
        code = np.where(sub, np.rint(r / 2.0 ** -9), (er + 7) * 8 + np.rint((r / 2.0 ** er - 1.0) * 8))
        sign = np.signbit(x).astype(np.uint8) << 7
        return itp.TensorHandle((code.astype(np.uint8) | sign).astype(np.uint8), dst_type.scalar)

    def narrow(src, dst_type):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            return to_bf16(src, dst_type)
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.float16:
            return to_f16(src, dst_type)
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.float8e4nv:
            return to_e4m3(src, dst_type)
        return None

    def cast_impl(self, src, dst_type):
        r = narrow(src, dst_type)
        return r if r is not None else orig_cast(self, src, dst_type)

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        r = narrow(src, dst_type)
        return r if r is not None else orig_fp2fp(self, src, dst_type, rounding_mode)

    B.create_dot = create_dot
    B.cast_impl = cast_impl
    B.create_fp_to_fp = create_fp_to_fp


def _reference_dir(argv):
    """The reference checkout: ``--reference DIR`` on the command line, else $HTRC_REFERENCE (required)."""
    if "--reference" in argv:
        i = argv.index("--reference")
        return Path(argv[i + 1]), argv[:i] + argv[i + 2:]
    env = os.environ.get("HTRC_REFERENCE")
    if not env:
        raise SystemExit("name the reference checkout: --reference DIR or HTRC_REFERENCE=DIR")
    return Path(env), argv


def _load_reference(ref):
    spec = importlib.util.spec_from_file_location("_ref_htrc_flat", ref / "h3" / "htrc_flat.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["_ref_htrc_flat"] = mod
    spec.loader.exec_module(mod)
    return mod


def _recorder(flat):
    """Wrap the reference's kernel wrappers (and its k-means order) to record what flows between them."""
    tri = flat._load_triton()
    rec = {"stats": [], "sel": [], "tile": [], "perm": []}
    o_km = flat.kmeans_order

    def kmeans_order(q, *a, **kw):
        perm = o_km(q, *a, **kw)
        rec["perm"].append(perm.clone())
        return perm

    flat.kmeans_order = kmeans_order
    o_stats, o_sel, o_tile = tri.leaf_stats, tri.rowmax_select, tri.tile_attention

    def leaf_stats(mu, kf, vf, nb, scale, **kw):
        g, lz, vb, sg, sv = o_stats(mu, kf, vf, nb, scale, **kw)
        ent = dict(mu=mu.clone(), g8=g.clone(), lz=lz.clone(), vb=vb.clone())
        if sg is not None:                         # int8 / fp8 store: slope row scales (bf16: none)
            ent["sg"] = sg.clone()
        if sv is not None:                         # fp8 store: value row scales too
            ent["sv"] = sv.clone()
        rec["stats"].append(ent)
        return g, lz, vb, sg, sv

    def rowmax_select(*a, **kw):
        sel = o_sel(*a, **kw)
        rec["sel"].append(sel.clone())
        return sel

    def tile_attention(q_c, mu_c, g, lz, vb, excl, idx, k_ex, v_ex, scale, **kw):
        ws = kw.get("ws")
        res = o_tile(q_c, mu_c, g, lz, vb, excl, idx, k_ex, v_ex, scale, **kw)
        ent = dict(q_c=q_c.clone(), excl=excl.clone(), k8=k_ex.clone(), out=res.clone())
        if kw.get("ks") is not None:
            ent["ks"] = kw["ks"].clone()
        if idx is not None:
            ent["idx"] = idx.clone()
        if ws is not None:
            ent["pm"], ent["pl"] = ws["pm"][: q_c.shape[0]].clone(), ws["pl"][: q_c.shape[0]].clone()
        rec["tile"].append(ent)
        return res

    tri.leaf_stats, tri.rowmax_select, tri.tile_attention = leaf_stats, rowmax_select, tile_attention
    return rec


def _cat(lst, key):
    return torch.cat([e[key] for e in lst], 0)


CASES = [
    # name, grid (t,h,w) or (n, m) low-rank, leaf, exact_leaves, sink, tail rows, n_query_trim
    dict(name="base", grid=(2, 16, 16), leaf=64, E=2, sink=0, tail=0, trim=0, seed=11),
    dict(name="ragged", grid=(2, 16, 16), leaf=64, E=3, sink=0, tail=0, trim=37, seed=12),
    dict(name="sink_tail", grid=(2, 16, 16), leaf=64, E=2, sink=1, tail=5, trim=0, seed=13),
    dict(name="all_exact", grid=(2, 16, 16), leaf=64, E=8, sink=0, tail=0, trim=0, seed=14),
    dict(name="no_exact", grid=(2, 16, 16), leaf=64, E=0, sink=0, tail=0, trim=0, seed=15),
    dict(name="big_tail", grid=(2, 16, 16), leaf=64, E=2, sink=0, tail=20, trim=0, seed=16),
    dict(name="leaf32", grid=(2, 16, 16), leaf=32, E=4, sink=0, tail=0, trim=0, seed=17),
    dict(name="wide", grid=(4, 16, 32), leaf=64, E=4, sink=0, tail=0, trim=0, seed=18),
    # groups of tiles sharing one centre (kern group) and the k-means query order (order="kmeans")
    dict(name="group2", grid=(2, 16, 16), leaf=64, E=2, sink=0, tail=0, trim=37, seed=19, group=2),
    dict(name="group4", grid=(2, 16, 20), leaf=64, E=2, sink=1, tail=0, trim=0, seed=20, group=4),
    dict(name="kmeans", grid=(2, 16, 16), leaf=64, E=2, sink=0, tail=0, trim=21, seed=21, order="kmeans"),
    dict(name="kmeans_g2_tail", grid=(2, 16, 16), leaf=64, E=2, sink=0, tail=5, trim=0, seed=22, order="kmeans",
         group=2),
    dict(name="kmeans_sampled", grid=(4, 32, 33), leaf=64, E=4, sink=0, tail=0, trim=67, seed=23, order="kmeans",
         slim=True, keys=1024),
    # 32-row tiles (the "max" mode: k-means order, tile 32)
    dict(name="tile32", grid=(2, 16, 16), leaf=64, E=2, sink=1, tail=5, trim=19, seed=24, tile=32),
    dict(name="max_mode", grid=(2, 16, 16), leaf=64, E=3, sink=0, tail=0, trim=0, seed=25, tile=32, order="kmeans"),
    dict(name="tile32_g2", grid=(2, 16, 16), leaf=64, E=2, sink=0, tail=0, trim=45, seed=26, tile=32, group=2),
    # low-bit simulation of the inputs (quant=): k/v int4 and q int8 with groups of 32
    dict(name="quant_kv_q", grid=(2, 16, 16), leaf=64, E=2, sink=0, tail=0, trim=0, seed=27,
         quant={"kv": "int4", "q": "int8", "group": 32}),
    # the fp8 (e4m3) leaf state with row scales (store="fp8"): fp16 far-field dots, bf16 near field
    dict(name="fp8_state", grid=(2, 16, 16), leaf=64, E=2, sink=0, tail=0, trim=23, seed=28, store="fp8"),
    dict(name="fp8_sink_tail", grid=(2, 16, 16), leaf=64, E=3, sink=1, tail=5, trim=0, seed=29, store="fp8"),
    # the bf16 leaf state (store="bf16"): bf16 g and vbar without scales, bf16 far- and near-field dots
    dict(name="bf16_state", grid=(2, 16, 16), leaf=64, E=2, sink=0, tail=0, trim=23, seed=30, store="bf16"),
    dict(name="bf16_sink_tail", grid=(2, 16, 16), leaf=64, E=3, sink=1, tail=5, trim=0, seed=31, store="bf16"),
]


def run_case(flat, c):
    q, k, v = synth.head_inputs(c["grid"], 128, base_seed=c["seed"])
    tk = tv = None
    if c["tail"]:
        tk = k[-c["tail"]:].float().clone()
        tv = v[-c["tail"]:].float().clone()
        k, v = k[: -c["tail"]], v[: -c["tail"]]
        keep = (k.shape[0] // c["leaf"]) * c["leaf"]
        k, v = k[:keep].contiguous(), v[:keep].contiguous()
    if c["trim"]:
        q = q[: -c["trim"]].contiguous()
    if c.get("keys"):
        k, v = k[: c["keys"]].contiguous(), v[: c["keys"]].contiguous()
    rec = _recorder(flat)
    ws = {}
    cfg = dict(flat.PROD)
    cfg.update(leaf=c["leaf"], exact_leaves=c["E"], sink_leaves=c["sink"], tile_chunk=4096,
               order=c.get("order", "seq"), tile=c.get("tile", 64), store=c.get("store", "int8"))
    if c.get("group", 1) > 1:
        cfg["kern"] = {**cfg["kern"], "group": c["group"]}
    if c.get("quant"):
        cfg["quant"] = dict(c["quant"])
    out = flat.flat_attention(q, k, v, tail=(tk, tv) if tk is not None else None, ws=ws, **cfg)
    st = rec["stats"]
    ti = rec["tile"]
    fp8 = c.get("store") == "fp8"
    bf16 = c.get("store") == "bf16"
    res = dict(q=q.float().numpy(), k=k.float().numpy(), v=v.float().numpy(),
               leaf=np.int64(c["leaf"]), exact_leaves=np.int64(c["E"]), sink_leaves=np.int64(c["sink"]),
               group=np.int64(c.get("group", 1)), tile=np.int64(c.get("tile", 64)),
               mu=_cat(st, "mu").numpy(), lz=_cat(st, "lz").numpy(),
               excl=_cat(ti, "excl").numpy().astype(np.uint8), out=out.float().numpy())
    if "sg" in st[0]:
        res["sg"] = _cat(st, "sg").numpy()
    if bf16:
        # bf16 state as its bit patterns; no INT8 keys, no scales
        res.update(store=np.array("bf16"), g_bf16=_cat(st, "g8").view(torch.int16).numpy().view(np.uint16),
                   vb_bf16=_cat(st, "vb").view(torch.int16).numpy().view(np.uint16))
    elif fp8:
        # e4m3 state as its codes (bytes), with the row scales of g and vbar; no INT8 keys
        res.update(store=np.array("fp8"), g_e4m3=_cat(st, "g8").view(torch.uint8).numpy(),
                   vb_e4m3=_cat(st, "vb").view(torch.uint8).numpy(), sv=_cat(st, "sv").numpy())
    else:
        res.update(g8=_cat(st, "g8").numpy(), vb=_cat(st, "vb").float().numpy(), k8=ti[0]["k8"].numpy(),
                   ks=ti[0]["ks"].numpy())
    if rec["sel"]:
        res["sel"] = torch.cat(rec["sel"], 0).numpy()
    if "idx" in ti[0]:
        res["idx"] = _cat(ti, "idx").numpy().astype(np.int32)
    if "pm" in ti[0] and c["tail"] <= 16:          # a >16-key tail is a host partial outside ws
        pm, pl = _cat(ti, "pm").double(), _cat(ti, "pl").double()
        mm = pm.amax(1, keepdim=True)
        lse = (mm[:, 0] + torch.log((pl * torch.exp(pm - mm)).sum(1))).float()
        lse = lse.reshape(-1)[: q.shape[0]]
        if rec["perm"]:                            # tile order -> the caller's row order
            full = torch.empty_like(lse)
            full[rec["perm"][0]] = lse
            lse = full
        res["lse"] = lse.numpy()
    if tk is not None:
        res["tail_k"], res["tail_v"] = tk.numpy(), tv.numpy()
    if rec["perm"]:
        res["perm"] = rec["perm"][0].numpy().astype(np.int64)
    if c.get("quant"):
        res["quant_kv"], res["quant_q"] = np.array(c["quant"]["kv"]), np.array(c["quant"]["q"])
        res["quant_group"] = np.int64(c["quant"]["group"])
    if c.get("slim"):
        # large case: inputs as bfloat16 bit patterns, no per-(tile, leaf) state (the tests recompute it)
        for name, t in (("q", q), ("k", k), ("v", v)):
            res.pop(name)
            res[name + "16"] = t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        for name in ("g8", "vb", "sg", "lz", "sel", "k8"):
            res.pop(name, None)
    return res


def fake_quant_fixture(flat):
    """The reference's fake_quant (h3/htrc_flat.py:68-97) on rows of varied scale, and its dequant_rows
    (h3/htrc_flat_triton.py:276-294) on e4m3 codes."""
    g = torch.Generator().manual_seed(31)
    x = torch.randn(64, 128, generator=g) * torch.rand(64, 1, generator=g).pow(3) * 20
    x[5] = 0.0
    x[6, :7] = 1e-30
    xb = x.to(torch.bfloat16)                        # bf16 inputs (the kv path)
    res = {"x": x.numpy(), "xb": xb.float().numpy()}
    for fmt in ("int8", "int4", "fp8", "fp4"):
        for grp in (0, 16, 32):
            res[f"y_{fmt}_{grp}"] = flat.fake_quant(x, fmt, grp).numpy()
            res[f"yb_{fmt}_{grp}"] = flat.fake_quant(xb, fmt, grp).numpy()
    codes = torch.randint(0, 256, (64, 128), generator=g, dtype=torch.uint8)
    codes[(codes & 0x7F) == 0x7F] = 0x3C               # no NaN codes
    sc = torch.rand(64, generator=g) * 3 + 1e-3
    tri = flat._load_triton()
    out = torch.empty(64, 128, dtype=torch.bfloat16)
    tri.dequant_rows(codes.view(torch.float8_e4m3fn), sc, out)
    res.update(codes=codes.numpy(), dq_scale=sc.numpy(), dq_out=out.float().numpy())
    return res


def torch_spec_fixture(flat):
    """The reference's float32 torch backend (h3/htrc_flat.py:279-388) with curvature lin and iso: the
    specification the INT8 path approximates, and the only place the reference defines the iso term."""
    q, k, v = synth.head_inputs((2, 16, 16), 128, base_seed=41)
    q = q[:-21].contiguous()
    res = {name + "16": t.view(torch.int16).numpy().view(np.uint16) for name, t in (("q", q), ("k", k), ("v", v))}
    for curv in ("lin", "iso"):
        for e in (0, 3, 8):
            out = flat.flat_attention(q, k, v, backend="torch", curvature=curv, leaf=64, exact_leaves=e, tile=64,
                                      tile_chunk=64, precision="fp32")
            res[f"out_{curv}_{e}"] = out.numpy()
    return res


def main():
    ref, argv = _reference_dir(sys.argv[1:])
    _shim()
    flat = _load_reference(ref)
    torch.manual_seed(0)
    only = set(argv)
    if not only or "torch_spec" in only:
        np.savez_compressed(HERE / "torch_spec.npz", **torch_spec_fixture(flat))
        print("torch_spec -> torch_spec.npz")
    if not only or "fake_quant" in only:
        np.savez_compressed(HERE / "fake_quant.npz", **fake_quant_fixture(flat))
        print("fake_quant -> fake_quant.npz")
    for c in CASES:
        if only and c["name"] not in only:
            continue
        res = run_case(flat, c)
        path = HERE / f"{c['name']}.npz"
        np.savez_compressed(path, **res)
        qs, ks = res.get("q", res.get("q16")).shape, res.get("k", res.get("k16")).shape
        print(f"{c['name']}: q{tuple(qs)} k{tuple(ks)} -> {path.name}")


if __name__ == "__main__":
    main()
