"""CPU oracle of the flat HTRC operator's production (INT8) path, in NumPy.

TEST INFRASTRUCTURE ONLY.  This module is the checker the parity tests, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg compare the CUDA library against.  Nothing in the shipped
operator (``htrc_b200``) imports it; the CUDA path never falls back to it.

It restates, step by step, the arithmetic of the reference operator
``flat_attention(**PROD, leaf=L)`` of ASarych/HTRC, i.e. ``backend="triton", store="int8",
dot="bf16", select="max", curvature="lin"``:

  K INT8 pack ............ h3/htrc_flat.py:213-219       (round-half-even, IEEE divide by the scale)
  k-means query order .... h3/htrc_flat.py:47-65         (order="kmeans": Lloyd on a sample, stable sort)
  tile centres ........... h3/htrc_flat.py:142-156       (mean over the tile's real rows)
  group centres .......... h3/htrc_flat.py:223-231       (kern group G: mean over G padded tiles)
  leaf statistics ........ h3/htrc_flat_triton.py:41-85  (lz, g -> g8/sg half-away, vbar -> bf16)
  row-max selection ...... h3/htrc_flat_triton.py:214-254 (dq8 . g8 * sdq * sg, max over rows, + lz)
  top-E routing .......... h3/htrc_flat.py:232-265       (sink leaves forced, topk, exclusion mask)
  far + near + tail ...... h3/htrc_flat_triton.py:88-211 (online softmax, bf16 P for PV)
  split merge ............ h3/htrc_flat_triton.py:257-273 (normalised output) + log-Z (addition)

Precision of the restatement: the leaf statistics are computed in float64 and rounded once to
float32, from float32 operands (precision "fp32") or from their tf32 operand values (precision "tf32",
the reference's production setting on the GPU: the low 13 mantissa bits of the centre and of the softmax
weights cleared, ``tf32_operand``); every quantisation
formula is evaluated in float32 exactly as written in the reference; the softmax sums are float64.
Division is IEEE float32 (the reference's torch code uses IEEE division; its Triton kernels use
``/`` whose GPU lowering may be approximate; the CUDA kernels divide with IEEE rounding too).

Parity status: pinned against outputs of the reference itself run in the build container
(``tests/golden/make_golden.py`` runs h3/htrc_flat.py on CPU; the fixtures it wrote live in
``tests/golden/*.npz``; ``tests/test_oracle.py`` checks this module against them).
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32
INV127 = F32(1.0 / 127.0)      # the constant (1.0 / 127.0) the reference multiplies by, as float32
EPS_ROW = F32(1e-20)           # row-scale floor (h3/htrc_flat.py:217, h3/htrc_flat_triton.py:112)
EPS_SLOPE = F32(1e-30)         # slope abs-max floor (h3/htrc_flat_triton.py:75)


# ----------------------------------------------------------------------------- bf16 helpers
def bf16_bits(x):
    """float32 -> bfloat16 bit pattern (uint16), round to nearest even (finite inputs)."""
    b = np.ascontiguousarray(x, dtype=F32).view(np.uint32)
    lsb = (b >> np.uint32(16)) & np.uint32(1)
    return ((b + (lsb + np.uint32(0x7FFF))) >> np.uint32(16)).astype(np.uint16)   # no overflow for finite x


def bf16_to_f32(bits):
    """bfloat16 bit pattern (uint16) -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


def bf16_round(x):
    """Round float32 values to the nearest bfloat16 value (ties to even), returned as float32."""
    return bf16_to_f32(bf16_bits(x))


# ----------------------------------------------------------------------------- INT8 packing
def pack_rows_half_even(x):
    """Per-row INT8 pack of the near-field keys (h3/htrc_flat.py:216-218).

    ks = max(amax_row|x| * (1/127), 1e-20);  x8 = clamp(round_half_even(x / ks), -127, 127).
    Returns (x8 int8 [R, D], ks float32 [R])."""
    x = np.asarray(x, dtype=F32)
    s = np.maximum(np.abs(x).max(-1) * INV127, EPS_ROW).astype(F32)
    y = (x / s[:, None]).astype(F32)
    return np.clip(np.rint(y), -127, 127).astype(np.int8), s


def _round_half_away_i8(y):
    y = np.asarray(y, dtype=F32)
    z = np.where(y >= 0, y + F32(0.5), y - F32(0.5)).astype(F32)
    return np.trunc(z).astype(np.int8)


def pack_rows_half_away(x):
    """Per-row INT8 pack of query rows q and offsets dq = q - mu (h3/htrc_flat_triton.py:110-117,
    :230-233): s = max(amax_row|x| * (1/127), 1e-20);  x8 = trunc(x / s +- 0.5) (half away).
    Returns (x8 int8 [R, D], s float32 [R])."""
    x = np.asarray(x, dtype=F32)
    s = np.maximum(np.abs(x).max(-1) * INV127, EPS_ROW).astype(F32)
    return _round_half_away_i8(x / s[..., None]), s


def pack_blocks(x, block, rounding):
    """Extension, not in the reference (its scales are per row): the INT8 pack with one scale per block
    of `block` consecutive rows (one absmax scale per 64-token block of keys or queries).
    s_b = max(amax_block|x| * (1/127), 1e-20); every row of the block is coded with s_b, half-even
    (rounding "even": the keys' rule, h3/htrc_flat.py:216-218) or half-away ("away": the query rows' rule,
    h3/htrc_flat_triton.py:110-117).  Returns (x8 int8 [R, D], s float32 [R]: the block's scale per row)."""
    x = np.asarray(x, dtype=F32)
    r = x.shape[0]
    nbk = -(-r // block)
    am = np.zeros(nbk * block, F32)
    am[:r] = np.abs(x).max(-1)
    s = np.maximum((am.reshape(nbk, block).max(1) * INV127).astype(F32), EPS_ROW).astype(F32)
    sr = np.repeat(s, block)[:r]
    y = (x / sr[:, None]).astype(F32)
    if rounding == "even":
        return np.clip(np.rint(y), -127, 127).astype(np.int8), sr
    return _round_half_away_i8(y), sr


def pack_slope(g):
    """INT8 far-field slope per (tile, leaf) row (h3/htrc_flat_triton.py:73-79):
    am = max(amax|g|, 1e-30); sg = am * (1/127); g8 = trunc(g * (127 / am) +- 0.5).
    Returns (g8 int8 [..., D], sg float32 [...])."""
    g = np.asarray(g, dtype=F32)
    am = np.maximum(np.abs(g).max(-1), EPS_SLOPE).astype(F32)
    sg = (am * INV127).astype(F32)
    r = (F32(127.0) / am).astype(F32)
    return _round_half_away_i8(g * r[..., None]), sg


# ----------------------------------------------------------------------------- low-bit simulation
FP4_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], F32)      # e2m1 magnitudes
FP4_THR = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], F32)         # bucket boundaries (h3/htrc_flat.py:66)


def e4m3_round(t):
    """Nearest-even float8 e4m3fn value of t (|t| <= 448): 3 mantissa bits, exponent bias 7,
    subnormal quantum 2^-9."""
    t = np.asarray(t, np.float64)
    a = np.abs(t)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -9)))
    quantum = np.where(a < 2.0 ** -6, 2.0 ** -9, 2.0 ** (e - 3))
    r = np.rint(a / quantum) * quantum                  # half-even on the exact quotient (a power of 2)
    return (np.sign(t) * np.minimum(r, 448.0)).astype(F32)


def fake_quant(x, fmt, group=0):
    """Low-bit round trip with symmetric per-group scales (h3/htrc_flat.py:68-97): float32 result."""
    x = np.asarray(x, F32)
    d = x.shape[-1]
    if fmt == "fp4" and not group:
        group = 16
    gsz = d if not group else int(group)
    if d % gsz:
        raise ValueError("quant group must divide the feature size")
    y = x.reshape(*x.shape[:-1], d // gsz, gsz)
    amax = np.maximum(np.abs(y).max(-1, keepdims=True), F32(1e-20))
    if fmt in ("int8", "int4"):
        qmax = F32(127.0 if fmt == "int8" else 7.0)
        sc = (amax / qmax).astype(F32)
        out = (np.clip(np.rint((y / sc).astype(F32)), -qmax, qmax) * sc).astype(F32)
    elif fmt == "fp8":
        sc = (amax / F32(448.0)).astype(F32)
        out = (e4m3_round(np.clip((y / sc).astype(F32), -448.0, 448.0)) * sc).astype(F32)
    elif fmt == "fp4":
        sc = (amax / F32(6.0)).astype(F32)
        a = np.abs((y / sc).astype(F32))
        idx = (a[..., None] > FP4_THR).sum(-1)
        out = ((np.sign(y).astype(F32) * FP4_GRID[idx]).astype(F32) * sc).astype(F32)
    else:
        raise ValueError(f"unknown quant format {fmt}")
    return out.reshape(x.shape)


def dequant_rows(x8_values, scale):
    """bf16(x8 * scale) per row (h3/htrc_flat_triton.py:276-294), x8 given as its float values."""
    return bf16_round((np.asarray(x8_values, F32) * np.asarray(scale, F32)[:, None]).astype(F32))


# ----------------------------------------------------------------------------- stages
def linspace_f32(hi, steps):
    """torch.linspace(0, hi, steps) in float32 on the CPU: step = hi / (steps - 1) in float32, the first
    half step * i, the second half hi - step * (steps - 1 - i) rounded once (checked against
    torch.linspace in tests/test_oracle.py)."""
    if steps <= 1:
        return np.zeros(max(steps, 0), F32)
    step = F32(F32(hi) / F32(steps - 1))
    i = np.arange(steps)
    up = (np.float64(step) * i).astype(F32)
    dn = (np.float64(F32(hi)) - np.float64(step) * (steps - 1 - i)).astype(F32)
    return np.where(i < steps // 2, up, dn).astype(F32)


def _round_index(x):
    """torch's .round().long(): half to even."""
    return np.rint(x.astype(np.float64)).astype(np.int64)


def _nearest(x, c):
    """Index of the nearest centre per row (first minimum), distances in float64."""
    x = np.asarray(x, np.float64)
    c = np.asarray(c, np.float64)
    d = (x * x).sum(1)[:, None] - 2.0 * (x @ c.T) + (c * c).sum(1)[None, :]
    return d.argmin(1)


def kmeans_order(q, clusters=32, sample=4096, iters=8, return_labels=False):
    """Permutation grouping queries by k-means (h3/htrc_flat.py:47-65): Lloyd's iterations on the
    rows round(linspace(0, n-1, min(sample, n))), seeded with the sample rows
    round(linspace(0, S-1, clusters)); an empty cluster keeps its centre; then every row's nearest
    centre and a stable sort by it.  Distances here are float64 (the reference's torch.cdist works in
    float32 through |x|^2 - 2 x.c + |c|^2), so assignments can differ at near-ties only."""
    x = np.asarray(q, dtype=F32)
    n = x.shape[0]
    sidx = _round_index(linspace_f32(n - 1, min(sample, n)))
    s = x[sidx]
    c = s[_round_index(linspace_f32(s.shape[0] - 1, clusters))].copy()
    for _ in range(iters):
        a = _nearest(s, c)
        sums = np.zeros((clusters, x.shape[1]), np.float64)
        np.add.at(sums, a, s.astype(np.float64))
        cnt = np.bincount(a, minlength=clusters)
        nz = cnt > 0
        c[nz] = (sums[nz] / cnt[nz][:, None]).astype(F32)
    assign = _nearest(x, c)
    perm = np.argsort(assign, kind="stable").astype(np.int64)
    return (perm, assign) if return_labels else perm


def group_centres(qt, group):
    """Centres of groups of `group` consecutive tiles (h3/htrc_flat.py:223-231): the tiles are padded
    with repeats of the last tile to a multiple of the group and each centre is the mean of all
    group * T rows (the last tile's padding rows included); float64 mean rounded once."""
    qt = np.asarray(qt, dtype=F32)
    nt, t, d = qt.shape
    ntp = -(-nt // group) * group
    if ntp > nt:
        qt = np.concatenate([qt, np.repeat(qt[-1:], ntp - nt, 0)], 0)
    return qt.reshape(ntp // group, group * t, d).astype(np.float64).mean(1).astype(F32)


def tile_centres(q, tile):
    """(qt float32 [nt, T, D], mu float32 [nt, D], n) with the last tile padded by repeats of the
    last row and its centre taken over its real rows (h3/htrc_flat.py:142-156).  The mean is
    evaluated in float64 and rounded once."""
    q = np.asarray(q, dtype=F32)
    n, d = q.shape
    nt = -(-n // tile)
    npad = nt * tile
    qs = q if npad == n else np.concatenate([q, np.repeat(q[-1:], npad - n, 0)], 0)
    qt = qs.reshape(nt, tile, d)
    mu = qt.astype(np.float64).mean(1)
    if npad > n:
        mu[-1] = qt[-1, : n - (nt - 1) * tile].astype(np.float64).mean(0)
    return qt, mu.astype(F32), n


def tf32_operand(x):
    """float32 values as a tf32 tensor-core dot reads them on sm_100: the low 13 mantissa bits cleared.  The
    reference's Triton dots with input_precision="tf32" (h3/htrc_flat_triton.py:57, :62-63) behave this way on
    B200: its log-partitions match a = scale (tf32(mu) . k) to ~1e-5, against ~1e-2 for rounding to nearest."""
    b = np.ascontiguousarray(x, dtype=F32).view(np.uint32) & np.uint32(0xFFFFE000)
    return b.view(F32)


def leaf_stats(mu, k, v, leaf, scale, precision="fp32"):
    """Exact leaf cumulants at the tile centres (h3/htrc_flat_triton.py:41-85):
    a = scale mu.k_s, lz = logsumexp_s a, w = softmax a, g = scale sum w k, vbar = sum w v.
    precision "tf32" (the reference's PREC="tf32", PROD's setting): mu and w enter the two dots as tf32
    operand values (``tf32_operand``; k and v are bf16, exact in tf32).
    Returns float32 (g [nt, nb, D], lz [nt, nb], vbar [nt, nb, D])."""
    tf32 = precision == "tf32"
    mu = np.asarray(tf32_operand(mu) if tf32 else mu, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    nb = k.shape[0] // leaf
    d = k.shape[1]
    k3 = k[: nb * leaf].reshape(nb, leaf, d)
    v3 = v[: nb * leaf].reshape(nb, leaf, d)
    a = np.einsum("td,lsd->tls", mu, k3) * float(scale)
    m = a.max(-1, keepdims=True)
    w = np.exp(a - m)
    z = w.sum(-1, keepdims=True)
    w /= z
    lz = (m + np.log(z))[..., 0]
    if tf32:
        w = tf32_operand(w.astype(F32)).astype(np.float64)
    g = np.einsum("tls,lsd->tld", w, k3) * float(scale)
    vb = np.einsum("tls,lsd->tld", w, v3)
    return g.astype(F32), lz.astype(F32), vb.astype(F32)


def iso_coeff(mu, k, leaf, scale):
    """Isotropic curvature coefficient per (centre, leaf) (h3/htrc_flat.py:331-333, the torch backend's
    curvature="iso"): 0.5 / D * max(tr, 0), tr = scale^2 (sum_s w_s |k_s|^2 - |sum_s w_s k_s|^2), in
    float64 rounded once."""
    mu = np.asarray(mu, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    nb = k.shape[0] // leaf
    d = k.shape[1]
    k3 = k[: nb * leaf].reshape(nb, leaf, d)
    a = np.einsum("td,lsd->tls", mu, k3) * float(scale)
    w = np.exp(a - a.max(-1, keepdims=True))
    w /= w.sum(-1, keepdims=True)
    kn2 = (k3 * k3).sum(-1)                                   # [nb, leaf]
    mean = np.einsum("tls,lsd->tld", w, k3)
    tr = float(scale) ** 2 * ((w * kn2[None]).sum(-1) - (mean * mean).sum(-1))
    return (0.5 / d * np.maximum(tr, 0.0)).astype(F32)


def offset_sqnorm(qt, mu):
    """|q_r - mu|^2 per tile row, from the float32 offsets (the iso term's row factor)."""
    dq = (np.asarray(qt, F32) - np.asarray(mu, F32)[:, None, :]).astype(F32)
    return (dq.astype(np.float64) ** 2).sum(-1).astype(F32)


def state_int8(g, vb):
    """The stored far-field state: (g8, sg, vbar as bf16-rounded float32)
    (h3/htrc_flat_triton.py:73-81)."""
    g8, sg = pack_slope(g)
    return g8, sg, bf16_round(vb)


def query_codes(qt, mu, q_block=False):
    """Per-row INT8 codes of the tile rows and of their offsets from the tile centre, as the tile
    and row-max kernels form them in-register (h3/htrc_flat_triton.py:103-117).  q_block (extension):
    one scale per tile for the rows' codes (`pack_blocks`); the offsets keep per-row scales."""
    qt = np.asarray(qt, dtype=F32)
    dq = (qt - np.asarray(mu, dtype=F32)[:, None, :]).astype(F32)
    if q_block:
        nt, t, d = qt.shape
        q8, sq = pack_blocks(qt.reshape(nt * t, d), t, "away")
        q8, sq = q8.reshape(nt, t, d), sq.reshape(nt, t)
    else:
        q8, sq = pack_rows_half_away(qt)
    dq8, sdq = pack_rows_half_away(dq)
    return q8, sq, dq8, sdq


def rowmax_select(dq8, sdq, g8, sg, lz, group=1, cv=None, dd=None):
    """SEL[t, l] = max_r (dq8_r . g8_l) * (sdq_r * sg_l) + lz_l (h3/htrc_flat_triton.py:240-254); with
    groups the rows are all G * T rows of a group (the reference calls the kernel with
    T = G * tile, h3/htrc_flat.py:243-249) and the state row is the group's: returns [ng, nb]."""
    nt = dq8.shape[0]
    st = np.arange(nt) // group
    dot = np.matmul(dq8.astype(np.float64), np.swapaxes(g8[st].astype(np.float64), 1, 2))
    sc = dot.astype(F32) * (sdq[:, :, None] * sg[st][:, None, :]).astype(F32)
    if cv is not None:                                        # iso curvature: + c_l |q_r - mu|^2
        sc = (sc + (cv[st][:, None, :] * dd[:, :, None]).astype(F32)).astype(F32)
    per_tile = (sc.max(1) + lz[st]).astype(F32)
    ng = -(-nt // group)
    out = np.full((ng, per_tile.shape[1]), -np.inf, F32)
    np.maximum.at(out, st, per_tile)
    return out


def route(sel, exact_leaves, sink_leaves=0):
    """Top-E near-leaf routing per tile (h3/htrc_flat.py:232-233, :250-265).

    Returns (idx int32 [nt, kx] sorted ascending, excl uint8 [nt, nb]).  The reference's
    torch.topk returns the same set in an unspecified order; ties at the boundary are broken
    here towards the lower leaf index."""
    sel = np.array(sel, dtype=F32, copy=True)
    nt, nb = sel.shape
    sink = max(0, min(int(sink_leaves), nb))
    kx = min(int(exact_leaves) + sink, nb)
    excl = np.zeros((nt, nb), np.uint8)
    if kx <= 0:
        return np.zeros((nt, 0), np.int32), excl
    if sink:
        sel[:, :sink] = np.inf
    order = np.argsort(-sel, axis=1, kind="stable")[:, :kx]
    idx = np.sort(order, axis=1).astype(np.int32)
    np.put_along_axis(excl, idx.astype(np.int64), 1, axis=1)
    return idx, excl


def tile_attention(qt, q8, sq, dq8, sdq, g8, sg, lz, vb, excl, idx, k8, ks, v, leaf, scale,
                   tail=None, group=1, cv=None, dd=None):
    """Far field + near field + tail of every tile, merged; returns (out float32 [nt*T, D],
    lse float32 [nt*T]) (h3/htrc_flat_triton.py:88-211, merge :257-273).

    far  : logit = (dq8 . g8_l) * (sdq * sg_l) + lz_l over the non-excluded leaves, value vbar_l
    near : logit = (q8 . k8_j) * (sq * ks_j * scale) over the tokens of the routed leaves, value v_j
    tail : logit = bf16(q) . bf16(tk_j) * scale (<= 16 keys) or the float32 product (> 16 keys),
           value tv_j (h3/htrc_flat_triton.py:187-207, :381-388)
    P is rounded to bfloat16 for the value product (not for a > 16-key tail, whose partial the
    reference forms in float32 on the host); the normaliser sums float32 P.  Tile t uses the state,
    exclusion and routing rows of its group t // group (h3/htrc_flat_triton.py:102)."""
    nt, T, d = qt.shape
    nb = lz.shape[1]
    v = np.asarray(v, dtype=F32)
    out = np.zeros((nt, T, d), F32)
    lse = np.zeros((nt, T), F32)
    ar = np.arange(leaf)
    if tail is not None and tail[0].shape[0] > 0:
        tk = np.asarray(tail[0], dtype=F32)
        tv = np.asarray(tail[1], dtype=F32)
        small = tk.shape[0] <= 16
        if small:
            tk, tv = bf16_round(tk), bf16_round(tv)
    else:
        tk = tv = None
    for t in range(nt):
        gt = t // group
        parts_s, parts_v, parts_r = [], [], []
        keep = excl[gt] == 0
        if keep.any():
            dot = dq8[t].astype(np.float64) @ g8[gt][keep].astype(np.float64).T
            sc = dot.astype(F32) * (sdq[t][:, None] * sg[gt][keep][None, :]).astype(F32) + lz[gt][keep][None, :]
            if cv is not None:
                sc = sc + (cv[gt][keep][None, :] * dd[t][:, None]).astype(F32)
            parts_s.append(sc.astype(F32))
            parts_v.append(vb[gt][keep])
            parts_r.append(np.ones(sc.shape[1], bool))
        if idx.shape[1]:
            tok = (idx[gt][:, None].astype(np.int64) * leaf + ar[None, :]).reshape(-1)
            dot = q8[t].astype(np.float64) @ k8[tok].astype(np.float64).T
            sc = dot.astype(F32) * ((sq[t][:, None] * ks[tok][None, :]).astype(F32) * F32(scale)).astype(F32)
            parts_s.append(sc.astype(F32))
            parts_v.append(v[tok])
            parts_r.append(np.ones(sc.shape[1], bool))
        if tk is not None:
            if small:
                sc = (bf16_round(qt[t]).astype(np.float64) @ tk.astype(np.float64).T).astype(F32) * F32(scale)
            else:
                sc = (qt[t].astype(np.float64) @ tk.astype(np.float64).T).astype(F32) * F32(scale)
            parts_s.append(sc.astype(F32))
            parts_v.append(tv)
            parts_r.append(np.full(sc.shape[1], small))
        s = np.concatenate(parts_s, 1).astype(np.float64)
        vv = np.concatenate(parts_v, 0).astype(np.float64)
        rnd = np.concatenate(parts_r)
        m = s.max(1, keepdims=True)
        p = np.exp(s - m)
        den = p.sum(1)
        pq = np.where(rnd[None, :], bf16_round(p.astype(F32)).astype(np.float64), p)
        num = pq @ vv
        out[t] = (num / np.maximum(den, 1e-30)[:, None]).astype(F32)
        lse[t] = (m[:, 0] + np.log(den)).astype(F32)
    return out.reshape(nt * T, d), lse.reshape(nt * T)


def _split(n, ns, bn):
    """Per-split extent rounded up to the block width (h3/htrc_flat_triton.py:297-299)."""
    per = -(-n // ns)
    return max(bn, -(-per // bn) * bn)


def tile_attention_ordered(qt, q8, sq, dq8, sdq, g8, sg, lz, vb, excl, idx, k8, ks, v, leaf, scale,
                           tail=None, splits=4, bn=64, group=1):
    """Same operator evaluated in the reference kernel's exact order: ``splits`` split programs per
    tile, blocks of ``bn`` leaves / tokens, float32 online softmax with P rounded to bfloat16
    against the running maximum, then the split merge (h3/htrc_flat_triton.py:118-211, :257-273).
    ``idx`` must be in the reference's (unsorted) order.  Pins the restatement bit-for-bit
    (up to float32 summation order) against fixtures recorded from the reference; returns
    (out [nt*T, D], lse [nt*T])."""
    nt, T, d = qt.shape
    nb = lz.shape[1]
    kx = idx.shape[1]
    lps = _split(nb, splits, bn)
    e_n = kx * leaf
    eps = _split(e_n, splits, bn)
    v = np.asarray(v, dtype=F32)
    small_tail = tail is not None and 0 < tail[0].shape[0] <= 16
    if small_tail:
        tk, tv = bf16_round(tail[0]), bf16_round(tail[1])
    out = np.zeros((nt, T, d), F32)
    lse = np.zeros((nt, T), F32)
    scale = F32(scale)

    def step(m, l, acc, sc, vals):
        mn = np.maximum(m, sc.max(1))
        ms = np.where(mn == -np.inf, F32(0), mn).astype(F32)
        p = np.exp(sc - ms[:, None]).astype(F32)
        al = np.exp(m - ms).astype(F32)
        l = (l * al + p.sum(1)).astype(F32)
        acc = (acc * al[:, None] + (bf16_round(p).astype(np.float64) @ vals.astype(np.float64))).astype(F32)
        return mn, l, acc

    for t in range(nt):
        gt = t // group
        pms, pls, paccs = [], [], []
        for sp in range(splits):
            m = np.full(T, -np.inf, F32)
            l = np.zeros(T, F32)
            acc = np.zeros((T, d), F32)
            lo, hi = sp * lps, min(nb, sp * lps + lps)
            for n0 in range(lo, hi, bn):
                c = np.arange(n0, min(n0 + bn, hi))
                dot = dq8[t].astype(np.int32) @ g8[gt][c].astype(np.int32).T
                sc = (dot.astype(F32) * (sdq[t][:, None] * sg[gt][c][None, :]).astype(F32) + lz[gt][c][None, :]).astype(F32)
                sc = np.where((excl[gt][c] == 0)[None, :], sc, F32(-np.inf))
                m, l, acc = step(m, l, acc, sc, vb[gt][c])
            e_lo, e_hi = sp * eps, min(e_n, sp * eps + eps)
            for e0 in range(e_lo, e_hi, bn):
                j = np.arange(e0, min(e0 + bn, e_hi))
                tok = idx[gt][j // leaf].astype(np.int64) * leaf + j % leaf
                dot = q8[t].astype(np.int32) @ k8[tok].astype(np.int32).T
                sc = (dot.astype(F32) * ((sq[t][:, None] * ks[tok][None, :]).astype(F32) * scale)).astype(F32)
                m, l, acc = step(m, l, acc, sc, v[tok])
            if small_tail and sp == splits - 1:
                sc = ((bf16_round(qt[t]).astype(np.float64) @ tk.astype(np.float64).T).astype(F32) * scale).astype(F32)
                m, l, acc = step(m, l, acc, sc, tv)
            pms.append(m)
            pls.append(l)
            paccs.append(acc)
        if tail is not None and tail[0].shape[0] > 16:
            tk32 = np.asarray(tail[0], F32)
            lg = (qt[t].astype(np.float64) @ tk32.astype(np.float64).T).astype(F32) * scale
            tm = lg.max(1)
            te = np.exp(lg - tm[:, None]).astype(F32)
            pms.append(tm.astype(F32))
            pls.append(te.sum(1).astype(F32))
            paccs.append((te.astype(np.float64) @ np.asarray(tail[1], np.float64)).astype(F32))
        pm, pl, pa = np.array(pms), np.array(pls), np.array(paccs)
        mm = pm.max(0)
        mm = np.where(mm == -np.inf, F32(0), mm)
        w = np.exp(pm - mm).astype(F32)
        den = (pl * w).sum(0)
        out[t] = ((pa * w[:, :, None]).sum(0) / np.maximum(den, F32(1e-30))[:, None]).astype(F32)
        lse[t] = (mm + np.log(np.maximum(den, F32(1e-30)))).astype(F32)
    return out.reshape(nt * T, d), lse.reshape(nt * T)


# ----------------------------------------------------------------------------- fp8 (e4m3) state
INV448 = F32(1.0 / 448.0)      # the constant (1.0 / 448.0) the reference multiplies by, as float32


def f16_round(x):
    """Nearest-even float16 value of float32 x, as float32."""
    return np.asarray(x, F32).astype(np.float16).astype(F32)


def e4m3_codes(vals):
    """e4m3fn code bytes of values already on the e4m3 grid (|v| <= 448); -0 for negative zeros."""
    x = np.asarray(vals, np.float64)
    a = np.abs(x)
    sub = a < 2.0 ** -6
    er = np.floor(np.log2(np.maximum(a, 2.0 ** -6)))
    code = np.where(sub, np.rint(a / 2.0 ** -9), (er + 7) * 8 + np.rint((a / 2.0 ** er - 1.0) * 8))
    return (code.astype(np.uint8) | (np.signbit(x).astype(np.uint8) << 7)).astype(np.uint8)


def e4m3_values(codes):
    """Float32 values of e4m3fn code bytes."""
    c = np.asarray(codes, np.uint8).astype(np.int64)
    sign = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 7
    v = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * 2.0 ** (e - 7.0))
    return (sign * v).astype(F32)


def state_fp8(g, vb):
    """The fp8 far-field state (h3/htrc_flat_triton.py:65-72): per (centre, leaf) row scales
    sg = max(amax|g| * (1/448), 1e-30), sv likewise for vbar, and the e4m3 values of g / sg and
    vbar / sv (nearest even, saturating at 448).  Returns (g values, sg, vbar values, sv)."""
    g = np.asarray(g, F32)
    vb = np.asarray(vb, F32)
    sg = np.maximum((np.abs(g).max(-1) * INV448).astype(F32), F32(1e-30)).astype(F32)
    sv = np.maximum((np.abs(vb).max(-1) * INV448).astype(F32), F32(1e-30)).astype(F32)
    gq = e4m3_round(np.clip((g / sg[..., None]).astype(F32), -448.0, 448.0))
    vq = e4m3_round(np.clip((vb / sv[..., None]).astype(F32), -448.0, 448.0))
    return gq, sg, vq, sv


def state_bf16(g, vb):
    """The bf16 far-field state (h3/htrc_flat_triton.py:82-84, store="bf16"): g and vbar rounded to bf16
    (nearest even), no row scales.  Returns (g values, vbar values) as float32."""
    return bf16_round(np.asarray(g, F32)), bf16_round(np.asarray(vb, F32))


def query_codes_bf16(qt, mu):
    """The bf16 state's query operands (h3/htrc_flat_triton.py:106-107, DOT=1): bf16(q) for the near field and
    bf16(q - mu) for the far field (float32 offsets rounded once)."""
    qt = np.asarray(qt, F32)
    dq = (qt - np.asarray(mu, F32)[:, None, :]).astype(F32)
    return bf16_round(qt), bf16_round(dq)


def rowmax_select_bf16(dqb, gb, lz, group=1):
    """SEL[t, l] = max_r (bf16(dq_r) . g_l) + lz_l (h3/htrc_flat_triton.py:247-248, DOT=1 with the bf16
    state): float32 sums of exact bf16 products; groups as rowmax_select."""
    return rowmax_select_fp8(dqb, gb, np.ones(np.asarray(lz).shape, F32), lz, group)


def query_codes_fp8(qt, mu):
    """The fp8 path's query operands (h3/htrc_flat_triton.py:103-109): bf16(q) for the near field and
    fp16(q - mu) for the far field (float32 offsets rounded once)."""
    qt = np.asarray(qt, F32)
    dq = (qt - np.asarray(mu, F32)[:, None, :]).astype(F32)
    return bf16_round(qt), f16_round(dq)


def rowmax_select_fp8(dqh, gq, sg, lz, group=1):
    """SEL[t, l] = max_r (fp16(dq_r) . g_l) * sg_l + lz_l (h3/htrc_flat_triton.py:240-254, FP8=1): float32
    products of fp16 operands; groups as rowmax_select."""
    nt = dqh.shape[0]
    st = np.arange(nt) // group
    dot = np.matmul(dqh.astype(np.float64), np.swapaxes(gq[st].astype(np.float64), 1, 2)).astype(F32)
    per_tile = ((dot * sg[st][:, None, :]).astype(F32).max(1) + lz[st]).astype(F32)
    ng = -(-nt // group)
    out = np.full((ng, per_tile.shape[1]), -np.inf, F32)
    np.maximum.at(out, st, per_tile)
    return out


def tile_attention_fp8(qt, qb, dqh, gq, sg, lz, vq, sv, excl, idx, kb, vbf, leaf, scale, tail=None, group=1,
                       far_weight="f16"):
    """Far + near (+ tail) of every tile with the fp8 state (h3/htrc_flat_triton.py:118-211, FP8=1, DOT=1),
    order-free: far logit = (fp16 dq . g) * sg + lz, value weight fp16(p * sv) on the e4m3 values of vbar;
    near logit = (bf16 q . bf16 k) * scale, weight bf16(p); the normaliser sums float32 p.
    far_weight="bf16" with sg = sv = 1, bf16 dq and the bf16 state is the bf16-state path (:139-140, :154):
    far logit = (bf16 dq . g) + lz, weight bf16(p).  Returns (out [nt*T, D], lse [nt*T])."""
    nt, T, d = qt.shape
    out = np.zeros((nt, T, d), F32)
    lse = np.zeros((nt, T), F32)
    ar = np.arange(leaf)
    vbf = np.asarray(vbf, F32)
    small_tail = tail is not None and 0 < tail[0].shape[0] <= 16
    for t in range(nt):
        gt = t // group
        ss, vs, ws = [], [], []          # scores, values, (kind, column multiplier)
        keep = excl[gt] == 0
        if keep.any():
            sc = (dqh[t].astype(np.float64) @ gq[gt][keep].astype(np.float64).T).astype(F32)
            ss.append((sc * sg[gt][keep][None, :]).astype(F32) + lz[gt][keep][None, :])
            vs.append(vq[gt][keep])
            ws.append((far_weight, sv[gt][keep]) if far_weight == "f16" else ("bf16", None))
        if idx.shape[1]:
            tok = (idx[gt][:, None].astype(np.int64) * leaf + ar[None, :]).reshape(-1)
            sc = (qb[t].astype(np.float64) @ kb[tok].astype(np.float64).T).astype(F32)
            ss.append((sc * F32(scale)).astype(F32))
            vs.append(vbf[tok])
            ws.append(("bf16", None))
        if tail is not None and tail[0].shape[0]:
            tk = np.asarray(tail[0], F32)
            tv = np.asarray(tail[1], F32)
            if small_tail:
                sc = (bf16_round(qt[t]).astype(np.float64) @ bf16_round(tk).astype(np.float64).T).astype(F32)
                ss.append((sc * F32(scale)).astype(F32))
                vs.append(bf16_round(tv))
                ws.append(("bf16", None))
            else:
                sc = (qt[t].astype(np.float64) @ tk.astype(np.float64).T).astype(F32)
                ss.append((sc * F32(scale)).astype(F32))
                vs.append(tv)
                ws.append(("none", None))
        m = np.max([x.max(1) for x in ss], axis=0)
        den = np.zeros(T)
        num = np.zeros((T, d))
        for sc, vv, (kind, mult) in zip(ss, vs, ws):
            pr = np.exp(sc.astype(np.float64) - m[:, None])
            den += pr.sum(1)
            if kind == "f16":
                w = f16_round((pr * mult[None, :]).astype(F32)).astype(np.float64)
            elif kind == "bf16":
                w = bf16_round(pr.astype(F32)).astype(np.float64)
            else:
                w = pr
            num += w @ vv.astype(np.float64)
        out[t] = (num / np.maximum(den, 1e-30)[:, None]).astype(F32)
        lse[t] = (m + np.log(den)).astype(F32)
    return out.reshape(nt * T, d), lse.reshape(nt * T)


def tile_attention_fp8_ordered(qt, qb, dqh, gq, sg, lz, vq, sv, excl, idx, kb, vbf, leaf, scale, tail=None,
                               splits=4, bn=64, group=1, far_weight="f16"):
    """The fp8 tile attention in the reference kernel's own order (splits, blocks of bn, float32 online
    softmax, weights rounded against the running maximum, split merge); idx in the reference's order.
    Pins the restatement against fixtures recorded from the reference."""
    nt, T, d = qt.shape
    nb = lz.shape[1]
    kx = idx.shape[1]
    lps = _split(nb, splits, bn)
    e_n = kx * leaf
    eps = _split(e_n, splits, bn)
    vbf = np.asarray(vbf, F32)
    scale = F32(scale)
    small_tail = tail is not None and 0 < tail[0].shape[0] <= 16
    out = np.zeros((nt, T, d), F32)
    lse = np.zeros((nt, T), F32)

    def step(m, l, acc, sc, vals, weight):
        mn = np.maximum(m, sc.max(1))
        ms = np.where(mn == -np.inf, F32(0), mn).astype(F32)
        p = np.exp(sc - ms[:, None]).astype(F32)
        al = np.exp(m - ms).astype(F32)
        l = (l * al + p.sum(1)).astype(F32)
        acc = (acc * al[:, None] + (weight(p).astype(np.float64) @ vals.astype(np.float64))).astype(F32)
        return mn, l, acc

    for t in range(nt):
        gt = t // group
        pms, pls, paccs = [], [], []
        for sp in range(splits):
            m = np.full(T, -np.inf, F32)
            l = np.zeros(T, F32)
            acc = np.zeros((T, d), F32)
            lo, hi = sp * lps, min(nb, sp * lps + lps)
            for n0 in range(lo, hi, bn):
                c = np.arange(n0, min(n0 + bn, hi))
                sc = (dqh[t].astype(np.float64) @ gq[gt][c].astype(np.float64).T).astype(F32)
                sc = ((sc * sg[gt][c][None, :]).astype(F32) + lz[gt][c][None, :]).astype(F32)
                sc = np.where((excl[gt][c] == 0)[None, :], sc, F32(-np.inf))
                svc = sv[gt][c]
                wf = (lambda p, svc=svc: f16_round((p * svc[None, :]).astype(F32))) if far_weight == "f16" else bf16_round
                m, l, acc = step(m, l, acc, sc, vq[gt][c], wf)
            e_lo, e_hi = sp * eps, min(e_n, sp * eps + eps)
            for e0 in range(e_lo, e_hi, bn):
                j = np.arange(e0, min(e0 + bn, e_hi))
                tok = idx[gt][j // leaf].astype(np.int64) * leaf + j % leaf
                sc = ((qb[t].astype(np.float64) @ kb[tok].astype(np.float64).T).astype(F32) * scale).astype(F32)
                m, l, acc = step(m, l, acc, sc, vbf[tok], bf16_round)
            if small_tail and sp == splits - 1:
                tk, tv = bf16_round(tail[0]), bf16_round(tail[1])
                sc = ((bf16_round(qt[t]).astype(np.float64) @ tk.astype(np.float64).T).astype(F32) * scale).astype(F32)
                m, l, acc = step(m, l, acc, sc, tv, bf16_round)
            pms.append(m)
            pls.append(l)
            paccs.append(acc)
        if tail is not None and tail[0].shape[0] > 16:
            tk32 = np.asarray(tail[0], F32)
            lg = (qt[t].astype(np.float64) @ tk32.astype(np.float64).T).astype(F32) * scale
            tm = lg.max(1)
            te = np.exp(lg - tm[:, None]).astype(F32)
            pms.append(tm.astype(F32))
            pls.append(te.sum(1).astype(F32))
            paccs.append((te.astype(np.float64) @ np.asarray(tail[1], np.float64)).astype(F32))
        pm, pl, pa = np.array(pms), np.array(pls), np.array(paccs)
        mm = pm.max(0)
        mm = np.where(mm == -np.inf, F32(0), mm)
        w = np.exp(pm - mm).astype(F32)
        den = (pl * w).sum(0)
        out[t] = ((pa * w[:, :, None]).sum(0) / np.maximum(den, F32(1e-30))[:, None]).astype(F32)
        lse[t] = (mm + np.log(np.maximum(den, F32(1e-30)))).astype(F32)
    return out.reshape(nt * T, d), lse.reshape(nt * T)


def pack_k(k):
    """Near-field key pack of bf16 keys: (k8, ks) (h3/htrc_flat.py:211-219)."""
    return pack_rows_half_even(bf16_round(np.asarray(k, dtype=F32)))


def flat_attention(q, k, v, *, tile=64, exact_leaves=256, leaf=64, scale=None, sink_leaves=0,
                   tail=None, return_stages=False, group=1, order="seq", perm=None, quant=None,
                   stats_bf16=False, curvature="lin", store="int8", qk_scale_block=0, precision="fp32"):
    """The whole production path for one head: q [N, D], k/v [M, D] (float32 arrays holding the
    caller's values; k and v are rounded to bfloat16 as the reference's bf16 path stores them).
    group: G tiles per centre (kern["group"]); order "kmeans" permutes the queries first (``perm``
    overrides the permutation, e.g. with the device's, to check the stages after it); precision: the leaf
    statistics' dots, "fp32" (the reference's "ieee"; its recorded fixtures, whose interpreter evaluates every
    dot in float32) or "tf32" (PROD's setting on the GPU, see ``tf32_operand``).
    Returns (out float32 [N, D], lse float32 [N]) and, with return_stages, a dict of every stage."""
    q = np.asarray(q, dtype=F32)
    group = max(1, int(group))
    k_stats = v_stats = None
    if quant:
        # h3/htrc_flat.py:190-195: inputs fake-quantised first (float32 results); the bf16 near field
        # rounds the quantised keys/values to bf16 while the leaf statistics use them unrounded
        # (stats_bf16=True models a device that reads bf16 keys for the statistics too)
        qg = int(quant.get("group", 0))
        if quant.get("kv"):
            k = fake_quant(k, quant["kv"], qg)
            v = fake_quant(v, quant["kv"], qg)
            if not stats_bf16:
                k_stats, v_stats = k, v
        if quant.get("q"):
            q = fake_quant(q, quant["q"], qg)
    if order == "kmeans" and perm is None:
        perm = kmeans_order(q)
    if order != "kmeans":
        perm = None
    q_caller = q
    if perm is not None:
        q = q[np.asarray(perm, np.int64)]
    k = bf16_round(np.asarray(k, dtype=F32))
    v = bf16_round(np.asarray(v, dtype=F32))
    n, d = q.shape
    m = k.shape[0]
    if m % leaf:
        raise ValueError("key count must be a multiple of the leaf size")
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    # qk_scale_block=64 (extension): one scale per 64 keys (a leaf) and per query tile
    k8, ks = pack_blocks(k, int(qk_scale_block), "even") if qk_scale_block else pack_rows_half_even(k)
    qt, mu, _ = tile_centres(q, tile)
    if group > 1:
        mu = group_centres(qt, group)
    g, lz, vbf = leaf_stats(mu, k if k_stats is None else k_stats, v if v_stats is None else v_stats, leaf, scale,
                            precision)
    if store in ("fp8", "bf16"):
        return _flat_fp8(qt, mu, g, lz, vbf, k, v, n, leaf, scale, exact_leaves, sink_leaves, tail, group, perm,
                         return_stages, store=store)
    g8, sg, vb = state_int8(g, vbf)
    mu_t = mu[np.arange(qt.shape[0]) // group]
    q8, sq, dq8, sdq = query_codes(qt, mu_t, q_block=bool(qk_scale_block))
    cv = dd = None
    if curvature == "iso":
        cv = iso_coeff(mu, k if k_stats is None else k_stats, leaf, scale)
        dd = offset_sqnorm(qt, mu_t)
    nb = m // leaf
    sink = max(0, min(int(sink_leaves), nb))
    kx = min(int(exact_leaves) + sink, nb)
    if kx > 0:
        sel = rowmax_select(dq8, sdq, g8, sg, lz, group, cv, dd)
    else:
        sel = np.zeros((mu.shape[0], nb), F32)
    idx, excl = route(sel, exact_leaves, sink)
    out, lse = tile_attention(qt, q8, sq, dq8, sdq, g8, sg, lz, vb, excl, idx, k8, ks, v, leaf,
                              scale, tail=tail, group=group, cv=cv, dd=dd)
    out, lse = out[:n], lse[:n]
    if perm is not None:
        full, full_l = np.empty_like(out), np.empty_like(lse)
        full[perm], full_l[perm] = out, lse
        out, lse = full, full_l
    if not return_stages:
        return out, lse
    return out, lse, dict(k8=k8, ks=ks, qt=qt, mu=mu, g=g, g8=g8, sg=sg, lz=lz, vb=vb, q8=q8,
                          sq=sq, dq8=dq8, sdq=sdq, sel=sel, idx=idx, excl=excl, perm=perm, q=q_caller, cv=cv, dd=dd)


def _flat_fp8(qt, mu, g, lz, vbf, kb, vb, n, leaf, scale, exact_leaves, sink_leaves, tail, group, perm, return_stages,
              store="fp8"):
    """store="fp8" after the leaf statistics: e4m3 state, fp16 far field, bf16 near field; store="bf16": the
    bf16 state without scales, bf16 far and near fields."""
    mu_t = mu[np.arange(qt.shape[0]) // group]
    if store == "bf16":
        gq, vq = state_bf16(g, vbf)
        sg = np.ones(np.asarray(lz).shape, F32)
        sv = sg
        qb, dqh = query_codes_bf16(qt, mu_t)
        far_weight = "bf16"
    else:
        gq, sg, vq, sv = state_fp8(g, vbf)
        qb, dqh = query_codes_fp8(qt, mu_t)
        far_weight = "f16"
    nb = kb.shape[0] // leaf
    sink = max(0, min(int(sink_leaves), nb))
    kx = min(int(exact_leaves) + sink, nb)
    sel = rowmax_select_fp8(dqh, gq, sg, lz, group) if kx > 0 else np.zeros((mu.shape[0], nb), F32)
    idx, excl = route(sel, exact_leaves, sink)
    out, lse = tile_attention_fp8(qt, qb, dqh, gq, sg, lz, vq, sv, excl, idx, kb, vb, leaf, scale, tail=tail,
                                  group=group, far_weight=far_weight)
    out, lse = out[:n], lse[:n]
    if perm is not None:
        full, full_l = np.empty_like(out), np.empty_like(lse)
        full[perm], full_l[perm] = out, lse
        out, lse = full, full_l
    if not return_stages:
        return out, lse
    return out, lse, dict(qt=qt, mu=mu, g=g, gq=gq, sg=sg, lz=lz, vq=vq, sv=sv, qb=qb, dqh=dqh, sel=sel, idx=idx,
                          excl=excl, perm=perm)


def prepare_head(q, k, v, *, tile=64, leaf=64):
    """Per-head work of the production path that does not depend on the query tile: bf16 keys and
    values, the key INT8 pack (h3/htrc_flat.py:211-219) and the tile centres (:142-156)."""
    q = np.asarray(q, dtype=F32)
    kb = bf16_round(np.asarray(k, dtype=F32))
    vb = bf16_round(np.asarray(v, dtype=F32))
    if kb.shape[0] % leaf:
        raise ValueError("key count must be a multiple of the leaf size")
    k8, ks = pack_rows_half_even(kb)
    qt, mu, n = tile_centres(q, tile)
    return dict(k=kb, v=vb, k8=k8, ks=ks, qt=qt, mu=mu, n=n, leaf=leaf)


def attention_tiles(prep, tiles, *, exact_leaves=256, scale=None, sink_leaves=0, tail=None, precision="fp32"):
    """The production path for a subset of query tiles of a prepared head (every tile is independent
    given the keys): returns (out float32 [len(tiles)*T, D], lse float32 [len(tiles)*T]) for the
    rows of those tiles, padding rows included."""
    k, v, leaf = prep["k"], prep["v"], prep["leaf"]
    d = k.shape[1]
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    tiles = np.asarray(tiles, dtype=np.int64)
    qt, mu = prep["qt"][tiles], prep["mu"][tiles]
    nb = k.shape[0] // leaf
    g, lz, vbf = leaf_stats(mu, k, v, leaf, scale, precision)
    g8, sg, vb = state_int8(g, vbf)
    q8, sq, dq8, sdq = query_codes(qt, mu)
    sink = max(0, min(int(sink_leaves), nb))
    kx = min(int(exact_leaves) + sink, nb)
    sel = rowmax_select(dq8, sdq, g8, sg, lz) if kx > 0 else np.zeros((len(tiles), nb), F32)
    idx, excl = route(sel, exact_leaves, sink)
    return tile_attention(qt, q8, sq, dq8, sdq, g8, sg, lz, vb, excl, idx, prep["k8"], prep["ks"], v, leaf, scale,
                          tail=tail)


def flat_attention_tiles(q, k, v, tiles, *, tile=64, exact_leaves=256, leaf=64, scale=None, sink_leaves=0,
                         tail=None):
    """``prepare_head`` + ``attention_tiles`` in one call."""
    return attention_tiles(prepare_head(q, k, v, tile=tile, leaf=leaf), tiles, exact_leaves=exact_leaves,
                           scale=scale, sink_leaves=sink_leaves, tail=tail)


def flat_attention_f32(q, k, v, *, tile=64, exact_leaves=64, leaf=16, scale=None, curvature="lin"):
    """The reference's float32 specification of the operator (the torch backend, h3/htrc_flat.py:279-388),
    evaluated in float64: exact leaf cumulants at the tile centres (real rows only), far logits
    lz + dq.g (+ the isotropic curvature 0.5/D max(tr, 0) |dq|^2 with curvature="iso", :331-333), the
    exact_leaves leaves with the largest row-maximum logit evaluated exactly, both parts merged.  No INT8
    and no bf16 rounding (the production path's quantisation is not part of this specification)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    n, d = q.shape
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    nb = k.shape[0] // leaf
    k3 = k[: nb * leaf].reshape(nb, leaf, d)
    v3 = v[: nb * leaf].reshape(nb, leaf, d)
    nt = -(-n // tile)
    qs = np.concatenate([q, np.repeat(q[-1:], nt * tile - n, 0)], 0) if nt * tile > n else q
    qt = qs.reshape(nt, tile, d)
    out = np.zeros((nt, tile, d))
    kx = min(int(exact_leaves), nb)
    for t in range(nt):
        real = min(tile, n - t * tile)
        mu = qt[t, :real].mean(0)
        a = np.einsum("d,lsd->ls", mu, k3) * scale
        m = a.max(-1, keepdims=True)
        w = np.exp(a - m)
        z = w.sum(-1, keepdims=True)
        w /= z
        lz = (m + np.log(z))[:, 0]
        g = np.einsum("ls,lsd->ld", w, k3) * scale
        vb = np.einsum("ls,lsd->ld", w, v3)
        dq = qt[t] - mu[None, :]
        lg = dq @ g.T + lz[None, :]
        if curvature == "iso":
            tr = (w * (k3 * k3).sum(-1)).sum(-1) * scale * scale - (g * g).sum(-1)
            lg = lg + 0.5 / d * np.maximum(tr, 0.0)[None, :] * (dq * dq).sum(-1)[:, None]
        parts_s, parts_v = [], []
        keep = np.ones(nb, bool)
        if kx > 0:
            idx = np.argsort(-lg.max(0), kind="stable")[:kx]
            keep[idx] = False
            tok = (idx[:, None] * leaf + np.arange(leaf)[None, :]).reshape(-1)
            parts_s.append(qt[t] @ k[tok].T * scale)
            parts_v.append(v[tok])
        if keep.any():
            parts_s.append(lg[:, keep])
            parts_v.append(vb[keep])
        s_ = np.concatenate(parts_s, 1)
        vv = np.concatenate(parts_v, 0)
        p_ = np.exp(s_ - s_.max(1, keepdims=True))
        out[t] = p_ @ vv / p_.sum(1, keepdims=True)
    return out.reshape(nt * tile, d)[:n].astype(F32)


def exact_attention(q, k, v, scale=None, tail=None):
    """Dense softmax attention in float64 (for reporting the operator's approximation error):
    returns (out float32 [N, D], lse float32 [N])."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    if tail is not None and tail[0].shape[0]:
        k = np.concatenate([k, np.asarray(tail[0], np.float64)], 0)
        v = np.concatenate([v, np.asarray(tail[1], np.float64)], 0)
    scale = 1.0 / math.sqrt(q.shape[1]) if scale is None else float(scale)
    s = (q @ k.T) * scale
    m = s.max(1, keepdims=True)
    p = np.exp(s - m)
    den = p.sum(1, keepdims=True)
    return (p @ v / den).astype(F32), (m[:, 0] + np.log(den[:, 0])).astype(F32)
