"""GPU parity of the query-order and grouping options of the flat operator against the CPU oracle and the
reference's fixtures, through the C ABI:

* ``order="kmeans"`` (accurate / max modes, h3/htrc_flat.py:47-65, :146-147, :159-165): the device
  permutation against the reference's recorded one and the oracle's, then every stage after it;
* ``kern={"group": G}`` (h3/htrc_flat.py:223-231): G consecutive tiles share one centre, far-field
  state row and routing;
* ``tile=32`` (the max mode, h3/htrc_flat_runner.py:52): 32-row tiles, held as 64 rows.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import flat_oracle as O  # noqa: E402

OUT_TOL = 2e-2
LSE_TOL = 1e-3
ROUTE_AGREE = 0.999


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from htrc_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


def _inputs(grid, seed):
    from htrc_b200 import synth
    return synth.head_inputs(grid, 128, base_seed=seed)


def _np(t):
    return t.detach().float().cpu().numpy() if t.dtype in (torch.bfloat16, torch.float16) else t.detach().cpu().numpy()


def _device_perm(q, dtype):
    from htrc_b200 import _lib
    from htrc_b200._lib import lib, ptr, stream_ptr
    n = int(q.shape[0])
    nbytes = ctypes.c_size_t()
    _lib.check(lib().htrc_kmeans_scratch_size(n, nbytes), "scratch size")
    scratch = torch.empty(int(nbytes.value), dtype=torch.uint8, device=q.device)
    perm = torch.full((n,), -1, dtype=torch.int32, device=q.device)
    code = _lib.DTYPE_BF16 if dtype == torch.bfloat16 else _lib.DTYPE_F32
    qd = q.to(dtype).contiguous()
    _lib.check(lib().htrc_kmeans_order(ptr(qd), code, n, 128, ptr(perm), ptr(scratch), int(nbytes.value),
                                       stream_ptr()), "kmeans order")
    torch.cuda.synchronize()
    return perm.cpu().numpy().astype(np.int64)


KMEANS_FIXTURES = ["kmeans", "kmeans_g2_tail", "kmeans_sampled", "max_mode"]
GROUP_FIXTURES = ["group2", "group4"]
TILE32_FIXTURES = ["tile32", "tile32_g2"]


def _tile(z):
    return int(z["tile"]) if "tile" in z else 64


@pytest.mark.parametrize("case", KMEANS_FIXTURES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_kmeans_order_equals_reference_permutation(dev, golden_cases, case, dtype):
    z = golden_cases[case]
    q = torch.from_numpy(z["q"]).to(dev)
    assert np.array_equal(_device_perm(q, dtype), z["perm"])


@pytest.mark.parametrize("grid,seed", [((16, 32, 64), 81), ((4, 8, 8), 82), ((1, 1, 7), 83)])
def test_kmeans_order_against_oracle(dev, grid, seed):
    """A permutation, sorted by the oracle's cluster labels (stable), except where a row sits at a
    near-tie between two centres (float32 device distances vs float64 oracle distances)."""
    q, _, _ = _inputs(grid, seed)
    n = q.shape[0]
    p = _device_perm(q.to(dev), torch.bfloat16)
    assert np.array_equal(np.sort(p), np.arange(n))
    ref, labels = O.kmeans_order(q.float().numpy(), return_labels=True)
    if np.array_equal(p, ref):
        return
    lab = labels[p]
    bad = (np.diff(lab) < 0) | ((np.diff(lab) == 0) & (np.diff(p) < 0))
    assert bad.sum() <= max(2, n // 10000), bad.sum()


def _check(out, lse, excl_dev, z_out, z_lse, z_excl, n, group, perm, tile=64):
    """Routing agreement >= 99.9% of (group, leaf) pairs; out max-abs on the rows of groups whose
    routing agrees (rows mapped through the permutation); log-Z mean-abs over all rows."""
    agree = (excl_dev == z_excl).mean()
    assert agree >= ROUTE_AGREE, agree
    same_tile_rows = np.repeat((excl_dev == z_excl).all(1), tile * group)[:n]
    rows = np.arange(n) if perm is None else np.asarray(perm)[:n]
    o = out.cpu().numpy()
    err = np.abs(o[rows[same_tile_rows]] - z_out[rows[same_tile_rows]]).max()
    assert err < OUT_TOL, err
    if z_lse is not None:
        assert np.abs(lse.cpu().numpy() - z_lse).mean() < LSE_TOL


@pytest.mark.parametrize("case", GROUP_FIXTURES + KMEANS_FIXTURES + TILE32_FIXTURES)
def test_end_to_end_against_reference_fixtures(dev, golden_cases, case):
    """The whole operator with kern group / order="kmeans" against outputs recorded from the reference."""
    import htrc_b200
    z = golden_cases[case]
    q = torch.from_numpy(z["q"]).to(torch.bfloat16).to(dev)
    k = torch.from_numpy(z["k"]).to(torch.bfloat16).to(dev)
    v = torch.from_numpy(z["v"]).to(torch.bfloat16).to(dev)
    tail = None
    if "tail_k" in z:
        tail = (torch.from_numpy(z["tail_k"]).to(dev), torch.from_numpy(z["tail_v"]).to(dev))
    g = int(z["group"])
    order = "kmeans" if "perm" in z else "seq"
    # the fixtures were recorded by Triton's interpreter, which evaluates the tf32 dots in float32
    cfg = {**htrc_b200.PROD, "leaf": 64, "exact_leaves": int(z["exact_leaves"]), "sink_leaves": int(z["sink_leaves"]),
           "order": order, "kern": {**htrc_b200.PROD["kern"], "group": g}, "tile": _tile(z), "precision": "fp32"}
    out, lse = htrc_b200.flat_attention(q, k, v, tail=tail, return_lse=True, **cfg)
    st = htrc_b200.run_stages(q, k, v, tail[0] if tail else None, tail[1] if tail else None,
                              exact_leaves=cfg["exact_leaves"], sink_leaves=cfg["sink_leaves"], group=g,
                              order=htrc_b200.flat.order_code(order), tile=_tile(z), precision=0)
    torch.cuda.synchronize()
    assert torch.equal(out, st["out"]) and torch.equal(lse, st["lse"])
    assert int(st["status"].item()) == 0
    n = z["q"].shape[0]
    perm = None
    if order == "kmeans":
        perm = _np(st["perm"]).astype(np.int64)
        assert np.array_equal(perm, z["perm"])
    nb = st["nb"]
    _check(out, lse, _np(st["excl"])[:, :nb], z["out"], z.get("lse"), z["excl"], n, g, perm, _tile(z))


def _held(x, nt, tile):
    """Device rows [nt * 64, ...] -> the oracle's [nt, tile, ...] (a 32-row tile is held as 64 rows)."""
    x = _np(x)
    return x.reshape(nt, 64, *x.shape[1:])[:, :tile]


def _oracle_on_device_state(q, v, st, group, perm, tail=None, tile=64):
    """The oracle's far + near attention on the device's own stage outputs, in the caller's row order."""
    nb, kx = st["nb"], st["kx"]
    qf = q.float().numpy()
    if perm is not None:
        qf = qf[perm]
    qt, _, n = O.tile_centres(qf, tile)
    nt = qt.shape[0]
    out, lse = O.tile_attention(qt, _held(st["q8"], nt, tile), _held(st["sq"], nt, tile),
                                _held(st["dq8"], nt, tile), _held(st["sdq"], nt, tile), _np(st["g8"]),
                                _np(st["sg"])[:, :nb], _np(st["lz"])[:, :nb], _np(st["vb"]), _np(st["excl"])[:, :nb],
                                _np(st["idx"])[:, :kx], _np(st["k8"]), _np(st["ks"]), O.bf16_round(v.float().numpy()),
                                64, 1 / math.sqrt(128), tail=tail, group=group)
    out, lse = out[:n], lse[:n]
    if perm is not None:
        fo, fl = np.empty_like(out), np.empty_like(lse)
        fo[perm], fl[perm] = out, lse
        out, lse = fo, fl
    return out, lse


@pytest.mark.parametrize("grid,seed,E,group,trim,order,tile", [
    ((4, 16, 32), 91, 6, 2, 0, "seq", 64), ((4, 16, 32), 92, 6, 3, 70, "seq", 64),
    ((4, 16, 32), 93, 9, 4, 0, "seq", 64), ((4, 16, 32), 94, 5, 1, 13, "kmeans", 64),
    ((4, 16, 32), 95, 8, 2, 0, "kmeans", 64), ((4, 16, 32), 96, 6, 1, 11, "seq", 32),
    ((4, 16, 32), 97, 7, 2, 40, "kmeans", 32)])
def test_stages_on_device_state(dev, grid, seed, E, group, trim, order, tile):
    """Group centres and query codes bit-exact; fed the device's own state, selection and routing equal
    the oracle's formulas bit for bit and far + near attention matches the oracle."""
    import htrc_b200
    q, k, v = _inputs(grid, seed)
    if trim:
        q = q[:-trim]
    oc = htrc_b200.flat.order_code(order)
    st = htrc_b200.run_stages(q.to(dev), k.to(dev), v.to(dev), exact_leaves=E, group=group, order=oc, tile=tile)
    torch.cuda.synchronize()
    assert int(st["status"].item()) == 0
    perm = _np(st["perm"]).astype(np.int64) if order == "kmeans" else None
    if perm is not None:
        assert np.array_equal(np.sort(perm), np.arange(q.shape[0]))
    qf = q.float().numpy() if perm is None else q.float().numpy()[perm]
    qt, mu1, _ = O.tile_centres(qf, tile)
    mu = O.group_centres(qt, group) if group > 1 else mu1
    assert np.array_equal(_np(st["mu"]).view(np.uint32), mu.view(np.uint32))
    nt, nb = qt.shape[0], st["nb"]
    q8, sq, dq8, sdq = O.query_codes(qt, mu[np.arange(nt) // group])
    assert np.array_equal(_held(st["q8"], nt, tile), q8)
    assert np.array_equal(_held(st["dq8"], nt, tile), dq8)
    assert np.array_equal(_held(st["sdq"], nt, tile).view(np.uint32), sdq.view(np.uint32))
    if tile == 32:                                   # held rows 32..63 repeat row 31
        held = _np(st["dq8"]).reshape(nt, 64, 128)
        assert (held[:, 32:] == held[:, 31:32]).all()
    gt = np.arange(nt) // group
    g8, sg, lz = _np(st["g8"]), _np(st["sg"])[:, :nb], _np(st["lz"])[:, :nb]
    per_tile = O.rowmax_select(dq8, sdq, g8[gt], sg[gt], lz[gt])
    assert np.array_equal(_np(st["sel"])[:nt, :nb].view(np.uint32), per_tile.view(np.uint32))
    sel = O.rowmax_select(dq8, sdq, g8, sg, lz, group)
    idx, excl = O.route(sel, E)
    assert np.array_equal(_np(st["idx"])[:, :idx.shape[1]], idx)
    assert np.array_equal(_np(st["excl"])[:, :nb], excl)
    out, lse = _oracle_on_device_state(q, v, st, group, perm, tile=tile)
    assert np.abs(_np(st["out"]) - out).max() < OUT_TOL
    assert np.abs(_np(st["lse"]) - lse).mean() < LSE_TOL


@pytest.mark.parametrize("group,order,chunk,tile", [(2, "seq", 6, 64), (3, "seq", 7, 64), (1, "kmeans", 10, 64),
                                                     (4, "kmeans", 9, 64), (1, "seq", 5, 32), (2, "kmeans", 8, 32)])
def test_chunked_forward_equals_staged(dev, group, order, chunk, tile):
    """The single-call forward with chunked state (groups per chunk = tile_chunk // G) equals the staged
    path; the tail partial is read in the caller's row order."""
    import htrc_b200
    q, k, v = _inputs((4, 16, 40), 101)
    tk, tv = k[-9:].float().to(dev), v[-9:].float().to(dev)
    qd, kd, vd = q.to(dev), k[:-64].to(dev), v[:-64].to(dev)
    cfg = {**htrc_b200.PROD, "leaf": 64, "exact_leaves": 5, "order": order, "tile": tile,
           "kern": {**htrc_b200.PROD["kern"], "group": group}}
    a, la = htrc_b200.flat_attention(qd, kd, vd, tail=(tk, tv), return_lse=True, **{**cfg, "tile_chunk": 0})
    b, lb = htrc_b200.flat_attention(qd, kd, vd, tail=(tk, tv), return_lse=True, **{**cfg, "tile_chunk": chunk})
    st = htrc_b200.run_stages(qd, kd, vd, tk, tv, exact_leaves=5, group=group, order=htrc_b200.flat.order_code(order),
                              tile=tile)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(la, lb)
    assert torch.equal(a, st["out"]) and torch.equal(la, st["lse"])
    perm = _np(st["perm"]).astype(np.int64) if order == "kmeans" else None
    out, lse = _oracle_on_device_state(q, v[:-64], st, group, perm, tail=(tk.cpu().numpy(), tv.cpu().numpy()),
                                       tile=tile)
    assert np.abs(a.cpu().numpy() - out).max() < OUT_TOL


@pytest.mark.parametrize("mode", ["accurate", "max"])
def test_runner_kmeans_modes(dev, mode):
    """FlatRunner(mode="accurate" / "max"): k-means order with 1024 routed leaves (tile 64 / 32),
    captured in a CUDA graph."""
    import htrc_b200
    from htrc_b200 import runner
    q, k, v = _inputs((8, 32, 48), 111)
    n = q.shape[0]
    r = runner.FlatRunner(n, n, mode=mode, lse=True, leaf=64)
    assert r.graph is not None, r.graph_error
    out, lse = r.head(q.to(dev), k.to(dev), v.to(dev))
    ref, rl = htrc_b200.flat_attention(q.to(dev), k.to(dev), v.to(dev), return_lse=True,
                                       **{**htrc_b200.PROD, **runner.MODES[mode], "leaf": 64})
    torch.cuda.synchronize()
    assert torch.equal(out, ref) and torch.equal(lse, rl)
    r.check_status()
    # 192 leaves, all routed: every row is exact INT8 attention, whatever tile the permutation puts it in
    ro, rl = O.flat_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), exact_leaves=1024)
    assert np.abs(out.cpu().numpy() - ro).max() < OUT_TOL
    assert np.abs(lse.cpu().numpy() - rl).mean() < LSE_TOL
    r.close()


@pytest.mark.parametrize("grid,seed,E,group,order,tile", [((4, 16, 32), 121, 6, 1, "seq", 64),
                                                          ((4, 16, 32), 122, 5, 2, "kmeans", 64),
                                                          ((4, 16, 32), 123, 7, 1, "seq", 32)])
def test_iso_curvature_on_device_state(dev, grid, seed, E, group, order, tile):
    """curvature="iso" (the torch backend's isotropic second-order far-field term, on the INT8 path): key
    norms, row offsets and curvature coefficients against the oracle; fed the device's own state, the
    selection and routing bit for bit and far + near attention within the tolerance."""
    import htrc_b200
    from htrc_b200 import _lib
    q, k, v = _inputs(grid, seed)
    st = htrc_b200.run_stages(q.to(dev), k.to(dev), v.to(dev), exact_leaves=E, group=group,
                              order=htrc_b200.flat.order_code(order), tile=tile, curvature=_lib.CURV_ISO,
                              precision=_lib.PREC_FP32)
    torch.cuda.synchronize()
    assert int(st["status"].item()) == 0
    perm = _np(st["perm"]).astype(np.int64) if order == "kmeans" else None
    kb = O.bf16_round(k.float().numpy())
    assert np.allclose(_np(st["kn2"]), (kb.astype(np.float64) ** 2).sum(1), rtol=1e-6)
    qf = q.float().numpy() if perm is None else q.float().numpy()[perm]
    qt, mu1, _ = O.tile_centres(qf, tile)
    mu = O.group_centres(qt, group) if group > 1 else mu1
    nt, nb = qt.shape[0], st["nb"]
    mu_t = mu[np.arange(nt) // group]
    assert np.allclose(_held(st["dd"], nt, tile), O.offset_sqnorm(qt, mu_t), rtol=1e-5, atol=1e-6)
    cv = _np(st["cv"])[:, :nb]
    want = O.iso_coeff(mu, kb, 64, 1 / math.sqrt(128))
    assert np.allclose(cv, want, rtol=2e-3, atol=2e-5), np.abs(cv - want).max()
    dq8 = _held(st["dq8"], nt, tile)
    sdq = _held(st["sdq"], nt, tile)
    dd = _held(st["dd"], nt, tile)
    gt = np.arange(nt) // group
    g8, sg, lz = _np(st["g8"]), _np(st["sg"])[:, :nb], _np(st["lz"])[:, :nb]
    per_tile = O.rowmax_select(dq8, sdq, g8[gt], sg[gt], lz[gt], 1, cv[gt], dd)
    assert np.array_equal(_np(st["sel"])[:nt, :nb].view(np.uint32), per_tile.view(np.uint32))
    idx, excl = O.route(O.rowmax_select(dq8, sdq, g8, sg, lz, group, cv, dd), E)
    assert np.array_equal(_np(st["idx"])[:, :idx.shape[1]], idx)
    assert np.array_equal(_np(st["excl"])[:, :nb], excl)
    out, lse = O.tile_attention(qt, _held(st["q8"], nt, tile), _held(st["sq"], nt, tile), dq8, sdq, g8, sg, lz,
                                _np(st["vb"]), excl, idx, _np(st["k8"]), _np(st["ks"]),
                                O.bf16_round(v.float().numpy()), 64, 1 / math.sqrt(128), group=group, cv=cv, dd=dd)
    n = q.shape[0]
    out, lse = out[:n], lse[:n]
    if perm is not None:
        fo, fl = np.empty_like(out), np.empty_like(lse)
        fo[perm], fl[perm] = out, lse
        out, lse = fo, fl
    assert np.abs(_np(st["out"]) - out).max() < OUT_TOL
    assert np.abs(_np(st["lse"]) - lse).mean() < LSE_TOL


def test_iso_curvature_end_to_end(dev):
    """flat_attention(backend="cuda", curvature="iso") and FlatRunner against the oracle computing its own
    statistics (routing agreement, output and log-Z tolerances); backend="triton" rejects it like the
    reference."""
    import htrc_b200
    from htrc_b200 import runner
    q, k, v = _inputs((8, 32, 32), 131)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    # the isotropic term is the reference's float32 torch-backend semantics: float32-accurate statistics
    cfg = {**htrc_b200.PROD, "leaf": 64, "exact_leaves": 24, "backend": "cuda", "curvature": "iso", "precision": "fp32"}
    out, lse = htrc_b200.flat_attention(qd, kd, vd, return_lse=True, **cfg)
    with pytest.raises(ValueError, match="curvature='lin'"):
        htrc_b200.flat_attention(qd, kd, vd, **{**cfg, "backend": "triton"})
    r = runner.FlatRunner(q.shape[0], k.shape[0], mode="fast", backend="cuda", curvature="iso", lse=True,
                          exact_leaves=24, precision="fp32", leaf=64)
    assert r.graph is not None, r.graph_error
    o2, l2 = r.head(qd, kd, vd)
    torch.cuda.synchronize()
    assert torch.equal(o2, out) and torch.equal(l2, lse)
    ro, rl, rst = O.flat_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), exact_leaves=24,
                                   curvature="iso", return_stages=True)
    st = htrc_b200.run_stages(qd, kd, vd, exact_leaves=24, curvature=htrc_b200.flat.curvature_code("iso"),
                              precision=0)
    torch.cuda.synchronize()
    nb = st["nb"]
    ex = _np(st["excl"])[:, :nb]
    assert (ex == rst["excl"]).mean() >= ROUTE_AGREE
    same = np.repeat((ex == rst["excl"]).all(1), 64)[:q.shape[0]]
    err = np.abs(out.cpu().numpy()[same] - ro[same]).max(1)
    assert (err < OUT_TOL).mean() >= 0.999 and err.max() < 2.5 * OUT_TOL
    assert np.abs(lse.cpu().numpy() - rl).mean() < LSE_TOL
    r.close()
