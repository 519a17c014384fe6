"""GPU parity of every stage of libhtrc_flat against the CPU oracle (oracle/flat_oracle.py), on the same
seeded inputs, through the C ABI.  Bit-exact for the INT8 codes and scales and for the integer/index
stages fed identical inputs; within the operator tolerance (out max-abs 2e-2, log-Z mean-abs 1e-3,
routing agreement >= 99.9%) end to end."""
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
    import htrc_b200  # noqa: F401
    from htrc_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


def _inputs(grid, seed):
    from htrc_b200 import synth
    return synth.head_inputs(grid, 128, base_seed=seed)


def _np(t):
    return t.detach().float().cpu().numpy() if t.dtype in (torch.bfloat16, torch.float16) else t.detach().cpu().numpy()


def test_key_pack_bit_exact(dev):
    from htrc_b200 import _lib
    from htrc_b200._lib import lib, ptr, stream_ptr
    g = torch.Generator().manual_seed(3)
    k = (torch.randn(4096, 128, generator=g) * torch.rand(4096, 1, generator=g) * 5).to(torch.bfloat16)
    k[17] = 0                                                     # all-zero row: scale floor 1e-20
    kd = k.to(dev)
    k8 = torch.empty((4096, 128), dtype=torch.int8, device=dev)
    ks = torch.empty((4096,), dtype=torch.float32, device=dev)
    kn2 = torch.empty((4096,), dtype=torch.float32, device=dev)
    _lib.check(lib().htrc_pack_int8(ptr(kd), _lib.DTYPE_BF16, 4096, 128, _lib.ROUND_HALF_EVEN, ptr(k8), ptr(ks),
                                    ptr(kn2), stream_ptr()), "pack")
    torch.cuda.synchronize()
    rk8, rks = O.pack_rows_half_even(k.float().numpy())
    assert np.array_equal(k8.cpu().numpy(), rk8)
    assert np.array_equal(ks.cpu().numpy().view(np.uint32), rks.view(np.uint32))
    assert np.allclose(kn2.cpu().numpy(), (k.double().numpy() ** 2).sum(1), rtol=1e-6)   # the iso key norms


def test_half_away_pack_bit_exact(dev):
    from htrc_b200 import _lib
    from htrc_b200._lib import lib, ptr, stream_ptr
    g = torch.Generator().manual_seed(4)
    x = torch.randn(2048, 128, generator=g) * torch.rand(2048, 1, generator=g) * 3
    x[5, :] = 0.0
    x[6, 3] = 1e-19
    xd = x.to(dev)
    x8 = torch.empty((2048, 128), dtype=torch.int8, device=dev)
    s = torch.empty((2048,), dtype=torch.float32, device=dev)
    _lib.check(lib().htrc_pack_int8(ptr(xd), _lib.DTYPE_F32, 2048, 128, _lib.ROUND_HALF_AWAY, ptr(x8), ptr(s), None,
                                    stream_ptr()), "pack")
    torch.cuda.synchronize()
    r8, rs = O.pack_rows_half_away(x.numpy())
    assert np.array_equal(x8.cpu().numpy(), r8)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))


@pytest.mark.parametrize("n", [1024, 1000, 64, 37])
@pytest.mark.parametrize("precision", ["fp32", "tf32"])
def test_tile_prep_bit_exact(dev, n, precision):
    import htrc_b200
    from htrc_b200 import _lib
    q, k, v = _inputs((2, 16, 32), 21)
    q = q[:n]
    st = htrc_b200.run_stages(q.to(dev), k.to(dev), v.to(dev), exact_leaves=2, precision=_lib.PRECISIONS[precision])
    torch.cuda.synchronize()
    qt, mu, _ = O.tile_centres(q.float().numpy(), 64)
    assert np.array_equal(_np(st["mu"]).view(np.uint32), mu.view(np.uint32))
    q8, sq, dq8, sdq = O.query_codes(qt, mu)
    nt = qt.shape[0]
    assert np.array_equal(_np(st["q8"]).reshape(nt, 64, 128), q8)
    assert np.array_equal(_np(st["dq8"]).reshape(nt, 64, 128), dq8)
    assert np.array_equal(_np(st["sq"]).reshape(nt, 64).view(np.uint32), sq.view(np.uint32))
    assert np.array_equal(_np(st["sdq"]).reshape(nt, 64).view(np.uint32), sdq.view(np.uint32))
    hi = _np(st["mu_hi"])
    lo = _np(st["mu_lo"])
    if precision == "tf32":                  # hi + lo is the centre's tf32 operand value, exactly
        assert np.array_equal((hi.astype(np.float64) + lo).astype(np.float32), O.tf32_operand(mu))
        return
    assert np.array_equal(hi, O.bf16_round(mu))
    assert np.abs(hi.astype(np.float64) + lo - mu).max() <= 2.0 ** -16 * np.abs(mu).max()


@pytest.mark.parametrize("grid,seed", [((2, 16, 32), 31), ((4, 16, 32), 32)])
@pytest.mark.parametrize("precision", ["fp32", "tf32"])
def test_leaf_stats(dev, grid, seed, precision):
    """lz, sg, g8 and vbar against the oracle at the same precision setting (tf32: the centre and the softmax
    weights enter the dots as tf32 operand values)."""
    import htrc_b200
    from htrc_b200 import _lib
    q, k, v = _inputs(grid, seed)
    st = htrc_b200.run_stages(q.to(dev), k.to(dev), v.to(dev), exact_leaves=2, precision=_lib.PRECISIONS[precision])
    torch.cuda.synchronize()
    nb = st["nb"]
    mu = _np(st["mu"])
    g, lz, vb = O.leaf_stats(mu, O.bf16_round(k.float().numpy()), O.bf16_round(v.float().numpy()), 64,
                             1 / math.sqrt(128), precision)
    g8, sg = O.pack_slope(g)
    lz_d = _np(st["lz"])[:, :nb]
    sg_d = _np(st["sg"])[:, :nb]
    assert np.abs(lz_d - lz).max() < 2e-4
    assert np.abs(sg_d / sg - 1).max() < 2e-3
    d = np.abs(_np(st["g8"]).astype(int) - g8.astype(int))
    assert d.max() <= 1 and (d > 0).mean() < 2e-3
    vbd = _np(st["vb"])
    assert np.abs(vbd - O.bf16_round(vb)).max() <= 2.0 ** -7 * max(1.0, np.abs(vb).max())


@pytest.mark.parametrize("grid,seed,E", [((2, 16, 32), 41, 4), ((4, 16, 32), 42, 7)])
def test_rowmax_and_route_bit_exact_on_device_state(dev, grid, seed, E):
    """Fed the device's own state, selection and routing equal the oracle's formulas bit for bit."""
    import htrc_b200
    q, k, v = _inputs(grid, seed)
    st = htrc_b200.run_stages(q.to(dev), k.to(dev), v.to(dev), exact_leaves=E)
    torch.cuda.synchronize()
    nb, nt = st["nb"], st["mu"].shape[0]
    dq8 = _np(st["dq8"]).reshape(nt, 64, 128)
    sdq = _np(st["sdq"]).reshape(nt, 64)
    sel = O.rowmax_select(dq8, sdq, _np(st["g8"]), _np(st["sg"])[:, :nb], _np(st["lz"])[:, :nb])
    assert np.array_equal(_np(st["sel"])[:, :nb].view(np.uint32), sel.view(np.uint32))
    idx, excl = O.route(sel, E)
    assert np.array_equal(_np(st["idx"])[:, :idx.shape[1]], idx)
    assert np.array_equal(_np(st["excl"])[:, :nb], excl)


def test_route_sink_and_ties(dev):
    from htrc_b200 import _lib
    from htrc_b200._lib import lib, ptr, stream_ptr
    nb = 40
    pitch = int(lib().htrc_leaf_pitch(nb))
    sel = torch.zeros((3, pitch), dtype=torch.float32)
    sel[0, :nb] = torch.arange(nb, dtype=torch.float32) % 7          # many ties
    sel[1, :nb] = -torch.arange(nb, dtype=torch.float32)
    sel[2, :nb] = torch.randn(nb, generator=torch.Generator().manual_seed(1))
    for E, sink in [(5, 0), (5, 3), (0, 2), (38, 0), (40, 1), (0, 0)]:
        kx = min(E + sink, nb)
        idx = torch.full((3, max(kx, 1)), -1, dtype=torch.int32, device=dev)
        excl = torch.full((3, pitch), 9, dtype=torch.uint8, device=dev)
        _lib.check(lib().htrc_route(ptr(sel.to(dev)), 3, nb, E, sink, 1, ptr(idx), ptr(excl), stream_ptr()), "route")
        torch.cuda.synchronize()
        ridx, rex = O.route(sel[:, :nb].numpy(), E, sink)
        assert np.array_equal(excl.cpu().numpy()[:, :nb], rex), (E, sink)
        assert (excl.cpu().numpy()[:, nb:] == 0).all()
        if kx:
            assert np.array_equal(idx.cpu().numpy()[:, :kx], ridx), (E, sink)


@pytest.mark.parametrize("grid,seed,E,trim", [((2, 16, 32), 51, 4, 0), ((2, 16, 32), 52, 16, 0),
                                              ((2, 16, 32), 53, 0, 0), ((4, 16, 32), 54, 9, 70)])
def test_tile_attention_on_device_state(dev, grid, seed, E, trim):
    """Fed the device's own stage outputs, far+near attention matches the order-free oracle."""
    import htrc_b200
    q, k, v = _inputs(grid, seed)
    if trim:
        q = q[:-trim]
    st = htrc_b200.run_stages(q.to(dev), k.to(dev), v.to(dev), exact_leaves=E)
    torch.cuda.synchronize()
    nb, nt = st["nb"], st["mu"].shape[0]
    kx = st["kx"]
    qt, _, n = O.tile_centres(q.float().numpy(), 64)
    out, lse = O.tile_attention(qt, _np(st["q8"]).reshape(nt, 64, 128), _np(st["sq"]).reshape(nt, 64),
                                _np(st["dq8"]).reshape(nt, 64, 128), _np(st["sdq"]).reshape(nt, 64), _np(st["g8"]),
                                _np(st["sg"])[:, :nb], _np(st["lz"])[:, :nb], _np(st["vb"]),
                                _np(st["excl"])[:, :nb], _np(st["idx"])[:, :kx], _np(st["k8"]), _np(st["ks"]),
                                O.bf16_round(v.float().numpy()), 64, 1 / math.sqrt(128))
    od, ld = _np(st["out"]), _np(st["lse"])
    assert np.isfinite(od).all() and np.isfinite(ld).all()
    assert np.abs(od - out[:n]).max() < OUT_TOL
    assert np.abs(ld - lse[:n]).mean() < LSE_TOL
    assert int(st["status"].item()) == 0


GOLDEN64 = ["base", "ragged", "sink_tail", "all_exact", "no_exact", "big_tail", "wide"]


def _check_against(out, lse, st, ref_out, ref_lse, ref_excl, ref_sel, n, kx, oracle_on_device_state, strict=True):
    """Operator parity in the presence of routing: agreement >= 99.9% of (tile, leaf) pairs; every
    disagreement a near-tie at the selection threshold; out max-abs on the tiles whose routing agrees;
    log-Z mean-abs over all rows; and, fed the device's own stage outputs, the oracle matches every row."""
    nb = st["nb"]
    ex = _np(st["excl"])[:, :nb]
    agree = (ex == ref_excl).mean()
    assert agree >= ROUTE_AGREE, agree
    flips = np.argwhere(ex != ref_excl)
    if len(flips) and ref_sel is not None:
        srt = -np.sort(-ref_sel, axis=1)
        for t, l in flips:
            thr = srt[t, kx - 1]
            assert abs(ref_sel[t, l] - thr) <= 2e-2 * max(1.0, abs(thr)), (t, l, ref_sel[t, l], thr)
    same = np.repeat((ex == ref_excl).all(1), 64)[:n]
    o = out.cpu().numpy()
    err = np.abs(o[same] - ref_out[same]).max(1)
    if strict:
        assert err.max() < OUT_TOL
    else:
        # independent leaf statistics: a one-LSB slope-code flip moves a far logit by up to
        # |dq|max * |g|max / 127, so a few far-dominated rows may pass 2e-2 (the reference's own GPU operator
        # is 0.031 max-abs from the same float64 restatement on sampled full-size tiles)
        assert (err < OUT_TOL).mean() >= 0.999 and err.max() < 2.5 * OUT_TOL, (err.max(), (err >= OUT_TOL).sum())
    if ref_lse is not None:
        assert np.abs(lse.cpu().numpy() - ref_lse).mean() < LSE_TOL
    if oracle_on_device_state is not None:
        o2, _ = oracle_on_device_state
        assert np.abs(o - o2[:n]).max() < OUT_TOL


def _oracle_on_device_state(q, v, st, tail):
    """The oracle's far + near attention evaluated on the device's own stage outputs (identical inputs)."""
    nb, kx, nt = st["nb"], st["kx"], st["mu"].shape[0]
    qt, _, _ = O.tile_centres(q.float().numpy(), 64)
    return O.tile_attention(qt, _np(st["q8"]).reshape(nt, 64, 128), _np(st["sq"]).reshape(nt, 64),
                            _np(st["dq8"]).reshape(nt, 64, 128), _np(st["sdq"]).reshape(nt, 64), _np(st["g8"]),
                            _np(st["sg"])[:, :nb], _np(st["lz"])[:, :nb], _np(st["vb"]), _np(st["excl"])[:, :nb],
                            _np(st["idx"])[:, :kx], _np(st["k8"]), _np(st["ks"]), O.bf16_round(v.float().numpy()), 64,
                            1 / math.sqrt(128), tail=tail)


@pytest.mark.parametrize("case", GOLDEN64)
def test_end_to_end_against_reference_fixtures(dev, golden_cases, case):
    """The whole operator against outputs recorded from the reference itself."""
    import htrc_b200
    z = golden_cases[case]
    q = torch.from_numpy(z["q"]).to(torch.bfloat16).to(dev)
    k = torch.from_numpy(z["k"]).to(torch.bfloat16).to(dev)
    v = torch.from_numpy(z["v"]).to(torch.bfloat16).to(dev)
    tail = None
    if "tail_k" in z:
        tail = (torch.from_numpy(z["tail_k"]).to(dev), torch.from_numpy(z["tail_v"]).to(dev))
    # the fixtures were recorded by Triton's interpreter, which evaluates the tf32 dots in float32
    cfg = {**htrc_b200.PROD, "leaf": 64, "exact_leaves": int(z["exact_leaves"]), "sink_leaves": int(z["sink_leaves"]),
           "precision": "fp32"}
    out, lse = htrc_b200.flat_attention(q, k, v, tail=tail, return_lse=True, **cfg)
    st = htrc_b200.run_stages(q, k, v, tail[0] if tail else None, tail[1] if tail else None,
                              exact_leaves=cfg["exact_leaves"], sink_leaves=cfg["sink_leaves"], precision=0)
    torch.cuda.synchronize()
    assert np.array_equal(_np(st["k8"]), z["k8"])
    assert np.array_equal(_np(st["ks"]).view(np.uint32), z["ks"].view(np.uint32))
    assert torch.equal(out, st["out"])
    n = z["q"].shape[0]
    _check_against(out, lse, st, z["out"], z.get("lse"), z["excl"], z.get("sel"), n, st["kx"], None)


@pytest.mark.parametrize("grid,seed,E,sink,ntail,drop", [((8, 32, 32), 61, 16, 0, 0, 0), ((8, 32, 32), 62, 40, 2, 9, 64),
                                                          ((4, 32, 64), 63, 128, 0, 0, 0), ((8, 32, 32), 64, 7, 3, 20, 128)])
def test_end_to_end_against_oracle(dev, grid, seed, E, sink, ntail, drop):
    import htrc_b200
    q, k, v = _inputs(grid, seed)
    tail = (k[-ntail:].float(), v[-ntail:].float()) if ntail else None
    if drop:
        k, v = k[:-drop], v[:-drop]
    tail_d = (tail[0].to(dev), tail[1].to(dev)) if tail else None
    cfg = {**htrc_b200.PROD, "leaf": 64, "exact_leaves": E, "sink_leaves": sink}
    out, lse = htrc_b200.flat_attention(q.to(dev), k.to(dev), v.to(dev), tail=tail_d, return_lse=True, **cfg)
    st = htrc_b200.run_stages(q.to(dev), k.to(dev), v.to(dev), *(tail_d or (None, None)), exact_leaves=E,
                              sink_leaves=sink)
    torch.cuda.synchronize()
    assert torch.equal(out, st["out"])
    tnp = (tail[0].numpy(), tail[1].numpy()) if tail else None
    ro, rl, rst = O.flat_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), leaf=64,
                                   exact_leaves=E, sink_leaves=sink, tail=tnp, return_stages=True, precision="tf32")
    same_state = _oracle_on_device_state(q, v, st, tnp)
    _check_against(out, lse, st, ro, rl, rst["excl"], rst["sel"], q.shape[0], st["kx"], same_state, strict=False)


def test_fused_forward_equals_staged(dev):
    """The single-call forward (chunked) and the staged path give identical outputs."""
    import htrc_b200
    q, k, v = _inputs((8, 32, 32), 71)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    cfg = {**htrc_b200.PROD, "leaf": 64, "exact_leaves": 24}
    a, la = htrc_b200.flat_attention(qd, kd, vd, return_lse=True, **{**cfg, "tile_chunk": 0})
    b, lb = htrc_b200.flat_attention(qd, kd, vd, return_lse=True, **{**cfg, "tile_chunk": 16})
    st = htrc_b200.run_stages(qd, kd, vd, exact_leaves=24)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(la, lb)
    assert torch.equal(a, st["out"]) and torch.equal(la, st["lse"])


def test_bounded_wait_runs_out_and_reports(dev):
    """The failure path every kernel shares, made to run out on purpose without a fault: a wait on a
    barrier nothing arrives at gives up after its bound, the status word reports it (and the library's
    status reader raises), and the context still runs the operator afterwards."""
    import htrc_b200
    from htrc_b200 import _lib
    from htrc_b200 import flat as F
    from htrc_b200._lib import lib, ptr, stream_ptr
    ws = F.new_workspace(4096, dev)                     # the status word is the workspace's first word
    _lib.check(lib().htrc_selftest_wait_timeout(ptr(ws), 2_000_000, stream_ptr()), "selftest")
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) == 1     # HTRC_STATUS_WAIT_TIMEOUT
    with pytest.raises(_lib.HtrcError, match="bounded wait"):
        F.device_status(ws)
    F.device_status(ws)                                   # read and cleared: no bit left
    q, k, v = _inputs((2, 16, 16), 141)
    out = htrc_b200.flat_attention(q.to(dev), k.to(dev), v.to(dev), **{**htrc_b200.PROD, "leaf": 64, "exact_leaves": 2})
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
