"""GPU parity of the bf16 state path (store="bf16": bf16 g and vbar without scales, bf16 far- and near-field
dots -- h3/htrc_flat_triton.py:82-84 and the DOT=1 branches of its row-max and tile kernels) against the CPU
oracle and against fixtures recorded from the reference, through the C ABI's bf16 stage entry points and the
whole operator.  Tolerances: output max-abs 2e-2 and log-Z mean-abs 1e-3 end to end, routing agreement >=
99.9%; the bf16 state values agree with the reference's except where the device's float32 statistics sit on the
other side of a bf16 rounding boundary (then within one bf16 step of the row's largest value)."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import flat_oracle as O  # noqa: E402

OUT_TOL = 2e-2
LSE_TOL = 1e-3
ROUTE_AGREE = 0.999
SCALE = 1.0 / math.sqrt(128)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from htrc_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


def _np(t):
    return t.detach().float().cpu().numpy() if t.dtype in (torch.bfloat16, torch.float16) else t.detach().cpu().numpy()


def _bits(t):
    """bf16 tensor -> uint16 bit patterns (numpy)."""
    return t.detach().view(torch.int16).cpu().numpy().view(np.uint16)


def _stages(dev, q, k, v, E, sink=0, tail=None, **kw):
    import htrc_b200
    from htrc_b200 import _lib
    tk = tv = None
    if tail is not None:
        tk = torch.from_numpy(np.asarray(tail[0], np.float32)).to(dev)
        tv = torch.from_numpy(np.asarray(tail[1], np.float32)).to(dev)
    st = htrc_b200.run_stages(torch.from_numpy(q).to(dev), torch.from_numpy(k).to(torch.bfloat16).to(dev),
                              torch.from_numpy(v).to(torch.bfloat16).to(dev), tk, tv, exact_leaves=E, sink_leaves=sink,
                              store=_lib.STORE_BF16, **{"precision": _lib.PREC_FP32, **kw})
    torch.cuda.synchronize()
    assert int(st["status"].item()) == 0
    return st


def _bf16_close(dev_bits, ref_bits):
    """Values equal except rarely; where not, within one bf16 step of the row's largest value (the device's
    statistics are float32-accurate sums, so an element that cancels to a small value can land several of its
    own bf16 steps away, never more than the row's rounding)."""
    a = (dev_bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    b = (ref_bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    row = np.abs(b).max(-1, keepdims=True)
    assert (np.abs(a - b) <= row * 2.0 ** -8).all(), float((np.abs(a - b) / np.maximum(row, 1e-30)).max())
    assert (dev_bits != ref_bits).mean() < 1e-2, float((dev_bits != ref_bits).mean())


@pytest.mark.parametrize("case", ["bf16_state", "bf16_sink_tail"])
def test_bf16_path_against_reference_fixture(dev, golden_cases, case):
    z = golden_cases[case]
    tail = (z["tail_k"], z["tail_v"]) if "tail_k" in z else None
    E, sink = int(z["exact_leaves"]), int(z["sink_leaves"])
    st = _stages(dev, z["q"], z["k"], z["v"], E, sink, tail)
    nb = st["nb"]
    # tile prep: the centres and the operand rows (bf16 q and bf16 offsets, bit for bit)
    assert np.allclose(_np(st["mu"]), z["mu"], rtol=0, atol=2e-6)
    qt, _, _ = O.tile_centres(z["q"], 64)
    qb, dqb = O.query_codes_bf16(qt, _np(st["mu"]))
    nt = qt.shape[0]
    assert np.array_equal(_np(st["qb"]).reshape(nt, 64, 128), qb)
    assert np.array_equal(_np(st["dqb"]).reshape(nt, 64, 128), dqb)
    # state
    _bf16_close(_bits(st["gb"])[:, :nb], z["g_bf16"])
    _bf16_close(_bits(st["vbb"])[:, :nb], z["vb_bf16"])
    assert np.abs(_np(st["lz"])[:, :nb] - z["lz"]).max() < 2e-4
    # selection and routing
    assert np.abs(_np(st["sel"])[:, :nb] - z["sel"]).max() < 1e-2 * max(1.0, np.abs(z["sel"]).max())
    assert (_np(st["excl"])[:, :nb] == z["excl"]).mean() >= ROUTE_AGREE
    # output
    out, lse = _np(st["out"]), _np(st["lse"])
    assert np.abs(out - z["out"]).max() < OUT_TOL
    assert np.abs(lse - z["lse"]).mean() < LSE_TOL


@pytest.mark.parametrize("case", ["bf16_state", "bf16_sink_tail"])
def test_bf16_operator_end_to_end(dev, golden_cases, case):
    """flat_attention(**PROD, store="bf16") against the reference's recorded output."""
    import htrc_b200
    z = golden_cases[case]
    tail = None
    if "tail_k" in z:
        tail = (torch.from_numpy(z["tail_k"]).to(dev), torch.from_numpy(z["tail_v"]).to(dev))
    q = torch.from_numpy(z["q"]).to(dev)
    k = torch.from_numpy(z["k"]).to(torch.bfloat16).to(dev)
    v = torch.from_numpy(z["v"]).to(torch.bfloat16).to(dev)
    # recorded by Triton's interpreter, which evaluates the tf32 dots in float32
    cfg = {**htrc_b200.PROD, "leaf": 64, "store": "bf16", "exact_leaves": int(z["exact_leaves"]),
           "sink_leaves": int(z["sink_leaves"]), "precision": "fp32"}
    out, lse = htrc_b200.flat_attention(q, k, v, tail=tail, return_lse=True, **cfg)
    torch.cuda.synchronize()
    assert np.abs(out.cpu().numpy() - z["out"]).max() < OUT_TOL
    assert np.abs(lse.cpu().numpy() - z["lse"]).mean() < LSE_TOL


def _synthetic(n, m, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(n, 128, generator=g) * 2.0
    k = torch.randn(m, 128, generator=g) * 2.0
    # smooth structure: nearby tokens share a direction, so leaves carry real far-field mass
    base = torch.randn(max(1, m // 64), 128, generator=g) * 2.5
    k += base.repeat_interleave(64, 0)[:m]
    q += base.repeat_interleave(64, 0)[torch.arange(n) * max(1, m // 64) // n]
    v = torch.randn(m, 128, generator=g)
    return q.numpy().astype(np.float32), O.bf16_round(k.numpy()), O.bf16_round(v.numpy())


@pytest.mark.parametrize("n,m,E,sink,n_tail", [(4096, 8192, 16, 1, 0),     # far and near steps
                                               (3000, 32768, 61, 2, 5),    # 8 far blocks, ragged tiles, tail
                                               (1024, 64 * 130, 0, 0, 0),  # far field only
                                               (640, 4096, 64, 0, 0),      # everything routed: near only
                                               (2048, 8192, 8, 0, 20)])    # a float32 tail (> 16 keys)
def test_bf16_tile_kernel_on_device_state(dev, n, m, E, sink, n_tail):
    """Fed the device's own bf16 state and routing, the tile kernel reproduces the oracle's bf16-state tile
    attention (weights rounded against the row's final maximum) within the bf16-weight rounding, and selection
    / routing equal the oracle's formulas on that state."""
    q, k, v = _synthetic(n, m, 200 + n_tail)
    tail = None
    if n_tail:
        g = np.random.default_rng(9)
        tail = (g.standard_normal((n_tail, 128)).astype(np.float32), g.standard_normal((n_tail, 128)).astype(np.float32))
    st = _stages(dev, q, k, v, E, sink, tail)
    nb = st["nb"]
    qt, _, _ = O.tile_centres(q, 64)
    nt = qt.shape[0]
    qb, dqb = _np(st["qb"]).reshape(nt, 64, 128), _np(st["dqb"]).reshape(nt, 64, 128)
    gq, lz, vq = _np(st["gb"])[:, :nb], _np(st["lz"])[:, :nb], _np(st["vbb"])[:, :nb]
    one = np.ones(lz.shape, np.float32)
    kx = st["kx"]
    if 0 < kx < nb:
        sel = O.rowmax_select_bf16(dqb, gq, lz)
        sel_d = _np(st["sel"])[:, :nb]
        assert np.abs(sel_d - sel).max() <= 1e-4 * max(1.0, np.abs(sel).max())
        idx, excl = O.route(sel_d, E, min(sink, nb))
        assert np.array_equal(_np(st["excl"])[:, :nb], excl)
        assert np.array_equal(np.sort(_np(st["idx"])[:, :kx], 1), np.sort(idx, 1))
    excl_d = _np(st["excl"])[:, :nb]
    idx_d = _np(st["idx"])[:, :kx] if kx else np.zeros((nt, 0), np.int32)
    o, l = O.tile_attention_fp8(qt, qb, dqb, gq, one, lz, vq, one, excl_d, idx_d, k, v, 64, SCALE, tail=tail,
                                far_weight="bf16")
    out, lse = _np(st["out"]), _np(st["lse"])
    assert np.abs(out - o[:n]).max() < 1e-2
    assert np.abs(lse - l[:n]).max() < 1e-3


@pytest.mark.parametrize("over", [{"kern": {"group": 2}}, {"order": "kmeans"}, {"tile": 32},
                                  {"order": "kmeans", "tile": 32, "kern": {"group": 4}}])
def test_bf16_modes_against_oracle(dev, over):
    """Groups, the k-means order and 32-row tiles on the bf16-state path, end to end against the oracle on the
    same inputs (with the device's k-means permutation)."""
    import htrc_b200
    from htrc_b200 import _lib
    q, k, v = _synthetic(2048, 16384, 56)
    cfg = {**htrc_b200.PROD, "leaf": 64, "store": "bf16", "exact_leaves": 24, "sink_leaves": 1, **over}
    st = htrc_b200.run_stages(torch.from_numpy(q).cuda(), torch.from_numpy(k).to(torch.bfloat16).cuda(),
                              torch.from_numpy(v).to(torch.bfloat16).cuda(), exact_leaves=24, sink_leaves=1,
                              store=_lib.STORE_BF16, group=htrc_b200.flat.group_of(cfg.get("kern")),
                              order=htrc_b200.flat.order_code(cfg.get("order", "seq")), tile=cfg["tile"])
    torch.cuda.synchronize()
    perm = _np(st["perm"]) if st["perm"] is not None else None
    ro, rl, rst = O.flat_attention(q, k, v, exact_leaves=24, sink_leaves=1, tile=cfg["tile"],
                                   group=htrc_b200.flat.group_of(cfg.get("kern")), order=cfg.get("order", "seq"),
                                   perm=perm, store="bf16", return_stages=True, precision="tf32")
    nb = st["nb"]
    assert (_np(st["excl"])[:, :nb] == rst["excl"]).mean() >= ROUTE_AGREE
    out, lse = htrc_b200.flat_attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).to(torch.bfloat16).cuda(),
                                        torch.from_numpy(v).to(torch.bfloat16).cuda(), return_lse=True, **cfg)
    torch.cuda.synchronize()
    agree = (_np(st["excl"])[:, :nb] == rst["excl"]).all(1)
    i = np.arange(q.shape[0])
    same = agree[(i // cfg["tile"]) // htrc_b200.flat.group_of(cfg.get("kern"))]
    o = out.cpu().numpy()
    rows = i if perm is None else perm.astype(np.int64)
    ok_rows = rows[same]
    assert np.abs(o[ok_rows] - ro[ok_rows]).max() < OUT_TOL
    assert np.abs(lse.cpu().numpy() - rl).mean() < LSE_TOL
    assert np.array_equal(o, _np(st["out"]))            # the fused forward and the stage launches agree


@pytest.mark.parametrize("chunk,group", [(8, 1), (6, 2)])
def test_bf16_chunked_state_matches_one_chunk(dev, chunk, group):
    """tile_chunk smaller than the tile count: the bf16 statistics, row-max and both tile passes run per chunk
    of centre rows; every row equals the single-chunk result."""
    import htrc_b200
    q, k, v = _synthetic(2000, 8192, 78)
    qd = torch.from_numpy(q).cuda()
    kd = torch.from_numpy(k).to(torch.bfloat16).cuda()
    vd = torch.from_numpy(v).to(torch.bfloat16).cuda()
    base = {**htrc_b200.PROD, "leaf": 64, "store": "bf16", "exact_leaves": 12, "sink_leaves": 1,
            "kern": {"group": group}}
    o1, l1 = htrc_b200.flat_attention(qd, kd, vd, return_lse=True, **{**base, "tile_chunk": 0})
    oc, lc = htrc_b200.flat_attention(qd, kd, vd, return_lse=True, **{**base, "tile_chunk": chunk})
    torch.cuda.synchronize()
    assert torch.equal(o1, oc) and torch.equal(l1, lc)
