"""GPU parity at the benchmark's own sizes, through the C ABI, against the CPU oracle on the same seeded inputs
(PROD's precision setting, tf32 leaf-statistics operands, on both sides).

Configuration 2 (16,384 tokens of a 16x32x32 latent, leaf 64, fast mode E = 256 = every leaf): the operator
reduces to exact attention through the near-field path, so there is no far field and no leaf statistic in
the way: the key and query codes must be bit-exact, every leaf routed, every output row within 2e-2 of the
oracle and log-Z within 1e-3 mean-abs; the error against float32 softmax attention is reported.

Configuration 3 (129,024 tokens of a 32x48x84 latent, E = 256 of 2016 leaves): the codes of every key and
query row are bit-exact at full size, and on a sample of query tiles (the oracle computes its own float64
leaf statistics, selection and routing for them) the routing masks agree on >= 99.9% of the (tile, leaf)
pairs, outputs of the agreeing tiles are within 2e-2 and log-Z within 1e-3 mean-abs.
"""
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


def _np(t):
    return t.detach().cpu().numpy()


def _codes_bit_exact(st, prep):
    nt = prep["qt"].shape[0]
    q8, sq, dq8, sdq = O.query_codes(prep["qt"], prep["mu"])
    assert np.array_equal(_np(st["k8"]), prep["k8"])
    assert np.array_equal(_np(st["ks"]).view(np.uint32), prep["ks"].view(np.uint32))
    assert np.array_equal(_np(st["mu"]).view(np.uint32), prep["mu"].view(np.uint32))
    assert np.array_equal(_np(st["q8"]).reshape(nt, 64, 128), q8)
    assert np.array_equal(_np(st["sq"]).reshape(nt, 64).view(np.uint32), sq.view(np.uint32))
    assert np.array_equal(_np(st["dq8"]).reshape(nt, 64, 128), dq8)
    assert np.array_equal(_np(st["sdq"]).reshape(nt, 64).view(np.uint32), sdq.view(np.uint32))


@pytest.mark.parametrize("head", [0, 7, 13, 23])
def test_cfg2_head_every_leaf_exact(dev, head):
    import htrc_b200
    from htrc_b200 import synth
    q, k, v = synth.head_inputs(synth.GRID_SMALL, 128, head=head)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    cfg = {**htrc_b200.PROD, "leaf": 64}
    out, lse = htrc_b200.flat_attention(qd, kd, vd, return_lse=True, **cfg)
    st = htrc_b200.run_stages(qd, kd, vd, exact_leaves=cfg["exact_leaves"])
    torch.cuda.synchronize()
    assert int(st["status"].item()) == 0
    assert torch.equal(out, st["out"]) and torch.equal(lse, st["lse"])
    nb = st["nb"]
    assert nb == 256 and st["kx"] == nb
    assert (_np(st["excl"])[:, :nb] == 1).all()                  # fast mode opens every leaf at this size
    qn, kn, vn = q.float().numpy(), k.float().numpy(), v.float().numpy()
    prep = O.prepare_head(qn, kn, vn)
    _codes_bit_exact(st, prep)
    ro, rl = O.attention_tiles(prep, np.arange(prep["qt"].shape[0]), exact_leaves=cfg["exact_leaves"],
                               precision="tf32")
    n = q.shape[0]
    err = np.abs(_np(out) - ro[:n]).max()
    assert err < OUT_TOL, err
    assert np.abs(_np(lse) - rl[:n]).mean() < LSE_TOL
    # the error against float32 softmax attention (INT8 QK, bf16 P and V): reported, bounded loosely
    rows = torch.arange(0, n, 61, device=dev)
    s_ = (qd[rows].float() @ kd.float().T) / math.sqrt(128)
    ex = torch.softmax(s_, -1) @ vd.float()
    rel = float((out[rows] - ex).norm() / ex.norm())
    print(f"cfg2 head {head}: out max-abs vs oracle {err:.3e}, rel-L2 vs exact attention {rel:.3e}")
    assert rel < 5e-2


def test_cfg3_head_codes_full_size_and_sampled_tiles(dev):
    import htrc_b200
    from htrc_b200 import flat as F
    from htrc_b200 import synth
    q, k, v = synth.head_inputs(synth.GRID_FULL, 128, head=5)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    n, m = q.shape[0], k.shape[0]
    nt, nb = -(-n // 64), m // 64
    E = htrc_b200.PROD["exact_leaves"]
    out = torch.empty((n, 128), dtype=torch.float32, device=dev)
    lse = torch.empty((n,), dtype=torch.float32, device=dev)
    mask = torch.zeros((nt, F.leaf_pitch(nb)), dtype=torch.uint8, device=dev)
    ws = F.new_workspace(F.workspace_bytes(n, m, E), dev)
    F.forward_into(qd, kd, vd, None, None, exact_leaves=E, out=out, lse=lse, workspace=ws, route_mask=mask)
    torch.cuda.synchronize()
    F.device_status(ws)
    qn, kn, vn = q.float().numpy(), k.float().numpy(), v.float().numpy()
    prep = O.prepare_head(qn, kn, vn)
    st = htrc_b200.run_stages(qd, kd, vd, exact_leaves=E)
    torch.cuda.synchronize()
    assert torch.equal(out, st["out"]) and torch.equal(lse, st["lse"])
    _codes_bit_exact(st, prep)
    del st
    tiles = np.sort(np.random.default_rng(3).choice(nt, size=8, replace=False))
    tiles[-1] = nt - 1                                            # the last tile too
    tiles = np.unique(tiles)
    mu, qt = prep["mu"][tiles], prep["qt"][tiles]
    g, lz, vbf = O.leaf_stats(mu, prep["k"], prep["v"], 64, 1 / math.sqrt(128), "tf32")
    g8, sg, _ = O.state_int8(g, vbf)
    _, _, dq8, sdq = O.query_codes(qt, mu)
    _, excl_o = O.route(O.rowmax_select(dq8, sdq, g8, sg, lz), E)
    excl_d = _np(mask)[tiles][:, :nb]
    agree = (excl_d == excl_o).mean()
    print(f"cfg3 head 5: routing agreement {agree:.5f} on {len(tiles)} tiles")
    assert agree >= ROUTE_AGREE, agree
    ro, rl = O.attention_tiles(prep, tiles, exact_leaves=E, precision="tf32")
    rows = (tiles[:, None] * 64 + np.arange(64)[None, :]).reshape(-1)
    valid = rows < n
    od, ld = _np(out)[rows[valid]], _np(lse)[rows[valid]]
    same = np.repeat((excl_d == excl_o).all(1), 64)[valid]
    assert same.mean() >= 0.5
    err = np.abs(od[same] - ro[valid][same]).max()
    assert err < OUT_TOL, err
    assert np.abs(ld - rl[valid]).mean() < LSE_TOL
