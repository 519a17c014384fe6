"""The hierarchical operator's CUDA path (htrc_b200.tree over include/htrc_tree.h) against the reference's
NumPy model: fixtures recorded from src/htrc_reference/model.py itself, the reference's own identities of
that model (its tests/test_reference.py, restated on the GPU), and the float64 oracle at larger sizes.

Tolerances: the kernels compute in float32 and the reference in float64.  Per-query counters
(visited_nodes, accepted_nodes, exact_leaves) must equal the reference's on at least 99% of the queries
(an opening decision whose score sits within float32 rounding of the threshold may flip); outputs must
agree within 2e-4 max-abs on queries whose counters agree (1e-3 for the RMS-3 video inputs, whose logits
reach ~100), within 2e-2 on every query, and log-Z within 1e-3 mean-abs."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE / "golden"))

pytestmark = pytest.mark.gpu

from oracle import tree_oracle as T  # noqa: E402
import make_tree_golden as G  # noqa: E402


def _np(x):
    return x.detach().float().cpu().numpy() if torch.is_tensor(x) else np.asarray(x)


def _check(out, counters, ref_out, ref_counters, lse=None, ref_lse=None, agree=0.99, same_tol=2e-4):
    out, ref_out = _np(out), np.asarray(ref_out)
    same = (np.asarray(counters) == np.asarray(ref_counters)).all(1)
    assert same.mean() >= agree, f"counters agree on {same.mean():.4f} of the queries"
    err = np.abs(out - ref_out).max(1)
    assert err.max() <= 2e-2, err.max()
    if same.any():
        assert err[same].max() <= same_tol, err[same].max()
    if lse is not None:
        assert np.abs(_np(lse) - np.asarray(ref_lse)).mean() <= 1e-3


@pytest.mark.parametrize("name", list(G.CASES))
def test_tree_matches_reference_fixtures(name):
    from htrc_b200 import tree
    fx = np.load(HERE / "golden" / f"tree_{name}.npz")
    q, k, v = G.inputs(name)
    assert G.digest(q, k, v) == str(fx["sha"])
    rows = fx["rows"]
    qs = torch.from_numpy(q[rows]).float() * float(fx["scale"])
    forest = tree.build_forest(k, v, fx["centres"], leaf_size=int(fx["leaf"]), fanout=int(fx["fanout"]))
    out, info, lse = tree.evaluate(k, v, qs, fx["centres"], forest, opening_threshold=float(fx["thr"]),
                                   assign=fx["assign"][rows], return_lse=True)
    cnt = np.stack([_np(info["visited_nodes"]), _np(info["accepted_nodes"]), _np(info["exact_leaves"])], 1)
    _, ref_lse, _, _ = T.evaluate_centres(k, v, q.astype(np.float64)[rows] * float(fx["scale"]), fx["centres"],
                                          fx["assign"][rows], leaf_size=int(fx["leaf"]), fanout=int(fx["fanout"]),
                                          opening_threshold=float(fx["thr"]))
    _check(out, cnt, fx["out"], fx["counters"], lse, ref_lse)


def test_tree_bf16_loaders_and_tensor_core_leaves():
    """bfloat16 inputs: with the CUDA-core leaf kernel (HTRC_TREE_SIMT_LEAVES=1) the result is bitwise the float32
    path's on the same values; the default tensor-core leaf kernel (bf16 MMAs, P as bf16 hi + lo) agrees with it
    within float32 rounding (counters on >= 99% of the queries)."""
    import os
    from htrc_b200 import tree
    q, k, v = G.inputs("field")
    fx = np.load(HERE / "golden" / "tree_field.npz")
    dev = torch.device("cuda")
    qb, kb, vb = (torch.from_numpy(x).to(dev).bfloat16() for x in (q, k, v))
    cen = torch.from_numpy(fx["centres"]).float().to(dev)
    asg = torch.from_numpy(fx["assign"]).int().to(dev)
    kw = dict(leaf_size=64, fanout=16, centres=cen, assign=asg, return_lse=True, return_info=True)
    of, lf, inf = tree.tree_attention(qb.float(), kb.float(), vb.float(), **kw)
    os.environ["HTRC_TREE_SIMT_LEAVES"] = "1"
    try:
        ob, lb, _ = tree.tree_attention(qb, kb, vb, **kw)
    finally:
        del os.environ["HTRC_TREE_SIMT_LEAVES"]
    assert torch.equal(ob, of) and torch.equal(lb, lf)
    ot, lt, intc = tree.tree_attention(qb, kb, vb, **kw)
    cnt = np.stack([_np(intc[x]) for x in ("visited_nodes", "accepted_nodes", "exact_leaves")], 1)
    ref = np.stack([_np(inf[x]) for x in ("visited_nodes", "accepted_nodes", "exact_leaves")], 1)
    _check(ot, cnt, _np(of), ref, lt, _np(lf), same_tol=1e-3)
    assert np.abs(_np(lt) - _np(lf)).mean() < 1e-4


def _small():
    rng = np.random.default_rng(1107)
    return rng.normal(size=(128, 8)), rng.normal(size=(128, 5)), rng.normal(size=8) * 0.2, rng.normal(size=8) * 0.1


def test_level_one_equals_merged_leaves():
    """Level-1 statistics from the keys equal the merge of the leaves' exact statistics (model.py:51-66), and a
    level merged on the GPU equals the oracle's merge."""
    from htrc_b200 import tree
    rng = np.random.default_rng(3)
    k, v, c = rng.normal(size=(512, 8)), rng.normal(size=(512, 5)), rng.normal(size=8) * 0.2
    f = tree.build_forest(k, v, c, leaf_size=16, fanout=4)
    assert f.nodes == [32, 8, 2]
    lv = T.forest(k, v, c, leaf_size=16, fanout=4)
    np.testing.assert_allclose(_np(f.level_stats(0)["L"]), lv[0]["L"], atol=2e-5)
    np.testing.assert_allclose(_np(f.level_stats(0)["a"]), k @ c, atol=2e-5)
    for level in (1, 2):
        got = f.level_stats(level)
        for fld, tol in (("L", 2e-5), ("g", 2e-5), ("u", 2e-5), ("H", 5e-5), ("J", 5e-5)):
            np.testing.assert_allclose(_np(got[fld]), lv[level][fld], atol=tol, err_msg=f"level {level} {fld}")


def test_collapse_at_the_centre_is_exact():
    from htrc_b200 import tree
    k, v, c, _ = _small()
    f = tree.build_forest(k, v, c)
    out, info = tree.evaluate(k, v, c, c, f)
    np.testing.assert_allclose(_np(out), T.exact_attention(k, v, c)[0][0], atol=1e-5)
    assert info["exact_leaves"] == 0
    assert out.shape == (5,)


def test_threshold_zero_opens_every_leaf():
    from htrc_b200 import tree
    k, v, c, d = _small()
    f = tree.build_forest(k, v, c)
    out, info, lse = tree.evaluate(k, v, c + d, c, f, opening_threshold=0, return_lse=True)
    ref, ref_lse = T.exact_attention(k, v, c + d)
    np.testing.assert_allclose(_np(out), ref[0], atol=1e-5)
    assert abs(float(lse) - ref_lse[0]) < 1e-5
    assert info["exact_leaves"] == 8 and info["visited_nodes"] >= 1


def test_validation():
    from htrc_b200 import tree
    k, v, c, d = _small()
    f = tree.build_forest(k, v, c)
    with pytest.raises(ValueError):
        tree.evaluate(k, v, c, c, f, opening_threshold=-1)
    with pytest.raises(ValueError):
        tree.evaluate(k, v, np.zeros(7), c, f)
    with pytest.raises(ValueError):
        tree.build_forest(k, v[:10], c)
    with pytest.raises(ValueError):
        tree.build_forest(k, v, np.zeros(3))
    with pytest.raises(ValueError):
        tree.evaluate(k, v, np.stack([c, c]), np.stack([c, c]), tree.build_forest(k, v, np.stack([c, c])))
    with pytest.raises(ValueError):      # an out-of-range centre index is reported by the device
        tree.evaluate(k, v, np.stack([c, c]), np.stack([c, c]), tree.build_forest(k, v, np.stack([c, c])),
                      assign=[0, 2])


def test_many_queries_match_single_queries_and_are_deterministic():
    from htrc_b200 import tree
    rng = np.random.default_rng(9)
    k, v = rng.normal(size=(1000, 16)), rng.normal(size=(1000, 12))
    c = rng.normal(size=16) * 0.15
    qs = c + rng.normal(size=(40, 16)) * 0.12
    f = tree.build_forest(k, v, c, leaf_size=16, fanout=4)
    out, info = tree.evaluate(k, v, qs, c, f, opening_threshold=0.001)
    out2, info2 = tree.evaluate(k, v, qs, c, f, opening_threshold=0.001)
    assert torch.equal(out, out2)
    for i in (0, 17, 39):
        o1, i1 = tree.evaluate(k, v, qs[i], c, f, opening_threshold=0.001)
        assert torch.equal(o1, out[i])
        assert i1["exact_leaves"] == int(info["exact_leaves"][i])
    ref, ref_lse, ref_info = T.evaluate(k, v, qs, c, T.forest(k, v, c, leaf_size=16, fanout=4), opening_threshold=0.001)
    cnt = np.stack([_np(info[x]) for x in ("visited_nodes", "accepted_nodes", "exact_leaves")], 1)
    rcnt = np.stack([ref_info[x] for x in ("visited_nodes", "accepted_nodes", "exact_leaves")], 1)
    _check(out, cnt, ref, rcnt)


def test_operator_on_the_video_generator():
    """tree_attention on 16,384 smooth-field tokens with its own k-means centres, against the oracle on a
    sample of queries of two centres."""
    from htrc_b200 import synth, tree
    q, k, v = synth.head_inputs((16, 32, 32), 128, head=3)
    dev = torch.device("cuda")
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    out, lse, info = tree.tree_attention(qd, kd, vd, return_lse=True, return_info=True)
    cen = _np(info["centres"])
    assert torch.isfinite(out).all() and torch.isfinite(lse).all()
    assign = _np(info["assign"]).astype(np.int64)
    sc = 1.0 / np.sqrt(128)
    qn, kn, vn = (x.float().numpy() for x in (q, k, v))
    for cidx in np.unique(assign)[:2]:
        rows = np.nonzero(assign == cidx)[0][:24]
        lv = T.forest(kn, vn, cen[cidx].astype(np.float64), leaf_size=64, fanout=16)
        ref, ref_lse, ref_info = T.evaluate(kn, vn, qn[rows].astype(np.float64) * sc, cen[cidx], lv,
                                            opening_threshold=0.02)
        cnt = np.stack([_np(info[x])[rows] for x in ("visited_nodes", "accepted_nodes", "exact_leaves")], 1)
        rcnt = np.stack([ref_info[x] for x in ("visited_nodes", "accepted_nodes", "exact_leaves")], 1)
        # RMS-3 inputs: logits up to ~100, whose float32 rounding (~1e-5 relative) moves outputs by a few 1e-4
        _check(_np(out)[rows], cnt, ref, rcnt, _np(lse)[rows], ref_lse, agree=0.95, same_tol=1e-3)


def test_tensor_core_nodes_match_cuda_core_nodes():
    """The internal nodes below the roots on tcgen05 (D and M as bf16 hi + lo parts, three MMA chains) against the
    float32 CUDA-core kernels (HTRC_TREE_SIMT_NODES=1) on the three-level fixtures."""
    import os
    from htrc_b200 import tree
    for name in ("cluster", "ragged"):
        fx = np.load(HERE / "golden" / f"tree_{name}.npz")
        q, k, v = G.inputs(name)
        qs = torch.from_numpy(q).float() * float(fx["scale"])
        forest = tree.build_forest(k, v, fx["centres"], leaf_size=int(fx["leaf"]), fanout=int(fx["fanout"]))
        assert forest.levels == 3
        args = (k, v, qs, fx["centres"], forest)
        kw = dict(opening_threshold=float(fx["thr"]), assign=fx["assign"], return_lse=True)
        ot, it, lt = tree.evaluate(*args, **kw)
        os.environ["HTRC_TREE_SIMT_NODES"] = "1"
        try:
            os_, is_, ls_ = tree.evaluate(*args, **kw)
        finally:
            del os.environ["HTRC_TREE_SIMT_NODES"]
        cnt = np.stack([_np(it[x]) for x in ("visited_nodes", "accepted_nodes", "exact_leaves")], 1)
        ref = np.stack([_np(is_[x]) for x in ("visited_nodes", "accepted_nodes", "exact_leaves")], 1)
        _check(ot, cnt, _np(os_), ref, lt, _np(ls_), same_tol=2e-4)


@pytest.mark.parametrize("m,leaf,fanout", [(1000, 16, 4), (4096, 16, 4), (3000, 40, 8)])
def test_tensor_core_path_on_other_shapes(m, leaf, fanout):
    """bfloat16 inputs through the tensor-core kernels (build, node products, leaf blocks) with leaves of 16 and
    40 keys, a ragged last leaf (1000 = 62 x 16 + 8, 3000 = 75 x 40) and four levels (4096 keys, leaf 16,
    fanout 4), against the float64 oracle on the same bfloat16 values."""
    from htrc_b200 import synth, tree
    q, k, v = synth.cluster_inputs(m, 128, clusters=32, seed=m + leaf)
    q, k, v = (torch.from_numpy(x).bfloat16() for x in (q, k, v))
    qn, kn, vn = (x.float().numpy().astype(np.float64) for x in (q, k, v))
    sc = 1.0 / np.sqrt(128)
    cen, asg = G.centres_of(qn * sc, 4)
    dev = torch.device("cuda")
    out, lse, info = tree.tree_attention(q.to(dev), k.to(dev), v.to(dev), leaf_size=leaf, fanout=fanout,
                                         centres=torch.from_numpy(cen).float().to(dev),
                                         assign=torch.from_numpy(asg).int().to(dev), return_lse=True, return_info=True)
    assert info["forest"].levels == (4 if m == 4096 else 3)
    rows = np.arange(0, m, max(1, m // 96))
    ref, ref_lse, ref_cnt, _ = T.evaluate_centres(kn, vn, qn[rows] * sc, cen, asg[rows], leaf_size=leaf, fanout=fanout,
                                                  opening_threshold=0.02)
    cnt = np.stack([_np(info[x])[rows] for x in ("visited_nodes", "accepted_nodes", "exact_leaves")], 1)
    rc = np.stack([ref_cnt[x] for x in ("visited_nodes", "accepted_nodes", "exact_leaves")], 1)
    _check(_np(out)[rows], cnt, ref, rc, _np(lse)[rows], ref_lse, agree=0.97, same_tol=1e-3)


def test_edge_cases():
    """One key; one query; a centre that no query uses; queries exactly at a centre."""
    from htrc_b200 import tree
    rng = np.random.default_rng(21)
    k1, v1 = rng.normal(size=(1, 8)), rng.normal(size=(1, 5))
    c = rng.normal(size=8) * 0.2
    qs = c + rng.normal(size=(3, 8)) * 0.1
    f = tree.build_forest(k1, v1, c)
    assert f.nodes == [1]
    out, info = tree.evaluate(k1, v1, qs, c, f, opening_threshold=0.01)
    np.testing.assert_allclose(_np(out), np.repeat(v1, 3, 0), atol=1e-6)     # one key: its value, exactly
    k, v = rng.normal(size=(300, 8)), rng.normal(size=(300, 5))
    cen = np.stack([c, c + 5.0])                                            # the second centre is never assigned
    f2 = tree.build_forest(k, v, cen, leaf_size=16, fanout=4)
    q1 = c + rng.normal(size=8) * 0.1
    o1, i1 = tree.evaluate(k, v, q1[None], cen, f2, assign=[0])
    lv = T.forest(k, v, c, leaf_size=16, fanout=4)
    ref, _, rinfo = T.evaluate(k, v, q1[None], c, lv)
    np.testing.assert_allclose(_np(o1)[0], ref[0], atol=2e-5)
    assert int(i1["exact_leaves"][0]) == int(rinfo["exact_leaves"][0])
    oc, ic = tree.evaluate(k, v, np.stack([c, c]), cen, f2, assign=[0, 0])  # at the centre: no leaf opens
    np.testing.assert_allclose(_np(oc), np.repeat(T.exact_attention(k, v, c)[0], 2, 0), atol=2e-5)
    assert int(ic["exact_leaves"].sum()) == 0
