"""The hierarchical-law oracle (oracle/tree_oracle.py) against fixtures recorded from the reference's own
NumPy model (tests/golden/make_tree_golden.py), and the reference's own identities of that model
(tests/test_reference.py of the reference, restated on the oracle)."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE / "golden"))

from oracle import tree_oracle as T  # noqa: E402
import make_tree_golden as G  # noqa: E402


def _case(name):
    fx = np.load(HERE / "golden" / f"tree_{name}.npz")
    q, k, v = G.inputs(name)
    assert G.digest(q, k, v) == str(fx["sha"]), "the input generator no longer reproduces the fixture's inputs"
    return fx, q, k, v


@pytest.mark.parametrize("name", list(G.CASES))
def test_oracle_matches_reference_model(name):
    fx, q, k, v = _case(name)
    rows = fx["rows"]
    qs = q.astype(np.float64)[rows] * float(fx["scale"])
    out, lse, cnt, _ = T.evaluate_centres(k, v, qs, fx["centres"], fx["assign"][rows], leaf_size=int(fx["leaf"]),
                                          fanout=int(fx["fanout"]), opening_threshold=float(fx["thr"]))
    np.testing.assert_allclose(out, fx["out"], atol=1e-9, rtol=1e-9)
    got = np.stack([cnt["visited_nodes"], cnt["accepted_nodes"], cnt["exact_leaves"]], 1)
    np.testing.assert_array_equal(got, fx["counters"])
    assert np.isfinite(lse).all()


def test_oracle_roots_match_reference_model():
    fx, q, k, v = _case("cluster")
    lv = T.forest(k, v, fx["centres"][0], leaf_size=int(fx["leaf"]), fanout=int(fx["fanout"]))
    top = lv[-1]
    np.testing.assert_allclose(top["L"], fx["root_L"], atol=1e-10)
    np.testing.assert_allclose(top["g"], fx["root_g"], atol=1e-10)
    np.testing.assert_allclose(top["u"], fx["root_u"], atol=1e-10)
    np.testing.assert_allclose(top["H"], fx["root_H"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(top["J"], fx["root_J"], rtol=1e-6, atol=1e-6)


def _small():
    rng = np.random.default_rng(1107)
    return rng.normal(size=(128, 8)), rng.normal(size=(128, 5)), rng.normal(size=8) * 0.2, rng.normal(size=8) * 0.1


def test_merge_equals_whole_block():
    """Merging eight leaves' statistics gives the statistics of the whole block (the law is exact)."""
    k, v, c, _ = _small()
    whole = T.leaf_stats(k, v, c, 128)
    merged = T.merge_level(T.leaf_stats(k, v, c, 16), 8)
    for f in ("L", "g", "H", "u", "J"):
        np.testing.assert_allclose(merged[f], whole[f], atol=1e-12)


def test_value_jacobian_is_the_derivative():
    k, v, c, d = _small()
    st = T.leaf_stats(k, v, c, 128)
    e = d / np.linalg.norm(d)
    h = 1e-5
    fd = (T.exact_attention(k, v, c + h * e)[0] - T.exact_attention(k, v, c - h * e)[0]) / (2 * h)
    np.testing.assert_allclose(fd[0], st["J"][0] @ e, atol=1e-9, rtol=1e-8)


def test_collapse_at_the_centre_is_exact():
    k, v, c, _ = _small()
    lv = T.forest(k, v, c)
    out, lse, info = T.evaluate(k, v, c, c, lv)
    ref, ref_lse = T.exact_attention(k, v, c)
    np.testing.assert_allclose(out, ref, atol=1e-12)
    np.testing.assert_allclose(lse, ref_lse, atol=1e-12)
    assert info["exact_leaves"][0] == 0


def test_threshold_zero_opens_every_leaf():
    k, v, c, d = _small()
    lv = T.forest(k, v, c)
    out, _, info = T.evaluate(k, v, c + d, c, lv, opening_threshold=0)
    np.testing.assert_allclose(out, T.exact_attention(k, v, c + d)[0], atol=1e-12)
    assert info["exact_leaves"][0] == 8


def test_negative_threshold_raises():
    k, v, c, _ = _small()
    with pytest.raises(ValueError):
        T.evaluate(k, v, c, c, T.forest(k, v, c), opening_threshold=-1)
