"""CPU oracle of the hierarchical HTRC law (the reference's NumPy teaching model), vectorised over queries.

TEST INFRASTRUCTURE ONLY.  The tree tests, ``__graft_entry__.smoke()`` and ``bench.py``'s baseline leg
compare the CUDA tree operator (``htrc_b200.tree``) against this module; nothing in the shipped package
imports it and the CUDA path never falls back to it.

It restates the law of src/htrc_reference/model.py in float64, for many queries at once:

  leaf statistics ..... model.py:35-49   (log-mass, mean key, Hessian, mean value, value Jacobian at a centre)
  merge ............... model.py:51-66   (log-sum-exp of the children, Hessian + outer(dg, dg), dipole merge)
  forest .............. model.py:68-86   (contiguous leaves of leaf_size keys, levels of `fanout` nodes
                                          merged while a level has more than `fanout` nodes; the last
                                          level is the list of roots)
  prediction .......... model.py:91-96   (second-order log-mass L + g.d + d.H.d / 2, value u + J.d)
  evaluation .......... model.py:98-137  (norm = log-sum-exp of the roots' predicted masses; a node
                                          opens when exp(min(0, lm - norm)) * expm1(min(|quad| / 2, 80))
                                          exceeds the threshold; an opened leaf is exact attention over
                                          its keys; the output is the softmax over accepted log-masses
                                          of the accepted values)

The reference walks one query depth-first; this restatement walks all queries level by level with a
per-query reach mask.  Both accept the same nodes in a different order, so outputs agree to float64
rounding.  Besides the output it returns the log-sum-exp of the accepted masses (the operator's log-Z),
the reference's per-query counters (visited_nodes, accepted_nodes, exact_leaves) and every node
decision, for the decision-agreement tests.

Parity status: pinned against the reference module itself (``tests/golden/make_tree_golden.py`` imports
src/htrc_reference/model.py and records its outputs and counters; ``tests/test_tree_oracle.py`` checks
this module against them).
"""
from __future__ import annotations

import numpy as np

F64 = np.float64


def _lse(x, axis):
    m = np.max(x, axis=axis, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    return np.squeeze(m, axis) + np.log(np.sum(np.exp(x - m), axis=axis))


def leaf_stats(keys, values, centre, leaf_size):
    """Exact statistics of every leaf (model.py:35-49) at one centre: dict of L [nl], g [nl, D],
    H [nl, D, D], u [nl, Dv], J [nl, Dv, D], and the key ranges."""
    keys = np.asarray(keys, F64)
    values = np.asarray(values, F64)
    c = np.asarray(centre, F64)
    m = keys.shape[0]
    starts = np.arange(0, m, leaf_size)
    out = {k: [] for k in ("L", "g", "H", "u", "J")}
    for s in starts:
        kb, vb = keys[s:s + leaf_size], values[s:s + leaf_size]
        a = kb @ c
        mx = a.max()
        e = np.exp(a - mx)
        z = e.sum()
        w = e / z
        mu = w @ kb
        val = w @ vb
        ck, cv = kb - mu, vb - val
        out["L"].append(mx + np.log(z))
        out["g"].append(mu)
        out["H"].append((ck * w[:, None]).T @ ck)
        out["u"].append(val)
        out["J"].append((cv * w[:, None]).T @ ck)
    st = {k: np.stack(v) for k, v in out.items()}
    st["start"] = starts
    st["stop"] = np.minimum(starts + leaf_size, m)
    return st


def merge_level(st, fanout):
    """One level up (model.py:51-66, :80-85): consecutive groups of `fanout` nodes, the last possibly
    shorter."""
    n = st["L"].shape[0]
    out = {k: [] for k in ("L", "g", "H", "u", "J")}
    for i in range(0, n, fanout):
        sl = slice(i, min(n, i + fanout))
        lg = st["L"][sl]
        mx = lg.max()
        e = np.exp(lg - mx)
        z = e.sum()
        w = e / z
        mu = w @ st["g"][sl]
        val = w @ st["u"][sl]
        dg = st["g"][sl] - mu
        dv = st["u"][sl] - val
        out["L"].append(mx + np.log(z))
        out["g"].append(mu)
        out["u"].append(val)
        out["H"].append(np.einsum("c,cde->de", w, st["H"][sl]) + np.einsum("c,cd,ce->de", w, dg, dg))
        out["J"].append(np.einsum("c,cde->de", w, st["J"][sl]) + np.einsum("c,cd,ce->de", w, dv, dg))
    return {k: np.stack(v) for k, v in out.items()}


def build_forest(keys, values, centre, *, leaf_size=16, fanout=4):
    """Levels of the forest, leaves first, roots last (model.py:68-86)."""
    if leaf_size < 1 or fanout < 2:
        raise ValueError("leaf_size must be positive and fanout >= 2")
    levels = [leaf_stats(keys, values, centre, leaf_size)]
    while levels[-1]["L"].shape[0] > fanout:
        levels.append(merge_level(levels[-1], fanout))
    return levels


def _predict(st, dq):
    """Second-order log-mass, value and quadratic term of every node for every query (model.py:91-96):
    returns lm [T, n], val [T, n, Dv], quad [T, n]."""
    quad = np.einsum("td,nde,te->tn", dq, st["H"], dq)
    lm = st["L"][None] + dq @ st["g"].T + 0.5 * quad
    val = st["u"][None] + np.einsum("nve,te->tnv", st["J"], dq)
    return lm, val, quad


def evaluate(keys, values, queries, centre, levels, *, opening_threshold=0.01):
    """Evaluate the law for queries [T, D] (already scaled, like the reference's `query`) against one
    centre's forest.  Returns (out [T, Dv], lse [T], info) where info has int arrays visited_nodes,
    accepted_nodes, exact_leaves [T] and, per level (leaves first), the boolean masks `reach` and
    `open` [T, n_level] of the walk."""
    if opening_threshold < 0:
        raise ValueError("opening_threshold must be nonnegative")
    keys = np.asarray(keys, F64)
    values = np.asarray(values, F64)
    q = np.atleast_2d(np.asarray(queries, F64))
    dq = q - np.asarray(centre, F64)[None]
    t = q.shape[0]
    top = len(levels) - 1
    lm_top, _, _ = _predict(levels[top], dq)
    norm = np.logaddexp.reduce(lm_top, axis=1)
    acc_lm, acc_val = [], []
    visited = np.zeros(t, np.int64)
    accepted = np.zeros(t, np.int64)
    exact = np.zeros(t, np.int64)
    reach = np.ones((t, levels[top]["L"].shape[0]), bool)
    masks = [None] * len(levels)
    for lev in range(top, -1, -1):
        st = levels[lev]
        lm, val, quad = _predict(st, dq)
        frac = np.exp(np.minimum(0.0, lm - norm[:, None]))
        score = frac * np.expm1(np.minimum(0.5 * np.abs(quad), 80.0))
        op = (score > opening_threshold) & reach
        masks[lev] = {"reach": reach.copy(), "open": op}
        visited += reach.sum(1)
        if lev > 0:
            far = reach & ~op
            accepted += far.sum(1)
            acc_lm.append(np.where(far, lm, -np.inf))
            acc_val.append(val)
            nchild = levels[lev - 1]["L"].shape[0]
            parent = np.minimum(np.arange(nchild) // fanout_of(levels, lev), st["L"].shape[0] - 1)
            reach = op[:, parent]
        else:
            accepted += reach.sum(1)
            exact += op.sum(1)
            ex_lm = np.full(lm.shape, -np.inf)
            ex_val = np.zeros_like(val)
            for li in range(st["L"].shape[0]):
                rows = np.nonzero(op[:, li])[0]
                if rows.size == 0:
                    continue
                s0, s1 = st["start"][li], st["stop"][li]
                lg = q[rows] @ keys[s0:s1].T
                lse = _lse(lg, 1)
                ex_lm[rows, li] = lse
                ex_val[rows, li] = np.exp(lg - lse[:, None]) @ values[s0:s1]
            acc_lm.append(np.where(op, ex_lm, np.where(reach, lm, -np.inf)))
            acc_val.append(np.where(op[..., None], ex_val, val))
    lms = np.concatenate(acc_lm, axis=1)
    vals = np.concatenate(acc_val, axis=1)
    lse = _lse(lms, 1)
    w = np.exp(lms - lse[:, None])
    out = np.einsum("tn,tnv->tv", w, vals)
    info = {"visited_nodes": visited, "accepted_nodes": accepted, "exact_leaves": exact, "levels": masks,
            "norm": norm}
    return out, lse, info


def fanout_of(levels, lev):
    """The fanout that made level `lev` from level lev - 1 (children per parent, the last parent possibly
    fewer): ceil(n_{lev-1} / n_lev) is ambiguous, so it is stored when the levels are built."""
    return levels[lev]["fanout"]


def forest(keys, values, centre, *, leaf_size=16, fanout=4):
    """build_forest with the fanout recorded on every merged level (used by evaluate)."""
    levels = build_forest(keys, values, centre, leaf_size=leaf_size, fanout=fanout)
    for lv in levels[1:]:
        lv["fanout"] = fanout
    return levels


def evaluate_centres(keys, values, queries, centres, assign, *, leaf_size=16, fanout=4, opening_threshold=0.01):
    """The law with one forest per centre: query i is evaluated against the forest of centres[assign[i]].
    Returns (out [N, Dv], lse [N], counters dict of [N] arrays, per-centre info list)."""
    q = np.asarray(queries, F64)
    n = q.shape[0]
    dv = np.asarray(values).shape[1]
    out = np.zeros((n, dv))
    lse = np.zeros(n)
    cnt = {k: np.zeros(n, np.int64) for k in ("visited_nodes", "accepted_nodes", "exact_leaves")}
    infos = []
    for c in range(np.asarray(centres).shape[0]):
        rows = np.nonzero(np.asarray(assign) == c)[0]
        if rows.size == 0:
            infos.append(None)
            continue
        lv = forest(keys, values, centres[c], leaf_size=leaf_size, fanout=fanout)
        o, s, info = evaluate(keys, values, q[rows], centres[c], lv, opening_threshold=opening_threshold)
        out[rows], lse[rows] = o, s
        for k in cnt:
            cnt[k][rows] = info[k]
        info["rows"] = rows
        infos.append(info)
    return out, lse, cnt, infos


def exact_attention(keys, values, queries):
    """Softmax attention for already-scaled queries (model.py:86-89), float64: (out, lse)."""
    lg = np.atleast_2d(np.asarray(queries, F64)) @ np.asarray(keys, F64).T
    lse = _lse(lg, 1)
    return np.exp(lg - lse[:, None]) @ np.asarray(values, F64), lse
