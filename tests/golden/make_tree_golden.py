"""Generate the golden fixtures of the hierarchical HTRC law by running the REFERENCE's NumPy model itself.

Run once, in a container that has the reference checkout, naming its directory with ``HTRC_REFERENCE``
or ``--reference``:

    python tests/golden/make_tree_golden.py --reference <checkout> [case ...]

It imports the reference's ``src/htrc_reference/model.py`` unmodified and calls ``build_forest`` and
``evaluate`` (one query at a time, as the reference does) on seeded synthetic inputs, recording the
outputs, the per-query counters and the roots' statistics.  Inputs are not stored: every case names
the committed generator (``htrc_b200.synth``) and seed that remake them, and stores a SHA-256 of the
float32 input bytes so that a test can see a generator that drifted.  The fixtures are written as
``tests/golden/tree_<case>.npz``; the reference is never needed at test time.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from htrc_b200 import synth  # noqa: E402

# case -> inputs, scale, centres, leaf size, fanout, threshold, evaluated query rows
CASES = {
    # clustered keys (the benchmark's configuration-1 generator at d 128), four centres, three levels
    "cluster": dict(gen="cluster", n=2048, d=128, seed=5, centres=4, leaf=64, fanout=4, thr=0.02, every=8,
                    roots=True),
    # 1000 keys: the last leaf of 16 keys holds 8; one centre; the reference's default threshold
    "ragged": dict(gen="cluster", n=1000, d=128, seed=11, centres=1, leaf=16, fanout=4, thr=0.01, every=4),
    # 200 keys in 4 leaves of 64 (the last 8): the leaves are the roots
    "single": dict(gen="cluster", n=200, d=128, seed=12, centres=1, leaf=64, fanout=4, thr=0.02, every=1),
    # the smooth-field video generator at 16,384 tokens, leaf 64, fanout 16, eight centres
    "field": dict(gen="field", grid=(16, 32, 32), d=128, seed=0, centres=8, leaf=64, fanout=16, thr=0.02,
                  every=128),
}


def inputs(case):
    """Remake a case's float32 (q, k, v) from the committed generator."""
    c = CASES[case]
    if c["gen"] == "cluster":
        q, k, v = synth.cluster_inputs(c["n"], c["d"], clusters=32, seed=c["seed"])
    else:
        q, k, v = synth.head_inputs(c["grid"], c["d"], head=c["seed"])
        q, k, v = (x.float().numpy() for x in (q, k, v))
    return np.ascontiguousarray(q, np.float32), np.ascontiguousarray(k, np.float32), np.ascontiguousarray(v, np.float32)


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def centres_of(qs, count, iters=8):
    """Deterministic Lloyd centres of the scaled queries (evenly spaced rows as the start) and the
    nearest centre of every query (first minimum)."""
    qs = np.asarray(qs, np.float64)
    if count == 1:
        return qs.mean(0, keepdims=True), np.zeros(qs.shape[0], np.int64)
    c = qs[np.linspace(0, qs.shape[0] - 1, count).round().astype(int)].copy()
    for _ in range(iters):
        a = np.argmin(((qs[:, None] - c[None]) ** 2).sum(-1), 1)
        for j in range(count):
            if (a == j).any():
                c[j] = qs[a == j].mean(0)
    return c, np.argmin(((qs[:, None] - c[None]) ** 2).sum(-1), 1)


def load_model(ref):
    path = Path(ref) / "src" / "htrc_reference" / "model.py"
    spec = importlib.util.spec_from_file_location("htrc_reference_model", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def make(case, model):
    c = CASES[case]
    q, k, v = inputs(case)
    scale = 1.0 / np.sqrt(q.shape[1])
    qs = q.astype(np.float64) * scale
    cen, assign = centres_of(qs, c["centres"])
    rows = np.arange(0, q.shape[0], c["every"])
    out = np.zeros((rows.size, v.shape[1]))
    cnt = np.zeros((rows.size, 3), np.int64)
    roots = {}
    for j in range(cen.shape[0]):
        sel = np.nonzero(assign[rows] == j)[0]
        forest = model.build_forest(k.astype(np.float64), v.astype(np.float64), cen[j], leaf_size=c["leaf"],
                                    fanout=c["fanout"])
        if j == 0 and c.get("roots"):
            st = [n.stats for n in forest]         # centre 0's roots, float32 to keep the fixture small
            roots = {"root_L": np.array([s.log_mass for s in st]), "root_g": np.stack([s.gradient for s in st]),
                     "root_H": np.stack([s.hessian for s in st]).astype(np.float32),
                     "root_u": np.stack([s.value for s in st]),
                     "root_J": np.stack([s.value_jacobian for s in st]).astype(np.float32)}
        for i in sel:
            o, info = model.evaluate(k.astype(np.float64), v.astype(np.float64), qs[rows[i]], cen[j], forest,
                                     opening_threshold=c["thr"])
            out[i] = o
            cnt[i] = (info["visited_nodes"], info["accepted_nodes"], info["exact_leaves"])
    np.savez_compressed(HERE / f"tree_{case}.npz", rows=rows, out=out, counters=cnt, centres=cen, assign=assign,
                        scale=scale, leaf=c["leaf"], fanout=c["fanout"], thr=c["thr"], sha=digest(q, k, v), **roots)
    print(case, "queries", rows.size, "mean counters", cnt.mean(0))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("HTRC_REFERENCE"))
    ap.add_argument("cases", nargs="*")
    a = ap.parse_args()
    if not a.reference:
        raise SystemExit("name the reference checkout with --reference or HTRC_REFERENCE")
    model = load_model(a.reference)
    for case in a.cases or list(CASES):
        make(case, model)


if __name__ == "__main__":
    main()
