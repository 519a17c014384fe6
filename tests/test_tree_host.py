"""Host-side checks of the hierarchical operator that need no GPU: forest shapes and buffer sizes through the
C ABI (include/htrc_tree.h), its argument validation, and the Python layer's reference ValueErrors."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from htrc_b200 import _lib, tree


def _levels(**kw):
    d = tree._dims(kw.get("m", 245952), kw.get("n", 245952), kw.get("c", 32), kw.get("leaf", 64), kw.get("fanout", 16),
                   _lib.DTYPE_BF16, _lib.DTYPE_BF16, 0.088, kw.get("thr", 0.02))
    n = _lib._i32()
    nodes = (_lib._i32 * _lib.TREE_MAX_LEVELS)()
    rc = _lib.lib().htrc_tree_levels(ctypes.byref(d), ctypes.byref(n), nodes)
    return rc, [int(nodes[i]) for i in range(n.value)]


def _model_levels(m, leaf, fanout):
    """Level sizes of model.py:75-85: ceil(m / leaf) leaves, then groups of fanout while more than fanout."""
    n = [-(-m // leaf)]
    while n[-1] > fanout:
        n.append(-(-n[-1] // fanout))
    return n


@pytest.mark.parametrize("m,leaf,fanout", [(245952, 64, 16), (4096, 64, 16), (1000, 16, 4), (200, 64, 4), (128, 16, 4),
                                           (129024, 64, 16), (1, 1, 2), (65, 64, 64)])
def test_levels_follow_the_reference(m, leaf, fanout):
    rc, got = _levels(m=m, leaf=leaf, fanout=fanout)
    assert rc == _lib.HTRC_OK
    assert got == _model_levels(m, leaf, fanout)


@pytest.mark.parametrize("kw", [dict(leaf=0), dict(leaf=65), dict(fanout=1), dict(fanout=65), dict(c=0), dict(c=257),
                                dict(thr=-1.0), dict(thr=float("nan")), dict(m=0)])
def test_invalid_dims_are_rejected(kw):
    rc, _ = _levels(**kw)
    assert rc == _lib.HTRC_ERR_ARG


def test_buffer_sizes():
    L = _lib.lib()
    d = tree._dims(245952, 245952, 32, 64, 16, _lib.DTYPE_BF16, _lib.DTYPE_BF16, 0.088, 0.02)
    f, w, r = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    assert L.htrc_tree_forest_size(ctypes.byref(d), ctypes.byref(f)) == _lib.HTRC_OK
    assert L.htrc_tree_walk_size(ctypes.byref(d), ctypes.byref(w)) == _lib.HTRC_OK
    assert L.htrc_tree_records_size(1000, ctypes.byref(r)) == _lib.HTRC_OK
    # level 1 (241 nodes) and the roots (16) carry H and J in float32 and as bf16 hi + lo operand copies:
    # 4 x 64 KiB per (centre, node)
    assert f.value >= 32 * (241 + 16) * 4 * 128 * 128 * 4
    assert f.value < 2.3e9 and w.value < 0.3e9
    assert r.value >= 1000 * (128 + 2) * 4
    assert L.htrc_tree_records_size(-1, ctypes.byref(r)) == _lib.HTRC_ERR_ARG


def test_entry_points_validate_before_the_device():
    L = _lib.lib()
    d = tree._dims(1000, 10, 1, 16, 4, _lib.DTYPE_F32, _lib.DTYPE_F32, 1.0, 0.01)
    nrec = _lib._i64(-5)
    # null inputs are argument errors; a missing walk buffer is a workspace error
    assert L.htrc_tree_build(ctypes.byref(d), None, None, None, None, 0, None) == _lib.HTRC_ERR_ARG
    assert L.htrc_tree_walk(ctypes.byref(d), None, None, None, None, None, 0, None, None, None, None, None) == \
        _lib.HTRC_ERR_ARG
    assert L.htrc_tree_walk(ctypes.byref(d), 1, 1, 1, 1, None, 0, 1, 1, None, ctypes.byref(nrec), None) == \
        _lib.HTRC_ERR_WORKSPACE
    assert nrec.value == 0
    d.q_dtype = _lib.DTYPE_BF16                            # queries and keys must share a dtype
    assert L.htrc_tree_walk(ctypes.byref(d), 1, 1, 1, 1, None, 0, 1, 1, None, ctypes.byref(nrec), None) == \
        _lib.HTRC_ERR_UNSUPPORTED
    d0 = tree._dims(1000, 0, 1, 16, 4, _lib.DTYPE_F32, _lib.DTYPE_F32, 1.0, 0.01)
    assert L.htrc_tree_walk(ctypes.byref(d0), None, None, None, None, None, 0, None, None, None, ctypes.byref(nrec),
                            None) == _lib.HTRC_OK
    assert nrec.value == 0


def test_python_layer_raises_the_reference_errors_without_a_device():
    k = np.zeros((16, 8))
    with pytest.raises(ValueError):
        tree.build_forest(k, k, np.zeros(8), leaf_size=0)
    with pytest.raises(ValueError):
        tree.build_forest(k, k, np.zeros(8), fanout=1)
    with pytest.raises(NotImplementedError):
        tree.build_forest(k, k, np.zeros(8), leaf_size=128)
    with pytest.raises(ValueError):
        tree.evaluate(k, k, np.zeros(8), np.zeros(8), None, opening_threshold=-1)
    with pytest.raises(TypeError):
        tree.evaluate(k, k, np.zeros(8), np.zeros(8), None)
