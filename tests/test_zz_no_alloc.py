"""The allocation-free forward entry point, htrc_flat_forward_static_ws.

It exists for callers that cannot allocate device memory: a plugin whose host owns every device
allocation and lends it only the input and output buffers, or an embedding whose device footprint must
not grow once it has started.  Such callers pass q, k, v, out and lse as usual; the operator's scratch
lives in a fixed 64 MiB array inside the library instead of a caller-provided workspace.

These tests call it through the C ABI twice in a row (different inputs and routing budgets each time,
so stale contents of the shared array would show) and require bitwise the results of the ordinary entry
point, htrc_flat_forward, on a caller-allocated workspace (the kernels fix every reduction order, so the
workspace's address cannot change a bit), a clean device status word after each call (read through
htrc_flat_static_ws_status), and an unchanged amount of free device memory across the calls.  This file is
named so that pytest collects it last; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from htrc_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


def _args(q, k, v, out, lse, E, ws=None):
    from htrc_b200 import _lib
    a = _lib.HtrcFlatArgs()
    a.q, a.q_dtype = q.data_ptr(), _lib.DTYPE_BF16
    a.k, a.v = k.data_ptr(), v.data_ptr()
    a.n_queries, a.n_keys = q.shape[0], k.shape[0]
    a.dim, a.tile, a.leaf = 128, 64, 64
    a.exact_leaves, a.sink_leaves, a.tile_chunk, a.scale = E, 0, 0, 0.0
    a.out, a.lse = out.data_ptr(), lse.data_ptr()
    if ws is not None:
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    return a


def _inputs(grid, seed, dev):
    from htrc_b200 import synth
    q, k, v = synth.head_inputs(grid, 128, base_seed=seed)
    return q.to(dev), k.to(dev), v.to(dev)


def _static_status(L, _lib, stream):
    st = ctypes.c_int32(-1)
    _lib.check(L.htrc_flat_static_ws_status(st, stream), "htrc_flat_static_ws_status")
    return st.value


CASES = [((4, 32, 32), 901, 16), ((8, 16, 32), 902, 5)]


def test_static_workspace_matches_allocated_workspace_twice_in_a_row(dev):
    from htrc_b200 import _lib
    L = _lib.lib()
    stream = _lib.stream_ptr()
    for grid, seed, E in CASES:
        q, k, v = _inputs(grid, seed, dev)
        n = q.shape[0]
        ref_out = torch.empty((n, 128), dtype=torch.float32, device=dev)
        ref_lse = torch.empty((n,), dtype=torch.float32, device=dev)
        need = ctypes.c_size_t()
        a = _args(q, k, v, ref_out, ref_lse, E)
        _lib.check(L.htrc_flat_workspace_size(a, need), "workspace size")
        ws = torch.zeros(need.value, dtype=torch.uint8, device=dev)
        a = _args(q, k, v, ref_out, ref_lse, E, ws)
        _lib.check(L.htrc_flat_forward(a, stream), "htrc_flat_forward")
        out = torch.full((n, 128), float("nan"), dtype=torch.float32, device=dev)
        lse = torch.full((n,), float("nan"), dtype=torch.float32, device=dev)
        b = _args(q, k, v, out, lse, E)
        _lib.check(L.htrc_flat_forward_static_ws(b, stream), "htrc_flat_forward_static_ws")
        assert _static_status(L, _lib, stream) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(out).all() and torch.isfinite(lse).all()
        assert torch.equal(out, ref_out)
        assert torch.equal(lse, ref_lse)


def test_static_workspace_allocates_nothing(dev):
    """Free device memory is the same before and after repeated calls (after one warm-up call per case, which
    loads the kernels' code)."""
    from htrc_b200 import _lib
    L = _lib.lib()
    stream = _lib.stream_ptr()
    calls = []
    for grid, seed, E in CASES:
        q, k, v = _inputs(grid, seed, dev)
        out = torch.empty((q.shape[0], 128), dtype=torch.float32, device=dev)
        lse = torch.empty((q.shape[0],), dtype=torch.float32, device=dev)
        calls.append((q, k, v, out, lse, _args(q, k, v, out, lse, E)))
    for c in calls:
        _lib.check(L.htrc_flat_forward_static_ws(c[-1], stream), "htrc_flat_forward_static_ws")
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(dev)[0]
    for _ in range(3):
        for c in calls:
            _lib.check(L.htrc_flat_forward_static_ws(c[-1], stream), "htrc_flat_forward_static_ws")
            assert _static_status(L, _lib, stream) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(dev)[0] == free0


def test_static_workspace_rejects_problems_beyond_its_size(dev):
    from htrc_b200 import _lib
    L = _lib.lib()
    a = _lib.HtrcFlatArgs()
    a.q = a.k = a.v = a.out = 256        # never dereferenced: the size check comes first
    a.q_dtype = _lib.DTYPE_BF16
    a.n_queries, a.n_keys = 129024, 129024
    a.dim, a.tile, a.leaf, a.exact_leaves = 128, 64, 64, 256
    rc = L.htrc_flat_forward_static_ws(a, _lib.stream_ptr())
    assert rc == _lib.HTRC_ERR_TOO_LARGE
    assert b"64 MiB" in L.htrc_strerror(rc)
