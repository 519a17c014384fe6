"""GPU parity of the per-block INT8 scale extension (`qk_scale_block=64`: one scale per 64-key leaf and
per query tile: one absmax scale per 64-token block; the reference's scales are per key and per row,
so this mode has no reference fixture and is pinned to the oracle's restatement, `pack_blocks`)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import flat_oracle as O  # noqa: E402

OUT_TOL = 2e-2
LSE_TOL = 1e-3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from htrc_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


@pytest.mark.parametrize("rows", [4096, 1000, 37])
@pytest.mark.parametrize("rounding", ["even", "away"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_pack_blocks_bit_exact(dev, rows, rounding, dtype):
    from htrc_b200 import _lib
    from htrc_b200._lib import lib, ptr, stream_ptr
    g = torch.Generator().manual_seed(rows)
    x = torch.randn(rows, 128, generator=g) * torch.rand(rows, 1, generator=g) * 4
    if rows > 128:
        x[64:128] = 0.0                                   # an all-zero block: the 1e-20 floor
    x = x.to(dtype)
    xd = x.to(dev)
    x8 = torch.empty((rows, 128), dtype=torch.int8, device=dev)
    s = torch.empty((rows,), dtype=torch.float32, device=dev)
    rc = _lib.ROUND_HALF_EVEN if rounding == "even" else _lib.ROUND_HALF_AWAY
    dt = _lib.DTYPE_BF16 if dtype == torch.bfloat16 else _lib.DTYPE_F32
    _lib.check(lib().htrc_pack_int8_blocks(ptr(xd), dt, rows, 128, rc, 64, ptr(x8), ptr(s), None, stream_ptr()),
               "pack blocks")
    torch.cuda.synchronize()
    r8, rs = O.pack_blocks(x.float().numpy(), 64, rounding)
    assert np.array_equal(x8.cpu().numpy(), r8)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), rs.view(np.uint32))


@pytest.mark.parametrize("tile", [64, 32])
def test_tile_prep_block_scales_bit_exact(dev, tile):
    import htrc_b200
    from htrc_b200 import synth
    q, k, v = synth.head_inputs((2, 16, 32), 128, base_seed=31)
    q = q[:1000]
    st = htrc_b200.run_stages(q.to(dev), k.to(dev), v.to(dev), exact_leaves=2, tile=tile, qk_scale_block=64)
    torch.cuda.synchronize()
    qt, mu, _ = O.tile_centres(q.float().numpy(), tile)
    assert np.array_equal(st["mu"].cpu().numpy().view(np.uint32), mu.view(np.uint32))
    q8, sq, dq8, sdq = O.query_codes(qt, mu, q_block=True)
    nt = qt.shape[0]
    held = lambda a: a.reshape(nt, 64, *a.shape[1:])[:, :tile]          # noqa: E731  the real rows of a tile
    assert np.array_equal(held(st["q8"].cpu().numpy()), q8)
    assert np.array_equal(held(st["sq"].cpu().numpy()).view(np.uint32), sq.view(np.uint32))
    assert np.array_equal(held(st["dq8"].cpu().numpy()), dq8)
    k8, ks = O.pack_blocks(O.bf16_round(k.float().numpy()), 64, "even")
    assert np.array_equal(st["k8"].cpu().numpy(), k8)
    assert np.array_equal(st["ks"].cpu().numpy().view(np.uint32), ks.view(np.uint32))


@pytest.mark.parametrize("E,sink", [(4, 0), (7, 1)])
def test_block_scales_end_to_end(dev, E, sink):
    """flat_attention(**PROD, qk_scale_block=64) against the oracle with the same scales: rows of tiles whose
    routing the oracle reproduces within the output tolerance, log-Z over all rows; the fused forward equals
    the stage launches."""
    import htrc_b200
    from htrc_b200 import synth
    q, k, v = synth.head_inputs((4, 16, 32), 128, base_seed=33)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    cfg = {**htrc_b200.PROD, "leaf": 64, "exact_leaves": E, "sink_leaves": sink, "qk_scale_block": 64}
    out, lse = htrc_b200.flat_attention(qd, kd, vd, return_lse=True, **cfg)
    st = htrc_b200.run_stages(qd, kd, vd, exact_leaves=E, sink_leaves=sink, qk_scale_block=64)
    torch.cuda.synchronize()
    ro, rl, rst = O.flat_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), exact_leaves=E,
                                   sink_leaves=sink, qk_scale_block=64, return_stages=True, precision="tf32")
    nb = st["nb"]
    agree = (st["excl"][:, :nb].cpu().numpy() == rst["excl"]).all(1)
    assert (st["excl"][:, :nb].cpu().numpy() == rst["excl"]).mean() >= 0.999
    rows = np.repeat(agree, 64)[: q.shape[0]]
    o = out.cpu().numpy()
    assert np.abs(o[rows] - ro[rows]).max() < OUT_TOL
    assert np.abs(lse.cpu().numpy() - rl).mean() < LSE_TOL
    assert np.array_equal(o, st["out"].cpu().numpy())
