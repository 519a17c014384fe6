"""Seeded random configurations of the whole operator (sizes, routing, sink and tail keys, groups, orders,
tile rows, state format, leaf size, chunking): the fused forward equals the stage-by-stage launches bit for bit, and
both agree with the oracle within the operator tolerance on the rows of tiles whose routing the oracle
reproduces (routing agreement >= 99.9%)."""
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


def _config(seed):
    r = np.random.default_rng(1000 + seed)
    n = int(r.integers(1, 2600))
    nb = int(r.integers(1, 90))
    c = dict(n=n, m=64 * nb, E=int(r.integers(0, nb + 3)), sink=int(r.integers(0, 3)),
             n_tail=int(r.choice([0, 0, 3, 16, 21])), group=int(r.choice([1, 1, 2, 3, 4])),
             order=str(r.choice(["seq", "kmeans"])), tile=int(r.choice([64, 64, 32])),
             store=str(r.choice(["int8", "int8", "fp8"])), chunk=int(r.choice([0, 0, 4, 7])),
             qdtype=str(r.choice(["bf16", "f32"])), seed=seed, leaf=64)
    if seed >= 32:
        # the later seeds also draw the bf16 state and leaves of 32 / 16 keys (INT8 state)
        c["store"] = str(r.choice(["int8", "fp8", "bf16"]))
        c["leaf"] = int(r.choice([64, 32, 16])) if c["store"] == "int8" else 64
        nbl = int(r.integers(1, 200))
        c["m"], c["E"] = c["leaf"] * nbl, int(r.integers(0, nbl + 3))
    return c


@pytest.mark.parametrize("seed", range(48))
def test_random_configuration(dev, seed):
    import htrc_b200
    from htrc_b200 import _lib
    from htrc_b200 import flat as F
    c = _config(seed)
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(max(1, -(-c["m"] // 64)), 128, generator=g) * 2.0
    k = torch.randn(c["m"], 128, generator=g) * 1.5 + base.repeat_interleave(64, 0)[: c["m"]]
    q = torch.randn(c["n"], 128, generator=g) * 1.5 + base[torch.randint(0, base.shape[0], (c["n"],), generator=g)]
    v = torch.randn(c["m"], 128, generator=g)
    k, v = k.to(torch.bfloat16), v.to(torch.bfloat16)
    q = q.to(torch.bfloat16) if c["qdtype"] == "bf16" else q
    tail = None
    if c["n_tail"]:
        tail = (torch.randn(c["n_tail"], 128, generator=g), torch.randn(c["n_tail"], 128, generator=g))
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    td = None if tail is None else (tail[0].to(dev), tail[1].to(dev))
    cfg = {**htrc_b200.PROD, "leaf": c["leaf"], "exact_leaves": c["E"], "sink_leaves": c["sink"], "tile": c["tile"],
           "order": c["order"], "kern": {"group": c["group"]}, "store": c["store"], "tile_chunk": c["chunk"]}
    out, lse = htrc_b200.flat_attention(qd, kd, vd, tail=td, return_lse=True, **cfg)
    st = htrc_b200.run_stages(qd, kd, vd, *(td if td else (None, None)), exact_leaves=c["E"], sink_leaves=c["sink"],
                              group=c["group"], order=F.order_code(c["order"]), tile=c["tile"],
                              store=_lib.STORES[c["store"]], leaf=c["leaf"])
    torch.cuda.synchronize()
    assert int(st["status"].item()) == 0, c
    assert torch.equal(out, st["out"]) and torch.equal(lse, st["lse"]), c
    perm = st["perm"].cpu().numpy() if st["perm"] is not None else None
    tn = None if tail is None else (tail[0].numpy(), tail[1].numpy())
    ro, rl, rst = O.flat_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), exact_leaves=c["E"],
                                   sink_leaves=c["sink"], tail=tn, tile=c["tile"], group=c["group"], leaf=c["leaf"],
                                   order=c["order"], perm=perm, store=c["store"], return_stages=True,
                                   precision="tf32")
    nb = st["nb"]
    ex_d = st["excl"][:, :nb].cpu().numpy()
    assert (ex_d == rst["excl"]).mean() >= 0.999, c
    agree = (ex_d == rst["excl"]).all(1)
    i = np.arange(c["n"])
    same = agree[(i // c["tile"]) // c["group"]]                 # tile-order rows whose routing agrees
    rows = i if perm is None else perm.astype(np.int64)
    o = out.cpu().numpy()
    if same.any():
        err = np.abs(o[rows[same]] - ro[rows[same]]).max(1)
        if c["store"] == "fp8":
            # independent statistics: an e4m3 code on the other side of a rounding boundary moves its value by
            # one step of a 3-bit mantissa (12.5%), which can carry a far-dominated row past 2e-2
            assert (err < OUT_TOL).mean() >= 0.99 and err.max() < 2.5 * OUT_TOL, (c, err.max())
        else:
            assert err.max() < OUT_TOL, c
    assert np.abs(lse.cpu().numpy() - rl).mean() < LSE_TOL, c
