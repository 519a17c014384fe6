"""GPU checks of the API additions: the routing-mask export of the fused forward (`route_mask`) and the
head-batched entry `flat_attention_heads`."""
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


def _head(seed, grid=(2, 16, 32)):
    from htrc_b200 import synth
    return synth.head_inputs(grid, 128, base_seed=seed)


@pytest.mark.parametrize("group,chunk,store", [(1, 0, "int8"), (2, 6, "int8"), (1, 4, "fp8")])
def test_route_mask_export_equals_the_stage_masks(dev, group, chunk, store):
    import htrc_b200
    from htrc_b200 import _lib
    from htrc_b200 import flat as F
    q, k, v = (t.to(dev) for t in _head(41))
    n, m = q.shape[0], k.shape[0]
    nt, nb = -(-n // 64), m // 64
    ng = -(-nt // group)
    sc = _lib.STORES[store]
    st = htrc_b200.run_stages(q, k, v, exact_leaves=3, sink_leaves=1, group=group, store=sc)
    mask = torch.full((ng, F.leaf_pitch(nb)), 7, dtype=torch.uint8, device=dev)
    out = torch.empty((n, 128), device=dev)
    w = F.new_workspace(F.workspace_bytes(n, m, 3, 1, chunk, group=group, store=sc), dev)
    F.forward_into(q, k, v, None, None, exact_leaves=3, sink_leaves=1, tile_chunk=chunk, out=out, workspace=w,
                   group=group, store=sc, route_mask=mask)
    torch.cuda.synchronize()
    F.device_status(w)
    assert torch.equal(mask[:, :nb], st["excl"][:, :nb])
    assert torch.equal(out, st["out"])


def test_head_batched_entry_equals_per_head_calls(dev):
    import htrc_b200
    heads = [_head(50 + h) for h in range(3)]
    q = torch.stack([h[0] for h in heads]).to(dev)
    k = torch.stack([h[1] for h in heads]).to(dev)
    v = torch.stack([h[2] for h in heads]).to(dev)
    cfg = {**htrc_b200.PROD, "leaf": 64, "exact_leaves": 4}
    out, lse = htrc_b200.flat_attention_heads(q, k, v, return_lse=True, **cfg)
    torch.cuda.synchronize()
    for h in range(3):
        o1, l1 = htrc_b200.flat_attention(q[h], k[h], v[h], return_lse=True, **cfg)
        assert torch.equal(out[h], o1) and torch.equal(lse[h], l1)
    with pytest.raises(ValueError):
        htrc_b200.flat_attention_heads(q[0], k[0], v[0], **cfg)
