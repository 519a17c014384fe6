"""GPU checks that the fused forward reads only workspace bytes it wrote and writes every output row:
runs over workspaces pre-filled with different byte patterns (zeros, ones, 0xFF, random) and outputs
pre-filled with NaN give bitwise identical results, also across repeated runs on one workspace."""
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


def _fill(w, pattern, gen):
    body = w[256:]
    if pattern == "random":
        body.copy_(torch.randint(0, 256, body.shape, dtype=torch.uint8, generator=gen).to(w.device))
    else:
        body.fill_(pattern)
    w[:256].zero_()          # the status word starts at zero


@pytest.mark.parametrize("store,group,chunk", [("int8", 1, 0), ("int8", 2, 8), ("fp8", 1, 0)])
def test_results_do_not_depend_on_workspace_contents(dev, store, group, chunk):
    from htrc_b200 import _lib, synth
    from htrc_b200 import flat as F
    q, k, v = (t.to(dev) for t in synth.head_inputs((4, 24, 40), 128, base_seed=23))
    n, m = q.shape[0], k.shape[0]
    sc = _lib.STORES[store]
    gen = torch.Generator().manual_seed(5)
    w = F.new_workspace(F.workspace_bytes(n, m, 12, 1, chunk, group=group, store=sc), dev)
    results = []
    for pattern in (0x00, 0xFF, 0x01, "random", None, None):
        if pattern is not None:
            _fill(w, pattern, gen)
        out = torch.full((n, 128), float("nan"), device=dev)
        lse = torch.full((n,), float("nan"), device=dev)
        F.forward_into(q, k, v, None, None, exact_leaves=12, sink_leaves=1, tile_chunk=chunk, out=out, lse=lse,
                       workspace=w, group=group, store=sc)
        torch.cuda.synchronize()
        F.device_status(w)
        assert not torch.isnan(out).any() and not torch.isnan(lse).any(), "an output row was not written"
        results.append((out, lse))
    o0, l0 = results[0]
    for o, l in results[1:]:
        assert torch.equal(o, o0) and torch.equal(l, l0)


@pytest.mark.parametrize("store", ["int8", "fp8"])
def test_heads_on_two_streams_equal_one_stream(dev, store):
    """Heads alternating over two streams with a workspace each (as the benchmark runs a layer: one head's
    small kernels and the tail of its tile kernel overlap the next head) give bitwise the results of the
    same heads one after another on one stream, over repeated layers."""
    from htrc_b200 import _lib, synth
    from htrc_b200 import flat as F
    heads = [tuple(t.to(dev) for t in synth.head_inputs((8, 48, 84), 128, head=h, base_seed=31)) for h in range(6)]
    n, m = heads[0][0].shape[0], heads[0][1].shape[0]
    sc = _lib.STORES[store]
    E = 256
    wsb = F.workspace_bytes(n, m, E, store=sc)
    main = torch.cuda.current_stream(dev)
    streams = [main, torch.cuda.Stream(dev)]
    wss = [F.new_workspace(wsb, dev), F.new_workspace(wsb, dev)]

    def layer(nstreams, outs):
        streams[1].wait_stream(main)
        for i, (q, k, v) in enumerate(heads):
            s = streams[i % nstreams]
            with torch.cuda.stream(s):
                F.forward_into(q, k, v, None, None, exact_leaves=E, out=outs[i][0], lse=outs[i][1],
                               workspace=wss[i % nstreams], stream=s, store=sc)
        main.wait_stream(streams[1])

    def fresh():
        return [(torch.full((n, 128), float("nan"), device=dev), torch.full((n,), float("nan"), device=dev))
                for _ in heads]

    ref = fresh()
    layer(1, ref)
    torch.cuda.synchronize()
    for w in wss:
        F.device_status(w)
    for _ in range(3):
        got = fresh()
        layer(2, got)
        torch.cuda.synchronize()
        for w in wss:
            F.device_status(w)
        for (o, l), (ro, rl) in zip(got, ref):
            assert torch.equal(o, ro) and torch.equal(l, rl)
