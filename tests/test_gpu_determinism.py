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


@pytest.mark.parametrize("store,group,chunk", [("int8", 1, 0), ("int8", 2, 8), ("fp8", 1, 0), ("bf16", 1, 0)])
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


@pytest.mark.parametrize("store", ["int8", "fp8", "bf16"])
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


@pytest.mark.parametrize("store,runs", [("int8", 10000), ("fp8", 5000), ("bf16", 5000)])
def test_row_max_stage_repeats_bitwise(dev, store, runs):
    """The row-max selection of one full-size head (129,024 tokens: 2,016 tiles x 16 blocks of 128 leaves),
    launched thousands of times on the same state, writes bitwise the same sel every time.  The reducing
    warps read each stage's sg / lz with ordinary shared-memory loads before releasing the stage to the TMA
    refill; without a generic-to-async proxy fence between those reads and the release, the refill could land
    first (about one warp-block in 10^7 read the next block's sg or lz), which this many blocks exposes."""
    from htrc_b200 import _lib, synth
    from htrc_b200 import flat as F
    from htrc_b200._lib import check, ptr
    q, k, v = (t.to(dev) for t in synth.head_inputs((32, 48, 84), 128, head=5, base_seed=31))
    sc = _lib.STORES[store]
    r = F.run_stages(q, k, v, exact_leaves=256, precision=F.precision_code("tf32", "triton"), store=sc)
    for key in ("vb", "vbb"):
        r.pop(key, None)
    torch.cuda.synchronize()
    L = _lib.lib()
    nt, nb = r["sel"].shape[0], r["nb"]
    s = torch.cuda.current_stream().cuda_stream
    stp = ptr(r["status"])
    sel0 = r["sel"][:, :nb].clone()
    buf = torch.zeros_like(r["sel"])
    bad = torch.zeros((), dtype=torch.int64, device=dev)
    for _ in range(runs):
        if sc == _lib.STORE_FP8:
            check(L.htrc_rowmax_select_fp8(ptr(r["dqh"]), 0, nt, 1, ptr(r["g8"]), ptr(r["sg"]), ptr(r["lz"]), nb,
                                           128, ptr(buf), stp, s), "htrc_rowmax_select_fp8")
        elif sc == _lib.STORE_BF16:
            check(L.htrc_rowmax_select_bf16(ptr(r["dqb"]), 0, nt, 1, ptr(r["gb"]), ptr(r["lz"]), nb, 128, ptr(buf),
                                            stp, s), "htrc_rowmax_select_bf16")
        else:
            check(L.htrc_rowmax_select(ptr(r["dq8"]), ptr(r["sdq"]), None, 0, nt, 1, ptr(r["g8"]), ptr(r["sg"]),
                                       ptr(r["lz"]), None, nb, 128, ptr(buf), stp, s), "htrc_rowmax_select")
        bad += (buf[:, :nb] != sel0).sum()
    torch.cuda.synchronize()
    assert int(r["status"].item()) == 0
    assert int(bad) == 0, f"{int(bad)} sel entries differed over {runs} runs"
