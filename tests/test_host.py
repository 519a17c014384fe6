"""Host-side checks that need no GPU: the C-ABI library loads and exports every function the header
declares, its argument validation and error names, and the Python layer's argument errors and memory
planning (h3/htrc_flat.py:118-132, :187-212; h3/htrc_flat_runner.py:61-84)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

import htrc_b200
from htrc_b200 import _lib, runner
from htrc_b200 import flat as F

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def _declared_functions():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(htrc_\w+)\s*\(", text))
    return sorted(names)


def _args(n=4096, m=4096, E=16, sink=0, dim=128, tile=64, leaf=64, chunk=0, ntail=0):
    a = _lib.HtrcFlatArgs()
    a.q_dtype = _lib.DTYPE_BF16
    a.n_queries, a.n_keys = n, m
    a.dim, a.tile, a.leaf = dim, tile, leaf
    a.exact_leaves, a.sink_leaves, a.tile_chunk, a.n_tail = E, sink, chunk, ntail
    return a


def test_library_exports_every_declared_symbol():
    names = _declared_functions()
    assert len(names) >= 13 and any(n.startswith("htrc_tree_") for n in names), names
    so = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in names if not hasattr(so, n)]
    assert not missing, missing
    # and the Python binding declares a signature for each
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_strerror_names_every_code():
    L = _lib.lib()
    seen = set()
    for code in range(7):
        s = L.htrc_strerror(code)
        assert isinstance(s, bytes) and s and s != b"unknown error"
        seen.add(s)
    assert len(seen) == 7
    assert L.htrc_strerror(99) == b"unknown error"


def test_leaf_pitch():
    for nb in (1, 15, 16, 17, 2016, 8192):
        p = F.leaf_pitch(nb)
        assert p >= nb and p % 16 == 0 and p - nb < 16


def test_workspace_size_validation():
    L = _lib.lib()
    nbytes = ctypes.c_size_t()
    size = lambda a: L.htrc_flat_workspace_size(ctypes.byref(a), ctypes.byref(nbytes))
    assert size(_args()) == _lib.HTRC_OK and nbytes.value > 0
    assert size(_args(m=4096 + 32)) == _lib.HTRC_ERR_ARG            # keys not a multiple of the leaf
    assert size(_args(n=0)) == _lib.HTRC_ERR_ARG
    assert size(_args(dim=64)) == _lib.HTRC_ERR_UNSUPPORTED
    assert size(_args(leaf=32)) == _lib.HTRC_OK                        # INT8 state, linear far field
    assert size(_args(leaf=16)) == _lib.HTRC_OK
    assert size(_args(leaf=8)) == _lib.HTRC_ERR_UNSUPPORTED
    assert size(_args(leaf=128)) == _lib.HTRC_ERR_UNSUPPORTED
    assert size(_args(tile=128)) == _lib.HTRC_ERR_UNSUPPORTED
    assert size(_args(tile=16)) == _lib.HTRC_ERR_UNSUPPORTED
    assert size(_args(tile=32)) == _lib.HTRC_OK                        # the "max" mode
    assert size(_args(E=-1)) == _lib.HTRC_ERR_ARG
    assert size(_args(m=64 * 9000)) == _lib.HTRC_ERR_UNSUPPORTED      # more leaves than the route kernel handles
    assert size(_args(m=64 * 2048, E=2000)) == _lib.HTRC_ERR_UNSUPPORTED  # more routed leaves than the tile kernel
    assert L.htrc_flat_workspace_size(ctypes.byref(_args()), None) == _lib.HTRC_ERR_ARG
    # chunking bounds the per-chunk leaf state, so a smaller chunk needs less
    assert size(_args(n=65536, m=65536, E=256, chunk=64)) == _lib.HTRC_OK
    small = nbytes.value
    assert size(_args(n=65536, m=65536, E=256, chunk=0)) == _lib.HTRC_OK
    assert small < nbytes.value
    assert F.workspace_bytes(65536, 65536, 256, 0, 64, 0) == small


def test_forward_rejects_missing_pointers_before_touching_a_device():
    L = _lib.lib()
    a = _args()
    assert L.htrc_flat_forward(ctypes.byref(a), None) == _lib.HTRC_ERR_ARG
    assert L.htrc_flat_forward(None, None) == _lib.HTRC_ERR_ARG


def test_static_workspace_entry_rejects_oversize_without_a_device():
    L = _lib.lib()
    a = _args(n=65536, m=65536, E=256)
    assert L.htrc_flat_forward_static_ws(ctypes.byref(a), None) == _lib.HTRC_ERR_TOO_LARGE
    assert b"64 MiB" in L.htrc_strerror(_lib.HTRC_ERR_TOO_LARGE)
    assert L.htrc_flat_forward_static_ws(None, None) == _lib.HTRC_ERR_ARG


def test_check_maps_codes_to_python_errors():
    _lib.check(_lib.HTRC_OK, "x")
    with pytest.raises(ValueError):
        _lib.check(_lib.HTRC_ERR_ARG, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.HTRC_ERR_UNSUPPORTED, "x")
    with pytest.raises(MemoryError):
        _lib.check(_lib.HTRC_ERR_WORKSPACE, "x")
    with pytest.raises(MemoryError):
        _lib.check(_lib.HTRC_ERR_TOO_LARGE, "x")
    with pytest.raises(_lib.HtrcError):
        _lib.check(_lib.HTRC_ERR_CUDA, "x")


def _qkv(n=256, m=256, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(0)
    return (torch.randn(n, 128, generator=g).to(dtype), torch.randn(m, 128, generator=g).to(dtype),
            torch.randn(m, 128, generator=g).to(dtype))


def test_flat_attention_argument_errors_match_the_reference():
    q, k, v = _qkv()
    cfg = dict(htrc_b200.PROD, leaf=64)
    with pytest.raises(ValueError, match="multiple of the leaf"):
        htrc_b200.flat_attention(q, k[:200], v[:200], **cfg)
    with pytest.raises(ValueError, match="curvature"):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "curvature": "iso"})
    with pytest.raises(ValueError, match="dot='bf16'"):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "store": "f32"})
    with pytest.raises(ValueError, match="unknown backend"):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "backend": "nope"})
    with pytest.raises(ValueError, match="store='fp8'"):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "select": "bound"})


def test_flat_attention_unimplemented_configurations_say_so():
    q, k, v = _qkv()
    cfg = dict(htrc_b200.PROD, leaf=64)
    with pytest.raises(NotImplementedError, match="tile=64 or 32"):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "tile": 16})
    with pytest.raises(NotImplementedError, match="leaf"):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "leaf": 8})
    with pytest.raises(NotImplementedError, match="leaf=32 is implemented for store='int8'"):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "leaf": 32, "store": "fp8"})
    with pytest.raises(NotImplementedError, match="leaf=16 is implemented for store='int8'"):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "leaf": 16, "backend": "cuda", "curvature": "iso"})
    with pytest.raises(NotImplementedError, match="one key scale per 64-key leaf"):
        htrc_b200.flat._check_scale_block(64, "int8", 16)
    with pytest.raises(NotImplementedError):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "store": "fp32", "dot": "tf32"})
    with pytest.raises(NotImplementedError, match="leaf=32 is implemented for store='int8'"):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "leaf": 32, "store": "bf16"})
    with pytest.raises(NotImplementedError):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "backend": "torch"})


def test_fp8_state_option_is_accepted_and_checked():
    """store='fp8' (the reference's e4m3 far-field state) passes the argument checks and then needs CUDA
    tensors like every other path; the iso curvature is refused on it; its workspace drops the INT8 key
    codes and halves the vbar state."""
    q, k, v = _qkv()
    cfg = dict(htrc_b200.PROD, leaf=64, store="fp8")
    for over in ({}, {"order": "kmeans"}, {"kern": {"group": 2}}, {"tile": 32}, {"sink_leaves": 1},
                 {"quant": {"kv": "int4", "q": "int8", "group": 32}}):
        with pytest.raises(ValueError, match="CUDA tensors"):
            htrc_b200.flat_attention(q, k, v, **{**cfg, **over})
    with pytest.raises(ValueError, match="store='fp8'"):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "quant": {"state": "int8"}})
    with pytest.raises(NotImplementedError, match="iso"):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "backend": "cuda", "curvature": "iso"})
    from htrc_b200 import flat as F
    n = m = 16384
    i8 = F.workspace_bytes(n, m, 256, store=_lib.STORE_INT8)
    f8 = F.workspace_bytes(n, m, 256, store=_lib.STORE_FP8)
    nt, nb = n // 64, m // 64
    # no k8/ks (m * 132), bf16 + fp16 query rows instead of two code rows and two scales (+ 512 - 264 bytes per
    # held row), vbar codes instead of bf16 (- nt*nb*128), plus sv (nt * pitch * 4); alignment slack
    want = i8 - m * 132 + nt * 64 * (512 - 264) - nt * nb * 128 + nt * F.leaf_pitch(nb) * 4
    assert abs(f8 - want) <= 8 * 256
    # with a far field the fp8 path also keeps one far partial row (dim + 2 floats) per query
    i8 = F.workspace_bytes(n, m, 64, store=_lib.STORE_INT8)
    f8 = F.workspace_bytes(n, m, 64, store=_lib.STORE_FP8)
    want = i8 - m * 132 + nt * 64 * (512 - 264) - nt * nb * 128 + nt * F.leaf_pitch(nb) * 4 + n * 130 * 4
    assert abs(f8 - want) <= 8 * 256
    a = _lib.HtrcFlatArgs()
    a.n_queries, a.n_keys, a.dim, a.tile, a.leaf, a.exact_leaves = n, m, 128, 64, 64, 256
    a.store, a.curvature = _lib.STORE_FP8, _lib.CURV_ISO
    nbytes = ctypes.c_size_t()
    assert _lib.lib().htrc_flat_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)) == _lib.HTRC_ERR_UNSUPPORTED
    a.store = 3
    assert _lib.lib().htrc_flat_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)) == _lib.HTRC_ERR_ARG


def test_orders_and_groups_need_no_cpu_path_either():
    q, k, v = _qkv()
    cfg = dict(htrc_b200.PROD, leaf=64)
    for over in ({"order": "kmeans"}, {"kern": {"group": 2}}, {"order": "kmeans", "kern": {"group": 4}},
                 {"order": "kmeans", "tile": 32}):
        with pytest.raises(ValueError, match="CUDA tensors"):
            htrc_b200.flat_attention(q, k, v, **{**cfg, **over})


def test_group_and_order_validation_and_workspace():
    L = _lib.lib()
    nbytes = ctypes.c_size_t()
    a = _args(n=65536, m=65536, E=256, chunk=64)
    assert L.htrc_flat_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)) == _lib.HTRC_OK
    base = nbytes.value
    a.group = 2                                     # half the centre rows: less far-field state per chunk
    assert L.htrc_flat_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)) == _lib.HTRC_OK
    assert nbytes.value < base
    a.group, a.order = 1, _lib.ORDER_KMEANS         # the permutation and the k-means scratch
    assert L.htrc_flat_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)) == _lib.HTRC_OK
    km = ctypes.c_size_t()
    assert L.htrc_kmeans_scratch_size(65536, ctypes.byref(km)) == _lib.HTRC_OK
    assert nbytes.value >= base + km.value + 65536 * 4
    a.order = 7
    assert L.htrc_flat_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)) == _lib.HTRC_ERR_ARG
    a.order, a.group = 0, 1 << 20
    assert L.htrc_flat_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)) == _lib.HTRC_ERR_ARG
    assert L.htrc_kmeans_scratch_size(0, ctypes.byref(km)) == _lib.HTRC_ERR_ARG
    assert L.htrc_kmeans_order(None, 0, 16, 128, None, None, 0, None) == _lib.HTRC_ERR_ARG


def test_group_and_order_of_the_reference_arguments():
    assert F.group_of(None) == 1 and F.group_of({}) == 1 and F.group_of({"group": 0}) == 1
    assert F.group_of({"group": 4, "tile_bn": 64}) == 4
    assert F.order_code("kmeans") == _lib.ORDER_KMEANS
    assert F.order_code("seq") == _lib.ORDER_SEQ and F.order_code("other") == _lib.ORDER_SEQ


def test_flat_attention_has_no_cpu_path():
    q, k, v = _qkv()
    with pytest.raises(ValueError, match="CUDA tensors"):
        htrc_b200.flat_attention(q, k, v, **htrc_b200.PROD, leaf=64)


def test_plan_chunk_takes_the_largest_chunk_that_fits():
    keys, q = 129024, 129024
    peaks = {c: runner.predicted_peak_mib(keys, 64, c, queries=q) for c in runner.CHUNKS}
    # the predicted peak grows with the chunk
    vals = [peaks[c] for c in sorted(peaks)]
    assert vals == sorted(vals)
    for c in runner.CHUNKS:
        free = int(peaks[c] * 2 ** 20) + 1
        got = runner.plan_chunk(free, keys, 64, queries=q)
        assert got == max(x for x in runner.CHUNKS if peaks[x] * 2 ** 20 <= free)
    with pytest.raises(MemoryError):
        runner.plan_chunk(1 << 20, keys, 64, queries=q)
    # with room for it, the whole sequence is one chunk (2016 tiles: every SM busy in one launch)
    assert runner.plan_chunk(1 << 40, keys, 64, queries=q) == -(-q // 64)
    assert runner.plan_chunk(1 << 40, 4096, 64, queries=4096) == 1024       # <= 1024 tiles: as the reference


def test_qk_scale_block_option_is_checked():
    """qk_scale_block (extension): None/0 or 64; INT8 store only; the C ABI says the same."""
    q, k, v = _qkv()
    cfg = dict(htrc_b200.PROD, leaf=64)
    with pytest.raises(ValueError, match="CUDA tensors"):
        htrc_b200.flat_attention(q, k, v, **{**cfg, "qk_scale_block": 64})
    with pytest.raises(ValueError, match="qk_scale_block"):
        htrc_b200.flat._check_scale_block(32, "int8")
    with pytest.raises(NotImplementedError, match="store='int8'"):
        htrc_b200.flat._check_scale_block(64, "fp8")
    assert htrc_b200.flat._check_scale_block(None, "int8") == 0
    a = _lib.HtrcFlatArgs()
    a.n_queries, a.n_keys, a.dim, a.tile, a.leaf, a.exact_leaves = 4096, 4096, 128, 64, 64, 16
    nbytes = ctypes.c_size_t()
    L = _lib.lib()
    a.qk_scale_block = 64
    assert L.htrc_flat_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)) == _lib.HTRC_OK
    a.qk_scale_block = 32
    assert L.htrc_flat_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)) == _lib.HTRC_ERR_ARG
    a.qk_scale_block, a.store = 64, _lib.STORE_FP8
    assert L.htrc_flat_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)) == _lib.HTRC_ERR_UNSUPPORTED


def test_forward_into_checks_every_buffer_before_any_launch():
    """forward_into rejects wrong shapes, dtypes, contiguity, an undersized route mask and buffers off the GPU
    with ValueError on the host (no kernel is launched: these tensors live on the CPU)."""
    n, m = 200, 256
    q = torch.zeros((n, 128), dtype=torch.float32)
    k = torch.zeros((m, 128), dtype=torch.bfloat16)
    v = torch.zeros((m, 128), dtype=torch.bfloat16)
    out = torch.zeros((n, 128), dtype=torch.float32)
    lse = torch.zeros((n,), dtype=torch.float32)
    ws = torch.zeros((1024,), dtype=torch.uint8)
    good = dict(exact_leaves=2, out=out, lse=lse, workspace=ws)

    def call(qd=q, kb=k, vb=v, tk=None, tv=None, **kw):
        F.forward_into(qd, kb, vb, tk, tv, **{**good, **kw})

    for kw, what in [(dict(kb=k.float()), "kb"), (dict(vb=v[:128]), "vb"), (dict(out=out[:, :64]), "out"),
                     (dict(out=out.double()), "out"), (dict(lse=lse[:10]), "lse"), (dict(qd=q.half()), "qd"),
                     (dict(out=torch.zeros((128, n)).T), "out"), (dict(workspace=ws.float()), "workspace"),
                     (dict(tk=torch.zeros((3, 128)), tv=None), "tv"),
                     (dict(route_mask=torch.zeros((3, 16), dtype=torch.uint8)), "route_mask"),
                     (dict(route_mask=torch.zeros((4, 16), dtype=torch.int32)), "route_mask")]:
        with pytest.raises(ValueError, match=what):
            call(**kw)
    # right shapes: ceil(200 / 64) = 4 tiles, leaf_pitch(256 / 64 = 4) = 16 -> 4 x 16 mask; still on the CPU
    with pytest.raises(ValueError, match="CUDA device"):
        call(route_mask=torch.zeros((4, 16), dtype=torch.uint8))
