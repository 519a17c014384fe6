"""Pins the CPU oracle (oracle/flat_oracle.py) against fixtures recorded from the reference operator
itself (tests/golden/make_golden.py ran h3/htrc_flat.py with PROD int8 settings)."""
import numpy as np
import pytest

from oracle import flat_oracle as O

CASES = ["base", "ragged", "sink_tail", "all_exact", "no_exact", "big_tail", "leaf32", "wide",
         "group2", "group4", "kmeans", "kmeans_g2_tail", "kmeans_sampled", "tile32", "max_mode", "tile32_g2",
         "quant_kv_q"]
SLIM = {"kmeans_sampled"}                      # no recorded per-(tile, leaf) state
STATE_CASES = [c for c in CASES if c not in SLIM]
KMEANS_CASES = ["kmeans", "kmeans_g2_tail", "kmeans_sampled", "max_mode"]


def _group(z):
    return int(z["group"]) if "group" in z else 1


def _quant(z):
    if "quant_kv" not in z:
        return None
    return {"kv": str(z["quant_kv"]), "q": str(z["quant_q"]), "group": int(z["quant_group"])}


def _stages(z):
    """The oracle on a fixture's inputs; a k-means case uses the reference's recorded permutation
    (the oracle's own is checked separately)."""
    tail = (z["tail_k"], z["tail_v"]) if "tail_k" in z else None
    order = "kmeans" if "perm" in z else "seq"
    return O.flat_attention(z["q"], z["k"], z["v"], leaf=int(z["leaf"]),
                            exact_leaves=int(z["exact_leaves"]), sink_leaves=int(z["sink_leaves"]),
                            tail=tail, return_stages=True, group=_group(z), order=order,
                            perm=z.get("perm"), tile=int(z["tile"]) if "tile" in z else 64,
                            quant=_quant(z)), tail


def _v_used(z):
    q = _quant(z)
    return O.fake_quant(z["v"], q["kv"], q["group"]) if q else z["v"]


def _tile_mu(z, nt):
    return z["mu"][np.arange(nt) // _group(z)]


@pytest.mark.parametrize("case", STATE_CASES)
def test_key_pack_bit_exact(golden_cases, case):
    z = golden_cases[case]
    q = _quant(z)
    k8, ks = O.pack_k(O.fake_quant(z["k"], q["kv"], q["group"]) if q else z["k"])
    assert np.array_equal(k8, z["k8"])
    assert np.array_equal(ks.view(np.uint32), z["ks"].view(np.uint32))


@pytest.mark.parametrize("case", CASES)
def test_centres(golden_cases, case):
    """Tile centres (group 1: over the real rows) and group centres (all G * 64 padded rows)."""
    z = golden_cases[case]
    (out, lse, st), _ = _stages(z)
    assert st["mu"].shape == z["mu"].shape
    assert np.abs(st["mu"] - z["mu"]).max() <= 1e-7 * max(1.0, np.abs(z["mu"]).max())


@pytest.mark.parametrize("case", STATE_CASES)
def test_centres_and_leaf_state(golden_cases, case):
    z = golden_cases[case]
    (out, lse, st), _ = _stages(z)
    assert np.abs(st["mu"] - z["mu"]).max() <= 1e-7 * max(1.0, np.abs(z["mu"]).max())
    # lz / sg / vbar: float32 products of the fp64 statistics vs the reference's float32 kernels
    assert np.abs(st["lz"] - z["lz"]).max() < 1e-5
    assert np.abs(st["sg"] / z["sg"] - 1).max() < 1e-5
    assert np.abs(st["vb"] - z["vb"]).max() <= 2.0 ** -8 * max(1.0, np.abs(z["vb"]).max())
    # int8 slope codes: identical except at most 1 LSB on the rare code sitting on a .5 boundary
    diff = np.abs(st["g8"].astype(int) - z["g8"].astype(int))
    assert diff.max() <= 1 and (diff > 0).mean() < 1e-4


def test_slope_pack_bit_exact_on_identical_input():
    rng = np.random.default_rng(5)
    g = (rng.standard_normal((64, 128)) * rng.uniform(0.01, 3, (64, 1))).astype(np.float32)
    g8, sg = O.pack_slope(g)
    # the formula, written out independently in float32
    am = np.maximum(np.abs(g).max(1), np.float32(1e-30))
    sg2 = am * np.float32(1 / 127)
    y = g * (np.float32(127) / am)[:, None]
    g82 = np.trunc(np.where(y >= 0, y + np.float32(0.5), y - np.float32(0.5))).astype(np.int8)
    assert np.array_equal(g8, g82) and np.array_equal(sg, sg2)
    assert np.abs(g8).max() <= 127


@pytest.mark.parametrize("case", [c for c in STATE_CASES if c != "no_exact"])
def test_rowmax_selection_and_routing(golden_cases, case):
    z = golden_cases[case]
    (out, lse, st), _ = _stages(z)
    # evaluated on the reference's own state, the selection is identical up to float32 rounding
    q8, sq, dq8, sdq = O.query_codes(st["qt"], _tile_mu(z, st["qt"].shape[0]))
    sel = O.rowmax_select(dq8, sdq, z["g8"], z["sg"], z["lz"], _group(z))
    assert np.abs(sel - z["sel"]).max() < 1e-4
    assert (st["excl"] == z["excl"]).mean() >= 0.999


@pytest.mark.parametrize("case", STATE_CASES)
def test_ordered_restatement_matches_reference(golden_cases, case):
    """With the reference's own state and block order, the restated online softmax reproduces the
    reference's output to float32 rounding."""
    z = golden_cases[case]
    (out, lse, st), tail = _stages(z)
    ng = z["mu"].shape[0]
    idx = z["idx"] if "idx" in z else np.zeros((ng, 0), np.int32)
    q8, sq, dq8, sdq = O.query_codes(st["qt"], _tile_mu(z, st["qt"].shape[0]))
    o2, l2 = O.tile_attention_ordered(st["qt"], q8, sq, dq8, sdq, z["g8"], z["sg"], z["lz"], z["vb"],
                                      z["excl"], idx, z["k8"], z["ks"], O.bf16_round(_v_used(z)),
                                      int(z["leaf"]), 1 / np.sqrt(128), tail=tail, group=_group(z))
    n = z["q"].shape[0]
    o2, l2 = o2[:n], l2[:n]
    if "perm" in z:                                      # tile order -> the caller's row order
        full, full_l = np.empty_like(o2), np.empty_like(l2)
        full[z["perm"]], full_l[z["perm"]] = o2, l2
        o2, l2 = full, full_l
    assert np.abs(o2 - z["out"]).max() < 2e-5
    if "lse" in z:
        assert np.abs(l2 - z["lse"]).max() < 2e-5


@pytest.mark.parametrize("case", CASES)
def test_order_free_oracle_within_tolerance(golden_cases, case):
    """The order-free oracle (the checker of the CUDA path) agrees with the reference's output to
    well inside the parity tolerance (out max-abs 2e-2, log-Z mean-abs 1e-3)."""
    z = golden_cases[case]
    (out, lse, st), _ = _stages(z)
    assert np.abs(out - z["out"]).max() < 1e-2
    if "lse" in z:
        assert np.abs(lse - z["lse"]).mean() < 1e-4


def test_all_leaves_exact_is_dequantised_softmax(golden_cases):
    """exact_leaves >= nb: the operator is softmax attention over the INT8-dequantised logits."""
    z = golden_cases["all_exact"]
    (out, lse, st), _ = _stages(z)
    n = z["q"].shape[0]
    qd = (st["q8"].astype(np.float64) * st["sq"][..., None]).reshape(-1, 128)[:n]
    kd = st["k8"].astype(np.float64) * st["ks"][:, None]
    s = qd @ kd.T / np.sqrt(128)
    m = s.max(1, keepdims=True)
    p = np.exp(s - m)
    ref = p @ O.bf16_round(z["v"]).astype(np.float64) / p.sum(1, keepdims=True)
    assert np.abs(out - ref).max() < 1e-2
    assert np.abs(lse - (m[:, 0] + np.log(p.sum(1)))).max() < 1e-4


@pytest.mark.parametrize("case", KMEANS_CASES)
def test_kmeans_order_matches_reference(golden_cases, case):
    """The restated k-means order reproduces the reference's permutation (sampled Lloyd + stable
    sort; the last case has more rows than the 4096-row sample)."""
    z = golden_cases[case]
    assert np.array_equal(O.kmeans_order(z["q"]), z["perm"])


def test_linspace_matches_torch():
    """The float32 linspace formula behind the k-means sample and seed rows."""
    torch = pytest.importorskip("torch")
    for n in list(range(1, 200)) + [4095, 4096, 4097, 40759, 129024, 245952, 1000003]:
        s = min(4096, n)
        assert np.array_equal(O.linspace_f32(n - 1, s), torch.linspace(0, n - 1, s).numpy()), n
        assert np.array_equal(O.linspace_f32(s - 1, 32), torch.linspace(0, s - 1, 32).numpy()), n


def test_groups_of_three_restate_the_rule():
    """G = 3 is outside what the reference's kernels compile for (tl.arange needs a power of two
    rows); the oracle applies the same rule: the centre of a group is the mean of its padded tiles,
    its selection the maximum over its tiles and every tile of a group uses one state row."""
    rng = np.random.default_rng(3)
    q = rng.standard_normal((7 * 64 - 5, 128)).astype(np.float32)
    k = rng.standard_normal((512, 128)).astype(np.float32)
    v = rng.standard_normal((512, 128)).astype(np.float32)
    out, lse, st = O.flat_attention(q, k, v, exact_leaves=2, group=3, return_stages=True)
    assert st["mu"].shape == (3, 128) and st["idx"].shape == (3, 2)
    qt = st["qt"]
    pad = np.concatenate([qt, qt[-1:], qt[-1:]], 0)             # 7 tiles -> 9 = 3 groups of 3
    assert np.allclose(st["mu"], pad.reshape(3, 192, 128).mean(1), atol=1e-6)
    gt = np.arange(7) // 3
    per_tile = O.rowmax_select(st["dq8"], st["sdq"], st["g8"][gt], st["sg"][gt], st["lz"][gt])
    for g in range(3):
        assert np.array_equal(st["sel"][g], per_tile[3 * g:3 * g + 3].max(0))
    # with every leaf exact the grouping of the centres does not matter
    o3 = O.flat_attention(q, k, v, exact_leaves=99, group=3)[0]
    o1 = O.flat_attention(q, k, v, exact_leaves=99, group=1)[0]
    assert np.array_equal(o3, o1)


def test_fake_quant_bit_exact_against_reference(golden_cases):
    """h3/htrc_flat.py:68-97 on float32 and bf16 rows of varied scale (a zero row, tiny values)."""
    z = golden_cases["fake_quant"]
    for fmt in ("int8", "int4", "fp8", "fp4"):
        for grp in (0, 16, 32):
            for xk, yk in (("x", "y"), ("xb", "yb")):
                got = O.fake_quant(z[xk], fmt, grp)
                assert np.array_equal(got, z[f"{yk}_{fmt}_{grp}"]), (fmt, grp, xk)


def test_e4m3_rounding_matches_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(0)
    t = np.concatenate([rng.uniform(-448, 448, 20000),
                        rng.uniform(-1, 1, 20000) * 2.0 ** rng.integers(-12, 0, 20000)]).astype(np.float32)
    ref = torch.from_numpy(t).to(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(O.e4m3_round(t), ref)


def test_dequant_rows_against_reference(golden_cases):
    import torch
    z = golden_cases["fake_quant"]
    vals = torch.from_numpy(z["codes"]).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(O.dequant_rows(vals, z["dq_scale"]), z["dq_out"])


@pytest.mark.parametrize("curv", ["lin", "iso"])
@pytest.mark.parametrize("e", [0, 3, 8])
def test_f32_specification_matches_reference_torch_backend(golden_cases, curv, e):
    """The reference's float32 torch backend, including the isotropic curvature term it alone defines."""
    z = golden_cases["torch_spec"]
    got = O.flat_attention_f32(z["q"], z["k"], z["v"], exact_leaves=e, leaf=64, curvature=curv)
    assert np.abs(got - z[f"out_{curv}_{e}"]).max() < 1e-4


def test_iso_term_properties():
    """On the INT8 path: the curvature coefficients are non-negative, the term changes only the far
    field (every leaf exact -> identical to lin), and with far leaves it changes the output."""
    rng = np.random.default_rng(7)
    q = rng.standard_normal((300, 128)).astype(np.float32)
    k = rng.standard_normal((512, 128)).astype(np.float32)
    v = rng.standard_normal((512, 128)).astype(np.float32)
    o_iso, _, st = O.flat_attention(q, k, v, exact_leaves=2, curvature="iso", return_stages=True)
    assert (st["cv"] >= 0).all() and st["cv"].max() > 0
    assert np.allclose(st["dd"], ((st["qt"] - st["mu"][:, None, :]) ** 2).sum(-1), rtol=1e-5)
    o_lin, _ = O.flat_attention(q, k, v, exact_leaves=2)
    assert np.abs(o_iso - o_lin).max() > 1e-3
    a, _ = O.flat_attention(q, k, v, exact_leaves=99, curvature="iso")
    b, _ = O.flat_attention(q, k, v, exact_leaves=99)
    assert np.array_equal(a, b)


def test_route_sink_and_ties():
    sel = np.array([[0.0, 5.0, 5.0, 1.0, 9.0]], np.float32)
    idx, excl = O.route(sel, 2, sink_leaves=1)
    assert idx.tolist() == [[0, 1, 4]]
    assert excl.tolist() == [[1, 1, 0, 0, 1]]
    idx, excl = O.route(sel, 0)
    assert idx.shape == (1, 0) and excl.sum() == 0
    idx, _ = O.route(sel, 99)
    assert idx.tolist() == [[0, 1, 2, 3, 4]]


FP8_CASES = ["fp8_state", "fp8_sink_tail"]


def _fp8(z):
    tail = (z["tail_k"], z["tail_v"]) if "tail_k" in z else None
    out, lse, st = O.flat_attention(z["q"], z["k"], z["v"], leaf=int(z["leaf"]),
                                    exact_leaves=int(z["exact_leaves"]), sink_leaves=int(z["sink_leaves"]),
                                    tail=tail, return_stages=True, store="fp8")
    return out, lse, st, tail


@pytest.mark.parametrize("case", FP8_CASES)
def test_fp8_state_bit_exact(golden_cases, case):
    """store="fp8": the e4m3 codes of g / sg and vbar / sv are the reference's, byte for byte, and the
    row scales agree to float32 rounding of the leaf statistics."""
    z = golden_cases[case]
    out, lse, st, _ = _fp8(z)
    assert np.array_equal(O.e4m3_codes(st["gq"]), z["g_e4m3"])
    assert np.array_equal(O.e4m3_codes(st["vq"]), z["vb_e4m3"])
    assert np.array_equal(O.e4m3_values(z["g_e4m3"]), st["gq"])
    assert np.allclose(st["sg"], z["sg"], rtol=2e-6, atol=0)
    assert np.allclose(st["sv"], z["sv"], rtol=2e-6, atol=0)
    assert np.allclose(st["sel"], z["sel"], rtol=0, atol=1e-4)
    assert np.array_equal(st["excl"], z["excl"])
    assert np.array_equal(np.sort(st["idx"], 1), np.sort(z["idx"], 1))


@pytest.mark.parametrize("case", FP8_CASES)
def test_fp8_ordered_restatement_matches_reference(golden_cases, case):
    """The fp8 tile attention in the reference kernel's order, fed the reference's own state, reproduces
    its output to float32 accumulation-order error."""
    z = golden_cases[case]
    out, lse, st, tail = _fp8(z)
    gq, vq = O.e4m3_values(z["g_e4m3"]), O.e4m3_values(z["vb_e4m3"])
    qb, dqh = O.query_codes_fp8(st["qt"], z["mu"])
    assert np.allclose(O.rowmax_select_fp8(dqh, gq, z["sg"], z["lz"]), z["sel"], rtol=0, atol=2e-5)
    o, l = O.tile_attention_fp8_ordered(st["qt"], qb, dqh, gq, z["sg"], z["lz"], vq, z["sv"], z["excl"], z["idx"],
                                        O.bf16_round(z["k"]), O.bf16_round(z["v"]), int(z["leaf"]),
                                        1.0 / np.sqrt(z["q"].shape[1]), tail=tail)
    n = z["q"].shape[0]
    assert np.abs(o[:n] - z["out"]).max() < 5e-5
    assert np.abs(l[:n] - z["lse"]).max() < 5e-5


@pytest.mark.parametrize("case", FP8_CASES)
def test_fp8_order_free_oracle_within_tolerance(golden_cases, case):
    """The order-free fp8 oracle (weights rounded against the row's final maximum) stays within the
    fp16-weight rounding of the reference."""
    z = golden_cases[case]
    out, lse, _, _ = _fp8(z)
    assert np.abs(out - z["out"]).max() < 1e-2
    assert np.abs(lse - z["lse"]).max() < 1e-4


BF16_CASES = ["bf16_state", "bf16_sink_tail"]


def _bf16_values(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _bf16(z):
    tail = (z["tail_k"], z["tail_v"]) if "tail_k" in z else None
    out, lse, st = O.flat_attention(z["q"], z["k"], z["v"], leaf=int(z["leaf"]),
                                    exact_leaves=int(z["exact_leaves"]), sink_leaves=int(z["sink_leaves"]),
                                    tail=tail, return_stages=True, store="bf16")
    return out, lse, st, tail


@pytest.mark.parametrize("case", BF16_CASES)
def test_bf16_state_matches_reference(golden_cases, case):
    """store="bf16": g and vbar are the reference's bf16 values (its float32 statistics rounded once: at most
    one bf16 step apart where the float64 restatement lands on the other side of a rounding boundary), the
    selection to float32 rounding, the routing equal."""
    z = golden_cases[case]
    out, lse, st, _ = _bf16(z)
    for mine, ref in ((st["gq"], z["g_bf16"]), (st["vq"], z["vb_bf16"])):
        bits = mine.view(np.uint32) >> 16
        diff = np.abs(bits.astype(np.int64) - ref.astype(np.int64))
        assert diff.max() <= 1 and (diff == 0).mean() >= 0.999, (diff.max(), (diff != 0).sum())
    assert "sg" not in z
    assert np.allclose(st["sel"], z["sel"], rtol=0, atol=1e-3)
    assert np.array_equal(st["excl"], z["excl"])
    assert np.array_equal(np.sort(st["idx"], 1), np.sort(z["idx"], 1))


@pytest.mark.parametrize("case", BF16_CASES)
def test_bf16_ordered_restatement_matches_reference(golden_cases, case):
    """The bf16-state tile attention in the reference kernel's order, fed the reference's own bf16 state,
    reproduces its output to float32 accumulation-order error."""
    z = golden_cases[case]
    out, lse, st, tail = _bf16(z)
    gq, vq = _bf16_values(z["g_bf16"]), _bf16_values(z["vb_bf16"])
    qb, dqb = O.query_codes_bf16(st["qt"], z["mu"])
    one = np.ones(z["lz"].shape, np.float32)
    assert np.allclose(O.rowmax_select_bf16(dqb, gq, z["lz"]), z["sel"], rtol=0, atol=2e-5)
    o, l = O.tile_attention_fp8_ordered(st["qt"], qb, dqb, gq, one, z["lz"], vq, one, z["excl"], z["idx"],
                                        O.bf16_round(z["k"]), O.bf16_round(z["v"]), int(z["leaf"]),
                                        1.0 / np.sqrt(z["q"].shape[1]), tail=tail, far_weight="bf16")
    n = z["q"].shape[0]
    # the float32 exponentials may differ in the last bit, which moves a bf16-rounded weight by one bf16 step
    # (2^-8 relative) where it sits on a rounding boundary: the row of that weight moves, bounded by the step
    err = np.abs(o[:n] - z["out"]).max(1)
    assert (err < 5e-5).mean() >= 0.99 and err.max() < 2e-3, (err.max(), (err >= 5e-5).sum())
    assert np.abs(l[:n] - z["lse"]).max() < 5e-5


@pytest.mark.parametrize("case", BF16_CASES)
def test_bf16_order_free_oracle_within_tolerance(golden_cases, case):
    """The order-free bf16-state oracle stays within the bf16-weight rounding of the reference."""
    z = golden_cases[case]
    out, lse, _, _ = _bf16(z)
    assert np.abs(out - z["out"]).max() < 1e-2
    assert np.abs(lse - z["lse"]).max() < 1e-4


def test_e4m3_codes_round_trip():
    c = np.arange(256, dtype=np.uint8)
    c = c[(c & 0x7F) != 0x7F]                       # 0x7F / 0xFF are NaN in e4m3fn
    assert np.array_equal(O.e4m3_codes(O.e4m3_values(c)), c)


def test_pack_blocks_restates_the_block_rule():
    """qk_scale_block extension: one scale per 64-row block from the block's abs-max, every row coded with
    it; a single-row block equals the per-row pack."""
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((130, 128)) * rng.random((130, 1)) * 3).astype(np.float32)
    x[64:128] = 0.0
    for rounding, per_row in (("even", O.pack_rows_half_even), ("away", O.pack_rows_half_away)):
        x8, s = O.pack_blocks(x, 64, rounding)
        assert x8.dtype == np.int8 and np.abs(x8.astype(int)).max() <= 127
        for b0 in (0, 64, 128):
            blk = slice(b0, min(b0 + 64, 130))
            assert np.all(s[blk] == s[b0])
            assert s[b0] == np.maximum(np.float32(np.abs(x[blk]).max()) * O.INV127, np.float32(1e-20))
        assert np.abs(x8[64:128]).max() == 0
        one8, one_s = O.pack_blocks(x, 1, rounding)
        r8, rs = per_row(x)
        assert np.array_equal(one8, r8) and np.array_equal(one_s, rs)
