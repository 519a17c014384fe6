"""GPU parity of the low-bit simulation (h3/htrc_flat.py:68-97 `fake_quant`, the `quant=` option of
flat_attention, :190-195) and of the fp8 row dequantisation (h3/htrc_flat_triton.py:276-294
`dequant_rows`) against values recorded from the reference."""
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


@pytest.mark.parametrize("fmt", ["int8", "int4", "fp8", "fp4"])
@pytest.mark.parametrize("grp", [0, 16, 32])
def test_fake_quant_bit_exact(dev, golden_cases, fmt, grp):
    import htrc_b200
    z = golden_cases["fake_quant"]
    for xk, yk in (("x", "y"), ("xb", "yb")):
        x = torch.from_numpy(z[xk]).to(dev)
        if xk == "xb":
            x = x.to(torch.bfloat16)
        y = htrc_b200.fake_quant(x, fmt, grp)
        torch.cuda.synchronize()
        want = z[f"{yk}_{fmt}_{grp}"]
        assert y.dtype == torch.float32
        assert np.array_equal(y.cpu().numpy(), want), (fmt, grp, xk)
        yb = htrc_b200.fake_quant(x, fmt, grp, out_dtype=torch.bfloat16)
        assert np.array_equal(yb.float().cpu().numpy(), O.bf16_round(want))


def test_fake_quant_rejects_what_the_reference_rejects(dev):
    import htrc_b200
    x = torch.randn(4, 128, device=dev)
    with pytest.raises(ValueError, match="divide"):
        htrc_b200.fake_quant(x, "int8", 48)
    with pytest.raises(ValueError, match="unknown quant format"):
        htrc_b200.fake_quant(x, "int3")


def test_dequant_rows_strided(dev, golden_cases):
    import htrc_b200
    z = golden_cases["fake_quant"]
    rows = z["codes"].shape[0]
    # the codes and scales as strided head views of a wider per-token cache
    cache = torch.zeros((rows, 3, 128), dtype=torch.uint8, device=dev)
    cache[:, 1] = torch.from_numpy(z["codes"]).to(dev)
    scales = torch.zeros((rows, 3), dtype=torch.float32, device=dev)
    scales[:, 1] = torch.from_numpy(z["dq_scale"]).to(dev)
    out = torch.empty((rows, 128), dtype=torch.bfloat16, device=dev)
    htrc_b200.dequant_rows(cache[:, 1], scales[:, 1], out)
    torch.cuda.synchronize()
    assert np.array_equal(out.float().cpu().numpy(), z["dq_out"])


def test_quant_option_end_to_end(dev, golden_cases):
    """flat_attention(**PROD, quant={"kv": "int4", "q": "int8", "group": 32}) against the reference's
    output.  The reference's leaf statistics read the quantised keys unrounded, this library's read them
    as bf16 (like its near field): the routing is checked for agreement, the rows of agreeing tiles for
    the output tolerance, and, fed the device's own state, the oracle for every row."""
    import htrc_b200
    z = golden_cases["quant_kv_q"]
    quant = {"kv": str(z["quant_kv"]), "q": str(z["quant_q"]), "group": int(z["quant_group"])}
    q = torch.from_numpy(z["q"]).to(torch.bfloat16).to(dev)
    k = torch.from_numpy(z["k"]).to(torch.bfloat16).to(dev)
    v = torch.from_numpy(z["v"]).to(torch.bfloat16).to(dev)
    # the fixture was recorded by Triton's interpreter, which evaluates the tf32 dots in float32
    cfg = {**htrc_b200.PROD, "leaf": 64, "exact_leaves": int(z["exact_leaves"]), "quant": quant, "precision": "fp32"}
    out, lse = htrc_b200.flat_attention(q, k, v, return_lse=True, **cfg)
    torch.cuda.synchronize()
    n = z["q"].shape[0]
    # the key codes the reference packed from its quantised keys
    kq = htrc_b200.fake_quant(k, quant["kv"], quant["group"], out_dtype=torch.bfloat16)
    k8, ks = O.pack_rows_half_even(kq.float().cpu().numpy())
    assert np.array_equal(k8, z["k8"]) and np.array_equal(ks.view(np.uint32), z["ks"].view(np.uint32))
    ro, rl, rst = O.flat_attention(z["q"], z["k"], z["v"], exact_leaves=int(z["exact_leaves"]), quant=quant,
                                   stats_bf16=True, return_stages=True)
    o = out.cpu().numpy()
    assert (rst["excl"] == z["excl"]).mean() >= 0.999
    assert np.abs(o - ro).max() < OUT_TOL                      # the oracle modelling bf16 statistics
    same = np.repeat((rst["excl"] == z["excl"]).all(1), 64)[:n]
    assert np.abs(o[same] - z["out"][same]).max() < 3 * OUT_TOL
    assert np.abs(lse.cpu().numpy() - z["lse"]).mean() < LSE_TOL
    assert np.abs(lse.cpu().numpy() - rl).mean() < LSE_TOL
