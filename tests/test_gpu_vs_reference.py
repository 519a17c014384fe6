"""Parity against the reference's own operator on the same GPU: ``flat_attention(**PROD, leaf=64)`` of the
unmodified reference (h3/htrc_flat.py:391-399, its Triton kernels h3/htrc_flat_triton.py), installed under
baseline/_ref by baseline/install_ref.sh; skipped when that install (or Triton) is absent.

On the same seeded inputs, with PROD's arithmetic as the reference runs it on the GPU (tf32 statistics
operands, ``division="triton"``): the INT8 key codes and scales bit-exact against the reference's formula
(h3/htrc_flat.py:213-219), routing masks (the reference's ``ws["excl"]``) agreeing on >= 99.9% of (tile, leaf)
pairs, outputs of tiles whose routing agrees within 2e-2 max-abs, and log-Z (logsumexp of the reference's split
partials ``ws["pm"]``, ``ws["pl"]``, one chunk) within 1e-3 mean-abs.

The query and offset codes are formed inside the reference's Triton kernels (h3/htrc_flat_triton.py:110-117),
whose float32 ``/`` is PTX div.full.f32 on the GPU; they are checked bit for bit against that formula compiled
by Triton on the same GPU (test-only, given this library's tile centres).
"""
import importlib.util
import os
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
OUT_TOL = 2e-2
LSE_TOL = 1e-3
ROUTE_AGREE = 0.999


@pytest.fixture(scope="module")
def ref():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    cands = [os.environ.get("HTRC_REFERENCE"), str(ROOT / "baseline" / "_ref")]
    root = next((Path(c) for c in cands if c and (Path(c) / "h3" / "htrc_flat.py").exists()), None)
    if root is None:
        pytest.skip("the reference is not installed (baseline/install_ref.sh)")
    try:
        import triton  # noqa: F401
    except ImportError:
        pytest.skip("triton is absent")
    name = "_apl_htrc_flat"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, root / "h3" / "htrc_flat.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


@pytest.mark.parametrize("grid,E,head", [((8, 32, 32), 16, 0), ((8, 48, 84), 256, 3), ((16, 32, 32), 256, 1)])
def test_against_the_reference_operator(ref, grid, E, head):
    import htrc_b200
    from htrc_b200 import flat as F
    from htrc_b200 import synth
    dev = torch.device("cuda:0")
    q, k, v = (t.to(dev) for t in synth.head_inputs(grid, 128, head=head, base_seed=77))
    n, m = q.shape[0], k.shape[0]
    nt, nb = -(-n // 64), m // 64
    cfg = {**ref.PROD, "leaf": 64, "exact_leaves": E}
    ws = {}
    out_r = ref.flat_attention(q, k, v, ws=ws, **{**cfg, "tile_chunk": nt}).float().clone()
    excl_r = ws["excl"][:nt].ne(0)
    pm, pl = ws["pm"][:nt].float(), ws["pl"][:nt].float()
    mm = pm.amax(1, keepdim=True)
    mm = torch.where(torch.isinf(mm), torch.zeros_like(mm), mm)
    lse_r = (mm[:, 0] + torch.log((pl * torch.exp(pm - mm)).sum(1))).reshape(-1)[:n]

    out = torch.empty((n, 128), dtype=torch.float32, device=dev)
    lse = torch.empty((n,), dtype=torch.float32, device=dev)
    mask = torch.zeros((nt, F.leaf_pitch(nb)), dtype=torch.uint8, device=dev)
    w = F.new_workspace(F.workspace_bytes(n, m, E), dev)
    pc = F.precision_code(cfg["precision"], "triton")
    F.forward_into(q, k, v, None, None, exact_leaves=E, out=out, lse=lse, workspace=w, route_mask=mask, precision=pc)
    st = htrc_b200.run_stages(q, k, v, exact_leaves=E, precision=pc)
    torch.cuda.synchronize()
    F.device_status(w)
    assert torch.equal(out, st["out"])
    # the key codes: the reference's formula (h3/htrc_flat.py:215-218), evaluated by torch on the same GPU
    kf = k.float()
    ks_r = (kf.abs().amax(-1) * (1.0 / 127.0)).clamp_min(1e-20)
    k8_r = (kf / ks_r[:, None]).round().clamp(-127, 127).to(torch.int8)
    assert torch.equal(st["k8"], k8_r) and torch.equal(st["ks"], ks_r)
    agree = (mask[:, :nb].ne(0) == excl_r)
    frac = agree.float().mean().item()
    tiles_ok = agree.all(1)
    rows_ok = tiles_ok.repeat_interleave(64)[:n]
    d_out = (out - out_r).abs().amax(1)
    d_lse = (lse - lse_r).abs().mean().item()
    print(f"vs reference {grid} E={E}: routing {frac:.5f}, tiles agreeing {tiles_ok.float().mean().item():.4f}, "
          f"out max-abs (agreeing tiles) {d_out[rows_ok].max().item():.3e}, lse mean-abs {d_lse:.3e}")
    assert frac >= ROUTE_AGREE, frac
    assert rows_ok.float().mean().item() >= 0.5
    assert d_out[rows_ok].max().item() < OUT_TOL
    assert d_lse < LSE_TOL


def _codes_kernel():
    import triton
    import triton.language as tl

    @triton.jit
    def codes(Q, MU, Q8, SQ, DQ8, SDQ, D: tl.constexpr, T: tl.constexpr):
        # the reference's per-row query and offset codes (h3/htrc_flat_triton.py:103-117), as its kernels form them
        t = tl.program_id(0)
        r = tl.arange(0, T)
        d = tl.arange(0, D)
        q = tl.load(Q + (t * T + r)[:, None] * D + d[None, :])
        mu = tl.load(MU + t * D + d)
        dq = q - mu[None, :]
        sdq = tl.maximum(tl.max(tl.abs(dq), axis=1) * (1.0 / 127.0), 1.0e-20)
        x = dq / sdq[:, None]
        dq8 = tl.where(x >= 0, x + 0.5, x - 0.5).to(tl.int8)
        sq = tl.maximum(tl.max(tl.abs(q), axis=1) * (1.0 / 127.0), 1.0e-20)
        x = q / sq[:, None]
        q8 = tl.where(x >= 0, x + 0.5, x - 0.5).to(tl.int8)
        tl.store(Q8 + (t * T + r)[:, None] * D + d[None, :], q8)
        tl.store(DQ8 + (t * T + r)[:, None] * D + d[None, :], dq8)
        tl.store(SQ + t * T + r, sq)
        tl.store(SDQ + t * T + r, sdq)
    return codes


@pytest.mark.parametrize("grid", [(8, 48, 84), (4, 32, 32)])
def test_triton_division_codes_bit_exact(ref, grid):
    """division="triton": this library's query and offset codes and scales equal the reference's formula as
    Triton compiles it on this GPU (div.full.f32), given the same tile centres; division="ieee" keeps the
    IEEE codes, which differ from them only rarely (at rounding boundaries)."""
    import htrc_b200
    from htrc_b200 import flat as F
    from htrc_b200 import synth
    dev = torch.device("cuda:0")
    q, k, v = (t.to(dev) for t in synth.head_inputs(grid, 128, head=2, base_seed=78))
    n = q.shape[0]
    nt = -(-n // 64)
    st = htrc_b200.run_stages(q, k, v, exact_leaves=4, precision=F.precision_code("tf32", "triton"))
    sti = htrc_b200.run_stages(q, k, v, exact_leaves=4, precision=F.precision_code("tf32", "ieee"))
    qt = q.float()
    if nt * 64 > n:
        qt = torch.cat([qt, qt[-1:].expand(nt * 64 - n, -1)], 0)
    q8 = torch.empty((nt * 64, 128), dtype=torch.int8, device=dev)
    dq8 = torch.empty_like(q8)
    sq = torch.empty((nt * 64,), dtype=torch.float32, device=dev)
    sdq = torch.empty_like(sq)
    _codes_kernel()[(nt,)](qt.contiguous(), st["mu"], q8, sq, dq8, sdq, D=128, T=64, num_warps=4)
    torch.cuda.synchronize()
    assert torch.equal(st["sq"], sq) and torch.equal(st["sdq"], sdq)
    assert torch.equal(st["q8"], q8) and torch.equal(st["dq8"], dq8)
    flips = (sti["q8"] != q8).float().mean().item() + (sti["dq8"] != dq8).float().mean().item()
    print(f"{grid}: IEEE vs Triton-division codes differ in {flips:.2e} of the codes")
    assert flips < 1e-3
