"""Flash pn_fir_tau forward+backward parity.

Tolerances (from the north star): fp32 inputs against the reference's golden
vectors at fp32-rounding level; bf16/fp16 outputs and gradients within 1e-2
relative L2 of an fp32 eager run on the same (rounded) inputs; silence-gate
and silent-tile decisions identical except for rows whose peak is within
1e-3 of the threshold.
"""
import math

import pytest
import torch

import paper_01_anti_decoy_pnfirtau_b200 as P
from conftest import rel_l2, rel_max
from oracle import pnfirtau_oracle as O
from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_ops import flash_pn_fir_tau_forward_stats

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2


def run_ours(q, k, v, tau, do, scale=None, gamma=0.5, causal=True):
    q, k, v = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    t = torch.tensor(float(tau), device=q.device, requires_grad=True)
    out = P.flash_pn_fir_tau_attention(q, k, v, t, scale=scale, gamma=gamma, causal_mask=causal)
    out.backward(do)
    P.check_device_status(q.device)
    return out.detach(), q.grad, k.grad, v.grad, t.grad


def run_oracle(q, k, v, tau, do, scale=None, gamma=0.5, causal=True, dtype=torch.float32):
    q, k, v = (t.detach().to(dtype).clone().requires_grad_(True) for t in (q, k, v))
    t = torch.tensor(float(tau), device=q.device, dtype=dtype, requires_grad=True)
    out = O.pn_fir_tau_attention(q, k, v, t, scale, gamma, causal)
    out.backward(do.to(dtype))
    return out.detach(), q.grad, k.grad, v.grad, t.grad


def assert_close_lowp(ours, ref, tol=BF16_TOL, names=("out", "dq", "dk", "dv"), dtau_tol=None):
    """Relative L2 of out/dq/dk/dv and relative error of the scalar dtau, which
    is a heavily cancelling sum (fp32 runs give it ~1e-5..1e-4 relative)."""
    for name, a, b in zip(names, ours[:4], ref[:4]):
        err = rel_l2(a, b)
        assert err < tol, f"{name}: rel L2 {err:.3e} >= {tol}"
    dtau_tol = tol if dtau_tol is None else dtau_tol
    da, db = float(ours[4]), float(ref[4])
    assert abs(da - db) <= dtau_tol * abs(db) + 1e-6, f"dtau {da} vs {db}"


@pytest.mark.parametrize(
    "case", ["b1h2n80d16_tau0", "b1h2n80d16_taup5", "b2h1n130d32_taum5", "b1h1n70d64_nc", "b1h2n96d16_quiet"]
)
def test_flash_fp32_golden(cuda, golden, case):
    c = golden("attention")[case]
    q, k, v, do = (c[n].to(cuda) for n in ("q", "k", "v", "do"))
    out, dq, dk, dv, dtau = run_ours(q, k, v, c["tau"], do, c["scale"], 0.5, c["causal"])
    assert rel_max(out, c["out"]) < 1e-5
    assert rel_max(dq, c["dq"]) < 5e-5
    assert rel_max(dk, c["dk"]) < 5e-5
    assert rel_max(dv, c["dv"]) < 5e-5
    assert abs(float(dtau) - float(c["dtau"])) <= 5e-5 * max(1.0, abs(float(c["dtau"])))


def _qkv(B, H, N, D, seed, dtype, device, quiet_frac=0.0, quiet_scale=0.05):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=g)
    if quiet_frac > 0:
        nb = (N + 63) // 64
        quiet = torch.rand(B, H, nb, generator=g) < quiet_frac
        fac = torch.where(quiet, quiet_scale, 1.0).repeat_interleave(64, dim=-1)[..., :N]
        q = q * fac[..., None]
    k = torch.randn(B, H, N, D, generator=g)
    v = torch.randn(B, H, N, D, generator=g)
    do = torch.randn(B, H, N, D, generator=g)
    return tuple(t.to(device=device, dtype=dtype) for t in (q, k, v, do))


def test_flash_config2_bf16(cuda):
    """B16 H4 N512 d64 bf16 vs fp32 eager."""
    q, k, v, do = _qkv(16, 4, 512, 64, 1234, torch.bfloat16, cuda)
    ours = run_ours(q, k, v, 0.0, do)
    ref = run_oracle(q, k, v, 0.0, do)
    assert ours[0].dtype == torch.bfloat16 and ours[1].dtype == torch.bfloat16
    assert_close_lowp(ours, ref)


@pytest.mark.parametrize("tau", [-0.5, 0.0, 0.5])
def test_flash_silent_regime_gate_and_tiles(cuda, tau):
    """Config-3 regime at reduced size: gate masks and 64x64 silent-tile flags
    match the exp4b oracle, and results stay within tolerance."""
    q, k, v, do = _qkv(2, 2, 1024, 64, 99, torch.bfloat16, cuda, quiet_frac=0.5)
    t = torch.tensor(tau, device=cuda)
    out, M, Z, Nmax, tiles = flash_pn_fir_tau_forward_stats(q, k, v, t)
    ref_tiles, ref_silent, ref_peak = O.tile_silence(q.float(), k.float(), tau)
    ref_peak_o, ref_z, ref_n = O.row_stats(q.float(), k.float(), torch.tensor(tau, device=cuda))
    near = ref_peak_o.abs() < 1e-3  # rows within 1e-3 of the threshold may flip
    gate_ours = M > 0
    gate_ref = ref_peak_o > 0
    assert torch.equal(gate_ours[~near], gate_ref[~near])
    # a tile is live iff some entry is positive; flags may differ only where a near-threshold row lives
    near_rows_tiles = torch.zeros_like(ref_tiles)
    nT = ref_tiles.shape[-1]
    near_rows_tiles |= near.reshape(2, 2, nT, 64).any(-1)[..., None]
    diff = tiles != ref_tiles
    assert not torch.any(diff & ~near_rows_tiles)
    assert rel_max(M, ref_peak_o) < 1e-2
    assert torch.equal(Nmax[~near], ref_n[~near])
    ours = run_ours(q, k, v, tau, do)
    ref = run_oracle(q, k, v, tau, do)
    assert_close_lowp(ours, ref)


@pytest.mark.parametrize("D", [16, 32, 64, 128])
@pytest.mark.parametrize("N", [1, 7, 63, 65, 129])
def test_flash_shapes_bf16(cuda, D, N):
    q, k, v, do = _qkv(1, 2, N, D, N * 1000 + D, torch.bfloat16, cuda)
    ours = run_ours(q, k, v, -0.2, do)
    ref = run_oracle(q, k, v, -0.2, do)
    assert_close_lowp(ours, ref)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_flash_dtypes(cuda, dtype):
    q, k, v, do = _qkv(2, 2, 200, 64, 5, dtype, cuda)
    ours = run_ours(q, k, v, 0.1, do)
    ref = run_oracle(q, k, v, 0.1, do, dtype=torch.float64)
    assert ours[0].dtype == dtype
    tol = 2e-5 if dtype == torch.float32 else BF16_TOL
    assert_close_lowp(ours, ref, tol=tol, dtau_tol=5e-4 if dtype == torch.float32 else BF16_TOL)


def test_flash_non_causal_and_no_gamma(cuda):
    q, k, v, do = _qkv(1, 3, 150, 64, 6, torch.bfloat16, cuda)
    assert_close_lowp(run_ours(q, k, v, 0.3, do, causal=False), run_oracle(q, k, v, 0.3, do, causal=False))
    assert_close_lowp(run_ours(q, k, v, 0.3, do, gamma=None), run_oracle(q, k, v, 0.3, do, gamma=None))
    assert_close_lowp(run_ours(q, k, v, 0.3, do, gamma=0.0), run_oracle(q, k, v, 0.3, do, gamma=0.0))


def test_flash_strided_qkv_views(cuda):
    """q/k/v as views of one [B,N,3,H,D] buffer (the module's layout): no copies needed."""
    B, N, H, D = 2, 192, 4, 64
    g = torch.Generator().manual_seed(8)
    buf = torch.randn(B, N, 3, H, D, generator=g).to(cuda, torch.bfloat16)
    do = torch.randn(B, H, N, D, generator=g).to(cuda, torch.bfloat16)
    q, k, v = (buf[:, :, i].transpose(1, 2) for i in range(3))
    assert not q.is_contiguous()
    ours = run_ours(q, k, v, 0.0, do)
    ref = run_oracle(q, k, v, 0.0, do)
    assert_close_lowp(ours, ref)


def test_flash_all_silent(cuda):
    q, k, v, do = _qkv(1, 1, 128, 64, 3, torch.bfloat16, cuda)
    out, dq, dk, dv, dtau = run_ours(q * 0.0, k, v, 0.5, do)
    assert torch.all(out == 0) and torch.all(dq == 0) and torch.all(dk == 0) and torch.all(dv == 0)
    assert float(dtau) == 0.0


def test_flash_exact_ties(cuda):
    """Duplicate keys give exact ties at the row peak: the gate gradient splits
    evenly over them (amax backward), fp32 inputs."""
    q, k, v, do = _qkv(1, 1, 64, 16, 4, torch.float32, cuda)
    k[:, :, 3] *= 3.0  # |k3|^2 dominates every other k3.kj, so the duplicates hold the peak
    k[:, :, 10] = k[:, :, 3]
    k[:, :, 20] = k[:, :, 3]
    q[:, :, 30:] = k[:, :, 3:4] * 2.0
    ours = run_ours(q, k, v, 0.0, do)
    ref = run_oracle(q, k, v, 0.0, do, dtype=torch.float64)
    _, _, _, Nmax, _ = flash_pn_fir_tau_forward_stats(q, k, v, torch.tensor(0.0, device=cuda))
    assert int(Nmax[0, 0, 40]) == 3
    assert_close_lowp(ours, ref, tol=2e-5, dtau_tol=2e-4)
