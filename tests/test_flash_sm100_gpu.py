"""tcgen05/TMA kernels (bf16, head dim 64/128) against the fp32 oracle and the
generic kernels: output, per-row statistics, gate masks and 64x64 silent-tile
flags."""
import math

import pytest
import torch

from conftest import rel_l2, rel_max
from oracle import pnfirtau_oracle as O
from paper_01_anti_decoy_pnfirtau_b200 import _lib
from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_ops import check_device_status, flash_pn_fir_tau_forward_stats

pytestmark = pytest.mark.gpu

SM100 = _lib.FLASH_PREFER_SM100
GENERIC = _lib.FLASH_FORCE_GENERIC


def _inputs(B, H, N, D, seed, device, quiet_frac=0.0, layout="bhnd"):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=g)
    if quiet_frac:
        nb = (N + 63) // 64
        quiet = torch.rand(B, H, nb, generator=g) < quiet_frac
        q = q * torch.where(quiet, 0.05, 1.0).repeat_interleave(64, dim=-1)[..., :N, None]
    k = torch.randn(B, H, N, D, generator=g)
    v = torch.randn(B, H, N, D, generator=g)
    q, k, v = (t.to(device, torch.bfloat16) for t in (q, k, v))
    if layout == "bnhd":  # the module's views of one [B,N,3,H,D] buffer
        buf = torch.stack([t.transpose(1, 2) for t in (q, k, v)], dim=2).contiguous()
        q, k, v = (buf[:, :, i].transpose(1, 2) for i in range(3))
    return q, k, v


def _check_fwd(q, k, v, tau, causal=True, gamma=0.5):
    dev = q.device
    t = torch.tensor(tau, device=dev)
    out, M, Z, Nmax, tiles = flash_pn_fir_tau_forward_stats(q, k, v, t, gamma=gamma, causal_mask=causal,
                                                            extra_flags=SM100)
    check_device_status(dev)
    ref = O.pn_fir_tau_attention(q.float(), k.float(), v.float(), t, gamma=gamma, causal=causal)
    assert rel_l2(out, ref) < 1e-2
    peak, z, nmax = O.row_stats(q.float(), k.float(), t, causal=causal)
    near = peak.abs() < 1e-3
    assert torch.equal((M > 0)[~near], (peak > 0)[~near])
    assert rel_max(M, peak) < 1e-3
    live = peak > 1e-3
    assert torch.allclose(Z[live], z[live], rtol=2e-4, atol=0)
    # rows whose two largest u are equal or a few ulps apart in the oracle's fp32
    # order may count a tie in one accumulation order and not in the other (genuine
    # ties from duplicated keys are checked in test_sm100_duplicate_key_ties)
    sc = O.thresholded_scores(q.float() @ k.float().transpose(-2, -1), t, 1.0 / math.sqrt(q.shape[-1]), causal)
    if sc.shape[-1] >= 2:
        top2 = torch.relu(sc).topk(2, dim=-1).values
        gap = top2[..., 0] - top2[..., 1]
        fuzzy = gap <= 1e-5 * top2[..., 0]
    else:
        fuzzy = torch.zeros_like(near)
    keep = ~near & ~fuzzy
    bad = keep & (Nmax != nmax)
    if bad.any():
        idx = bad.nonzero()[:4].tolist()
        info = [(i, int(Nmax[tuple(i)]), int(nmax[tuple(i)]), float(peak[tuple(i)]),
                 [float(v) for v in torch.relu(sc[tuple(i)]).topk(min(3, sc.shape[-1])).values]) for i in idx]
        raise AssertionError(f"Nmax differs on {int(bad.sum())} rows (row, ours, ref, peak, top3 u): {info}")
    if causal:
        ref_tiles, _, _ = O.tile_silence(q.float(), k.float(), tau)
        nT = ref_tiles.shape[-1]
        Np = nT * 64
        nr = torch.nn.functional.pad(near, (0, Np - near.shape[-1]))
        near_t = nr.reshape(*near.shape[:2], nT, 64).any(-1)[..., None].expand_as(ref_tiles)
        assert not torch.any((tiles != ref_tiles) & ~near_t)
    # same decisions and nearly the same numbers as the generic kernels
    out_g, M_g, _, N_g, tiles_g = flash_pn_fir_tau_forward_stats(q, k, v, t, gamma=gamma, causal_mask=causal,
                                                                 extra_flags=GENERIC)
    assert rel_l2(out, out_g) < 1e-2
    assert rel_max(M, M_g) < 1e-5
    return out


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("N", [128, 256, 200, 64, 1])
def test_sm100_fwd_shapes(cuda, D, N):
    q, k, v = _inputs(2, 2, N, D, 100 + N + D, cuda)
    _check_fwd(q, k, v, 0.0)


@pytest.mark.parametrize("tau", [-0.5, 0.0, 0.5])
def test_sm100_fwd_silent_regime(cuda, tau):
    q, k, v = _inputs(2, 2, 1024, 64, 7, cuda, quiet_frac=0.5)
    _check_fwd(q, k, v, tau)


def test_sm100_fwd_module_layout(cuda):
    q, k, v = _inputs(2, 4, 384, 64, 11, cuda, layout="bnhd")
    assert not q.is_contiguous()
    _check_fwd(q, k, v, 0.1)


def test_sm100_fwd_non_causal_and_no_gamma(cuda):
    q, k, v = _inputs(1, 2, 320, 64, 12, cuda)
    _check_fwd(q, k, v, 0.2, causal=False)
    _check_fwd(q, k, v, 0.2, gamma=None)


def test_sm100_fwd_all_silent(cuda):
    q, k, v = _inputs(1, 1, 256, 64, 13, cuda)
    t = torch.tensor(0.5, device=cuda)
    out, M, Z, Nmax, tiles = flash_pn_fir_tau_forward_stats(q * 0, k, v, t, extra_flags=SM100)
    check_device_status(cuda)
    assert torch.all(out == 0) and torch.all(M == 0) and torch.all(Nmax == 0) and not tiles.any()
    assert torch.all(Z == 1e-12)


def test_sm100_fwd_config3_slices(cuda):
    """Full config-3 size through the tcgen05 forward; per-head parity on a sample of heads."""
    B, H, N, D = 8, 8, 4096, 64
    q, k, v = _inputs(B, H, N, D, 2024, cuda, quiet_frac=0.5)
    for tau in (0.0, 0.5):
        t = torch.tensor(tau, device=cuda)
        out, M, Z, Nmax, tiles = flash_pn_fir_tau_forward_stats(q, k, v, t, extra_flags=SM100)
        check_device_status(cuda)
        assert torch.isfinite(out.float()).all()
        for bh in (0, 27, 63):
            b, h = divmod(bh, H)
            sl = (slice(b, b + 1), slice(h, h + 1))
            ref = O.pn_fir_tau_attention(q[sl].float(), k[sl].float(), v[sl].float(), t)
            assert rel_l2(out[sl], ref) < 1e-2
            peak, _, _ = O.row_stats(q[sl].float(), k[sl].float(), t)
            near = peak.abs() < 1e-3
            assert torch.equal((M[sl] > 0)[~near], (peak > 0)[~near])


def _fwd_bwd(q, k, v, do, tau, generic):
    from paper_01_anti_decoy_pnfirtau_b200 import pnfirtau_ops

    import paper_01_anti_decoy_pnfirtau_b200 as P

    old = pnfirtau_ops._FORCE_GENERIC
    pnfirtau_ops._FORCE_GENERIC = generic
    try:
        qq, kk, vv = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
        assert P.flash_kernel_path(qq, kk, vv) == ("generic" if generic else "sm100")
        tt = torch.tensor(tau, device=q.device, requires_grad=True)
        out = P.flash_pn_fir_tau_attention(qq, kk, vv, tt)
        out.backward(do)
        check_device_status(q.device)
        return out.detach(), qq.grad, kk.grad, vv.grad, tt.grad
    finally:
        pnfirtau_ops._FORCE_GENERIC = old


# head dims below 64 (or between 64 and 128) run zero-padded to 64 (128) through the TMA loads
@pytest.mark.parametrize("D", [16, 32, 48, 64, 96, 128])
@pytest.mark.parametrize("N,tau", [(128, 0.0), (192, -0.3), (320, 0.4), (70, 0.1)])
def test_sm100_fwd_bwd_vs_oracle_and_generic(cuda, D, N, tau):
    q, k, v = _inputs(2, 2, N, D, 300 + N + D, cuda)
    do = torch.randn(q.shape, generator=torch.Generator().manual_seed(N)).to(cuda, torch.bfloat16)
    ours = _fwd_bwd(q, k, v, do, tau, generic=False)
    gen = _fwd_bwd(q, k, v, do, tau, generic=True)
    qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
    tr = torch.tensor(tau, device=cuda, requires_grad=True)
    outr = O.pn_fir_tau_attention(qr, kr, vr, tr)
    outr.backward(do.float())
    ref = (outr.detach(), qr.grad, kr.grad, vr.grad, tr.grad)
    for name, a, g, r in zip(("out", "dq", "dk", "dv"), ours[:4], gen[:4], ref[:4]):
        assert rel_l2(a, r) < 1e-2, (name, rel_l2(a, r))
        assert rel_l2(g, r) < 1e-2, (name, rel_l2(g, r))
    assert abs(float(ours[4]) - float(ref[4])) <= 1e-2 * abs(float(ref[4])) + 1e-6


def test_sm100_bwd_silent_regime(cuda):
    q, k, v = _inputs(2, 2, 1024, 64, 77, cuda, quiet_frac=0.5)
    do = torch.randn(q.shape, generator=torch.Generator().manual_seed(5)).to(cuda, torch.bfloat16)
    for tau in (-0.5, 0.0, 0.5):
        ours = _fwd_bwd(q, k, v, do, tau, generic=False)
        qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
        tr = torch.tensor(tau, device=cuda, requires_grad=True)
        outr = O.pn_fir_tau_attention(qr, kr, vr, tr)
        outr.backward(do.float())
        for name, a, r in zip(("out", "dq", "dk", "dv"), ours[:4], (outr, qr.grad, kr.grad, vr.grad)):
            assert rel_l2(a, r) < 1e-2, (tau, name, rel_l2(a, r))
        assert abs(float(ours[4]) - float(tr.grad)) <= 1e-2 * abs(float(tr.grad)) + 1e-6, tau


def test_sm100_duplicate_key_ties(cuda):
    """Duplicated keys tie exactly in any arithmetic: the tcgen05 forward counts
    them and the backward splits the gate gradient over them (eager amax rule)."""
    g = torch.Generator().manual_seed(21)
    B, H, N, D = 1, 1, 192, 64
    q = torch.randn(B, H, N, D, generator=g)
    k = torch.randn(B, H, N, D, generator=g)
    v = torch.randn(B, H, N, D, generator=g)
    k[:, :, 3] *= 5.0  # |k3|^2 ~ 1600 dominates every other k3.kj (std ~ 320)
    for j in (40, 130):
        k[:, :, j] = k[:, :, 3]
    q[:, :, 60:] = k[:, :, 3:4] * 0.3  # rows 60..129 see two copies, rows >= 130 three
    q, k, v = (t.to(cuda, torch.bfloat16) for t in (q, k, v))
    do = torch.randn(q.shape, generator=g).to(cuda, torch.bfloat16)
    t = torch.tensor(0.0, device=cuda)
    _, M, _, Nmax, _ = flash_pn_fir_tau_forward_stats(q, k, v, t, extra_flags=SM100)
    check_device_status(cuda)
    assert int(Nmax[0, 0, 150]) == 3 and int(Nmax[0, 0, 100]) == 2
    ours = _fwd_bwd(q, k, v, do, 0.0, generic=False)
    qr, kr, vr = (x.double().requires_grad_(True) for x in (q, k, v))
    tr = torch.tensor(0.0, dtype=torch.float64, device=cuda, requires_grad=True)
    outr = O.pn_fir_tau_attention(qr, kr, vr, tr)
    outr.backward(do.double())
    for name, a, r in zip(("out", "dq", "dk", "dv"), ours[:4], (outr, qr.grad, kr.grad, vr.grad)):
        assert rel_l2(a, r) < 1e-2, (name, rel_l2(a, r))
    assert abs(float(ours[4]) - float(tr.grad)) <= 1e-2 * abs(float(tr.grad)) + 1e-6


def test_sm100_ties_within_one_key_quarter(cuda):
    """Duplicates inside one 32-key quarter of one tile (keys 5 and 12) and two more
    in a later tile's same quarter (140, 150): the per-row tie counts 1/2/3/4 and
    the gradients that follow the first maximal key."""
    g = torch.Generator().manual_seed(22)
    B, H, N, D = 1, 1, 192, 64
    q = torch.randn(B, H, N, D, generator=g)
    k = torch.randn(B, H, N, D, generator=g)
    v = torch.randn(B, H, N, D, generator=g)
    k[:, :, 5] *= 5.0
    for j in (12, 140, 150):
        k[:, :, j] = k[:, :, 5]
    q[:, :, 5:] = k[:, :, 5:6] * 0.3
    q, k, v = (t.to(cuda, torch.bfloat16) for t in (q, k, v))
    do = torch.randn(q.shape, generator=g).to(cuda, torch.bfloat16)
    t = torch.tensor(0.0, device=cuda)
    _, M, _, Nmax, _ = flash_pn_fir_tau_forward_stats(q, k, v, t, extra_flags=SM100)
    check_device_status(cuda)
    want = torch.tensor([1] * 7 + [2] * 128 + [3] * 10 + [4] * 42, dtype=torch.int32)
    assert torch.equal(Nmax[0, 0, 5:].cpu(), want)
    ours = _fwd_bwd(q, k, v, do, 0.0, generic=False)
    qr, kr, vr = (x.double().requires_grad_(True) for x in (q, k, v))
    tr = torch.tensor(0.0, dtype=torch.float64, device=cuda, requires_grad=True)
    outr = O.pn_fir_tau_attention(qr, kr, vr, tr)
    outr.backward(do.double())
    for name, a, r in zip(("out", "dq", "dk", "dv"), ours[:4], (outr, qr.grad, kr.grad, vr.grad)):
        assert rel_l2(a, r) < 1e-2, (name, rel_l2(a, r))
    assert abs(float(ours[4]) - float(tr.grad)) <= 1e-2 * abs(float(tr.grad)) + 1e-6
