"""Causal FIR on the keys in the tcgen05 kernels' K-tile load
(flash_pn_fir_tau_attention_fir: pnft_flash_bwd_fir always, pnft_flash_fwd_fir
with fused_forward) against the unfused composition flash(q, triton_causal_fir(k),
v) and the fp32 oracle. The tile filter is bit-exact, so the forward and every
gradient but dQ (whose cross-CTA accumulation order varies) agree bitwise."""
import pytest
import torch

import paper_01_anti_decoy_pnfirtau_b200 as P
from conftest import rel_l2
from oracle import pnfirtau_oracle as O
from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_ops import check_device_status

pytestmark = pytest.mark.gpu


def _module_layout(B, H, N, D, seed, device):
    """q, k, v as [B,H,N,D] views of one [B,N,3*H*D] projection output (the
    module's layout: head dims adjacent, rows 3*H*D apart)."""
    g = torch.Generator().manual_seed(seed)
    buf = torch.randn(B, N, 3 * H * D, generator=g).to(device, torch.bfloat16)
    q, k, v = buf.chunk(3, dim=-1)
    return tuple(t.view(B, N, H, D).transpose(1, 2) for t in (q, k, v))


def _taps(device):
    return O.gaussian_taps(7).to(device)


def _run(q, k, v, do, tau, taps, fused, fused_forward=False):
    qq, kk, vv = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    tt = torch.tensor(tau, device=q.device, requires_grad=True)
    hh = taps.detach().clone().requires_grad_(True)
    if fused:
        out = P.flash_pn_fir_tau_attention_fir(qq, kk, vv, tt, hh, fused_forward=fused_forward)
    else:
        B, H, N, D = kk.shape
        kt = P.triton_causal_fir(kk.transpose(1, 2).reshape(B, N, H * D), hh).view(B, N, H, D).transpose(1, 2)
        out = P.flash_pn_fir_tau_attention(qq, kt, vv, tt)
    out.backward(do)
    check_device_status(q.device)
    return out.detach(), qq.grad, kk.grad, vv.grad, tt.grad, hh.grad


@pytest.mark.parametrize("fused_forward", [False, True])
@pytest.mark.parametrize("D", [16, 32, 64, 128])
@pytest.mark.parametrize("N,tau", [(128, 0.0), (300, -0.2), (520, 0.3), (70, 0.1)])
def test_fused_fir_matches_unfused(cuda, D, N, tau, fused_forward):
    q, k, v = _module_layout(2, 2, N, D, 11 + N + D, cuda)
    do = torch.randn(q.shape, generator=torch.Generator().manual_seed(N)).to(cuda, torch.bfloat16)
    taps = _taps(cuda)
    assert P.flash_kernel_path(q, k, v) == "sm100"
    fu = _run(q, k, v, do, tau, taps, fused=True, fused_forward=fused_forward)
    un = _run(q, k, v, do, tau, taps, fused=False)
    assert torch.equal(fu[0], un[0]), "forward output"
    assert rel_l2(fu[1], un[1]) < 1e-3, ("dq", rel_l2(fu[1], un[1]))
    assert torch.equal(fu[2], un[2]), "dk"
    assert torch.equal(fu[3], un[3]), "dv"
    assert torch.equal(fu[4], un[4]), "dtau"
    assert rel_l2(fu[5], un[5]) < 1e-5, ("dtaps", rel_l2(fu[5], un[5]))


@pytest.mark.parametrize("D", [16, 64, 128])
def test_fused_fir_vs_oracle(cuda, D):
    B, H, N = 2, 2, 256
    q, k, v = _module_layout(B, H, N, D, 5 + D, cuda)
    do = torch.randn(q.shape, generator=torch.Generator().manual_seed(9)).to(cuda, torch.bfloat16)
    taps = _taps(cuda)
    ours = _run(q, k, v, do, 0.0, taps, fused=True)
    qr, kr, vr = (t.float().detach().requires_grad_(True) for t in (q, k, v))
    tr = torch.tensor(0.0, device=cuda, requires_grad=True)
    hr = taps.detach().clone().requires_grad_(True)
    kt = O.causal_fir(kr.transpose(1, 2).reshape(B, N, H * D), hr).view(B, N, H, D).transpose(1, 2)
    # the filtered keys rounded to bf16 as the kernels (and the reference's
    # triton_causal_fir, output in the input dtype) hold them; the cast passes
    # gradients through unchanged
    kt = kt.to(torch.bfloat16).float()
    outr = O.pn_fir_tau_attention(qr, kt, vr, tr)
    outr.backward(do.float())
    for name, a, r in zip(("out", "dq", "dk", "dv", "dtaps"), (ours[0], ours[1], ours[2], ours[3], ours[5]),
                          (outr, qr.grad, kr.grad, vr.grad, hr.grad)):
        assert rel_l2(a, r) < 1e-2, (name, rel_l2(a, r))
    assert abs(float(ours[4]) - float(tr.grad)) <= 1e-2 * abs(float(tr.grad)) + 1e-6


@pytest.mark.parametrize("fused_forward", [False, True])
def test_fused_fir_contiguous_keys(cuda, fused_forward):
    """k as a contiguous [B,H,N,D] tensor (b and h adjacent) also serves."""
    B, H, N, D = 2, 3, 200, 64
    g = torch.Generator().manual_seed(3)
    q, k, v, do = (torch.randn(B, H, N, D, generator=g).to(cuda, torch.bfloat16) for _ in range(4))
    taps = _taps(cuda)
    fu = _run(q, k, v, do, 0.1, taps, fused=True, fused_forward=fused_forward)
    un = _run(q, k, v, do, 0.1, taps, fused=False)
    assert torch.equal(fu[0], un[0])
    assert torch.equal(fu[2], un[2]) and torch.equal(fu[3], un[3])


def test_module_fuse_fir_is_identical(cuda):
    cfg = P.PnFirConfig(d_model=256, n_heads=4)
    torch.manual_seed(0)
    m0 = P.PnFirTauFlashMHA(cfg, fuse_fir=False).to(cuda)
    m1 = P.PnFirTauFlashMHA(cfg).to(cuda)
    m1.load_state_dict(m0.state_dict())
    x = torch.randn(2, 384, 256, device=cuda)
    outs, grads = [], []
    for m in (m0, m1):
        xx = x.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = m(xx)
        y.float().square().mean().backward()
        outs.append(y.detach())
        grads.append((xx.grad, m.qkv.weight.grad, m.score_tau.grad))
        m.zero_grad()
    assert torch.equal(outs[0], outs[1])
    for a, b in zip(grads[0], grads[1]):
        assert rel_l2(a, b) < 1e-3
