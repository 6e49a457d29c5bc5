"""Deterministic backward (PNFT_FLASH_DETERMINISTIC, ``deterministic=True`` or
``torch.use_deterministic_algorithms(True)``): the key tiles add their dQ
contributions to each query tile in key order, so two runs give bitwise-equal
gradients. The output equals the default path's bit for bit; the gradients equal
the default (atomic-order) backward's within fp32 rounding of the accumulation
orders (the deterministic walk visits the query tiles top down); everything
stays within the north-star tolerance of the fp32 oracle. The reference's backward accumulates dQ with atomics
(src/triton_pnfirtau.py:596-602) although its docstring promises a deterministic
backward (:15-17)."""
import pytest
import torch

import paper_01_anti_decoy_pnfirtau_b200 as P
from conftest import rel_l2
from oracle import pnfirtau_oracle as O
from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_ops import check_device_status

pytestmark = pytest.mark.gpu


def _inputs(B, H, N, D, seed, device, dtype, quiet_frac=0.0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=g)
    if quiet_frac:
        nb = (N + 63) // 64
        quiet = torch.rand(B, H, nb, generator=g) < quiet_frac
        q = q * torch.where(quiet, 0.05, 1.0).repeat_interleave(64, dim=-1)[..., :N, None]
    k, v, do = (torch.randn(B, H, N, D, generator=g) for _ in range(3))
    return tuple(t.to(device, dtype) for t in (q, k, v, do))


def _run(q, k, v, do, tau, deterministic, fir=False, causal=True):
    qq, kk, vv = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    tt = torch.tensor(tau, device=q.device, requires_grad=True)
    if fir:
        hh = O.gaussian_taps(7).to(q.device).requires_grad_(True)
        out = P.flash_pn_fir_tau_attention_fir(qq, kk, vv, tt, hh, deterministic=deterministic)
    else:
        hh = None
        out = P.flash_pn_fir_tau_attention(qq, kk, vv, tt, causal_mask=causal, deterministic=deterministic)
    out.backward(do)
    check_device_status(q.device)
    return [out.detach(), qq.grad, kk.grad, vv.grad, tt.grad] + ([hh.grad] if fir else [])


def _oracle(q, k, v, do, tau, fir=False, causal=True):
    qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
    tr = torch.tensor(tau, device=q.device, requires_grad=True)
    kt = kr
    if fir:
        B, H, N, D = kr.shape
        kt = O.causal_fir(kr.reshape(B * H, N, D), O.gaussian_taps(7).to(q.device)).reshape(kr.shape)
        kt = kt + (kt.to(torch.bfloat16).float() - kt).detach()  # the bf16 rounding of the fused path
    out = O.pn_fir_tau_attention(qr, kt, vr, tr, causal=causal)
    out.backward(do.float())
    return out.detach(), qr.grad, kr.grad, vr.grad, tr.grad


CASES = {
    # name: (B, H, N, D, dtype, tau, quiet, fir, causal, kernel family)
    "sm100_d64_silent": (2, 2, 1024, 64, torch.bfloat16, 0.5, 0.5, False, True, "sm100"),
    "sm100_d64_dense": (2, 3, 700, 64, torch.bfloat16, -0.2, 0.0, False, True, "sm100"),
    "sm100_d128": (1, 2, 640, 128, torch.bfloat16, 0.1, 0.0, False, True, "sm100"),
    "sm100_noncausal": (1, 2, 384, 64, torch.bfloat16, 0.3, 0.0, False, False, "sm100"),
    "sm100_fused_fir": (2, 2, 520, 64, torch.bfloat16, 0.0, 0.0, True, True, "sm100"),
    "generic_fp32": (1, 2, 300, 64, torch.float32, 0.1, 0.0, False, True, "generic"),
    "generic_bf16_d24": (2, 1, 257, 24, torch.bfloat16, 0.0, 0.0, False, True, "generic"),
    "sm100_d32_padded": (2, 2, 384, 32, torch.bfloat16, 0.2, 0.3, False, True, "sm100"),
    "sm100_d16_fused_fir": (1, 2, 300, 16, torch.bfloat16, 0.0, 0.0, True, True, "sm100"),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_deterministic_backward(cuda, case):
    B, H, N, D, dtype, tau, quiet, fir, causal, family = CASES[case]
    q, k, v, do = _inputs(B, H, N, D, 600 + N + D, cuda, dtype, quiet)
    assert P.flash_kernel_path(q, k, v) == family
    a = _run(q, k, v, do, tau, True, fir, causal)
    b = _run(q, k, v, do, tau, True, fir, causal)
    names = ["out", "dq", "dk", "dv", "dtau", "dtaps"]
    for n, x, y in zip(names, a, b):
        assert torch.equal(x, y), f"{n} differs between two deterministic runs"
    c = _run(q, k, v, do, tau, False, fir, causal)
    assert torch.equal(a[0], c[0]), "the forward does not depend on the backward's mode"
    for n, x, y in zip(names[1:], a[1:], c[1:]):
        # the deterministic walk visits query tiles in the opposite order, so the
        # fp32 accumulations of dQ (and of dK, dV, dtau) round differently
        assert rel_l2(x, y) < 2e-3, (n, rel_l2(x, y))
    ref = _oracle(q, k, v, do, tau, fir, causal)
    tol = 2e-5 if dtype == torch.float32 else 1e-2
    for n, x, r in zip(names[:4], a[:4], ref[:4]):
        assert rel_l2(x, r) < tol, (n, rel_l2(x, r))
    assert abs(float(a[4]) - float(ref[4])) <= max(tol, 5e-4) * abs(float(ref[4])) + 1e-6


def test_torch_deterministic_flag_selects_ordered_dq(cuda):
    """With torch.use_deterministic_algorithms(True) the default call is deterministic."""
    q, k, v, do = _inputs(2, 2, 768, 64, 91, cuda, torch.bfloat16)
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True)
    try:
        runs = [_run(q, k, v, do, 0.0, None) for _ in range(3)]
    finally:
        torch.use_deterministic_algorithms(prev)
    for r in runs[1:]:
        for x, y in zip(runs[0], r):
            assert torch.equal(x, y)
