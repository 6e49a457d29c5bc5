"""Row-fused score->weight kernels: every silence mode and p of the eager
power_norm_peak_gate, the reference's triton_pn_fir_tau_scores contract, and
rows longer than the reference's 4096 limit."""
import pytest
import torch

import paper_01_anti_decoy_pnfirtau_b200 as P
from conftest import rel_l2, rel_max
from oracle import pnfirtau_oracle as O

pytestmark = pytest.mark.gpu


def test_pngate_golden_all_modes(cuda, golden):
    for name, c in golden("pngate").items():
        s = c["scores"].to(cuda).requires_grad_(True)
        w = P.power_norm_peak_gate(s, c["p"], c["gamma"], c["mode"])
        w.backward(c["dy"].to(cuda))
        assert rel_max(w, c["w"]) < 2e-6, name
        assert rel_max(s.grad, c["dscores"]) < 2e-5, name


@pytest.mark.parametrize("N,causal,tau", [(300, True, 0.3), (64, True, -0.5), (129, False, 0.8), (1, True, 0.0)])
def test_scores_op_vs_oracle(cuda, N, causal, tau):
    g = torch.Generator().manual_seed(N)
    raw = (torch.randn(2, 4, N, N, generator=g) * 8).to(cuda).requires_grad_(True)
    t = torch.tensor(tau, device=cuda, requires_grad=True)
    w = P.triton_pn_fir_tau_scores(raw, t, scale=0.125, p=10.0, gamma=0.5, causal_mask=causal)
    dy = torch.randn_like(w)
    w.backward(dy)
    raw_r = raw.detach().double().requires_grad_(True)
    t_r = torch.tensor(tau, dtype=torch.float64, device=cuda, requires_grad=True)
    w_r = O.pn_scores(raw_r, t_r, 0.125, 10.0, 0.5, causal)
    w_r.backward(dy.double())
    assert rel_max(w, w_r) < 1e-5
    assert rel_max(raw.grad, raw_r.grad) < 1e-4
    assert abs(float(t.grad) - float(t_r.grad)) <= 1e-4 * max(1.0, abs(float(t_r.grad)))


def test_scores_op_beyond_reference_row_limit(cuda):
    N = 4100  # the reference falls back to eager above 4096
    g = torch.Generator().manual_seed(7)
    raw = (torch.randn(1, 1, N, N, generator=g) * 8).to(cuda)
    t = torch.tensor(0.2, device=cuda)
    w = P.triton_pn_fir_tau_scores(raw, t, scale=0.125)
    ref = O.pn_scores(raw.double(), t.double(), 0.125)
    assert rel_max(w, ref) < 1e-5


def test_scores_op_bf16(cuda):
    g = torch.Generator().manual_seed(3)
    raw = (torch.randn(2, 2, 256, 256, generator=g) * 8).to(cuda, torch.bfloat16).requires_grad_(True)
    t = torch.tensor(0.1, device=cuda, requires_grad=True)
    w = P.triton_pn_fir_tau_scores(raw, t, scale=0.125)
    assert w.dtype == torch.bfloat16
    dy = torch.randn_like(w)
    w.backward(dy)
    raw_r = raw.detach().float().requires_grad_(True)
    t_r = torch.tensor(0.1, device=cuda, requires_grad=True)
    w_r = O.pn_scores(raw_r, t_r, 0.125)
    w_r.backward(dy.float())
    assert rel_l2(w, w_r) < 1e-2
    assert rel_l2(raw.grad, raw_r.grad) < 1e-2
    assert abs(float(t.grad) - float(t_r.grad)) <= 1e-2 * abs(float(t_r.grad)) + 1e-6


@pytest.mark.parametrize("mode", ["peak", "mass_relu", "mass_pow"])
@pytest.mark.parametrize("p", [10.0, 2.0, 3.0])
def test_row_modes_with_tau_grad(cuda, mode, p):
    g = torch.Generator().manual_seed(11)
    raw = (torch.randn(1, 3, 90, 90, generator=g) * 4).to(cuda).requires_grad_(True)
    t = torch.tensor(0.25, device=cuda, requires_grad=True)
    w = P.pn_rows(raw, t, 0.25, p, 0.5, True, mode)
    dy = torch.randn_like(w)
    w.backward(dy)
    raw_r = raw.detach().double().requires_grad_(True)
    t_r = torch.tensor(0.25, dtype=torch.float64, device=cuda, requires_grad=True)
    w_r = O.pn_scores(raw_r, t_r, 0.25, p, 0.5, True, mode)
    w_r.backward(dy.double())
    assert rel_max(w, w_r) < 1e-5
    assert rel_max(raw.grad, raw_r.grad) < 1e-4
    assert abs(float(t.grad) - float(t_r.grad)) <= 1e-4 * max(1.0, abs(float(t_r.grad)))


def test_row_stats_and_silent_rows(cuda):
    raw = torch.full((1, 1, 8, 8), -5.0, device=cuda)
    raw[0, 0, 3, :2] = 4.0  # a two-way tie at the peak
    t = torch.tensor(0.0, device=cuda)
    w = P.triton_pn_fir_tau_scores(raw, t)
    assert torch.all(w[0, 0, :3] == 0) and torch.all(w[0, 0, 4:] == 0)
    assert torch.allclose(w[0, 0, 3, :2], torch.full((2,), 0.5 * 4.0 / 4.5, device=cuda))
