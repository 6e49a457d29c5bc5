"""Module-level parity: the three pn_fir_tau modules on CUDA against the
reference's golden vectors (BASELINE config 1 and an exp4-style case), the
port of the reference's fp32 parity harness (exp4_wikitext2_lm.py:385-455)
and its causality gate (exp4_wikitext2_lm.py:293-307)."""
import pytest
import torch

import paper_01_anti_decoy_pnfirtau_b200 as P
from conftest import rel_l2, rel_max
from oracle import pnfirtau_oracle as O

pytestmark = pytest.mark.gpu

CLASSES = [P.PnFirTauMHA, P.PnFirTauTritonMHA, P.PnFirTauFlashMHA]


@pytest.mark.parametrize("cls", CLASSES)
@pytest.mark.parametrize("case", ["config1_b8n64d64h4", "exp4_b2n40d64h4_tau03"])
def test_module_golden_fp32(cuda, golden, cls, case):
    c = golden("mha")[case]
    m = cls(P.PnFirConfig(d_model=c["d_model"], n_heads=c["n_heads"], tau_init=c["tau_init"])).to(cuda)
    m.load_state_dict(c["state_dict"])
    x = c["x"].to(cuda).requires_grad_(True)
    y = m(x)
    if c["loss"] == "mean":
        y.mean().backward()
    else:
        y.backward(c["dy"].to(cuda))
    assert rel_max(y, c["out"]) < 1e-5
    assert rel_max(x.grad, c["dx"]) < 5e-5
    for n, p in m.named_parameters():
        ref = c["grads"][n]
        if n == "score_tau":
            assert abs(float(p.grad) - float(ref)) <= 5e-5 * max(1e-3, abs(float(ref))), n
        else:
            assert rel_max(p.grad, ref) < 5e-5, n


def test_exp4_parity_harness(cuda):
    """fp32, TF32 off, x [8,128,64], dy ~ N(0,1), seed 42: the three modules
    agree with the eager oracle (reference: 2.4e-7 out, 6.1e-7 dx, 5.7e-6 dtau)."""
    torch.manual_seed(42)
    cfg = P.PnFirConfig(d_model=64, n_heads=4, dropout=0.0)
    mods = [cls(cfg).to(cuda) for cls in CLASSES]
    for m in mods[1:]:
        m.load_state_dict(mods[0].state_dict())
    x0 = torch.randn(8, 128, 64, device=cuda)
    dy = torch.randn_like(x0)
    sd = {k: v.detach().clone().double() for k, v in mods[0].state_dict().items()}
    sd_r = {k: v.requires_grad_(k != "fir_taps") for k, v in sd.items()}
    xr = x0.double().requires_grad_(True)
    yr = O.mha_forward(xr, sd_r["qkv.weight"], sd_r["out.weight"], sd_r["score_tau"], sd_r["fir_taps"], 4)
    yr.backward(dy.double())
    for m in mods:
        x = x0.clone().requires_grad_(True)
        y = m(x)
        y.backward(dy)
        assert rel_max(y, yr) < 1e-5, type(m).__name__
        assert rel_max(x.grad, xr.grad) < 1e-5, type(m).__name__
        dt, dtr = float(m.score_tau.grad), float(sd_r["score_tau"].grad)
        assert abs(dt - dtr) <= 1e-4 * max(1e-3, abs(dtr)), type(m).__name__


@pytest.mark.parametrize("cls", CLASSES)
def test_causality_gate(cuda, cls):
    torch.manual_seed(0)
    m = cls(P.PnFirConfig(d_model=64, n_heads=4)).to(cuda)
    x = torch.randn(2, 96, 64, device=cuda)
    y1 = m(x)
    x2 = x.clone()
    x2[:, -1] += 5.0 * torch.randn_like(x2[:, -1])
    y2 = m(x2)
    assert (y1[:, :-1] - y2[:, :-1]).abs().max().item() < 1e-4


@pytest.mark.parametrize("mode", ["peak", "mass_relu", "mass_pow"])
@pytest.mark.parametrize("p,gamma", [(10.0, 0.5), (2.0, 0.5), (3.0, 0.25), (10.0, None)])
def test_eager_module_all_config_fields(cuda, mode, p, gamma):
    if gamma is None and mode != "peak":
        pytest.skip("the mode is only read when a gate is applied")
    torch.manual_seed(1)
    cfg = P.PnFirConfig(d_model=64, n_heads=4, p=p, silence_gamma=gamma, silence_mode=mode, tau_init=0.1)
    m = P.PnFirTauMHA(cfg).to(cuda)
    x = torch.randn(2, 50, 64, device=cuda, requires_grad=True)
    y = m(x)
    dy = torch.randn_like(y)
    y.backward(dy)
    sd = {k: v.detach().double().requires_grad_(k != "fir_taps") for k, v in m.state_dict().items()}
    xr = x.detach().double().requires_grad_(True)
    yr = O.mha_forward(xr, sd["qkv.weight"], sd["out.weight"], sd["score_tau"], sd["fir_taps"], 4, p, gamma, mode)
    yr.backward(dy.double())
    assert rel_max(y, yr) < 1e-5
    assert rel_max(x.grad, xr.grad) < 1e-4
    # dtau is a cancelling sum over every weight: fp32 vs fp64 agree to ~1e-4 relative
    assert abs(float(m.score_tau.grad) - float(sd["score_tau"].grad)) <= 1e-3 * max(1e-3, abs(float(sd["score_tau"].grad)))


def test_return_weights_path(cuda):
    torch.manual_seed(2)
    m = P.PnFirTauFlashMHA(P.PnFirConfig(d_model=64, n_heads=4)).to(cuda)
    x = torch.randn(2, 70, 64, device=cuda)
    out, w = m(x, return_weights=True)
    out2 = m(x)
    assert w.shape == (2, 4, 70, 70)
    assert rel_max(out, out2) < 1e-5
    assert torch.all(w.sum(-1) <= 1.0 + 1e-6)


def test_bf16_autocast_module(cuda):
    """Under bf16 autocast the projections run in bf16, so the module-level error
    against fp32 is dominated by them: ours must be no worse than the reference's
    own eager path under the same autocast (with a small margin)."""
    torch.manual_seed(3)
    m = P.PnFirTauFlashMHA(P.PnFirConfig(d_model=256, n_heads=4)).to(cuda)
    x = torch.randn(4, 512, 256, device=cuda, requires_grad=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x)
    y.float().pow(2).mean().backward()
    sd = {k: v.detach().float().requires_grad_(k != "fir_taps") for k, v in m.state_dict().items()}

    def eager(autocast):
        xr = x.detach().clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            yr = O.mha_forward(xr, sd["qkv.weight"], sd["out.weight"], sd["score_tau"], sd["fir_taps"], 4)
        yr.float().pow(2).mean().backward()
        for v in sd.values():
            v.grad = None
        return yr.float().detach(), xr.grad

    y32, dx32 = eager(False)
    y16, dx16 = eager(True)
    assert rel_l2(y.float(), y32) <= max(2e-2, 1.25 * rel_l2(y16, y32))
    assert rel_l2(x.grad, dx32) <= max(2e-2, 1.25 * rel_l2(dx16, dx32))


@pytest.mark.parametrize("return_weights", [False, True])
@pytest.mark.parametrize("case", ["b4n48d64h4", "b2n33d32h2_noncausal"])
def test_smfir_golden_fp32(cuda, golden, case, return_weights):
    """SmFirMHA (softmax on the FIR-filtered keys, the FIR on this library's
    kernel) against the reference's golden forward/backward, fp32."""
    c = golden("smfir")[case]
    m = P.SmFirMHA(P.PnFirConfig(d_model=c["d_model"], n_heads=c["n_heads"], causal_mask=c["causal"])).to(cuda)
    m.load_state_dict(c["state_dict"])
    x = c["x"].to(cuda).requires_grad_(True)
    if return_weights:
        y, w = m(x, return_weights=True)
        assert rel_max(w, c["weights"]) < 1e-5
    else:
        y = m(x)
    y.backward(c["dy"].to(cuda))
    assert rel_max(y, c["out"]) < 1e-5
    assert rel_max(x.grad, c["dx"]) < 5e-5
    for n, p in m.named_parameters():
        assert rel_max(p.grad, c["grads"][n]) < 5e-5, n


def test_smfir_bf16_autocast_lm_shape(cuda):
    """The LM's attention shape (d_model 256, 4 heads of 64, seq 512) under bf16
    autocast against the fp32 oracle with the same parameters."""
    torch.manual_seed(3)
    m = P.SmFirMHA(P.PnFirConfig(d_model=256, n_heads=4)).to(cuda)
    x = torch.randn(4, 512, 256, device=cuda)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x)
    sd = m.state_dict()
    yr, _ = O.smfir_forward(x, sd["qkv.weight"], sd["out.weight"], sd["fir_taps"], 4)
    assert rel_l2(y.float(), yr) < 1e-2
