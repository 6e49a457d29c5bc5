"""Pins the CPU oracle (oracle/pnfirtau_oracle.py) to golden vectors produced
by running the reference's own eager code (tests/golden/make_golden.py).

All comparisons are fp32 against fp32: the oracle restates the same
arithmetic, so differences are reordering-level (<= ~1e-6 relative).
"""
import math

import pytest
import torch

from conftest import rel_max
from oracle import pnfirtau_oracle as O

TIGHT = 2e-6


def test_taps_match_reference(golden):
    taps = golden("taps")
    for k in (1, 3, 5, 7, 9, 11):
        assert torch.allclose(O.gaussian_taps(k, 3.0), taps[f"k{k}_sf3"], rtol=1e-6, atol=1e-7)
    assert torch.allclose(O.gaussian_taps(7, 2.0), taps["k7_sf2"], rtol=1e-6, atol=1e-7)
    # the values quoted in the reference docstring (lag-0 first), src/pnfirtau_attention.py:14
    h = taps["k7_sf3"].flip(0)
    quoted = torch.tensor([0.3329, 0.2938, 0.2019, 0.1081, 0.0451, 0.0146, 0.0037])
    assert torch.allclose(h, quoted, atol=6e-5)


@pytest.mark.parametrize("case", ["b2n20c12k7", "b1n5c3k7", "b3n33c40k5", "b2n17c8k9"])
def test_fir_matches_reference(golden, case):
    c = golden("fir")[case]
    K = c["taps"].numel()
    assert rel_max(O.causal_fir(c["x"], c["taps"]), c["y"]) < TIGHT
    assert rel_max(O.causal_fir_transpose(c["gy"], c["taps"]), c["gx"]) < TIGHT
    assert rel_max(O.causal_fir_dtaps(c["gy"], c["x"], K), c["dtaps"]) < 1e-5


def test_pngate_matches_reference(golden):
    cases = golden("pngate")
    assert len(cases) == 12
    for name, c in cases.items():
        s = c["scores"].clone().requires_grad_(True)
        w = O.power_norm_peak_gate(s, c["p"], c["gamma"], c["mode"])
        w.backward(c["dy"])
        assert rel_max(w, c["w"]) < TIGHT, name
        assert rel_max(s.grad, c["dscores"]) < 1e-5, name


def test_pngate_edge_rows_present(golden):
    c = golden("pngate")["p10.0_g0.5_peak"]
    w = c["w"]
    assert torch.all(w[1, 2, 5] == 0)  # silent row -> zero weights
    assert w[0, 0, 9, :4].unique().numel() == 1  # 4-way tie at the peak


@pytest.mark.parametrize(
    "case", ["b1h2n80d16_tau0", "b1h2n80d16_taup5", "b2h1n130d32_taum5", "b1h1n70d64_nc", "b1h2n96d16_quiet"]
)
def test_attention_matches_reference(golden, case):
    c = golden("attention")[case]
    q, k, v = (c[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
    tau = torch.tensor(c["tau"], requires_grad=True)
    out = O.pn_fir_tau_attention(q, k, v, tau, c["scale"], 0.5, c["causal"])
    out.backward(c["do"])
    assert rel_max(out, c["out"]) < TIGHT
    for got, ref in ((q.grad, c["dq"]), (k.grad, c["dk"]), (v.grad, c["dv"])):
        assert rel_max(got, ref) < 1e-5
    assert abs(float(tau.grad) - float(c["dtau"])) <= 1e-5 * max(1.0, abs(float(c["dtau"])))


@pytest.mark.parametrize("case", ["config1_b8n64d64h4", "exp4_b2n40d64h4_tau03"])
def test_mha_matches_reference(golden, case):
    c = golden("mha")[case]
    sd = {k: v.clone().requires_grad_(v.is_floating_point() and k != "fir_taps") for k, v in c["state_dict"].items()}
    x = c["x"].clone().requires_grad_(True)
    y = O.mha_forward(x, sd["qkv.weight"], sd["out.weight"], sd["score_tau"], sd["fir_taps"], c["n_heads"])
    if c["loss"] == "mean":
        y.mean().backward()
    else:
        y.backward(c["dy"])
    assert rel_max(y, c["out"]) < TIGHT
    assert rel_max(x.grad, c["dx"]) < 1e-5
    for n in ("qkv.weight", "out.weight"):
        assert rel_max(sd[n].grad, c["grads"][n]) < 1e-5
    ref_dtau = float(c["grads"]["score_tau"])
    assert abs(float(sd["score_tau"].grad) - ref_dtau) <= 1e-5 * max(1e-3, abs(ref_dtau))


def test_tile_silence_matches_reference(golden):
    t = golden("tiles")
    k_t = O.causal_fir(t["k_raw"].transpose(1, 2).reshape(1, 256, 32), t["taps"]).view(1, 256, 2, 16).transpose(1, 2)
    assert rel_max(k_t, t["k_tilde"]) < TIGHT
    for tau, r in t["per_tau"].items():
        tiles, row_silent, _ = O.tile_silence(t["q"], t["k_tilde"], tau, 1.0 / math.sqrt(16))
        assert torch.equal(tiles, r["tile_present"]), tau
        assert torch.equal(row_silent, r["row_silent"]), tau


def test_row_stats_consistent_with_weights(golden):
    c = golden("attention")["b1h2n80d16_taup5"]
    tau = torch.tensor(c["tau"])
    peak, z, nmax = O.row_stats(c["q"], c["k"], tau, c["scale"])
    s = O.thresholded_scores(c["q"] @ c["k"].transpose(-2, -1), tau, c["scale"], True)
    w = O.power_norm_peak_gate(s)
    gate = torch.where(peak > 0, peak / (peak + 0.5), torch.zeros_like(peak))
    # rows sum to gate * mass / (mass + 1e-12): below the gate only when u^10 is tiny
    assert torch.allclose(w.sum(-1), gate * (1 - 1e-12 / z), rtol=1e-5, atol=1e-6)
    assert torch.all((nmax == 0) == (peak == 0))


@pytest.mark.parametrize("case", ["b4n48d64h4", "b2n33d32h2_noncausal"])
def test_smfir_matches_reference(golden, case):
    c = golden("smfir")[case]
    sd = {k: v.clone().requires_grad_(k != "fir_taps") for k, v in c["state_dict"].items()}
    x = c["x"].clone().requires_grad_(True)
    y, w = O.smfir_forward(x, sd["qkv.weight"], sd["out.weight"], sd["fir_taps"], c["n_heads"], c["causal"])
    y.backward(c["dy"])
    assert rel_max(y, c["out"]) < TIGHT
    assert rel_max(w, c["weights"]) < TIGHT
    assert rel_max(x.grad, c["dx"]) < 1e-5
    for n in ("qkv.weight", "out.weight"):
        assert rel_max(sd[n].grad, c["grads"][n]) < 1e-5, n
