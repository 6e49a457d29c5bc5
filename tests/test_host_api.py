"""Host-side API surface checks (CPU only): names, defaults, state_dict keys
and the no-CPU-path contract of the reference-facing Python API."""
import inspect
import math

import pytest
import torch

import paper_01_anti_decoy_pnfirtau_b200 as P
from oracle import pnfirtau_oracle as O


def test_config_defaults_match_reference():
    # src/pnfirtau_attention.py:35-47
    c = P.PnFirConfig()
    assert (c.d_model, c.n_heads, c.p, c.silence_gamma, c.silence_mode) == (64, 4, 10.0, 0.5, "peak")
    assert (c.tau_init, c.fir_k, c.fir_sigma_frac, c.dropout, c.causal_mask, c.bias) == (0.0, 7, 3.0, 0.0, True, False)
    with pytest.raises(Exception):
        c.p = 2.0  # frozen


def test_public_signatures_match_reference():
    s = inspect.signature(P.flash_pn_fir_tau_attention)
    # the reference's positional parameters, in order; additions are keyword-only
    positional = [n for n, q in s.parameters.items() if q.kind is not inspect.Parameter.KEYWORD_ONLY]
    assert positional == ["q", "k_tilde", "v", "score_tau", "scale", "gamma", "causal_mask"]
    assert [n for n in s.parameters if n not in positional] == ["deterministic"]
    assert s.parameters["scale"].default is None and s.parameters["gamma"].default == 0.5
    assert s.parameters["causal_mask"].default is True
    s = inspect.signature(P.triton_pn_fir_tau_scores)
    assert list(s.parameters) == ["raw_scores", "score_tau", "scale", "p", "gamma", "causal_mask"]
    assert [s.parameters[n].default for n in ("scale", "p", "gamma", "causal_mask")] == [1.0, 10.0, 0.5, True]
    assert list(inspect.signature(P.triton_causal_fir).parameters) == ["x", "taps"]
    s = inspect.signature(P.power_norm_peak_gate)
    assert [s.parameters[n].default for n in ("p", "gamma", "silence_mode")] == [10.0, 0.5, "peak"]


def test_taps_function_matches_golden(golden):
    taps = golden("taps")
    for k in (1, 3, 5, 7, 9, 11):
        assert torch.allclose(P.causal_gaussian_taps(k), taps[f"k{k}_sf3"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("cls", [P.PnFirTauMHA, P.PnFirTauTritonMHA, P.PnFirTauFlashMHA])
def test_state_dict_keys_match_reference(golden, cls):
    ref_sd = golden("mha")["config1_b8n64d64h4"]["state_dict"]
    m = cls(P.PnFirConfig(d_model=64, n_heads=4))
    assert set(m.state_dict()) == set(ref_sd)
    m.load_state_dict(ref_sd)  # loads both ways
    for k, v in m.state_dict().items():
        assert v.shape == ref_sd[k].shape and v.dtype == ref_sd[k].dtype


def test_module_init_matches_reference_under_seed(golden):
    c = golden("mha")["config1_b8n64d64h4"]
    torch.manual_seed(0)
    m = P.PnFirTauMHA(P.PnFirConfig(d_model=64, n_heads=4))
    for k, v in m.state_dict().items():
        assert torch.equal(v, c["state_dict"][k]), k


def test_cpu_inputs_raise_no_fallback():
    x = torch.randn(2, 16, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        P.triton_causal_fir(x, P.causal_gaussian_taps(7))
    q = torch.randn(1, 1, 16, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        P.flash_pn_fir_tau_attention(q, q, q, torch.tensor(0.0))
    with pytest.raises(RuntimeError, match="CUDA"):
        P.triton_pn_fir_tau_scores(torch.randn(1, 8, 8), torch.tensor(0.0))
    m = P.PnFirTauFlashMHA(P.PnFirConfig())
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(1, 8, 64))


def test_row_op_shape_contract():
    with pytest.raises(AssertionError, match="N, N"):
        P.triton_pn_fir_tau_scores(torch.randn(1, 8, 9), torch.tensor(0.0))


def test_oracle_flash_defaults_scale():
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 1, 8, 16, generator=g) for _ in range(3))
    a = O.pn_fir_tau_attention(q, k, v, torch.tensor(0.0))
    b = O.pn_fir_tau_attention(q, k, v, torch.tensor(0.0), scale=1.0 / math.sqrt(16))
    assert torch.equal(a, b)
