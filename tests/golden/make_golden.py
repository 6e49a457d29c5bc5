"""Generates the golden fixtures under tests/golden/ by running the REFERENCE
implementation (mcfax-arch/paper_01_anti_decoy_pnfirtau, its eager PyTorch
code in src/pnfirtau_attention.py) on seeded inputs on the CPU in fp32.

Run from the repository root, with the reference checkout importable:

    python tests/golden/make_golden.py /path/to/reference [fixture names ...]

Only this script touches the reference; the fixtures it writes (small .pt
files) travel with the tests. The reference's Triton/Flash functions need a
GPU and are not run here; their eager counterparts (which the reference's
own fp32 parity harness, experiments/exp4_wikitext2_lm.py:385-455, treats as
ground truth) are.
"""
from __future__ import annotations

import math
import sys
from pathlib import Path

import torch

OUT = Path(__file__).resolve().parent


def _import_reference(root: str):
    sys.path.insert(0, root)
    import src.pnfirtau_attention as ref  # noqa: E402

    return ref


def gen_taps(ref):
    taps = {}
    for k in (1, 3, 5, 7, 9, 11):
        taps[f"k{k}_sf3"] = ref.causal_gaussian_taps(k, "cpu", torch.float32, 3.0)
    taps["k7_sf2"] = ref.causal_gaussian_taps(7, "cpu", torch.float32, 2.0)
    torch.save(taps, OUT / "taps.pt")


def gen_fir(ref):
    cases = {}
    g = torch.Generator().manual_seed(1)
    for name, (B, N, C, k) in {
        "b2n20c12k7": (2, 20, 12, 7),
        "b1n5c3k7": (1, 5, 3, 7),
        "b3n33c40k5": (3, 33, 40, 5),
        "b2n17c8k9": (2, 17, 8, 9),
    }.items():
        x = torch.randn(B, N, C, generator=g)
        taps = ref.causal_gaussian_taps(k, "cpu", torch.float32, 3.0)
        x_req = x.clone().requires_grad_(True)
        taps_req = taps.clone().requires_grad_(True)
        y = ref.causal_fir(x_req, taps_req)
        gy = torch.randn(B, N, C, generator=g)
        y.backward(gy)
        cases[name] = {"x": x, "taps": taps, "y": y.detach(), "gy": gy, "gx": x_req.grad, "dtaps": taps_req.grad}
    torch.save(cases, OUT / "fir.pt")


def gen_pngate(ref):
    """power_norm_peak_gate on thresholded, causally masked scores, with grads."""
    cases = {}
    g = torch.Generator().manual_seed(2)
    N = 17
    base = torch.randn(2, 3, N, N, generator=g) * 1.5
    # exact ties and silent rows
    base[0, 0, 9, :4] = 2.0
    base[0, 0, 9, 4:10] = -1.0
    base[1, 2, 5, :] = -3.0
    mask = torch.triu(torch.ones(N, N, dtype=torch.bool), diagonal=1)
    for p in (10.0, 2.0, 3.5):
        for gamma in (0.5, None):
            for mode in ("peak", "mass_relu", "mass_pow"):
                if gamma is None and mode != "peak":
                    continue
                s = base.masked_fill(mask, -1e4).clone().requires_grad_(True)
                w = ref.power_norm_peak_gate(s, p=p, gamma=gamma, silence_mode=mode)
                dy = torch.randn(w.shape, generator=g)
                w.backward(dy)
                cases[f"p{p}_g{gamma}_{mode}"] = {
                    "scores": base.masked_fill(mask, -1e4), "p": p, "gamma": gamma, "mode": mode,
                    "w": w.detach(), "dy": dy, "dscores": s.grad,
                }
    torch.save(cases, OUT / "pngate.pt")


def gen_attention(ref):
    """Operator-level composition of the flash op from the reference's eager
    pieces: scores = q k~^T*scale - tau, causal mask, power_norm_peak_gate, @v."""
    cases = {}
    g = torch.Generator().manual_seed(3)
    for name, (B, H, N, D, tau, causal, qscale) in {
        "b1h2n80d16_tau0": (1, 2, 80, 16, 0.0, True, 1.0),
        "b1h2n80d16_taup5": (1, 2, 80, 16, 0.5, True, 1.0),
        "b2h1n130d32_taum5": (2, 1, 130, 32, -0.5, True, 1.0),
        "b1h1n70d64_nc": (1, 1, 70, 64, 0.2, False, 1.0),
        "b1h2n96d16_quiet": (1, 2, 96, 16, 0.5, True, 0.05),
    }.items():
        q = torch.randn(B, H, N, D, generator=g) * qscale
        k = torch.randn(B, H, N, D, generator=g)
        v = torch.randn(B, H, N, D, generator=g)
        do = torch.randn(B, H, N, D, generator=g)
        tau_t = torch.tensor(float(tau), requires_grad=True)
        qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
        scale = 1.0 / math.sqrt(D)
        scores = torch.matmul(qr, kr.transpose(-2, -1)) * scale - tau_t
        if causal:
            scores = scores.masked_fill(torch.triu(torch.ones(N, N, dtype=torch.bool), diagonal=1), -1e4)
        w = ref.power_norm_peak_gate(scores, 10.0, 0.5, "peak")
        out = torch.matmul(w, vr)
        out.backward(do)
        cases[name] = {
            "q": q, "k": k, "v": v, "do": do, "tau": float(tau), "causal": causal, "scale": scale,
            "out": out.detach(), "dq": qr.grad, "dk": kr.grad, "dv": vr.grad, "dtau": tau_t.grad.detach(),
        }
    torch.save(cases, OUT / "attention.pt")


def gen_mha(ref):
    """PnFirTauMHA forward+backward (BASELINE config 1 and an exp4-style dy case)."""
    cases = {}
    for name, (B, N, Dm, H, seed, tau0, loss) in {
        "config1_b8n64d64h4": (8, 64, 64, 4, 0, 0.0, "mean"),
        "exp4_b2n40d64h4_tau03": (2, 40, 64, 4, 42, 0.3, "dy"),
    }.items():
        torch.manual_seed(seed)
        cfg = ref.PnFirConfig(d_model=Dm, n_heads=H, tau_init=tau0)
        m = ref.PnFirTauMHA(cfg)
        x = torch.randn(B, N, Dm)
        xr = x.clone().requires_grad_(True)
        y = m(xr)
        if loss == "mean":
            y.mean().backward()
            dy = None
        else:
            dy = torch.randn_like(y)
            y.backward(dy)
        cases[name] = {
            "d_model": Dm, "n_heads": H, "tau_init": tau0, "x": x, "dy": dy, "loss": loss,
            "state_dict": {k: v.clone() for k, v in m.state_dict().items()},
            "out": y.detach(), "dx": xr.grad,
            "grads": {n: p.grad.clone() for n, p in m.named_parameters()},
        }
    torch.save(cases, OUT / "mha.pt")


def gen_smfir(ref):
    """SmFirMHA (softmax attention on the causally filtered keys,
    src/pnfirtau_attention.py:152-192) forward+backward."""
    cases = {}
    for name, (B, N, Dm, H, seed, causal) in {
        "b4n48d64h4": (4, 48, 64, 4, 7, True),
        "b2n33d32h2_noncausal": (2, 33, 32, 2, 8, False),
    }.items():
        torch.manual_seed(seed)
        cfg = ref.PnFirConfig(d_model=Dm, n_heads=H, causal_mask=causal)
        m = ref.SmFirMHA(cfg)
        x = torch.randn(B, N, Dm)
        xr = x.clone().requires_grad_(True)
        y, w = m(xr, return_weights=True)
        dy = torch.randn_like(y)
        y.backward(dy)
        cases[name] = {
            "d_model": Dm, "n_heads": H, "causal": causal, "x": x, "dy": dy,
            "state_dict": {k: v.clone() for k, v in m.state_dict().items()},
            "out": y.detach(), "weights": w.detach(), "dx": xr.grad,
            "grads": {n: p.grad.clone() for n, p in m.named_parameters()},
        }
    torch.save(cases, OUT / "smfir.pt")


def gen_tiles(ref):
    """exp4b's silent-tile definition (experiments/exp4b_mha6_instrumentation.py:91-111)
    evaluated with the reference's own reshape/permute expression."""
    g = torch.Generator().manual_seed(4)
    B, H, N, D = 1, 2, 256, 16
    q = torch.randn(B, H, N, D, generator=g)
    blocks = torch.rand(B, H, N // 64, generator=g) < 0.5
    q = q * torch.where(blocks, 0.05, 1.0).repeat_interleave(64, dim=-1)[..., None]
    k = torch.randn(B, H, N, D, generator=g)
    taps = ref.causal_gaussian_taps(7)
    k_t = ref.causal_fir(k.transpose(1, 2).reshape(B, N, H * D), taps).view(B, N, H, D).transpose(1, 2)
    scale = 1.0 / math.sqrt(D)
    causal = torch.arange(N)[:, None] >= torch.arange(N)[None, :]
    out = {"q": q, "k_raw": k, "taps": taps, "k_tilde": k_t, "per_tau": {}}
    for tau in (-0.5, 0.0, 0.5):
        raw = torch.matmul(q, k_t.transpose(-2, -1)) * scale
        present = (raw > tau) & causal
        n_rt = n_ct = N // 64
        blk = (~present).reshape(B, H, n_rt, 64, n_ct, 64).permute(0, 1, 2, 4, 3, 5)
        tile_present = (~blk).any(dim=(-2, -1))
        out["per_tau"][tau] = {
            "tile_present": tile_present,
            "row_silent": ~present.any(dim=-1),
            "fully_silent_tiles_u": 1.0 - tile_present.float().mean().item(),
            "silent_rows_u": 1.0 - present.any(dim=-1).float().mean().item(),
        }
    torch.save(out, OUT / "tiles.pt")


GENERATORS = {"taps": gen_taps, "fir": gen_fir, "pngate": gen_pngate, "attention": gen_attention, "mha": gen_mha,
              "smfir": gen_smfir, "tiles": gen_tiles}


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else None
    if root is None:
        raise SystemExit("usage: make_golden.py <reference checkout root> [fixture names ...]")
    ref = _import_reference(root)
    torch.set_num_threads(1)
    for name in sys.argv[2:] or list(GENERATORS):
        GENERATORS[name](ref)
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
