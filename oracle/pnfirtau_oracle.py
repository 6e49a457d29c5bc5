"""TEST INFRASTRUCTURE ONLY - the parity oracle of the pn_fir_tau operator.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs may import this module, and only as the checker or the timed CPU
baseline. The product package (paper_01_anti_decoy_pnfirtau_b200) never
imports it and has no CPU path.

It restates, in plain PyTorch fp32 (or fp64) tensor arithmetic, the reference's
eager algorithm for the hot path (mcfax-arch/paper_01_anti_decoy_pnfirtau,
files under src/). Each function cites the reference lines it follows. The
restatement is pinned by tests/test_oracle_golden.py against golden vectors
that tests/golden/make_golden.py produced by importing and running the
reference itself.

Precision: every function computes in the dtype of its inputs; callers pass
fp32 (the north-star tolerance base) or fp64 (for tight checks).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


# ---------------------------------------------------------------------------
# primitives
# ---------------------------------------------------------------------------


def gaussian_taps(k: int = 7, sigma_frac: float = 3.0, dtype=torch.float32) -> torch.Tensor:
    """Causal half-Gaussian taps; index k-1 is lag 0 (src/pnfirtau_attention.py:50-62)."""
    t = torch.arange(k, dtype=dtype)
    lag = (k - 1) - t
    sigma = max((k - 1) / sigma_frac, 0.5)
    w = torch.exp(-0.5 * (lag / sigma) ** 2)
    return w / w.sum()


def causal_fir(x: torch.Tensor, taps: torch.Tensor) -> torch.Tensor:
    """y[b,n,c] = sum_u taps[K-1-u] * x[b,n-u,c] (src/pnfirtau_attention.py:65-74).

    The reference convolves with F.conv1d after left-padding K-1 zeros; this is
    the same sum written as shifted copies, accumulated lag 0 first.
    """
    K = taps.numel()
    if K <= 1:
        return x
    B, N, C = x.shape
    taps = taps.to(dtype=x.dtype, device=x.device)
    y = x * taps[K - 1]
    for u in range(1, K):
        if u >= N:
            break
        y = y + F.pad(x[:, : N - u, :], (0, 0, u, 0)) * taps[K - 1 - u]
    return y


def causal_fir_transpose(gy: torch.Tensor, taps: torch.Tensor) -> torch.Tensor:
    """Adjoint of causal_fir: gx[b,n,c] = sum_u taps[K-1-u] * gy[b,n+u,c]
    (src/triton_pnfirtau.py:89-135)."""
    K = taps.numel()
    B, N, C = gy.shape
    taps = taps.to(dtype=gy.dtype, device=gy.device)
    gx = gy * taps[K - 1]
    for u in range(1, K):
        if u >= N:
            break
        gx = gx + F.pad(gy[:, u:, :], (0, 0, 0, u)) * taps[K - 1 - u]
    return gx


def power_norm_peak_gate(scores: torch.Tensor, p: float = 10.0, gamma: float | None = 0.5,
                         silence_mode: str = "peak") -> torch.Tensor:
    """relu -> u^p -> normalise by (mass + 1e-12) -> gate strength/(strength+gamma)
    (src/pnfirtau_attention.py:87-119)."""
    pos = F.relu(scores)
    if p == 10.0:
        x2 = pos * pos
        x4 = x2 * x2
        pw = x4 * x4 * x2
    elif p == 2.0:
        pw = pos * pos
    else:
        pw = torch.where(pos > 0, pos.pow(p), torch.zeros_like(pos))
    mass = pw.sum(dim=-1, keepdim=True)
    w = pw / (mass + 1e-12)
    if gamma is not None and gamma > 0:
        if silence_mode == "peak":
            strength = pos.amax(dim=-1, keepdim=True)
        elif silence_mode == "mass_relu":
            strength = pos.sum(dim=-1, keepdim=True)
        elif silence_mode == "mass_pow":
            strength = mass
        else:
            raise ValueError(f"unknown silence_mode={silence_mode}")
        w = w * (strength / (strength + gamma))
    return w


def thresholded_scores(raw: torch.Tensor, tau: torch.Tensor, scale: float, causal: bool) -> torch.Tensor:
    """raw*scale - tau with the future masked to -1e4 (src/pnfirtau_attention.py:232-237,
    the eager fallback of triton_pn_fir_tau_scores src/triton_pnfirtau.py:804-810)."""
    s = raw * scale - tau
    if causal:
        N = s.shape[-1]
        mask = torch.triu(torch.ones(N, N, dtype=torch.bool, device=s.device), diagonal=1)
        s = s.masked_fill(mask, -1e4)
    return s


def pn_scores(raw: torch.Tensor, tau: torch.Tensor, scale: float = 1.0, p: float = 10.0,
              gamma: float | None = 0.5, causal: bool = True, silence_mode: str = "peak") -> torch.Tensor:
    """Weights of the row op (the eager path behind triton_pn_fir_tau_scores)."""
    return power_norm_peak_gate(thresholded_scores(raw, tau, scale, causal), p, gamma, silence_mode)


def pn_fir_tau_attention(q: torch.Tensor, k_tilde: torch.Tensor, v: torch.Tensor, tau: torch.Tensor,
                         scale: float | None = None, gamma: float | None = 0.5, causal: bool = True,
                         p: float = 10.0, silence_mode: str = "peak") -> torch.Tensor:
    """The flash op's result, composed from the eager pieces
    (src/pnfirtau_attention.py:231-243 on already-filtered keys): q,k,v [B,H,N,D]."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    raw = torch.matmul(q, k_tilde.transpose(-2, -1))
    w = pn_scores(raw, tau, scale, p, gamma, causal, silence_mode)
    return torch.matmul(w, v)


def row_stats(q: torch.Tensor, k_tilde: torch.Tensor, tau: torch.Tensor, scale: float | None = None,
              causal: bool = True):
    """Per-row peak M, mass+1e-12 Z and tie count Nmax of the flash forward
    (the statistics stored by src/triton_pnfirtau.py:440-443)."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    s = thresholded_scores(torch.matmul(q, k_tilde.transpose(-2, -1)), tau, scale, causal)
    u = F.relu(s)
    peak = u.amax(dim=-1)
    x2 = u * u
    x4 = x2 * x2
    z = (x4 * x4 * x2).sum(dim=-1) + 1e-12
    nmax = ((u == peak[..., None]) & (peak[..., None] > 0)).sum(dim=-1).to(torch.int32)
    return peak, z, nmax


# ---------------------------------------------------------------------------
# module-level forward (PnFirTauMHA) as a function of its parameters
# ---------------------------------------------------------------------------


def mha_forward(x: torch.Tensor, qkv_weight: torch.Tensor, out_weight: torch.Tensor, score_tau: torch.Tensor,
                fir_taps: torch.Tensor, n_heads: int, p: float = 10.0, gamma: float | None = 0.5,
                silence_mode: str = "peak", causal: bool = True, qkv_bias=None, out_bias=None) -> torch.Tensor:
    """PnFirTauMHA.forward without dropout (src/pnfirtau_attention.py:214-247)."""
    B, N, Dm = x.shape
    H, hd = n_heads, Dm // n_heads
    qkv = F.linear(x, qkv_weight, qkv_bias).reshape(B, N, 3, H, hd)
    q, k, v = qkv.unbind(2)
    k = causal_fir(k.reshape(B, N, H * hd), fir_taps).view(B, N, H, hd)
    q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    scale = 1.0 / math.sqrt(hd)
    w = pn_scores(torch.matmul(q, k.transpose(-2, -1)), score_tau, scale, p, gamma, causal, silence_mode)
    out = torch.matmul(w, v).transpose(1, 2).reshape(B, N, -1)
    return F.linear(out, out_weight, out_bias)


def smfir_forward(x: torch.Tensor, qkv_weight: torch.Tensor, out_weight: torch.Tensor, fir_taps: torch.Tensor,
                  n_heads: int, causal: bool = True, qkv_bias=None, out_bias=None):
    """SmFirMHA.forward without dropout (src/pnfirtau_attention.py:152-192):
    softmax attention on causally filtered keys, the future masked to -1e4.
    Returns (out, weights)."""
    B, N, Dm = x.shape
    H, hd = n_heads, Dm // n_heads
    qkv = F.linear(x, qkv_weight, qkv_bias).reshape(B, N, 3, H, hd)
    q, k, v = qkv.unbind(2)
    k = causal_fir(k.reshape(B, N, H * hd), fir_taps).view(B, N, H, hd)
    q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    att = torch.matmul(q, k.transpose(-2, -1)) * (1.0 / math.sqrt(hd))
    if causal:
        mask = torch.triu(torch.ones(N, N, dtype=torch.bool, device=x.device), diagonal=1)
        att = att.masked_fill(mask, -1e4)
    w = torch.softmax(att, dim=-1)
    out = torch.matmul(w, v).transpose(1, 2).reshape(B, N, -1)
    return F.linear(out, out_weight, out_bias), w


# ---------------------------------------------------------------------------
# silent-tile oracle (experiments/exp4b_mha6_instrumentation.py:80-128)
# ---------------------------------------------------------------------------


def tile_silence(q: torch.Tensor, k_tilde: torch.Tensor, tau: float, scale: float | None = None,
                 tile: int = 64, causal: bool = True):
    """Per-(row-tile, col-tile) "has a positive score" flags and per-row silence.

    present = (raw*scale > tau) & causal; a tile is fully silent when it holds
    no present entry (exp4b_mha6_instrumentation.py:91-111). Returns
    (tile_present [B,H,nT,nT] bool, row_silent [B,H,N] bool, row_peak [B,H,N]).
    """
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    B, H, N, _ = q.shape
    raw = torch.matmul(q, k_tilde.transpose(-2, -1)) * scale
    present = raw > tau
    c = torch.arange(N, device=q.device)
    if causal:
        present = present & (c[:, None] >= c[None, :])
    nT = (N + tile - 1) // tile
    pad = nT * tile - N
    pp = F.pad(present, (0, pad, 0, pad))
    tiles = pp.reshape(B, H, nT, tile, nT, tile).any(dim=5).any(dim=3)
    row_silent = ~present.any(dim=-1)
    s = raw - tau
    if causal:
        s = s.masked_fill(~(c[:, None] >= c[None, :]), -1e4)
    row_peak = F.relu(s).amax(dim=-1)
    return tiles, row_silent, row_peak


def causal_fir_dtaps(gy: torch.Tensor, x: torch.Tensor, K: int) -> torch.Tensor:
    """Gradient of causal_fir with respect to its taps: dtaps[K-1-u] =
    sum_{b,n,c} gy[b,n,c] * x[b,n-u,c] (the weight gradient of the reference's
    conv1d, src/pnfirtau_attention.py:72-73)."""
    N = x.shape[1]
    d = torch.zeros(K, dtype=x.dtype, device=x.device)
    for u in range(K):
        if u >= N:
            continue
        d[K - 1 - u] = (gy[:, u:, :] * x[:, : N - u, :]).sum()
    return d
