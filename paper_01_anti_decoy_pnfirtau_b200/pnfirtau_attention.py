"""pn_fir_tau attention modules and primitives on CUDA (counterpart of the
reference's ``src/pnfirtau_attention.py``).

Per head:
  1. causal FIR on the keys along N:  K~[t] = sum_u h[u] K[t-u]
  2. thresholded scores:              S[t,j] = <Q[t], K~[j]>/sqrt(d) - tau
  3. ReLU + p-th power normalisation: w^[t,j] = relu(S)^p / (sum_m relu(S)^p + 1e-12)
  4. peak silence gate:               W = w^ * peak/(peak + gamma)
  5. output:                          O = W V

Names, constructor arguments, ``forward`` signatures, parameter/buffer names
(``qkv.weight``, ``out.weight``, ``score_tau``, ``fir_taps``) and defaults match
the reference so ``state_dict``s load both ways. The three module classes route
to the CUDA operators of ``pnfirtau_ops``; there is no eager or CPU path, and a
CPU input raises ``RuntimeError``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .pnfirtau_ops import (
    _flash_bnhd,
    _flash_fir_qkv,
    _qkv_views,
    fused_fir_applies,
    pn_rows,
    triton_causal_fir,
    triton_pn_fir_tau_scores,
)

__all__ = [
    "PnFirConfig",
    "causal_gaussian_taps",
    "causal_fir",
    "power_norm_peak_gate",
    "PnFirTauMHA",
    "PnFirTauTritonMHA",
    "PnFirTauFlashMHA",
    "SmFirMHA",
]


@dataclass(frozen=True)
class PnFirConfig:
    """Hyper-parameters; fields and defaults as src/pnfirtau_attention.py:35-47."""

    d_model: int = 64
    n_heads: int = 4
    p: float = 10.0
    silence_gamma: float | None = 0.5
    silence_mode: str = "peak"
    tau_init: float = 0.0
    fir_k: int = 7
    fir_sigma_frac: float = 3.0
    dropout: float = 0.0
    causal_mask: bool = True
    bias: bool = False


def causal_gaussian_taps(
    k: int,
    device: torch.device | str = "cpu",
    dtype: torch.dtype = torch.float32,
    sigma_frac: float = 3.0,
) -> torch.Tensor:
    """Half-Gaussian causal FIR taps ``[k]``; index k-1 is lag 0, index 0 the oldest lag.

    h[k-1-u] = exp(-u^2 / (2 sigma^2)) / Z with sigma = max((k-1)/sigma_frac, 0.5)
    (src/pnfirtau_attention.py:50-62). This is parameter initialisation, not
    part of the operator.
    """
    assert k % 2 == 1 and k >= 1
    lag = (k - 1) - torch.arange(k, device=device, dtype=dtype)
    sigma = max((k - 1) / sigma_frac, 0.5)
    w = torch.exp(-0.5 * (lag / sigma) ** 2)
    return w / w.sum()


def causal_fir(x: torch.Tensor, taps: torch.Tensor) -> torch.Tensor:
    """Depthwise causal FIR along N of x ``[B, N, C]`` (src/pnfirtau_attention.py:65-74), on CUDA."""
    return triton_causal_fir(x, taps)


def power_norm_peak_gate(
    scores: torch.Tensor,
    p: float = 10.0,
    gamma: float | None = 0.5,
    silence_mode: str = "peak",
) -> torch.Tensor:
    """ReLU power-norm with optional soft silence gate on ``scores [..., Nk]``.

    src/pnfirtau_attention.py:87-119: rows sum to the gate (<= 1). Runs the
    row-fused CUDA kernel with scale 1, tau 0 and no mask (the caller's
    ``scores`` already carry the threshold and any masking).
    """
    zero = torch.zeros((), device=scores.device, dtype=torch.float32)
    return pn_rows(scores, zero, 1.0, p, gamma, False, silence_mode)


class _PnFirTauBase(nn.Module):
    def __init__(self, cfg: PnFirConfig):
        super().__init__()
        assert cfg.d_model % cfg.n_heads == 0
        assert cfg.fir_k % 2 == 1
        self.cfg = cfg
        self.n_heads = cfg.n_heads
        self.head_dim = cfg.d_model // cfg.n_heads
        self.qkv = nn.Linear(cfg.d_model, 3 * cfg.d_model, bias=cfg.bias)
        self.out = nn.Linear(cfg.d_model, cfg.d_model, bias=cfg.bias)
        self.drop = nn.Dropout(cfg.dropout)
        self.score_tau = nn.Parameter(torch.tensor(float(cfg.tau_init)))
        taps = causal_gaussian_taps(cfg.fir_k, torch.device("cpu"), torch.float32, cfg.fir_sigma_frac)
        self.register_buffer("fir_taps", taps, persistent=True)

    def _qkv_heads(self, x: torch.Tensor):
        B, N, _ = x.shape
        H, hd = self.n_heads, self.head_dim
        q_raw, k_raw, v_raw = self.qkv(x).chunk(3, dim=-1)
        k = triton_causal_fir(k_raw, self.fir_taps).view(B, N, H, hd).transpose(1, 2)
        q = q_raw.view(B, N, H, hd).transpose(1, 2)
        v = v_raw.view(B, N, H, hd).transpose(1, 2)
        return q, k, v

    def _weights_path(self, x: torch.Tensor, rows_fn, return_weights: bool):
        B, N, _ = x.shape
        q, k, v = self._qkv_heads(x)
        scale = 1.0 / math.sqrt(self.head_dim)
        raw_scores = torch.matmul(q, k.transpose(-2, -1))
        w = rows_fn(raw_scores, scale)
        w = self.drop(w)
        out = torch.matmul(w, v).transpose(1, 2).reshape(B, N, -1)
        out = self.out(out)
        if return_weights:
            return out, w
        return out


class PnFirTauMHA(_PnFirTauBase):
    """Canonical pn_fir_tau multi-head attention (src/pnfirtau_attention.py:195-247).

    Honors every ``PnFirConfig`` field: general ``p``, all three silence modes,
    ``silence_gamma=None``, attention dropout and ``causal_mask=False``.
    """

    def forward(self, x: torch.Tensor, return_weights: bool = False):
        cfg = self.cfg
        return self._weights_path(
            x,
            lambda raw, scale: pn_rows(raw, self.score_tau, scale, cfg.p, cfg.silence_gamma, cfg.causal_mask,
                                       cfg.silence_mode),
            return_weights,
        )


class PnFirTauTritonMHA(PnFirTauMHA):
    """Row-fused path (src/pnfirtau_attention.py:250-282): FIR kernel, cuBLAS
    scores, row kernel (peak silence, as the reference), dropout, PV."""

    def forward(self, x: torch.Tensor, return_weights: bool = False):
        cfg = self.cfg
        return self._weights_path(
            x,
            lambda raw, scale: triton_pn_fir_tau_scores(raw, self.score_tau, scale=scale, p=cfg.p,
                                                        gamma=cfg.silence_gamma, causal_mask=cfg.causal_mask),
            return_weights,
        )


class PnFirTauFlashMHA(PnFirTauMHA):
    """O(N)-memory tiled path with silent-tile skipping (src/pnfirtau_attention.py:285-316).

    As in the reference it uses p = 10 and the peak gate regardless of
    ``cfg.p`` / ``cfg.silence_mode`` and applies no attention dropout;
    ``return_weights=True`` takes the row-fused path.

    ``fuse_fir`` (default) routes the keys' causal filter through
    flash_pn_fir_tau_attention_fir where that path serves the inputs (7 taps,
    bf16, head dims that are multiples of 16 up to 128): the backward filters its key tile inside the
    attention kernel (no filtered-key tensor is kept for it, no separate
    filter backward node) and the forward runs one filter pass before the
    attention kernel. The results equal the unfused path's (the tile filter is
    bit-exact); ``fuse_fir=False`` keeps the separate ``triton_causal_fir``.
    """

    def __init__(self, cfg: PnFirConfig, fuse_fir: bool = True):
        super().__init__(cfg)
        self.fuse_fir = fuse_fir

    def forward(self, x: torch.Tensor, return_weights: bool = False):
        if return_weights:
            return PnFirTauTritonMHA.forward(self, x, return_weights=True)
        cfg = self.cfg
        B, N, _ = x.shape
        scale = 1.0 / math.sqrt(self.head_dim)
        if self.fuse_fir:
            H = self.n_heads
            qkv = self.qkv(x)
            if fused_fir_applies(*_qkv_views(qkv, H), cfg.fir_k):
                out = _flash_fir_qkv(qkv, H, self.score_tau, self.fir_taps, scale, cfg.silence_gamma,
                                     cfg.causal_mask)
                return self.out(out.transpose(1, 2).reshape(B, N, -1))
        q, k, v = self._qkv_heads(x)
        out = _flash_bnhd(q, k, v, self.score_tau, scale, cfg.silence_gamma, cfg.causal_mask)
        out = out.transpose(1, 2).reshape(B, N, -1)
        return self.out(out)


class SmFirMHA(nn.Module):
    """Softmax attention on causally filtered keys (src/pnfirtau_attention.py:152-192).

    The keys' causal FIR runs on this library's FIR kernel (triton_causal_fir,
    the same kernel the pn_fir_tau modules use, with its tap gradient); only the
    normaliser differs from PnFirTauMHA. Scores, the causal mask (-1e4 on the
    future, as the reference; equal to -inf under softmax since every row keeps
    its diagonal), softmax, dropout and PV are PyTorch's: fused
    scaled_dot_product_attention when no weights are returned, explicit matmul +
    softmax when ``return_weights=True``. Parameter and buffer names (``qkv``,
    ``out``, ``fir_taps``) match the reference. CUDA only, like the other modules.
    """

    def __init__(self, cfg: PnFirConfig):
        super().__init__()
        assert cfg.d_model % cfg.n_heads == 0
        self.cfg = cfg
        self.n_heads = cfg.n_heads
        self.head_dim = cfg.d_model // cfg.n_heads
        self.qkv = nn.Linear(cfg.d_model, 3 * cfg.d_model, bias=cfg.bias)
        self.out = nn.Linear(cfg.d_model, cfg.d_model, bias=cfg.bias)
        self.drop = nn.Dropout(cfg.dropout)
        taps = causal_gaussian_taps(cfg.fir_k, torch.device("cpu"), torch.float32, cfg.fir_sigma_frac)
        self.register_buffer("fir_taps", taps, persistent=True)

    def forward(self, x: torch.Tensor, return_weights: bool = False):
        B, N, _ = x.shape
        H, hd = self.n_heads, self.head_dim
        q_raw, k_raw, v_raw = self.qkv(x).chunk(3, dim=-1)
        k = triton_causal_fir(k_raw, self.fir_taps).view(B, N, H, hd).transpose(1, 2)
        q = q_raw.view(B, N, H, hd).transpose(1, 2)
        v = v_raw.view(B, N, H, hd).transpose(1, 2)
        if return_weights:
            att = torch.matmul(q, k.transpose(-2, -1)) * (1.0 / math.sqrt(hd))
            if self.cfg.causal_mask:
                causal = torch.triu(torch.ones(N, N, device=x.device, dtype=torch.bool), diagonal=1)
                att = att.masked_fill(causal, -1e4)
            w = self.drop(F.softmax(att, dim=-1))
            out = torch.matmul(w, v)
        else:
            out = F.scaled_dot_product_attention(q, k, v, dropout_p=self.drop.p if self.training else 0.0,
                                                 is_causal=self.cfg.causal_mask)
        out = self.out(out.transpose(1, 2).reshape(B, N, -1))
        if return_weights:
            return out, w
        return out
