"""Multi-GPU layout of the flash pn_fir_tau operator: one process per GPU,
each owning a contiguous block of the flattened batch x heads range.

Every (b, h) slice of the operator is independent (the reference's kernels
run one program per (query block, b*h), src/triton_pnfirtau.py:313-443 and
445-621), so out, dq, dk and dv need no collective. The one value shared by
all slices is the threshold tau: its gradient is the sum of every rank's
partial, reduced once per backward in fp64 (the reference sums its per-tile
partials in fp64, src/triton_pnfirtau.py:955-960).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch


def bh_range(B: int, H: int, rank: int, world: int) -> tuple[int, int]:
    """Half-open range [lo, hi) of flattened b*H + h indices owned by `rank`.

    Contiguous blocks; the first (B*H) % world ranks take one extra slice, so
    the blocks cover the range exactly once for any world size.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bh_range: rank {rank} outside world of {world}")
    if B < 0 or H < 0:
        raise ValueError(f"bh_range: negative size B={B} H={H}")
    n = B * H
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_bh(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's [1, hi-lo, N, d] block of a [B, H, N, d] tensor (a view when
    the B and H dimensions can be flattened without a copy)."""
    if x.dim() != 4:
        raise ValueError(f"shard_bh expects [B, H, N, d], got {tuple(x.shape)}")
    B, H = x.shape[:2]
    lo, hi = bh_range(B, H, rank, world)
    return x.flatten(0, 1)[lo:hi].unsqueeze(0)


def unshard_bh(parts: list[torch.Tensor], B: int, H: int) -> torch.Tensor:
    """Inverse of shard_bh over all ranks' blocks (rank order)."""
    flat = torch.cat([p.flatten(0, 1) for p in parts], dim=0)
    if flat.shape[0] != B * H:
        raise ValueError(f"unshard_bh: {flat.shape[0]} slices for B*H = {B * H}")
    return flat.reshape(B, H, *flat.shape[1:])


class _SumTauGrad(torch.autograd.Function):
    """Identity on tau whose backward all-reduces the gradient (fp64 sum)."""

    @staticmethod
    def forward(ctx, tau, group):
        ctx.group = group
        return tau.view_as(tau)

    @staticmethod
    def backward(ctx, g):
        import torch.distributed as dist

        t = g.to(torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=ctx.group)
        return t.to(g.dtype), None


def share_tau(tau: torch.Tensor, group=None) -> torch.Tensor:
    """tau as seen by this rank's slices: its gradient becomes the sum over the
    process group. Without an initialised process group it is tau itself."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return tau
    return _SumTauGrad.apply(tau, group)


def sharded_flash_pn_fir_tau_attention(q: torch.Tensor, k_tilde: torch.Tensor, v: torch.Tensor,
                                       score_tau: torch.Tensor, scale: Optional[float] = None,
                                       gamma: Optional[float] = 0.5, causal_mask: bool = True, group=None,
                                       attention: Optional[Callable] = None) -> torch.Tensor:
    """flash_pn_fir_tau_attention on this rank's [1, S, N, d] shard (see
    shard_bh) with tau's gradient summed over `group`.

    `attention` defaults to the CUDA operator; it takes the reference's
    argument list (q, k_tilde, v, score_tau, scale, gamma, causal_mask).
    """
    if attention is None:
        from .pnfirtau_ops import flash_pn_fir_tau_attention as attention
    return attention(q, k_tilde, v, share_tau(score_tau, group), scale, gamma, causal_mask)
