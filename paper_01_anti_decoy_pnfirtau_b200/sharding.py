"""Multi-GPU layout of the flash pn_fir_tau operator: one process per GPU,
each owning a contiguous block of the flattened batch x heads range.

Every (b, h) slice of the operator is independent (the reference's kernels
run one program per (query block, b*h), src/triton_pnfirtau.py:313-443 and
445-621), so out, dq, dk and dv need no collective. The one value shared by
all slices is the threshold tau: its gradient is the sum of every rank's
partial, reduced once per backward in fp64 (the reference sums its per-tile
partials in fp64, src/triton_pnfirtau.py:955-960), either inside the backward
or, through a TauGradReducer, on a side stream whose result the consumer of
tau's gradient waits for.
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


class TauGradReducer:
    """Sum of tau's gradient over the process group, reduced off the critical path.

    The backward of ``share_tau(tau, group, reducer)`` hands this rank's partial
    to :meth:`push`, which converts it to fp64 and all-reduces it on a side stream
    of the gradient's device (the compute stream only records an event): the
    collective overlaps the next kernels instead of putting every rank in
    lock-step once per backward (the side stream has high priority; with NCCL
    on a high-priority stream too, the collective's kernel takes the next free SM
    slot instead of queueing behind long compute kernels). The partial sums of
    successive backwards
    accumulate here until the consumer of tau's gradient calls :meth:`result`
    (its current stream then waits for the side stream) or :meth:`accumulate_into`
    (which adds the sum to ``tau.grad``), as data-parallel training finalises its
    gradient buckets before the optimizer step. Every rank must push the same
    number of times, in the same order (one collective per backward).
    On CPU tensors (``gloo``) the all-reduce runs inline. ``group`` may be a
    communicator of its own whose kernels take one CTA (NCCL options
    ``min_ctas = max_ctas = 1``): the 8-byte collective then runs beside the
    next step's kernels without queueing behind them.
    """

    def __init__(self, group=None):
        self.group = group
        self._sum: Optional[torch.Tensor] = None
        self._streams: dict = {}
        self.pushes = 0

    def push(self, g: torch.Tensor) -> None:
        import torch.distributed as dist

        self.pushes += 1
        if not g.is_cuda:
            t = g.detach().to(torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
            self._sum = t if self._sum is None else self._sum + t
            return
        cur = torch.cuda.current_stream(g.device)
        side = self._streams.get(g.device)
        if side is None:
            side = self._streams[g.device] = torch.cuda.Stream(g.device, priority=-1)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            t = g.detach().to(torch.float64)
            # blocking form: `side` (not the compute stream) waits for NCCL
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
            self._sum = t if self._sum is None else self._sum + t
        g.record_stream(side)

    def result(self) -> Optional[torch.Tensor]:
        """The fp64 sum of every push since the last call (None if none), valid
        on the caller's current stream."""
        s, self._sum = self._sum, None
        if s is not None and s.is_cuda:
            cur = torch.cuda.current_stream(s.device)
            side = self._streams.get(s.device)
            if side is not None:
                cur.wait_stream(side)
            s.record_stream(cur)
        return s

    def accumulate_into(self, tau: torch.Tensor) -> None:
        """Adds the pending sum to ``tau.grad`` (creating it) in tau's dtype."""
        s = self.result()
        if s is None:
            return
        s = s.to(tau.dtype).reshape(tau.shape)
        if tau.grad is None:
            tau.grad = s
        else:
            tau.grad.add_(s)


class _SumTauGrad(torch.autograd.Function):
    """Identity on tau whose backward sums the gradient over the process group
    (fp64): inline (the summed gradient flows on through autograd) or, with a
    TauGradReducer, deferred to the reducer (autograd then sees no gradient for
    tau: request it with ``allow_unused=True`` in ``torch.autograd.grad``)."""

    @staticmethod
    def forward(ctx, tau, group, reducer):
        ctx.group = group
        ctx.reducer = reducer
        return tau.view_as(tau)

    @staticmethod
    def backward(ctx, g):
        import torch.distributed as dist

        if ctx.reducer is not None:
            ctx.reducer.push(g)
            return None, None, None
        t = g.to(torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=ctx.group)
        return t.to(g.dtype), None, None


def share_tau(tau: torch.Tensor, group=None, reducer: Optional[TauGradReducer] = None) -> torch.Tensor:
    """tau as seen by this rank's slices: its gradient becomes the sum over the
    process group, inline or through ``reducer`` (see TauGradReducer). Without an
    initialised process group it is tau itself."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return tau
    return _SumTauGrad.apply(tau, group, reducer)


def sharded_flash_pn_fir_tau_attention(q: torch.Tensor, k_tilde: torch.Tensor, v: torch.Tensor,
                                       score_tau: torch.Tensor, scale: Optional[float] = None,
                                       gamma: Optional[float] = 0.5, causal_mask: bool = True, group=None,
                                       attention: Optional[Callable] = None,
                                       reducer: Optional[TauGradReducer] = None) -> torch.Tensor:
    """flash_pn_fir_tau_attention on this rank's [1, S, N, d] shard (see
    shard_bh) with tau's gradient summed over `group`.

    `attention` defaults to the CUDA operator; it takes the reference's
    argument list (q, k_tilde, v, score_tau, scale, gamma, causal_mask).
    With `reducer`, tau's gradient is summed off the critical path (see
    TauGradReducer) instead of inside this backward.
    """
    if attention is None:
        from .pnfirtau_ops import flash_pn_fir_tau_attention as attention
    return attention(q, k_tilde, v, share_tau(score_tau, group, reducer), scale, gamma, causal_mask)
