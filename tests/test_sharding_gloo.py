"""Multi-rank layout of the operator on CPU: world_size-2 `gloo` process
groups, with the CPU oracle standing in for the CUDA attention (the sharding
layer takes the attention callable as an argument).

Checks that the B*H partition covers every slice once, that each rank's
outputs and q/k/v gradients equal the matching slices of a single-process
run, and that tau's gradient is the all-reduced sum of the ranks' partials.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import pnfirtau_oracle as O
from paper_01_anti_decoy_pnfirtau_b200.sharding import (
    TauGradReducer,
    bh_range,
    shard_bh,
    share_tau,
    sharded_flash_pn_fir_tau_attention,
    unshard_bh,
)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("B,H,world", [(1, 1, 1), (2, 3, 2), (3, 5, 4), (1, 2, 8), (8, 8, 8), (4, 4, 3)])
def test_bh_range_covers_once(B, H, world):
    seen = []
    for r in range(world):
        lo, hi = bh_range(B, H, r, world)
        assert 0 <= lo <= hi <= B * H
        seen.extend(range(lo, hi))
    assert seen == list(range(B * H))
    sizes = [bh_range(B, H, r, world)[1] - bh_range(B, H, r, world)[0] for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


def test_bh_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        bh_range(2, 2, 2, 2)
    with pytest.raises(ValueError):
        bh_range(2, 2, 0, 0)


def test_shard_unshard_roundtrip():
    x = torch.arange(3 * 5 * 4 * 2, dtype=torch.float32).reshape(3, 5, 4, 2)
    parts = [shard_bh(x, r, 4) for r in range(4)]
    assert sum(p.shape[1] for p in parts) == 15
    assert torch.equal(unshard_bh(parts, 3, 5), x)


def test_share_tau_without_group_is_identity():
    t = torch.tensor(0.25, requires_grad=True)
    assert share_tau(t) is t


def _oracle_attention(q, k, v, tau, scale, gamma, causal):
    return O.pn_fir_tau_attention(q, k, v, tau, scale=scale, gamma=gamma, causal=causal)


def _inputs(B, H, N, D, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn(B, H, N, D, generator=g, dtype=torch.float64) for _ in range(4))
    return q, k, v, do


def _worker(rank, world, port, B, H, N, D, tau0, result_q, deferred=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        q, k, v, do = _inputs(B, H, N, D, seed=7)
        ql, kl, vl, dol = (shard_bh(t, rank, world).clone().requires_grad_(True) for t in (q, k, v, do))
        tau = torch.tensor(tau0, dtype=torch.float64, requires_grad=True)
        reducer = TauGradReducer() if deferred else None
        out = sharded_flash_pn_fir_tau_attention(ql, kl, vl, tau, None, 0.5, True, attention=_oracle_attention,
                                                 reducer=reducer)
        out.backward(dol.detach())
        if deferred:
            assert tau.grad is None  # nothing reaches tau until the reducer is finalised
            # a second backward accumulates a second partial sum in the reducer
            out2 = sharded_flash_pn_fir_tau_attention(ql.detach(), kl.detach(), vl.detach(), tau, None, 0.5, True,
                                                      attention=_oracle_attention, reducer=reducer)
            out2.backward(dol.detach())
            assert reducer.pushes == 2
            reducer.accumulate_into(tau)
            assert reducer.result() is None
            tau.grad /= 2
        result_q.put((rank, out.detach(), ql.grad, kl.grad, vl.grad, tau.grad.item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("deferred", [False, True], ids=["inline", "reducer"])
@pytest.mark.parametrize("world", [2])
def test_two_rank_gloo_matches_single_process(world, deferred):
    B, H, N, D, tau0 = 2, 3, 40, 8, 0.1
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, H, N, D, tau0, result_q, deferred))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, *vals = result_q.get(timeout=120)
            results[r] = vals
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)

    q, k, v, do = _inputs(B, H, N, D, seed=7)
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    tr = torch.tensor(tau0, dtype=torch.float64, requires_grad=True)
    ref = O.pn_fir_tau_attention(qr, kr, vr, tr, scale=None, gamma=0.5, causal=True)
    ref.backward(do)

    for i, want in enumerate((ref.detach(), qr.grad, kr.grad, vr.grad)):
        got = unshard_bh([results[r][i] for r in range(world)], B, H)
        torch.testing.assert_close(got, want, rtol=1e-12, atol=1e-12)
    for r in range(world):  # every rank holds the same all-reduced tau gradient
        assert results[r][4] == pytest.approx(tr.grad.item(), rel=1e-12, abs=1e-12)
    # ... which is the sum of the ranks' own partials, not one rank's share
    parts = []
    for r in range(world):
        t = torch.tensor(tau0, dtype=torch.float64, requires_grad=True)
        o = O.pn_fir_tau_attention(*(shard_bh(x, r, world) for x in (q, k, v)), t, scale=None, gamma=0.5,
                                   causal=True)
        o.backward(shard_bh(do, r, world))
        parts.append(t.grad.item())
    assert abs(parts[0]) > 0 and abs(parts[1]) > 0
    assert sum(parts) == pytest.approx(results[0][4], rel=1e-12, abs=1e-12)
