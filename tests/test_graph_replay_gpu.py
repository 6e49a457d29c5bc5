"""The operator captured in a CUDA graph and replayed: the port of the reference's
graph-replay determinism check (experiments/exp4c_cuda_graphs.py:161-175, which
compares the input gradients of two replays of the captured step).

flash_pn_fir_tau_attention fwd+bwd (bf16, config-3-like quiet regime) is captured
once; replays on the captured inputs, and on new values copied into them, are
compared with eager calls. With deterministic=True every replay equals the
eager deterministic call bit for bit; the default backward's dQ accumulation
order varies between runs, so there the gradients agree to fp32 rounding."""
import pytest
import torch

import paper_01_anti_decoy_pnfirtau_b200 as P
from conftest import rel_l2
from paper_01_anti_decoy_pnfirtau_b200.pnfirtau_ops import check_device_status

pytestmark = pytest.mark.gpu


def _inputs(seed, device, B=2, H=4, N=1024, D=64):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=g)
    quiet = torch.rand(B, H, N // 64, generator=g) < 0.5
    q = q * torch.where(quiet, 0.05, 1.0).repeat_interleave(64, dim=-1)[..., None]
    k, v, do = (torch.randn(B, H, N, D, generator=g) for _ in range(3))
    return [t.to(device, torch.bfloat16) for t in (q, k, v, do)]


def _step(q, k, v, do, tau, deterministic):
    out = P.flash_pn_fir_tau_attention(q, k, v, tau, deterministic=deterministic)
    return (out, *torch.autograd.grad(out, (q, k, v, tau), do))


@pytest.mark.parametrize("deterministic", [False, True], ids=["default", "deterministic"])
def test_operator_graph_replay(cuda, deterministic):
    q0, k0, v0, do0 = _inputs(11, cuda)
    q, k, v = (t.clone().requires_grad_(True) for t in (q0, k0, v0))
    do = do0.clone()
    tau = torch.tensor(0.5, device=cuda, requires_grad=True)
    side = torch.cuda.Stream(cuda)
    side.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(side):
        for _ in range(2):
            _step(q, k, v, do, tau, deterministic)
    torch.cuda.current_stream(cuda).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static = _step(q, k, v, do, tau, deterministic)
    runs = []
    for _ in range(2):
        graph.replay()
        torch.cuda.synchronize()
        runs.append([t.detach().clone() for t in static])
    check_device_status(cuda)
    eager = [t.detach() for t in _step(q, k, v, do, tau, deterministic)]
    names = ("out", "dq", "dk", "dv", "dtau")
    for n, a, b, e in zip(names, runs[0], runs[1], eager):
        assert torch.equal(a, b) or (not deterministic and rel_l2(a, b) < 1e-3), (n, "replay vs replay")
        if deterministic:
            assert torch.equal(a, e), (n, "replay vs eager")
        else:
            assert rel_l2(a, e) < 1e-3, (n, rel_l2(a, e))
    # new values in the captured inputs: the replay follows them
    q1, k1, v1, do1 = _inputs(12, cuda)
    with torch.no_grad():
        q.copy_(q1), k.copy_(k1), v.copy_(v1), do.copy_(do1)
    graph.replay()
    torch.cuda.synchronize()
    eager = [t.detach() for t in _step(q, k, v, do, tau, deterministic)]
    for n, a, e in zip(names, static, eager):
        if deterministic:
            assert torch.equal(a, e), n
        else:
            assert rel_l2(a, e) < 1e-3, (n, rel_l2(a, e))
    del graph
