"""lm.GraphedTrainStep: the config-4 training step captured in one CUDA graph
(the reference's exp4c technique, experiments/exp4c_cuda_graphs.py, applied to
the whole step), on one GPU against the eager step, and data parallel on two
GPUs (child processes over NCCL) against one process on the concatenated
batch. The two-GPU case is skipped where fewer than two GPUs are visible."""
import os
import socket

import pytest
import torch

from conftest import rel_l2
from paper_01_anti_decoy_pnfirtau_b200.lm import GraphedTrainStep, LMConfig, PnFirLM, lm_loss, make_optimizer, train_step

pytestmark = pytest.mark.gpu

CFG = LMConfig(max_seq=128)


def _batches(device, n, B=4, seed=5):
    g = torch.Generator(device=device).manual_seed(seed)
    return [torch.randint(0, CFG.vocab, (B, CFG.max_seq), device=device, generator=g) for _ in range(n)]


def test_graphed_step_tracks_eager(cuda):
    batches = _batches(cuda, 3)
    torch.manual_seed(1)
    m_graph = PnFirLM(CFG).to(cuda)
    m_eager = PnFirLM(CFG).to(cuda)
    m_eager.load_state_dict(m_graph.state_dict())
    before = [p.detach().clone() for p in m_graph.parameters()]
    graphed = GraphedTrainStep(m_graph, make_optimizer(m_graph, capturable=True), batches[0])
    # construction (warm-up + capture) leaves the weights as they were
    for p, b in zip(m_graph.parameters(), before):
        assert torch.equal(p.detach(), b)
    opt_e = make_optimizer(m_eager)
    lg = [float(graphed.step(b)) for b in batches]
    le = [float(train_step(m_eager, opt_e, b)) for b in batches]
    for a, b in zip(lg, le):
        assert abs(a - b) < 2e-3 * abs(b), (lg, le)
    for (n, p), q in zip(m_graph.named_parameters(), m_eager.parameters()):
        assert rel_l2(p.detach(), q.detach()) < 1e-3, n
    graphed.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        batches = _batches(dev, 2 * world, seed=11)
        mine = batches[rank::world]
        torch.manual_seed(100 + rank)  # different inits: the constructor broadcasts rank 0's weights
        model = PnFirLM(CFG).to(dev)
        graphed = GraphedTrainStep(model, make_optimizer(model, capturable=True), mine[0],
                                   group=dist.group.WORLD)
        graphed.step(mine[0])
        torch.cuda.synchronize()
        grads = [p.grad.detach().clone() for p in graphed.params]
        params = [p.detach().clone() for p in graphed.params]
        torch.save({"grads": [g.cpu() for g in grads], "params": [p.cpu() for p in params]},
                   os.path.join(out_dir, f"rank{rank}.pt"))
        graphed.close()
        del graphed
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_graphed_step_data_parallel_two_gpus(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    res = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    # every rank applied the same averaged update
    for a, b in zip(res[0]["params"], res[1]["params"]):
        assert torch.equal(a, b)
    # the averaged, clipped gradient equals one process's on the concatenated batch
    dev = torch.device("cuda", 0)
    batches = _batches(dev, 2 * world, seed=11)
    torch.manual_seed(100)
    model = PnFirLM(CFG).to(dev)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = lm_loss(model, torch.cat([batches[0], batches[1]]))
    loss.backward()
    torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
    for g, p in zip(res[0]["grads"], [p for p in model.parameters() if p.requires_grad]):
        assert rel_l2(g.to(dev), p.grad) < 2e-2
