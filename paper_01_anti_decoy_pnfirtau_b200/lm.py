"""Pre-LN decoder LM with pn_fir_tau attention in every layer - the caller of
the operator in the reference's language-model experiments
(experiments/exp4_wikitext2_lm.py:183-259, ``Block`` and ``WikiLM``;
experiments/exp4f_scaleout.py:260-271 for the D=256 / N=512 shape).

Token embedding + learned positions -> n_layers x Block(x + attn(ln1 x);
x + ffn(ln2 x)) -> ln_f -> head tied to the embedding.

With ``fused_step_ops`` (default) the step's non-attention work runs on this
library's kernels (lm_ops): each residual add fused with the LayerNorm after
it (output written in the autocast dtype), the MLP's GELU backward fused with
its bias gradients, the weight gradients of the projections and the MLP from a
split-K tcgen05 GEMM, and the head's loss and logit gradient in one pass over
the logits. With ``fused_step_ops=False`` the blocks are nn.LayerNorm, nn.Linear,
nn.GELU and F.cross_entropy. Parameters and state_dict keys are the same either
way.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .lm_ops import Bf16Casts, LayerNorm, Linear, add_layer_norm, head_cross_entropy, mlp_gelu
from .pnfirtau_attention import PnFirConfig, PnFirTauFlashMHA, PnFirTauMHA, PnFirTauTritonMHA

_VARIANTS = {"pn_fir_tau": PnFirTauMHA, "pn_fir_tau_triton": PnFirTauTritonMHA, "pn_fir_tau_flash": PnFirTauFlashMHA}


@dataclass(frozen=True)
class LMConfig:
    vocab: int = 33278
    d_model: int = 256
    n_heads: int = 4
    n_layers: int = 6
    d_ff: int = 1024
    max_seq: int = 512
    dropout: float = 0.0
    p: float = 10.0
    silence_gamma: float | None = 0.5
    tau_init: float = 0.0
    fir_k: int = 7


class Block(nn.Module):
    """exp4_wikitext2_lm.py:183-200."""

    def __init__(self, d_model: int, attn: nn.Module, dropout: float, d_ff: int, norm=nn.LayerNorm):
        super().__init__()
        self.ln1 = norm(d_model)
        self.attn = attn
        self.ln2 = norm(d_model)
        self.ffn = nn.Sequential(nn.Linear(d_model, d_ff), nn.GELU(), nn.Linear(d_ff, d_model), nn.Dropout(dropout))
        self.drop = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self.drop(self.attn(self.ln1(x)))
        return x + self.ffn(self.ln2(x))


class PnFirLM(nn.Module):
    """exp4_wikitext2_lm.py:203-247 (``WikiLM``) with a pn_fir_tau variant."""

    def __init__(self, cfg: LMConfig = LMConfig(), variant: str = "pn_fir_tau_flash", fused_step_ops: bool = True):
        super().__init__()
        self.cfg = cfg
        self.variant = variant
        self.fused_step_ops = fused_step_ops
        norm = LayerNorm if fused_step_ops else nn.LayerNorm
        self.embed = nn.Embedding(cfg.vocab, cfg.d_model)
        self.pos = nn.Embedding(cfg.max_seq, cfg.d_model)
        self.drop = nn.Dropout(cfg.dropout)
        acfg = PnFirConfig(d_model=cfg.d_model, n_heads=cfg.n_heads, p=cfg.p, silence_gamma=cfg.silence_gamma,
                           tau_init=cfg.tau_init, fir_k=cfg.fir_k, dropout=cfg.dropout, causal_mask=True, bias=False)
        cls = _VARIANTS[variant]
        self.blocks = nn.ModuleList(
            Block(cfg.d_model, cls(acfg), cfg.dropout, cfg.d_ff, norm) for _ in range(cfg.n_layers))
        self.ln_f = norm(cfg.d_model)
        if fused_step_ops:
            # the attention's projections with the library's weight-gradient GEMM (same parameters)
            for blk in self.blocks:
                for name in ("qkv", "out"):
                    setattr(blk.attn, name, Linear.sharing(getattr(blk.attn, name)))
        self.head = nn.Linear(cfg.d_model, cfg.vocab, bias=False)
        self.head.weight = self.embed.weight
        self._casts: Bf16Casts | None = None  # bf16 copies of the GEMM parameters (_step_casts)

    def forward(self, idx: torch.Tensor, for_loss: bool = False, targets: torch.Tensor | None = None) -> torch.Tensor:
        """Logits ``[B, N, vocab]``. ``for_loss``: the logits the next-token loss
        scores, ``[B, N-1, vocab_pad]`` for positions 0..N-2, with the vocabulary
        padded to a multiple of 64 (the padded logits are -inf, so they add nothing
        to a softmax): the head GEMM then has 16-byte aligned rows and no slice
        copy of the logits is needed. ``targets`` (``[B, N-1]``, the ids of
        positions 1..N-1): the mean next-token cross-entropy of positions 0..N-2
        instead of logits (one kernel pass over the logits with
        ``fused_step_ops``, else F.cross_entropy)."""
        B, N = idx.shape
        pos = torch.arange(N, device=idx.device).unsqueeze(0)
        h = self.drop(self.embed(idx) + self.pos(pos))
        casts = self._step_casts(idx.device)
        h = self._trunk_fused(h, casts) if self.fused_step_ops else self._trunk(h)
        if targets is not None:
            if self.fused_step_ops:
                return head_cross_entropy(h[:, :-1], self.head.weight, targets, casts=casts)
            logits = self._padded_logits(h)
            return nn.functional.cross_entropy(logits.reshape(-1, logits.size(-1)), targets.reshape(-1))
        if not for_loss:
            return self.head(h)
        return self._padded_logits(h)

    def _trunk(self, h: torch.Tensor) -> torch.Tensor:
        for blk in self.blocks:
            h = blk(h)
        return self.ln_f(h)

    def _step_casts(self, dev: torch.device) -> Bf16Casts | None:
        """With the fused step ops under bf16 CUDA autocast: the bf16 copies of
        every GEMM weight and bias (the head's padded to a multiple of 64 rows),
        refreshed by one kernel launch, which the GEMMs of this forward and its
        backward use instead of one cast per GEMM. None otherwise."""
        if not (self.fused_step_ops and dev.type == "cuda" and torch.is_autocast_enabled("cuda")
                and torch.get_autocast_dtype("cuda") == torch.bfloat16):
            return None
        if self._casts is None:
            lins = [lin for blk in self.blocks for lin in (blk.attn.qkv, blk.attn.out)]
            params = [t for lin in lins for t in (lin.weight, lin.bias)]
            params += [t for blk in self.blocks for t in (blk.ffn[0].weight, blk.ffn[0].bias, blk.ffn[2].weight,
                                                          blk.ffn[2].bias)]
            params.append(self.head.weight)
            if torch.cuda.is_current_stream_capturing() or any(
                    t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.device != dev)
                    for t in params):
                return None
            vp = (self.cfg.vocab + 63) // 64 * 64
            self._casts = Bf16Casts(params, padded={id(self.head.weight): vp})
            for lin in lins:
                lin.casts = self._casts
        self._casts.refresh()
        return self._casts

    def _trunk_fused(self, h: torch.Tensor, casts: Bf16Casts | None = None) -> torch.Tensor:
        """The same blocks with every residual add fused into the LayerNorm
        that follows it (the MLP's add into the next block's ln1, the last one
        into ln_f) and the MLP on mlp_gelu; returns ln_f's output."""
        blocks = list(self.blocks)
        a = blocks[0].ln1(h)
        for i, blk in enumerate(blocks):
            att = blk.drop(blk.attn(a))
            ln2 = blk.ln2
            h, b = add_layer_norm(h, att, ln2.normalized_shape, ln2.weight, ln2.bias, ln2.eps)
            f = blk.ffn[3](mlp_gelu(b, blk.ffn[0], blk.ffn[2], casts))
            nxt = blocks[i + 1].ln1 if i + 1 < len(blocks) else self.ln_f
            h, a = add_layer_norm(h, f, nxt.normalized_shape, nxt.weight, nxt.bias, nxt.eps)
        return a

    def _padded_logits(self, h: torch.Tensor) -> torch.Tensor:
        V = self.cfg.vocab
        Vp = (V + 63) // 64 * 64
        w = F.pad(self.head.weight, (0, 0, 0, Vp - V))
        logits = F.linear(h[:, :-1], w)
        if Vp > V:
            logits[..., V:] = float("-inf")
        return logits

    def param_count(self) -> int:
        return sum(p.numel() for p in {id(p): p for p in self.parameters()}.values())


def lm_loss(model: nn.Module, idx: torch.Tensor) -> torch.Tensor:
    """Next-token cross-entropy of positions 0..N-2 scored on the shifted ids
    (exp4_wikitext2_lm.py:714-719, which slices the logits of all N positions:
    the same loss)."""
    return model(idx, targets=idx[:, 1:])


def train_step(model: nn.Module, opt: torch.optim.Optimizer, idx: torch.Tensor, clip: float = 1.0) -> torch.Tensor:
    """One bf16-autocast step: loss, backward, clip_grad_norm_(1.0), AdamW
    (exp4_wikitext2_lm.py:712-729). Returns the loss tensor (no host sync)."""
    opt.zero_grad(set_to_none=True)
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        loss = lm_loss(model, idx)
    loss.backward()
    torch.nn.utils.clip_grad_norm_(model.parameters(), clip)
    opt.step()
    return loss.detach()


def make_optimizer(model: nn.Module, lr: float = 3e-4, capturable: bool = False) -> torch.optim.Optimizer:
    """AdamW(betas=(0.9, 0.95), weight_decay=0.1) as exp4_wikitext2_lm.py:684-689,
    with PyTorch's single-kernel (fused) implementation of the same update when
    the parameters are on a CUDA device."""
    fused = all(p.is_cuda for p in model.parameters())
    return torch.optim.AdamW(model.parameters(), lr=lr, betas=(0.9, 0.95), weight_decay=0.1, fused=fused,
                             capturable=capturable)


class GraphedTrainStep:
    """``train_step`` captured once in a CUDA graph and replayed (the technique
    of the reference's exp4c, experiments/exp4c_cuda_graphs.py, applied to the
    whole training step): bf16-autocast loss, backward, the gradient average
    over a data-parallel group, clip_grad_norm_ and the optimizer step run as
    one graph launch; ``step(idx)`` copies the batch into the captured input.

    Data parallelism without DDP's hooks: after the backward every gradient is
    gathered into one flat fp32 buffer, averaged across ``group`` by one NCCL
    all-reduce inside the graph, and copied back. The ranks' weights start
    equal (rank 0's are broadcast at construction).

    ``opt`` must be capturable (``make_optimizer(model, capturable=True)``).
    Construction runs ``warmup`` steps on ``example_idx`` (a side stream; the
    optimizer creates its state and NCCL its communicator there), captures a
    step, and then restores the parameters and the optimizer state, so it
    leaves the model as it found it. The graph's NCCL call must be released
    (``close()``) before the process group is destroyed."""

    def __init__(self, model: nn.Module, opt: torch.optim.Optimizer, example_idx: torch.Tensor, group=None,
                 clip: float = 1.0, warmup: int = 3):
        import torch.distributed as dist

        self.model, self.opt, self.clip, self.group = model, opt, clip, group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.params = [p for p in model.parameters() if p.requires_grad]
        dev = self.params[0].device
        if self.world > 1:
            src = dist.get_global_rank(group, 0)
            with torch.no_grad():
                for p in self.params:
                    dist.broadcast(p, src=src, group=group)
        self.sizes = [p.numel() for p in self.params]
        self.flat = torch.empty(sum(self.sizes), dtype=torch.float32, device=dev) if self.world > 1 else None
        # per-parameter views of the flat buffer: gradients are gathered into it and
        # scattered back with multi-tensor copies (torch.cat of the 77 gradients runs the
        # 34 MB embedding gradient on few blocks: 179 us against ~15 us)
        self.flat_views = ([t.view_as(p) for t, p in zip(self.flat.split(self.sizes), self.params)]
                           if self.world > 1 else None)
        self.idx = example_idx.detach().clone()
        saved_p = [p.detach().clone() for p in self.params]
        saved_s = {id(p): {k: (v.clone() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()}
                   for p in self.params if p in opt.state}
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                opt.zero_grad(set_to_none=True)
                self._step()
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        opt.zero_grad(set_to_none=True)
        with torch.cuda.graph(self.graph):
            self.loss = self._step()
        torch.cuda.synchronize(dev)
        # back to the state before construction
        with torch.no_grad():
            for p, s in zip(self.params, saved_p):
                p.copy_(s)
            for p in self.params:
                st = opt.state.get(p, {})
                old = saved_s.get(id(p))
                for k, v in st.items():
                    if torch.is_tensor(v):
                        v.copy_(old[k]) if old is not None and k in old else v.zero_()

    def _step(self) -> torch.Tensor:
        import torch.distributed as dist

        with torch.autocast(device_type="cuda", dtype=torch.bfloat16, cache_enabled=False):
            loss = lm_loss(self.model, self.idx)
        loss.backward()
        if self.world > 1:
            grads = [p.grad for p in self.params]
            torch._foreach_copy_(self.flat_views, grads)
            dist.all_reduce(self.flat, op=dist.ReduceOp.AVG, group=self.group)
            torch._foreach_copy_(grads, self.flat_views)
        torch.nn.utils.clip_grad_norm_(self.params, self.clip)
        self.opt.step()
        return loss.detach()

    def step(self, idx: torch.Tensor) -> torch.Tensor:
        """One replayed training step on ``idx``; returns the loss tensor (no host sync)."""
        self.idx.copy_(idx)
        self.graph.replay()
        return self.loss

    def close(self) -> None:
        self.graph = None
