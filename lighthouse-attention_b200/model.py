"""Llama3-style model harness with Lighthouse layers.

The reference trains a 270M Llama3 variant through a torchtitan patch
(lighthouse-attention.patch): flavour at :283-296 (dim 1024, 30 layers,
FFN hidden 1536, 8 heads, 8 KV heads, rope theta 1e4, byte vocabulary 256),
the attention call site at :700-737 (q/k/v after RoPE in (B, S, H, D) go to
the Lighthouse module, its (B, H, S, D) output is transposed back before wo)
and full SDPA attention on layers [0, 1, 28, 29] (:754-766).  torchtitan at
the patched revision is not available here, so this module restates that
architecture in plain PyTorch with the package's Lighthouse layer in the
attention of every other layer.

Data parallelism is plain DDP over NCCL (gradient all-reduce, bucketed and
overlapped with backward by torch).  Context parallelism (the reference's
`*_cp` flavours, PATCH:325-413, with set_cp_info plumbing PATCH:801-816):
every rank holds the load-balanced shard (global chunks r and 2W-1-r) of the
tokens, labels and RoPE positions (PATCH:822-829); Lighthouse layers run
LighthouseCP and the full-attention layers run causal attention over the
all-gathered K/V (cp.py); gradients are averaged over ranks by DDP.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from .library import ops as _ops
from . import cp as _cp
from .lighthouse_selection import (DilatedLighthouseGLAScorer, DilatedLighthouseScorer, LighthouseLocal,
                                   lighthouse_attention)


@dataclass
class ModelArgs:
    """Field names follow the torchtitan TransformerModelArgs the patch extends
    (lighthouse-attention.patch:551-579)."""
    dim: int = 1024
    n_layers: int = 30
    n_heads: int = 8
    n_kv_heads: int = 8
    vocab_size: int = 256
    hidden_dim: int = 1536
    norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    max_seq_len: int = 65536
    use_selection_lighthouse: bool = True
    lighthouse_num_levels: int = 3
    lighthouse_pooling_factor: int = 4
    lighthouse_topk: int = 2048
    lighthouse_scorer: str = "norm"          # "norm" | "dilated" | "gla"  (context parallelism: "norm" only)
    dilation: int = 4
    lighthouse_full_attn_layers: list = field(default_factory=lambda: [0, 1, 28, 29])


def rope_freqs(head_dim: int, seq_len: int, theta: float, device) -> torch.Tensor:
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim))
    t = torch.arange(seq_len, device=device, dtype=torch.float32)
    ang = torch.outer(t, inv)
    return torch.polar(torch.ones_like(ang), ang)          # (S, D/2) complex64


def apply_rope(x: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """x (B, S, H, D); rotation of adjacent pairs as in the Llama3 reference model."""
    xc = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    out = torch.view_as_real(xc * freqs[None, :, None, :]).flatten(-2)
    return out.to(x.dtype)


class _RopeFn(torch.autograd.Function):
    """Fused RoPE of q and k on the GPU (csrc/rope.cu); backward = inverse rotation."""

    @staticmethod
    def forward(ctx, xq, xk, table):
        ctx.save_for_backward(table)
        return _ops.rope_apply(xq.contiguous(), xk.contiguous(), table)

    @staticmethod
    def backward(ctx, gq, gk):
        (table,) = ctx.saved_tensors
        dq, dk = _ops.rope_apply(gq.contiguous(), gk.contiguous(), table, True)
        return dq, dk, None


def rope_qk(xq: torch.Tensor, xk: torch.Tensor, freqs: torch.Tensor):
    """RoPE of q and k: one fused kernel for CUDA tensors, the complex-multiply
    formulation (apply_rope) on the CPU."""
    if xq.is_cuda:
        return _RopeFn.apply(xq, xk, torch.view_as_real(freqs).contiguous())
    return apply_rope(xq, freqs), apply_rope(xk, freqs)


class Attention(nn.Module):
    def __init__(self, args: ModelArgs, layer_id: int):
        super().__init__()
        self.n_heads = args.n_heads
        self.head_dim = args.dim // args.n_heads
        if args.n_kv_heads != args.n_heads:
            raise NotImplementedError("Lighthouse selection path requires n_kv_heads == n_heads")
        self.wq = nn.Linear(args.dim, args.n_heads * self.head_dim, bias=False)
        self.wk = nn.Linear(args.dim, args.n_heads * self.head_dim, bias=False)
        self.wv = nn.Linear(args.dim, args.n_heads * self.head_dim, bias=False)
        self.wo = nn.Linear(args.n_heads * self.head_dim, args.dim, bias=False)
        self.lighthouse = args.use_selection_lighthouse and layer_id not in args.lighthouse_full_attn_layers
        self.L, self.p, self.k = args.lighthouse_num_levels, args.lighthouse_pooling_factor, args.lighthouse_topk
        # scorer from the config (PATCH:601-637); the GLA scorer adds a per-token
        # gate projection, gk = logsigmoid(wg(x)) / 16 (PATCH:662-664, 708-710)
        self.scorer_name = (args.lighthouse_scorer or "norm").lower()
        self.layer = None
        if self.scorer_name not in ("norm", "dilated", "gla"):
            raise ValueError(f"unknown lighthouse_scorer {args.lighthouse_scorer!r}")
        if self.lighthouse and self.scorer_name != "norm":
            kw = dict(dilation=args.dilation, pooling_factor=self.p, levels=self.L)
            scorer = (DilatedLighthouseGLAScorer(self.head_dim, **kw) if self.scorer_name == "gla"
                      else DilatedLighthouseScorer(head_dim=self.head_dim, **kw))
            self.layer = LighthouseLocal(None, scorer, num_levels=self.L, pooling_factor=self.p, topk=self.k)
            if self.scorer_name == "gla":
                self.wg = nn.Linear(args.dim, args.n_heads, bias=True)
                self.gate_logit_normalizer = 16

    def forward(self, x, freqs, cp_info=None):
        B, S, _ = x.shape
        xq = self.wq(x).view(B, S, self.n_heads, self.head_dim)
        xk = self.wk(x).view(B, S, self.n_heads, self.head_dim)
        xv = self.wv(x).view(B, S, self.n_heads, self.head_dim)
        xq, xk = rope_qk(xq, xk, freqs)
        if cp_info is not None:
            rank, world, group = cp_info
            if self.layer is not None:
                raise ValueError(f"lighthouse_scorer={self.scorer_name!r} is not supported under context "
                                 "parallelism (PATCH:610-615); use 'norm'")
            if self.lighthouse:
                out = _cp.lighthouse_cp_forward(xq, xk, xv, self.L, self.p, self.k, rank, world, group)
            else:
                out = _cp.full_cp_attention(xq, xk, xv, rank, world, group)
        elif self.layer is not None:
            gk = F.logsigmoid(self.wg(x).float()) / self.gate_logit_normalizer if self.scorer_name == "gla" else None
            out = self.layer(xq, xk, xv, gk=gk)
        elif self.lighthouse:
            out = lighthouse_attention(xq, xk, xv, self.L, self.p, self.k)          # (B, H, S, D)
        else:
            out = F.scaled_dot_product_attention(xq.transpose(1, 2), xk.transpose(1, 2), xv.transpose(1, 2),
                                                 is_causal=True)
        return self.wo(out.transpose(1, 2).reshape(B, S, -1))


class FeedForward(nn.Module):
    def __init__(self, dim: int, hidden: int):
        super().__init__()
        self.w1 = nn.Linear(dim, hidden, bias=False)
        self.w2 = nn.Linear(hidden, dim, bias=False)
        self.w3 = nn.Linear(dim, hidden, bias=False)

    def forward(self, x):
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class Block(nn.Module):
    def __init__(self, args: ModelArgs, layer_id: int):
        super().__init__()
        self.attention_norm = nn.RMSNorm(args.dim, eps=args.norm_eps)
        self.attention = Attention(args, layer_id)
        self.ffn_norm = nn.RMSNorm(args.dim, eps=args.norm_eps)
        self.feed_forward = FeedForward(args.dim, args.hidden_dim)

    def forward(self, x, freqs, cp_info=None):
        h = x + self.attention(_to_compute_dtype(self.attention_norm(x)), freqs, cp_info)
        return h + self.feed_forward(_to_compute_dtype(self.ffn_norm(h)))


def _to_compute_dtype(t):
    """Under autocast, cast a normalised fp32 activation to the autocast dtype
    once.  Autocast would otherwise cast it separately for every projection that
    reads it (wq, wk, wv; w1, w3), with one more conversion per projection in
    backward.  The projections see the same bf16 values either way."""
    if t.is_cuda and torch.is_autocast_enabled("cuda"):
        return t.to(torch.get_autocast_dtype("cuda"))
    return t


class Transformer(nn.Module):
    def __init__(self, args: ModelArgs):
        super().__init__()
        self.args = args
        self.tok_embeddings = nn.Embedding(args.vocab_size, args.dim)
        self.layers = nn.ModuleList(Block(args, i) for i in range(args.n_layers))
        self.norm = nn.RMSNorm(args.dim, eps=args.norm_eps)
        self.output = nn.Linear(args.dim, args.vocab_size, bias=False)
        self._freqs = None
        self.cp_info = None          # (rank, world_size, group) once set_cp_info is called

    def set_cp_info(self, rank: int, world_size: int, group) -> None:
        """Context-parallel mode (PATCH:801-816): forward then takes this rank's
        load-balanced token shard and applies RoPE at its global positions."""
        self.cp_info = (rank, world_size, group) if world_size > 1 else None

    def init_weights(self, seed: int = 0):
        g = torch.Generator(device="cpu").manual_seed(seed)
        for name, p in self.named_parameters():
            with torch.no_grad():
                if p.dim() == 2:
                    p.copy_(torch.randn(p.shape, generator=g) * 0.02)
                elif name.endswith("wg.bias"):                # gate projection bias (PATCH:687-689)
                    p.zero_()

    def forward(self, tokens):
        B, S = tokens.shape
        W = self.cp_info[1] if self.cp_info else 1
        S_glob = S * W
        if self._freqs is None or self._freqs.shape[0] < S_glob or self._freqs.device != tokens.device:
            self._freqs = rope_freqs(self.args.dim // self.args.n_heads, max(S_glob, 1), self.args.rope_theta,
                                     tokens.device)
        freqs = self._freqs[:S_glob]
        if self.cp_info:
            freqs = _cp.shard_sequence(freqs, self.cp_info[0], W, dim=0)   # global positions of the shard
        h = self.tok_embeddings(tokens)
        for layer in self.layers:
            h = layer(h, freqs, self.cp_info)
        return self.output(self.norm(h))


def num_params(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())


def train_step(model, optimizer, tokens: torch.Tensor) -> torch.Tensor:
    """One next-byte-prediction step on tokens (B, S+1): inputs are the first S
    bytes, labels the last S.  bf16 autocast over fp32 master weights (the
    reference trains with bf16 mixed precision).  In context-parallel mode
    (model.set_cp_info) every rank passes the same global tokens and trains on
    its load-balanced shard of inputs and labels; the returned loss is this
    rank's shard mean.  Returns the loss tensor."""
    inputs, labels = tokens[:, :-1], tokens[:, 1:]
    core = model.module if hasattr(model, "module") else model
    if core.cp_info:
        rank, W, _ = core.cp_info
        inputs = _cp.shard_sequence(inputs, rank, W, dim=1)
        labels = _cp.shard_sequence(labels, rank, W, dim=1)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits = model(inputs)
    loss = F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), labels.reshape(-1))
    loss.backward()
    optimizer.step()
    optimizer.zero_grad(set_to_none=True)
    return loss.detach()
