"""Drop-in for the reference module ``lighthouse_selection`` (norm scorer path).

Exports the names the torchtitan patch imports (lighthouse-attention.patch:591-598)
with the reference's constructor arguments and forward contracts
(src/lighthouse_selection.py of the reference, cited as SEL):

  DialatedLighthouseNormScorer / DialatedLighthouseNormScorerCP   SEL:578-616, 943-982
  LighthouseLocal                                                  SEL:772-825
  LighthouseCP (+ set_cp_info)                                     SEL:985-1054
  scatter_to_base_sequence                                         SEL:758-770
  compute_output_indices_selection                                 SEL:338-354
  DilatedLighthouseScorer, DilatedLighthouseGLAScorer              SEL:618, 692 (not provided:
                                                                   constructing works, forward raises)

``LighthouseLocal.forward`` runs the whole layer as one autograd node over
the sm_100a kernels: pyramid + scores -> selection -> gather -> tcgen05
causal attention -> deterministic fan-out scatter, and in backward the
scatter adjoint -> attention backward -> un-pool.  No Triton, no fallback.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import _native
from ._native import LighthouseShapeError
from .library import ops as _ops
from .lighthouse_selection_cuda import (LighthouseSelectionQkKqChunkedTopkNvrtc,  # noqa: F401
                                        compute_output_indices_selection)

__all__ = [
    "DialatedLighthouseNormScorer", "DialatedLighthouseNormScorerCP", "DilatedLighthouseScorer",
    "DilatedLighthouseGLAScorer", "LighthouseLocal", "LighthouseCP", "scatter_to_base_sequence",
    "compute_output_indices_selection", "LighthouseSelectionQkKqChunkedTopkNvrtc", "lighthouse_attention",
]


# ----------------------------------------------------------------------------- scorer
class _PyramidFn(torch.autograd.Function):
    """Scorer as an autograd node: forward = pyramid kernel; backward = un-pool
    kernel with the identity slot map (every pyramid entry is its own slot)."""

    @staticmethod
    def forward(ctx, xq, xk, xv, L, p):
        B, S, H, D = xq.shape
        pq, pk, pv, sqk, skq = _ops.pyramid_score(xq, xk, xv, L, p)
        cat = lambda x, pooled: torch.cat([x.transpose(1, 2), pooled], dim=2)
        ctx.L, ctx.p, ctx.S = L, p, S
        ctx.mark_non_differentiable(sqk, skq)
        return sqk.to(xq.dtype), skq.to(xq.dtype), cat(xq, pq), cat(xk, pk), cat(xv, pv)

    @staticmethod
    def backward(ctx, _gs1, _gs2, gq, gk, gv):
        given = next(g for g in (gq, gk, gv) if g is not None)
        B, H, S_tot = given.shape[:3]
        gq, gk, gv = (torch.zeros_like(given) if g is None else g for g in (gq, gk, gv))
        ident = torch.arange(S_tot, dtype=torch.int32, device=given.device).expand(B, H, S_tot).contiguous()
        dq, dk, dv = _ops.unpool_bwd(gq, gk, gv, ident, ctx.S, ctx.L, ctx.p)
        return dq, dk, dv, None, None


class DialatedLighthouseNormScorer(nn.Module):
    """Norm scorer + pyramid (SEL:578-616).

    forward(xq, xk, xv) with (B, S, H, D) inputs returns
    (scores_qk_cat, scores_kq_cat, xq_cat, xk_cat, xv_cat): scores (B, H, S_tot)
    in the input dtype, pyramids (B, H, S_tot, D).  The scores carry no
    gradient (the reference only ever uses them under no_grad, SEL:794).
    """

    def __init__(self, pooling_factor: int = 4, levels: int = 3):
        super().__init__()
        self.pooling_factor = pooling_factor
        self.levels = levels

    def forward(self, xq, xk, xv):
        return _PyramidFn.apply(xq, xk, xv, self.levels, self.pooling_factor)


class DialatedLighthouseNormScorerCP(DialatedLighthouseNormScorer):
    """CP twin of the norm scorer (SEL:943-982); identical computation."""

    def __init__(self, pooling_factor: int = 4, levels: int = 3):
        super().__init__(pooling_factor, levels)
        self._checked = False


def _causal_attention(q, k, v):
    """(B, H, S, D) causal attention on this package's tcgen05 kernel.  It is
    defined for bf16 CUDA tensors with D = 128 only; anything else raises (a
    caller that wants another attention passes it as ``attention=``)."""
    if not (q.dtype == torch.bfloat16 and q.shape[-1] == 128 and q.is_cuda):
        raise LighthouseShapeError(
            "dilated scorer: the default attention needs bf16 CUDA tensors with head_dim 128 "
            f"(got {q.dtype}, head_dim {q.shape[-1]}, device {q.device}); pass attention= for other inputs")
    o, _ = _ops.attn_fwd(q.contiguous(), k.contiguous(), v.contiguous(), 1.0 / math.sqrt(q.shape[-1]))
    return o


class DilatedLighthouseScorer(nn.Module):
    """Dilated scorer (SEL:618-689): the scores are the norms of attention
    outputs over dilated views of the sequence (every `dilation`-th token forms
    one of dilation*H sub-sequences), q attending to k (qk) and k to q (kq);
    the pyramids are the same level means as the norm scorer's.

    The reference's own wiring of this scorer does not run: the torchtitan
    patch constructs it with ``head_dim=`` and no ``attention`` (PATCH:623-628
    vs SEL:619-625), and its forward calls ``view`` on transposed tensors.
    Here ``attention`` defaults to causal attention (the tcgen05 kernel of this
    package for bf16 / D = 128), ``head_dim`` is accepted and unused, and the
    outputs are reshaped back to token order as the reference intends.  The
    scores only feed the selection (under no_grad in LighthouseLocal, SEL:794),
    so the scorer attention runs without autograd."""

    def __init__(self, attention=None, dilation: int = 4, pooling_factor: int = 4, levels: int = 3,
                 head_dim: int | None = None):
        super().__init__()
        self.attention = attention if attention is not None else _causal_attention
        self.dilation = dilation
        self.pooling_factor = pooling_factor
        self.levels = levels

    def scores(self, xq, xk, xv):
        """(scores_qk, scores_kq) over the pyramid, (B, H, S_tot) fp32."""
        b, s, h, d = xq.shape
        di = self.dilation
        if s % di:
            raise ValueError("dilated scorer: sequence length must be a multiple of the dilation")
        with torch.no_grad():
            view = lambda x: x.reshape(b, s // di, di * h, d).transpose(1, 2)     # (b, di*h, s/di, d)
            back = lambda o: o.transpose(1, 2).reshape(b, s, h, d).contiguous()
            out_qk = back(self.attention(view(xq), view(xk), view(xv)))
            out_kq = back(self.attention(view(xk), view(xq), view(xv)))
            # norms of the outputs, rounded to the dtype, max-pooled per level:
            # what the pyramid kernel computes for its first two inputs
            _, _, _, sqk, skq = _ops.pyramid_score(out_qk, out_kq, out_kq, self.levels, self.pooling_factor)
        return sqk, skq

    def forward(self, xq, xk, xv):
        sqk, skq = self.scores(xq, xk, xv)
        _, _, xq_cat, xk_cat, xv_cat = _PyramidFn.apply(xq, xk, xv, self.levels, self.pooling_factor)
        return sqk.to(xq.dtype), skq.to(xq.dtype), xq_cat, xk_cat, xv_cat


class DilatedLighthouseGLAScorer(nn.Module):
    """Gated-linear-attention scorer (SEL:692-755): the scores are the norms of
    simple-GLA outputs over the dilated views (dilation*H sub-sequences of every
    `dilation`-th token), q->k and k->q sharing v and the per-(token, head)
    log-gate gk; the pyramids are the norm scorer's level means.

    The reference takes simple GLA from the external fla package
    (chunk_simple_gla, SEL:725-726); here both passes run in one launch of this
    package's kernel (csrc/gla.cu, bf16, head_dim 128), and the norms and level
    maxima come from the pyramid kernel.  Like the reference, the scores are
    used for selection only and carry no gradient (the gate gets none either)."""

    def __init__(self, head_dim: int, dilation: int = 4, pooling_factor: int = 4, levels: int = 3):
        super().__init__()
        self.head_dim = head_dim
        self.dilation = dilation
        self.pooling_factor = pooling_factor
        self.levels = levels
        self.scaling = 1.0 / math.sqrt(head_dim)

    def scores(self, xq, xk, xv, gk):
        """(scores_qk, scores_kq) over the pyramid, (B, H, S_tot) fp32."""
        b, s, h, d = xq.shape
        di = self.dilation
        if s % di:
            raise ValueError("gla scorer: sequence length must be a multiple of the dilation")
        if gk is None or tuple(gk.shape) != (b, s, h):
            raise ValueError("gla scorer: needs the gate gk of shape (B, S, H)")
        with torch.no_grad():
            view = lambda x: x.reshape(b, s // di, di * h, d)          # fla's (B, T, H, D) layout
            gd = gk.detach().reshape(b, s // di, di * h)
            o_qk, o_kq = _ops.simple_gla_fwd2(view(xq).contiguous(), view(xk).contiguous(), view(xv).contiguous(),
                                              gd.float().contiguous(), self.scaling, view(xk).contiguous(),
                                              view(xq).contiguous())
            o_qk, o_kq = o_qk.view(b, s, h, d), o_kq.view(b, s, h, d)
            _, _, _, sqk, skq = _ops.pyramid_score(o_qk, o_kq, o_kq, self.levels, self.pooling_factor)
        return sqk, skq

    def forward(self, xq, xk, xv, gk):
        sqk, skq = self.scores(xq, xk, xv, gk)
        _, _, xq_cat, xk_cat, xv_cat = _PyramidFn.apply(xq, xk, xv, self.levels, self.pooling_factor)
        return sqk.to(xq.dtype), skq.to(xq.dtype), xq_cat, xk_cat, xv_cat


# ----------------------------------------------------------------------------- scatter
class _ScatterFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, attn, indices, N_shard, N_total, L, p):
        idx = indices.to(torch.int32).contiguous()
        inv = _ops.build_inverse(idx, _native.pyramid_len(N_shard, L, p))
        ctx.save_for_backward(idx)
        ctx.args = (N_shard, N_total, L, p)
        return _ops.scatter_fwd(attn.contiguous(), inv, N_shard, N_total, L, p)

    @staticmethod
    def backward(ctx, dout):
        (idx,) = ctx.saved_tensors
        return _ops.scatter_bwd(dout.contiguous(), idx, *ctx.args), None, None, None, None, None


def scatter_to_base_sequence(attn_out, indices_hp, rank_ids_hp, N_shard: int, N_total: int, num_levels: int,
                             pooling_factor: int):
    """Fan-out of selected outputs to base positions (SEL:758-770, kernels SEL:408-576).

    The reference adds rank_id * N_shard to every position; its callers always
    pass zeros (SEL:817, 1048-1049), which is the only case supported here.
    """
    if rank_ids_hp is not None and bool((rank_ids_hp != 0).any()):
        raise ValueError("scatter_to_base_sequence: non-zero rank_ids are not supported")
    return _ScatterFn.apply(attn_out, indices_hp, N_shard, N_total, num_levels, pooling_factor)


# ----------------------------------------------------------------------------- fused layer
class _LighthouseLayerFn(torch.autograd.Function):
    """One Lighthouse layer (SEL:789-825) as a single autograd node."""

    @staticmethod
    def forward(ctx, xq, xk, xv, L, p, k, scores=None):
        B, S, H, D = xq.shape
        xq, xk, xv = xq.contiguous(), xk.contiguous(), xv.contiguous()
        pq, pk, pv, sqk, skq = _ops.pyramid_score(xq, xk, xv, L, p)
        if scores is not None:                  # another scorer's (qk, kq) scores, fp32
            sqk, skq = (t.to(torch.float32).contiguous() for t in scores)
        idx, inv = _ops.select_topk(sqk, skq, L, p, k, S)
        qs, ks, vs = _ops.gather_selected(xq, xk, xv, pq, pk, pv, idx)
        scale = 1.0 / math.sqrt(D)
        o, lse = _ops.attn_fwd(qs, ks, vs, scale)
        # Token-major output (B, S, H, D), returned as a (B, H, S, D) view: the
        # caller's transpose before the output projection (PATCH:737) is then
        # free.  Same values as the (B, H, S, D) kernel.
        if _native.token_major_ok(B, H, D, o.dtype):
            out = _ops.scatter_fwd_token_major(o, inv, S, S, L, p).transpose(1, 2)
        else:
            out = _ops.scatter_fwd(o, inv, S, S, L, p)
        ctx.save_for_backward(qs, ks, vs, o, lse, idx, inv)
        ctx.args = (S, L, p, scale)
        ctx.mark_non_differentiable(idx)
        return out, idx

    @staticmethod
    def backward(ctx, dout, _didx):
        qs, ks, vs, o, lse, idx, inv = ctx.saved_tensors
        S, L, p, scale = ctx.args
        B, H, _, D = dout.shape
        if not dout.is_contiguous() and _native.token_major_ok(B, H, D, dout.dtype):
            dattn = _ops.scatter_bwd_token_major(dout.transpose(1, 2).contiguous(), idx, S, S, L, p)
        else:
            dattn = _ops.scatter_bwd(dout.contiguous(), idx, S, S, L, p)
        dqs, dks, dvs = _ops.attn_bwd(qs, ks, vs, o, lse, dattn, scale)
        dxq, dxk, dxv = _ops.unpool_bwd(dqs, dks, dvs, inv, S, L, p)
        return dxq, dxk, dxv, None, None, None, None


def lighthouse_attention(xq, xk, xv, num_levels: int = 3, pooling_factor: int = 4, topk: int = 1024,
                         return_indices: bool = False):
    """Functional form of LighthouseLocal.forward: (B,S,H,D) x3 -> (B,H,S,D)."""
    if xq.dtype != torch.bfloat16:
        raise ValueError("lighthouse_attention computes in bf16")
    out, idx = _LighthouseLayerFn.apply(xq, xk, xv, num_levels, pooling_factor, topk)
    return (out, idx) if return_indices else out


class LighthouseLocal(nn.Module):
    """Single-device Lighthouse layer (SEL:772-825).

    ``attention`` is kept for signature compatibility; the gathered causal
    attention runs in this package's tcgen05 kernels.
    """

    def __init__(self, attention, scorer, num_levels: int = 3, pooling_factor: int = 4, topk: int = 1024):
        super().__init__()
        self.scorer = scorer
        self.num_levels = num_levels
        self.pooling_factor = pooling_factor
        self.topk = topk
        self.attention = attention

    def forward(self, xq, xk, xv, gk=None):
        """``gk`` is the GLA scorer's gate (B, S, H); the torchtitan patch passes it
        by keyword (PATCH:708-710), which the reference's forward does not accept."""
        if isinstance(self.scorer, DialatedLighthouseNormScorer):
            return lighthouse_attention(xq, xk, xv, self.num_levels, self.pooling_factor, self.topk)
        if isinstance(self.scorer, (DilatedLighthouseScorer, DilatedLighthouseGLAScorer)):
            if xq.dtype != torch.bfloat16:
                raise ValueError("lighthouse_attention computes in bf16")
            if isinstance(self.scorer, DilatedLighthouseGLAScorer):
                scores = self.scorer.scores(xq, xk, xv, gk)
            else:
                scores = self.scorer.scores(xq, xk, xv)
            out, _ = _LighthouseLayerFn.apply(xq, xk, xv, self.num_levels, self.pooling_factor, self.topk, scores)
            return out
        raise NotImplementedError(f"unsupported scorer {type(self.scorer).__name__}")


class LighthouseCP(nn.Module):
    """Context-parallel Lighthouse layer (SEL:985-1054).

    The local shard holds the head/tail load-balanced chunks r and 2W-1-r of
    the global sequence.  Each half is pooled and selected on its own with
    topk / (2W) (SEL:1009-1029); attention runs causally over the selections
    of all 2W chunks in global order, K/V of the other ranks arriving through
    one NCCL all-gather (see ``cp.py``); each half is scattered back into its
    own half (SEL:1046-1054).
    """

    def __init__(self, attention, scorer, num_levels: int = 3, pooling_factor: int = 4, topk: int = 1024):
        super().__init__()
        self.scorer = scorer
        self.num_levels = num_levels
        self.pooling_factor = pooling_factor
        self.topk = topk
        self.attention = attention
        self._rank = 0
        self._world_size = 1
        self._cp_group = None

    def set_cp_info(self, rank: int, world_size: int, cp_group):
        self._rank = rank
        self._world_size = world_size
        self._cp_group = cp_group

    def forward(self, xq, xk, xv):
        from . import cp
        return cp.lighthouse_cp_forward(xq, xk, xv, self.num_levels, self.pooling_factor, self.topk,
                                        self._rank, self._world_size, self._cp_group)
