"""The C-ABI ops as torch.library custom ops (namespace ``lighthouse_b200``).

Each op wraps one entry point of liblighthouse_b200.so (through ``_native``) and
carries a fake kernel that gives its output shapes and dtypes without running
it, so torch.compile / torch.export trace the Lighthouse layer as one graph with
the kernels as opaque nodes (no graph breaks at the ctypes calls), and meta
tensors propagate through it.  The autograd nodes of the layer
(``lighthouse_selection``) call these ops.

Geometry (reference: CU:346-357, SEL:600-614):
    S_tot = sum_{l<L} S // p^l,   S_pool = S_tot - S,   S_sel = S // p^(L-1) + (L-1) p k
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _native

NS = "lighthouse_b200"


def _pyr_len(S, L: int, p: int):
    return sum(S // p ** l for l in range(L))


# --------------------------------------------------------------------------- pyramid + scores
@torch.library.custom_op(f"{NS}::pyramid_score", mutates_args=())
def pyramid_score(xq: Tensor, xk: Tensor, xv: Tensor, L: int, p: int) -> tuple[Tensor, Tensor, Tensor, Tensor,
                                                                                 Tensor]:
    """(B,S,H,D) x3 -> pooled q/k/v (B,H,S_pool,D), scores_qk/kq (B,H,S_tot) fp32."""
    return tuple(_native.pyramid_score(xq, xk, xv, L, p))


@pyramid_score.register_fake
def _(xq, xk, xv, L, p):
    B, S, H, D = xq.shape
    S_tot = _pyr_len(S, L, p)
    pooled = [xq.new_empty(B, H, S_tot - S, D) for _ in range(3)]
    return (*pooled, xq.new_empty(B, H, S_tot, dtype=torch.float32), xq.new_empty(B, H, S_tot, dtype=torch.float32))


# --------------------------------------------------------------------------- selection
@torch.library.custom_op(f"{NS}::select_topk", mutates_args=())
def select_topk(scores_qk: Tensor, scores_kq: Tensor, L: int, p: int, k: int, N: int) -> tuple[Tensor, Tensor]:
    """Selected pyramid indices (B,H,S_sel) int32 and the inverse map (B,H,S_tot) int32."""
    idx, inv = _native.select_topk(scores_qk, scores_kq, L, p, k, N)
    return idx, inv


@select_topk.register_fake
def _(scores_qk, scores_kq, L, p, k, N):
    B, H, S_tot = scores_qk.shape
    S_sel = N // p ** (L - 1) + (L - 1) * p * k
    return (scores_qk.new_empty(B, H, S_sel, dtype=torch.int32),
            scores_qk.new_empty(B, H, S_tot, dtype=torch.int32))


@torch.library.custom_op(f"{NS}::build_inverse", mutates_args=())
def build_inverse(indices: Tensor, S_tot: int) -> Tensor:
    """Inverse of a selection: inv[b,h,i] = slot of pyramid entry i, -1 when not selected."""
    return _native.build_inverse(indices, S_tot)


@build_inverse.register_fake
def _(indices, S_tot):
    B, H, _ = indices.shape
    return indices.new_empty(B, H, S_tot, dtype=torch.int32)


# --------------------------------------------------------------------------- gathers
@torch.library.custom_op(f"{NS}::gather_selected", mutates_args=())
def gather_selected(xq: Tensor, xk: Tensor, xv: Tensor, pq: Tensor, pk: Tensor, pv: Tensor,
                    indices: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """Rows of the pyramids [x (B,S,H,D) | pooled (B,H,S_pool,D)] at the indices -> (B,H,S_sel,D) x3."""
    return tuple(_native.gather_selected([xq, xk, xv], [pq, pk, pv], indices))


@gather_selected.register_fake
def _(xq, xk, xv, pq, pk, pv, indices):
    B, S, H, D = xq.shape
    S_sel = indices.shape[-1]
    return tuple(x.new_empty(B, H, S_sel, D) for x in (xq, xk, xv))


# --------------------------------------------------------------------------- attention
@torch.library.custom_op(f"{NS}::attn_fwd", mutates_args=())
def attn_fwd(q: Tensor, k: Tensor, v: Tensor, scale: float, q_off: int = 0) -> tuple[Tensor, Tensor]:
    """Causal attention (B,H,S_q,128) bf16 -> O (B,H,S_q,128), LSE (B,H,S_q) fp32."""
    o, lse = _native.attn_fwd(q, k, v, scale, q_off)
    return o, lse


@attn_fwd.register_fake
def _(q, k, v, scale, q_off=0):
    B, H, S_q, D = q.shape
    return q.new_empty(B, H, S_q, D), q.new_empty(B, H, S_q, dtype=torch.float32)


@torch.library.custom_op(f"{NS}::attn_bwd", mutates_args=())
def attn_bwd(q: Tensor, k: Tensor, v: Tensor, o: Tensor, lse: Tensor, do: Tensor, scale: float,
             q_off: int = 0) -> tuple[Tensor, Tensor, Tensor]:
    """Backward of attn_fwd: dQ, dK, dV."""
    return tuple(_native.attn_bwd(q, k, v, o, lse, do, scale, q_off))


@attn_bwd.register_fake
def _(q, k, v, o, lse, do, scale, q_off=0):
    return q.new_empty(q.shape), k.new_empty(k.shape), v.new_empty(v.shape)


# --------------------------------------------------------------------------- scatter / un-pool
@torch.library.custom_op(f"{NS}::scatter_fwd", mutates_args=())
def scatter_fwd(attn: Tensor, inverse: Tensor, N_shard: int, N_total: int, L: int, p: int) -> Tensor:
    """Fan-out of the selected rows (B,H,S_sel,D) to base positions (B,H,N_total,D)."""
    return _native.scatter_fwd(attn, inverse, N_shard, N_total, L, p)


@scatter_fwd.register_fake
def _(attn, inverse, N_shard, N_total, L, p):
    B, H, _, D = attn.shape
    return attn.new_empty(B, H, N_total, D)


@torch.library.custom_op(f"{NS}::scatter_bwd", mutates_args=())
def scatter_bwd(dout: Tensor, indices: Tensor, N_shard: int, N_total: int, L: int, p: int) -> Tensor:
    """Adjoint of scatter_fwd: window sums of dout for every selected row."""
    return _native.scatter_bwd(dout, indices, N_shard, N_total, L, p)


@scatter_bwd.register_fake
def _(dout, indices, N_shard, N_total, L, p):
    B, H, _, D = dout.shape
    return dout.new_empty(B, H, indices.shape[-1], D)


@torch.library.custom_op(f"{NS}::scatter_fwd_token_major", mutates_args=())
def scatter_fwd_token_major(attn: Tensor, inverse: Tensor, N_shard: int, N_total: int, L: int, p: int) -> Tensor:
    """scatter_fwd with the output as (B, N_total, H, D)."""
    return _native.scatter_fwd_token_major(attn, inverse, N_shard, N_total, L, p)


@scatter_fwd_token_major.register_fake
def _(attn, inverse, N_shard, N_total, L, p):
    B, H, _, D = attn.shape
    return attn.new_empty(B, N_total, H, D)


@torch.library.custom_op(f"{NS}::scatter_bwd_token_major", mutates_args=())
def scatter_bwd_token_major(dout: Tensor, indices: Tensor, N_shard: int, N_total: int, L: int, p: int) -> Tensor:
    """Adjoint of scatter_fwd_token_major: dout (B, N_total, H, D)."""
    return _native.scatter_bwd_token_major(dout, indices, N_shard, N_total, L, p)


@scatter_bwd_token_major.register_fake
def _(dout, indices, N_shard, N_total, L, p):
    B, _, H, D = dout.shape
    return dout.new_empty(B, H, indices.shape[-1], D)


@torch.library.custom_op(f"{NS}::unpool_bwd", mutates_args=())
def unpool_bwd(dq: Tensor, dk: Tensor, dv: Tensor, inverse: Tensor, S: int, L: int,
               p: int) -> tuple[Tensor, Tensor, Tensor]:
    """Gradients of the selected rows (B,H,S_sel,D) back to the inputs (B,S,H,D) through
    the gathers and the level means."""
    return tuple(_native.unpool_bwd([dq, dk, dv], inverse, S, L, p))


@unpool_bwd.register_fake
def _(dq, dk, dv, inverse, S, L, p):
    B, H, _, D = dq.shape
    return tuple(d.new_empty(B, S, H, D) for d in (dq, dk, dv))


# --------------------------------------------------------------------------- model harness / scorers
@torch.library.custom_op(f"{NS}::rope_apply", mutates_args=())
def rope_apply(xq: Tensor, xk: Tensor, table: Tensor, inverse: bool = False) -> tuple[Tensor, Tensor]:
    """Rotary embedding of q and k (B,S,H,D) with the (S, D/2, 2) fp32 (cos, sin) table."""
    oq, ok = _native.rope_apply(xq, xk, table, inverse)
    return oq, ok


@rope_apply.register_fake
def _(xq, xk, table, inverse=False):
    return xq.new_empty(xq.shape), xk.new_empty(xk.shape)


@torch.library.custom_op(f"{NS}::simple_gla_fwd2", mutates_args=())
def simple_gla_fwd2(q: Tensor, k: Tensor, v: Tensor, g: Tensor, scale: float, q2: Tensor,
                    k2: Tensor) -> tuple[Tensor, Tensor]:
    """Two simple-GLA passes sharing v and g ((B,T,H,128) bf16, g (B,T,H)): (q, k) and (q2, k2)."""
    o, o2 = _native.simple_gla_fwd(q, k, v, g, scale, q2=q2, k2=k2)
    return o, o2


@simple_gla_fwd2.register_fake
def _(q, k, v, g, scale, q2, k2):
    return q.new_empty(q.shape), q.new_empty(q.shape)


ops = torch.ops.lighthouse_b200
