"""Context-parallel Lighthouse layer (LighthouseCP, reference src/lighthouse_selection.py:985-1054).

Sharding (head/tail load balance, as torch's context_parallel load balancer
does for the reference): the global sequence is cut into 2W equal chunks and
rank r holds chunks r and 2W-1-r, concatenated, as its local shard.

Per rank:
  1. each local half is pooled, scored and selected on its own with
     k / (2W) (pooling restarts per chunk: SEL:1014-1029);
  2. the selected K and V of both halves are all-gathered over the CP group
     (one NCCL all_gather, overlapped with the diagonal blocks' attention)
     and laid out in global chunk order;
  3. the selected queries of chunk c attend causally to the selections of
     chunks 0..c (query row r of chunk c sits at global selected position
     c * S_c + r) -- the same result torch's ring attention gives the
     reference under context_parallel;
  4. each half's output is scattered back into its half (SEL:1046-1054).
Backward: dQ stays local; the off-diagonal dK/dV partials for every chunk
are summed over ranks with one reduce-scatter (fp32, overlapped with the
diagonal blocks' backward) so each rank receives its own chunks'.

``ops`` is the kernel namespace (``_native`` on the GPU); tests may pass a
namespace with the same functions to exercise the host logic on CPU ranks.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import _native


def _owner(c: int, W: int) -> tuple[int, int]:
    """(rank, slot) holding global chunk c: slot 0 = head half, 1 = tail half."""
    return (c, 0) if c < W else (2 * W - 1 - c, 1)


class _SelectHalfFn(torch.autograd.Function):
    """Pyramid + selection + gather of one chunk; backward = un-pool."""

    @staticmethod
    def forward(ctx, xq, xk, xv, L, p, k, ops):
        B, S, H, D = xq.shape
        pq, pk, pv, sqk, skq = ops.pyramid_score(xq, xk, xv, L, p)
        idx, inv = ops.select_topk(sqk, skq, L, p, k, S)
        qs, ks, vs = ops.gather_selected([xq, xk, xv], [pq, pk, pv], idx)
        ctx.save_for_backward(inv)
        ctx.args = (S, L, p, ops)
        ctx.mark_non_differentiable(idx, inv)
        return qs, ks, vs, idx, inv

    @staticmethod
    def backward(ctx, dqs, dks, dvs, _di, _dv):
        (inv,) = ctx.saved_tensors
        S, L, p, ops = ctx.args
        dxq, dxk, dxv = ops.unpool_bwd([dqs, dks, dvs], inv, S, L, p)
        return dxq, dxk, dxv, None, None, None, None


class _ScatterInvFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, attn, idx, inv, N, L, p, ops):
        ctx.save_for_backward(idx)
        ctx.args = (N, L, p, ops)
        return ops.scatter_fwd(attn, inv, N, N, L, p)

    @staticmethod
    def backward(ctx, dout):
        (idx,) = ctx.saved_tensors
        N, L, p, ops = ctx.args
        return ops.scatter_bwd(dout, idx, N, N, L, p), None, None, None, None, None, None


class _CPAttentionFn(torch.autograd.Function):
    """Causal attention of the two local query chunks against all ranks' K/V.

    Local chunks a = rank (head) and b = 2W-1-rank (tail).  Chunk c's queries
    see the keys of chunks 0..c-1 in full and their own chunk causally, so
    each query chunk's attention splits into a diagonal block (its own
    chunk, causal, local data) and an off-diagonal block (the earlier chunks,
    unmasked, gathered data), merged by log-sum-exp as the ring attention the
    reference runs under torch's context parallelism merges its per-step
    blocks.  The all-gather of the selected K/V runs while the diagonal
    blocks compute; in backward the reduce-scatter of the off-diagonal dK/dV
    partials runs while the diagonal blocks' backward computes."""

    @staticmethod
    def forward(ctx, qh, qt, kh, kt, vh, vt, rank, W, group, ops):
        B, H, S_c, D = qh.shape
        scale = 1.0 / math.sqrt(D)
        a, b = rank, 2 * W - 1 - rank
        kv = torch.stack([kh, kt, vh, vt])                    # (4, B, H, S_c, D)
        gathered, work = _all_gather_async(kv, W, group)      # rank order
        oh, lh = ops.attn_fwd(qh, kh, vh, scale)              # diagonal blocks, local
        ot, lt = ops.attn_fwd(qt, kt, vt, scale)
        if work is not None:
            work.wait()
        K, V = _global_kv(gathered, W, b)                     # chunks 0..b-1, global order
        if a > 0:
            oo, lo = ops.attn_fwd(qh, K[:, :, :a * S_c], V[:, :, :a * S_c], scale, q_off=a * S_c)
            oh, lh = ops.attn_merge(oh, lh, oo, lo)
        oo, lo = ops.attn_fwd(qt, K, V, scale, q_off=b * S_c)
        ot, lt = ops.attn_merge(ot, lt, oo, lo)
        ctx.save_for_backward(qh, qt, kh, kt, vh, vt, K, V, oh, ot, lh, lt)
        ctx.args = (rank, W, group, ops, scale, S_c)
        return oh, ot

    @staticmethod
    def backward(ctx, doh, dot):
        qh, qt, kh, kt, vh, vt, K, V, oh, ot, lh, lt = ctx.saved_tensors
        rank, W, group, ops, scale, S_c = ctx.args
        a, b = rank, 2 * W - 1 - rank
        B, H, _, D = qh.shape
        # off-diagonal blocks first: their dK / dV belong to chunks 0..b-1 of
        # every rank and go out with one reduce-scatter (fp32 sums, as torch's
        # ring attention accumulates in fp32)
        dqt, dKt, dVt = ops.attn_bwd(qt, K, V, ot, lt, dot, scale, q_off=b * S_c)
        if a > 0:
            dqh, dKh, dVh = ops.attn_bwd(qh, K[:, :, :a * S_c], V[:, :, :a * S_c], oh, lh, doh, scale, q_off=a * S_c)
        blocks = torch.zeros(W, 4, B, H, S_c, D, dtype=torch.float32, device=qh.device)
        for c in range(b):
            r, slot = _owner(c, W)
            sl = slice(c * S_c, (c + 1) * S_c)
            blocks[r, slot].copy_(dKt[:, :, sl])
            blocks[r, 2 + slot].copy_(dVt[:, :, sl])
            if c < a:
                blocks[r, slot] += dKh[:, :, sl]
                blocks[r, 2 + slot] += dVh[:, :, sl]
        mine, work = _reduce_scatter_async(blocks, W, group)
        # diagonal blocks (local chunks) while the partials travel
        dqh_d, dkh, dvh = ops.attn_bwd(qh, kh, vh, oh, lh, doh, scale)
        dqt_d, dkt, dvt = ops.attn_bwd(qt, kt, vt, ot, lt, dot, scale)
        dqh = dqh_d if a == 0 else (dqh_d.float() + dqh.float()).to(qh.dtype)
        dqt = (dqt_d.float() + dqt.float()).to(qt.dtype)
        if work is not None:
            work.wait()
        mine = mine if W > 1 else blocks[0]
        out = [(mine[i] + d.float()).to(qh.dtype) for i, d in enumerate((dkh, dkt, dvh, dvt))]
        return dqh, dqt, out[0], out[1], out[2], out[3], None, None, None, None


def _all_gather_async(t: torch.Tensor, W: int, group):
    """Start an all-gather of t over the group; (list of per-rank tensors, work or None)."""
    if W == 1:
        return [t], None
    outs = [torch.empty_like(t) for _ in range(W)]
    work = dist.all_gather(outs, t.contiguous(), group=group, async_op=True)
    return outs, work


def _global_kv(gathered, W: int, n_chunks: int):
    """K and V of global chunks 0..n_chunks-1 in chunk order from the
    rank-ordered gathered (4, B, H, S_c, D) blocks."""
    ks, vs = [], []
    for c in range(n_chunks):
        r, slot = _owner(c, W)
        ks.append(gathered[r][slot])
        vs.append(gathered[r][2 + slot])
    return torch.cat(ks, dim=2).contiguous(), torch.cat(vs, dim=2).contiguous()


def _reduce_scatter_async(t: torch.Tensor, W: int, group):
    """Start summing the rank-ordered blocks t (W, ...) over the group; this
    rank receives its own block.  Returns (result tensor, work or None)."""
    if W == 1:
        return t[0], None
    if dist.get_backend(group) == "nccl":
        out = torch.empty_like(t[0])
        work = dist.reduce_scatter_tensor(out, t.contiguous(), group=group, async_op=True)
        return out, work
    dist.all_reduce(t, group=group)          # gloo (CPU test ranks) has no reduce-scatter
    return t[dist.get_rank(group)], None


def lighthouse_cp_forward(xq, xk, xv, L: int, p: int, k: int, rank: int, world_size: int, group, ops=None):
    """LighthouseCP.forward (SEL:1009-1054): (B, S_local, H, D) x3 -> (B, H, S_local, D)."""
    ops = ops or _native
    W = max(1, int(world_size))
    _, s, _, _ = xq.shape
    half = s // 2
    k_chunk = k // (2 * W)
    sel = []
    for part in (slice(0, half), slice(half, s)):
        sel.append(_SelectHalfFn.apply(xq[:, part].contiguous(), xk[:, part].contiguous(),
                                       xv[:, part].contiguous(), L, p, k_chunk, ops))
    (qh, kh, vh, ih, invh), (qt, kt, vt, it, invt) = sel
    oh, ot = _CPAttentionFn.apply(qh, qt, kh, kt, vh, vt, rank, W, group, ops)
    out_h = _ScatterInvFn.apply(oh, ih, invh, half, L, p, ops)
    out_t = _ScatterInvFn.apply(ot, it, invt, half, L, p, ops)
    return torch.cat([out_h, out_t], dim=2)


def full_cp_attention(xq, xk, xv, rank: int, world_size: int, group, ops=None):
    """Causal attention over the whole (load-balanced, sharded) sequence: the
    full-attention layers of a context-parallel model (the reference runs them
    under torch's context_parallel ring attention, PATCH:754-766).
    (B, S_local, H, D) x3, local shard = global chunks (rank, 2W-1-rank)
    -> (B, H, S_local, D).  Same collectives as the Lighthouse layer: one
    all-gather of K/V, one reduce-scatter of the dK/dV partials."""
    ops = ops or _native
    W = max(1, int(world_size))
    _, s, _, _ = xq.shape
    half = s // 2
    t = lambda x, part: x[:, part].transpose(1, 2).contiguous()
    hp, tp = slice(0, half), slice(half, s)
    oh, ot = _CPAttentionFn.apply(t(xq, hp), t(xq, tp), t(xk, hp), t(xk, tp), t(xv, hp), t(xv, tp),
                                  rank, W, group, ops)
    return torch.cat([oh, ot], dim=2)


def shard_sequence(x: torch.Tensor, rank: int, world_size: int, dim: int = 1) -> torch.Tensor:
    """This rank's load-balanced shard: global chunks rank and 2W-1-rank of 2W."""
    W = max(1, int(world_size))
    chunks = x.chunk(2 * W, dim=dim)
    return torch.cat([chunks[rank], chunks[2 * W - 1 - rank]], dim=dim)
