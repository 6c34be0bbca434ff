"""CPU stand-ins for the kernel namespace used by the context-parallel host
logic (TEST INFRASTRUCTURE ONLY).

Same function names, argument meaning and output layouts as the product's
``_native`` module, computed with the oracle's restatements in fp32 on the
CPU, so that the multi-rank orchestration in the package's ``cp.py`` can run
on `gloo` CPU ranks in tests.  The product never imports this module.
"""
from __future__ import annotations

import math

import torch

from . import oracle as O


def pyramid_score(xq, xk, xv, L, p):
    B, S, H, D = xq.shape
    sqk, skq, qc, kc, vc = O.norm_scorer(xq, xk, xv, p, L)
    return (qc[:, :, S:].contiguous(), kc[:, :, S:].contiguous(), vc[:, :, S:].contiguous(),
            sqk.float().contiguous(), skq.float().contiguous())


def select_topk(sqk, skq, L, p, k, N, with_inverse=True):
    idx = O.select(sqk, skq, L, p, k, N)
    return idx, O.inverse_map(idx, sqk.shape[-1])


def gather_selected(raws, pooleds, idx):
    outs = []
    for x, pooled in zip(raws, pooleds):
        cat = torch.cat([x.transpose(1, 2), pooled], dim=2)
        outs.append(O.gather_rows(cat, idx).contiguous())
    return outs


def _attn(q, k, v, q_off):
    S_q, S_kv = q.shape[2], k.shape[2]
    s = q @ k.transpose(-1, -2) / math.sqrt(q.shape[-1])
    pq = torch.arange(S_q)[:, None] + q_off
    pk = torch.arange(S_kv)[None, :]
    s = s.masked_fill(pk > pq, float("-inf"))
    return torch.softmax(s, -1) @ v, torch.logsumexp(s, -1)


def attn_fwd(q, k, v, scale, q_off=0):
    o, lse = _attn(q.float(), k.float(), v.float(), q_off)
    return o.to(q.dtype), lse


def attn_bwd(q, k, v, o, lse, do, scale, q_off=0):
    """Backward of one key block given the row statistics of the whole
    attention (o, lse), as the product kernel computes it:
    P = exp(scale QK^T - lse), Delta = rowsum(dO o), dS = P (dO V^T - Delta)."""
    qf, kf, vf, of, dof = (t.float() for t in (q, k, v, o, do))
    S_q, S_kv = q.shape[2], k.shape[2]
    s = qf @ kf.transpose(-1, -2) * scale
    pq = torch.arange(S_q)[:, None] + q_off
    pk = torch.arange(S_kv)[None, :]
    p = torch.exp(s - lse.float()[..., None]).masked_fill(pk > pq, 0.0)
    delta = (dof * of).sum(-1, keepdim=True)
    ds = p * (dof @ vf.transpose(-1, -2) - delta)
    dq = ds @ kf * scale
    dk = ds.transpose(-1, -2) @ qf * scale
    dv = p.transpose(-1, -2) @ dof
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


def attn_merge(o1, lse1, o2, lse2):
    lse = torch.logaddexp(lse1, lse2)
    o = torch.exp(lse1 - lse)[..., None] * o1.float() + torch.exp(lse2 - lse)[..., None] * o2.float()
    return o.to(o1.dtype), lse


def scatter_fwd(attn, inv, N, N_total, L, p):
    S_sel = attn.shape[2]
    # rebuild the index list from the inverse map (slot -> pyramid index)
    B, H, S_tot = inv.shape
    idx = torch.full((B, H, S_sel), -1, dtype=torch.long)
    pos = torch.arange(S_tot).expand(B, H, S_tot)
    m = inv >= 0
    idx[m.nonzero(as_tuple=True)[0], m.nonzero(as_tuple=True)[1], inv[m].long()] = pos[m]
    return O.scatter_to_base(attn, idx, N, N_total, L, p)


def scatter_bwd(dout, idx, N, N_total, L, p):
    B, H, S_sel = idx.shape
    with torch.enable_grad():
        a = torch.zeros(B, H, S_sel, dout.shape[-1], dtype=dout.dtype, requires_grad=True)
        O.scatter_to_base(a, idx.long(), N, N_total, L, p).backward(dout)
    return a.grad


def unpool_bwd(dsels, inv, S, L, p):
    outs = []
    for d in dsels:
        B, H, S_sel, D = d.shape
        idx = torch.full((B, H, S_sel), 0, dtype=torch.long)
        m = inv >= 0
        b, h = m.nonzero(as_tuple=True)[0], m.nonzero(as_tuple=True)[1]
        idx[b, h, inv[m].long()] = torch.arange(inv.shape[-1]).expand_as(inv)[m]
        with torch.enable_grad():
            x = torch.zeros(B, S, H, D, dtype=d.dtype, requires_grad=True)
            _, _, qc, _, _ = O.norm_scorer(x, x, x, p, L)
            O.gather_rows(qc, idx).backward(d)
        outs.append(x.grad)
    return outs
