"""CPU oracle for the Lighthouse selection-attention path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference legs may import this module; the product package never does.

Parity status: the selection restatement (``lh_oracle.c``) is pinned against
the reference's own kernel source run on host threads (``oracle/_ref``,
``build.py``) and, on the GPU box, compiled with the reference's NVRTC flags.
The scorer, gathers, SDPA and scatter are restated with the same ATen calls
the reference makes; the GLA scorer's sequence mixer (the external fla
package's simple GLA) is restated as its defining recurrence; golden vectors from the reference's own Python code
(scorer on CPU, Triton scatter kernels in Triton's interpreter) are committed
under ``tests/golden/`` with the script that made them.

Reference citations (paths inside the reference project):
  SEL = src/lighthouse_selection.py, CU = src/lighthouse_selection_cuda.py
"""
from __future__ import annotations

import ctypes
import math
import pathlib

import numpy as np
import torch
import torch.nn.functional as F

HERE = pathlib.Path(__file__).resolve().parent
_REF = HERE / "_ref"
_lib = None
_ref_cpu = {}
_ref_gpu = {}


def _oracle_lib():
    global _lib
    if _lib is None:
        so = _REF / "liblh_oracle.so"
        if not so.exists():
            import importlib.util
            spec = importlib.util.spec_from_file_location("_lh_oracle_build", HERE / "build.py")
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            mod.build_oracle()
        _lib = ctypes.CDLL(str(so))
        _lib.lho_select.restype = ctypes.c_int
        _lib.lho_sel_len.restype = ctypes.c_int
    return _lib


# --------------------------------------------------------------------------- sizes
def sel_len(N: int, L: int, p: int, k: int) -> int:
    """S_sel, as CU:346-357."""
    total = 0
    for level in range(L, 0, -1):
        total += N // p ** (level - 1) if level == L else p * k
    return total


def pyramid_len(N: int, L: int, p: int) -> int:
    """S_tot = sum_{l<L} N // p^l, the concatenated pyramid length (SEL:600-614)."""
    return sum(N // p ** l for l in range(L))


def level_offsets(N: int, L: int, p: int) -> list[int]:
    offs, acc = [], 0
    for l in range(L):
        offs.append(acc)
        acc += N // p ** l
    return offs


def shape_defined(N: int, L: int, p: int, k: int) -> bool:
    """True when the reference kernel is well defined (k%128, C%T, NCC>=128, NCC%64)."""
    if k % 128 or (p & (p - 1)) or k // 2 < p:
        return False
    T = k // 128
    C = N // p ** (L - 1)
    if N % p ** (L - 1) or C % T:
        return False
    ncc = C // T
    return ncc >= 128 and ncc % 64 == 0


# --------------------------------------------------------------------------- selection
def select(scores_qk: torch.Tensor, scores_kq: torch.Tensor, L: int, p: int, k: int, N: int,
           return_raw: bool = False):
    """C restatement of LighthouseSelectionQkKqChunkedTopkNvrtc.forward (CU:362-429)."""
    lib = _oracle_lib()
    B, H, S_tot = scores_qk.shape
    sq = np.ascontiguousarray(scores_qk.detach().float().cpu().numpy())
    sk = np.ascontiguousarray(scores_kq.detach().float().cpu().numpy())
    S_sel = sel_len(N, L, p, k)
    out = np.empty((B, H, S_sel), np.int32)
    keys = np.empty((B, H, S_sel), np.int32) if return_raw else None
    vals = np.empty((B, H, S_sel), np.int32) if return_raw else None
    P = ctypes.c_void_p
    rc = lib.lho_select(sq.ctypes.data_as(P), sk.ctypes.data_as(P), B * H, S_tot, N, L, p, k,
                        out.ctypes.data_as(P),
                        keys.ctypes.data_as(P) if return_raw else None,
                        vals.ctypes.data_as(P) if return_raw else None)
    if rc != 0:
        raise ValueError(f"oracle select: shape outside the reference's domain (N={N}, L={L}, p={p}, k={k})")
    if return_raw:
        return torch.from_numpy(out), torch.from_numpy(keys), torch.from_numpy(vals)
    return torch.from_numpy(out)


def _ref_geometry(N, L, p, k):
    T = k // 128
    ncc = (N // p ** (L - 1)) // T
    chunk = sel_len(N // T, L, p, 128)
    return T, ncc, chunk


def ref_select_cpu(scores_qk: torch.Tensor, scores_kq: torch.Tensor, L: int, p: int, k: int, N: int,
                   return_raw: bool = False):
    """The reference kernel's own source run on host threads, then the stable
    sort + gather of CU:426-427 (torch.sort stable on int32 keys)."""
    if p not in _ref_cpu:
        so = _REF / f"libref_cpu_p{p}.so"
        if not so.exists():
            raise FileNotFoundError(f"{so} not built (oracle/build.py build_ref needs the reference tree)")
        lib = ctypes.CDLL(str(so))
        lib.ref_cpu_topk.restype = ctypes.c_int
        _ref_cpu[p] = lib
    lib = _ref_cpu[p]
    B, H, S_tot = scores_qk.shape
    S_sel = sel_len(N, L, p, k)
    T, ncc, chunk = _ref_geometry(N, L, p, k)
    assert ncc >= 128
    sq = np.ascontiguousarray(scores_qk.detach().float().cpu().numpy())
    sk = np.ascontiguousarray(scores_kq.detach().float().cpu().numpy())
    # slack after the last row: the reference kernel writes past its row on
    # undefined shapes; the slack keeps that inside this buffer.
    slack = (ncc // 64 + 1) * 64 * 4
    keys = np.full(B * H * S_sel + slack, -1, np.int32)
    vals = np.full(B * H * S_sel + slack, -1, np.int32)
    P = ctypes.c_void_p
    lib.ref_cpu_topk(sq.ctypes.data_as(P), sk.ctypes.data_as(P), keys.ctypes.data_as(P),
                     vals.ctypes.data_as(P), B, H, S_tot, S_sel, L, p, N, ncc, chunk, T)
    keys_t = torch.from_numpy(keys[: B * H * S_sel].reshape(B, H, S_sel).copy())
    vals_t = torch.from_numpy(vals[: B * H * S_sel].reshape(B, H, S_sel).copy())
    order = torch.sort(keys_t, dim=-1, stable=True).indices
    out = torch.gather(vals_t, -1, order)
    if return_raw:
        return out, keys_t, vals_t
    return out


def ref_gpu_lib(p: int):
    """ctypes handle of the reference kernel built for sm_100a (oracle/_ref)."""
    if p not in _ref_gpu:
        so = _REF / f"libref_gpu_p{p}.so"
        lib = ctypes.CDLL(str(so))
        lib.ref_gpu_topk.restype = ctypes.c_int
        _ref_gpu[p] = lib
    return _ref_gpu[p]


def ref_select_gpu(scores_qk: torch.Tensor, scores_kq: torch.Tensor, L: int, p: int, k: int, N: int):
    """The reference kernel on the GPU with its own flags, then CU:426-427."""
    lib = ref_gpu_lib(p)
    B, H, S_tot = scores_qk.shape
    S_sel = sel_len(N, L, p, k)
    T, ncc, chunk = _ref_geometry(N, L, p, k)
    assert shape_defined(N, L, p, k), "reference kernel only runs on defined shapes here"
    sq = scores_qk.float().contiguous()
    sk = scores_kq.float().contiguous()
    keys = torch.full((B, H, S_sel), -1, dtype=torch.int32, device=sq.device)
    vals = torch.full((B, H, S_sel), -1, dtype=torch.int32, device=sq.device)
    P = ctypes.c_void_p
    rc = lib.ref_gpu_topk(P(sq.data_ptr()), P(sk.data_ptr()), P(keys.data_ptr()), P(vals.data_ptr()),
                          B, H, S_tot, S_sel, L, p, N, ncc, chunk, T,
                          P(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, f"reference kernel launch failed: {rc}"
    order = torch.sort(keys, dim=-1, stable=True).indices
    return torch.gather(vals, -1, order)


# --------------------------------------------------------------------------- scorer
def norm_scorer(xq, xk, xv, p: int, L: int):
    """DialatedLighthouseNormScorer.forward (SEL:589-616), same ATen calls."""
    b, s, h, d = xq.shape
    sqk = xq.norm(dim=-1)
    skq = xk.norm(dim=-1)
    lq, lk, lv, lsq, lsk = [xq], [xk], [xv], [sqk], [skq]
    for level in range(1, L):
        pf = p ** level
        n = s // pf
        lq.append(xq[:, : n * pf].view(b, n, pf, h, d).mean(2))
        lk.append(xk[:, : n * pf].view(b, n, pf, h, d).mean(2))
        lv.append(xv[:, : n * pf].view(b, n, pf, h, d).mean(2))
        lsq.append(sqk[:, : n * pf].view(b, n, pf, h).max(2).values)
        lsk.append(skq[:, : n * pf].view(b, n, pf, h).max(2).values)
    cat = lambda xs: torch.cat(xs, dim=1).transpose(1, 2)
    return cat(lsq), cat(lsk), cat(lq), cat(lk), cat(lv)


def simple_gla(q, k, v, g, scale: float):
    """Simple gated linear attention, forward, zero initial state: the function the
    reference's GLA scorer takes from the external flash-linear-attention package
    (fla 0.5.1, ``fla.ops.simple_gla.chunk_simple_gla``, called at SEL:725-726).
    Its published definition, stepped as the recurrence over time
        S_t = exp(g_t) S_{t-1} + k_t v_t^T,     o_t = scale * q_t S_t
    in fp32.  q, k, v (B, T, H, D); g (B, T, H); returns o in q's dtype."""
    dt = q.dtype
    q, k, v, g = (x.float() for x in (q, k, v, g))
    B, T, H, D = q.shape
    state = torch.zeros(B, H, D, v.shape[-1], dtype=torch.float32, device=q.device)
    out = torch.empty(B, T, H, v.shape[-1], dtype=torch.float32, device=q.device)
    for t in range(T):
        state = state * g[:, t].exp()[..., None, None] + k[:, t, :, :, None] * v[:, t, :, None, :]
        out[:, t] = scale * torch.einsum("bhd,bhde->bhe", q[:, t], state)
    return out.to(dt)


def gla_scorer(xq, xk, xv, gk, dilation: int, p: int, L: int):
    """DilatedLighthouseGLAScorer.forward (SEL:711-755): simple GLA over the
    dilated views (b, s/di, di*h, d) in both directions (q->k, k->q) sharing v
    and the gate, output norms as scores, then the pyramid of the norm scorer
    (level means of x, level maxima of the scores)."""
    b, s, h, d = xq.shape
    di = dilation
    view = lambda x: x.reshape(b, s // di, di * h, *x.shape[3:])
    gd = gk.reshape(b, s // di, di * h)
    scale = 1.0 / math.sqrt(d)
    o_qk = simple_gla(view(xq), view(xk), view(xv), gd, scale).reshape(b, s, h, d)
    o_kq = simple_gla(view(xk), view(xq), view(xv), gd, scale).reshape(b, s, h, d)
    sqk, skq = o_qk.norm(dim=-1), o_kq.norm(dim=-1)
    lq, lk, lv, lsq, lsk = [xq], [xk], [xv], [sqk], [skq]
    for level in range(1, L):
        pf = p ** level
        n = s // pf
        lq.append(xq[:, : n * pf].view(b, n, pf, h, d).mean(2))
        lk.append(xk[:, : n * pf].view(b, n, pf, h, d).mean(2))
        lv.append(xv[:, : n * pf].view(b, n, pf, h, d).mean(2))
        lsq.append(sqk[:, : n * pf].view(b, n, pf, h).max(2).values)
        lsk.append(skq[:, : n * pf].view(b, n, pf, h).max(2).values)
    cat = lambda xs: torch.cat(xs, dim=1).transpose(1, 2)
    return cat(lsq), cat(lsk), cat(lq), cat(lk), cat(lv)


# --------------------------------------------------------------------------- scatter
def fanout_windows(indices: torch.Tensor, N_shard: int, N_total: int, L: int, p: int):
    """Per selected slot: (base position + fan - 1, fan) as in SEL:428-455."""
    idx = indices.long()
    base = torch.zeros_like(idx)
    fan = torch.ones_like(idx)
    start = 0
    for l in range(L):
        size = N_shard // p ** l
        inl = (idx >= start) & (idx < start + size)
        base = torch.where(inl, (idx - start) * p ** l, base)
        fan = torch.where(inl, torch.full_like(idx, p ** l), fan)
        start += size
    return base + fan - 1, fan


def scatter_to_base(attn, indices, N_shard: int, N_total: int, L: int, p: int):
    """Differentiable restatement of _ScatterToBaseAutograd (SEL:408-576):
    out[bh, pos] += attn[bh, s] for pos in [base+fan-1, base+2fan-1) & [0, N_total)."""
    B, H, S_sel, D = attn.shape
    first, fan = fanout_windows(indices, N_shard, N_total, L, p)
    maxfan = p ** (L - 1)
    out = attn.new_zeros(B * H * N_total, D)
    flat_attn = attn.reshape(B * H * S_sel, D)
    bh = torch.arange(B * H, device=attn.device).view(B, H, 1).expand(B, H, S_sel)
    for c in range(maxfan):
        pos = first + c
        m = (c < fan) & (pos >= 0) & (pos < N_total)
        sel = m.reshape(-1).nonzero().squeeze(1)
        tgt = (bh.reshape(-1)[sel] * N_total + pos.reshape(-1)[sel])
        out = out.index_add(0, tgt, flat_attn[sel])
    return out.view(B, H, N_total, D)


def gather_rows(x_cat, indices):
    d = x_cat.shape[-1]
    return torch.gather(x_cat, 2, indices.long().unsqueeze(-1).expand(-1, -1, -1, d))


def sdpa_causal(q, k, v):
    return F.scaled_dot_product_attention(q, k, v, is_causal=True)


# --------------------------------------------------------------------------- layer
def lighthouse_local(xq, xk, xv, L: int, p: int, k: int, indices=None, select_fn=None):
    """LighthouseLocal.forward (SEL:789-825) on CPU tensors. Differentiable in
    xq/xk/xv. ``indices`` may be given to skip selection."""
    s = xq.shape[1]
    sqk, skq, q_cat, k_cat, v_cat = norm_scorer(xq, xk, xv, p, L)
    if indices is None:
        with torch.no_grad():
            indices = (select_fn or select)(sqk.float(), skq.float(), L, p, k, s)
    qs, ks, vs = gather_rows(q_cat, indices), gather_rows(k_cat, indices), gather_rows(v_cat, indices)
    attn = sdpa_causal(qs, ks, vs)
    return scatter_to_base(attn, indices, s, s, L, p), indices


def lighthouse_cp_global(xq, xk, xv, world_size: int, L: int, p: int, k: int, indices=None):
    """Semantics of LighthouseCP (SEL:1009-1054) under load-balanced CP with
    world size W, emulated in one process on the global sequence: 2W equal
    chunks, per-chunk scorer + selection with k/(2W), one causal attention over
    the selections concatenated in global chunk order, per-chunk scatter.
    ``indices`` (one tensor per chunk) may be given to skip selection."""
    B, S, H, D = xq.shape
    nch = 2 * world_size
    n = S // nch
    kc = k // nch
    sels, idxs = [], []
    qs, ks, vs = [], [], []
    for c in range(nch):
        sl = slice(c * n, (c + 1) * n)
        sqk, skq, qc, kc_, vc = norm_scorer(xq[:, sl], xk[:, sl], xv[:, sl], p, L)
        if indices is not None:
            idx = indices[c]
        else:
            with torch.no_grad():
                idx = select(sqk.float(), skq.float(), L, p, kc, n)
        idxs.append(idx)
        qs.append(gather_rows(qc, idx)); ks.append(gather_rows(kc_, idx)); vs.append(gather_rows(vc, idx))
    attn = sdpa_causal(torch.cat(qs, 2), torch.cat(ks, 2), torch.cat(vs, 2))
    outs, off = [], 0
    for c in range(nch):
        m = idxs[c].shape[-1]
        outs.append(scatter_to_base(attn[:, :, off:off + m], idxs[c], n, n, L, p))
        off += m
    return torch.cat(outs, dim=2), idxs


def inverse_map(indices: torch.Tensor, S_tot: int) -> torch.Tensor:
    """inv[bh, pyramid_index] = selected slot, -1 when not selected."""
    B, H, S_sel = indices.shape
    inv = torch.full((B, H, S_tot), -1, dtype=torch.int32)
    inv.scatter_(2, indices.long(), torch.arange(S_sel, dtype=torch.int32).expand(B, H, S_sel).contiguous())
    return inv
