"""ctypes binding of liblighthouse_b200.so (the C ABI in include/lighthouse_b200.h).

Every wrapper takes torch CUDA tensors, checks dtype / layout / device,
allocates outputs with torch's caching allocator on the input's device and
enqueues the kernels on ``torch.cuda.current_stream()``.  There is no CPU or
eager-PyTorch fallback: if the library is missing or the device is not a
B200 the call raises.
"""
from __future__ import annotations

import ctypes
import pathlib

import torch

_LIB_PATH = pathlib.Path(__file__).resolve().parent / "liblighthouse_b200.so"
_lib = None

LH_DTYPE = {torch.bfloat16: 0, torch.float32: 1}
_VP = ctypes.c_void_p


class LighthouseError(RuntimeError):
    """Raised when a C-ABI entry point returns a non-zero status."""


class LighthouseShapeError(ValueError):
    """The C ABI rejected a shape (LH_ERR_SHAPE)."""


_SIGS = {
    "lh_last_error": (ctypes.c_char_p, []),
    "lh_abi_version": (ctypes.c_int, []),
    "lh_device_status": (ctypes.c_int, [ctypes.c_int]),
    "lh_pyramid_score_fwd": (ctypes.c_int, [_VP, _VP, _VP, ctypes.c_int] + [ctypes.c_int] * 6 + [_VP] * 6),
    "lh_select_topk": (ctypes.c_int, [_VP, _VP] + [ctypes.c_int] * 6 + [_VP, _VP, _VP]),
    "lh_build_inverse": (ctypes.c_int, [_VP] + [ctypes.c_int] * 4 + [_VP, _VP]),
    "lh_gather_selected": (ctypes.c_int, [_VP] * 6 + [ctypes.c_int] * 6 + [_VP, ctypes.c_int] + [_VP] * 4),
    "lh_attn_fwd": (ctypes.c_int, [_VP] * 3 + [ctypes.c_int] * 6 + [ctypes.c_float, _VP, _VP, _VP]),
    "lh_attn_bwd_workspace_size": (ctypes.c_size_t, [ctypes.c_int] * 5),
    "lh_attn_merge": (ctypes.c_int, [_VP] * 4 + [ctypes.c_longlong, ctypes.c_int, _VP, _VP, _VP]),
    "lh_attn_bwd": (ctypes.c_int, [_VP] * 6 + [ctypes.c_int] * 6 + [ctypes.c_float] + [_VP] * 4
                    + [ctypes.c_size_t, _VP]),
    "lh_attn_bwd_noalloc": (ctypes.c_int, [_VP] * 6 + [ctypes.c_int] * 6 + [ctypes.c_float] + [_VP] * 4),
    "lh_scatter_fwd": (ctypes.c_int, [_VP, _VP] + [ctypes.c_int] * 9 + [_VP, _VP]),
    "lh_scatter_bwd": (ctypes.c_int, [_VP, _VP] + [ctypes.c_int] * 9 + [_VP, _VP]),
    "lh_scatter_fwd_token_major": (ctypes.c_int, [_VP, _VP] + [ctypes.c_int] * 9 + [_VP, _VP]),
    "lh_scatter_bwd_token_major": (ctypes.c_int, [_VP, _VP] + [ctypes.c_int] * 9 + [_VP, _VP]),
    "lh_unpool_bwd": (ctypes.c_int, [_VP] * 4 + [ctypes.c_int] * 8 + [_VP] * 4),
    "lh_rope_apply": (ctypes.c_int, [_VP] * 5 + [ctypes.c_int] * 6 + [_VP]),
    "lh_simple_gla_fwd": (ctypes.c_int, [_VP] * 8 + [ctypes.c_int] * 5 + [ctypes.c_float, _VP]),
}


def lib_path() -> pathlib.Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            raise ImportError(
                f"{_LIB_PATH} is not built; run `python lighthouse-attention_b200/build.py` "
                "(the CUDA path has no fallback)")
        lib = ctypes.CDLL(str(_LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def _check(rc: int) -> None:
    if rc != 0:
        msg = load().lh_last_error().decode(errors="replace")
        if rc == 1:
            raise LighthouseShapeError(msg)
        raise LighthouseError(f"lighthouse_b200 error {rc}: {msg}")


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("lighthouse_b200 ops take CUDA tensors (no CPU path)")


def device_status(reset: bool = True) -> int:
    return load().lh_device_status(1 if reset else 0)


# --------------------------------------------------------------------------- geometry
def pyramid_len(N: int, L: int, p: int) -> int:
    return sum(N // p ** l for l in range(L))


def sel_len(N: int, L: int, p: int, k: int) -> int:
    return N // p ** (L - 1) + (L - 1) * p * k


# --------------------------------------------------------------------------- ops
def pyramid_score(xq, xk, xv, L: int, p: int):
    """(B,S,H,D) x3 -> pooled q/k/v (B,H,S_pool,D), scores_qk/kq (B,H,S_tot) fp32."""
    _require_cuda(xq, xk, xv)
    xq, xk, xv = xq.contiguous(), xk.contiguous(), xv.contiguous()
    B, S, H, D = xq.shape
    S_tot = pyramid_len(S, L, p)
    S_pool = S_tot - S
    pq = torch.empty(B, H, S_pool, D, dtype=xq.dtype, device=xq.device)
    pk, pv = torch.empty_like(pq), torch.empty_like(pq)
    sqk = torch.empty(B, H, S_tot, dtype=torch.float32, device=xq.device)
    skq = torch.empty_like(sqk)
    _check(load().lh_pyramid_score_fwd(_ptr(xq), _ptr(xk), _ptr(xv), LH_DTYPE[xq.dtype], B, S, H, D, L, p,
                                       _ptr(pq), _ptr(pk), _ptr(pv), _ptr(sqk), _ptr(skq), _stream()))
    return pq, pk, pv, sqk, skq


def select_topk(scores_qk, scores_kq, L: int, p: int, k: int, N: int, with_inverse: bool = True):
    """Selection indices (B,H,S_sel) int32 and inverse map (B,H,S_tot) int32."""
    _require_cuda(scores_qk, scores_kq)
    if scores_qk.shape != scores_kq.shape:
        raise AssertionError("scores_qk and scores_kq must have the same shape")
    sq = scores_qk.float().contiguous()
    sk = scores_kq.float().contiguous()
    B, H, S_tot = sq.shape
    if S_tot != pyramid_len(N, L, p):
        raise LighthouseShapeError(f"scores length {S_tot} != pyramid length {pyramid_len(N, L, p)}")
    S_sel = sel_len(N, L, p, k)
    idx = torch.empty(B, H, S_sel, dtype=torch.int32, device=sq.device)
    inv = torch.empty(B, H, S_tot, dtype=torch.int32, device=sq.device) if with_inverse else None
    _check(load().lh_select_topk(_ptr(sq), _ptr(sk), B, H, N, L, p, k, _ptr(idx), _ptr(inv), _stream()))
    return idx, inv


def build_inverse(indices, S_tot: int):
    _require_cuda(indices)
    indices = indices.to(torch.int32).contiguous()
    B, H, S_sel = indices.shape
    inv = torch.empty(B, H, S_tot, dtype=torch.int32, device=indices.device)
    _check(load().lh_build_inverse(_ptr(indices), B, H, S_sel, S_tot, _ptr(inv), _stream()))
    return inv


def gather_selected(raws, pooleds, indices):
    """raws: 3 tensors (B,S,H,D) (or None); pooleds: 3 tensors (B,H,S_pool,D)."""
    first = next(r for r in raws if r is not None)
    B, S, H, D = first.shape
    S_pool = next(p for p in pooleds if p is not None).shape[2]
    S_sel = indices.shape[-1]
    outs = [None if r is None else torch.empty(B, H, S_sel, D, dtype=r.dtype, device=r.device) for r in raws]
    raws = [None if r is None else r.contiguous() for r in raws]
    pooleds = [None if p is None else p.contiguous() for p in pooleds]
    _check(load().lh_gather_selected(*[_ptr(r) for r in raws], *[_ptr(p) for p in pooleds],
                                     LH_DTYPE[first.dtype], B, S, H, D, S_pool, _ptr(indices), S_sel,
                                     *[_ptr(o) for o in outs], _stream()))
    return outs


def _attn_operands(*ts):
    _require_cuda(*ts)
    for t in ts:
        if t.dtype != torch.bfloat16 or t.shape[-1] != 128:
            raise ValueError("attention kernels take bf16 tensors with head dim 128")
    return [t.contiguous() for t in ts]


def attn_fwd(q, k, v, scale: float, q_off: int = 0):
    """Causal attention; query row r at position q_off + r, key row c at c."""
    q, k, v = _attn_operands(q, k, v)
    B, H, S_q, D = q.shape
    S_kv = k.shape[2]
    o = torch.empty_like(q)
    lse = torch.empty(B, H, S_q, dtype=torch.float32, device=q.device)
    _check(load().lh_attn_fwd(_ptr(q), _ptr(k), _ptr(v), B, H, S_q, S_kv, q_off, D, scale, _ptr(o), _ptr(lse),
                              _stream()))
    return o, lse


def attn_merge(o1, lse1, o2, lse2):
    """Log-sum-exp merge of two partial attentions of the same queries over
    disjoint key sets: (o, lse), o bf16 (..., D), lse fp32 (...)."""
    o1, o2 = _attn_operands(o1, o2)
    lse1, lse2 = lse1.float().contiguous(), lse2.float().contiguous()
    if o1.shape != o2.shape or lse1.shape != o1.shape[:-1] or lse2.shape != lse1.shape:
        raise LighthouseShapeError("attn_merge: o1/o2 and lse1/lse2 must agree")
    o = torch.empty_like(o1)
    lse = torch.empty_like(lse1)
    _check(load().lh_attn_merge(_ptr(o1), _ptr(lse1), _ptr(o2), _ptr(lse2), lse1.numel(), o1.shape[-1], _ptr(o),
                                _ptr(lse), _stream()))
    return o, lse


def attn_bwd_workspace_size(B: int, H: int, S_q: int, S_kv: int, D: int) -> int:
    return int(load().lh_attn_bwd_workspace_size(B, H, S_q, S_kv, D))


def attn_bwd(q, k, v, o, lse, do, scale: float, q_off: int = 0):
    q, k, v, o, do = _attn_operands(q, k, v, o, do)
    B, H, S_q, D = q.shape
    S_kv = k.shape[2]
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ws_bytes = attn_bwd_workspace_size(B, H, S_q, S_kv, D)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    _check(load().lh_attn_bwd(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse.contiguous()), _ptr(do), B, H, S_q,
                              S_kv, q_off, D, scale, _ptr(dq), _ptr(dk), _ptr(dv), _ptr(ws), ws_bytes, _stream()))
    return dq, dk, dv


def scatter_fwd(attn, inverse, N_shard: int, N_total: int, L: int, p: int):
    attn = attn.contiguous()
    B, H, S_sel, D = attn.shape
    out = torch.empty(B, H, N_total, D, dtype=attn.dtype, device=attn.device)
    _check(load().lh_scatter_fwd(_ptr(attn), _ptr(inverse), LH_DTYPE[attn.dtype], B, H, S_sel, D, N_shard, N_total,
                                 L, p, _ptr(out), _stream()))
    return out


def token_major_ok(B: int, H: int, D: int, dtype) -> bool:
    """Whether the token-major scatter kernels cover this geometry."""
    row = D * (2 if dtype == torch.bfloat16 else 4)
    return row in (256, 512) and (B * H) % (32 // (row // 16)) == 0


def scatter_fwd_token_major(attn, inverse, N_shard: int, N_total: int, L: int, p: int):
    """scatter_fwd with the output as (B, N_total, H, D) (token-major)."""
    attn = attn.contiguous()
    B, H, S_sel, D = attn.shape
    out = torch.empty(B, N_total, H, D, dtype=attn.dtype, device=attn.device)
    _check(load().lh_scatter_fwd_token_major(_ptr(attn), _ptr(inverse), LH_DTYPE[attn.dtype], B, H, S_sel, D,
                                             N_shard, N_total, L, p, _ptr(out), _stream()))
    return out


def scatter_bwd_token_major(dout, indices, N_shard: int, N_total: int, L: int, p: int):
    """scatter_bwd for dout given as (B, N_total, H, D) (token-major)."""
    dout = dout.contiguous()
    B, _, H, D = dout.shape
    S_sel = indices.shape[-1]
    dattn = torch.empty(B, H, S_sel, D, dtype=dout.dtype, device=dout.device)
    _check(load().lh_scatter_bwd_token_major(_ptr(dout), _ptr(indices), LH_DTYPE[dout.dtype], B, H, S_sel, D,
                                             N_shard, N_total, L, p, _ptr(dattn), _stream()))
    return dattn


def scatter_bwd(dout, indices, N_shard: int, N_total: int, L: int, p: int):
    dout = dout.contiguous()
    B, H, _, D = dout.shape
    S_sel = indices.shape[-1]
    dattn = torch.empty(B, H, S_sel, D, dtype=dout.dtype, device=dout.device)
    _check(load().lh_scatter_bwd(_ptr(dout), _ptr(indices), LH_DTYPE[dout.dtype], B, H, S_sel, D, N_shard,
                                 N_total, L, p, _ptr(dattn), _stream()))
    return dattn


def unpool_bwd(dsels, inverse, S: int, L: int, p: int):
    first = next(d for d in dsels if d is not None)
    B, H, S_sel, D = first.shape
    dsels = [None if d is None else d.contiguous() for d in dsels]
    outs = [None if d is None else torch.empty(B, S, H, D, dtype=d.dtype, device=d.device) for d in dsels]
    _check(load().lh_unpool_bwd(*[_ptr(d) for d in dsels], _ptr(inverse), LH_DTYPE[first.dtype], B, S, H, D, L, p,
                                S_sel, *[_ptr(o) for o in outs], _stream()))
    return outs


def rope_apply(xq, xk, table, inverse: bool = False):
    """Rotary embedding of q and k (B, S, H, D) with the (S, D/2, 2) fp32 (cos, sin)
    table; returns new tensors.  inverse=True rotates by minus the angles."""
    xq, xk, table = xq.contiguous(), xk.contiguous(), table.contiguous()
    B, S, H, D = xq.shape
    if xk.shape != xq.shape or xk.dtype != xq.dtype or tuple(table.shape) != (S, D // 2, 2):
        raise LighthouseShapeError("rope: q, k and the table must agree")
    oq, ok = torch.empty_like(xq), torch.empty_like(xk)
    _check(load().lh_rope_apply(_ptr(xq), _ptr(xk), _ptr(oq), _ptr(ok), _ptr(table), LH_DTYPE[xq.dtype],
                                B, S, H, D, int(inverse), _stream()))
    return oq, ok



def simple_gla_fwd(q, k, v, g, scale: float, q2=None, k2=None):
    """Simple GLA forward (fla's chunk_simple_gla, zero initial state) of (B, T, H, 128)
    bf16 q/k/v with the (B, T, H) log-gate g; returns o, or (o, o2) when the second
    pass (q2, k2) sharing v and g is given."""
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    g = g.float().contiguous()
    B, T, H, D = q.shape
    if k.shape != q.shape or v.shape != q.shape or tuple(g.shape) != (B, T, H):
        raise LighthouseShapeError("gla: q, k, v (B, T, H, D) and g (B, T, H) must agree")
    o = torch.empty_like(q)
    o2 = None
    if q2 is not None:
        q2, k2 = q2.contiguous(), k2.contiguous()
        if q2.shape != q.shape or k2.shape != q.shape:
            raise LighthouseShapeError("gla: the second pass must have the shape of the first")
        o2 = torch.empty_like(q)
    _check(load().lh_simple_gla_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(o), _ptr(q2), _ptr(k2), _ptr(o2),
                                    LH_DTYPE[q.dtype], B, T, H, D, scale, _stream()))
    return o if q2 is None else (o, o2)
