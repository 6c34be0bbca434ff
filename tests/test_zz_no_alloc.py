"""lh_attn_bwd_noalloc: the attention backward for callers that may not
allocate device memory during a step (for example a non-Python host that has
no caching allocator and must not call cudaMalloc mid-step).  It uses a
static device array inside the library as its workspace.

Checked through the C ABI against lh_attn_bwd (which takes a caller-owned
workspace) on two calls in a row with different inputs, so that contents the
first call leaves in the shared array cannot leak into the second.  Runs last
(file name) so that a failure here does not hide the other tests."""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def _close(a, b, what):
    a, b = a.float(), b.float()
    m = (a - b).abs().max().item()
    r = ((a - b).norm() / b.norm().clamp_min(1e-12)).item()
    assert m <= MAX_ABS and r <= REL_L2, f"{what}: max-abs {m:.3e} rel-L2 {r:.3e}"


def _case(lh, cuda, B, H, S_q, S_kv, q_off, seed):
    g = torch.Generator().manual_seed(seed)
    mk = lambda n: torch.randn(B, H, n, 128, generator=g).to(torch.bfloat16).to(cuda)
    q, k, v, do = mk(S_q), mk(S_kv), mk(S_kv), mk(S_q)
    scale = 1 / math.sqrt(128)
    o, lse = lh._native.attn_fwd(q, k, v, scale, q_off=q_off)
    ref = lh._native.attn_bwd(q, k, v, o, lse, do, scale, q_off=q_off)       # workspace entry point
    lib = lh._native.load()
    outs = [torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)]
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = lib.lh_attn_bwd_noalloc(P(q), P(k), P(v), P(o), P(lse), P(do), B, H, S_q, S_kv, q_off, 128, scale,
                                 P(outs[0]), P(outs[1]), P(outs[2]),
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.lh_last_error()
    torch.cuda.synchronize()
    for a, b, n in zip(outs, ref, ("dQ", "dK", "dV")):
        _close(a, b, n)


def test_noalloc_matches_workspace_entry_point_twice(lh, cuda):
    _case(lh, cuda, 1, 4, 2048, 2048, 0, seed=1)       # 8192 rows
    _case(lh, cuda, 2, 2, 1000, 3000, 2000, seed=2)    # different geometry; stale contents must not matter
    assert lh._native.device_status() == 0


def test_noalloc_rejects_over_limit(lh, cuda):
    lib = lh._native.load()
    t = torch.empty(1, device=cuda)
    p = ctypes.c_void_p(t.data_ptr())
    rc = lib.lh_attn_bwd_noalloc(p, p, p, p, p, p, 1, 8, 4096, 4096, 0, 128, 1.0, p, p, p, None)
    assert rc == 1 and b"limit" in lib.lh_last_error()
