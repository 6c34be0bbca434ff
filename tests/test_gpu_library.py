"""The lighthouse_b200:: custom ops on the GPU: torch.library.opcheck (schema:
no input mutation or aliasing; fake kernels agree with the real outputs'
shapes, dtypes and strides) and the layer compiled by torch.compile (inductor,
full graph) against eager, bit for bit."""
import math

import pytest
import torch

from inputs import make_qkv

pytestmark = pytest.mark.gpu

UTILS = ("test_schema", "test_faketensor")


def _layer_args(cuda, B=1, S=4096, H=2, L=3, p=4, k=256):
    xq, xk, xv = (t.to(cuda) for t in make_qkv(B, S, H, 128, torch.bfloat16, 71))
    return xq, xk, xv, L, p, k


def test_opcheck_every_op(lh, cuda):
    ops = torch.ops.lighthouse_b200
    xq, xk, xv, L, p, k = _layer_args(cuda)
    S = xq.shape[1]
    torch.library.opcheck(ops.pyramid_score, (xq, xk, xv, L, p), test_utils=UTILS)
    pq, pk, pv, sqk, skq = ops.pyramid_score(xq, xk, xv, L, p)
    torch.library.opcheck(ops.select_topk, (sqk, skq, L, p, k, S), test_utils=UTILS)
    idx, inv = ops.select_topk(sqk, skq, L, p, k, S)
    torch.library.opcheck(ops.build_inverse, (idx, sqk.shape[-1]), test_utils=UTILS)
    torch.library.opcheck(ops.gather_selected, (xq, xk, xv, pq, pk, pv, idx), test_utils=UTILS)
    qs, ks, vs = ops.gather_selected(xq, xk, xv, pq, pk, pv, idx)
    scale = 1 / math.sqrt(128)
    torch.library.opcheck(ops.attn_fwd, (qs, ks, vs, scale, 0), test_utils=UTILS)
    o, lse = ops.attn_fwd(qs, ks, vs, scale, 0)
    torch.library.opcheck(ops.attn_bwd, (qs, ks, vs, o, lse, o, scale, 0), test_utils=UTILS)
    torch.library.opcheck(ops.scatter_fwd, (o, inv, S, S, L, p), test_utils=UTILS)
    out = ops.scatter_fwd(o, inv, S, S, L, p)
    torch.library.opcheck(ops.scatter_bwd, (out, idx, S, S, L, p), test_utils=UTILS)
    torch.library.opcheck(ops.unpool_bwd, (qs, ks, vs, inv, S, L, p), test_utils=UTILS)
    table = torch.randn(S, 64, 2, device=cuda)
    torch.library.opcheck(ops.rope_apply, (xq, xk, table, False), test_utils=UTILS)
    y = xq.reshape(1, S // 4, 8, 128)
    g = torch.nn.functional.logsigmoid(torch.randn(1, S // 4, 8, device=cuda))
    torch.library.opcheck(ops.simple_gla_fwd2, (y, y, y, g, 0.1, y, y), test_utils=UTILS)
    assert lh._native.device_status() == 0


def test_compiled_layer_equals_eager(lh, cuda):
    xq, xk, xv, L, p, k = _layer_args(cuda, B=2, S=8192, H=2, L=3, p=4, k=256)
    dout = torch.randn(2, 2, 8192, 128, device=cuda).to(torch.bfloat16)

    def f(a, b, c):
        return lh.lighthouse_attention(a, b, c, L, p, k)

    def run(fn):
        xs = [t.detach().clone().requires_grad_(True) for t in (xq, xk, xv)]
        out = fn(*xs)
        out.backward(dout)
        return out.detach(), [x.grad for x in xs]

    torch._dynamo.reset()
    out_c, g_c = run(torch.compile(f, fullgraph=True))
    out_e, g_e = run(f)
    assert torch.equal(out_c, out_e)
    for a, b in zip(g_c, g_e):
        assert torch.equal(a, b)
    assert lh._native.device_status() == 0
