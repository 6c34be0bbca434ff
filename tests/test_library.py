"""The C-ABI ops registered as torch.library custom ops: fake kernels give the
reference geometry on meta tensors, and torch.compile traces the whole layer
(forward and backward) as one graph.  CPU only: meta tensors never reach the
CUDA library."""
import pytest
import torch

from inputs import pyramid_len

GEOMS = [(1, 4096, 2, 128, 3, 4, 256), (2, 8192, 1, 128, 2, 8, 128), (1, 16384, 3, 128, 4, 2, 256)]


def _meta(*shape, dtype=torch.bfloat16):
    return torch.empty(*shape, dtype=dtype, device="meta")


@pytest.mark.parametrize("g", GEOMS)
def test_fake_kernels_give_the_reference_geometry(lh, O, g):
    B, S, H, D, L, p, k = g
    ops = torch.ops.lighthouse_b200
    x = _meta(B, S, H, D)
    S_tot, S_sel = pyramid_len(S, L, p), O.sel_len(S, L, p, k)
    pq, pk, pv, sqk, skq = ops.pyramid_score(x, x, x, L, p)
    assert pq.shape == (B, H, S_tot - S, D) and pq.dtype == x.dtype
    assert sqk.shape == (B, H, S_tot) and sqk.dtype == torch.float32
    idx, inv = ops.select_topk(sqk, skq, L, p, k, S)
    assert idx.shape == (B, H, S_sel) and inv.shape == (B, H, S_tot) and idx.dtype == inv.dtype == torch.int32
    assert ops.build_inverse(idx, S_tot).shape == (B, H, S_tot)
    qs, ks, vs = ops.gather_selected(x, x, x, pq, pk, pv, idx)
    assert qs.shape == (B, H, S_sel, D)
    o, lse = ops.attn_fwd(qs, ks, vs, 0.1, 0)
    assert o.shape == qs.shape and lse.shape == (B, H, S_sel) and lse.dtype == torch.float32
    assert all(t.shape == qs.shape for t in ops.attn_bwd(qs, ks, vs, o, lse, o, 0.1, 0))
    out = ops.scatter_fwd(o, inv, S, S, L, p)
    assert out.shape == (B, H, S, D)
    assert ops.scatter_bwd(out, idx, S, S, L, p).shape == (B, H, S_sel, D)
    assert all(t.shape == (B, S, H, D) for t in ops.unpool_bwd(qs, ks, vs, inv, S, L, p))
    xq, xk = ops.rope_apply(x, x, _meta(S, D // 2, 2, dtype=torch.float32), False)
    assert xq.shape == x.shape
    T = S // 4
    y = _meta(B, T, 4 * H, D)
    o1, o2 = ops.simple_gla_fwd2(y, y, y, _meta(B, T, 4 * H, dtype=torch.float32), 0.1, y, y)
    assert o1.shape == o2.shape == y.shape


def test_layer_compiles_as_one_graph_forward_and_backward(lh):
    B, S, H, D, L, p, k = GEOMS[0]
    from torch._dynamo.testing import CompileCounterWithBackend

    def f(xq, xk, xv):
        return lh.lighthouse_attention(xq, xk, xv, L, p, k)

    torch._dynamo.reset()
    cnt = CompileCounterWithBackend("aot_eager")
    xs = [_meta(B, S, H, D).requires_grad_(True) for _ in range(3)]
    out = torch.compile(f, backend=cnt, fullgraph=True)(*xs)       # fullgraph: a graph break raises
    out.sum().backward()
    assert cnt.frame_count == 1
    assert out.shape == (B, H, S, D) and all(x.grad.shape == x.shape for x in xs)


def test_scorers_trace_on_meta_tensors(lh):
    B, S, H, D, L, p = 1, 4096, 2, 128, 3, 4
    xs = [_meta(B, S, H, D) for _ in range(3)]
    gk = _meta(B, S, H, dtype=torch.float32)
    S_tot = pyramid_len(S, L, p)
    sqk, skq = lh.DilatedLighthouseGLAScorer(D, dilation=4, pooling_factor=p, levels=L).scores(*xs, gk)
    assert sqk.shape == skq.shape == (B, H, S_tot)
    outs = lh.DialatedLighthouseNormScorer(p, L)(*xs)
    assert outs[2].shape == (B, H, S_tot, D)
