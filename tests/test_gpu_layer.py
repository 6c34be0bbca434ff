"""End-to-end Lighthouse layer (the drop-in module API) on the GPU vs the oracle."""
import pytest
import torch

from inputs import make_qkv

pytestmark = pytest.mark.gpu


def _err(a, b):
    """(max-abs error beyond one bf16 ulp of the reference value, rel-L2 error).

    The layer's outputs and gradients are stored in bf16, so a result that is
    exact up to its own storage rounding differs from an fp32 reference by up
    to one bf16 ulp (2^-7 |x|); the max-abs bar of 2e-2 applies on top of it."""
    a, b = a.float(), b.float()
    beyond = ((a - b).abs() - b.abs() * 2.0 ** -7).clamp_min(0).max().item()
    return beyond, ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("shape", [(1, 4096, 2, 3, 4, 256), (1, 8192, 2, 3, 2, 256), (1, 16384, 2, 4, 2, 256),
                                   (2, 8192, 2, 2, 8, 128), (1, 8192, 3, 5, 2, 128), (1, 16384, 1, 3, 8, 128),
                                   (3, 4096, 4, 3, 4, 128), (1, 24576, 2, 3, 4, 1536)])
def test_lighthouse_local_fwd_bwd_vs_oracle(lh, O, cuda, shape):
    B, S, H, L, p, k = shape
    D = 128
    xq, xk, xv = make_qkv(B, S, H, D, torch.bfloat16, 17)
    g = torch.Generator().manual_seed(18)
    dout = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    layer = lh.LighthouseLocal(None, lh.DialatedLighthouseNormScorer(p, L), num_levels=L, pooling_factor=p, topk=k)
    xs = [t.to(cuda).requires_grad_(True) for t in (xq, xk, xv)]
    out = layer(*xs)
    out.backward(dout.to(cuda))
    # oracle on the same selection (selection parity is tested on its own)
    _, _, _, sqk, skq = lh._native.pyramid_score(*[t.detach() for t in xs], L, p)
    idx = O.select(sqk.cpu(), skq.cpu(), L, p, k, S)
    xr = [t.float().requires_grad_(True) for t in (xq, xk, xv)]
    ref, _ = O.lighthouse_local(*xr, L, p, k, indices=idx)
    ref.backward(dout.float())
    m, r = _err(out.cpu(), ref)
    assert m <= 2e-2 and r <= 1e-2, f"out max-abs {m:.3e} rel {r:.3e}"
    for a, b, n in zip(xs, xr, "qkv"):
        m, r = _err(a.grad.cpu(), b.grad)
        assert m <= 2e-2 and r <= 1e-2, f"d{n} max-abs {m:.3e} rel {r:.3e}"
    assert lh._native.device_status() == 0


def test_lighthouse_cp_single_rank_vs_oracle(lh, O, cuda):
    B, S, H, D, L, p, k = 1, 16384, 2, 128, 3, 4, 1024
    xq, xk, xv = make_qkv(B, S, H, D, torch.bfloat16, 19)
    layer = lh.LighthouseCP(None, lh.DialatedLighthouseNormScorerCP(p, L), num_levels=L, pooling_factor=p, topk=k)
    xs = [t.to(cuda).requires_grad_(True) for t in (xq, xk, xv)]
    out = layer(*xs)
    dout = torch.randn_like(out)
    out.backward(dout)
    # per-chunk selections from the kernels (selection parity is tested on its own)
    half = S // 2
    idxs = []
    for part in (slice(0, half), slice(half, S)):
        _, _, _, sqk, skq = lh._native.pyramid_score(*[t.detach()[:, part].contiguous() for t in xs], L, p)
        idxs.append(O.select(sqk.cpu(), skq.cpu(), L, p, k // 2, half))
    xr = [t.float().requires_grad_(True) for t in (xq, xk, xv)]
    ref, _ = O.lighthouse_cp_global(*xr, 1, L, p, k, indices=idxs)
    ref.backward(dout.float().cpu())
    m, r = _err(out.cpu(), ref)
    assert m <= 2e-2 and r <= 1e-2, f"cp out max-abs {m:.3e} rel {r:.3e}"
    for a, b, n in zip(xs, xr, "qkv"):
        m, r = _err(a.grad.cpu(), b.grad)
        assert m <= 2e-2 and r <= 1e-2, f"cp d{n} max-abs {m:.3e} rel {r:.3e}"


def test_scorer_module_api(lh, O, cuda):
    B, S, H, D, L, p = 1, 4096, 2, 128, 3, 4
    xq, xk, xv = (t.to(cuda).requires_grad_(True) for t in make_qkv(B, S, H, D, torch.bfloat16, 20))
    sqk, skq, qc, kc, vc = lh.DialatedLighthouseNormScorer(p, L)(xq, xk, xv)
    rq, rk, rqc, rkc, rvc = O.norm_scorer(xq.detach(), xk.detach(), xv.detach(), p, L)
    assert sqk.dtype == torch.bfloat16 and sqk.shape == rq.shape and qc.shape == rqc.shape
    assert (sqk.float() - rq.float()).abs().max().item() <= 0.1
    (qc.float().sum() + 2 * kc.float().sum() + 3 * vc.float().sum()).backward()
    xr = [t.detach().float().requires_grad_(True) for t in (xq, xk, xv)]
    _, _, a, b, c = O.norm_scorer(*xr, p, L)
    (a.sum() + 2 * b.sum() + 3 * c.sum()).backward()
    for x, y in zip((xq, xk, xv), xr):
        assert (x.grad.float() - y.grad).abs().max().item() < 1e-2


def _ref_dilated_scores(xq, xk, xv, di, L, p):
    """The reference dilated scorer's scores (SEL:635-689) in plain PyTorch:
    causal SDPA over the dilated views, bf16 output norms, max over windows."""
    import torch.nn.functional as F
    b, s, h, d = xq.shape
    view = lambda x: x.reshape(b, s // di, di * h, d).transpose(1, 2)
    back = lambda o: o.transpose(1, 2).reshape(b, s, h, d)
    outs = [back(F.scaled_dot_product_attention(view(a), view(c), view(xv), is_causal=True))
            for a, c in ((xq, xk), (xk, xq))]
    res = []
    for o in outs:
        sc = o.norm(dim=-1).transpose(1, 2)                      # (b, h, s) in the input dtype
        levels = [sc] + [sc[..., : (s // p ** l) * p ** l].reshape(b, h, s // p ** l, p ** l).amax(-1)
                         for l in range(1, L)]
        res.append(torch.cat(levels, dim=-1).float())
    return res


@pytest.mark.parametrize("shape", [(1, 8192, 2, 3, 4, 256, 4), (1, 16384, 2, 3, 4, 512, 2)])
def test_dilated_scorer_and_layer(lh, O, cuda, shape):
    B, S, H, L, p, k, di = shape
    D = 128
    xq, xk, xv = make_qkv(B, S, H, D, torch.bfloat16, 23)
    scorer = lh.DilatedLighthouseScorer(head_dim=D, dilation=di, pooling_factor=p, levels=L)   # patch signature
    xs = [t.to(cuda).requires_grad_(True) for t in (xq, xk, xv)]
    sqk, skq = scorer.scores(*[t.detach() for t in xs])
    rqk, rkq = _ref_dilated_scores(*[t.detach() for t in xs], di, L, p)
    for ours, ref in ((sqk, rqk), (skq, rkq)):       # different attention kernels: within two bf16 ulps
        assert ((ours - ref).abs() <= 2 * 2.0 ** -7 * ref.abs() + 1e-6).all()
    # the scorer module's outputs have the reference's shapes and pyramids
    s_qk, s_kq, qc, kc, vc = scorer(*xs)
    assert s_qk.shape == (B, H, O.pyramid_len(S, L, p)) and qc.shape == (B, H, O.pyramid_len(S, L, p), D)
    _, _, rqc, _, _ = O.norm_scorer(xq.to(cuda), xk.to(cuda), xv.to(cuda), p, L)
    assert ((qc.detach().float() - rqc.float()).abs() <= 2.0 ** -7 * rqc.float().abs() + 1e-6).all()
    # the layer with the dilated scores vs the oracle on the same selection
    g = torch.Generator().manual_seed(24)
    dout = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    layer = lh.LighthouseLocal(None, scorer, num_levels=L, pooling_factor=p, topk=k)
    out = layer(*xs)
    out.backward(dout.to(cuda))
    idx = O.select(sqk.cpu(), skq.cpu(), L, p, k, S)
    xr = [t.float().requires_grad_(True) for t in (xq, xk, xv)]
    ref, _ = O.lighthouse_local(*xr, L, p, k, indices=idx)
    ref.backward(dout.float())
    m, r = _err(out.cpu(), ref)
    assert m <= 2e-2 and r <= 1e-2, f"out max-abs {m:.3e} rel {r:.3e}"
    for a, b, n in zip(xs, xr, "qkv"):
        m, r = _err(a.grad.cpu(), b.grad)
        assert m <= 2e-2 and r <= 1e-2, f"d{n} max-abs {m:.3e} rel {r:.3e}"
    assert lh._native.device_status() == 0


def test_lighthouse_local_baseline_config2_vs_oracle(lh, O, cuda):
    """BASELINE config 2 (B=1, S=65536, H=8, D=128, L=3, p=4, k=2048) through the
    module API, forward + backward, all eight heads on the GPU; heads 0 and 5
    checked against the fp32 oracle layer (run on the GPU, math SDPA) on the
    kernels' own selection."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    B, S, H, D, L, p, k = 1, 65536, 8, 128, 3, 4, 2048
    xq, xk, xv = make_qkv(B, S, H, D, torch.bfloat16, 0)
    g = torch.Generator().manual_seed(1)
    dout = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    layer = lh.LighthouseLocal(None, lh.DialatedLighthouseNormScorer(p, L), num_levels=L, pooling_factor=p, topk=k)
    xs = [t.to(cuda).requires_grad_(True) for t in (xq, xk, xv)]
    out = layer(*xs)
    out.backward(dout.to(cuda))
    _, _, _, sqk, skq = lh._native.pyramid_score(*[t.detach() for t in xs], L, p)
    idx = lh._native.select_topk(sqk, skq, L, p, k, S)[0]
    assert idx.shape == (B, H, O.sel_len(S, L, p, k))
    heads = [0, 5]
    xr = [t[:, :, heads].float().to(cuda).requires_grad_(True) for t in (xq, xk, xv)]
    with sdpa_kernel(SDPBackend.MATH):
        ref, _ = O.lighthouse_local(*xr, L, p, k, indices=idx[:, heads])
        ref.backward(dout[:, heads].float().to(cuda))
    m, r = _err(out[:, heads].detach(), ref.detach())
    assert m <= 2e-2 and r <= 1e-2, f"out max-abs {m:.3e} rel {r:.3e}"
    for a, b, n in zip(xs, xr, "qkv"):
        m, r = _err(a.grad[:, :, heads], b.grad)
        assert m <= 2e-2 and r <= 1e-2, f"d{n} max-abs {m:.3e} rel {r:.3e}"
    assert lh._native.device_status() == 0
