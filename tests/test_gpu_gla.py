"""The `gla` scorer on the GPU: the simple-GLA kernel (csrc/gla.cu) against the
oracle's recurrence, a plain PyTorch fp32 evaluation of the closed form, and the
reference's own dependency (fla's chunk_simple_gla) where it imports; the scorer
against the reference golden vectors; the layer with GLA scores against the oracle."""
import math

import pytest
import torch

from inputs import GLA_CASES, make_gate, make_qkv

pytestmark = pytest.mark.gpu

# bf16 operands inside the chunked evaluation (scores, decayed values, the state
# as a matmul operand) and bf16 outputs: relative L2 error at most 1e-2, no
# element off by more than 3 % of the largest output magnitude.
REL_L2 = 1e-2
MAX_FRAC = 3e-2


def _close(a, b, what):
    a, b = a.float(), b.float()
    r = ((a - b).norm() / b.norm().clamp_min(1e-12)).item()
    m = ((a - b).abs().max() / b.abs().max().clamp_min(1e-12)).item()
    assert r <= REL_L2 and m <= MAX_FRAC, f"{what}: rel-L2 {r:.3e} max/|max| {m:.3e}"


def _inputs(B, T, H, div, seed, device):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, T, H, 128, generator=g).to(torch.bfloat16).to(device) for _ in range(3))
    gate = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, generator=g)) / div).to(device)
    return q, k, v, gate


def _closed_form(q, k, v, g, scale):
    """o_t = scale sum_{s<=t} exp(G_t - G_s) (q_t . k_s) v_s in fp32 (quadratic in T)."""
    q, k, v = q.float(), k.float(), v.float()
    G = g.float().cumsum(1)
    T = q.shape[1]
    dec = (G[:, :, None, :] - G[:, None, :, :]).clamp_max(0).exp()
    A = torch.einsum("bthd,bshd->btsh", q, k) * dec * torch.ones(T, T, dtype=torch.bool, device=q.device).tril()[
        None, :, :, None]
    return scale * torch.einsum("btsh,bshd->bthd", A, v)


@pytest.mark.parametrize("shape", [(1, 10, 1, 16.0), (1, 64, 2, 16.0), (2, 200, 3, 1.0), (1, 333, 2, 1000.0)])
def test_simple_gla_vs_oracle_recurrence(lh, O, cuda, shape):
    B, T, H, div = shape
    q, k, v, g = _inputs(B, T, H, div, 61, cuda)
    scale = 1 / math.sqrt(128)
    o = lh._native.simple_gla_fwd(q, k, v, g, scale)
    assert o.dtype == torch.bfloat16 and o.shape == q.shape
    _close(o.cpu(), O.simple_gla(q.cpu().float(), k.cpu().float(), v.cpu().float(), g.cpu(), scale), "o")
    assert lh._native.device_status() == 0


@pytest.mark.parametrize("shape", [(1, 2048, 8, 16.0), (2, 1000, 4, 4.0), (1, 4096, 4, 200.0)])
def test_simple_gla_two_passes_vs_closed_form(lh, cuda, shape):
    B, T, H, div = shape
    q, k, v, g = _inputs(B, T, H, div, 62, cuda)
    scale = 1 / math.sqrt(128)
    o1, o2 = lh._native.simple_gla_fwd(q, k, v, g, scale, q2=k, k2=q)
    _close(o1, _closed_form(q, k, v, g, scale), "q->k")
    _close(o2, _closed_form(k, q, v, g, scale), "k->q")
    # the single-pass launch computes the same first pass bit for bit
    assert torch.equal(lh._native.simple_gla_fwd(q, k, v, g, scale), o1)


def test_simple_gla_vs_fla_chunk_simple_gla(lh, cuda):
    """The function the reference scorer calls (fla 0.5.1), on its Triton kernels."""
    try:
        from fla.ops.simple_gla import chunk_simple_gla
    except Exception as e:                                    # noqa: BLE001
        pytest.skip(f"fla not importable: {e}")
    B, T, H = 1, 8192, 8
    q, k, v, g = _inputs(B, T, H, 16.0, 63, cuda)
    scale = 1 / math.sqrt(128)
    try:
        ref, _ = chunk_simple_gla(q, k, v, g, scale=scale)
    except Exception as e:                                    # noqa: BLE001
        pytest.skip(f"fla's Triton kernels did not run here: {type(e).__name__}")
    _close(lh._native.simple_gla_fwd(q, k, v, g, scale), ref, "vs fla")


@pytest.mark.parametrize("name", [n for n, c in GLA_CASES.items() if c[3] == 128])
def test_gla_scorer_vs_reference_golden(lh, O, golden, cuda, name):
    B, S, H, D, di, L, p, dtype, div, seed = GLA_CASES[name]
    xq, xk, xv = make_qkv(B, S, H, D, dtype, seed)
    gk = make_gate(B, S, H, div, seed)
    scorer = lh.DilatedLighthouseGLAScorer(head_dim=D, dilation=di, pooling_factor=p, levels=L)
    sqk, skq, qc, _, _ = scorer(*(t.to(cuda) for t in (xq, xk, xv, gk)))
    g = golden["gla"]
    for ours, key in ((sqk, "scores_qk"), (skq, "scores_kq")):
        ref = torch.from_numpy(g[f"{name}/{key}"])
        ours = ours.float().cpu()
        # norms of 128 bf16 outputs: within four bf16 ulps of the reference's
        assert ((ours - ref).abs() <= 2.0 ** -5 * ref.abs() + 1e-3).all(), key
        assert ((ours - ref).norm() / ref.norm()).item() < 4e-3, key
    _, _, rqc, _, _ = O.norm_scorer(xq, xk, xv, p, L)
    assert ((qc.float().cpu() - rqc.float()).abs() <= 2.0 ** -7 * rqc.float().abs() + 1e-6).all()


def _err(a, b):
    a, b = a.float(), b.float()
    beyond = ((a - b).abs() - b.abs() * 2.0 ** -7).clamp_min(0).max().item()
    return beyond, ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("shape", [(1, 8192, 2, 3, 4, 256, 4), (2, 4096, 2, 2, 4, 256, 2)])
def test_layer_with_gla_scores_vs_oracle(lh, O, cuda, shape):
    B, S, H, L, p, k, di = shape
    D = 128
    xq, xk, xv = make_qkv(B, S, H, D, torch.bfloat16, 64)
    gk = make_gate(B, S, H, 16.0, 64)
    scorer = lh.DilatedLighthouseGLAScorer(head_dim=D, dilation=di, pooling_factor=p, levels=L)
    layer = lh.LighthouseLocal(None, scorer, num_levels=L, pooling_factor=p, topk=k)
    xs = [t.to(cuda).requires_grad_(True) for t in (xq, xk, xv)]
    sqk, skq = scorer.scores(*[t.detach() for t in xs], gk.to(cuda))
    g = torch.Generator().manual_seed(65)
    dout = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    out = layer(*xs, gk=gk.to(cuda))                           # the patch's keyword call
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
    with pytest.raises(ValueError):
        layer(*xs)                                             # the GLA scorer needs its gate
    assert lh._native.device_status() == 0


def test_simple_gla_rejects_bad_shapes(lh, cuda):
    q = torch.zeros(1, 64, 2, 64, dtype=torch.bfloat16, device=cuda)
    g = torch.zeros(1, 64, 2, device=cuda)
    with pytest.raises(lh._native.LighthouseShapeError):
        lh._native.simple_gla_fwd(q, q, q, g, 0.1)             # head_dim 64
