"""GPU parity of the tcgen05 causal attention (forward / backward) against a
plain PyTorch fp32 reference of the same op.  Tolerances (bf16): max-abs 2e-2
and rel-L2 1e-2, the bar stated for attention outputs and gradients."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def ref_attention(q, k, v, q_off):
    """fp32 causal attention: query row r at position q_off + r, key c at c."""
    qf, kf, vf = q.float(), k.float(), v.float()
    S_q, S_kv = q.shape[2], k.shape[2]
    s = qf @ kf.transpose(-1, -2) / math.sqrt(q.shape[-1])
    pos_q = torch.arange(S_q, device=q.device)[:, None] + q_off
    pos_k = torch.arange(S_kv, device=q.device)[None, :]
    s = s.masked_fill(pos_k > pos_q, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    return torch.softmax(s, dim=-1) @ vf, lse


def _check(ours, ref, what):
    ours, ref = ours.float(), ref.float()
    max_abs = (ours - ref).abs().max().item()
    rel = ((ours - ref).norm() / ref.norm().clamp_min(1e-12)).item()
    assert max_abs <= MAX_ABS and rel <= REL_L2, f"{what}: max-abs {max_abs:.3e} rel-L2 {rel:.3e}"


def _inputs(B, H, S_q, S_kv, seed, device):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, S_q, 128, generator=g).to(torch.bfloat16).to(device)
    k = torch.randn(B, H, S_kv, 128, generator=g).to(torch.bfloat16).to(device)
    v = torch.randn(B, H, S_kv, 128, generator=g).to(torch.bfloat16).to(device)
    do = torch.randn(B, H, S_q, 128, generator=g).to(torch.bfloat16).to(device)
    return q, k, v, do


CASES = [  # (B, H, S_q, S_kv, q_off)
    (1, 1, 128, 128, 0), (1, 2, 256, 256, 0), (2, 3, 1000, 1000, 0), (1, 2, 4096, 4096, 0),
    (1, 2, 256, 1024, 512), (1, 1, 384, 1152, 768), (1, 2, 200, 700, 500),
]


@pytest.mark.parametrize("case", CASES)
def test_attn_fwd_vs_fp32_reference(lh, cuda, case):
    B, H, S_q, S_kv, q_off = case
    q, k, v, _ = _inputs(B, H, S_q, S_kv, 1, cuda)
    o, lse = lh._native.attn_fwd(q, k, v, 1 / math.sqrt(128), q_off=q_off)
    ro, rlse = ref_attention(q, k, v, q_off)
    assert lh._native.device_status() == 0
    _check(o, ro, "O")
    assert (lse - rlse).abs().max().item() < 1e-3


def test_attn_fwd_matches_sdpa_at_selected_length(lh, cuda):
    q, k, v, _ = _inputs(1, 8, 20480, 20480, 2, cuda)
    o, _ = lh._native.attn_fwd(q, k, v, 1 / math.sqrt(128))
    ro = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=True)
    _check(o, ro, "O @ S_sel=20480")


def test_attn_fwd_large_logits(lh, cuda):
    # scaled scores well beyond the 2^8 rescale threshold exercise the O rescale path
    q, k, v, _ = _inputs(1, 2, 1024, 1024, 3, cuda)
    q = (q.float() * 6).to(torch.bfloat16)
    o, _ = lh._native.attn_fwd(q, k, v, 1 / math.sqrt(128))
    ro, _ = ref_attention(q, k, v, 0)
    _check(o, ro, "O large logits")


@pytest.mark.parametrize("case", CASES)
def test_attn_bwd_vs_fp32_reference(lh, cuda, case):
    B, H, S_q, S_kv, q_off = case
    q, k, v, do = _inputs(B, H, S_q, S_kv, 4, cuda)
    scale = 1 / math.sqrt(128)
    o, lse = lh._native.attn_fwd(q, k, v, scale, q_off=q_off)
    dq, dk, dv = lh._native.attn_bwd(q, k, v, o, lse, do, scale, q_off=q_off)
    qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
    ro, _ = ref_attention(qr, kr, vr, q_off)
    ro.backward(do.float())
    assert lh._native.device_status() == 0
    _check(dq, qr.grad, "dQ")
    _check(dk, kr.grad, "dK")
    _check(dv, vr.grad, "dV")


def _ref_fwd_bwd_chunked(q, k, v, do, scale, chunk=2048):
    """fp32 causal attention forward + backward for one (b, h) slice, in query
    chunks so that no S x S matrix is held at once:
    P = softmax(scale QK^T + mask), O = PV, Delta = rowsum(dO * O),
    dS = P * (dO V^T - Delta), dQ = scale dS K, dK = scale dS^T Q, dV = P^T dO."""
    qf, kf, vf, dof = q.float(), k.float(), v.float(), do.float()
    S = qf.shape[0]
    o = torch.empty_like(qf)
    dq = torch.empty_like(qf)
    dk = torch.zeros_like(kf)
    dv = torch.zeros_like(vf)
    kpos = torch.arange(S, device=q.device)[None, :]
    for c0 in range(0, S, chunk):
        c1 = min(S, c0 + chunk)
        qpos = torch.arange(c0, c1, device=q.device)[:, None]
        s = (qf[c0:c1] @ kf[:c1].T) * scale
        s = s.masked_fill(kpos[:, :c1] > qpos, float("-inf"))
        p = torch.softmax(s, dim=-1)
        del s
        o[c0:c1] = p @ vf[:c1]
        delta = (dof[c0:c1] * o[c0:c1]).sum(-1, keepdim=True)
        ds = p * (dof[c0:c1] @ vf[:c1].T - delta)
        dv[:c1] += p.T @ dof[c0:c1]
        del p
        dq[c0:c1] = (ds @ kf[:c1]) * scale
        dk[:c1] += (ds.T @ qf[c0:c1]) * scale
    return o, dq, dk, dv


@pytest.mark.parametrize("S_sel", [20480, 24576])
def test_attn_fwd_bwd_at_product_selected_lengths(lh, cuda, S_sel):
    """The selected lengths the layer runs at BASELINE configs 2 (S=65536,
    k=2048: S_sel=20480) and 3 (S=131072, k=2048: S_sel=24576), all 8 heads in
    one launch (the grid and the fp32 dQ accumulation as in the product),
    each head checked against the chunked fp32 reference."""
    B, H = 1, 8
    q, k, v, do = _inputs(B, H, S_sel, S_sel, 5, cuda)
    scale = 1 / math.sqrt(128)
    o, lse = lh._native.attn_fwd(q, k, v, scale)
    dq, dk, dv = lh._native.attn_bwd(q, k, v, o, lse, do, scale)
    torch.cuda.synchronize()
    assert lh._native.device_status() == 0
    for h in range(H):
        ro, rdq, rdk, rdv = _ref_fwd_bwd_chunked(q[0, h], k[0, h], v[0, h], do[0, h], scale)
        _check(o[0, h], ro, f"O head {h}")
        _check(dq[0, h], rdq, f"dQ head {h}")
        _check(dk[0, h], rdk, f"dK head {h}")
        _check(dv[0, h], rdv, f"dV head {h}")
