"""The CPU oracle pinned against the reference's own code (golden vectors) and,
where oracle/_ref is built, against the reference kernel source run on host threads."""
import numpy as np
import pytest
import torch

from inputs import (GLA_CASES, LAYER_CASES, SCATTER_CASES, SCORER_CASES, SELECT_CASES, checksum, make_gate, make_qkv,
                    make_scores, pyramid_len)


@pytest.mark.parametrize("name", list(SCORER_CASES))
def test_scorer_matches_reference_golden(O, golden, name):
    B, S, H, D, L, p, dtype, seed = SCORER_CASES[name]
    xq, xk, xv = make_qkv(B, S, H, D, dtype, seed)
    g = golden["scorer"]
    assert str(g[f"{name}/checksum"]) == checksum(xq, xk, xv), "seeded inputs drifted"
    sqk, skq, qc, kc, vc = O.norm_scorer(xq, xk, xv, p, L)
    assert np.array_equal(sqk.float().numpy(), g[f"{name}/scores_qk"])
    assert np.array_equal(skq.float().numpy(), g[f"{name}/scores_kq"])
    for t, c in (("q", qc), ("k", kc), ("v", vc)):
        assert np.array_equal(c[:, :, S:].float().numpy(), g[f"{name}/pooled_{t}"])


@pytest.mark.parametrize("name", list(SELECT_CASES))
def test_selection_matches_reference_kernel_golden(O, golden, name):
    B, H, N, L, p, k, mode, seed = SELECT_CASES[name]
    sq, sk = make_scores(B, H, N, L, p, mode, seed)
    g = golden["select"]
    assert str(g[f"{name}/checksum"]) == checksum(sq, sk)
    idx = O.select(sq, sk, L, p, k, N)
    assert np.array_equal(idx.numpy(), g[f"{name}/indices"])


@pytest.mark.parametrize("name", list(SELECT_CASES))
def test_selection_properties(O, name):
    B, H, N, L, p, k, mode, seed = SELECT_CASES[name]
    sq, sk = make_scores(B, H, N, L, p, mode, seed)
    idx = O.select(sq, sk, L, p, k, N).long()
    S_sel = O.sel_len(N, L, p, k)
    assert idx.shape == (B, H, S_sel)
    S_tot = pyramid_len(N, L, p)
    assert int(idx.min()) >= 0 and int(idx.max()) < S_tot
    for row in idx.reshape(-1, S_sel):
        assert row.unique().numel() == S_sel                      # unique
        # positions covered: every base token is covered exactly once by the
        # leaves + rejected coarse entries (refined entries cover their children)
        first, fan = O.fanout_windows(row.view(1, 1, -1), N, N, L, p)
        start = (first - fan + 1).view(-1)
        starts_sorted = torch.sort(start).values
        assert torch.all(starts_sorted[1:] >= starts_sorted[:-1])
    # per-level counts: coarsest level fully present, every other level p*k entries
    offs = O.level_offsets(N, L, p)
    for l in range(L):
        n = ((idx >= offs[l]) & (idx < offs[l] + N // p ** l)).sum(-1)
        expect = N // p ** (L - 1) if l == L - 1 else p * k
        assert torch.all(n == expect)


def test_selection_refuses_undefined_shapes(O):
    sq, sk = make_scores(1, 1, 4096, 3, 4, "randn", 0)
    with pytest.raises(ValueError):
        O.select(sq, sk, 3, 4, 1536, 4096)          # NCC=21 < 128


@pytest.mark.parametrize("case", [(4096, 3, 4, 256), (512, 2, 2, 128), (8192, 3, 2, 256), (8192, 2, 8, 128)])
def test_oracle_vs_reference_kernel_on_host_threads(O, case):
    N, L, p, k = case
    try:
        O.ref_select_cpu
        sq, sk = make_scores(1, 2, N, L, p, "bf16norm", 5)
        ref, rk, rv = O.ref_select_cpu(sq, sk, L, p, k, N, return_raw=True)
    except FileNotFoundError:
        pytest.skip("oracle/_ref not built (needs the reference tree)")
    ours, ok, ov = O.select(sq, sk, L, p, k, N, return_raw=True)
    assert torch.equal(ours, ref)
    assert torch.equal(ok, rk) and torch.equal(ov, rv)          # same unsorted (key, value) slots too


@pytest.mark.parametrize("name", list(SCATTER_CASES))
def test_scatter_matches_reference_triton_golden(O, golden, name):
    B, H, N, D, L, p, k, seed = SCATTER_CASES[name]
    g = golden["scatter"]
    idx = torch.from_numpy(g[f"{name}/indices"])
    attn = torch.from_numpy(g[f"{name}/attn"]).requires_grad_(True)
    out = O.scatter_to_base(attn, idx, N, N, L, p)
    out.backward(torch.from_numpy(g[f"{name}/dout"]))
    np.testing.assert_allclose(out.detach().numpy(), g[f"{name}/out"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(attn.grad.numpy(), g[f"{name}/dattn"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name", list(LAYER_CASES))
def test_layer_forward_matches_reference_golden(O, golden, name):
    B, S, H, D, L, p, k, seed = LAYER_CASES[name]
    xq, xk, xv = make_qkv(B, S, H, D, torch.float32, seed)
    g = golden["layer"]
    assert str(g[f"{name}/checksum"]) == checksum(xq, xk, xv)
    out, idx = O.lighthouse_local(xq, xk, xv, L, p, k)
    assert np.array_equal(idx.numpy(), g[f"{name}/indices"])
    np.testing.assert_allclose(out.detach().numpy(), g[f"{name}/out"], rtol=1e-5, atol=1e-5)


def test_cp_emulation_with_one_rank_equals_local_on_halves(O):
    # W=1: LighthouseCP = per-half selection, one causal attention over both selections
    xq, xk, xv = make_qkv(1, 8192, 1, 16, torch.float32, 3)
    out, idxs = O.lighthouse_cp_global(xq, xk, xv, 1, 3, 4, 512)
    assert out.shape == (1, 1, 8192, 16) and len(idxs) == 2
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("name", list(GLA_CASES))
def test_gla_scorer_matches_reference_golden(O, golden, name):
    """The GLA scorer restatement vs the reference scorer run on CPU with fla's own
    reference recurrence as its sequence mixer.  fp32: summation order only;
    bf16 outputs: the two fp32 recurrences may round an output element to
    neighbouring bf16 values, so scores agree to one bf16 ulp."""
    B, S, H, D, di, L, p, dtype, div, seed = GLA_CASES[name]
    xq, xk, xv = make_qkv(B, S, H, D, dtype, seed)
    gk = make_gate(B, S, H, div, seed)
    g = golden["gla"]
    assert str(g[f"{name}/checksum"]) == checksum(xq, xk, xv, gk), "seeded inputs drifted"
    sqk, skq, qc, _, _ = O.gla_scorer(xq, xk, xv, gk, di, p, L)
    for ours, key in ((sqk, "scores_qk"), (skq, "scores_kq")):
        ref = torch.from_numpy(g[f"{name}/{key}"])
        tol = 1e-5 * ref.abs() + 1e-6 if dtype == torch.float32 else 2.0 ** -7 * ref.abs() + 1e-6
        assert ((ours.float() - ref).abs() <= tol).all(), key
    if f"{name}/pooled_q" in g:
        assert np.array_equal(qc[:, :, S:].float().numpy(), g[f"{name}/pooled_q"])


def test_gla_recurrence_equals_closed_form(O):
    """The recurrence equals the closed form o_t = scale sum_{s<=t} exp(G_t-G_s)(q_t.k_s) v_s
    (quadratic) that the chunked kernels evaluate, including ragged T."""
    g = torch.Generator().manual_seed(7)
    B, T, H, D = 2, 100, 3, 8
    q, k, v = (torch.randn(B, T, H, D, generator=g, dtype=torch.float64) for _ in range(3))
    gate = torch.nn.functional.logsigmoid(torch.randn(B, T, H, generator=g, dtype=torch.float64))
    o = O.simple_gla(q, k, v, gate, 0.3).double()
    G = gate.cumsum(1)                                                       # (B, T, H)
    dec = (G[:, :, None, :] - G[:, None, :, :]).exp()                        # (B, t, s, H)
    mask = torch.ones(T, T, dtype=torch.bool).tril()[None, :, :, None]
    A = torch.einsum("bthd,bshd->btsh", q, k) * dec * mask
    ref = 0.3 * torch.einsum("btsh,bshd->bthd", A, v)
    assert torch.allclose(o, ref, rtol=1e-5, atol=1e-5)
