"""GPU parity of the pyramid, selection and row-mover kernels (through the C ABI)."""
import numpy as np
import pytest
import torch

from inputs import SCORER_CASES, SELECT_CASES, make_qkv, make_scores, pyramid_len

pytestmark = pytest.mark.gpu

BF16_ULP = 2.0 ** -7   # relative spacing of bf16


def _rel_close(a, b, rel, atol=0.0):
    return ((a - b).abs() <= rel * b.abs() + atol)


# ----------------------------------------------------------------------------- pyramid
@pytest.mark.parametrize("name", list(SCORER_CASES))
def test_pyramid_vs_reference_golden(lh, golden, cuda, name):
    B, S, H, D, L, p, dtype, seed = SCORER_CASES[name]
    xq, xk, xv = (t.to(cuda) for t in make_qkv(B, S, H, D, dtype, seed))
    pq, pk, pv, sqk, skq = lh._native.pyramid_score(xq, xk, xv, L, p)
    g = golden["scorer"]
    tol = 1e-6 if dtype == torch.float32 else BF16_ULP
    for ours, key in ((sqk, "scores_qk"), (skq, "scores_kq")):
        ref = torch.from_numpy(g[f"{name}/{key}"])
        assert _rel_close(ours.cpu(), ref, tol).all()
    for ours, key in ((pq, "pooled_q"), (pk, "pooled_k"), (pv, "pooled_v")):
        ref = torch.from_numpy(g[f"{name}/{key}"])
        assert _rel_close(ours.float().cpu(), ref, tol, 1e-6).all()


@pytest.mark.parametrize("shape", [(1, 8192, 8, 128, 3, 4), (2, 4096, 4, 128, 4, 2), (1, 8192, 8, 128, 3, 8),
                                   (1, 4096, 8, 64, 5, 2), (1, 65536, 8, 128, 3, 4)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_pyramid_vs_aten_on_gpu(lh, O, cuda, shape, dtype):
    B, S, H, D, L, p = shape
    xq, xk, xv = (t.to(cuda) for t in make_qkv(B, S, H, D, dtype, 7))
    pq, pk, pv, sqk, skq = lh._native.pyramid_score(xq, xk, xv, L, p)
    rq, rk, rqc, rkc, rvc = O.norm_scorer(xq, xk, xv, p, L)     # the reference's ATen calls, on the GPU
    tol = 2e-6 if dtype == torch.float32 else BF16_ULP
    for ours, ref in ((sqk, rq.float()), (skq, rk.float())):
        close = _rel_close(ours, ref, tol)
        assert close.all()
        if dtype == torch.bfloat16:
            assert (ours == ref).float().mean() > 0.999   # identical bits except rare rounding ties
    for ours, ref in ((pq, rqc[:, :, S:]), (pk, rkc[:, :, S:]), (pv, rvc[:, :, S:])):
        assert _rel_close(ours.float(), ref.float(), tol, 1e-6).all()


# ----------------------------------------------------------------------------- selection
@pytest.mark.parametrize("name", list(SELECT_CASES))
def test_select_vs_reference_golden(lh, golden, cuda, name):
    B, H, N, L, p, k, mode, seed = SELECT_CASES[name]
    sq, sk = make_scores(B, H, N, L, p, mode, seed)
    idx, inv = lh._native.select_topk(sq.to(cuda), sk.to(cuda), L, p, k, N)
    assert np.array_equal(idx.cpu().numpy(), golden["select"][f"{name}/indices"])


# Every defined BASELINE shape plus the reference's own seq_len (98304) sweeps.
SWEEP = [
    (65536, 3, 4, 2048), (131072, 3, 4, 2048), (131072, 3, 4, 4096),
    (98304, 3, 4, 1536), (98304, 3, 4, 2048), (98304, 3, 4, 3072), (98304, 3, 4, 4096), (98304, 3, 4, 6144),
    (98304, 3, 2, 1536), (98304, 4, 2, 1536), (98304, 5, 2, 1536), (98304, 3, 8, 1536),
    (49152, 3, 4, 384), (24576, 3, 4, 1536), (4096, 3, 4, 256),
]


@pytest.mark.parametrize("case", SWEEP)
def test_select_bit_exact_vs_reference_kernel_and_oracle(lh, O, cuda, case):
    N, L, p, k = case
    assert O.shape_defined(N, L, p, k)
    B, H = 1, 8
    sq, sk = make_scores(B, H, N, L, p, "bf16norm", 100 + N % 997 + k)
    sq_d, sk_d = sq.to(cuda), sk.to(cuda)
    idx, inv = lh._native.select_topk(sq_d, sk_d, L, p, k, N)
    ref_gpu = O.ref_select_gpu(sq_d, sk_d, L, p, k, N)           # the reference kernel, fast-math, on the GPU
    oracle = O.select(sq, sk, L, p, k, N)
    assert torch.equal(ref_gpu.cpu(), oracle), "oracle restatement != reference kernel"
    assert torch.equal(idx.cpu(), oracle), "product kernel != reference"
    assert torch.equal(inv.cpu(), O.inverse_map(oracle, pyramid_len(N, L, p)))


@pytest.mark.parametrize("mode", ["ties2", "allsame", "randn"])
def test_select_tie_patterns_at_scale(lh, O, cuda, mode):
    N, L, p, k = 65536, 3, 4, 2048
    sq, sk = make_scores(1, 8, N, L, p, mode, 77)
    idx, _ = lh._native.select_topk(sq.to(cuda), sk.to(cuda), L, p, k, N)
    assert torch.equal(idx.cpu(), O.ref_select_gpu(sq.to(cuda), sk.to(cuda), L, p, k, N).cpu())


def test_select_end_to_end_from_raw_qkv(lh, O, cuda):
    """Selection from the kernel's scores vs the reference pipeline (ATen scorer +
    reference kernel) from the same q/k: indices equal except where a bf16 norm
    rounded differently; the mismatch rate is reported."""
    B, S, H, D, L, p, k = 1, 65536, 8, 128, 3, 4, 2048
    xq, xk, xv = (t.to(cuda) for t in make_qkv(B, S, H, D, torch.bfloat16, 5))
    _, _, _, sqk, skq = lh._native.pyramid_score(xq, xk, xv, L, p)
    idx, _ = lh._native.select_topk(sqk, skq, L, p, k, S)
    rq, rk, *_ = O.norm_scorer(xq, xk, xv, p, L)
    ref = O.ref_select_gpu(rq.float(), rk.float(), L, p, k, S)
    same_scores = torch.equal(sqk, rq.float()) and torch.equal(skq, rk.float())
    mismatch = (idx != ref).float().mean().item()
    print(f"end-to-end index mismatch rate {mismatch:.2e} (scores identical: {same_scores})")
    if same_scores:
        assert mismatch == 0.0
    assert mismatch < 0.05


def test_select_rejects_undefined_shape(lh, cuda):
    sq = torch.rand(1, 1, pyramid_len(4096, 3, 4), device=cuda)
    with pytest.raises(lh._native.LighthouseShapeError):
        lh._native.select_topk(sq, sq, 3, 4, 1536, 4096)


# ----------------------------------------------------------------------------- row movers
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 4096, 2, 128, 3, 4, 256), (2, 8192, 3, 64, 3, 2, 256),
                                   (1, 8192, 2, 128, 2, 8, 128)])
def test_gather_scatter_unpool_vs_oracle(lh, O, cuda, dtype, shape):
    B, S, H, D, L, p, k = shape
    xq, xk, xv = (t.to(cuda) for t in make_qkv(B, S, H, D, dtype, 9))
    pq, pk, pv, sqk, skq = lh._native.pyramid_score(xq, xk, xv, L, p)
    idx, inv = lh._native.select_topk(sqk, skq, L, p, k, S)
    qs, ks, vs = lh._native.gather_selected([xq, xk, xv], [pq, pk, pv], idx)
    # gather: exact copy of pyramid rows
    for x, pooled, sel in ((xq, pq, qs), (xk, pk, ks), (xv, pv, vs)):
        cat = torch.cat([x.transpose(1, 2), pooled], dim=2)
        assert torch.equal(sel, O.gather_rows(cat, idx))
    # scatter forward: deterministic pull vs oracle push (fp32)
    g = torch.Generator().manual_seed(1)
    attn = torch.randn(B, H, idx.shape[-1], D, generator=g).to(dtype).to(cuda)
    out = lh._native.scatter_fwd(attn, inv, S, S, L, p)
    ref = O.scatter_to_base(attn.float(), idx.long(), S, S, L, p)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert (out.float() - ref).abs().max().item() <= tol
    # scatter adjoint
    dout = torch.randn(B, H, S, D, generator=g).to(dtype).to(cuda)
    dattn = lh._native.scatter_bwd(dout, idx, S, S, L, p)
    a = attn.float().clone().requires_grad_(True)
    O.scatter_to_base(a, idx.long(), S, S, L, p).backward(dout.float())
    assert (dattn.float() - a.grad).abs().max().item() <= (1e-4 if dtype == torch.float32 else 0.1)
    # un-pool backward vs autograd of gather + means
    dq = torch.randn_like(qs.float())
    dxq, _, _ = lh._native.unpool_bwd([dq.to(dtype), None, None], inv, S, L, p)
    x = xq.float().clone().requires_grad_(True)
    _, _, qc, _, _ = O.norm_scorer(x, x, x, p, L)
    O.gather_rows(qc, idx).backward(dq.to(dtype).float())
    assert (dxq.float() - x.grad).abs().max().item() <= (1e-5 if dtype == torch.float32 else 3e-2)


def test_scatter_with_longer_output(lh, O, cuda):
    B, S, H, D, L, p, k = 1, 4096, 1, 128, 3, 4, 256
    sq, sk = make_scores(B, H, S, L, p, "randn", 3)
    idx, inv = lh._native.select_topk(sq.to(cuda), sk.to(cuda), L, p, k, S)
    attn = torch.randn(B, H, idx.shape[-1], D, device=cuda)
    out = lh._native.scatter_fwd(attn, inv, S, S + 100, L, p)
    ref = O.scatter_to_base(attn, idx.long(), S, S + 100, L, p)
    assert (out - ref).abs().max().item() < 1e-5


# Geometries of the grouped scatter / un-pool path (two heads per warp for bf16 D=128):
# windows wider than the 16-token group (L=3, p=8), many levels (L=5, p=2), and an
# output longer than the pooled shard.
@pytest.mark.parametrize("shape", [(1, 8192, 2, 128, 3, 8, 128), (1, 8192, 4, 128, 5, 2, 256),
                                   (2, 4096, 2, 128, 2, 4, 256)])
def test_grouped_scatter_and_unpool_vs_oracle(lh, O, cuda, shape):
    B, S, H, D, L, p, k = shape
    xq, xk, xv = (t.to(cuda) for t in make_qkv(B, S, H, D, torch.bfloat16, 21))
    pq, pk, pv, sqk, skq = lh._native.pyramid_score(xq, xk, xv, L, p)
    idx, inv = lh._native.select_topk(sqk, skq, L, p, k, S)
    g = torch.Generator().manual_seed(5)
    attn = torch.randn(B, H, idx.shape[-1], D, generator=g).to(torch.bfloat16).to(cuda)
    for n_out in (S, S + 37):
        out = lh._native.scatter_fwd(attn, inv, S, n_out, L, p)
        ref = O.scatter_to_base(attn.float(), idx.long(), S, n_out, L, p)
        assert _rel_close(out.float(), ref, BF16_ULP, 1e-6).all()     # the fp32 sum rounded once to bf16
    dsel = torch.randn(B, H, idx.shape[-1], D, generator=g).to(torch.bfloat16).to(cuda)
    dxq, _, _ = lh._native.unpool_bwd([dsel, None, None], inv, S, L, p)
    x = xq.float().clone().requires_grad_(True)
    _, _, qc, _, _ = O.norm_scorer(x, x, x, p, L)
    O.gather_rows(qc, idx).backward(dsel.float())
    assert _rel_close(dxq.float(), x.grad, BF16_ULP, 1e-6).all()


def test_select_faster_than_reference_kernel(lh, O, cuda):
    """BASELINE config 3 shape (S=131072, L=3, p=4, k=2048, H=8): the product
    selection (indices + inverse map, one launch) against the reference
    kernel compiled from its own source plus its stable sort and gather
    (CU:404-427), CUDA events on the current stream, 20 launches each after
    3 warm-up launches.  Prints both times; asserts the product is faster."""
    N, L, p, k = 131072, 3, 4, 2048
    sq, sk = make_scores(1, 8, N, L, p, "bf16norm", 5)
    sq, sk = sq.to(cuda), sk.to(cuda)

    def timed(fn):
        for _ in range(3):
            fn()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(20):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / 20

    ours = timed(lambda: lh._native.select_topk(sq, sk, L, p, k, N))
    ref = timed(lambda: O.ref_select_gpu(sq, sk, L, p, k, N))
    print(f"\nselection at S=131072, k=2048, H=8: product {ours * 1e3:.1f} us, reference kernel + sort/gather "
          f"{ref * 1e3:.1f} us")
    assert ours < ref


@pytest.mark.parametrize("shape", [(1, 16384, 8, 3, 4, 1024), (2, 8192, 2, 3, 2, 256)])
def test_scatter_token_major_matches_head_major(lh, O, cuda, shape):
    """The token-major fan-out (B, N, H, D) and its adjoint give the same values,
    bit for bit, as the (B, H, N, D) kernels; the layer returns them as a
    (B, H, S, D) view whose transpose the output projection reads for free."""
    B, S, H, L, p, k = shape
    D = 128
    g = torch.Generator().manual_seed(9)
    sq, sk = make_scores(B, H, S, L, p, "randn", 41)
    idx, inv = lh._native.select_topk(sq.to(cuda), sk.to(cuda), L, p, k, S)
    attn = torch.randn(B, H, idx.shape[-1], D, generator=g).to(torch.bfloat16).to(cuda)
    ref = lh._native.scatter_fwd(attn, inv, S, S, L, p)
    tm = lh._native.scatter_fwd_token_major(attn, inv, S, S, L, p)
    assert tm.shape == (B, S, H, D) and torch.equal(tm.transpose(1, 2), ref)
    dout = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16).to(cuda)
    assert torch.equal(lh._native.scatter_bwd_token_major(dout.transpose(1, 2).contiguous(), idx, S, S, L, p),
                       lh._native.scatter_bwd(dout, idx, S, S, L, p))
    xq, xk, xv = (torch.randn(B, S, H, D, generator=g).to(torch.bfloat16).to(cuda).requires_grad_(True)
                  for _ in range(3))
    out = lh.lighthouse_attention(xq, xk, xv, L, p, k)
    assert out.shape == (B, H, S, D) and out.transpose(1, 2).is_contiguous()
    out.transpose(1, 2).reshape(B, S, H * D).float().sum().backward()   # grad arrives token-major
    assert all(torch.isfinite(t.grad).all() for t in (xq, xk, xv))
