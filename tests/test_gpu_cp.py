"""LighthouseCP across 2 GPUs over NCCL (one process per GPU): the all-gather of
selected K/V, causal chunk attention with query offsets and the reduce-scatter
of dK/dV, against the single-process emulation of the reference semantics."""
import os
import pathlib
import sys

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = pathlib.Path(__file__).resolve().parent.parent

B, S, H, D, L, P, K = 1, 16384, 2, 128, 3, 4, 1024


def _shard(x, rank, W, dim):
    chunks = x.chunk(2 * W, dim=dim)
    return torch.cat([chunks[rank], chunks[2 * W - 1 - rank]], dim=dim)


def _err(a, b):
    a, b = a.float(), b.float()
    beyond = ((a - b).abs() - b.abs() * 2.0 ** -7).clamp_min(0).max().item()
    return beyond, ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def _worker(rank, W, port, q):
    try:
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        sys.path.insert(0, str(ROOT))
        sys.path.insert(0, str(ROOT / "tests" / "golden"))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=W, device_id=torch.device("cuda", rank))
        import __graft_entry__ as ge
        from oracle import oracle as O
        from inputs import make_qkv
        lh = ge.load_package()
        dev = torch.device("cuda", rank)
        xq, xk, xv = make_qkv(B, S, H, D, torch.bfloat16, 31)
        dout = torch.randn(B, H, S, D, generator=torch.Generator().manual_seed(32)).to(torch.bfloat16)
        layer = lh.LighthouseCP(None, lh.DialatedLighthouseNormScorerCP(P, L), num_levels=L, pooling_factor=P, topk=K)
        layer.set_cp_info(rank, W, dist.group.WORLD)
        local = [_shard(x, rank, W, 1).to(dev).requires_grad_(True) for x in (xq, xk, xv)]
        out = layer(*local)
        out.backward(_shard(dout, rank, W, 2).to(dev))
        torch.cuda.synchronize()
        # reference on the global sequence with per-chunk selections from the kernels
        n = S // (2 * W)
        idxs = []
        for c in range(2 * W):
            sl = slice(c * n, (c + 1) * n)
            _, _, _, sqk, skq = lh._native.pyramid_score(*[x[:, sl].contiguous().to(dev) for x in (xq, xk, xv)], L, P)
            idxs.append(O.select(sqk.cpu(), skq.cpu(), L, P, K // (2 * W), n))
        xr = [x.float().requires_grad_(True) for x in (xq, xk, xv)]
        ref, _ = O.lighthouse_cp_global(*xr, W, L, P, K, indices=idxs)
        ref.backward(dout.float())
        errs = [_err(out.detach().cpu(), _shard(ref.detach(), rank, W, 2))]
        errs += [_err(a.grad.cpu(), _shard(b.grad, rank, W, 1)) for a, b in zip(local, xr)]
        status = lh._native.device_status()
        dist.destroy_process_group()
        q.put((rank, errs, status, None))
    except Exception:
        import traceback
        q.put((rank, None, None, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_cp_two_gpus_vs_global_semantics():
    W = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, W, port, q)) for r in range(W)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(W)]
    for p in procs:
        p.join(timeout=120)
    for rank, errs, status, tb in results:
        assert tb is None, tb
        assert status == 0
        for m, r in errs:
            assert m <= 2e-2 and r <= 1e-2, (rank, errs)


def _model_worker(rank, W, port, q):
    try:
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        sys.path.insert(0, str(ROOT))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=W, device_id=torch.device("cuda", rank))
        import __graft_entry__ as ge
        lh = ge.load_package()
        from lighthouse_b200 import model as M
        dev = torch.device("cuda", rank)
        cp_group = dist.new_group(list(range(W)))          # CP collectives apart from DDP's
        args = M.ModelArgs(dim=256, n_layers=4, n_heads=2, n_kv_heads=2, hidden_dim=384, max_seq_len=16384,
                           lighthouse_topk=1024, lighthouse_full_attn_layers=[0])
        torch.manual_seed(0)
        m = M.Transformer(args).to(dev)
        m.init_weights(0)
        m.set_cp_info(rank, W, cp_group)
        ddp = torch.nn.parallel.DistributedDataParallel(m, device_ids=[rank])
        opt = torch.optim.AdamW(ddp.parameters(), lr=3e-3, fused=True)
        g = torch.Generator().manual_seed(1)
        base = torch.randint(0, 256, (1, 64), generator=g)
        tokens = base.repeat(1, 16384 // 64 + 1)[:, :16385].to(dev)   # the same global tokens on every rank
        losses = []
        for _ in range(8):
            loss = M.train_step(ddp, opt, tokens).detach()
            dist.all_reduce(loss)
            losses.append(loss.item() / W)
        flat = torch.cat([p.detach().float().flatten() for p in m.parameters()])
        lo, hi = flat.clone(), flat.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        spread = (hi - lo).abs().max().item()
        status = lh._native.device_status()
        dist.destroy_process_group()
        q.put((rank, (losses, spread), status, None))
    except Exception:
        import traceback
        q.put((rank, None, None, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_context_parallel_model_trains_on_two_gpus():
    """Context-parallel training loop: sharded tokens / labels / RoPE positions,
    LighthouseCP and sharded full attention, DDP gradient averaging."""
    W = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29800 + os.getpid() % 150
    procs = [ctx.Process(target=_model_worker, args=(r, W, port, q)) for r in range(W)]
    for p in procs:
        p.start()
    results = [q.get(timeout=900) for _ in range(W)]
    for p in procs:
        p.join(timeout=60)
    for rank, res, status, tb in results:
        assert tb is None, tb
        losses, spread = res
        assert all(torch.isfinite(torch.tensor(losses))), losses
        assert losses[-1] < losses[0] - 0.5, losses
        assert spread == 0.0, spread            # replicas stay identical
        assert status == 0
