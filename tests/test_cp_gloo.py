"""Context-parallel host logic on 2 and 4 gloo CPU ranks.

The package's cp.py (sharding, per-chunk selection with k/(2W), all-gather of
selected K/V into global chunk order, causal chunk attention with query
offsets, reduce of dK/dV partials) runs with the oracle's CPU kernel stand-ins
(oracle/cp_ops.py) and is compared with the single-process emulation of the
reference semantics (oracle.lighthouse_cp_global)."""
import os
import pathlib
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = pathlib.Path(__file__).resolve().parent.parent

B, S, H, D, L, P, K = 1, 16384, 2, 16, 3, 4, 1024


def _shard(x, rank, W, dim):
    chunks = x.chunk(2 * W, dim=dim)
    return torch.cat([chunks[rank], chunks[2 * W - 1 - rank]], dim=dim)


def _worker(rank, W, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        sys.path.insert(0, str(ROOT))
        dist.init_process_group("gloo", rank=rank, world_size=W)
        import __graft_entry__ as ge
        from oracle import cp_ops, oracle as O
        lh = ge.load_package()
        g = torch.Generator().manual_seed(0)
        xs = [torch.randn(B, S, H, D, generator=g) for _ in range(3)]
        dout = torch.randn(B, H, S, D, generator=g)
        local = [_shard(x, rank, W, 1).requires_grad_(True) for x in xs]
        layer = lh.LighthouseCP(None, lh.DialatedLighthouseNormScorerCP(P, L), num_levels=L, pooling_factor=P, topk=K)
        layer.set_cp_info(rank, W, dist.group.WORLD)
        from lighthouse_b200 import cp
        out = cp.lighthouse_cp_forward(*local, L, P, K, rank, W, dist.group.WORLD, ops=cp_ops)
        out.backward(_shard(dout, rank, W, 2))
        # reference semantics on the global sequence, in this process
        xr = [x.clone().requires_grad_(True) for x in xs]
        ref, _ = O.lighthouse_cp_global(*xr, W, L, P, K)
        ref.backward(dout)
        errs = [(out - _shard(ref, rank, W, 2)).abs().max().item()]
        errs += [(a.grad - _shard(b.grad, rank, W, 1)).abs().max().item() for a, b in zip(local, xr)]
        q.put((rank, errs, None))
        dist.destroy_process_group()
    except Exception as e:  # surfaced to the parent
        import traceback
        q.put((rank, None, traceback.format_exc()))


@pytest.mark.parametrize("W", [2, 4])
def test_cp_matches_global_semantics(W):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + W * 7 + os.getpid() % 100
    procs = [ctx.Process(target=_worker, args=(r, W, port, q)) for r in range(W)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(W)]
    for p in procs:
        p.join(timeout=60)
    for rank, errs, tb in results:
        assert tb is None, tb
        assert max(errs) < 1e-4, (rank, errs)


def test_owner_map():
    import __graft_entry__ as ge
    ge.load_package()
    from lighthouse_b200 import cp
    W = 4
    owners = [cp._owner(c, W) for c in range(2 * W)]
    assert owners == [(0, 0), (1, 0), (2, 0), (3, 0), (3, 1), (2, 1), (1, 1), (0, 1)]


def _full_worker(rank, W, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        sys.path.insert(0, str(ROOT))
        dist.init_process_group("gloo", rank=rank, world_size=W)
        import __graft_entry__ as ge
        from oracle import cp_ops
        ge.load_package()
        from lighthouse_b200 import cp
        S_full, H_, D_ = 2048, 2, 16
        g = torch.Generator().manual_seed(3)
        xs = [torch.randn(1, S_full, H_, D_, generator=g) for _ in range(3)]
        dout = torch.randn(1, H_, S_full, D_, generator=g)
        local = [cp.shard_sequence(x, rank, W, dim=1).requires_grad_(True) for x in xs]
        out = cp.full_cp_attention(*local, rank, W, dist.group.WORLD, ops=cp_ops)
        out.backward(cp.shard_sequence(dout, rank, W, dim=2))
        xr = [x.clone().requires_grad_(True) for x in xs]
        ref = torch.nn.functional.scaled_dot_product_attention(*(x.transpose(1, 2) for x in xr), is_causal=True)
        ref.backward(dout)
        errs = [(out - cp.shard_sequence(ref, rank, W, dim=2)).abs().max().item()]
        errs += [(a.grad - cp.shard_sequence(b.grad, rank, W, dim=1)).abs().max().item() for a, b in zip(local, xr)]
        q.put((rank, errs, None))
        dist.destroy_process_group()
    except Exception:
        import traceback
        q.put((rank, None, traceback.format_exc()))


@pytest.mark.parametrize("W", [2, 4])
def test_full_cp_attention_matches_causal_sdpa(W):
    """The full-attention layers of the context-parallel model: sharded causal
    attention over all-gathered K/V equals causal SDPA over the whole sequence."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + W * 7 + os.getpid() % 100
    procs = [ctx.Process(target=_full_worker, args=(r, W, port, q)) for r in range(W)]
    for p_ in procs:
        p_.start()
    results = [q.get(timeout=600) for _ in range(W)]
    for p_ in procs:
        p_.join(timeout=60)
    for rank, errs, tb in results:
        assert tb is None, tb
        assert max(errs) < 1e-4, (rank, errs)
