"""Benchmark: Lighthouse attention layer forward+backward tokens/s (BASELINE metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE.json config 3 at k=2048, the metric's "@S=128K k=2048"):
B=1, S=131072, H=8, D=128, norm scorer, L=3, p=4, k=2048, causal, bf16,
q/k/v/dO seeded N(0,1).  One step = forward + backward of one layer.  Inputs
(3 x 268 MB + dO) are larger than the 126 MB L2, so no flush is needed
between steps.

N > 1 (torchrun): every rank runs an independent replica (the layer has no
parameters and the path does not shard across ranks: "replicas only"), value =
all ranks' tokens / the max over ranks of the device time.

``--impl reference`` times the reference's CPU implementation of the path
(the oracle's restatement: ATen scorer, C selection, torch.gather, CPU SDPA,
index_add scatter -- the reference itself has no CPU selection or scatter)
on the host cores, on rank 0 only: the whole layer (all heads) per step, at
most 3 timed steps after 1 warm-up (each step takes several seconds).

The default line also carries, from the same run: every kernel group's time
and HBM fraction (CUDA events inside the timed steps), the attention roofline
against the measured bf16 peak (burst for a timed region under 2 s), the
same-run cuDNN SDPA timing on the identical gathered tensors, the end-to-end
figure through ``lighthouse_attention`` with host inputs, and the SM clocks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(B=1, S=131072, H=8, D=128, L=3, p=4, k=2048)
METRIC = "Lighthouse attn fwd+bwd tokens/s @S=128K k=2048"


def _sel_len(S, L, p, k):
    return S // p ** (L - 1) + (L - 1) * p * k


def _config(extra=None):
    c = {"workload": "lighthouse_layer_fwd_bwd", "batch": CFG["B"], "seq_len": CFG["S"], "heads": CFG["H"],
         "head_dim": CFG["D"], "levels": CFG["L"], "pooling_factor": CFG["p"], "topk": CFG["k"],
         "selected_len": _sel_len(CFG["S"], CFG["L"], CFG["p"], CFG["k"]), "scorer": "norm",
         "l2": "inputs larger than L2 (no flush needed)"}
    c.update(extra or {})
    return c


def _inputs(device, dtype=torch.bfloat16, heads=None):
    B, S, H, D = CFG["B"], CFG["S"], CFG["H"], CFG["D"]
    g = torch.Generator().manual_seed(0)
    xs = [torch.randn(B, S, H, D, generator=g) for _ in range(3)]
    dout = torch.randn(B, H, S, D, generator=g)
    if heads is not None:
        xs = [x[:, :, heads].contiguous() for x in xs]
        dout = dout[:, heads].contiguous()
    return [x.to(dtype).to(device) for x in xs], dout.to(dtype).to(device)


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    def __init__(self, index: int):
        self.proc = None
        self.index = index

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.proc is None:
            return
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=5)
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 7:
                self.rows.append(parts)

    def summary(self):
        if not getattr(self, "rows", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[3:7]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(self.rows[0][1]) if self.rows[0][1].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(self.rows)}


# ----------------------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    import __graft_entry__ as ge
    lh = ge.load_package()
    N = lh._native
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B, S, H, D, L, p, k = (CFG[x] for x in ("B", "S", "H", "D", "L", "p", "k"))
    (xq, xk, xv), dout = _inputs(dev)
    scale = 1.0 / math.sqrt(D)
    ev = {}

    def mark(name):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        ev.setdefault(name, []).append(e)

    # segment boundaries inside one step: every kernel group of the layer gets
    # its own pair of events on the launching (current) stream
    SEG = ["pyramid", "select", "gather", "attn_fwd", "scatter_fwd", "scatter_bwd", "attn_bwd", "unpool_bwd"]

    def step(timed):
        # the fused layer of lighthouse_selection._LighthouseLayerFn, instrumented
        if timed: mark("start")
        pq, pk, pv, sqk, skq = N.pyramid_score(xq, xk, xv, L, p)
        if timed: mark("pyramid")
        idx, inv = N.select_topk(sqk, skq, L, p, k, S)
        if timed: mark("select")
        qs, ks, vs = N.gather_selected([xq, xk, xv], [pq, pk, pv], idx)
        if timed: mark("gather")
        o, lse = N.attn_fwd(qs, ks, vs, scale)
        if timed: mark("attn_fwd")
        out = N.scatter_fwd(o, inv, S, S, L, p)
        if timed: mark("scatter_fwd")
        dattn = N.scatter_bwd(dout, idx, S, S, L, p)
        if timed: mark("scatter_bwd")
        dqs, dks, dvs = N.attn_bwd(qs, ks, vs, o, lse, dattn, scale)
        if timed: mark("attn_bwd")
        dx = N.unpool_bwd([dqs, dks, dvs], inv, S, L, p)
        if timed: mark("unpool_bwd")
        return out, dx

    for _ in range(args.warmup):
        step(False)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            step(True)
        t1.record()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
    ms = t0.elapsed_time(t1) / args.steps
    seg_ms = {}
    prev = "start"
    for name in SEG:
        seg_ms[name] = statistics.mean(a.elapsed_time(b) for a, b in zip(ev[prev], ev[name]))
        prev = name
    fwd_ms, bwd_ms = seg_ms["attn_fwd"], seg_ms["attn_bwd"]
    assert N.device_status() == 0, "an attention kernel left a bounded wait"

    # The reference runs F.scaled_dot_product_attention (cuDNN on sm_100) on
    # the gathered sequence: time it here on the same q/k/v/dO, same stream.
    sdpa_fwd_ms = sdpa_bwd_ms = None
    if not args.no_sdpa:
        with torch.no_grad():
            pq, pk, pv, sqk, skq = N.pyramid_score(xq, xk, xv, L, p)
            idx, inv = N.select_topk(sqk, skq, L, p, k, S)
            qs, ks, vs = N.gather_selected([xq, xk, xv], [pq, pk, pv], idx)
            dattn = N.scatter_bwd(dout, idx, S, S, L, p)
            del pq, pk, pv, sqk, skq, inv
        qg, kg, vg = (t.detach().requires_grad_(True) for t in (qs, ks, vs))
        sf, sb = [], []
        for it in range(args.warmup + min(args.steps, 10)):
            a0, a1, a2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            a0.record()
            og = torch.nn.functional.scaled_dot_product_attention(qg, kg, vg, is_causal=True)
            a1.record()
            og.backward(dattn)
            a2.record()
            if it >= args.warmup:
                sf.append((a0, a1)); sb.append((a1, a2))
            qg.grad = kg.grad = vg.grad = None
        torch.cuda.synchronize()
        sdpa_fwd_ms = statistics.mean(a.elapsed_time(b) for a, b in sf)
        sdpa_bwd_ms = statistics.mean(a.elapsed_time(b) for a, b in sb)
        del qg, kg, vg, og, qs, ks, vs, dattn, idx

    # end to end through the public API: pinned host inputs -> device, scalar loss back
    (hq, hk, hv), _ = _inputs("cpu")
    hq, hk, hv = (t.pin_memory() for t in (hq, hk, hv))
    w = dout  # resident upstream weight: loss = <out, w>
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))

    # Input pipeline as in training: step i+1's host->device copy runs on a
    # second stream while step i computes (two device buffers ordered by
    # events).  Every step's copy and its loss read-back are inside the timed
    # region; only their overlap with compute changes.
    copy_stream = torch.cuda.Stream(device=dev)
    bufs = [[torch.empty(t.shape, dtype=t.dtype, device=dev) for t in (hq, hk, hv)] for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]
    w_f = w.float()  # the resident upstream weight, converted once

    def enqueue_copy(slot, after=None):
        with torch.cuda.stream(copy_stream):
            if after is not None:
                copy_stream.wait_event(after)
            copy_stream.wait_event(freed[slot])      # the step that last read this buffer is done
            for d_, h_ in zip(bufs[slot], (hq, hk, hv)):
                d_.copy_(h_, non_blocking=True)
            copied[slot].record(copy_stream)

    def e2e_run(n, start=None):
        enqueue_copy(0, start)
        loss = None
        for i in range(n):
            slot = i % 2
            if i + 1 < n:
                enqueue_copy((i + 1) % 2)
            torch.cuda.current_stream().wait_event(copied[slot])
            xs = [b_.detach().requires_grad_(True) for b_ in bufs[slot]]
            out = lh.lighthouse_attention(*xs, num_levels=L, pooling_factor=p, topk=k)
            loss_t = (out * w_f).sum()
            loss_t.backward()
            freed[slot].record()
            loss = loss_t.item()                     # device -> host read of the step's result
        return loss

    e2e_run(max(2, args.warmup // 2))
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_steps = max(2, min(args.steps, 5))
    e0.record()
    e2e_run(e_steps, start=e0)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e_steps

    clocks = clk.summary()
    per_rank = None
    if world > 1:
        # every rank's figures, so that a slow GPU setting the max shows by itself
        mine = torch.tensor([ms, e2e_ms, fwd_ms, bwd_ms, float(clocks["sm_mhz"] or 0)]
                            + [seg_ms[n] for n in SEG], device=dev)
        allr = torch.empty(world, mine.numel(), device=dev)
        torch.distributed.all_gather_into_tensor(allr, mine)
        per_rank = [{"ms_per_step": r[0], "e2e_ms": r[1], "attn_fwd_ms": r[2], "attn_bwd_ms": r[3], "sm_mhz": r[4]}
                    for r in allr.tolist()]
        mx = allr.max(dim=0).values.tolist()
        ms, e2e_ms, fwd_ms, bwd_ms = mx[:4]
        seg_ms = dict(zip(SEG, mx[5:]))
    if rank != 0:
        return

    S_sel = _sel_len(S, L, p, k)
    P = S_sel * (S_sel + 1) / 2
    bwd_flops = 10 * B * H * D * P
    fwd_flops = 4 * B * H * D * P
    pk_ = _peak_for(ms * args.steps * 1e-3)
    peak = pk_["tflops"]
    achieved = bwd_flops / (bwd_ms * 1e-3) / 1e12
    hbm = pk_["gbs"]
    # algorithmic bytes of the HBM-bound kernels (per launch)
    S_tot = sum(S // p ** l for l in range(L))
    S_pool = S_tot - S
    row = D * 2
    hb = {
        "pyramid": 3 * B * S * H * row + 3 * B * H * S_pool * row + 2 * B * H * S_tot * 4,
        "select": 2 * B * H * 4 * (S // p ** (L - 1) + 2 * (L - 1) * p * k) + B * H * (S_sel + S_tot) * 4,
        "gather": 2 * 3 * B * H * S_sel * row,
        "scatter_fwd": B * H * S * row + B * H * S_sel * row,
        "scatter_bwd": B * H * S * row + B * H * S_sel * row,
        "unpool_bwd": 3 * B * S * H * row + 3 * B * H * S_sel * row,
    }
    hbm_kernels = {n: {"ms": seg_ms[n], "bytes": hb[n], "gbs": hb[n] / (seg_ms[n] * 1e-3) / 1e9,
                       "frac": hb[n] / (seg_ms[n] * 1e-3) / 1e9 / hbm} for n in hb}
    pss_bytes = hb["pyramid"] + hb["select"]
    pss_ms = seg_ms["pyramid"] + seg_ms["select"]
    hbm_kernels["pool_score_select"] = {"ms": pss_ms, "bytes": pss_bytes, "gbs": pss_bytes / (pss_ms * 1e-3) / 1e9,
                                        "frac": pss_bytes / (pss_ms * 1e-3) / 1e9 / hbm}
    attn_tf = (fwd_flops + bwd_flops) / ((fwd_ms + bwd_ms) * 1e-3) / 1e12
    tokens = B * S * world
    line = {
        "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) q/k/v/dO)",
        "config": _config({"parallelism": f"replicas x{world}"}),
        "roofline": {"kernel": "attn_bwd (prep + tcgen05 main + post)", "bound": "tensor",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "peak_source": pk_["tf_src"], "traffic": None,
                     "traffic_note": "not measured in this run (ncu DRAM counters of a small-shape capture "
                                     "are summarised under profiles/)",
                     "flops_per_launch": bwd_flops, "ms_per_launch": bwd_ms,
                     "attn_fwd": {"achieved": fwd_flops / (fwd_ms * 1e-3) / 1e12,
                                  "frac": fwd_flops / (fwd_ms * 1e-3) / 1e12 / peak, "ms_per_launch": fwd_ms,
                                  "flops_per_launch": fwd_flops},
                     "attn_fwd_bwd": {"achieved": attn_tf, "frac": attn_tf / peak},
                     "hbm_peak_gbs": hbm, "hbm_peak_source": pk_["gbs_src"], "hbm_kernels": hbm_kernels},
        "kernels": {"attn_fwd_ms": fwd_ms, "attn_fwd_tflops": fwd_flops / (fwd_ms * 1e-3) / 1e12,
                    "attn_bwd_ms": bwd_ms, "attn_bwd_tflops": achieved,
                    "rest_ms": ms - fwd_ms - bwd_ms, "segments_ms": seg_ms,
                    "cudnn_fwd_ms": sdpa_fwd_ms, "cudnn_bwd_ms": sdpa_bwd_ms,
                    "cudnn_note": "torch scaled_dot_product_attention(is_causal=True), the reference's attention "
                                  "call, on the identical gathered q/k/v and scattered dO, same run"},
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": 4, "ms_per_step": e2e_ms, "api": "lighthouse_attention",
                "input_pipeline": "step i+1 host->device copy on a second stream during step i"},
        "gpu_launches": 10 * args.steps,
        "timed_region_s": ms * args.steps * 1e-3,
        "clocks": clocks,
    }
    if per_rank:
        line["per_rank"] = per_rank
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_sample(steps=1, warmup=1)["cpu_baseline"]   # warm, as the reference arm
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- model workload
def run_model(args, rank, world, local_rank, cp=False):
    """270M Llama3-style training step (Lighthouse on 26 of 30
    layers), bf16 autocast, AdamW, seq 65536, uniform random bytes; DDP over NCCL
    for N > 1 (weak scaling: every rank trains on its own sequence).  With
    cp=True (the reference's *_cp flavours) the N ranks
    train one sequence together: context parallelism over the sequence,
    gradients averaged by DDP (strong scaling)."""
    import __graft_entry__ as ge
    lh = ge.load_package()
    from lighthouse_b200 import model as M
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    # config 5 (CP): seq 262144 with k=1536 is outside the reference's defined
    # domain (its selection writes holes there); its defined twin is seq 196608
    seq = args.seq_len or (196608 if cp else 65536)
    margs = M.ModelArgs(max_seq_len=seq, lighthouse_topk=args.topk or (1536 if cp else 2048))
    torch.manual_seed(0)
    model = M.Transformer(margs).to(dev)
    model.init_weights(0)
    cpn = min(args.cp or 2, world) if cp else 1       # context-parallel group size (config 5: 2)
    if cp and world % cpn:
        raise SystemExit(f"--cp {cpn} must divide the {world} ranks")
    dp = world // cpn
    if cp and world > 1:
        # ranks [g*cpn, (g+1)*cpn) train one sequence together; every rank
        # creates every group (new_group is collective over the world)
        groups = [torch.distributed.new_group(list(range(g * cpn, (g + 1) * cpn))) for g in range(dp)]
        if cpn > 1:
            model.set_cp_info(rank % cpn, cpn, groups[rank // cpn])
    if world > 1:
        model = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local_rank], bucket_cap_mb=100,
                                                          gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True)
    # CP: one sequence per context-parallel group, shared by its ranks
    g = torch.Generator().manual_seed(1000 + (rank // cpn if cp else rank))
    host = [torch.randint(0, 256, (1, seq + 1), generator=g, dtype=torch.long).pin_memory() for _ in range(2)]
    toks = [h.to(dev) for h in host]
    for i in range(args.warmup):
        M.train_step(model, opt, toks[i % 2])
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    with ClockSampler(local_rank) as clk:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for i in range(args.steps):
            M.train_step(model, opt, toks[i % 2])
        t1.record()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
    ms = t0.elapsed_time(t1) / args.steps
    # end to end: tokens copied from pinned host memory each step, loss read back
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_steps = max(1, min(args.steps, 3))
    e0.record()
    for i in range(e_steps):
        loss = M.train_step(model, opt, host[i % 2].to(dev, non_blocking=True)).item()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e_steps
    assert lh._native.device_status() == 0
    clocks = clk.summary()
    per_rank = None
    if world > 1:
        t = torch.tensor([ms, e2e_ms, float(clocks["sm_mhz"] or 0)], device=dev)
        allr = torch.empty(world, 3, device=dev)
        torch.distributed.all_gather_into_tensor(allr, t)
        per_rank = [{"ms_per_step": r[0], "e2e_ms": r[1], "sm_mhz": r[2]} for r in allr.tolist()]
        ms, e2e_ms = allr[:, :2].max(dim=0).values.tolist()
    if rank != 0:
        return
    tokens = seq * dp if cp else seq * world
    n_layers_lh = sum(1 for i in range(margs.n_layers) if i not in margs.lighthouse_full_attn_layers)
    line = {
        "metric": f"270M train tok/s (Lighthouse norm, k={margs.lighthouse_topk}, p=4, L=3)", "value": tokens / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": ("strong" if dp == 1 else "weak over dp, strong over cp") if cp else "weak",
        "vs_baseline": None,
        "dtype": "bf16 autocast, fp32 master",
        "data": "synthetic (uniform random bytes, seeded)",
        "config": {"workload": "llama3_270m_train_step", "params": M.num_params(model), "seq_len": seq,
                   "global_batch": dp if cp else world, "lighthouse_layers": n_layers_lh,
                   "parallelism": (f"cp{cpn} x dp{dp} (LighthouseCP + sharded full attention, NCCL; DDP across)"
                                   if cp else f"dp{world} (DDP/NCCL)"),
                   "l2": "activations far larger than L2"},
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": (seq + 1) * 8,
                "d2h_bytes_per_step": 4, "ms_per_step": e2e_ms, "final_loss": loss},
        "gpu_launches": 10 * n_layers_lh * args.steps,
        "clocks": clocks,
    }
    if per_rank:
        line["per_rank"] = per_rank
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- sweep workload
# S=131072 with top-k, levels and pooling factor varied.  The
# reference kernel is defined at S=131072 only for p=4, L=3, k in {2048, 4096};
# every other point runs at S=98304, the reference's own seq_len, where all of
# them are defined (the package raises LighthouseShapeError, as the reference
# writes holes, on undefined shapes).
SWEEP = [  # (S, L, p, k); the first point is BASELINE config 2
    (65536, 3, 4, 2048),
    (131072, 3, 4, 2048), (131072, 3, 4, 4096),
    (98304, 3, 4, 1536), (98304, 3, 4, 2048), (98304, 3, 4, 3072), (98304, 3, 4, 4096), (98304, 3, 4, 6144),
    (98304, 3, 2, 1536), (98304, 4, 2, 1536), (98304, 5, 2, 1536),
    (98304, 3, 8, 1536),
]


def run_sweep(args, rank, world, local_rank):
    """One line per sweep point: layer fwd+bwd tokens/s on resident inputs and the
    attention kernels' TFLOP/s.  Inputs are drawn on the device (timing only; parity
    of these shapes is covered by the GPU tests)."""
    import __graft_entry__ as ge
    lh = ge.load_package()
    N = lh._native
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B, H, D = CFG["B"], CFG["H"], CFG["D"]
    scale = 1.0 / math.sqrt(D)
    g = torch.Generator(device=dev).manual_seed(0)
    for (S, L, p, k) in SWEEP:
        xq, xk, xv = (torch.randn(B, S, H, D, generator=g, device=dev, dtype=torch.bfloat16) for _ in range(3))
        dout = torch.randn(B, H, S, D, generator=g, device=dev, dtype=torch.bfloat16)
        ev = {n: [] for n in ("f0", "f1", "b0", "b1")}

        def step(timed):
            pq, pk, pv, sqk, skq = N.pyramid_score(xq, xk, xv, L, p)
            idx, inv = N.select_topk(sqk, skq, L, p, k, S)
            qs, ks, vs = N.gather_selected([xq, xk, xv], [pq, pk, pv], idx)
            marks = []
            for name in ("f0", "f1", "b0", "b1"):
                marks.append(torch.cuda.Event(enable_timing=True))
                if timed:
                    ev[name].append(marks[-1])
            marks[0].record()
            o, lse = N.attn_fwd(qs, ks, vs, scale)
            marks[1].record()
            out = N.scatter_fwd(o, inv, S, S, L, p)
            dattn = N.scatter_bwd(dout, idx, S, S, L, p)
            marks[2].record()
            dqs, dks, dvs = N.attn_bwd(qs, ks, vs, o, lse, dattn, scale)
            marks[3].record()
            N.unpool_bwd([dqs, dks, dvs], inv, S, L, p)

        for _ in range(args.warmup):
            step(False)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            step(True)
        t1.record()
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1) / args.steps
        fwd_ms = statistics.mean(a.elapsed_time(b) for a, b in zip(ev["f0"], ev["f1"]))
        bwd_ms = statistics.mean(a.elapsed_time(b) for a, b in zip(ev["b0"], ev["b1"]))
        if world > 1:
            t = torch.tensor([ms, fwd_ms, bwd_ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms, fwd_ms, bwd_ms = t.tolist()
        assert N.device_status() == 0, "an attention kernel left a bounded wait"
        del xq, xk, xv, dout
        if rank != 0:
            continue
        S_sel = _sel_len(S, L, p, k)
        P = S_sel * (S_sel + 1) / 2
        print(json.dumps({
            "metric": "Lighthouse attn fwd+bwd tokens/s (sweep point)", "value": B * S * world / (ms * 1e-3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "dtype": "bf16", "data": "synthetic (seeded N(0,1) on the device)",
            "config": {"workload": "lighthouse_layer_sweep", "seq_len": S, "levels": L, "pooling_factor": p,
                       "topk": k, "selected_len": S_sel, "batch": B, "heads": H, "head_dim": D,
                       "l2": "inputs larger than L2 (no flush needed)"},
            "kernels": {"attn_fwd_ms": fwd_ms, "attn_fwd_tflops": 4 * B * H * D * P / (fwd_ms * 1e-3) / 1e12,
                        "attn_bwd_ms": bwd_ms, "attn_bwd_tflops": 10 * B * H * D * P / (bwd_ms * 1e-3) / 1e12,
                        "rest_ms": ms - fwd_ms - bwd_ms},
        }), flush=True)


# ----------------------------------------------------------------------------- GLA scorer workload
def _peak_for(timed_s: float):
    """Roofline denominators from MEASURED_PEAKS.json.  The burst bf16 figure
    applies to a timed region shorter than 2 s; the sustained (power-capped)
    one to longer regions."""
    try:
        m = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        m = {}
    if timed_s >= 2.0 and "bf16_tflops_sustained" in m:
        tf, src = m["bf16_tflops_sustained"], "measured sustained (timed region >= 2 s)"
    elif "bf16_tflops" in m:
        tf, src = m["bf16_tflops"], "measured burst (timed region < 2 s)"
    else:
        tf, src = (1400.0, "fallback sustained") if timed_s >= 2.0 else (1590.0, "fallback burst")
    gbs, gsrc = (m["hbm_gbs"], "measured") if "hbm_gbs" in m else (6650.0, "fallback")
    return {"tflops": tf, "tf_src": src, "gbs": gbs, "gbs_src": gsrc}


def _peaks():
    """Dense bf16 peak for a kernel timed on its own: the measured burst figure."""
    return _peak_for(0.0)


def run_scorer_gla(args, rank, world, local_rank):
    """The `gla` scorer (SEL:692-755) at the layer configuration: simple GLA over
    the dilated views (dilation 4: 32 sub-sequences of 32768 steps per pass),
    both passes, then norms, level maxima and pyramid means.  Forward only (the
    scores carry no gradient).  N ranks run independent replicas."""
    import __graft_entry__ as ge
    lh = ge.load_package()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B, S, H, D, L, p = CFG["B"], CFG["S"], CFG["H"], CFG["D"], CFG["L"], CFG["p"]
    di = 4
    scorer = lh.DilatedLighthouseGLAScorer(D, dilation=di, pooling_factor=p, levels=L)
    g = torch.Generator().manual_seed(0)
    host = [torch.randn(B, S, H, D, generator=g).to(torch.bfloat16).pin_memory() for _ in range(3)]
    host.append((torch.nn.functional.logsigmoid(torch.randn(B, S, H, generator=g)) / 16).pin_memory())
    xs = [h.to(dev) for h in host]
    T, Hd = S // di, H * di
    view = lambda x: x.reshape(B, T, Hd, *x.shape[3:])
    kern = lambda: lh._native.simple_gla_fwd(view(xs[0]), view(xs[1]), view(xs[2]), view(xs[3]), scorer.scaling,
                                             q2=view(xs[1]), k2=view(xs[0]))
    for _ in range(args.warmup):
        scorer.scores(*xs)
        kern()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ev = lambda: torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        t0, t1 = ev(), ev()
        t0.record()
        for _ in range(args.steps):
            scorer.scores(*xs)
        t1.record()
        k0, k1 = ev(), ev()
        k0.record()
        for _ in range(args.steps):
            kern()
        k1.record()
        torch.cuda.synchronize()
    ms, kms = t0.elapsed_time(t1) / args.steps, k0.elapsed_time(k1) / args.steps
    e0, e1 = ev(), ev()
    e0.record()
    for _ in range(args.steps):
        d = [h.to(dev, non_blocking=True) for h in host]
        sqk, skq = scorer.scores(*d)
        (sqk[0, 0, 0] + skq[0, 0, 0]).item()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    assert lh._native.device_status() == 0
    if world > 1:
        t = torch.tensor([ms, kms, e2e_ms], device=dev)
        allr = torch.empty(world, 3, device=dev)
        torch.distributed.all_gather_into_tensor(allr, t)
        per_rank = [{"ms_per_step": r[0], "kernel_ms": r[1], "e2e_ms": r[2]} for r in allr.tolist()]
        ms, kms, e2e_ms = allr.max(dim=0).values.tolist()
    else:
        per_rank = None
    if rank != 0:
        return
    # algorithmic FLOPs: the recurrence's state update k v^T and read-out q S, 2 D^2 multiply-adds
    # per (step, sub-head, pass); the chunked evaluation's intra-chunk products are extra work
    flops = 2 * B * Hd * T * 4 * D * D
    peaks = _peaks()
    line = {
        "metric": "GLA scorer tokens/s @S=128K (dilation 4, both passes + pyramid)", "value": B * S * world / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v, gate logsigmoid(N(0,1))/16)",
        "config": _config({"workload": "gla_scorer_fwd", "scorer": "gla", "dilation": di,
                           "parallelism": f"replicas x{world}"}),
        "roofline": {"kernel": "simple_gla_fwd_kernel (warp MMA, both passes)", "bound": "tensor",
                     "achieved": flops / (kms * 1e-3) / 1e12, "peak": peaks["tflops"], "unit": "TFLOP/s",
                     "frac": flops / (kms * 1e-3) / 1e12 / peaks["tflops"], "peak_source": peaks["tf_src"],
                     "traffic": None, "flops_per_launch": flops, "ms_per_launch": kms},
        "e2e": {"value": B * S * world / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": sum(h.numel() * h.element_size() for h in host), "d2h_bytes_per_step": 4,
                "ms_per_step": e2e_ms, "api": "DilatedLighthouseGLAScorer.scores"},
        "gpu_launches": 3 * args.steps,          # scorer: GLA + pyramid; kernel leg: GLA
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        # the oracle (fp32 recurrence, ATen on the host threads) on the first 8192 tokens;
        # its cost is linear in the sequence length, so tokens/s carries over
        from oracle import oracle as O
        n = 8192
        cs = [h[:, :n].float() for h in host[:3]] + [host[3][:, :n]]
        t = time.perf_counter()
        O.gla_scorer(*cs, di, p, L)
        dt = time.perf_counter() - t
        line["cpu_baseline"] = {"value": B * n / dt, "unit": "tokens/s", "cores": torch.get_num_threads(),
                                "kind": "port", "dtype": "f32",
                                "sample": f"first {n} of {S} tokens, all heads, both passes + pyramid; oracle "
                                          "recurrence (fla's published simple-GLA definition)"}
    if per_rank:
        line["per_rank"] = per_rank
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- CPU arm
def cpu_sample(steps: int, warmup: int):
    """The reference path on the host cores: the whole layer (all heads)
    forward + backward per step, fp32, on all host threads."""
    from oracle import oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    B, S, H, D, L, p, k = (CFG[x] for x in ("B", "S", "H", "D", "L", "p", "k"))
    (xq, xk, xv), dout = _inputs("cpu", torch.float32)

    def one():
        xs = [t.clone().requires_grad_(True) for t in (xq, xk, xv)]
        out, _ = O.lighthouse_local(*xs, L, p, k)
        out.backward(dout)

    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    dt = (time.perf_counter() - t0) / steps
    value = (B * S) / dt
    return {"value": value, "sec_per_step": dt, "cpu_baseline": {
        "value": value, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
        "dtype": "f32",
        "sample": f"the whole S={S} layer (all {H} heads) fwd+bwd, {steps} timed step(s) after {warmup} warm-up; "
                  "oracle restatement (ATen scorer, C selection, gather, CPU SDPA, index_add scatter)"}}


def run_reference(args, rank):
    if rank != 0:
        return
    steps = max(1, min(args.steps, 3))
    warm = min(args.warmup, 1)
    r = cpu_sample(steps, warm)
    line = {"metric": METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": warm, "ms_per_step": r["sec_per_step"] * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
            "config": _config({"parallelism": "cpu"}), "impl": "reference",
            "cpu_baseline": r["cpu_baseline"],
            "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sdpa", action="store_true", help="skip the same-run cuDNN SDPA comparison")
    ap.add_argument("--workload", default="layer", choices=["layer", "model", "model_cp", "scorer_gla", "sweep"],
                    help="layer: BASELINE config 3 (default); model: config 4, the 270M training step; "
                         "model_cp: config 5, one sequence context-parallel over the N ranks; "
                         "scorer_gla: the `gla` scorer at the layer configuration; "
                         "sweep: config 3's k / L / p sweep, one line per point")
    ap.add_argument("--seq-len", type=int, default=None, help="profiling only: override S")
    ap.add_argument("--cp", type=int, default=None,
                    help="model_cp: context-parallel group size (default 2, BASELINE config 5); the rest is data parallel")
    ap.add_argument("--topk", type=int, default=None, help="profiling only: override k")
    args = ap.parse_args()
    if args.seq_len and args.workload in ("layer", "scorer_gla"):
        CFG["S"] = args.seq_len
    if args.topk:
        CFG["k"] = args.topk
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl")
    try:
        if args.workload in ("model", "model_cp"):
            run_model(args, rank, world, local_rank, cp=args.workload == "model_cp")
        elif args.workload == "sweep":
            run_sweep(args, rank, world, local_rank)
        elif args.workload == "scorer_gla":
            run_scorer_gla(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
