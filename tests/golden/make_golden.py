"""Generate the golden vectors in this folder from the REFERENCE's own code.

Run in the build container (the reference tree is not on the GPU box):

    python tests/golden/make_golden.py          # every fixture
    python tests/golden/make_golden.py gla      # only gla.npz

What produces each fixture (reference paths inside the reference project):
  scorer.npz     DialatedLighthouseNormScorer.forward (src/lighthouse_selection.py:589-616),
                 imported unmodified and run on CPU in fp32 and bf16.
  select.npz     lighthouse_selection_chunked_topk_kernel (src/lighthouse_selection_cuda.py:114-330),
                 its own source rendered by _make_kernel_source and run on host threads
                 (oracle/build.py, oracle/_ref/libref_cpu_p*.so), followed by the
                 stable sort + gather of src/lighthouse_selection_cuda.py:425-427.
  scatter.npz    _ScatterToBaseAutograd forward/backward with the reference Triton
                 kernels (src/lighthouse_selection.py:408-576) in Triton's CPU interpreter.
  gla.npz        DilatedLighthouseGLAScorer.forward (src/lighthouse_selection.py:711-755),
                 imported unmodified and run on CPU, with its `chunk_simple_gla` (the
                 external flash-linear-attention package, fla 0.5.1, whose Triton
                 kernels need a GPU) replaced by that package's own reference
                 implementation of the same function, `naive_recurrent_simple_gla`.
  layer.npz      LighthouseLocal's forward (src/lighthouse_selection.py:789-825) composed
                 from the pieces above and CPU SDPA (selection from the reference kernel
                 source on host threads, since the reference asserts CUDA for it).
Inputs are regenerated from torch.Generator seeds by tests/golden/inputs.py;
the fixtures store a checksum of them.
"""
from __future__ import annotations

import importlib.util
import os
import pathlib
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from inputs import (GLA_CASES, SCORER_CASES, SELECT_CASES, SCATTER_CASES, LAYER_CASES, checksum, make_gate,
                    make_scores, make_qkv)  # noqa: E402

# The reference tree: LH_REFERENCE_ROOT, else the build container's mount point.
REF = pathlib.Path(os.environ.get("LH_REFERENCE_ROOT", "/root/reference")) / "src"


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    m = importlib.util.module_from_spec(spec)
    sys.modules[name] = m
    spec.loader.exec_module(m)
    return m


def load_reference():
    for pkg in ["torchtitan", "torchtitan.models", "torchtitan.models.llama3", "torchtitan.models.llama3.model"]:
        if pkg not in sys.modules:
            try:
                __import__(pkg)
            except Exception:
                sys.modules[pkg] = types.ModuleType(pkg)
    _load("torchtitan.models.llama3.model.lighthouse_selection_cuda", REF / "lighthouse_selection_cuda.py")
    return _load("torchtitan.models.llama3.model.lighthouse_selection", REF / "lighthouse_selection.py")


def make_gla(sel):
    from fla.ops.simple_gla.naive import naive_recurrent_simple_gla

    def chunk_simple_gla(q, k, v, g, scale=None):
        o, _ = naive_recurrent_simple_gla(q, k, v, g, scale=scale, output_final_state=False)
        return o.contiguous(), None          # chunk_simple_gla returns a contiguous (B, T, H, D) tensor

    sel.chunk_simple_gla = chunk_simple_gla
    out = {}
    for name, (B, S, H, D, di, L, p, dtype, div, seed) in GLA_CASES.items():
        xq, xk, xv = make_qkv(B, S, H, D, dtype, seed)
        gk = make_gate(B, S, H, div, seed)
        with torch.no_grad():
            sqk, skq, qc, kc, vc = sel.DilatedLighthouseGLAScorer(D, dilation=di, pooling_factor=p, levels=L)(
                xq, xk, xv, gk)
        out[f"{name}/checksum"] = np.array(checksum(xq, xk, xv, gk))
        out[f"{name}/scores_qk"] = sqk.float().numpy()
        out[f"{name}/scores_kq"] = skq.float().numpy()
        if D <= 32:                               # the pooling is the norm scorer's; keep the file small
            out[f"{name}/pooled_q"] = qc[:, :, S:].float().numpy()
    np.savez_compressed(HERE / "gla.npz", **out)
    print("gla", (HERE / "gla.npz").stat().st_size, "bytes")


def main():
    if sys.argv[1:] == ["gla"]:
        make_gla(load_reference())
        return
    from oracle import build as ob, oracle as O
    ob.build_oracle()
    ob.build_ref(gpu=False)
    sel = load_reference()

    out = {}
    for name, (B, S, H, D, L, p, dtype, seed) in SCORER_CASES.items():
        xq, xk, xv = make_qkv(B, S, H, D, dtype, seed)
        with torch.no_grad():
            sqk, skq, qc, kc, vc = sel.DialatedLighthouseNormScorer(p, L)(xq, xk, xv)
        out[f"{name}/checksum"] = np.array(checksum(xq, xk, xv))
        out[f"{name}/scores_qk"] = sqk.float().numpy()
        out[f"{name}/scores_kq"] = skq.float().numpy()
        for t, c in (("q", qc), ("k", kc), ("v", vc)):
            out[f"{name}/pooled_{t}"] = c[:, :, S:].float().numpy()  # levels >= 1
    np.savez_compressed(HERE / "scorer.npz", **out)

    out = {}
    for name, (B, H, N, L, p, k, mode, seed) in SELECT_CASES.items():
        sq, sk = make_scores(B, H, N, L, p, mode, seed)
        idx = O.ref_select_cpu(sq, sk, L, p, k, N)
        out[f"{name}/checksum"] = np.array(checksum(sq, sk))
        out[f"{name}/indices"] = idx.numpy()
    np.savez_compressed(HERE / "select.npz", **out)

    out = {}
    for name, (B, H, N, D, L, p, k, seed) in SCATTER_CASES.items():
        sq, sk = make_scores(B, H, N, L, p, "randn", seed)
        idx = O.ref_select_cpu(sq, sk, L, p, k, N)
        g = torch.Generator().manual_seed(seed + 1)
        attn = torch.randn(B, H, idx.shape[-1], D, generator=g).requires_grad_(True)
        dout = torch.randn(B, H, N, D, generator=g)
        res = sel.scatter_to_base_sequence(attn, idx, torch.zeros_like(idx), N, N, L, p)
        res.backward(dout)
        out[f"{name}/indices"] = idx.numpy()
        out[f"{name}/attn"] = attn.detach().numpy()
        out[f"{name}/dout"] = dout.numpy()
        out[f"{name}/out"] = res.detach().numpy()
        out[f"{name}/dattn"] = attn.grad.numpy()
    np.savez_compressed(HERE / "scatter.npz", **out)

    out = {}
    for name, (B, S, H, D, L, p, k, seed) in LAYER_CASES.items():
        xq, xk, xv = make_qkv(B, S, H, D, torch.float32, seed)
        with torch.no_grad():
            sqk, skq, qc, kc, vc = sel.DialatedLighthouseNormScorer(p, L)(xq, xk, xv)
            idx = O.ref_select_cpu(sqk.float(), skq.float(), L, p, k, S)
            g = lambda x: torch.gather(x, 2, idx.long().unsqueeze(-1).expand(-1, -1, -1, D))
            attn = torch.nn.functional.scaled_dot_product_attention(g(qc), g(kc), g(vc), is_causal=True)
            res = sel.scatter_to_base_sequence(attn, idx, torch.zeros_like(idx), S, S, L, p)
        out[f"{name}/checksum"] = np.array(checksum(xq, xk, xv))
        out[f"{name}/indices"] = idx.numpy()
        out[f"{name}/out"] = res.numpy()
    np.savez_compressed(HERE / "layer.npz", **out)
    make_gla(sel)
    for f in ("scorer", "select", "scatter", "layer"):
        print(f, (HERE / f"{f}.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
