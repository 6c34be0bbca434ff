"""Seeded inputs for the golden fixtures (shared by make_golden.py and the tests).

Inputs are drawn on the CPU from torch.Generator seeds, so every machine with
the same torch version produces the same bits; the fixtures store a checksum
to detect any drift.
"""
from __future__ import annotations

import hashlib

import torch

# name: (B, S, H, D, L, p, dtype, seed)
SCORER_CASES = {
    "f32_L3p4": (1, 256, 2, 128, 3, 4, torch.float32, 11),
    "bf16_L3p4": (1, 256, 2, 128, 3, 4, torch.bfloat16, 12),
    "bf16_L4p2": (1, 128, 2, 64, 4, 2, torch.bfloat16, 13),
    "bf16_L3p8": (1, 256, 1, 128, 3, 8, torch.bfloat16, 14),
}

# name: (B, H, N, L, p, k, score mode, seed)
SELECT_CASES = {
    "n512_L2p2_k128_randn": (1, 2, 512, 2, 2, 128, "randn", 21),
    "n512_L2p2_k128_ties": (1, 2, 512, 2, 2, 128, "ties2", 22),
    "n4096_L3p4_k256_randn": (1, 2, 4096, 3, 4, 256, "randn", 23),
    "n4096_L3p4_k256_bf16norm": (1, 2, 4096, 3, 4, 256, "bf16norm", 24),
    "n4096_L3p4_k256_allsame": (1, 1, 4096, 3, 4, 256, "allsame", 25),
    "n8192_L3p2_k256_ties": (1, 2, 8192, 3, 2, 256, "ties2", 26),
    "n16384_L4p2_k256_bf16norm": (1, 1, 16384, 4, 2, 256, "bf16norm", 27),
    "n8192_L2p8_k128_randn": (1, 1, 8192, 2, 8, 128, "randn", 28),
    "n24576_L3p4_k1536_bf16norm": (1, 1, 24576, 3, 4, 1536, "bf16norm", 29),
}

# name: (B, H, N, D, L, p, k, seed)
SCATTER_CASES = {
    "n512_L2p2": (1, 2, 512, 16, 2, 2, 128, 31),
    "n4096_L3p4": (1, 1, 4096, 8, 3, 4, 256, 32),
}

# name: (B, S, H, D, L, p, k, seed)
LAYER_CASES = {
    "s4096_L3p4_k256": (1, 4096, 1, 16, 3, 4, 256, 41),
}

# name: (B, S, H, D, dilation, L, p, dtype, gate divisor, seed); the gate is
# logsigmoid(N(0,1)) / divisor per (token, head), as PATCH:709 makes it
GLA_CASES = {
    "f32_d16_di4": (1, 256, 2, 16, 4, 3, 4, torch.float32, 16.0, 51),
    "f32_d32_di2": (2, 512, 1, 32, 2, 2, 2, torch.float32, 1.0, 52),
    "bf16_d128_di4": (1, 2048, 2, 128, 4, 3, 4, torch.bfloat16, 16.0, 53),
    "bf16_d128_ragged": (1, 1600, 2, 128, 4, 3, 4, torch.bfloat16, 2.0, 54),
}


def pyramid_len(N, L, p):
    return sum(N // p ** l for l in range(L))


def make_qkv(B, S, H, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(B, S, H, D, generator=g).to(dtype) for _ in range(3))


def make_gate(B, S, H, div, seed):
    g = torch.Generator().manual_seed(seed + 1000)
    return torch.nn.functional.logsigmoid(torch.randn(B, S, H, generator=g)) / div


def make_scores(B, H, N, L, p, mode, seed):
    """(scores_qk, scores_kq) fp32 (B, H, S_tot) pyramids built like the norm
    scorer: level-l score = max over the p^l raw scores it covers."""
    g = torch.Generator().manual_seed(seed)
    if mode == "randn":
        raw = torch.randn(2, B, H, N, generator=g).abs()
    elif mode == "ties2":
        raw = torch.randint(0, 2, (2, B, H, N), generator=g).float()
    elif mode == "allsame":
        raw = torch.ones(2, B, H, N)
    elif mode == "bf16norm":   # bf16-rounded norms of N(0,1) rows of width 128: heavy ties
        raw = torch.randn(2, B, H, N, 128, generator=g).norm(dim=-1).to(torch.bfloat16).float()
    else:
        raise ValueError(mode)
    out = []
    for r in raw:
        levels = [r]
        for l in range(1, L):
            f = p ** l
            n = N // f
            levels.append(r[..., : n * f].reshape(B, H, n, f).amax(-1))
        out.append(torch.cat(levels, dim=-1).contiguous())
    return out[0], out[1]


def checksum(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(t.detach().contiguous().view(torch.uint8).numpy().tobytes() if t.dtype != torch.bfloat16
                 else t.detach().contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()
