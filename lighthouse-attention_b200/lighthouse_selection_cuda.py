"""Drop-in for the reference module ``lighthouse_selection_cuda``.

Same names, arguments and error behaviour as src/lighthouse_selection_cuda.py
of the reference (:346-429); the NVRTC kernel + torch.sort + torch.gather are
replaced by one sm_100a selection kernel (``lh_select_topk``) that writes the
position-ordered indices directly.
"""
from __future__ import annotations

from functools import lru_cache

import torch

from . import _native


@lru_cache(maxsize=100, typed=False)
def compute_output_indices_selection(N: int, num_levels: int, pooling_factor: int, topk: int) -> int:
    """Selected-sequence length S_sel (reference :346-357)."""
    total = 0
    for level in range(num_levels, 0, -1):
        c_l = pooling_factor ** (level - 1)
        total += N // c_l if level == num_levels else pooling_factor * topk
    return total


class LighthouseSelectionQkKqChunkedTopkNvrtc:
    """Hierarchical qk/kq chunked top-k (reference :359-429)."""

    @torch.no_grad()
    @staticmethod
    def forward(scores_qk: torch.Tensor, scores_kq: torch.Tensor, num_levels: int, pooling_factor: int,
                topk: int, actual_seq_len: int) -> torch.Tensor:
        # Preconditions as asserted by the reference (:370-375, 385, 391)
        assert scores_qk.shape == scores_kq.shape
        assert scores_qk.is_cuda and scores_kq.is_cuda
        assert scores_qk.dtype == torch.float32
        assert topk % 128 == 0, "topk must be a multiple of 128"
        assert (pooling_factor & (pooling_factor - 1)) == 0, "pf must be power of 2"
        assert topk // 2 >= pooling_factor
        assert topk // 128 >= 1, "topk must be >= 128"
        coarsest = actual_seq_len
        for _ in range(num_levels - 1):
            coarsest //= pooling_factor
        n_chunk_coarsest = coarsest // (topk // 128)
        assert n_chunk_coarsest >= 128, (
            f"N_CHUNK_COARSEST={n_chunk_coarsest} must be >= TOPK_PER_TILE=128")
        idx, _ = _native.select_topk(scores_qk, scores_kq, num_levels, pooling_factor, topk, actual_seq_len,
                                     with_inverse=False)
        return idx
