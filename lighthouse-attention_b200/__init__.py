"""lighthouse_b200 — B200 (sm_100a) implementation of Lighthouse selection attention.

The directory is named ``lighthouse-attention_b200``; it is imported under the
package name ``lighthouse_b200`` (``load_package`` in __graft_entry__.py does
that with importlib).  Modules:

  lighthouse_selection       drop-in for the reference module of the same name
  lighthouse_selection_cuda  drop-in for the reference module of the same name
  cp                         context-parallel layer (NCCL all-gather of selected K/V)
  _native                    ctypes binding of liblighthouse_b200.so (include/lighthouse_b200.h)
"""
from . import _native  # noqa: F401
from . import library  # noqa: F401  (registers the lighthouse_b200:: custom ops)
from .lighthouse_selection import (DialatedLighthouseNormScorer, DialatedLighthouseNormScorerCP,  # noqa: F401
                                   DilatedLighthouseGLAScorer, DilatedLighthouseScorer, LighthouseCP,
                                   LighthouseLocal, compute_output_indices_selection, lighthouse_attention,
                                   scatter_to_base_sequence)
from .lighthouse_selection_cuda import LighthouseSelectionQkKqChunkedTopkNvrtc  # noqa: F401
