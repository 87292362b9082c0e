"""Inference-only SOL routed block-sparse BF16 attention for NVIDIA B200 (sm_100a).

Drop-in for the public API of zihaomu/SolAttn-AMD (``src/sol_attn_amd/__init__.py:6``).
"""

from .attention import SolStats, dense_attention, dense_attention_rows, sol_attention
from .host import sol_attention_host
from .indexed import IndexedPlan, sol_attention_indexed

# The reference's public names (``__init__.py:6``) plus the host-buffer entry point and the
# in-place dense step for global query rows.
__all__ = ["SolStats", "dense_attention", "sol_attention", "IndexedPlan", "sol_attention_indexed",
           "sol_attention_host", "dense_attention_rows"]
