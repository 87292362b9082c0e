"""Inference-only SOL routed block-sparse BF16 attention for NVIDIA B200 (sm_100a).

Drop-in for the public API of zihaomu/SolAttn-AMD (``src/sol_attn_amd/__init__.py:6``).
"""

from .attention import SolStats, dense_attention, sol_attention
from .indexed import IndexedPlan, sol_attention_indexed

__all__ = ["SolStats", "dense_attention", "sol_attention", "IndexedPlan", "sol_attention_indexed"]
