"""htrc_b200: the flat (tree-free) HTRC attention operator for NVIDIA B200 (sm_100a).

Drop-in for the production path of ASarych/HTRC's flat operator (h3/htrc_flat.py,
h3/htrc_flat_runner.py): PyTorch host code over the C-ABI library libhtrc_flat.so of hand-written
sm_100a kernels.  See include/htrc_flat.h for the C ABI.
"""
from .flat import (PROD, dequant_rows, fake_quant, flat_attention, flat_attention_heads,  # noqa: F401
                   flat_attention_prod, forward_into, run_stages, workspace_bytes)
from .runner import CHUNKS, MODES, FlatRunner, plan_chunk, predicted_peak_mib  # noqa: F401

__all__ = ["PROD", "MODES", "CHUNKS", "flat_attention", "flat_attention_heads", "flat_attention_prod", "FlatRunner",
           "plan_chunk",
           "predicted_peak_mib", "run_stages", "workspace_bytes", "forward_into", "fake_quant", "dequant_rows"]
