"""B200 (sm_100a) backend for the vxg-tensor Q8-KV decode attention / gated-DeltaNet hot path.

The compute lives in ``libvxg_attn_cuda.so`` (hand-written CUDA behind the C ABI of
``include/vxg_attn_cuda.h``); this package is its Python host layer.  There is no CPU fallback:
importing the operators requires the built library and calling them requires an sm_100 GPU.
"""
from ._lib import VxgError, lib  # noqa: F401
from .attn import (Context, KvF32Pool, KvQ8Block, KvQ8Pool, deltanet_prefill,  # noqa: F401
                   deltanet_step, lse_combine, lse_combine_packed, step_deltanet_recurrent,
                   step_full_gqa, step_full_gqa_q8)

__all__ = ["VxgError", "Context", "KvF32Pool", "KvQ8Block", "KvQ8Pool", "step_full_gqa", "deltanet_prefill", "deltanet_step",
           "lse_combine", "lse_combine_packed", "step_deltanet_recurrent", "step_full_gqa_q8",
           "lib"]
