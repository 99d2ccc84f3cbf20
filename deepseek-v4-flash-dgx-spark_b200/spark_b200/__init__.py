"""spark_b200: B200 (sm_100a) routed-expert MoE hot path of DeepSeek-V4-Flash.

Drop-in for the reference runtime's MoE layer (``LazyMoE`` / official ``MoE``,
``Gate``, ``Expert``), its expert arena and its native packed-slab loader.
Compute runs in libdsv4moe.so (hand-written CUDA for sm_100a) through the C
ABI in include/dsv4moe.h, reached from torch as ``torch.ops.dsv4moe.*``
(libdsv4moe_torch.so); there is no CPU fallback.
"""

from ._lib import load as load_library  # noqa: F401
from .ops import load as load_ops  # noqa: F401
from .moe import Expert, ExpertArena, Gate, ModelArgs, MoE, packed_block_bytes, packed_block_layout  # noqa: F401

__all__ = ["Expert", "ExpertArena", "Gate", "ModelArgs", "MoE", "load_library", "load_ops", "packed_block_bytes",
           "packed_block_layout"]
