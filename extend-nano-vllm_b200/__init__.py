"""B200-native (sm_100a) Qwen3-MoE expert-execution path for extend-nano-vLLM.

Import as ``extend_nano_vllm_b200`` (the repository root module of that name
loads this directory).  The public surface is ``ExpertParallelMoE``, a drop-in
for ``nanovllm.layers.moe.ExpertParallelMoE``, plus the tensor-level kernel
wrappers in ``ops`` and the ctypes binding in ``_lib``.
"""

from ._lib import B200MoEError, LIB_PATH, device_status
from .moe import (
    DISPATCH_BACKENDS, MOE_MAX_GRAPH_TOKENS_PER_RANK, STREAM_ENGINE_MAX_ROUTES,
    ExpertParallelMoE, SharedExpertMLP, reduce_fp64_to_bf16,
)
from . import ops

__all__ = [
    "B200MoEError", "LIB_PATH", "device_status", "DISPATCH_BACKENDS",
    "MOE_MAX_GRAPH_TOKENS_PER_RANK", "STREAM_ENGINE_MAX_ROUTES", "ExpertParallelMoE",
    "SharedExpertMLP", "reduce_fp64_to_bf16", "ops",
]
