"""mosaic_b200 — B200-native (sm_100a) MoE-layer hot path of Mosaic.

Router (sigmoid / sqrt-softplus / softmax scores, group-limited top-k,
selection-only bias; hash routing by token id), histogram / scan
permutation, MXFP4 x E4M3 block-scaled tcgen05 expert GEMMs with a fused
SwiGLU epilogue, shared expert and ordered combine, behind the reference's
MoE module / operator API; expert parallelism across GPUs in ``ep``.  The
CUDA library is loaded lazily; building it is ``python -m mosaic_b200.build``.
"""
from .moe import (  # noqa: F401
    ExactContractError,
    ExpertBank,
    HashMoELayer,
    HashRouter,
    MoEConfig,
    MoELayer,
    Router,
    exact_moe,
    exact_target,
    grouped_expert_forward,
)
from .ep import ExpertParallelMoELayer, PeerFailure, PeerHealth, expert_range, shard_bank  # noqa: F401
from .pipeline import HostPipeline  # noqa: F401

__all__ = [
    "ExactContractError",
    "ExpertBank",
    "ExpertParallelMoELayer",
    "HashMoELayer",
    "HashRouter",
    "HostPipeline",
    "MoEConfig",
    "MoELayer",
    "PeerFailure",
    "PeerHealth",
    "Router",
    "exact_moe",
    "exact_target",
    "expert_range",
    "grouped_expert_forward",
    "shard_bank",
]
