"""nano_ktrans_b200 — B200 (sm_100a) device backend for nano-ktrans's routed-expert MoE path.

Public API (mirrors the reference's names):

* ``GPTQLinearWeight``, ``quantize_symmetric`` — quantized-weight container
* ``ExpertOffloadBackend``, ``normalize_offload_backend_name`` — plugin interface
* ``CudaMoEBackend`` — the ``"cuda"`` expert backend
* ``HybridMoE`` — the MoE layer using it
* ``MoeLayer`` — direct access to the C-ABI handle (route / experts / fused forward)
* ``EpMoeLayer``, ``plan_placement``, ``shard_layer``, ``TorchDistComm``,
  ``PeerExchange`` — expert parallelism over the ranks of a process group (NCCL
  all-to-alls, or the library's kernels over peer memory)
"""
from .offload_backend import ExpertOffloadBackend, normalize_offload_backend_name
from .weights import GPTQLinearWeight, LayerWeights, quantize_symmetric, stack_layer

__all__ = [
    "ExpertOffloadBackend", "normalize_offload_backend_name", "GPTQLinearWeight", "LayerWeights",
    "quantize_symmetric", "stack_layer", "CudaMoEBackend", "HybridMoE", "MoeLayer",
    "EpMoeLayer", "plan_placement", "shard_layer", "TorchDistComm", "PeerExchange",
]


def __getattr__(name):
    if name == "CudaMoEBackend":
        from .cuda_moe import CudaMoEBackend
        return CudaMoEBackend
    if name == "HybridMoE":
        from .hybrid_moe import HybridMoE
        return HybridMoE
    if name == "MoeLayer":
        from .moe_layer import MoeLayer
        return MoeLayer
    if name in ("EpMoeLayer", "plan_placement", "shard_layer", "TorchDistComm", "PeerExchange"):
        from . import expert_parallel
        return getattr(expert_parallel, name)
    raise AttributeError(name)
