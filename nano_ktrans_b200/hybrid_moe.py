"""``HybridMoE`` with the routed experts served by ``CudaMoEBackend``.

Keeps the reference layer's constructor keywords and ``forward(hidden_states,
router_logits)`` contract (nano_ktrans/layers/hybrid_moe.py:54-290,
:3310-3570).  Routing semantics are the reference's (:3321-3329), computed by
the router kernel; the offloaded experts go through the backend's
``submit_forward`` / ``sync_forward`` (:3373-3378, :3563-3567); experts marked
GPU-resident in ``gpu_experts_mask`` are served one of two ways, chosen by
``resident_experts``:

* ``"kernels"`` (default): by the same kernels, from the backend's quantized
  weights of every expert (the backend holds all of them), so route + all
  routed experts + combine are one ``moe_forward`` launch set with no host
  synchronisation — the resident/offloaded split then only decides who owns
  the weights, not how the output is computed;
* ``"modules"``: as dense ``nn.Module``s in the reference's per-expert loop
  (:3501-3533, with its host reads of the routed ids), summed with the
  backend's part (:3570) — bit-for-bit the reference's split semantics.

The reference's residency machinery (migration queues, prefetch caches,
schedulers; hybrid_moe.py:109-254, :2841-3300) is not part of this path; its
constructor keywords are accepted and ignored so existing call sites keep
working.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
from torch import nn

from .cuda_moe import CudaMoEBackend
from .offload_backend import normalize_offload_backend_name


class HybridMoE(nn.Module):
    def __init__(
        self,
        num_experts: int,
        top_k: int,
        hidden_size: int,
        moe_intermediate_size: int,
        gpu_experts: nn.ModuleDict,
        gpu_experts_mask: torch.Tensor,
        layer_idx: int,
        weight_path: str,
        num_threads: int = 16,
        numa_pools: int = 1,
        chunked_prefill_size: int = 512,
        method: str = "GPTQ",
        offload_backend: str = "cuda",
        offload_backend_kwargs: Optional[Dict[str, object]] = None,
        router_use_softmax: bool = False,
        normalize_topk_prob: bool = True,
        expert_key_template: Optional[str] = None,
        expert_proj_names: Optional[Dict[str, str]] = None,
        experts_are_packed: bool = False,
        hidden_act: str = "silu",
        resident_experts: str = "kernels",
        **_residency_kwargs,
    ):
        super().__init__()
        self.num_experts = num_experts
        self.top_k = top_k
        self.hidden_size = hidden_size
        self.gpu_experts_mask = gpu_experts_mask
        self.gpu_experts = gpu_experts
        self.layer_idx = layer_idx
        self.router_use_softmax = router_use_softmax
        self.normalize_topk_prob = normalize_topk_prob
        self.experts_are_packed = experts_are_packed
        self.hidden_act = hidden_act
        if resident_experts not in ("kernels", "modules"):
            raise ValueError("resident_experts must be 'kernels' or 'modules'")
        self.resident_experts = resident_experts
        self.has_cpu_experts = bool((~gpu_experts_mask.bool()).any().item())
        self.offload_backend_name = normalize_offload_backend_name(offload_backend)
        if self.offload_backend_name != "cuda":
            raise NotImplementedError(f"this package provides the 'cuda' backend, not '{self.offload_backend_name}'")
        if not self.has_cpu_experts and resident_experts == "modules":
            raise ValueError("every expert is GPU-resident: there is no routed-expert work for the cuda backend")
        kwargs = dict(layer_idx=layer_idx, num_experts=num_experts, top_k=top_k, hidden_size=hidden_size,
                      intermediate_size=moe_intermediate_size, gpu_experts_mask=gpu_experts_mask,
                      weight_path=weight_path, num_threads=num_threads, numa_pools=numa_pools,
                      chunked_prefill_size=chunked_prefill_size, method=method,
                      expert_key_template=expert_key_template, expert_proj_names=expert_proj_names,
                      router_use_softmax=router_use_softmax, normalize_topk_prob=normalize_topk_prob)
        kwargs.update(offload_backend_kwargs or {})
        self.offload_backend = CudaMoEBackend(**kwargs)
        self.last_topk_ids: Optional[torch.Tensor] = None
        self.last_topk_weights: Optional[torch.Tensor] = None

    def forward(self, hidden_states: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        layer = self.offload_backend.layer
        if self.resident_experts == "kernels" or not bool(self.gpu_experts_mask.bool().any()):
            t = hidden_states.shape[0]
            ids = torch.empty(t, self.top_k, dtype=torch.int64, device=hidden_states.device)
            w = torch.empty(t, self.top_k, dtype=torch.bfloat16, device=hidden_states.device)
            out = layer.forward(hidden_states, router_logits, out_ids=ids, out_weights=w)
            self.offload_backend.submit_calls += 1
            self.offload_backend.sync_calls += 1
            self.last_topk_ids, self.last_topk_weights = ids, w
            return out

        topk_ids, topk_weights = layer.route(router_logits)
        self.last_topk_ids, self.last_topk_weights = topk_ids, topk_weights
        stream = torch.cuda.current_stream(hidden_states.device).cuda_stream
        self.offload_backend.submit_forward(hidden_states, topk_ids, topk_weights, stream)

        final_gpu_states = torch.zeros_like(hidden_states)
        mask_host = self.gpu_experts_mask.bool().cpu().tolist()
        for expert_idx in torch.unique(topk_ids).cpu().tolist():
            if not mask_host[expert_idx] or str(expert_idx) not in self.gpu_experts:
                continue
            match = topk_ids == expert_idx
            token_indices = torch.where(match.any(dim=1))[0]
            expert_output = self.gpu_experts[str(expert_idx)](hidden_states[token_indices])
            weights = topk_weights[token_indices][match[token_indices]]
            final_gpu_states.index_add_(0, token_indices, expert_output * weights.unsqueeze(1))

        cpu_output = self.offload_backend.sync_forward(hidden_states, stream)
        return final_gpu_states + cpu_output

    def diagnostics(self) -> dict:
        return {"layer_idx": self.layer_idx, "offload_backend": self.offload_backend.diagnostics()}
