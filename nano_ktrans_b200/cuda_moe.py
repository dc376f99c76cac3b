"""``CudaMoEBackend``: the routed-expert backend served by the B200 kernels.

A drop-in ``ExpertOffloadBackend`` (nano_ktrans/kernels/offload_backend.py:29-90)
taking the same constructor keywords as the reference ``CPUMoEBackend``
(nano_ktrans/kernels/cpu_moe.py:160-175).  It computes the experts whose
``gpu_experts_mask`` entry is False — the part the reference's CPU backend
computes with its GPTQ W4A32 path (cpu_moe.py:491-539) — on the device, from
quantized weights, with no host round trip:

* ``submit_forward`` enqueues the whole routed-expert step on ``cuda_stream``
  (the stream ``HybridMoE.forward`` passes, hybrid_moe.py:3373-3378) and
  returns immediately;
* ``sync_forward`` returns the bf16 ``[T, H]`` result, ordered after the
  submit on the caller's stream.

Weights come either from ``weight_path`` (GPTQ safetensors, as the reference
loads them, cpu_moe.py:324-387) or, for synthetic layers, from
``gptq_experts`` / ``layer_weights`` keyword arguments.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

from .moe_layer import MoeLayer
from .offload_backend import ExpertOffloadBackend
from .weight_loader import ExpertWeightLoader
from .weights import GPTQLinearWeight, LayerWeights, stack_layer


class CudaMoEBackend(ExpertOffloadBackend):
    backend_name = "cuda"

    def __init__(
        self,
        layer_idx: int,
        num_experts: int,
        top_k: int,
        hidden_size: int,
        intermediate_size: int,
        gpu_experts_mask: torch.Tensor,
        weight_path: str = "",
        num_threads: int = 16,
        numa_pools: int = 1,
        chunked_prefill_size: int = 512,
        method: str = "GPTQ",
        expert_key_template: Optional[str] = None,
        expert_proj_names: Optional[Dict[str, str]] = None,
        *,
        device: Optional[torch.device] = None,
        gptq_experts: Optional[Dict[int, Dict[str, GPTQLinearWeight]]] = None,
        layer_weights: Optional[LayerWeights] = None,
        router_use_softmax: bool = True,
        normalize_topk_prob: bool = True,
        max_tokens: int = 4096,
    ):
        super().__init__()
        self.layer_idx = layer_idx
        self.num_experts = num_experts
        self.top_k = top_k
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.method = method
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise ValueError("CudaMoEBackend runs on a CUDA device only")
        self.gpu_experts_mask = gpu_experts_mask.to(dtype=torch.bool, device="cpu").clone()
        self._offload_mask_dev = (~self.gpu_experts_mask).to(dtype=torch.uint8, device=self.device)
        if layer_weights is None:
            if gptq_experts is None:
                gptq_experts = self._load_gptq(weight_path, expert_key_template, expert_proj_names)
            missing = [e for e in range(num_experts) if e not in gptq_experts]
            if missing:
                raise ValueError(f"GPTQ weights missing for experts {missing[:8]}")
            layer_weights = stack_layer([gptq_experts[e] for e in range(num_experts)], self.device)
        self.layer = MoeLayer(layer_weights, top_k=top_k, router_use_softmax=router_use_softmax,
                              normalize_topk_prob=normalize_topk_prob, max_tokens=max_tokens)
        self._pending: Optional[torch.Tensor] = None
        self._pending_event: Optional[torch.cuda.Event] = None
        self.last_launches = 0

    def _load_gptq(self, weight_path, key_template, proj_names) -> Dict[int, Dict[str, GPTQLinearWeight]]:
        loader = ExpertWeightLoader(weight_path)
        tmpl = key_template or "model.layers.{layer}.block_sparse_moe.experts.{expert}.{proj}.weight"
        names = proj_names or {"gate": "w1", "up": "w3", "down": "w2"}
        out: Dict[int, Dict[str, GPTQLinearWeight]] = {}
        for e in range(self.num_experts):
            out[e] = {p: loader.load_gptq_expert_linear(layer_idx=self.layer_idx, expert_idx=e, proj_name=p,
                                                        key_template=tmpl, proj_name_map=names)
                      for p in ("gate", "up", "down")}
        return out

    # ------------------------------------------------------------------
    def submit_forward(self, hidden_states: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                       cuda_stream: int | None) -> None:
        self.submit_calls += 1
        flat = hidden_states.view(-1, hidden_states.shape[-1])
        if not flat.is_cuda:
            raise ValueError("CudaMoEBackend.submit_forward needs CUDA hidden states")
        x = flat if flat.dtype == torch.bfloat16 else flat.to(torch.bfloat16)
        stream = cuda_stream if cuda_stream is not None else torch.cuda.current_stream(flat.device).cuda_stream
        out = self.layer.experts_forward(x, topk_ids.view(x.shape[0], -1), topk_weights.view(x.shape[0], -1),
                                         offload_mask=self._offload_mask_dev, stream=stream)
        self.last_launches = self.layer.last_launch_count()
        ev = torch.cuda.Event()
        ev.record(torch.cuda.ExternalStream(stream) if cuda_stream is not None else torch.cuda.current_stream())
        self._pending, self._pending_event = out, ev

    def sync_forward(self, hidden_states: torch.Tensor, cuda_stream: int | None) -> torch.Tensor:
        self.sync_calls += 1
        if self._pending is None:
            return torch.zeros_like(hidden_states)
        stream = torch.cuda.ExternalStream(cuda_stream) if cuda_stream is not None else torch.cuda.current_stream()
        stream.wait_event(self._pending_event)
        out = self._pending
        self._pending, self._pending_event = None, None
        if out.dtype != hidden_states.dtype:
            out = out.to(hidden_states.dtype)
        return out.view_as(hidden_states)

    def update_gpu_expert_mask(self, gpu_experts_mask: torch.Tensor) -> None:
        self.gpu_experts_mask = gpu_experts_mask.to(dtype=torch.bool, device="cpu").clone()
        self._offload_mask_dev = (~self.gpu_experts_mask).to(dtype=torch.uint8, device=self.device)

    def diagnostics(self) -> dict:
        d = super().diagnostics()
        d.update({
            "backend_name": self.backend_name,
            "layer_idx": self.layer_idx,
            "method": self.method,
            "bits": self.layer.weights.bits,
            "offloaded_experts": int((~self.gpu_experts_mask).sum().item()),
            "last_kernel_launches": self.last_launches,
            "expert_bytes": self.layer.weights.expert_bytes(),
        })
        return d
