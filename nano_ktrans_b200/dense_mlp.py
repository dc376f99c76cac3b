"""``QuantizedDenseMLP``: a dense decoder layer's MLP served by the routed-expert
kernels.

The reference builds, for the layers that are not MoE layers
(``first_k_dense_replace``, ``mlp_only_layers``, ``decoder_sparse_step``;
nano_ktrans/models/config.py:184-197), a plain ``SparseExpertMLP``
(nano_ktrans/models/mixtral.py:180-189, layers/expert_mlp.py:9-25):
``w2(silu(w1 x) * w3 x)``.  Here that MLP holds GPTQ-quantized weights and runs
as one always-on expert over every token: expert ids all 0, routing weights
all 1.0, so the combine's single bf16 rounding of ``1.0 * y`` returns
``bf16(y)`` with ``y`` accumulated in fp32 exactly as a routed expert's.  The
projections take the same kernels as routed experts: the single-launch decode
kernels for a few tokens, the weight-streaming kernels for small batches and
the tensor-core grouped GEMM for long prefills.
"""
from __future__ import annotations

from typing import Optional

import torch

from .moe_layer import MoeLayer
from .weights import GPTQLinearWeight, LayerWeights, stack_layer


def is_moe_layer(layer_idx: int, *, first_k_dense_replace: int = 0, mlp_only_layers=(),
                 decoder_sparse_step: int = 1, num_local_experts: int = 1, num_experts_per_tok: int = 1,
                 attention_backend: str = "standard") -> bool:
    """Whether decoder layer ``layer_idx`` has an MoE block (models/config.py:184-197)."""
    if attention_backend != "standard" or num_local_experts <= 0 or num_experts_per_tok <= 0:
        return False
    if layer_idx < first_k_dense_replace or layer_idx in set(mlp_only_layers):
        return False
    step = max(int(decoder_sparse_step or 1), 1)
    return (layer_idx + 1) % step == 0


class QuantizedDenseMLP:
    """``forward(x [T, H] bf16) -> [T, H] bf16`` = ``down(silu(gate(x)) * up(x))``.

    Built from ``gate`` / ``up`` / ``down`` ``GPTQLinearWeight`` (the reference's
    ``w1`` / ``w3`` / ``w2``) or from a one-expert ``LayerWeights``.
    """

    def __init__(self, gate: Optional[GPTQLinearWeight] = None, up: Optional[GPTQLinearWeight] = None,
                 down: Optional[GPTQLinearWeight] = None, *, device=None, layer_weights: Optional[LayerWeights] = None,
                 max_tokens: int = 4096):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if layer_weights is None:
            if gate is None or up is None or down is None:
                raise ValueError("QuantizedDenseMLP needs gate, up and down weights (or layer_weights)")
            layer_weights = stack_layer([{"gate": gate, "up": up, "down": down}], self.device)
        if layer_weights.num_experts != 1 or layer_weights.shared is not None:
            raise ValueError("a dense MLP is one expert without a shared expert")
        self.weights = layer_weights
        self.hidden_size = layer_weights.hidden_size
        self.intermediate_size = layer_weights.inter_size
        self.max_tokens = max_tokens
        self.layer = MoeLayer(layer_weights, top_k=1, router_use_softmax=False, normalize_topk_prob=False,
                              max_tokens=max_tokens)
        # the always-on routing: expert 0 with weight 1.0 for every token
        self._ids = torch.zeros(max_tokens, 1, dtype=torch.int64, device=self.device)
        self._w = torch.ones(max_tokens, 1, dtype=torch.bfloat16, device=self.device)

    def forward(self, x: torch.Tensor, *, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        t = int(x.shape[0])
        if t > self.max_tokens:
            raise ValueError(f"{t} tokens above max_tokens {self.max_tokens}")
        return self.layer.experts_forward(x, self._ids[:t], self._w[:t], out=out, stream=stream)

    __call__ = forward

    def last_launch_count(self) -> int:
        return self.layer.last_launch_count()

    def close(self) -> None:
        self.layer.close()
