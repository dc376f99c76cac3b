"""GPTQ safetensors reader for routed-expert weights.

Follows the reference loader's on-disk contract
(nano_ktrans/kernels/weight_loader.py:99-141 key index, :278-325
``load_gptq_linear``, :327-353 ``load_gptq_expert_linear``):

* ``<prefix>.qweight`` int32 ``[K*bits/32, N]`` (transposed on disk),
* ``<prefix>.scales`` ``[K/group, N]`` or ``[N, K/group]``,
* optional ``<prefix>.g_idx`` — only sequential grouping is accepted,
* optional ``<prefix>.qzeros`` — accepted only for symmetric checkpoints
  (asymmetric raises, as the reference does),
* ``quantize_config.json`` (or ``config.json``) supplies bits / group_size / sym.
"""
from __future__ import annotations

import json
import os
from glob import glob
from typing import Dict, Optional

import torch
from safetensors import safe_open

from .weights import GPTQLinearWeight


class ExpertWeightLoader:
    def __init__(self, weight_path: str):
        self.weight_path = weight_path
        self._key_to_file: Dict[str, str] = {}
        self._quantize_config: Dict[str, object] = {}
        if not weight_path:
            return
        files = sorted(glob(os.path.join(weight_path, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"No .safetensors files found in {weight_path}")
        for f in files:
            with safe_open(f, "pt", "cpu") as sf:
                for key in sf.keys():
                    self._key_to_file[key] = f
        for name in ("quantize_config.json", "config.json"):
            p = os.path.join(weight_path, name)
            if os.path.exists(p):
                with open(p) as fh:
                    cfg = json.load(fh)
                self._quantize_config = cfg.get("quantization_config", cfg) if name == "config.json" else cfg
                break

    @property
    def quantize_config(self) -> Dict[str, object]:
        return self._quantize_config

    def has_key(self, key: str) -> bool:
        return key in self._key_to_file

    def _load_tensor(self, key: str) -> torch.Tensor:
        f = self._key_to_file.get(key)
        if f is None:
            raise KeyError(f"Weight key '{key}' not found in safetensors files.")
        with safe_open(f, "pt", "cpu") as sf:
            return sf.get_tensor(key).contiguous()

    @staticmethod
    def _normalize_scale_layout(scales: torch.Tensor, *, output_dim: int, num_groups: int) -> torch.Tensor:
        if tuple(scales.shape) == (output_dim, num_groups):
            return scales.to(torch.float32).contiguous()
        if tuple(scales.shape) == (num_groups, output_dim):
            return scales.transpose(0, 1).to(torch.float32).contiguous()
        raise ValueError(f"Unsupported GPTQ scales shape: expected {(output_dim, num_groups)} or "
                         f"{(num_groups, output_dim)}, got {tuple(scales.shape)}")

    def load_gptq_linear(self, linear_prefix: str, *, bits: Optional[int] = None, group_size: Optional[int] = None,
                         sym: Optional[bool] = None) -> GPTQLinearWeight:
        bits = int(bits or self._quantize_config.get("bits", 4))
        group_size = int(group_size or self._quantize_config.get("group_size", 128))
        sym = bool(self._quantize_config.get("sym", True) if sym is None else sym)
        qweight = self._load_tensor(f"{linear_prefix}.qweight").transpose(0, 1).to(torch.int32).contiguous()
        output_dim = qweight.shape[0]
        input_dim = qweight.shape[1] * (32 // bits)
        if group_size <= 0:
            group_size = input_dim
        num_groups = (input_dim + group_size - 1) // group_size
        g_key = f"{linear_prefix}.g_idx"
        if g_key in self._key_to_file:
            g_idx = self._load_tensor(g_key).to(torch.long)
            expected = torch.arange(input_dim, dtype=torch.long) // group_size
            if g_idx.numel() < input_dim or not torch.equal(g_idx[:input_dim], expected):
                raise NotImplementedError("Only sequential GPTQ grouping is supported.")
        scales = self._normalize_scale_layout(self._load_tensor(f"{linear_prefix}.scales"), output_dim=output_dim,
                                              num_groups=num_groups)
        if f"{linear_prefix}.qzeros" in self._key_to_file and not sym:
            raise NotImplementedError("Asymmetric GPTQ is not supported.")
        return GPTQLinearWeight(qweight=qweight, scales=scales, zero_points=None, group_size=group_size, bits=bits,
                                sym=sym, linear_prefix=linear_prefix)

    def load_gptq_expert_linear(self, *, layer_idx: int, expert_idx: int, proj_name: str,
                                key_template: str = "model.layers.{layer}.mlp.experts.{expert}.{proj}.weight",
                                proj_name_map: Optional[Dict[str, str]] = None, **kw) -> GPTQLinearWeight:
        proj_map = proj_name_map or {"gate": "gate_proj", "up": "up_proj", "down": "down_proj"}
        if proj_name not in proj_map:
            raise KeyError(f"Unknown expert projection name: {proj_name}")
        key = key_template.format(layer=layer_idx, expert=expert_idx, proj=proj_map[proj_name])
        prefix = key[: -len(".weight")] if key.endswith(".weight") else key
        return self.load_gptq_linear(prefix, **kw)
