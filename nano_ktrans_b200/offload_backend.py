"""Expert-backend plugin interface.

``ExpertOffloadBackend`` keeps the reference ABC's methods and counters
(nano_ktrans/kernels/offload_backend.py:29-90); ``normalize_offload_backend_name``
keeps its aliases (:11-22) and adds ``"cuda"``, the backend this package
provides.
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Any

import torch


def normalize_offload_backend_name(name: str | None) -> str:
    if not name:
        return "cpu"
    normalized = name.lower().replace("-", "_")
    aliases = {
        "cpu": "cpu",
        "pim": "pim",
        "pim_shadow": "pim_shadow",
        "cuda": "cuda",
        "b200": "cuda",
    }
    if normalized not in aliases:
        raise ValueError(f"Unsupported offload backend: {name}")
    return aliases[normalized]


class ExpertOffloadBackend(ABC):
    backend_name = "unknown"

    def __init__(self) -> None:
        self.submit_calls = 0
        self.sync_calls = 0
        self.migration_submit_calls = 0
        self.last_migration_plan_size = 0
        self.last_migration_phase = ""

    @abstractmethod
    def submit_forward(self, hidden_states: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                       cuda_stream: int | None) -> None:
        raise NotImplementedError

    @abstractmethod
    def sync_forward(self, hidden_states: torch.Tensor, cuda_stream: int | None) -> torch.Tensor:
        raise NotImplementedError

    def update_gpu_expert_mask(self, gpu_experts_mask: torch.Tensor) -> None:
        raise NotImplementedError

    def export_expert_weights(self, expert_idx: int) -> dict[str, torch.Tensor] | None:
        return None

    def notify_expert_evicted(self, expert_idx: int, residency_before: str) -> None:
        pass

    def queue_migration_plan(self, ops: list[Any], *, phase: str = "") -> None:
        self.migration_submit_calls += 1
        self.last_migration_plan_size = len(ops)
        self.last_migration_phase = phase

    def diagnostics(self) -> dict[str, Any]:
        return {
            "backend_name": self.backend_name,
            "submit_calls": self.submit_calls,
            "sync_calls": self.sync_calls,
            "migration_submit_calls": self.migration_submit_calls,
            "last_migration_plan_size": self.last_migration_plan_size,
            "last_migration_phase": self.last_migration_phase,
        }
