"""A CPU stand-in for the device steps of an expert-parallel step (TEST
INFRASTRUCTURE ONLY).

``NumpyEpStep`` implements route / dispatch / expert_rows / combine with the
oracle's arithmetic on CPU tensors, so the rank-side sequence that
``nano_ktrans_b200.expert_parallel.EpStep.forward`` runs (placement, split
sizes, both all-to-alls, row order, combine order) can be exercised with
``gloo`` ranks on a machine without a GPU.  The CUDA steps are checked
against the same oracle in the GPU tests.
"""
from __future__ import annotations

import numpy as np
import torch

from nano_ktrans_b200.expert_parallel import DispatchState, EpStep, experts_of_rank
from oracle import moe_oracle as mo


def bf16_from_bits(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


class NumpyEpStep(EpStep):
    def __init__(self, experts: dict, *, num_experts, top_k, slot_of_expert, rank, world, hidden,
                 use_softmax=True, renorm=True):
        self.num_experts, self.top_k, self.rank, self.world = num_experts, top_k, rank, world
        self.epr = num_experts // world
        self.hidden = hidden
        self.max_rows = 1 << 30
        self.device = torch.device("cpu")
        self.slot = np.asarray(slot_of_expert)
        self.use_softmax, self.renorm = use_softmax, renorm
        # this rank's experts in local order: (gate, up, down) QuantLinear
        self.local = [experts.get(int(e)) for e in experts_of_rank(self.slot, rank, world)]

    def route(self, logits: torch.Tensor):
        ids, w, _ = mo.route(bits_of(logits), self.top_k, self.use_softmax, self.renorm)
        return torch.from_numpy(ids.astype(np.int64)), bf16_from_bits(w)

    def dispatch(self, x, ids, w) -> DispatchState:
        g = self.slot[ids.numpy()].reshape(-1)
        order = np.argsort(g, kind="stable")  # by slot, pair index ascending within a slot
        self._pos = np.empty_like(order)
        self._pos[order] = np.arange(order.size)
        xb = bits_of(x)
        send = bf16_from_bits(xb[order // self.top_k]) if order.size else torch.empty(0, self.hidden,
                                                                                          dtype=torch.bfloat16)
        counts = torch.from_numpy(np.bincount(g, minlength=self.num_experts).astype(np.int32))
        return DispatchState(ids=ids, weights=w, send_rows=send, slot_counts=counts, send_splits=None)

    def expert_rows(self, st: DispatchState) -> None:
        rows = mo.bf16_bits_to_f32(bits_of(st.recv_rows)) if st.recv_rows.numel() else np.zeros((0, self.hidden))
        local = np.repeat(np.tile(np.arange(self.epr), self.world), st.recv_counts.reshape(-1))
        y = np.zeros((rows.shape[0], self.hidden), dtype=np.float32)
        for i in range(rows.shape[0]):  # one row at a time: results independent of how rows are batched
            y[i] = mo.expert_forward(rows[i:i + 1], *self.local[local[i]])[0]
        st.y_rows = torch.from_numpy(y)

    def combine(self, st: DispatchState, out=None):
        t = st.ids.shape[0]
        ids = st.ids.numpy()
        w = mo.bf16_bits_to_f32(bits_of(st.weights))
        ret = st.ret_rows.numpy()
        acc = np.zeros((t, self.hidden), dtype=np.float32)
        for i in range(t):
            for j in sorted(range(self.top_k), key=lambda j: ids[i, j]):  # experts ascending
                acc[i] += ret[self._pos[i * self.top_k + j]] * w[i, j]
        return bf16_from_bits(mo.f32_to_bf16_bits(acc))


def per_row_reference(x_bits: np.ndarray, ids: np.ndarray, w_bits: np.ndarray, experts: dict) -> np.ndarray:
    """The single-device combine (experts ascending, fp32, one bf16 rounding)
    with every (token, expert) output computed one row at a time."""
    x = mo.bf16_bits_to_f32(x_bits)
    w = mo.bf16_bits_to_f32(w_bits)
    t, k = ids.shape
    acc = np.zeros((t, x.shape[1]), dtype=np.float32)
    for i in range(t):
        for j in sorted(range(k), key=lambda j: ids[i, j]):
            acc[i] += mo.expert_forward(x[i:i + 1], *experts[int(ids[i, j])])[0] * w[i, j]
    return mo.f32_to_bf16_bits(acc)
