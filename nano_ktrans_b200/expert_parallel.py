"""Expert parallelism: the routed experts of a layer split across the ranks of
a process group, tokens exchanged with two all-to-alls.

No counterpart in nano-ktrans (its offload backends serve one device); the
arithmetic each token sees is the single-device path's: the same routing
(nano_ktrans/layers/hybrid_moe.py:3321-3329), the same expert MLP
(nano_ktrans/kernels/cpu_moe.py:419-450) and the same combine order, experts
ascending, fp32, one bf16 rounding (cpu_moe.py:515-538).

One step of a layer on rank r (``EpMoeLayer.forward``):

1. route r's tokens (``moe_route``);
2. ``moe_ep_dispatch``: sort the (token, slot) pairs by slot, i.e. by owning
   rank then local expert, and gather the token rows into that order;
3. all-to-all of the per-slot row counts, then of the rows (bf16);
4. ``moe_rows_forward``: every received row through its local expert (fp32);
5. all-to-all of the fp32 output rows back, in the order they came;
6. ``moe_ep_combine``: weighted sum per token into bf16.

With a ``PeerExchange`` (``moe_ep_peer_*``) the same step runs without a
collective and without a host read: every rank publishes its token rows and
their expert slots in its own device region; each owner's kernels read every
rank's rows through CUDA IPC mappings, run the pairs it owns and store each
fp32 output row straight into the token's rank's region; the token's rank
then combines from its region.  Ranks hand over with epoch flags in the
regions (bounded waits).

Expert placement (``plan_placement``) balances expected load: experts sorted
by routing frequency, each given to the least-loaded rank that still has a
free slot, so a Zipf-skewed router does not pile its popular experts on one
rank.  The device steps are the C-ABI calls of ``include/moe_b200.h``; the
exchanges go through ``torch.distributed`` (NCCL on GPUs).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib
from .moe_layer import MoeLayer, _stream_handle
from .weights import LayerWeights


# ---------------------------------------------------------------------------
# placement
# ---------------------------------------------------------------------------


def plan_placement(num_experts: int, world: int, freq: Optional[Sequence[float]] = None) -> np.ndarray:
    """slot_of_expert [E] int32: expert e lives on rank slot // (E/world) as local
    expert slot % (E/world).

    Greedy longest-processing-time assignment with equal expert counts per
    rank: experts in decreasing ``freq`` (ties: lower id first), each to the
    rank with the least assigned load among ranks with a free slot (ties:
    lower rank).  Local indices follow ascending global id within a rank.
    ``freq`` None means uniform, which gives round-robin ownership.
    """
    if world < 1 or num_experts % world:
        raise ValueError(f"num_experts ({num_experts}) must be a multiple of the world size ({world})")
    epr = num_experts // world
    f = np.ones(num_experts, dtype=np.float64) if freq is None else np.asarray(freq, dtype=np.float64)
    if f.shape != (num_experts,) or (f < 0).any() or not np.isfinite(f).all():
        raise ValueError("freq must be num_experts non-negative finite values")
    order = sorted(range(num_experts), key=lambda e: (-f[e], e))
    load = np.zeros(world, dtype=np.float64)
    owned: list[list[int]] = [[] for _ in range(world)]
    for e in order:
        cands = [r for r in range(world) if len(owned[r]) < epr]
        r = min(cands, key=lambda q: (load[q], q))
        owned[r].append(e)
        load[r] += f[e]
    slot = np.empty(num_experts, dtype=np.int32)
    for r in range(world):
        for local, e in enumerate(sorted(owned[r])):
            slot[e] = r * epr + local
    return slot


def experts_of_rank(slot_of_expert: np.ndarray, rank: int, world: int) -> np.ndarray:
    """Global ids of rank's experts, in local order."""
    epr = len(slot_of_expert) // world
    out = np.empty(epr, dtype=np.int64)
    for e, g in enumerate(np.asarray(slot_of_expert)):
        if g // epr == rank:
            out[g % epr] = e
    return out


def shard_layer(lw: LayerWeights, slot_of_expert: np.ndarray, rank: int, world: int) -> LayerWeights:
    """The experts of ``rank`` (local order) as their own stacked LayerWeights."""
    idx = torch.as_tensor(experts_of_rank(slot_of_expert, rank, world), device=lw.gate_q.device)
    sel = {k: getattr(lw, k).index_select(0, idx).contiguous()
           for k in ("gate_q", "gate_s", "up_q", "up_s", "down_q", "down_s")}
    return LayerWeights(bits=lw.bits, group_size=lw.group_size, shared=None, **sel)


# ---------------------------------------------------------------------------
# exchanges
# ---------------------------------------------------------------------------


class TorchDistComm:
    """all_to_all over a torch.distributed process group (NCCL for CUDA tensors)."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor, out_splits=None, in_splits=None) -> None:
        self.dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits,
                                    group=self.group)


@dataclass
class DispatchState:
    """Per-step bookkeeping between the phases of one rank."""
    ids: torch.Tensor
    weights: torch.Tensor
    send_rows: torch.Tensor
    slot_counts: torch.Tensor
    send_splits: list
    recv_splits: list = None
    recv_counts: np.ndarray = None
    recv_rows: torch.Tensor = None
    y_rows: torch.Tensor = None
    ret_rows: torch.Tensor = None


class _LayerHandle:
    """A handle for routing, dispatch and combine: layer shape only, no weights."""

    def __init__(self, num_experts, top_k, hidden, inter, bits, group, use_softmax, renorm, max_tokens, device):
        self.device = device
        desc = _lib.MoeLayerDesc(num_experts, top_k, hidden, inter, bits, group, int(use_softmax), int(renorm),
                                 max_tokens, 0)
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(1024)
        with torch.cuda.device(device):
            rc = _lib.lib().moe_create(ctypes.byref(desc), ctypes.byref(h), err, len(err))
        if rc != _lib.MOE_OK:
            raise _lib.MoeError(rc, err.value.decode())
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().moe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class LoopbackComm:
    """The exchange of a one-rank group: every all-to-all is a copy."""

    rank, world = 0, 1

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor, out_splits=None, in_splits=None) -> None:
        out.copy_(inp)


class PeerExchange:
    """One rank's side of a peer-memory exchange group (``moe_ep_group_*``).

    The rank's region (its published token rows and slots, and the fp32
    expert outputs the other ranks store for its tokens) is mapped into every
    other rank's process through CUDA IPC (``connect_ipc``), or, for ranks
    emulated in one process on one device, handed over directly
    (``connect_emulated``).  One group serves every expert-parallel layer of
    the rank that runs on the same stream: a step completes all of its
    exchanges before the next one publishes.  ``max_tokens`` bounds the tokens
    any rank publishes per step.
    """

    def __init__(self, rank: int, world: int, *, max_tokens: int, top_k: int, hidden: int, num_experts: int,
                 device=None):
        self.rank, self.world = int(rank), int(world)
        self.max_tokens, self.top_k, self.hidden = int(max_tokens), int(top_k), int(hidden)
        self.num_experts = int(num_experts)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        g = ctypes.c_void_p()
        err = ctypes.create_string_buffer(1024)
        with torch.cuda.device(self.device):
            rc = _lib.lib().moe_ep_group_create(self.rank, self.world, self.max_tokens, self.top_k, self.hidden,
                                                self.num_experts, ctypes.byref(g), err, len(err))
        if rc != _lib.MOE_OK:
            raise _lib.MoeError(rc, err.value.decode())
        self._g = g

    @property
    def handle(self):
        return self._g

    def ipc_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(_lib.EP_IPC_HANDLE_BYTES)
        _lib.check_group(_lib.lib().moe_ep_group_ipc_handle(self._g, buf), self._g, "moe_ep_group_ipc_handle")
        return buf.raw

    def region_ptr(self) -> int:
        p = ctypes.c_void_p()
        _lib.check_group(_lib.lib().moe_ep_group_region(self._g, ctypes.byref(p)), self._g, "moe_ep_group_region")
        return int(p.value)

    def connect_ipc(self, group=None) -> None:
        """Exchange IPC handles over a torch.distributed group and map every
        other rank's region (collective: every rank calls it)."""
        import torch.distributed as dist

        handles = [None] * self.world
        dist.all_gather_object(handles, self.ipc_handle(), group=group)
        with torch.cuda.device(self.device):
            for peer, h in enumerate(handles):
                if peer != self.rank:
                    _lib.check_group(_lib.lib().moe_ep_group_open_peer(self._g, peer, h), self._g,
                                     "moe_ep_group_open_peer")

    @staticmethod
    def connect_emulated(groups: Sequence["PeerExchange"]) -> None:
        """Ranks emulated in one process: every group sees every other's region."""
        ptrs = [g.region_ptr() for g in groups]
        for g in groups:
            for peer, p in enumerate(ptrs):
                if peer != g.rank:
                    _lib.check_group(_lib.lib().moe_ep_group_set_peer(g._g, peer, p), g._g, "moe_ep_group_set_peer")

    def read_status(self, stream=None) -> int:
        st = ctypes.c_int32(0)
        _lib.check_group(_lib.lib().moe_ep_group_read_status(self._g, ctypes.byref(st), _stream_handle(stream)),
                         self._g, "moe_ep_group_read_status")
        return int(st.value)

    def close(self, barrier=None) -> None:
        """Release the group.  ``barrier`` (e.g. torch.distributed.barrier) is
        called after this rank's work has drained and again after it unmapped
        the other regions, so no rank frees a region another still maps."""
        if getattr(self, "_g", None) is None:
            return
        torch.cuda.synchronize(self.device)
        if barrier is not None:
            barrier()
        _lib.lib().moe_ep_group_close_peers(self._g)
        if barrier is not None:
            barrier()
        _lib.lib().moe_ep_group_destroy(self._g)
        self._g = None


class EpStep:
    """The rank-side sequence of one expert-parallel step, independent of how
    the device steps are carried out (``EpMoeLayer`` binds them to the CUDA
    library).  Subclasses provide route / dispatch / expert_rows / combine."""

    num_experts: int
    top_k: int
    rank: int
    world: int
    epr: int
    hidden: int
    max_rows: int
    device: torch.device

    def exchange_counts(self, st: DispatchState, recv_counts: torch.Tensor) -> None:
        """recv_counts [world * epr] int32: rows each source sends to each of my local experts."""
        both = torch.cat([st.slot_counts, recv_counts]).cpu().numpy()  # one device->host read per step
        mine = both[: self.num_experts].reshape(self.world, self.epr)
        theirs = both[self.num_experts:].reshape(self.world, self.epr)
        st.send_splits = mine.sum(axis=1).tolist()
        st.recv_splits = theirs.sum(axis=1).tolist()
        st.recv_counts = theirs

    def forward(self, x: torch.Tensor, logits: torch.Tensor, comm=None, out: Optional[torch.Tensor] = None,
                tokens_per_rank: int = 0):
        """This rank's routed-expert output for its tokens x [T, H] bf16, with the
        ids and weights it routed them to.  Layers built with a peer exchange
        ignore ``comm`` and take ``tokens_per_rank`` (see ``peer_experts``)."""
        if getattr(self, "exchange", None) is not None:
            return self.forward_peer(x, logits, out, tokens_per_rank=tokens_per_rank)
        ids, w = self.route(logits)
        st = self.dispatch(x, ids, w)
        recv_counts = torch.empty_like(st.slot_counts)
        comm.all_to_all(recv_counts, st.slot_counts)
        self.exchange_counts(st, recv_counts)
        st.recv_rows = torch.empty(int(sum(st.recv_splits)), self.hidden, dtype=torch.bfloat16, device=self.device)
        comm.all_to_all(st.recv_rows, st.send_rows, st.recv_splits, st.send_splits)
        self.expert_rows(st)
        st.ret_rows = torch.empty(st.send_rows.shape[0], self.hidden, dtype=torch.float32, device=self.device)
        comm.all_to_all(st.ret_rows, st.y_rows, st.send_splits, st.recv_splits)
        return self.combine(st, out), ids, w


class EpMoeLayer(EpStep):
    """One MoE layer whose routed experts are split across ranks.

    ``local_weights`` holds this rank's ``num_experts / world`` experts in
    local order (``shard_layer``); ``slot_of_expert`` comes from
    ``plan_placement`` and must be identical on every rank.  ``max_tokens``
    bounds the tokens a rank routes per call; ``max_rows`` bounds the rows a
    rank receives (default: every rank's pairs, world * max_tokens * top_k).
    """

    def __init__(self, local_weights: LayerWeights, *, num_experts: int, top_k: int, slot_of_expert,
                 rank: int, world: int, router_use_softmax: bool = True, normalize_topk_prob: bool = True,
                 max_tokens: int = 4096, max_rows: Optional[int] = None,
                 exchange: Optional[PeerExchange] = None):
        if local_weights.shared is not None:
            raise ValueError("expert parallelism covers routed experts only (no shared expert)")
        self.num_experts, self.top_k = int(num_experts), int(top_k)
        self.rank, self.world = int(rank), int(world)
        if self.num_experts % self.world:
            raise ValueError("num_experts must be a multiple of the world size")
        self.epr = self.num_experts // self.world
        if local_weights.num_experts != self.epr:
            raise ValueError(f"local weights hold {local_weights.num_experts} experts, expected {self.epr}")
        self.device = local_weights.gate_q.device
        self.hidden = local_weights.hidden_size
        self.max_tokens = int(max_tokens)
        self.max_rows = int(max_rows) if max_rows else self.world * self.max_tokens * self.top_k
        slot = np.asarray(slot_of_expert, dtype=np.int32)
        if sorted(slot.tolist()) != list(range(self.num_experts)):
            raise ValueError("slot_of_expert must be a permutation of 0..num_experts-1")
        self.slot_of_expert = torch.as_tensor(slot, device=self.device)
        self.router = _LayerHandle(self.num_experts, self.top_k, self.hidden, local_weights.inter_size,
                                   local_weights.bits, local_weights.group_size, router_use_softmax,
                                   normalize_topk_prob, self.max_tokens, self.device)
        self.exchange = exchange
        if exchange is None:
            # rows through the local experts: top_k 1, one row per received pair
            self.experts = MoeLayer(local_weights, top_k=1, router_use_softmax=router_use_softmax,
                                    normalize_topk_prob=normalize_topk_prob, max_tokens=self.max_rows)
        else:
            if (exchange.rank, exchange.world, exchange.num_experts, exchange.top_k, exchange.hidden) != \
                    (self.rank, self.world, self.num_experts, self.top_k, self.hidden):
                raise ValueError("the peer exchange group was made for another rank, world or layer shape")
            if exchange.max_tokens < self.max_tokens:
                raise ValueError("the peer exchange group's max_tokens is below the layer's")
            if self.top_k > self.epr:
                raise ValueError("the peer exchange needs top_k <= experts per rank")
            # every rank's tokens through the local experts: pairs owned elsewhere are skipped
            self.experts = MoeLayer(local_weights, top_k=self.top_k, router_use_softmax=router_use_softmax,
                                    normalize_topk_prob=normalize_topk_prob,
                                    max_tokens=self.world * exchange.max_tokens)
        self._send_local = torch.empty(self.max_tokens * self.top_k, dtype=torch.int64, device=self.device)
        self._local_ids = torch.arange(self.epr, dtype=torch.int64, device=self.device).repeat(self.world)

    # -- argument checks: every tensor whose pointer reaches a kernel ----------
    def _check(self, t: torch.Tensor, name: str, shape, dtype) -> None:
        if (tuple(t.shape) != tuple(shape) or t.dtype is not dtype or not t.is_cuda
                or t.get_device() != self.slot_of_expert.get_device()):
            raise ValueError(f"{name} must be {dtype} {list(shape)} on {self.device}, got "
                             f"{t.dtype} {list(t.shape)} on {t.device}")

    # -- phases -------------------------------------------------------------
    def route(self, logits: torch.Tensor, stream=None):
        if logits.dim() != 2:
            raise ValueError("router logits must be [T, E]")
        t = int(logits.shape[0])
        self._check(logits, "router logits", (t, self.num_experts), torch.bfloat16)
        ids = torch.empty(t, self.top_k, dtype=torch.int64, device=self.device)
        w = torch.empty(t, self.top_k, dtype=torch.bfloat16, device=self.device)
        _lib.check(_lib.lib().moe_route(self.router._h, logits.contiguous().data_ptr(), t, ids.data_ptr(),
                                        w.data_ptr(), _stream_handle(stream)), self.router._h, "moe_route")
        return ids, w

    def dispatch(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, stream=None) -> DispatchState:
        if x.dim() != 2:
            raise ValueError("activations must be [T, H]")
        t = int(x.shape[0])
        if t > self.max_tokens:
            raise ValueError(f"{t} tokens above max_tokens {self.max_tokens}")
        self._check(x, "activations", (t, self.hidden), torch.bfloat16)
        self._check(ids, "topk_ids", (t, self.top_k), torch.int64)
        self._check(w, "topk_weights", (t, self.top_k), torch.bfloat16)
        ids, w = ids.contiguous(), w.contiguous()
        send_rows = torch.empty(t * self.top_k, self.hidden, dtype=torch.bfloat16, device=self.device)
        counts = torch.empty(self.num_experts, dtype=torch.int32, device=self.device)
        _lib.check(_lib.lib().moe_ep_dispatch(self.router._h, x.contiguous().data_ptr(), ids.data_ptr(), t,
                                              self.slot_of_expert.data_ptr(), self.epr, self.world,
                                              send_rows.data_ptr(), self._send_local.data_ptr(), counts.data_ptr(),
                                              _stream_handle(stream)), self.router._h, "moe_ep_dispatch")
        return DispatchState(ids=ids, weights=w, send_rows=send_rows, slot_counts=counts, send_splits=None)

    def expert_rows(self, st: DispatchState, stream=None) -> None:
        n = int(sum(st.recv_splits))
        if n > self.max_rows:
            raise RuntimeError(f"{n} rows received, above max_rows {self.max_rows}")
        st.y_rows = torch.empty(n, self.hidden, dtype=torch.float32, device=self.device)
        if n == 0:
            return
        # rows from each source arrive grouped by local expert, in local order
        row_expert = torch.repeat_interleave(self._local_ids,
                                             torch.as_tensor(st.recv_counts.reshape(-1), device=self.device),
                                             output_size=n)
        _lib.check(_lib.lib().moe_rows_forward(self.experts.handle, st.recv_rows.data_ptr(), row_expert.data_ptr(),
                                               n, st.y_rows.data_ptr(), _stream_handle(stream)),
                   self.experts.handle, "moe_rows_forward")

    def combine(self, st: DispatchState, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
        t = int(st.ids.shape[0])
        if out is not None:
            self._check(out, "out", (t, self.hidden), torch.bfloat16)
            if not out.is_contiguous():
                raise ValueError("out must be contiguous")
        out = out if out is not None else torch.empty(t, self.hidden, dtype=torch.bfloat16, device=self.device)
        if t:
            _lib.check(_lib.lib().moe_ep_combine(self.router._h, st.ids.data_ptr(), st.weights.data_ptr(), t,
                                                 st.ret_rows.data_ptr(), out.data_ptr(), _stream_handle(stream)),
                       self.router._h, "moe_ep_combine")
        return out

    # -- the peer-memory step (exchange given) ----------------------------------
    def peer_publish(self, x: torch.Tensor, ids: torch.Tensor, stream=None) -> None:
        """Phase 1: this rank's tokens and their expert slots into its region."""
        if self.exchange is None:
            raise RuntimeError("this layer was built without a peer exchange")
        t = int(x.shape[0]) if x.dim() == 2 else -1
        if t < 0:
            raise ValueError("activations must be [T, H]")
        if t > self.exchange.max_tokens:
            raise ValueError(f"{t} tokens above the exchange's max_tokens {self.exchange.max_tokens}")
        self._check(x, "activations", (t, self.hidden), torch.bfloat16)
        self._check(ids, "topk_ids", (t, self.top_k), torch.int64)
        g = self.exchange.handle
        _lib.check_group(_lib.lib().moe_ep_peer_publish(g, x.contiguous().data_ptr(), ids.contiguous().data_ptr(), t,
                                                        self.slot_of_expert.data_ptr(), _stream_handle(stream)),
                         g, "moe_ep_peer_publish")

    def peer_experts(self, pairs_hint: int, tokens_per_rank: int = 0, stream=None) -> None:
        """Phase 2: every rank's pairs owned here through the local experts, the
        outputs stored into their token's rank's region.  ``tokens_per_rank``
        (0: the exchange's max_tokens) bounds every rank's tokens in this step;
        ``pairs_hint`` only picks the kernels."""
        if self.exchange is None:
            raise RuntimeError("this layer was built without a peer exchange")
        g = self.exchange.handle
        _lib.check_group(_lib.lib().moe_ep_peer_experts(g, self.experts.handle, int(tokens_per_rank),
                                                        int(pairs_hint), _stream_handle(stream)),
                         g, "moe_ep_peer_experts")

    def peer_combine(self, ids: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
                     stream=None) -> torch.Tensor:
        """Phase 3: the weighted combine of this rank's tokens from its region."""
        if self.exchange is None:
            raise RuntimeError("this layer was built without a peer exchange")
        if ids.dim() != 2:
            raise ValueError("topk_ids must be [T, top_k]")
        t = int(ids.shape[0])
        self._check(ids, "topk_ids", (t, self.top_k), torch.int64)
        self._check(w, "topk_weights", (t, self.top_k), torch.bfloat16)
        if out is not None:
            self._check(out, "out", (t, self.hidden), torch.bfloat16)
            if not out.is_contiguous():
                raise ValueError("out must be contiguous")
        out = out if out is not None else torch.empty(t, self.hidden, dtype=torch.bfloat16, device=self.device)
        g = self.exchange.handle
        _lib.check_group(_lib.lib().moe_ep_peer_combine(g, ids.contiguous().data_ptr(), w.contiguous().data_ptr(), t,
                                                        out.data_ptr(), _stream_handle(stream)),
                         g, "moe_ep_peer_combine")
        return out

    def forward_peer(self, x: torch.Tensor, logits: torch.Tensor, out: Optional[torch.Tensor] = None, stream=None,
                     tokens_per_rank: int = 0):
        """One step over the peer exchange: no host synchronisation, no
        collective.  ``tokens_per_rank`` as in ``peer_experts``."""
        ids, w = self.route(logits, stream)
        self.peer_publish(x, ids, stream)
        self.peer_experts(int(x.shape[0]) * self.top_k, tokens_per_rank, stream)
        return self.peer_combine(ids, w, out, stream), ids, w

    def set_gemm(self, mode: int) -> None:
        """Kernel selection of the local expert rows (see MoeLayer.set_gemm)."""
        self.experts.set_gemm(mode)

    def read_status(self) -> int:
        st = ctypes.c_int32(0)
        _lib.check(_lib.lib().moe_read_status(self.router._h, ctypes.byref(st), _stream_handle(None)),
                   self.router._h, "moe_read_status")
        return int(st.value) | self.experts.read_status()

    def close(self):
        self.router.close()
        self.experts.close()
