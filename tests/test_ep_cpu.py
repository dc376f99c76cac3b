"""Expert parallelism on CPU: placement and the rank-side step sequence.

Two ``gloo`` ranks run ``EpStep.forward`` (the same sequence the GPU path
runs over NCCL) with the device steps replaced by the oracle's arithmetic
(``tests/ep_numpy.py``).  Each rank's output must equal the single-device
oracle on that rank's tokens: nothing may be lost, duplicated, reordered or
combined in another order by the exchanges.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

from nano_ktrans_b200.expert_parallel import LoopbackComm, experts_of_rank, plan_placement
from oracle import moe_oracle as mo
from tests import helpers as hp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ---------------------------------------------------------------------------
# placement
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_placement_is_balanced_permutation(world):
    E = 128
    z = np.arange(1, E + 1, dtype=np.float64) ** -1.2
    freq = np.random.Generator(np.random.PCG64(3)).permutation(z)
    slot = plan_placement(E, world, freq)
    assert sorted(slot.tolist()) == list(range(E))
    epr = E // world
    loads = [freq[experts_of_rank(slot, r, world)].sum() for r in range(world)]
    # contiguous sharding for comparison: ranks own experts [r*epr, (r+1)*epr)
    contiguous = [freq[r * epr:(r + 1) * epr].sum() for r in range(world)]
    assert max(loads) <= max(contiguous) + 1e-12
    # no rank above 1.15x the larger of the mean load and the heaviest single expert
    assert max(loads) <= 1.15 * max(sum(loads) / world, freq.max())
    for r in range(world):
        own = experts_of_rank(slot, r, world)
        assert list(own) == sorted(own)  # local order = ascending global id
        assert all(slot[e] // epr == r for e in own)


def test_placement_rejects_bad_inputs():
    with pytest.raises(ValueError):
        plan_placement(60, 8)
    with pytest.raises(ValueError):
        plan_placement(8, 2, [1.0] * 7)
    with pytest.raises(ValueError):
        plan_placement(8, 2, [1.0] * 7 + [-1.0])


# ---------------------------------------------------------------------------
# the step sequence, one rank (loopback) and two gloo ranks
# ---------------------------------------------------------------------------

CFG = dict(E=8, k=2, H=64, I=64, bits=4, group=32)


def _experts(seed=5):
    return {e: hp.make_expert(seed, e, CFG["H"], CFG["I"], CFG["bits"], CFG["group"]) for e in range(CFG["E"])}


def _rank_inputs(rank, tokens):
    return hp.make_inputs(40 + rank, tokens, CFG["H"], CFG["E"], zipf=1.2)


def _run_rank(rank, world, port, tokens_per_rank, result_path):
    import torch.distributed as dist

    from nano_ktrans_b200.expert_parallel import TorchDistComm
    from tests.ep_numpy import NumpyEpStep, bf16_from_bits, bits_of, per_row_reference

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        experts = _experts()
        freq = np.bincount(np.concatenate([mo.route(_rank_inputs(r, tokens_per_rank[r])[1], CFG["k"], True, True)[0]
                                           .reshape(-1) for r in range(world)]), minlength=CFG["E"])
        slot = plan_placement(CFG["E"], world, freq)
        step = NumpyEpStep(experts, num_experts=CFG["E"], top_k=CFG["k"], slot_of_expert=slot, rank=rank,
                           world=world, hidden=CFG["H"])
        x, logits = _rank_inputs(rank, tokens_per_rank[rank])
        out, ids, w = step.forward(bf16_from_bits(x), bf16_from_bits(logits), TorchDistComm())
        ref = per_row_reference(x, ids.numpy(), bits_of(w), experts)
        np.save(result_path, np.stack([bits_of(out), ref]) if x.shape[0] else np.zeros((2, 0, CFG["H"]), np.uint16))
    finally:
        dist.destroy_process_group()


def _spawn(world, tokens_per_rank, tmp_path):
    import torch.multiprocessing as mp

    port = _free_port()
    paths = [str(tmp_path / f"rank{r}.npy") for r in range(world)]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_run_rank, args=(r, world, port, tokens_per_rank, paths[r])) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return [np.load(p) for p in paths]


def test_ep_step_loopback_matches_single_device():
    from tests.ep_numpy import NumpyEpStep, bf16_from_bits, bits_of, per_row_reference

    experts = _experts()
    x, logits = _rank_inputs(0, 9)
    step = NumpyEpStep(experts, num_experts=CFG["E"], top_k=CFG["k"], slot_of_expert=plan_placement(CFG["E"], 1),
                       rank=0, world=1, hidden=CFG["H"])
    out, ids, w = step.forward(bf16_from_bits(x), bf16_from_bits(logits), LoopbackComm())
    ref = per_row_reference(x, ids.numpy(), bits_of(w), experts)
    assert np.array_equal(bits_of(out), ref)
    # the per-row reference is the oracle's combine up to BLAS batching
    hp.assert_paths_agree(ref, mo.offload_forward(x, ids.numpy(), bits_of(w), experts), 1e-4, 5e-3)


@pytest.mark.parametrize("tokens", [(7, 5), (12, 0)], ids=["uneven", "one_rank_empty"])
def test_ep_two_gloo_ranks_match_single_device(tokens, tmp_path):
    res = _spawn(2, list(tokens), tmp_path)
    for r, arr in enumerate(res):
        got, ref = arr[0], arr[1]
        assert got.shape == (tokens[r], CFG["H"])
        assert np.array_equal(got, ref), f"rank {r}: EP output differs from the single-device oracle"


# ---------------------------------------------------------------------------
# peer-memory exchange: the host protocol (handle exchange and teardown order)
# ---------------------------------------------------------------------------


class _FakePeerLib:
    """Stands in for libmoe_b200's group calls: records what PeerExchange asks
    of the library; the device side is covered by tests/test_ep_peer_gpu.py."""

    def __init__(self, rank, slow_close=0.0):
        self.rank, self.slow_close = rank, slow_close
        self.opened, self.peers_set, self.events = {}, {}, []

    def moe_ep_group_create(self, rank, world, max_tokens, top_k, hidden, num_experts, gptr, err, n):
        gptr._obj.value = 0x1000 * (rank + 1)
        return 0

    def moe_ep_group_ipc_handle(self, g, buf):
        ctypes.memmove(buf, bytes([65 + self.rank]) * 64, 64)
        return 0

    def moe_ep_group_open_peer(self, g, peer, handle):
        self.opened[int(peer)] = bytes(handle)
        return 0

    def moe_ep_group_region(self, g, pptr):
        pptr._obj.value = 0x100000 * (self.rank + 1)
        return 0

    def moe_ep_group_set_peer(self, g, peer, region):
        self.peers_set[int(peer)] = int(region)
        return 0

    def moe_ep_group_close_peers(self, g):
        import time

        time.sleep(self.slow_close)
        self.events.append(("close", time.time()))
        return 0

    def moe_ep_group_destroy(self, g):
        import time

        self.events.append(("destroy", time.time()))
        return 0

    def moe_ep_group_last_error(self, g, buf, n):
        return 0


def _patch_for_fake(monkeypatch_like, fake):
    import contextlib

    from nano_ktrans_b200 import _lib

    monkeypatch_like(_lib, "lib", lambda: fake)
    monkeypatch_like(torch.cuda, "device", lambda d: contextlib.nullcontext())
    monkeypatch_like(torch.cuda, "synchronize", lambda *a, **k: None)


def _peer_protocol_rank(rank, world, port, path):
    import json

    import torch.distributed as dist

    from nano_ktrans_b200.expert_parallel import PeerExchange

    fake = _FakePeerLib(rank, slow_close=0.5 if rank == 0 else 0.0)
    _patch_for_fake(setattr, fake)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        ex = PeerExchange(rank, world, max_tokens=8, top_k=2, hidden=64, num_experts=4 * world, device="cpu")
        ex.connect_ipc()
        ex.close(barrier=dist.barrier)
        with open(path, "w") as f:
            json.dump({"opened": {str(k): v.hex() for k, v in fake.opened.items()}, "events": fake.events}, f)
    finally:
        dist.destroy_process_group()


def test_peer_exchange_handles_and_teardown_order_on_gloo_ranks(tmp_path):
    """Three gloo ranks: every rank maps exactly the other ranks' regions with
    their own IPC handles, and no rank frees its region before every rank has
    unmapped the others (rank 0 is slow to unmap)."""
    import json

    import torch.multiprocessing as mp

    world, port = 3, _free_port()
    paths = [str(tmp_path / f"peer{r}.json") for r in range(world)]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_peer_protocol_rank, args=(r, world, port, paths[r])) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [json.load(open(p)) for p in paths]
    for r, got in enumerate(res):
        assert got["opened"] == {str(s): (bytes([65 + s]) * 64).hex() for s in range(world) if s != r}
        assert [e[0] for e in got["events"]] == ["close", "destroy"]
    last_close = max(e[1] for got in res for e in got["events"] if e[0] == "close")
    first_destroy = min(e[1] for got in res for e in got["events"] if e[0] == "destroy")
    assert last_close <= first_destroy


def test_peer_exchange_emulated_ranks_see_each_other(monkeypatch):
    from nano_ktrans_b200.expert_parallel import PeerExchange

    fakes = [_FakePeerLib(r) for r in range(3)]
    exs = []
    for r, fake in enumerate(fakes):
        _patch_for_fake(monkeypatch.setattr, fake)
        exs.append(PeerExchange(r, 3, max_tokens=8, top_k=2, hidden=64, num_experts=12, device="cpu"))
    # one library serves all emulated ranks in a real process; here each group keeps its own recorder
    calls = {}

    class _Router:
        def __getattr__(self, name):
            return getattr(fakes[0], name)

        def moe_ep_group_region(self, g, pptr):
            pptr._obj.value = 0x100000 * (g.value // 0x1000)
            return 0

        def moe_ep_group_set_peer(self, g, peer, region):
            calls.setdefault(g.value // 0x1000 - 1, {})[int(peer)] = int(region)
            return 0

    _patch_for_fake(monkeypatch.setattr, _Router())
    PeerExchange.connect_emulated(exs)
    for r in range(3):
        assert calls[r] == {s: 0x100000 * (s + 1) for s in range(3) if s != r}
