"""Expert parallelism over peer memory (moe_ep_group_*, moe_ep_peer_*): the
exchanges done by the library's kernels through every rank's region, with
epoch flags instead of host reads and collectives.

On one GPU the ranks are emulated in one process (every group sees the
others' regions directly) and run phase by phase on one stream: every rank's
publish, then every rank's experts, then every rank's combine, so each wait
finds its flags already set.  With two or more GPUs the same layers run as
one process per GPU with the regions mapped through CUDA IPC.  Each rank's
output must be bit-identical to the single-GPU moe_experts_forward of the same
tokens with the same kernel selection, over several consecutive steps (the
epochs advance and the buffers are reused)."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from tests import helpers as hp
from tests.test_ep_gpu import MAX_ABS, MEAN_REL, _free_port, _random_layer, _single_gpu

pytestmark = pytest.mark.gpu


def _peer_setup(lw, world, slot, k, max_tokens, use_softmax=True, renorm=True):
    from nano_ktrans_b200.expert_parallel import EpMoeLayer, PeerExchange, shard_layer

    E, H = lw.num_experts, lw.hidden_size
    groups = [PeerExchange(r, world, max_tokens=max_tokens, top_k=k, hidden=H, num_experts=E) for r in range(world)]
    PeerExchange.connect_emulated(groups)
    layers = [EpMoeLayer(shard_layer(lw, slot, r, world), num_experts=E, top_k=k, slot_of_expert=slot, rank=r,
                         world=world, router_use_softmax=use_softmax, normalize_topk_prob=renorm,
                         max_tokens=max_tokens, exchange=groups[r]) for r in range(world)]
    return groups, layers


def _peer_step(layers, xs, lgs):
    routed = []
    for L, x, lg in zip(layers, xs, lgs):
        ids, w = L.route(lg)
        L.peer_publish(x, ids)
        routed.append((ids, w))
    bound = max(x.shape[0] for x in xs)
    for L, x in zip(layers, xs):
        L.peer_experts(x.shape[0] * L.top_k, bound)
    return [(L.peer_combine(ids, w), ids, w) for L, (ids, w) in zip(layers, routed)]


def _close(groups, layers):
    for L in layers:
        L.close()
    for g in groups:
        g.close()


def _inputs(E, H, tokens, dev, seed):
    gen = torch.Generator(device=dev).manual_seed(seed)
    wr = (torch.randn(E, H, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    bias = torch.log(torch.arange(1, E + 1, device=dev, dtype=torch.float32) ** -1.2)[
        torch.randperm(E, device=dev, generator=gen)]
    xs, lgs = [], []
    for t in tokens:
        x = torch.randn(t, H, device=dev, generator=gen).to(torch.bfloat16)
        xs.append(x)
        lgs.append(((x @ wr.T).float() + bias).to(torch.bfloat16))
    return xs, lgs


@pytest.mark.parametrize("mode", [0, 2], ids=["stream", "gemm"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_emulated_ranks_bit_identical_to_single_gpu(world, mode, cuda_device):
    """Qwen3-shaped layer (128 experts, top-8, W4 g128), Zipf-skewed routing,
    uneven token counts (one rank without tokens at 4 and 8 ranks), three
    consecutive steps with fresh tokens."""
    from nano_ktrans_b200.expert_parallel import plan_placement

    E, k, H, I = 128, 8, 2048, 768
    lw = _random_layer(E, H, I, 4, 128, cuda_device, 7)
    tokens = [40 + 13 * r for r in range(world)]
    tokens[-1] = 0 if world > 2 else tokens[-1]
    groups, layers = _peer_setup(lw, world, plan_placement(E, world), k, max(tokens))
    for L in layers:
        L.set_gemm(mode)
    for step in range(3):
        xs, lgs = _inputs(E, H, tokens, cuda_device, 3 + step)
        res = _peer_step(layers, xs, lgs)
        torch.cuda.synchronize()
        for r, (out, ids, w) in enumerate(res):
            assert out.shape == (tokens[r], H)
            if tokens[r] == 0:
                continue
            ref = _single_gpu(lw, k, xs[r], ids, w, mode)
            torch.cuda.synchronize()
            assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"step {step} rank {r} differs"
    assert all(g.read_status() == 0 for g in groups)
    assert all(L.read_status() == 0 for L in layers)
    _close(groups, layers)


def test_peer_emulated_matches_oracle(cuda_device):
    """Small layer with oracle-quantized experts (16 experts, top-4, 4 ranks):
    within the parity bar of the reference's CPU path, through forward()."""
    from nano_ktrans_b200.expert_parallel import plan_placement

    E, k, H, I, world = 16, 4, 256, 256, 4
    experts = {e: hp.make_expert(12, e, H, I, 4, 128) for e in range(E)}
    lw = hp.device_layer(experts, E, H, I, 4, 128, cuda_device)
    tokens = [9, 0, 17, 5]
    ins = [hp.make_inputs(60 + r, t, H, E) for r, t in enumerate(tokens)]
    groups, layers = _peer_setup(lw, world, plan_placement(E, world), k, max(tokens))
    res = _peer_step(layers, [hp.bf16_tensor(x, cuda_device) for x, _ in ins],
                     [hp.bf16_tensor(lg, cuda_device) for _, lg in ins])
    torch.cuda.synchronize()
    for r, (out, ids, w) in enumerate(res):
        if tokens[r] == 0:
            assert out.shape[0] == 0
            continue
        ref = mo.offload_forward_f32(ins[r][0], ids.cpu().numpy(), hp.bf16_bits(w), experts)
        hp.assert_parity(hp.bf16_bits(out), ref, MAX_ABS, MEAN_REL)
    assert all(g.read_status() == 0 for g in groups)
    _close(groups, layers)


def test_peer_one_rank_is_the_single_gpu_path(cuda_device):
    """world 1: publish, experts and combine on the rank's own region equal
    MoeLayer.experts_forward bit for bit (decode-sized and prefill-sized)."""
    from nano_ktrans_b200.expert_parallel import plan_placement

    E, k, H, I = 128, 8, 2048, 768
    lw = _random_layer(E, H, I, 4, 128, cuda_device, 11)
    groups, layers = _peer_setup(lw, 1, plan_placement(E, 1), k, 256)
    for t in (5, 256):
        xs, lgs = _inputs(E, H, [t], cuda_device, 20 + t)
        out, ids, w = layers[0].forward(xs[0], lgs[0])
        ref = _single_gpu(lw, k, xs[0], ids, w, 1)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), t
    assert groups[0].read_status() == 0
    _close(groups, layers)


def test_peer_wait_runs_out_and_reports(cuda_device):
    """A rank that never publishes: the other rank's expert step waits its
    bounded time (5 s), records MOE_EP_STATUS_TIMEOUT and selects no pairs;
    the combine then returns at once with zeros; reading the status clears it
    and the group works again once both ranks step together."""
    from nano_ktrans_b200 import _lib
    from nano_ktrans_b200.expert_parallel import plan_placement

    E, k, H, I, world = 16, 4, 256, 256, 2
    lw = _random_layer(E, H, I, 4, 128, cuda_device, 5)
    groups, layers = _peer_setup(lw, world, plan_placement(E, world), k, 8)
    xs, lgs = _inputs(E, H, [8, 8], cuda_device, 9)
    ids, w = layers[0].route(lgs[0])
    layers[0].peer_publish(xs[0], ids)
    layers[0].peer_experts(8 * k, 8)
    out = layers[0].peer_combine(ids, w)
    torch.cuda.synchronize()
    assert groups[0].read_status() & _lib.EP_STATUS_TIMEOUT
    assert int(out.view(torch.int16).abs().sum()) == 0
    # rank 1 catches up on its step; then both ranks step together again
    ids1, w1 = layers[1].route(lgs[1])
    layers[1].peer_publish(xs[1], ids1)
    layers[1].peer_experts(8 * k, 8)
    layers[1].peer_combine(ids1, w1)
    torch.cuda.synchronize()
    assert groups[1].read_status() == 0
    res = _peer_step(layers, xs, lgs)
    torch.cuda.synchronize()
    for r, (o, i, ww) in enumerate(res):
        ref = _single_gpu(lw, k, xs[r], i, ww, 1)
        torch.cuda.synchronize()
        assert torch.equal(o.view(torch.int16), ref.view(torch.int16)), r
    assert all(g.read_status() == 0 for g in groups)
    _close(groups, layers)


def test_peer_step_refuses_out_of_order_calls(cuda_device):
    from nano_ktrans_b200 import _lib
    from nano_ktrans_b200.expert_parallel import plan_placement

    E, k, H, I = 16, 4, 256, 256
    lw = _random_layer(E, H, I, 4, 128, cuda_device, 5)
    groups, layers = _peer_setup(lw, 1, plan_placement(E, 1), k, 8)
    xs, lgs = _inputs(E, H, [8], cuda_device, 9)
    ids, w = layers[0].route(lgs[0])
    with pytest.raises(_lib.MoeError):
        layers[0].peer_experts(8)  # before publish
    with pytest.raises(_lib.MoeError):
        layers[0].peer_combine(ids, w)
    layers[0].peer_publish(xs[0], ids)
    with pytest.raises(_lib.MoeError):
        layers[0].peer_publish(xs[0], ids)  # twice
    layers[0].peer_experts(8 * k)
    layers[0].peer_combine(ids, w)
    torch.cuda.synchronize()
    assert groups[0].read_status() == 0
    _close(groups, layers)


def test_peer_step_bound_below_a_rank_is_reported(cuda_device):
    """tokens_per_rank below another rank's token count: that rank's extra
    tokens are not served and MOE_EP_STATUS_OVERFLOW is set; a bound below the
    caller's own count is refused on the host."""
    from nano_ktrans_b200 import _lib
    from nano_ktrans_b200.expert_parallel import plan_placement

    E, k, H, I, world = 16, 4, 256, 256, 2
    lw = _random_layer(E, H, I, 4, 128, cuda_device, 5)
    groups, layers = _peer_setup(lw, world, plan_placement(E, world), k, 16)
    xs, lgs = _inputs(E, H, [4, 12], cuda_device, 9)
    routed = []
    for L, x, lg in zip(layers, xs, lgs):
        ids, w = L.route(lg)
        L.peer_publish(x, ids)
        routed.append((ids, w))
    with pytest.raises(_lib.MoeError):
        layers[1].peer_experts(12 * k, 4)  # below rank 1's own 12 tokens
    layers[0].peer_experts(4 * k, 4)
    layers[1].peer_experts(12 * k, 12)
    for L, (ids, w) in zip(layers, routed):
        L.peer_combine(ids, w)
    torch.cuda.synchronize()
    assert groups[0].read_status() & _lib.EP_STATUS_OVERFLOW
    assert groups[1].read_status() == 0
    _close(groups, layers)


def _ipc_rank(rank, world, port, path):
    import datetime

    import torch.distributed as dist

    from nano_ktrans_b200.expert_parallel import EpMoeLayer, PeerExchange, plan_placement, shard_layer

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        E, k, H, I = 128, 8, 2048, 768
        lw = _random_layer(E, H, I, 4, 128, dev, 7)  # same seed: identical weights on every rank
        slot = plan_placement(E, world)
        ex = PeerExchange(rank, world, max_tokens=96, top_k=k, hidden=H, num_experts=E, device=dev)
        ex.connect_ipc()
        ep = EpMoeLayer(shard_layer(lw, slot, rank, world), num_experts=E, top_k=k, slot_of_expert=slot, rank=rank,
                        world=world, max_tokens=96, exchange=ex)
        ep.set_gemm(2)
        gen = torch.Generator(device=dev).manual_seed(100 + rank)
        results = []
        for step in range(3):
            t = 96 - 31 * rank - 7 * step
            x = torch.randn(t, H, device=dev, generator=gen).to(torch.bfloat16)
            lg = torch.randn(t, E, device=dev, generator=gen).to(torch.bfloat16)
            out, ids, w = ep.forward(x, lg)
            ref = _single_gpu(lw, k, x, ids, w, 2)
            torch.cuda.synchronize()
            results.append(bool(torch.equal(out.view(torch.int16), ref.view(torch.int16))))
        ok = ex.read_status() == 0 and ep.read_status() == 0
        np.save(path, np.array([all(results), ok]))
        ep.close()
        ex.close(barrier=dist.barrier)
    finally:
        dist.destroy_process_group()


def test_peer_ipc_ranks_bit_identical_to_single_gpu(tmp_path):
    """Two (or more) GPUs, one process each, regions mapped through CUDA IPC."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = min(n, 4)
    port = _free_port()
    ctx = mp.get_context("spawn")
    paths = [str(tmp_path / f"r{r}.npy") for r in range(world)]
    procs = [ctx.Process(target=_ipc_rank, args=(r, world, port, paths[r])) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        same, ok = np.load(paths[r])
        assert ok and same, f"rank {r}: equal={same} status_ok={ok}"
