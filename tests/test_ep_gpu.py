"""Expert parallelism on B200: the CUDA device steps (moe_ep_dispatch,
moe_rows_forward, moe_ep_combine) through the C ABI.

On one GPU the ranks are emulated phase by phase (every rank's dispatch, then
the exchanges as tensor copies, then every rank's expert rows, ...); with two
or more GPUs the same layers run as NCCL ranks.  Each rank's output must be
bit-identical to the single-GPU moe_experts_forward of the same tokens with
the same kernel selection (per-row expert arithmetic does not depend on how
rows are batched or which rank computes them), and within the parity bar of
the oracle.
"""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from tests import helpers as hp

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 5e-3


def _random_layer(E, H, I, bits, group, dev, seed):
    from nano_ktrans_b200.weights import LayerWeights, scale_stride

    g = torch.Generator(device=dev).manual_seed(seed)

    def proj(n, k):
        q = torch.randint(0, 256, (E, n, k * bits // 8), dtype=torch.uint8, device=dev, generator=g)
        G = k // (group if group else k)
        s = torch.zeros(E, n, scale_stride(G), dtype=torch.bfloat16, device=dev)
        s[:, :, :G] = (torch.rand(E, n, G, device=dev, generator=g) * 2e-3 + 1e-3).to(torch.bfloat16)
        return q, s

    gq, gs = proj(I, H)
    uq, us = proj(I, H)
    dq, ds = proj(H, I)
    return LayerWeights(bits=bits, group_size=group, gate_q=gq, gate_s=gs, up_q=uq, up_s=us, down_q=dq, down_s=ds)


def _emulate(layers, xs, logits):
    """All ranks of one step on one GPU; exchanges as tensor copies."""
    W, epr = len(layers), layers[0].epr
    sts = []
    for L, x, lg in zip(layers, xs, logits):
        ids, w = L.route(lg)
        sts.append(L.dispatch(x, ids, w))
    for r, L in enumerate(layers):
        L.exchange_counts(sts[r], torch.cat([sts[s].slot_counts[r * epr:(r + 1) * epr] for s in range(W)]))
    for r in range(W):
        segs = []
        for s in range(W):
            off = sum(sts[s].send_splits[:r])
            segs.append(sts[s].send_rows[off:off + sts[s].send_splits[r]])
        sts[r].recv_rows = torch.cat(segs)
    for r, L in enumerate(layers):
        L.expert_rows(sts[r])
    for s in range(W):
        segs = []
        for r in range(W):
            off = sum(sts[r].recv_splits[:s])
            segs.append(sts[r].y_rows[off:off + sts[r].recv_splits[s]])
        sts[s].ret_rows = torch.cat(segs)
    return [(L.combine(st), st.ids, st.weights) for L, st in zip(layers, sts)]


def _ep_layers(lw, world, slot, top_k, max_tokens, use_softmax=True, renorm=True):
    from nano_ktrans_b200.expert_parallel import EpMoeLayer, shard_layer

    return [EpMoeLayer(shard_layer(lw, slot, r, world), num_experts=lw.num_experts, top_k=top_k, slot_of_expert=slot,
                       rank=r, world=world, router_use_softmax=use_softmax, normalize_topk_prob=renorm,
                       max_tokens=max_tokens) for r in range(world)]


def _single_gpu(lw, top_k, x, ids, w, mode, use_softmax=True, renorm=True):
    from nano_ktrans_b200.moe_layer import MoeLayer

    layer = MoeLayer(lw, top_k=top_k, router_use_softmax=use_softmax, normalize_topk_prob=renorm,
                     max_tokens=x.shape[0])
    layer.set_decode_fused(False)
    layer.set_gemm(mode)
    return layer.experts_forward(x, ids, w)


@pytest.mark.parametrize("mode", [0, 2], ids=["matvec", "gemm"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_emulated_ranks_bit_identical_to_single_gpu(world, mode, cuda_device):
    """Qwen3-shaped layer (128 experts, top-8, W4 g128), Zipf-skewed routing,
    frequency-balanced placement, uneven token counts per rank."""
    from nano_ktrans_b200.expert_parallel import plan_placement

    E, k, H, I = 128, 8, 2048, 768
    lw = _random_layer(E, H, I, 4, 128, cuda_device, 7)
    tokens = [40 + 13 * r for r in range(world)]
    tokens[-1] = 0 if world > 2 else tokens[-1]  # a rank without tokens still serves its experts
    gen = torch.Generator(device=cuda_device).manual_seed(3)
    wr = (torch.randn(E, H, device=cuda_device, generator=gen) * 0.02).to(torch.bfloat16)
    bias = torch.log(torch.arange(1, E + 1, device=cuda_device, dtype=torch.float32) ** -1.2)[
        torch.randperm(E, device=cuda_device, generator=gen)]
    xs, lgs = [], []
    for t in tokens:
        x = torch.randn(t, H, device=cuda_device, generator=gen).to(torch.bfloat16)
        xs.append(x)
        lgs.append(((x @ wr.T).float() + bias).to(torch.bfloat16))
    freq = torch.zeros(E)
    probe = _ep_layers(lw, 1, plan_placement(E, 1), k, max(tokens))[0]
    for lg in lgs:
        if lg.shape[0]:
            ids, _ = probe.route(lg)
            freq += torch.bincount(ids.reshape(-1).cpu(), minlength=E)
    probe.close()
    slot = plan_placement(E, world, freq.numpy())
    layers = _ep_layers(lw, world, slot, k, max(tokens))
    for L in layers:
        L.set_gemm(mode)
    res = _emulate(layers, xs, lgs)
    torch.cuda.synchronize()
    for r, (out, ids, w) in enumerate(res):
        assert out.shape == (tokens[r], H)
        if tokens[r] == 0:
            continue
        ref = _single_gpu(lw, k, xs[r], ids, w, mode)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"rank {r} differs from single GPU"
    assert all(L.read_status() == 0 for L in layers)


def test_ep_emulated_matches_oracle(cuda_device):
    """Small layer with oracle-quantized experts: EP output within the parity bar of the oracle."""
    from nano_ktrans_b200.expert_parallel import plan_placement

    E, k, H, I, world = 16, 4, 256, 256, 4
    experts = {e: hp.make_expert(12, e, H, I, 4, 128) for e in range(E)}
    lw = hp.device_layer(experts, E, H, I, 4, 128, cuda_device)
    tokens = [9, 0, 17, 5]
    ins = [hp.make_inputs(60 + r, t, H, E) for r, t in enumerate(tokens)]
    layers = _ep_layers(lw, world, plan_placement(E, world), k, max(tokens))
    res = _emulate(layers, [hp.bf16_tensor(x, cuda_device) for x, _ in ins],
                   [hp.bf16_tensor(lg, cuda_device) for _, lg in ins])
    torch.cuda.synchronize()
    for r, (out, ids, w) in enumerate(res):
        if tokens[r] == 0:
            assert out.shape[0] == 0
            continue
        ref = mo.offload_forward_f32(ins[r][0], ids.cpu().numpy(), hp.bf16_bits(w), experts)
        hp.assert_parity(hp.bf16_bits(out), ref, MAX_ABS, MEAN_REL)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, path):
    import datetime

    import torch.distributed as dist

    from nano_ktrans_b200.expert_parallel import TorchDistComm, plan_placement

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        E, k, H, I = 128, 8, 2048, 768
        lw = _random_layer(E, H, I, 4, 128, dev, 7)  # same seed: identical weights on every rank
        slot = plan_placement(E, world)
        from nano_ktrans_b200.expert_parallel import EpMoeLayer, shard_layer

        ep = EpMoeLayer(shard_layer(lw, slot, rank, world), num_experts=E, top_k=k, slot_of_expert=slot, rank=rank,
                        world=world, max_tokens=96)
        ep.set_gemm(2)
        gen = torch.Generator(device=dev).manual_seed(100 + rank)
        t = 96 - 31 * rank
        x = torch.randn(t, H, device=dev, generator=gen).to(torch.bfloat16)
        lg = torch.randn(t, E, device=dev, generator=gen).to(torch.bfloat16)
        out, ids, w = ep.forward(x, lg, TorchDistComm())
        torch.cuda.synchronize()
        ref = _single_gpu(lw, k, x, ids, w, 2)
        torch.cuda.synchronize()
        same = bool(torch.equal(out.view(torch.int16), ref.view(torch.int16)))
        np.save(path, np.array([same, ep.read_status() == 0, t == out.shape[0]]))
        ep.close()
    finally:
        dist.destroy_process_group()


def test_ep_nccl_ranks_bit_identical_to_single_gpu(tmp_path):
    """Two (or more) GPUs: the same step over NCCL all_to_all_single."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = min(n, 4)
    port = _free_port()
    ctx = mp.get_context("spawn")
    paths = [str(tmp_path / f"r{r}.npy") for r in range(world)]
    procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, paths[r])) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        same, ok, shape = np.load(paths[r])
        assert shape and ok and same, f"rank {r}: equal={same} status_ok={ok}"
