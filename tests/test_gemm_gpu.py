"""GPU parity of the prefill path: tensor-core grouped GEMM (grouped_gemm.cu).

The GEMM path replaces the per-expert matvec loop of nano-ktrans's CPU
backend (nano_ktrans/kernels/cpu_moe.py:515-536) for batches where experts see
many tokens.  Every test runs it through the C ABI and compares with the
oracle's restatement of the reference (fp32 accumulation, one bf16 rounding)
at the parity bar of the rest of the suite, and with the matvec path on the
same inputs.  Token counts per expert are chosen to hit the tile edges
(1, 127, 128, 129, 257 tokens; experts with none).
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from tests import helpers as hp

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 5e-3
GEMM_LAUNCHES = 6  # permute, tile table, pack, gate/up GEMM, down GEMM, combine


def _layer(lw, top_k, use_softmax=True, renorm=True, max_tokens=64):
    from nano_ktrans_b200.moe_layer import MoeLayer

    return MoeLayer(lw, top_k=top_k, router_use_softmax=use_softmax, normalize_topk_prob=renorm,
                    max_tokens=max_tokens)


def _ids_with_counts(counts, top_k, seed):
    """[T, top_k] expert ids in which expert e occurs counts[e] times, each
    token's ids distinct (sum(counts) = T * top_k, max(counts) <= T)."""
    total = int(sum(counts))
    assert total % top_k == 0
    t = total // top_k
    assert max(counts) <= t
    flat = np.repeat(np.arange(len(counts)), counts)  # sorted by expert
    ids = flat.reshape(top_k, t).T.copy()  # slot j takes flat[j*t + i]: distinct since max count <= t
    rng = np.random.Generator(np.random.PCG64([seed, 3]))
    ids = ids[rng.permutation(t)]
    for row in ids:
        rng.shuffle(row)
    return ids.astype(np.int64)


def _weights(t, top_k, seed):
    rng = np.random.Generator(np.random.PCG64([seed, 4]))
    w = rng.uniform(0.05, 1.0, size=(t, top_k)).astype(np.float32)
    return mo.f32_to_bf16_bits(w / w.sum(axis=1, keepdims=True))


def _run(layer, x, ids, w, dev, mode, mask=None, tile=0):
    layer.set_decode_fused(False)
    layer.set_gemm(mode)
    layer.set_gemm_tile(tile)
    out = layer.experts_forward(hp.bf16_tensor(x, dev), torch.from_numpy(ids).to(dev), hp.bf16_tensor(w, dev),
                                offload_mask=None if mask is None else torch.from_numpy(mask).to(dev))
    torch.cuda.synchronize()
    return hp.bf16_bits(out), layer.last_launch_count()


@pytest.mark.parametrize("tile", [16, 32, 64, 128])
@pytest.mark.parametrize("bits,group", [(4, 64), (4, 128), (4, 0), (8, 0)], ids=["w4g64", "w4g128", "w4pc", "w8pc"])
def test_gemm_ragged_tiles(bits, group, tile, cuda_device):
    """Per-expert token counts 129, 128, 1, 0, 257, 6, 127 against the oracle,
    and against the matvec path, at every token-tile width."""
    E, k, H, I = 7, 2, 256, 384
    counts = [129, 128, 1, 0, 257, 6, 127]
    ids = _ids_with_counts(counts, k, 11)
    t = ids.shape[0]
    x, _ = hp.make_inputs(5, t, H, E)
    w = _weights(t, k, 5)
    experts = {e: hp.make_expert(9, e, H, I, bits, group) for e in range(E) if counts[e]}
    lw = hp.device_layer(experts, E, H, I, bits, group, cuda_device)
    layer = _layer(lw, k, max_tokens=t)
    got, n = _run(layer, x, ids, w, cuda_device, 2, tile=tile)
    assert n == GEMM_LAUNCHES
    ref = mo.offload_forward_f32(x, ids, w, experts)
    hp.assert_parity(got, ref, MAX_ABS, MEAN_REL)
    mv, n_mv = _run(layer, x, ids, w, cuda_device, 0)
    assert n_mv < GEMM_LAUNCHES
    hp.assert_paths_agree(got, mv, MAX_ABS, MEAN_REL)
    assert layer.read_status() == 0


def test_gemm_offload_mask(cuda_device):
    """Experts excluded by the offload mask contribute nothing; the others
    match the oracle restricted to the same mask."""
    E, k, H, I = 7, 2, 256, 384
    counts = [129, 128, 1, 0, 257, 6, 127]
    ids = _ids_with_counts(counts, k, 12)
    t = ids.shape[0]
    x, _ = hp.make_inputs(6, t, H, E)
    w = _weights(t, k, 6)
    experts = {e: hp.make_expert(10, e, H, I, 4, 128) for e in range(E) if counts[e]}
    layer = _layer(hp.device_layer(experts, E, H, I, 4, 128, cuda_device), k, max_tokens=t)
    mask = np.array([1, 0, 1, 1, 0, 1, 1], dtype=np.uint8)
    got, n = _run(layer, x, ids, w, cuda_device, 2, mask)
    assert n == GEMM_LAUNCHES
    hp.assert_parity(got, mo.offload_forward_f32(x, ids, w, experts, mask.astype(bool)), MAX_ABS, MEAN_REL)


def test_gemm_deterministic(cuda_device):
    E, k, H, I = 7, 2, 256, 384
    counts = [129, 128, 1, 0, 257, 6, 127]
    ids = _ids_with_counts(counts, k, 13)
    t = ids.shape[0]
    x, _ = hp.make_inputs(7, t, H, E)
    w = _weights(t, k, 7)
    experts = {e: hp.make_expert(11, e, H, I, 4, 64) for e in range(E) if counts[e]}
    layer = _layer(hp.device_layer(experts, E, H, I, 4, 64, cuda_device), k, max_tokens=t)
    a, _ = _run(layer, x, ids, w, cuda_device, 2)
    b, _ = _run(layer, x, ids, w, cuda_device, 2)
    assert np.array_equal(a, b)
    # the tile width changes which tokens share an MMA, not any token's arithmetic
    for tile in (16, 32, 64, 128):
        c, _ = _run(layer, x, ids, w, cuda_device, 2, tile=tile)
        assert np.array_equal(a, c), tile


@pytest.mark.parametrize("tokens", [64, 256])
def test_gemm_qwen3_w4(tokens, cuda_device):
    """Qwen3-30B-A3B-shaped W4 g128 layer at 64 and 256 tokens, routed on the
    device."""
    cfg = hp.QWEN3
    x, logits = hp.make_inputs(300 + tokens, tokens, cfg["hidden"], cfg["experts"])
    ids_ref, w_ref, ranked = mo.route(logits, cfg["top_k"], True, True)
    check = np.arange(tokens) if tokens <= 64 else np.arange(0, tokens, 16)
    needed = sorted(set(ids_ref.reshape(-1).tolist()))
    experts = {e: hp.make_expert(300, e, cfg["hidden"], cfg["inter"], 4, 128) for e in needed}
    layer = _layer(hp.device_layer(experts, cfg["experts"], cfg["hidden"], cfg["inter"], 4, 128, cuda_device),
                   cfg["top_k"], max_tokens=tokens)
    layer.set_gemm(2)
    xd, ld = hp.bf16_tensor(x, cuda_device), hp.bf16_tensor(logits, cuda_device)
    ids = torch.empty(tokens, cfg["top_k"], dtype=torch.int64, device=cuda_device)
    w = torch.empty(tokens, cfg["top_k"], dtype=torch.bfloat16, device=cuda_device)
    out = layer.forward(xd, ld, out_ids=ids, out_weights=w)
    torch.cuda.synchronize()
    assert layer.last_launch_count() == GEMM_LAUNCHES + 1  # + routing
    ids_np = ids.cpu().numpy()
    assert mo.tie_aware_match(ids_np, ids_ref, ranked).all()
    got = hp.bf16_bits(out)
    ref = mo.offload_forward_f32(x[check], ids_np[check], hp.bf16_bits(w)[check], experts)
    hp.assert_parity(got[check], ref, MAX_ABS, MEAN_REL)
    # the whole batch against the matvec path
    mv, _ = _run(layer, x, ids_np, hp.bf16_bits(w), cuda_device, 0)
    hp.assert_paths_agree(got, mv, MAX_ABS, MEAN_REL)
    assert layer.read_status() == 0


def test_gemm_qwen2_shared_expert(cuda_device):
    """Qwen2-MoE-shaped W4 layer (60 experts, top-4, shared expert) at 128
    tokens with Zipf-skewed routing: routed experts on the GEMM path, the
    shared expert added before the single bf16 rounding."""
    cfg = hp.QWEN2
    tokens, seed = 128, 77
    x, logits = hp.make_inputs(seed, tokens, cfg["hidden"], cfg["experts"], zipf=1.2)
    ids_ref, w_ref, _ = mo.route(logits, cfg["top_k"], True, False)
    check = np.arange(0, tokens, 8)
    needed = sorted(set(ids_ref.reshape(-1).tolist()))
    experts = {e: hp.make_expert(seed, e, cfg["hidden"], cfg["inter"], 4, 128) for e in needed}
    rng = np.random.Generator(np.random.PCG64([seed, 99]))
    shared = tuple(mo.make_quant_linear(rng.standard_normal(s, dtype=np.float32) * np.float32(0.02), 128, 4)
                   for s in ((cfg["shared_inter"], cfg["hidden"]), (cfg["shared_inter"], cfg["hidden"]),
                             (cfg["hidden"], cfg["shared_inter"])))
    gate_vec = mo.f32_to_bf16_bits(rng.standard_normal(cfg["hidden"], dtype=np.float32) * np.float32(0.02))
    lw = hp.device_layer(experts, cfg["experts"], cfg["hidden"], cfg["inter"], 4, 128, cuda_device, shared, gate_vec)
    layer = _layer(lw, cfg["top_k"], True, False, max_tokens=tokens)
    layer.set_gemm(2)
    ids = torch.empty(tokens, cfg["top_k"], dtype=torch.int64, device=cuda_device)
    w = torch.empty(tokens, cfg["top_k"], dtype=torch.bfloat16, device=cuda_device)
    out = layer.forward(hp.bf16_tensor(x, cuda_device), hp.bf16_tensor(logits, cuda_device), out_ids=ids,
                        out_weights=w)
    torch.cuda.synchronize()
    ids_np, w_np = ids.cpu().numpy(), hp.bf16_bits(w)
    ref = mo.offload_forward_f32(x[check], ids_np[check], w_np[check], experts) + \
        mo.shared_expert_f32(x[check], gate_vec, shared)
    hp.assert_parity(hp.bf16_bits(out)[check], ref, MAX_ABS, MEAN_REL)
    assert layer.read_status() == 0


def test_gemm_mixtral_w8_prefill(cuda_device):
    """Mixtral-8x7B-shaped W8 per-channel layer (8 experts, top-2, hidden
    4096, inter 14336) at 2048 prefill tokens, Mixtral top-k -> softmax
    routing; sample tokens against the oracle, every token against the matvec
    path."""
    cfg = hp.MIXTRAL
    tokens, seed = 2048, 21
    x, logits = hp.make_inputs(seed, tokens, cfg["hidden"], cfg["experts"])
    ids_ref, w_ref, ranked = mo.route(logits, cfg["top_k"], False, True)
    check = np.arange(0, tokens, 256)
    needed = sorted(set(ids_ref[check].reshape(-1).tolist()))
    experts = {e: hp.make_expert(seed, e, cfg["hidden"], cfg["inter"], 8, 0) for e in needed}
    lw = hp.device_layer(experts, cfg["experts"], cfg["hidden"], cfg["inter"], 8, 0, cuda_device)
    layer = _layer(lw, cfg["top_k"], False, True, max_tokens=tokens)
    ids = torch.empty(tokens, cfg["top_k"], dtype=torch.int64, device=cuda_device)
    w = torch.empty(tokens, cfg["top_k"], dtype=torch.bfloat16, device=cuda_device)
    out = layer.forward(hp.bf16_tensor(x, cuda_device), hp.bf16_tensor(logits, cuda_device), out_ids=ids,
                        out_weights=w)
    torch.cuda.synchronize()
    assert layer.last_launch_count() == GEMM_LAUNCHES + 1
    ids_np, w_np = ids.cpu().numpy(), hp.bf16_bits(w)
    assert mo.tie_aware_match(ids_np, ids_ref, ranked).all()
    got = hp.bf16_bits(out)
    hp.assert_parity(got[check], mo.offload_forward_f32(x[check], ids_np[check], w_np[check], experts),
                     MAX_ABS, MEAN_REL)
    mv, _ = _run(layer, x, ids_np, w_np, cuda_device, 0)
    hp.assert_paths_agree(got, mv, MAX_ABS, MEAN_REL)
    assert layer.read_status() == 0


def test_gemm_refused_outside_shape_rules(cuda_device):
    """inter = 96 is not a multiple of the 128-row tile: forcing the GEMM path
    is refused with a message, the default selection keeps the matvec path."""
    E, k, H, I = 4, 2, 256, 96
    experts = {e: hp.make_expert(1, e, H, I, 4, 32) for e in range(E)}
    layer = _layer(hp.device_layer(experts, E, H, I, 4, 32, cuda_device), k, max_tokens=64)
    with pytest.raises(RuntimeError, match="GEMM"):
        layer.set_gemm(2)
    ids = _ids_with_counts([16, 16, 16, 16], k, 1)
    t = ids.shape[0]
    x, _ = hp.make_inputs(2, t, H, E)
    w = _weights(t, k, 2)
    got, n = _run(layer, x, ids, w, cuda_device, 1)
    assert n < GEMM_LAUNCHES
    hp.assert_parity(got, mo.offload_forward_f32(x, ids, w, experts), MAX_ABS, MEAN_REL)
