"""GPU parity: the CUDA path through the C-ABI against the oracle and against
golden vectors recorded from nano-ktrans itself.

Bars (from the north star): routing ids bit-exact (tie-aware), dequantized
weights bit-exact, bf16 outputs within max-abs 2e-2 and mean-rel 5e-3 of the
reference fp32-accumulated path, where mean-rel = mean|got-ref| / mean|ref|.
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from tests import helpers as hp
from tests.golden.cases import CASES
from tests.golden.load import load, oracle_experts, oracle_shared

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 5e-3


def _layer(weights, top_k, use_softmax, renorm, max_tokens=64):
    from nano_ktrans_b200.moe_layer import MoeLayer

    return MoeLayer(weights, top_k=top_k, router_use_softmax=use_softmax, normalize_topk_prob=renorm,
                    max_tokens=max_tokens)


def _golden_layer(name, dev):
    g = load(name)
    c = g["case"]
    experts = oracle_experts(c)
    group = c["group_size"]
    shared = gate_vec = None
    if c.get("shared_inter"):
        shared, gate_vec = oracle_shared(c)
    lw = hp.device_layer(experts, c["experts"], c["hidden"], c["inter"], c["bits"], group, dev, shared, gate_vec)
    return g, c, experts, _layer(lw, c["top_k"], c["use_softmax"], c["renormalize"])


# ---------------------------------------------------------------------------
# Golden vectors from the reference
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("name", sorted(CASES))
def test_route_matches_reference(name, cuda_device):
    g, c, _, layer = _golden_layer(name, cuda_device)
    ids, w = layer.route(hp.bf16_tensor(g["logits"], cuda_device))
    ids = ids.cpu().numpy()
    assert mo.tie_aware_match(ids, g["ids"], g["ranked"]).all()
    # weights per selected expert equal the reference's, bit for bit
    wb = hp.bf16_bits(w)
    for t in range(ids.shape[0]):
        ref = dict(zip(g["ids"][t].tolist(), g["weights"][t].tolist()))
        mine = dict(zip(ids[t].tolist(), wb[t].tolist()))
        if set(ref) == set(mine):
            assert ref == mine, (t, ref, mine)


@pytest.mark.parametrize("fused", [1, 2, 0], ids=["fused", "fused_multi", "chain"])
@pytest.mark.parametrize("name", sorted(CASES))
def test_experts_match_reference(name, fused, cuda_device):
    g, c, _, layer = _golden_layer(name, cuda_device)
    layer.set_decode_fused(fused)
    x = hp.bf16_tensor(g["x"], cuda_device)
    ids = torch.from_numpy(g["ids"]).to(cuda_device)
    w = hp.bf16_tensor(g["weights"], cuda_device)
    mask = None
    if c.get("gpu_experts"):
        m = np.ones(c["experts"], dtype=np.uint8)
        m[c["gpu_experts"]] = 0
        mask = torch.from_numpy(m).to(cuda_device)
    out = layer.experts_forward(x, ids, w, offload_mask=mask)
    torch.cuda.synchronize()
    hp.assert_parity(hp.bf16_bits(out), g["out_f32"], MAX_ABS, MEAN_REL)
    # tighter than the bar: only fp32 summation order differs from the reference
    got = mo.bf16_bits_to_f32(hp.bf16_bits(out))
    assert np.abs(got - mo.bf16_bits_to_f32(g["out_bf16"])).max() <= 2 * np.abs(g["out_f32"]).max() * 2 ** -8
    if "shared_f32" in g:
        out2 = layer.experts_forward(x, ids, w, add_shared=True)
        hp.assert_parity(hp.bf16_bits(out2), g["out_f32"] + g["shared_f32"], MAX_ABS, MEAN_REL)


@pytest.mark.parametrize("name", ["qwen3_w4_t7", "qwen3_w8_t3", "mixtral_w8_t9"])
def test_dequant_bit_exact(name, cuda_device):
    g, c, experts, layer = _golden_layer(name, cuda_device)
    for e in (0, c["experts"] - 1):
        for proj, ql in enumerate(experts[e]):
            got = layer.dequant_rows(proj, e, 0, ql.output_dim).cpu().numpy()
            np.testing.assert_array_equal(got, ql.dequantize())


@pytest.mark.parametrize("bits", [4, 8])
def test_dequant_exhaustive_codes(bits, cuda_device):
    """Every code at every position of a word, with scales spanning exponents."""
    n_codes = 1 << bits
    H, I = 256, 64
    rng = np.random.Generator(np.random.PCG64(9))
    trip = []
    for n, k in ((I, H), (I, H), (H, I)):
        codes = rng.integers(0, n_codes, size=(n, k), dtype=np.uint8)
        m = min(n_codes, k)
        codes[0, :m] = np.arange(m)
        codes[1, :] = np.arange(k) % n_codes
        g = 32 if bits == 4 else 16
        scales = mo.round_bf16(np.exp2(rng.uniform(-20, 4, size=(n, k // g))).astype(np.float32))
        trip.append(mo.QuantLinear(mo.pack_words(codes, bits), scales, g, bits))
    lw = hp.device_layer({0: tuple(trip)}, 1, H, I, bits, 32 if bits == 4 else 16, cuda_device)
    layer = _layer(lw, 1, True, True)
    for proj, ql in enumerate(trip):
        got = layer.dequant_rows(proj, 0, 0, ql.output_dim).cpu().numpy()
        np.testing.assert_array_equal(got, ql.dequantize())


def test_hybrid_moe_from_gptq_checkpoint(tmp_path, cuda_device):
    """Drop-in path: HybridMoE(offload_backend="cuda") loading the same GPTQ
    safetensors layout the reference loads, vs the reference's output."""
    import json

    from safetensors.torch import save_file

    from nano_ktrans_b200.hybrid_moe import HybridMoE

    name = "qwen3_w4_t7"
    g = load(name)
    c = g["case"]
    tensors = {}
    for e, trip in oracle_experts(c).items():
        for p, ql in zip(("gate_proj", "up_proj", "down_proj"), trip):
            pre = f"model.layers.0.mlp.experts.{e}.{p}"
            tensors[pre + ".qweight"] = torch.from_numpy(ql.qweight.T.copy())
            tensors[pre + ".scales"] = torch.from_numpy(ql.scales.T.copy())
    save_file(tensors, str(tmp_path / "model.safetensors"))
    (tmp_path / "quantize_config.json").write_text(json.dumps({"bits": 4, "group_size": 128, "sym": True}))
    moe = HybridMoE(num_experts=c["experts"], top_k=c["top_k"], hidden_size=c["hidden"],
                    moe_intermediate_size=c["inter"], gpu_experts=torch.nn.ModuleDict(),
                    gpu_experts_mask=torch.zeros(c["experts"], dtype=torch.bool), layer_idx=0,
                    weight_path=str(tmp_path), router_use_softmax=True, normalize_topk_prob=True,
                    expert_key_template="model.layers.{layer}.mlp.experts.{expert}.{proj}.weight",
                    expert_proj_names={"gate": "gate_proj", "up": "up_proj", "down": "down_proj"},
                    offload_backend_kwargs={"device": cuda_device, "max_tokens": 16})
    out = moe(hp.bf16_tensor(g["x"], cuda_device), hp.bf16_tensor(g["logits"], cuda_device))
    torch.cuda.synchronize()
    hp.assert_parity(hp.bf16_bits(out), g["out_f32"], MAX_ABS, MEAN_REL)
    assert mo.tie_aware_match(moe.last_topk_ids.cpu().numpy(), g["ids"], g["ranked"]).all()


def test_backend_submit_sync_with_gpu_experts(cuda_device):
    """Backend contract with a GPU-expert mask: only offloaded experts computed."""
    from nano_ktrans_b200.cuda_moe import CudaMoEBackend
    from nano_ktrans_b200.weights import GPTQLinearWeight

    name = "qwen3_w4_mask"
    g = load(name)
    c = g["case"]
    experts = {}
    for e, trip in oracle_experts(c).items():
        experts[e] = {p: GPTQLinearWeight(torch.from_numpy(ql.qweight), torch.from_numpy(ql.scales), None,
                                          ql.group_size, ql.bits, True, f"e{e}.{p}")
                      for p, ql in zip(("gate", "up", "down"), trip)}
    mask = torch.zeros(c["experts"], dtype=torch.bool)
    mask[c["gpu_experts"]] = True
    be = CudaMoEBackend(0, c["experts"], c["top_k"], c["hidden"], c["inter"], mask, gptq_experts=experts,
                        device=cuda_device, max_tokens=8)
    x = hp.bf16_tensor(g["x"], cuda_device)
    stream = torch.cuda.Stream(cuda_device)
    with torch.cuda.stream(stream):
        be.submit_forward(x, torch.from_numpy(g["ids"]).to(cuda_device), hp.bf16_tensor(g["weights"], cuda_device),
                          stream.cuda_stream)
    out = be.sync_forward(x, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    hp.assert_parity(hp.bf16_bits(out), g["out_f32"], MAX_ABS, MEAN_REL)
    assert be.submit_calls == 1 and be.sync_calls == 1
    assert be.diagnostics()["offloaded_experts"] == c["experts"] - len(c["gpu_experts"])


# ---------------------------------------------------------------------------
# BASELINE shapes against the oracle
# ---------------------------------------------------------------------------


def _full_case(cfg, tokens, bits, group, seed, cuda_device, zipf=None, sample_tokens=None):
    x, logits = hp.make_inputs(seed, tokens, cfg["hidden"], cfg["experts"], zipf)
    ids_ref, w_ref, ranked = mo.route(logits, cfg["top_k"], cfg["use_softmax"], cfg["renormalize"])
    check_tok = np.arange(tokens) if sample_tokens is None else sample_tokens
    needed = sorted(set(ids_ref[check_tok].reshape(-1).tolist()))
    experts = {e: hp.make_expert(seed, e, cfg["hidden"], cfg["inter"], bits, group) for e in needed}
    shared = gate_vec = None
    if cfg.get("shared_inter"):
        rng = np.random.Generator(np.random.PCG64([seed, 99]))
        shared = tuple(mo.make_quant_linear(rng.standard_normal(s, dtype=np.float32) * np.float32(0.02), group, bits)
                       for s in ((cfg["shared_inter"], cfg["hidden"]), (cfg["shared_inter"], cfg["hidden"]),
                                 (cfg["hidden"], cfg["shared_inter"])))
        gate_vec = mo.f32_to_bf16_bits(rng.standard_normal(cfg["hidden"], dtype=np.float32) * np.float32(0.02))
    lw = hp.device_layer(experts, cfg["experts"], cfg["hidden"], cfg["inter"], bits, group, cuda_device, shared,
                         gate_vec)
    layer = _layer(lw, cfg["top_k"], cfg["use_softmax"], cfg["renormalize"], max_tokens=tokens)
    return dict(x=x, logits=logits, ids=ids_ref, w=w_ref, ranked=ranked, experts=experts, layer=layer,
                check=check_tok, shared=shared, gate_vec=gate_vec)


@pytest.mark.parametrize("fused", [1, 2, 0], ids=["fused", "fused_multi", "chain"])
@pytest.mark.parametrize("tokens", [1, 3, 8, 32, 64])
def test_qwen3_w4_decode_sweep(tokens, fused, cuda_device):
    """Config 2: Qwen3-30B-A3B-shaped W4 g128 decode at batch 1/8/32/64 (and 3),
    through the single-launch kernel (where the batch allows) and the chain."""
    d = _full_case(hp.QWEN3, tokens, 4, 128, 100 + tokens, cuda_device)
    layer = d["layer"]
    layer.set_decode_fused(fused)
    ids, w = layer.route(hp.bf16_tensor(d["logits"], cuda_device))
    assert mo.tie_aware_match(ids.cpu().numpy(), d["ids"], d["ranked"]).all()
    x = hp.bf16_tensor(d["x"], cuda_device)
    out = layer.experts_forward(x, torch.from_numpy(d["ids"]).to(cuda_device), hp.bf16_tensor(d["w"], cuda_device))
    fused = layer.forward(x, hp.bf16_tensor(d["logits"], cuda_device))
    torch.cuda.synchronize()
    ref = mo.offload_forward_f32(d["x"], d["ids"], d["w"], d["experts"])
    hp.assert_parity(hp.bf16_bits(out), ref)
    # the in-kernel-routed output against the oracle run on the device's own
    # routing (which may differ from the oracle's only on exact ties)
    # (experts the oracle's routing never picked hold zero weights on the device)
    ids_d, w_d = layer.route(hp.bf16_tensor(d["logits"], cuda_device))
    present = np.isin(np.arange(hp.QWEN3["experts"]), list(d["experts"]))
    ref_d = mo.offload_forward_f32(d["x"], ids_d.cpu().numpy(), hp.bf16_bits(w_d), d["experts"], present)
    hp.assert_parity(hp.bf16_bits(fused), ref_d)
    assert layer.read_status() == 0


@pytest.mark.parametrize("fused", [1, 2, 0], ids=["fused", "fused_multi", "chain"])
def test_qwen3_w8_per_channel_decode(fused, cuda_device):
    """Config 1: W8 symmetric per-output-channel, batch 1."""
    d = _full_case(hp.QWEN3, 1, 8, 0, 7, cuda_device)
    d["layer"].set_decode_fused(fused)
    out = d["layer"].forward(hp.bf16_tensor(d["x"], cuda_device), hp.bf16_tensor(d["logits"], cuda_device))
    torch.cuda.synchronize()
    ref = mo.offload_forward_f32(d["x"], d["ids"], d["w"], d["experts"])
    hp.assert_parity(hp.bf16_bits(out), ref)


def test_qwen2_shared_expert_zipf(cuda_device):
    """Config 4 shapes (60 experts, top-4 no renorm, W4 shared expert) on a token
    sample: every 37th token plus every token routed to the busiest expert."""
    x, logits = hp.make_inputs(21, 256, hp.QWEN2["hidden"], hp.QWEN2["experts"], 1.2)
    ids0, _, _ = mo.route(logits, hp.QWEN2["top_k"], hp.QWEN2["use_softmax"], hp.QWEN2["renormalize"])
    head = np.bincount(ids0.reshape(-1), minlength=hp.QWEN2["experts"]).argmax()
    sample = np.union1d(np.arange(0, 256, 37), np.where((ids0 == head).any(axis=1))[0])
    d = _full_case(hp.QWEN2, 256, 4, 128, 21, cuda_device, zipf=1.2, sample_tokens=sample)
    out = d["layer"].forward(hp.bf16_tensor(d["x"], cuda_device), hp.bf16_tensor(d["logits"], cuda_device))
    torch.cuda.synchronize()
    xs = d["x"][sample]
    ref = mo.offload_forward_f32(xs, d["ids"][sample], d["w"][sample], d["experts"])
    ref = ref + mo.shared_expert_f32(xs, d["gate_vec"], d["shared"])
    hp.assert_parity(hp.bf16_bits(out)[sample], ref)


# ---------------------------------------------------------------------------
# Properties and edge cases
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("tokens", [4, 32])
def test_deterministic_and_permutation_equivariant(tokens, cuda_device):
    d = _full_case(hp.QWEN3, tokens, 4, 128, 5, cuda_device)
    layer = d["layer"]
    x = hp.bf16_tensor(d["x"], cuda_device)
    lg = hp.bf16_tensor(d["logits"], cuda_device)
    a = layer.forward(x, lg).clone()
    b = layer.forward(x, lg).clone()
    perm = torch.randperm(tokens, generator=torch.Generator().manual_seed(1)).to(cuda_device)
    c = layer.forward(x[perm].contiguous(), lg[perm].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(a[perm], c)


@pytest.mark.parametrize("tokens", [2, 8])
def test_mask_split_sums_to_whole(tokens, cuda_device):
    d = _full_case(hp.QWEN3, tokens, 4, 128, 6, cuda_device)
    layer = d["layer"]
    x = hp.bf16_tensor(d["x"], cuda_device)
    ids = torch.from_numpy(d["ids"]).to(cuda_device)
    w = hp.bf16_tensor(d["w"], cuda_device)
    m = (torch.arange(128, device=cuda_device) % 3 == 0).to(torch.uint8)
    whole = layer.experts_forward(x, ids, w).float()
    part = layer.experts_forward(x, ids, w, offload_mask=m).float() + \
        layer.experts_forward(x, ids, w, offload_mask=1 - m).float()
    torch.cuda.synchronize()
    assert (whole - part).abs().max().item() <= 2 * whole.abs().max().item() * 2 ** -8


@pytest.mark.parametrize("fused", [1, 2, 0], ids=["fused", "fused_multi", "chain"])
def test_empty_and_bad_inputs(fused, cuda_device):
    d = _full_case(hp.QWEN3, 4, 4, 128, 8, cuda_device)
    layer = d["layer"]
    layer.set_decode_fused(fused)
    x = hp.bf16_tensor(d["x"], cuda_device)
    empty = layer.forward(x[:0], hp.bf16_tensor(d["logits"], cuda_device)[:0])
    assert empty.shape == (0, 2048)
    # all routed experts masked out -> zeros
    ids = torch.from_numpy(d["ids"]).to(cuda_device)
    w = hp.bf16_tensor(d["w"], cuda_device)
    z = layer.experts_forward(x, ids, w, offload_mask=torch.zeros(128, dtype=torch.uint8, device=cuda_device))
    torch.cuda.synchronize()
    assert torch.count_nonzero(z).item() == 0
    # out-of-range expert ids are skipped and reported, never dereferenced
    bad = ids.clone()
    bad[0, 0] = 500
    bad[1, 1] = -3
    layer.experts_forward(x, bad, w)
    assert layer.read_status() == 1
    assert layer.read_status() == 0
    # above max_tokens is refused on the host
    from nano_ktrans_b200._lib import MoeError

    big = torch.zeros(5, 2048, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(MoeError):
        layer.forward(big, torch.zeros(5, 128, dtype=torch.bfloat16, device=cuda_device))


def test_top_k_equals_num_experts(cuda_device):
    cfg = dict(hp.QWEN3, experts=8, top_k=8, hidden=256, inter=128)
    d = _full_case(cfg, 3, 4, 128, 9, cuda_device)
    out = d["layer"].forward(hp.bf16_tensor(d["x"], cuda_device), hp.bf16_tensor(d["logits"], cuda_device))
    torch.cuda.synchronize()
    hp.assert_parity(hp.bf16_bits(out), mo.offload_forward_f32(d["x"], d["ids"], d["w"], d["experts"]))


def test_fused_decode_is_one_launch_and_matches_chain(cuda_device):
    """The single-launch decode step equals the multi-kernel chain on the CUDA-core
    matvec kernels bit for bit (same per-row arithmetic and combine order), and
    the chain on the tensor-core streaming kernels within the parity bar."""
    d = _full_case(hp.QWEN3, 2, 4, 128, 31, cuda_device)
    layer = d["layer"]
    x = hp.bf16_tensor(d["x"], cuda_device)
    lg = hp.bf16_tensor(d["logits"], cuda_device)
    ids_f = torch.empty(2, 8, dtype=torch.int64, device=cuda_device)
    w_f = torch.empty(2, 8, dtype=torch.bfloat16, device=cuda_device)
    fused = layer.forward(x, lg, out_ids=ids_f, out_weights=w_f).clone()
    assert layer.last_launch_count() == 1
    layer.set_decode_fused(False)
    layer.set_stream(False)
    ids_c = torch.empty_like(ids_f)
    w_c = torch.empty_like(w_f)
    chain = layer.forward(x, lg, out_ids=ids_c, out_weights=w_c).clone()
    assert layer.last_launch_count() == 5
    layer.set_stream(True)
    streamed = layer.forward(x, lg)
    assert layer.last_launch_count() == 5
    torch.cuda.synchronize()
    assert torch.equal(ids_f, ids_c) and torch.equal(w_f, w_c)
    assert torch.equal(fused, chain)
    hp.assert_paths_agree(hp.bf16_bits(streamed), hp.bf16_bits(fused), MAX_ABS, MEAN_REL)
    assert layer.read_status() == 0


@pytest.mark.parametrize("mode", [1, 2], ids=["single_token", "multi_token"])
def test_single_token_decode_is_one_launch_and_matches_chain(mode, cuda_device):
    """One token: both single-launch kernels route bit-identically to the
    multi-kernel chain and match its output (same per-row arithmetic class,
    same combine order), and the oracle within the parity bar."""
    d = _full_case(hp.QWEN3, 1, 4, 128, 77, cuda_device)
    layer = d["layer"]
    x = hp.bf16_tensor(d["x"], cuda_device)
    lg = hp.bf16_tensor(d["logits"], cuda_device)
    ids_f = torch.empty(1, 8, dtype=torch.int64, device=cuda_device)
    w_f = torch.empty(1, 8, dtype=torch.bfloat16, device=cuda_device)
    layer.set_decode_fused(mode)
    fused = layer.forward(x, lg, out_ids=ids_f, out_weights=w_f).clone()
    assert layer.last_launch_count() == 1
    layer.set_decode_fused(0)
    ids_c = torch.empty_like(ids_f)
    w_c = torch.empty_like(w_f)
    chain = layer.forward(x, lg, out_ids=ids_c, out_weights=w_c)
    torch.cuda.synchronize()
    assert torch.equal(ids_f, ids_c) and torch.equal(w_f, w_c)
    hp.assert_paths_agree(hp.bf16_bits(fused), hp.bf16_bits(chain), MAX_ABS, MEAN_REL)
    ref = mo.offload_forward_f32(d["x"], ids_f.cpu().numpy(), hp.bf16_bits(w_f), d["experts"])
    hp.assert_parity(hp.bf16_bits(fused), ref, MAX_ABS, MEAN_REL)
    assert layer.read_status() == 0


def test_single_token_decode_repeated_and_masked(cuda_device):
    """The single-token kernel on consecutive calls (the grid-barrier counter
    carries over) and with an offload mask, through moe_experts_forward."""
    d = _full_case(hp.QWEN3, 1, 4, 128, 78, cuda_device)
    layer = d["layer"]
    x = hp.bf16_tensor(d["x"], cuda_device)
    ids = torch.from_numpy(d["ids"]).to(cuda_device)
    w = hp.bf16_tensor(d["w"], cuda_device)
    first = layer.experts_forward(x, ids, w).clone()
    assert layer.last_launch_count() == 1
    for _ in range(5):
        again = layer.experts_forward(x, ids, w)
    torch.cuda.synchronize()
    assert torch.equal(first, again)
    mask = np.ones(hp.QWEN3["experts"], dtype=np.uint8)
    mask[d["ids"][0, ::2]] = 0
    part = layer.experts_forward(x, ids, w, offload_mask=torch.from_numpy(mask).to(cuda_device))
    torch.cuda.synchronize()
    assert layer.last_launch_count() == 1
    ref = mo.offload_forward_f32(d["x"], d["ids"], d["w"], d["experts"], mask.astype(bool))
    hp.assert_parity(hp.bf16_bits(part), ref, MAX_ABS, MEAN_REL)
    assert layer.read_status() == 0


_T1_SHAPES = {
    # 7 output rows per CTA, 4 tensor-core groups per down row
    "h1024": dict(experts=64, top_k=4, hidden=1024, inter=512, use_softmax=True, renormalize=True),
    # 28 output rows per CTA: two 16-row down tiles, the second one partial
    "h4096": dict(experts=32, top_k=4, hidden=4096, inter=1024, use_softmax=True, renormalize=True),
    # 56 output rows per CTA (warps take two combine rows each), Mixtral routing, 16 experts
    "h8192_mixtral": dict(experts=16, top_k=2, hidden=8192, inter=512, use_softmax=False, renormalize=True),
}


@pytest.mark.parametrize("name", sorted(_T1_SHAPES))
def test_single_token_decode_shapes(name, cuda_device):
    """The single-token kernel away from the Qwen3 shape: other row counts per CTA,
    multi-tile down projections and both routing modes, against the oracle and
    the multi-kernel chain."""
    cfg = _T1_SHAPES[name]
    d = _full_case(cfg, 1, 4, 128, 90, cuda_device)
    layer = d["layer"]
    x = hp.bf16_tensor(d["x"], cuda_device)
    lg = hp.bf16_tensor(d["logits"], cuda_device)
    k = cfg["top_k"]
    ids_f = torch.empty(1, k, dtype=torch.int64, device=cuda_device)
    w_f = torch.empty(1, k, dtype=torch.bfloat16, device=cuda_device)
    layer.set_decode_fused(1)
    fused = layer.forward(x, lg, out_ids=ids_f, out_weights=w_f).clone()
    assert layer.last_launch_count() == 1
    torch.cuda.synchronize()
    assert mo.tie_aware_match(ids_f.cpu().numpy(), d["ids"], d["ranked"]).all()
    layer.set_decode_fused(0)
    chain = layer.forward(x, lg)
    torch.cuda.synchronize()
    hp.assert_paths_agree(hp.bf16_bits(fused), hp.bf16_bits(chain), MAX_ABS, MEAN_REL)
    ref = mo.offload_forward_f32(d["x"], ids_f.cpu().numpy(), hp.bf16_bits(w_f), d["experts"])
    hp.assert_parity(hp.bf16_bits(fused), ref, MAX_ABS, MEAN_REL)
    assert layer.read_status() == 0


def test_forward_rejects_unsafe_output_buffers(cuda_device):
    """A caller's out buffer is checked before any kernel may write [T, H] bf16 into it."""
    d = _full_case(hp.QWEN3, 2, 4, 128, 5, cuda_device)
    layer = d["layer"]
    x = hp.bf16_tensor(d["x"], cuda_device)
    lg = hp.bf16_tensor(d["logits"], cuda_device)
    H = hp.QWEN3["hidden"]
    bad = [torch.empty(1, H, dtype=torch.bfloat16, device=cuda_device),        # too few rows
           torch.empty(2, H, dtype=torch.float32, device=cuda_device),         # wrong dtype
           torch.empty(H, 2, dtype=torch.bfloat16, device=cuda_device).t(),    # not contiguous
           torch.empty(2, H, dtype=torch.bfloat16)]                            # host memory
    for out in bad:
        with pytest.raises(ValueError):
            layer.forward(x, lg, out=out)
    good = torch.empty(2, H, dtype=torch.bfloat16, device=cuda_device)
    assert layer.forward(x, lg, out=good) is good
