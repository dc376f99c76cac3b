"""CPU-only tests: the C-ABI library builds, loads and exports every declared
symbol; argument validation needs no GPU; the host-side container, quantizer,
device layout and GPTQ loader agree with the oracle."""
import ctypes
import json

import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo


@pytest.fixture(scope="module")
def lib():
    from nano_ktrans_b200 import _lib, build

    build.build()
    return _lib.lib()


def test_library_exports_every_header_symbol(lib):
    from nano_ktrans_b200 import _lib

    syms = _lib.header_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/moe_b200.h but not exported"
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"
    assert lib.moe_abi_version() == 1


@pytest.mark.parametrize("field,value,needle", [
    ("bits", 3, "bits"),
    ("top_k", 0, "top_k"),
    ("hidden_size", 100, "hidden_size"),
    ("group_size", 48, "group_size"),
    ("num_experts", 2000, "num_experts"),
    ("max_tokens", 0, "max_tokens"),
])
def test_create_rejects_bad_descriptions_without_gpu(lib, field, value, needle):
    from nano_ktrans_b200 import _lib

    d = dict(num_experts=128, top_k=8, hidden_size=2048, inter_size=768, bits=4, group_size=128,
             router_use_softmax=1, normalize_topk_prob=1, max_tokens=64, shared_inter=0)
    d[field] = value
    desc = _lib.MoeLayerDesc(*[d[n] for n in _lib._DESC_FIELDS])
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(256)
    rc = lib.moe_create(ctypes.byref(desc), ctypes.byref(h), err, len(err))
    assert rc == _lib.MOE_EINVAL
    assert needle in err.value.decode()
    assert not h.value


def test_null_handle_calls_fail_cleanly(lib):
    from nano_ktrans_b200 import _lib

    assert lib.moe_route(None, None, 0, None, None, None) == _lib.MOE_EINVAL
    assert lib.moe_experts_forward(None, None, None, None, 0, None, 0, None, None) == _lib.MOE_EINVAL
    lib.moe_destroy(None)


@pytest.mark.parametrize("args,needle", [
    ((0, 0, 64, 8, 2048, 128), "world"),
    ((0, 9, 64, 8, 2048, 128), "world"),
    ((2, 2, 64, 8, 2048, 128), "rank"),
    ((0, 2, 0, 8, 2048, 128), "max_tokens"),
    ((0, 2, 64, 0, 2048, 128), "top_k"),
    ((0, 2, 64, 8, 2044, 128), "hidden_size"),
    ((0, 3, 64, 8, 2048, 128), "num_experts"),
    ((0, 2, 64, 8, 2048, 4), "num_experts"),
])
def test_peer_group_rejects_bad_shapes_without_gpu(lib, args, needle):
    from nano_ktrans_b200 import _lib

    g = ctypes.c_void_p()
    err = ctypes.create_string_buffer(256)
    assert lib.moe_ep_group_create(*args, ctypes.byref(g), err, len(err)) == _lib.MOE_EINVAL
    assert needle in err.value.decode()
    assert not g.value


def test_peer_group_null_calls_fail_cleanly(lib):
    from nano_ktrans_b200 import _lib

    assert lib.moe_ep_peer_publish(None, None, None, 0, None, None) == _lib.MOE_EINVAL
    assert lib.moe_ep_peer_experts(None, None, 0, 0, None) == _lib.MOE_EINVAL
    assert lib.moe_ep_peer_combine(None, None, None, 0, None, None) == _lib.MOE_EINVAL
    assert lib.moe_ep_group_destroy(None) == _lib.MOE_EINVAL


@pytest.mark.parametrize("bits,group", [(4, 128), (4, 64), (8, 0), (8, 128)])
def test_torch_quantizer_matches_oracle(bits, group):
    from nano_ktrans_b200.weights import quantize_symmetric

    rng = np.random.Generator(np.random.PCG64(5))
    w = rng.standard_normal((48, 256), dtype=np.float32) * np.float32(0.02)
    q = quantize_symmetric(torch.from_numpy(w), group_size=group, bits=bits)
    ref = mo.make_quant_linear(w, group if group else 256, bits)
    np.testing.assert_array_equal(q.qweight.numpy(), ref.qweight)
    np.testing.assert_array_equal(q.scales.numpy(), ref.scales)
    np.testing.assert_array_equal(q.dequantize().numpy(), ref.dequantize())


def test_device_layout_is_the_reference_word_bytes():
    from nano_ktrans_b200.weights import quantize_symmetric, stack_layer

    rng = np.random.Generator(np.random.PCG64(6))
    experts = []
    for _ in range(3):
        experts.append({p: quantize_symmetric(torch.from_numpy(rng.standard_normal(s, dtype=np.float32) * 0.02),
                                              group_size=64)
                        for p, s in (("gate", (64, 256)), ("up", (64, 256)), ("down", (256, 64)))})
    lw = stack_layer(experts, "cpu")
    assert lw.gate_q.shape == (3, 64, 128) and lw.gate_q.dtype == torch.uint8
    assert lw.down_s.shape == (3, 256, 8) and lw.down_s.dtype == torch.bfloat16
    for e in range(3):
        words = lw.gate_q[e].numpy().view(np.int32)
        np.testing.assert_array_equal(words, experts[e]["gate"].qweight.numpy())
        codes = mo.unpack_words(words, 4)
        assert codes.shape == (64, 256)
    assert lw.group_size == 64
    assert lw.expert_bytes() == 2 * (64 * 128 + 64 * 4 * 2) + 256 * 32 + 256 * 1 * 2


def test_gptq_loader_reads_reference_layout(tmp_path):
    """The on-disk layout the reference's own loader test writes
    (tests/test_quantized_ops.py:20-52 of nano-ktrans)."""
    from safetensors.torch import save_file

    from nano_ktrans_b200.weight_loader import ExpertWeightLoader
    from nano_ktrans_b200.weights import quantize_symmetric

    dense = torch.randn(32, 128, generator=torch.Generator().manual_seed(0))
    q = quantize_symmetric(dense, group_size=64, scale_dtype=torch.float32)
    save_file({
        "model.layers.0.mlp.experts.0.gate_proj.qweight": q.qweight.t().contiguous(),
        "model.layers.0.mlp.experts.0.gate_proj.scales": q.scales.t().contiguous(),
        "model.layers.0.mlp.experts.0.gate_proj.g_idx": (torch.arange(128) // 64).to(torch.int32),
    }, str(tmp_path / "model.safetensors"))
    (tmp_path / "quantize_config.json").write_text(json.dumps({"bits": 4, "group_size": 64, "sym": True}))
    loaded = ExpertWeightLoader(str(tmp_path)).load_gptq_expert_linear(layer_idx=0, expert_idx=0, proj_name="gate")
    assert torch.equal(loaded.qweight, q.qweight)
    assert torch.equal(loaded.scales, q.scales)
    assert loaded.group_size == 64 and loaded.sym


def test_loader_rejects_nonsequential_g_idx(tmp_path):
    from safetensors.torch import save_file

    from nano_ktrans_b200.weight_loader import ExpertWeightLoader
    from nano_ktrans_b200.weights import quantize_symmetric

    q = quantize_symmetric(torch.randn(16, 128), group_size=64)
    g_idx = (torch.arange(128) // 64).flip(0).to(torch.int32)
    save_file({"l.qweight": q.qweight.t().contiguous(), "l.scales": q.scales.t().contiguous(), "l.g_idx": g_idx},
              str(tmp_path / "m.safetensors"))
    (tmp_path / "quantize_config.json").write_text(json.dumps({"bits": 4, "group_size": 64}))
    with pytest.raises(NotImplementedError):
        ExpertWeightLoader(str(tmp_path)).load_gptq_linear("l")


def test_backend_name_registry():
    from nano_ktrans_b200 import normalize_offload_backend_name

    assert normalize_offload_backend_name("cuda") == "cuda"
    assert normalize_offload_backend_name("B200") == "cuda"
    assert normalize_offload_backend_name(None) == "cpu"
    assert normalize_offload_backend_name("pim-shadow") == "pim_shadow"
    with pytest.raises(ValueError):
        normalize_offload_backend_name("tpu")


def test_moe_layer_refuses_cpu_tensors():
    from nano_ktrans_b200.moe_layer import MoeLayer
    from nano_ktrans_b200.weights import quantize_symmetric, stack_layer

    ex = [{p: quantize_symmetric(torch.randn(*s) * 0.02, group_size=64) for p, s in
           (("gate", (64, 256)), ("up", (64, 256)), ("down", (256, 64)))}]
    with pytest.raises(ValueError, match="CUDA"):
        MoeLayer(stack_layer(ex, "cpu"), top_k=1)


def test_routing_oracle_properties():
    rng = np.random.Generator(np.random.PCG64(3))
    logits = mo.f32_to_bf16_bits(rng.standard_normal((64, 128), dtype=np.float32))
    ids, w, probs = mo.route(logits, 8, True, True)
    wf = mo.bf16_bits_to_f32(w)
    assert np.all(np.diff(mo.bf16_bits_to_f32(probs)[np.arange(64)[:, None], ids], axis=1) <= 0)
    np.testing.assert_allclose(wf.sum(1), 1.0, atol=2e-2)
    ids2, w2, _ = mo.route(logits, 2, False, True)
    np.testing.assert_allclose(mo.bf16_bits_to_f32(w2).sum(1), 1.0, atol=1e-2)


def _stub_layer():
    """A MoeLayer with the attributes the argument checks read and no handle
    (the checks must reject before anything reaches the library)."""
    from nano_ktrans_b200.moe_layer import MoeLayer

    lay = MoeLayer.__new__(MoeLayer)
    lay.device, lay._dev_index, lay._h = torch.device("cuda", 0), 0, None
    lay.num_experts, lay.top_k, lay.hidden_size = 8, 2, 64
    return lay


def test_moe_layer_rejects_host_tensors_before_any_launch():
    lay = _stub_layer()
    x = torch.zeros(3, 64, dtype=torch.bfloat16)
    lg = torch.zeros(3, 8, dtype=torch.bfloat16)
    for call in (lambda: lay.route(lg), lambda: lay.forward(x, lg),
                 lambda: lay.experts_forward(x, torch.zeros(3, 2, dtype=torch.int64),
                                             torch.zeros(3, 2, dtype=torch.bfloat16))):
        with pytest.raises(ValueError, match="cuda"):
            call()


@pytest.mark.parametrize("which", ["ids_shape", "ids_dtype", "ids_strided", "w_shape", "w_dtype", "logits_dtype",
                                   "logits_rank", "logits_rows"])
def test_moe_layer_rejects_bad_routing_buffers(which, monkeypatch):
    """Every routing buffer a kernel writes or reads is checked for exact shape,
    dtype and contiguity (device placement is taken as given here, no GPU)."""
    from nano_ktrans_b200.moe_layer import MoeLayer

    monkeypatch.setattr(MoeLayer, "_on_device", lambda self, t: True)
    lay = _stub_layer()
    x = torch.zeros(3, 64, dtype=torch.bfloat16)
    lg = torch.zeros(3, 8, dtype=torch.bfloat16)
    ids = torch.zeros(3, 2, dtype=torch.int64)
    w = torch.zeros(3, 2, dtype=torch.bfloat16)
    bad = {"ids_shape": dict(out_ids=torch.zeros(2, 2, dtype=torch.int64)),
           "ids_dtype": dict(out_ids=torch.zeros(3, 2, dtype=torch.int32)),
           "ids_strided": dict(out_ids=torch.zeros(2, 3, dtype=torch.int64).t()),
           "w_shape": dict(out_weights=torch.zeros(3, 3, dtype=torch.bfloat16)),
           "w_dtype": dict(out_weights=torch.zeros(3, 2, dtype=torch.float32)),
           "logits_dtype": dict(logits=lg.float()),
           "logits_rank": dict(logits=lg.reshape(-1)),
           "logits_rows": dict(logits=torch.zeros(4, 8, dtype=torch.bfloat16))}[which]
    logits = bad.pop("logits", lg)
    kw = dict(out_ids=ids, out_weights=w)
    kw.update(bad)
    with pytest.raises(ValueError):
        lay.forward(x, logits, **kw)
    if "logits" not in which:
        with pytest.raises(ValueError):
            lay.route(lg, **kw)


def test_is_moe_layer_follows_reference_config_rule():
    """models/config.py:184-197: dense below first_k_dense_replace, in
    mlp_only_layers, off the decoder_sparse_step grid, or without experts."""
    from nano_ktrans_b200.dense_mlp import is_moe_layer

    assert is_moe_layer(0) and is_moe_layer(5)
    assert not is_moe_layer(0, first_k_dense_replace=1) and is_moe_layer(1, first_k_dense_replace=1)
    assert not is_moe_layer(3, mlp_only_layers=[3])
    assert [is_moe_layer(i, decoder_sparse_step=2) for i in range(4)] == [False, True, False, True]
    assert not is_moe_layer(2, num_local_experts=0) and not is_moe_layer(2, num_experts_per_tok=0)
    assert not is_moe_layer(2, attention_backend="mla")
