"""moe_decode_noalloc: the decode step for callers that cannot allocate.

moe_forward() works through a handle whose workspace moe_create() obtains
with cudaMalloc.  A caller running under a memory budget fixed up front, or
one that may only use pre-registered buffers, cannot do that when it runs a
layer; moe_decode_noalloc() takes inputs and outputs directly and keeps its
scratch in a fixed device array inside the library.  These tests call it
through the C ABI and check it against moe_forward().

This file is collected last on purpose (its name sorts after the others), so a
run that stops at the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from tests import helpers as hp

MAX_ABS, MEAN_REL = 2e-2, 5e-3  # the parity bar used by every output test


def _desc_and_weights(layer):
    from nano_ktrans_b200 import _lib

    w = layer.weights
    desc = _lib.MoeLayerDesc(layer.num_experts, layer.top_k, layer.hidden_size, layer.inter_size, w.bits,
                             w.group_size, int(layer.router_use_softmax), int(layer.normalize_topk_prob),
                             layer.max_tokens, 0)
    ptrs = _lib.MoeWeights(w.gate_q.data_ptr(), w.gate_s.data_ptr(), w.up_q.data_ptr(), w.up_s.data_ptr(),
                           w.down_q.data_ptr(), w.down_s.data_ptr(), None, None, None, None, None, None, None)
    return desc, ptrs


def _noalloc(desc, ptrs, x, logits, status=None):
    from nano_ktrans_b200 import _lib

    t = x.shape[0]
    out = torch.empty_like(x)
    ids = torch.empty(t, desc.top_k, dtype=torch.int64, device=x.device)
    wts = torch.empty(t, desc.top_k, dtype=torch.bfloat16, device=x.device)
    err = ctypes.create_string_buffer(512)
    rc = _lib.lib().moe_decode_noalloc(ctypes.byref(desc), ctypes.byref(ptrs), x.data_ptr(), logits.data_ptr(), t,
                                       out.data_ptr(), ids.data_ptr(), wts.data_ptr(),
                                       None if status is None else status.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream, err, len(err))
    return rc, err.value.decode(), out, ids, wts


@pytest.mark.gpu
def test_noalloc_matches_moe_forward_on_two_calls_in_a_row(cuda_device):
    from nano_ktrans_b200 import _lib
    from nano_ktrans_b200.moe_layer import MoeLayer

    cfg = hp.QWEN3
    seed = 41
    xa, la = hp.make_inputs(seed, 3, cfg["hidden"], cfg["experts"])
    xb, lb = hp.make_inputs(seed + 1, 1, cfg["hidden"], cfg["experts"])
    routed = set()
    for lg in (la, lb):
        ids, _, _ = mo.route(lg, cfg["top_k"], True, True)
        routed |= set(ids.reshape(-1).tolist())
    experts = {e: hp.make_expert(seed, e, cfg["hidden"], cfg["inter"], 4, 128) for e in sorted(routed)}
    lw = hp.device_layer(experts, cfg["experts"], cfg["hidden"], cfg["inter"], 4, 128, cuda_device)
    layer = MoeLayer(lw, top_k=cfg["top_k"], router_use_softmax=True, normalize_topk_prob=True, max_tokens=8)
    desc, ptrs = _desc_and_weights(layer)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)

    # two calls in a row, different batches: the second reuses the scratch the first left behind
    for x_bits, l_bits in ((xa, la), (xb, lb)):
        x = hp.bf16_tensor(x_bits, cuda_device)
        lg = hp.bf16_tensor(l_bits, cuda_device)
        ids_ref = torch.empty(x.shape[0], cfg["top_k"], dtype=torch.int64, device=cuda_device)
        w_ref = torch.empty(x.shape[0], cfg["top_k"], dtype=torch.bfloat16, device=cuda_device)
        ref = layer.forward(x, lg, out_ids=ids_ref, out_weights=w_ref)
        rc, msg, out, ids, wts = _noalloc(desc, ptrs, x, lg, status)
        torch.cuda.synchronize()
        assert rc == _lib.MOE_OK, msg
        assert torch.equal(ids, ids_ref) and torch.equal(wts, w_ref)
        hp.assert_parity(hp.bf16_bits(out), mo.bf16_bits_to_f32(hp.bf16_bits(ref)), MAX_ABS, MEAN_REL)
        # and against the CPU oracle of the reference's path
        hp.assert_parity(hp.bf16_bits(out), mo.offload_forward_f32(x_bits, ids.cpu().numpy(), hp.bf16_bits(wts),
                                                                  experts), MAX_ABS, MEAN_REL)
    assert int(status.item()) == 0


@pytest.mark.gpu
def test_noalloc_rejects_batches_beyond_its_scratch(cuda_device):
    from nano_ktrans_b200 import _lib
    from nano_ktrans_b200.moe_layer import MoeLayer

    cfg = hp.QWEN3
    lw = hp.device_layer({}, cfg["experts"], cfg["hidden"], cfg["inter"], 4, 128, cuda_device)
    layer = MoeLayer(lw, top_k=cfg["top_k"], max_tokens=64)
    desc, ptrs = _desc_and_weights(layer)
    x = torch.zeros(16, cfg["hidden"], dtype=torch.bfloat16, device=cuda_device)
    lg = torch.zeros(16, cfg["experts"], dtype=torch.bfloat16, device=cuda_device)
    rc, msg, *_ = _noalloc(desc, ptrs, x, lg)
    assert rc == _lib.MOE_ERANGE
    assert "scratch" in msg or "limits" in msg
