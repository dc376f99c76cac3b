"""GPU parity of the weight-streaming tensor-core projections (stream.cu):
against the oracle (the reference's fp32 CPU path) and against the CUDA-core
matvec kernels, on the Qwen3 decode shape at the batches the sweep reports,
on small shapes where experts get several 8-token chunks, per-channel W4, and
the Qwen2 down shape (11 groups, four K-parts)."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from tests import helpers as hp
from tests.test_parity_gpu import MAX_ABS, MEAN_REL, _full_case

pytestmark = pytest.mark.gpu


def _both_paths(d, dev):
    layer = d["layer"]
    layer.set_decode_fused(0)
    layer.set_gemm(0)
    x = hp.bf16_tensor(d["x"], dev)
    ids = torch.from_numpy(d["ids"]).to(dev)
    w = hp.bf16_tensor(d["w"], dev)
    layer.set_stream(True)
    streamed = layer.experts_forward(x, ids, w).clone()
    launches = layer.last_launch_count()
    layer.set_stream(False)
    matvec = layer.experts_forward(x, ids, w).clone()
    torch.cuda.synchronize()
    assert layer.read_status() == 0
    layer.set_stream(True)
    return streamed, matvec, launches


@pytest.mark.parametrize("tokens", [5, 8, 16, 32, 64])
def test_stream_qwen3_decode_batches(tokens, cuda_device):
    d = _full_case(hp.QWEN3, tokens, 4, 128, 300 + tokens, cuda_device)
    streamed, matvec, launches = _both_paths(d, cuda_device)
    assert launches == 4  # permute, streaming gate/up, streaming down, combine
    ref = mo.offload_forward_f32(d["x"], d["ids"], d["w"], d["experts"])
    hp.assert_parity(hp.bf16_bits(streamed), ref, MAX_ABS, MEAN_REL)
    hp.assert_paths_agree(hp.bf16_bits(streamed), hp.bf16_bits(matvec), MAX_ABS, MEAN_REL)


_SMALL = dict(experts=16, top_k=4, hidden=256, inter=256, use_softmax=True, renormalize=True)


@pytest.mark.parametrize("group", [128, 0], ids=["g128", "per_channel"])
@pytest.mark.parametrize("tokens", [40, 64])
def test_stream_multi_chunk_experts(tokens, group, cuda_device):
    """16 experts, top-4: 10-16 tokens per expert on average, so experts span
    two or more 8-token chunks, and chunks end mid-chunk."""
    d = _full_case(_SMALL, tokens, 4, group, 400 + tokens, cuda_device)
    counts = np.bincount(d["ids"].reshape(-1), minlength=_SMALL["experts"])
    assert counts.max() > 8
    streamed, matvec, _ = _both_paths(d, cuda_device)
    ref = mo.offload_forward_f32(d["x"], d["ids"], d["w"], d["experts"])
    hp.assert_parity(hp.bf16_bits(streamed), ref, MAX_ABS, MEAN_REL)
    hp.assert_paths_agree(hp.bf16_bits(streamed), hp.bf16_bits(matvec), MAX_ABS, MEAN_REL)


def test_stream_qwen2_shapes_zipf(cuda_device):
    """Qwen2-MoE expert shapes (I = 1408: the down projection's 11 groups over
    four K-parts) with Zipf(1.2) routing, whose head experts take many tokens."""
    cfg = {k: v for k, v in hp.QWEN2.items() if k != "shared_inter"}
    d = _full_case(cfg, 48, 4, 128, 501, cuda_device, zipf=1.2)
    streamed, matvec, _ = _both_paths(d, cuda_device)
    ref = mo.offload_forward_f32(d["x"], d["ids"], d["w"], d["experts"])
    hp.assert_parity(hp.bf16_bits(streamed), ref, MAX_ABS, MEAN_REL)
    hp.assert_paths_agree(hp.bf16_bits(streamed), hp.bf16_bits(matvec), MAX_ABS, MEAN_REL)


def test_stream_results_do_not_depend_on_batch_company(cuda_device):
    """A token's output is the same bits whether it shares its experts' chunks
    with other tokens or runs alone (the mma columns are independent and the
    K-part sums are added in a fixed order)."""
    d = _full_case(_SMALL, 64, 4, 128, 601, cuda_device)
    layer = d["layer"]
    layer.set_decode_fused(0)
    layer.set_gemm(0)
    x = hp.bf16_tensor(d["x"], cuda_device)
    ids = torch.from_numpy(d["ids"]).to(cuda_device)
    w = hp.bf16_tensor(d["w"], cuda_device)
    full = layer.experts_forward(x, ids, w).clone()
    for t in (0, 13, 63):
        part = layer.experts_forward(x[t:t + 5], ids[t:t + 5], w[t:t + 5]).clone()
        torch.cuda.synchronize()
        n = part.shape[0]
        assert torch.equal(part.view(torch.int16), full[t:t + n].view(torch.int16)), t
