"""GPU tests of the two callers either side of the routed-expert path:
GPU-resident experts served by the same kernels inside HybridMoE.forward (one
launch set, no host synchronisation), and a dense decoder layer's MLP run as
one always-on expert (QuantizedDenseMLP), both against the oracle."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from tests import helpers as hp
from tests.golden.load import load, oracle_experts
from tests.test_parity_gpu import MAX_ABS, MEAN_REL

pytestmark = pytest.mark.gpu


def _gptq(ql):
    from nano_ktrans_b200.weights import GPTQLinearWeight

    return GPTQLinearWeight(torch.from_numpy(ql.qweight), torch.from_numpy(ql.scales), None, ql.group_size, ql.bits,
                            True, "w")


def test_hybrid_moe_resident_experts_through_kernels(cuda_device):
    """A mixed residency mask: every routed expert, resident or offloaded, goes
    through one moe_forward launch set with no host sync, and the output is
    the oracle's over all routed experts."""
    from nano_ktrans_b200.hybrid_moe import HybridMoE

    g = load("qwen3_w4_mask")
    c = g["case"]
    trips = oracle_experts(c)
    experts = {e: {p: _gptq(ql) for p, ql in zip(("gate", "up", "down"), trip)} for e, trip in trips.items()}
    mask = torch.zeros(c["experts"], dtype=torch.bool)
    mask[c["gpu_experts"]] = True
    moe = HybridMoE(num_experts=c["experts"], top_k=c["top_k"], hidden_size=c["hidden"],
                    moe_intermediate_size=c["inter"], gpu_experts=torch.nn.ModuleDict(), gpu_experts_mask=mask,
                    layer_idx=0, weight_path="", router_use_softmax=True, normalize_topk_prob=True,
                    offload_backend_kwargs={"device": cuda_device, "max_tokens": 8, "gptq_experts": experts})
    x = hp.bf16_tensor(g["x"], cuda_device)
    lg = hp.bf16_tensor(g["logits"], cuda_device)
    moe(x, lg)
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        out = moe(x, lg)
    finally:
        torch.cuda.set_sync_debug_mode(0)
    torch.cuda.synchronize()
    ids = moe.last_topk_ids.cpu().numpy()
    assert mo.tie_aware_match(ids, g["ids"], g["ranked"]).all()
    assert np.isin(ids, c["gpu_experts"]).any(), "the case must route to a resident expert"
    ref = mo.offload_forward_f32(g["x"], ids, hp.bf16_bits(moe.last_topk_weights), trips)
    hp.assert_parity(hp.bf16_bits(out), ref, MAX_ABS, MEAN_REL)
    assert moe.offload_backend.layer.last_launch_count() <= 5
    assert moe.offload_backend.layer.read_status() == 0


@pytest.mark.parametrize("tokens", [1, 3, 8, 40, 300])
def test_quantized_dense_mlp(tokens, cuda_device):
    """A dense layer's W4 g128 MLP through the routed-expert kernels (single-token
    kernel, multi-token kernel, streaming or GEMM path by batch) against the
    oracle's expert MLP."""
    from nano_ktrans_b200.dense_mlp import QuantizedDenseMLP

    H, I = 512, 1024
    trip = hp.make_expert(900, 0, H, I, 4, 128)
    mlp = QuantizedDenseMLP(*[_gptq(ql) for ql in trip], device=cuda_device, max_tokens=512)
    rng = np.random.Generator(np.random.PCG64([900, tokens]))
    xb = mo.f32_to_bf16_bits(rng.standard_normal((tokens, H), dtype=np.float32))
    y = mlp(hp.bf16_tensor(xb, cuda_device))
    torch.cuda.synchronize()
    ref = mo.expert_forward(mo.bf16_bits_to_f32(xb), *trip)
    hp.assert_parity(hp.bf16_bits(y), ref, MAX_ABS, MEAN_REL)
    assert mlp.layer.read_status() == 0
    mlp.close()
