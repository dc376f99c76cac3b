"""GPU parity of the router projection (moe_router_logits / moe_forward_x)
against the reference's bf16 nn.Linear gate (nano_ktrans/models/mixtral.py:127,
:212), run here as torch's bf16 F.linear on the same device: logits within one
bf16 unit in the last place, routing tie-aware equal to routing on the
kernel's own logits, and any token whose ids differ from routing on the
nn.Linear logits sits on a near-tie (its boundary values within one ulp)."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from tests import helpers as hp
from tests.test_parity_gpu import MAX_ABS, MEAN_REL

pytestmark = pytest.mark.gpu


def _ulp_bf16(v: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 values at |v| (fp32)."""
    a = v.abs().float().clamp_min(1e-30)
    return torch.exp2(torch.floor(torch.log2(a)) - 7)


def _layer(cfg, dev, tokens, seed):
    experts = {e: hp.make_expert(seed, e, cfg["hidden"], cfg["inter"], 4, 128) for e in range(cfg["experts"])}
    lw = hp.device_layer(experts, cfg["experts"], cfg["hidden"], cfg["inter"], 4, 128, dev)
    from nano_ktrans_b200.moe_layer import MoeLayer

    layer = MoeLayer(lw, top_k=cfg["top_k"], router_use_softmax=cfg["use_softmax"],
                     normalize_topk_prob=cfg["renormalize"], max_tokens=tokens)
    return layer, experts


@pytest.mark.parametrize("cfg_name,tokens", [("QWEN3", 1), ("QWEN3", 8), ("QWEN3", 64), ("MIXTRAL", 37)])
def test_router_logits_match_nn_linear(cfg_name, tokens, cuda_device):
    cfg = getattr(hp, cfg_name)
    g = torch.Generator(device=cuda_device).manual_seed(tokens)
    x = torch.randn(tokens, cfg["hidden"], generator=g, device=cuda_device).to(torch.bfloat16)
    wr = (torch.randn(cfg["experts"], cfg["hidden"], generator=g, device=cuda_device) * 0.02).to(torch.bfloat16)
    ref = torch.nn.functional.linear(x, wr)  # the reference gate: bf16 nn.Linear without bias
    from nano_ktrans_b200.moe_layer import MoeLayer
    from nano_ktrans_b200.weights import LayerWeights

    E, H, I = cfg["experts"], cfg["hidden"], 128
    z8 = lambda *s: torch.zeros(*s, dtype=torch.uint8, device=cuda_device)  # noqa: E731
    zs = lambda *s: torch.zeros(*s, dtype=torch.bfloat16, device=cuda_device)  # noqa: E731
    lw = LayerWeights(bits=4, group_size=128, gate_q=z8(E, I, H // 2), gate_s=zs(E, I, 16),
                      up_q=z8(E, I, H // 2), up_s=zs(E, I, 16), down_q=z8(E, H, I // 2), down_s=zs(E, H, 8))
    layer = MoeLayer(lw, top_k=cfg["top_k"], router_use_softmax=cfg["use_softmax"],
                     normalize_topk_prob=cfg["renormalize"], max_tokens=tokens)
    mine = layer.router_logits(x, wr)
    torch.cuda.synchronize()
    diff = (mine.float() - ref.float()).abs()
    assert (diff <= _ulp_bf16(ref.float()) * 1.0001).all(), float(diff.max())
    # routing: the in-block ids equal routing on the kernel's logits; against the
    # nn.Linear logits they agree except at near-ties
    ids_k, _ = layer.route(mine)
    ids_r, _ = layer.route(ref)
    torch.cuda.synchronize()
    ids_o, _, ranked = mo.route(hp.bf16_bits(mine), cfg["top_k"], cfg["use_softmax"], cfg["renormalize"])
    assert mo.tie_aware_match(ids_k.cpu().numpy(), ids_o, ranked).all()
    differ = (np.sort(ids_k.cpu().numpy(), 1) != np.sort(ids_r.cpu().numpy(), 1)).any(1)
    for t in np.nonzero(differ)[0]:
        a = set(ids_k[t].tolist()) ^ set(ids_r[t].tolist())
        vals = ref[t, list(a)].float()
        assert (vals.max() - vals.min()) <= 2 * _ulp_bf16(vals.abs().max()), (t, a)
    layer.close()


@pytest.mark.parametrize("tokens", [1, 8])
def test_forward_x_matches_oracle(tokens, cuda_device):
    """moe_forward_x (router projection + routing + experts + combine) against
    the oracle on the kernel's own logits and ids; the launch count includes
    the router kernel."""
    cfg = dict(experts=16, top_k=4, hidden=256, inter=256, use_softmax=True, renormalize=True)
    layer, experts = _layer(cfg, cuda_device, tokens, 700 + tokens)
    g = torch.Generator(device=cuda_device).manual_seed(tokens)
    x = torch.randn(tokens, cfg["hidden"], generator=g, device=cuda_device).to(torch.bfloat16)
    wr = (torch.randn(cfg["experts"], cfg["hidden"], generator=g, device=cuda_device) * 0.02).to(torch.bfloat16)
    ids = torch.empty(tokens, 4, dtype=torch.int64, device=cuda_device)
    w = torch.empty(tokens, 4, dtype=torch.bfloat16, device=cuda_device)
    lg = torch.empty(tokens, 16, dtype=torch.bfloat16, device=cuda_device)
    out = layer.forward_x(x, wr, out_ids=ids, out_weights=w, out_logits=lg)
    torch.cuda.synchronize()
    assert layer.last_launch_count() >= 2
    assert torch.equal(lg, layer.router_logits(x, wr))
    ref = mo.offload_forward_f32(hp.bf16_bits(x), ids.cpu().numpy(), hp.bf16_bits(w), experts)
    hp.assert_parity(hp.bf16_bits(out), ref, MAX_ABS, MEAN_REL)
    assert layer.read_status() == 0
    layer.close()


@pytest.mark.parametrize("host_io", [0, 1, 2])
def test_forward_host_matches_forward(host_io, cuda_device):
    """moe_forward_host (host buffers in and out) gives the bits of forward(), for
    copy-engine transfers, kernel reads of mapped host memory (and direct stores
    of the output), pinned and pageable buffers, on the single-token kernel and
    the multi-kernel path."""
    cfg = dict(experts=16, top_k=4, hidden=256, inter=256, use_softmax=True, renormalize=True)
    for tokens in (1, 6):
        layer, _ = _layer(cfg, cuda_device, tokens, 800 + tokens)
        layer.set_host_io(host_io)
        g = torch.Generator(device=cuda_device).manual_seed(tokens)
        x = torch.randn(tokens, 256, generator=g, device=cuda_device).to(torch.bfloat16)
        lg = (torch.randn(tokens, 16, generator=g, device=cuda_device)).to(torch.bfloat16)
        want = layer.forward(x, lg).cpu()
        for pinned in (True, False):
            xh, lh = x.cpu(), lg.cpu()
            oh = torch.empty_like(xh)
            if pinned:
                xh, lh, oh = xh.pin_memory(), lh.pin_memory(), oh.pin_memory()
            layer.forward_host(xh, lh, oh)
            torch.cuda.synchronize()
            assert torch.equal(oh.view(torch.int16), want.view(torch.int16)), (tokens, pinned)
        assert layer.read_status() == 0
        layer.close()
