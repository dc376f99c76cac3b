"""Shared test helpers: synthetic layers built with the oracle's quantizer."""
from __future__ import annotations

import numpy as np

from oracle import moe_oracle as mo

# BASELINE configurations (shapes only; the tests choose token counts)
QWEN3 = dict(experts=128, top_k=8, hidden=2048, inter=768, use_softmax=True, renormalize=True)
MIXTRAL = dict(experts=8, top_k=2, hidden=4096, inter=14336, use_softmax=False, renormalize=True)
QWEN2 = dict(experts=60, top_k=4, hidden=2048, inter=1408, use_softmax=True, renormalize=False, shared_inter=5632)


def expert_rng(seed: int, e: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64([seed, 1000 + e]))


def make_expert(seed: int, e: int, hidden: int, inter: int, bits: int, group: int):
    """(gate, up, down) QuantLinear from N(0, 0.02) weights (group 0 = per-channel)."""
    rng = expert_rng(seed, e)
    trip = []
    for n, k in ((inter, hidden), (inter, hidden), (hidden, inter)):
        w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
        trip.append(mo.make_quant_linear(w, group if group > 0 else k, bits))
    return tuple(trip)


def make_inputs(seed: int, tokens: int, hidden: int, experts: int, zipf: float | None = None):
    rng = np.random.Generator(np.random.PCG64([seed, 7]))
    x = mo.f32_to_bf16_bits(rng.standard_normal((tokens, hidden), dtype=np.float32))
    wr = mo.round_bf16(rng.standard_normal((experts, hidden), dtype=np.float32) * np.float32(0.02))
    logits = mo.bf16_bits_to_f32(x) @ wr.T
    if zipf:
        from tests.golden.cases import zipf_bias

        logits = logits + zipf_bias(experts, zipf, 1.0, np.random.Generator(np.random.PCG64([seed, 8])))
    return x, mo.f32_to_bf16_bits(logits.astype(np.float32))


def device_layer(experts: dict, num_experts: int, hidden: int, inter: int, bits: int, group: int, device,
                 shared=None, shared_gate_vec=None):
    """LayerWeights with the given experts' codes/scales; absent experts are zero."""
    import torch

    from nano_ktrans_b200.weights import LayerWeights

    g_h = hidden // (group if group > 0 else hidden)
    g_i = inter // (group if group > 0 else inter)

    def alloc(n, k, g):
        return (np.zeros((num_experts, n, k * bits // 8), dtype=np.uint8),
                np.zeros((num_experts, n, (g + 7) // 8 * 8), dtype=np.float32))

    gq, gs = alloc(inter, hidden, g_h)
    uq, us = alloc(inter, hidden, g_h)
    dq, ds = alloc(hidden, inter, g_i)
    for e, (g, u, d) in experts.items():
        gq[e], gs[e, :, :g_h] = g.qweight.view(np.uint8), g.scales
        uq[e], us[e, :, :g_h] = u.qweight.view(np.uint8), u.scales
        dq[e], ds[e, :, :g_i] = d.qweight.view(np.uint8), d.scales

    def tq(a):
        return torch.from_numpy(a).to(device)

    def ts(a):
        return torch.from_numpy(a).to(torch.bfloat16).to(device)

    sh = None
    if shared is not None:
        sh = {}
        for p, ql in zip(("gate", "up", "down"), shared):
            sh[p + "_q"] = tq(ql.qweight.view(np.uint8)[None].copy())
            g = ql.scales.shape[1]
            padded = np.zeros((1, ql.scales.shape[0], (g + 7) // 8 * 8), dtype=np.float32)
            padded[0, :, :g] = ql.scales
            sh[p + "_s"] = ts(padded)
        sh["gate_vec"] = torch.from_numpy(shared_gate_vec.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return LayerWeights(bits=bits, group_size=group, gate_q=tq(gq), gate_s=ts(gs), up_q=tq(uq), up_s=ts(us),
                        down_q=tq(dq), down_s=ts(ds), shared=sh)


def bf16_tensor(bits: np.ndarray, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).view(torch.bfloat16).to(device)


def bf16_bits(t) -> np.ndarray:
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def assert_parity(out_bf16_bits: np.ndarray, ref_f32: np.ndarray, max_abs: float = 2e-2, mean_rel: float = 5e-3):
    """The north-star bar: bf16 output vs the reference fp32-accumulated path."""
    got = mo.bf16_bits_to_f32(out_bf16_bits).astype(np.float64)
    ref = ref_f32.astype(np.float64)
    err = np.abs(got - ref)
    denom = np.abs(ref).mean() + 1e-30
    assert err.max() <= max_abs, f"max-abs {err.max():.3e} > {max_abs}"
    assert err.mean() / denom <= mean_rel, f"mean-rel {err.mean() / denom:.3e} > {mean_rel}"
    return float(err.max()), float(err.mean() / denom)


def assert_paths_agree(a_bf16_bits: np.ndarray, b_bf16_bits: np.ndarray, max_abs: float = 2e-2,
                       mean_rel: float = 5e-3):
    """Two device paths, each rounded to bf16 once, agree: |a - b| within the
    absolute bar plus one bf16 unit in the last place of b (each output may sit
    half a unit from the common fp32 value; 1 ulp <= |b| * 2^-7), and the
    mean-relative bar as in assert_parity."""
    a = mo.bf16_bits_to_f32(a_bf16_bits).astype(np.float64)
    b = mo.bf16_bits_to_f32(b_bf16_bits).astype(np.float64)
    err = np.abs(a - b)
    bound = max_abs + np.abs(b) * 2.0 ** -7
    worst = int(np.argmax(err - bound))
    assert (err <= bound).all(), f"|a-b| {err.flat[worst]:.3e} > {bound.flat[worst]:.3e} at |b| {abs(b.flat[worst]):.3e}"
    denom = np.abs(b).mean() + 1e-30
    assert err.mean() / denom <= mean_rel, f"mean-rel {err.mean() / denom:.3e} > {mean_rel}"
