"""CPU oracle for the HybridMoE routed-expert path (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The shipped path (``nano_ktrans_b200``) never calls into it and has no CPU
fallback.

It restates, in numpy, the arithmetic of nano-ktrans's own CPU path for this
layer.  Every function cites the reference file:line it follows (paths are
relative to the nano-ktrans project root):

* routing ............ nano_ktrans/layers/hybrid_moe.py:3321-3329
* quantizer .......... nano_ktrans/kernels/quantized_ops.py:17-59 (W4), and the
                       same formula with bits=8, group=K (the reference
                       quantizer rejects bits!=4 at :24-25; its container and
                       matvec are bit-width generic, weight_loader.py:48,51-69)
* packer ............. nano_ktrans/kernels/quantized_ops.py:62-72
* unpack/dequantize .. nano_ktrans/kernels/weight_loader.py:51-69
* grouped matvec ..... nano_ktrans/kernels/quantized_ops.py:86-124
* expert MLP ......... nano_ktrans/kernels/cpu_moe.py:419-450
* offload combine .... nano_ktrans/kernels/cpu_moe.py:491-539
* shared expert ...... nano_ktrans/models/mixtral.py:170-179, 215-218

Parity of this restatement is pinned by ``tests/test_oracle_golden.py`` against
golden vectors produced by running the reference itself
(``tests/golden/make_golden.py`` drives the reference ``HybridMoE.forward`` ->
``CPUMoEBackend`` GPTQ path live and records its outputs).

Scale convention for bf16 scales: scales and codes are
computed in fp32 exactly as the reference quantizer does, then the stored
scales are rounded to bf16; every consumer dequantizes with the bf16-valued
scale, which makes ``(q - z) * s`` exact in fp32.
"""
from __future__ import annotations

import numpy as np

# --------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, as torch's float->bfloat16 cast)
# --------------------------------------------------------------------------


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit pattern (uint16), round to nearest even, NaN kept quiet."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r = r.copy()
        r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(a: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bf16 value (returned as fp32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(a))


# --------------------------------------------------------------------------
# Quantized-weight container arithmetic
# --------------------------------------------------------------------------


def quantize_symmetric(weight: np.ndarray, group_size: int, bits: int):
    """Symmetric per-group quantizer.

    Follows nano_ktrans/kernels/quantized_ops.py:17-59 step by step (fp32
    ``max|w_g| clamp(min=1e-6) / (2^(b-1)-1)``, ``round`` half-to-even,
    ``clamp(-2^(b-1), 2^(b-1)-1) + 2^(b-1)``); bits=8 uses the same formula.
    Returns (qvalues uint8 [N,K], scales fp32 [N,G]) with fp32 scales.
    """
    w = np.ascontiguousarray(weight, dtype=np.float32)
    n, k = w.shape
    if k % group_size:
        raise ValueError("input_dim must be divisible by group_size")
    qmax = np.float32((1 << (bits - 1)) - 1)
    zero = 1 << (bits - 1)
    g = k // group_size
    chunks = w.reshape(n, g, group_size)
    max_abs = np.maximum(np.abs(chunks).max(axis=2), np.float32(1e-6)).astype(np.float32)
    scales = (max_abs / qmax).astype(np.float32)
    q = np.round(chunks / scales[:, :, None]).astype(np.float32)
    q = np.clip(q, -(1 << (bits - 1)), (1 << (bits - 1)) - 1)
    qvalues = (q + zero).astype(np.uint8).reshape(n, k)
    return qvalues, scales


def pack_words(qvalues: np.ndarray, bits: int) -> np.ndarray:
    """Pack codes LSB-first along K into int32 words.

    nano_ktrans/kernels/quantized_ops.py:62-72 for bits=4 (8 codes per word,
    code j at bits 4j); bits=8 packs 4 codes per word at bits 8j.  The result
    is the reference's ``GPTQLinearWeight.qweight`` layout [N, K*bits/32].
    """
    n, k = qvalues.shape
    vpw = 32 // bits
    if k % vpw:
        raise ValueError("input_dim must be divisible by values-per-word")
    q = qvalues.astype(np.uint32).reshape(n, k // vpw, vpw)
    shifts = (np.arange(vpw, dtype=np.uint32) * bits)[None, None, :]
    words = np.bitwise_or.reduce(q << shifts, axis=2).astype(np.uint32)
    return words.view(np.int32)


def unpack_words(qweight: np.ndarray, bits: int) -> np.ndarray:
    """weight_loader.py:51-55 / quantized_ops.py:75-83: words -> codes [N, K]."""
    w = np.ascontiguousarray(qweight).view(np.uint32)
    vpw = 32 // bits
    shifts = (np.arange(vpw, dtype=np.uint32) * bits)[None, None, :]
    vals = (w[:, :, None] >> shifts) & np.uint32((1 << bits) - 1)
    return vals.reshape(w.shape[0], w.shape[1] * vpw).astype(np.uint8)


def dequantize(qweight: np.ndarray, scales: np.ndarray, group_size: int, bits: int) -> np.ndarray:
    """weight_loader.py:57-69: ``(q - 2^(b-1)) * scale[:, g]`` in fp32."""
    q = unpack_words(qweight, bits).astype(np.float32)
    n, k = q.shape
    zero = np.float32(1 << (bits - 1))
    out = np.empty((n, k), dtype=np.float32)
    for gi in range(scales.shape[1]):
        s, e = gi * group_size, min((gi + 1) * group_size, k)
        out[:, s:e] = (q[:, s:e] - zero) * scales[:, gi:gi + 1].astype(np.float32)
    return out


def matvec_grouped(x: np.ndarray, qweight: np.ndarray, scales: np.ndarray, group_size: int, bits: int) -> np.ndarray:
    """quantized_ops.py:86-124 ``cpu_w4a32_matvec_grouped``.

    Per K-group, in group order: unpack the group's words, dequantize with the
    group's scale, and accumulate ``x_g @ W_g^T`` into an fp32 output.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    vpw = 32 // bits
    n = qweight.shape[0]
    k = qweight.shape[1] * vpw
    if x.shape[1] != k:
        raise ValueError(f"input dim mismatch: {x.shape} vs K={k}")
    zero = np.float32(1 << (bits - 1))
    out = np.zeros((x.shape[0], n), dtype=np.float32)
    for gi in range(scales.shape[1]):
        s = gi * group_size
        e = min(s + group_size, k)
        sw, ew = s // vpw, (e + vpw - 1) // vpw
        q = unpack_words(qweight[:, sw:ew], bits).astype(np.float32)
        off = s - sw * vpw
        q = q[:, off:off + (e - s)]
        deq = (q - zero) * scales[:, gi:gi + 1].astype(np.float32)
        out += x[:, s:e] @ deq.T
    return out


def silu(v: np.ndarray) -> np.ndarray:
    v = v.astype(np.float32)
    return (v / (np.float32(1.0) + np.exp(-v))).astype(np.float32)


class QuantLinear:
    """The fields of ``GPTQLinearWeight`` (weight_loader.py:25-69) the path reads."""

    def __init__(self, qweight: np.ndarray, scales: np.ndarray, group_size: int, bits: int):
        self.qweight = np.ascontiguousarray(qweight, dtype=np.int32)
        self.scales = np.ascontiguousarray(scales, dtype=np.float32)
        self.group_size = int(group_size)
        self.bits = int(bits)

    @property
    def output_dim(self) -> int:
        return self.qweight.shape[0]

    @property
    def input_dim(self) -> int:
        return self.qweight.shape[1] * (32 // self.bits)

    def matvec(self, x: np.ndarray) -> np.ndarray:
        return matvec_grouped(x, self.qweight, self.scales, self.group_size, self.bits)

    def dequantize(self) -> np.ndarray:
        return dequantize(self.qweight, self.scales, self.group_size, self.bits)


def make_quant_linear(weight: np.ndarray, group_size: int, bits: int) -> QuantLinear:
    """Quantize (reference formula), pack, and round the stored scales to bf16."""
    q, s = quantize_symmetric(weight, group_size, bits)
    return QuantLinear(pack_words(q, bits), round_bf16(s), group_size, bits)


# --------------------------------------------------------------------------
# Expert MLP, offload combine, shared expert
# --------------------------------------------------------------------------


def expert_forward(x: np.ndarray, gate: QuantLinear, up: QuantLinear, down: QuantLinear) -> np.ndarray:
    """cpu_moe.py:419-450: ``down(silu(gate(x)) * up(x))``, fp32 throughout."""
    g = gate.matvec(x)
    u = up.matvec(x)
    h = (silu(g) * u).astype(np.float32)
    return down.matvec(h)


def offload_forward_f32(x_bf16: np.ndarray, topk_ids: np.ndarray, topk_w_bf16: np.ndarray,
                        experts: dict, offload_mask: np.ndarray | None = None) -> np.ndarray:
    """cpu_moe.py:491-539, GPTQ branch, returning the fp32 accumulator.

    ``x_bf16``/``topk_w_bf16`` are uint16 bf16 bit patterns.  Experts are
    visited in ascending index (:515); each contributes
    ``index_add_(tok, y * w)`` in fp32 (:528-536).  ``experts[e]`` is a
    (gate, up, down) tuple of QuantLinear; ``offload_mask[e]`` False skips
    expert e (it is GPU-resident and not the backend's job).
    """
    x = bf16_bits_to_f32(x_bf16)
    w = bf16_bits_to_f32(topk_w_bf16)
    t, h = x.shape
    out = np.zeros((t, h), dtype=np.float32)
    # experts may hold only the routed subset; scan every id that can occur
    num_experts = max(max(experts) + 1, int(topk_ids.max()) + 1 if topk_ids.size else 0)
    for e in range(num_experts):
        if offload_mask is not None and not offload_mask[e]:
            continue
        match = topk_ids == e
        rows = np.nonzero(match.any(axis=1))[0]
        if rows.size == 0:
            continue
        if e not in experts:
            raise KeyError(f"expert {e} is routed but its weights were not provided")
        y = expert_forward(x[rows], *experts[e])
        r_idx, c_idx = np.nonzero(match[rows])
        wt = w[rows[r_idx], c_idx][:, None]
        np.add.at(out, rows[r_idx], y[r_idx] * wt)
    return out


def offload_forward(x_bf16, topk_ids, topk_w_bf16, experts, offload_mask=None) -> np.ndarray:
    """Same as :func:`offload_forward_f32` with the final bf16 cast (:538)."""
    return f32_to_bf16_bits(offload_forward_f32(x_bf16, topk_ids, topk_w_bf16, experts, offload_mask))


def shared_expert_f32(x_bf16: np.ndarray, gate_proj: np.ndarray, shared: tuple) -> np.ndarray:
    """models/mixtral.py:215-218 with a W4 shared expert.

    ``sigmoid(x @ g_s) * SparseExpertMLP_s(x)``; the reference's shared expert
    is dense bf16, the configs quantize it W4 group-128, so the oracle runs it
    through the grouped matvec (cpu_moe.py:419-450 arithmetic).  The gate
    logit is computed in fp32 from bf16 ``x`` and bf16 ``gate_proj`` [H].
    """
    x = bf16_bits_to_f32(x_bf16)
    g = bf16_bits_to_f32(gate_proj).reshape(-1)
    logit = x @ g
    gate = (np.float32(1.0) / (np.float32(1.0) + np.exp(-logit.astype(np.float32)))).astype(np.float32)
    return expert_forward(x, *shared) * gate[:, None]


# --------------------------------------------------------------------------
# Routing
# --------------------------------------------------------------------------


def softmax_f32(v: np.ndarray) -> np.ndarray:
    v = v.astype(np.float32)
    m = v.max(axis=-1, keepdims=True)
    e = np.exp(v - m).astype(np.float32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def topk_stable(values: np.ndarray, k: int):
    """Top-k by (value desc, index asc) — the kernel's documented tie rule."""
    order = np.lexsort((np.arange(values.shape[-1])[None, :].repeat(values.shape[0], 0), -values), axis=-1)
    ids = order[:, :k]
    return np.take_along_axis(values, ids, axis=1), ids.astype(np.int64)


def route(logits_bf16: np.ndarray, top_k: int, use_softmax: bool, renormalize: bool):
    """hybrid_moe.py:3321-3329.

    Qwen (``use_softmax``): ``p = bf16(softmax_fp32(logits))``; ``topk(p)``;
    if ``renormalize``: ``w = bf16(w / bf16(sum w))``.
    Mixtral: ``topk(logits)``; ``w = bf16(softmax_fp32(w))``.
    Returns (ids int64 [T,k], weights bf16 bits [T,k], probs bf16 bits [T,E])
    where ``probs`` are the values top-k ranked.  Ties follow (value desc,
    index asc); the reference's ``torch.topk`` leaves tie order unspecified,
    which ``tie_aware_match`` accounts for.
    """
    logits = bf16_bits_to_f32(logits_bf16)
    if use_softmax:
        probs = round_bf16(softmax_f32(logits))
        vals, ids = topk_stable(probs, top_k)
        if renormalize:
            s = round_bf16(vals.sum(axis=-1, keepdims=True, dtype=np.float32))
            vals = round_bf16((vals / s).astype(np.float32))
        return ids, f32_to_bf16_bits(vals), f32_to_bf16_bits(probs)
    vals, ids = topk_stable(logits, top_k)
    w = round_bf16(softmax_f32(vals))
    return ids, f32_to_bf16_bits(w), f32_to_bf16_bits(logits)


def tie_aware_match(ids_a: np.ndarray, ids_b: np.ndarray, ranked_bf16: np.ndarray) -> np.ndarray:
    """Per token: True when ``ids_a`` is a valid top-k ordering equal to ``ids_b``
    up to permutations among equal ranked values.

    ``ranked_bf16`` are the values the reference ranks (bf16 probabilities for
    softmax routing, bf16 logits for Mixtral).  Positions whose values are
    strictly ordered must hold the same id; within a run of equal values the
    ids may be permuted, and at the k-th boundary any id of equal value is
    accepted.
    """
    vals = bf16_bits_to_f32(ranked_bf16)
    t = ids_a.shape[0]
    ok = np.ones(t, dtype=bool)
    for i in range(t):
        va = vals[i, ids_a[i]]
        vb = vals[i, ids_b[i]]
        if len(set(ids_a[i].tolist())) != ids_a.shape[1]:
            ok[i] = False
            continue
        if not np.array_equal(va, vb) or np.any(np.diff(va) > 0):
            ok[i] = False
            continue
        kth = va[-1]
        # every unselected expert must not beat the k-th value
        sel = np.zeros(vals.shape[1], dtype=bool)
        sel[ids_a[i]] = True
        if np.any(vals[i, ~sel] > kth):
            ok[i] = False
            continue
        # strictly ordered positions must agree exactly
        for j in range(ids_a.shape[1]):
            v = va[j]
            if np.count_nonzero(vals[i] == v) == 1 and ids_a[i, j] != ids_b[i, j]:
                ok[i] = False
                break
    return ok


# --------------------------------------------------------------------------
# Whole layer (routing + offload path + optional shared expert)
# --------------------------------------------------------------------------


def moe_layer_f32(x_bf16, logits_bf16, experts, top_k, use_softmax, renormalize,
                  shared=None, shared_gate=None, offload_mask=None) -> dict:
    """HybridMoE.forward with every expert offloaded (hybrid_moe.py:3310-3570),
    plus the decoder layer's shared-expert add (mixtral.py:212-218).

    Returns a dict with ``out`` (fp32 [T,H], routed + gated shared part, no
    intermediate bf16 rounding: the "fp32-accumulated path" the parity bar is
    stated against), ``routed`` (fp32), ``ids``, ``weights`` (bf16 bits) and
    ``ranked`` (bf16 bits of the values top-k ranks).
    """
    ids, w, ranked = route(logits_bf16, top_k, use_softmax, renormalize)
    routed = offload_forward_f32(x_bf16, ids, w, experts, offload_mask)
    out = routed
    if shared is not None:
        out = routed + shared_expert_f32(x_bf16, shared_gate, shared)
    return {"out": out.astype(np.float32), "routed": routed, "ids": ids, "weights": w, "ranked": ranked}
