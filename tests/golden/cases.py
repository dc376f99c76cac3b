"""Golden-vector cases: shapes, routing flavour and seeded input generators.

Shared by ``make_golden.py`` (which runs nano-ktrans on these inputs) and by
the tests (which regenerate the same inputs and compare against the stored
reference outputs).  Weights are N(0, 0.02) fp32 from numpy PCG64 and are not
stored: the fixture keeps only their SHA-256 after quantization.
"""
from __future__ import annotations

import numpy as np

# group_size 0 means per output channel (group = K)
CASES: dict[str, dict] = {
    # Qwen3-MoE flavour: softmax -> top-k -> renormalise; W4 group 128
    "qwen3_w4_t1": dict(seed=11, experts=16, top_k=4, hidden=256, inter=128, bits=4, group_size=128,
                        use_softmax=True, renormalize=True, tokens=1),
    "qwen3_w4_t7": dict(seed=12, experts=16, top_k=4, hidden=256, inter=256, bits=4, group_size=128,
                        use_softmax=True, renormalize=True, tokens=7),
    # W8 per-channel (config 1 style)
    "qwen3_w8_t3": dict(seed=13, experts=16, top_k=4, hidden=256, inter=128, bits=8, group_size=0,
                        use_softmax=True, renormalize=True, tokens=3),
    # Mixtral flavour: top-k on logits -> softmax over the k; W8 per-channel
    "mixtral_w8_t9": dict(seed=14, experts=8, top_k=2, hidden=256, inter=384, bits=8, group_size=0,
                          use_softmax=False, renormalize=True, tokens=9),
    # Qwen2-MoE flavour: softmax top-k without renormalisation, W4 g128,
    # Zipf-biased router, gated W4 shared expert
    "qwen2_w4_shared_t6": dict(seed=15, experts=12, top_k=4, hidden=256, inter=128, bits=4, group_size=128,
                               use_softmax=True, renormalize=False, tokens=6, zipf=1.2, shared_inter=256),
    # ties: rows with exactly equal logits around and inside the top-k
    "qwen3_w4_ties": dict(seed=16, experts=16, top_k=4, hidden=256, inter=128, bits=4, group_size=128,
                          use_softmax=True, renormalize=True, tokens=4, ties=True),
    # some experts GPU-resident: the backend returns only the offloaded part
    "qwen3_w4_mask": dict(seed=17, experts=16, top_k=4, hidden=256, inter=128, bits=4, group_size=128,
                          use_softmax=True, renormalize=True, tokens=5, gpu_experts=[0, 3, 5, 9]),
}


def _rng(case: dict, stream: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64([case["seed"], stream]))


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def expert_weights_f32(case: dict) -> dict:
    """{expert: {"gate"|"up"|"down": fp32 [N, K]}}, N(0, 0.02)."""
    rng = _rng(case, 1)
    H, I = case["hidden"], case["inter"]
    out = {}
    for e in range(case["experts"]):
        out[e] = {
            "gate": (rng.standard_normal((I, H), dtype=np.float32) * np.float32(0.02)),
            "up": (rng.standard_normal((I, H), dtype=np.float32) * np.float32(0.02)),
            "down": (rng.standard_normal((H, I), dtype=np.float32) * np.float32(0.02)),
        }
    return out


def shared_weights_f32(case: dict):
    rng = _rng(case, 4)
    H, S = case["hidden"], case["shared_inter"]
    ws = {
        "gate": rng.standard_normal((S, H), dtype=np.float32) * np.float32(0.02),
        "up": rng.standard_normal((S, H), dtype=np.float32) * np.float32(0.02),
        "down": rng.standard_normal((H, S), dtype=np.float32) * np.float32(0.02),
    }
    gate_vec = f32_to_bf16_bits(rng.standard_normal(H, dtype=np.float32) * np.float32(0.02))
    return ws, gate_vec


def zipf_bias(num_experts: int, alpha: float, beta: float, rng: np.random.Generator) -> np.ndarray:
    """Router bias b_e = beta * log(z_e), z ∝ rank^-alpha over a seeded expert permutation."""
    ranks = np.empty(num_experts, dtype=np.float64)
    ranks[rng.permutation(num_experts)] = np.arange(1, num_experts + 1)
    z = ranks ** (-alpha)
    z /= z.sum()
    return (beta * np.log(z)).astype(np.float32)


def inputs_for_case(case: dict):
    """(x bf16 bits [T,H], router logits bf16 bits [T,E])."""
    rng = _rng(case, 2)
    T, H, E = case["tokens"], case["hidden"], case["experts"]
    x = f32_to_bf16_bits(rng.standard_normal((T, H), dtype=np.float32))
    wr = bf16_bits_to_f32(f32_to_bf16_bits(rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.02)))
    logits = bf16_bits_to_f32(x) @ wr.T
    if case.get("zipf"):
        logits = logits + zipf_bias(E, case["zipf"], 1.0, _rng(case, 3))
    if case.get("ties"):
        # token 0: all logits equal; token 1: a tie straddling the k-th slot;
        # token 2: a tie inside the top-k; token 3 left as drawn
        k = case["top_k"]
        logits[0, :] = 0.5
        order = np.argsort(-logits[1])
        logits[1, order[k - 1]] = logits[1, order[k]]
        order = np.argsort(-logits[2])
        logits[2, order[1]] = logits[2, order[0]]
    return x, f32_to_bf16_bits(logits.astype(np.float32))
