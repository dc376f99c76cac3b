"""Pin the CPU oracle to golden vectors recorded from nano-ktrans itself.

The fixtures under tests/golden/ were produced by running the reference's
HybridMoE.forward -> CPUMoEBackend (GPTQ) path (tests/golden/make_golden.py).
"""
import numpy as np
import pytest

from oracle import moe_oracle as mo
from tests.golden.cases import CASES
from tests.golden.load import load, oracle_experts, oracle_shared, sha

NAMES = sorted(CASES)


@pytest.mark.parametrize("name", NAMES)
def test_quantizer_bit_exact_vs_reference(name):
    g = load(name)
    experts = oracle_experts(g["case"])
    for e, trip in experts.items():
        for p, ql in zip(("gate", "up", "down"), trip):
            assert sha(ql.qweight) == g["digests"][f"{e}.{p}.qweight"], (e, p)
            assert sha(ql.scales) == g["digests"][f"{e}.{p}.scales"], (e, p)
    if "shared_digests" in g:
        trip, _ = oracle_shared(g["case"])
        for p, ql in zip(("gate", "up", "down"), trip):
            assert sha(ql.qweight) == g["shared_digests"][f"shared.{p}.qweight"]
            assert sha(ql.scales) == g["shared_digests"][f"shared.{p}.scales"]


@pytest.mark.parametrize("name", NAMES)
def test_routing_vs_reference(name):
    g = load(name)
    c = g["case"]
    ids, w, ranked = mo.route(g["logits"], c["top_k"], c["use_softmax"], c["renormalize"])
    np.testing.assert_array_equal(ranked, g["ranked"])
    assert mo.tie_aware_match(ids, g["ids"], g["ranked"]).all()
    # weights: same multiset per token (tie order may differ)
    np.testing.assert_array_equal(np.sort(w, axis=1), np.sort(g["weights"], axis=1))


@pytest.mark.parametrize("name", NAMES)
def test_expert_path_vs_reference(name):
    g = load(name)
    c = g["case"]
    experts = oracle_experts(c)
    mask = None
    if c.get("gpu_experts"):
        mask = np.ones(c["experts"], dtype=bool)
        mask[c["gpu_experts"]] = False
    out = mo.offload_forward_f32(g["x"], g["ids"], g["weights"], experts, mask)
    np.testing.assert_allclose(out, g["out_f32"], rtol=1e-5, atol=1e-6)
    bf = mo.f32_to_bf16_bits(out)
    diff = np.abs(bf.astype(np.int32) - g["out_bf16"].astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() < 0.01


def test_shared_expert_vs_reference():
    g = load("qwen2_w4_shared_t6")
    trip, gate_vec = oracle_shared(g["case"])
    out = mo.shared_expert_f32(g["x"], gate_vec, trip)
    np.testing.assert_allclose(out, g["shared_f32"], rtol=1e-5, atol=1e-6)


def test_dequantize_exhaustive_codes():
    """All 16 (W4) and 256 (W8) codes dequantize to (q - 2^(b-1)) * s exactly."""
    for bits in (4, 8):
        n = 1 << bits
        vpw = 32 // bits
        codes = np.arange(n, dtype=np.uint8)
        k = max(n, vpw * 16)
        q = np.tile(codes, k // n)[None, :].repeat(3, 0)
        words = mo.pack_words(q, bits)
        np.testing.assert_array_equal(mo.unpack_words(words, bits), q)
        scales = mo.round_bf16(np.array([[0.0123], [1.5], [3e-4]], dtype=np.float32))
        deq = mo.dequantize(words, scales, k, bits)
        exp = (q.astype(np.float32) - (1 << (bits - 1))) * scales
        np.testing.assert_array_equal(deq, exp)


def test_tie_checker_rejects_planted_error():
    g = load("qwen3_w4_t7")
    bad = g["ids"].copy()
    # swap a strictly ranked id for an unselected one in token 0
    vals = mo.bf16_bits_to_f32(g["ranked"][0])
    unselected = [e for e in range(g["case"]["experts"]) if e not in bad[0] and vals[e] < vals[bad[0, -1]]]
    bad[0, 0] = unselected[0]
    ok = mo.tie_aware_match(bad, g["ids"], g["ranked"])
    assert not ok[0] and ok[1:].all()


def test_ties_case_has_ties():
    g = load("qwen3_w4_ties")
    vals = mo.bf16_bits_to_f32(g["ranked"])
    k = g["case"]["top_k"]
    # token 0: all equal -> any k distinct ids are valid
    assert np.unique(vals[0]).size == 1
    ids, _, _ = mo.route(g["logits"], k, True, True)
    assert list(ids[0]) == list(range(k))  # documented rule: index ascending among ties
