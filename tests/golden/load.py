"""Load a golden case and rebuild its quantized weights with the oracle."""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np

from oracle import moe_oracle as mo
from tests.golden.cases import CASES, expert_weights_f32, shared_weights_f32

HERE = os.path.dirname(os.path.abspath(__file__))


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load(name: str) -> dict:
    with np.load(os.path.join(HERE, f"{name}.npz")) as z:
        d = {k: z[k] for k in z.files}
    d["digests"] = json.loads(str(d["digests"]))
    if "shared_digests" in d:
        d["shared_digests"] = json.loads(str(d["shared_digests"]))
    d["case"] = CASES[name]
    return d


def oracle_experts(case: dict) -> dict:
    """{e: (gate, up, down)} QuantLinear built with the oracle's quantizer."""
    out = {}
    for e, projs in expert_weights_f32(case).items():
        trip = []
        for p in ("gate", "up", "down"):
            w = projs[p]
            g = case["group_size"] if case["group_size"] > 0 else w.shape[1]
            trip.append(mo.make_quant_linear(w, g, case["bits"]))
        out[e] = tuple(trip)
    return out


def oracle_shared(case: dict):
    ws, gate_vec = shared_weights_f32(case)
    trip = tuple(mo.make_quant_linear(ws[p], case["group_size"], case["bits"]) for p in ("gate", "up", "down"))
    return trip, gate_vec
