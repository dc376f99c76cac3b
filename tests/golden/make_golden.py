"""Generate golden vectors for the routed-expert path by running nano-ktrans itself.

Run from the repository root in a container that has the nano-ktrans sources
(pass their location with ``--reference``)::

    python tests/golden/make_golden.py --reference <nano-ktrans checkout>

For every case it

1. draws seeded synthetic weights (numpy PCG64, N(0, 0.02) fp32), quantizes
   them with the reference's own ``quantize_symmetric_w4a32`` (W4) or with the
   same formula at bits=8 (W8: the reference quantizer only accepts bits=4,
   nano_ktrans/kernels/quantized_ops.py:24-25), rounds the stored scales to
   bf16, and writes a GPTQ-layout safetensors checkpoint plus
   ``quantize_config.json`` (the layout tests/test_quantized_ops.py:20-52 of the
   reference writes);
2. builds the reference ``HybridMoE`` with every expert offloaded to the
   GPTQ ``CPUMoEBackend`` (or the backend alone when a GPU-expert mask is
   given) and runs ``forward`` on seeded bf16 activations and router logits;
3. records the routing the reference passed to ``submit_forward``, its bf16
   output, and the fp32 accumulator recomputed with the reference's own
   per-expert functions in the reference's order (asserted to round to the
   very same bf16 output);
4. stores SHA-256 digests of the reference-quantized weights so the oracle's
   restated quantizer can be checked bit-exactly without committing the
   weights.

The fixtures are written to ``tests/golden/<case>.npz``.  Nothing on the GPU
box runs this script; tests only read the ``.npz`` files.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden.cases import CASES, expert_weights_f32, inputs_for_case  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def quantize_reference(w: np.ndarray, group: int, bits: int):
    """Reference quantizer for W4; the same formula restated for W8."""
    from nano_ktrans.kernels.quantized_ops import pack_int4_matrix, quantize_symmetric_w4a32

    wt = torch.from_numpy(w)
    if bits == 4:
        q = quantize_symmetric_w4a32(wt, group_size=group, bits=4)
        qweight, scales = q.qweight, q.scales
    else:
        n, k = wt.shape
        qv = torch.empty(n, k, dtype=torch.uint8)
        scales = torch.empty(n, k // group, dtype=torch.float32)
        for gi in range(k // group):
            chunk = wt[:, gi * group:(gi + 1) * group]
            scale = chunk.abs().amax(dim=1).clamp(min=1e-6) / 127
            qq = torch.round(chunk / scale.unsqueeze(1)).clamp(-128, 127)
            qv[:, gi * group:(gi + 1) * group] = (qq + 128).to(torch.uint8)
            scales[:, gi] = scale
        # 4 codes per int32 word, LSB first: pack_int4_matrix's layout at 8 bits
        words = qv.to(torch.int64).reshape(n, k // 4, 4)
        shifts = (torch.arange(4, dtype=torch.int64) * 8).view(1, 1, 4)
        packed = torch.sum(words << shifts, dim=2).numpy().astype(np.uint32).view(np.int32)
        qweight = torch.from_numpy(packed.copy())
        _ = pack_int4_matrix
    scales = scales.to(torch.bfloat16).to(torch.float32)
    return qweight.contiguous(), scales.contiguous()


def build_checkpoint(case: dict, tmpdir: str):
    experts = expert_weights_f32(case)
    tensors, digests = {}, {}
    tmpl = "model.layers.0.mlp.experts.{e}.{p}"
    for e, projs in experts.items():
        for p, w in projs.items():
            group = case["group_size"] if case["group_size"] > 0 else w.shape[1]
            qweight, scales = quantize_reference(w, group, case["bits"])
            prefix = tmpl.format(e=e, p=p + "_proj")
            tensors[prefix + ".qweight"] = qweight.t().contiguous()
            tensors[prefix + ".scales"] = scales.t().contiguous()
            digests[f"{e}.{p}.qweight"] = sha(qweight.numpy())
            digests[f"{e}.{p}.scales"] = sha(scales.numpy())
    from safetensors.torch import save_file

    save_file(tensors, os.path.join(tmpdir, "model.safetensors"))
    # per-channel: one checkpoint-wide group size covering every K, so each
    # projection has exactly one group (weight_loader.py:288-290 derives the
    # group count as ceil(K / group_size))
    group = case["group_size"] if case["group_size"] > 0 else max(case["hidden"], case["inter"])
    with open(os.path.join(tmpdir, "quantize_config.json"), "w") as f:
        json.dump({"bits": case["bits"], "group_size": group, "sym": True, "checkpoint_format": "gptq"}, f)
    return digests


def run_case(case: dict) -> dict:
    from nano_ktrans.layers.hybrid_moe import HybridMoE
    from nano_ktrans.kernels.cpu_moe import CPUMoEBackend
    from nano_ktrans.utils.context import set_context
    from nano_ktrans.kernels.quantized_ops import cpu_w4a32_matvec

    E, k, H, I = case["experts"], case["top_k"], case["hidden"], case["inter"]
    x_bits, logits_bits = inputs_for_case(case)
    x = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16)
    logits = torch.from_numpy(logits_bits.view(np.int16)).view(torch.bfloat16)
    mask = torch.zeros(E, dtype=torch.bool)
    for e in case.get("gpu_experts", []):
        mask[e] = True
    with tempfile.TemporaryDirectory() as tmpdir:
        digests = build_checkpoint(case, tmpdir)
        tmpl = "model.layers.{layer}.mlp.experts.{expert}.{proj}.weight"
        names = {"gate": "gate_proj", "up": "up_proj", "down": "down_proj"}
        set_context(is_prefill=case["tokens"] > 1)
        captured = {}
        if mask.any():
            # GPU experts present: drive the backend alone with the routing
            # computed exactly as HybridMoE.forward does (hybrid_moe.py:3321-3329).
            backend = CPUMoEBackend(layer_idx=0, num_experts=E, top_k=k, hidden_size=H, intermediate_size=I,
                                    gpu_experts_mask=mask, weight_path=tmpdir,
                                    expert_key_template=tmpl, expert_proj_names=names)
            probs = torch.softmax(logits, dim=-1, dtype=torch.float32).to(logits.dtype)
            tw, tid = torch.topk(probs, k, dim=-1)
            if case["renormalize"]:
                tw = tw / tw.sum(dim=-1, keepdim=True)
            backend.submit_forward(x, tid, tw, None)
            out = backend.sync_forward(x, None)
            captured.update(ids=tid, weights=tw)
            ref_backend = backend
        else:
            moe = HybridMoE(num_experts=E, top_k=k, hidden_size=H, moe_intermediate_size=I,
                            gpu_experts=torch.nn.ModuleDict(), gpu_experts_mask=mask, layer_idx=0,
                            weight_path=tmpdir, router_use_softmax=case["use_softmax"],
                            normalize_topk_prob=case["renormalize"], expert_key_template=tmpl,
                            expert_proj_names=names)
            ref_backend = moe.offload_backend
            orig = ref_backend.submit_forward

            def spy(hidden_states, topk_ids, topk_weights, cuda_stream):
                captured["ids"] = topk_ids.clone()
                captured["weights"] = topk_weights.clone()
                return orig(hidden_states, topk_ids, topk_weights, cuda_stream)

            ref_backend.submit_forward = spy
            out = moe(x, logits)
        assert ref_backend.is_gptq, "reference backend did not take the GPTQ path"
        # fp32 accumulator, recomputed with the reference's own per-expert
        # function in its own order (cpu_moe.py:515-536)
        ids, w = captured["ids"], captured["weights"]
        flat = x.to(torch.float32)
        acc = torch.zeros(x.shape[0], H, dtype=torch.float32)
        for e in range(E):
            if mask[e]:
                continue
            match = ids == e
            rows = torch.where(match.any(dim=1))[0]
            if len(rows) == 0:
                continue
            y = ref_backend._compute_expert_output_cpu_gptq(flat[rows], ref_backend.cpu_expert_lookup[e])
            r, c = torch.where(match[rows])
            acc.index_add_(0, rows[r], y[r] * w.to(torch.float32)[rows[r], c].unsqueeze(1))
        assert torch.equal(acc.to(torch.bfloat16), out), "fp32 recomputation does not round to the reference output"
        if case["use_softmax"]:
            ranked = torch.softmax(logits, dim=-1, dtype=torch.float32).to(logits.dtype)
        else:
            ranked = logits
        res = {
            "x": x_bits, "logits": logits_bits,
            "ids": ids.numpy().astype(np.int64), "weights": bf16_bits(w), "ranked": bf16_bits(ranked),
            "out_bf16": bf16_bits(out), "out_f32": acc.numpy(),
            "digests": np.array(json.dumps(digests, sort_keys=True)),
        }
        if case.get("shared_inter"):
            res.update(shared_reference(case, x))
        return res


def shared_reference(case: dict, x: torch.Tensor) -> dict:
    """Gated shared expert through the reference's W4 matvec (mixtral.py:215-218)."""
    from nano_ktrans.kernels.quantized_ops import cpu_w4a32_matvec
    from tests.golden.cases import shared_weights_f32
    from nano_ktrans.kernels.weight_loader import GPTQLinearWeight

    ws, gate_bits = shared_weights_f32(case)
    xs = x.to(torch.float32)
    qs, digests = {}, {}
    for p, w in ws.items():
        qweight, scales = quantize_reference(w, case["group_size"], case["bits"])
        qs[p] = GPTQLinearWeight(qweight=qweight, scales=scales, zero_points=None, group_size=case["group_size"],
                                 bits=case["bits"], sym=True, linear_prefix=f"shared.{p}")
        digests[f"shared.{p}.qweight"] = sha(qweight.numpy())
        digests[f"shared.{p}.scales"] = sha(scales.numpy())
    g = cpu_w4a32_matvec(xs, qs["gate"]).output
    u = cpu_w4a32_matvec(xs, qs["up"]).output
    y = cpu_w4a32_matvec(torch.nn.functional.silu(g) * u, qs["down"]).output
    gvec = torch.from_numpy(gate_bits.view(np.int16)).view(torch.bfloat16).to(torch.float32)
    sg = torch.sigmoid(xs @ gvec)
    return {"shared_f32": (y * sg.unsqueeze(1)).numpy(), "shared_digests": np.array(json.dumps(digests, sort_keys=True))}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="nano-ktrans source checkout")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, case in CASES.items():
        if args.only and name != args.only:
            continue
        res = run_case(case)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **res)
        print(f"{name}: T={case['tokens']} out|mean|={np.abs(res['out_f32']).mean():.4g}")


if __name__ == "__main__":
    main()
