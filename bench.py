#!/usr/bin/env python
"""Routed-expert MoE layer benchmark on B200.

Workload (the one the metric is quoted on): a
Qwen3-30B-A3B-shaped MoE layer — hidden 2048, 128 experts, moe_intermediate
768, top-8 renormalised softmax routing, W4 symmetric group-128 weights with
bf16 scales — in decode at batch 1.  One *step* is one pass of the hot path
(router top-k -> permutation -> W4 gate/up + SiLU*up -> W4 down -> weighted
combine) over one batch of tokens through one layer.  Steps cycle through a
stack of 48 distinct layers (15 GB of expert weights), so consecutive steps
never hit the previous layer's weights in the 126 MB L2.

Synthetic data: weights N(0, 0.02) fp32 quantized on the device with the
reference quantizer's formula; 8 distinct quantized layers are replicated into
48 separate buffers.  Activations bf16 N(0, 1); router weights bf16
N(0, 0.02); logits = bf16(x @ Wr^T), one router per layer.

Output: one JSON line (rank 0).  ``value`` is device-timed (CUDA-graph replay
of the steps with inputs resident in HBM, events on the launching stream,
max over ranks); ``e2e`` is the same metric through ``MoeLayer.forward`` (the
public API) with host->device copies of each step's inputs from pinned memory
and a device->host copy of its output inside the timed region.
``--impl reference`` times the CPU restatement of the reference's own CPU path
(nano_ktrans CPUMoEBackend GPTQ branch) on the host cores instead.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE-layer routed tokens/s and expert-weight HBM GB/s (% peak) at 1/2/4/8 B200"
CFG = dict(hidden=2048, experts=128, inter=768, top_k=8, bits=4, group=128)
UNIQUE_LAYERS = 8
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=48 * 2000)
    ap.add_argument("--warmup", type=int, default=96)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--sweep", default="8,32,64", help="extra decode batch sizes to report ('' = none)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=960)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--prefill", default="mixtral,qwen2",
                    help="prefill workloads to report beside the decode line: mixtral (config 3), qwen2 (config 4)")
    ap.add_argument("--prefill-steps", type=int, default=20)
    ap.add_argument("--ep", default="4096,64",
                    help="config 5: global prefill,decode token counts of the 48-layer expert-parallel stack "
                         "('' = skip)")
    ap.add_argument("--ep-steps", type=int, default=3)
    ap.add_argument("--ep-exchange", default="peer", choices=("peer", "nccl"),
                    help="expert-parallel exchanges: the library's kernels over peer memory (CUDA IPC), or two "
                         "NCCL all_to_all_single calls per layer with a host read of the split sizes")
    ap.add_argument("--ep-graph", type=int, default=1,
                    help="with the peer exchange, replay the 48-layer step as one CUDA graph (1) or launch it "
                         "eagerly (0)")
    ap.add_argument("--m32", type=int, default=200,
                    help="steps of the dense bf16 stacked-bmm batch-1 comparator (0 = skip)")
    ap.add_argument("--no-c1", action="store_true", help="skip the config-1 (W8 per-channel, batch 1) decode line")
    ap.add_argument("--trace", action="store_true",
                    help="after the timed region, record the single-token kernel's per-CTA phase stamps "
                         "and add their median / slowest-CTA times to the JSON line")
    ap.add_argument("--ncu-case", type=int, default=0,
                    help="small profiling workload: this many tokens per step through MoeLayer.forward over 4 "
                         "distinct Qwen3-shaped layers (1.2 GB of weights), 2 passes, then exit")
    ap.add_argument("--skip-decode", action="store_true",
                    help="report only the prefill workloads (profiling runs of the grouped GEMM)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# peaks, clocks
# ---------------------------------------------------------------------------


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi sampled every 200 ms while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self._t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# synthetic stack
# ---------------------------------------------------------------------------


def make_unique_layer(gen, device):
    import torch

    from nano_ktrans_b200.weights import LayerWeights, quantize_symmetric, scale_stride

    E, H, I, bits, g = CFG["experts"], CFG["hidden"], CFG["inter"], CFG["bits"], CFG["group"]
    out = {}
    for proj, (n, k) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
        q = torch.empty(E, n, k * bits // 8, dtype=torch.uint8, device=device)
        s = torch.zeros(E, n, scale_stride(k // g), dtype=torch.bfloat16, device=device)
        for e0 in range(0, E, 16):
            w = torch.randn(16 * n, k, generator=gen, device=device) * 0.02
            qw = quantize_symmetric(w, group_size=g, bits=bits)
            q[e0:e0 + 16] = qw.qweight.view(torch.uint8).view(16, n, -1)
            s[e0:e0 + 16, :, :k // g] = qw.scales.view(16, n, -1).to(torch.bfloat16)
            del w, qw
        out[proj] = (q, s)
    return LayerWeights(bits=bits, group_size=g, gate_q=out["gate"][0], gate_s=out["gate"][1],
                        up_q=out["up"][0], up_s=out["up"][1], down_q=out["down"][0], down_s=out["down"][1])


def clone_layer(lw):
    from nano_ktrans_b200.weights import LayerWeights

    return LayerWeights(bits=lw.bits, group_size=lw.group_size, gate_q=lw.gate_q.clone(), gate_s=lw.gate_s.clone(),
                        up_q=lw.up_q.clone(), up_s=lw.up_s.clone(), down_q=lw.down_q.clone(), down_s=lw.down_s.clone())


def make_inputs(gen, n_layers, batch, device, with_router=False):
    import torch

    H, E = CFG["hidden"], CFG["experts"]
    x = torch.randn(n_layers, batch, H, generator=gen, device=device).to(torch.bfloat16)
    wr = (torch.randn(n_layers, E, H, generator=gen, device=device) * 0.02).to(torch.bfloat16)
    logits = torch.bmm(x, wr.transpose(1, 2))  # bf16 GEMM, as nn.Linear in bf16 computes the router
    return (x, logits.contiguous(), wr) if with_router else (x, logits.contiguous())


def expert_proj_bytes(lw):
    """Algorithmic bytes of one expert: (gate+up, down) codes + scales."""
    gu = sum(q[0].numel() + q.shape[1] * lw.groups(q) * 2 for q in (lw.gate_q, lw.up_q))
    dn = lw.down_q[0].numel() + lw.down_q.shape[1] * lw.groups(lw.down_q) * 2
    return gu, dn


# ---------------------------------------------------------------------------
# timed device loop
# ---------------------------------------------------------------------------


def run_device(layers, x, logits, outs, steps, warmup, profile_layer_class=None):
    """Warm up eagerly, capture the L-step cycle in a CUDA graph, replay it to
    cover `steps` steps; the timed graphs hold only the layers' own kernels.
    With profile_layer_class, a second graph of the same cycle brackets that
    kernel class with CUDA-event record nodes and is replayed after the timed
    region to measure the kernel alone.  Returns (ms, per-kernel avg ms or
    None, launches/step)."""
    import torch

    L = len(layers)
    for i in range(warmup):
        layers[i % L].forward(x[i % L], logits[i % L], out=outs[i % L])
    torch.cuda.synchronize()
    launches = layers[0].last_launch_count()
    full, rem = divmod(steps, L)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(n):
                layers[i].forward(x[i], logits[i], out=outs[i])
        return g

    g_full = capture(L)
    g_rem = capture(rem) if rem else None
    g_full.replay()  # one untimed replay
    torch.cuda.synchronize()
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(full):
        g_full.replay()
    if g_rem is not None:
        g_rem.replay()
    e1.record(st)
    torch.cuda.synchronize()
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    ms = e0.elapsed_time(e1)
    kern = None
    if profile_layer_class is not None:
        for lay in layers:
            lay.profile_begin(profile_layer_class, 1)
        g_prof = capture(L)
        g_prof.replay()  # warm
        g_prof.replay()  # the event nodes now hold this replay's times
        torch.cuda.synchronize()
        tot, n = 0.0, 0
        for lay in layers:
            a, b = lay.profile_end()
            tot += a
            n += b
        kern = tot / max(n, 1)
        del g_prof
    del g_full, g_rem
    return ms, kern, launches


def run_router_step(layers, x, wr, outs, steps, warmup):
    """The decode step from hidden states (MoeLayer.forward_x: the router
    projection kernel, then the single-launch step), captured for the L-layer
    cycle in a CUDA graph and replayed like run_device.  Returns (ms for
    `steps` steps, launches per step)."""
    import torch

    L = len(layers)
    for i in range(warmup):
        layers[i % L].forward_x(x[i % L], wr[i % L], out=outs[i % L])
    torch.cuda.synchronize()
    launches = layers[0].last_launch_count()
    full, rem = divmod(steps, L)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(n):
                layers[i].forward_x(x[i], wr[i], out=outs[i])
        return g

    g_full = capture(L)
    g_rem = capture(rem) if rem else None
    g_full.replay()
    torch.cuda.synchronize()
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(full):
        g_full.replay()
    if g_rem is not None:
        g_rem.replay()
    e1.record(st)
    torch.cuda.synchronize()
    del g_full, g_rem
    return e0.elapsed_time(e1), launches


def distinct_experts(layers, logits):
    import torch

    out = []
    for lay, lg in zip(layers, logits):
        ids, _ = lay.route(lg)
        out.append(int(torch.unique(ids).numel()))
    return out


T1_PHASES = ["inputs landed", "routing done", "chunk table built", "prologue done", "copies queued",
             "own gate/up rows done", "h written", "grid barrier passed", "h staged", "down blocks landed",
             "down tiles done", "exit"]


def trace_phases(layers, x, logits, outs, sm_mhz, reps=6):
    """Per-CTA phase stamps of the single-token kernel (SM clock cycles since CTA
    entry), over `reps` traced passes of the layer cycle, outside any timed region.
    Returns {phase: [median us, slowest-CTA us]}."""
    import numpy as np
    import torch

    L = len(layers)
    for lay in layers:
        lay.set_trace(True)
    rows = []
    try:
        for _ in range(reps):
            for i in range(L):
                layers[i].forward(x[i], logits[i], out=outs[i])
            torch.cuda.synchronize()
            rows.append(layers[L - 1].read_trace().astype(np.int64))
    finally:
        for lay in layers:
            lay.set_trace(False)
    tr = np.concatenate(rows[1:])
    return {name: [round(float(np.median(tr[:, i + 1])) / sm_mhz, 3), round(float(tr[:, i + 1].max()) / sm_mhz, 3)]
            for i, name in enumerate(T1_PHASES)}


def run_e2e(layers, x, logits, steps, call=None):
    """Public API with host buffers: H2D inputs, MoeLayer.forward (or
    call(j, x, logits, out)), D2H output."""
    import torch

    L = len(layers)
    if call is None:
        def call(j, xj, lj, oj):
            layers[j].forward(xj, lj, out=oj)
    xh = x.cpu().pin_memory()
    lh = logits.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    xd, ld = torch.empty_like(x), torch.empty_like(logits)
    od = torch.empty_like(x)
    for i in range(2 * L):
        j = i % L
        xd[j].copy_(xh[j], non_blocking=True)
        ld[j].copy_(lh[j], non_blocking=True)
        call(j, xd[j], ld[j], od[j])
        oh[j].copy_(od[j], non_blocking=True)
    torch.cuda.synchronize()
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(steps):
        j = i % L
        xd[j].copy_(xh[j], non_blocking=True)
        ld[j].copy_(lh[j], non_blocking=True)
        call(j, xd[j], ld[j], od[j])
        oh[j].copy_(od[j], non_blocking=True)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    h2d = xh[0].numel() * 2 + lh[0].numel() * 2
    d2h = oh[0].numel() * 2
    return ms, h2d, d2h


# ---------------------------------------------------------------------------
# CPU (reference algorithm) timing
# ---------------------------------------------------------------------------


def run_e2e_host(layers, x, logits, steps):
    """The C-ABI host-buffer call: moe_forward_host per step (H2D of x and the
    logits, the step, D2H of the output, all on the stream) from pinned
    buffers."""
    import torch

    L = len(layers)
    xh = x.cpu().pin_memory()
    lh = logits.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    for i in range(2 * L):
        layers[i % L].forward_host(xh[i % L], lh[i % L], oh[i % L])
    torch.cuda.synchronize()
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(steps):
        layers[i % L].forward_host(xh[i % L], lh[i % L], oh[i % L])
    e1.record(st)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1), xh[0].numel() * 2 + lh[0].numel() * 2, oh[0].numel() * 2


def hybrid_layers(lws, device):
    """HybridMoE layers (the reference's layer class and forward contract) over
    the same weights, every expert offloaded to the cuda backend."""
    import torch
    from torch import nn

    from nano_ktrans_b200.hybrid_moe import HybridMoE

    E, H, I, k = CFG["experts"], CFG["hidden"], CFG["inter"], CFG["top_k"]
    return [HybridMoE(num_experts=E, top_k=k, hidden_size=H, moe_intermediate_size=I, gpu_experts=nn.ModuleDict(),
                      gpu_experts_mask=torch.zeros(E, dtype=torch.bool), layer_idx=j, weight_path="",
                      router_use_softmax=True, normalize_topk_prob=True,
                      offload_backend_kwargs={"layer_weights": lw, "device": device, "max_tokens": 1})
            for j, lw in enumerate(lws)]


def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [p.get("num_threads", 1) for p in threadpool_info() if p.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:
        return 1


def host_expert(lw, e):
    """Copy one expert's codes/scales to the host as oracle QuantLinear triple."""
    import numpy as np
    import torch

    from oracle import moe_oracle as mo

    g = lw.group_size if lw.group_size > 0 else None
    trip = []
    for q, s in ((lw.gate_q, lw.gate_s), (lw.up_q, lw.up_s), (lw.down_q, lw.down_s)):
        words = q[e].contiguous().cpu().numpy().view(np.int32)
        k = words.shape[1] * 32 // lw.bits
        sc = s[e, :, :lw.groups(q)].to(torch.float32).cpu().numpy()
        trip.append(mo.QuantLinear(words, sc, g or k, lw.bits))
    return tuple(trip)


def cpu_reference_rate(layer_w, x, logits, seconds: float, max_steps: int):
    """Run the reference CPU algorithm (oracle port of CPUMoEBackend's GPTQ
    branch) on whole layer-steps until `seconds` elapse; tokens/s."""
    import numpy as np
    import torch

    from oracle import moe_oracle as mo

    L = len(layer_w)
    T = x.shape[1]
    xb = x.view(torch.int16).cpu().numpy().view(np.uint16)
    lb = logits.view(torch.int16).cpu().numpy().view(np.uint16)
    done, tokens, busy = 0, 0, 0.0
    cache = {}
    while done < max_steps and busy < seconds:
        j = done % L
        ids, w, _ = mo.route(lb[j], CFG["top_k"], True, True)
        experts = {}
        for e in sorted(set(ids.reshape(-1).tolist())):
            key = (id(layer_w[j]), e)
            if key not in cache:
                cache[key] = host_expert(layer_w[j], e)
            experts[e] = cache[key]
        t0 = time.perf_counter()
        mo.offload_forward(xb[j], ids, w, _Dense(experts, CFG["experts"]))
        busy += time.perf_counter() - t0
        done += 1
        tokens += T
    return tokens / busy, done, busy


class _Dense(dict):
    """Expert table with len() == num_experts for the oracle's expert scan."""

    def __init__(self, d, n):
        super().__init__(d)
        self.n = n

    def __len__(self):
        return self.n


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------


def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def max_over_ranks(v: float) -> float:
    import torch

    if not torch.distributed.is_initialized():
        return v
    t = torch.tensor([v], device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def config_block(args, world):
    return {"workload": "qwen3-30b-a3b moe layer decode (BASELINE config 2)", "hidden": CFG["hidden"],
            "experts": CFG["experts"], "moe_intermediate": CFG["inter"], "top_k": CFG["top_k"],
            "routing": "softmax top-k renormalised", "weights": "W4 symmetric group-128, bf16 scales",
            "batch_tokens": args.batch, "layers_cycled": args.layers, "unique_layer_contents": UNIQUE_LAYERS,
            "l2": "inputs larger than L2: steps cycle 48 distinct layer buffers (15 GB)",
            "parallelism": f"replicas x{world} (decode does not shard)"}


def main_reference(args):
    """CPU restatement of the reference path on the host cores."""
    import numpy as np
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # every host core, also under torch.distributed.run (which sets OMP_NUM_THREADS=1)
    ncores = len(os.sched_getaffinity(0))
    torch.set_num_threads(ncores)
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=ncores)
    except Exception:
        pass
    torch.manual_seed(args.seed)
    gen = torch.Generator().manual_seed(args.seed)
    from nano_ktrans_b200.weights import quantize_symmetric

    # one layer of 128 experts generated on the CPU (torch) with the same formula
    E, H, I = CFG["experts"], CFG["hidden"], CFG["inter"]
    from oracle import moe_oracle as mo

    experts = {}
    for e in range(E):
        trip = []
        for n, k in ((I, H), (I, H), (H, I)):
            q = quantize_symmetric(torch.randn(n, k, generator=gen) * 0.02, group_size=CFG["group"])
            trip.append(mo.QuantLinear(q.qweight.numpy(), q.scales.numpy(), CFG["group"], 4))
        experts[e] = tuple(trip)
    n_in = 16
    x = torch.randn(n_in, args.batch, H, generator=gen).to(torch.bfloat16)
    wr = (torch.randn(E, H, generator=gen) * 0.02).to(torch.bfloat16)
    logits = (x.float() @ wr.float().T).to(torch.bfloat16)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    lb = logits.view(torch.int16).numpy().view(np.uint16)
    table = _Dense(experts, E)
    for i in range(min(args.warmup, 2)):
        ids, w, _ = mo.route(lb[i % n_in], CFG["top_k"], True, True)
        mo.offload_forward(xb[i % n_in], ids, w, table)
    done, busy = 0, 0.0
    while done < args.steps and busy < 60.0:
        ids, w, _ = mo.route(lb[done % n_in], CFG["top_k"], True, True)
        t0 = time.perf_counter()
        mo.offload_forward(xb[done % n_in], ids, w, table)
        busy += time.perf_counter() - t0
        done += 1
    v = done * args.batch / busy
    cores = blas_threads()
    line = {
        "impl": "reference", "host_cores": ncores, "torch_threads": torch.get_num_threads(), "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "steps_run": done, "warmup": args.warmup, "ms_per_step": 1000 * busy / done,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(args, 1),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{done} whole layer-steps of the workload (bounded at 60 s of CPU time); "
                                   "oracle port of CPUMoEBackend GPTQ grouped W4A32 path"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        return main_reference(args)
    import torch

    from nano_ktrans_b200 import _lib
    from nano_ktrans_b200.moe_layer import MoeLayer

    world, rank, local = dist_setup(args)
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev).manual_seed(args.seed + 1000 * rank)
    if args.ncu_case:
        return ncu_case(gen, dev, args.ncu_case)
    if args.skip_decode:
        pre = prefill_block(args, dev, rank)
        if rank == 0:
            print(json.dumps({"metric": METRIC, "n_gpus": world, "data": "synthetic", "prefill": pre}), flush=True)
        if torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()
        return
    # expert weights are the same on every rank (the expert-parallel leg shards one
    # model across the ranks); inputs differ per rank
    wgen = torch.Generator(device=dev).manual_seed(args.seed)
    uniq = [make_unique_layer(wgen, dev) for _ in range(min(UNIQUE_LAYERS, args.layers))]
    lws = [uniq[i] if i < len(uniq) else clone_layer(uniq[i % len(uniq)]) for i in range(args.layers)]
    max_b = max([args.batch] + [int(b) for b in args.sweep.split(",") if b])
    layers = [MoeLayer(lw, top_k=CFG["top_k"], router_use_softmax=True, normalize_topk_prob=True, max_tokens=max_b)
              for lw in lws]
    x, logits, wr = make_inputs(gen, args.layers, args.batch, dev, with_router=True)
    outs = torch.empty_like(x)
    gu_bytes, dn_bytes = expert_proj_bytes(lws[0])
    peak, peak_kind = hbm_peak()

    distinct = distinct_experts(layers, logits)
    L = args.layers
    steps_bytes = [distinct[i % L] * (gu_bytes + dn_bytes) for i in range(args.steps)]

    # dominant kernel: the single-launch decode step when the batch fits it,
    # else the gate/up matvec of the multi-kernel chain
    fused = args.batch <= 4
    kclass = _lib.K_DECODE_FUSED if fused else _lib.K_GATEUP
    with ClockSampler(local) as clk:
        ms, k_ms, launches = run_device(layers, x, logits, outs, args.steps, args.warmup, profile_layer_class=kclass)
    ms = max_over_ranks(ms)
    tokens = args.steps * args.batch * world
    value = tokens / (ms / 1e3)
    alg_bytes = sum(steps_bytes)
    gbs = alg_bytes * world / (ms / 1e3) / 1e9
    # roofline: the kernel's algorithmic bytes per launch (codes + scales of the
    # distinct routed experts it reads) / its CUDA-event duration
    per_launch = statistics.mean(d * ((gu_bytes + dn_bytes) if fused else gu_bytes) for d in distinct)
    # kernel time of the roofline: with one launch per step (the single-launch
    # kernel) it is the graph-replay step time itself, measured without anything
    # inserted between the launches; the event-bracketed replay (which breaks the
    # programmatic-dependent-launch overlap) is reported beside it, not used
    one_launch = fused and launches == 1
    kern_ms = ms / args.steps if one_launch else k_ms
    achieved = per_launch / (kern_ms / 1e3) / 1e9
    kname = ("moe_decode_t1_kernel" if args.batch == 1 else "moe_decode_fused_kernel<4>") if fused \
        else "expert_matvec_kernel<4,32,gate/up>"
    traffic = read_traffic(("decode_t1" if args.batch == 1 else "decode_fused") if fused else "gateup", args.batch)

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u4 codes, f32 accumulate, bf16 io", "data": "synthetic",
        "config": config_block(args, world),
        "expert_weight_gbs": gbs, "expert_weight_frac_of_peak": gbs / world / peak,
        "roofline": {"bound": "hbm", "kernel": kname, "achieved": achieved,
                     "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_kind,
                     "traffic": traffic, "algorithmic_bytes_per_launch": per_launch,
                     "avg_launch_ms": kern_ms,
                     "kernel_time_source": ("graph-replay step time (one launch per step)" if one_launch
                                            else "CUDA events bracketing the kernel in a second graph replay"),
                     "event_bracketed_launch_ms": k_ms,
                     "traffic_source": "ncu dram__bytes_read+write per launch recorded in profiles/ncu_traffic.txt"},
        "gpu_launches": launches * args.steps,
        "clocks": clk.summary(),
    }

    if fused:
        # the same step from hidden states: the router projection (bf16 [E, H] per
        # layer) runs in the timed graph too
        r_ms, r_launch = run_router_step(layers, x, wr, outs, args.steps, args.warmup)
        r_ms = max_over_ranks(r_ms)
        router_bytes = CFG["experts"] * CFG["hidden"] * 2
        r_step = r_ms / args.steps
        line["decode_with_router"] = {
            "value": args.steps * args.batch * world / (r_ms / 1e3), "unit": "tokens/s", "ms_per_step": r_step,
            "launches_per_step": r_launch,
            "bytes_per_step": statistics.mean(steps_bytes) + router_bytes, "router_bytes_per_step": router_bytes,
            "frac_of_peak": (statistics.mean(steps_bytes) + router_bytes) / (r_step / 1e3) / 1e9 / peak,
            "api": "MoeLayer.forward_x (moe_forward_x: router projection kernel + the single-launch step)"}

    if not args.no_c1 and args.batch == 1:
        line["c1_w8_decode_b1"] = run_c1(gen, dev, 48 * 500, 48,
                                         cpu_seconds=0.0 if (args.no_cpu_baseline or world > 1) else 5.0)

    if args.m32 and args.batch == 1:
        line["m32_dense_bmm_b1"] = run_m32_bmm(gen, dev, args.m32, max(args.warmup, 3))

    if args.trace and fused and args.batch == 1:
        line["phase_timeline_us"] = trace_phases(layers, x, logits, outs, clk.summary().get("sm_mhz") or 1965.0)

    if not args.no_e2e:
        e_ms, h2d, d2h = run_e2e_host(layers, x, logits, args.e2e_steps)
        e_ms = max_over_ranks(e_ms)
        line["e2e"] = {"value": args.e2e_steps * args.batch * world / (e_ms / 1e3), "unit": "tokens/s",
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": args.e2e_steps,
                       "api": "moe_forward_host per step (C ABI via MoeLayer.forward_host): pinned host x and "
                              "logits read by the device through their mapped addresses, bf16 output stored by "
                              "the step's last kernel into pinned host memory"}
        for lay in layers:
            lay.set_host_io(0)
        d_ms, _, _ = run_e2e_host(layers, x, logits, args.e2e_steps)
        for lay in layers:
            lay.set_host_io(2)
        line["e2e"]["copy_engine"] = {
            "value": args.e2e_steps * args.batch * world / (max_over_ranks(d_ms) / 1e3), "unit": "tokens/s",
            "api": "moe_forward_host with copy-engine copies in and out"}
        t_ms, _, _ = run_e2e(layers, x, logits, args.e2e_steps)
        t_ms = max_over_ranks(t_ms)
        line["e2e"]["moe_layer_forward"] = {
            "value": args.e2e_steps * args.batch * world / (t_ms / 1e3), "unit": "tokens/s",
            "api": "torch copies of pinned host tensors + MoeLayer.forward on device tensors, per step"}
        if args.batch == 1:
            hyb = hybrid_layers(lws, dev)

            def hcall(j, xj, lj, oj):
                oj.copy_(hyb[j](xj, lj))
            h_ms, _, _ = run_e2e(layers, x, logits, args.e2e_steps, call=hcall)
            h_ms = max_over_ranks(h_ms)
            line["e2e"]["hybrid_moe_forward"] = {
                "value": args.e2e_steps * args.batch * world / (h_ms / 1e3), "unit": "tokens/s",
                "api": "HybridMoE.forward (all experts offloaded to the cuda backend) per step, pinned host buffers"}
            del hyb

    sweep = {}
    for b in [int(b) for b in args.sweep.split(",") if b]:
        xb_, lb_ = make_inputs(gen, args.layers, b, dev)
        ob_ = torch.empty_like(xb_)
        d_b = distinct_experts(layers, lb_)
        st = 48 * 100
        s_ms, s_k, _ = run_device(layers, xb_, lb_, ob_, st, 48, profile_layer_class=_lib.K_GATEUP)
        s_ms = max_over_ranks(s_ms)
        byt = sum(d_b[i % L] * (gu_bytes + dn_bytes) for i in range(st))
        step_gbs = byt / (s_ms / 1e3) / 1e9
        sweep[str(b)] = {"tokens_per_s": st * b * world / (s_ms / 1e3), "ms_per_step": s_ms / st,
                         "expert_weight_gbs": byt * world / (s_ms / 1e3) / 1e9,
                         "gateup_kernel_gbs": statistics.mean(d * gu_bytes for d in d_b) / (s_k / 1e3) / 1e9,
                         "distinct_experts_mean": statistics.mean(d_b),
                         "launches_per_step": layers[0].last_launch_count(),
                         "roofline": {"bound": "hbm", "scope": "whole step (every kernel of the step)",
                                      "achieved": step_gbs, "peak": peak, "unit": "GB/s", "frac": step_gbs / peak,
                                      "peak_source": peak_kind,
                                      "algorithmic_bytes_per_step": byt / st,
                                      "traffic": read_traffic("sweep", b)}}
    if sweep:
        line["sweep"] = sweep

    pre = prefill_block(args, dev, rank)
    if pre:
        line["prefill"] = pre
    if args.ep:
        line["ep"] = run_ep(args, world, rank, dev, uniq, lws)

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, n, busy = cpu_reference_rate(lws, x, logits, args.cpu_seconds, 10 ** 6)
        line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": blas_threads(), "kind": "port",
                                "sample": f"{n} layer-steps at batch {args.batch} ({busy:.1f} s), oracle port of "
                                          "CPUMoEBackend GPTQ grouped W4A32 path on the same weights"}
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if torch.distributed.is_initialized():
        torch.distributed.destroy_process_group()


# ---------------------------------------------------------------------------
# prefill workloads (tensor-core grouped GEMM path)
# ---------------------------------------------------------------------------

PREFILL = {
    # config 3: Mixtral-8x7B-shaped layer, 2048-token prefill, W8 per-channel,
    # top-2 softmax over the top-k logits
    "mixtral": dict(experts=8, hidden=4096, inter=14336, top_k=2, bits=8, group=0, softmax=False, renorm=True,
                    tokens=2048, shared=0, zipf=None),
    # config 4: Qwen2-MoE-A2.7B-shaped layer, 256 tokens, W4 g128, top-4 without
    # renormalisation, shared expert 5632 with a sigmoid gate, Zipf(1.2) routing
    "qwen2": dict(experts=60, hidden=2048, inter=1408, top_k=4, bits=4, group=128, softmax=True, renorm=False,
                  tokens=256, shared=5632, zipf=1.2),
}


def quantized_stack(gen, device, E, n, k, bits, group):
    """[E, n, k*bits/8] codes + padded bf16 scales of N(0, 0.02) weights."""
    import torch

    from nano_ktrans_b200.weights import quantize_symmetric, scale_stride

    g = group if group > 0 else k
    q = torch.empty(E, n, k * bits // 8, dtype=torch.uint8, device=device)
    s = torch.zeros(E, n, scale_stride(k // g), dtype=torch.bfloat16, device=device)
    for e in range(E):
        qw = quantize_symmetric(torch.randn(n, k, generator=gen, device=device) * 0.02, group_size=group, bits=bits)
        q[e] = qw.qweight.view(torch.uint8).view(n, -1)
        s[e, :, :k // g] = qw.scales.view(n, -1).to(torch.bfloat16)
        del qw
    return q, s


def zipf_router_bias(E: int, alpha: float, gen, device, beta: float = 1.0):
    """b_e = beta * log(z_e), z proportional to rank^-alpha over a seeded expert permutation."""
    import torch

    perm = torch.randperm(E, generator=gen, device=device)
    ranks = torch.empty(E, device=device)
    ranks[perm] = torch.arange(1, E + 1, device=device, dtype=torch.float32)
    z = ranks ** (-alpha)
    return beta * torch.log(z / z.sum())


_ZIPF_BETA = {}


def calibrate_zipf_beta(E: int, top_k: int, H: int, alpha: float, device, renorm: bool = True, tokens: int = 8192):
    """The router bias scale beta for which the empirical top-k selection
    frequency of N(0, 1) tokens through an N(0, 0.02) bf16 router follows
    Zipf(alpha) over the bias ranks: bisection on beta so that the slope of
    log(frequency) against log(rank), fitted over the ranks that are selected
    at all, equals -alpha.  Seeded and cached per (E, k, H, alpha)."""
    import numpy as np
    import torch

    key = (E, top_k, H, alpha)
    if key in _ZIPF_BETA:
        return _ZIPF_BETA[key]
    gen = torch.Generator(device=device).manual_seed(4242)
    x = torch.randn(tokens, H, generator=gen, device=device).to(torch.bfloat16)
    wr = (torch.randn(E, H, generator=gen, device=device) * 0.02).to(torch.bfloat16)
    base = (x @ wr.T).float()
    perm = torch.randperm(E, generator=gen, device=device)
    ranks = torch.empty(E, device=device)
    ranks[perm] = torch.arange(1, E + 1, device=device, dtype=torch.float32)
    logz = torch.log(ranks ** (-alpha) / (ranks ** (-alpha)).sum())

    def fitted(beta):
        lg = (base + beta * logz).to(torch.bfloat16).float()
        p = torch.softmax(lg, dim=-1).to(torch.bfloat16)
        ids = torch.topk(p, top_k, dim=-1).indices
        freq = torch.bincount(ids.reshape(-1), minlength=E).float()
        f = freq[perm].cpu().numpy()  # by bias rank 1..E
        r = np.arange(1, E + 1, dtype=np.float64)
        sel = f > 0
        return -np.polyfit(np.log(r[sel]), np.log(f[sel]), 1)[0]

    lo, hi = 0.0, 8.0
    for _ in range(30):
        mid = 0.5 * (lo + hi)
        if fitted(mid) < alpha:
            lo = mid
        else:
            hi = mid
    beta = 0.5 * (lo + hi)
    _ZIPF_BETA[key] = (beta, float(fitted(beta)))
    return _ZIPF_BETA[key]


def qlin(q, s, e: int, bits: int, group: int):
    """Expert e of a stacked [E, N, K*bits/8] code / [E, N, SS] scale pair as the
    oracle's QuantLinear (the host copy of the same device weights)."""
    import numpy as np
    import torch

    from oracle import moe_oracle as mo

    words = q[e].contiguous().cpu().numpy().view(np.int32)
    kdim = words.shape[1] * 32 // bits
    g = group if group > 0 else kdim
    sc = s[e, :, :kdim // g].to(torch.float32).cpu().numpy()
    return mo.QuantLinear(words, sc, g, bits)


def prefill_cpu_baseline(name, lw, x, ids, wts, shared, E, k, T, seconds):
    """The oracle port of the reference CPU path (CPUMoEBackend GPTQ branch and
    the shared-expert add) on the same weights, routing and tokens.  Mixtral's
    1.4 TFLOP layer is sampled: the experts are run in ascending order until
    `seconds` of CPU time, and the time is scaled by the (token, expert) pairs
    of all experts over those run."""
    import numpy as np
    import torch

    from oracle import moe_oracle as mo

    xb = x.view(torch.int16).cpu().numpy().view(np.uint16)
    ib = ids.cpu().numpy()
    wb = wts.view(torch.int16).cpu().numpy().view(np.uint16)
    g = lw.group_size
    counts = np.bincount(ib.reshape(-1), minlength=E)
    busy, pairs_done, run = 0.0, 0, []
    for e in range(E):
        if counts[e] == 0:
            continue
        ex = {e: tuple(qlin(q, s_, e, lw.bits, g) for q, s_ in ((lw.gate_q, lw.gate_s), (lw.up_q, lw.up_s),
                                                                   (lw.down_q, lw.down_s)))}
        sel = np.where(ib == e, ib, -1)
        t0 = time.perf_counter()
        mo.offload_forward_f32(xb, sel, wb, ex, None) if sel.max() >= 0 else None
        busy += time.perf_counter() - t0
        pairs_done += int(counts[e])
        run.append(e)
        if busy > seconds:
            break
    total = busy * counts.sum() / max(pairs_done, 1)
    sample = f"experts {run[0]}..{run[-1]} ({len(run)} of {int((counts > 0).sum())} routed, {pairs_done} of " \
             f"{int(counts.sum())} pairs) timed once, scaled by pairs"
    if shared is not None:
        sh = tuple(qlin(shared[a], shared[b], 0, lw.bits, g) for a, b in (("gate_q", "gate_s"), ("up_q", "up_s"),
                                                                        ("down_q", "down_s")))
        gv = shared["gate_vec"].view(torch.int16).cpu().numpy().view(np.uint16)
        t0 = time.perf_counter()
        mo.shared_expert_f32(xb, gv, sh)
        total += time.perf_counter() - t0
        sample += "; shared expert timed once"
    return {"value": T / total, "unit": "tokens/s", "cores": blas_threads(), "kind": "port",
            "sample": f"{name} layer of {T} tokens: {sample}; oracle port of CPUMoEBackend GPTQ path"}


def bf16_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (burst)"
    except Exception:
        return 1590.0, "fallback"


def run_prefill(name: str, gen, device, steps: int, warmup: int, cpu_seconds: float = 0.0):
    """Device time of MoeLayer.forward (route + permute + pack + grouped GEMMs +
    combine, shared expert included) on one prefill batch, CUDA events on the
    launching stream; the expert weights (> L2) are re-read every step."""
    import torch

    from nano_ktrans_b200 import _lib
    from nano_ktrans_b200.moe_layer import MoeLayer
    from nano_ktrans_b200.weights import LayerWeights

    c = PREFILL[name]
    E, H, I, k, T, bits, grp = c["experts"], c["hidden"], c["inter"], c["top_k"], c["tokens"], c["bits"], c["group"]
    gq, gs = quantized_stack(gen, device, E, I, H, bits, grp)
    uq, us = quantized_stack(gen, device, E, I, H, bits, grp)
    dq, ds = quantized_stack(gen, device, E, H, I, bits, grp)
    shared = None
    if c["shared"]:
        S = c["shared"]
        sg = quantized_stack(gen, device, 1, S, H, bits, grp)
        su = quantized_stack(gen, device, 1, S, H, bits, grp)
        sd = quantized_stack(gen, device, 1, H, S, bits, grp)
        vec = (torch.randn(H, generator=gen, device=device) * 0.02).to(torch.bfloat16)
        shared = {"gate_q": sg[0], "gate_s": sg[1], "up_q": su[0], "up_s": su[1], "down_q": sd[0], "down_s": sd[1],
                  "gate_vec": vec}
    lw = LayerWeights(bits=bits, group_size=grp, gate_q=gq, gate_s=gs, up_q=uq, up_s=us, down_q=dq, down_s=ds,
                      shared=shared)
    layer = MoeLayer(lw, top_k=k, router_use_softmax=c["softmax"], normalize_topk_prob=c["renorm"], max_tokens=T)
    x = torch.randn(T, H, generator=gen, device=device).to(torch.bfloat16)
    wr = (torch.randn(E, H, generator=gen, device=device) * 0.02).to(torch.bfloat16)
    logits = x @ wr.T
    zipf = None
    if c["zipf"]:
        beta, fit = calibrate_zipf_beta(E, k, H, c["zipf"], device, renorm=c["renorm"])
        zipf = {"alpha": c["zipf"], "beta": beta, "fitted_alpha": fit}
        logits = (logits.float() + zipf_router_bias(E, c["zipf"], gen, device, beta)).to(torch.bfloat16)
    out = torch.empty_like(x)
    for _ in range(max(warmup, 3)):
        layer.forward(x, logits, out=out)
    torch.cuda.synchronize()
    launches = layer.last_launch_count()
    kern = {}
    for cls, nm in ((_lib.K_GATEUP, "gateup"), (_lib.K_DOWN, "down")):
        layer.profile_begin(cls, steps)
        for _ in range(steps):
            layer.forward(x, logits, out=out)
        ms_k, n_k = layer.profile_end()
        kern[nm] = ms_k / max(n_k, 1)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(steps):
        layer.forward(x, logits, out=out)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    ids, wts = layer.route(logits)
    per_expert = torch.bincount(ids.reshape(-1), minlength=E)
    flops_routed = 2.0 * T * k * 3 * H * I
    flops_gateup = 2.0 * T * k * 2 * H * I
    peak, peak_kind = bf16_peak()
    gu_tf = flops_gateup / (kern["gateup"] / 1e3) / 1e12
    res = {
        "config": f"{name}: E={E} H={H} I={I} top{k} W{bits} group={grp or 'per-channel'} tokens={T}"
                  + (f" shared={c['shared']} zipf={c['zipf']}" if c["shared"] else ""),
        "tokens_per_s": T / (ms / 1e3), "ms_per_step": ms, "launches_per_step": launches,
        "routed_tflops": flops_routed / (ms / 1e3) / 1e12,
        "tokens_per_expert": {"max": int(per_expert.max()), "min": int(per_expert.min()),
                              "mean": float(per_expert.float().mean())},
        "down_kernel_tflops": 2.0 * T * k * H * I / (kern["down"] / 1e3) / 1e12,
        "down_avg_launch_ms": kern["down"],
    }
    gemm_roof = {"bound": "tensor", "kernel": f"grouped_gemm_kernel<{bits},gate/up>", "achieved": gu_tf,
                 "peak": peak, "unit": "TFLOP/s", "frac": gu_tf / peak, "peak_source": peak_kind,
                 "algorithmic_flops_per_launch": flops_gateup, "avg_launch_ms": kern["gateup"],
                 "kernel_time_source": "CUDA events bracketing the kernel (eager launches)"}
    if name == "qwen2":
        # about 124 FLOP per weight byte: below the ridge, so the bound is HBM: the
        # distinct routed experts' codes + scales plus the shared expert, once per step
        def proj_bytes(q):
            kdim = q.shape[2] * 8 // bits
            return q[0].numel() + q.shape[1] * (kdim // (grp if grp > 0 else kdim)) * 2  # codes + bf16 scales

        per_e = proj_bytes(gq) + proj_bytes(uq) + proj_bytes(dq)
        distinct = int((per_expert > 0).sum())
        sh_bytes = sum(proj_bytes(shared[a]) for a in ("gate_q", "up_q", "down_q"))
        step_bytes = distinct * per_e + sh_bytes
        gbs = step_bytes / (ms / 1e3) / 1e9
        hpeak, hkind = hbm_peak()
        res["roofline"] = {"bound": "hbm", "scope": "whole step", "achieved": gbs, "peak": hpeak, "unit": "GB/s",
                           "frac": gbs / hpeak, "peak_source": hkind, "algorithmic_bytes_per_step": step_bytes,
                           "distinct_routed_experts": distinct, "shared_expert_bytes": sh_bytes}
        res["gateup_gemm_tensor_roofline"] = gemm_roof
        res["zipf"] = zipf
    else:
        res["roofline"] = gemm_roof
    if cpu_seconds > 0:
        res["cpu_baseline"] = prefill_cpu_baseline(name, lw, x, ids, wts, shared, E, k, T, cpu_seconds)
    del layer, lw, gq, gs, uq, us, dq, ds
    torch.cuda.empty_cache()
    return res


def ncu_case(gen, dev, batch: int, n_layers: int = 4, passes: int = 2):
    """A small, bounded workload for kernel captures: `passes` eager passes of
    MoeLayer.forward over n_layers distinct Qwen3-shaped W4 layers at `batch`
    tokens (launch i of a kernel class belongs to layer i % n_layers)."""
    import torch

    from nano_ktrans_b200.moe_layer import MoeLayer

    lws = [make_unique_layer(gen, dev) for _ in range(n_layers)]
    layers = [MoeLayer(lw, top_k=CFG["top_k"], router_use_softmax=True, normalize_topk_prob=True, max_tokens=batch)
              for lw in lws]
    x, logits = make_inputs(gen, n_layers, batch, dev)
    out = torch.empty_like(x)
    for _ in range(passes):
        for i, lay in enumerate(layers):
            lay.forward(x[i], logits[i], out=out[i])
    torch.cuda.synchronize()
    bad = sum(lay.read_status() for lay in layers)
    print(json.dumps({"ncu_case": batch, "layers": n_layers, "passes": passes,
                      "launches_per_step": layers[0].last_launch_count(), "status": bad}), flush=True)
    for lay in layers:
        lay.close()
    return 0 if bad == 0 else 1


def run_m32_bmm(gen, device, steps: int, warmup: int, n_layers: int = 4):
    """The reference's GPU-resident batch-1 comparator (the fused stacked-bmm
    decode of hybrid_moe.py:3442-3500) restated in PyTorch on dense bf16
    Qwen3-shaped experts: unique routed ids read to the host, the routed
    experts' gate/up/down stacked, three bmm + SiLU * up, and the weighted sum
    over the routed experts.  n_layers distinct layers (1.2 GB of bf16 experts
    each) are cycled so every step reads its experts from HBM.  CUDA events
    around `steps` steps; the block's host reads are inside the timed region,
    as they are in the reference."""
    import torch
    import torch.nn.functional as F

    E, H, I, k = CFG["experts"], CFG["hidden"], CFG["inter"], CFG["top_k"]
    w1 = [(torch.randn(E, I, H, generator=gen, device=device) * 0.02).to(torch.bfloat16) for _ in range(n_layers)]
    w3 = [(torch.randn(E, I, H, generator=gen, device=device) * 0.02).to(torch.bfloat16) for _ in range(n_layers)]
    w2 = [(torch.randn(E, H, I, generator=gen, device=device) * 0.02).to(torch.bfloat16) for _ in range(n_layers)]
    xs = [torch.randn(1, H, generator=gen, device=device).to(torch.bfloat16) for _ in range(n_layers)]
    wr = [(torch.randn(E, H, generator=gen, device=device) * 0.02).to(torch.bfloat16) for _ in range(n_layers)]
    route = []
    for x, r in zip(xs, wr):
        p = torch.softmax((x @ r.T).float(), dim=-1)
        w, ids = torch.topk(p, k, dim=-1)
        route.append((ids, (w / w.sum(dim=-1, keepdim=True)).to(torch.bfloat16)))
    gpu_mask = torch.ones(E, dtype=torch.bool, device=device)
    outs = [torch.zeros(1, H, dtype=torch.bfloat16, device=device) for _ in range(n_layers)]

    def block(j):
        ids, w = route[j]
        unique_routed = torch.unique(ids).cpu().tolist()
        mask = gpu_mask.cpu().tolist()
        routed = [e for e in unique_routed if mask[e]]
        g1 = torch.stack([w1[j][e] for e in routed])
        g3 = torch.stack([w3[j][e] for e in routed])
        g2 = torch.stack([w2[j][e] for e in routed])
        xb = xs[j].expand(len(routed), -1).unsqueeze(1)
        h = F.silu(torch.bmm(xb, g1.transpose(1, 2))) * torch.bmm(xb, g3.transpose(1, 2))
        o = torch.bmm(h, g2.transpose(1, 2)).squeeze(1)
        rt = torch.tensor(routed, device=device, dtype=torch.long)
        match = (rt.unsqueeze(1) == ids[0].unsqueeze(0)).to(w.dtype)
        outs[j][0] = (o * (match * w[0].unsqueeze(0)).sum(dim=1).unsqueeze(1)).sum(dim=0)

    for i in range(warmup):
        block(i % n_layers)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        block(i % n_layers)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    per_step = k * 3 * H * I * 2  # the routed experts' bf16 weights
    peak, peak_kind = hbm_peak()
    gbs = per_step / (ms / 1e3) / 1e9
    del w1, w2, w3
    torch.cuda.empty_cache()
    return {"ms_per_step": ms, "tokens_per_s": 1e3 / ms, "expert_weight_gbs": gbs, "frac_of_hbm_peak": gbs / peak,
            "peak_source": peak_kind, "algorithmic_bytes_per_step": per_step, "steps": steps,
            "weights": "dense bf16, 8 routed experts of E=128 H=2048 I=768", "layers_cycled": n_layers,
            "note": "stacks copy the routed weights each step (reads + writes 2x the algorithmic bytes)"}


def run_c1(gen, device, steps: int, warmup: int, n_layers: int = 6, cpu_seconds: float = 0.0):
    """Config 1: Qwen3-shaped W8 per-output-channel decode at batch 1 (the
    single-launch multi-token kernel; the single-token kernel is W4 only).
    n_layers distinct layers (0.6 GB of expert weights each) are cycled in a
    CUDA graph, so every step reads its 8 experts (37.8 MB) from HBM."""
    import torch

    from nano_ktrans_b200 import _lib
    from nano_ktrans_b200.moe_layer import MoeLayer
    from nano_ktrans_b200.weights import LayerWeights

    E, H, I, k = CFG["experts"], CFG["hidden"], CFG["inter"], CFG["top_k"]
    layers, x, logits, lws = [], [], [], []
    for _ in range(n_layers):
        gq, gs = quantized_stack(gen, device, E, I, H, 8, 0)
        uq, us = quantized_stack(gen, device, E, I, H, 8, 0)
        dq, ds = quantized_stack(gen, device, E, H, I, 8, 0)
        lw = LayerWeights(bits=8, group_size=0, gate_q=gq, gate_s=gs, up_q=uq, up_s=us, down_q=dq, down_s=ds)
        layers.append(MoeLayer(lw, top_k=k, router_use_softmax=True, normalize_topk_prob=True, max_tokens=1))
        lws.append(lw)
        xi = torch.randn(1, H, generator=gen, device=device).to(torch.bfloat16)
        wr = (torch.randn(E, H, generator=gen, device=device) * 0.02).to(torch.bfloat16)
        x.append(xi)
        logits.append(xi @ wr.T)
    outs = [torch.empty_like(xi) for xi in x]
    ms, k_ms, launches = run_device(layers, x, logits, outs, steps, warmup, profile_layer_class=_lib.K_DECODE_FUSED)
    ev_ms = k_ms
    if launches == 1:
        k_ms = ms / steps  # one launch per step: the graph-replay step time is the kernel time
    per_expert = 3 * H * I + (2 * I + H) * 2  # int8 codes + one bf16 scale per output row: 4,725,760 B
    distinct = [int(torch.unique(lay.route(lg)[0]).numel()) for lay, lg in zip(layers, logits)]
    step_bytes = sum(distinct[i % n_layers] for i in range(steps)) / steps * per_expert
    peak, peak_kind = hbm_peak()
    gbs = step_bytes / (ms / steps / 1e3) / 1e9
    kgbs = step_bytes / (k_ms / 1e3) / 1e9
    cpu = None
    if cpu_seconds > 0:
        rate, n, busy = cpu_reference_rate(lws, torch.stack(x), torch.stack(logits), cpu_seconds, 10 ** 6)
        cpu = {"value": rate, "unit": "tokens/s", "cores": blas_threads(), "kind": "port",
               "sample": f"{n} layer-steps at batch 1 ({busy:.1f} s), oracle port of CPUMoEBackend GPTQ path "
                         "(W8 per-channel) on the same weights"}
    del layers
    torch.cuda.empty_cache()
    return {"cpu_baseline": cpu,
            "config": "C1: E=128 H=2048 I=768 top8 renormalised, W8 per-channel, bf16 scales, batch 1",
            "tokens_per_s": steps / (ms / 1e3), "ms_per_step": ms / steps, "launches_per_step": launches,
            "expert_weight_gbs": gbs, "expert_weight_frac_of_peak": gbs / peak,
            "roofline": {"bound": "hbm", "kernel": "moe_decode_fused_kernel<8>", "achieved": kgbs, "peak": peak,
                         "unit": "GB/s", "frac": kgbs / peak, "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": step_bytes, "avg_launch_ms": k_ms,
                         "kernel_time_source": "graph-replay step time (one launch per step)" if launches == 1
                         else "CUDA events bracketing the kernel", "event_bracketed_launch_ms": ev_ms,
                         "traffic": read_traffic("decode_fused_w8", 1)},
            "layers_cycled": n_layers}


def prefill_block(args, dev, rank):
    """Prefill workloads, one replica per rank; ms is the max over ranks."""
    import torch

    out = {}
    for name in [n for n in args.prefill.split(",") if n]:
        gen = torch.Generator(device=dev).manual_seed(args.seed + 17 + 1000 * rank)
        r = run_prefill(name, gen, dev, args.prefill_steps, args.warmup,
                        0.0 if (args.no_cpu_baseline or rank != 0) else args.cpu_seconds)
        ms = max_over_ranks(r["ms_per_step"])
        world = torch.distributed.get_world_size() if torch.distributed.is_initialized() else 1
        r["ms_per_step"] = ms
        r["tokens_per_s"] = PREFILL[name]["tokens"] * world / (ms / 1e3)
        r["replicas"] = world
        out[name] = r
    return out


# ---------------------------------------------------------------------------
# config 5: 48-layer stack, experts split across the ranks
# ---------------------------------------------------------------------------


def run_ep(args, world, rank, dev, uniq, lws):
    """Config 5: the 48-layer Qwen3-shaped stack (W4 g128, Zipf(1.2) routing)
    with each layer's 128 experts split over the ranks (frequency-balanced
    placement; exchanges over peer memory, or NCCL all-to-alls with
    --ep-exchange nccl); global prefill and decode batches split evenly over
    the ranks.  One GPU runs the same layers through the single-GPU path.
    Times are CUDA events around a pass over all 48 layers (max over ranks);
    with --ep-graph (default) the pass is one CUDA graph replay at every N
    (the NCCL exchange, which reads split sizes on the host, runs eagerly)."""
    import torch

    from nano_ktrans_b200.expert_parallel import EpMoeLayer, TorchDistComm, plan_placement, shard_layer
    from nano_ktrans_b200.moe_layer import MoeLayer

    E, H, k = CFG["experts"], CFG["hidden"], CFG["top_k"]
    n_prefill, n_decode = [int(v) for v in args.ep.split(",")]
    L = len(lws)
    gen = torch.Generator(device=dev).manual_seed(args.seed + 5000)  # same router and bias on every rank
    routers = [(torch.randn(E, H, generator=gen, device=dev) * 0.02).to(torch.bfloat16) for _ in range(L)]
    beta, fit_alpha = calibrate_zipf_beta(E, k, H, 1.2, dev, renorm=True)
    biases = [zipf_router_bias(E, 1.2, gen, dev, beta) for _ in range(L)]
    tgen = torch.Generator(device=dev).manual_seed(args.seed + 6000 + rank)  # this rank's tokens

    def batch(n_global):
        t = n_global // world + (1 if rank < n_global % world else 0)
        xs = [torch.randn(t, H, generator=tgen, device=dev).to(torch.bfloat16) for _ in range(L)]
        lg = [((x @ r.T).float() + b).to(torch.bfloat16) for x, r, b in zip(xs, routers, biases)]
        return t, xs, lg

    tp, xp, lp = batch(n_prefill)
    td, xd, ld = batch(n_decode)
    res = {"placement": "frequency-balanced (prefill batch routing counts, all ranks)", "world": world,
           "zipf": {"alpha": 1.2, "beta": beta, "fitted_alpha": fit_alpha}}

    exchange = None
    if world == 1:
        layers = [MoeLayer(lw, top_k=k, router_use_softmax=True, normalize_topk_prob=True, max_tokens=tp)
                  for lw in lws]

        def step(xs, lg):
            for lay, x, g in zip(layers, xs, lg):
                lay.forward(x, g)
        res["path"] = "single GPU: moe_forward per layer (all experts local)" + (
            "; the 48-layer step replayed as one CUDA graph" if args.ep_graph else "")
    else:
        comm = TorchDistComm()
        if args.ep_exchange == "peer":
            from nano_ktrans_b200.expert_parallel import PeerExchange

            exchange = PeerExchange(rank, world, max_tokens=max(tp, td), top_k=k, hidden=H, num_experts=E, device=dev)
            exchange.connect_ipc()
        probe = EpMoeLayer(shard_layer(uniq[0], plan_placement(E, world), rank, world), num_experts=E, top_k=k,
                           slot_of_expert=plan_placement(E, world), rank=rank, world=world, max_tokens=tp)
        layers = []
        max_ratio = 0.0
        for i in range(L):
            ids, _ = probe.route(lp[i])
            freq = torch.bincount(ids.reshape(-1), minlength=E).to(torch.float64)
            torch.distributed.all_reduce(freq)
            slot = plan_placement(E, world, freq.cpu().numpy())
            epr = E // world
            loads = [0.0] * world
            for e in range(E):
                loads[int(slot[e]) // epr] += float(freq[e])
            max_ratio = max(max_ratio, max(loads) / (sum(loads) / world))
            layers.append(EpMoeLayer(shard_layer(uniq[i % len(uniq)], slot, rank, world), num_experts=E, top_k=k,
                                     slot_of_expert=slot, rank=rank, world=world, max_tokens=max(tp, td),
                                     exchange=exchange))
        probe.close()
        res["max_rank_load_over_mean"] = max_ratio

        def step(xs, lg):
            # every rank's token count is at most ceil(global / world): the peer step's work bound
            bound = -(-(n_prefill if xs is xp else n_decode) // world)
            for lay, x, g in zip(layers, xs, lg):
                lay.forward(x, g, comm, tokens_per_rank=bound)
        if exchange is not None:
            res["path"] = ("expert parallel over peer memory: moe_route -> moe_ep_peer_publish -> "
                           "moe_ep_peer_experts (token rows read from every rank's region over NVLink, outputs "
                           "stored into the token's rank's region) -> moe_ep_peer_combine; epoch flags, no host "
                           "read, no collective" + ("; the 48-layer step replayed as one CUDA graph"
                                                    if args.ep_graph else ""))
        else:
            res["path"] = ("expert parallel: moe_ep_dispatch -> NCCL all_to_all -> moe_rows_forward -> "
                           "all_to_all -> moe_ep_combine")

    def timed(xs, lg, steps):
        step(xs, lg)  # warm-up pass
        torch.cuda.synchronize()
        run = lambda: step(xs, lg)  # noqa: E731
        graph = None
        if (exchange is not None or world == 1) and args.ep_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step(xs, lg)
            run = graph.replay
        if torch.distributed.is_initialized():
            torch.distributed.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            run()
        e1.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1) / steps)
        del graph
        return ms

    flops_layer = 2.0 * n_prefill * k * 3 * H * CFG["inter"]
    ms = timed(xp, lp, args.ep_steps)
    res["prefill"] = {"global_tokens": n_prefill, "ms_per_48_layers": ms, "tokens_per_s": n_prefill / (ms / 1e3),
                      "routed_tflops": flops_layer * L / (ms / 1e3) / 1e12}
    ms = timed(xd, ld, 3 * args.ep_steps)
    res["decode"] = {"global_tokens": n_decode, "ms_per_48_layers": ms, "tokens_per_s": n_decode / (ms / 1e3)}
    res["ep_parity"] = ep_parity(layers, uniq, xp, lp, xd, ld, world, rank, tp)
    if exchange is not None:
        res["ep_parity"]["exchange_status"] = exchange.read_status()
    if world == 1 and not args.no_cpu_baseline and args.cpu_seconds > 0:
        res["cpu_baseline"] = ep_cpu_baseline(layers[0], lws[0], xp[0], lp[0], xd[0], ld[0], L, args.cpu_seconds)
    for lay in layers:
        lay.close()
    if exchange is not None:
        exchange.close(barrier=torch.distributed.barrier)
    torch.cuda.empty_cache()
    if world > 1:
        # the N = 1 configuration measured in the same run: every rank puts the
        # whole global batch through the single-GPU path on its own GPU (local
        # work; then every rank takes the same collective steps)
        one = single_gpu_same_run(args, lws, routers, biases, n_prefill, n_decode, dev)
        ok = torch.tensor([1.0 if one is not None else 0.0], device=dev)
        torch.distributed.all_reduce(ok, op=torch.distributed.ReduceOp.MIN)
        p1 = max_over_ranks(one[0] if one is not None else 0.0)
        d1 = max_over_ranks(one[1] if one is not None else 0.0)
        if float(ok.item()) == 1.0:
            res["single_gpu_same_run"] = {
                "prefill_ms_per_48_layers": p1, "decode_ms_per_48_layers": d1,
                "path": "moe_forward per layer, all experts on one GPU, the global batches, max over ranks"}
            res["prefill"]["scaling_efficiency"] = p1 / (world * res["prefill"]["ms_per_48_layers"])
            res["decode"]["scaling_efficiency"] = d1 / (world * res["decode"]["ms_per_48_layers"])
    return res


def single_gpu_same_run(args, lws, routers, biases, n_prefill, n_decode, dev):
    """The global prefill and decode batches through the single-GPU path
    (MoeLayer.forward per layer, every expert local) on this rank's GPU, timed
    like the expert-parallel passes (a CUDA graph of the 48-layer pass when
    --ep-graph).  Local work only.  Returns (prefill ms, decode ms) per pass,
    or None when it could not run (the reason goes to stderr)."""
    import torch

    from nano_ktrans_b200.moe_layer import MoeLayer

    k, H = CFG["top_k"], CFG["hidden"]
    layers1 = []
    try:
        gen = torch.Generator(device=dev).manual_seed(args.seed + 7000)  # the same batches on every rank

        def gbatch(n):
            xs = [torch.randn(n, H, generator=gen, device=dev).to(torch.bfloat16) for _ in range(len(lws))]
            lg = [((x @ r.T).float() + b).to(torch.bfloat16) for x, r, b in zip(xs, routers, biases)]
            return xs, lg

        xp1, lp1 = gbatch(n_prefill)
        xd1, ld1 = gbatch(n_decode)
        layers1 = [MoeLayer(lw, top_k=k, router_use_softmax=True, normalize_topk_prob=True, max_tokens=n_prefill)
                   for lw in lws]

        def time_pass(xs, lg, steps):
            def step():
                for lay, x, g in zip(layers1, xs, lg):
                    lay.forward(x, g)
            step()
            torch.cuda.synchronize()
            run, graph = step, None
            if args.ep_graph:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    step()
                run = graph.replay
                run()
                torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                run()
            e1.record()
            torch.cuda.synchronize()
            del graph
            return e0.elapsed_time(e1) / steps

        return time_pass(xp1, lp1, args.ep_steps), time_pass(xd1, ld1, 3 * args.ep_steps)
    except Exception as exc:  # reported, and the efficiency keys are left out on every rank
        print(f"single-GPU reference pass not run: {exc}", file=sys.stderr, flush=True)
        return None
    finally:
        for lay in layers1:
            lay.close()
        torch.cuda.empty_cache()


def ep_cpu_baseline(layer, lw, xp, lp, xd, ld, n_layers, seconds):
    """The oracle port of the reference CPU path on one layer of the stack
    (the prefill batch sampled by experts, the decode batch by whole steps),
    stated per pass over all n_layers layers (one layer x n_layers)."""
    import torch

    E, k = CFG["experts"], CFG["top_k"]
    ids, w = layer.route(lp)
    pre = prefill_cpu_baseline("c5-layer0", lw, xp, ids, w, None, E, k, xp.shape[0], seconds / 2)
    rate, n, busy = cpu_reference_rate([lw], xd[None], ld[None], seconds / 2, 10 ** 6)
    return {"prefill": {"value": pre["value"] / n_layers, "unit": "tokens/s", "cores": pre["cores"], "kind": "port",
                        "sample": pre["sample"] + f"; one layer x {n_layers}"},
            "decode": {"value": rate / n_layers, "unit": "tokens/s", "cores": blas_threads(), "kind": "port",
                       "sample": f"{n} steps of layer 0 at {xd.shape[0]} tokens ({busy:.1f} s); one layer x "
                                 f"{n_layers}; oracle port of CPUMoEBackend GPTQ path"}}


def ep_parity(layers, uniq, xp, lp, xd, ld, world, rank, max_tokens, n_check: int = 2):
    """Bit-compare the expert-parallel output of this rank's tokens with the
    single-GPU MoeLayer.forward of the same tokens on this rank's GPU, for the
    prefill and decode batches of the first n_check layers; the mismatch
    counts are summed over ranks.  At one rank the expert-parallel layer runs
    with a loopback exchange."""
    import torch

    from nano_ktrans_b200.expert_parallel import (EpMoeLayer, LoopbackComm, TorchDistComm, plan_placement,
                                                  shard_layer)
    from nano_ktrans_b200.moe_layer import MoeLayer

    E, k = CFG["experts"], CFG["top_k"]
    own = []
    if world == 1:
        comm = LoopbackComm()
        slot = plan_placement(E, 1)
        ep = [EpMoeLayer(shard_layer(uniq[i % len(uniq)], slot, 0, 1), num_experts=E, top_k=k,
                         slot_of_expert=slot, rank=0, world=1, max_tokens=max_tokens) for i in range(n_check)]
        own = ep
    else:
        comm = TorchDistComm()
        ep = layers[:n_check]
    # checked tokens, mismatching tokens, mismatching elements, max |difference| (summed / maxed over ranks)
    tokens = torch.zeros(3, dtype=torch.float64, device=xp[0].device)
    worst = torch.zeros(1, dtype=torch.float64, device=xp[0].device)
    for i in range(n_check):
        ref = MoeLayer(uniq[i % len(uniq)], top_k=k, router_use_softmax=True, normalize_topk_prob=True,
                       max_tokens=max_tokens)
        for xs, lg in ((xp, lp), (xd, ld)):
            got = ep[i].forward(xs[i], lg[i], comm)[0].clone()
            want = ref.forward(xs[i], lg[i]).clone()
            diff = got.view(torch.int16) != want.view(torch.int16)
            tokens[0] += got.shape[0]
            tokens[1] += diff.any(dim=1).sum()
            tokens[2] += diff.sum()
            worst = torch.maximum(worst, (got.float() - want.float()).abs().max().double().reshape(1))
        torch.cuda.synchronize()
        ref.close()
    for lay in own:
        lay.close()
    if torch.distributed.is_initialized():
        torch.distributed.all_reduce(tokens)
        torch.distributed.all_reduce(worst, op=torch.distributed.ReduceOp.MAX)
    return {"checked_tokens": int(tokens[0]), "mismatches": int(tokens[1]), "mismatching_elements": int(tokens[2]),
            "max_abs_diff": float(worst[0]), "layers": n_check, "batches": "prefill and decode",
            "compare": "bf16 bit pattern vs MoeLayer.forward on the same GPU", "ranks": world}


def read_traffic(kernel: str, batch: int):
    """DRAM bytes per launch recorded from an ncu capture (profiles/ncu_traffic.txt):
    lines `<kernel> <batch> <bytes_per_launch>`."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    try:
        with open(p) as f:
            for ln in f:
                parts = ln.split()
                if len(parts) >= 3 and not ln.startswith("#") and parts[0] == kernel and int(parts[1]) == batch:
                    return float(parts[2])
    except OSError:
        pass
    return None


if __name__ == "__main__":
    sys.exit(main() or 0)
