"""Quantized-weight container and its device layout.

``GPTQLinearWeight`` keeps the reference container's fields and methods
(nano_ktrans/kernels/weight_loader.py:25-69): ``qweight`` int32
``[N, K*bits/32]`` with codes LSB-first along K, ``scales`` ``[N, K/group]``,
implicit zero point ``2^(bits-1)`` when ``zero_points`` is None.

``quantize_symmetric`` is the reference quantizer
(nano_ktrans/kernels/quantized_ops.py:17-59) generalised to bits=8 (the
reference raises for bits != 4 at :24-25, while its container and matvec are
bit-width generic), with an option to round the stored scales to bf16.

``LayerWeights`` is the device layout the kernels read: for each projection
the qweight bytes stacked over experts, ``uint8 [E, N, K*bits/8]`` (exactly
the little-endian bytes of the int32 words, so no repacking), and the scales
as ``bf16 [E, N, SS]`` with SS = K/group rounded up to 8 (16-byte rows).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch


@dataclass
class GPTQLinearWeight:
    qweight: torch.Tensor
    scales: torch.Tensor
    zero_points: Optional[torch.Tensor]
    group_size: int
    bits: int
    sym: bool
    linear_prefix: str

    @property
    def input_dim(self) -> int:
        return int(self.qweight.shape[1]) * self.values_per_word

    @property
    def output_dim(self) -> int:
        return int(self.qweight.shape[0])

    @property
    def num_groups(self) -> int:
        return int(self.scales.shape[1])

    @property
    def values_per_word(self) -> int:
        return 32 // self.bits

    def unpack_qvalues(self) -> torch.Tensor:
        shifts = torch.arange(self.values_per_word, dtype=torch.int32, device=self.qweight.device) * self.bits
        packed = self.qweight.to(dtype=torch.int32).contiguous()
        unpacked = ((packed.unsqueeze(-1) >> shifts) & ((1 << self.bits) - 1)).to(dtype=torch.float32)
        return unpacked.reshape(self.output_dim, self.qweight.shape[1] * self.values_per_word)

    def dequantize(self) -> torch.Tensor:
        q = self.unpack_qvalues()
        zero = float(1 << (self.bits - 1))
        gs = min(self.group_size, self.input_dim)
        s = self.scales.to(torch.float32).repeat_interleave(gs, dim=1)[:, : self.input_dim]
        if self.zero_points is not None:
            z = self.zero_points.to(torch.float32).repeat_interleave(gs, dim=1)[:, : self.input_dim]
            return (q - z) * s
        return (q - zero) * s


def pack_codes(qvalues: torch.Tensor, bits: int) -> torch.Tensor:
    """Pack uint8 codes [N, K] into int32 words LSB-first (quantized_ops.py:62-72 at any bit width)."""
    n, k = qvalues.shape
    vpw = 32 // bits
    if k % vpw:
        raise ValueError(f"input_dim {k} must be divisible by {vpw} for {bits}-bit packing")
    words = qvalues.to(torch.int64).reshape(n, k // vpw, vpw)
    shifts = (torch.arange(vpw, dtype=torch.int64, device=qvalues.device) * bits).view(1, 1, vpw)
    packed = torch.sum(words << shifts, dim=2)
    packed = torch.where(packed >= 2**31, packed - 2**32, packed)
    return packed.to(torch.int32).contiguous()


def quantize_symmetric(weight: torch.Tensor, *, group_size: int = 128, bits: int = 4,
                       scale_dtype: torch.dtype = torch.bfloat16,
                       linear_prefix: str = "synthetic") -> GPTQLinearWeight:
    """Symmetric per-group quantizer (quantized_ops.py:17-59), bits 4 or 8.

    Scales and codes are computed in fp32 exactly as the reference does; the
    stored scales are then rounded to ``scale_dtype`` (bf16 for the
    benchmark configurations) and kept as fp32 values in the container.
    ``group_size=0`` means one group per output channel.
    """
    if bits not in (4, 8):
        raise NotImplementedError("Only 4- and 8-bit symmetric quantization is supported.")
    w = weight.to(torch.float32).contiguous()
    n, k = w.shape
    g = k if group_size in (0, None) else group_size
    if k % g:
        raise ValueError("input_dim must be divisible by group_size")
    qmax = (1 << (bits - 1)) - 1
    chunks = w.view(n, k // g, g)
    max_abs = chunks.abs().amax(dim=2).clamp(min=1e-6)
    scales = max_abs / qmax
    q = torch.round(chunks / scales.unsqueeze(2)).clamp(-(1 << (bits - 1)), qmax)
    codes = (q + (1 << (bits - 1))).to(torch.uint8).view(n, k)
    scales = scales.to(scale_dtype).to(torch.float32)
    return GPTQLinearWeight(qweight=pack_codes(codes, bits), scales=scales.contiguous(), zero_points=None,
                            group_size=g, bits=bits, sym=True, linear_prefix=linear_prefix)


def scale_stride(num_groups: int) -> int:
    """bf16 scale elements per row on the device: groups rounded up to 8 (16 bytes)."""
    return (num_groups + 7) // 8 * 8


def pad_scales(s: torch.Tensor) -> torch.Tensor:
    """[..., G] -> [..., scale_stride(G)] bf16, zero padding."""
    g = s.shape[-1]
    out = torch.zeros(*s.shape[:-1], scale_stride(g), dtype=torch.bfloat16, device=s.device)
    out[..., :g] = s.to(torch.bfloat16)
    return out


def _codes_bytes(w: GPTQLinearWeight) -> torch.Tensor:
    return w.qweight.contiguous().view(torch.uint8)


def _check(w: GPTQLinearWeight, n: int, k: int, bits: int, name: str) -> None:
    if w.bits != bits:
        raise ValueError(f"{name}: bits {w.bits} != layer bits {bits}")
    if w.zero_points is not None or not w.sym:
        raise NotImplementedError(f"{name}: only symmetric GPTQ weights (implicit zero point) are supported")
    if (w.output_dim, w.input_dim) != (n, k):
        raise ValueError(f"{name}: shape {(w.output_dim, w.input_dim)} != expected {(n, k)}")


@dataclass
class LayerWeights:
    """Device-resident stacked expert weights of one MoE layer."""

    bits: int
    group_size: int  # 0 = per output channel
    gate_q: torch.Tensor
    gate_s: torch.Tensor
    up_q: torch.Tensor
    up_s: torch.Tensor
    down_q: torch.Tensor
    down_s: torch.Tensor
    shared: Optional[dict] = None  # {"gate_q","gate_s","up_q","up_s","down_q","down_s","gate_vec"}
    keepalive: list = field(default_factory=list)

    @property
    def num_experts(self) -> int:
        return int(self.gate_q.shape[0])

    @property
    def inter_size(self) -> int:
        return int(self.gate_q.shape[1])

    @property
    def hidden_size(self) -> int:
        return int(self.down_q.shape[1])

    @property
    def shared_inter(self) -> int:
        return 0 if self.shared is None else int(self.shared["gate_q"].shape[1])

    def expert_bytes(self) -> int:
        """Packed code + scale bytes of one routed expert (all three projections)."""
        per = 0
        for q, s in ((self.gate_q, self.gate_s), (self.up_q, self.up_s), (self.down_q, self.down_s)):
            per += q[0].numel() + q.shape[1] * self.groups(q) * 2
        return per

    def groups(self, q: torch.Tensor) -> int:
        """Scale groups per row of a projection whose codes are ``q``."""
        k = q.shape[2] * 8 // self.bits
        return 1 if self.group_size == 0 else k // self.group_size

    def shared_bytes(self) -> int:
        if self.shared is None:
            return 0
        return sum(self.shared[p + "_q"].numel() + self.shared[p + "_q"].shape[1] * self.groups(self.shared[p + "_q"]) * 2
                   for p in ("gate", "up", "down"))


def layer_group_size(experts: list[dict]) -> int:
    """0 when every projection is per-channel (one group spanning its K)."""
    ws = [w for ex in experts for w in ex.values()]
    if all(w.num_groups == 1 for w in ws):
        return 0
    g = min(w.input_dim // w.num_groups for w in ws)
    for w in ws:
        if w.input_dim % g or w.num_groups != w.input_dim // g:
            raise ValueError(f"projection {w.linear_prefix}: K={w.input_dim} with {w.num_groups} groups "
                             f"does not match the layer group size {g}")
    return g


def stack_layer(experts: list[dict], device, shared: Optional[dict] = None,
                shared_gate_vec: Optional[torch.Tensor] = None) -> LayerWeights:
    """Stack per-expert ``{"gate","up","down": GPTQLinearWeight}`` into the device layout."""
    if not experts:
        raise ValueError("no experts")
    bits = experts[0]["gate"].bits
    h = experts[0]["gate"].input_dim
    i = experts[0]["gate"].output_dim
    for e, ex in enumerate(experts):
        _check(ex["gate"], i, h, bits, f"expert {e} gate")
        _check(ex["up"], i, h, bits, f"expert {e} up")
        _check(ex["down"], h, i, bits, f"expert {e} down")
    group = layer_group_size(experts + ([shared] if shared else []))

    def stack(proj: str):
        q = torch.stack([_codes_bytes(ex[proj]) for ex in experts]).to(device).contiguous()
        s = torch.stack([ex[proj].scales.to(torch.float32) for ex in experts])
        return q, pad_scales(s).to(device).contiguous()

    gq, gsc = stack("gate")
    uq, usc = stack("up")
    dq, dsc = stack("down")
    sh = None
    if shared is not None:
        si = shared["gate"].output_dim
        _check(shared["gate"], si, h, bits, "shared gate")
        _check(shared["up"], si, h, bits, "shared up")
        _check(shared["down"], h, si, bits, "shared down")
        if shared_gate_vec is None:
            raise ValueError("a shared expert needs its sigmoid gate vector")
        sh = {}
        for p in ("gate", "up", "down"):
            sh[p + "_q"] = _codes_bytes(shared[p]).unsqueeze(0).to(device).contiguous()
            sh[p + "_s"] = pad_scales(shared[p].scales.to(torch.float32).unsqueeze(0)).to(device).contiguous()
        sh["gate_vec"] = shared_gate_vec.reshape(-1).to(torch.bfloat16).to(device).contiguous()
    return LayerWeights(bits=bits, group_size=group, gate_q=gq, gate_s=gsc, up_q=uq, up_s=usc,
                        down_q=dq, down_s=dsc, shared=sh)
