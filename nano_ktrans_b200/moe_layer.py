"""``MoeLayer``: one routed-expert MoE layer bound to ``libmoe_b200.so``.

Thin Python owner of a C-ABI handle (include/moe_b200.h).  Tensors cross the
boundary as raw device pointers; every call enqueues on a CUDA stream (the
current torch stream unless one is given) and returns without synchronising.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from .weights import LayerWeights


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream_handle(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class MoeLayer:
    def __init__(self, weights: LayerWeights, *, top_k: int, router_use_softmax: bool = True,
                 normalize_topk_prob: bool = True, max_tokens: int = 4096):
        if not weights.gate_q.is_cuda:
            raise ValueError("MoeLayer weights must be CUDA tensors (there is no CPU path)")
        self.weights = weights
        self.device = weights.gate_q.device
        self.num_experts = weights.num_experts
        self.hidden_size = weights.hidden_size
        self.inter_size = weights.inter_size
        self.top_k = int(top_k)
        self.router_use_softmax = bool(router_use_softmax)
        self.normalize_topk_prob = bool(normalize_topk_prob)
        self.max_tokens = int(max_tokens)
        self._dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        L = _lib.lib()
        desc = _lib.MoeLayerDesc(self.num_experts, self.top_k, self.hidden_size, self.inter_size, weights.bits,
                                 weights.group_size, int(self.router_use_softmax), int(self.normalize_topk_prob),
                                 self.max_tokens, weights.shared_inter)
        handle = ctypes.c_void_p()
        err = ctypes.create_string_buffer(1024)
        with torch.cuda.device(self.device):
            rc = L.moe_create(ctypes.byref(desc), ctypes.byref(handle), err, len(err))
        if rc != _lib.MOE_OK:
            raise _lib.MoeError(rc, err.value.decode())
        self._h = handle
        sh = weights.shared or {}
        w = _lib.MoeWeights(
            _ptr(weights.gate_q), _ptr(weights.gate_s), _ptr(weights.up_q), _ptr(weights.up_s),
            _ptr(weights.down_q), _ptr(weights.down_s),
            _ptr(sh.get("gate_q")), _ptr(sh.get("gate_s")), _ptr(sh.get("up_q")), _ptr(sh.get("up_s")),
            _ptr(sh.get("down_q")), _ptr(sh.get("down_s")), _ptr(sh.get("gate_vec")))
        rc = L.moe_set_weights(self._h, ctypes.byref(w), err, len(err))
        if rc != _lib.MOE_OK:
            L.moe_destroy(self._h)
            self._h = None
            raise _lib.MoeError(rc, err.value.decode())

    @property
    def handle(self):
        return self._h

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().moe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------
    # Argument checks.  Every tensor whose pointer reaches a kernel is checked
    # for device, dtype, exact shape and contiguity first: a wrong buffer must
    # raise here, never be handed to the device as a raw pointer.
    def _on_device(self, t: torch.Tensor) -> bool:
        return t.is_cuda and t.get_device() == self._dev_index

    def _check_tokens(self, x: torch.Tensor) -> int:
        if x.dim() != 2 or x.shape[1] != self.hidden_size:
            raise ValueError(f"expected [T, {self.hidden_size}] activations, got {tuple(x.shape)}")
        if x.dtype is not torch.bfloat16 or not self._on_device(x):
            raise ValueError(f"activations must be bf16 on {self.device}")
        return int(x.shape[0])

    def _check_logits(self, logits: torch.Tensor, t: Optional[int] = None) -> int:
        if logits.dim() != 2 or logits.shape[1] != self.num_experts or (t is not None and logits.shape[0] != t):
            raise ValueError(f"router logits must be [T, {self.num_experts}], got {tuple(logits.shape)}")
        if logits.dtype is not torch.bfloat16 or not self._on_device(logits):
            raise ValueError(f"router logits must be bf16 on {self.device}")
        return int(logits.shape[0])

    def _check_routing_out(self, t: int, out_ids, out_weights) -> None:
        """Caller-provided routing outputs: exactly [T, top_k], int64 ids and bf16 weights,
        contiguous, on this device (the kernels write T * top_k entries into each)."""
        for buf, dt, name in ((out_ids, torch.int64, "out_ids"), (out_weights, torch.bfloat16, "out_weights")):
            if buf is None:
                continue
            if (tuple(buf.shape) != (t, self.top_k) or buf.dtype is not dt or not self._on_device(buf)
                    or not buf.is_contiguous()):
                raise ValueError(f"{name} must be a contiguous {dt} [{t}, {self.top_k}] tensor on {self.device}")

    def _out_for(self, xc: torch.Tensor, out: Optional[torch.Tensor]) -> torch.Tensor:
        """The caller's output buffer after checking that the kernels may write
        [T, H] bf16 into it, or a new one."""
        if out is None:
            return torch.empty_like(xc)
        if (out.shape != xc.shape or out.dtype is not torch.bfloat16 or not self._on_device(out)
                or not out.is_contiguous()):
            raise ValueError(f"out must be a contiguous bf16 {tuple(xc.shape)} tensor on {self.device}")
        return out

    def route(self, router_logits: torch.Tensor, *, out_ids=None, out_weights=None, stream=None):
        t = self._check_logits(router_logits)
        self._check_routing_out(t, out_ids, out_weights)
        logits = router_logits.contiguous()
        ids = out_ids if out_ids is not None else torch.empty(t, self.top_k, dtype=torch.int64, device=self.device)
        w = out_weights if out_weights is not None else torch.empty(t, self.top_k, dtype=torch.bfloat16,
                                                                    device=self.device)
        _lib.check(_lib.lib().moe_route(self._h, logits.data_ptr(), t, ids.data_ptr(), w.data_ptr(),
                                        _stream_handle(stream)), self._h, "moe_route")
        return ids, w

    def experts_forward(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, *,
                        offload_mask: Optional[torch.Tensor] = None, add_shared: bool = False, out=None,
                        stream=None) -> torch.Tensor:
        t = self._check_tokens(x)
        if not self._on_device(topk_ids) or not self._on_device(topk_weights):
            raise ValueError(f"routing tensors must be on {self.device}")
        ids = topk_ids
        if ids.dtype != torch.int64:
            ids = ids.to(torch.int64)
        w = topk_weights
        if w.dtype != torch.bfloat16:
            w = w.to(torch.bfloat16)
        ids, w, xc = ids.contiguous(), w.contiguous(), x.contiguous()
        if tuple(ids.shape) != (t, self.top_k) or tuple(w.shape) != (t, self.top_k):
            raise ValueError(f"routing tensors must be [{t}, {self.top_k}]")
        mask = None
        if offload_mask is not None:
            if offload_mask.numel() != self.num_experts:
                raise ValueError(f"offload_mask must hold {self.num_experts} entries")
            mask = offload_mask.reshape(-1).to(device=self.device, dtype=torch.uint8).contiguous()
        out = self._out_for(xc, out)
        _lib.check(_lib.lib().moe_experts_forward(self._h, xc.data_ptr(), ids.data_ptr(), w.data_ptr(), t,
                                                  _ptr(mask), int(add_shared), out.data_ptr(),
                                                  _stream_handle(stream)), self._h, "moe_experts_forward")
        return out

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor, *, out=None, out_ids=None, out_weights=None,
                stream=None) -> torch.Tensor:
        t = self._check_tokens(x)
        self._check_logits(router_logits, t)
        self._check_routing_out(t, out_ids, out_weights)
        xc, lc = x.contiguous(), router_logits.contiguous()
        out = self._out_for(xc, out)
        _lib.check(_lib.lib().moe_forward(self._h, xc.data_ptr(), lc.data_ptr(), t, out.data_ptr(), _ptr(out_ids),
                                          _ptr(out_weights), _stream_handle(stream)), self._h, "moe_forward")
        return out

    def forward_host(self, x: torch.Tensor, router_logits: torch.Tensor, out: torch.Tensor, stream=None) -> None:
        """forward() on host tensors (bf16, contiguous, ideally pinned): copies in,
        runs the step and copies the result into `out`, all enqueued on the
        stream — `out` is valid after the stream is synchronised."""
        # one combined test on the per-step path (a few attribute reads per tensor);
        # the per-tensor loop below only names the offending argument
        bf, t = torch.bfloat16, x.shape[0] if x.dim() == 2 else -1
        if not (x.is_cpu and router_logits.is_cpu and out.is_cpu and x.dtype is bf and router_logits.dtype is bf
                and out.dtype is bf and x.shape == (t, self.hidden_size)
                and router_logits.shape == (t, self.num_experts) and out.shape == (t, self.hidden_size)
                and x.is_contiguous() and router_logits.is_contiguous() and out.is_contiguous()):
            for name, tsr, cols in (("x", x, self.hidden_size), ("router_logits", router_logits, self.num_experts),
                                    ("out", out, self.hidden_size)):
                if (tsr.device.type != "cpu" or tsr.dtype is not bf or tsr.dim() != 2
                        or tsr.shape[1] != cols or tsr.shape[0] != t or not tsr.is_contiguous()):
                    raise ValueError(f"{name} must be a contiguous bf16 host tensor [T, {cols}]")
            raise ValueError("x, router_logits and out must be contiguous bf16 host tensors of T rows")
        _lib.check(_lib.lib().moe_forward_host(self._h, x.data_ptr(), router_logits.data_ptr(), int(x.shape[0]),
                                               out.data_ptr(), _stream_handle(stream)), self._h, "moe_forward_host")

    def _check_router(self, router_weight: torch.Tensor) -> None:
        if (not self._on_device(router_weight) or router_weight.dtype != torch.bfloat16
                or tuple(router_weight.shape) != (self.num_experts, self.hidden_size)
                or not router_weight.is_contiguous()):
            raise ValueError(f"router weight must be a contiguous bf16 [{self.num_experts}, {self.hidden_size}] "
                             f"tensor on {self.device}")

    def router_logits(self, x: torch.Tensor, router_weight: torch.Tensor, *, out=None, stream=None) -> torch.Tensor:
        """bf16(x . router_weight^T) with fp32 accumulation: the reference's
        `self.gate(hidden_states)` (nano_ktrans/models/mixtral.py:127, :212)."""
        t = self._check_tokens(x)
        self._check_router(router_weight)
        xc = x.contiguous()
        if out is None:
            out = torch.empty(t, self.num_experts, dtype=torch.bfloat16, device=self.device)
        elif (not self._on_device(out) or out.dtype != torch.bfloat16 or tuple(out.shape) != (t, self.num_experts)
              or not out.is_contiguous()):
            raise ValueError(f"out must be a contiguous bf16 [{t}, {self.num_experts}] tensor on {self.device}")
        _lib.check(_lib.lib().moe_router_logits(self._h, xc.data_ptr(), router_weight.data_ptr(), t, out.data_ptr(),
                                                _stream_handle(stream)), self._h, "moe_router_logits")
        return out

    def forward_x(self, x: torch.Tensor, router_weight: torch.Tensor, *, out=None, out_ids=None, out_weights=None,
                  out_logits=None, stream=None) -> torch.Tensor:
        """The MoE block from hidden states: router projection, routing, routed
        experts and combine (models/mixtral.py:212-218 with every expert on
        this backend).  out_logits, when given, receives the router logits."""
        t = self._check_tokens(x)
        self._check_router(router_weight)
        self._check_routing_out(t, out_ids, out_weights)
        if out_logits is not None:
            self._check_logits(out_logits, t)
            if not out_logits.is_contiguous():
                raise ValueError("out_logits must be contiguous")
        xc = x.contiguous()
        out = self._out_for(xc, out)
        _lib.check(_lib.lib().moe_forward_x(self._h, xc.data_ptr(), router_weight.data_ptr(), t, out.data_ptr(),
                                            _ptr(out_ids), _ptr(out_weights), _ptr(out_logits),
                                            _stream_handle(stream)), self._h, "moe_forward_x")
        return out

    def dequant_rows(self, proj: int, expert: int, row0: int, nrows: int, stream=None) -> torch.Tensor:
        k = self.hidden_size if proj in (0, 1, 3, 4) else (self.inter_size if proj == 2 else
                                                            self.weights.shared_inter)
        out = torch.empty(nrows, k, dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().moe_dequant_rows(self._h, proj, expert, row0, nrows, out.data_ptr(),
                                               _stream_handle(stream)), self._h, "moe_dequant_rows")
        return out

    def read_status(self, stream=None) -> int:
        st = ctypes.c_int32(0)
        _lib.check(_lib.lib().moe_read_status(self._h, ctypes.byref(st), _stream_handle(stream)), self._h,
                   "moe_read_status")
        return int(st.value)

    def set_decode_fused(self, mode) -> None:
        """Small batches as one cooperative launch: True/1 (default; the single-token
        kernel for T == 1 where it applies), 2 (the multi-token kernel also for T == 1),
        False/0 (always the multi-kernel chain)."""
        _lib.check(_lib.lib().moe_set_option(self._h, _lib.OPT_DECODE_FUSED, int(mode)), self._h, "moe_set_option")

    def set_gemm(self, mode: int) -> None:
        """Expert projections of the multi-kernel path: 0 matvec only, 1 tensor-core
        grouped GEMM for large batches (default), 2 grouped GEMM for every batch."""
        _lib.check(_lib.lib().moe_set_option(self._h, _lib.OPT_GEMM, int(mode)), self._h, "moe_set_option")

    def set_stream(self, enabled: bool) -> None:
        """Expert projections of the multi-kernel path below the GEMM threshold:
        True (default) the weight-streaming tensor-core kernels where the layer's
        shapes allow, False the CUDA-core matvec kernels."""
        _lib.check(_lib.lib().moe_set_option(self._h, _lib.OPT_STREAM, int(bool(enabled))), self._h,
                   "moe_set_option")

    def set_host_io(self, mode: int) -> None:
        """forward_host with page-locked buffers: 0 copy-engine copies, 1 a kernel
        reads the inputs from mapped host memory, 2 (default) also the output is
        stored straight into host memory."""
        _lib.check(_lib.lib().moe_set_option(self._h, _lib.OPT_HOST_IO, int(mode)), self._h, "moe_set_option")

    def set_gemm_tile(self, width: int) -> None:
        """Token-tile width of the grouped GEMM: 0 chooses by batch, else 16, 32, 64 or 128."""
        _lib.check(_lib.lib().moe_set_option(self._h, _lib.OPT_GEMM_TILE, int(width)), self._h, "moe_set_option")

    def set_trace(self, enabled: bool) -> None:
        """Record per-CTA phase timestamps in the single-launch decode kernel."""
        _lib.check(_lib.lib().moe_set_option(self._h, _lib.OPT_TRACE, int(bool(enabled))), self._h, "moe_set_option")

    def read_trace(self, stream=None):
        """[num_ctas][16] phase stamps of the last traced single-token decode launch.

        Column 0 is %globaltimer at CTA entry (ns); columns 1-12 are SM clock cycles since
        entry: inputs landed, routing done, chunk table built, prologue done, copies
        requested, own gate/up rows done, h written, grid barrier passed, h staged, down
        blocks landed, down rows done, exit."""
        import numpy as np

        buf = (ctypes.c_uint64 * (1024 * 16))()
        n = ctypes.c_int32(0)
        _lib.check(_lib.lib().moe_read_trace(self._h, buf, len(buf), ctypes.byref(n), _stream_handle(stream)),
                   self._h, "moe_read_trace")
        return np.frombuffer(buf, dtype=np.uint64)[: n.value * 16].reshape(n.value, 16).copy()

    def profile_begin(self, kernel_class: int, max_samples: int) -> None:
        _lib.check(_lib.lib().moe_profile_begin(self._h, kernel_class, max_samples), self._h, "moe_profile_begin")

    def profile_end(self):
        """(summed kernel ms, number of bracketed launches)"""
        ms = ctypes.c_float(0.0)
        n = ctypes.c_int32(0)
        _lib.check(_lib.lib().moe_profile_end(self._h, ctypes.byref(ms), ctypes.byref(n)), self._h, "moe_profile_end")
        return float(ms.value), int(n.value)

    def last_launch_count(self) -> int:
        return int(_lib.lib().moe_last_launch_count(self._h))
