"""ctypes binding of ``libmoe_b200.so`` (declared in ``include/moe_b200.h``).

The library is loaded from this package directory.  There is no fallback: if
the library is missing the import of any compute entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import re

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libmoe_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(PKG_DIR), "include", "moe_b200.h")

MOE_OK, MOE_EINVAL, MOE_ECUDA, MOE_ENOWEIGHTS, MOE_ERANGE, MOE_EDEVICE = range(6)
K_ROUTE, K_PERMUTE, K_GATEUP, K_DOWN, K_COMBINE, K_DECODE_FUSED = range(1, 7)
OPT_DECODE_FUSED, OPT_TRACE, OPT_GEMM, OPT_GEMM_TILE, OPT_STREAM, OPT_HOST_IO = 1, 2, 3, 4, 5, 6

_DESC_FIELDS = ("num_experts", "top_k", "hidden_size", "inter_size", "bits", "group_size",
                "router_use_softmax", "normalize_topk_prob", "max_tokens", "shared_inter")
_WEIGHT_FIELDS = ("gate_q_dev", "gate_s_dev", "up_q_dev", "up_s_dev", "down_q_dev", "down_s_dev",
                  "shared_gate_q_dev", "shared_gate_s_dev", "shared_up_q_dev", "shared_up_s_dev",
                  "shared_down_q_dev", "shared_down_s_dev", "shared_gate_vec_dev")


class MoeLayerDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in _DESC_FIELDS]


class MoeWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in _WEIGHT_FIELDS]


class MoeError(RuntimeError):
    """A C-ABI call returned a nonzero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[moe_b200 status {code}] {message}")
        self.code = code


_vp, _i32, _sz, _cp = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t, ctypes.c_char_p

# name -> (restype, argtypes)
SIGNATURES = {
    "moe_abi_version": (_i32, []),
    "moe_create": (_i32, [ctypes.POINTER(MoeLayerDesc), ctypes.POINTER(_vp), _cp, _sz]),
    "moe_set_weights": (_i32, [_vp, ctypes.POINTER(MoeWeights), _cp, _sz]),
    "moe_route": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp]),
    "moe_experts_forward": (_i32, [_vp, _vp, _vp, _vp, _i32, _vp, _i32, _vp, _vp]),
    "moe_forward": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp]),
    "moe_forward_host": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp]),
    "moe_router_logits": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp]),
    "moe_forward_x": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp]),
    "moe_dequant_rows": (_i32, [_vp, _i32, _i32, _i32, _i32, _vp, _vp]),
    "moe_read_status": (_i32, [_vp, ctypes.POINTER(_i32), _vp]),
    "moe_last_launch_count": (_i32, [_vp]),
    "moe_profile_begin": (_i32, [_vp, _i32, _i32]),
    "moe_set_option": (_i32, [_vp, _i32, _i32]),
    "moe_read_trace": (_i32, [_vp, ctypes.POINTER(ctypes.c_uint64), _i32, ctypes.POINTER(_i32), _vp]),
    "moe_profile_end": (_i32, [_vp, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(_i32)]),
    "moe_last_error": (_i32, [_vp, _cp, _sz]),
    "moe_destroy": (None, [_vp]),
    "moe_decode_noalloc": (_i32, [ctypes.POINTER(MoeLayerDesc), ctypes.POINTER(MoeWeights), _vp, _vp, _i32, _vp, _vp,
                                  _vp, _vp, _vp, _cp, _sz]),
    "moe_ep_dispatch": (_i32, [_vp, _vp, _vp, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _vp]),
    "moe_rows_forward": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp]),
    "moe_ep_combine": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp, _vp]),
    "moe_ep_group_create": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, ctypes.POINTER(_vp), _cp, _sz]),
    "moe_ep_group_ipc_handle": (_i32, [_vp, _vp]),
    "moe_ep_group_open_peer": (_i32, [_vp, _i32, _vp]),
    "moe_ep_group_region": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "moe_ep_group_set_peer": (_i32, [_vp, _i32, _vp]),
    "moe_ep_peer_publish": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp]),
    "moe_ep_peer_experts": (_i32, [_vp, _vp, _i32, _i32, _vp]),
    "moe_ep_peer_combine": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp]),
    "moe_ep_group_read_status": (_i32, [_vp, ctypes.POINTER(_i32), _vp]),
    "moe_ep_group_last_error": (_i32, [_vp, _cp, _sz]),
    "moe_ep_group_close_peers": (_i32, [_vp]),
    "moe_ep_group_destroy": (_i32, [_vp]),
}

EP_IPC_HANDLE_BYTES = 64
EP_STATUS_BAD_ID, EP_STATUS_TIMEOUT, EP_STATUS_OVERFLOW = 1, 2, 4

_lib = None


def header_symbols() -> list[str]:
    """Function names declared in include/moe_b200.h."""
    with open(HEADER_PATH) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:int|void)\s+(moe_\w+)\s*\(", text, flags=re.M)))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built; run `python -m nano_ktrans_b200.build` "
                               "(there is no CPU fallback for this path)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        if L.moe_abi_version() != 1:
            raise RuntimeError("libmoe_b200.so ABI version mismatch")
        _lib = L
    return _lib


def last_error(handle) -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().moe_last_error(handle, buf, len(buf))
    return buf.value.decode(errors="replace")


def group_error(group) -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().moe_ep_group_last_error(group, buf, len(buf))
    return buf.value.decode(errors="replace")


def check_group(rc: int, group, what: str) -> None:
    if rc != MOE_OK:
        raise MoeError(rc, f"{what}: {group_error(group) if group else ''}")


def check(rc: int, handle=None, what: str = "") -> None:
    if rc != MOE_OK:
        msg = last_error(handle) if handle else ""
        raise MoeError(rc, f"{what}: {msg}" if what else msg)
