"""ctypes binding of ``libmoe_b200.so`` (the C ABI declared in include/moe_b200.h).

The library is loaded from the package's ``_lib`` directory.  There is no
fallback: if it is missing or fails to load, every operation raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "_lib", "libmoe_b200.so")

MOE_OK = 0
MOE_ERR_INVALID = -1
MOE_ERR_UNSUPPORTED = -2
MOE_ERR_WORKSPACE = -3
MOE_ERR_CUDA = -4
MOE_ERR_DEVICE = -5

MOE_F32 = 0
MOE_Q4_0 = 2
MOE_Q5_1 = 7
MOE_Q8_0 = 8
MOE_Q4_K = 12
MOE_Q6_K = 14
MOE_ACT_SWIGLU = 0
MOE_ACT_GEGLU_TANH = 1
MOE_KERNELS_AUTO, MOE_KERNELS_GEMV, MOE_KERNELS_BLOCKSCALE, MOE_KERNELS_SPLIT_GEMM = 0, 1, 2, 3
MOE_ROUTE_TOPK_SOFTMAX = 0
MOE_ROUTE_SOFTMAX_TOPK_RENORM = 1
MOE_ROUTER_D_E = 0
MOE_ROUTER_E_D = 1

MOE_STATUS_BAD_EXPERT_ID = 1
MOE_STATUS_ROW_OVERFLOW = 2
MOE_STATUS_TIMEOUT = 4

vp = ctypes.c_void_p
ci = ctypes.c_int
csz = ctypes.c_size_t
ci64 = ctypes.c_int64
cf = ctypes.c_float


class MoEExpertOpts(ctypes.Structure):
    """Mirror of ``moe_expert_opts``."""
    _fields_ = [("act", ci), ("down_qtype", ci), ("gate_up_stride", csz), ("down_scale", vp),
                ("kernels", ci), ("chunk_rows", ci)]


class MoELayerWeights(ctypes.Structure):
    """Mirror of ``moe_layer_weights``."""
    _fields_ = [
        ("gate_w", vp), ("bias", vp), ("w_gate", vp), ("w_up", vp), ("w_down", vp),
        ("s_gate", vp), ("s_up", vp), ("s_down", vp),
        ("router_layout", ci), ("qtype", ci), ("shared_qtype", ci),
        ("E", ci), ("k", ci), ("d", ci), ("F", ci), ("Fs", ci), ("mode", ci),
        ("opts", ctypes.POINTER(MoEExpertOpts)),
    ]


# name -> (argtypes) ; every function returns int
SIGNATURES = {
    "moe_version": [],
    "moe_last_error": [ctypes.c_char_p, csz],
    "moe_block_geometry": [ci, ctypes.POINTER(ci), ctypes.POINTER(ci)],
    "moe_read_status": [vp, ctypes.POINTER(ci), vp],
    "moe_profile_enable": [ci],
    "moe_profile_collect": [ctypes.POINTER(cf), ctypes.POINTER(ci), ci],
    "moe_dequantize": [vp, vp, ci, ci64, vp],
    "moe_packed_bytes": [ci, ci, ci, ci, ctypes.POINTER(csz)],
    "moe_pack_weights": [vp, vp, ci, ci, ci, ci, vp],
    "moe_unpack_weights": [vp, vp, ci, ci, ci, ci, vp],
    "moe_router_workspace_bytes": [ci, ci, ci, ctypes.POINTER(csz)],
    "moe_router": [vp, vp, vp, ci, ci, ci, ci, ci, ci, vp, vp, vp, csz, vp],
    "moe_router_noalloc": [vp, vp, vp, ci, ci, ci, ci, ci, ci, vp, vp, vp],
    "moe_dispatch_workspace_bytes": [ci, ci, ci, ctypes.POINTER(csz)],
    "moe_dispatch": [vp, ci, ci, ci, vp, vp, vp, vp, csz, vp],
    "moe_experts_workspace_bytes": [ci, ci, ci, ci, ctypes.POINTER(csz)],
    "moe_experts": [vp, vp, vp, ci, vp, ci, ci, vp, vp, ci, ci, ci, vp, vp, vp, csz, vp],
    "moe_experts_ex": [vp, vp, vp, ci, ctypes.POINTER(MoEExpertOpts), vp, ci, ci, vp, vp, ci, ci,
                       ci, vp, vp, vp, csz, vp],
    "moe_router_input": [vp, vp, cf, ci, ci, vp, vp],
    "moe_layer_forward_ex": [ctypes.POINTER(MoELayerWeights), vp, vp, ci, vp, vp, vp, vp, vp, csz,
                             vp],
    "moe_combine": [vp, vp, vp, vp, vp, ci, ci, ci, vp, vp],
    "moe_rms_norm": [vp, vp, cf, ci, ci, vp, vp],
    "moe_rms_norm_ex": [vp, vp, cf, ci, ci, ci, vp, vp],
    "moe_gather_rows": [vp, vp, ci, ci, ci, vp, vp],
    "moe_ep_local_order": [vp, ci, ci, ci, vp, vp, vp, vp],
    "moe_ipc_alloc": [csz, ctypes.POINTER(ctypes.c_void_p)],
    "moe_ipc_free": [vp],
    "moe_ipc_handle": [vp, vp],
    "moe_ipc_open": [vp, ctypes.POINTER(ctypes.c_void_p)],
    "moe_ipc_close": [vp],
    "moe_ep_window_bytes": [ci, ci, ci, ci, ci, ctypes.POINTER(csz)],
    "moe_ep_workspace_bytes": [vp, ci, ci, ctypes.POINTER(csz)],
    "moe_ep_forward": [vp, ci, ci, vp, vp, vp, ci, vp, vp, ci, vp, csz, vp],
    "moe_ep_forward_phases": [vp, ci, ci, vp, vp, vp, ci, vp, vp, ci, ci, vp, csz, vp],
    "moe_layer_workspace_bytes": [ctypes.POINTER(MoELayerWeights), ci, ctypes.POINTER(csz)],
    "moe_layer_forward": [ctypes.POINTER(MoELayerWeights), vp, ci, vp, vp, vp, vp, vp, csz, vp],
}


KERNEL_NAMES = ["router", "router_select", "dispatch", "plan", "xprep", "gateup", "down",
                "combine", "rms_norm", "pack", "dequant", "aux", "ep_send", "ep_recv_plan",
                "ep_return", "ep_wait"]

MOE_EP_PHASE_SEND = 1
MOE_EP_PHASE_SERVE = 2
MOE_EP_PHASE_COMBINE = 4
MOE_EP_PHASE_ALL = 7


def profile_enable(on: bool) -> None:
    check(load().moe_profile_enable(1 if on else 0))


def profile_collect():
    """{kernel name: (total device ms, launches)} since the last collect."""
    n = len(KERNEL_NAMES)
    ms = (cf * n)()
    cnt = (ci * n)()
    check(load().moe_profile_collect(ms, cnt, n))
    return {KERNEL_NAMES[i]: (float(ms[i]), int(cnt[i])) for i in range(n)}


class MoEError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"moe status {status}: {message}")
        self.status = status


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Loads the library once; raises if it is absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m linuxnightmaresuite_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ci
        _lib = lib
        return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    load().moe_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != MOE_OK:
        raise MoEError(status, last_error())


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
