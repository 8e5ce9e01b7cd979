"""Torch-tensor wrappers over the C ABI.

Every function takes CUDA tensors, allocates outputs and workspaces with torch
and enqueues the library's kernels on the current CUDA stream.  Inputs that
are not contiguous CUDA tensors of the right dtype are rejected.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import call

QTYPE_F32 = _lib.MOE_F32
QTYPE_Q4_0 = _lib.MOE_Q4_0
QTYPE_Q5_1 = _lib.MOE_Q5_1
QTYPE_Q8_0 = _lib.MOE_Q8_0
QTYPE_Q4_K = _lib.MOE_Q4_K
QTYPE_Q6_K = _lib.MOE_Q6_K
ACT_SWIGLU = _lib.MOE_ACT_SWIGLU
ACT_GEGLU_TANH = _lib.MOE_ACT_GEGLU_TANH
KERNELS_AUTO = _lib.MOE_KERNELS_AUTO
KERNELS_GEMV = _lib.MOE_KERNELS_GEMV
KERNELS_BLOCKSCALE = _lib.MOE_KERNELS_BLOCKSCALE
KERNELS_SPLIT_GEMM = _lib.MOE_KERNELS_SPLIT_GEMM
# GGML type -> (weights per block, bytes per block), dequant_fast.py:723-754
BLOCK_GEOMETRY = {QTYPE_F32: (1, 4), QTYPE_Q4_0: (32, 18), QTYPE_Q5_1: (32, 24),
                  QTYPE_Q8_0: (32, 34), QTYPE_Q4_K: (256, 144), QTYPE_Q6_K: (256, 210)}
BLOCK_BYTES = {QTYPE_Q4_0: 18, QTYPE_Q8_0: 34}
PACKED_QTYPES = (QTYPE_Q4_0, QTYPE_Q8_0)


def row_bytes(qtype: int, cols: int) -> int:
    e, b = BLOCK_GEOMETRY[qtype]
    if cols % e:
        raise ValueError(f"row of {cols} weights is not whole blocks of type {qtype}")
    return cols // e * b


def packed_path(qtype: int, down_qtype: int) -> bool:
    """Whether a layer's expert matrices are repacked into MMA tiles (Q4_0 /
    Q8_0 on all three) or used as stored (every other combination)."""
    return qtype in PACKED_QTYPES and down_qtype == qtype


class ExpertOpts:
    """Expert variant (``moe_expert_opts``): activation, down matrix type,
    gate/up stride of a fused stack, per-expert down scale (device f32), and
    the kernel family (``KERNELS_*``, 0 = automatic) with its chunk rows."""

    def __init__(self, act: int = ACT_SWIGLU, down_qtype: int = 0, gate_up_stride: int = 0,
                 down_scale: Optional[torch.Tensor] = None, kernels: int = 0,
                 chunk_rows: int = 0):
        if down_scale is not None:
            _need(down_scale, torch.float32, "down_scale")
        self.down_scale = down_scale
        self.c = _lib.MoEExpertOpts(act, down_qtype, gate_up_stride,
                                    0 if down_scale is None else down_scale.data_ptr(),
                                    kernels, chunk_rows)

    @property
    def ref(self):
        return ctypes.byref(self.c)


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _need(t: torch.Tensor, dtype, name: str, pinned_ok: bool = False) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not (t.is_cuda or (pinned_ok and t.is_pinned())):
        raise TypeError(f"{name} must be a CUDA tensor" + (" or pinned host memory"
                                                          if pinned_ok else ""))
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def _size_out(fn: str, *args) -> int:
    out = ctypes.c_size_t(0)
    call(fn, *args, ctypes.byref(out))
    return int(out.value)


def workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def block_geometry(qtype: int) -> Tuple[int, int]:
    e, b = ctypes.c_int(0), ctypes.c_int(0)
    call("moe_block_geometry", qtype, ctypes.byref(e), ctypes.byref(b))
    return e.value, b.value


# --------------------------------------------------------------------------- weights

def router_input(x: torch.Tensor, scale: Optional[torch.Tensor], eps: float = 1e-6,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """gemma4's router input, x / sqrt(mean(x^2) + eps) * f32(1/sqrt(d)) * scale
    (nightmare_stream.py:4662-4667)."""
    _need(x, torch.float32, "x")
    if scale is not None:
        _need(scale, torch.float32, "scale")
    T, d = x.shape
    if out is None:
        out = torch.empty_like(x)
    call("moe_router_input", _ptr(x), _ptr(scale), ctypes.c_float(eps), T, d, _ptr(out),
         _stream())
    return out


def dequantize(raw: torch.Tensor, qtype: int, n_elements: int) -> torch.Tensor:
    _need(raw, torch.uint8, "raw")
    out = torch.empty(n_elements, dtype=torch.float32, device=raw.device)
    call("moe_dequantize", _ptr(raw), _ptr(out), qtype, n_elements, _stream())
    return out


def pack_weights(raw: torch.Tensor, qtype: int, n_mats: int, rows: int, cols: int) -> torch.Tensor:
    _need(raw, torch.uint8, "raw")
    nbytes = _size_out("moe_packed_bytes", qtype, n_mats, rows, cols)
    if raw.numel() != nbytes:
        raise ValueError(f"raw blocks hold {raw.numel()} bytes, expected {nbytes}")
    out = torch.empty(nbytes, dtype=torch.uint8, device=raw.device)
    call("moe_pack_weights", _ptr(raw), _ptr(out), qtype, n_mats, rows, cols, _stream())
    return out


def unpack_weights(packed: torch.Tensor, qtype: int, n_mats: int, rows: int, cols: int) -> torch.Tensor:
    _need(packed, torch.uint8, "packed")
    out = torch.empty_like(packed)
    call("moe_unpack_weights", _ptr(packed), _ptr(out), qtype, n_mats, rows, cols, _stream())
    return out


# --------------------------------------------------------------------------- stages

def router(x: torch.Tensor, gate_w: torch.Tensor, k: int, mode: int = 0,
           bias: Optional[torch.Tensor] = None, layout: int = _lib.MOE_ROUTER_D_E):
    """(ids int32 (T,k), weights f32 (T,k)) for x (T, d)."""
    _need(x, torch.float32, "x")
    _need(gate_w, torch.float32, "gate_w")
    if bias is not None:
        _need(bias, torch.float32, "bias")
    T, d = x.shape
    E = gate_w.shape[1] if layout == _lib.MOE_ROUTER_D_E else gate_w.shape[0]
    ids = torch.empty((T, k), dtype=torch.int32, device=x.device)
    w = torch.empty((T, k), dtype=torch.float32, device=x.device)
    ws = workspace(_size_out("moe_router_workspace_bytes", T, d, E), x.device)
    call("moe_router", _ptr(x), _ptr(gate_w), _ptr(bias), T, d, E, k, layout, mode,
         _ptr(ids), _ptr(w), _ptr(ws), ws.numel(), _stream())
    return ids, w


def dispatch(ids: torch.Tensor, n_experts: int, ws: Optional[torch.Tensor] = None):
    """(expert_offsets (E+1), perm_rows (T*k), inv_perm (T*k)), all int32."""
    _need(ids, torch.int32, "ids")
    T, k = ids.shape
    dev = ids.device
    off = torch.empty(n_experts + 1, dtype=torch.int32, device=dev)
    perm = torch.empty(T * k, dtype=torch.int32, device=dev)
    inv = torch.empty(T * k, dtype=torch.int32, device=dev)
    if ws is None:
        ws = workspace(_size_out("moe_dispatch_workspace_bytes", T, k, n_experts), dev)
        ws[:256].zero_()
    call("moe_dispatch", _ptr(ids), T, k, n_experts, _ptr(off), _ptr(perm), _ptr(inv),
         _ptr(ws), ws.numel(), _stream())
    return off, perm, inv


def read_status(ws: torch.Tensor) -> int:
    st = ctypes.c_int(0)
    rc = _lib.load().moe_read_status(_ptr(ws), ctypes.byref(st), _stream())
    if rc not in (_lib.MOE_OK, _lib.MOE_ERR_DEVICE):
        _lib.check(rc)
    return st.value


def experts(w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, qtype: int,
            offsets: torch.Tensor, x: torch.Tensor, d: int, F: int,
            x_rows: Optional[torch.Tensor] = None, x_rows_div: int = 1,
            y: Optional[torch.Tensor] = None, y_rows: Optional[torch.Tensor] = None,
            rows: Optional[int] = None, ws: Optional[torch.Tensor] = None,
            opts: Optional[ExpertOpts] = None) -> torch.Tensor:
    """Grouped experts on packed weights (Q4_0 / Q8_0) or raw matrices (other
    types, or a down matrix of another type); returns y (rows, d) f32."""
    for t, n in ((w_gate, "w_gate"), (w_up, "w_up"), (w_down, "w_down")):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or not t.is_contiguous():
            raise TypeError(f"{n} must be a contiguous CUDA tensor")
    _need(offsets, torch.int32, "offsets")
    _need(x, torch.float32, "x")
    E = offsets.numel() - 1
    if rows is None:
        rows = int(offsets[-1].item())
    if y is None:
        y = torch.empty((rows, d), dtype=torch.float32, device=x.device)
    if ws is None:
        ws = workspace(_size_out("moe_experts_workspace_bytes", rows, E, d, F), x.device)
        ws[:256].zero_()
    call("moe_experts_ex", _ptr(w_gate), _ptr(w_up), _ptr(w_down), qtype,
         None if opts is None else opts.ref, _ptr(offsets), E, rows, _ptr(x), _ptr(x_rows),
         x_rows_div, d, F, _ptr(y), _ptr(y_rows), _ptr(ws), ws.numel(), _stream())
    return y


def combine(y: torch.Tensor, inv_perm: torch.Tensor, weights: torch.Tensor,
            shared: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    T, k = weights.shape
    d = y.shape[1]
    if out is None:
        out = torch.empty((T, d), dtype=torch.float32, device=y.device)
    call("moe_combine", _ptr(y), _ptr(inv_perm), _ptr(weights), _ptr(shared), _ptr(residual),
         T, k, d, _ptr(out), _stream())
    return out


def gather_rows(x: torch.Tensor, rows: torch.Tensor, div: int = 1,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _need(x, torch.float32, "x")
    _need(rows, torch.int32, "rows")
    n, d = rows.numel(), x.shape[1]
    if out is None:
        out = torch.empty((n, d), dtype=torch.float32, device=x.device)
    call("moe_gather_rows", _ptr(x), _ptr(rows), div, n, d, _ptr(out), _stream())
    return out


def ep_local_order(recv_counts: torch.Tensor, max_rows: int, ws: torch.Tensor):
    """(local_offsets (E_local+1), row_map (max_rows)) on the device."""
    _need(recv_counts, torch.int32, "recv_counts")
    W, El = recv_counts.shape
    loff = torch.empty(El + 1, dtype=torch.int32, device=recv_counts.device)
    row_map = torch.empty(max(max_rows, 1), dtype=torch.int32, device=recv_counts.device)
    call("moe_ep_local_order", _ptr(recv_counts), W, El, max_rows, _ptr(loff), _ptr(row_map),
         _ptr(ws), _stream())
    return loff, row_map


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
             out: Optional[torch.Tensor] = None, gemma_style: bool = False) -> torch.Tensor:
    _need(x, torch.float32, "x")
    _need(weight, torch.float32, "weight")
    T, d = x.shape
    if out is None:
        out = torch.empty_like(x)
    call("moe_rms_norm_ex", _ptr(x), _ptr(weight), ctypes.c_float(eps), 1 if gemma_style else 0,
         T, d, _ptr(out), _stream())
    return out


# --------------------------------------------------------------------------- layer

class LayerWeights:
    """Device-resident weights of one MoE layer in the library's layout."""

    def __init__(self, gate_w: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
                 w_down: torch.Tensor, qtype: int, E: int, k: int, d: int, F: int,
                 mode: int = 0, bias: Optional[torch.Tensor] = None,
                 router_layout: int = _lib.MOE_ROUTER_D_E,
                 shared: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None,
                 shared_qtype: int = QTYPE_Q8_0, Fs: int = 0,
                 opts: Optional[ExpertOpts] = None):
        self.gate_w, self.bias = gate_w, bias
        self.opts = opts
        self.w_gate, self.w_up, self.w_down = w_gate, w_up, w_down
        self.shared = shared
        self.qtype, self.E, self.k, self.d, self.F, self.mode = qtype, E, k, d, F, mode
        self.shared_qtype, self.Fs = shared_qtype, Fs
        s = shared or (None, None, None)
        self.c = _lib.MoELayerWeights(
            gate_w.data_ptr(), 0 if bias is None else bias.data_ptr(),
            w_gate.data_ptr(), w_up.data_ptr(), w_down.data_ptr(),
            0 if s[0] is None else s[0].data_ptr(), 0 if s[1] is None else s[1].data_ptr(),
            0 if s[2] is None else s[2].data_ptr(),
            router_layout, qtype, shared_qtype, E, k, d, F, Fs, mode,
            ctypes.pointer(opts.c) if opts is not None else None)

    def workspace_bytes(self, T: int) -> int:
        out = ctypes.c_size_t(0)
        call("moe_layer_workspace_bytes", ctypes.byref(self.c), T, ctypes.byref(out))
        return int(out.value)


def layer_forward(lw: LayerWeights, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                  residual: Optional[torch.Tensor] = None, ws: Optional[torch.Tensor] = None,
                  ids: Optional[torch.Tensor] = None,
                  weights: Optional[torch.Tensor] = None,
                  router_x: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x and out may be pinned host tensors: the layer then reads x and writes
    out over the bus from its own kernels (no separate copies)."""
    _need(x, torch.float32, "x", pinned_ok=True)
    if out is not None:
        _need(out, torch.float32, "out", pinned_ok=True)
    if router_x is not None:
        _need(router_x, torch.float32, "router_x")
        if router_x.shape != x.shape:
            raise ValueError("router_x must have the shape of x")
    T = x.shape[0]
    if out is None:
        out = torch.empty_like(x) if x.is_cuda else torch.empty(x.shape, dtype=x.dtype,
                                                                 pin_memory=True)
    dev = x.device if x.is_cuda else torch.device("cuda", torch.cuda.current_device())
    if ws is None:
        ws = workspace(lw.workspace_bytes(T), dev)
        ws[:256].zero_()
    call("moe_layer_forward_ex", ctypes.byref(lw.c), _ptr(x), _ptr(router_x), T, _ptr(out),
         _ptr(residual), _ptr(ids), _ptr(weights), _ptr(ws), ws.numel(), _stream())
    return out


def layer_forward_ptr(lw: LayerWeights, x_ptr: int, T: int, out_ptr: int, ws: torch.Tensor,
                      router_x_ptr: int = 0, residual_ptr: int = 0) -> None:
    """moe_layer_forward_ex on raw device pointers (f32 (T, d) rows on the
    current device), for callers that hold their own device buffers."""
    call("moe_layer_forward_ex", ctypes.byref(lw.c), ctypes.c_void_p(int(x_ptr)),
         ctypes.c_void_p(int(router_x_ptr)), T, ctypes.c_void_p(int(out_ptr)),
         ctypes.c_void_p(int(residual_ptr)), None, None, _ptr(ws), ws.numel(), _stream())
