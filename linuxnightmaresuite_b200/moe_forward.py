"""Drop-in B200 counterpart of the reference's ``moe_forward.py`` MoE classes.

Same names, constructor arguments and call results as the reference:

* ``MoERouter(gate_weight, n_experts, top_k=2)`` with ``route(x) ->
  (List[int], np.ndarray)`` for one token (moe_forward.py:78-109);
* ``ExpertFFN`` with ``forward(x)`` (moe_forward.py:116-133);
* ``MoELayer(router, experts, shared_expert=None)`` with ``forward(x)``
  (moe_forward.py:140-174);
* ``rms_norm(x, weight, eps=1e-6)`` (moe_forward.py:34-40).

Everything runs in the CUDA library (``libmoe_b200.so``); there is no CPU path.
Inputs may be numpy float32 arrays (results come back as numpy, like the
reference) or CUDA tensors (results stay on the device).  A 2-D input of T
tokens is processed as one batch whose row t equals the single-token result.

Experts are built from GGUF Q4_0 / Q8_0 block bytes (``ExpertFFN.from_blocks``
/ ``MoELayer.from_blocks``) -- exactly what ``gguf_parser.load_tensor_raw``
(gguf_parser.py:532-558) or a per-expert slice of an ``ffn_*_exps`` tensor
(nightmare_stream.py:3361-3441) yields.  ``ExpertFFN(w_gate, w_up, w_down)``
takes the reference's f32 matrices, or such block arrays when given ``qtype``.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

from . import _lib
from . import kernels as K

Array = Union[np.ndarray, torch.Tensor]

QTYPE_F32 = K.QTYPE_F32
QTYPE_Q4_0 = K.QTYPE_Q4_0
QTYPE_Q5_1 = K.QTYPE_Q5_1
QTYPE_Q8_0 = K.QTYPE_Q8_0
QTYPE_Q4_K = K.QTYPE_Q4_K
QTYPE_Q6_K = K.QTYPE_Q6_K
ACT_SWIGLU = K.ACT_SWIGLU
ACT_GEGLU_TANH = K.ACT_GEGLU_TANH


def _device(device=None) -> torch.device:
    if device is not None:
        return torch.device(device)
    if not torch.cuda.is_available():
        raise RuntimeError("the B200 MoE layer needs a CUDA device")
    return torch.device("cuda", torch.cuda.current_device())


def _to_dev_f32(a: Array, device) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(device=device, dtype=torch.float32).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device)


def _to_dev_u8(a: Array, device) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(device=device).contiguous().view(torch.uint8).reshape(-1)
    return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1)).to(device)


def rms_norm(x: Array, weight: Array, eps: float = 1e-6, gemma_style: bool = False):
    """moe_forward.rms_norm (moe_forward.py:34-40); rows normalised
    independently; ``gemma_style`` scales by (1 + weight)."""
    dev = _device(x.device if isinstance(x, torch.Tensor) and x.is_cuda else None)
    xt = _to_dev_f32(x, dev)
    one = xt.dim() == 1
    out = K.rms_norm(xt.reshape(1, -1) if one else xt, _to_dev_f32(weight, dev), eps,
                     gemma_style=gemma_style)
    out = out.reshape(-1) if one else out
    return out if isinstance(x, torch.Tensor) else out.cpu().numpy()


class MoERouter:
    """Top-k expert routing (moe_forward.py:78-109).

    ``mode=0`` is the reference's MoERouter (top-k logits, softmax over them,
    descending); ``mode=1`` is the production rule of nightmare_stream.py:3227-3238
    (softmax over all experts, top-k, renormalised, ascending).  ``bias`` is an
    optional per-expert logit offset."""

    def __init__(self, gate_weight: Array, n_experts: int, top_k: int = 2, mode: int = 0,
                 bias: Optional[Array] = None, device=None, layout: int = _lib.MOE_ROUTER_D_E):
        if top_k > n_experts:
            raise ValueError(f"top_k {top_k} exceeds n_experts {n_experts}")
        self.gate_weight = gate_weight
        self.n_experts = n_experts
        self.top_k = top_k
        self.mode = mode
        self.layout = layout
        self.device = _device(device)
        self.g = _to_dev_f32(gate_weight, self.device)
        e_axis = 1 if layout == _lib.MOE_ROUTER_D_E else 0
        if self.g.shape[e_axis] != n_experts:
            raise ValueError(f"gate_weight is {tuple(self.g.shape)}, expected {n_experts} experts "
                             f"on axis {e_axis}")
        self.bias = None if bias is None else _to_dev_f32(bias, self.device)

    def route_batch(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """(ids int32 (T,k), weights f32 (T,k)) on the device."""
        return K.router(x, self.g, self.top_k, self.mode, self.bias, self.layout)

    def route(self, x: Array):
        xt = _to_dev_f32(x, self.device)
        if xt.dim() == 1:
            ids, w = self.route_batch(xt.reshape(1, -1))
            return ids[0].cpu().tolist(), w[0].cpu().numpy()
        ids, w = self.route_batch(xt)
        if isinstance(x, torch.Tensor):
            return ids, w
        return ids.cpu().numpy(), w.cpu().numpy()


def _weights(raw: Array, qtype: int, n_mats: int, rows: int, cols: int, device,
             pack: bool) -> torch.Tensor:
    """Raw GGUF blocks of n_mats (rows, cols) matrices on the device: packed
    into MMA tiles for the Q4_0 / Q8_0 kernels, else kept as stored."""
    t = _to_dev_u8(raw, device)
    need = n_mats * rows * K.row_bytes(qtype, cols)
    if t.numel() != need:
        raise ValueError(f"{t.numel()} bytes of type-{qtype} blocks, expected {need} for "
                         f"{n_mats} x ({rows}, {cols})")
    return K.pack_weights(t, qtype, n_mats, rows, cols) if pack else t


def _is_float(a) -> bool:
    if isinstance(a, torch.Tensor):
        return a.is_floating_point()
    return np.issubdtype(np.asarray(a).dtype, np.floating)


class ExpertFFN:
    """One SwiGLU expert (moe_forward.py:116-133).

    As in the reference, ``ExpertFFN(w_gate, w_up, w_down)`` takes f32
    matrices: w_gate / w_up (hidden_dim, dim), w_down (dim, hidden_dim); they
    are used on the GPU as given (4 bytes per weight).  With ``qtype`` (GGML
    type 2 = Q4_0, 8 = Q8_0) plus ``dim`` / ``hidden_dim`` the arguments are
    GGUF block bytes instead, packed once into the device layout."""

    def __init__(self, w_gate: Array, w_up: Array, w_down: Array, qtype: Optional[int] = None,
                 dim: Optional[int] = None, hidden_dim: Optional[int] = None, device=None):
        self.device = _device(device)
        if qtype is None or qtype == QTYPE_F32:
            if not (_is_float(w_gate) and _is_float(w_up) and _is_float(w_down)):
                raise TypeError("ExpertFFN(w_gate, w_up, w_down) takes float matrices; for GGUF "
                                "block bytes pass qtype (2 = Q4_0, 8 = Q8_0), dim and hidden_dim")
            wg, wu, wd = (_to_dev_f32(a, self.device) for a in (w_gate, w_up, w_down))
            if wg.dim() != 2 or wu.shape != wg.shape or wd.shape != (wg.shape[1], wg.shape[0]):
                raise ValueError(f"expected w_gate, w_up (hidden_dim, dim) and w_down (dim, "
                                 f"hidden_dim); got {tuple(wg.shape)}, {tuple(wu.shape)}, "
                                 f"{tuple(wd.shape)}")
            self.qtype, self.hidden_dim, self.dim = QTYPE_F32, int(wg.shape[0]), int(wg.shape[1])
            self.w_gate, self.w_up, self.w_down = wg, wu, wd
            return
        if qtype not in K.BLOCK_GEOMETRY:
            raise ValueError(f"unsupported GGML type {qtype}")
        self.qtype, self.dim, self.hidden_dim = qtype, int(dim), int(hidden_dim)
        d, F = self.dim, self.hidden_dim
        pack = K.packed_path(qtype, qtype)
        self.w_gate = _weights(w_gate, qtype, 1, F, d, self.device, pack)
        self.w_up = _weights(w_up, qtype, 1, F, d, self.device, pack)
        self.w_down = _weights(w_down, qtype, 1, d, F, self.device, pack)

    @classmethod
    def from_blocks(cls, gate_bytes: Array, up_bytes: Array, down_bytes: Array, qtype: int,
                    dim: int, hidden_dim: int, device=None) -> "ExpertFFN":
        return cls(gate_bytes, up_bytes, down_bytes, qtype, dim, hidden_dim, device)

    def forward(self, x: Array):
        xt = _to_dev_f32(x, self.device)
        one = xt.dim() == 1
        xt = xt.reshape(1, -1) if one else xt
        T = xt.shape[0]
        off = torch.tensor([0, T], dtype=torch.int32, device=self.device)
        y = K.experts(self.w_gate, self.w_up, self.w_down, self.qtype, off, xt, self.dim,
                      self.hidden_dim, rows=T)
        y = y.reshape(-1) if one else y
        return y if isinstance(x, torch.Tensor) else y.cpu().numpy()


class MoELayer:
    """Router + routed experts + optional shared expert (moe_forward.py:140-174)."""

    def __init__(self, router: MoERouter, experts: Sequence[ExpertFFN],
                 shared_expert: Optional[ExpertFFN] = None):
        self.router = router
        self.experts = list(experts)
        self.shared_expert = shared_expert
        if len(self.experts) != router.n_experts:
            raise ValueError(f"{len(self.experts)} experts for a router over {router.n_experts}")
        e0 = self.experts[0]
        for ex in self.experts:
            if (ex.qtype, ex.dim, ex.hidden_dim) != (e0.qtype, e0.dim, e0.hidden_dim):
                raise ValueError("all routed experts must share quant type and shape")
        dev = router.device
        self._build(router, torch.cat([ex.w_gate for ex in self.experts]).to(dev),
                    torch.cat([ex.w_up for ex in self.experts]).to(dev),
                    torch.cat([ex.w_down for ex in self.experts]).to(dev),
                    e0.qtype, e0.dim, e0.hidden_dim, shared_expert)

    def _build(self, router, wg, wu, wd, qtype, d, F, shared, opts=None):
        self.dim, self.hidden_dim, self.qtype = d, F, qtype
        sh = None
        sq, Fs = QTYPE_Q8_0, 0
        if shared is not None:
            if shared.dim != d:
                raise ValueError("shared expert dim differs from the routed experts")
            sh = (shared.w_gate, shared.w_up, shared.w_down)
            sq, Fs = shared.qtype, shared.hidden_dim
        self.weights = K.LayerWeights(router.g, wg, wu, wd, qtype, router.n_experts,
                                      router.top_k, d, F, router.mode, router.bias,
                                      router.layout, sh, sq, Fs, opts)
        self._ws = None

    @classmethod
    def from_blocks(cls, gate_weight: Array, w_gate: Array, w_up: Array, w_down: Array,
                    qtype: int, top_k: int, shared: Optional[Tuple[Array, Array, Array]] = None,
                    shared_qtype: int = QTYPE_Q8_0, shared_hidden: int = 0, mode: int = 0,
                    bias: Optional[Array] = None, device=None, *, act: int = K.ACT_SWIGLU,
                    down_qtype: Optional[int] = None, down_scale: Optional[Array] = None,
                    gate_up: Optional[Array] = None,
                    router_layout: int = _lib.MOE_ROUTER_D_E) -> "MoELayer":
        """Layer from stacked expert blocks: ``w_gate`` / ``w_up`` (E, F, row
        bytes), ``w_down`` (E, d, row bytes), i.e. the bytes of GGUF
        ``ffn_*_exps`` tensors (nightmare_stream.py:3361-3441).

        Expert variants (the gemma4 MoE, nightmare_stream.py:4655-4693):
        ``gate_up`` a fused (E, 2F, row bytes) ``ffn_gate_up_exps`` stack in
        place of w_gate / w_up (pass None for those); ``down_qtype`` the type
        of w_down when it differs; ``down_scale`` (E,) per-expert factor of the
        down projection (``ffn_down_exps.scale``); ``act`` K.ACT_GEGLU_TANH for
        GeGLU-tanh experts; ``router_layout`` MOE_ROUTER_E_D for a (E, d)
        router matrix (the production ``moe_router`` tensor)."""
        dev = _device(device)
        G = gate_weight
        if router_layout == _lib.MOE_ROUTER_E_D:
            E, d = int(G.shape[0]), int(G.shape[1])
        else:
            d, E = int(G.shape[0]), int(G.shape[1])
        router = MoERouter(G, E, top_k, mode, bias, dev, layout=router_layout)
        self = cls.__new__(cls)
        self.router, self.experts = router, None
        dq = qtype if down_qtype is None else down_qtype
        pack = K.packed_path(qtype, dq)
        stride = 0
        if gate_up is not None:
            if w_gate is not None or w_up is not None:
                raise ValueError("pass either gate_up or w_gate / w_up")
            F = int(gate_up.shape[1]) // 2
            guw = _weights(gate_up, qtype, E, 2 * F, d, dev, pack)
            mat = F * K.row_bytes(qtype, d)
            wg, wu = guw, guw[mat:]
            stride = 2 * mat
        else:
            F = int(w_gate.shape[1])
            wg = _weights(w_gate, qtype, E, F, d, dev, pack)
            wu = _weights(w_up, qtype, E, F, d, dev, pack)
        wd = _weights(w_down, dq, E, d, F, dev, pack)
        sh_ex = None
        if shared is not None:
            sh_ex = ExpertFFN(shared[0], shared[1], shared[2], shared_qtype, d, shared_hidden, dev)
        self.shared_expert = sh_ex
        opts = None
        if act != K.ACT_SWIGLU or dq != qtype or stride or down_scale is not None:
            ds = None if down_scale is None else _to_dev_f32(down_scale, dev).reshape(-1)
            if ds is not None and ds.numel() != E:
                raise ValueError(f"down_scale has {ds.numel()} entries for {E} experts")
            opts = K.ExpertOpts(act, dq if dq != qtype else 0, stride, ds)
        self._build(router, wg, wu, wd, qtype, d, F, sh_ex, opts)
        self._keep = (wg, wu)   # the fused stack's views
        return self

    def _workspace(self, T: int) -> torch.Tensor:
        need = self.weights.workspace_bytes(T)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=self.router.device)
        return self._ws

    def forward_batch(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                      out: Optional[torch.Tensor] = None, return_routing: bool = False,
                      router_x: Optional[torch.Tensor] = None):
        """(T, d) tokens on the device, or in pinned host memory (with ``out``
        then also pinned host memory or on the device): the layer's kernels
        read and write host tensors over the bus themselves.  ``router_x``
        (T, d) is what the router reads when it differs from the experts'
        input (gemma4)."""
        T = x.shape[0]
        ids = weights = None
        if return_routing:
            dev = self.router.device
            ids = torch.empty((T, self.router.top_k), dtype=torch.int32, device=dev)
            weights = torch.empty((T, self.router.top_k), dtype=torch.float32, device=dev)
        out = K.layer_forward(self.weights, x, out=out, residual=residual,
                              ws=self._workspace(T), ids=ids, weights=weights, router_x=router_x)
        return (out, ids, weights) if return_routing else out

    def device_status(self) -> int:
        """Reads and clears the device status bits (synchronises)."""
        return 0 if self._ws is None else K.read_status(self._ws)

    def forward(self, x: Array):
        xt = _to_dev_f32(x, self.router.device)
        one = xt.dim() == 1
        out = self.forward_batch(xt.reshape(1, -1) if one else xt)
        out = out.reshape(-1) if one else out
        return out if isinstance(x, torch.Tensor) else out.cpu().numpy()
