"""Stacked decode step: L MoE layers, each with an always-on shared expert,
with the residual and RMSNorm of MoETransformerModel._layer_forward
(moe_forward.py:348-359): ``x = x + moe(rms_norm(x, w))``."""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from . import kernels as K
from .moe_forward import MoELayer


class StackedMoE:
    def __init__(self, layers: Sequence[MoELayer], norms: Sequence[torch.Tensor], eps: float = 1e-6):
        self.layers = list(layers)
        self.norms = list(norms)
        self.eps = eps
        self._buf: Optional[torch.Tensor] = None

    @classmethod
    def from_layers(cls, datas, device=None, eps: float = 1e-6) -> "StackedMoE":
        """From synthetic layer data (``synth.MoELayerData`` per layer)."""
        layers, norms = [], []
        for data in datas:
            cfg = data.cfg
            shared = None
            if cfg.shared_ffn:
                shared = (data.s_gate[0], data.s_up[0], data.s_down[0])
            layer = MoELayer.from_blocks(data.gate_w, data.w_gate, data.w_up, data.w_down,
                                         cfg.qtype, cfg.top_k, shared=shared,
                                         shared_qtype=cfg.shared_qtype,
                                         shared_hidden=cfg.shared_ffn, bias=data.bias,
                                         device=device)
            layers.append(layer)
            norms.append(torch.from_numpy(data.norm_w).to(layer.router.device))
        return cls(layers, norms, eps)

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x (T, d) f32 on the device -> (T, d).  The residual stream lives in
        ``out`` (allocated once if not given): the first layer adds x into it,
        later layers update it in place (the combine may write over its own
        residual input), so a step allocates nothing after the first."""
        if self._buf is None or self._buf.shape != x.shape:
            self._buf = torch.empty_like(x)
        xn = self._buf
        res = out if out is not None else torch.empty_like(x)
        cur = x
        for layer, nw in zip(self.layers, self.norms):
            K.rms_norm(cur, nw, self.eps, out=xn)
            layer.forward_batch(xn, residual=cur, out=res)
            cur = res
        return res


class StackedEP:
    """The stacked step with every layer expert-parallel over ``group``: the
    layers share one exchange window; RMSNorm and the residual are local."""

    def __init__(self, layers, norms, eps: float = 1e-6):
        self.layers = list(layers)
        self.norms = list(norms)
        self.eps = eps
        self._buf: Optional[torch.Tensor] = None

    @classmethod
    def build(cls, cfg, seed: int, tokens: int, group=None, device=None, eps: float = 1e-6,
              layers: Optional[int] = None) -> "StackedEP":
        """Synthetic layers (seed + layer index); each rank generates and packs
        only its own experts."""
        import torch.distributed as dist
        from . import synth
        from .ep import EPExchange, EPMoELayer, expert_range
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        e0, e1 = expert_range(rank, world, cfg.n_experts)
        ex = EPExchange(group, device)
        ls, ns = [], []
        for li in range(cfg.n_layers if layers is None else layers):
            data = synth.make_layer_slice(cfg, seed + li, tokens * world, e0, e1)
            shared = (data.s_gate, data.s_up, data.s_down) if cfg.shared_ffn else None
            layer = EPMoELayer(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype,
                               cfg.top_k, cfg.route_mode, None, group=group, device=device,
                               shared=shared, shared_qtype=cfg.shared_qtype, local=True,
                               exchange=ex)
            ls.append(layer)
            ns.append(torch.from_numpy(data.norm_w).to(layer.device))
        return cls(ls, ns, eps)

    @classmethod
    def from_layers(cls, datas, group=None, device=None, eps: float = 1e-6) -> "StackedEP":
        """From per-layer data whose expert stacks hold this rank's experts
        only (``synth.make_layer_device`` / ``make_layer_slice`` for the rank's
        expert range); the layers share one exchange window."""
        from .ep import EPExchange, EPMoELayer
        ex = EPExchange(group, device)
        ls, ns = [], []
        for data in datas:
            cfg = data.cfg
            shared = (data.s_gate, data.s_up, data.s_down) if cfg.shared_ffn else None
            layer = EPMoELayer(data.gate_w, data.w_gate, data.w_up, data.w_down, cfg.qtype,
                               cfg.top_k, cfg.route_mode, data.bias, group=group, device=device,
                               shared=shared, shared_qtype=cfg.shared_qtype, local=True,
                               exchange=ex)
            ls.append(layer)
            ns.append(torch.from_numpy(data.norm_w).to(layer.device))
        return cls(ls, ns, eps)

    def close(self) -> None:
        if self.layers:
            self.layers[0].exchange.close()

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """As ``StackedMoE.forward``, every layer expert-parallel."""
        if self._buf is None or self._buf.shape != x.shape:
            self._buf = torch.empty_like(x)
        xn = self._buf
        res = out if out is not None else torch.empty_like(x)
        cur = x
        for layer, nw in zip(self.layers, self.norms):
            K.rms_norm(cur, nw, self.eps, out=xn)
            layer.forward(xn, out=res, residual=cur)
            cur = res
        return res
