"""gemma4's MoE feed-forward block on the B200 layer.

A gemma4 MoE layer's FFN is the SUM of a dense shared expert and the routed
experts, each with its own pair of RMS norms, and the router reads a
different vector than the experts (nightmare_stream.py:4630-4693):

    mlp_in  = rms(attn_out, ffn_norm)
    cur_mlp = rms(down(geglu(gate(mlp_in)) * up(mlp_in)), post_ffw_norm_1)
    r_in    = attn_out / sqrt(mean(attn_out^2) + eps) * f32(1/sqrt(dim)) * ffn_gate_inp.scale
    moe_in  = rms(attn_out, pre_ffw_norm_2)
    cur_moe = rms(sum_k w_k * expert_k(moe_in), post_ffw_norm_2)
              (softmax over all experts -> top-k -> renormalised)
    f       = cur_mlp + cur_moe

The experts are the gemma4 GGUF layout: a fused ``ffn_gate_up_exps`` stack
(2F rows per expert: gate then up, Q4_K), ``ffn_down_exps`` (Q5_1) times the
per-expert ``ffn_down_exps.scale``, GeGLU-tanh activation
(nightmare_stream.py:3256-3271, :3361-3441).  Every step runs in the CUDA
library: the norms and the router input in the RMSNorm kernels, the shared
MLP as a one-expert grouped call, the routed experts as one layer forward
whose router reads the router input.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import _lib
from . import kernels as K
from .moe_forward import ExpertFFN, MoELayer, _device, _to_dev_f32, _weights


class Gemma4MoEBlock:
    """``forward(attn_out)`` returns f (T, d): the gemma4 FFN block output
    before the layer's post_ffw_norm and residual.

    router (E, d) f32 (``ffn_gate_inp``); gate_inp_scale (d,) or None;
    gate_up (E, 2F, row bytes) raw blocks of type gu_qtype; down (E, d, row
    bytes) of type down_qtype; down_scale (E,) or None; shared (gate, up,
    down) raw blocks of type shared_qtype with hidden size shared_hidden;
    the four norm weights (d,)."""

    def __init__(self, router, gate_inp_scale, gate_up, gu_qtype: int, down, down_qtype: int,
                 down_scale, top_k: int, shared, shared_qtype: int, shared_hidden: int,
                 ffn_norm, post_ffw_norm_1, pre_ffw_norm_2, post_ffw_norm_2,
                 eps: float = 1e-6, device=None):
        dev = _device(device)
        self.device, self.eps = dev, float(eps)
        E, d = int(router.shape[0]), int(router.shape[1])
        self.d, self.E = d, E
        self.layer = MoELayer.from_blocks(router, None, None, down, gu_qtype, top_k,
                                          mode=_lib.MOE_ROUTE_SOFTMAX_TOPK_RENORM, device=dev,
                                          act=K.ACT_GEGLU_TANH, down_qtype=down_qtype,
                                          down_scale=down_scale, gate_up=gate_up,
                                          router_layout=_lib.MOE_ROUTER_E_D)
        self.shared = ExpertFFN(shared[0], shared[1], shared[2], shared_qtype, d, shared_hidden,
                                dev)
        self.shared_opts = K.ExpertOpts(K.ACT_GEGLU_TANH)
        self._sum_T = None
        self.gis = None if gate_inp_scale is None else _to_dev_f32(gate_inp_scale, dev)
        norms = (ffn_norm, post_ffw_norm_1, pre_ffw_norm_2, post_ffw_norm_2)
        self.ffn_norm, self.post1, self.pre2, self.post2 = (
            None if n is None else _to_dev_f32(n, dev) for n in norms)
        if self.ffn_norm is None or self.pre2 is None:
            raise ValueError("gemma4 MoE blocks need ffn_norm and pre_ffw_norm_2")

    def _shared_mlp(self, mlp_in: torch.Tensor) -> torch.Tensor:
        sh = self.shared
        T = mlp_in.shape[0]
        off = torch.tensor([0, T], dtype=torch.int32, device=self.device)
        return K.experts(sh.w_gate, sh.w_up, sh.w_down, sh.qtype, off, mlp_in, sh.dim,
                         sh.hidden_dim, rows=T, opts=self.shared_opts)

    def forward(self, attn_out, return_routing: bool = False):
        x = _to_dev_f32(attn_out, self.device)
        one = x.dim() == 1
        x = x.reshape(1, -1) if one else x
        eps = self.eps
        mlp_in = K.rms_norm(x, self.ffn_norm, eps)
        cur_mlp = self._shared_mlp(mlp_in)
        if self.post1 is not None:
            cur_mlp = K.rms_norm(cur_mlp, self.post1, eps)
        r_in = K.router_input(x, self.gis, eps)
        moe_in = K.rms_norm(x, self.pre2, eps)
        res = self.layer.forward_batch(moe_in, return_routing=return_routing, router_x=r_in)
        cur_moe = res[0] if return_routing else res
        if self.post2 is not None:
            cur_moe = K.rms_norm(cur_moe, self.post2, eps)
        # f = cur_mlp + cur_moe: the combine kernel with one unit-weight slot
        # per token adds the shared output in f32 (1.0 * y is exact)
        T = x.shape[0]
        if self._sum_T != T:
            self._ident = torch.arange(T, dtype=torch.int32, device=self.device)
            self._ones = torch.ones((T, 1), dtype=torch.float32, device=self.device)
            self._sum_T = T
        f = K.combine(cur_moe, self._ident, self._ones, shared=cur_mlp)
        f = f.reshape(-1) if one else f
        out = f if isinstance(attn_out, torch.Tensor) else f.cpu().numpy()
        return (out, res[1], res[2]) if return_routing else out

    def routed(self, attn_out: torch.Tensor, moe_in: torch.Tensor,
               eps: Optional[float] = None) -> torch.Tensor:
        """The routed experts' sum alone, before post_ffw_norm_2, for a caller
        that has normalised the experts' input itself -- what
        _moe_ffn_g4_gpu returns (nightmare_stream.py:4330-4459)."""
        e = self.eps if eps is None else float(eps)
        r_in = K.router_input(attn_out, self.gis, e)
        return self.layer.forward_batch(moe_in, router_x=r_in)

    def device_status(self) -> int:
        return self.layer.device_status()
