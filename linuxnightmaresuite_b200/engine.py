"""The reference engines' MoE feed-forward calls, served by the B200 layer.

The reference runs its MoE FFN from four engine methods, each of which routes
on the host and launches three matvecs per selected expert, with a
device->host copy of every expert's output and a host-side weighted sum:

* ``GPUStreamEngine._moe_ffn(xn, layer_idx, weights)`` -- CPU path
  (nightmare_stream.py:3220-3253);
* ``GPUStreamEngine._moe_ffn_gpu(xn_ptr, layer_idx, weights, out_ptr)`` --
  activations on the device (nightmare_stream.py:3280-3334);
* ``GPUStreamEngine._moe_ffn_g4_gpu(attn_out, moe_in, weights, layer, eps)`` --
  gemma4's routed experts (nightmare_stream.py:4330-4459);
* ``GpuNativeEngine._moe_ffn_gpu_native(gpu, bufs, layer)``
  (nightmare_gpu_native.py:1542-1590).

``MoEEngineAdapter`` offers the same four calls with the same arguments and
results, each one whole layer forward in the library (router -> dispatch ->
grouped experts -> combine on the device, no per-expert round trip).  Layers
come from the model's GGUF file (``gguf.load_moe_layer``, loaded on first use
and kept resident) or are given.  ``install(engine)`` binds the calls onto an
engine object in place of its own.

Pointer arguments (``xn_ptr``, ``out_ptr``, ``bufs[...]``) are device
addresses of f32 vectors on the adapter's device, in the context the library
runs in (the device's primary context, which torch uses).
"""
from __future__ import annotations

import ctypes
from typing import Dict, Optional

import numpy as np
import torch

from . import _lib
from . import kernels as K
from .gemma4 import Gemma4MoEBlock


class MoEEngineAdapter:
    def __init__(self, parser=None, model=None, device=None, layers: Optional[Dict] = None,
                 top_k: Optional[int] = None):
        self.parser, self.model = parser, model
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.layers: Dict[int, object] = dict(layers or {})
        self.top_k = top_k
        self._stager = None
        self.calls = 0

    # ------------------------------------------------------------- layers
    def layer(self, idx: int):
        """The resident MoE of block ``idx`` (loaded from the file once)."""
        lay = self.layers.get(int(idx))
        if lay is None:
            if self.parser is None:
                raise KeyError(f"no MoE layer {idx} and no GGUF file to load it from")
            from . import gguf
            if self._stager is None:
                self._stager = gguf.PinnedStager(self.device)
            lay = gguf.load_moe_layer(self.parser, self.model, int(idx), self.device,
                                      top_k=self.top_k, stager=self._stager)
            self.layers[int(idx)] = lay
        return lay

    def _routed_layer(self, idx: int):
        lay = self.layer(idx)
        return lay.layer if isinstance(lay, Gemma4MoEBlock) else lay

    def _dim(self, lay) -> int:
        return int(lay.weights.d)

    # ------------------------------------------------------------- calls
    def moe_ffn(self, xn, layer_idx: int, weights=None) -> np.ndarray:
        """GPUStreamEngine._moe_ffn: xn (dim,) or (1, dim) host f32 ->
        (1, dim) f32 (softmax over all experts -> top-k -> renormalised).
        The token and the result go through pinned host buffers that the
        layer's kernels read and write themselves."""
        lay = self._routed_layer(layer_idx)
        d = self._dim(lay)
        xin, xout = self._pinned(d)
        xin.numpy()[0] = np.asarray(xn, dtype=np.float32).reshape(-1)
        with torch.cuda.device(self.device):
            lay.forward_batch(xin, out=xout)
            torch.cuda.current_stream().synchronize()
        self.calls += 1
        return xout.numpy().copy()

    def _pinned(self, d: int):
        buf = getattr(self, "_pin", None)
        if buf is None or buf[0].shape[1] != d:
            self._pin = buf = (torch.empty((1, d), dtype=torch.float32, pin_memory=True),
                               torch.empty((1, d), dtype=torch.float32, pin_memory=True))
        return buf

    def moe_ffn_gpu(self, xn_ptr: int, layer_idx: int, weights=None, out_ptr: Optional[int] = None):
        """GPUStreamEngine._moe_ffn_gpu: reads dim f32 at device address
        ``xn_ptr``, writes the layer output to ``out_ptr`` (device) and returns
        it; nothing crosses to the host.  Without ``out_ptr`` the result goes
        to an adapter-owned device buffer whose address is returned."""
        lay = self._routed_layer(layer_idx)
        if out_ptr is None:
            buf = getattr(self, "_out_buf", None)
            if buf is None or buf.numel() < self._dim(lay):
                self._out_buf = buf = torch.empty(self._dim(lay), dtype=torch.float32,
                                                  device=self.device)
            out_ptr = buf.data_ptr()
        K.layer_forward_ptr(lay.weights, int(xn_ptr), 1, int(out_ptr), lay._workspace(1))
        self.calls += 1
        return out_ptr

    def moe_ffn_g4_gpu(self, attn_out, moe_in, weights, layer: int, eps: float):
        """GPUStreamEngine._moe_ffn_g4_gpu: gemma4's routed experts for one
        token; the router reads attn_out (its own RMS, 1/sqrt(dim) and
        ffn_gate_inp.scale), the experts moe_in.  Returns cur_moe (dim,) host
        f32, before post_ffw_norm_2, as the reference does."""
        blk = self.layer(layer)
        if not isinstance(blk, Gemma4MoEBlock):
            raise TypeError(f"layer {layer} is not a gemma4 MoE block")
        a = torch.from_numpy(np.ascontiguousarray(np.asarray(attn_out, np.float32)
                                                  .reshape(1, -1))).to(self.device)
        m = torch.from_numpy(np.ascontiguousarray(np.asarray(moe_in, np.float32)
                                                  .reshape(1, -1))).to(self.device)
        self.calls += 1
        return blk.routed(a, m, eps).cpu().numpy().reshape(-1)

    def moe_ffn_gpu_native(self, gpu, bufs, layer: int) -> None:
        """GpuNativeEngine._moe_ffn_gpu_native: reads bufs['xn'] and writes
        the layer output back into bufs['xn'] (device addresses)."""
        lay = self._routed_layer(layer)
        d = self._dim(lay)
        tmp = getattr(self, "_native_in", None)
        if tmp is None or tmp.numel() < d:
            self._native_in = tmp = torch.empty(d, dtype=torch.float32, device=self.device)
        # the layer's output must not alias its input: take a device copy
        _lib.call("moe_gather_rows", ctypes.c_void_p(int(bufs["xn"])), K._ptr(self._zero_row()),
                  1, 1, d, K._ptr(tmp), K._stream())
        K.layer_forward_ptr(lay.weights, tmp.data_ptr(), 1, int(bufs["xn"]), lay._workspace(1))
        self.calls += 1

    def _zero_row(self) -> torch.Tensor:
        z = getattr(self, "_zero", None)
        if z is None:
            self._zero = z = torch.zeros(1, dtype=torch.int32, device=self.device)
        return z

    # ------------------------------------------------------------- binding
    def install(self, engine) -> None:
        """Replaces the engine's MoE methods by this adapter's (the ones the
        engine has): _moe_ffn, _moe_ffn_gpu, _moe_ffn_g4_gpu,
        _moe_ffn_gpu_native."""
        adapter = self

        def _moe_ffn(xn, layer_idx, weights):
            return adapter.moe_ffn(xn, layer_idx, weights)

        def _moe_ffn_gpu(xn_ptr, layer_idx, weights, out_ptr=None):
            return adapter.moe_ffn_gpu(xn_ptr, layer_idx, weights, out_ptr)

        def _moe_ffn_g4_gpu(attn_out, moe_in, weights, layer, eps):
            return adapter.moe_ffn_g4_gpu(attn_out, moe_in, weights, layer, eps)

        def _moe_ffn_gpu_native(gpu, bufs, layer):
            return adapter.moe_ffn_gpu_native(gpu, bufs, layer)

        for name, fn in (("_moe_ffn", _moe_ffn), ("_moe_ffn_gpu", _moe_ffn_gpu),
                         ("_moe_ffn_g4_gpu", _moe_ffn_g4_gpu),
                         ("_moe_ffn_gpu_native", _moe_ffn_gpu_native)):
            if hasattr(engine, name) or name == "_moe_ffn":
                setattr(engine, name, fn)
        engine._b200_moe = adapter
