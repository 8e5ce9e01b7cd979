"""GGUF files and expert-slice upload for the B200 MoE layer.

The reference reads GGUF model files with ``gguf_parser.GGUFParser``
(gguf_parser.py:325-556: header, metadata, tensor infos, a memory map) and
slices one expert at a time out of the 3-D ``ffn_*_exps`` tensors
(nightmare_stream.py:3361-3441): with ggml's ``ne = [in, out, E]`` the expert
axis is outermost and every expert is a contiguous, block-aligned byte range.

This module keeps that surface -- ``GGUFParser(path).parse()`` returning a
``GGUFModel`` with ``metadata`` / ``tensors`` / ``tensor_data_offset``, and
``load_tensor_raw`` -- and adds the B200 side:

* ``ExpertSlices`` lists the byte range of every expert of a layer;
* ``PinnedStager`` moves ranges of the memory-mapped file into the GPU through
  a ring of pinned host buffers: while one buffer's host->device copy runs on
  the stream, the next range is copied out of the page cache into the other,
  so file reads overlap the transfers and the expert stacks land in HBM
  without an intermediate pageable copy;
* ``load_moe_layer`` builds a ``MoELayer`` (or a gemma4 ``Gemma4MoEBlock``)
  of one block straight from the file, raw blocks uploaded as stored;
* ``write_gguf`` writes GGUF v3 files (synthetic models, tests).
"""
from __future__ import annotations

import dataclasses
import mmap
import os
import struct
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

GGUF_MAGIC = 0x46554747
GGUF_DEFAULT_ALIGNMENT = 32

# metadata value types (GGUF specification)
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i",
           T_F32: "<f", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}

# GGML type -> (weights per block, bytes per block) for the types this layer
# takes (dequant_fast.py:723-754), plus F16 for plain tensors
BLOCK_GEOMETRY = {0: (1, 4), 1: (1, 2), 2: (32, 18), 7: (32, 24), 8: (32, 34), 12: (256, 144),
                  14: (256, 210)}


@dataclasses.dataclass
class TensorInfo:
    """A tensor of the file (gguf_parser.py:177-184): ``shape`` in ggml order
    (contiguous dimension first), ``offset`` from the tensor data section."""
    name: str
    n_dims: int
    shape: tuple
    dtype: int
    offset: int

    @property
    def n_elements(self) -> int:
        n = 1
        for v in self.shape:
            n *= int(v)
        return n

    @property
    def nbytes(self) -> int:
        be, bb = BLOCK_GEOMETRY[self.dtype]
        return self.n_elements // be * bb


@dataclasses.dataclass
class GGUFModel:
    """Parsed header of a GGUF file (gguf_parser.py:187-199)."""
    version: int
    metadata: dict = dataclasses.field(default_factory=dict)
    tensors: Dict[str, TensorInfo] = dataclasses.field(default_factory=dict)
    tensor_data_offset: int = 0
    file_path: str = ""

    @property
    def architecture(self) -> str:
        return str(self.metadata.get("general.architecture", "unknown"))

    def _arch_int(self, key: str, default: int = 0) -> int:
        v = self.metadata.get(f"{self.architecture}.{key}", default)
        if isinstance(v, list):
            v = v[0] if v else default
        try:
            return int(v)
        except (TypeError, ValueError):
            return default

    @property
    def embedding_length(self) -> int:
        return self._arch_int("embedding_length")

    @property
    def expert_count(self) -> int:
        return self._arch_int("expert_count")

    @property
    def expert_used_count(self) -> int:
        return self._arch_int("expert_used_count")

    @property
    def expert_feed_forward_length(self) -> int:
        return self._arch_int("expert_feed_forward_length")

    @property
    def norm_eps(self) -> float:
        v = self.metadata.get(f"{self.architecture}.attention.layer_norm_rms_epsilon", 1e-6)
        return float(v)


class GGUFParser:
    """Reads a GGUF v2 / v3 file: header, metadata, tensor infos, then a
    read-only memory map of the whole file (gguf_parser.py:325-448)."""

    def __init__(self, file_path: str):
        self.file_path = str(file_path)
        self._mm: Optional[mmap.mmap] = None
        self._fh = None

    # --------------------------------------------------------------- parsing
    def parse(self) -> GGUFModel:
        if not os.path.exists(self.file_path):
            raise FileNotFoundError(f"model file not found: {self.file_path}")
        self._fh = open(self.file_path, "rb")
        self._mm = mmap.mmap(self._fh.fileno(), 0, access=mmap.ACCESS_READ)
        buf = self._mm
        pos = 0

        def take(fmt):
            nonlocal pos
            v = struct.unpack_from(fmt, buf, pos)
            pos += struct.calcsize(fmt)
            return v[0]

        def string():
            nonlocal pos
            n = take("<Q")
            if n > (1 << 24):
                raise ValueError(f"string length {n} at {pos}: corrupt file")
            s = bytes(buf[pos:pos + n]).decode("utf-8", errors="replace")
            pos += n
            return s

        def value(t):
            nonlocal pos
            if t in _SCALAR:
                return take(_SCALAR[t])
            if t == T_BOOL:
                return take("<B") != 0
            if t == T_STR:
                return string()
            if t == T_ARR:
                et, n = take("<I"), take("<Q")
                if n > 50_000_000:
                    raise ValueError(f"array of {n} elements: corrupt file")
                if et in _SCALAR and et != T_BOOL:
                    fmt = _SCALAR[et]
                    sz = struct.calcsize(fmt)
                    arr = list(struct.unpack_from(f"<{n}{fmt[1]}", buf, pos))
                    pos += n * sz
                    return arr
                return [value(et) for _ in range(n)]
            raise ValueError(f"unknown metadata type {t}")

        if len(buf) < 24 or take("<I") != GGUF_MAGIC:
            raise ValueError(f"{self.file_path} is not a GGUF file")
        model = GGUFModel(version=take("<I"), file_path=self.file_path)
        if model.version not in (2, 3):
            raise ValueError(f"unsupported GGUF version {model.version}")
        n_tensors, n_kv = take("<Q"), take("<Q")
        for _ in range(n_kv):
            key = string()
            model.metadata[key] = value(take("<I"))
        for _ in range(n_tensors):
            name = string()
            nd = take("<I")
            shape = tuple(take("<Q") for _ in range(nd))
            dtype = take("<I")
            off = take("<Q")
            model.tensors[name] = TensorInfo(name, nd, shape, dtype, off)
        align = int(model.metadata.get("general.alignment", GGUF_DEFAULT_ALIGNMENT))
        model.tensor_data_offset = pos + (align - pos % align) % align
        return model

    def close(self) -> None:
        if self._mm is not None:
            self._mm.close()
            self._mm = None
        if self._fh is not None:
            self._fh.close()
            self._fh = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # --------------------------------------------------------------- access
    def view(self, model: GGUFModel, offset: int, nbytes: int) -> memoryview:
        """Zero-copy bytes [offset, offset + nbytes) of the tensor data section."""
        if self._mm is None:
            raise RuntimeError("parse() the file first")
        a = model.tensor_data_offset + int(offset)
        if a + nbytes > len(self._mm):
            raise ValueError(f"range {a}+{nbytes} beyond the end of {self.file_path}")
        return memoryview(self._mm)[a:a + nbytes]

    def load_tensor_raw(self, model: GGUFModel, tensor_name: str):
        """(raw uint8 copy, GGML type, ggml shape, elements), as
        gguf_parser.load_tensor_raw (gguf_parser.py:527-555)."""
        if tensor_name not in model.tensors:
            raise KeyError(f"tensor '{tensor_name}' not in the model")
        info = model.tensors[tensor_name]
        raw = np.frombuffer(self.view(model, info.offset, info.nbytes), dtype=np.uint8).copy()
        return raw, info.dtype, info.shape, info.n_elements

    def load_f32(self, model: GGUFModel, tensor_name: str) -> np.ndarray:
        """An F32 tensor in logical (reversed ggml) shape."""
        info = model.tensors[tensor_name]
        if info.dtype != 0:
            raise TypeError(f"{tensor_name} is GGML type {info.dtype}, not F32")
        a = np.frombuffer(self.view(model, info.offset, info.nbytes), dtype=np.float32).copy()
        return a.reshape(tuple(int(v) for v in info.shape[::-1]))


# ------------------------------------------------------------------- slices

@dataclasses.dataclass
class ExpertSlice:
    offset: int      # from the tensor data section
    nbytes: int
    dtype: int
    rows: int        # logical (out) rows of one expert
    cols: int        # logical (in) columns


def expert_slices(model: GGUFModel, tensor_name: str) -> List[ExpertSlice]:
    """Byte ranges of every expert of a 3-D ``ffn_*_exps`` tensor with ggml
    ``ne = [in, out, E]``: expert e is ``out * in / block_elems`` blocks at
    ``e`` times that (nightmare_stream.py:3361-3441)."""
    info = model.tensors[tensor_name]
    if len(info.shape) != 3:
        raise ValueError(f"{tensor_name} has shape {info.shape}, expected [in, out, experts]")
    cols, rows, E = (int(v) for v in info.shape)
    be, bb = BLOCK_GEOMETRY[info.dtype]
    if cols % be:
        raise ValueError(f"{tensor_name}: rows of {cols} are not whole blocks")
    per = rows * (cols // be) * bb
    return [ExpertSlice(info.offset + e * per, per, info.dtype, rows, cols) for e in range(E)]


class PinnedStager:
    """Host->device upload of file byte ranges through ``n_buffers`` pinned
    staging buffers of ``chunk_bytes`` each, on one CUDA stream.  A buffer is
    refilled only after the event recorded behind its previous copy has
    completed, so the host's memcpy out of the page cache for chunk i+1 runs
    while chunk i is on the wire."""

    def __init__(self, device, chunk_bytes: int = 64 << 20, n_buffers: int = 2, stream=None):
        import torch
        self.torch = torch
        self.device = torch.device(device)
        self.chunk = int(chunk_bytes)
        self.bufs = [torch.empty(self.chunk, dtype=torch.uint8).pin_memory()
                     for _ in range(n_buffers)]
        self.events = [None] * n_buffers
        self.stream = stream if stream is not None else torch.cuda.current_stream(self.device)
        self.turn = 0
        self.bytes_moved = 0

    def upload(self, src: memoryview, dst, dst_offset: int = 0) -> None:
        """Copies ``src`` (bytes) into the uint8 device tensor ``dst`` at
        ``dst_offset``, chunk by chunk."""
        torch = self.torch
        n = len(src)
        done = 0
        with torch.cuda.stream(self.stream):
            while done < n:
                k = min(self.chunk, n - done)
                i = self.turn
                self.turn = (self.turn + 1) % len(self.bufs)
                if self.events[i] is not None:
                    self.events[i].synchronize()
                host = self.bufs[i][:k]
                host.numpy()[:] = np.frombuffer(src[done:done + k], dtype=np.uint8)
                dst[dst_offset + done:dst_offset + done + k].copy_(host, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.stream)
                self.events[i] = ev
                done += k
        self.bytes_moved += n

    def finish(self) -> None:
        for ev in self.events:
            if ev is not None:
                ev.synchronize()


def upload_experts(parser: GGUFParser, model: GGUFModel, tensor_name: str,
                   experts: Sequence[int], stager: PinnedStager):
    """The raw blocks of the given experts of one ``ffn_*_exps`` tensor as one
    (len(experts), rows, row bytes) uint8 device tensor, in the given order
    (consecutive experts are one range of the file and one upload)."""
    torch = stager.torch
    sl = expert_slices(model, tensor_name)
    per = sl[0].nbytes
    out = torch.empty(len(experts) * per, dtype=torch.uint8, device=stager.device)
    i = 0
    experts = [int(e) for e in experts]
    while i < len(experts):
        j = i + 1
        while j < len(experts) and experts[j] == experts[j - 1] + 1:
            j += 1
        src = parser.view(model, sl[experts[i]].offset, (j - i) * per)
        stager.upload(src, out, i * per)
        i = j
    rb = per // sl[0].rows
    return out.view(len(experts), sl[0].rows, rb), sl[0]


def upload_tensor(parser: GGUFParser, model: GGUFModel, tensor_name: str, stager: PinnedStager):
    """A whole tensor's raw bytes as a uint8 device tensor."""
    info = model.tensors[tensor_name]
    out = stager.torch.empty(info.nbytes, dtype=stager.torch.uint8, device=stager.device)
    stager.upload(parser.view(model, info.offset, info.nbytes), out)
    return out, info


# ------------------------------------------------------------------- layers

def load_moe_layer(parser: GGUFParser, model: GGUFModel, layer: int, device=None,
                   top_k: Optional[int] = None, mode: Optional[int] = None,
                   experts: Optional[Sequence[int]] = None, stager: Optional[PinnedStager] = None):
    """One block's MoE from the file, on the device.

    * ``ffn_gate_exps`` / ``ffn_up_exps`` / ``ffn_down_exps`` (+ optional
      ``ffn_*_shexp`` shared expert): a ``MoELayer`` with SwiGLU experts and
      the (E, d) ``ffn_gate_inp`` router;
    * ``ffn_gate_up_exps`` (gemma4): a ``Gemma4MoEBlock`` -- fused gate/up,
      ``ffn_down_exps.scale``, ``ffn_gate_inp.scale``, the dense shared MLP
      ``ffn_gate/up/down`` and the four norms.

    ``experts`` limits the upload to those experts (expert-parallel ranks; the
    layer then holds them as experts 0..len-1 and routing is the caller's
    concern -- see ``ep.EPMoELayer(..., local=True)``)."""
    import torch
    from . import _lib
    from .moe_forward import MoELayer
    dev = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    own = stager is None
    stager = stager or PinnedStager(dev)
    p = f"blk.{layer}."
    T = model.tensors
    E = model.expert_count or int(T[p + "ffn_gate_inp.weight"].shape[1])
    k = top_k or model.expert_used_count or 2
    sel = list(range(E)) if experts is None else [int(e) for e in experts]
    router = parser.load_f32(model, p + "ffn_gate_inp.weight")       # (E, d)
    d = int(router.shape[1])
    try:
        if p + "ffn_gate_up_exps.weight" in T:
            from .gemma4 import Gemma4MoEBlock
            gu, gsl = upload_experts(parser, model, p + "ffn_gate_up_exps.weight", sel, stager)
            dn, dsl = upload_experts(parser, model, p + "ffn_down_exps.weight", sel, stager)
            F = gsl.rows // 2
            scale = None
            if p + "ffn_down_exps.scale" in T:
                scale = parser.load_f32(model, p + "ffn_down_exps.scale").reshape(-1)[sel]
            gis = parser.load_f32(model, p + "ffn_gate_inp.scale").reshape(-1) \
                if p + "ffn_gate_inp.scale" in T else None
            sh = [upload_tensor(parser, model, p + f"ffn_{m}.weight", stager) for m in
                  ("gate", "up", "down")]
            Fs = int(sh[0][1].shape[1])
            norms = [parser.load_f32(model, p + f"{n}.weight") if p + f"{n}.weight" in T
                     else None for n in ("ffn_norm", "post_ffw_norm_1", "pre_ffw_norm_2",
                                         "post_ffw_norm_2")]
            stager.finish()
            return Gemma4MoEBlock(router[sel] if experts is not None else router, gis, gu,
                                  gsl.dtype, dn, dsl.dtype, scale, k,
                                  tuple(t for t, _ in sh), sh[0][1].dtype, Fs, *norms,
                                  eps=model.norm_eps, device=dev)
        wg, gsl = upload_experts(parser, model, p + "ffn_gate_exps.weight", sel, stager)
        wu, _ = upload_experts(parser, model, p + "ffn_up_exps.weight", sel, stager)
        wd, dsl = upload_experts(parser, model, p + "ffn_down_exps.weight", sel, stager)
        shared, s_qt, Fs = None, 8, 0
        if p + "ffn_gate_shexp.weight" in T:
            sh = [upload_tensor(parser, model, p + f"ffn_{m}_shexp.weight", stager) for m in
                  ("gate", "up", "down")]
            shared = tuple(t for t, _ in sh)
            s_qt, Fs = sh[0][1].dtype, int(sh[0][1].shape[1])
        stager.finish()
        rmode = _lib.MOE_ROUTE_SOFTMAX_TOPK_RENORM if mode is None else mode
        return MoELayer.from_blocks(router, wg, wu, wd, gsl.dtype, k, shared=shared,
                                    shared_qtype=s_qt, shared_hidden=Fs, mode=rmode, device=dev,
                                    down_qtype=dsl.dtype, router_layout=_lib.MOE_ROUTER_E_D)
    finally:
        if own:
            stager.finish()


# ------------------------------------------------------------------- writing

def _pack_value(v) -> Tuple[int, bytes]:
    if isinstance(v, bool):
        return T_BOOL, struct.pack("<B", int(v))
    if isinstance(v, int):
        return (T_U32, struct.pack("<I", v)) if 0 <= v < (1 << 32) else (T_I64, struct.pack("<q", v))
    if isinstance(v, float):
        return T_F32, struct.pack("<f", v)
    if isinstance(v, str):
        b = v.encode("utf-8")
        return T_STR, struct.pack("<Q", len(b)) + b
    if isinstance(v, (list, tuple)):
        if not v:
            return T_ARR, struct.pack("<IQ", T_U32, 0)
        et, _ = _pack_value(v[0])
        body = b"".join(_pack_value(x)[1] for x in v)
        return T_ARR, struct.pack("<IQ", et, len(v)) + body
    raise TypeError(f"cannot store {type(v).__name__} in GGUF metadata")


def write_gguf(path: str, metadata: dict, tensors: Sequence[Tuple[str, tuple, int, bytes]],
               alignment: int = GGUF_DEFAULT_ALIGNMENT) -> None:
    """Writes a GGUF v3 file.  ``tensors``: (name, ggml shape [contiguous
    dimension first], GGML type, raw bytes); each tensor's data starts on an
    ``alignment`` boundary of the data section."""
    meta = dict(metadata)
    if alignment != GGUF_DEFAULT_ALIGNMENT:
        meta["general.alignment"] = int(alignment)
    head = bytearray(struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(meta)))
    for key, v in meta.items():
        kb = key.encode("utf-8")
        t, body = _pack_value(v)
        head += struct.pack("<Q", len(kb)) + kb + struct.pack("<I", t) + body
    offs, off = [], 0
    for name, shape, dtype, raw in tensors:
        nb = name.encode("utf-8")
        head += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(shape))
        head += b"".join(struct.pack("<Q", int(s)) for s in shape)
        head += struct.pack("<IQ", int(dtype), off)
        offs.append(off)
        off += len(raw)
        off += (alignment - off % alignment) % alignment
    pad = (alignment - len(head) % alignment) % alignment
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * pad)
        pos = 0
        for (name, shape, dtype, raw), o in zip(tensors, offs):
            if o > pos:
                f.write(b"\0" * (o - pos))
                pos = o
            f.write(bytes(raw))
            pos += len(raw)
