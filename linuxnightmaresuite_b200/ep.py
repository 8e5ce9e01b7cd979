"""Expert-parallel MoE layer, one process per GPU of a node.

Each of the W ranks owns a contiguous block of E / W experts and its own
tokens.  ``EPMoELayer`` runs one layer step as device work only, through
``moe_ep_forward``: router -> dispatch -> the routed rows are stored straight
into the owners' exchange windows over NVLink (CUDA IPC mappings) -> each owner
runs its experts on the rows it received -> the outputs are stored straight
back into the sources' windows -> combine.  Release/acquire flags carrying a
step counter order the two exchanges; there is no host synchronisation and no
collective library on the data path (torch.distributed only shares the IPC
handles at set-up).

The reference has no collective at all: its multi-GPU MoE uploads the token
to every card and sums per-expert outputs on the host
(nightmare_stream.py:4381-4449).

The bookkeeping of the exchange (``exchange_plan``, ``local_order``) is also
written out in numpy, with a collective version (``ep_exchange``) that runs on
CPU ranks (gloo); it states what the device kernels compute.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist


def _rows(a, sl=slice(None)):
    """Contiguous expert rows of a raw block stack (numpy array or tensor)."""
    if isinstance(a, torch.Tensor):
        return a[sl].contiguous()
    return np.ascontiguousarray(a[sl])


def expert_range(rank: int, world: int, n_experts: int) -> Tuple[int, int]:
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split over {world} ranks")
    per = n_experts // world
    return rank * per, (rank + 1) * per


def exchange_plan(offsets: np.ndarray, world: int) -> Tuple[np.ndarray, np.ndarray]:
    """From this rank's expert offsets (E+1, sorted-row boundaries) return
    (send_rows[W], send_counts[W, E/W]): rows bound for each owner and the
    per-expert split inside each owner's block."""
    offsets = np.asarray(offsets, dtype=np.int64)
    E = offsets.size - 1
    per = E // world
    counts = np.diff(offsets).reshape(world, per)
    return counts.sum(axis=1), counts


def local_order(recv_counts: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """recv_counts[src, e]: rows source ``src`` sent for local expert ``e``,
    laid out in the receive buffer source-major, expert-minor (each source's
    block is its sorted rows).  Returns (local_offsets[E_local+1], row_map[R]):
    expert-sorted row r of this rank reads (and writes) receive-buffer row
    row_map[r]; inside an expert, rows keep source order, then the source's
    own (token, slot) order."""
    rc = np.asarray(recv_counts, dtype=np.int64)
    W, El = rc.shape
    src_base = np.zeros((W, El), dtype=np.int64)
    flat = rc.reshape(-1)
    starts = np.concatenate([[0], np.cumsum(flat)[:-1]]).reshape(W, El)
    src_base[:] = starts
    per_expert = rc.sum(axis=0)
    offs = np.zeros(El + 1, dtype=np.int64)
    offs[1:] = np.cumsum(per_expert)
    row_map = np.empty(int(offs[-1]), dtype=np.int64)
    for e in range(El):
        pos = offs[e]
        for s in range(W):
            n = rc[s, e]
            row_map[pos:pos + n] = np.arange(src_base[s, e], src_base[s, e] + n)
            pos += n
    return offs.astype(np.int32), row_map.astype(np.int32)


def all_to_all_rows(send: torch.Tensor, send_rows: Sequence[int], recv_rows: Sequence[int],
                    group=None) -> torch.Tensor:
    """Variable-split all-to-all of row blocks (any device / backend)."""
    d = send.shape[1]
    recv = torch.empty((int(sum(recv_rows)), d), dtype=send.dtype, device=send.device)
    dist.all_to_all_single(recv, send, output_split_sizes=[int(v) for v in recv_rows],
                           input_split_sizes=[int(v) for v in send_rows], group=group)
    return recv


def ep_exchange(send: torch.Tensor, counts: torch.Tensor, expert_fn, group=None) -> torch.Tensor:
    """Steps 3-6.  ``send``: this rank's routed rows in expert-sorted order;
    ``counts`` (W, E/W) int32: rows per destination expert.  ``expert_fn(recv,
    local_offsets, row_map)`` returns the expert outputs for the received rows,
    in receive order.  Returns the outputs of this rank's rows, in its sorted
    order."""
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts, group=group)
    c_host = counts.cpu().numpy()
    rc_host = recv_counts.cpu().numpy()
    send_rows = c_host.sum(axis=1)
    recv_rows = rc_host.sum(axis=1)
    recv = all_to_all_rows(send, send_rows, recv_rows, group)
    loff, row_map = local_order(rc_host)
    y_recv = expert_fn(recv, loff, row_map)
    return all_to_all_rows(y_recv, recv_rows, send_rows, group)


class EPExchange:
    """The exchange window of this rank (and the mapped windows of the other
    ranks), a step workspace and the step counter.  Layers of the same shape
    can share one: each step's exchange completes before the next starts."""

    def __init__(self, group, device):
        from . import kernels as K
        from . import _lib
        self.K, self._lib = K, _lib
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device
        self.key = None
        self.window = None
        self._mapped = []
        self.epoch = 0

    def ensure(self, lw, T: int) -> None:
        """(Re)build the windows for steps of T tokens (collective)."""
        key = (lw.E, lw.k, lw.d, lw.F, lw.Fs, T)
        if self.key == key:
            return
        _lib, K = self._lib, self.K
        self.close()
        W, rank = self.world, self.rank
        nbytes = ctypes.c_size_t(0)
        _lib.call("moe_ep_window_bytes", W, lw.E, T, lw.k, lw.d, ctypes.byref(nbytes))
        win = ctypes.c_void_p(0)
        _lib.call("moe_ipc_alloc", nbytes.value, ctypes.byref(win))
        self.window = win.value
        handle = (ctypes.c_uint8 * 64)()
        _lib.call("moe_ipc_handle", ctypes.c_void_p(self.window), ctypes.cast(handle, ctypes.c_void_p))
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        allh = [torch.empty_like(mine) for _ in range(W)]
        dist.all_gather(allh, mine, group=self.group)
        ptrs = []
        for s_ in range(W):
            if s_ == rank:
                ptrs.append(self.window)
                continue
            h = (ctypes.c_uint8 * 64)(*allh[s_].cpu().tolist())
            p = ctypes.c_void_p(0)
            _lib.call("moe_ipc_open", ctypes.cast(h, ctypes.c_void_p), ctypes.byref(p))
            self._mapped.append(p.value)
            ptrs.append(p.value)
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        wsb = ctypes.c_size_t(0)
        _lib.call("moe_ep_workspace_bytes", ctypes.byref(lw.c), W, T, ctypes.byref(wsb))
        self.ws = K.workspace(wsb.value, self.device)
        self.ws[:256].zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.key = key
        self.epoch = 0

    def close(self) -> None:
        """Unmap the peers' windows and free this rank's (collective)."""
        if self.window is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._mapped:
            self._lib.call("moe_ipc_close", ctypes.c_void_p(p))
        self._mapped = []
        dist.barrier(group=self.group)
        self._lib.call("moe_ipc_free", ctypes.c_void_p(self.window))
        self.window = None
        self.key = None


class EPMoELayer:
    """One MoE layer sharded over the ranks of ``group`` by expert; this rank
    holds experts ``expert_range(rank, W, E)`` and routes its own tokens.

    w_gate / w_up / w_down: raw block stacks of all E experts, or of this
    rank's experts only with ``local=True``.  ``shared``: an always-on shared
    expert (three raw block arrays), run on this rank's own tokens.
    ``exchange``: an ``EPExchange`` to share with other layers."""

    def __init__(self, gate_weight, w_gate, w_up, w_down, qtype: int, top_k: int,
                 mode: int = 0, bias=None, group=None, device=None, shared=None,
                 shared_qtype: int = 8, local: bool = False,
                 exchange: Optional[EPExchange] = None):
        from . import kernels as K
        from . import _lib
        from .moe_forward import _to_dev_u8, _device
        self.K, self._lib = K, _lib
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = _device(device)
        d, E = int(gate_weight.shape[0]), int(gate_weight.shape[1])
        self.d, self.E, self.k, self.qtype, self.mode = d, E, top_k, qtype, mode
        self.e0, self.e1 = expert_range(self.rank, self.world, E)
        self.F = int(w_gate.shape[1])
        dev = self.device
        self.gate_w = torch.as_tensor(np.ascontiguousarray(gate_weight, dtype=np.float32)).to(dev)
        self.bias = None if bias is None else torch.as_tensor(
            np.ascontiguousarray(bias, dtype=np.float32)).to(dev)
        El = self.e1 - self.e0
        sl = slice(0, El) if local else slice(self.e0, self.e1)
        if local and int(w_gate.shape[0]) != El:
            raise ValueError(f"local weights hold {w_gate.shape[0]} experts, rank owns {El}")
        self.w_gate = K.pack_weights(_to_dev_u8(_rows(w_gate, sl), dev), qtype, El, self.F, d)
        self.w_up = K.pack_weights(_to_dev_u8(_rows(w_up, sl), dev), qtype, El, self.F, d)
        self.w_down = K.pack_weights(_to_dev_u8(_rows(w_down, sl), dev), qtype, El, d, self.F)
        sh, Fs = None, 0
        if shared is not None:
            sg, su, sd = shared
            Fs = int(sg.shape[-2])
            sh = (K.pack_weights(_to_dev_u8(_rows(sg), dev), shared_qtype, 1, Fs, d),
                  K.pack_weights(_to_dev_u8(_rows(su), dev), shared_qtype, 1, Fs, d),
                  K.pack_weights(_to_dev_u8(_rows(sd), dev), shared_qtype, 1, d, Fs))
        self.lw = K.LayerWeights(self.gate_w, self.w_gate, self.w_up, self.w_down, qtype, E,
                                 top_k, d, self.F, mode, self.bias, shared=sh,
                                 shared_qtype=shared_qtype, Fs=Fs)
        self.exchange = exchange if exchange is not None else EPExchange(group, dev)

    def close(self) -> None:
        self.exchange.close()

    # ------------------------------------------------------------------ step
    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One expert-parallel step for this rank's tokens x (T, d); every rank
        calls it with the same T.  x and out may be pinned host tensors (the
        layer's kernels read and write them over the bus)."""
        K, ex = self.K, self.exchange
        K._need(x, torch.float32, "x", pinned_ok=True)
        if out is not None:
            K._need(out, torch.float32, "out", pinned_ok=True)
        T = int(x.shape[0])
        ex.ensure(self.lw, T)
        if out is None:
            out = torch.empty_like(x) if x.is_cuda else torch.empty(x.shape, dtype=x.dtype,
                                                                     pin_memory=True)
        ex.epoch += 1
        self._lib.call("moe_ep_forward", ctypes.byref(self.lw.c), self.world, self.rank,
                       ctypes.c_void_p(ex.peers.data_ptr()), ctypes.c_void_p(ex.window),
                       K._ptr(x), T, K._ptr(out), K._ptr(residual), ex.epoch, K._ptr(ex.ws),
                       ex.ws.numel(), K._stream())
        return out

    def device_status(self) -> int:
        ex = self.exchange
        return self.K.read_status(ex.ws) if ex.window is not None else 0

    def routing_stats(self, x: torch.Tensor) -> Tuple[int, int]:
        """(active local experts, rows this rank's experts receive) for a step
        on x: routes every rank's tokens and sums the per-expert counts over
        the ranks (a collective with a host read; not for timed regions)."""
        K = self.K
        ids, _ = K.router(x, self.gate_w, self.k, self.mode, self.bias)
        cnt = torch.bincount(ids.reshape(-1).long(), minlength=self.E).to(torch.int64)
        dist.all_reduce(cnt, group=self.group)
        local = cnt[self.e0:self.e1].cpu().numpy()
        return int(np.count_nonzero(local)), int(local.sum())


class EPLocalRanks:
    """All W ranks of an expert-parallel layer driven by one process on one
    device: W windows, W workspaces and W expert shards in the same HBM, the
    same device code as one process per GPU (``moe_ep_forward_phases``).

    A step runs the send phase of every rank, then the serve phase of every
    rank, then the combine phase of every rank, all on one stream.  Each wait
    in a phase is then satisfied by work that has already completed in stream
    order, so no kernel depends on another one being scheduled at the same
    time.  This exercises the exchange windows, the counts and positions, the
    owner-side expert order and the return path on a single GPU.

    Arguments as ``EPMoELayer`` (all E experts' raw blocks), plus ``world``."""

    def __init__(self, gate_weight, w_gate, w_up, w_down, qtype: int, top_k: int, world: int,
                 mode: int = 0, bias=None, device=None, shared=None, shared_qtype: int = 8):
        from . import kernels as K
        from . import _lib
        from .moe_forward import _to_dev_u8, _device
        self.K, self._lib = K, _lib
        self.world = int(world)
        self.device = _device(device)
        dev = self.device
        d, E = int(gate_weight.shape[0]), int(gate_weight.shape[1])
        self.d, self.E, self.k, self.qtype, self.mode = d, E, top_k, qtype, mode
        self.F = int(w_gate.shape[1])
        self.gate_w = torch.as_tensor(np.ascontiguousarray(gate_weight, dtype=np.float32)).to(dev)
        self.bias = None if bias is None else torch.as_tensor(
            np.ascontiguousarray(bias, dtype=np.float32)).to(dev)
        sh, Fs = None, 0
        if shared is not None:
            sg, su, sd = shared
            Fs = int(sg.shape[-2])
            sh = (K.pack_weights(_to_dev_u8(_rows(sg), dev), shared_qtype, 1, Fs, d),
                  K.pack_weights(_to_dev_u8(_rows(su), dev), shared_qtype, 1, Fs, d),
                  K.pack_weights(_to_dev_u8(_rows(sd), dev), shared_qtype, 1, d, Fs))
        self.lws = []
        for r in range(self.world):
            e0, e1 = expert_range(r, self.world, E)
            El = e1 - e0
            sl = slice(e0, e1)
            wg = K.pack_weights(_to_dev_u8(_rows(w_gate, sl), dev), qtype, El, self.F, d)
            wu = K.pack_weights(_to_dev_u8(_rows(w_up, sl), dev), qtype, El, self.F, d)
            wd = K.pack_weights(_to_dev_u8(_rows(w_down, sl), dev), qtype, El, d, self.F)
            self.lws.append(K.LayerWeights(self.gate_w, wg, wu, wd, qtype, E, top_k, d, self.F,
                                           mode, self.bias, shared=sh, shared_qtype=shared_qtype,
                                           Fs=Fs))
        self.T = None
        self.epoch = 0

    def _ensure(self, T: int) -> None:
        if self.T == T:
            return
        _lib, K = self._lib, self.K
        W = self.world
        nbytes = ctypes.c_size_t(0)
        _lib.call("moe_ep_window_bytes", W, self.E, T, self.k, self.d, ctypes.byref(nbytes))
        self.windows = [torch.zeros(nbytes.value, dtype=torch.uint8, device=self.device)
                        for _ in range(W)]
        self.peers = torch.tensor([w.data_ptr() for w in self.windows], dtype=torch.int64,
                                  device=self.device)
        wsb = ctypes.c_size_t(0)
        _lib.call("moe_ep_workspace_bytes", ctypes.byref(self.lws[0].c), W, T, ctypes.byref(wsb))
        self.wss = [torch.zeros(max(wsb.value, 256), dtype=torch.uint8, device=self.device)
                    for _ in range(W)]
        self.T = T
        self.epoch = 0

    def forward(self, xs, residuals=None, outs=None):
        """xs: W tensors (T, d) f32, rank r's tokens in xs[r].  Returns the W
        outputs.  Device work only."""
        K, _lib = self.K, self._lib
        W = self.world
        if len(xs) != W:
            raise ValueError(f"{len(xs)} token blocks for {W} ranks")
        T = int(xs[0].shape[0])
        for x in xs:
            K._need(x, torch.float32, "x", pinned_ok=True)
            if int(x.shape[0]) != T:
                raise ValueError("every rank must bring the same number of tokens")
        self._ensure(T)
        if outs is None:
            outs = [torch.empty_like(x) if x.is_cuda else
                    torch.empty(x.shape, dtype=x.dtype, pin_memory=True) for x in xs]
        res = residuals if residuals is not None else [None] * W
        self.epoch += 1
        for phase in (_lib.MOE_EP_PHASE_SEND, _lib.MOE_EP_PHASE_SERVE, _lib.MOE_EP_PHASE_COMBINE):
            for r in range(W):
                _lib.call("moe_ep_forward_phases", ctypes.byref(self.lws[r].c), W, r,
                          ctypes.c_void_p(self.peers.data_ptr()),
                          ctypes.c_void_p(self.windows[r].data_ptr()), K._ptr(xs[r]), T,
                          K._ptr(outs[r]), K._ptr(res[r]), self.epoch, phase,
                          K._ptr(self.wss[r]), self.wss[r].numel(), K._stream())
        return outs

    def device_status(self):
        """Per-rank device status words (reads and clears them; synchronises)."""
        if self.T is None:
            return [0] * self.world
        return [self.K.read_status(ws) for ws in self.wss]
