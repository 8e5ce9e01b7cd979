"""Expert-parallel MoE layer over torch.distributed (NCCL on B200s).

Each of the W ranks owns a contiguous block of E / W experts and its own
tokens.  One layer forward:

1. route the rank's tokens with the full router (all E experts);
2. stable-sort the (token, slot) pairs by expert (``moe_dispatch``); because
   experts are contiguous per rank, the sorted rows are grouped by owner;
3. exchange per-expert row counts (one small all-to-all) -- this fixes every
   split of the payload exchange;
4. all-to-all the routed activation rows to the experts' owners;
5. run the owner's experts on the received rows, in expert order
   (``moe_experts`` with a gather / scatter row map), writing each result back
   into its received position;
6. all-to-all the results back (the reverse splits);
7. combine each token's k results in router order (``moe_combine``).

The reference has no collective at all: its multi-GPU MoE uploads the token
to every card and sums per-expert outputs on the host
(nightmare_stream.py:4381-4449).

The bookkeeping of steps 3-5 (``exchange_plan``, ``local_order``) is plain
numpy so it can be checked on CPU ranks; ``EPMoELayer`` drives the device
kernels.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist


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


class EPMoELayer:
    """One MoE layer sharded over the ranks of ``group`` by expert."""

    def __init__(self, gate_weight, w_gate, w_up, w_down, qtype: int, top_k: int,
                 mode: int = 0, bias=None, group=None, device=None):
        from . import kernels as K
        from .moe_forward import MoERouter, _to_dev_u8, _device
        self.K = K
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = _device(device)
        d, E = int(gate_weight.shape[0]), int(gate_weight.shape[1])
        self.d, self.E, self.k, self.qtype = d, E, top_k, qtype
        self.e0, self.e1 = expert_range(self.rank, self.world, E)
        self.F = int(w_gate.shape[1])
        self.router = MoERouter(gate_weight, E, top_k, mode, bias, self.device)
        sl = slice(self.e0, self.e1)
        El = self.e1 - self.e0
        self.w_gate = K.pack_weights(_to_dev_u8(np.ascontiguousarray(w_gate[sl]), self.device),
                                     qtype, El, self.F, d)
        self.w_up = K.pack_weights(_to_dev_u8(np.ascontiguousarray(w_up[sl]), self.device),
                                   qtype, El, self.F, d)
        self.w_down = K.pack_weights(_to_dev_u8(np.ascontiguousarray(w_down[sl]), self.device),
                                     qtype, El, d, self.F)
        self._ws = None
        self.last = {}

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """All device work; one small device->host read per step (the row
        counts, which NCCL needs as split sizes)."""
        K = self.K
        ids, w = self.router.route_batch(x)
        off, perm, inv = K.dispatch(ids, self.E)
        counts = torch.diff(off).to(torch.int32).reshape(self.world, -1)
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        send = K.gather_rows(x, perm, self.k)          # expert-sorted, owner-grouped
        both = torch.stack([counts, recv_counts]).cpu().numpy()
        send_rows = both[0].sum(axis=1)
        recv_rows = both[1].sum(axis=1)
        recv = all_to_all_rows(send, send_rows, recv_rows, self.group)
        R = int(recv_rows.sum())
        self.last = {"rows": R, "active": int(np.count_nonzero(both[1].sum(axis=0)))}
        y_recv = torch.empty((R, self.d), dtype=torch.float32, device=x.device)
        if R:
            if self._ws is None or self._ws.device != x.device:
                self._ws = torch.zeros(256, dtype=torch.uint8, device=x.device)
            loff, row_map = K.ep_local_order(recv_counts, R, self._ws)
            K.experts(self.w_gate, self.w_up, self.w_down, self.qtype, loff, recv, self.d, self.F,
                      x_rows=row_map, x_rows_div=1, y=y_recv, y_rows=row_map, rows=R)
        y_sorted = all_to_all_rows(y_recv, recv_rows, send_rows, self.group)
        return K.combine(y_sorted, inv, w)
