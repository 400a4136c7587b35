"""Peer-memory row exchange for the expert-parallel layer.

Replaces the two ``all_to_all_single`` calls of the token-dispatch EP forward
(the rows themselves; reframework/parallel/dist.py:194-206) with one-sided
NVLink stores: every rank owns a receive buffer, a return buffer and a control
block of flag words, allocated with CUDA IPC by the rf_moe library and mapped
by every peer.  ``push`` copies this rank's rows straight into the peers'
buffers (one kernel, folding in the row gather) and raises this rank's flag in
every peer; ``wait`` is a stream-ordered, bounded wait for all sources' flags.
``exchange_counts`` carries the per-step counts all-gather the same way.

Buffer growth is collective: every rank derives the same needed capacity from
the step's all-to-all matrix, so all ranks grow (and re-exchange handles) in
the same step.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import numpy as np
import torch
import torch.distributed as tdist

from .._lib import check, lib, stream_of

__all__ = ["PeerExchange"]

DISPATCH, RETURN = 0, 1


class _Buf:
    """One IPC allocation of this rank and its 64-byte handle."""

    def __init__(self, nbytes: int):
        self.nbytes = int(nbytes)
        p = ctypes.c_void_p()
        h = ctypes.create_string_buffer(64)
        check(lib().rf_moe_peer_alloc(self.nbytes, ctypes.byref(p), h), "rf_moe_peer_alloc")
        self.ptr = int(p.value)
        self.handle = h.raw

    def free(self) -> None:
        if self.ptr:
            check(lib().rf_moe_peer_free(self.ptr), "rf_moe_peer_free")
            self.ptr = 0


class PeerExchange:
    """Receive / return buffers of ``rows x row_bytes`` per rank plus flags."""

    GROWTH = 1.25

    def __init__(self, rank: int, world: int, device: torch.device, group=None, num_experts: int = 0):
        if world > 64:
            raise ValueError("peer exchange supports at most 64 ranks")
        self.rank, self.world, self.device, self.group = rank, world, device, group
        self.num_experts = int(num_experts)
        self.epoch = 0
        self.row_bytes = 0
        self.recv_rows = self.back_rows = 0
        self.own: List[Optional[_Buf]] = [None, None, None]  # recv, back, ctrl
        self.peer: List[List[int]] = [[0] * world for _ in range(3)]
        # control block: dispatch / return flags [2R], the push kernels' block
        # counter, counts flags [R]; then two [R][E] counts tables (step parity)
        self._counts_flags_off = (2 * world + 1) * 4
        self._counts_off = ((3 * world + 1) * 4 + 15) // 16 * 16
        self._ctrl_bytes = self._counts_off + 2 * world * max(self.num_experts, 1) * 4

    # ------------------------------------------------------------ buffers
    def ensure(self, recv_rows: int, back_rows: int, row_bytes: int) -> None:
        """Collective: grow the buffers when any rank needs more rows (every
        rank passes the same maxima, derived from the same matrix)."""
        if (self.own[2] is not None and row_bytes == self.row_bytes and recv_rows <= self.recv_rows
                and back_rows <= self.back_rows):
            return
        torch.cuda.synchronize(self.device)
        if self.own[2] is not None:
            tdist.barrier(group=self.group)  # every peer is done with the old buffers
            self._release()
        self.row_bytes = int(row_bytes)
        self.recv_rows = max(int(recv_rows * self.GROWTH), 1024)
        self.back_rows = max(int(back_rows * self.GROWTH), 1024)
        self.own = [_Buf(self.recv_rows * self.row_bytes), _Buf(self.back_rows * self.row_bytes),
                    _Buf(self._ctrl_bytes)]
        handles = [b.handle for b in self.own]
        allh: List[Optional[list]] = [None] * self.world
        tdist.all_gather_object(allh, handles, group=self.group)
        for r in range(self.world):
            for k in range(3):
                if r == self.rank:
                    self.peer[k][r] = self.own[k].ptr
                else:
                    p = ctypes.c_void_p()
                    check(lib().rf_moe_peer_open(allh[r][k], ctypes.byref(p)), "rf_moe_peer_open")
                    self.peer[k][r] = int(p.value)
        self.epoch = 0
        tdist.barrier(group=self.group)

    def _release(self) -> None:
        for k in range(3):
            for r in range(self.world):
                if r != self.rank and self.peer[k][r]:
                    check(lib().rf_moe_peer_close(self.peer[k][r]), "rf_moe_peer_close")
                self.peer[k][r] = 0
        for b in self.own:
            if b is not None:
                b.free()
        self.own = [None, None, None]

    def close(self) -> None:
        """Collective teardown (all ranks, after their last forward)."""
        if self.own[2] is None:
            return
        torch.cuda.synchronize(self.device)
        tdist.barrier(group=self.group)
        self._release()

    # ------------------------------------------------------------- steps
    def recv_ptr(self) -> int:
        return self.own[0].ptr

    def back_ptr(self) -> int:
        return self.own[1].ptr

    def next_epoch(self) -> int:
        self.epoch = (self.epoch % 0x7FFFFFFF) + 1
        return self.epoch

    def push(self, direction: int, src: torch.Tensor, chunk_off: Sequence[int], dst_row0: Sequence[int],
             idx1: Optional[torch.Tensor] = None, idx2: Optional[torch.Tensor] = None, div: int = 1) -> None:
        """Rows [chunk_off[d], chunk_off[d+1]) of this rank (through idx1/idx2)
        into rank d's receive (DISPATCH) or return (RETURN) buffer at dst_row0[d]."""
        R = self.world
        c_off = (ctypes.c_int64 * (R + 1))(*[int(v) for v in chunk_off])
        c_row0 = (ctypes.c_int64 * R)(*[int(v) for v in dst_row0])
        bufs = self.peer[0] if direction == DISPATCH else self.peer[1]
        c_dst = (ctypes.c_void_p * R)(*bufs)
        flag_off = (direction * R + self.rank) * 4
        c_flag = (ctypes.c_void_p * R)(*[self.peer[2][d] + flag_off for d in range(R)])
        done = self.own[2].ptr + 2 * R * 4
        rc = lib().rf_moe_ep_push_rows(
            src.data_ptr() if src.numel() else None, self.row_bytes,
            None if idx1 is None else idx1.data_ptr(), None if idx2 is None else idx2.data_ptr(), int(div),
            R, self.rank, c_off, c_row0, c_dst, c_flag, self.epoch, done, stream_of(self.device))
        check(rc, "rf_moe_ep_push_rows")

    def exchange_counts(self, counts: torch.Tensor, epoch: int) -> torch.Tensor:
        """The step's counts all-gather over peer memory: this rank's routed
        rows per expert (int32 [E], device) into every rank's table, then a
        bounded wait for every rank's row; returns the [R, E] table (device)."""
        R, E = self.world, self.num_experts
        st = stream_of(self.device)
        toff = self._counts_off + (epoch & 1) * R * E * 4
        dst = (ctypes.c_void_p * R)(*[self.peer[2][d] + toff for d in range(R)])
        flag = (ctypes.c_void_p * R)(*[self.peer[2][d] + self._counts_flags_off + 4 * self.rank for d in range(R)])
        check(lib().rf_moe_ep_counts_push(counts.data_ptr(), E, R, self.rank, dst, flag, epoch, st),
              "rf_moe_ep_counts_push")
        out = torch.empty(R, E, dtype=torch.int32, device=self.device)
        check(lib().rf_moe_ep_counts_collect(self.own[2].ptr + self._counts_flags_off, self.own[2].ptr + toff, R, E,
                                             epoch, out.data_ptr(), st), "rf_moe_ep_counts_collect")
        return out

    def wait(self, direction: int) -> None:
        flags = self.own[2].ptr + direction * self.world * 4
        check(lib().rf_moe_ep_wait(flags, self.world, self.epoch, stream_of(self.device)), "rf_moe_ep_wait")


def matrix_offsets(M: np.ndarray, rank: int):
    """From the all-to-all matrix M[s, d]: this rank's send chunk bounds, the
    first row of its chunk in every destination's receive buffer, its receive
    chunk bounds, and (for the return trip) the first row of each source's
    chunk in that source's return buffer."""
    R = M.shape[0]
    send_off = np.concatenate([[0], np.cumsum(M[rank])])
    dst_row0 = M[:rank].sum(0) if rank else np.zeros(R, np.int64)
    recv_off = np.concatenate([[0], np.cumsum(M[:, rank])])
    back_row0 = M[:, :rank].sum(1) if rank else np.zeros(R, np.int64)
    return send_off, dst_row0, recv_off, back_row0
