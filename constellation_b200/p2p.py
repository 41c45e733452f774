"""Peer-memory exchange buffers for expert parallelism (one process per GPU on one node).

Each rank allocates one device buffer through ``cst_ipc_alloc``:

* ``world * tl_cap`` receive slots of ``hidden`` fp32 (slot r holds what rank r pushed for
  this rank's tokens);
* ``world * tl_cap`` gathered rows of ``hidden`` 2-byte elements (the all-gather of the
  tokens, rank-major);
* 64 int32: combine arrival counters at [0, world), gather arrival counters at [8, 8 +
  world), the combine epoch at [32], a reserved word at [33], the gather epoch at [34];
* ``world * tl_cap`` presence words (int32): rank r writes 0 for a token of this rank it
  has no row for and pushes nothing for it; the reduce skips that slot (at a decode batch
  about a third of the (rank, token) partials are empty, at a skewed prefill most are).

The ranks swap the CUDA IPC handles with one all-gather, so every rank maps every other
rank's buffer.  ``cst_gather_rows`` stores each rank's rows into every rank's gathered
rows; ``cst_moe_routed_push`` stores each gathered token's partial sum straight into its
owner's slot over NVLink and ``cst_reduce_pushed`` adds the slots in rank order on the
owner.  Both halves of the all-gather exchange thus run over peer memory
(``constellation_b200.ep``, mode ``"p2p"``).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _dlpack, _lib
from ._lib import CST_MAX_PEERS, CstIpcHandle, CstPeerSet, check

_TAIL_INTS = 64  # combine flags [0, world), gather flags [8, 8 + world), epochs at [32] and [34]


class PeerExchange:
    """One rank's exchange buffers and its mappings of every other rank's.  Other ranks may
    still push into this rank's buffer, so nothing frees it implicitly: ``close()`` -- on
    every rank, after a barrier -- releases it, or the process exit does."""

    def __init__(self, device, *, world: int, rank: int, tl_cap: int, hidden: int, group=None):
        if not 1 <= world <= CST_MAX_PEERS:
            raise ValueError(f"peer exchange supports 1..{CST_MAX_PEERS} ranks, got {world}")
        self.device = torch.device(device)
        self.world, self.rank, self.tl_cap, self.hidden = int(world), int(rank), int(tl_cap), int(hidden)
        self.slot_bytes = self.world * self.tl_cap * self.hidden * 4
        self.x_off = self.slot_bytes
        self.x_bytes = self.world * self.tl_cap * self.hidden * 2
        self.tail_off = self.x_off + self.x_bytes
        # presence words [world][tl_cap]: a rank with no row for a token pushes only a 0 here
        self.pres_off = self.tail_off + _TAIL_INTS * 4
        nbytes = self.pres_off + self.world * self.tl_cap * 4
        own = ctypes.c_void_p()
        handle = CstIpcHandle()
        with torch.cuda.device(self.device):
            check(_lib.lib.cst_ipc_alloc(nbytes, ctypes.byref(own), ctypes.byref(handle)))
        self._own = own.value
        self._opened: list[int] = []
        mine = torch.tensor(list(bytes(handle.bytes)), dtype=torch.uint8, device=self.device)
        every = torch.empty((self.world, 64), dtype=torch.uint8, device=self.device)
        if self.world > 1:
            dist.all_gather_into_tensor(every, mine, group=group)
        else:
            every[0].copy_(mine)
        rows = every.cpu().tolist()
        bases = []
        with torch.cuda.device(self.device):
            for q in range(self.world):
                if q == self.rank:
                    bases.append(self._own)
                    continue
                h = CstIpcHandle()
                h.bytes[:] = rows[q]
                p = ctypes.c_void_p()
                check(_lib.lib.cst_ipc_open(ctypes.byref(h), ctypes.byref(p)))
                self._opened.append(p.value)
                bases.append(p.value)
        self.bases = bases

    def peer_set(self, tl: int) -> CstPeerSet:
        """The ABI view of the buffers for an exchange with ``tl`` tokens per rank."""
        if not 0 < tl <= self.tl_cap:
            raise ValueError(f"tl={tl} outside (0, {self.tl_cap}]")
        ps = CstPeerSet()
        ps.world, ps.rank, ps.tl, ps.tl_cap = self.world, self.rank, int(tl), self.tl_cap
        for q, b in enumerate(self.bases):
            ps.recv[q] = b
            ps.flags[q] = b + self.tail_off
        tail = self._own + self.tail_off
        ps.epoch = tail + 32 * 4
        ps.done = tail + 33 * 4
        ps.x_offset = self.x_off
        ps.gather_epoch = tail + 34 * 4
        ps.presence_offset = self.pres_off
        return ps

    def gathered(self, tl: int, dtype: torch.dtype) -> torch.Tensor:
        """This rank's gathered rows ``[world * tl, hidden]`` (a view of the exchange buffer,
        valid until ``close()``), filled by ``ExpertContext.gather_rows``."""
        if dtype not in (torch.bfloat16, torch.float16):
            raise TypeError(f"gathered rows are 2-byte, got {dtype}")
        return _dlpack.view(self._own + self.x_off, (self.world * int(tl), self.hidden), dtype, self.device)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after every rank stopped using them)."""
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.lib.cst_ipc_close(p)
            self._opened = []
            if self._own:
                _lib.lib.cst_ipc_free(self._own)
                self._own = 0
