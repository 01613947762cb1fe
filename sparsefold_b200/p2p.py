"""Peer exchanges over NVLink for the row-sharded path (one process per GPU, one box).

``PeerExchange`` maps every rank's receive buffers into its peers once (CUDA IPC through
``sf_ipc_export`` / ``sf_ipc_import``, the handles passed over the process group), and an
exchange is then: this rank writes each block straight into the owning peer's buffer with
16-byte stores from the SMs (``sf_scatter_peers``), raises its flag word in every peer
(``sf_peer_signal``), and the stream waits, bounded, for every peer's flag of the same
exchange (``sf_peer_wait``).  It replaces the all-to-all and all-gather of
runtime/dist.py:477-565 between the ranks of one box; everything stays on the current stream.

Buffers: a pool of ``slots`` receive buffers per size, in turn; a result is overwritten
``slots`` exchanges of its size later.  When rank r writes exchange e into a peer's buffer it
has seen every peer's flag of exchange e-1, which a peer raises only after the work queued
before it (the consumers of its earlier exchanges) has run, so a buffer is never written while
its previous contents are still to be read, for any ``slots`` >= 2.  All ranks must call the
exchanges in the same order (as they do collectives).
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from sparsefold_b200 import _native as N


def _stream() -> int:
  return torch.cuda.current_stream().cuda_stream


class PeerExchange:
  def __init__(self, group=None, slots: int = 3, polls: int = 1 << 24):
    if slots < 2:
      raise ValueError("PeerExchange needs at least two buffers per size")
    self.group = group
    self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
    if self.world > 32:
      raise ValueError("PeerExchange takes at most 32 ranks")
    self.slots, self.polls = slots, polls
    self.epoch = 0
    self.flags = torch.zeros(self.world, dtype=torch.int32, device="cuda")   # flags[q]: raised by rank q
    self._flag_ptrs = self._share(self.flags)
    self._pool: dict[int, dict] = {}

  def _share(self, t: torch.Tensor) -> list[int]:
    """Pointers to every rank's copy of t (this rank's own, the peers' mapped here)."""
    handle, off = C.create_string_buffer(64), C.c_uint64()
    N.call("sf_ipc_export", C.c_void_p(t.data_ptr()), handle, C.byref(off))
    mine = (handle.raw, off.value)
    every = [None] * self.world
    dist.all_gather_object(every, mine, group=self.group)
    ptrs = []
    for q, (hb, o) in enumerate(every):
      if q == self.rank:
        ptrs.append(t.data_ptr())
        continue
      p = C.c_void_p()
      N.call("sf_ipc_import", C.create_string_buffer(hb, 64), o, C.byref(p))
      ptrs.append(p.value)
    return ptrs

  def _buffer(self, nbytes: int):
    ent = self._pool.setdefault(nbytes, {"bufs": [], "next": 0})
    i = ent["next"]
    ent["next"] = (i + 1) % self.slots
    if i == len(ent["bufs"]):
      t = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
      ptrs = self._share(t)
      ent["bufs"].append((t, torch.tensor(ptrs, dtype=torch.int64, device="cuda")))
    return ent["bufs"][i]

  def _sync(self) -> None:
    self.epoch += 1
    for q in range(self.world):
      if q != self.rank:
        N.call("sf_peer_signal", C.c_void_p(self._flag_ptrs[q] + 4 * self.rank), self.epoch & 0xFFFFFFFF, _stream())
    N.call("sf_peer_wait", C.c_void_p(self.flags.data_ptr()), self.world, self.rank, self.epoch & 0xFFFFFFFF,
           self.polls, _stream())

  def all_to_all(self, send: torch.Tensor) -> torch.Tensor:
    """send [P * m, ...] -> recv [P * m, ...]: block q of send goes to rank q, block q of recv came from
    rank q (the semantics of ``all_to_all_single`` with equal splits)."""
    send = send.contiguous()
    nbytes = send.numel() * send.element_size()
    if nbytes % (16 * self.world):
      raise ValueError("PeerExchange.all_to_all needs blocks of a multiple of 16 bytes")
    blk = nbytes // self.world
    buf, dptrs = self._buffer(nbytes)
    N.call("sf_scatter_peers", C.c_void_p(send.data_ptr()), C.c_void_p(dptrs.data_ptr()), self.world, blk, blk,
           self.rank * blk, _stream())
    self._sync()
    return buf.view(send.dtype).view(send.shape)

  def all_gather(self, x: torch.Tensor) -> torch.Tensor:
    """x [m, ...] on every rank -> [P * m, ...], rank q's x at block q."""
    x = x.contiguous()
    nbytes = x.numel() * x.element_size()
    if nbytes % 16:
      raise ValueError("PeerExchange.all_gather needs a multiple of 16 bytes")
    buf, dptrs = self._buffer(nbytes * self.world)
    N.call("sf_scatter_peers", C.c_void_p(x.data_ptr()), C.c_void_p(dptrs.data_ptr()), self.world, nbytes, 0,
           self.rank * nbytes, _stream())
    self._sync()
    return buf.view(x.dtype).view((self.world * x.shape[0],) + tuple(x.shape[1:]))

  def close(self) -> None:
    """Unmap the peers' buffers (every rank, after its last exchange has run)."""
    torch.cuda.synchronize()
    dist.barrier(group=self.group)
    N.call("sf_ipc_close_all")
    dist.barrier(group=self.group)
    self._pool.clear()
