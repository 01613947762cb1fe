"""Row sharding of the pair tensor across the GPUs of one node.

The pair tensor z [N, N, 128] is split by rows over P ranks (one process per
GPU, torch.distributed over NCCL): rank r owns rows [offset_r, offset_r + rows_r)
and all N columns, and the single representation rows with the same indices.
The exchanges are the reference's (runtime/dist.py:173-577, trunk/blocks.py):

* triangle multiplication, outgoing: all-gather of b (blocks.py:542-546);
* incoming: all-gather of a and an all-to-all of b (blocks.py:547-555), which
  here arrive as K-chunks that the contraction reads in place;
* triangle attention: all-gather of the pair bias (blocks.py:321-325); the
  ending node also transposes the pair tensor with an all-to-all there and back
  (blocks.py:335-346, :363-364);
* single attention: all-gather of k and v (diffusion/transformer.py:322-330).

Every kernel runs on the rank's own shard through the phase entry points of
``libsparsefold_b200.so``; the collectives are NCCL calls on the current stream.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch
import torch.distributed as dist

from sparsefold_b200 import _native as N
from sparsefold_b200 import ops


class Shard:
  """Row partition of a length-N axis over P ranks (runtime/dist.py:173-235).

  even=True requires N % P == 0; otherwise the sizes are the rounded cumulative
  split with the largest share moved to rank 0.
  """

  def __init__(self, length: int, num_shards: int, rank: int, even: bool = True):
    if even and length % num_shards:
      raise ValueError(f"even partition needs length {length} divisible by {num_shards}")
    self.length, self.num_shards, self.rank, self.is_even = length, num_shards, rank, even
    if even:
      sizes = [length // num_shards] * num_shards
    elif length <= num_shards:
      sizes = [1] * length + [0] * (num_shards - length)
    else:
      sizes, off = [], 0
      step = length / num_shards
      for i in range(num_shards):
        end = int(round((i + 1) * step))
        sizes.append(end - off)
        off = end
      mx = int(np.argmax(sizes))
      sizes[0], sizes[mx] = sizes[mx], sizes[0]
    self._sizes = sizes
    self._offsets = [0] + [int(x) for x in np.cumsum(sizes)[:-1]]

  def sizes(self) -> list[int]:
    return list(self._sizes)

  def offsets(self) -> list[int]:
    return list(self._offsets)

  def size(self, rank: int | None = None) -> int:
    return self._sizes[self.rank if rank is None else rank]

  def offset(self, rank: int | None = None) -> int:
    return self._offsets[self.rank if rank is None else rank]

  def shard(self, x: torch.Tensor, dim: int = 0) -> torch.Tensor:
    return x.narrow(dim, self.offset(), self.size())


class RankFailure(RuntimeError):
  """A peer rank did not reach a step of the sharded path within the time limit."""


def step_barrier(store, step: int, rank: int, world: int, timeout_s: float = 10.0, prefix: str = "sf_step") -> None:
  """Host-side liveness check before the collectives of one sharded step.

  Every rank posts ``{prefix}/{step}/{rank}`` in the process group's key-value
  store and waits, at most ``timeout_s`` seconds, for the other ranks' keys.  A
  rank that raised, exited or never started is reported by index with
  ``RankFailure`` before any collective or kernel of the step is launched, so
  the surviving ranks leave between steps with nothing in flight on their GPUs
  (the reference detects a lost rank only when a collective times out).
  """
  import datetime
  import time
  store.set(f"{prefix}/{step}/{rank}", "1")
  deadline = time.monotonic() + timeout_s
  missing = [r for r in range(world) if r != rank]
  while missing:
    left = deadline - time.monotonic()
    if left <= 0:
      raise RankFailure(f"step {step}: ranks {missing} did not arrive within {timeout_s:.1f} s")
    try:
      store.wait([f"{prefix}/{step}/{missing[0]}"], datetime.timedelta(seconds=max(left, 0.05)))
      missing.pop(0)
    except Exception:   # the store's own timeout (DistStoreError) or a closed connection
      if time.monotonic() >= deadline:
        raise RankFailure(f"step {step}: ranks {missing} did not arrive within {timeout_s:.1f} s") from None
      time.sleep(0.05)


def world_size(group=None) -> int:
  return dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1


# CUDA ranks exchange through sparsefold_b200.p2p (NVLink peer stores, CUDA IPC mappings made
# once per buffer); SF_PEER_EXCHANGE=0 keeps NCCL's all-gather / all-to-all.  A result of the
# peer path lives in the exchange's buffer pool and stays valid for at least two more exchanges
# of its size, which every caller here consumes before.
_PEER: dict = {}


def peer_exchange(group=None):
  """The PeerExchange of a process group (made on first use by every rank), or None when disabled."""
  import os
  if os.environ.get("SF_PEER_EXCHANGE", "1").strip() == "0":
    return None
  key = id(group) if group is not None else 0
  if key not in _PEER:
    from sparsefold_b200 import p2p
    _PEER[key] = p2p.PeerExchange(group)
  return _PEER[key]


def close_peer_exchanges() -> None:
  """Unmap every peer buffer (all ranks, before the process group goes away)."""
  for ex in list(_PEER.values()):
    ex.close()
  _PEER.clear()


def _peer_for(t: torch.Tensor, group, block_bytes: int):
  """The peer exchange for t's blocks of block_bytes each (16-byte multiples), or None (NCCL / gloo)."""
  return peer_exchange(group) if t.is_cuda and block_bytes % 16 == 0 else None


def all_gather_rows(x: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
  """Concatenate every rank's x along dim 0 (equal shards)."""
  world = world_size(group)
  x = x.contiguous()
  if world > 1 and (px := _peer_for(x, group, x.numel() * x.element_size())) is not None:
    res = px.all_gather(x)
    if out is None:
      return res
    out.copy_(res)
    return out
  if out is None:
    out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
  if world == 1:
    out.copy_(x)
  else:
    dist.all_gather_into_tensor(out, x, group=group)
  return out


def all_to_all_rows(send: torch.Tensor, group=None) -> torch.Tensor:
  """send [P * m, ...] -> recv [P * m, ...]: block p of send goes to rank p, block p of recv came from rank p."""
  send = send.contiguous()
  world = world_size(group)
  if world > 1 and (px := _peer_for(send, group, send.numel() * send.element_size() // world)) is not None:
    return px.all_to_all(send)
  recv = torch.empty_like(send)
  dist.all_to_all_single(recv, send, group=group)
  return recv


def _pack_blocks(dst: torch.Tensor, src: torch.Tensor, nblk: int, rows: int, width: int, sbs: int, srs: int,
                 dbs: int, drs: int) -> None:
  """Strided block copy (element strides) on the device: one sf_copy_blocks launch when the layout allows
  16-byte chunks (CUDA tensors), else a torch copy of the same views (CPU ranks)."""
  es = src.element_size()
  if src.is_cuda and (width * es) % 16 == 0 and all((v * es) % 16 == 0 for v in (sbs, srs, dbs, drs)) \
      and src.data_ptr() % 16 == 0 and dst.data_ptr() % 16 == 0:
    N.call("sf_copy_blocks", _p(dst), _p(src), nblk, rows, width * es, sbs * es, srs * es, dbs * es, drs * es,
           _stream())
    return
  d = dst.as_strided((nblk, rows, width), (dbs, drs, 1))
  d.copy_(src.as_strided((nblk, rows, width), (sbs, srs, 1)))


def pair_transpose_to_columns(z_loc: torch.Tensor, shard: Shard, group=None) -> torch.Tensor:
  """[rows_loc, N, C] (row shard) -> [N, cols_loc, C] (column shard), the reshard of
  runtime/dist.py:477-565: block q of the send buffer holds my rows x the columns of rank q."""
  p = shard.num_shards
  r, n, c = z_loc.shape
  cl = n // p
  z_loc = z_loc.contiguous()
  send = torch.empty(p * r, cl, c, dtype=z_loc.dtype, device=z_loc.device)
  _pack_blocks(send, z_loc, p, r, cl * c, cl * c, n * c, r * cl * c, cl * c)
  return all_to_all_rows(send, group).view(n, cl, c)


def pair_transpose_to_rows(z_col: torch.Tensor, shard: Shard, group=None) -> torch.Tensor:
  """[N, cols_loc, C] (column shard) -> [rows_loc, N, C] (row shard)."""
  p = shard.num_shards
  n, cl, c = z_col.shape
  r = n // p
  recv = all_to_all_rows(z_col, group)              # block q: my rows x columns of rank q, [p][r][cl][c]
  out = torch.empty(r, n, c, dtype=z_col.dtype, device=z_col.device)
  _pack_blocks(out, recv, p, r, cl * c, r * cl * c, cl * c, cl * c, n * c)
  return out


def _stream() -> int:
  return torch.cuda.current_stream().cuda_stream


def _p(t):
  return None if t is None else t.data_ptr()


# ---------------------------------------------------------------------------
# sharded ops (bf16)
# ---------------------------------------------------------------------------
# Triangle multiplication on P ranks moves its operands one of two ways:
#  * "rows" (the reference's choreography, blocks.py:541-555): every rank all-gathers the
#    whole b (outgoing) or a^T (incoming) operand, (P-1)/P of [N][C][N] per rank and op;
#  * "channels": every rank contracts C/P channels over all N x N positions; a and b go out
#    by channel block and the product comes back by row block, three all-to-alls of
#    (P-1)/P of the rank's [rows][C][N] each, i.e. 3/P of what "rows" moves (fewer bytes from
#    P = 4 on).
CHANNELS_FROM_RANKS = 4


def tri_mult_mode(p: int) -> str:
  """"rows" or "channels" for P ranks; SF_TRIMULT_SHARDING=rows|channels overrides the choice."""
  import os
  forced = os.environ.get("SF_TRIMULT_SHARDING", "").strip().lower()
  if forced in ("rows", "channels"):
    return forced
  return "channels" if p >= CHANNELS_FROM_RANKS else "rows"


# Channel sub-chunks per rank in the "channels" mode: the all-to-alls of chunk s+1 run on NCCL's
# stream while chunk s contracts, and chunk s's product goes back while chunk s+1 contracts
# (SF_TRIMULT_CHUNKS overrides; 1 = no pipelining).
TRIMULT_CHUNKS = 2


def _trimult_chunks(cl: int) -> int:
  import os
  want = int(os.environ.get("SF_TRIMULT_CHUNKS", TRIMULT_CHUNKS))
  return want if want >= 1 and cl % want == 0 else 1


def _channel_send(op: torch.Tensor, p: int, s: int, sub: int) -> torch.Tensor:
  """[P][m][sub][kp]: block q = channels [q C/P + s sub, + sub) of op [m][C][kp]."""
  m, c, kp = op.shape
  cl = c // p
  op = op.contiguous()
  send = torch.empty(p, m, sub, kp, dtype=op.dtype, device=op.device)
  _pack_blocks(send, op.view(-1)[s * sub * kp:], p, m, sub * kp, cl * kp, c * kp, m * sub * kp, sub * kp)
  return send


def channel_blocks_out_async(op: torch.Tensor, p: int, s: int, sub: int, group=None):
  """Start the all-to-all that takes channels [q C/P + s sub, q C/P + (s+1) sub) of every rank's op
  [m][C][kp] to rank q.  Returns (work, recv [P][m_src][sub][kp], send); keep send alive until the work
  is waited for."""
  m, c, kp = op.shape
  send = _channel_send(op, p, s, sub)
  recv = torch.empty_like(send)
  work = dist.all_to_all_single(recv.view(p * m, sub, kp), send.view(p * m, sub, kp), group=group, async_op=True)
  return work, recv, send


def channel_blocks_out(op: torch.Tensor, p: int, group=None) -> torch.Tensor:
  """op [m][C][kp] (this rank's rows of a contraction operand) -> [P][m_src][C/P][kp]: channel block r
  of every rank's op on rank r (all-to-all; block q of the send buffer = channels q C/P ..)."""
  work, recv, _send = channel_blocks_out_async(op, p, 0, op.shape[1] // p, group)
  work.wait()
  return recv


def _unpack_product(out: torch.Tensor, recv: torch.Tensor, p: int, s: int, sub: int) -> None:
  """recv [P (channel block q)][rows][sub][pn] -> out[:, q C/P + s sub .. + sub, :] of out [rows][C][pn]."""
  rows, c, pn = out.shape
  _pack_blocks(out.view(-1)[s * sub * pn:], recv, p, rows, sub * pn, rows * sub * pn, sub * pn, (c // p) * pn, c * pn)


def channel_blocks_back(prod_c: torch.Tensor, p: int, rows: int, c: int, group=None) -> torch.Tensor:
  """prod_c [N][C/P][pn] (this rank's channels, all rows) -> [rows][C][pn] (all channels, this rank's rows)."""
  n, cl, pn = prod_c.shape
  recv = all_to_all_rows(prod_c.contiguous().view(n, cl, pn), group)      # [P (channel block)][rows][cl][pn]
  out = torch.empty(rows, c, pn, dtype=prod_c.dtype, device=prod_c.device)
  _unpack_product(out, recv.view(p, rows, cl, pn), p, 0, cl)
  return out


def channel_pipeline(a_op: torch.Tensor, b_op: torch.Tensor, p: int, rows: int, pn: int, contract, group=None,
                     chunks: int | None = None) -> torch.Tensor:
  """The data movement of the "channels" mode, in channel sub-chunks.

  a_op, b_op [m][C][kp] are this rank's contraction operands; rank q contracts channels
  [q C/P, (q+1) C/P).  For sub-chunk s (sub = C/P / chunks channels) the operands go out
  by one all-to-all each, ``contract(a_s, b_s, sub)`` (a_s, b_s [P][m_src][sub][kp]) returns
  the sub-chunk's product [N][sub][pn] over all rows, and that goes back by row block.  The
  all-to-alls are asynchronous (NCCL's stream): chunk s+1's operands move while chunk s
  contracts, and chunk s's product returns while chunk s+1 contracts.  Returns this rank's
  rows of the product for every channel, [rows][C][pn]."""
  m, c, kp = a_op.shape
  cl = c // p
  if a_op.is_cuda and peer_exchange(group) is not None:
    # the peer exchanges are synchronous on the stream (and faster than NCCL's all-to-all):
    # operands out, contraction, product back, one chunk
    a_s = all_to_all_rows(_channel_send(a_op, p, 0, cl).view(p * m, cl, kp), group).view(p, m, cl, kp)
    b_s = all_to_all_rows(_channel_send(b_op, p, 0, cl).view(p * m, cl, kp), group).view(p, m, cl, kp)
    prod_s = contract(a_s, b_s, cl).contiguous()
    prod = torch.empty(rows, c, pn, dtype=a_op.dtype, device=a_op.device)
    _unpack_product(prod, all_to_all_rows(prod_s, group).view(p, rows, cl, pn), p, 0, cl)
    return prod
  chunks = _trimult_chunks(cl) if chunks is None else chunks
  sub = cl // chunks
  outs = [(channel_blocks_out_async(a_op, p, s, sub, group), channel_blocks_out_async(b_op, p, s, sub, group))
          for s in range(chunks)]
  prod = torch.empty(rows, c, pn, dtype=a_op.dtype, device=a_op.device)
  backs = []
  for s in range(chunks):
    (wa, ra, _sa), (wb, rb, _sb) = outs[s]
    wa.wait()
    wb.wait()
    prod_s = contract(ra, rb, sub).contiguous()                                   # [N][sub][pn]
    recv = torch.empty_like(prod_s)
    work = dist.all_to_all_single(recv, prod_s, group=group, async_op=True)
    backs.append((work, recv, prod_s))
  for s, (work, recv, _ps) in enumerate(backs):
    work.wait()
    _unpack_product(prod, recv.view(p, rows, sub, pn), p, s, sub)
  return prod


def _tri_mult_channels(mod, z_loc, mask_u8, shard: Shard, w, group=None) -> torch.Tensor:
  rows, n, c = z_loc.shape
  p = shard.num_shards
  if not shard.is_even or c % p:
    raise ValueError("channel-sharded triangle multiplication needs an even row split and C divisible by P")
  dt = N.SF_BF16
  if not mod.incoming:
    pitch = ops.pitch(n)
    a_op = torch.empty(rows, c, pitch, dtype=z_loc.dtype, device=z_loc.device)
    b_op = torch.empty_like(a_op)
    N.call("sf_tri_mult_project_rows", dt, _p(z_loc), _p(mask_u8), rows, n, shard.offset(), 0, C.byref(w), _p(a_op),
           _p(b_op), _stream())
    kchunks = 1                    # each rank's a/b sub-chunk is [P][rows][sub][pitch] = all rows i, K whole
  else:
    if rows % 64 or ops.pitch(rows) != rows:
      raise ValueError(f"incoming triangle multiplication needs shard rows ({rows}) that are multiples of 64")
    a_op = torch.empty(n, c, rows, dtype=z_loc.dtype, device=z_loc.device)   # b^T: [i][C][k_loc]
    b_op = torch.empty_like(a_op)                                             # a^T: [j][C][k_loc]
    N.call("sf_tri_mult_project_rows", dt, _p(z_loc), _p(mask_u8), rows, n, shard.offset(), 1, C.byref(w),
           _p(a_op), _p(b_op), _stream())
    kchunks = p                    # [P (k chunk)][N][sub][k_loc]: K arrives in per-rank chunks
  pn = ops.pitch(n)

  def contract(a_s, b_s, sub):
    prod_s = torch.empty(n, sub, pn, dtype=z_loc.dtype, device=z_loc.device)
    N.call("sf_tri_mult_contract_chunked", dt, _p(a_s), kchunks, _p(b_s), kchunks, _p(prod_s), sub, n, n, n,
           _stream())
    return prod_s

  prod = channel_pipeline(a_op, b_op, p, rows, pn, contract, group)
  out = torch.empty_like(z_loc)
  N.call("sf_tri_mult_output", dt, _p(z_loc), _p(prod), rows, n, C.byref(w), _p(out), None, 0, _stream())
  return out


def tri_mult(mod, z_loc: torch.Tensor, mask_u8: torch.Tensor, shard: Shard, group=None) -> torch.Tensor:
  """TriangleMultiplication (blocks.py:484-566) on a row shard."""
  rows, n, c = z_loc.shape
  p = shard.num_shards
  w = mod.native_weights(z_loc.dtype)
  dt = N.SF_BF16
  if p > 1 and tri_mult_mode(p) == "channels":
    return _tri_mult_channels(mod, z_loc, mask_u8, shard, w, group)
  if not mod.incoming:
    pitch = ops.pitch(n)
    a_op = torch.empty(rows, c, pitch, dtype=z_loc.dtype, device=z_loc.device)
    b_op = torch.empty_like(a_op)
    N.call("sf_tri_mult_project_rows", dt, _p(z_loc), _p(mask_u8), rows, n, shard.offset(), 0, C.byref(w), _p(a_op),
           _p(b_op), _stream())
    b_full = all_gather_rows(b_op, group)                                   # [N][C][pitch]
    chunks_a = chunks_b = 1
  else:
    if p > 1 and (rows % 64 or ops.pitch(rows) != rows):
      raise ValueError(f"incoming triangle multiplication needs shard rows ({rows}) that are multiples of 64")
    pitch = ops.pitch(rows)
    a_send = torch.empty(n, c, pitch, dtype=z_loc.dtype, device=z_loc.device)   # b^T: [i][C][k_loc]
    b_send = torch.empty_like(a_send)                                           # a^T: [j][C][k_loc]
    N.call("sf_tri_mult_project_rows", dt, _p(z_loc), _p(mask_u8), rows, n, shard.offset(), 1, C.byref(w),
           _p(a_send), _p(b_send), _stream())
    a_op = all_to_all_rows(a_send, group) if p > 1 else a_send              # [P][i_loc][C][k_loc]
    b_full = all_gather_rows(b_send, group) if p > 1 else b_send            # [P][N][C][k_loc]
    chunks_a = chunks_b = p
  prod = torch.empty(rows, c, ops.pitch(n), dtype=z_loc.dtype, device=z_loc.device)
  N.call("sf_tri_mult_contract_chunked", dt, _p(a_op), chunks_a, _p(b_full), chunks_b, _p(prod), c, rows, n, n,
         _stream())
  out = torch.empty_like(z_loc)
  N.call("sf_tri_mult_output", dt, _p(z_loc), _p(prod), rows, n, C.byref(w), _p(out), None, 0, _stream())
  return out


def _att_buffers(nb: int, nq: int, dtype, device):
  qp = int(N.load().sf_tri_attention_query_pitch(nq))
  q = torch.empty(nb, 4, qp, 32, dtype=dtype, device=device)
  return qp, q, torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)   # Q, K, V^T, G


def tri_attention(mod, z_loc: torch.Tensor, mask_u8: torch.Tensor, shard: Shard, group=None) -> torch.Tensor:
  """GridSelfAttention (blocks.py:293-366) on a row shard."""
  rows, n, c = z_loc.shape
  w = mod.native_weights(z_loc.dtype)
  dt = N.SF_BF16
  qp = int(N.load().sf_tri_attention_query_pitch(n))
  bias_full = torch.empty(qp, 4, qp, dtype=z_loc.dtype, device=z_loc.device)
  bias_loc = torch.empty(rows, 4, qp, dtype=z_loc.dtype, device=z_loc.device)
  if not mod.transpose:
    _, q, k, vt, g = _att_buffers(rows, n, z_loc.dtype, z_loc.device)
    N.call("sf_tri_attention_project", dt, _p(z_loc), rows, n, 0, 1, C.byref(w), _p(q), _p(k), _p(vt), _p(g),
           _p(bias_loc), _stream())
    all_gather_rows(bias_loc, group, out=bias_full[:n])
    out = torch.empty_like(z_loc)
    N.call("sf_tri_attention_core", dt, _p(q), _p(k), _p(vt), _p(g), _p(bias_full), _p(mask_u8), _p(z_loc), _p(out),
           rows, n, 0, shard.offset(), C.byref(w), _stream())
    return out
  # ending node: the bias comes from the untransposed local rows, the attention runs on columns
  N.call("sf_tri_attention_bias", dt, _p(z_loc), rows, n, C.byref(w), _p(bias_loc), qp, _stream())
  all_gather_rows(bias_loc, group, out=bias_full[:n])
  z_col = pair_transpose_to_columns(z_loc, shard, group) if shard.num_shards > 1 else z_loc
  cols = z_col.shape[1]
  _, q, k, vt, g = _att_buffers(cols, n, z_loc.dtype, z_loc.device)
  N.call("sf_tri_attention_project", dt, _p(z_col), n, cols, 1, 0, C.byref(w), _p(q), _p(k), _p(vt), _p(g), None,
         _stream())
  out_col = torch.empty_like(z_col)
  N.call("sf_tri_attention_core", dt, _p(q), _p(k), _p(vt), _p(g), _p(bias_full), _p(mask_u8), _p(z_col),
         _p(out_col), n, cols, 1, shard.offset(), C.byref(w), _stream())
  return pair_transpose_to_rows(out_col, shard, group) if shard.num_shards > 1 else out_col


def single_update(mod, z_loc: torch.Tensor, s_loc: torch.Tensor, mask: torch.Tensor, shard: Shard,
                  group=None) -> torch.Tensor:
  """SingleActUpdate (blocks.py:739-763) on a row shard: k and v are all-gathered (transformer.py:322-330)."""
  dt = z_loc.dtype
  heads = mod.single_pair_logits_projection.output_shape[0]
  logits = ops.pair_logits(z_loc.contiguous(), mod._kept("ln_w"), mod._kept("ln_b"), mod._packed("logits", dt), heads)
  att = mod.single_attention
  h, d = att._hd
  xn = ops.layer_norm(s_loc, att._kept("ln_ln_w"), att._kept("ln_ln_b"))
  y = ops.linear(xn, att._packed("qkvg", dt), bias=att._kept("qkvg_bias"))     # [rows, 4*H*D]
  y_full = all_gather_rows(y, group) if shard.num_shards > 1 else y
  rows = s_loc.shape[0]
  yl = y.view(rows, 4, h, d)
  yf = y_full.view(-1, 4, h, d)
  o = ops.attention(yl[:, 0], yf[:, 1], yf[:, 2], mask_k=mask, bias=logits, gate=yl[:, 3])
  s_loc = ops.linear(o.reshape(rows, h * d), att._packed("zi_t2", dt), residual=s_loc)
  return mod.single_transition(s_loc, broadcast_dim=None)


def pairformer_block(block, z_loc: torch.Tensor, s_loc: torch.Tensor, mask: torch.Tensor, shard: Shard,
                     group=None):
  """PairFormerIteration.forward (blocks.py:862-910) on a row shard of the pair tensor."""
  if z_loc.dtype != torch.bfloat16:
    raise TypeError("the sharded pair track runs in bf16")
  m8 = ops.mask_u8(mask)
  z_loc = tri_mult(block.triangle_multiplication_outgoing, z_loc, m8, shard, group)
  z_loc = tri_mult(block.triangle_multiplication_incoming, z_loc, m8, shard, group)
  z_loc = tri_attention(block.pair_attention1, z_loc, m8, shard, group)
  z_loc = tri_attention(block.pair_attention2, z_loc, m8, shard, group)
  z_loc = block.pair_transition(z_loc)
  s_loc = single_update(block.single_act_update, z_loc, s_loc, m8, shard, group)
  return z_loc, s_loc


def pairformer_trunk(trunk, z_loc, s_loc, mask, shard: Shard, group=None):
  mask = ops.mask_u8(mask)
  for blk in trunk.blocks:
    z_loc, s_loc = pairformer_block(blk, z_loc, s_loc, mask, shard, group)
  return z_loc, s_loc
