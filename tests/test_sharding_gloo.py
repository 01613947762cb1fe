"""Host logic of the row-sharded path on CPU ranks (gloo, world sizes 2 and 4).

The kernels are CUDA-only; these tests cover the partition rule, the collective
helpers, the pair transpose between row and column shards, and the layout
choreography of the incoming triangle multiplication (operands assembled as
per-rank K-chunks), with the contraction emulated in torch against the oracle.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sparsefold_b200.sharding import Shard, all_gather_rows, all_to_all_rows, pair_transpose_to_columns, \
    pair_transpose_to_rows


def test_shard_even_and_ragged_rules():
  s = Shard(2048, 8, rank=3)
  assert s.sizes() == [256] * 8 and s.offset() == 768 and s.size() == 256
  r = Shard(10, 4, rank=0, even=False)          # rounded cumulative split, largest share on rank 0
  assert sum(r.sizes()) == 10 and r.sizes()[0] == max(r.sizes())
  assert r.offsets() == [0] + list(torch.tensor(r.sizes()).cumsum(0)[:-1].tolist())
  assert Shard(3, 4, rank=3, even=False).sizes() == [1, 1, 1, 0]
  with pytest.raises(ValueError):
    Shard(10, 4, rank=0, even=True)


def _free_port():
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    return s.getsockname()[1]


def _worker(rank, world, port, fn, q):
  os.environ["MASTER_ADDR"] = "127.0.0.1"
  os.environ["MASTER_PORT"] = str(port)
  dist.init_process_group("gloo", rank=rank, world_size=world)
  try:
    fn(rank, world)
    q.put((rank, "ok"))
  except Exception as e:  # reported to the parent
    q.put((rank, repr(e)))
  finally:
    dist.destroy_process_group()


def _run(fn, world=2):
  ctx = mp.get_context("spawn")
  q = ctx.Queue()
  port = _free_port()
  procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
  for p in procs:
    p.start()
  for p in procs:
    p.join(120)
    assert p.exitcode == 0, f"rank exited with {p.exitcode}"
  results = dict(q.get() for _ in range(world))
  assert all(v == "ok" for v in results.values()), results


def _collectives(rank, world):
  g = torch.Generator().manual_seed(0)
  n, c = 8, 3
  z = torch.randn(n, n, c, generator=g)
  sh = Shard(n, world, rank)
  z_loc = sh.shard(z).contiguous()
  full = all_gather_rows(z_loc)
  assert torch.equal(full, z)
  z_col = pair_transpose_to_columns(z_loc, sh)
  assert torch.equal(z_col, z[:, sh.offset():sh.offset() + sh.size()])
  assert torch.equal(pair_transpose_to_rows(z_col, sh), z_loc)
  send = torch.arange(world * 2.0).reshape(world * 2, 1) + 100 * rank
  recv = all_to_all_rows(send)
  assert recv.flatten().tolist() == [2 * rank + 100 * p + e for p in range(world) for e in range(2)]


@pytest.mark.parametrize("world", [2, 4])
def test_collectives_and_pair_transpose(world):
  _run(_collectives, world)


def _incoming_choreography(rank, world):
  """Incoming tri-mult: P[c,i,j] = sum_k a[c,k,j] b[c,k,i] with k split over ranks (blocks.py:547-558)."""
  g = torch.Generator().manual_seed(1)
  n, c = 8, 4
  a = torch.randn(c, n, n, generator=g)          # a[c, k, j]
  b = torch.randn(c, n, n, generator=g)          # b[c, k, i]
  ref = torch.einsum("ckj,cki->cij", a, b)
  sh = Shard(n, world, rank)
  kl, off = sh.size(), sh.offset()
  # what the projection writes on this rank (local rows k): b^T and a^T as [n][C][k_loc]
  a_send = b[:, off:off + kl, :].permute(2, 0, 1).contiguous()   # A[i][c][k_loc] = b[c,k,i]
  b_send = a[:, off:off + kl, :].permute(2, 0, 1).contiguous()   # B[j][c][k_loc] = a[c,k,j]
  a_op = all_to_all_rows(a_send).view(world, kl, c, kl)           # [src][i_loc][C][k_chunk]
  b_op = all_gather_rows(b_send).view(world, n, c, kl)            # [src][j][C][k_chunk]
  # the contraction reads K chunk `src` of both operands: K index = src * kl + k
  a_full = a_op.permute(1, 2, 0, 3).reshape(kl, c, n)             # [i_loc][C][K]
  b_full = b_op.permute(1, 2, 0, 3).reshape(n, c, n)              # [j][C][K]
  p = torch.einsum("ick,jck->icj", a_full, b_full)                # [i_loc][C][j]
  assert torch.allclose(p, ref[:, off:off + kl, :].permute(1, 0, 2), atol=1e-5)


@pytest.mark.parametrize("world", [2, 4])
def test_incoming_triangle_multiplication_choreography(world):
  _run(_incoming_choreography, world)


def _channel_choreography(rank, world):
  """Channel-sharded triangle multiplication (the "channels" mode of sharding.tri_mult): a and b leave by
  channel block, each rank contracts its channels over all positions, the product returns by row block.
  The contraction is emulated with einsum; everything else is the module's own data movement."""
  from sparsefold_b200.sharding import channel_blocks_back, channel_blocks_out
  g = torch.Generator().manual_seed(2)
  n, c = 8, 4 * world
  a = torch.randn(n, c, n, generator=g)           # A[i][c][k] (outgoing operand layout, rows i)
  b = torch.randn(n, c, n, generator=g)           # B[j][c][k]
  ref = torch.einsum("ick,jck->icj", a, b)        # P[i][c][j]
  sh = Shard(n, world, rank)
  rows, off = sh.size(), sh.offset()
  a_c = channel_blocks_out(a[off:off + rows].contiguous(), world).reshape(n, c // world, n)   # all i, my channels
  b_c = channel_blocks_out(b[off:off + rows].contiguous(), world).reshape(n, c // world, n)
  cl = c // world
  assert torch.equal(a_c, a[:, rank * cl:(rank + 1) * cl])
  prod_c = torch.einsum("ick,jck->icj", a_c, b_c)                                          # [N][my channels][N]
  prod = channel_blocks_back(prod_c, world, rows, c)
  assert torch.allclose(prod, ref[off:off + rows], atol=1e-5)
  # incoming: operands hold K in per-rank chunks ([i][C][k_loc] on every rank)
  at = torch.randn(n, c, rows, generator=torch.Generator().manual_seed(10 + rank))
  got = channel_blocks_out(at, world)                                                      # [P][N][cl][k_loc]
  full = all_gather_rows(at.unsqueeze(0)).view(world, n, c, rows)                          # every rank's chunk
  assert torch.equal(got, full[:, :, rank * cl:(rank + 1) * cl, :])


@pytest.mark.parametrize("world", [2, 4])
def test_channel_sharded_triangle_multiplication_choreography(world):
  _run(_channel_choreography, world)


def _channel_pipeline_choreography(rank, world):
  """The pipelined "channels" mode (sharding.channel_pipeline): operands out and products back in
  channel sub-chunks with asynchronous all-to-alls, for 1, 2 and 4 sub-chunks, outgoing (K whole on
  every rank) and incoming (K in per-rank chunks); the contraction is emulated with einsum."""
  from sparsefold_b200.sharding import channel_pipeline
  g = torch.Generator().manual_seed(3)
  n, c = 8, 4 * world
  sh = Shard(n, world, rank)
  rows, off = sh.size(), sh.offset()
  a = torch.randn(n, c, n, generator=g)           # A[i][c][k]
  b = torch.randn(n, c, n, generator=g)           # B[j][c][k]
  ref = torch.einsum("ick,jck->icj", a, b)[off:off + rows]

  def contract_out(a_s, b_s, sub):                # [P][rows][sub][k] -> [N][sub][N]
    return torch.einsum("ick,jck->icj", a_s.reshape(n, sub, n), b_s.reshape(n, sub, n))

  # incoming layout: each rank holds every i with its own K chunk, [i][C][k_loc]
  at, bt = a[:, :, off:off + rows].contiguous(), b[:, :, off:off + rows].contiguous()

  def contract_in(a_s, b_s, sub):                 # [P (k chunk)][N][sub][k_loc] -> [N][sub][N]
    af = a_s.permute(1, 2, 0, 3).reshape(n, sub, n)
    bf = b_s.permute(1, 2, 0, 3).reshape(n, sub, n)
    return torch.einsum("ick,jck->icj", af, bf)

  for chunks in (1, 2, 4):
    got = channel_pipeline(a[off:off + rows].contiguous(), b[off:off + rows].contiguous(), world, rows, n,
                           contract_out, chunks=chunks)
    assert torch.allclose(got, ref, atol=1e-5), chunks
    got = channel_pipeline(at, bt, world, rows, n, contract_in, chunks=chunks)
    assert torch.allclose(got, ref, atol=1e-5), chunks


@pytest.mark.parametrize("world", [2, 4])
def test_channel_pipeline_choreography(world):
  _run(_channel_pipeline_choreography, world)
