"""Failure detection of the sharded path on the host (gloo ranks on CPU, no GPU).

The failures are made on the host, never on a device: a rank that raises
before a step, a rank that never joins the process group, and a rank that
leaves before a collective.  The surviving ranks must get a bounded error
rather than wait forever:

* ``sharding.step_barrier`` (the liveness check the sharded trunk can run
  between steps) names the missing rank within its time limit;
* ``init_process_group`` with a short timeout fails when a rank never joins;
* a collective of the sharded path (``all_gather_rows``) on a group whose peer
  has gone ends with an error within the process group's timeout.
"""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sparsefold_b200 import sharding


def _free_port():
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    return s.getsockname()[1]


def _put(q, item):
  """Queue a result and flush it: the ranks below leave with os._exit, which skips the queue's feeder."""
  q.put(item)
  q.close()
  q.join_thread()


def _init(rank, world, port, timeout_s):
  os.environ["MASTER_ADDR"] = "127.0.0.1"
  os.environ["MASTER_PORT"] = str(port)
  dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _raises_before_step(rank, world, port, q):
  _init(rank, world, port, 20)
  store = dist.distributed_c10d._get_default_store()
  sharding.step_barrier(store, 0, rank, world, timeout_s=10)     # everyone is alive at step 0
  if rank == world - 1:
    _put(q, (rank, "raised"))
    raise SystemExit(3)                                         # this rank fails between steps
  t0 = time.monotonic()
  try:
    sharding.step_barrier(store, 1, rank, world, timeout_s=2)
    _put(q, (rank, "no error"))
  except sharding.RankFailure as e:
    _put(q, (rank, f"failure {time.monotonic() - t0:.1f} {e}"))
  os._exit(0)   # leave without destroying the group: the failed rank will never join a teardown


def test_step_barrier_names_a_rank_that_raised():
  ctx = mp.get_context("spawn")
  q = ctx.Queue()
  port = _free_port()
  world = 3
  procs = [ctx.Process(target=_raises_before_step, args=(r, world, port, q)) for r in range(world)]
  for p in procs:
    p.start()
  for p in procs:
    p.join(60)
  assert [p.exitcode for p in procs] == [0, 0, 3]
  res = dict(q.get(timeout=10) for _ in range(world))
  assert res[2] == "raised"
  for r in (0, 1):
    assert res[r].startswith("failure"), res[r]
    assert "[2]" in res[r]
    assert float(res[r].split()[1]) < 10.0


def _never_joined(rank, world, port, q):
  t0 = time.monotonic()
  try:
    _init(rank, world, port, 3)
    _put(q, (rank, "joined"))
  except Exception as e:   # DistStoreError / RuntimeError: the missing rank never connected
    _put(q, (rank, f"error {time.monotonic() - t0:.1f} {type(e).__name__}"))


def test_init_fails_in_bounded_time_when_a_rank_never_joins():
  ctx = mp.get_context("spawn")
  q = ctx.Queue()
  port = _free_port()
  world = 3   # rank 2 is never started
  procs = [ctx.Process(target=_never_joined, args=(r, world, port, q)) for r in range(2)]
  for p in procs:
    p.start()
  for p in procs:
    p.join(60)
    assert p.exitcode == 0
  res = dict(q.get(timeout=10) for _ in range(2))
  for r in (0, 1):
    assert res[r].startswith("error"), res[r]
    assert float(res[r].split()[1]) < 30.0


def _peer_leaves(rank, world, port, q):
  _init(rank, world, port, 5)
  x = torch.full((4, 3), float(rank))
  full = sharding.all_gather_rows(x)                 # step 0: both ranks take part
  assert full.shape == (8, 3)
  if rank == 1:
    _put(q, (rank, "left"))
    os._exit(0)                                      # leaves between steps, nothing in flight
  t0 = time.monotonic()
  try:
    sharding.all_gather_rows(x)
    _put(q, (rank, "no error"))
  except Exception as e:   # gloo: peer closed the connection, or the group's timeout
    _put(q, (rank, f"error {time.monotonic() - t0:.1f} {type(e).__name__}"))
  os._exit(0)


def test_collective_of_the_sharded_path_errors_when_a_peer_left():
  ctx = mp.get_context("spawn")
  q = ctx.Queue()
  port = _free_port()
  procs = [ctx.Process(target=_peer_leaves, args=(r, 2, port, q)) for r in range(2)]
  for p in procs:
    p.start()
  for p in procs:
    p.join(60)
  assert [p.exitcode for p in procs] == [0, 0]
  res = dict(q.get(timeout=10) for _ in range(2))
  assert res[1] == "left"
  assert res[0].startswith("error"), res[0]
  assert float(res[0].split()[1]) < 30.0
