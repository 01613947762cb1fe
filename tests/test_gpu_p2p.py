"""The NVLink peer exchange (sparsefold_b200/p2p.py) on 2 GPUs against NCCL's collectives.

Two spawned ranks map each other's receive buffers with CUDA IPC; ``all_to_all`` and ``all_gather``
through peer stores must equal ``all_to_all_single`` / ``all_gather_into_tensor`` bit for bit, for
several sizes (buffer pool reuse included) and dtypes, with the device status clear.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
  with socket.socket() as sk:
    sk.bind(("127.0.0.1", 0))
    return sk.getsockname()[1]


def _rank(rank, world, port, q):
  import datetime
  import torch.distributed as dist
  from sparsefold_b200 import _native, p2p
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
  torch.cuda.set_device(rank)
  dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                          device_id=torch.device("cuda", rank))
  try:
    ex = p2p.PeerExchange()
    g = torch.Generator(device="cuda").manual_seed(rank)
    bad = []
    for rnd in range(2):                                   # the second round reuses pooled buffers
      for rows, dt in ((64, torch.bfloat16), (4096, torch.bfloat16), (96, torch.float32)):
        x = torch.randn(world * rows, 40, device="cuda", generator=g).to(dt)
        ref = torch.empty_like(x)
        dist.all_to_all_single(ref, x)
        if not torch.equal(ex.all_to_all(x), ref):
          bad.append(f"all_to_all {rows} {dt} round {rnd}")
        y = x[:rows]
        refg = torch.empty(world * rows, 40, device="cuda", dtype=dt)
        dist.all_gather_into_tensor(refg, y)
        if not torch.equal(ex.all_gather(y), refg):
          bad.append(f"all_gather {rows} {dt} round {rnd}")
    torch.cuda.synchronize()
    st = _native.device_status()
    dist.barrier()
    ex.close()
    if rank == 0:
      q.put("ok" if not bad and st == 0 else f"{bad} status {st}")
  except Exception as e:
    q.put(repr(e))
    raise
  finally:
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_exchange_matches_nccl_on_two_gpus():
  ctx = mp.get_context("spawn")
  q = ctx.Queue()
  port = _free_port()
  procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
  for p in procs:
    p.start()
  for p in procs:
    p.join(300)
  for p in procs:
    if p.is_alive():
      p.kill()
      p.join(10)
  assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
  assert q.get(timeout=10) == "ok"
