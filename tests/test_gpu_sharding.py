"""Row-sharded Pairformer block on GPUs vs the single-device block (bf16).

The sharded path runs the same kernels on each rank's rows with the exchanges of the
reference (all-gathers of b / a / bias / k,v, all-to-alls for the incoming operand and the
ending-node transpose), through NVLink peer stores (sparsefold_b200.p2p) or NCCL; its
gathered output must match the single-device block.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from sparsefold_b200 import _native, modules, sharding, synth
from tests.golden_io import max_rel_err

pytestmark = pytest.mark.gpu
N_TOK = 128


@pytest.fixture(scope="module", autouse=True)
def _device():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")


def _block(device):
  blk = modules.PairFormerIteration()
  synth.init_params(blk, seed=5)
  blk = blk.to(device)
  modules.prepare(blk)
  return blk


def _inputs(device):
  z, s, mask = synth.pair_inputs(N_TOK, n_real=119, seed=6)
  return z.to(device, torch.bfloat16), s.to(device, torch.bfloat16), mask.to(device)


def test_single_rank_sharded_block_matches_block():
  blk = _block("cuda")
  z, s, mask = _inputs("cuda")
  zr, sr = blk(z, seq_mask=mask, single_act=s)
  zs, ss = sharding.pairformer_block(blk, z, s, mask, sharding.Shard(N_TOK, 1, 0))
  torch.cuda.synchronize()
  assert max_rel_err(zs.float().cpu(), zr.float().cpu()) < 1e-2
  assert max_rel_err(ss.float().cpu(), sr.float().cpu()) < 1e-2
  assert _native.device_status() == 0


def _free_port():
  with socket.socket() as sk:
    sk.bind(("127.0.0.1", 0))
    return sk.getsockname()[1]


def _rank(rank, world, port, q, mode="rows", peer="1"):
  import datetime
  import torch.distributed as dist
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", SF_TRIMULT_SHARDING=mode,
                    SF_PEER_EXCHANGE=peer)
  torch.cuda.set_device(rank)
  dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                          device_id=torch.device("cuda", rank))
  try:
    dev = torch.device("cuda", rank)
    blk = _block(dev)
    z, s, mask = _inputs(dev)
    sh = sharding.Shard(N_TOK, world, rank)
    zl, sl = sharding.pairformer_block(blk, sh.shard(z).contiguous(), sh.shard(s).contiguous(), mask, sh)
    zg = sharding.all_gather_rows(zl)
    sg = sharding.all_gather_rows(sl)
    if rank == 0:
      zr, sr = blk(z, seq_mask=mask, single_act=s)
      torch.cuda.synchronize()
      ez = max_rel_err(zg.float().cpu(), zr.float().cpu())
      es = max_rel_err(sg.float().cpu(), sr.float().cpu())
      st = _native.device_status()
      q.put(("ok" if ez < 1e-2 and es < 1e-2 and st == 0 else f"mismatch z {ez:.3e} s {es:.3e} status {st}"))
    dist.barrier()
    sharding.close_peer_exchanges()
  except Exception as e:
    q.put(repr(e))
    raise
  finally:
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("peer", ["1", "0"], ids=["nvlink-peer-stores", "nccl"])
@pytest.mark.parametrize("mode", ["rows", "channels"])
def test_two_gpu_sharded_block_matches_block(mode, peer):
  """Both ways of moving the triangle-multiplication operands: all-gathers of whole operands ("rows", the
  reference's choreography) and channel blocks out / product rows back ("channels"); each over the
  NVLink peer exchange and over NCCL."""
  ctx = mp.get_context("spawn")
  q = ctx.Queue()
  port = _free_port()
  procs = [ctx.Process(target=_rank, args=(r, 2, port, q, mode, peer)) for r in range(2)]
  for p in procs:
    p.start()
  for p in procs:
    p.join(300)
  for p in procs:   # a rank still waiting after the limit is ended, not left behind
    if p.is_alive():
      p.kill()
      p.join(10)
  assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
  assert q.get(timeout=10) == "ok"
