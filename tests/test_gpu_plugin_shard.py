"""The reference's PairFormerIteration in its distributed mode, on 2 GPUs through the b200 plugin.

Each rank initialises the reference's runtime/dist.py with NCCL (NVLS off),
sets ``dist.current_shard`` over the token axis as model/network.py:143 does,
builds the reference block with ``distributed=True`` under the b200 backend and
runs it on its row shard: the B200 mixins route to the sharded phase entry points
(NCCL all-gathers and all-to-alls) and the single attention gathers every rank's
keys and values (diffusion/transformer.py:322-330).  The gathered output must
match the unsharded standalone block (bf16, 1e-2).
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tests.golden_io import max_rel_err
from tests.refsrc import reference_src

pytestmark = pytest.mark.gpu
N_TOK = 128


def _free_port():
  with socket.socket() as sk:
    sk.bind(("127.0.0.1", 0))
    return sk.getsockname()[1]


def _rank(rank, world, port, q):
  os.environ["NCCL_NVLS_ENABLE"] = "0"
  torch.cuda.set_device(rank)
  from tests.refsrc import import_reference
  import_reference()
  from sparsefold.runtime import config, dist as rdist
  from sparsefold import backends
  import sparsefold_b200.backend as b200
  from sparsefold_b200 import modules, sharding, synth
  try:
    rdist.init(rank=rank, world_size=world, master_addr="127.0.0.1", master_port=port, backend="nccl")
    b200.register()
    config.configure_runtime(backend="b200", device="cuda", sdpa_implementation="math", enable_sharding=False,
                             enable_compile=False, logs=set())
    backends.init()
    from sparsefold.model.trunk import blocks, network
    from sparsefold.model import config as mc
    rdist.current_shard = rdist.Shard(N_TOK)
    dev = torch.device("cuda", rank)
    blk = blocks.PairFormerIteration(network.Evoformer.Config().pairformer, mc.GlobalConfig(), with_single=True,
                                     num_channels=128, seq_channels=384, distributed=True)
    p = synth.init_params(blk, 5)
    backends.prepare(blk)
    blk = blk.to(dev)
    z, s, mask = synth.pair_inputs(N_TOK, n_real=119, seed=6)
    z, s, mask = z.to(dev, torch.bfloat16), s.to(dev, torch.bfloat16), mask.to(dev)
    sh = sharding.Shard(N_TOK, world, rank)
    with torch.no_grad():
      zl, sl = blk(sh.shard(z).contiguous(), seq_mask=mask, single_act=sh.shard(s).contiguous())
    zg, sg = sharding.all_gather_rows(zl), sharding.all_gather_rows(sl)
    if rank == 0:
      mine = modules.PairFormerIteration()
      mine.load_state_dict(p, strict=True)
      modules.prepare(mine)
      mine = mine.to(dev)
      with torch.no_grad():
        zr, sr = mine(z, seq_mask=mask, single_act=s)
      torch.cuda.synchronize()
      ez = max_rel_err(zg.float().cpu(), zr.float().cpu())
      es = max_rel_err(sg.float().cpu(), sr.float().cpu())
      q.put("ok" if ez < 1e-2 and es < 1e-2 else f"mismatch z {ez:.3e} s {es:.3e}")
    torch.distributed.barrier()
    sharding.close_peer_exchanges()
  except Exception as e:
    q.put(repr(e))
    raise
  finally:
    b200.unapply()
    if torch.distributed.is_initialized():
      torch.distributed.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.skipif(reference_src() is None, reason="reference package not present")
def test_reference_block_sharded_over_two_gpus_through_the_plugin():
  ctx = mp.get_context("spawn")
  q = ctx.Queue()
  port = _free_port()
  procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
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
