"""The B200 mixins follow the reference's distributed mode (gloo ranks on CPU).

With the reference's runtime/dist.py initialised and ``dist.current_shard`` set
(as model/network.py:143 does), a reference ``PairFormerIteration`` built with
``distributed=True`` under the b200 backend must route its triangle
multiplications and triangle attentions to the sharded phase entry points with
the reference's own partition.  The kernels need a GPU, so on the CPU the two
sharded entry points are replaced by recorders; the 2-GPU test in
test_gpu_plugin_shard.py runs the real kernels through the same path.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tests.refsrc import reference_src


def _free_port():
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    return s.getsockname()[1]


def _rank(rank, world, port, q):
  from tests.refsrc import import_reference
  import_reference()
  from sparsefold.runtime import config, dist as rdist
  from sparsefold import backends
  import sparsefold_b200.backend as b200
  from sparsefold_b200 import modules, sharding, synth
  try:
    rdist.init(rank=rank, world_size=world, master_addr="127.0.0.1", master_port=port, backend="gloo")
    b200.register()
    config.configure_runtime(backend="b200", device="cpu", sdpa_implementation="math", enable_sharding=False,
                             enable_compile=False, logs=set())
    backends.init()
    from sparsefold.model.trunk import blocks, network
    from sparsefold.model import config as mc
    n = 16
    rdist.current_shard = rdist.Shard(n)
    blk = blocks.PairFormerIteration(network.Evoformer.Config().pairformer, mc.GlobalConfig(), with_single=True,
                                     num_channels=128, seq_channels=384, distributed=True)
    synth.init_params(blk, 0)
    backends.prepare(blk)
    seen = []

    def record(kind):
      def fn(mod, act, mask_u8, shard, group=None):
        seen.append((kind, type(mod).__name__, tuple(act.shape), shard.offset(), shard.size(), shard.num_shards,
                     int(mask_u8.sum())))
        return act
      return fn
    sharding.tri_mult = record("tri_mult")
    sharding.tri_attention = record("tri_attention")
    z, s, mask = synth.pair_inputs(n, n_real=13)
    rows = n // world
    z_loc = z[rank * rows:(rank + 1) * rows]
    for m in (blk.triangle_multiplication_outgoing, blk.triangle_multiplication_incoming, blk.pair_attention1,
              blk.pair_attention2):
      out = m(z_loc, mask)
      assert out.shape == z_loc.shape
    assert [k for k, *_ in seen] == ["tri_mult", "tri_mult", "tri_attention", "tri_attention"], seen
    for _, _, shape, off, size, ns, nreal in seen:
      assert shape == (rows, n, 128) and off == rank * rows and size == rows and ns == world and nreal == 13
    # a standalone (non-reference) module never routes: no shard without the reference's distributed mode
    assert modules._reference_shard(modules.TriangleMultiplication()) is None
    q.put((rank, "ok"))
  except Exception as e:   # reported to the parent
    q.put((rank, repr(e)))
  finally:
    b200.unapply()
    if torch.distributed.is_initialized():
      torch.distributed.destroy_process_group()


@pytest.mark.skipif(reference_src() is None, reason="reference package not present")
def test_reference_block_routes_to_sharded_entry_points_two_ranks():
  ctx = mp.get_context("spawn")
  q = ctx.Queue()
  port = _free_port()
  procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
  for p in procs:
    p.start()
  for p in procs:
    p.join(120)
    assert p.exitcode == 0
  res = dict(q.get(timeout=10) for _ in range(2))
  assert res == {0: "ok", 1: "ok"}, res
