"""The token transformer as a denoising loop uses it: pair-logit pack computed once, each step one
CUDA-graph replay (model/diffusion/generator.py:393-501 calls it 200 times with fixed shapes).

Replayed steps must equal eager steps bit for bit (same kernels, same order), chained over three
steps, and the cached pack must give the same result as recomputing it from pair_cond.
"""
import pytest
import torch

from sparsefold_b200 import _native, modules, synth
from sparsefold_b200.graphs import GraphedCall

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  _native.check(_native.load().sf_device_check(), "sf_device_check")


def test_cached_pack_and_graph_replay_match_eager_steps():
  g = torch.Generator().manual_seed(1)
  s_, n, c, sc, pc = 3, 96, 128, 64, 16
  m = modules.DiffusionTransformer(c, sc, pc, num_head=4, num_blocks=4, super_block_size=2)
  synth.init_params(m, seed=2)
  m = m.cuda()
  modules.prepare(m)
  dt = torch.bfloat16
  act = torch.randn(s_, n, c, generator=g).to("cuda", dt)
  single = torch.randn(n, sc, generator=g).to("cuda", dt)
  pair = torch.randn(n, n, pc, generator=g).to("cuda", dt)
  mask = (torch.arange(n) < 90).cuda()
  with torch.no_grad():
    pack = m.pair_logits_pack(pair, dt)
    ref = m(act, mask, single, pair)
    cached = m(act, mask, single, pair_logits_pack=pack)
    assert torch.equal(ref, cached)
    step = GraphedCall(lambda a: m(a, mask, single, pair_logits_pack=pack), act)
    a_eager, a_graph = act, act
    for _ in range(3):
      a_eager = m(a_eager, mask, single, pair_logits_pack=pack)
      a_graph = step(a_graph).clone()
    torch.cuda.synchronize()
  assert torch.equal(a_eager, a_graph)
  assert _native.device_status() == 0
