"""The diffusion and MSA modules at the per-block dimensions of configs[2] and configs[3] (reduced token,
atom and MSA counts so the CPU oracle finishes in seconds), bf16 on the GPU against the fp32 oracle on
the same parameter values (weight matrices rounded to bf16, LayerNorm parameters and biases fp32, as
the kernels take them) and bf16-rounded inputs; tolerance 2e-2.

* token transformer: c = 768, 16 heads x 48, single_cond 384, pair_cond 128 (transformer.py:348-477);
* atom CrossAttTransformer: c_atom = 128, 4 heads x 32, windows of 32 queries x 128 keys, pair_cond 16,
  3 blocks (transformer.py:588-693);
* MSA pair-weighted averaging (8 x 8) and outer-product mean (32 -> 128) with c_m = 64 and 15 % gaps
  (trunk/blocks.py:99-185, :569-689).
"""
import types

import pytest
import torch

from oracle import diffusion as dif
from sparsefold_b200 import _native, modules, synth
from tests.golden_io import max_rel_err

pytestmark = pytest.mark.gpu
DT = torch.bfloat16


@pytest.fixture(scope="module", autouse=True)
def _device():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  _native.check(_native.load().sf_device_check(), "sf_device_check")


def _kernel_values(p):
  keep = lambda k: k.split(".")[-1] in ("bias", "output_b") or "norm" in k
  return {k: (v.float() if keep(k) else v.to(DT).float()) for k, v in p.items()}


def _bf(t):
  return t.to(DT).float()


def _prep(m, seed):
  p = synth.init_params(m, seed)
  modules.prepare(m)
  return m.cuda(), _kernel_values(p)


def test_token_transformer_configs2_dims():
  g = torch.Generator().manual_seed(1)
  s_, n, c, sc, pc, h = 2, 128, 768, 384, 128, 16
  m, p = _prep(modules.DiffusionTransformer(c, sc, pc, num_head=h, num_blocks=4, super_block_size=2), 31)
  act, single, pair = torch.randn(s_, n, c, generator=g), torch.randn(n, sc, generator=g), torch.randn(n, n, pc, generator=g)
  mask = torch.arange(n) < 121
  with torch.no_grad():
    got = m(act.to(DT).cuda(), mask.cuda(), single.to(DT).cuda(), pair.to(DT).cuda())
  torch.cuda.synchronize()
  assert _native.device_status() == 0
  ref = dif.transformer(_bf(act), mask, _bf(single), _bf(pair), p, 2, 2)
  assert max_rel_err(got.float().cpu(), ref) < 2e-2


def test_atom_transformer_configs2_dims():
  g = torch.Generator().manual_seed(2)
  s_, nsub, q_, k_, c, pc = 2, 24, 32, 128, 128, 16
  m, p = _prep(modules.CrossAttTransformer(c, pc, num_head=4, key_dim=128, num_blocks=3, num_intermediate_factor=2), 32)
  starts = torch.clamp(32 * torch.arange(nsub) + 16 - 64, 0, nsub * q_ - k_)
  idx = (starts[:, None] + torch.arange(k_)[None, :]).to(torch.int32)
  gmask = torch.rand(nsub, k_, generator=g) > 0.05
  kmask = gmask & (torch.rand(nsub, k_, generator=g) > 0.1)
  qmask = torch.rand(nsub, q_, generator=g) > 0.1
  qact = torch.randn(s_, nsub, q_, c, generator=g)
  qsc, ksc = torch.randn(nsub, q_, c, generator=g), torch.randn(nsub, k_, c, generator=g)
  pcq = torch.randn(nsub, q_, k_, pc, generator=g)
  info = types.SimpleNamespace(gather_idxs=idx.cuda(), gather_mask=gmask.cuda())
  with torch.no_grad():
    got = m(qact.to(DT).cuda(), qmask.cuda(), info, kmask.cuda(), qsc.to(DT).cuda(), ksc.to(DT).cuda(),
            pcq.to(DT).cuda())
  torch.cuda.synchronize()
  assert _native.device_status() == 0
  ref = dif.cross_att_transformer(_bf(qact), qmask, idx, gmask, kmask, _bf(qsc), _bf(ksc), _bf(pcq), p, 3)
  assert max_rel_err(got.float().cpu(), ref) < 2e-2


def _msa_inputs(m_, n, seed):
  g = torch.Generator().manual_seed(seed)
  onehot = torch.nn.functional.one_hot(torch.randint(0, 32, (m_, n), generator=g), 32).float()
  act = torch.cat([onehot, torch.randn(m_, n, 32, generator=g)], -1)   # c_m = 64
  mask = torch.rand(m_, n, generator=g) > 0.15
  return act, mask


def test_msa_pair_weighted_averaging_configs3_dims():
  act, mask = _msa_inputs(64, 96, 3)
  pair = torch.randn(96, 96, 128, generator=torch.Generator().manual_seed(4))
  m, p = _prep(modules.MSAAttention(64, 128, 8), 33)
  with torch.no_grad():
    got = m(act.to(DT).cuda(), mask.cuda(), pair.to(DT).cuda())
  torch.cuda.synchronize()
  assert _native.device_status() == 0
  ref = dif.msa_attention(_bf(act), mask, _bf(pair), p)
  assert max_rel_err(got.float().cpu(), ref) < 2e-2


def test_outer_product_mean_configs3_dims():
  act, mask = _msa_inputs(128, 96, 5)
  m, p = _prep(modules.OuterProductMean(64, 128, 32), 34)
  with torch.no_grad():
    got = m(act.to(DT).cuda(), mask.cuda())
  torch.cuda.synchronize()
  assert _native.device_status() == 0
  ref = dif.outer_product_mean(_bf(act), mask, p)
  assert max_rel_err(got.float().cpu(), ref) < 2e-2
