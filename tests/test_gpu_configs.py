"""Parity at the benchmark configurations' own shapes.

* one PairFormerIteration at N=256 (all tokens real), seed 0, fp32,
  against the fp32 oracle at matmul precision "highest"; tolerance 1e-4 on the
  pair and single outputs (max|y - ref| / max|ref|).
* configs[1] per op: each pair op and the single update at N=512 with 475 real
  tokens, bf16, against the fp32 oracle on bf16-rounded inputs and weights;
  tolerance 2e-2.
* configs[1] trunk: the 48-block trunk that bench.py times (same weights, same
  inputs), bf16 on the GPU, against the fp32 oracle run block by block on the
  host with the parameter values the kernels use (weight matrices rounded to
  bf16; LayerNorm parameters and biases fp32, as the C ABI takes them) and
  bf16-rounded inputs.  The acceptance criterion is cosine similarity >= 0.999
  for the pair and the single representation, over all positions and over the
  real tokens only.

Reference composition: trunk/network.py:400-413 (layer_stack of
PairFormerIteration), trunk/blocks.py:862-910 (the block).
"""
import os

import pytest
import torch

from oracle import pairformer as orc
from sparsefold_b200 import _native, modules, synth
from tests.golden_io import cosine, max_rel_err

pytestmark = pytest.mark.gpu

N1, N1_REAL = 512, 475


@pytest.fixture(scope="module", autouse=True)
def _device():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  _native.check(_native.load().sf_device_check(), "sf_device_check")
  n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
  torch.set_num_threads(n)


def _round(p, dtype):
  """The parameter values the bf16 kernels compute with: weight matrices rounded to bf16 (prepare()
  packs them so), LayerNorm scales/offsets and Linear biases kept in fp32 (the C ABI takes them as
  fp32).  Rounding those too would compare against a model with different parameters."""
  keep = lambda k: k.split(".")[-1] == "bias" or "norm" in k
  return {k: (v.float() if keep(k) else v.to(dtype).float()) for k, v in p.items()}


def test_configs0_block_fp32():
  """N=256, all-ones mask, z, s ~ N(0,1) seed 0, random-init weights seed 0, fp32."""
  n = 256
  z, s, mask = synth.pair_inputs(n, seed=0)
  assert bool(mask.all())
  blk = modules.PairFormerIteration()
  p = synth.init_params(blk, seed=0)
  modules.prepare(blk)
  blk = blk.cuda()
  with torch.no_grad():
    zo, so = blk(z.cuda(), seq_mask=mask.cuda(), single_act=s.cuda())
  torch.cuda.synchronize()
  assert _native.device_status() == 0
  zr, sr = orc.pairformer_block(z, s, mask, p)
  ez, es = max_rel_err(zo.cpu(), zr), max_rel_err(so.cpu(), sr)
  print(f"configs[0] fp32 N=256: pair max rel err {ez:.3e}, single {es:.3e}")
  assert ez < 1e-4 and es < 1e-4


_OPS = {
    "tri_mult_out": (lambda: modules.TriangleMultiplication(128, "...ikc,...jkc->...ijc"),
                     lambda p, z, m, s: orc.triangle_multiplication(z, m, p, outgoing=True)),
    "tri_mult_in": (lambda: modules.TriangleMultiplication(128, "...kjc,...kic->...ijc"),
                    lambda p, z, m, s: orc.triangle_multiplication(z, m, p, outgoing=False)),
    "tri_att_start": (lambda: modules.GridSelfAttention(128, 4, transpose=False),
                      lambda p, z, m, s: orc.grid_self_attention(z, m, p, transpose=False)),
    "tri_att_end": (lambda: modules.GridSelfAttention(128, 4, transpose=True),
                    lambda p, z, m, s: orc.grid_self_attention(z, m, p, transpose=True)),
    "transition": (lambda: modules.TransitionBlock(128, 4), lambda p, z, m, s: orc.transition_block(z, p)),
    "single_update": (lambda: modules.SingleActUpdate(128, 384),
                      lambda p, z, m, s: orc.single_act_update(z, s, m, p, prefix="")),
}


@pytest.mark.parametrize("op", list(_OPS))
def test_configs1_op_bf16(op):
  """configs[1] shape, one op: N=512 with the last 37 tokens masked, bf16 I/O, fp32 accumulation."""
  make, oracle = _OPS[op]
  z, s, mask = synth.pair_inputs(N1, n_real=N1_REAL, seed=1)
  m = make()
  p = synth.init_params(m, seed=2)
  modules.prepare(m)
  m = m.cuda()
  dt = torch.bfloat16
  zd, sd, md = z.to(dt).cuda(), s.to(dt).cuda(), mask.cuda()
  with torch.no_grad():
    if op == "transition":
      got = m(zd)
    elif op == "single_update":
      got = m(zd, sd, md)
    else:
      got = m(zd, md)
  torch.cuda.synchronize()
  assert _native.device_status() == 0
  ref = oracle(_round(p, dt), z.to(dt).float(), mask, s.to(dt).float())
  err = max_rel_err(got.float().cpu(), ref)
  print(f"configs[1] {op} bf16 N=512 (475 real): max rel err {err:.3e}")
  assert err < 2e-2


def test_configs1_trunk48_cosine_bf16():
  """The bench workload end to end: 48 blocks, N=512 (475 real), bf16, cosine >= 0.999."""
  from bench import build_trunk
  blocks = 48
  z, s, mask = synth.pair_inputs(N1, 128, 384, n_real=N1_REAL, seed=0)
  dt = torch.bfloat16
  trunk = build_trunk(torch.device("cuda", 0), n_blocks=blocks, seed=0)
  with torch.no_grad():
    zo, so = trunk(z.to(dt).cuda(), s.to(dt).cuda(), mask.cuda())
  torch.cuda.synchronize()
  assert _native.device_status() == 0
  zo, so = zo.float().cpu(), so.float().cpu()
  del trunk
  torch.cuda.empty_cache()

  holder = modules.PairformerTrunk(blocks)
  p0 = synth.init_params(holder, seed=0)
  del holder
  p = _round(p0, dt)
  zr, sr = z.to(dt).float(), s.to(dt).float()
  with torch.no_grad():
    for i in range(blocks):
      zr, sr = orc.pairformer_block(zr, sr, mask, orc._sub(p, f"blocks.{i}."))
  real2 = mask[:, None] & mask[None, :]
  cos = {"pair": cosine(zo, zr), "pair_real": cosine(zo[real2], zr[real2]),
         "single": cosine(so, sr), "single_real": cosine(so[mask], sr[mask])}
  print("configs[1] 48-block trunk bf16 vs fp32 oracle, cosine: " +
        ", ".join(f"{k} {v:.6f}" for k, v in cos.items()) +
        f"; max rel err pair {max_rel_err(zo, zr):.3e}, single {max_rel_err(so, sr):.3e}")
  for k, v in cos.items():
    assert v >= 0.999, (k, v)
