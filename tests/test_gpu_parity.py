"""CUDA path vs the CPU oracle and the reference-generated golden fixtures.

Tolerances (max|y - ref| / max|ref| over the whole tensor): 1e-4 in fp32 mode,
2e-2 in bf16 mode where the reference is the fp32 oracle on bf16-rounded
inputs and weights.
"""
import pytest
import torch

from oracle import pairformer as orc
from sparsefold_b200 import _native, modules, ops, synth
from tests.golden_io import load, max_rel_err

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}
DTYPES = [torch.float32, torch.bfloat16]


@pytest.fixture(scope="module", autouse=True)
def _device():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  _native.check(_native.load().sf_device_check(), "sf_device_check")


def _round(p, dtype):
  return {k: v.to(dtype).float() for k, v in p.items()}


def _make(op):
  return {
      "tri_mult_out": lambda: modules.TriangleMultiplication(128, "...ikc,...jkc->...ijc"),
      "tri_mult_in": lambda: modules.TriangleMultiplication(128, "...kjc,...kic->...ijc"),
      "tri_att_start": lambda: modules.GridSelfAttention(128, 4, transpose=False),
      "tri_att_end": lambda: modules.GridSelfAttention(128, 4, transpose=True),
      "transition": lambda: modules.TransitionBlock(128, 4),
      "single_update": lambda: modules.SingleActUpdate(128, 384),
      "pairformer": lambda: modules.PairFormerIteration(),
  }[op]()


def _native_module(op, params):
  m = _make(op)
  m.load_state_dict(params, strict=True)
  modules.prepare(m)
  return m.cuda()


def _oracle(op, p, z, mask, s=None):
  if op == "tri_mult_out":
    return orc.triangle_multiplication(z, mask, p, outgoing=True)
  if op == "tri_mult_in":
    return orc.triangle_multiplication(z, mask, p, outgoing=False)
  if op == "tri_att_start":
    return orc.grid_self_attention(z, mask, p, transpose=False)
  if op == "tri_att_end":
    return orc.grid_self_attention(z, mask, p, transpose=True)
  if op == "transition":
    return orc.transition_block(z, p)
  if op == "single_update":
    return orc.single_act_update(z, s, mask, p, prefix="")
  raise ValueError(op)


def _run(m, op, z, mask, s=None):
  if op == "transition":
    return m(z)
  if op == "single_update":
    return m(z, s, mask)
  return m(z, mask)


PAIR_OPS = ["tri_mult_out", "tri_mult_in", "tri_att_start", "tri_att_end", "transition"]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [8, 16])
@pytest.mark.parametrize("op", PAIR_OPS + ["single_update"])
def test_golden_fixture(op, n, dtype):
  arrays, p = load(f"{op}_n{n}")
  z, mask = arrays["z"], arrays["mask"]
  s = arrays.get("s")
  m = _native_module(op, p)
  args = [z.to(dtype).cuda(), mask.cuda()]
  got = _run(m, op, args[0], args[1], None if s is None else s.to(dtype).cuda())
  if dtype == torch.float32:
    ref = arrays["out"]
  else:
    ref = _oracle(op, _round(p, dtype), z.to(dtype).float(), mask,
                  None if s is None else s.to(dtype).float())
  assert max_rel_err(got.float().cpu(), ref) < TOL[dtype]


@pytest.mark.parametrize("dtype", DTYPES)
def test_pairformer_block_golden(dtype):
  arrays, p = load("pairformer_n24")
  m = _native_module("pairformer", p)
  z, s, mask = arrays["z"], arrays["s"], arrays["mask"]
  zo, so = m(z.to(dtype).cuda(), seq_mask=mask.cuda(), single_act=s.to(dtype).cuda())
  if dtype == torch.float32:
    zr, sr = arrays["z_out"], arrays["s_out"]
  else:
    zr, sr = orc.pairformer_block(z.to(dtype).float(), s.to(dtype).float(), mask, _round(p, dtype))
  assert max_rel_err(zo.float().cpu(), zr) < TOL[dtype]
  assert max_rel_err(so.float().cpu(), sr) < TOL[dtype]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n,n_real", [(1, 1), (3, 2), (17, 11), (33, 33), (64, 50), (130, 127)])
@pytest.mark.parametrize("op", PAIR_OPS)
def test_edge_sizes(op, n, n_real, dtype):
  z, _, mask = synth.pair_inputs(n, n_real=n_real, seed=n)
  m = _make(op)
  p = synth.init_params(m, seed=7)
  modules.prepare(m)
  m = m.cuda()
  got = _run(m, op, z.to(dtype).cuda(), mask.cuda())
  ref = _oracle(op, _round(p, dtype), z.to(dtype).float(), mask)
  assert max_rel_err(got.float().cpu(), ref) < TOL[dtype]


@pytest.mark.parametrize("op", PAIR_OPS + ["single_update"])
def test_many_tiles_bf16(op):
  """Several tiles per SM (persistent pipelines wrap their stages many times), ragged N."""
  n, n_real = 320, 301
  z, s, mask = synth.pair_inputs(n, n_real=n_real, seed=3)
  m = _make(op)
  p = synth.init_params(m, seed=9)
  modules.prepare(m)
  m = m.cuda()
  dt = torch.bfloat16
  s_in = s.to(dt) if op == "single_update" else None
  got = _run(m, op, z.to(dt).cuda(), mask.cuda(), None if s_in is None else s_in.cuda())
  ref = _oracle(op, _round(p, dt), z.to(dt).float(), mask, None if s_in is None else s_in.float())
  assert max_rel_err(got.float().cpu(), ref) < TOL[dt]
  assert _native.device_status() == 0


@pytest.mark.parametrize("dtype", DTYPES)
def test_all_masked_tokens(dtype):
  """Every pair row padded: attention rows average V uniformly, tri-mult operands are zero."""
  n = 12
  z, s, _ = synth.pair_inputs(n, seed=9)
  mask = torch.zeros(n, dtype=torch.bool)
  blk = modules.PairFormerIteration()
  p = synth.init_params(blk, seed=3)
  modules.prepare(blk)
  blk = blk.cuda()
  zo, so = blk(z.to(dtype).cuda(), seq_mask=mask.cuda(), single_act=s.to(dtype).cuda())
  zr, sr = orc.pairformer_block(z.to(dtype).float(), s.to(dtype).float(), mask, _round(p, dtype))
  assert max_rel_err(zo.float().cpu(), zr) < TOL[dtype]
  assert max_rel_err(so.float().cpu(), sr) < TOL[dtype]


def test_attention_golden_semantics():
  arrays, _ = load("attention")
  for bi in range(3):
    for masked in (0, 1):
      t = f"b{bi}_m{masked}"
      q, k, v = (arrays[f"{t}_{x}"] for x in "qkv")   # includes the reference's Dv != Dqk cases
      got = ops.attention(q.cuda(), k.cuda(), v.cuda(), scale=0.4,
                          mask_q=None if not masked else arrays[f"{t}_mask_q"].cuda(),
                          mask_k=None if not masked else arrays[f"{t}_mask_k"].cuda(),
                          bias=arrays[f"{t}_bias"].cuda())
      torch.testing.assert_close(got.cpu(), arrays[f"{t}_out"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("dq,dv", [(16, 12), (24, 32), (8, 40)])
def test_attention_value_dim_differs(dq, dv, dtype):
  """sdpa.py:22-121 takes v with its own head dim; out and gate follow v."""
  g = torch.Generator().manual_seed(dq * 100 + dv)
  q = torch.randn(2, 37, 3, dq, generator=g).to(dtype)
  k = torch.randn(2, 45, 3, dq, generator=g).to(dtype)
  v = torch.randn(2, 45, 3, dv, generator=g).to(dtype)
  bias = torch.randn(2, 3, 37, 45, generator=g).to(dtype)
  gate = torch.randn(2, 37, 3, dv, generator=g).to(dtype)
  mk = torch.rand(2, 45, generator=g) > 0.2
  ref = orc.dot_product_attention(q.float(), k.float(), v.float(), mask_k=mk, bias=bias.float())
  ref = ref * torch.sigmoid(gate.float())
  got = ops.attention(q.cuda(), k.cuda(), v.cuda(), mask_k=mk.cuda(), bias=bias.cuda(), gate=gate.cuda())
  assert got.shape == (2, 37, 3, dv)
  assert max_rel_err(got.float().cpu(), ref) < TOL[dtype]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch", [(), (2,), (2, 3)])
def test_attention_masks_bias_batch(batch, dtype):
  g = torch.Generator().manual_seed(808)
  q = torch.randn(*batch, 7, 3, 16, generator=g).to(dtype)
  k = torch.randn(*batch, 9, 3, 16, generator=g).to(dtype)
  v = torch.randn(*batch, 9, 3, 16, generator=g).to(dtype)
  bias = torch.randn(*batch, 3, 7, 9, generator=g).to(dtype)
  mq = torch.tensor([True, False, True, True, True, False, True]).expand(*batch, 7)
  mk = torch.tensor([True, False, True, True, True, False, True, False, True]).expand(*batch, 9)
  ref = orc.dot_product_attention(q.float(), k.float(), v.float(), scale=0.3, mask_q=mq, mask_k=mk,
                                  bias=bias.float())
  got = ops.attention(q.cuda(), k.cuda(), v.cuda(), scale=0.3, mask_q=mq.cuda(), mask_k=mk.cuda(),
                      bias=bias.cuda())
  assert max_rel_err(got.float().cpu(), ref) < TOL[dtype]


def test_larger_block_bf16():
  n = 128
  z, s, mask = synth.pair_inputs(n, n_real=119, seed=11)
  blk = modules.PairFormerIteration()
  p = synth.init_params(blk, seed=1)
  modules.prepare(blk)
  blk = blk.cuda()
  dt = torch.bfloat16
  zo, so = blk(z.to(dt).cuda(), seq_mask=mask.cuda(), single_act=s.to(dt).cuda())
  zr, sr = orc.pairformer_block(z.to(dt).float(), s.to(dt).float(), mask, _round(p, dt))
  assert max_rel_err(zo.float().cpu(), zr) < 2e-2
  assert max_rel_err(so.float().cpu(), sr) < 2e-2


@pytest.mark.parametrize("op", ["tri_att_start", "tri_att_end"])
def test_triangle_attention_wide_logits_bf16(op):
  """Query/key and pair-bias weights scaled up so each row's logits span tens of units: later
  key blocks exceed the running max by more than 2^8 and block sums pass 2^8, which sends the
  attention core through its exact path (block max from S and the bias, running max moved,
  O rescaled).  Same bf16 tolerance as every other parity test."""
  n, n_real = 200, 187
  z, _, mask = synth.pair_inputs(n, n_real=n_real, seed=21)
  m = _make(op)
  p = synth.init_params(m, seed=13)
  for name in ("q_projection.weight", "k_projection.weight", "pair_bias_projection.weight"):
    p[name] = p[name] * 2.0
  m = _native_module(op, p)
  dt = torch.bfloat16
  got = _run(m, op, z.to(dt).cuda(), mask.cuda())
  ref = _oracle(op, _round(p, dt), z.to(dt).float(), mask)
  assert max_rel_err(got.float().cpu(), ref) < TOL[dt]
  assert _native.device_status() == 0


def test_tri_attention_row_bias_bf16():
  """sf_tri_attention_bias (the pair bias of a block of pair rows, which the ending-node attention of a
  row shard needs) against the projection's own bias for the same rows and against
  log2(e) * bf16(LN(z)) . W_b in fp32, on a ragged block."""
  from sparsefold_b200 import sharding
  rows, n = 37, 130
  z = (torch.randn(rows, n, 128, generator=torch.Generator().manual_seed(11)) * 1.5 + 0.3).to(torch.bfloat16)
  m = _make("tri_att_start")
  p = synth.init_params(m, seed=5)
  modules.prepare(m)
  m = m.cuda()
  w = m.native_weights(torch.bfloat16)
  lib = _native.load()
  qp = int(lib.sf_tri_attention_query_pitch(n))
  zc = z.cuda()
  got = torch.zeros(rows, 4, qp, dtype=torch.bfloat16, device="cuda")
  _native.call("sf_tri_attention_bias", _native.SF_BF16, sharding._p(zc), rows, n, sharding.C.byref(w), sharding._p(got),
               qp, sharding._stream())
  _, q, k, vt, g = sharding._att_buffers(rows, n, torch.bfloat16, zc.device)
  ref_proj = torch.zeros_like(got)
  _native.call("sf_tri_attention_project", _native.SF_BF16, sharding._p(zc), rows, n, 0, 1, sharding.C.byref(w),
               sharding._p(q), sharding._p(k), sharding._p(vt), sharding._p(g), sharding._p(ref_proj), sharding._stream())
  torch.cuda.synchronize()
  assert _native.device_status() == 0
  got_v = got[:, :, :n].float().cpu()
  assert max_rel_err(got_v, ref_proj[:, :, :n].float().cpu()) < 1e-2
  ln = (torch.nn.functional.layer_norm(z.float(), (128,), eps=1e-5) * p["act_norm.weight"]).to(torch.bfloat16).float()
  ref = torch.einsum("rsc,ch->rhs", ln, p["pair_bias_projection.weight"].to(torch.bfloat16).float()) * 1.4426950408889634
  assert max_rel_err(got_v, ref) < TOL[torch.bfloat16]
