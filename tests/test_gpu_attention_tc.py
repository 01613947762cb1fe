"""The tcgen05 attention kernel (k_mha_tc) behind sf_attention for bf16 inputs, against the oracle.

bf16 calls with head dims that are multiples of 8 (up to 64) run on the tensor
cores; the reference semantics (backends/torch/attention/sdpa.py:22-121) are
checked on ragged query/key lengths, per-batch key masks including fully
masked batches, masked query rows, bf16 and fp32 biases broadcast over the
batch, the sigmoid gate, strided q/k/v/gate views of one fused projection
buffer (the single-attention layout), and logits wide enough that the running
max moves by more than 2^8 (O rescaled in TMEM).  Tolerance: 2e-2 max relative
error against the fp32 oracle on the same bf16 inputs.
"""
import pytest
import torch

from oracle import pairformer as orc
from sparsefold_b200 import _native, ops
from tests.golden_io import max_rel_err

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module", autouse=True)
def _device():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  _native.check(_native.load().sf_device_check(), "sf_device_check")


def _ref(q, k, v, scale, mask_q, mask_k, bias, gate):
  o = orc.dot_product_attention(q.float(), k.float(), v.float(), scale=scale, mask_q=mask_q, mask_k=mask_k,
                                bias=None if bias is None else bias.float())
  return o if gate is None else o * torch.sigmoid(gate.float())


@pytest.mark.parametrize("d", [8, 16, 24, 32, 48, 64])
@pytest.mark.parametrize("qlen,klen", [(1, 1), (37, 45), (128, 128), (200, 129), (130, 513)])
def test_shapes_masks_bias_gate(d, qlen, klen):
  g = torch.Generator().manual_seed(d * 1000 + qlen + klen)
  B, H = 2, 3
  dt = torch.bfloat16
  q = torch.randn(B, qlen, H, d, generator=g).to(dt)
  k = torch.randn(B, klen, H, d, generator=g).to(dt)
  v = torch.randn(B, klen, H, d, generator=g).to(dt)
  bias = torch.randn(B, H, qlen, klen, generator=g).to(dt)
  gate = torch.randn(B, qlen, H, d, generator=g).to(dt)
  mq = torch.rand(B, qlen, generator=g) > 0.1
  mk = torch.rand(B, klen, generator=g) > 0.3
  mk[1] = False                          # a batch whose keys are all masked: uniform average of v
  got = ops.attention(q.cuda(), k.cuda(), v.cuda(), mask_q=mq.cuda(), mask_k=mk.cuda(), bias=bias.cuda(),
                      gate=gate.cuda())
  ref = _ref(q, k, v, None, mq, mk, bias, gate)
  assert max_rel_err(got.float().cpu(), ref) < TOL
  assert _native.device_status() == 0


@pytest.mark.parametrize("bias_kind", ["none", "bf16_broadcast", "f32"])
def test_bias_forms(bias_kind):
  g = torch.Generator().manual_seed(7)
  B, H, Q, K, d = 3, 4, 96, 160, 32
  dt = torch.bfloat16
  q, k, v = (torch.randn(B, n, H, d, generator=g).to(dt) for n in (Q, K, K))
  bias = None
  if bias_kind == "bf16_broadcast":
    bias = torch.randn(H, Q, K, generator=g).to(dt)          # shared by every batch entry
  elif bias_kind == "f32":
    bias = torch.randn(B, H, Q, K, generator=g)
  mk = torch.rand(B, K, generator=g) > 0.2
  got = ops.attention(q.cuda(), k.cuda(), v.cuda(), scale=0.3, mask_k=mk.cuda(),
                      bias=None if bias is None else bias.cuda())
  ref = _ref(q, k, v, 0.3, None, mk, bias, None)
  assert max_rel_err(got.float().cpu(), ref) < TOL


def test_fused_projection_views_single_attention_layout():
  """q, k, v, gate as strided views of one [N, 4, H, D] buffer (SelfAttentionB200's layout), N=512, 16 x 24."""
  g = torch.Generator().manual_seed(11)
  n, H, d = 512, 16, 24
  y = torch.randn(n, 4, H, d, generator=g).to(torch.bfloat16)
  bias = torch.randn(H, n, n, generator=g).to(torch.bfloat16)
  mk = torch.arange(n) < 475
  yc = y.cuda()
  got = ops.attention(yc[:, 0], yc[:, 1], yc[:, 2], mask_k=mk.cuda(), bias=bias.cuda(), gate=yc[:, 3])
  ref = _ref(y[:, 0], y[:, 1], y[:, 2], None, None, mk, bias, y[:, 3])
  assert max_rel_err(got.float().cpu(), ref) < TOL


def test_wide_logits_move_the_running_max():
  """Logits spanning tens of units in rising order: later key blocks exceed the running max by more
  than 2^8 many times, so O is rescaled in TMEM between P V products."""
  g = torch.Generator().manual_seed(5)
  B, H, Q, K, d = 2, 2, 128, 640, 64
  dt = torch.bfloat16
  q = (torch.randn(B, Q, H, d, generator=g) * 2).to(dt)
  k = (torch.randn(B, K, H, d, generator=g) * 2).to(dt)
  v = torch.randn(B, K, H, d, generator=g).to(dt)
  ramp = torch.linspace(0, 60, K)[None, None, None, :]
  bias = (torch.randn(B, H, Q, K, generator=g) + ramp).to(dt)
  got = ops.attention(q.cuda(), k.cuda(), v.cuda(), bias=bias.cuda())
  ref = _ref(q, k, v, None, None, None, bias, None)
  assert max_rel_err(got.float().cpu(), ref) < TOL
  assert _native.device_status() == 0


def test_masked_query_rows_and_rows_without_valid_keys():
  g = torch.Generator().manual_seed(3)
  B, H, Q, K, d = 4, 2, 70, 90, 16
  dt = torch.bfloat16
  q, k, v = (torch.randn(B, n, H, d, generator=g).to(dt) for n in (Q, K, K))
  mq = torch.ones(B, Q, dtype=torch.bool)
  mq[0, ::3] = False
  mk = torch.ones(B, K, dtype=torch.bool)
  mk[2, :64] = False                     # the first key block of batch 2 masked, valid keys after it
  mk[3] = False
  bias = torch.randn(B, H, Q, K, generator=g).to(dt)
  got = ops.attention(q.cuda(), k.cuda(), v.cuda(), mask_q=mq.cuda(), mask_k=mk.cuda(), bias=bias.cuda())
  ref = _ref(q, k, v, None, mq, mk, bias, None)
  assert max_rel_err(got.float().cpu(), ref) < TOL


@pytest.mark.parametrize("nsub,q,k,d", [(10, 32, 128, 32), (4, 32, 128, 16), (7, 20, 100, 24), (2, 1, 16, 8)])
def test_windows_four_per_cta(nsub, q, k, d):
  """Entries of at most 32 queries (atom windows: 32 queries x 128 keys of their own) run four to a
  CTA; a batch that is not a multiple of four, ragged keys, per-window masks, a fully masked window."""
  g = torch.Generator().manual_seed(nsub * 100 + q + k + d)
  H, dt = 4, torch.bfloat16
  qq = torch.randn(2, nsub, q, H, d, generator=g).to(dt)      # 2 samples x nsub windows
  kk = torch.randn(2, nsub, k, H, d, generator=g).to(dt)
  vv = torch.randn(2, nsub, k, H, d, generator=g).to(dt)
  gate = torch.randn(2, nsub, q, H, d, generator=g).to(dt)
  bias = torch.randn(nsub, H, q, k, generator=g).to(dt)          # per window, shared by the samples
  mq = torch.rand(nsub, q, generator=g) > 0.1
  mk = torch.rand(nsub, k, generator=g) > 0.2
  mk[nsub // 2] = False
  got = ops.attention(qq.cuda(), kk.cuda(), vv.cuda(), mask_q=mq.cuda(), mask_k=mk.cuda(), bias=bias.cuda(),
                      gate=gate.cuda())
  ref = _ref(qq, kk, vv, None, mq.expand(2, nsub, q), mk.expand(2, nsub, k), bias, gate)
  assert max_rel_err(got.float().cpu(), ref) < TOL
  assert _native.device_status() == 0
