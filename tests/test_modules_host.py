"""Host-side contract of the B200 modules (no GPU): parameters, buffers, packing layouts.

Mirrors the reference's native-preparation contract
(tests/test_native_preparation.py:107-132): forward refuses to run before
prepare, Parameters and state_dict keys are unchanged, only non-persistent
buffers are added, and re-preparation is idempotent.  The packing tests
recompute an op's first stage on the CPU from the *packed* weights and compare
it with the oracle, which pins the row orders the kernels rely on.
"""
import types

import pytest
import torch

from oracle import pairformer as orc
from sparsefold_b200 import modules, synth


def _block():
  b = modules.PairFormerIteration()
  synth.init_params(b, seed=0)
  return b


def test_forward_refuses_before_prepare():
  b = _block()
  z, s, mask = synth.pair_inputs(8)
  with pytest.raises(RuntimeError, match="not prepared"):
    b.triangle_multiplication_outgoing(z, mask)


def test_prepare_keeps_parameters_and_state_dict():
  b = _block()
  keys = set(b.state_dict())
  params = {k: v.detach().clone() for k, v in b.named_parameters()}
  counts = modules.prepare(b)
  assert counts["opaque"] == 8
  assert set(b.state_dict()) == keys
  for k, v in b.named_parameters():
    torch.testing.assert_close(v, params[k], rtol=0, atol=0)
  for m in b.modules():
    assert set(m._buffers) <= m._non_persistent_buffers_set
  modules.prepare(b)
  assert set(b.state_dict()) == keys


def test_tri_mult_glu_packing_matches_reference_channel_split():
  b = _block()
  modules.prepare(b)
  t = b.triangle_multiplication_outgoing
  p = {k: v for k, v in t.state_dict().items()}
  z, _, mask = synth.pair_inputs(6, seed=3)
  x = orc.layer_norm(z, p["left_norm_input.weight"], p["left_norm_input.bias"])
  proj = torch.sigmoid(x @ p["gate_projection.weight"]) * (x @ p["projection.weight"])
  y = x @ t._packed("glu", torch.float32).T
  c = 128
  a_pk = torch.sigmoid(y[..., :c]) * y[..., c:2 * c]
  b_pk = torch.sigmoid(y[..., 2 * c:3 * c]) * y[..., 3 * c:]
  torch.testing.assert_close(a_pk, proj[..., 0::2], rtol=1e-5, atol=1e-5)
  torch.testing.assert_close(b_pk, proj[..., 1::2], rtol=1e-5, atol=1e-5)


def test_grid_attention_qkvg_packing():
  b = _block()
  modules.prepare(b)
  g = b.pair_attention1
  p = g.state_dict()
  z, _, _ = synth.pair_inputs(5, seed=4)
  x = orc.layer_norm(z, p["act_norm.weight"], None)
  y = x @ g._packed("qkvg", torch.float32).T
  q = torch.einsum("bnc,hdc->bnhd", x, p["q_projection.weight"]).reshape(5, 5, 128)
  v = torch.einsum("bnc,chd->bnhd", x, p["v_projection.weight"]).reshape(5, 5, 128)
  gate = torch.einsum("bnc,oc->bno", x, p["gating_query.weight"])
  torch.testing.assert_close(y[..., :128], q, rtol=1e-5, atol=1e-5)
  torch.testing.assert_close(y[..., 256:384], v, rtol=1e-5, atol=1e-5)
  torch.testing.assert_close(y[..., 384:], gate, rtol=1e-5, atol=1e-5)


def test_ops_reject_host_tensors():
  from sparsefold_b200 import ops
  x = torch.zeros(4, 8)
  with pytest.raises(ValueError, match="CUDA"):
    ops.layer_norm(x, None, None)


def test_prepare_after_move_keeps_every_buffer_on_the_parameter_device():
  """prepare() on an already-moved module must not leave any buffer behind on the host."""
  b = modules.PairFormerIteration().to("meta")
  modules.prepare(b)
  for name, buf in b.named_buffers():
    assert buf.device.type == "meta", name


def test_diffusion_pair_logit_pack_reused_for_an_unchanged_pair_cond():
  """The diffusion transformer computes its pair-logit pack once while the denoising loop passes the
  same, unchanged pair_cond (generator.py:338-346), and again after an in-place change, for another
  dtype or another tensor; inference tensors (no version counter) are never memoised, and the memo
  goes when its pair_cond is freed."""
  import gc

  t = modules.DiffusionTransformerB200.__new__(modules.DiffusionTransformerB200)
  t._pack_memo = None
  calls = []

  def fake_pack(pair_cond, dtype):
    calls.append((pair_cond, dtype))
    return torch.full((1,), float(len(calls)))

  t.pair_logits_pack = fake_pack
  pc = torch.zeros(4, 4, 8)
  p1 = t._pack_of(pc, torch.bfloat16)
  assert t._pack_of(pc, torch.bfloat16) is p1 and len(calls) == 1
  pc.add_(1.0)                                   # in place: the version counter moves
  p2 = t._pack_of(pc, torch.bfloat16)
  assert p2 is not p1 and len(calls) == 2
  assert t._pack_of(pc, torch.float32) is not p2 and len(calls) == 3
  other = pc.clone()
  t._pack_of(other, torch.float32)
  assert len(calls) == 4
  with torch.inference_mode():
    inf = torch.zeros(4, 4, 8)
  t._pack_of(inf, torch.bfloat16)
  t._pack_of(inf, torch.bfloat16)
  assert len(calls) == 6
  t._pack_of(other, torch.bfloat16)
  assert t._pack_memo is not None
  calls.clear()
  del other
  gc.collect()
  assert t._pack_memo is None


def test_diffusion_pair_logit_pack_not_memoised_under_graph_capture(monkeypatch):
  """A CUDA graph must record the pack's computation (a replay re-reads pair_cond without running
  Python), so while the current stream captures, every call computes the pack and none is kept."""
  t = modules.DiffusionTransformerB200.__new__(modules.DiffusionTransformerB200)
  t._pack_memo = None
  calls = []
  t.pair_logits_pack = lambda pc, dt: calls.append(dt) or torch.zeros(1)
  pc = types.SimpleNamespace(is_cuda=True)   # a CUDA pair_cond, as far as the memo looks
  monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: True)
  t._pack_of(pc, torch.bfloat16)
  t._pack_of(pc, torch.bfloat16)
  assert len(calls) == 2 and t._pack_memo is None
