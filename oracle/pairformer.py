"""CPU oracle for the AF3 trunk hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this file, and only as the
checker or the timed CPU baseline.  The product path (``sparsefold_b200``)
never calls it.

It restates, in plain torch CPU arithmetic, what the reference Torch backend
computes (paths relative to HenryRenYz/SparseFold ``src/sparsefold/``).  Every
function takes a flat parameter dict with the reference's own parameter names
(``module.state_dict()`` keys relative to the module).  Parity is pinned by
``tests/golden/*.npz``, which ``tests/golden/make_golden.py`` produced by
running the reference modules themselves; ``tests/test_oracle_golden.py`` checks
this file against those fixtures.

Numerics: callers pass fp32 (or fp64) tensors; matmuls use whatever
``torch.get_float32_matmul_precision`` is set (tests set "highest").
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _w(p, name, dtype):
  return p[name].to(dtype)


def layer_norm(x, weight, bias, eps=1e-5):
  """``primitives.LayerNorm.forward`` (model/layers/primitives.py:471-497), dim=-1."""
  return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)


def sigmoid(x):
  return torch.sigmoid(x)


def swish(x):
  """``primitives.swish`` (primitives.py:688-699)."""
  return x * torch.sigmoid(x)


def dot_product_attention(q, k, v, scale=None, mask_q=None, mask_k=None, bias=None):
  """``backends/torch/attention/sdpa.py:22-121`` with the math backend.

  q [..., Q, H, D], k [..., K, H, D], v [..., K, H, Dv], mask_q [..., Q],
  mask_k [..., K], bias broadcastable to [..., H, Q, K].  Masked positions get
  an additive ``-finfo(dtype).max`` (sdpa.py:61-80), so a fully masked query
  row averages V uniformly over all keys.
  """
  dtype = q.dtype
  if scale is None:
    scale = 1.0 / math.sqrt(q.shape[-1])
  batch = q.shape[:-3]
  attn_bias = None
  if mask_q is not None or mask_k is not None or bias is not None:
    attn_bias = torch.zeros(batch + (1, q.shape[-3], k.shape[-3]), dtype=dtype)
    min_val = -float(torch.finfo(dtype).max)
    if mask_q is not None:
      attn_bias.masked_fill_(~mask_q[..., None, :, None].bool(), min_val)
    if mask_k is not None:
      attn_bias.masked_fill_(~mask_k[..., None, None, :].bool(), min_val)
    if bias is not None:
      attn_bias = attn_bias + bias.to(dtype)
  qh = q.transpose(-3, -2)  # [..., H, Q, D]
  kh = k.transpose(-3, -2)
  vh = v.transpose(-3, -2)
  logits = torch.einsum("...qd,...kd->...qk", qh, kh) * scale
  if attn_bias is not None:
    logits = logits + attn_bias
  probs = torch.softmax(logits, dim=-1)
  out = torch.einsum("...qk,...kd->...qd", probs, vh)
  return out.transpose(-3, -2)


def triangle_multiplication(z, mask, p, outgoing: bool):
  """``TriangleMultiplication.forward`` (model/trunk/blocks.py:484-566), single device.

  z [N, N, C]; mask [N] bool.  GLU projection: gate columns first, then value
  (blocks.py:513-520 stacks (gate, projection)); a = even channels, b = odd
  (blocks.py:538 "(c i2)").  Outgoing: P[c,i,j] = sum_k a[c,i,k] b[c,j,k];
  incoming: P[c,i,j] = sum_k a[c,k,j] b[c,k,i] (blocks.py:447-450, :558).
  """
  dt = z.dtype
  pm = (mask[:, None] & mask[None, :])  # blocks.py:503
  x = layer_norm(z, _w(p, "left_norm_input.weight", dt), _w(p, "left_norm_input.bias", dt))
  g = x @ _w(p, "gate_projection.weight", dt)          # [N, N, 2C]
  v = x @ _w(p, "projection.weight", dt)
  proj = torch.sigmoid(g) * v                          # primitives.py:624-631
  proj = proj.permute(2, 0, 1)                         # [2C, N, N]  blocks.py:522
  proj = proj.masked_fill(~pm[None], 0.0)              # blocks.py:523
  a = proj[0::2]
  b = proj[1::2]
  if outgoing:
    pc = torch.einsum("cik,cjk->cij", a, b)
  else:
    pc = torch.einsum("ckj,cki->cij", a, b)
  y = pc.permute(1, 2, 0)                              # center_norm dim=-3 (blocks.py:467-472)
  y = layer_norm(y, _w(p, "center_norm.weight", dt), _w(p, "center_norm.bias", dt))
  out = y @ _w(p, "output_projection.weight", dt)
  gate = torch.sigmoid(x @ _w(p, "gating_linear.weight", dt))  # blocks.py:564
  return z + out * gate


def grid_self_attention(z, mask, p, transpose: bool):
  """``GridSelfAttention.forward`` / ``_attention`` (blocks.py:270-366), single device.

  act_norm has no bias (blocks.py:260-264).  The pair bias comes from the
  *untransposed* normalised pair (blocks.py:317-329); for ``transpose`` the
  attention runs along columns (blocks.py:335-346, :363-364).
  """
  dt = z.dtype
  n = z.shape[0]
  pm = (mask[:, None] & mask[None, :])                              # blocks.py:314
  x = layer_norm(z, _w(p, "act_norm.weight", dt), None)
  bias = torch.einsum("qkc,ch->hqk", x, _w(p, "pair_bias_projection.weight", dt))  # [H, N, N]
  if transpose:
    x = x.transpose(0, 1)
  wq = _w(p, "q_projection.weight", dt)   # (H, D, C) transpose_weights
  wk = _w(p, "k_projection.weight", dt)
  wv = _w(p, "v_projection.weight", dt)   # (C, H, D)
  q = torch.einsum("bnc,hdc->bnhd", x, wq)
  k = torch.einsum("bnc,hdc->bnhd", x, wk)
  v = torch.einsum("bnc,chd->bnhd", x, wv)
  o = dot_product_attention(q, k, v, mask_k=pm, bias=bias[None])   # blocks.py:281-285
  o = o.reshape(n, n, -1)
  gate = torch.sigmoid(torch.einsum("bnc,oc->bno", x, _w(p, "gating_query.weight", dt)))
  out = (o * gate) @ _w(p, "output_projection.weight", dt)
  if transpose:
    out = out.transpose(0, 1)
  return z + out


def transition_block(x, p, prefix=""):
  """``TransitionBlock.forward`` (blocks.py:79-96): LN -> SwiGLU -> down proj + residual.

  transition1.weight [C, 2*I] is split "a (i2 n)" (blocks.py:88-90): the first
  I columns go through swish, the second I are the linear half.
  """
  dt = x.dtype
  h = layer_norm(x, _w(p, prefix + "input_layer_norm.weight", dt), _w(p, prefix + "input_layer_norm.bias", dt))
  w1 = _w(p, prefix + "transition1.weight", dt)
  inter = w1.shape[1] // 2
  y = h @ w1
  c = swish(y[..., :inter]) * y[..., inter:]
  return x + c @ _w(p, prefix + "transition2.weight", dt)


def self_attention(s, mask, p, pair_logits=None, prefix=""):
  """Diffusion ``SelfAttention.forward`` without single_cond (transformer.py:306-345).

  Plain LayerNorm (AdaptiveLayerNorm with single_cond=None, transformer.py:94-95),
  q has a bias, k/v do not; softmax over keys with mask_k and pair_logits bias;
  sigmoid gate from gating_query; zero_init.transition2 projection; residual.
  """
  dt = s.dtype
  x = layer_norm(s, _w(p, prefix + "layer_norm.layer_norm.weight", dt), _w(p, prefix + "layer_norm.layer_norm.bias", dt))
  wq = _w(p, prefix + "q_projection.weight", dt)   # (C, H, D)
  q = torch.einsum("nc,chd->nhd", x, wq) + _w(p, prefix + "q_projection.bias", dt)
  k = torch.einsum("nc,chd->nhd", x, _w(p, prefix + "k_projection.weight", dt))
  v = torch.einsum("nc,chd->nhd", x, _w(p, prefix + "v_projection.weight", dt))
  o = dot_product_attention(q, k, v, mask_k=mask, bias=pair_logits)
  o = o.reshape(s.shape[0], -1)
  gate = torch.sigmoid(x @ _w(p, prefix + "gating_query.weight", dt))
  return s + (o * gate) @ _w(p, prefix + "zero_init.transition2.weight", dt)


def single_act_update(z, s, mask, p, prefix="single_act_update."):
  """``SingleActUpdate.forward`` (blocks.py:739-763)."""
  dt = z.dtype
  x = layer_norm(z, _w(p, prefix + "single_pair_logits_norm.weight", dt), _w(p, prefix + "single_pair_logits_norm.bias", dt))
  logits = x @ _w(p, prefix + "single_pair_logits_projection.weight", dt)   # [N, N, H]
  logits = logits.permute(2, 0, 1)                                          # blocks.py:749
  s = self_attention(s, mask, p, pair_logits=logits, prefix=prefix + "single_attention.")
  return transition_block(s, p, prefix=prefix + "single_transition.")


def _sub(p, prefix):
  return {k[len(prefix):]: v for k, v in p.items() if k.startswith(prefix)}


def pairformer_block(z, s, mask, p):
  """``PairFormerIteration.forward`` (blocks.py:862-910), with_single=True."""
  z = triangle_multiplication(z, mask, _sub(p, "triangle_multiplication_outgoing."), outgoing=True)
  z = triangle_multiplication(z, mask, _sub(p, "triangle_multiplication_incoming."), outgoing=False)
  z = grid_self_attention(z, mask, _sub(p, "pair_attention1."), transpose=False)
  z = grid_self_attention(z, mask, _sub(p, "pair_attention2."), transpose=True)
  z = transition_block(z, _sub(p, "pair_transition."))
  s = single_act_update(z, s, mask, p)
  return z, s
