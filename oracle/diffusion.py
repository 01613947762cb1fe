"""CPU oracle for the diffusion-transformer and MSA ops — TEST INFRASTRUCTURE ONLY.

Restates the reference Torch path (paths relative to HenryRenYz/SparseFold
``src/sparsefold/``) in plain torch CPU arithmetic, for the parity tests.
Parameter dicts use the reference parameter names relative to each module.
Pinned by ``tests/golden/*.npz`` (written by ``tests/golden/make_golden.py``
from the reference modules themselves).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle.pairformer import dot_product_attention, layer_norm, swish


def adaptive_layer_norm(x, p, pre, single_cond):
  """``AdaptiveLayerNorm.forward`` (model/diffusion/transformer.py:80-96)."""
  if single_cond is None:
    return layer_norm(x, p[pre + "layer_norm.weight"], p[pre + "layer_norm.bias"])
  xn = F.layer_norm(x, (x.shape[-1],))
  sc = layer_norm(single_cond, p[pre + "single_cond_layer_norm.weight"], None)
  scale = torch.sigmoid(sc @ p[pre + "single_cond_scale.weight"] + p[pre + "single_cond_scale.bias"])
  bias = sc @ p[pre + "single_cond_bias.weight"]
  return scale * xn + bias


def adaptive_zero_init(x, p, pre, single_cond):
  """``AdaptiveZeroInit.forward`` (transformer.py:138-154)."""
  out = x @ p[pre + "transition2.weight"]
  if single_cond is not None:
    out = out * torch.sigmoid(single_cond @ p[pre + "adaptive_zero_cond.weight"] + p[pre + "adaptive_zero_cond.bias"])
  return out


def self_attention(x, mask, p, pair_logits=None, single_cond=None, pre=""):
  """Diffusion ``SelfAttention.forward`` (transformer.py:306-345)."""
  xn = adaptive_layer_norm(x, p, pre + "layer_norm.", single_cond)
  q = torch.einsum("...c,chd->...hd", xn, p[pre + "q_projection.weight"]) + p[pre + "q_projection.bias"]
  k = torch.einsum("...c,chd->...hd", xn, p[pre + "k_projection.weight"])
  v = torch.einsum("...c,chd->...hd", xn, p[pre + "v_projection.weight"])
  o = dot_product_attention(q, k, v, mask_k=mask, bias=pair_logits)
  o = o.reshape(*o.shape[:-2], -1)
  gate = torch.sigmoid(xn @ p[pre + "gating_query.weight"])
  return x + adaptive_zero_init(o * gate, p, pre + "zero_init.", single_cond)


def transition(x, p, single_cond=None, pre=""):
  """Diffusion ``TransitionBlock.forward`` (transformer.py:208-231)."""
  xn = adaptive_layer_norm(x, p, pre + "layer_norm.", single_cond)
  w = p[pre + "transition.weight"]
  inter = w.shape[1] // 2
  y = xn @ w
  c = swish(y[..., :inter]) * y[..., inter:]
  return x + adaptive_zero_init(c, p, pre + "zero_init.", single_cond)


def cross_attention(x_q, x_k, mask_q, mask_k, p, pair_logits=None, single_cond_q=None, single_cond_k=None, pre=""):
  """``CrossAttention.forward`` (transformer.py:549-585)."""
  xq = adaptive_layer_norm(x_q, p, pre + "q_layernorm.", single_cond_q)
  xk = adaptive_layer_norm(x_k, p, pre + "k_layernorm.", single_cond_k)
  q = torch.einsum("...c,chd->...hd", xq, p[pre + "q_projection.weight"]) + p[pre + "q_projection.bias"]
  k = torch.einsum("...c,chd->...hd", xk, p[pre + "k_projection.weight"])
  v = torch.einsum("...c,chd->...hd", xk, p[pre + "v_projection.weight"])
  o = dot_product_attention(q, k, v, mask_q=mask_q, mask_k=mask_k, bias=pair_logits)
  o = o.reshape(*o.shape[:-2], -1)
  gate = torch.sigmoid(xq @ p[pre + "gating_query.weight"])
  return x_q + adaptive_zero_init(o * gate, p, pre + "zero_init.", single_cond_q)


def transformer(act, mask, single_cond, pair_cond, p, n_super, super_block):
  """Diffusion ``Transformer.forward`` (transformer.py:422-477) with the pair-logit pack (:429-447)."""
  pair = layer_norm(pair_cond, p["pair_input_layer_norm.weight"], None)
  for sb in range(n_super):
    logits = torch.einsum("bnc,csh->shbn", pair, p[f"pair_logits_projection.{sb}.weight"])
    for s in range(super_block):
      act = self_attention(act, mask, p, pair_logits=logits[s], single_cond=single_cond,
                           pre=f"self_attention.{sb}.{s}.")
      act = transition(act, p, single_cond, pre=f"transition_block.{sb}.{s}.")
  return act


def gather(arr, idx, gmask):
  """``atom_layout.convert`` with layout_axes=(-3, -2) (schema/atom_layout.py:52-83)."""
  flat = arr.reshape(*arr.shape[:-3], -1, arr.shape[-1])
  out = flat[..., idx.long(), :]
  return out.masked_fill(~gmask[..., None], 0.0)


def cross_att_transformer(queries_act, queries_mask, gather_idxs, gather_mask, keys_mask, q_sc, k_sc, pair_cond, p,
                          num_blocks):
  """``CrossAttTransformer.forward`` (transformer.py:644-693)."""
  pair = layer_norm(pair_cond, p["pair_input_layer_norm.weight"], None)
  logits = torch.einsum("sqkc,cbh->bshqk", pair, p["pair_logits_projection.weight"])
  for blk in range(num_blocks):
    keys = gather(queries_act, gather_idxs, gather_mask)
    queries_act = cross_attention(queries_act, keys, queries_mask, keys_mask, p, pair_logits=logits[blk],
                                  single_cond_q=q_sc, single_cond_k=k_sc, pre=f"cross_attention.{blk}.")
    queries_act = transition(queries_act, p, q_sc, pre=f"transition_block.{blk}.")
  return queries_act


def msa_attention(act, mask, pair_act, p):
  """``MSAAttention.forward`` pair-weighted averaging (model/trunk/blocks.py:155-185)."""
  a = layer_norm(act, p["act_norm.weight"], p["act_norm.bias"])
  z = layer_norm(pair_act, p["pair_norm.weight"], p["pair_norm.bias"])
  logits = torch.einsum("bnc,ch->hbn", z, p["pair_logits.weight"])
  logits = logits + 1e9 * (mask.to(torch.bfloat16).amax(0).float() - 1.0).to(torch.bfloat16).float()
  w = torch.softmax(logits, dim=-1)
  v = torch.einsum("mkc,chd->mkhd", a, p["v_projection.weight"])
  avg = torch.einsum("hqk,mkhd->mqhd", w, v).reshape(act.shape[0], pair_act.shape[0], -1)
  gate = torch.sigmoid(a @ p["gating_query.weight"])
  return (avg * gate) @ p["output_projection.weight"]


def outer_product_mean(act, mask, p):
  """``OuterProductMean.forward`` (model/trunk/blocks.py:630-689)."""
  x = layer_norm(act, p["layer_norm_input.weight"], p["layer_norm_input.bias"])
  m = mask[..., None].to(x.dtype)
  left = (x @ p["left_projection.weight"]) * m
  right = (x @ p["right_projection.weight"]) * m
  o = torch.einsum("mia,mjb->ijab", left, right)
  out = torch.einsum("ijab,abc->ijc", o, p["output_w"]) + p["output_b"]
  # the normaliser is formed in bf16 arithmetic whatever the activation dtype (blocks.py:683-689)
  norm = torch.einsum("mi,mj->ij", mask.float(), mask.float()).to(torch.bfloat16)
  inv = (1 / (1e-3 + norm)).float()
  return out * inv[..., None]
