"""CPU oracle for the embedding-side pair ops — TEST INFRASTRUCTURE ONLY.

Restates, in plain torch CPU arithmetic (paths relative to HenryRenYz/SparseFold
``src/sparsefold/``), the pair embedding of the trunk's ``Evoformer`` and the base
conditioning of the ``DiffusionHead``, for the parity tests.  Parameter dicts use the
reference parameter names relative to the owning module.  Pinned by
``tests/golden/embedding_n16.npz`` (written by ``tests/golden/make_golden.py`` from the
reference modules themselves).
"""
from __future__ import annotations

import torch

from oracle.diffusion import transition
from oracle.pairformer import layer_norm


def seq_pair_embedding(target_feat_shard, target_feat, p):
  """``Evoformer._get_seq_pair_embedding`` (model/trunk/network.py:195-212):
  left_single(t_shard)[:, None] + right_single(t)[None, :]."""
  left = target_feat_shard @ p["left_single.weight"]
  right = target_feat @ p["right_single.weight"]
  return left[:, None] + right[None, :]


def position_feat(rel_features, p):
  """``Evoformer._get_position_feat`` (network.py:188-193): a bias-free linear over the relative
  encoding (139 features)."""
  return rel_features @ p["position_activations.weight"]


def contact_matrix(n, pl_idx, pl_mask, ll_idx, ll_mask):
  """The bond contact map of ``Evoformer._get_bonds_act`` (network.py:214-251): gather index pairs of
  the polymer-ligand and ligand-ligand bonds, zeroed where a gather is masked, set to 1, and the
  padding position (0, 0) cleared."""
  idx = []
  for g, m in ((pl_idx, pl_mask), (ll_idx, ll_mask)):
    keep = m.prod(dim=1).to(g.dtype)[:, None]
    idx.append(g * keep)
  idx = torch.cat(idx)
  c = torch.zeros(n, n)
  c[idx[:, 0].long(), idx[:, 1].long()] = 1.0
  c[0, 0] = 0.0
  return c


def bonds_act(contact, p):
  """``Evoformer._get_bonds_act`` (network.py:253-256): Linear(1 -> C) of the contact map."""
  return contact[:, :, None] @ p["bond_embedding.weight"]


def prev_embedding(prev_pair, pair, p):
  """The recycling step of ``Evoformer.forward`` (network.py:369-372):
  prev_embedding(LayerNorm(prev pair), residual=pair)."""
  xn = layer_norm(prev_pair, p["prev_embedding_layer_norm.weight"], p["prev_embedding_layer_norm.bias"])
  return xn @ p["prev_embedding.weight"] + pair


def base_cond(rel_features, single, pair, target_feat, use_conditioning, p):
  """``DiffusionHead._get_base_cond`` (model/diffusion/generator.py:367-391)."""
  single_e = use_conditioning * single
  pair_e = use_conditioning * pair
  f2 = torch.cat((pair_e, rel_features), dim=-1)
  pc = layer_norm(f2, p["pair_cond_initial_norm.weight"], None) @ p["pair_cond_initial_projection.weight"]
  for i in range(2):
    pc = transition(pc, p, pre=f"pair_transitions.{i}.")
  f1 = torch.cat((single_e, target_feat), dim=-1)
  sc = layer_norm(f1, p["single_cond_initial_norm.weight"], None) @ p["single_cond_initial_projection.weight"]
  return sc, pc
