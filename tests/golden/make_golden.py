"""Generate the golden fixtures by running the *reference* SparseFold modules.

Run in a container that has the reference source tree (it is read-only and is
never needed at test time):

    python tests/golden/make_golden.py /path/to/SparseFold/src

The reference is configured exactly as its own CPU tests do
(tests/test_runtime_reference.py:22-29): backend "torch", device "cpu", math
SDPA, no sharding/compile; fp32 matmuls at "highest" precision.  Weights come
from ``sparsefold_b200.synth`` (keyed by parameter name), inputs from seeded
generators.  Each fixture stores inputs, outputs and the parameter spec list
(name, shape, kind, fan_in) so the weights can be regenerated without the
reference.  ``weights/records.py`` imports ``zstandard``; it is unused without
checkpoints, so a stub module is injected when the package is absent.
"""
from __future__ import annotations

import json
import math
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from sparsefold_b200 import synth  # noqa: E402


def _setup_reference(src: str):
  sys.path.insert(0, src)
  try:
    import zstandard  # noqa: F401
  except ImportError:
    sys.modules["zstandard"] = types.ModuleType("zstandard")
  from sparsefold.runtime import config
  config.configure_runtime(backend="torch", device="cpu", sdpa_implementation="math",
                           enable_sharding=False, enable_compile=False, logs=set())
  from sparsefold import backends
  backends.init()
  torch.set_float32_matmul_precision("highest")
  # A Linear built with precision="highest" restores the reference's default fp32 matmul
  # precision ("medium", runtime/util.py:28) after its einsum (layers/primitives.py:359-364);
  # the fixtures keep every fp32 matmul at "highest".
  from sparsefold.runtime import util
  util.DEFAULT_FP32_MATMUL_PRECISION = "highest"


def _spec(module) -> list:
  out = []
  for mod_name, mod in module.named_modules():
    for pname, p in mod.named_parameters(recurse=False):
      full = f"{mod_name}.{pname}" if mod_name else pname
      if synth._is_layernorm(mod):
        kind, fan = ("ln_weight" if pname == "weight" else "ln_bias"), 1
      elif synth._is_linear(mod):
        kind, fan = ("weight" if pname == "weight" else "bias"), int(math.prod(mod.input_shape))
      elif pname == "output_w":
        kind, fan = "weight", int(p.shape[0] * p.shape[1])
      elif pname == "output_b":
        kind, fan = "bias", 1
      else:
        raise ValueError(full)
      out.append([full, list(p.shape), kind, fan])
  return out


def _save(name, module_spec, seed, **arrays):
  path = os.path.join(HERE, f"{name}.npz")
  meta = json.dumps({"seed": seed, "params": module_spec})
  np.savez_compressed(path, meta=np.array(meta), **{k: np.asarray(v) for k, v in arrays.items()})
  print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def main(src: str):
  _setup_reference(src)
  from sparsefold.model.trunk import blocks, network
  from sparsefold.model import config as mc
  from sparsefold.backends.torch.attention import dot_product_attention

  gc = mc.GlobalConfig()
  pcfg = network.Evoformer.Config().pairformer
  seed = 0

  # 1. dot_product_attention semantics (tests/test_runtime_reference.py:117-138 shapes, seed 808)
  arrays = {}
  for bi, batch in enumerate([(), (2,), (2, 3)]):
    for masked in (False, True):
      g = torch.Generator().manual_seed(808)
      q = torch.randn(*batch, 3, 2, 4, generator=g)
      k = torch.randn(*batch, 5, 2, 4, generator=g)
      v = torch.randn(*batch, 5, 2, 6, generator=g)
      bias = torch.randn(*batch, 2, 3, 5, generator=g)
      mq = torch.tensor([True, False, True]).expand(*batch, 3) if masked else None
      mk = torch.tensor([True, False, True, True, False]).expand(*batch, 5) if masked else None
      out = dot_product_attention(q, k, v, scale=0.4, mask_q=mq, mask_k=mk, bias=bias)
      tag = f"b{bi}_m{int(masked)}"
      arrays.update({f"{tag}_q": q, f"{tag}_k": k, f"{tag}_v": v, f"{tag}_bias": bias, f"{tag}_out": out})
      if masked:
        arrays.update({f"{tag}_mask_q": mq.contiguous(), f"{tag}_mask_k": mk.contiguous()})
  # A larger case shaped like tests/test_runtime_gpu.py:28-41 (seed 610, scale 0.3).
  g = torch.Generator().manual_seed(610)
  q = torch.randn(2, 7, 3, 16, generator=g)
  k = torch.randn(2, 9, 3, 16, generator=g)
  v = torch.randn(2, 9, 3, 12, generator=g)
  bias = torch.randn(2, 3, 7, 9, generator=g)
  mk = torch.tensor([[True, False, True, True, True, False, True, False, True]]).expand(2, 9)
  out = dot_product_attention(q, k, v, mask_k=mk, bias=bias, scale=0.3)
  arrays.update({"g610_q": q, "g610_k": k, "g610_v": v, "g610_bias": bias,
                 "g610_mask_k": mk.contiguous(), "g610_out": out})
  _save("attention", [], 808, **arrays)

  # 2. Per-op fixtures on a ragged pair (N=16, 13 real tokens) and a full one (N=8).
  for n, n_real in ((16, 13), (8, 8)):
    z, s, mask = synth.pair_inputs(n, n_real=n_real, seed=1)
    tag = f"n{n}"
    for name, make in (
        ("tri_mult_out", lambda: blocks.TriangleMultiplication(pcfg.triangle_multiplication_outgoing, gc, num_channels=128, name="t")),
        ("tri_mult_in", lambda: blocks.TriangleMultiplication(pcfg.triangle_multiplication_incoming, gc, num_channels=128, name="t")),
        ("tri_att_start", lambda: blocks.GridSelfAttention(pcfg.pair_attention, gc, transpose=False, num_channels=128, name="g")),
        ("tri_att_end", lambda: blocks.GridSelfAttention(pcfg.pair_attention, gc, transpose=True, num_channels=128, name="g")),
        ("transition", lambda: blocks.TransitionBlock(pcfg.pair_transition, gc, num_channels=128, name="p")),
    ):
      mod = make()
      synth.init_params(mod, seed)
      with torch.no_grad():
        out = mod(z, mask) if name != "transition" else mod(z)
      _save(f"{name}_{tag}", _spec(mod), seed, z=z, mask=mask, out=out)
    mod = blocks.SingleActUpdate(gc, 128, 384, pcfg.single_attention, pcfg.single_transition)
    synth.init_params(mod, seed)
    with torch.no_grad():
      out = mod(z, s, mask)
    _save(f"single_update_{tag}", _spec(mod), seed, z=z, s=s, mask=mask, out=out)

  # 3. Full Pairformer block, ragged N=24 (21 real).
  z, s, mask = synth.pair_inputs(24, n_real=21, seed=2)
  blk = blocks.PairFormerIteration(pcfg, gc, with_single=True, num_channels=128, seq_channels=384)
  synth.init_params(blk, seed)
  with torch.no_grad():
    zo, so = blk(z, seq_mask=mask, single_act=s)
  _save("pairformer_n24", _spec(blk), seed, z=z, s=s, mask=mask, z_out=zo, s_out=so)


def diffusion_and_msa():
  """Fixtures of the diffusion-transformer and MSA modules (small AF3-like shapes)."""
  from sparsefold.model.diffusion import transformer as T
  from sparsefold.model.trunk import blocks
  from sparsefold.model import config as mc
  from sparsefold.schema.atom_layout import GatherInfo
  gc = mc.GlobalConfig()
  seed = 0
  g = torch.Generator().manual_seed(11)
  rn = lambda *s: torch.randn(*s, generator=g)

  # token self-attention with AdaLN (2 samples, 24 tokens, 21 real, c=128, 4 heads, single cond 64)
  n, c, sc_c = 24, 128, 64
  x, sc, pl = rn(2, n, c), rn(n, sc_c), rn(4, n, n)
  mask = torch.arange(n) < 21
  mod = T.SelfAttention(T.SelfAttention.Config(num_head=4), gc, num_channels=c, single_cond_size=sc_c, name="x")
  synth.init_params(mod, seed)
  with torch.no_grad():
    out = mod(x, mask, pair_logits=pl, single_cond=sc)
  _save("diff_self_attention", _spec(mod), seed, x=x, single_cond=sc, pair_logits=pl, mask=mask, out=out)

  mod = T.TransitionBlock(gc, num_channels=c, num_intermediate_factor=2, single_cond_size=sc_c, name="x")
  synth.init_params(mod, seed)
  with torch.no_grad():
    out = mod(x, single_cond=sc)
  _save("diff_transition", _spec(mod), seed, x=x, single_cond=sc, out=out)

  # transformer: 4 blocks in super-blocks of 2, pair_cond 16 channels
  pc = rn(n, n, 16)
  mod = T.Transformer(T.Transformer.Config(attention=T.SelfAttention.Config(num_head=4), num_blocks=4,
                                           super_block_size=2), gc, num_channels=c, single_cond_size=sc_c,
                      pair_cond_size=16)
  synth.init_params(mod, seed)
  with torch.no_grad():
    out = mod(x, mask, sc, pc)
  _save("diff_transformer", _spec(mod), seed, x=x, single_cond=sc, pair_cond=pc, mask=mask, out=out)

  # atom cross attention: 4 subsets x 32 queries over 128 atoms, 128-key windows, c_atom=64, 4 heads x 16
  s_, q_, k_, ca = 4, 32, 128, 64
  xq = rn(2, s_, q_, ca)
  qsc, ksc = rn(s_, q_, ca), rn(s_, k_, ca)
  qmask = torch.rand(s_, q_, generator=g) > 0.1
  starts = torch.clamp(32 * torch.arange(s_) + 16 - 64, 0, s_ * q_ - k_)
  idx = (starts[:, None] + torch.arange(k_)[None, :]).to(torch.int32)
  gmask = torch.rand(s_, k_, generator=g) > 0.05
  kmask = gmask & (torch.rand(s_, k_, generator=g) > 0.1)
  pcq = rn(s_, q_, k_, 8)
  cfg = T.CrossAttention.Config(num_head=4, key_dim=64, value_dim=64)
  mod = T.CrossAttention(cfg, gc, num_channels=ca, name="x")
  synth.init_params(mod, seed)
  xk = rn(2, s_, k_, ca)
  plq = rn(s_, 4, q_, k_)
  with torch.no_grad():
    out = mod(xq, xk, qmask, kmask, pair_logits=plq, single_cond_q=qsc, single_cond_k=ksc)
  _save("diff_cross_attention", _spec(mod), seed, x_q=xq, x_k=xk, mask_q=qmask, mask_k=kmask, pair_logits=plq,
        single_cond_q=qsc, single_cond_k=ksc, out=out)

  mod = T.CrossAttTransformer(T.CrossAttTransformer.Config(num_intermediate_factor=2, num_blocks=2, attention=cfg), gc,
                              pair_cond_size=8, num_channels=ca, super_name="a")
  synth.init_params(mod, seed)
  info = GatherInfo(gather_idxs=idx, gather_mask=gmask, input_shape=torch.tensor([s_, q_], dtype=torch.int32))
  with torch.no_grad():
    out = mod(xq, qmask, info, kmask, qsc, ksc, pcq)
  _save("diff_cross_att_transformer", _spec(mod), seed, queries_act=xq, queries_mask=qmask, gather_idxs=idx,
        gather_mask=gmask, keys_mask=kmask, queries_single_cond=qsc, keys_single_cond=ksc, pair_cond=pcq, out=out)

  # MSA pair-weighted averaging and outer-product mean: 6 MSA rows x 16 tokens, c_m=64, c_z=128
  m_, nn_ = 6, 16
  act, pair = rn(m_, nn_, 64), rn(nn_, nn_, 128)
  msa_mask = torch.rand(m_, nn_, generator=g) > 0.15
  msa_mask[:, 3] = False                        # a key masked in every row
  mod = blocks.MSAAttention(blocks.MSAAttention.Config(), gc, num_channels=64, num_output_channel=128, name="x")
  synth.init_params(mod, seed)
  with torch.no_grad():
    out = mod(act, msa_mask, pair_act=pair)
  _save("msa_attention", _spec(mod), seed, act=act, mask=msa_mask, pair_act=pair, out=out)

  mod = blocks.OuterProductMean(blocks.OuterProductMean.Config(), gc, num_channels=64, num_output_channel=128, name="x")
  mod.output_w = torch.nn.Parameter(torch.empty(32, 32, 128), requires_grad=False)
  mod.output_b = torch.nn.Parameter(torch.empty(128), requires_grad=False)
  synth.init_params(mod, seed)
  with torch.no_grad():
    out = mod(act, msa_mask)
  _save("outer_product_mean", _spec(mod), seed, act=act, mask=msa_mask, out=out)


def _spec_sub(module, names) -> list:
  """The parameter spec of the named submodules only, with their full names."""
  out = []
  for name in names:
    for full, shape, kind, fan in _spec(getattr(module, name)):
      out.append([f"{name}.{full}", shape, kind, fan])
  return out


def embedding():
  """Fixture of the embedding-side pair ops: the Evoformer's pair embedding and recycling step and the
  DiffusionHead's base conditioning, N=16 tokens in two chains, the reference's own relative encoding."""
  import types as _types
  from sparsefold.model.trunk import network
  from sparsefold.model.diffusion import generator
  from sparsefold.model.embeddings import features as emb
  from sparsefold.model import config as mc
  gc = mc.GlobalConfig()
  seed = 0
  g = torch.Generator().manual_seed(13)
  rn = lambda *s: torch.randn(*s, generator=g)
  n, tf_size = 16, 447
  tok = _types.SimpleNamespace(
      token_index=torch.arange(n), residue_index=torch.cat([torch.arange(10), torch.arange(6)]),
      asym_id=torch.cat([torch.zeros(10), torch.ones(6)]).long(), entity_id=torch.cat([torch.zeros(10), torch.ones(6)]).long(),
      sym_id=torch.zeros(n).long())
  rel = emb.create_relative_encoding(tok, 32, 2).float()
  assert rel.shape == (n, n, 139)
  evo = network.Evoformer(network.Evoformer.Config(), gc, target_feat_size=tf_size)
  names = ("left_single", "right_single", "position_activations", "bond_embedding", "prev_embedding_layer_norm",
           "prev_embedding")
  for name in names:
    synth.init_params(getattr(evo, name), seed, prefix=f"{name}.")
  target_feat = rn(n, tf_size)
  pl_idx = torch.tensor([[2, 12], [5, 14], [0, 0]], dtype=torch.int32)
  pl_mask = torch.tensor([[1, 1], [1, 1], [0, 1]], dtype=torch.int32)
  ll_idx = torch.tensor([[12, 13], [14, 15]], dtype=torch.int32)
  ll_mask = torch.tensor([[1, 1], [1, 0]], dtype=torch.int32)
  batch = _types.SimpleNamespace(
      token_features=tok,
      polymer_ligand_bond_info=_types.SimpleNamespace(
          tokens_to_polymer_ligand_bonds=_types.SimpleNamespace(gather_idxs=pl_idx, gather_mask=pl_mask)),
      ligand_ligand_bond_info=_types.SimpleNamespace(
          tokens_to_ligand_ligand_bonds=_types.SimpleNamespace(gather_idxs=ll_idx, gather_mask=ll_mask)))
  prev_pair = rn(n, n, 128)
  with torch.no_grad():
    seq_pair = evo._get_seq_pair_embedding(tok, target_feat, target_feat)
    pos = evo._get_position_feat(rel, torch.float32)
    bonds = evo._get_bonds_act(batch, torch.float32)
    pair = seq_pair + pos + bonds
    prev_out = evo.prev_embedding(evo.prev_embedding_layer_norm(prev_pair), residual=pair)
  spec = _spec_sub(evo, names)

  head = generator.DiffusionHead(generator.DiffusionHead.Config(), gc, pair_channels=128, seq_channels=384,
                                 target_feat_size=tf_size)
  hnames = ("pair_cond_initial_norm", "pair_cond_initial_projection", "pair_transitions", "single_cond_initial_norm",
            "single_cond_initial_projection")
  for name in hnames:
    synth.init_params(getattr(head, name), seed, prefix=f"head.{name}.")
  single = rn(n, 384)
  with torch.no_grad():
    sc, pc = head._get_base_cond(rel, {"single": single, "pair": prev_out, "target_feat": target_feat}, True)
  spec_h = [[f"head.{f}", s, k, fan] for f, s, k, fan in _spec_sub(head, hnames)]
  meta_seed = seed
  _save("embedding_n16", spec + spec_h, meta_seed, target_feat=target_feat, rel_features=rel, pl_idx=pl_idx,
        pl_mask=pl_mask, ll_idx=ll_idx, ll_mask=ll_mask, prev_pair=prev_pair, seq_pair=seq_pair, position_feat=pos,
        bonds_act=bonds, prev_out=prev_out, single=single, single_cond=sc, pair_cond=pc)


if __name__ == "__main__":
  src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SPARSEFOLD_REF_SRC")
  if not src:
    raise SystemExit("usage: make_golden.py <path of the reference's src/ directory> (or set SPARSEFOLD_REF_SRC)")
  main(src)
  diffusion_and_msa()
  embedding()
