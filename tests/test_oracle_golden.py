"""Pin the CPU oracle against fixtures produced by the reference modules themselves."""
import pytest
import torch

from oracle import pairformer as orc
from tests.golden_io import load, max_rel_err


def test_attention_semantics_golden():
  arrays, _ = load("attention")
  for bi in range(3):
    for masked in (0, 1):
      t = f"b{bi}_m{masked}"
      out = orc.dot_product_attention(
          arrays[f"{t}_q"], arrays[f"{t}_k"], arrays[f"{t}_v"], scale=0.4,
          mask_q=arrays.get(f"{t}_mask_q"), mask_k=arrays.get(f"{t}_mask_k"),
          bias=arrays[f"{t}_bias"])
      torch.testing.assert_close(out, arrays[f"{t}_out"], rtol=1e-6, atol=1e-6)
  out = orc.dot_product_attention(arrays["g610_q"], arrays["g610_k"], arrays["g610_v"],
                                  scale=0.3, mask_k=arrays["g610_mask_k"], bias=arrays["g610_bias"])
  torch.testing.assert_close(out, arrays["g610_out"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("n", [8, 16])
@pytest.mark.parametrize("op", ["tri_mult_out", "tri_mult_in", "tri_att_start", "tri_att_end", "transition"])
def test_pair_ops_golden(op, n):
  arrays, p = load(f"{op}_n{n}")
  z, mask = arrays["z"], arrays["mask"]
  if op == "tri_mult_out":
    out = orc.triangle_multiplication(z, mask, p, outgoing=True)
  elif op == "tri_mult_in":
    out = orc.triangle_multiplication(z, mask, p, outgoing=False)
  elif op == "tri_att_start":
    out = orc.grid_self_attention(z, mask, p, transpose=False)
  elif op == "tri_att_end":
    out = orc.grid_self_attention(z, mask, p, transpose=True)
  else:
    out = orc.transition_block(z, p)
  assert max_rel_err(out, arrays["out"]) < 2e-6


@pytest.mark.parametrize("n", [8, 16])
def test_single_update_golden(n):
  arrays, p = load(f"single_update_n{n}")
  out = orc.single_act_update(arrays["z"], arrays["s"], arrays["mask"], p, prefix="")
  assert max_rel_err(out, arrays["out"]) < 2e-6


def test_pairformer_block_golden():
  arrays, p = load("pairformer_n24")
  zo, so = orc.pairformer_block(arrays["z"], arrays["s"], arrays["mask"], p)
  assert max_rel_err(zo, arrays["z_out"]) < 5e-6
  assert max_rel_err(so, arrays["s_out"]) < 5e-6


def test_fully_masked_row_averages_values():
  """A fully masked query row returns the uniform mean of V (sdpa.py:61-80 -finfo.max bias)."""
  g = torch.Generator().manual_seed(3)
  q = torch.randn(4, 1, 8, generator=g)
  k = torch.randn(6, 1, 8, generator=g)
  v = torch.randn(6, 1, 8, generator=g)
  mk = torch.zeros(6, dtype=torch.bool)
  out = orc.dot_product_attention(q, k, v, mask_k=mk)
  torch.testing.assert_close(out, v.mean(0, keepdim=True).expand(4, 1, 8), rtol=1e-6, atol=1e-6)


# ---- diffusion transformer and MSA ------------------------------------------
from oracle import diffusion as dif  # noqa: E402


def test_diffusion_self_attention_golden():
  a, p = load("diff_self_attention")
  out = dif.self_attention(a["x"], a["mask"], p, pair_logits=a["pair_logits"], single_cond=a["single_cond"])
  assert max_rel_err(out, a["out"]) < 2e-6


def test_diffusion_transition_golden():
  a, p = load("diff_transition")
  assert max_rel_err(dif.transition(a["x"], p, a["single_cond"]), a["out"]) < 2e-6


def test_diffusion_transformer_golden():
  a, p = load("diff_transformer")
  out = dif.transformer(a["x"], a["mask"], a["single_cond"], a["pair_cond"], p, n_super=2, super_block=2)
  assert max_rel_err(out, a["out"]) < 5e-6


def test_cross_attention_golden():
  a, p = load("diff_cross_attention")
  out = dif.cross_attention(a["x_q"], a["x_k"], a["mask_q"], a["mask_k"], p, pair_logits=a["pair_logits"],
                            single_cond_q=a["single_cond_q"], single_cond_k=a["single_cond_k"])
  assert max_rel_err(out, a["out"]) < 2e-6


def test_cross_att_transformer_golden():
  a, p = load("diff_cross_att_transformer")
  out = dif.cross_att_transformer(a["queries_act"], a["queries_mask"], a["gather_idxs"], a["gather_mask"],
                                  a["keys_mask"], a["queries_single_cond"], a["keys_single_cond"], a["pair_cond"], p,
                                  num_blocks=2)
  assert max_rel_err(out, a["out"]) < 5e-6


def test_msa_attention_golden():
  a, p = load("msa_attention")
  assert max_rel_err(dif.msa_attention(a["act"], a["mask"], a["pair_act"], p), a["out"]) < 1e-5


def test_outer_product_mean_golden():
  a, p = load("outer_product_mean")
  assert max_rel_err(dif.outer_product_mean(a["act"], a["mask"], p), a["out"]) < 2e-6


def test_embedding_golden():
  """The embedding-side pair ops: Evoformer pair embedding + recycling step and the DiffusionHead base
  conditioning, against the reference's own outputs (N=16, two chains, its relative encoding)."""
  from oracle import embedding as emb
  a, p = load("embedding_n16")
  n = a["target_feat"].shape[0]
  assert max_rel_err(emb.seq_pair_embedding(a["target_feat"], a["target_feat"], p), a["seq_pair"]) < 1e-6
  assert max_rel_err(emb.position_feat(a["rel_features"], p), a["position_feat"]) < 1e-6
  contact = emb.contact_matrix(n, a["pl_idx"], a["pl_mask"], a["ll_idx"], a["ll_mask"])
  assert int(contact.sum()) == 3 and contact[0, 0] == 0
  assert max_rel_err(emb.bonds_act(contact, p), a["bonds_act"]) < 1e-6
  pair = a["seq_pair"] + a["position_feat"] + a["bonds_act"]
  assert max_rel_err(emb.prev_embedding(a["prev_pair"], pair, p), a["prev_out"]) < 2e-6
  hp = {k[len("head."):]: v for k, v in p.items() if k.startswith("head.")}
  sc, pc = emb.base_cond(a["rel_features"], a["single"], a["prev_out"], a["target_feat"], True, hp)
  assert max_rel_err(sc, a["single_cond"]) < 2e-6
  assert max_rel_err(pc, a["pair_cond"]) < 2e-6
