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
