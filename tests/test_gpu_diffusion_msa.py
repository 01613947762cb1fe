"""Diffusion-transformer and MSA modules on the CUDA path vs the reference fixtures / oracle.

fp32 runs are compared with the reference outputs in tests/golden (tolerance 1e-4);
bf16 runs with the oracle on bf16-rounded inputs and weights (tolerance 2e-2).
"""
import types

import pytest
import torch

from oracle import diffusion as dif
from sparsefold_b200 import _native, modules
from tests.golden_io import load, max_rel_err

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


@pytest.fixture(scope="module", autouse=True)
def _device():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  _native.check(_native.load().sf_device_check(), "sf_device_check")


def _build(mod, params):
  mod.load_state_dict(params, strict=True)
  modules.prepare(mod)
  return mod.cuda()


def _cast(arrays, dtype):
  return {k: (v.to(dtype) if v.is_floating_point() else v) for k, v in arrays.items()}


def _round(p, dtype):
  return {k: v.to(dtype).float() for k, v in p.items()}


def _check(got, a, ref_fn, p, dtype):
  ref = a["out"] if dtype == torch.float32 else ref_fn(_cast(_cast(a, dtype), torch.float32), _round(p, dtype))
  err = max_rel_err(got.float().cpu(), ref)
  assert err < TOL[dtype], err
  assert _native.device_status() == 0


DTYPES = [torch.float32, torch.bfloat16]


@pytest.mark.parametrize("dtype", DTYPES)
def test_token_self_attention(dtype):
  a, p = load("diff_self_attention")
  m = _build(modules.SelfAttention(128, 4, single_cond_size=64), p)
  g = {k: v.cuda() for k, v in _cast(a, dtype).items()}
  got = m(g["x"], g["mask"], pair_logits=g["pair_logits"], single_cond=g["single_cond"])
  _check(got, a, lambda t, q: dif.self_attention(t["x"], t["mask"], q, pair_logits=t["pair_logits"],
                                                 single_cond=t["single_cond"]), p, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_adaln_transition(dtype):
  a, p = load("diff_transition")
  m = _build(modules.DiffusionTransitionBlock(128, 2, 64), p)
  g = {k: v.cuda() for k, v in _cast(a, dtype).items()}
  got = m(g["x"], single_cond=g["single_cond"])
  _check(got, a, lambda t, q: dif.transition(t["x"], q, t["single_cond"]), p, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_token_transformer(dtype):
  a, p = load("diff_transformer")
  m = _build(modules.DiffusionTransformer(128, 64, 16, num_head=4, num_blocks=4, super_block_size=2), p)
  g = {k: v.cuda() for k, v in _cast(a, dtype).items()}
  got = m(g["x"], g["mask"], g["single_cond"], g["pair_cond"])
  _check(got, a, lambda t, q: dif.transformer(t["x"], t["mask"], t["single_cond"], t["pair_cond"], q, 2, 2), p, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_atom_cross_attention(dtype):
  a, p = load("diff_cross_attention")
  m = _build(modules.CrossAttention(64, 4, 64), p)
  g = {k: v.cuda() for k, v in _cast(a, dtype).items()}
  got = m(g["x_q"], g["x_k"], g["mask_q"], g["mask_k"], pair_logits=g["pair_logits"],
          single_cond_q=g["single_cond_q"], single_cond_k=g["single_cond_k"])
  _check(got, a, lambda t, q: dif.cross_attention(t["x_q"], t["x_k"], t["mask_q"], t["mask_k"], q,
                                                  pair_logits=t["pair_logits"], single_cond_q=t["single_cond_q"],
                                                  single_cond_k=t["single_cond_k"]), p, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_atom_cross_att_transformer(dtype):
  a, p = load("diff_cross_att_transformer")
  m = _build(modules.CrossAttTransformer(64, 8, num_head=4, key_dim=64, num_blocks=2, num_intermediate_factor=2), p)
  g = {k: v.cuda() for k, v in _cast(a, dtype).items()}
  info = types.SimpleNamespace(gather_idxs=g["gather_idxs"], gather_mask=g["gather_mask"])
  got = m(g["queries_act"], g["queries_mask"], info, g["keys_mask"], g["queries_single_cond"],
          g["keys_single_cond"], g["pair_cond"])
  _check(got, a, lambda t, q: dif.cross_att_transformer(t["queries_act"], t["queries_mask"], t["gather_idxs"],
                                                        t["gather_mask"], t["keys_mask"], t["queries_single_cond"],
                                                        t["keys_single_cond"], t["pair_cond"], q, 2), p, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_msa_pair_weighted_averaging(dtype):
  a, p = load("msa_attention")
  m = _build(modules.MSAAttention(64, 128, 8), p)
  g = {k: v.cuda() for k, v in _cast(a, dtype).items()}
  got = m(g["act"], g["mask"], g["pair_act"])
  _check(got, a, lambda t, q: dif.msa_attention(t["act"], t["mask"], t["pair_act"], q), p, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_outer_product_mean(dtype):
  a, p = load("outer_product_mean")
  m = _build(modules.OuterProductMean(64, 128, 32), p)
  g = {k: v.cuda() for k, v in _cast(a, dtype).items()}
  got = m(g["act"], g["mask"])
  _check(got, a, lambda t, q: dif.outer_product_mean(t["act"], t["mask"], q), p, dtype)
