"""Embedding-side pair ops on the GPU (trunk/network.py:195-285, diffusion/generator.py:367-391).

* The two kernels against plain fp32 PyTorch on the host: ``sf_pair_outer_sum`` (vector and scalar
  paths, with an addend) and ``sf_pair_sparse_linear`` (one-hot relative encodings, dense inputs,
  a 0/1 contact map, a residual, 32 to 256 channels, weights staged in shared memory or read from
  global memory).
* The reference's own ``Evoformer`` and ``DiffusionHead`` built under the b200 backend: their pair
  embedding, bond embedding, recycling step and base conditioning against the fixture the reference
  itself wrote (fp32, 1e-4) and against the oracle on bf16-rounded inputs (bf16, 2e-2).
"""
import types

import pytest
import torch

from oracle import embedding as emb
from sparsefold_b200 import _native, ops
from tests.golden_io import load, max_rel_err
from tests.refsrc import import_reference, loaded_shapes

pytestmark = pytest.mark.gpu
DT = torch.bfloat16


@pytest.fixture(scope="module", autouse=True)
def _device():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  _native.check(_native.load().sf_device_check(), "sf_device_check")


def _one_hot_rel(n, seed):
  """Relative-encoding-shaped features: four one-hot groups (66 + 66 + 1 + 6 = 139) per position."""
  g = torch.Generator().manual_seed(seed)
  x = torch.zeros(n, n, 139)
  i = torch.arange(n)
  x[i[:, None], i[None, :], torch.clamp(i[:, None] - i[None, :] + 32, 0, 64)] = 1.0
  x[i[:, None], i[None, :], 66 + torch.randint(0, 66, (n, n), generator=g)] = 1.0
  x[..., 132] = (torch.rand(n, n, generator=g) > 0.5).float()
  x[i[:, None], i[None, :], 133 + torch.randint(0, 6, (n, n), generator=g)] = 1.0
  return x


@pytest.mark.parametrize("dtype", [torch.float32, DT])
@pytest.mark.parametrize("c", [128, 13])
def test_pair_outer_sum(dtype, c):
  g = torch.Generator().manual_seed(1)
  b, n = 37, 53
  left, right, add = torch.randn(b, c, generator=g), torch.randn(n, c, generator=g), torch.randn(b, n, c, generator=g)
  l_, r_, a_ = (t.to(dtype) for t in (left, right, add))
  got = ops.pair_outer_sum(l_.cuda(), r_.cuda())
  got_a = ops.pair_outer_sum(l_.cuda(), r_.cuda(), a_.cuda())
  torch.cuda.synchronize()
  want = l_.float()[:, None] + r_.float()[None, :]
  tol = 1e-7 if dtype == torch.float32 else 4e-3
  assert max_rel_err(got.float().cpu(), want) < tol
  assert max_rel_err(got_a.float().cpu(), want + a_.float()) < tol
  assert _native.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float32, DT])
@pytest.mark.parametrize("kind", ["one_hot", "dense", "contact"])
@pytest.mark.parametrize("c", [32, 128, 256])
def test_pair_sparse_linear(dtype, kind, c):
  g = torch.Generator().manual_seed(2)
  n = 40
  if kind == "one_hot":
    x = _one_hot_rel(n, 3)
  elif kind == "dense":
    x = torch.randn(n, n, 139, generator=g)
  else:
    x = (torch.rand(n, n, 1, generator=g) > 0.9).float()
  w = torch.randn(x.shape[-1], c, generator=g) / x.shape[-1] ** 0.5
  res = torch.randn(n, n, c, generator=g)
  xd = x.to(dtype)
  got = ops.pair_sparse_linear(xd.cuda(), w.cuda())
  got_r = ops.pair_sparse_linear(xd.cuda(), w.cuda(), residual=res.to(dtype).cuda())
  torch.cuda.synchronize()
  want = xd.double() @ w.double()
  tol = 1e-6 if dtype == torch.float32 else 4e-3
  assert max_rel_err(got.float().cpu(), want) < tol
  assert max_rel_err(got_r.float().cpu(), want + res.to(dtype).double()) < tol
  assert _native.device_status() == 0


def test_pair_sparse_linear_weights_from_global_memory():
  """k * channels * 4 bytes above the shared-memory staging limit (512 x 128 fp32 = 256 KB)."""
  g = torch.Generator().manual_seed(4)
  x = torch.randn(300, 512, generator=g) * (torch.rand(300, 512, generator=g) > 0.7)
  w = torch.randn(512, 128, generator=g)
  got = ops.pair_sparse_linear(x.cuda(), w.cuda())
  torch.cuda.synchronize()
  assert max_rel_err(got.cpu(), x.double() @ w.double()) < 1e-6


# ---------------------------------------------------------------------------------------------------
@pytest.fixture(scope="module")
def ref_models():
  if import_reference() is None:
    pytest.skip("reference package not present")
  from sparsefold.runtime import config
  from sparsefold import backends
  import sparsefold_b200.backend as b200
  b200.register()
  config.configure_runtime(backend="b200", device="cuda", sdpa_implementation="math", enable_sharding=False,
                           enable_compile=False, logs=set())
  backends.init()
  from sparsefold.model.trunk import network
  from sparsefold.model.diffusion import generator
  from sparsefold.model import config as mc
  gc = mc.GlobalConfig()
  cfg = network.Evoformer.Config()
  cfg.pairformer.num_layer = 1            # the stacks are not exercised here; one block each keeps it small
  cfg.msa_stack.num_layer = 1
  evo = loaded_shapes(network.Evoformer(cfg, gc, target_feat_size=447))
  head = generator.DiffusionHead(generator.DiffusionHead.Config(), gc, pair_channels=128, seq_channels=384,
                                 target_feat_size=447)
  a, p = load("embedding_n16")
  with torch.no_grad():
    for mod, pre in ((evo, ""), (head, "head.")):
      for name, prm in mod.named_parameters():
        prm.copy_(p[pre + name] if pre + name in p else torch.randn(prm.shape) * 0.02)
  backends.prepare(evo)
  backends.prepare(head)
  yield evo, head, a, p
  b200.unapply()
  config.configure_runtime(backend="torch", device="cpu", sdpa_implementation="math", enable_sharding=False,
                           enable_compile=False, logs=set())
  backends._current_library = None
  backends._applied_libraries.discard("b200")


def _batch(a, dev):
  ns = types.SimpleNamespace
  return ns(token_features=ns(token_index=torch.arange(a["target_feat"].shape[0], device=dev)),
            polymer_ligand_bond_info=ns(tokens_to_polymer_ligand_bonds=ns(gather_idxs=a["pl_idx"].to(dev),
                                                                          gather_mask=a["pl_mask"].to(dev))),
            ligand_ligand_bond_info=ns(tokens_to_ligand_ligand_bonds=ns(gather_idxs=a["ll_idx"].to(dev),
                                                                        gather_mask=a["ll_mask"].to(dev))))


@pytest.mark.parametrize("dtype", [torch.float32, DT])
def test_reference_evoformer_pair_embedding_on_b200(ref_models, dtype):
  evo, head, a, p = ref_models
  cu = lambda t: t.to(dtype).cuda()
  tf, rel, prev = a["target_feat"], a["rel_features"], a["prev_pair"]
  with torch.no_grad():
    seq_pair = evo._get_seq_pair_embedding(None, cu(tf), cu(tf))
    pos = evo._get_position_feat(rel.cuda(), dtype)
    bonds = evo._get_bonds_act(_batch(a, "cuda"), dtype)
    pair = seq_pair + pos + bonds
    prev_out = evo.prev_embedding(evo.prev_embedding_layer_norm(cu(prev)), residual=pair)
  torch.cuda.synchronize()
  assert _native.device_status() == 0
  if dtype == torch.float32:
    want = {"seq_pair": a["seq_pair"], "pos": a["position_feat"], "bonds": a["bonds_act"], "prev": a["prev_out"]}
    tol = 1e-4
  else:
    r = lambda t: t.to(dtype).float()
    pw = {k: (v.float() if "norm" in k else r(v)) for k, v in p.items()}
    contact = emb.contact_matrix(tf.shape[0], a["pl_idx"], a["pl_mask"], a["ll_idx"], a["ll_mask"])
    sp, ps, bd = (emb.seq_pair_embedding(r(tf), r(tf), pw), emb.position_feat(r(rel), p), emb.bonds_act(contact, p))
    want = {"seq_pair": sp, "pos": ps, "bonds": bd, "prev": emb.prev_embedding(r(prev), r(r(sp) + r(ps) + r(bd)), pw)}
    tol = 2e-2
  assert max_rel_err(seq_pair.float().cpu(), want["seq_pair"]) < tol
  assert max_rel_err(pos.float().cpu(), want["pos"]) < tol
  assert max_rel_err(bonds.float().cpu(), want["bonds"]) < tol
  assert max_rel_err(prev_out.float().cpu(), want["prev"]) < tol


@pytest.mark.parametrize("dtype", [torch.float32, DT])
def test_reference_diffusion_head_base_cond_on_b200(ref_models, dtype):
  evo, head, a, p = ref_models
  cu = lambda t: t.to(dtype).cuda()
  with torch.no_grad():
    sc, pc = head._get_base_cond(cu(a["rel_features"]), {"single": cu(a["single"]), "pair": cu(a["prev_out"]),
                                                         "target_feat": cu(a["target_feat"])}, True)
  torch.cuda.synchronize()
  assert _native.device_status() == 0
  if dtype == torch.float32:
    want_s, want_p, tol = a["single_cond"], a["pair_cond"], 1e-4
  else:
    r = lambda t: t.to(dtype).float()
    hp = {k[len("head."):]: v for k, v in p.items() if k.startswith("head.")}
    hp = {k: (v.float() if ("norm" in k or "projection" in k) else r(v)) for k, v in hp.items()}
    want_s, want_p = emb.base_cond(r(a["rel_features"]), r(a["single"]), r(a["prev_out"]), r(a["target_feat"]), True,
                                   hp)
    tol = 2e-2
  assert max_rel_err(sc.float().cpu(), want_s) < tol
  assert max_rel_err(pc.float().cpu(), want_p) < tol
