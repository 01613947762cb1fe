"""The b200 backend behind the reference's own plugin API (backends/__init__.py:28-102).

Runs only where the reference package is importable ($SPARSEFOLD_REF_SRC or the
pip-installed copy under baseline/_ref, see tests/refsrc.py); it checks factory
replacement, class identity, and that preparing a reference PairFormerIteration
keeps its state_dict contract.
"""
import pytest

from tests.refsrc import import_reference, loaded_shapes


@pytest.fixture(scope="module")
def ref():
  if import_reference() is None:
    pytest.skip("reference package not present")
  from sparsefold.runtime import config
  from sparsefold import backends
  import sparsefold_b200.backend as b200
  b200.register()
  config.configure_runtime(backend="b200", device="cpu", sdpa_implementation="math",
                           enable_sharding=False, enable_compile=False, logs=set())
  backends.init()
  yield backends
  b200.unapply()
  config.configure_runtime(backend="torch", device="cpu", sdpa_implementation="math",
                           enable_sharding=False, enable_compile=False, logs=set())
  backends._current_library = None
  backends._applied_libraries.discard("b200")


def test_apply_replaces_factories(ref):
  from sparsefold.model.trunk import blocks
  from sparsefold.model.diffusion import transformer
  from sparsefold_b200 import modules
  for name in ("GridSelfAttention", "TriangleMultiplication", "TransitionBlock", "SingleActUpdate"):
    assert issubclass(getattr(blocks, name), modules.B200Module), name
  assert issubclass(transformer.SelfAttention, modules.SelfAttentionB200)


def test_reference_block_prepares_with_same_state_dict(ref):
  import torch
  from sparsefold.model.trunk import blocks, network
  from sparsefold.model import config as mc
  from sparsefold_b200 import synth
  blk = blocks.PairFormerIteration(network.Evoformer.Config().pairformer, mc.GlobalConfig(),
                                   with_single=True, num_channels=128, seq_channels=384)
  synth.init_params(blk, 0)
  keys = set(blk.state_dict())
  z, s, mask = synth.pair_inputs(8)
  with pytest.raises(RuntimeError, match="not prepared"):
    blk(z, seq_mask=mask, single_act=s)
  counts = ref.prepare(blk)
  assert counts["opaque"] >= 6
  assert set(blk.state_dict()) == keys
  for m in blk.modules():
    assert set(m._buffers) <= m._non_persistent_buffers_set
  # The standalone block has the same parameter names, so weights transfer 1:1.
  from sparsefold_b200 import modules
  mine = modules.PairFormerIteration()
  mine.load_state_dict(blk.state_dict(), strict=True)
  for k, v in mine.state_dict().items():
    torch.testing.assert_close(v, blk.state_dict()[k], rtol=0, atol=0)


def test_evoformer_and_diffusion_head_pair_layers_take_b200_classes(ref):
  """The embedding-side pair layers (trunk/network.py:195-285, diffusion/generator.py:367-391): prepare()
  gives the Evoformer's and the DiffusionHead's pair-side Linear / LayerNorm instances B200 classes, keeps
  the state_dict, and the product path refuses host tensors (no CPU fallback)."""
  import torch
  from sparsefold.model.trunk import network
  from sparsefold.model.diffusion import generator
  from sparsefold.model import config as mc
  from sparsefold_b200 import modules
  assert issubclass(network.Evoformer, modules.EvoformerB200)
  assert issubclass(generator.DiffusionHead, modules.DiffusionHeadB200)
  evo = loaded_shapes(network.Evoformer(network.Evoformer.Config(), mc.GlobalConfig(), target_feat_size=447))
  head = generator.DiffusionHead(generator.DiffusionHead.Config(), mc.GlobalConfig(), pair_channels=128,
                                 seq_channels=384, target_feat_size=447)
  for mod in (evo, head):
    with torch.no_grad():
      for p in mod.parameters():
        p.normal_(0.0, 0.02)
    keys = set(mod.state_dict())
    ref.prepare(mod)
    assert set(mod.state_dict()) == keys
  for name, sparse in modules.EvoformerB200._LINEARS.items():
    sub = getattr(evo, name)
    assert isinstance(sub, modules.LinearB200) and sub._sf_sparse == sparse, name
  assert isinstance(evo.prev_embedding_layer_norm, modules.LayerNormB200)
  assert isinstance(head.pair_cond_initial_projection, modules.LinearB200)
  assert isinstance(head.pair_cond_initial_norm, modules.LayerNormB200)
  with pytest.raises(ValueError, match="CUDA tensors only"):
    evo._get_position_feat(torch.zeros(4, 4, 139), torch.float32)
  with pytest.raises(ValueError, match="CUDA tensors only"):
    evo._get_seq_pair_embedding(None, torch.zeros(4, 447), torch.zeros(4, 447))
