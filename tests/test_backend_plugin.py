"""The b200 backend behind the reference's own plugin API (backends/__init__.py:28-102).

Runs only where the reference package is importable ($SPARSEFOLD_REF_SRC or the
pip-installed copy under baseline/_ref, see tests/refsrc.py); it checks factory
replacement, class identity, and that preparing a reference PairFormerIteration
keeps its state_dict contract.
"""
import pytest

from tests.refsrc import import_reference


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
