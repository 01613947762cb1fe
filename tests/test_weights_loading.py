"""Real-weight loading (SURVEY next-step f4): AF3-layout parameters through the reference's loader, then
the b200 packing, on the CPU.

A synthetic bf16 checkpoint in the AF3 layout (tests/af3_layout.py) is loaded into the reference's
``PairFormerIteration`` built under the b200 backend with ``backend.load_and_prepare``; the reference's
strict loader must accept it completely, the state_dict keys must stay the reference's, and the packed
kernel buffers must equal the packing of the same (bf16-valued) parameters done without the loader.
"""
import pytest
import torch

from tests.refsrc import import_reference


@pytest.fixture(scope="module")
def ref():
  if import_reference() is None:
    pytest.skip("reference package not present")
  from sparsefold.runtime import config
  from sparsefold import backends
  import sparsefold_b200.backend as b200
  b200.register()
  config.configure_runtime(backend="b200", device="cpu", sdpa_implementation="math", enable_sharding=False,
                           enable_compile=False, logs=set())
  backends.init()
  yield
  b200.unapply()
  config.configure_runtime(backend="torch", device="cpu", sdpa_implementation="math", enable_sharding=False,
                           enable_compile=False, logs=set())
  backends._current_library = None
  backends._applied_libraries.discard("b200")


def _block():
  from sparsefold.model.trunk import blocks, network
  from sparsefold.model import config as mc
  return blocks.PairFormerIteration(network.Evoformer.Config().pairformer, mc.GlobalConfig(), with_single=True,
                                    num_channels=128, seq_channels=384)


def test_af3_layout_checkpoint_loads_and_packs(ref):
  from sparsefold_b200 import backend, modules, synth
  from tests.af3_layout import checkpoint_from_module
  src = _block()
  synth.init_params(src, 3)
  ckpt = checkpoint_from_module(src)
  assert all(t.dtype == torch.bfloat16 for scope in ckpt.values() for t in scope.values())
  blk = _block()
  keys = set(blk.state_dict())
  report = backend.load_and_prepare(blk, ckpt)
  assert report.complete and len(report.entries) == len(keys)
  assert set(blk.state_dict()) == keys
  for k, v in blk.state_dict().items():                          # values are the bf16 checkpoint values
    assert torch.equal(v, src.state_dict()[k].to(torch.bfloat16).to(v.dtype)), k
  mine = modules.PairFormerIteration()                            # the same values packed without the loader
  mine.load_state_dict({k: v.to(torch.bfloat16).float() for k, v in src.state_dict().items()}, strict=True)
  modules.prepare(mine)
  got = {k: v for k, v in blk.named_buffers() if "._sf_" in k or k.startswith("_sf_")}
  want = {k: v for k, v in mine.named_buffers() if "._sf_" in k or k.startswith("_sf_")}
  assert got.keys() == want.keys() and got
  for k in got:
    assert torch.equal(got[k], want[k]), k


def test_misshaped_checkpoint_is_refused_and_nothing_is_packed(ref):
  from sparsefold.weights import WeightLoadError
  from sparsefold_b200 import backend, synth
  from tests.af3_layout import checkpoint_from_module
  src = _block()
  synth.init_params(src, 3)
  ckpt = checkpoint_from_module(src)
  scope = next(k for k in ckpt if k.endswith("pair_attention1/q_projection"))
  ckpt[scope]["weights"] = ckpt[scope]["weights"][..., :-1]
  blk = _block()
  with pytest.raises(WeightLoadError):
    backend.load_and_prepare(blk, ckpt)
  assert not any(getattr(m, "_native_prepared", False) for m in blk.modules())
