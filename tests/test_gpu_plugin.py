"""The reference's own module classes on the GPU through the b200 plugin.

The reference package (tests/refsrc.py: $SPARSEFOLD_REF_SRC or the pip-installed
copy under baseline/_ref) is configured with ``backend="b200"``, so
``backends.init()`` runs this package's ``apply()`` and the reference's
``PairFormerIteration`` is built from the replaced factories
(trunk/blocks.py:766-860).  Its forward (blocks.py:862-910) is the reference's
own code; every sub-module is a ``(B200 mixin, reference class)``.  The outputs
are checked against the golden fixture the reference itself produced (fp32,
1e-4) and against the oracle on bf16-rounded inputs (bf16, 2e-2), and must equal
the standalone modules' outputs bit for bit (same kernels, same packing).
"""
import pytest
import torch

from oracle import pairformer as orc
from sparsefold_b200 import _native, modules
from tests.golden_io import load, max_rel_err
from tests.refsrc import import_reference

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref_blocks():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  if import_reference() is None:
    pytest.skip("reference package not present")
  _native.check(_native.load().sf_device_check(), "sf_device_check")
  from sparsefold.runtime import config
  from sparsefold import backends
  import sparsefold_b200.backend as b200
  b200.register()
  config.configure_runtime(backend="b200", device="cuda", sdpa_implementation="math",
                           enable_sharding=False, enable_compile=False, logs=set())
  backends.init()
  from sparsefold.model.trunk import blocks, network
  from sparsefold.model import config as mc
  yield blocks, network, mc, backends
  b200.unapply()
  config.configure_runtime(backend="torch", device="cpu", sdpa_implementation="math",
                           enable_sharding=False, enable_compile=False, logs=set())
  backends._current_library = None
  backends._applied_libraries.discard("b200")


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 2e-2)])
def test_reference_pairformer_block_on_b200(ref_blocks, dtype, tol):
  blocks, network, mc, backends = ref_blocks
  arrays, p = load("pairformer_n24")
  blk = blocks.PairFormerIteration(network.Evoformer.Config().pairformer, mc.GlobalConfig(), with_single=True,
                                   num_channels=128, seq_channels=384)
  assert isinstance(blk.pair_attention1, modules.GridSelfAttentionB200)
  assert isinstance(blk.triangle_multiplication_incoming, modules.TriangleMultiplicationB200)
  blk.load_state_dict(p, strict=True)
  backends.prepare(blk)
  blk = blk.cuda()
  z, s, mask = arrays["z"], arrays["s"], arrays["mask"]
  with torch.no_grad():
    zo, so = blk(z.to(dtype).cuda(), seq_mask=mask.cuda(), single_act=s.to(dtype).cuda())
  torch.cuda.synchronize()
  assert _native.device_status() == 0
  if dtype == torch.float32:
    zr, sr = arrays["z_out"], arrays["s_out"]
  else:
    pr = {k: v.to(dtype).float() for k, v in p.items()}
    zr, sr = orc.pairformer_block(z.to(dtype).float(), s.to(dtype).float(), mask, pr)
  assert max_rel_err(zo.float().cpu(), zr) < tol
  assert max_rel_err(so.float().cpu(), sr) < tol
  mine = modules.PairFormerIteration()
  mine.load_state_dict(p, strict=True)
  modules.prepare(mine)
  mine = mine.cuda()
  with torch.no_grad():
    zm, sm = mine(z.to(dtype).cuda(), seq_mask=mask.cuda(), single_act=s.to(dtype).cuda())
  assert torch.equal(zm, zo) and torch.equal(sm, so)


def test_af3_layout_checkpoint_through_the_reference_loader_on_b200(ref_blocks):
  """Weights in the AF3 layout (bf16, tests/af3_layout.py) loaded by the reference's own loader into its
  PairFormerIteration, packed by prepare(), run on the GPU in bf16 against the oracle on the same values."""
  blocks, network, mc, backends = ref_blocks
  from sparsefold_b200 import backend, synth
  from tests.af3_layout import checkpoint_from_module

  def make():
    return blocks.PairFormerIteration(network.Evoformer.Config().pairformer, mc.GlobalConfig(), with_single=True,
                                      num_channels=128, seq_channels=384)
  src = make()
  synth.init_params(src, 11)
  blk = make()
  report = backend.load_and_prepare(blk, checkpoint_from_module(src))
  assert report.complete
  blk = blk.cuda()
  z, s, mask = synth.pair_inputs(64, n_real=57, seed=12)
  dt = torch.bfloat16
  with torch.no_grad():
    zo, so = blk(z.to(dt).cuda(), seq_mask=mask.cuda(), single_act=s.to(dt).cuda())
  torch.cuda.synchronize()
  assert _native.device_status() == 0
  p = {k: v.to(dt).float().cpu() for k, v in src.state_dict().items()}   # the checkpoint's bf16 values
  zr, sr = orc.pairformer_block(z.to(dt).float(), s.to(dt).float(), mask, p)
  assert max_rel_err(zo.float().cpu(), zr) < 2e-2
  assert max_rel_err(so.float().cpu(), sr) < 2e-2
