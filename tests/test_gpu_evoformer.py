"""The other trunk stacks that reuse the hot-path kernels, through the b200 plugin on the GPU.

* The MSA-stack block, the reference's ``EvoformerIteration`` (trunk/blocks.py:913-1058: outer-product
  mean, MSA pair-weighted averaging, MSA transition, both triangle multiplications, both triangle
  attentions, pair transition), built from the replaced factories.
* ``PairFormerIteration`` without the single track (``with_single=False``), the form the template stack
  and the confidence head use.

Both run on the GPU under the b200 backend and are checked against the reference's own Torch path on the
CPU (backend "torch", math SDPA, fp32 "highest") on the same parameters and inputs: fp32 within 1e-4,
bf16 within 2e-2 (the reference run in fp32 on bf16-rounded inputs and weight matrices, LayerNorm
parameters and biases in fp32 as the kernels take them).
"""
import pytest
import torch

from sparsefold_b200 import _native, synth
from tests.golden_io import max_rel_err
from tests.refsrc import import_reference, loaded_shapes

pytestmark = pytest.mark.gpu
TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


@pytest.fixture(scope="module")
def ref():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  if import_reference() is None:
    pytest.skip("reference package not present")
  _native.check(_native.load().sf_device_check(), "sf_device_check")
  from sparsefold.runtime import config
  from sparsefold import backends
  import sparsefold_b200.backend as b200
  b200.register()
  config.configure_runtime(backend="b200", device="cuda", sdpa_implementation="math", enable_sharding=False,
                           enable_compile=False, logs=set())
  backends.init()
  from sparsefold.model.trunk import blocks, network
  from sparsefold.model import config as mc
  yield blocks, network, mc, backends, b200
  b200.unapply()
  config.configure_runtime(backend="torch", device="cpu", sdpa_implementation="math", enable_sharding=False,
                           enable_compile=False, logs=set())
  backends._current_library = None
  backends._applied_libraries.discard("b200")


def _kernel_values(p, dtype):
  keep = lambda k: k.split(".")[-1] in ("bias", "output_b") or "norm" in k
  return {k: (v.float() if keep(k) else v.to(dtype).float()) for k, v in p.items()}


def _twins(ref, make, seed):
  """(module under b200, module of the reference's own Torch path on the CPU) with the same parameters."""
  blocks, network, mc, backends, b200 = ref
  mine = loaded_shapes(make())
  p = synth.init_params(mine, seed)
  backends.prepare(mine)
  b200.unapply()                      # the reference's own classes for the second copy
  try:
    theirs = loaded_shapes(make()).cpu()
  finally:
    b200.apply()
  return mine, theirs, p


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_evoformer_iteration_msa_stack_block(ref, dtype):
  blocks, network, mc, backends, b200 = ref
  make = lambda: blocks.EvoformerIteration(blocks.EvoformerIteration.Config(), mc.GlobalConfig(), num_channels=64,
                                           num_output_channel=128)
  mine, theirs, p = _twins(ref, make, 21)
  assert type(mine.outer_product_mean).__name__.endswith("B200") and not type(theirs.outer_product_mean).__name__.endswith("B200")
  g = torch.Generator().manual_seed(5)
  m_, n = 8, 32
  msa = torch.randn(m_, n, 64, generator=g)
  pair = torch.randn(n, n, 128, generator=g)
  msa_mask = torch.rand(m_, n, generator=g) > 0.15
  seq_mask = torch.arange(n) < 29
  with torch.no_grad():
    out = mine.cuda()({"msa": msa.to(dtype).cuda(), "pair": pair.to(dtype).cuda()},
                      {"msa": msa_mask.cuda(), "seq": seq_mask.cuda()})
    torch.cuda.synchronize()
    theirs.load_state_dict(_kernel_values(p, dtype), strict=True)
    want = theirs({"msa": msa.to(dtype).float(), "pair": pair.to(dtype).float()}, {"msa": msa_mask, "seq": seq_mask})
  assert _native.device_status() == 0
  assert max_rel_err(out["pair"].float().cpu(), want["pair"]) < TOL[dtype]
  assert max_rel_err(out["msa"].float().cpu(), want["msa"]) < TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_pairformer_without_single_track(ref, dtype):
  blocks, network, mc, backends, b200 = ref
  make = lambda: blocks.PairFormerIteration(network.Evoformer.Config().pairformer, mc.GlobalConfig(),
                                            with_single=False, num_channels=128)
  mine, theirs, p = _twins(ref, make, 22)
  z, _, mask = synth.pair_inputs(40, n_real=37, seed=6)
  with torch.no_grad():
    got = mine.cuda()(z.to(dtype).cuda(), seq_mask=mask.cuda())
    torch.cuda.synchronize()
    theirs.load_state_dict(_kernel_values(p, dtype), strict=True)
    want = theirs(z.to(dtype).float(), seq_mask=mask)
  assert _native.device_status() == 0
  assert max_rel_err(got.float().cpu(), want) < TOL[dtype]
