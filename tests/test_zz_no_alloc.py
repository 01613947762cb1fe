"""sf_transition_noalloc, the TransitionBlock entry point for callers that cannot allocate.

Callers that may not call cudaMalloc (code that must not touch the device
memory map, embedders with a fixed memory budget, bindings without a place to
keep a workspace) use this entry point; it runs the same kernels as
sf_transition on a fixed 16 MiB scratch array inside the library.  The test
calls both entry points through the C ABI on the same inputs, twice in a row
(the scratch keeps the previous call's contents), and checks that they agree
with each other and with the CPU oracle of TransitionBlock; it also checks
that a size beyond the fixed scratch is refused before anything is launched.  This file is
collected last so that a run stopping at the first failure has already run
every other test.
"""
import pytest
import torch

from oracle import pairformer as orc
from sparsefold_b200 import _native as N
from tests.golden_io import max_rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  N.check(N.load().sf_device_check(), "sf_device_check")


def _inputs(rows, c, inter, dtype, seed):
  g = torch.Generator().manual_seed(seed)
  x = torch.randn(rows, c, generator=g).to(dtype).cuda()
  ln_w = (1 + 0.1 * torch.randn(c, generator=g)).cuda()
  ln_b = (0.1 * torch.randn(c, generator=g)).cuda()
  w1 = (torch.randn(2 * inter, c, generator=g) / c ** 0.5).to(dtype).cuda()
  w2 = (torch.randn(c, inter, generator=g) / inter ** 0.5).to(dtype).cuda()
  return x, ln_w, ln_b, w1, w2


def _with_workspace(dt, x, ln_w, ln_b, w1, w2, rows, c, inter):
  lib = N.load()
  ws = torch.empty(max(lib.sf_transition_workspace(dt, rows, inter), 256), dtype=torch.uint8, device="cuda")
  y = torch.empty_like(x)
  N.check(lib.sf_transition(dt, x.data_ptr(), ln_w.data_ptr(), ln_b.data_ptr(), w1.data_ptr(), w2.data_ptr(),
                            y.data_ptr(), rows, c, inter, ws.data_ptr(), ws.numel(),
                            torch.cuda.current_stream().cuda_stream), "sf_transition")
  return y


def _no_alloc(dt, x, ln_w, ln_b, w1, w2, rows, c, inter):
  y = torch.empty_like(x)
  N.check(N.load().sf_transition_noalloc(dt, x.data_ptr(), ln_w.data_ptr(), ln_b.data_ptr(), w1.data_ptr(),
                                         w2.data_ptr(), y.data_ptr(), rows, c, inter,
                                         torch.cuda.current_stream().cuda_stream), "sf_transition_noalloc")
  return y


def _oracle(x, ln_w, ln_b, w1, w2):
  """TransitionBlock on the CPU (blocks.py:79-96) on the same (dtype-rounded) inputs, in fp32."""
  p = {"input_layer_norm.weight": ln_w.cpu(), "input_layer_norm.bias": ln_b.cpu(),
       "transition1.weight": w1.float().cpu().T, "transition2.weight": w2.float().cpu().T}
  return orc.transition_block(x.float().cpu(), p)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 2e-2)])
def test_no_alloc_matches_workspace_entry_point_twice(dtype, tol):
  dt = N.SF_F32 if dtype == torch.float32 else N.SF_BF16
  rows, c, inter = 512, 384, 1536   # the Pairformer single transition at N_token = 512
  for seed in (1, 2):               # two calls in a row on the shared scratch
    args = _inputs(rows, c, inter, dtype, seed)
    ref = _with_workspace(dt, *args, rows, c, inter)
    got = _no_alloc(dt, *args, rows, c, inter)
    torch.cuda.synchronize()
    assert max_rel_err(got.float().cpu(), ref.float().cpu()) < tol
    assert max_rel_err(got.float().cpu(), _oracle(*args)) < tol


def test_no_alloc_rejects_sizes_beyond_the_fixed_scratch():
  lib = N.load()
  limit = lib.sf_transition_noalloc_max_scratch()
  rows, c, inter = 4096, 384, 1536
  assert lib.sf_transition_workspace(N.SF_BF16, rows, inter) > limit
  # Null tensor pointers: the size check refuses the call first; were it ever to run later,
  # sf_transition's own argument check would still refuse null pointers before any launch.
  st = lib.sf_transition_noalloc(N.SF_BF16, None, None, None, None, None, None, rows, c, inter, None)
  assert st == N.SF_ERR_WORKSPACE
  assert "scratch" in N.last_error()
