"""Failure detection on the GPU without a fault: a bounded wait that runs out.

``sf_selftest_wait`` launches one warp that waits on an mbarrier nothing
arrives on, through the same bounded wait every tcgen05 kernel of the library
uses (with a short bound).  The kernel must return, the library's status word
must read SF_ERR_TIMEOUT, reading it with clear must reset it, and the CUDA
context must stay usable (a later op gives the right answer).  No trap, assert,
bad address or endless loop is involved.
"""
import time

import pytest
import torch

from sparsefold_b200 import _native as N
from sparsefold_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  N.check(N.load().sf_device_check(), "sf_device_check")


def _stream():
  return torch.cuda.current_stream().cuda_stream


def test_wait_that_nothing_completes_times_out_and_is_reported():
  lib = N.load()
  assert N.device_status(clear=True) == 0
  t0 = time.monotonic()
  N.check(lib.sf_selftest_wait(1 << 12, 0, _stream()), "sf_selftest_wait")
  torch.cuda.synchronize()
  assert time.monotonic() - t0 < 5.0                       # the kernel returned
  assert N.device_status(clear=False) == N.SF_ERR_TIMEOUT   # read without clearing
  assert N.device_status(clear=True) == N.SF_ERR_TIMEOUT    # read and clear
  assert N.device_status() == 0


def test_completed_wait_leaves_status_clear():
  lib = N.load()
  assert N.device_status(clear=True) == 0
  N.check(lib.sf_selftest_wait(1 << 12, 1, _stream()), "sf_selftest_wait")
  torch.cuda.synchronize()
  assert N.device_status() == 0


def test_context_usable_after_a_timeout():
  lib = N.load()
  N.check(lib.sf_selftest_wait(1 << 10, 0, _stream()), "sf_selftest_wait")
  assert N.device_status() == N.SF_ERR_TIMEOUT
  x = torch.randn(64, 384, device="cuda")
  w = torch.rand(384, device="cuda") + 0.5
  b = torch.randn(384, device="cuda")
  y = ops.layer_norm(x, w, b)
  ref = torch.nn.functional.layer_norm(x.cpu(), (384,), w.cpu(), b.cpu(), 1e-5)
  torch.testing.assert_close(y.cpu(), ref, rtol=1e-4, atol=1e-4)
  assert N.device_status() == 0


def test_selftest_rejects_unbounded_polls():
  lib = N.load()
  assert lib.sf_selftest_wait(0, 0, None) == N.SF_ERR_ARG
  assert lib.sf_selftest_wait(0xFFFFFFFF, 0, None) == N.SF_ERR_ARG
  assert "polls" in N.last_error()


def test_peer_wait_on_a_flag_nothing_raises_times_out():
  """The flag wait of the NVLink peer exchange (sf_peer_wait), on one GPU: a 'peer' flag nobody raises
  (a local array of zeros) makes the bounded wait run out; the kernel returns and reports SF_ERR_TIMEOUT.
  A flag that is already raised passes at once and leaves the status clear."""
  lib = N.load()
  flags = torch.zeros(4, dtype=torch.int32, device="cuda")
  assert N.device_status(clear=True) == 0
  t0 = time.monotonic()
  N.call("sf_peer_wait", flags.data_ptr(), 4, 0, 1, 1 << 12, _stream())
  torch.cuda.synchronize()
  assert time.monotonic() - t0 < 5.0
  assert N.device_status(clear=True) == N.SF_ERR_TIMEOUT
  flags.fill_(7)
  N.call("sf_peer_wait", flags.data_ptr(), 4, 0, 7, 1 << 12, _stream())
  torch.cuda.synchronize()
  assert N.device_status() == 0
  assert lib.sf_peer_wait(flags.data_ptr(), 0, 0, 1, 1, None) == N.SF_ERR_ARG       # no ranks
  assert lib.sf_peer_wait(flags.data_ptr(), 4, 0, 1, 0, None) == N.SF_ERR_ARG       # unbounded
