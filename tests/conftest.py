import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
  sys.path.insert(0, REPO)


def pytest_configure(config):
  config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(autouse=True)
def _highest_precision():
  import torch
  old = torch.get_float32_matmul_precision()
  torch.set_float32_matmul_precision("highest")
  yield
  torch.set_float32_matmul_precision(old)
