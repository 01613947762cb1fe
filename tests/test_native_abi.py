"""The C-ABI library loads and exports every entry point include/sparsefold_b200.h declares."""
import os
import re

import pytest

from sparsefold_b200 import _native

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "sparsefold_b200.h")


def _declared():
  text = open(HEADER).read()
  text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
  return sorted(set(re.findall(r"\b(sf_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
  if not os.path.exists(_native.LIB_PATH):
    from sparsefold_b200 import build
    build.build()
  return _native.load()


def test_header_declares_entry_points():
  names = _declared()
  assert "sf_tri_mult_project" in names and "sf_attention" in names
  assert len(names) >= 15


def test_library_exports_every_declared_symbol(lib):
  for name in _declared():
    assert hasattr(lib, name), f"{name} declared in the header but not exported"


def test_binding_covers_every_declared_symbol():
  assert set(_declared()) <= set(_native.exported_symbols())


def test_version_and_error_plumbing(lib):
  assert b"sm_100a" in lib.sf_version()
  # A bad argument is rejected on the host without touching a device.
  st = lib.sf_layernorm(0, None, None, None, None, 1, 1, 1e-5, None)
  assert st == _native.SF_ERR_ARG
  assert "sf_layernorm" in _native.last_error()


def test_workspace_queries_need_no_device(lib):
  assert lib.sf_tri_mult_project_workspace(_native.SF_BF16, 64) > 64 * 64 * 128 * 2
  assert lib.sf_tri_attention_workspace(_native.SF_F32, 16, 4) > 0
