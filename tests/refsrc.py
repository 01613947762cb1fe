"""Locate and import the reference package (SparseFold) for the tests that run it.

The reference is found, in order, at ``$SPARSEFOLD_REF_SRC`` (a directory that
holds the ``sparsefold`` package, e.g. the reference's ``src/``) or at
``baseline/_ref`` in this repository, where ``pip install --target
baseline/_ref`` puts the unmodified reference.  Tests that need it skip when
neither exists.  ``weights/records.py`` of the reference imports
``zstandard``, which only checkpoint loading uses; an empty stand-in module is
registered when the package is absent.
"""
from __future__ import annotations

import os
import sys
import types

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_src() -> str | None:
  cands = []
  if os.environ.get("SPARSEFOLD_REF_SRC"):
    cands.append(os.environ["SPARSEFOLD_REF_SRC"])
  cands.append(os.path.join(REPO, "baseline", "_ref"))
  for c in cands:
    if os.path.isdir(os.path.join(c, "sparsefold")):
      return c
  return None


def import_reference() -> str | None:
  """Put the reference on sys.path (stubbing zstandard if needed); returns its path or None."""
  src = reference_src()
  if src is None:
    return None
  if src not in sys.path:
    sys.path.insert(0, src)
  try:
    import zstandard  # noqa: F401
  except ImportError:
    sys.modules["zstandard"] = types.ModuleType("zstandard")
  return src


def loaded_shapes(module):
  """The reference's OuterProductMean creates output_w / output_b only when weights are loaded
  (trunk/blocks.py:608-628, set_parameters); give them their loaded shapes so a module built without a
  checkpoint carries every parameter."""
  import torch
  for mod in module.modules():
    if type(mod).__name__.startswith("OuterProductMean") and "output_w" not in mod._parameters:
      outer, dev = tuple(mod.left_projection.output_shape), mod.left_projection.weight.device
      mod.output_w = torch.nn.Parameter(torch.empty(*outer, *outer, mod.num_output_channel, device=dev),
                                        requires_grad=False)
      mod.output_b = torch.nn.Parameter(torch.empty(mod.num_output_channel, device=dev), requires_grad=False)
  return module
