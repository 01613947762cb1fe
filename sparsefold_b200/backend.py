"""The ``b200`` backend for SparseFold's plugin API (backends/__init__.py:25-137).

Registration, as a user of the reference does it::

    import sparsefold_b200.backend as b200
    b200.register()                                   # backends.register_library(apply, "b200", hooks)
    config.configure_runtime(backend="b200", device="cuda")
    backends.init()                                   # runs apply(): factory replacement
    model = ...construct...; load weights
    backends.prepare(model)                           # prepare_native() on every B200 module

``apply`` replaces the module factories exactly as vecops/backend.py:187-223
does, with classes built as ``(Mixin, ReferenceClass)`` so the reference
``__init__`` and parameter layout stay untouched (state_dict keys unchanged,
tests/test_native_preparation.py:107-132).
"""
from __future__ import annotations

from contextlib import nullcontext

import torch

from sparsefold_b200 import modules as _m

_PATCHED: list[tuple[object, str, object]] = []
_MADE: dict[str, type] = {}


def _native_class(ref_cls: type, mixin: type) -> type:
  key = f"{ref_cls.__module__}.{ref_cls.__qualname__}"
  if key not in _MADE:
    _MADE[key] = type(ref_cls.__name__ + "B200", (mixin, ref_cls), {"__module__": __name__})
  return _MADE[key]


def replacement_map():
  """(module, attribute, replacement) for each reference factory this backend replaces."""
  from sparsefold.model.trunk import blocks
  from sparsefold.model.diffusion import transformer
  orig = {name: getattr(blocks, name) for name in ("GridSelfAttention", "TriangleMultiplication",
                                                     "TransitionBlock", "SingleActUpdate")}
  for name, cls in list(orig.items()):
    if issubclass(cls, _m.B200Module):   # already applied: recover the reference base
      orig[name] = next(b for b in cls.__mro__[1:] if not issubclass(b, _m.B200Module))
  for name in ("MSAAttention", "OuterProductMean"):
    orig[name] = _reference_base(getattr(blocks, name))
  diff = {name: _reference_base(getattr(transformer, name))
          for name in ("SelfAttention", "TransitionBlock", "CrossAttention", "Transformer", "CrossAttTransformer")}
  from sparsefold.model.trunk import network
  from sparsefold.model.diffusion import generator
  evoformer = _reference_base(network.Evoformer)
  head = _reference_base(generator.DiffusionHead)
  return [
      (blocks, "GridSelfAttention", _native_class(orig["GridSelfAttention"], _m.GridSelfAttentionB200)),
      (blocks, "TriangleMultiplication", _native_class(orig["TriangleMultiplication"], _m.TriangleMultiplicationB200)),
      (blocks, "TransitionBlock", _native_class(orig["TransitionBlock"], _m.TransitionBlockB200)),
      (blocks, "SingleActUpdate", _native_class(orig["SingleActUpdate"], _m.SingleActUpdateB200)),
      (blocks, "MSAAttention", _native_class(orig["MSAAttention"], _m.MSAAttentionB200)),
      (blocks, "OuterProductMean", _native_class(orig["OuterProductMean"], _m.OuterProductMeanB200)),
      (transformer, "SelfAttention", _native_class(diff["SelfAttention"], _m.SelfAttentionB200)),
      (transformer, "TransitionBlock", _native_class(diff["TransitionBlock"], _m.DiffusionTransitionBlockB200)),
      (transformer, "CrossAttention", _native_class(diff["CrossAttention"], _m.CrossAttentionB200)),
      (transformer, "Transformer", _native_class(diff["Transformer"], _m.DiffusionTransformerB200)),
      (transformer, "CrossAttTransformer", _native_class(diff["CrossAttTransformer"], _m.CrossAttTransformerB200)),
      (network, "Evoformer", _native_class(evoformer, _m.EvoformerB200)),
      (generator, "DiffusionHead", _native_class(head, _m.DiffusionHeadB200)),
  ]


def _reference_base(cls: type) -> type:
  """The reference class behind an already applied B200 class (apply() is idempotent)."""
  if issubclass(cls, _m.B200Module):
    return next(b for b in cls.__mro__[1:] if not issubclass(b, _m.B200Module))
  return cls


def apply() -> None:
  """Swap the reference factories for B200 classes (construct models afterwards)."""
  for module, name, repl in replacement_map():
    current = getattr(module, name)
    if current is repl:
      continue
    _PATCHED.append((module, name, current))
    setattr(module, name, repl)


def unapply() -> None:
  for module, name, original in reversed(_PATCHED):
    setattr(module, name, original)
  _PATCHED.clear()


def manual_seed(seed: int) -> None:
  torch.manual_seed(seed)


def prepare(module: torch.nn.Module) -> dict[str, int]:
  return _m.prepare(module)


def load_and_prepare(module: torch.nn.Module, checkpoint, *, strict: bool = True):
  """Load AF3 parameters with the reference's own loader, then pack them for the kernels.

  ``checkpoint`` is what ``sparsefold.weights.load_checkpoint`` takes (weights/loading.py:145):
  a ``Checkpoint`` read from disk or the nested ``{scope: {name: tensor}}`` mapping of the AF3
  parameter layout (bf16 in the released weights).  The reference assigns the tensors to the
  module's parameters (state_dict keys and shapes unchanged by the b200 factories), and
  ``prepare`` then packs the weight matrices as bf16 (and fp32) "out x in" buffers and keeps the
  LayerNorm parameters and biases in fp32.  Returns the loader's report."""
  from sparsefold.weights import load_checkpoint
  report = load_checkpoint(module, checkpoint, strict=strict)
  _m.prepare(module)
  return report


def materialize(*, parallelism: int | None = None) -> int:
  return 0


def precompile(module, *args, **kwargs):
  return None


def is_precompiling() -> bool:
  return False


def execution_context():
  return nullcontext()


HOOKS = {"manual_seed": manual_seed, "prepare": prepare, "precompile": precompile,
         "materialize": materialize, "is_precompiling": is_precompiling,
         "execution_context": execution_context}


def register(name: str = "b200") -> None:
  """``backends.register_library(apply, name, hooks)`` on the reference package."""
  from sparsefold import backends
  if name not in backends._registered_impl:
    backends.register_library(apply, name, dict(HOOKS))
