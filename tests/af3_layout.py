"""A checkpoint in the AF3 parameter layout, built from a module's own parameters (test infrastructure).

The AF3 weights are not on this machine, so the loading tests write a synthetic checkpoint the way
the released ones are laid out: one scope per parameterised module, named by the chain of module
names (a name ending in "_" is joined to its children's names without "/", as Haiku does, and
unnamed modules add no level), LayerNorm parameters as "scale" / "offset", Linear parameters as
"weights" / "bias" in the JAX layout (input dims first, the shape the reference keeps), bf16 values.
The reference's own loader (weights/loading.py:145-265) then decides whether the layout is right:
a strict load fails on any missing, unexpected or misshaped entry.
"""
from __future__ import annotations

import torch

_NAMES = {"LayerNorm": {"weight": "scale", "bias": "offset"}}


def checkpoint_from_module(module: torch.nn.Module, dtype=torch.bfloat16) -> dict:
  def walk(mod, prefix: str, out: dict) -> None:
    for _, child in mod.named_children():
      nm = getattr(child, "name", None)
      if nm in ("<none>", ""):
        nm = None
      sep = "" if prefix.endswith("_") else "/"
      walk(child, (prefix + sep + nm) if (nm and prefix) else (nm or prefix), out)
    own = dict(mod.named_parameters(recurse=False))
    if own:
      ren = _NAMES.get(type(mod).__name__, {"weight": "weights", "bias": "bias"})
      out[prefix] = {ren[n]: t.detach().to(dtype).clone() for n, t in own.items()}
  out: dict = {}
  walk(module, getattr(module, "name", ""), out)
  return out
