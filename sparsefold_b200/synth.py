"""Seeded synthetic inputs and random-init AF3-shaped weights.

There are no AF3 checkpoints on this machine, so every parity case and every
benchmark runs on weights drawn from the recipe below.  The recipe is keyed by
parameter *name*, so the reference modules (``sparsefold.model.trunk.blocks``)
and the standalone modules of this package (which keep the same parameter
names, ``sparsefold_b200.layers``) receive bit-identical values.

Recipe (per parameter, own ``torch.Generator`` seeded with crc32(f"{seed}:{name}")):

* Linear weight: N(0, 1) / sqrt(fan_in), fan_in = prod(input_shape)
  (``primitives.Linear`` keeps the input dims first unless ``transpose_weights``,
  primitives.py:251-255).
* Linear bias: 0.1 * N(0, 1).
* LayerNorm scale: 1 + 0.1 * N(0, 1); LayerNorm offset: 0.1 * N(0, 1).
* OuterProductMean ``output_w`` [32, 32, C]: N(0, 1) / sqrt(1024); ``output_b``: 0.1 * N(0, 1).
"""
from __future__ import annotations

import math
import zlib

import torch


def _gen(seed: int, name: str) -> torch.Generator:
  return torch.Generator().manual_seed(zlib.crc32(f"{seed}:{name}".encode()) & 0x7FFFFFFF)


def _is_layernorm(mod) -> bool:
  return hasattr(mod, "normalized_shape") and hasattr(mod, "eps")


def _is_linear(mod) -> bool:
  return hasattr(mod, "input_shape") and hasattr(mod, "output_shape")


def param_value(seed: int, full_name: str, shape, kind: str, fan_in: int = 1) -> torch.Tensor:
  g = _gen(seed, full_name)
  r = torch.randn(tuple(shape), generator=g, dtype=torch.float32)
  if kind == "ln_weight":
    return 1.0 + 0.1 * r
  if kind in ("ln_bias", "bias"):
    return 0.1 * r
  if kind == "weight":
    return r / math.sqrt(max(fan_in, 1))
  raise ValueError(kind)


@torch.no_grad()
def init_params(module: torch.nn.Module, seed: int = 0, prefix: str = "") -> dict[str, torch.Tensor]:
  """Fill every parameter of ``module`` from the recipe; returns {name: value}."""
  values: dict[str, torch.Tensor] = {}
  for mod_name, mod in module.named_modules():
    for pname, p in mod.named_parameters(recurse=False):
      full = f"{prefix}{mod_name}.{pname}" if mod_name else f"{prefix}{pname}"
      if _is_layernorm(mod):
        kind = "ln_weight" if pname == "weight" else "ln_bias"
        fan_in = 1
      elif _is_linear(mod):
        kind = "weight" if pname == "weight" else "bias"
        fan_in = int(math.prod(mod.input_shape))
      elif pname == "output_w":
        kind, fan_in = "weight", int(p.shape[0] * p.shape[1])
      elif pname == "output_b":
        kind, fan_in = "bias", 1
      else:
        raise ValueError(f"no init rule for parameter {full}")
      v = param_value(seed, full, p.shape, kind, fan_in)
      p.data.copy_(v.to(p.dtype))
      values[full] = v
  return values


def pair_inputs(n_token: int, c_z: int = 128, c_s: int = 384, n_real: int | None = None,
                seed: int = 0):
  """z ~ N(0,1) [N,N,c_z], s ~ N(0,1) [N,c_s], mask True for the first n_real tokens."""
  g = torch.Generator().manual_seed(seed)
  z = torch.randn(n_token, n_token, c_z, generator=g)
  s = torch.randn(n_token, c_s, generator=g)
  mask = torch.zeros(n_token, dtype=torch.bool)
  mask[: (n_token if n_real is None else n_real)] = True
  return z, s, mask
