"""Parameter holders with the reference's shapes and names.

``Linear`` and ``LayerNorm`` mirror the parameter layout of
``model/layers/primitives.py`` (Linear: primitives.py:192-280, weight
``input_shape + output_shape`` or, with ``transpose_weights``,
``output_shape + input_shape``; LayerNorm: primitives.py:382-421).  They hold
parameters only: the B200 modules read them in ``prepare_native`` and never
run them on the host.  With these, the standalone modules of
``sparsefold_b200.modules`` have exactly the reference ``state_dict`` keys.
"""
from __future__ import annotations

import numbers

import torch


def _shape(v) -> tuple:
  return (int(v),) if isinstance(v, numbers.Integral) else tuple(int(x) for x in v)


class Linear(torch.nn.Module):
  def __init__(self, num_input, num_output, *, bias: bool = False, transpose_weights: bool = False,
               name: str | None = None):
    super().__init__()
    self.name = name
    self.input_shape = _shape(num_input)
    self.output_shape = _shape(num_output)
    self.transpose_weights = transpose_weights
    self.use_bias = bias
    shape = self.output_shape + self.input_shape if transpose_weights else self.input_shape + self.output_shape
    self.weight = torch.nn.Parameter(torch.empty(shape), requires_grad=False)
    if bias:
      self.bias = torch.nn.Parameter(torch.empty(self.output_shape), requires_grad=False)
    else:
      self.register_parameter("bias", None)

  def forward(self, *args, **kwargs):
    raise RuntimeError("parameter holder: B200 modules never run Linear on the host")


class LayerNorm(torch.nn.Module):
  def __init__(self, normalized_shape: int, *, eps: float = 1e-5, elementwise_affine: bool = True,
               dim: int = -1, bias: bool = True, name: str | None = None):
    super().__init__()
    self.name = name
    self.normalized_shape = _shape(normalized_shape)
    self.eps = eps
    self.dim = dim
    self.elementwise_affine = elementwise_affine
    if elementwise_affine:
      self.weight = torch.nn.Parameter(torch.empty(self.normalized_shape), requires_grad=False)
      if bias:
        self.bias = torch.nn.Parameter(torch.empty(self.normalized_shape), requires_grad=False)
      else:
        self.register_parameter("bias", None)
    else:
      self.register_parameter("weight", None)
      self.register_parameter("bias", None)

  def forward(self, *args, **kwargs):
    raise RuntimeError("parameter holder: B200 modules never run LayerNorm on the host")
