"""CUDA-graph replay of a fixed-shape call, for loops that repeat one step many times.

The diffusion sampler calls the token transformer once per denoising step with
the same shapes every time (model/diffusion/generator.py:393-501: 200 steps of
24 blocks each).  Launching its ~400 kernels from Python every step costs host
time that a step of a few milliseconds cannot hide; ``GraphedCall`` captures the
call once into a CUDA graph on static input buffers and replays it, so a step
costs one graph launch.  The library's entry points only enqueue work on the
current stream (their one-time set-up runs in the warm-up calls before
capture), so they record into a graph like any other kernel launch.
"""
from __future__ import annotations

import torch


class GraphedCall:
  """``fn(*inputs)`` captured once; calling the object copies new inputs into the captured
  buffers and replays the graph.  The returned tensor is the graph's static output: it is
  overwritten by the next replay (clone it to keep it)."""

  def __init__(self, fn, *example_inputs: torch.Tensor, warmup: int = 2):
    self._fn = fn
    self._static_in = [t.clone() for t in example_inputs]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
      for _ in range(warmup):   # one-time set-up (kernel attributes, tensor-map encoders) outside capture
        fn(*self._static_in)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    self._graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(self._graph):
      self._static_out = fn(*self._static_in)

  def __call__(self, *inputs: torch.Tensor) -> torch.Tensor:
    for dst, src in zip(self._static_in, inputs):
      if src.data_ptr() != dst.data_ptr():
        dst.copy_(src)
    self._graph.replay()
    return self._static_out
