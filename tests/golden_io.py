"""Load the committed golden fixtures and regenerate their weights from the recipe."""
import json
import os

import numpy as np
import torch

from sparsefold_b200 import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
  data = np.load(os.path.join(GOLDEN, f"{name}.npz"))
  meta = json.loads(str(data["meta"]))
  arrays = {k: torch.from_numpy(np.array(data[k])) for k in data.files if k != "meta"}
  params = {full: synth.param_value(meta["seed"], full, shape, kind, fan)
            for full, shape, kind, fan in meta["params"]}
  return arrays, params


def max_rel_err(y, ref):
  """max|y - ref| / max|ref| over the whole tensor (the per-op tolerance metric)."""
  y = y.double()
  ref = ref.double()
  return float((y - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


def cosine(a, b):
  a = a.double().flatten()
  b = b.double().flatten()
  return float((a @ b) / (a.norm() * b.norm()).clamp_min(1e-300))
