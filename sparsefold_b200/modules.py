"""B200 module mixins and standalone modules of the Pairformer hot path.

Each ``*B200`` mixin supplies ``prepare_native()`` (packs the reference
parameters into non-persistent device buffers, never new Parameters) and a
``forward`` that calls the C ABI through ``sparsefold_b200.ops``.  The mixins
read parameters by the reference attribute names only, so they combine with

* the reference classes (``backend.apply`` builds ``type(name, (Mixin, RefClass), {})``
  and patches the factories, the pattern of vecops/backend.py:187-223), or
* the parameter holders of ``sparsefold_b200.layers`` (the standalone classes
  at the end of this file, used by the tests and ``bench.py``).

Calling ``forward`` before ``prepare_native`` raises, as the reference native
modules do (backends/vecops/modules.py:88-94).
"""
from __future__ import annotations

import functools

import torch

from sparsefold_b200 import ops

_DTYPES = (torch.float32, torch.bfloat16)


def _set_buffer(module: torch.nn.Module, name: str, value: torch.Tensor) -> None:
  value = value.detach().contiguous()
  if name in module._buffers:
    module._buffers[name] = value
  else:
    module.register_buffer(name, value, persistent=False)


def _tag(dtype: torch.dtype) -> str:
  return "f32" if dtype == torch.float32 else "bf16"


def _require_prepared(fn):
  @functools.wraps(fn)
  def wrapped(self, *args, **kwargs):
    if not getattr(self, "_native_prepared", False):
      raise RuntimeError("Native buffers are not prepared; call backends.prepare(model) after weight loading")
    dev = args[0].device if args and isinstance(args[0], torch.Tensor) else None
    for name, buf in self._buffers.items():
      if dev is not None and name.startswith("_sf_") and buf.device != dev:
        raise RuntimeError(f"prepared buffer {name} is on {buf.device}, activation on {dev}; "
                           "move the module before or after prepare, consistently")
    return fn(self, *args, **kwargs)
  return wrapped


def _f32(t):
  return None if t is None else t.detach().to(torch.float32).contiguous()


class B200Module:
  """Common helpers: per-dtype weight packs stored as non-persistent buffers."""

  def _pack(self, name: str, value: torch.Tensor) -> None:
    for dt in _DTYPES:
      _set_buffer(self, f"_sf_{name}_{_tag(dt)}", value.detach().to(dt))

  def _packed(self, name: str, dtype: torch.dtype) -> torch.Tensor:
    return self._buffers[f"_sf_{name}_{_tag(dtype)}"]

  def _keep(self, name: str, value: torch.Tensor) -> None:
    _set_buffer(self, f"_sf_{name}", _f32(value))

  def _kept(self, name: str) -> torch.Tensor:
    return self._buffers[f"_sf_{name}"]


def _check_pair(act: torch.Tensor, mask: torch.Tensor, c: int) -> None:
  if act.ndim != 3 or act.shape[0] != act.shape[1] or act.shape[2] != c:
    raise ValueError(f"pair activation must be [N, N, {c}] on one device, got {tuple(act.shape)}")
  if mask.shape != (act.shape[0],):
    raise ValueError(f"mask must be [N], got {tuple(mask.shape)}")


# ---------------------------------------------------------------------------
class TriangleMultiplicationB200(B200Module):
  """``TriangleMultiplication`` (blocks.py:425-566) on the C ABI.

  Packing: the GLU weight stack (gate, projection) of blocks.py:513-517 is
  split into a-channels (reference channel 2c) and b-channels (2c+1),
  blocks.py:538, as rows [gate_a; value_a; gate_b; value_b] of ``w_glu``.
  """

  def prepare_native(self):
    c = self.num_channels
    wg = self.gate_projection.weight.detach().float()   # [C, 2C] (x @ W)
    wp = self.projection.weight.detach().float()
    glu = torch.cat([wg[:, 0::2].T, wp[:, 0::2].T, wg[:, 1::2].T, wp[:, 1::2].T], 0)
    assert glu.shape == (4 * c, c)
    self._pack("glu", glu)
    self._pack("out", self.output_projection.weight.detach().float().T)
    self._pack("gate", self.gating_linear.weight.detach().float().T)
    self._keep("ln_w", self.left_norm_input.weight)
    self._keep("ln_b", self.left_norm_input.bias)
    self._keep("center_w", self.center_norm.weight)
    self._keep("center_b", self.center_norm.bias)
    self._native_prepared = True

  @property
  def incoming(self) -> bool:
    return self.equation == "...ckj,...cki->...cij"

  def native_weights(self, dtype):
    return ops.tri_mult_weights(self._packed("glu", dtype), self._kept("ln_w"), self._kept("ln_b"),
                                self._kept("center_w"), self._kept("center_b"),
                                self._packed("out", dtype), self._packed("gate", dtype))

  @_require_prepared
  def forward(self, act: torch.Tensor, mask: torch.Tensor):
    _check_pair(act, mask, self.num_channels)
    w = self.native_weights(act.dtype)
    return ops.tri_mult(act.contiguous(), ops.mask_u8(mask), w, self.incoming)


class GridSelfAttentionB200(B200Module):
  """``GridSelfAttention`` (blocks.py:188-366) on the C ABI.

  Packing: q/k (H, D, C) with transpose_weights -> rows (h, d); v (C, H, D)
  -> transposed; gating_query (H*D, C) as is; rows stacked [q; k; v; g].
  """

  def prepare_native(self):
    c = self.num_channels
    h = self.config.num_head if hasattr(self, "config") else self.num_head
    d = self.qkv_dim
    if h * d != c:
      raise ValueError("B200 GridSelfAttention needs num_head * head_dim == num_channels")
    wq = self.q_projection.weight.detach().float().reshape(h * d, c)
    wk = self.k_projection.weight.detach().float().reshape(h * d, c)
    wv = self.v_projection.weight.detach().float().reshape(c, h * d).T
    wg = self.gating_query.weight.detach().float()
    self._pack("qkvg", torch.cat([wq, wk, wv, wg], 0))
    self._pack("bias", self.pair_bias_projection.weight.detach().float().T)   # [H, C]
    self._pack("out", self.output_projection.weight.detach().float().T)       # [C, H*D]
    self._keep("ln_w", self.act_norm.weight)
    self._heads = h
    self._native_prepared = True

  def native_weights(self, dtype):
    return ops.tri_attention_weights(self._kept("ln_w"), self._packed("qkvg", dtype),
                                     self._packed("bias", dtype), self._packed("out", dtype), self._heads)

  @_require_prepared
  def forward(self, act: torch.Tensor, seq_mask: torch.Tensor):
    _check_pair(act, seq_mask, self.num_channels)
    w = self.native_weights(act.dtype)
    return ops.tri_attention(act.contiguous(), ops.mask_u8(seq_mask), w, bool(self.transpose))


class TransitionBlockB200(B200Module):
  """``TransitionBlock`` (blocks.py:38-96): LN -> SwiGLU -> down projection + residual."""

  def prepare_native(self):
    self._pack("w1", self.transition1.weight.detach().float().T)   # [2I, C]
    self._pack("w2", self.transition2.weight.detach().float().T)   # [C, I]
    self._keep("ln_w", self.input_layer_norm.weight)
    self._keep("ln_b", self.input_layer_norm.bias)
    self._native_prepared = True

  @_require_prepared
  def forward(self, act: torch.Tensor, *, broadcast_dim: int | None = 0):
    dt = act.dtype
    return ops.transition(act.contiguous(), self._kept("ln_w"), self._kept("ln_b"),
                          self._packed("w1", dt), self._packed("w2", dt))


class SelfAttentionB200(B200Module):
  """Diffusion ``SelfAttention`` without ``single_cond`` (transformer.py:234-345).

  This is the Pairformer single attention (blocks.py:724-730).  q, k, v and the
  gate come from one GEMM whose bias is q's bias (zeros elsewhere); the
  attention kernel applies sigmoid(gate); ``zero_init.transition2`` adds the
  residual in its epilogue.
  """

  def prepare_native(self):
    if getattr(self.layer_norm, "single_cond", False):
      raise NotImplementedError("B200 SelfAttention with single_cond is not implemented yet")
    c = self.q_projection.input_shape[0]
    h, d = self.q_projection.output_shape
    wq = self.q_projection.weight.detach().float().reshape(c, h * d).T
    wk = self.k_projection.weight.detach().float().reshape(c, h * d).T
    wv = self.v_projection.weight.detach().float().reshape(c, h * d).T
    wg = self.gating_query.weight.detach().float().T
    self._pack("qkvg", torch.cat([wq, wk, wv, wg], 0))
    bias = torch.zeros(4 * h * d, device=self.q_projection.weight.device)
    bias[: h * d] = self.q_projection.bias.detach().float().reshape(-1)
    self._keep("qkvg_bias", bias)
    self._pack("out", self.zero_init.transition2.weight.detach().float().T)
    self._keep("ln_w", self.layer_norm.layer_norm.weight)
    self._keep("ln_b", self.layer_norm.layer_norm.bias)
    self._hd = (h, d)
    self._native_prepared = True

  @_require_prepared
  def forward(self, x: torch.Tensor, mask: torch.Tensor, *, pair_logits=None, single_cond=None):
    if single_cond is not None:
      raise NotImplementedError("B200 SelfAttention with single_cond is not implemented yet")
    dt = x.dtype
    h, d = self._hd
    n = x.shape[-2]
    xn = ops.layer_norm(x, self._kept("ln_w"), self._kept("ln_b"))
    y = ops.linear(xn, self._packed("qkvg", dt), bias=self._kept("qkvg_bias"))   # [..., N, 4*H*D]
    y = y.view(*x.shape[:-1], 4, h, d)
    q, k, v, g = (y[..., i, :, :] for i in range(4))
    o = ops.attention(q, k, v, mask_k=mask, bias=pair_logits, gate=g)
    return ops.linear(o.reshape(*x.shape[:-1], h * d), self._packed("out", dt), residual=x)


class SingleActUpdateB200(B200Module):
  """``SingleActUpdate`` (blocks.py:692-763): pair logits, single attention, transition."""

  def prepare_native(self):
    self._pack("logits", self.single_pair_logits_projection.weight.detach().float().T)   # [H, C]
    self._keep("ln_w", self.single_pair_logits_norm.weight)
    self._keep("ln_b", self.single_pair_logits_norm.bias)
    self._native_prepared = True

  @_require_prepared
  def forward(self, pair_act: torch.Tensor, single_act: torch.Tensor, seq_mask: torch.Tensor):
    dt = pair_act.dtype
    heads = self.single_pair_logits_projection.output_shape[0]
    logits = ops.pair_logits(pair_act.contiguous(), self._kept("ln_w"), self._kept("ln_b"),
                             self._packed("logits", dt), heads)
    single_act = self.single_attention(single_act, seq_mask, pair_logits=logits)
    return self.single_transition(single_act, broadcast_dim=None)


# ---------------------------------------------------------------------------
# Standalone modules: the reference module trees (same attribute names, shapes
# and state_dict keys) built from the parameter holders of layers.py.
# ---------------------------------------------------------------------------
from sparsefold_b200.layers import LayerNorm, Linear  # noqa: E402

_EQUATIONS = {
    "...ikc,...jkc->...ijc": "...cik,...cjk->...cij",   # outgoing (blocks.py:447-450)
    "...kjc,...kic->...ijc": "...ckj,...cki->...cij",   # incoming
}


class TriangleMultiplication(TriangleMultiplicationB200, torch.nn.Module):
  def __init__(self, num_channels: int = 128, equation: str = "...ikc,...jkc->...ijc", name: str = ""):
    torch.nn.Module.__init__(self)
    self.name = name
    self.num_channels = c = num_channels
    self.equation = _EQUATIONS[equation]
    self.left_norm_input = LayerNorm(c, bias=True, name="left_norm_input")
    self.projection = Linear(c, 2 * c, name="projection")
    self.gate_projection = Linear(c, 2 * c, name="gate")
    self.center_norm = LayerNorm(c, bias=True, dim=-3, name="center_norm")
    self.output_projection = Linear(c, c, name="output_projection")
    self.gating_linear = Linear(c, c, name="gating_linear")


class GridSelfAttention(GridSelfAttentionB200, torch.nn.Module):
  def __init__(self, num_channels: int = 128, num_head: int = 4, transpose: bool = False, name: str = ""):
    torch.nn.Module.__init__(self)
    self.name = name
    self.num_channels = c = num_channels
    self.num_head = num_head
    self.transpose = transpose
    self.qkv_dim = d = max(c // num_head, 16)
    self.q_projection = Linear(c, (num_head, d), transpose_weights=True, name="q_projection")
    self.k_projection = Linear(c, (num_head, d), transpose_weights=True, name="k_projection")
    self.v_projection = Linear(c, (num_head, d), name="v_projection")
    self.gating_query = Linear(c, num_head * d, transpose_weights=True, name="gating_query")
    self.output_projection = Linear(num_head * d, c, name="output_projection")
    self.act_norm = LayerNorm(c, bias=False, name="act_norm")
    self.pair_bias_projection = Linear(c, num_head, name="pair_bias_projection")


class TransitionBlock(TransitionBlockB200, torch.nn.Module):
  def __init__(self, num_channels: int = 128, num_intermediate_factor: int = 4, name: str = ""):
    torch.nn.Module.__init__(self)
    self.name = name
    self.num_channels = c = num_channels
    self.num_intermediate = i = c * num_intermediate_factor
    self.input_layer_norm = LayerNorm(c, name="input_layer_norm")
    self.transition1 = Linear(c, 2 * i, name="transition1")
    self.transition2 = Linear(i, c, name="transition2")


class _AdaptiveLayerNorm(torch.nn.Module):
  """Parameter tree of transformer.AdaptiveLayerNorm with single_cond=None (transformer.py:70-75)."""

  def __init__(self, c: int):
    super().__init__()
    self.single_cond = False
    self.layer_norm = LayerNorm(c, name="layer_norm")


class _AdaptiveZeroInit(torch.nn.Module):
  """Parameter tree of transformer.AdaptiveZeroInit with single_cond=None (transformer.py:128-133)."""

  def __init__(self, hidden: int, c: int):
    super().__init__()
    self.single_cond = False
    self.transition2 = Linear(hidden, c, name="transition2")


class SelfAttention(SelfAttentionB200, torch.nn.Module):
  def __init__(self, num_channels: int = 384, num_head: int = 16, name: str = ""):
    torch.nn.Module.__init__(self)
    self.name = name
    c = num_channels
    d = c // num_head
    self.key_dim = self.value_dim = d
    self.layer_norm = _AdaptiveLayerNorm(c)
    self.q_projection = Linear(c, (num_head, d), bias=True, name="q_projection")
    self.k_projection = Linear(c, (num_head, d), name="k_projection")
    self.v_projection = Linear(c, (num_head, d), name="v_projection")
    self.gating_query = Linear(c, num_head * d, name="gating_query")
    self.zero_init = _AdaptiveZeroInit(c, c)


class SingleActUpdate(SingleActUpdateB200, torch.nn.Module):
  def __init__(self, num_channels: int = 128, seq_channels: int = 384, num_head: int = 16,
               num_intermediate_factor: int = 4):
    torch.nn.Module.__init__(self)
    self.name = "<none>"
    self.num_channels = num_channels
    self.seq_channels = seq_channels
    self.num_head = num_head
    self.single_pair_logits_norm = LayerNorm(num_channels, name="single_pair_logits_norm")
    self.single_pair_logits_projection = Linear(num_channels, num_head, name="single_pair_logits_projection")
    self.single_attention = SelfAttention(seq_channels, num_head, name="single_attention_")
    self.single_transition = TransitionBlock(seq_channels, num_intermediate_factor, name="single_transition")


class PairFormerIteration(torch.nn.Module):
  """``PairFormerIteration`` (blocks.py:766-910) with with_single=True.

  The composition is the reference's own (blocks.py:883-908); every sub-module
  is a B200 module.  Its forward is what the reference runs once the factories
  are replaced, so this class is only the standalone container.
  """

  def __init__(self, num_channels: int = 128, seq_channels: int = 384):
    super().__init__()
    self.name = "pairformer_stack"
    c = num_channels
    self.triangle_multiplication_outgoing = TriangleMultiplication(c, "...ikc,...jkc->...ijc")
    self.triangle_multiplication_incoming = TriangleMultiplication(c, "...kjc,...kic->...ijc")
    self.pair_attention1 = GridSelfAttention(c, 4, transpose=False)
    self.pair_attention2 = GridSelfAttention(c, 4, transpose=True)
    self.pair_transition = TransitionBlock(c, 4)
    self.single_act_update = SingleActUpdate(c, seq_channels)

  def forward(self, act, *, seq_mask, single_act=None):
    act = self.triangle_multiplication_outgoing(act, seq_mask)
    act = self.triangle_multiplication_incoming(act, seq_mask)
    act = self.pair_attention1(act, seq_mask)
    act = self.pair_attention2(act, seq_mask)
    act = self.pair_transition(act)
    single_act = self.single_act_update(act, single_act, seq_mask)
    return act, single_act


def prepare(module: torch.nn.Module) -> dict[str, int]:
  """Call ``prepare_native`` on every B200 module (the backend ``prepare`` hook)."""
  counts = {"packed": 0, "fallback": 0, "opaque": 0}
  for m in module.modules():
    if isinstance(m, B200Module):
      m.prepare_native()
      counts["opaque"] += 1
  return counts


class PairformerTrunk(torch.nn.Module):
  """48 ``PairFormerIteration`` blocks applied in order, as ``Evoformer.forward``
  runs ``layer_stack(pairformer_fn)`` (trunk/network.py:400-413)."""

  def __init__(self, num_layers: int = 48, num_channels: int = 128, seq_channels: int = 384):
    super().__init__()
    self.blocks = torch.nn.ModuleList(PairFormerIteration(num_channels, seq_channels) for _ in range(num_layers))

  def forward(self, pair, single, seq_mask):
    for blk in self.blocks:
      pair, single = blk(pair, seq_mask=seq_mask, single_act=single)
    return pair, single
