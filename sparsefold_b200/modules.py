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
import weakref

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


def _check_pair(act: torch.Tensor, mask: torch.Tensor, c: int, shard=None) -> None:
  rows = act.shape[1] if shard is None else shard.size()
  if act.ndim != 3 or act.shape[0] != rows or act.shape[2] != c:
    raise ValueError(f"pair activation must be [{'N' if shard is None else 'N/P'}, N, {c}], got {tuple(act.shape)}")
  if mask.shape != (act.shape[1],):
    raise ValueError(f"mask must be [N], got {tuple(mask.shape)}")


def _reference_shard(mod):
  """The row shard of the reference's distributed mode, or None.

  A reference module built with ``distributed=True`` while the reference's
  runtime/dist.py is initialised reads ``dist.current_shard`` (trunk/blocks.py:309-314,
  :499-503); the B200 mixins then run the sharded phase entry points with the same
  partition (``sharding.Shard`` follows the reference's even / ragged rule)."""
  if not getattr(mod, "distributed", False):
    return None
  from sparsefold.runtime import dist as rdist   # only reference-built modules get here
  cs = rdist.current_shard
  if cs is None:
    return None
  from sparsefold_b200 import sharding
  return sharding.Shard(cs.length, rdist.get_world_size(), rdist.get_rank(), even=cs.is_even)


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
    shard = _reference_shard(self)
    _check_pair(act, mask, self.num_channels, shard)
    if shard is not None:   # rows sharded over the ranks (blocks.py:540-556)
      from sparsefold_b200 import sharding
      return sharding.tri_mult(self, act.contiguous(), ops.mask_u8(mask), shard)
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
    shard = _reference_shard(self)
    _check_pair(act, seq_mask, self.num_channels, shard)
    if shard is not None:   # rows sharded over the ranks (blocks.py:309-346)
      from sparsefold_b200 import sharding
      return sharding.tri_attention(self, act.contiguous(), ops.mask_u8(seq_mask), shard)
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


def _pack_adaln(mod: "B200Module", ln, tag: str) -> None:
  """Weights of an AdaptiveLayerNorm (diffusion/transformer.py:27-96) under prefix `tag`."""
  if getattr(ln, "single_cond", False):
    mod._keep(f"{tag}_sc_w", ln.single_cond_layer_norm.weight)
    mod._pack(f"{tag}_scale_w", ln.single_cond_scale.weight.detach().float().T)
    mod._keep(f"{tag}_scale_b", ln.single_cond_scale.bias)
    mod._pack(f"{tag}_bias_w", ln.single_cond_bias.weight.detach().float().T)
  else:
    mod._keep(f"{tag}_ln_w", ln.layer_norm.weight)
    mod._keep(f"{tag}_ln_b", ln.layer_norm.bias)


def _apply_adaln(mod: "B200Module", ln, tag: str, x: torch.Tensor, single_cond) -> torch.Tensor:
  """AdaptiveLayerNorm.forward (transformer.py:80-96) on the C ABI."""
  if not getattr(ln, "single_cond", False):
    return ops.layer_norm(x, mod._kept(f"{tag}_ln_w"), mod._kept(f"{tag}_ln_b"))
  dt = x.dtype
  sc = ops.layer_norm(single_cond.to(dt), mod._kept(f"{tag}_sc_w"), None)
  scale = ops.linear(sc, mod._packed(f"{tag}_scale_w", dt), bias=mod._kept(f"{tag}_scale_b"), post_op="sigmoid")
  bias = ops.linear(sc, mod._packed(f"{tag}_bias_w", dt))
  return ops.adaln(x, scale, bias)


def _pack_zero_init(mod: "B200Module", zi) -> None:
  """AdaptiveZeroInit (transformer.py:99-154): transition2 and, with single_cond, the sigmoid gate."""
  mod._pack("zi_t2", zi.transition2.weight.detach().float().T)
  if getattr(zi, "single_cond", False):
    mod._pack("zi_cond_w", zi.adaptive_zero_cond.weight.detach().float().T)
    mod._keep("zi_cond_b", zi.adaptive_zero_cond.bias)


def _apply_zero_init(mod: "B200Module", zi, u: torch.Tensor, single_cond, residual: torch.Tensor) -> torch.Tensor:
  """residual + AdaptiveZeroInit(u, single_cond)."""
  dt = u.dtype
  if not getattr(zi, "single_cond", False):
    return ops.linear(u, mod._packed("zi_t2", dt), residual=residual)
  v = ops.linear(u, mod._packed("zi_t2", dt))
  cond = ops.linear(single_cond.to(dt), mod._packed("zi_cond_w", dt), bias=mod._kept("zi_cond_b"), post_op="sigmoid")
  return ops.gated_residual(residual, v, cond)


class SelfAttentionB200(B200Module):
  """Diffusion ``SelfAttention`` (transformer.py:234-345), with or without ``single_cond``.

  Used as the Pairformer single attention (blocks.py:724-730, no single_cond)
  and as the diffusion token attention (AdaLN + adaptive-zero output).  q, k,
  v and the gate come from one GEMM whose bias is q's bias; the attention
  kernel applies sigmoid(gate) to its output.
  """

  def prepare_native(self):
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
    _pack_adaln(self, self.layer_norm, "ln")
    _pack_zero_init(self, self.zero_init)
    self._hd = (h, d)
    self._native_prepared = True

  @_require_prepared
  def forward(self, x: torch.Tensor, mask: torch.Tensor, *, pair_logits=None, single_cond=None):
    dt = x.dtype
    h, d = self._hd
    xn = _apply_adaln(self, self.layer_norm, "ln", x, single_cond)
    y = ops.linear(xn, self._packed("qkvg", dt), bias=self._kept("qkvg_bias"))   # [..., N, 4*H*D]
    y = y.view(*x.shape[:-1], 4, h, d)
    q, k, v, g = (y[..., i, :, :] for i in range(4))
    shard = _reference_shard(self)
    if shard is not None:   # keys and values of every rank's rows (diffusion/transformer.py:322-330)
      from sparsefold_b200 import sharding
      yf = sharding.all_gather_rows(y.reshape(y.shape[-4], -1)).view(-1, 4, h, d)
      k, v = yf[:, 1], yf[:, 2]
    o = ops.attention(q, k, v, mask_k=mask, bias=pair_logits, gate=g)
    return _apply_zero_init(self, self.zero_init, o.reshape(*x.shape[:-1], h * d), single_cond, x)


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


class DiffusionTransitionBlockB200(B200Module):
  """Diffusion ``TransitionBlock`` (transformer.py:157-231): AdaLN -> SwiGLU -> adaptive-zero output + residual."""

  def prepare_native(self):
    _pack_adaln(self, self.layer_norm, "ln")
    self._pack("w1", self.transition.weight.detach().float().T)    # [2I, C]; first I rows = swish half
    _pack_zero_init(self, self.zero_init)
    self._native_prepared = True

  @_require_prepared
  def forward(self, x: torch.Tensor, *, single_cond=None):
    xn = _apply_adaln(self, self.layer_norm, "ln", x, single_cond)
    hidden = ops.swiglu(ops.linear(xn, self._packed("w1", x.dtype)))
    return _apply_zero_init(self, self.zero_init, hidden, single_cond, x)


class CrossAttentionB200(B200Module):
  """Diffusion ``CrossAttention`` (transformer.py:480-585): local-window atom attention."""

  def prepare_native(self):
    c = self.q_projection.input_shape[0]
    h, d = self.q_projection.output_shape
    wq = self.q_projection.weight.detach().float().reshape(c, h * d).T
    wg = self.gating_query.weight.detach().float().T
    self._pack("qg", torch.cat([wq, wg], 0))
    bias = torch.zeros(2 * h * d, device=self.q_projection.weight.device)
    bias[: h * d] = self.q_projection.bias.detach().float().reshape(-1)
    self._keep("qg_bias", bias)
    wk = self.k_projection.weight.detach().float().reshape(c, h * d).T
    wv = self.v_projection.weight.detach().float().reshape(c, h * d).T
    self._pack("kv", torch.cat([wk, wv], 0))
    _pack_adaln(self, self.q_layernorm, "lnq")
    _pack_adaln(self, self.k_layernorm, "lnk")
    _pack_zero_init(self, self.zero_init)
    self._hd = (h, d)
    self._native_prepared = True

  @_require_prepared
  def forward(self, x_q, x_k, mask_q, mask_k, pair_logits=None, single_cond_q=None, single_cond_k=None):
    dt = x_q.dtype
    h, d = self._hd
    xq = _apply_adaln(self, self.q_layernorm, "lnq", x_q, single_cond_q)
    xk = _apply_adaln(self, self.k_layernorm, "lnk", x_k.to(dt), single_cond_k)
    qg = ops.linear(xq, self._packed("qg", dt), bias=self._kept("qg_bias")).view(*x_q.shape[:-1], 2, h, d)
    kv = ops.linear(xk, self._packed("kv", dt)).view(*x_k.shape[:-1], 2, h, d)
    o = ops.attention(qg[..., 0, :, :], kv[..., 0, :, :], kv[..., 1, :, :], mask_q=mask_q, mask_k=mask_k,
                      bias=pair_logits, gate=qg[..., 1, :, :])
    return _apply_zero_init(self, self.zero_init, o.reshape(*x_q.shape[:-1], h * d), single_cond_q, x_q)


class DiffusionTransformerB200(B200Module):
  """Diffusion ``Transformer`` (transformer.py:348-477): 24 blocks in super-blocks of 4 with the
  pair-logit pack of every super-block computed once from LN(pair_cond) (transformer.py:429-447)."""

  def prepare_native(self):
    ws = [lin.weight.detach().float() for lin in self.pair_logits_projection]     # each [P, sbs, H]
    p = ws[0].shape[0]
    self._pack("pack_w", torch.cat([w.reshape(p, -1) for w in ws], 1).T)          # [nsb*sbs*H, P]
    self._keep("pair_ln_w", self.pair_input_layer_norm.weight)
    self._shape = (len(ws), ws[0].shape[1], ws[0].shape[2])
    self._pack_memo = None
    self._native_prepared = True

  def pair_logits_pack(self, pair_cond: torch.Tensor, dtype) -> torch.Tensor:
    nsb, sbs, h = self._shape
    n = pair_cond.shape[0]
    x = ops.layer_norm(pair_cond.to(dtype), self._kept("pair_ln_w"), None)
    lg = ops.linear(x, self._packed("pack_w", dtype)).reshape(n * n, nsb * sbs * h)
    out = torch.empty(nsb * sbs * h, n * n, dtype=dtype, device=lg.device)
    ops.transpose_(lg, out, 1, 1, n * n, nsb * sbs * h, 0, 0, nsb * sbs * h, 0, 0, n * n)
    return out.view(nsb, sbs, h, n, n)

  def _pack_of(self, pair_cond: torch.Tensor, dtype) -> torch.Tensor:
    """The pair-logit pack of ``pair_cond``, reused while the same tensor object comes back with
    the same version counter (no in-place change since) and dtype.  The reference's denoising
    loop (generator.py:393-501, _denoising at :338-346) hands every step the same base pair
    conditioning (``torch.asarray`` of a tensor already in the compute dtype returns the tensor
    itself), so through the plugin the pack is computed once per loop, not once per step.  The
    memo is dropped when that tensor is freed and when the weights are prepared again; inference
    tensors keep no version counter and are not memoised.  Under CUDA-graph capture the memo is
    neither used nor filled: the graph must record the pack's own computation, since a replay
    re-reads pair_cond's buffer without running this code."""
    if pair_cond.is_cuda and torch.cuda.is_current_stream_capturing():
      return self.pair_logits_pack(pair_cond, dtype)
    try:
      version = pair_cond._version
    except RuntimeError:
      return self.pair_logits_pack(pair_cond, dtype)
    memo = self._pack_memo
    if memo is not None and memo[0]() is pair_cond and memo[1] == version and memo[2] == dtype:
      return memo[3]
    pack = self.pair_logits_pack(pair_cond, dtype)
    token = object()
    self._pack_memo = (weakref.ref(pair_cond), version, dtype, pack, token)
    weakref.finalize(pair_cond, _forget_pack, weakref.ref(self), token)
    return pack

  @_require_prepared
  def forward(self, act, mask, single_cond, pair_cond=None, *, pair_logits_pack=None):
    """transformer.py:422-477.  ``pair_logits_pack`` (from ``pair_logits_pack(pair_cond)``) lets a
    denoising loop compute the pack once for all its steps, as pair_cond does not change between
    them; without it the pack of an unchanged ``pair_cond`` is reused (``_pack_of``)."""
    nsb, sbs, _ = self._shape
    pack = pair_logits_pack
    if pack is None and pair_cond is not None:
      pack = self._pack_of(pair_cond, act.dtype)
    for sb in range(nsb):
      for s in range(sbs):
        act = self.self_attention[sb][s](act, mask, pair_logits=None if pack is None else pack[sb, s],
                                         single_cond=single_cond)
        act = self.transition_block[sb][s](act, single_cond=single_cond)
    return act


def _forget_pack(module_ref, token) -> None:
  """Drops a diffusion transformer's pack memo once its pair_cond is freed."""
  m = module_ref()
  if m is not None and getattr(m, "_pack_memo", None) is not None and m._pack_memo[4] is token:
    m._pack_memo = None


class CrossAttTransformerB200(B200Module):
  """Diffusion ``CrossAttTransformer`` (transformer.py:588-693): atom-window cross attention blocks."""

  def prepare_native(self):
    w = self.pair_logits_projection.weight.detach().float()                        # [P, blocks, H]
    wt = w.reshape(w.shape[0], -1).T                                               # [blocks * H, P]
    width = (wt.shape[0] + 7) // 8 * 8   # output width padded to 8 so the projection runs on tcgen05
    self._pack("pl_w", torch.cat([wt, wt.new_zeros(width - wt.shape[0], wt.shape[1])], 0))
    self._keep("pair_ln_w", self.pair_input_layer_norm.weight)
    self._bh = (w.shape[1], w.shape[2])
    self._plw = width
    self._native_prepared = True

  @_require_prepared
  def forward(self, queries_act, queries_mask, queries_to_keys, keys_mask, queries_single_cond, keys_single_cond,
              pair_cond):
    nb, h = self._bh
    dt = queries_act.dtype
    s_, q_, k_, _ = pair_cond.shape
    x = ops.layer_norm(pair_cond.to(dt), self._kept("pair_ln_w"), None)
    wd = self._plw
    lg = ops.linear(x, self._packed("pl_w", dt)).reshape(s_ * q_ * k_, wd)      # columns (b, h), padded to wd
    # "s q k b h -> b s h q k" (transformer.py:661)
    pl = torch.empty(nb, s_, h, q_, k_, dtype=dt, device=lg.device)
    qk = q_ * k_
    ops.transpose_(lg, pl, s_, nb, qk, h, qk * wd, h, wd, h * qk, s_ * h * qk, qk)
    idx = queries_to_keys.gather_idxs
    gmask = queries_to_keys.gather_mask
    lead = queries_act.shape[:-3]
    for blk in range(nb):
      src = queries_act.reshape(-1, s_ * q_, queries_act.shape[-1])
      keys = ops.gather_rows(src, idx, gmask).view(*lead, *idx.shape, queries_act.shape[-1])
      queries_act = self.cross_attention[blk](x_q=queries_act, x_k=keys, mask_q=queries_mask, mask_k=keys_mask,
                                              pair_logits=pl[blk], single_cond_q=queries_single_cond,
                                              single_cond_k=keys_single_cond)
      queries_act = self.transition_block[blk](queries_act, single_cond=queries_single_cond)
    return queries_act


class MSAAttentionB200(B200Module):
  """``MSAAttention`` pair-weighted averaging (trunk/blocks.py:99-185).

  weights[h,q,k] = softmax_k(LN(pair) W_h + 1e9 (max_m mask[m,k] - 1));
  v_avg[m,q,h,:] = sum_k weights[h,q,k] v[m,k,h,:] runs as one batched tensor-core
  contraction per head over (m, d) rows; gated by sigmoid(LN(msa) W_g); output projection.
  """

  def prepare_native(self):
    c = self.num_channels
    h, d = self.v_projection.output_shape
    self._pack("logits", self.pair_logits.weight.detach().float().T)                # [H, C2]
    self._pack("v", self.v_projection.weight.detach().float().reshape(c, h * d).T)  # [H*D, C]
    self._pack("gate", self.gating_query.weight.detach().float().T)
    self._pack("out", self.output_projection.weight.detach().float().T)
    self._keep("act_w", self.act_norm.weight)
    self._keep("act_b", self.act_norm.bias)
    self._keep("pair_w", self.pair_norm.weight)
    self._keep("pair_b", self.pair_norm.bias)
    self._hd = (h, d)
    self._native_prepared = True

  @_require_prepared
  def forward(self, act: torch.Tensor, mask: torch.Tensor, pair_act: torch.Tensor):
    dt = act.dtype
    h, d = self._hd
    m_, n_, _ = act.shape
    nq = pair_act.shape[0]
    x = ops.layer_norm(act, self._kept("act_w"), self._kept("act_b"))
    logits = ops.pair_logits(pair_act.to(dt).contiguous(), self._kept("pair_w"), self._kept("pair_b"),
                             self._packed("logits", dt), h)                              # [H, q, k]
    # the reference forms the key bias in bf16 (blocks.py:166-167)
    kbias = (1e9 * (mask.to(torch.bfloat16).amax(0) - 1.0)).float()
    kp = ops.pitch(n_)
    # contraction operands are [row][channel = head][k]: w [q][h][k], vt [(m,d)][h][k]
    wsm = torch.empty(h, nq, n_, dtype=dt, device=act.device)
    ops.softmax_rows(logits.reshape(h * nq, n_), kbias, out=wsm)
    w = torch.zeros(nq, h, kp, dtype=dt, device=act.device)
    ops.transpose_(wsm, w, h, nq, 1, n_, nq * n_, n_, n_, kp, h * kp, 1)           # [h][q][k] -> [q][h][k]
    v = ops.linear(x, self._packed("v", dt))                                         # [M, N, H*D]
    vt = torch.zeros(m_ * d, h, kp, dtype=dt, device=act.device)
    # v[m][k][h][d] -> vt[(m, d)][h][k]
    ops.transpose_(v, vt, m_, h, n_, d, n_ * h * d, d, h * d, d * h * kp, kp, h * kp)
    pavg = ops.contract(vt, w, h, m_ * d, nq, n_)                                    # [(m,d)][h][pitch(q)]
    qp = pavg.shape[-1]
    avg = torch.empty(m_, nq, h * d, dtype=dt, device=act.device)
    # pavg[m][d][h][q] -> avg[m][q][h][d]
    ops.transpose_(pavg, avg, m_, h, d, nq, d * h * qp, qp, h * qp, nq * h * d, d, h * d)
    gate = ops.linear(x, self._packed("gate", dt), post_op="sigmoid")
    return ops.linear(ops.gated_residual(None, avg, gate), self._packed("out", dt))


class OuterProductMeanB200(B200Module):
  """``OuterProductMean`` (trunk/blocks.py:569-689).

  O[(i,a),(j,b)] = sum_m L[m,i,a] R[m,j,b] is one tensor-core GEMM over the MSA
  axis; the 32x32 blocks are regrouped per pair position and projected to the pair
  channels with the bias, then scaled by 1/(1e-3 + sum_m mask[m,i] mask[m,j]).
  """

  def prepare_native(self):
    self._pack("left", self.left_projection.weight.detach().float().T)     # [32, C]
    self._pack("right", self.right_projection.weight.detach().float().T)
    if "output_w" not in self._parameters:
      # the reference creates output_w / output_b when its weights are set (blocks.py:608-628)
      raise RuntimeError(f"{getattr(self, 'name', type(self).__name__)}: output_w / output_b are not loaded; "
                         "load the weights before backends.prepare(model)")
    w = self.output_w.detach().float()                                       # [32, 32, C2]
    self._pack("out", w.reshape(-1, w.shape[-1]).T)                          # [C2, 1024]
    self._keep("out_b", self.output_b)
    self._keep("ln_w", self.layer_norm_input.weight)
    self._keep("ln_b", self.layer_norm_input.bias)
    self._d = w.shape[0]
    self._native_prepared = True

  @_require_prepared
  def forward(self, act: torch.Tensor, mask: torch.Tensor):
    dt = act.dtype
    d = self._d
    m_, n_, _ = act.shape
    x = ops.layer_norm(act, self._kept("ln_w"), self._kept("ln_b"))
    left = ops.mask_rows_(ops.linear(x, self._packed("left", dt)), mask)     # [M, N, 32]
    right = ops.mask_rows_(ops.linear(x, self._packed("right", dt)), mask)
    mp = ops.pitch(m_)
    lt = torch.zeros(n_ * d, mp, dtype=dt, device=act.device)     # [(i,a)][1 channel][m]
    rt = torch.zeros(n_ * d, mp, dtype=dt, device=act.device)
    ops.transpose_(left, lt, 1, 1, m_, n_ * d, 0, 0, n_ * d, 0, 0, mp)        # [M][(i,a)] -> [(i,a)][M]
    ops.transpose_(right, rt, 1, 1, m_, n_ * d, 0, 0, n_ * d, 0, 0, mp)
    o = ops.contract(lt, rt, 1, n_ * d, n_ * d, m_)                           # [1][(i,a)][pitch((j,b))]
    blocks = ops.opm_repack(o.reshape(n_ * d, -1), n_, d)                    # [(i,j)][(a,b)]
    out = ops.linear(blocks, self._packed("out", dt), bias=self._kept("out_b")).view(n_, n_, -1)
    norm = ops.opm_norm(mask, dt)
    return ops.scale_rows_(out, norm.reshape(-1))


# ---------------------------------------------------------------------------
# Embedding-side pair layers (trunk/network.py:195-285, diffusion/generator.py:367-391).
# The Evoformer and the DiffusionHead hold plain primitives (Linear, LayerNorm) for their
# pair-side embeddings; at prepare time those instances take a B200 class of their own
# (``(LinearB200, primitives.Linear)``), so the reference's methods run unchanged and call
# the kernels, and parameters and state_dict keys stay where they were.
# ---------------------------------------------------------------------------
_ADOPTED: dict[tuple[type, type], type] = {}


def _adopt(mod: torch.nn.Module, mixin: type) -> torch.nn.Module:
  """Give one module instance the class (mixin, its class); returns it."""
  if not isinstance(mod, mixin):
    base = type(mod)
    key = (base, mixin)
    if key not in _ADOPTED:
      _ADOPTED[key] = type(base.__name__ + "B200", (mixin, base), {"__module__": __name__})
    mod.__class__ = _ADOPTED[key]
  return mod


class LinearB200(B200Module):
  """``Linear`` (layers/primitives.py:192-365) with one input and one output axis on the C ABI.

  Dense mode: ``sf_linear`` (tcgen05 for bf16 with K, N multiples of 8, CUDA cores otherwise) in the
  activation dtype, or in fp32 where the reference asks ``precision="highest"``; bias, residual and
  post_op in the reference's order (output + bias + residual, then post_op, primitives.py:347-365).
  Sparse mode (``_sf_sparse``, for one-hot or 0/1 inputs): ``sf_pair_sparse_linear`` over the nonzero
  features with the fp32 weight.  The result has the input's dtype, as the reference's.
  """
  _sf_sparse = False

  def prepare_native(self):
    if len(self.input_shape) != 1 or len(self.output_shape) != 1:
      raise ValueError(f"{self.name}: B200 Linear takes one input and one output axis, got "
                       f"{self.input_shape} -> {self.output_shape}")
    w = self.weight.detach().float()
    w_kc = w.T if self.transpose_weights else w                     # [K, C]
    if self._sf_sparse and (self.use_bias or w_kc.shape[1] not in (32, 64, 128, 256)):
      raise ValueError(f"{self.name}: sparse pair linear needs no bias and 32/64/128/256 outputs")
    self._keep("w_kc", w_kc)
    self._pack("wt", w_kc.T)                                        # [C, K] per activation dtype
    if self.use_bias:
      self._keep("bias", self.bias)
    self._native_prepared = True

  @_require_prepared
  def forward(self, inputs: torch.Tensor, *, post_op=None, residual: torch.Tensor | None = None):
    dt = inputs.dtype
    if self._sf_sparse:
      if post_op is not None:
        raise ValueError(f"{self.name}: post_op on a sparse pair linear")
      return ops.pair_sparse_linear(inputs, self._kept("w_kc"), residual)
    cdt = torch.float32 if getattr(self, "precision", None) == "highest" else dt
    bias = self._kept("bias") if self.use_bias else None
    res = None if residual is None else residual.to(cdt)
    return ops.linear(inputs.to(cdt), self._packed("wt", cdt), bias, residual=res, post_op=post_op).to(dt)


class LayerNormB200(B200Module):
  """``LayerNorm`` (layers/primitives.py:368-497) over the last axis on ``sf_layernorm`` (fp32
  statistics, affine parameters in fp32, output in the input's dtype)."""

  def prepare_native(self):
    if len(self.normalized_shape) != 1:
      raise ValueError(f"{self.name}: B200 LayerNorm normalises one axis")
    if self.weight is not None:
      self._keep("w", self.weight)
    if self.bias is not None:
      self._keep("b", self.bias)
    self._native_prepared = True

  @_require_prepared
  def forward(self, input: torch.Tensor) -> torch.Tensor:
    if self.dim not in (-1, input.ndim - 1):
      raise ValueError(f"{self.name}: B200 LayerNorm normalises the last axis only (dim={self.dim})")
    w = self._kept("w") if self.weight is not None else None
    b = self._kept("b") if self.bias is not None else None
    return ops.layer_norm(input, w, b, self.eps)


class EvoformerB200(B200Module):
  """The pair embedding of ``Evoformer`` (trunk/network.py:195-285, :344-376) on the C ABI.

  * ``_get_seq_pair_embedding``: left_single / right_single on ``sf_linear``, then one
    ``sf_pair_outer_sum`` pass for left[:, None] + right[None, :] (network.py:195-212);
  * ``_get_position_feat`` and ``_get_bonds_act`` run the reference's code, whose
    ``position_activations`` (139 one-hot features) and ``bond_embedding`` (one 0/1 feature) are
    sparse B200 Linears (``sf_pair_sparse_linear``);
  * the recycling step prev_embedding(LayerNorm(prev pair), residual=pair) (:369-372) runs on
    ``sf_layernorm`` and ``sf_linear`` with the residual in its epilogue.
  The template, MSA and Pairformer stacks are the reference's, built from the B200 factories.
  """
  _LINEARS = {"left_single": False, "right_single": False, "prev_embedding": False,
              "position_activations": True, "bond_embedding": True}
  _NORMS = ("prev_embedding_layer_norm",)

  def prepare_native(self):
    for name, sparse in self._LINEARS.items():
      sub = _adopt(getattr(self, name), LinearB200)
      sub._sf_sparse = sparse
      sub.prepare_native()
    for name in self._NORMS:
      _adopt(getattr(self, name), LayerNormB200).prepare_native()
    self._native_prepared = True

  @_require_prepared
  def _get_seq_pair_embedding(self, token_features, target_feat: torch.Tensor, target_feat_shard: torch.Tensor):
    left = self.left_single(target_feat_shard)    # (B, C)
    right = self.right_single(target_feat)        # (N, C)
    return ops.pair_outer_sum(left, right)        # (B, N, C)


class DiffusionHeadB200(B200Module):
  """The base conditioning of ``DiffusionHead._get_base_cond`` (diffusion/generator.py:367-391): the
  LayerNorms over [pair embedding | 139 relative features] and [single | target features] on
  ``sf_layernorm`` and the two ``precision="highest"`` projections on ``sf_linear`` in fp32; the
  pair transitions are the B200 diffusion TransitionBlock of the factory swap."""
  _LINEARS = ("pair_cond_initial_projection", "single_cond_initial_projection")
  _NORMS = ("pair_cond_initial_norm", "single_cond_initial_norm")

  def prepare_native(self):
    for name in self._LINEARS:
      _adopt(getattr(self, name), LinearB200).prepare_native()
    for name in self._NORMS:
      _adopt(getattr(self, name), LayerNormB200).prepare_native()
    self._native_prepared = True


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
  """Parameter tree of transformer.AdaptiveLayerNorm (transformer.py:33-75)."""

  def __init__(self, c: int, single_cond_size: int | None = None):
    super().__init__()
    self.single_cond = single_cond_size is not None
    if self.single_cond:
      self.layer_norm = LayerNorm(c, elementwise_affine=False, name="layer_norm")
      self.single_cond_layer_norm = LayerNorm(single_cond_size, bias=False, name="single_cond_layer_norm")
      self.single_cond_scale = Linear(single_cond_size, c, bias=True, name="single_cond_scale")
      self.single_cond_bias = Linear(single_cond_size, c, name="single_cond_bias")
    else:
      self.layer_norm = LayerNorm(c, name="layer_norm")


class _AdaptiveZeroInit(torch.nn.Module):
  """Parameter tree of transformer.AdaptiveZeroInit (transformer.py:102-133)."""

  def __init__(self, hidden: int, c: int, single_cond_size: int | None = None):
    super().__init__()
    self.single_cond = single_cond_size is not None
    self.transition2 = Linear(hidden, c, name="transition2")
    if self.single_cond:
      self.adaptive_zero_cond = Linear(single_cond_size, c, bias=True, name="adaptive_zero_cond")


class SelfAttention(SelfAttentionB200, torch.nn.Module):
  def __init__(self, num_channels: int = 384, num_head: int = 16, name: str = "", single_cond_size: int | None = None):
    torch.nn.Module.__init__(self)
    self.name = name
    c = num_channels
    d = c // num_head
    self.key_dim = self.value_dim = d
    self.layer_norm = _AdaptiveLayerNorm(c, single_cond_size)
    self.q_projection = Linear(c, (num_head, d), bias=True, name="q_projection")
    self.k_projection = Linear(c, (num_head, d), name="k_projection")
    self.v_projection = Linear(c, (num_head, d), name="v_projection")
    self.gating_query = Linear(c, num_head * d, name="gating_query")
    self.zero_init = _AdaptiveZeroInit(c, c, single_cond_size)


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
    # every kernel reads the token mask as bytes: convert once, not once per op
    seq_mask = ops.mask_u8(seq_mask)
    act = self.triangle_multiplication_outgoing(act, seq_mask)
    act = self.triangle_multiplication_incoming(act, seq_mask)
    act = self.pair_attention1(act, seq_mask)
    act = self.pair_attention2(act, seq_mask)
    act = self.pair_transition(act)
    single_act = self.single_act_update(act, single_act, seq_mask)
    return act, single_act


class DiffusionTransitionBlock(DiffusionTransitionBlockB200, torch.nn.Module):
  def __init__(self, num_channels: int, num_intermediate_factor: int = 2, single_cond_size: int | None = None):
    torch.nn.Module.__init__(self)
    c = num_channels
    i = c * num_intermediate_factor
    self.layer_norm = _AdaptiveLayerNorm(c, single_cond_size)
    self.transition = Linear(c, 2 * i, name="ffw_transition1")
    self.zero_init = _AdaptiveZeroInit(i, c, single_cond_size)


class CrossAttention(CrossAttentionB200, torch.nn.Module):
  def __init__(self, num_channels: int = 128, num_head: int = 4, key_dim: int = 128):
    torch.nn.Module.__init__(self)
    c = num_channels
    d = key_dim // num_head
    self.q_layernorm = _AdaptiveLayerNorm(c, c)
    self.k_layernorm = _AdaptiveLayerNorm(c, c)
    self.q_projection = Linear(c, (num_head, d), bias=True, name="q_projection")
    self.k_projection = Linear(c, (num_head, d), name="k_projection")
    self.v_projection = Linear(c, (num_head, d), name="v_projection")
    self.gating_query = Linear(c, num_head * d, name="gating_query")
    self.zero_init = _AdaptiveZeroInit(c, c, c)


class DiffusionTransformer(DiffusionTransformerB200, torch.nn.Module):
  def __init__(self, num_channels: int = 768, single_cond_size: int = 384, pair_cond_size: int = 128,
               num_head: int = 16, num_blocks: int = 24, super_block_size: int = 4, num_intermediate_factor: int = 2):
    torch.nn.Module.__init__(self)
    nsb = num_blocks // super_block_size
    mk = lambda f: torch.nn.ModuleList(torch.nn.ModuleList(f() for _ in range(super_block_size)) for _ in range(nsb))
    self.self_attention = mk(lambda: SelfAttention(num_channels, num_head, single_cond_size=single_cond_size))
    self.transition_block = mk(lambda: DiffusionTransitionBlock(num_channels, num_intermediate_factor, single_cond_size))
    self.pair_logits_projection = torch.nn.ModuleList(
        Linear(pair_cond_size, (super_block_size, num_head), name="pair_logits_projection") for _ in range(nsb))
    self.pair_input_layer_norm = LayerNorm(pair_cond_size, bias=False, name="pair_input_layer_norm")


class CrossAttTransformer(CrossAttTransformerB200, torch.nn.Module):
  def __init__(self, num_channels: int = 128, pair_cond_size: int = 16, num_head: int = 4, key_dim: int = 128,
               num_blocks: int = 3, num_intermediate_factor: int = 2):
    torch.nn.Module.__init__(self)
    self.pair_input_layer_norm = LayerNorm(pair_cond_size, bias=False, name="pair_input_layer_norm")
    self.pair_logits_projection = Linear(pair_cond_size, (num_blocks, num_head), name="pair_logits_projection")
    self.cross_attention = torch.nn.ModuleList(CrossAttention(num_channels, num_head, key_dim) for _ in range(num_blocks))
    self.transition_block = torch.nn.ModuleList(
        DiffusionTransitionBlock(num_channels, num_intermediate_factor, num_channels) for _ in range(num_blocks))


class MSAAttention(MSAAttentionB200, torch.nn.Module):
  def __init__(self, num_channels: int = 64, num_output_channel: int = 128, num_head: int = 8):
    torch.nn.Module.__init__(self)
    self.num_channels = c = num_channels
    self.num_output_channel = c2 = num_output_channel
    d = c // num_head
    self.act_norm = LayerNorm(c, name="act_norm")
    self.pair_norm = LayerNorm(c2, name="pair_norm")
    self.pair_logits = Linear(c2, num_head, name="pair_logits")
    self.v_projection = Linear(c, (num_head, d), name="v_projection")
    self.gating_query = Linear(c, num_head * d, name="gating_query")
    self.output_projection = Linear(num_head * d, c, name="output_projection")


class OuterProductMean(OuterProductMeanB200, torch.nn.Module):
  def __init__(self, num_channels: int = 64, num_output_channel: int = 128, num_outer_channel: int = 32):
    torch.nn.Module.__init__(self)
    self.num_channels = num_channels
    self.num_output_channel = num_output_channel
    self.layer_norm_input = LayerNorm(num_channels, name="layer_norm_input")
    self.left_projection = Linear(num_channels, num_outer_channel, name="left_projection")
    self.right_projection = Linear(num_channels, num_outer_channel, name="right_projection")
    self.output_w = torch.nn.Parameter(torch.empty(num_outer_channel, num_outer_channel, num_output_channel),
                                       requires_grad=False)
    self.output_b = torch.nn.Parameter(torch.empty(num_output_channel), requires_grad=False)


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
    seq_mask = ops.mask_u8(seq_mask)
    for blk in self.blocks:
      pair, single = blk(pair, seq_mask=seq_mask, single_act=single)
    return pair, single
