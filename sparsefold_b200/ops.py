"""Torch-facing wrappers of the C ABI: tensors in, tensors out, current stream.

Each wrapper validates shapes/dtypes, allocates outputs and workspace with the
torch caching allocator, and calls one entry point of libsparsefold_b200.so.
Nothing here computes on the host; a missing library raises NativeError.
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from sparsefold_b200 import _native as N


def _dt(t: torch.Tensor) -> int:
  if t.dtype == torch.float32:
    return N.SF_F32
  if t.dtype == torch.bfloat16:
    return N.SF_BF16
  raise TypeError(f"unsupported dtype {t.dtype}; use float32 or bfloat16")


def _stream() -> int:
  return torch.cuda.current_stream().cuda_stream


def _p(t) -> int | None:
  return None if t is None else t.data_ptr()


def _cuda(*ts):
  for t in ts:
    if t is not None and not t.is_cuda:
      raise ValueError("sparsefold_b200 ops take CUDA tensors only")


def _ws(nbytes: int, device) -> torch.Tensor:
  return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def mask_u8(mask: torch.Tensor) -> torch.Tensor:
  return mask.to(torch.uint8).contiguous()


# ---------------------------------------------------------------------------
def layer_norm(x: torch.Tensor, weight, bias, eps: float = 1e-5) -> torch.Tensor:
  _cuda(x, weight, bias)
  x = x.contiguous()
  y = torch.empty_like(x)
  cols = x.shape[-1]
  N.call("sf_layernorm", _dt(x), _p(x), _p(y), _p(weight), _p(bias), x.numel() // cols, cols,
         C.c_float(eps), _stream())
  return y


def linear(x: torch.Tensor, wt: torch.Tensor, bias=None, residual=None, post_op=None) -> torch.Tensor:
  """y = post_op(x @ wt.T + bias + residual); wt is [out, in] in x's dtype."""
  _cuda(x, wt, bias, residual)
  x = x.contiguous()
  k = x.shape[-1]
  n = wt.shape[0]
  assert wt.shape[1] == k and wt.dtype == x.dtype
  rows = x.numel() // k
  y = torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=x.device)
  if residual is not None:
    residual = residual.to(x.dtype).expand_as(y).contiguous()
  N.call("sf_linear", _dt(x), _p(x), _p(wt), _p(bias), _p(residual), _p(y), rows, k, n,
         N.POST_OPS[post_op], _stream())
  return y


def attention(q, k, v, *, scale=None, mask_q=None, mask_k=None, bias=None, gate=None,
              mask_row=None) -> torch.Tensor:
  """Drop-in for backends/torch/attention/sdpa.py:22 dot_product_attention.

  q [..., Q, H, D], k [..., K, H, D], v [..., K, H, Dv] (Dv may differ from D,
  as sdpa.py allows), masks [..., Q] / [..., K] (broadcast), bias broadcastable
  to [..., H, Q, K]; optional gate [..., Q, H, Dv] applies sigmoid(gate) to the
  output.  Returns [..., Q, H, Dv] in q's dtype.
  """
  _cuda(q, k, v)
  batch = q.shape[:-3]
  Q, H, D = q.shape[-3:]
  K = k.shape[-3]
  Dv = v.shape[-1]
  B = math.prod(batch) if batch else 1
  dt = _dt(q)
  q3 = q.reshape(B, Q, H, D)
  k3 = k.expand(*batch, K, H, D).reshape(B, K, H, D)
  v3 = v.expand(*batch, K, H, Dv).reshape(B, K, H, Dv)
  q3, k3, v3 = (t if t.stride(-1) == 1 else t.contiguous() for t in (q3, k3, v3))
  out = torch.empty(B, Q, H, Dv, dtype=q.dtype, device=q.device)
  a = N.AttentionArgs()
  a.dtype = dt
  a.batch, a.heads, a.q_len, a.k_len, a.head_dim = B, H, Q, K, D
  a.value_dim = Dv
  a.q, a.q_sb, a.q_sh, a.q_sq = _p(q3), q3.stride(0), q3.stride(2), q3.stride(1)
  a.k, a.k_sb, a.k_sh, a.k_sk = _p(k3), k3.stride(0), k3.stride(2), k3.stride(1)
  a.v, a.v_sb, a.v_sh, a.v_sk = _p(v3), v3.stride(0), v3.stride(2), v3.stride(1)
  a.out, a.o_sb, a.o_sh, a.o_sq = _p(out), out.stride(0), out.stride(2), out.stride(1)
  keep = [q3, k3, v3, out]
  if bias is not None:
    b4 = bias.to(q.dtype) if bias.dtype not in (torch.float32, q.dtype) else bias
    b4 = b4.expand(*batch, H, Q, K)
    try:
      b4 = b4.view(B, H, Q, K)
    except RuntimeError:
      b4 = b4.reshape(B, H, Q, K)
    if b4.stride(-1) != 1:
      b4 = b4.contiguous()
    a.bias, a.bias_dtype = _p(b4), _dt(b4)
    a.b_sb, a.b_sh, a.b_sq = b4.stride(0), b4.stride(1), b4.stride(2)
    keep.append(b4)
  if mask_q is not None:
    mq = mask_u8(mask_q.expand(*batch, Q).reshape(B, Q))
    a.mask_q, a.mq_sb = _p(mq), mq.stride(0)
    keep.append(mq)
  if mask_k is not None:
    mk = mask_u8(mask_k.expand(*batch, K).reshape(B, K))
    a.mask_k, a.mk_sb = _p(mk), mk.stride(0)
    keep.append(mk)
  if mask_row is not None:
    mr = mask_u8(mask_row.reshape(B))
    a.mask_row = _p(mr)
    keep.append(mr)
  if gate is not None:
    g3 = gate.reshape(B, Q, H, Dv)
    a.gate, a.g_sb, a.g_sh, a.g_sq = _p(g3), g3.stride(0), g3.stride(2), g3.stride(1)
    keep.append(g3)
  a.scale = float(1.0 / math.sqrt(D) if scale is None else scale)
  N.call("sf_attention", C.byref(a), _stream())
  return out.reshape(*batch, Q, H, Dv)


# ---------------------------------------------------------------------------
def tri_mult_weights(glu, ln_w, ln_b, center_w, center_b, w_out, w_gate) -> N.TriMultWeights:
  return N.TriMultWeights(_p(ln_w), _p(ln_b), _p(glu), _p(center_w), _p(center_b), _p(w_out), _p(w_gate))


def tri_mult(z: torch.Tensor, mask_u8_: torch.Tensor, w: N.TriMultWeights, incoming: bool,
             out: torch.Tensor | None = None) -> torch.Tensor:
  """Whole TriangleMultiplication on one device: returns z + update."""
  _cuda(z)
  n, n2, c = z.shape
  assert n == n2 and c == 128 and z.is_contiguous()
  dt = _dt(z)
  lib = N.load()
  pitch = lib.sf_pair_pitch(n)
  a_op = torch.empty(n, c, pitch, dtype=z.dtype, device=z.device)     # [row][channel][pitch]
  b_op = torch.empty_like(a_op)
  p = torch.empty_like(a_op)
  ws = _ws(max(lib.sf_tri_mult_project_workspace(dt, n), lib.sf_tri_mult_output_workspace(dt, n, n)), z.device)
  N.call("sf_tri_mult_project", dt, _p(z), _p(mask_u8_), n, int(incoming), C.byref(w), _p(a_op), _p(b_op),
         _p(ws), ws.numel(), _stream())
  N.call("sf_tri_mult_contract", dt, _p(a_op), _p(b_op), _p(p), c, n, n, n, _stream())
  out = torch.empty_like(z) if out is None else out
  N.call("sf_tri_mult_output", dt, _p(z), _p(p), n, n, C.byref(w), _p(out), _p(ws), ws.numel(), _stream())
  return out


def tri_attention_weights(ln_w, w_qkvg, w_bias, w_out, heads: int) -> N.TriAttentionWeights:
  return N.TriAttentionWeights(_p(ln_w), _p(w_qkvg), _p(w_bias), _p(w_out), heads)


def tri_attention(z: torch.Tensor, mask_u8_: torch.Tensor, w: N.TriAttentionWeights, transpose: bool,
                  out: torch.Tensor | None = None) -> torch.Tensor:
  _cuda(z)
  n, n2, c = z.shape
  assert n == n2 and c == 128 and z.is_contiguous()
  dt = _dt(z)
  ws = _ws(N.load().sf_tri_attention_workspace(dt, n, w.heads), z.device)
  out = torch.empty_like(z) if out is None else out
  N.call("sf_tri_attention", dt, _p(z), _p(mask_u8_), n, int(transpose), C.byref(w), _p(out), _p(ws),
         ws.numel(), _stream())
  return out


def transition(x: torch.Tensor, ln_w, ln_b, w1, w2, out: torch.Tensor | None = None) -> torch.Tensor:
  _cuda(x)
  x = x.contiguous()
  c = x.shape[-1]
  inter = w1.shape[0] // 2
  rows = x.numel() // c
  dt = _dt(x)
  ws = _ws(N.load().sf_transition_workspace(dt, rows, inter), x.device)
  out = torch.empty_like(x) if out is None else out
  N.call("sf_transition", dt, _p(x), _p(ln_w), _p(ln_b), _p(w1), _p(w2), _p(out), rows, c, inter,
         _p(ws), ws.numel(), _stream())
  return out


def pair_logits(z: torch.Tensor, ln_w, ln_b, w, heads: int) -> torch.Tensor:
  """[H, rows, n] logits of LN(z) @ W (SingleActUpdate, blocks.py:745-749)."""
  _cuda(z)
  rows, n, c = z.shape
  dt = _dt(z)
  out = torch.empty(heads, rows, n, dtype=z.dtype, device=z.device)
  ws = _ws(N.load().sf_pair_logits_workspace(dt, rows, n, c), z.device)
  N.call("sf_pair_logits", dt, _p(z.contiguous()), _p(ln_w), _p(ln_b), _p(w), _p(out), rows, n, c, heads,
         _p(ws), ws.numel(), _stream())
  return out


# ---------------------------------------------------------------------------
# diffusion-transformer and MSA helpers
# ---------------------------------------------------------------------------
def _trailing_period(t: torch.Tensor, like: torch.Tensor):
  """(t, period) with t contiguous and like's trailing shape: the elements of t repeat every
  `period` elements of like (t broadcasts over like's leading dims), or t expanded in full."""
  t = t.to(like.dtype)
  lead = like.ndim - t.ndim
  if lead >= 0 and tuple(t.shape) == tuple(like.shape[lead:]):
    t = t.contiguous()
    return t, t.numel()
  t = t.expand_as(like).contiguous()
  return t, t.numel()


def adaln(x: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
  """scale * LN(x) + bias, all [..., C] of x's dtype (AdaptiveLayerNorm with single_cond); scale and
  bias may have fewer leading dims than x (one conditioning for every sample) and are not copied then."""
  _cuda(x, scale, bias)
  x = x.contiguous()
  c = x.shape[-1]
  if scale.shape != bias.shape:
    scale, bias = torch.broadcast_tensors(scale, bias)
  scale, per = _trailing_period(scale, x)
  bias, per_b = _trailing_period(bias, x)
  if per_b != per:
    scale, per = scale.expand_as(x).contiguous(), x.numel()
    bias = bias.expand_as(x).contiguous()
  y = torch.empty_like(x)
  N.call("sf_adaln", _dt(x), _p(x), _p(scale), _p(bias), _p(y), x.numel() // c, c, per // c, _stream())
  return y


def gated_residual(base, u: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
  """base + u * gate (base may be None); gate broadcasts to u's shape (over leading dims without a copy)."""
  _cuda(u, gate, base)
  u = u.contiguous()
  gate, per = _trailing_period(gate, u)
  if base is not None:
    base = base.to(u.dtype).expand_as(u).contiguous()
  out = torch.empty_like(u)
  N.call("sf_gated_residual", _dt(u), _p(base), _p(u), _p(gate), _p(out), u.numel(), per, _stream())
  return out


def gather_rows(src: torch.Tensor, idx: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
  """src [B, R, C] -> out [B, n_out, C] with out[b, i] = mask[i] ? src[b, idx[i]] : 0."""
  _cuda(src, idx, mask)
  src = src.contiguous()
  b, r, c = src.shape
  idx = idx.reshape(-1).to(torch.int32).contiguous()
  m = mask_u8(mask.reshape(-1))
  out = torch.empty(b, idx.numel(), c, dtype=src.dtype, device=src.device)
  N.call("sf_gather_rows", _dt(src), _p(src), b, r, _p(idx), _p(m), idx.numel(), c, _p(out), _stream())
  return out


def mask_rows_(x: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
  """In place: x[..., :] = 0 where !mask[...] (mask has x's leading shape)."""
  _cuda(x, mask)
  assert x.is_contiguous()
  c = x.shape[-1]
  m = mask_u8(mask.expand(x.shape[:-1]).reshape(-1))
  N.call("sf_mask_rows", _dt(x), _p(x), _p(m), x.numel() // c, c, _stream())
  return x


def softmax_rows(x: torch.Tensor, key_bias=None, out=None, ldy=None) -> torch.Tensor:
  _cuda(x, key_bias)
  x = x.contiguous()
  k = x.shape[-1]
  rows = x.numel() // k
  if out is None:
    out = torch.empty_like(x)
  N.call("sf_softmax_rows", _dt(x), _p(x), _p(key_bias), _p(out), rows, k, ldy or k, _stream())
  return out


def transpose_(src: torch.Tensor, dst: torch.Tensor, nb1, nb2, rows, cols, ib1, ib2, is_r, ob1, ob2, os_c) -> None:
  """Batched strided transpose between two CUDA buffers (strides in elements)."""
  _cuda(src, dst)
  N.call("sf_transpose", _dt(src), _p(src), _p(dst), nb1, nb2, rows, cols, ib1, ib2, is_r, ob1, ob2, os_c, _stream())


def pitch(n: int) -> int:
  return int(N.load().sf_pair_pitch(n))


def contract(a_op: torch.Tensor, b_op: torch.Tensor, channels: int, rows: int, cols: int, kdim: int) -> torch.Tensor:
  """P[i][c][j] = sum_k A[i][c][k] B[j][c][k]; A [rows][c][pitch(k)], B [cols][c][pitch(k)] -> [rows][c][pitch(cols)]."""
  _cuda(a_op, b_op)
  p = torch.empty(rows, channels, pitch(cols), dtype=a_op.dtype, device=a_op.device)
  N.call("sf_tri_mult_contract", _dt(a_op), _p(a_op), _p(b_op), _p(p), channels, rows, cols, kdim, _stream())
  return p


def opm_norm(mask: torch.Tensor, dtype) -> torch.Tensor:
  """[n_res, n_res] fp32 = 1/(1e-3 + sum_m mask[m,i] mask[m,j]) (count rounded to dtype)."""
  _cuda(mask)
  m = mask_u8(mask)
  n_seq, n_res = m.shape
  ws = _ws(N.load().sf_opm_norm_workspace(n_seq, n_res), m.device)
  norm = torch.empty(n_res, n_res, dtype=torch.float32, device=m.device)
  dt = N.SF_F32 if dtype == torch.float32 else N.SF_BF16
  N.call("sf_opm_norm", dt, _p(m), n_seq, n_res, _p(norm), _p(ws), ws.numel(), _stream())
  return norm


def opm_repack(o: torch.Tensor, n_res: int, d: int) -> torch.Tensor:
  _cuda(o)
  out = torch.empty(n_res * n_res, d * d, dtype=o.dtype, device=o.device)
  N.call("sf_opm_repack", _dt(o), _p(o), o.shape[-1], n_res, d, _p(out), _stream())
  return out


def scale_rows_(x: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
  _cuda(x, s)
  assert x.is_contiguous() and s.dtype == torch.float32
  c = x.shape[-1]
  N.call("sf_scale_rows", _dt(x), _p(x), _p(s.contiguous()), x.numel() // c, c, _stream())
  return x


def swiglu(h: torch.Tensor) -> torch.Tensor:
  """[..., 2I] -> swish(h[..., :I]) * h[..., I:]."""
  _cuda(h)
  h = h.contiguous()
  i2 = h.shape[-1]
  out = torch.empty(*h.shape[:-1], i2 // 2, dtype=h.dtype, device=h.device)
  N.call("sf_swiglu", _dt(h), _p(h), _p(out), h.numel() // i2, i2 // 2, _stream())
  return out


def pair_outer_sum(left: torch.Tensor, right: torch.Tensor, addend=None) -> torch.Tensor:
  """out[i, j] = left[i] + right[j] (+ addend[i, j]): [B, C] x [N, C] -> [B, N, C] in left's dtype
  (Evoformer._get_seq_pair_embedding, trunk/network.py:195-212)."""
  _cuda(left, right, addend)
  assert left.ndim == 2 and right.ndim == 2 and left.shape[1] == right.shape[1] and left.dtype == right.dtype
  b, c = left.shape
  n = right.shape[0]
  left, right = left.contiguous(), right.contiguous()
  if addend is not None:
    addend = addend.to(left.dtype).expand(b, n, c).contiguous()
  out = torch.empty(b, n, c, dtype=left.dtype, device=left.device)
  N.call("sf_pair_outer_sum", _dt(left), _p(left), _p(right), _p(addend), _p(out), b, n, c, _stream())
  return out


def pair_sparse_linear(x: torch.Tensor, w_kc: torch.Tensor, residual=None) -> torch.Tensor:
  """out[..., :] = sum over the nonzero x[..., k] of x[..., k] * w_kc[k, :] (+ residual): the linear layers
  on one-hot / 0-1 pair features (trunk/network.py:188-193, :214-256).  w_kc is fp32 [K, C]."""
  _cuda(x, w_kc, residual)
  assert w_kc.dtype == torch.float32 and w_kc.ndim == 2 and x.shape[-1] == w_kc.shape[0]
  x = x.contiguous()
  k, c = w_kc.shape
  out = torch.empty(*x.shape[:-1], c, dtype=x.dtype, device=x.device)
  if residual is not None:
    residual = residual.to(x.dtype).expand_as(out).contiguous()
  N.call("sf_pair_sparse_linear", _dt(x), _p(x), _p(w_kc.contiguous()), _p(residual), _p(out), x.numel() // k, k, c,
         _stream())
  return out
