"""ctypes binding of ``libsparsefold_b200.so`` (declared in include/sparsefold_b200.h).

There is no fallback: if the library is missing or the device is not sm_100,
every op raises.  Build it with ``python -m sparsefold_b200.build``.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libsparsefold_b200.so")

SF_F32, SF_BF16 = 0, 1
SF_OK, SF_ERR_ARG, SF_ERR_CUDA, SF_ERR_WORKSPACE, SF_ERR_DEVICE, SF_ERR_TIMEOUT = range(6)
POST_OPS = {None: 0, "none": 0, "relu": 1, "silu": 2, "sigmoid": 3}

_vp = C.c_void_p
_i64 = C.c_int64
_f32p = C.c_void_p  # float* passed as raw address


class AttentionArgs(C.Structure):
  _fields_ = [
      ("dtype", C.c_int),
      ("batch", _i64), ("heads", _i64), ("q_len", _i64), ("k_len", _i64), ("head_dim", _i64),
      ("q", _vp), ("q_sb", _i64), ("q_sh", _i64), ("q_sq", _i64),
      ("k", _vp), ("k_sb", _i64), ("k_sh", _i64), ("k_sk", _i64),
      ("v", _vp), ("v_sb", _i64), ("v_sh", _i64), ("v_sk", _i64),
      ("out", _vp), ("o_sb", _i64), ("o_sh", _i64), ("o_sq", _i64),
      ("bias", _vp), ("bias_dtype", C.c_int), ("b_sb", _i64), ("b_sh", _i64), ("b_sq", _i64),
      ("mask_q", _vp), ("mq_sb", _i64),
      ("mask_k", _vp), ("mk_sb", _i64),
      ("mask_row", _vp),
      ("gate", _vp), ("g_sb", _i64), ("g_sh", _i64), ("g_sq", _i64),
      ("scale", C.c_float),
      ("value_dim", _i64),
  ]


class TriMultWeights(C.Structure):
  _fields_ = [("ln_w", _vp), ("ln_b", _vp), ("w_glu", _vp), ("center_w", _vp), ("center_b", _vp),
              ("w_out", _vp), ("w_gate", _vp)]


class TriAttentionWeights(C.Structure):
  _fields_ = [("ln_w", _vp), ("w_qkvg", _vp), ("w_bias", _vp), ("w_out", _vp), ("heads", _i64)]


# name -> (restype, argtypes)
_SIGNATURES = {
    "sf_version": (C.c_char_p, []),
    "sf_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "sf_device_check": (C.c_int, []),
    "sf_launch_count": (C.c_uint64, []),
    "sf_pair_pitch": (C.c_int64, [_i64]),
    "sf_device_status": (C.c_int, [C.POINTER(C.c_uint32), C.c_int]),
    "sf_selftest_wait": (C.c_int, [C.c_uint32, C.c_int, _vp]),
    "sf_attention": (C.c_int, [C.POINTER(AttentionArgs), _vp]),
    "sf_layernorm": (C.c_int, [C.c_int, _vp, _vp, _vp, _vp, _i64, _i64, C.c_float, _vp]),
    "sf_linear": (C.c_int, [C.c_int, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, C.c_int, _vp]),
    "sf_tri_mult_project": (C.c_int, [C.c_int, _vp, _vp, _i64, C.c_int, C.POINTER(TriMultWeights),
                                      _vp, _vp, _vp, C.c_size_t, _vp]),
    "sf_tri_mult_project_workspace": (C.c_size_t, [C.c_int, _i64]),
    "sf_tri_mult_contract": (C.c_int, [C.c_int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "sf_tri_mult_output": (C.c_int, [C.c_int, _vp, _vp, _i64, _i64, C.POINTER(TriMultWeights), _vp,
                                     _vp, C.c_size_t, _vp]),
    "sf_tri_mult_output_workspace": (C.c_size_t, [C.c_int, _i64, _i64]),
    "sf_tri_attention": (C.c_int, [C.c_int, _vp, _vp, _i64, C.c_int, C.POINTER(TriAttentionWeights), _vp,
                                   _vp, C.c_size_t, _vp]),
    "sf_tri_attention_workspace": (C.c_size_t, [C.c_int, _i64, _i64]),
    "sf_transition": (C.c_int, [C.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, C.c_size_t, _vp]),
    "sf_transition_workspace": (C.c_size_t, [C.c_int, _i64, _i64]),
    "sf_transition_noalloc": (C.c_int, [C.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "sf_transition_noalloc_max_scratch": (C.c_size_t, []),
    "sf_pair_logits": (C.c_int, [C.c_int, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, C.c_size_t, _vp]),
    "sf_pair_logits_workspace": (C.c_size_t, [C.c_int, _i64, _i64, _i64]),
    "sf_adaln": (C.c_int, [C.c_int, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "sf_gated_residual": (C.c_int, [C.c_int, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "sf_gather_rows": (C.c_int, [C.c_int, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _vp]),
    "sf_mask_rows": (C.c_int, [C.c_int, _vp, _vp, _i64, _i64, _vp]),
    "sf_softmax_rows": (C.c_int, [C.c_int, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "sf_swiglu": (C.c_int, [C.c_int, _vp, _vp, _i64, _i64, _vp]),
    "sf_transpose": (C.c_int, [C.c_int, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "sf_opm_norm": (C.c_int, [C.c_int, _vp, _i64, _i64, _vp, _vp, C.c_size_t, _vp]),
    "sf_opm_norm_workspace": (C.c_size_t, [_i64, _i64]),
    "sf_opm_repack": (C.c_int, [C.c_int, _vp, _i64, _i64, _i64, _vp, _vp]),
    "sf_scale_rows": (C.c_int, [C.c_int, _vp, _vp, _i64, _i64, _vp]),
    "sf_copy_blocks": (C.c_int, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "sf_pair_outer_sum": (C.c_int, [C.c_int, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "sf_pair_sparse_linear": (C.c_int, [C.c_int, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "sf_ipc_export": (C.c_int, [_vp, _vp, C.POINTER(C.c_uint64)]),
    "sf_ipc_import": (C.c_int, [_vp, C.c_uint64, C.POINTER(C.c_void_p)]),
    "sf_ipc_close_all": (C.c_int, []),
    "sf_scatter_peers": (C.c_int, [_vp, _vp, C.c_int32, _i64, _i64, _i64, _vp]),
    "sf_peer_signal": (C.c_int, [_vp, C.c_uint32, _vp]),
    "sf_peer_wait": (C.c_int, [_vp, C.c_int32, C.c_int32, C.c_uint32, C.c_uint32, _vp]),
    "sf_tri_mult_project_rows": (C.c_int, [C.c_int, _vp, _vp, _i64, _i64, _i64, C.c_int, C.POINTER(TriMultWeights),
                                           _vp, _vp, _vp]),
    "sf_tri_mult_contract_chunked": (C.c_int, [C.c_int, _vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp]),
    "sf_tri_attention_query_pitch": (C.c_int64, [_i64]),
    "sf_tri_attention_bias": (C.c_int, [C.c_int, _vp, _i64, _i64, C.POINTER(TriAttentionWeights), _vp, _i64, _vp]),
    "sf_tri_attention_project": (C.c_int, [C.c_int, _vp, _i64, _i64, C.c_int, C.c_int, C.POINTER(TriAttentionWeights),
                                           _vp, _vp, _vp, _vp, _vp, _vp]),
    "sf_tri_attention_core": (C.c_int, [C.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, C.c_int, _i64,
                                        C.POINTER(TriAttentionWeights), _vp]),
}

_lib = None
_lock = threading.Lock()


class NativeError(RuntimeError):
  pass


def load(path: str = LIB_PATH):
  """Load the library (once) and declare every exported entry point."""
  global _lib
  with _lock:
    if _lib is not None:
      return _lib
    if not os.path.exists(path):
      raise NativeError(f"{path} is missing; build it with `python -m sparsefold_b200.build`")
    lib = C.CDLL(path)
    for name, (res, args) in _SIGNATURES.items():
      fn = getattr(lib, name)
      fn.restype = res
      fn.argtypes = args
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
  return list(_SIGNATURES)


def last_error() -> str:
  buf = C.create_string_buffer(2048)
  load().sf_last_error(buf, len(buf))
  return buf.value.decode(errors="replace")


def check(status: int, what: str) -> None:
  if status != SF_OK:
    raise NativeError(f"{what} failed (status {status}): {last_error()}")


def call(name: str, *args) -> None:
  check(getattr(load(), name)(*args), name)


def device_status(clear: bool = True) -> int:
  """0, or SF_ERR_TIMEOUT if a kernel's bounded wait gave up since the last clear."""
  v = C.c_uint32(0)
  check(load().sf_device_status(C.byref(v), int(clear)), "sf_device_status")
  return int(v.value)


def launch_count() -> int:
  return int(load().sf_launch_count())
