"""Python wrappers of the kernel-level C ABI (include/af_cuda.h). Tensors are torch CUDA tensors used
only as device memory; every call goes through libaf_cuda.so on torch's current stream and raises on
a non-zero return code. No CPU path exists."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _runtime as R


def _stream(t) -> int:
  import torch
  return torch.cuda.current_stream(t.device).cuda_stream


def _p(t) -> int:
  return 0 if t is None else t.data_ptr()


def _need(cond, msg):
  if not cond:
    raise ValueError(msg)


def quantize_per_row_i8(W):
  """Per-row int8 codes [N,K] + fp16 scales [N] (bit-exact to the reference numpy encoder)."""
  import torch
  _need(W.is_cuda and W.dim() == 2 and W.is_contiguous(), "W must be a contiguous 2-D CUDA tensor")
  _need(W.dtype in (torch.float16, torch.float32), "W must be fp16 or fp32")
  N, K = W.shape
  q = torch.empty((N, K), dtype=torch.int8, device=W.device)
  s = torch.empty((N,), dtype=torch.float16, device=W.device)
  R.check(R.lib().af_quantize_per_row_i8(_p(W), int(W.dtype == torch.float16), N, K, _p(q), _p(s), _stream(W)),
          "af_quantize_per_row_i8")
  return q, s


def quantize_g32_i4(W):
  """Group-32 int4: packed [N, K/2] uint8 + fp16 scales [N, K/32]."""
  import torch
  _need(W.is_cuda and W.dim() == 2 and W.is_contiguous(), "W must be a contiguous 2-D CUDA tensor")
  N, K = W.shape
  _need(K % 32 == 0, "K must be a multiple of 32")
  p = torch.empty((N, K // 2), dtype=torch.uint8, device=W.device)
  s = torch.empty((N, K // 32), dtype=torch.float16, device=W.device)
  R.check(R.lib().af_quantize_g32_i4(_p(W), int(W.dtype == torch.float16), N, K, _p(p), _p(s), _stream(W)),
          "af_quantize_g32_i4")
  return p, s


def gemv(x, w, scales=None, bias=None, wf=R.W_I8, epi=R.EPI_F32, y=None, n_out=None):
  """y = epi(scales (.) (x . W^T) + bias). x [NB, K] fp16; w rows [N, ...]."""
  import torch
  _need(x.is_cuda and x.dtype == torch.float16 and x.dim() == 2, "x must be [NB, K] fp16 CUDA")
  NB, K = x.shape
  N = w.shape[0]
  cols = N // 2 if epi == R.EPI_SWIGLU else N
  if y is None:
    dt = torch.float16 if epi in (R.EPI_F16, R.EPI_SWIGLU) else torch.float32
    y = torch.zeros((NB, cols), dtype=dt, device=x.device)
  R.check(R.lib().af_gemv(wf, epi, _p(x), x.stride(0), _p(w), _p(scales), _p(bias), _p(y), y.stride(0), NB, N, K,
                          _stream(x)), "af_gemv")
  return y


def lm_head_argmax(x, w, scales=None, wf=R.W_F16, logits=True, pos=None, scratch=None, out=None):
  """Greedy token per row of x [NB, K] fp16 against head rows w [V, K]; optional fp32 logits.
  `scratch` (zeroed, left zeroed) may be reused across calls of one shape; `out` = (tok, logits)
  preallocated outputs."""
  import torch
  NB, K = x.shape
  V = w.shape[0]
  L = R.lib()
  nbytes = ctypes.c_size_t()
  R.check(L.af_lm_head_argmax_scratch(wf, V, K, NB, ctypes.byref(nbytes)), "scratch")
  if scratch is None:
    scratch = torch.zeros((nbytes.value,), dtype=torch.uint8, device=x.device)
  _need(scratch.numel() >= nbytes.value, "lm_head scratch too small")
  if out is not None:
    tok, lg = out
  else:
    tok = torch.zeros((NB,), dtype=torch.int32, device=x.device)
    lg = torch.zeros((NB, V), dtype=torch.float32, device=x.device) if logits else None
  R.check(L.af_lm_head_argmax(wf, _p(x), x.stride(0), _p(w), _p(scales), _p(lg), NB, V, K, _p(tok), _p(pos),
                              _p(scratch), scratch.numel(), _stream(x)), "af_lm_head_argmax")
  return tok, lg


def rmsnorm(x, g, floor):
  import torch
  NB, D = x.shape
  out = torch.empty((NB, D), dtype=torch.float16, device=x.device)
  R.check(R.lib().af_rmsnorm(_p(x), int(x.dtype == torch.float16), x.stride(0), _p(g), float(floor), _p(out),
                             out.stride(0), NB, D, _stream(x)), "af_rmsnorm")
  return out


def attn_decode_scratch_bytes(nb, kv, n_split, g, dh) -> int:
  n = ctypes.c_size_t()
  R.check(R.load_library().af_attn_decode_scratch(nb, kv, n_split, g, dh, ctypes.byref(n)), "scratch")
  return n.value


def attn_decode(qkv, kc, vc, pos, cos_t, sin_t, H, KV, dh, scale, kv_c=1.0, expand=False, n_split=1, scratch=None,
                err=None, out=None):
  """Decode attention; updates kc/vc at pos in place; returns fp16 [NB, H*dh]."""
  import torch
  NB = qkv.shape[0]
  M = kc.shape[2]
  if out is None:
    out = torch.zeros((NB, H * dh), dtype=torch.float16, device=qkv.device)
  if n_split > 1 and scratch is None:
    scratch = torch.zeros((attn_decode_scratch_bytes(NB, KV, n_split, H // KV, dh),), dtype=torch.uint8,
                          device=qkv.device)
  nbytes = 0 if scratch is None else scratch.numel()
  R.check(R.lib().af_attn_decode(_p(qkv), qkv.stride(0), _p(kc), _p(vc), _p(pos), _p(cos_t), _p(sin_t), _p(out),
                                 out.stride(0), NB, H, KV, dh, M, n_split, float(scale), float(kv_c), int(expand),
                                 _p(scratch), nbytes, _p(err), _stream(qkv)), "af_attn_decode")
  return out


def pack_i8_tiles(q):
  """Per-row int8 codes [N, K] -> the tensor-core fragment-tile layout (uint8, flat)."""
  import torch
  N, K = q.shape
  L = R.lib()
  out = torch.empty((L.af_pack_i8_tiles_bytes(N, K),), dtype=torch.uint8, device=q.device)
  R.check(L.af_pack_i8_tiles(_p(q), N, K, _p(out), _stream(q)), "af_pack_i8_tiles")
  return out


def gemv_tc_scratch(N, K, NB, device):
  import torch
  n = R.load_library().af_gemv_tc_scratch_bytes(N, K, NB)
  return torch.zeros((max(n, 1),), dtype=torch.uint8, device=device), n


def pack_i4_tiles(packed, scales, N, K):
  """Group-32 int4 (packed [N, K/2] + scales [N, K/32]) -> tensor-core tiles with the scales inside."""
  import torch
  L = R.lib()
  out = torch.empty((L.af_pack_i4_tiles_bytes(N, K),), dtype=torch.uint8, device=packed.device)
  R.check(L.af_pack_i4_tiles(_p(packed), _p(scales), N, K, _p(out), _stream(packed)), "af_pack_i4_tiles")
  return out


def gemv_tc_i4(x, tiles, N, K, bias=None, epi=R.EPI_F32, y=None, scratch=None):
  """Tensor-core group-32 int4 GEMV over pack_i4_tiles output. x [NB, K] fp16."""
  import torch
  NB = x.shape[0]
  cols = N // 2 if epi == R.EPI_SWIGLU else N
  if y is None:
    dt = torch.float16 if epi in (R.EPI_F16, R.EPI_SWIGLU) else torch.float32
    y = torch.zeros((NB, cols), dtype=dt, device=x.device)
  if scratch is None:
    scratch, nbytes = gemv_tc_scratch(N, K, NB, x.device)
  else:
    nbytes = scratch.numel()
  R.check(R.lib().af_gemv_tc_i4(epi, _p(x), x.stride(0), _p(tiles), _p(bias), _p(y), y.stride(0), NB, N, K,
                                _p(scratch), nbytes, _stream(x)), "af_gemv_tc_i4")
  return y


def gemv_tc(x, tiles, scales, N, K, bias=None, epi=R.EPI_F32, y=None, scratch=None):
  """Tensor-core int8 GEMV over packed tiles. x [NB, K] fp16."""
  import torch
  NB = x.shape[0]
  cols = N // 2 if epi == R.EPI_SWIGLU else N
  if y is None:
    dt = torch.float16 if epi in (R.EPI_F16, R.EPI_SWIGLU) else torch.float32
    y = torch.zeros((NB, cols), dtype=dt, device=x.device)
  if scratch is None:
    scratch, nbytes = gemv_tc_scratch(N, K, NB, x.device)
  else:
    nbytes = scratch.numel()
  R.check(R.lib().af_gemv_tc(epi, _p(x), x.stride(0), _p(tiles), _p(scales), _p(bias), _p(y), y.stride(0), NB, N, K,
                             _p(scratch), nbytes, _stream(x)), "af_gemv_tc")
  return y


def attn_decode_noalloc(qkv, kc, vc, pos, cos_t, sin_t, H, KV, dh, scale, kv_c=1.0, expand=False, n_split=1, err=None):
  """Decode attention using the library's built-in scratch (no allocation by the entry point).
  Returns (rc, out); rc != 0 means the shape was rejected (reason in _runtime.last_error())."""
  import torch
  NB = qkv.shape[0]
  M = kc.shape[2]
  out = torch.zeros((NB, H * dh), dtype=torch.float16, device=qkv.device)
  rc = R.lib().af_attn_decode_noalloc(_p(qkv), qkv.stride(0), _p(kc), _p(vc), _p(pos), _p(cos_t), _p(sin_t),
                                      _p(out), out.stride(0), NB, H, KV, dh, M, n_split, float(scale), float(kv_c),
                                      int(expand), _p(err), _stream(qkv))
  return rc, out


def moe_gate(logits, k, renorm=True):
  """Router logits [NB, E] fp32 -> (gw [NB, E] fp32, sel [NB, k] int32) on the device."""
  import torch
  NB, E = logits.shape
  gw = torch.zeros((NB, E), dtype=torch.float32, device=logits.device)
  sel = torch.zeros((NB, k), dtype=torch.int32, device=logits.device)
  R.check(R.lib().af_moe_gate(_p(logits), logits.stride(0), NB, E, k, int(renorm), _p(gw), _p(sel), _stream(logits)),
          "af_moe_gate")
  return gw, sel


def gemv_tc_expert(x, tiles, scales, N, K, E, wf=R.W_I8, epi=R.EPI_F32, y=None, sel=None, slot=0, fixed_e=0, rw=None,
                   scratch=None):
  """Tensor-core GEMV over E experts' tiles stored back to back; expert = sel[slot] or fixed_e."""
  import torch
  if sel is None and not 0 <= fixed_e < E:
    raise ValueError(f"fixed_e={fixed_e} outside the {E} experts of these tiles")
  NB = x.shape[0]
  cols = N // 2 if epi == R.EPI_SWIGLU else N
  if y is None:
    dt = torch.float16 if epi in (R.EPI_F16, R.EPI_SWIGLU) else torch.float32
    y = torch.zeros((NB, cols), dtype=dt, device=x.device)
  if scratch is None:
    scratch, nbytes = gemv_tc_scratch(N, K, NB, x.device)
  else:
    nbytes = scratch.numel()
  stride = tiles.numel() // E
  R.check(R.lib().af_gemv_tc_expert(wf, epi, _p(x), x.stride(0), _p(tiles), _p(scales), _p(y), y.stride(0), NB, N, K,
                                    _p(sel), slot, fixed_e, stride, N if scales is not None else 0, _p(rw), E,
                                    _p(scratch), nbytes, _stream(x)), "af_gemv_tc_expert")
  return y


def gemm_tc(x, tiles, scales, N, K, wf=R.W_I8, bias=None, epi=R.EPI_F32, y=None):
  """Prefill GEMM on tcgen05 over packed tiles: x [M, K] fp16 -> y [M, N] (or [M, N/2] for SWIGLU)."""
  import torch
  M = x.shape[0]
  cols = N // 2 if epi == R.EPI_SWIGLU else N
  if y is None:
    dt = torch.float16 if epi in (R.EPI_F16, R.EPI_SWIGLU) else torch.float32
    y = torch.zeros((M, cols), dtype=dt, device=x.device)
  R.check(R.lib().af_gemm_tc(wf, epi, _p(x), x.stride(0), _p(tiles), _p(scales), _p(bias), _p(y), y.stride(0), M, N, K,
                             _stream(x)), "af_gemm_tc")
  return y
