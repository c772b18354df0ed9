"""Weight encoders and the per-weight encoding policy, re-targeted at the B200 device layouts.

Restates the reference's `aneforge/_blob.py` encoders and `aneforge/_compile.py:112-188`
(`_Emitter.weight`) so that `compress=` means the same thing here:

  None        -> fp16
  "int8"      -> per-output-row int8 (`quantize_per_row`, _blob.py:20-25)
  "int4"      -> per-tensor 16-entry LUT when its relative Frobenius error <= compress_atol
                 (`palettize_lut4`, _blob.py:28-43, gate _compile.py:135-153), else per-row int8
  "blockwise" -> int8 in 32-column blocks when within compress_atol (_blob.py:46-56), else fp16
  "sparse"    -> bitmask sparse when >= half zeros (_blob.py:59-64), else fp16
  "int4_g32"  -> this build's group-32 symmetric 4-bit format (no reference counterpart)

Large int8 / int4_g32 weights are quantized on the GPU (csrc/quant.cu, bit-identical to the numpy
code below); the numpy encoders serve small tensors and the LUT/blockwise/sparse gates.
"""
from __future__ import annotations

import numpy as np

F16, F32 = np.float16, np.float32


def quantize_per_row(W):
  W = np.asarray(W).astype(F32)
  scale = np.clip(np.abs(W).max(axis=1, keepdims=True) / 127.0, 1e-8, None)
  q = np.round(W / scale).clip(-127, 127).astype(np.int8)
  return np.ascontiguousarray(q), scale[:, 0].astype(F16)


def palettize_lut4(W):
  flat = np.asarray(W).reshape(-1).astype(F32)
  edges = np.quantile(flat, np.linspace(0.0, 1.0, 17))
  cent = ((edges[:-1] + edges[1:]) / 2.0).astype(F32)
  for _ in range(20):
    idx = np.abs(flat[:, None] - cent[None, :]).argmin(axis=1)
    for k in range(16):
      sel = flat[idx == k]
      if sel.size:
        cent[k] = sel.mean()
  idx = np.abs(flat[:, None] - cent[None, :]).argmin(axis=1).astype(np.uint8).reshape(W.shape[0], -1)
  if idx.shape[1] % 2:
    idx = np.pad(idx, ((0, 0), (0, 1)))
  packed = (idx[:, 0::2] | (idx[:, 1::2] << 4)).astype(np.uint8)
  return np.ascontiguousarray(packed), cent.astype(F16)


def lut4_dense(W2, packed, lut):
  raw = packed.reshape(-1)
  idx = np.empty(raw.size * 2, np.uint8)
  idx[0::2], idx[1::2] = raw & 0x0F, (raw >> 4) & 0x0F
  return lut.astype(F32)[idx][: W2.size].reshape(W2.shape)


def quantize_blockwise(W, block_size=32):
  W = np.asarray(W).astype(F32)
  OUT, IN = W.shape
  bs = int(block_size)
  while bs > 1 and IN % bs:
    bs -= 1
  nb = IN // bs
  Wb = W.reshape(OUT, nb, bs)
  scale = np.clip(np.abs(Wb).max(axis=2) / 127.0, 1e-8, None)
  q = np.round(Wb / scale[:, :, None]).clip(-127, 127).astype(np.int8).reshape(OUT, IN)
  return np.ascontiguousarray(q), scale.astype(F16), nb


def quantize_g32_int4(W, group=32):
  W = np.asarray(W).astype(F32)
  OUT, IN = W.shape
  Wg = W.reshape(OUT, IN // group, group)
  scale = np.clip(np.abs(Wg).max(axis=2) / 7.0, 1e-8, None)
  q = np.round(Wg / scale[:, :, None]).clip(-7, 7).astype(np.int8).reshape(OUT, IN)
  nib = (q + 8).astype(np.uint8)
  return np.ascontiguousarray((nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)), scale.astype(F16)


def _rel(a, b):
  b = np.asarray(b, F32)
  return float(np.linalg.norm(np.asarray(a, F32) - b) / (np.linalg.norm(b) + 1e-12))


def decide(W, compress, compress_atol=0.05, block_size=32, allow_int8=True, allow_int4=True,
           allow_sparse=True, int8=None):
  """The encoding kind the reference's policy picks for W (`_compile.py:112-188`).
  Returns (kind, payload) with payload None for kinds the device quantizes itself."""
  W2 = np.asarray(W).reshape(W.shape[0], -1)
  auto = compress == "auto"
  if compress == "int4_g32" and allow_int8 and W2.shape[1] % 32 == 0:
    return "int4_g32", None
  if (compress == "sparse" or auto) and allow_sparse:
    nz = np.count_nonzero(W2)
    if 0 < nz <= W2.size // 2:
      return "sparse", None
  if (compress == "int4" or auto) and allow_int4 and W2.shape[1] % 2 == 0:
    packed, lut = palettize_lut4(W2)
    if _rel(lut4_dense(W2, packed, lut), W2) <= compress_atol:
      return "lut4", (packed, lut)
  if compress == "blockwise" and allow_int8:
    q, s, nb = quantize_blockwise(W2, block_size)
    OUT, IN = W2.shape
    deq = (q.astype(F32).reshape(OUT, nb, IN // nb) * s.astype(F32)[:, :, None]).reshape(OUT, IN)
    if _rel(deq, W2) <= compress_atol:
      return "blockwise", (q, s, nb)
  use_int8 = int8 if int8 is not None else (compress in ("int8", "int4") or auto)
  if use_int8 and allow_int8:
    return "int8", None
  return "fp16", None


def dense_of(W, compress, **kw) -> np.ndarray:
  """The fp32 matrix the device multiplies by for W under `compress` (small tensors only)."""
  kind, payload = decide(W, compress, **kw)
  W2 = np.asarray(W).reshape(W.shape[0], -1)
  if kind == "int8":
    q, s = quantize_per_row(W2)
    return (q.astype(F32) * s.astype(F32)[:, None]).reshape(W.shape)
  if kind == "lut4":
    return lut4_dense(W2, *payload).reshape(W.shape)
  if kind == "blockwise":
    q, s, nb = payload
    OUT, IN = W2.shape
    return (q.astype(F32).reshape(OUT, nb, IN // nb) * s.astype(F32)[:, :, None]).reshape(W.shape)
  if kind == "int4_g32":
    p, s = quantize_g32_int4(W2)
    nib = np.stack([p & 15, p >> 4], -1).reshape(W2.shape).astype(F32) - 8
    return (nib.reshape(W2.shape[0], -1, 32) * s.astype(F32)[:, :, None]).reshape(W.shape)
  return np.asarray(W, F16).astype(F32)


def gqa_expand_factor(n_kv: int, group: int, compress, compress_atol=0.05, block_size=32) -> float:
  """The value a 1 of the reference's 0/1 GQA expansion matrix (`llm.py:205-211`) decodes to under
  `compress`: 127*f16(1/127) for per-row int8, exactly 1 for fp16 or an accepted LUT."""
  if group == 1:
    return 1.0
  Mx = np.repeat(np.eye(n_kv, dtype=F16), group, axis=0)
  d = dense_of(Mx, compress, compress_atol=compress_atol, block_size=block_size)
  return float(d[0, 0])
