"""Weight encoders: numpy restatement of the reference's `aneforge/_blob.py` quantizers and of the
per-weight encoding decision in `aneforge/_compile.py:_Emitter.weight`.

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`).

Every encoder returns arrays (not bytes); `tests/test_oracle_golden.py` compares their bytes with
the golden blobs the reference itself produced.
"""
from __future__ import annotations

import numpy as np

F16, F32 = np.float16, np.float32


def quantize_per_row(W: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
  """Per-output-row symmetric int8 (reference `aneforge/_blob.py:20-25`).

  scale = clip(max|row| / 127, 1e-8) in f32; codes = round-half-even(W / scale) clipped to
  [-127, 127]; the STORED scale is f16(scale). Dequant is `codes * scale_f16[:, None]`
  (`aneforge/_compile.py:173-179`, axis 0, zero point 0). Codes come from the f32 scale, the
  dequant uses the f16 one - both exactly as the reference does.
  """
  W = np.asarray(W).astype(F32)
  scale = np.clip(np.abs(W).max(axis=1, keepdims=True) / 127.0, 1e-8, None)
  q = np.round(W / scale).clip(-127, 127).astype(np.int8)
  return np.ascontiguousarray(q), scale[:, 0].astype(F16)


def dequant_per_row(q: np.ndarray, s: np.ndarray) -> np.ndarray:
  return q.astype(F32) * s.astype(F32)[:, None]


def palettize_lut4(W: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
  """Per-tensor 16-entry LUT (reference `aneforge/_blob.py:28-43`).

  Centroids start at the midpoints of the 17 quantile edges, then 20 Lloyd iterations
  (nearest centroid by |w - c|, first index on ties; empty clusters keep their value). Indices
  are packed two per byte, low nibble first, odd rows padded with index 0; codebook stored f16.
  Returns (packed [OUT, ceil(IN/2)] uint8, codebook [16] f16).
  """
  flat = np.asarray(W).reshape(-1).astype(F32)
  edges = np.quantile(flat, np.linspace(0.0, 1.0, 17))
  cent = ((edges[:-1] + edges[1:]) / 2.0).astype(F32)
  for _ in range(20):
    idx = np.abs(flat[:, None] - cent[None, :]).argmin(axis=1)
    for k in range(16):
      sel = flat[idx == k]
      if sel.size:
        cent[k] = sel.mean()
  idx = np.abs(flat[:, None] - cent[None, :]).argmin(axis=1).astype(np.uint8)
  idx = idx.reshape(W.shape[0], -1)
  if idx.shape[1] % 2:
    idx = np.pad(idx, ((0, 0), (0, 1)))
  packed = (idx[:, 0::2] | (idx[:, 1::2] << 4)).astype(np.uint8)
  return np.ascontiguousarray(packed), cent.astype(F16)


def unpack_lut4(packed: np.ndarray, lut: np.ndarray, shape) -> np.ndarray:
  """Inverse of `palettize_lut4` as the reference's gate reconstructs it (`_compile.py:93-101`)."""
  raw = np.asarray(packed, np.uint8).reshape(-1)
  idx = np.empty(raw.size * 2, np.uint8)
  idx[0::2], idx[1::2] = raw & 0x0F, (raw >> 4) & 0x0F
  out, inn = shape
  pad_in = inn + (inn % 2)
  idx = idx.reshape(out, pad_in)[:, :inn]
  return lut.astype(F32)[idx]


def lut4_rel_error(W2: np.ndarray, packed: np.ndarray, lut: np.ndarray) -> float:
  """Relative Frobenius error of the LUT reconstruction (reference `_compile.py:93-101`).

  The reference flattens the packed indices and truncates to W.size, which only equals the
  per-row unpacking when IN is even - the reference gates int4 on an even IN (`_compile.py:136`).
  """
  cb = lut.astype(F32)
  raw = np.asarray(packed, np.uint8).reshape(-1)
  idx = np.empty(raw.size * 2, np.uint8)
  idx[0::2], idx[1::2] = raw & 0x0F, (raw >> 4) & 0x0F
  recon = cb[idx][: W2.size].reshape(W2.shape)
  W2 = W2.astype(F32)
  return float(np.linalg.norm(recon - W2) / (np.linalg.norm(W2) + 1e-12))


def quantize_blockwise(W: np.ndarray, block_size: int = 32) -> tuple[np.ndarray, np.ndarray, int]:
  """Per-block symmetric int8 along IN (reference `aneforge/_blob.py:46-56`).

  The block size clamps down to the largest divisor of IN. Returns (codes [OUT, IN] int8,
  scales [OUT, nblocks] f16, nblocks).
  """
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


def blockwise_rel_error(W2, q, scale, nb) -> float:
  """Reference `_compile.py:103-110`."""
  OUT, IN = W2.shape
  recon = (q.astype(F32).reshape(OUT, nb, IN // nb) * scale.astype(F32)[:, :, None]).reshape(OUT, IN)
  W2 = W2.astype(F32)
  return float(np.linalg.norm(recon - W2) / (np.linalg.norm(W2) + 1e-12))


def sparsify(W: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
  """Bitmask sparse encoding, LSB first (reference `aneforge/_blob.py:59-64`)."""
  flat = np.asarray(W).reshape(-1)
  nz = flat != 0.0
  mask = np.packbits(nz.astype(np.uint8), bitorder="little")
  return mask, flat[nz].astype(F16)


def quantize_g32_int4(W: np.ndarray, group: int = 32) -> tuple[np.ndarray, np.ndarray]:
  """Group-32 symmetric 4-bit format (Q4_0-like). NOT in the reference: parity unpinned.

  Modelled on `quantize_blockwise` (`aneforge/_blob.py:46-56`) with 7 levels per sign instead of
  127: per 32-column group g, scale = clip(max|g| / 7, 1e-8) in f32; code = round-half-even(w /
  scale) clipped to [-7, 7]; stored nibble = code + 8 (1..15); scale stored f16. Two codes per
  byte, element 2i in the low nibble (the LUT4 packing order of `_blob.py:41`). IN must be a
  multiple of `group`. Returns (packed [OUT, IN/2] uint8, scales [OUT, IN/group] f16).
  """
  W = np.asarray(W).astype(F32)
  OUT, IN = W.shape
  if IN % group:
    raise ValueError(f"int4 group-{group}: IN={IN} is not a multiple of {group}")
  Wg = W.reshape(OUT, IN // group, group)
  scale = np.clip(np.abs(Wg).max(axis=2) / 7.0, 1e-8, None)
  q = np.round(Wg / scale[:, :, None]).clip(-7, 7).astype(np.int8).reshape(OUT, IN)
  nib = (q + 8).astype(np.uint8)
  packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
  return np.ascontiguousarray(packed), scale.astype(F16)


def dequant_g32_int4(packed: np.ndarray, scale: np.ndarray, group: int = 32) -> np.ndarray:
  OUT = packed.shape[0]
  IN = packed.shape[1] * 2
  nib = np.empty((OUT, IN), np.int8)
  nib[:, 0::2] = (packed & 0x0F).astype(np.int8)
  nib[:, 1::2] = (packed >> 4).astype(np.int8)
  q = (nib - 8).astype(F32).reshape(OUT, IN // group, group)
  return (q * scale.astype(F32)[:, :, None]).reshape(OUT, IN)


class Encoded:
  """One weight after the encoding decision: `kind` in {fp16, int8, lut4, blockwise, sparse,
  int4_g32} and `deq` the fp32 matrix the device multiplies by (the reference's constexpr
  dequant output). `int8_rows` keeps (codes, scale) for int8 so callers can apply the scale
  after the dot product, as the device kernels do."""
  __slots__ = ("kind", "deq", "parts")

  def __init__(self, kind, deq, parts=()):
    self.kind, self.deq, self.parts = kind, deq, parts


def encode_weight(W: np.ndarray, compress: str | None, compress_atol: float = 0.05,
                  block_size: int = 32, allow_int8: bool = True, allow_int4: bool = True,
                  allow_sparse: bool = True, int8: bool | None = None) -> Encoded:
  """Encoding precedence of reference `aneforge/_compile.py:112-188` (`_Emitter.weight`):
  sparse (only if >= half zeros) -> int4 LUT (gated by `compress_atol`, even IN) -> blockwise
  (gated) -> per-row int8 (compress in {"int8", "int4"} or a per-node int8 override) -> fp16.
  `compress="int4_g32"` is this build's group-32 format (no reference counterpart).
  The "auto" mode is the reference's family-dependent union; the B200 build treats every
  encoding as streamable, which is the reference's default set (`_compile.py:73`).
  """
  W2 = np.asarray(W).reshape(W.shape[0], -1)
  auto = compress == "auto"
  if compress == "int4_g32" and allow_int8 and W2.shape[1] % 32 == 0:
    p, s = quantize_g32_int4(W2)
    return Encoded("int4_g32", dequant_g32_int4(p, s).reshape(W.shape), (p, s))
  if (compress == "sparse" or auto) and allow_sparse:
    mask, vals = sparsify(W2)
    if 0 < vals.size <= W2.size // 2:
      return Encoded("sparse", np.asarray(W2, F16).astype(F32).reshape(W.shape), (mask, vals))
  if (compress == "int4" or auto) and allow_int4 and W2.shape[1] % 2 == 0:
    packed, lut = palettize_lut4(W2)
    if lut4_rel_error(W2, packed, lut) <= compress_atol:
      return Encoded("lut4", unpack_lut4(packed, lut, W2.shape).reshape(W.shape), (packed, lut))
  if compress == "blockwise" and allow_int8:
    q, s, nb = quantize_blockwise(W2, block_size)
    if blockwise_rel_error(W2, q, s, nb) <= compress_atol:
      OUT, IN = W2.shape
      deq = (q.astype(F32).reshape(OUT, nb, IN // nb) * s.astype(F32)[:, :, None]).reshape(W.shape)
      return Encoded("blockwise", deq, (q, s, nb))
  use_int8 = int8 if int8 is not None else (compress in ("int8", "int4") or auto)
  if use_int8 and allow_int8:
    q, s = quantize_per_row(W2)
    return Encoded("int8", dequant_per_row(q, s).reshape(W.shape), (q, s))
  return Encoded("fp16", np.asarray(W, F16).astype(F32), ())
