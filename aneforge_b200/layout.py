"""Device weight layouts (the B200 re-pack of the reference's `_blob.py` payloads).

* int8 per-row: codes [N][K] row-major + fp16 scales [N] - each 16-byte load is 16 codes of one row,
  so a warp streams 512 contiguous bytes.
* int4 group-32: packed [N][K/2] (element 2i in the low nibble) + fp16 scales [N][K/32]; one 16-byte
  load is exactly one group.
* int8 on the tensor-core GEMV: the per-row codes are re-packed into 16x32 fragment tiles
  (csrc/gemv_tc.cu) so each lane's 16-byte load is exactly its mma.sync A fragment.
* Fused projections: q|k|v rows are concatenated (one GEMV over the shared normalised input); gate
  and up rows are interleaved in blocks (4+4 rows for the CUDA-core GEMV, 8+8 rows = one 16-row
  tile for the tensor-core GEMV) so the epilogue produces silu(gate)*up from rows it already holds.

Packers accept numpy arrays or torch tensors (on any device) and return the same kind.
"""
from __future__ import annotations

import numpy as np

SWIGLU_BLOCK = 8          # rows per gate/up block for the CUDA-core GEMV (must match gemv.cu)
SWIGLU_HALF = SWIGLU_BLOCK // 2
SWIGLU_HALF_TC = 8        # the tensor-core GEMV: each 16-row tile = 8 gate rows + 8 up rows (gemv_tc.cu)


def _cat(parts, like):
  if isinstance(like, np.ndarray):
    return np.concatenate(parts, axis=0)
  import torch
  return torch.cat(parts, dim=0)


def interleave_blocks(g, u, half: int = SWIGLU_HALF):
  """Rows [g0..g3, u0..u3, g4..g7, u4..u7, ...]: blocks of `half` rows of g then of u."""
  F = g.shape[0]
  if F % half:
    raise ValueError(f"gate/up rows ({F}) must be a multiple of {half}")
  rest = tuple(g.shape[1:])
  if isinstance(g, np.ndarray):
    out = np.stack([g.reshape((F // half, half) + rest), u.reshape((F // half, half) + rest)], axis=1)
    return np.ascontiguousarray(out.reshape((2 * F,) + rest))
  import torch
  out = torch.stack([g.reshape((F // half, half) + rest), u.reshape((F // half, half) + rest)], dim=1)
  return out.reshape((2 * F,) + rest).contiguous()


def pack_gate_up(qg, qu, sg, su):
  """int8 codes and per-row scales of gate and up -> the packed swiglu matrix."""
  return interleave_blocks(qg, qu), interleave_blocks(sg, su)


def concat_rows(*mats):
  return _cat(list(mats), mats[0])
