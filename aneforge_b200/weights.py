"""Packing reference-layout weights (numpy or torch, host or device) into device-resident fused
projections: the B200 replacement for baking weights into the e5rt BLOBFILE
(`aneforge/_compile.py:112-188`, `_blob.py:67-86`)."""
from __future__ import annotations

import hashlib
import os
from dataclasses import dataclass

import numpy as np

from . import _blob
from . import _runtime as R
from . import layout

F16, F32 = np.float16, np.float32
_HOST_DECIDE_LIMIT = 1 << 22        # run the host encoding gates only on tensors this small


def torch_mod():
  import torch
  return torch


def to_device(a, device, dtype=None):
  """numpy / torch (any device) -> contiguous CUDA tensor on `device`."""
  torch = torch_mod()
  if isinstance(a, torch.Tensor):
    t = a.to(device=device, non_blocking=False)
  else:
    t = torch.from_numpy(np.ascontiguousarray(np.asarray(a))).to(device)
  if dtype is not None:
    t = t.to(dtype)
  return t.contiguous()


def fp16_bits_exact(a) -> bool:
  """True when every value of `a` is exactly representable in fp16."""
  torch = torch_mod()
  if isinstance(a, torch.Tensor):
    return bool(a.dtype == torch.float16 or torch.equal(a.float(), a.half().float()))
  a = np.asarray(a)
  return a.dtype == F16 or bool(np.array_equal(a.astype(F32), a.astype(F16).astype(F32)))


@dataclass
class DevLinear:
  kind: str            # "int8" | "fp16" | "int4_g32"
  w: object            # packed codes / fp16 weights (torch CUDA)
  s: object            # int8: [N] fp16 scales; int4_g32: [N, K/32] fp16; fp16: None
  bias: object         # [N] fp16 or None
  N: int
  K: int
  tiled: bool = False  # int8 / int4_g32 in tensor-core fragment tiles (K % 32 == 0) vs row-major
  group: int = 0       # blockwise: elements per scale
  rowoff: object = None  # sparse: [N + 1] int32 offsets of each row's values in `s`

  @property
  def wf(self) -> str:
    if self.kind == "int8":
      return "i8t" if self.tiled else "i8"
    if self.kind == "int4_g32":
      return "i4t" if self.tiled else "i4"
    if self.kind == "lut4":
      return "l4"
    if self.kind == "blockwise":
      return "i8g"
    if self.kind == "sparse":
      return "sp"
    return "f16"

  @property
  def nbytes(self) -> int:
    n = self.w.numel() * self.w.element_size()
    for t in (self.s, self.rowoff):
      if t is not None:
        n += t.numel() * t.element_size()
    return n


def decide_kind(W, compress, atol=0.05, block_size=32) -> str:
  """The reference policy's encoding kind for one matmul weight (`_compile.py:112-188`)."""
  K = int(W.shape[1])
  if compress is None:
    return "fp16"
  if compress == "int8":
    return "int8"
  if compress == "int4_g32":
    return "int4_g32" if K % 32 == 0 else "fp16"
  numel = int(np.prod(W.shape))
  if numel > _HOST_DECIDE_LIMIT and compress == "int4":
    # the reference's LUT gate on a large near-Gaussian weight: run it on a host copy
    pass
  Wh = W.detach().float().cpu().numpy() if hasattr(W, "detach") else np.asarray(W, F32)
  kind, _ = _blob.decide(Wh, compress, atol, block_size)
  return kind


# Accepted LUT4, blockwise and sparse weights stream packed (`_packed`: 4-bit codes + per-row
# codebook, int8 codes + per-block scales, or a keep bitmask + the kept fp16 values, on the CUDA-core
# GEMVs) when every part of a fused projection takes that encoding and the shape fits (LUT4 and
# sparse: K % 32 == 0; blockwise: blocks a multiple of 16). The rest - projections whose parts
# encode differently, other shapes - run as fp16 matrices of their decoded values on the fp16-weight
# kernels: exact for LUT4 and sparse values; a blockwise weight's int8 x fp16-scale product is then
# rounded to fp16 once.
DENSE_KINDS = ("lut4", "blockwise", "sparse")


def _decoded_fp16(W, compress, atol, block_size):
  """(kind, fp32 matrix of decoded values or None) for one weight: None for the kinds the
  device quantizes itself (int8, int4_g32, fp16)."""
  if compress in (None, "int8", "int4_g32"):
    return decide_kind(W, compress, atol, block_size), None
  Wh = W.detach().float().cpu().numpy() if hasattr(W, "detach") else np.asarray(W, F32)
  W2 = Wh.reshape(Wh.shape[0], -1)
  kind, payload = _blob.decide(Wh, compress, atol, block_size)
  if kind == "lut4":
    return kind, _blob.lut4_dense(W2, *payload).reshape(Wh.shape)
  if kind == "blockwise":
    q, sc, nb = payload
    OUT, IN = W2.shape
    return kind, (q.astype(F32).reshape(OUT, nb, IN // nb) * sc.astype(F32)[:, :, None]).reshape(Wh.shape)
  if kind == "sparse":
    return kind, np.asarray(Wh, np.float16).astype(F32)
  if kind not in ("int8", "fp16", "int4_g32"):
    raise NotImplementedError(f"compress={compress!r}: the {kind} device decoder is not built yet")
  return kind, None


def _quantize(W, kind, device):
  """One matrix -> (codes, scales) on the device (bit-exact to the reference encoders)."""
  from . import kernels
  torch = torch_mod()
  Wd = to_device(W, device)
  if Wd.dtype not in (torch.float16, torch.float32):
    Wd = Wd.float()
  if kind == "int8":
    return kernels.quantize_per_row_i8(Wd)
  if kind == "int4_g32":
    return kernels.quantize_g32_i4(Wd)
  return Wd.half().contiguous(), None


def _packed(parts, compress, atol, block_size):
  """(kind, [(codes, side data)] per part, group) when every part takes the same packed encoding the
  device streams as such - an accepted LUT4 palette (codes 4-bit, one 16-entry fp16 codebook per row,
  K a multiple of 32) or accepted blockwise int8 (one fp16 scale per block, block a multiple of 16)
  - else None."""
  if compress not in ("int4", "blockwise", "auto", "sparse"):
    return None
  hosts = [P.detach().float().cpu().numpy() if hasattr(P, "detach") else np.asarray(P, F32) for P in parts]
  K = hosts[0].shape[1]
  decided = [_blob.decide(W, compress, atol, block_size) for W in hosts]
  kinds = {k for k, _ in decided}
  if len(kinds) != 1:
    return None
  kind = kinds.pop()
  if kind == "sparse" and K % 32 == 0:
    return kind, [(np.asarray(W, np.float16), None) for W in hosts], 0
  if kind == "lut4" and K % 32 == 0:
    return kind, [(packed, np.tile(lut.astype(F16), (W.shape[0], 1))) for W, (_, (packed, lut)) in zip(hosts, decided)], 0
  if kind == "blockwise":
    nbs = {nb for _, (_, _, nb) in decided}
    group = K // nbs.pop() if len(nbs) == 1 else 0
    if group and group % 16 == 0:
      return kind, [(q, s) for _, (q, s, _) in decided], group
  return None


def _encode_sparse(mats, device, swiglu):
  """(mask words [N][K/32] int32, kept values fp16, row offsets [N+1] int32) of the fused fp16
  matrix: the reference's `sparsify` bit order (LSB first) per row, values in column order."""
  torch = torch_mod()
  W = (layout.interleave_blocks(mats[0], mats[1], layout.SWIGLU_HALF) if swiglu
       else np.concatenate(mats, 0) if len(mats) > 1 else mats[0])
  nz = W != 0
  mask = np.packbits(nz, axis=1, bitorder="little").view("<u4").view(np.int32)
  counts = nz.sum(axis=1, dtype=np.int64)
  if counts.sum() >= 2 ** 31:
    raise NotImplementedError("a sparse projection with 2^31 or more kept values")
  rowoff = np.zeros(W.shape[0] + 1, np.int32)
  rowoff[1:] = np.cumsum(counts)
  dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
  vals = W[nz].astype(np.float16)
  return dev(mask), dev(vals if vals.size else np.zeros(1, np.float16)), dev(rowoff)


def _encode_packed(parts, kind, enc, group, device, biases, swiglu) -> DevLinear:
  torch = torch_mod()
  dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
  if kind == "sparse":
    mask, vals, rowoff = _encode_sparse([m for m, _ in enc], device, swiglu)
    N, K = int(mask.shape[0]), int(parts[0].shape[1])
    b = None
    if biases is not None and any(x is not None for x in biases):
      if swiglu:
        raise NotImplementedError("bias on a gate/up projection")
      b = torch.cat([torch.zeros(int(P.shape[0]), dtype=torch.float16, device=device) if x is None
                     else to_device(x, device).float().half() for P, x in zip(parts, biases)]).contiguous()
    return DevLinear("sparse", mask, vals, b, N, K, False, 0, rowoff)
  if swiglu:
    (cg, sg), (cu, su) = enc
    codes = layout.interleave_blocks(cg, cu, layout.SWIGLU_HALF)
    side = layout.interleave_blocks(sg, su, layout.SWIGLU_HALF)
  else:
    codes = np.concatenate([c for c, _ in enc], 0)
    side = np.concatenate([s for _, s in enc], 0)
  N, K = int(codes.shape[0]), int(parts[0].shape[1])
  b = None
  if biases is not None and any(x is not None for x in biases):
    if swiglu:
      raise NotImplementedError("bias on a gate/up projection")
    b = torch.cat([torch.zeros(int(P.shape[0]), dtype=torch.float16, device=device) if x is None
                   else to_device(x, device).float().half() for P, x in zip(parts, biases)]).contiguous()
  w = dev(codes.view(np.uint8) if kind == "lut4" else codes.astype(np.int8))
  return DevLinear(kind, w, dev(side.astype(F16)), b, N, K, False, group)


# ---- content-addressed cache of packed projections (the B200 counterpart of the reference's
# content-addressed program cache, `aneforge/_compile.py:898-923`): the device payload of a
# projection keyed by the SHA-256 of everything that decides it - the format version, compress=,
# the gate tolerance and block size, the fused layout, and every part's and bias's dtype, shape and
# bytes. Host-heavy encodings (the LUT4 palettizer, blockwise, sparse) are then paid once per
# checkpoint. On when AF_WEIGHT_CACHE names a directory (or `set_weight_cache`); AF_FORCE_REPACK=1
# re-encodes and overwrites. Weights given as device tensors are not hashed (no host copy is made).
CACHE_FORMAT = 1
_cache_dir = None


def set_weight_cache(path) -> None:
  """Directory of the packed-projection cache (None: AF_WEIGHT_CACHE, unset: off)."""
  global _cache_dir
  _cache_dir = None if path is None else str(path)


def weight_cache_dir():
  return _cache_dir or os.environ.get("AF_WEIGHT_CACHE") or None


def _host_bytes(a):
  if a is None:
    return b"-"
  if hasattr(a, "detach"):
    if a.device.type != "cpu":
      return None
    a = a.detach().numpy()
  a = np.ascontiguousarray(np.asarray(a))
  return f"{a.dtype.str}{a.shape}".encode(), memoryview(a).cast("B")


def _cache_key(parts, biases, compress, swiglu, atol, block_size):
  h = hashlib.sha256(f"afw{CACHE_FORMAT}|{compress}|{int(swiglu)}|{atol!r}|{block_size}|{len(parts)}".encode())
  for a in list(parts) + list(biases or [None] * len(parts)):
    hb = _host_bytes(a)
    if hb is None:
      return None
    for piece in (hb if isinstance(hb, tuple) else (hb,)):
      h.update(piece)
  return h.hexdigest()


def _cache_load(path, device):
  torch = torch_mod()
  d = torch.load(path, map_location=device, weights_only=True)
  m = d["meta"]
  return DevLinear(m["kind"], d["w"], d.get("s"), d.get("bias"), int(m["N"]), int(m["K"]), bool(m["tiled"]),
                   int(m["group"]), d.get("rowoff"))


def _cache_store(path, lin: DevLinear):
  torch = torch_mod()
  d = {"meta": {"kind": lin.kind, "N": lin.N, "K": lin.K, "tiled": lin.tiled, "group": lin.group},
       "w": lin.w.detach().cpu()}
  for k in ("s", "bias", "rowoff"):
    t = getattr(lin, k)
    if t is not None:
      d[k] = t.detach().cpu()
  os.makedirs(os.path.dirname(path), exist_ok=True)
  tmp = f"{path}.{os.getpid()}.tmp"
  torch.save(d, tmp)
  os.replace(tmp, path)                       # atomic: a concurrent reader sees all or nothing


def encode_linear(parts, compress, device, biases=None, swiglu=False, atol=0.05, block_size=32) -> DevLinear:
  """Encode one or more [N_i, K] matrices sharing their input into one device projection.
  `swiglu=True` takes (gate, up) and interleaves them for the fused silu(gate)*up epilogue;
  otherwise the rows are concatenated (q|k|v). Goes through the packed-projection cache when one is
  configured."""
  root = weight_cache_dir()
  key = _cache_key(parts, biases, compress, swiglu, atol, block_size) if root else None
  if key is None:
    return _encode_linear(parts, compress, device, biases, swiglu, atol, block_size)
  path = os.path.join(root, key[:2], key + ".pt")
  if os.path.exists(path) and os.environ.get("AF_FORCE_REPACK", "0") == "0":
    return _cache_load(path, device)
  lin = _encode_linear(parts, compress, device, biases, swiglu, atol, block_size)
  _cache_store(path, lin)
  return lin


def _encode_linear(parts, compress, device, biases=None, swiglu=False, atol=0.05, block_size=32) -> DevLinear:
  torch = torch_mod()
  packed = _packed(parts, compress, atol, block_size)
  if packed is not None:
    kind, enc, group = packed
    return _encode_packed(parts, kind, enc, group, device, biases, swiglu)
  dec = [_decoded_fp16(P, compress, atol, block_size) for P in parts]
  # a decoded encoding runs as an fp16 matrix of its values (DENSE_KINDS)
  kinds = {"fp16" if k in DENSE_KINDS else k for k, _ in dec}
  if len(kinds) > 1 and "fp16" in kinds:
    # parts of one fused projection that the reference encodes differently (e.g. an accepted LUT
    # for q, per-row int8 for k): all parts run as fp16 matrices of their decoded values
    dec = [(k, d) if d is not None else ("fp16", _blob.dense_of(
        P.detach().float().cpu().numpy() if hasattr(P, "detach") else np.asarray(P, F32), compress,
        compress_atol=atol, block_size=block_size)) for P, (k, d) in zip(parts, dec)]
    kinds = {"fp16"}
  if len(kinds) != 1:
    raise NotImplementedError(f"fused projection parts encode differently: {sorted(k for k, _ in dec)}")
  kind = kinds.pop()
  parts = [P if d is None else torch.from_numpy(np.ascontiguousarray(d)) for P, (_, d) in zip(parts, dec)]
  K = int(parts[0].shape[1])
  enc = [_quantize(P, kind, device) for P in parts]
  if swiglu:
    (wg, sg), (wu, su) = enc
    half = layout.SWIGLU_HALF_TC if kind in ("int8", "int4_g32") else layout.SWIGLU_HALF
    w = layout.interleave_blocks(wg, wu, half)
    s = None if sg is None else layout.interleave_blocks(sg, su, half)
  else:
    w = torch.cat([e[0] for e in enc], 0) if len(enc) > 1 else enc[0][0]
    s = None if enc[0][1] is None else (torch.cat([e[1] for e in enc], 0) if len(enc) > 1 else enc[0][1])
  N = int(w.shape[0])
  b = None
  if biases is not None and any(x is not None for x in biases):
    if swiglu:
      raise NotImplementedError("bias on a gate/up projection")
    cols = []
    for P, x in zip(parts, biases):
      cols.append(torch.zeros(int(P.shape[0]), dtype=torch.float16, device=device) if x is None
                  else to_device(x, device).float().half())
    b = torch.cat(cols, 0).contiguous()
  tiled = False
  if kind == "int8" and K % 32 == 0:
    from . import kernels
    w = kernels.pack_i8_tiles(w.contiguous())          # tensor-core fragment tiles
    tiled = True
  elif kind == "int4_g32":
    from . import kernels
    w = kernels.pack_i4_tiles(w.contiguous(), s.contiguous(), N, K)   # tiles carry their group scales
    s = None
    tiled = True
  elif kind == "int8" and swiglu:
    # the CUDA-core GEMV pairs gate/up rows in blocks of 4: re-interleave at that granularity
    g, u = enc[0][0], enc[1][0]
    w = layout.interleave_blocks(g, u, layout.SWIGLU_HALF)
    s = layout.interleave_blocks(enc[0][1], enc[1][1], layout.SWIGLU_HALF)
  return DevLinear(kind, w.contiguous(), None if s is None else s.contiguous(), b, N, K, tiled)


def rms_weights(gamma, eps, device):
  """(g_eff fp16 tensor, floor float) as the reference bakes them (`_compile.py:738-748`)."""
  g = np.asarray(gamma.detach().float().cpu().numpy() if hasattr(gamma, "detach") else gamma)
  D = int(g.shape[-1])
  g_eff = (g.reshape(1, D).astype(F32) * float(np.sqrt(D))).astype(F16).reshape(D)
  floor = float(np.float16((D * float(eps)) ** 0.5))
  return to_device(g_eff, device), floor


@dataclass
class DevExperts:
  """E experts' SwiGLU weights on the device, each expert's tiles back to back (the layout the expert
  GEMVs index with `w_stride`): gate|up rows interleaved for the fused silu(gate)*up epilogue, down
  with the FFN axis as its contraction."""
  kind: str            # "int8" | "int4_g32"
  gu_w: object         # uint8 [E * gu_bytes]
  gu_s: object         # int8: fp16 [E * 2F] per-row scales; int4_g32: None (scales inside the tiles)
  down_w: object       # uint8 [E * down_bytes]
  down_s: object       # int8: fp16 [E * D] (one scale per expert, repeated per row); int4_g32: None
  E: int
  F: int
  D: int

  @property
  def wf(self) -> str:
    return "i4t" if self.kind == "int4_g32" else "i8t"

  @property
  def nbytes(self) -> int:
    n = self.gu_w.numel() + self.down_w.numel()
    for s in (self.gu_s, self.down_s):
      if s is not None:
        n += s.numel() * 2
    return n


def _per_expert_int8(W):
  """The reference's `bmm_weight` encoding of one expert's down matrix (`aneforge/moe.py:60`, encoded
  as one row of [E, ffn*dim]): one fp32 scale max|W|/127 for the whole expert, codes round-half-even
  of W / scale clipped to +-127, scale stored fp16 - `_blob.quantize_per_row` on that row."""
  torch = torch_mod()
  W32 = W.float()
  s = torch.clamp(W32.abs().max() / 127.0, min=1e-8)
  q = torch.round(W32 / s).clamp(-127, 127).to(torch.int8)
  return q, s.to(torch.float16)


def encode_experts(wgate, wup, wdown, compress, device) -> DevExperts:
  """wgate / wup / wdown: [E, F, D] (reference `moe.py` layout: down stored transposed for act @ w)."""
  from . import kernels
  torch = torch_mod()
  E, F, D = (int(v) for v in wgate.shape)
  kind = "int4_g32" if compress == "int4_g32" else "int8"
  if kind == "int8" and compress not in ("int8", "int4", None):
    raise NotImplementedError(f"expert compress={compress!r}")
  if compress is None:
    raise NotImplementedError("fp16 experts have no tiled device path; use compress='int8' or 'int4_g32'")
  gu_w, gu_s, dn_w, dn_s = [], [], [], []
  for e in range(E):
    g = to_device(wgate[e], device); u = to_device(wup[e], device)
    dT = to_device(wdown[e], device).t().contiguous()         # [D, F]: contraction over F
    if kind == "int8":
      qg, sg = kernels.quantize_per_row_i8(g.half() if g.dtype != torch.float32 else g)
      qu, su = kernels.quantize_per_row_i8(u.half() if u.dtype != torch.float32 else u)
      gu_w.append(kernels.pack_i8_tiles(layout.interleave_blocks(qg, qu, layout.SWIGLU_HALF_TC).contiguous()))
      gu_s.append(layout.interleave_blocks(sg, su, layout.SWIGLU_HALF_TC))
      q, s = _per_expert_int8(dT)
      dn_w.append(kernels.pack_i8_tiles(q.contiguous()))
      dn_s.append(s.reshape(1).expand(D).contiguous())
    else:
      pg, sg = kernels.quantize_g32_i4(g if g.dtype in (torch.float16, torch.float32) else g.float())
      pu, su = kernels.quantize_g32_i4(u if u.dtype in (torch.float16, torch.float32) else u.float())
      pp = layout.interleave_blocks(pg, pu, layout.SWIGLU_HALF_TC).contiguous()
      sp = layout.interleave_blocks(sg, su, layout.SWIGLU_HALF_TC).contiguous()
      gu_w.append(kernels.pack_i4_tiles(pp, sp, 2 * F, D))
      pd, sd = kernels.quantize_g32_i4(dT if dT.dtype in (torch.float16, torch.float32) else dT.float())
      dn_w.append(kernels.pack_i4_tiles(pd, sd, D, F))
  cat = lambda xs: torch.cat(xs).contiguous() if xs else None
  return DevExperts(kind, cat(gu_w), cat(gu_s), cat(dn_w), cat(dn_s), E, F, D)
