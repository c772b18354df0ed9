"""Tensor parallelism for the decoder: one process per GPU, Megatron-style shards, NCCL collectives
issued inside each rank's program (so they are part of its CUDA graph).

Shards of rank r out of T (no reference counterpart: the ANE runtime is single-device):
  * attention: query heads [r H/T, (r+1) H/T) and kv heads [r KV/T, ...) - q/k/v rows (and biases)
    column-parallel, o_proj columns row-parallel; the KV cache holds only the local kv heads;
  * MLP: gate/up rows column-parallel, down columns row-parallel, split on 32-column groups so the
    group-32 int4 format stays aligned (uneven when F/32 is not a multiple of T);
  * lm_head: vocabulary rows split as evenly as possible; each rank's greedy candidate (best logit,
    global index) is all-gathered and the lowest index among equal best logits wins;
  * embedding, norms and the fp32 residual stream are replicated.
Per layer the exchanges are two all-reduces of the fp32 residual update [NB, D]; per token one
all-gather of NB (value, index) pairs.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace

import numpy as np

from . import _runtime as R


def split_even(n: int, parts: int, quantum: int = 1) -> list[tuple[int, int]]:
  """[start, end) of `parts` contiguous pieces of range(n) in units of `quantum`, sizes differing by
  at most one quantum (the first pieces take the remainder)."""
  if n % quantum:
    raise ValueError(f"{n} is not a multiple of {quantum}")
  units = n // quantum
  base, extra = divmod(units, parts)
  out, s = [], 0
  for i in range(parts):
    u = base + (1 if i < extra else 0)
    out.append((s * quantum, (s + u) * quantum))
    s += u
  return out


@dataclass
class Shard:
  rank: int
  world: int
  q_heads: tuple[int, int]       # local query heads [h0, h1)
  kv_heads: tuple[int, int]      # local kv heads
  ffn: tuple[int, int]           # local FFN rows / down columns
  vocab: tuple[int, int]         # local lm_head rows
  experts: tuple[int, int] = (0, 0)   # mixture of experts: the experts this rank holds (expert parallel)


def plan_shard(cfg, rank: int, world: int) -> Shard:
  """Rank `rank`'s shard. Dense layers split heads and FFN rows (tensor parallel); the experts of a
  mixture-of-experts layer are split whole over the ranks (expert parallel: E / world experts per
  GPU, each with its full FFN), their router replicated."""
  H, KV, F, V = cfg.n_heads, cfg.n_kv_heads, cfg.ffn_dim, cfg.vocab
  if H % world or KV % world:
    raise ValueError(f"tensor parallel {world} needs heads ({H}) and kv heads ({KV}) divisible by it")
  hq, hk = H // world, KV // world
  E = int(cfg.extra.get("n_experts", 0) or 0)
  if E and E % world:
    raise ValueError(f"expert parallel {world} needs the expert count ({E}) divisible by it")
  ex = (rank * E // world, (rank + 1) * E // world) if E else (0, 0)
  return Shard(rank, world, (rank * hq, (rank + 1) * hq), (rank * hk, (rank + 1) * hk),
               split_even(F, world, 32 if F % 32 == 0 else 1)[rank], split_even(V, world)[rank], ex)


def _rows(a, lo, hi):
  return a[lo:hi]


def _cols(a, lo, hi):
  c = a[:, lo:hi]
  return c.contiguous() if hasattr(c, "contiguous") else np.ascontiguousarray(c)


def shard_layer(lw: dict, cfg, s: Shard) -> dict:
  """One layer's weights (reference dict layout) restricted to shard `s`."""
  dh = cfg.dh
  q0, q1 = s.q_heads[0] * dh, s.q_heads[1] * dh
  k0, k1 = s.kv_heads[0] * dh, s.kv_heads[1] * dh
  f0, f1 = s.ffn
  out = {}
  for k, v in lw.items():
    if k in ("wq", "q_bias"):
      out[k] = _rows(v, q0, q1)
    elif k in ("wk", "wv", "k_bias", "v_bias"):
      out[k] = _rows(v, k0, k1)
    elif k == "wo":
      out[k] = _cols(v, q0, q1)
    elif k == "o_bias":
      if s.rank == 0:
        out[k] = v                       # a row-parallel bias is added once
    elif k in ("wgate", "wup"):
      out[k] = _rows(v, f0, f1)
    elif k == "wdown":
      out[k] = _cols(v, f0, f1)
    elif k in ("wgate_exps", "wup_exps", "wdown_exps"):
      out[k] = v[s.experts[0]:s.experts[1]]        # whole experts (expert parallel)
    else:
      out[k] = v                         # norms (attention / MLP / QK-norm) are replicated
  return out


class _ShardedLayers:
  """The layer list of a weights dict, sharded on access (works with lazily generated layers)."""

  def __init__(self, layers, cfg, s: Shard):
    self.layers, self.cfg, self.s = layers, cfg, s

  def __len__(self):
    return len(self.layers)

  def __getitem__(self, i):
    return shard_layer(self.layers[i], self.cfg, self.s)

  def __iter__(self):
    return (self[i] for i in range(len(self)))


def shard_model(cfg, weights: dict, s: Shard):
  """(local config, local weights) of shard `s`. The local config has the local head / FFN counts;
  vocabulary, model width and the embedding stay full; `lm_head` holds the local vocabulary rows."""
  extra = dict(cfg.extra)
  if extra.get("n_experts"):
    extra["ep_experts"] = tuple(s.experts)          # global ids of the local experts; n_experts stays global
  local = replace(cfg, n_heads=s.q_heads[1] - s.q_heads[0], n_kv_heads=s.kv_heads[1] - s.kv_heads[0],
                  ffn_dim=s.ffn[1] - s.ffn[0], head_dim=cfg.dh, extra=extra)
  w = dict(weights)
  w["layers"] = _ShardedLayers(weights["layers"], cfg, s)
  w["lm_head"] = _rows(weights["lm_head"], *s.vocab)
  return local, w


class TensorParallel:
  """A rank's NCCL communicator in libaf_cuda.so plus its shard plan."""

  def __init__(self, rank: int, world: int, device: int, handle):
    self.rank, self.world, self.device, self.handle = rank, world, device, handle
    self.p2p = False

  @staticmethod
  def unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    R.check(R.lib().af_comm_unique_id(buf, 128), "af_comm_unique_id")
    return buf.raw

  @classmethod
  def create(cls, rank: int, world: int, device: int, uid: bytes) -> "TensorParallel":
    h = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(uid, 128)
    R.check(R.lib().af_comm_init(buf, world, rank, device, ctypes.byref(h)), "af_comm_init")
    return cls(rank, world, device, h)

  @classmethod
  def from_torch_distributed(cls, device: int, p2p: bool | None = None, p2p_floats: int = 16 * 8192) -> "TensorParallel":
    """Every rank of the default torch.distributed group calls this: rank 0 makes the NCCL id and
    broadcasts it over the group, then each rank joins with its GPU. With `p2p` (default: on, env
    AF_TP_P2P=0 turns it off) the ranks also map each other's exchange buffers so that the decode's
    residual all-reduces (up to `p2p_floats` fp32 per call) run as one-shot peer-memory kernels;
    if that setup fails on any rank, every rank keeps NCCL for them."""
    import os
    import torch.distributed as dist
    rank, world = dist.get_rank(), dist.get_world_size()
    obj = [cls.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    tp = cls.create(rank, world, device, obj[0])
    if p2p is None:
      p2p = os.environ.get("AF_TP_P2P", "1") != "0"
    if p2p and world > 1:
      tp._p2p_setup(p2p_floats)
    return tp

  def _p2p_setup(self, cap_floats: int) -> None:
    import torch.distributed as dist
    lib = R.lib()
    buf = ctypes.create_string_buffer(64)
    ok = lib.af_comm_p2p_handle(self.handle, cap_floats, buf, 64) == 0
    handles = [None] * self.world
    dist.all_gather_object(handles, buf.raw if ok else None)
    if all(h is not None for h in handles):
      joined = ctypes.create_string_buffer(b"".join(handles), 64 * self.world)
      ok = lib.af_comm_p2p_open(self.handle, joined, 64) == 0
    else:
      ok = False
    flags = [None] * self.world
    dist.all_gather_object(flags, ok)
    self.p2p = all(flags)
    if ok and not self.p2p:
      # a peer could not map the buffers: nobody uses the peer path (it needs every rank)
      lib.af_comm_p2p_disable(self.handle)

  def close(self) -> None:
    if self.handle:
      R.lib().af_comm_destroy(self.handle)
      self.handle = None
