"""Tensor-parallel host logic on the CPU: the shard plan, the sharded weights' algebra (row-parallel
partials sum to the unsharded product, column-parallel pieces concatenate to it), the cross-rank
argmax rule, and the communicator-id exchange over a 2-rank gloo group."""
import os

import numpy as np
import pytest

from aneforge_b200 import tp as TP
from aneforge_b200.llm import LlamaConfig

F32 = np.float32


def test_split_even_covers_and_aligns():
  assert TP.split_even(10, 3) == [(0, 4), (4, 7), (7, 10)]
  parts = TP.split_even(29568, 8, 32)                 # Qwen2-72B FFN: 924 groups of 32 over 8 ranks
  sizes = [(b - a) // 32 for a, b in parts]
  assert sizes == [116, 116, 116, 116, 115, 115, 115, 115]
  assert parts[0][0] == 0 and parts[-1][1] == 29568
  assert all(parts[i][1] == parts[i + 1][0] for i in range(7))
  with pytest.raises(ValueError):
    TP.split_even(100, 3, 32)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_shard_partitions_every_axis(world):
  cfg = LlamaConfig(dim=4096, n_layers=1, n_heads=32, n_kv_heads=8, ffn_dim=14336, vocab=128256)
  shards = [TP.plan_shard(cfg, r, world) for r in range(world)]
  for axis, total in (("q_heads", 32), ("kv_heads", 8), ("ffn", 14336), ("vocab", 128256)):
    spans = [getattr(s, axis) for s in shards]
    assert spans[0][0] == 0 and spans[-1][1] == total
    assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
  assert all((s.ffn[1] - s.ffn[0]) % 32 == 0 for s in shards)
  with pytest.raises(ValueError):
    TP.plan_shard(LlamaConfig(dim=64, n_layers=1, n_heads=4, n_kv_heads=2, ffn_dim=64, vocab=10), 0, 4)


def _layer(rng, D, H, KV, dh, F, bias=True):
  R = lambda *s: rng.standard_normal(s).astype(F32)
  lw = {"wq": R(H * dh, D), "wk": R(KV * dh, D), "wv": R(KV * dh, D), "wo": R(D, H * dh),
        "wgate": R(F, D), "wup": R(F, D), "wdown": R(D, F), "attn_norm": R(D), "mlp_norm": R(D)}
  if bias:
    lw.update(q_bias=R(H * dh), k_bias=R(KV * dh), v_bias=R(KV * dh))
  return lw


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_layer_algebra(world):
  rng = np.random.default_rng(world)
  D, H, KV, dh, F = 64, 8, 4, 8, 96
  cfg = LlamaConfig(dim=D, n_layers=1, n_heads=H, n_kv_heads=KV, ffn_dim=F, vocab=50, head_dim=dh)
  lw = _layer(rng, D, H, KV, dh, F)
  x = rng.standard_normal(D).astype(F32)
  att = rng.standard_normal(H * dh).astype(F32)
  act_full = (x @ lw["wgate"].T) * (x @ lw["wup"].T)
  q, k, v = [], [], []
  o_sum = np.zeros(D, F32)
  d_sum = np.zeros(D, F32)
  for r in range(world):
    s = TP.plan_shard(cfg, r, world)
    sl = TP.shard_layer(lw, cfg, s)
    q.append(x @ sl["wq"].T + sl["q_bias"]); k.append(x @ sl["wk"].T + sl["k_bias"]); v.append(x @ sl["wv"].T + sl["v_bias"])
    a0, a1 = s.q_heads[0] * dh, s.q_heads[1] * dh
    o_sum += att[a0:a1] @ sl["wo"].T
    d_sum += ((x @ sl["wgate"].T) * (x @ sl["wup"].T)) @ sl["wdown"].T
    assert np.array_equal(sl["attn_norm"], lw["attn_norm"])
  np.testing.assert_allclose(np.concatenate(q), x @ lw["wq"].T + lw["q_bias"], rtol=1e-5, atol=1e-4)
  np.testing.assert_allclose(np.concatenate(k), x @ lw["wk"].T + lw["k_bias"], rtol=1e-5, atol=1e-4)
  np.testing.assert_allclose(np.concatenate(v), x @ lw["wv"].T + lw["v_bias"], rtol=1e-5, atol=1e-4)
  np.testing.assert_allclose(o_sum, att @ lw["wo"].T, rtol=1e-4, atol=1e-3)
  np.testing.assert_allclose(d_sum, act_full @ lw["wdown"].T, rtol=1e-4, atol=1e-2)


def test_shard_model_local_config_and_head():
  cfg = LlamaConfig(dim=64, n_layers=2, n_heads=8, n_kv_heads=4, ffn_dim=96, vocab=50, head_dim=8)
  rng = np.random.default_rng(0)
  w = {"embed": rng.standard_normal((50, 64)), "lm_head": rng.standard_normal((50, 64)),
       "final_norm": np.ones(64), "layers": [_layer(rng, 64, 8, 4, 8, 96) for _ in range(2)]}
  s = TP.plan_shard(cfg, 1, 2)
  local, lw = TP.shard_model(cfg, w, s)
  assert (local.n_heads, local.n_kv_heads, local.ffn_dim, local.dim, local.vocab) == (4, 2, 32, 64, 50)
  assert local.dh == 8
  assert np.array_equal(lw["lm_head"], w["lm_head"][25:50]) and lw["embed"] is w["embed"]
  assert lw["layers"][1]["wq"].shape == (32, 64) and lw["layers"][1]["wdown"].shape == (64, 32)


def test_cross_rank_argmax_rule():
  """The combine kernel's rule: best value over the ranks' candidates, ties to the lowest global
  index - identical to the single-device argmax of the concatenated logits."""
  rng = np.random.default_rng(3)
  for _ in range(200):
    V, T = 37, 4
    logits = rng.integers(-3, 3, V).astype(F32)           # many exact ties
    spans = TP.split_even(V, T)
    cands = [(float(logits[a:b].max()), a + int(np.argmax(logits[a:b]))) for a, b in spans]
    best, bi = -np.inf, None
    for v, i in cands:
      if bi is None or v > best or (v == best and i < bi):
        best, bi = v, i
    assert bi == int(np.argmax(logits))


def _gloo_rank(rank, world, port, q):
  import torch.distributed as dist
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world)
  made = {}
  TP.TensorParallel.unique_id = staticmethod(lambda: bytes(range(128)))
  TP.TensorParallel.create = classmethod(lambda cls, r, w, d, uid: made.setdefault("x", (r, w, d, uid)))
  TP.TensorParallel.from_torch_distributed(device=rank, p2p=False)
  dist.barrier()
  dist.destroy_process_group()
  q.put(made["x"])


def test_communicator_id_exchange_over_gloo():
  import multiprocessing as mp
  import socket
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
  ctx = mp.get_context("spawn")
  q = ctx.Queue()
  procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
  for p in procs:
    p.start()
  got = sorted(q.get(timeout=120) for _ in procs)
  for p in procs:
    p.join(timeout=60)
    assert p.exitcode == 0
  assert [g[0] for g in got] == [0, 1] and all(g[1] == 2 and g[3] == bytes(range(128)) for g in got)


class _FakeP2pLib:
  """Stands in for libaf_cuda.so's peer-buffer entry points: a 64-byte handle derived from the rank,
  and a record of the handles each rank opens."""

  def __init__(self, rank, fail=False):
    self.rank, self.fail, self.opened, self.disabled = rank, fail, None, False

  def af_comm_p2p_handle(self, comm, cap, buf, nbytes):
    import ctypes
    ctypes.memmove(buf, bytes([self.rank]) * 64, 64)
    return 0

  def af_comm_p2p_open(self, comm, joined, each):
    self.opened = bytes(joined.raw)
    return -1 if self.fail else 0

  def af_comm_p2p_disable(self, comm):
    self.disabled = True


def _p2p_rank(rank, world, port, fail_rank, q):
  import torch.distributed as dist
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world)
  fake = _FakeP2pLib(rank, fail=rank == fail_rank)
  TP.R.lib = lambda: fake
  tp = TP.TensorParallel(rank, world, rank, handle=object())
  tp._p2p_setup(1024)
  dist.barrier()
  dist.destroy_process_group()
  q.put((rank, tp.p2p, fake.opened, fake.disabled))


@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_peer_buffer_handles_exchanged_in_rank_order(fail_rank):
  """Every rank opens all ranks' handles in rank order; if one rank cannot open them, every rank
  falls back (the peer all-reduce needs all of them)."""
  import multiprocessing as mp
  import socket
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
  ctx = mp.get_context("spawn")
  q = ctx.Queue()
  world = 3
  procs = [ctx.Process(target=_p2p_rank, args=(r, world, port, fail_rank, q)) for r in range(world)]
  for p in procs:
    p.start()
  got = sorted(q.get(timeout=120) for _ in procs)
  for p in procs:
    p.join(timeout=60)
    assert p.exitcode == 0
  want = b"".join(bytes([r]) * 64 for r in range(world))
  for rank, on, opened, disabled in got:
    assert opened == want
    assert on == (fail_rank < 0)
    assert disabled == (fail_rank >= 0 and rank != fail_rank)


# ---------------------------------------------------------------------------- expert parallel

def _ep_rank(rank, world, port, q):
  """One gloo rank of the expert-parallel MoE algebra: route the (replicated) rows with the full
  router, run only the experts this rank's shard holds, and all-reduce the partial outputs."""
  import torch
  import torch.distributed as dist
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world)
  from oracle.model import topk_gate, softmax, silu
  cfg, lw, x = _ep_case()
  s = TP.plan_shard(cfg, rank, world)
  local = TP.shard_layer(lw, cfg, s)
  probs = softmax(x @ local["router"].T)
  gw = topk_gate(probs, 2)
  gw = gw / gw.sum(1, keepdims=True)
  part = np.zeros_like(x)
  for j, e in enumerate(range(*s.experts)):
    act = silu(x @ local["wgate_exps"][j].T) * (x @ local["wup_exps"][j].T)
    part += gw[:, e:e + 1] * (act @ local["wdown_exps"][j])
  t = torch.from_numpy(part)
  dist.all_reduce(t)
  q.put((rank, s.experts, t.numpy()))
  dist.barrier()
  dist.destroy_process_group()


def _ep_case():
  rng = np.random.default_rng(7)
  E, D, F = 8, 32, 48
  cfg = LlamaConfig(dim=D, n_layers=1, n_heads=8, n_kv_heads=4, ffn_dim=F, vocab=20,
                    extra={"n_experts": E, "n_experts_per_tok": 2})
  lw = {"router": rng.standard_normal((E, D)).astype(F32), "wgate_exps": rng.standard_normal((E, F, D)).astype(F32) * 0.2,
        "wup_exps": rng.standard_normal((E, F, D)).astype(F32) * 0.2,
        "wdown_exps": rng.standard_normal((E, F, D)).astype(F32) * 0.2, "mlp_norm": np.ones(D, F32)}
  return cfg, lw, rng.standard_normal((5, D)).astype(F32)


@pytest.mark.parametrize("world", [2])
def test_expert_parallel_dispatch_and_combine_over_gloo(world):
  """Experts split whole over `world` gloo ranks: every expert is held once, and the all-reduce of
  the ranks' partial outputs equals the dense all-expert MoE of the reference (`aneforge/moe.py:48-63`)."""
  import multiprocessing as mp
  import socket
  from oracle.model import topk_gate, softmax, silu
  with socket.socket() as sk:
    sk.bind(("127.0.0.1", 0))
    port = sk.getsockname()[1]
  ctx = mp.get_context("spawn")
  q = ctx.Queue()
  procs = [ctx.Process(target=_ep_rank, args=(r, world, port, q)) for r in range(world)]
  for p in procs:
    p.start()
  got = dict((r, (ex, y)) for r, ex, y in (q.get(timeout=120) for _ in procs))
  for p in procs:
    p.join(timeout=60)
    assert p.exitcode == 0
  spans = sorted(got[r][0] for r in range(world))
  assert spans[0][0] == 0 and spans[-1][1] == 8 and all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
  cfg, lw, x = _ep_case()
  gw = topk_gate(softmax(x @ lw["router"].T), 2)
  gw = gw / gw.sum(1, keepdims=True)
  ref = np.zeros_like(x)
  for e in range(8):
    act = silu(x @ lw["wgate_exps"][e].T) * (x @ lw["wup_exps"][e].T)
    ref += gw[:, e:e + 1] * (act @ lw["wdown_exps"][e])
  for r in range(world):
    np.testing.assert_allclose(got[r][1], ref, rtol=1e-5, atol=1e-5)


def test_expert_parallel_shard_plan():
  cfg = LlamaConfig(dim=4096, n_layers=1, n_heads=32, n_kv_heads=8, ffn_dim=14336, vocab=32000,
                    extra={"n_experts": 8, "n_experts_per_tok": 2})
  for world in (1, 2, 4, 8):
    shards = [TP.plan_shard(cfg, r, world) for r in range(world)]
    assert [s.experts for s in shards] == [(r * 8 // world, (r + 1) * 8 // world) for r in range(world)]
    local, _ = TP.shard_model(cfg, {"layers": [], "lm_head": np.zeros((32000, 4))}, shards[-1])
    assert local.extra["n_experts"] == 8 and local.extra["ep_experts"] == shards[-1].experts
  with pytest.raises(ValueError):
    TP.plan_shard(LlamaConfig(dim=64, n_layers=1, n_heads=4, n_kv_heads=4, ffn_dim=64, vocab=10,
                              extra={"n_experts": 6}), 0, 4)
