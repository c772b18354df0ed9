"""Tensor-parallel decode on 2 GPUs (needs >= 2 CUDA devices; skipped otherwise): each rank runs its
shard (local heads / FFN rows / vocabulary rows) with NCCL all-reduces inside its program; the
greedy tokens must pass the same oracle check as the single-GPU path (equal to the oracle's argmax
except inside the reference's tie margin), for int8 and group-32 int4 weights."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _cfg(case):
  from oracle.model import Config
  if case == "moe":
    # Mixtral-like: attention int8 (tensor parallel), 8 group-32 int4 experts (expert parallel, 4 per GPU)
    return Config(dim=512, n_layers=2, n_heads=8, n_kv_heads=2, ffn_dim=384, vocab=2048, rope_base=10000.0,
                  head_dim=64, extra={"n_experts": 8, "n_experts_per_tok": 2, "norm_topk_prob": True}), {"moe": True}
  if case == "int8":
    return Config(dim=1024, n_layers=2, n_heads=8, n_kv_heads=2, ffn_dim=3584, vocab=4096, rope_base=500000.0), {}
  return Config(dim=1024, n_layers=2, n_heads=8, n_kv_heads=2, ffn_dim=2816, vocab=4096, rope_base=1e6), {"qkv_bias": True}


def _rank(rank, world, port, case, prompt, q, p2p):
  import torch.distributed as dist
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  torch.cuda.set_device(rank)
  dist.init_process_group("gloo", rank=rank, world_size=world)
  from oracle.model import random_llama_weights
  from tests.test_llm_gpu import to_b200_cfg
  from aneforge_b200.llm import LlamaPrefill
  from aneforge_b200.tp import TensorParallel
  cfg, extra = _cfg(case)
  w = _weights(case, cfg, extra)
  tp = TensorParallel.from_torch_distributed(rank, p2p=p2p)
  assert tp.p2p == p2p
  if case == "moe":
    from tests.test_moe_gpu import _b200_cfg
    m = LlamaPrefill(_b200_cfg(cfg), w, compress="int8", device=rank, tp=tp, moe_compress="int4_g32")
  else:
    m = LlamaPrefill(to_b200_cfg(cfg), w, compress="int8" if case == "int8" else "int4_g32", device=rank, tp=tp)
  toks = m.generate(prompt, 24, max_len=64)
  m.release()
  tp.close()
  dist.barrier()
  dist.destroy_process_group()
  q.put((rank, toks))


def _weights(case, cfg, extra):
  from oracle.model import random_llama_weights
  if case != "moe":
    return random_llama_weights(cfg, seed=21, **extra)
  w = random_llama_weights(cfg, seed=21, std=0.05, moe=True)
  for lw in w["layers"]:
    # a well-separated router: no top-k choice sits on a near tie (see tests/test_moe_gpu.py)
    lw["router"] = (lw["router"].astype(np.float32) * 10).astype(np.float16)
  return w


@pytest.mark.parametrize("case,p2p", [("int8", False), ("int8", True), ("int4_g32", True), ("moe", True)])
def test_tensor_parallel_2_gpus_matches_oracle(case, p2p):
  """NCCL for every collective, or the residual all-reduces over NVLink peer memory; `moe`: the
  Mixtral-like model with tensor-parallel attention and expert-parallel experts (4 of 8 per GPU,
  combined by the all-reduce)."""
  if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs 2 GPUs")
  import multiprocessing as mp
  import socket
  from oracle.model import OracleModel, random_llama_weights
  from tests.test_llm_gpu import teacher_forced_check
  cfg, extra = _cfg(case)
  prompt = [int(t) for t in np.random.default_rng(22).integers(0, cfg.vocab, 31)]
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
  ctx = mp.get_context("spawn")
  q = ctx.Queue()
  procs = [ctx.Process(target=_rank, args=(r, 2, port, case, prompt, q, p2p)) for r in range(2)]
  for p in procs:
    p.start()
  got = dict(q.get(timeout=600) for _ in procs)
  for p in procs:
    p.join(timeout=120)
    assert p.exitcode == 0
  assert got[0] == got[1] and len(got[0]) == 24
  w = _weights(case, cfg, extra)
  if case == "moe":
    om = OracleModel(cfg, w, "int8", precision="device", moe_compress="int4_g32")
  else:
    om = OracleModel(cfg, w, "int8" if case == "int8" else "int4_g32", precision="device")
  assert teacher_forced_check(om, prompt, got[0], 64, n_check=24) <= 2
