"""Benchmark: int8 decode tokens/s of a Llama-3-8B-shaped model (the headline decode workload) on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl reference]

One step = one decode token for each of the B sequences (B = 1 by default), all 32 layers, the
final norm, the lm_head and the greedy argmax, replayed as one CUDA graph over a device-resident
KV cache. Weights are random N(0, 0.02) (no checkpoints here), quantized per row to int8 on the
GPU with the reference's encoder; the prompt is 512 uniform token ids, prefilled before timing.

Under torchrun (N > 1) the model runs tensor parallel over the N GPUs (strong scaling: heads, FFN
rows and vocabulary split, residual all-reduces over NVLink peer memory; experts split whole for the
MoE model); `--replicas` runs N independent copies instead (weak scaling). The timed region is
bracketed by a barrier + device sync on every rank and the slowest rank's time is reported.

`--impl reference` times the reference algorithm's CPU path (the numpy restatement of ANEForge's
decode driver in `oracle/`, run with every host thread BLAS offers) on the same workload, on a
bounded sample: a few decode steps of a 2-layer slice of the same model plus its lm_head, scaled to
32 layers.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# The benchmarked models (random-init, seeded; no checkpoints). `--model` picks one; the default is
# the Llama-3-8B-shaped int8 decode the headline metric is quoted on.
MODELS = {
  "llama3-8b": dict(
    cfg=dict(dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, ffn_dim=14336, vocab=128256, rope_base=500000.0,
             norm_eps=1e-5),
    compress="int8", prompt=512, qkv_bias=False, traffic_profile="gemv_tc_gate_up_llama8b.md",
    chain_traffic_profile="gemv_chain_llama8b.md",
    metric="int8 decode tokens/s (Llama-3-8B-shaped, greedy)",
    workload="config 3: Llama-3-8B-shaped int8 per-row greedy decode",
    dtype="int8 weights, fp16 activations, fp32 accumulation"),
  "qwen2-72b": dict(
    cfg=dict(dim=8192, n_layers=80, n_heads=64, n_kv_heads=8, ffn_dim=29568, vocab=152064, rope_base=1e6,
             norm_eps=1e-6),
    compress="int4_g32", prompt=2048, qkv_bias=True, traffic_profile="gemv_tc_i4_gate_up_qwen72b.md",
    chain_traffic_profile="gemv_chain_i4_qwen72b.md",
    metric="int4 decode tokens/s (Qwen2-72B-shaped, greedy)",
    workload="config 4: Qwen2-72B-shaped group-32 int4 greedy decode",
    dtype="int4 group-32 weights, fp16 activations, fp32 accumulation"),
  "mixtral-8x7b": dict(
    cfg=dict(dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, ffn_dim=14336, vocab=32000, rope_base=1e6,
             norm_eps=1e-5, extra={"n_experts": 8, "n_experts_per_tok": 2, "norm_topk_prob": True}),
    compress="int8", moe_compress="int4_g32", prompt=1024, qkv_bias=False, moe=True,
    traffic_profile="gemv_tc_i4_expert_gate_up_mixtral.md",
    metric="int4-expert MoE decode tokens/s (Mixtral-8x7B-shaped, greedy)",
    workload="config 5: Mixtral-8x7B-shaped MoE greedy decode, group-32 int4 experts, int8 attention",
    dtype="int4 group-32 expert weights, int8 attention weights, fp16 activations, fp32 accumulation"),
}
MODEL = "llama3-8b"
CFG = MODELS[MODEL]["cfg"]
PROMPT = MODELS[MODEL]["prompt"]
METRIC = MODELS[MODEL]["metric"]


def select_model(name):
  global MODEL, CFG, PROMPT, METRIC
  MODEL, CFG, PROMPT, METRIC = name, MODELS[name]["cfg"], MODELS[name]["prompt"], MODELS[name]["metric"]


def _dist():
  ws = int(os.environ.get("WORLD_SIZE", "1"))
  rank = int(os.environ.get("RANK", "0"))
  local = int(os.environ.get("LOCAL_RANK", "0"))
  return ws, rank, local


def _peaks():
  try:
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
      p = json.load(f)
    return float(p["hbm_gbs"]), "measured"
  except Exception:
    return 6650.0, "fallback"


class ClockSampler:
  """SM clocks and throttle reasons of one GPU sampled every 200 ms through NVML (in-process: no
  nvidia-smi child processes competing with the timed region)."""

  _REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20), ("hw_thermal_slowdown", 0x40),
              ("sw_power_cap", 0x4))

  def __init__(self, index: int):
    self.index, self.samples, self._stop = index, [], threading.Event()
    self._t = threading.Thread(target=self._run, daemon=True)
    self._h = None
    try:
      import pynvml
      pynvml.nvmlInit()
      self._nv = pynvml
      self._h = pynvml.nvmlDeviceGetHandleByIndex(self._physical_index(index))
    except Exception:
      self._h = None

  @staticmethod
  def _physical_index(index):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v.strip() for v in vis.split(",") if v.strip()]
    return int(ids[index]) if index < len(ids) and ids[index].isdigit() else index

  def _sample(self):
    nv, h = self._nv, self._h
    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
    mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
    mask = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
    self.samples.append((sm, mx, mask))

  def _run(self):
    while not self._stop.is_set():
      try:
        self._sample()
      except Exception:
        pass
      self._stop.wait(0.2)

  def __enter__(self):
    if self._h is not None:
      self._t.start()
    return self

  def __exit__(self, *a):
    self._stop.set()
    if self._t.is_alive():
      self._t.join(timeout=10)
    if self._h is not None:
      try:
        self._sample()                      # at least one sample at the end of the region
      except Exception:
        pass

  def summary(self):
    if not self.samples:
      return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
    sm = [s[0] for s in self.samples]
    reasons = sorted({n for s in self.samples for n, bit in self._REASONS if s[2] & bit})
    return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(s[1] for s in self.samples), "reasons": reasons,
            "samples": len(self.samples), "source": "nvml"}


def make_weights(cfg, device, seed=0, qkv_bias=False, moe=False):
  """Seeded N(0, 0.02) fp16 weights generated on the device (`aneforge_b200.synthetic`)."""
  from aneforge_b200.synthetic import make_weights as mw
  return mw(cfg, device, seed=seed, qkv_bias=qkv_bias, moe=moe)


def decode_cache_len(args):
  """Cache rows of the timed decode program: every step (warm-up, timed, e2e) fits."""
  e2e_steps = max(8, args.steps // 2)
  return PROMPT + args.warmup + args.steps + e2e_steps + 8, e2e_steps


def workload_config(args, ws, tp_on):
  """The `config` object of the JSON line; both arms print the same one."""
  spec = MODELS[MODEL]
  NB = args.batch
  units = 1 if tp_on else ws
  M, _ = decode_cache_len(args)
  from types import SimpleNamespace
  cfg = SimpleNamespace(**{k: v for k, v in CFG.items() if k != "extra"}, extra=CFG.get("extra", {}),
                        dh=CFG["dim"] // CFG["n_heads"])
  step_bytes = algorithmic_bytes_per_step(cfg, NB, PROMPT + args.warmup + args.steps // 2, spec["compress"],
                                          spec["qkv_bias"], spec.get("moe_compress"))
  return {"workload": spec["workload"], "model": MODEL + "-shaped", "global_batch": NB * units, "batch_per_gpu": NB,
          "seq_len": PROMPT, "decode_pos": f"{PROMPT}..{M}",
          "parallelism": f"tp{ws}" if tp_on else (f"replicas{ws}" if ws > 1 else "single"),
          "l2": f"weights {step_bytes / 1e9:.1f} GB per step >> 126 MB L2 (no flush needed)"}


def host_info():
  """The host cores the CPU baseline ran on."""
  model = None
  try:
    out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
    for line in out.splitlines():
      if line.lower().startswith("model name"):
        model = line.split(":", 1)[1].strip()
        break
  except Exception:
    pass
  return {"cpu_count": os.cpu_count(), "lscpu_model": model, "blas_threads": blas_threads()}


def _proj_bytes(n_params, rows, fmt):
  """Codes + fp16 scales of one projection in a weight format."""
  if fmt == "int4_g32":
    return n_params // 2 + 2 * (n_params // 32)
  return n_params + 2 * rows


def algorithmic_bytes_per_step(cfg, NB, pos, compress="int8", qkv_bias=False, moe_compress=None):
  """Bytes a decode step must move once (each byte counted once per step): codes + fp16 scales of every
  projection (int8: 1 B/param + one scale per row; int4_g32: 0.5 B/param + one scale per 32), qkv
  biases, the fp16 lm_head, norms, KV cache read (positions 0..pos) + the new slot write, and the
  step's activations in/out."""
  D, H, KV, dh, F, V, L = cfg.dim, cfg.n_heads, cfg.n_kv_heads, cfg.dh, cfg.ffn_dim, cfg.vocab, cfg.n_layers
  if cfg.extra.get("n_experts"):
    # MoE: attention + router in `compress`; the experts a step reads in `moe_compress` - the top k at
    # batch 1, every expert once for larger batches (each expert's routed rows share one pass)
    E, k = cfg.extra["n_experts"], cfg.extra["n_experts_per_tok"]
    attn = _proj_bytes((H + 2 * KV) * dh * D, (H + 2 * KV) * dh, compress) + _proj_bytes(D * H * dh, D, compress)
    router = _proj_bytes(E * D, E, compress)
    expert = _proj_bytes(2 * F * D, 2 * F, moe_compress) + _proj_bytes(D * F, D, moe_compress)
    per_layer = attn + router + (k if NB == 1 else E) * expert + 2 * D * 2
    kv = L * NB * (2 * KV * (pos + 1) * dh * 2)
    return L * per_layer + V * D * 2 + D * 2 + kv + NB * (4 + 4)
  proj_rows = (H + 2 * KV) * dh + D + 2 * F + D
  proj_params = ((H + 2 * KV) * dh * D) + D * H * dh + 2 * F * D + D * F
  if compress == "int4_g32":
    per_layer = proj_params // 2 + 2 * (proj_params // 32) + 2 * D * 2
  else:
    per_layer = proj_params + 2 * proj_rows + 2 * D * 2
  if qkv_bias:
    per_layer += 2 * (H + 2 * KV) * dh
  kv = L * NB * (2 * KV * (pos + 1) * dh * 2)
  return L * per_layer + V * D * 2 + D * 2 + kv + NB * (4 + 4)


class _ExpertGU:
  """Expert e's fused gate|up projection of a layer, shaped like a DevLinear for the timing loop."""

  def __init__(self, ex, e):
    self.ex, self.e, self.kind = ex, e, "expert-" + ex.kind
    self.N, self.K = 2 * ex.F, ex.D
    self.nbytes = (ex.gu_w.numel() + (ex.gu_s.numel() * 2 if ex.gu_s is not None else 0)) // ex.E


def _run_lin(kernels, R, x, lin, y, scr):
  """One fused gate|up projection launch in whatever tiled format the loader chose."""
  if isinstance(lin, _ExpertGU):
    ex = lin.ex
    kernels.gemv_tc_expert(x, ex.gu_w, ex.gu_s, lin.N, lin.K, ex.E, wf=R.W_I4G32 if ex.kind == "int4_g32" else R.W_I8,
                           epi=R.EPI_SWIGLU, y=y, fixed_e=lin.e, scratch=scr)
  elif lin.kind == "int4_g32":
    kernels.gemv_tc_i4(x, lin.w, lin.N, lin.K, epi=R.EPI_SWIGLU, y=y, scratch=scr)
  else:
    kernels.gemv_tc(x, lin.w, lin.s, lin.N, lin.K, epi=R.EPI_SWIGLU, y=y, scratch=scr)


def chain_bytes(pb, kv, NB):
  """Algorithmic bytes of one `gemv_chain` launch: every job's packed weights, scales and bias,
  its x rows in, its y rows out (plus the residual read for a residual epilogue), and each norm's
  fp32 rows in, gamma and fp16 rows out."""
  total = 0
  for j in range(int(kv["jobs"])):
    p = f"j{j}."
    n, k, epi = int(kv[p + "n"]), int(kv[p + "k"]), kv[p + "epi"]
    for key in ("w", "s", "b"):
      if p + key in kv:
        total += pb.bufs[kv[p + key]].nbytes
    out = n // 2 if epi == "swiglu" else n
    total += NB * k * 2 + NB * out * (2 if epi in ("swiglu", "f16") else 4) + (NB * n * 4 if epi == "resid" else 0)
    if p + "nd" in kv:
      d = int(kv[p + "nd"])
      total += NB * d * 4 + d * 2 + NB * d * 2
  return total


def time_chains(m, dec, NB, reps=4):
  """The decode step's `gemv_chain` launches (o, norm, gate|up, down, norm, next qkv of every layer)
  replayed alone as one program on its own stream, timed with CUDA events: (us per launch,
  algorithmic bytes per launch). The layers' weights (several GB, above L2) stream from HBM."""
  import torch
  from aneforge_b200 import _runtime as R
  from aneforge_b200.plan import PlanBuilder
  pb = dec["plan"]
  ops = [(k, kv) for k, kv in pb.ops if k == "gemv_chain"]
  if not ops:
    return None
  # the layers' weights (bound below), the chain's own buffers and the final norm; not the embedding,
  # head or rope tables of the decode program
  keep = {n: b for n, b in pb.bufs.items() if b.role != "weight" or n.startswith("L") or n == "final_g"}
  sub = PlanBuilder(bufs=keep, ops=list(ops))
  prog = R.Program.from_text(sub.text(), {}, {}, m.device)
  d = m._load()
  for li in range(m.cfg.n_layers):
    m._bind_layer(prog, li, d["layers"][li])
  prog.bind("final_g", d["final_g"])
  for _ in range(2):
    prog.execute_async()
  prog.sync()
  stream = torch.cuda.ExternalStream(prog.stream(), device=torch.device("cuda", m.device))
  e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  e0.record(stream)
  for _ in range(reps):
    prog.execute_async()
  e1.record(stream)
  prog.sync()
  torch.cuda.synchronize()
  us = e0.elapsed_time(e1) * 1e3 / (reps * len(ops))
  nbytes = sum(chain_bytes(pb, kv, NB) for _, kv in ops) / len(ops)
  del stream
  prog.release()
  return us, nbytes


def run_b200(args):
  import torch
  import torch.distributed as dist
  from aneforge_b200 import llm as L, _runtime as R, kernels
  ws, rank, local = _dist()
  torch.cuda.set_device(local)
  dev = torch.device("cuda", local)
  if ws > 1:
    dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=600))
  tp = None
  if ws > 1 and not args.replicas:
    # one model sharded over the ranks (tensor parallel, strong scaling): same weights and prompt on
    # every rank; with --replicas every rank runs its own replica on its own sequences (weak scaling)
    from aneforge_b200.tp import TensorParallel
    tp = TensorParallel.from_torch_distributed(local)
  spec = MODELS[MODEL]
  mlp = "moe" if spec.get("moe") else "swiglu"
  cfg = L.LlamaConfig(**CFG, layers=[L.LayerSpec(mlp=mlp) for _ in range(CFG["n_layers"])])
  NB = args.batch
  t_load = time.perf_counter()
  w = make_weights(cfg, dev, seed=1234 + (0 if tp else rank), qkv_bias=spec["qkv_bias"], moe=bool(spec.get("moe")))
  m = L.LlamaPrefill(cfg, w, compress=spec["compress"], device=local, tp=tp,
                     moe_compress=spec.get("moe_compress", "same"))
  m._load()
  del w
  torch.cuda.empty_cache()
  load_s = time.perf_counter() - t_load
  M, e2e_steps = decode_cache_len(args)
  rng = np.random.default_rng(99 + (0 if tp else rank))
  prompts = [list(rng.integers(0, cfg.vocab, PROMPT)) for _ in range(NB)]
  dec = m._decoder(M, NB)
  prog = dec["prog"]
  m._reset_state(dec)
  first, pos = [], []
  t_pf = time.perf_counter()
  for b, p in enumerate(prompts):
    pre, real, _ = m._prefill_hidden(p)
    hid = pre["prog"].read_output("hid")
    first.append(int(np.argmax(m._logits(hid[real - 1]))))
    m._seed_cache(dec, pre, real, slot=b)
    pos.append(real)
  torch.cuda.synchronize()
  prefill_s = time.perf_counter() - t_pf
  prog.set_input("tok", np.array(first, np.int32)); prog.set_input("pos", np.array(pos, np.int32))
  stream = torch.cuda.ExternalStream(prog.stream(), device=dev)
  for _ in range(args.warmup):
    prog.execute_async()
  prog.sync()
  # the clock sampler (NVML set-up can take a while, differently on each rank) starts before the
  # barrier, so every rank enters the timed region together: a rank that started late would hold
  # the others in their all-reduce waits and their timers would count it
  clk = ClockSampler(local)
  with clk:
    if ws > 1:
      dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.profile_region:
      torch.cuda.profiler.start()       # ncu --profile-from-start off sees the timed steps only
    e0.record(stream)
    for _ in range(args.steps):
      prog.execute_async()
    e1.record(stream)
    prog.sync()
  if args.profile_region:
    torch.cuda.profiler.stop()
  torch.cuda.synchronize()
  ms = e0.elapsed_time(e1)
  if ws > 1:
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    dist.barrier()
  ms_step = ms / args.steps
  units = 1 if tp else ws                                  # sequences advanced per step, whole job
  tok_s = NB * args.steps * units / (ms / 1e3)
  launches_per_step = sum(1 for _ in dec["plan"].ops)

  # ---- end-to-end through the public program API with host buffers: per step one H2D of the
  # input token ids (pinned host -> tok port) and one D2H of the produced ids
  host_tok = torch.empty(NB, dtype=torch.int32).pin_memory()
  host_out = torch.empty(NB, dtype=torch.int32).pin_memory()
  tok_dev = prog.tensor("tok", (NB,), "int32")
  out_dev = prog.tensor("tok_out", (NB,), "int32")
  host_tok.copy_(out_dev.cpu())
  torch.cuda.synchronize()
  t0 = time.perf_counter()
  with torch.cuda.stream(stream):
    for _ in range(e2e_steps):
      tok_dev.copy_(host_tok, non_blocking=True)
      prog.execute_async()
      host_out.copy_(out_dev, non_blocking=True)
      stream.synchronize()
      host_tok.copy_(host_out)
  e2e_s = time.perf_counter() - t0
  prog.sync()                                              # raises if any step recorded a device error
  e2e_tok_s = NB * e2e_steps * units / e2e_s

  # ---- dominant kernel: the fused gate|up int8 GEMV, timed alone on the program stream over the
  # 32 layers' own weights (3.7 GB > L2, so every launch streams from HBM)
  if "experts" in m._dev["layers"][0]:
    # MoE: one expert's gate|up (2 F x D) per launch, cycling over the layers' experts (the ones this
    # GPU holds: all of them, or its share under expert parallelism)
    E = m._dev["layers"][0]["experts"].E
    gu = [_ExpertGU(m._dev["layers"][i]["experts"], e) for i in range(cfg.n_layers) for e in range(E)][:4 * cfg.n_layers]
  else:
    gu = [m._dev["layers"][i]["gu"] for i in range(cfg.n_layers)]
  x = torch.randn(NB, cfg.dim, device=dev).half()
  y = torch.empty(NB, cfg.ffn_dim, device=dev, dtype=torch.float16)
  reps = 3 * len(gu)
  scr, _ = kernels.gemv_tc_scratch(gu[0].N, gu[0].K, NB, dev)
  with torch.cuda.stream(stream):
    for l in gu:
      _run_lin(kernels, R, x, l, y, scr)
    torch.cuda.synchronize()
    kgraph = torch.cuda.CUDAGraph()                       # launches back to back, not paced by the host
    with torch.cuda.graph(kgraph, stream=stream):
      for i in range(reps):
        _run_lin(kernels, R, x, gu[i % len(gu)], y, scr)
    kgraph.replay()
    torch.cuda.synchronize()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record(stream)
    kgraph.replay()
    k1.record(stream)
  torch.cuda.synchronize()
  k_us = k0.elapsed_time(k1) * 1e3 / reps
  del kgraph
  gu_bytes = gu[0].nbytes + NB * cfg.dim * 2 + NB * cfg.ffn_dim * 2
  chain = time_chains(m, dec, NB)
  peak, peak_kind = _peaks()
  step_bytes = algorithmic_bytes_per_step(cfg, NB, PROMPT + args.warmup + args.steps // 2, spec["compress"],
                                          spec["qkv_bias"], spec.get("moe_compress"))
  result = None
  if rank == 0:
    achieved = gu_bytes / (k_us * 1e-6) / 1e9
    peak_note = f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback"
    gate_up = {"kernel": f"gemv_tc {gu[0].kind} gate|up + silu*mul ({gu[0].N}x{gu[0].K}, mma.sync)",
               "achieved": round(achieved, 1), "frac": round(achieved / peak, 4), "launch_us": round(k_us, 2),
               "algorithmic_bytes": gu_bytes}
    if chain is not None:
      c_us, c_bytes = chain
      c_ach = c_bytes / (c_us * 1e-6) / 1e9
      roofline = {"bound": "hbm", "kernel": "gemv_chain_kernel: o, rmsnorm, gate|up, down, rmsnorm, next qkv "
                                            "(one persistent launch per layer, mma.sync)",
                  "achieved": round(c_ach, 1), "peak": peak, "unit": "GB/s", "frac": round(c_ach / peak, 4),
                  "traffic": profile_traffic(spec.get("chain_traffic_profile", "")),
                  "traffic_source": f"ncu dram__bytes_read.sum + dram__bytes_write.sum, profiles/{spec.get('chain_traffic_profile')}",
                  "peak_kind": peak_note, "launch_us": round(c_us, 2), "algorithmic_bytes": int(c_bytes),
                  "how": "the step's chain launches replayed alone as one program, CUDA events on its stream",
                  "gate_up_alone": gate_up}
    else:
      roofline = {"bound": "hbm", "kernel": gate_up["kernel"], "achieved": gate_up["achieved"], "peak": peak,
                  "unit": "GB/s", "frac": gate_up["frac"], "traffic": profile_traffic(spec["traffic_profile"]),
                  "traffic_source": f"ncu dram__bytes_read.sum + dram__bytes_write.sum, profiles/{spec['traffic_profile']}",
                  "peak_kind": peak_note, "launch_us": gate_up["launch_us"], "algorithmic_bytes": gu_bytes}
    result = {
      "metric": METRIC, "value": round(tok_s, 2), "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
      "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
      "scaling": "strong" if tp else "weak",
      "vs_baseline": None, "dtype": spec["dtype"], "data": "synthetic",
      "config": workload_config(args, ws, tp is not None),
      "e2e": {"value": round(e2e_tok_s, 2), "unit": "tokens/s", "h2d_bytes_per_step": 4 * NB,
              "d2h_bytes_per_step": 4 * NB,
              "how": "program API, pinned host token ids in/out every step, host sync per step"},
      "roofline": roofline,
      "step_roofline": {"algorithmic_bytes": int(step_bytes), "achieved_gbs": round(step_bytes / (ms_step * 1e-3) / 1e9, 1),
                        "frac": round(step_bytes / (ms_step * 1e-3) / 1e9 / peak / (ws if tp else 1), 4),
                        "per": "GPU (the model's bytes are split over the tensor-parallel ranks)" if tp else "GPU"},
      "gpu_launches": launches_per_step * args.steps,
      "clocks": clk.summary(),
      "load_s": round(load_s, 2), "prefill_s": round(prefill_s, 3),
    }
  # torch objects that touched the program's stream go before the stream itself
  del host_tok, host_out, tok_dev, out_dev, x, y, gu, scr, stream
  torch.cuda.synchronize()
  import gc
  gc.collect()

  # ---- end to end through `LlamaPrefill.generate` (the reference's public call, llm.py:560-633):
  # host prompt ids in, the benchmark prompt prefilled, `--gen-tokens` greedy tokens back on the
  # host. One untimed call builds the programs; then the time to first token (prefill + the head's
  # argmax) and the whole call are timed on the host clock (each call ends with a device sync)
  gen = None
  G = args.gen_tokens
  if NB == 1 and G > 0:
    Mg = PROMPT + G + 8
    p0 = prompts[0]
    m.generate(p0, G, max_len=Mg)
    if ws > 1:
      dist.barrier()
    t0 = time.perf_counter()
    m.generate(p0, 1, max_len=Mg)
    ttft = time.perf_counter() - t0
    if ws > 1:
      dist.barrier()
    t0 = time.perf_counter()
    toks = m.generate(p0, G, max_len=Mg)
    total = time.perf_counter() - t0
    if ws > 1:
      t = torch.tensor([ttft, total], device=dev, dtype=torch.float64)
      dist.all_reduce(t, op=dist.ReduceOp.MAX)
      ttft, total = (float(v) for v in t.tolist())
    gen = {"tokens": len(toks), "prompt": PROMPT, "ttft_ms": round(ttft * 1e3, 2), "total_s": round(total, 4),
           "tokens_per_s": round(len(toks) / total, 2),
           "decode_tokens_per_s": round((len(toks) - 1) / max(total - ttft, 1e-9), 2),
           "h2d_bytes": 4 * PROMPT, "d2h_bytes": 4 * len(toks),
           "how": "LlamaPrefill.generate(prompt, max_new_tokens) on host ids, TTFT included, max over ranks"}
  if result is not None and gen is not None:
    result["e2e"]["generate"] = gen
  m.release()
  if tp is not None:
    tp.close()
  if ws > 1:
    dist.barrier()
    dist.destroy_process_group()
  return result


def kernel_bench(name, reps, warmup, nb=1):
  """One hot kernel alone on the device (the `--kernel` mode; the small case the ncu summaries in
  profiles/ are captured on). Weights rotate over enough copies that every launch streams from HBM.
  Returns a dict with the launch time (CUDA events on the launching stream) and algorithmic GB/s."""
  import torch
  from aneforge_b200 import kernels as K, _runtime as R
  from aneforge_b200.llm import rope_tables
  dev = torch.device("cuda", 0)
  torch.cuda.set_device(dev)
  g = torch.Generator(device=dev)
  g.manual_seed(7)
  D, F, H, KV, dh, V = CFG["dim"], CFG["ffn_dim"], CFG["n_heads"], CFG["n_kv_heads"], 128, CFG["vocab"]
  st = torch.cuda.Stream(dev)
  if name in ("prefill", "prefill_1layer"):
    # the whole prefill program of the selected model over its benchmark prompt (time to first hidden
    # state: embed, per layer norm + tcgen05 GEMMs + RoPE / cache write + causal attention, final norm);
    # `prefill_1layer` is one layer of it with a 4096-token vocabulary (the small case for captures
    # of the prefill attention kernel)
    from aneforge_b200 import llm as L
    spec = MODELS[MODEL]
    mlp = "moe" if spec.get("moe") else "swiglu"
    cd = dict(CFG, n_layers=1, vocab=4096) if name == "prefill_1layer" else CFG
    cfg = L.LlamaConfig(**cd, layers=[L.LayerSpec(mlp=mlp) for _ in range(cd["n_layers"])])
    w = make_weights(cfg, dev, seed=1234, qkv_bias=spec["qkv_bias"], moe=bool(spec.get("moe")))
    m = L.LlamaPrefill(cfg, w, compress=spec["compress"], device=0, moe_compress=spec.get("moe_compress", "same"))
    m._load()
    del w
    torch.cuda.empty_cache()
    ids = np.random.default_rng(99).integers(0, cfg.vocab, PROMPT).astype(np.int32)
    pre = m._prefiller(PROMPT)
    prog = pre["prog"]
    prog.set_input("ids", ids)
    for _ in range(warmup):
      prog.execute_async()
    prog.sync()
    ps = torch.cuda.ExternalStream(prog.stream(), device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ps)
    for _ in range(reps):
      prog.execute_async()             # weights (GBs) exceed L2: every run streams them from HBM
    e1.record(ps)
    prog.sync()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    nl, hd = cd["n_layers"], CFG.get("head_dim") or D // H
    ex = CFG.get("extra", {}).get("n_experts_per_tok", 1) if spec.get("moe") else 1
    lin = 2.0 * PROMPT * nl * (D * (H + 2 * KV) * hd + H * hd * D + 3 * D * F * ex)
    att = 2.0 * nl * H * hd * PROMPT * (PROMPT + 1)      # causal QK^T + PV
    del ps
    m.release()
    return {"kernel": name, "what": f"prefill program, {MODEL} {spec['compress']}, {nl} layers, {PROMPT} tokens",
            "ms_per_prefill": round(ms, 3), "tokens_per_s": round(PROMPT / (ms * 1e-3), 1),
            "tflops": round((lin + att) / (ms * 1e-3) / 1e12, 1), "reps": reps, "warmup": warmup}

  if name == "chain":
    # the decode step's chained GEMV launch (o, norm, gate|up, down, norm, next qkv) of a 4-layer
    # model of the selected shape with a 4096-token vocabulary: ~0.9 GB of layer weights for the
    # 8B shape, above L2; the small case for captures of gemv_chain_kernel
    from aneforge_b200 import llm as L
    spec = MODELS[MODEL]
    cd = dict(CFG, n_layers=4, vocab=4096)
    cfg = L.LlamaConfig(**cd, layers=[L.LayerSpec() for _ in range(4)])
    w = make_weights(cfg, dev, seed=1234, qkv_bias=spec["qkv_bias"])
    m = L.LlamaPrefill(cfg, w, compress=spec["compress"], device=0)
    m._load()
    del w
    dec = m._decoder(PROMPT + 64, 1)
    us, nbytes = time_chains(m, dec, 1, reps=max(reps // 4, 2))
    peak, _ = _peaks()
    m.release()
    return {"kernel": name, "what": f"gemv_chain {MODEL} {spec['compress']}: o, norm, gate|up, down, norm, next qkv",
            "us_per_launch": round(us, 2), "algorithmic_bytes": int(nbytes),
            "gbs": round(nbytes / (us * 1e-6) / 1e9, 1), "frac": round(nbytes / (us * 1e-6) / 1e9 / peak, 4)}

  def int8_tiles(N, Kd, copies):
    W = (torch.randn(N, Kd, generator=g, device=dev) * 0.02).half()
    q, sc = K.quantize_per_row_i8(W)
    t = K.pack_i8_tiles(q)
    return [t] + [t.clone() for _ in range(copies - 1)], sc

  I4 = {"gemv_i4_gu": (2 * 29568, 8192, R.EPI_SWIGLU), "gemv_i4_qkv": (80 * 128, 8192, R.EPI_F32),
        "gemv_i4_o": (8192, 8192, R.EPI_RESID), "gemv_i4_down": (8192, 29568, R.EPI_RESID),
        "gemv_i4_moe_gu": (2 * 14336, 4096, R.EPI_SWIGLU)}   # one Mixtral expert's gate|up
  if name in ("gemm_gu", "gemm_i4_gu", "gemm_qkv", "gemm_o", "gemm_down"):
    # prefill: the tcgen05 GEMM over a 512-row (8B) / 2048-row (72B) prompt; FLOP-bound. qkv / o /
    # down are the 8B prompt shapes with fewer 256-column tiles than SMs (128-column tiles)
    i4 = name == "gemm_i4_gu"
    M, N, Kd = {"gemm_gu": (512, 2 * F, D), "gemm_i4_gu": (2048, 2 * 29568, 8192),
                "gemm_qkv": (512, (H + 2 * KV) * dh, D), "gemm_o": (512, D, H * dh),
                "gemm_down": (512, D, F)}[name]
    # the prefill program's epilogues: SwiGLU for gate|up, f32 for qkv, the residual add for o / down
    epi = {"gemm_gu": R.EPI_SWIGLU, "gemm_i4_gu": R.EPI_SWIGLU, "gemm_qkv": R.EPI_F32}.get(name, R.EPI_RESID)
    W = (torch.randn(N, Kd, generator=g, device=dev) * 0.02).half()
    if i4:
      pk, sc = K.quantize_g32_i4(W); tiles = K.pack_i4_tiles(pk, sc, N, Kd); sc = None
    else:
      q, sc = K.quantize_per_row_i8(W); tiles = K.pack_i8_tiles(q)
    del W
    x = torch.randn(M, Kd, generator=g, device=dev).half()
    y = (torch.empty(M, N // 2, device=dev, dtype=torch.float16) if epi == R.EPI_SWIGLU
         else torch.zeros(M, N, device=dev, dtype=torch.float32))
    fn = lambda i: K.gemm_tc(x, tiles, sc, N, Kd, wf=R.W_I4G32 if i4 else R.W_I8, epi=epi, y=y)
    flops = 2.0 * M * N * Kd
    with torch.cuda.stream(st):
      for i in range(warmup):
        fn(i)
      torch.cuda.synchronize()
      e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
      e0.record(st)
      for i in range(reps):
        fn(i)
      e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    try:
      with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
        tpk, tkind = float(json.load(f)["bf16_tflops"]), "measured bf16 dense (cuBLAS burst)"
    except Exception:
      tpk, tkind = 1590.0, "fallback"
    tf = flops / (us * 1e-6) / 1e12
    return {"kernel": name, "what": f"gemm_tc {'int4_g32' if i4 else 'int8'} M={M} N={N} K={Kd} "
                                    f"{ {R.EPI_SWIGLU: 'swiglu', R.EPI_F32: 'f32'}.get(epi, 'resid') }",
            "us_per_launch": round(us, 1), "tflops": round(tf, 1), "peak_tflops": tpk, "peak_kind": tkind,
            "frac": round(tf / tpk, 4), "reps": reps, "warmup": warmup}
  if name in I4:                                            # Qwen2-72B shapes, group-32 int4
    N, Kd, epi = I4[name]
    copies = max(2, -(-300_000_000 // (N * Kd // 2)))
    W = (torch.randn(N, Kd, generator=g, device=dev) * 0.02).half()
    pk, sc = K.quantize_g32_i4(W)
    del W
    t0 = K.pack_i4_tiles(pk, sc, N, Kd)
    tiles = [t0] + [t0.clone() for _ in range(copies - 1)]
    x = torch.randn(nb, Kd, generator=g, device=dev).half()
    y = K.gemv_tc_i4(x, tiles[0], N, Kd, epi=epi)
    scr, _ = K.gemv_tc_scratch(N, Kd, nb, dev)
    nbytes = N * Kd // 2 + 2 * (N * Kd // 32) + 2 * Kd * nb + y.numel() * y.element_size() * (2 if epi == R.EPI_RESID else 1)
    fn = lambda i: K.gemv_tc_i4(x, tiles[i % copies], N, Kd, epi=epi, y=y, scratch=scr)
    what = f"gemv_tc int4_g32 {N}x{Kd} epi={epi} rows={nb}"
  elif name in ("gemv_gu", "gemv_cfg1", "gemv_qkv", "gemv_o", "gemv_down"):
    N, Kd, epi = {"gemv_gu": (2 * F, D, R.EPI_SWIGLU), "gemv_cfg1": (4096, 4096, R.EPI_F16),
                  "gemv_qkv": ((H + 2 * KV) * dh, D, R.EPI_F32), "gemv_o": (D, H * dh, R.EPI_RESID),
                  "gemv_down": (D, F, R.EPI_RESID)}[name]
    copies = max(2, -(-300_000_000 // (N * Kd)))            # > 2x L2 of weights in rotation
    tiles, sc = int8_tiles(N, Kd, copies)
    x = torch.randn(nb, Kd, generator=g, device=dev).half()
    y = K.gemv_tc(x, tiles[0], sc, N, Kd, epi=epi)
    scr, _ = K.gemv_tc_scratch(N, Kd, nb, dev)
    nbytes = N * Kd + 2 * N + 2 * Kd * nb + y.numel() * y.element_size() * (2 if epi == R.EPI_RESID else 1)
    fn = lambda i: K.gemv_tc(x, tiles[i % copies], sc, N, Kd, epi=epi, y=y, scratch=scr)
    what = f"gemv_tc int8 {N}x{Kd} epi={epi} rows={nb}"
  elif name == "attn":
    M, pos = 1024, 576
    kc = torch.randn(1, KV, M, dh, generator=g, device=dev).half()
    vc = torch.randn(1, KV, M, dh, generator=g, device=dev).half()
    qkv = torch.randn(1, (H + 2 * KV) * dh, generator=g, device=dev)
    p = torch.tensor([pos], dtype=torch.int32, device=dev)
    c, s_ = (torch.from_numpy(a).to(dev) for a in rope_tables(M, dh, CFG["rope_base"]))
    from aneforge_b200.llm import decode_nsplit
    nsplit = decode_nsplit(M, KV)                            # the decode program's split count
    scr = torch.zeros(K.attn_decode_scratch_bytes(1, KV, nsplit, H // KV, dh), dtype=torch.uint8, device=dev)
    kv_c = 127 * float(np.float16(1 / 127))
    nbytes = 2 * KV * (pos + 1) * dh * 2 + qkv.numel() * 4 + H * dh * 2
    o = torch.zeros(1, H * dh, dtype=torch.float16, device=dev)
    fn = lambda i: K.attn_decode(qkv, kc, vc, p, c, s_, H, KV, dh, float(np.float16(1 / np.sqrt(dh))), kv_c, True,
                                 nsplit, scr, out=o)
    what = f"attn_decode H{H}/KV{KV} dh{dh} pos {pos} nsplit {nsplit} (KV cache {2 * KV * (pos + 1) * dh * 2} B)"
  elif name == "rmsnorm":
    # the decode's pre-attention / pre-MLP norm: one fp32 residual row -> fp16
    xs = [torch.randn(1, D, generator=g, device=dev) for _ in range(64)]
    gam = (torch.randn(D, generator=g, device=dev) * 0.5 + 1.0).half()
    nbytes = D * 4 + D * 2 + D * 2
    fn = lambda i: K.rmsnorm(xs[i % 64], gam, float(np.float16(np.sqrt(D * 1e-5))))
    what = f"rmsnorm fp32 row of {D} -> fp16"
  elif name == "moe_gate":
    # Mixtral router tail: softmax over 8 experts, top-2, renormalise
    lg = [torch.randn(1, 8, generator=g, device=dev) for _ in range(64)]
    nbytes = 8 * 4 + 8 * 4 + 2 * 4
    fn = lambda i: K.moe_gate(lg[i % 64], 2)
    what = "moe_gate E=8 k=2, one row"
  elif name == "lm_head":
    W = (torch.randn(V, D, generator=g, device=dev) * 0.02).half()
    x = torch.randn(1, D, generator=g, device=dev).half()
    nbytes = V * D * 2 + D * 2 + V * 4
    scr = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)
    outs = (torch.zeros(1, dtype=torch.int32, device=dev), torch.zeros(1, V, dtype=torch.float32, device=dev))
    fn = lambda i: K.lm_head_argmax(x, W, scratch=scr, out=outs)
    what = f"lm_head fp16 {V}x{D} + argmax"
  else:
    raise SystemExit(f"unknown --kernel {name}")
  # the launches are captured in one CUDA graph so that host-side call overhead does not pace them
  with torch.cuda.stream(st):
    for i in range(warmup):
      fn(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
      for i in range(reps):
        fn(warmup + i)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    graph.replay()
    e1.record(st)
  torch.cuda.synchronize()
  us = e0.elapsed_time(e1) * 1e3 / reps
  del graph
  peak, kind = _peaks()
  gbs = nbytes / (us * 1e-6) / 1e9
  return {"kernel": name, "what": what, "us_per_launch": round(us, 2), "algorithmic_bytes": int(nbytes),
          "achieved_gbs": round(gbs, 1), "peak_gbs": peak, "peak_kind": kind, "frac": round(gbs / peak, 4),
          "reps": reps, "warmup": warmup, "timing": "CUDA events around one CUDA-graph replay of `reps` back-to-back launches"}


def timeline(args):
  """Kernel timeline of decode-step graph replays (the `--timeline` mode): CUPTI kernel records
  through torch.profiler over 3 steps after warm-up, each kernel's wall share = its end minus the
  previous kernel's end (overlapped launches count once), summed per kernel kind and per layer."""
  import collections
  import torch
  from aneforge_b200 import llm as L
  spec = MODELS[MODEL]
  dev = torch.device("cuda", 0)
  torch.cuda.set_device(dev)
  mlp = "moe" if spec.get("moe") else "swiglu"
  cfg = L.LlamaConfig(**CFG, layers=[L.LayerSpec(mlp=mlp) for _ in range(CFG["n_layers"])])
  w = make_weights(cfg, dev, seed=1234, qkv_bias=spec["qkv_bias"], moe=bool(spec.get("moe")))
  m = L.LlamaPrefill(cfg, w, compress=spec["compress"], moe_compress=spec.get("moe_compress", "same"))
  m._load()
  del w
  NB = args.batch
  M = PROMPT + 64
  dec = m._decoder(M, NB)
  prog = dec["prog"]
  m._reset_state(dec)
  rng = np.random.default_rng(99)
  for b in range(NB):
    pre, real, _ = m._prefill_hidden(list(rng.integers(0, cfg.vocab, PROMPT)))
    m._seed_cache(dec, pre, real, slot=b)
  torch.cuda.synchronize()
  prog.set_input("tok", np.full(NB, 7, np.int32)); prog.set_input("pos", np.full(NB, PROMPT, np.int32))
  for _ in range(max(args.warmup, 3)):
    prog.execute_async()
  prog.sync()
  with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
    for _ in range(3):
      prog.execute_async()
    prog.sync()
    torch.cuda.synchronize()
  ev = sorted((e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA),
              key=lambda e: e.time_range.start)
  per = len(ev) // 3
  step = ev[per:2 * per]                                   # the middle step
  kinds = {"gemv_chain_kernel": "chain (o, norm, gate|up, down, norm, next qkv)", "gemv_tc_kernel<1, 0": "qkv (f32 epi)", "gemv_tc_kernel<1, 2": "o / down (resid epi)",
           "gemv_tc_kernel<1, 3": "gate|up (swiglu epi)", "attn_decode": "attention", "rmsnorm": "rmsnorm",
           "gemv_kernel": "lm_head + argmax", "embed": "embed", "moe_gate": "moe gate", "lm_head_tc": "lm_head (tensor pipe)"}
  share, busy, count = collections.defaultdict(float), collections.defaultdict(float), collections.Counter()
  t0 = step[0].time_range.start
  prev = t0
  for e in step:
    k = next((v for s, v in kinds.items() if s in e.name), e.name[:40])
    end = e.time_range.end
    share[k] += max(0.0, end - prev)
    busy[k] += e.time_range.end - e.time_range.start
    count[k] += 1
    prev = max(prev, end)
  span = prev - t0
  return {"mode": "timeline", "model": MODEL, "batch": NB, "kernels_per_step": per, "step_us": round(span, 1),
          "per_kind": {k: {"launches": count[k], "wall_share_us": round(share[k], 1), "busy_us": round(busy[k], 1),
                           "wall_share_frac": round(share[k] / span, 4)} for k in share},
          "how": "torch.profiler CUDA kernel records of 3 CUDA-graph replays after warm-up; the middle step"}


def profile_traffic(name="gemv_tc_gate_up_llama8b.md"):
  """DRAM bytes per launch of the dominant kernel from the committed ncu summary (or None)."""
  import re
  try:
    with open(os.path.join(ROOT, "profiles", name)) as f:
      m = re.search(r"traffic_bytes_per_launch:\s*([0-9,]+)", f.read())
    return int(m.group(1).replace(",", "")) if m else None
  except OSError:
    return None


def cpu_reference(steps=3, warmup=1, layers=1, max_steps=30):
  """The reference path on the host: the oracle's decode of a `layers`-deep slice of the same model
  plus the full lm_head and argmax, each step scaled to the model's depth (layer time x depth / layers
  + head time). `warmup` untimed then `steps` timed steps (at most `max_steps`, so a run stays within
  about a minute of host time). Returns (tokens/s, description, seconds per scaled step)."""
  from oracle.model import OracleModel, Config, random_llama_weights
  spec = MODELS[MODEL]
  steps = max(1, min(int(steps), max_steps))
  warmup = max(1, min(int(warmup), 5))
  cfg = Config(dim=CFG["dim"], n_layers=layers, n_heads=CFG["n_heads"], n_kv_heads=CFG["n_kv_heads"],
               ffn_dim=CFG["ffn_dim"], vocab=CFG["vocab"], rope_base=CFG["rope_base"], norm_eps=CFG["norm_eps"])
  w = random_llama_weights(cfg, seed=5, qkv_bias=spec["qkv_bias"])
  w["embed"] = np.zeros((cfg.vocab, cfg.dim), np.float16)   # only gathered rows are read; values do not change the time
  om = OracleModel(cfg, w, spec["compress"], precision="device")
  M = PROMPT + warmup + steps + 2
  om._tables(M)
  caches = om.new_caches(M)
  rng = np.random.default_rng(1)
  for Kc, Vc in caches:
    Kc[:, :PROMPT] = rng.standard_normal(Kc[:, :PROMPT].shape, dtype=np.float32).astype(np.float16)
    Vc[:, :PROMPT] = rng.standard_normal(Vc[:, :PROMPT].shape, dtype=np.float32).astype(np.float16)
  tok, pos = 7, PROMPT
  for _ in range(warmup):                                  # warm BLAS / page in
    hid = om.decode_step(tok, pos, caches)
    tok = int(np.argmax(om.logits(hid.astype(np.float32))))
    pos += 1
  t_layers, t_head = 0.0, 0.0
  for _ in range(steps):
    t0 = time.perf_counter()
    hid = om.decode_step(tok, pos, caches)
    t1 = time.perf_counter()
    tok = int(np.argmax(om.logits(hid.astype(np.float32))))
    t2 = time.perf_counter()
    t_layers += t1 - t0; t_head += t2 - t1
    pos += 1
  per_tok = t_layers / steps * (CFG["n_layers"] / layers) + t_head / steps
  return 1.0 / per_tok, (f"{steps} timed decode steps (after {warmup}) of a {layers}-layer slice at positions "
                         f"{PROMPT}.., each plus the full {CFG['vocab']}-row lm_head and argmax, layer time scaled "
                         f"to {CFG['n_layers']} layers"), per_tok


def blas_threads():
  try:
    from threadpoolctl import threadpool_info
    return max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
  except Exception:
    return os.cpu_count() or 1


class _JsonOut:
  """stdout carries the JSON line(s) only: everything else written to file descriptor 1 while the
  bench runs (NCCL's version banner, library messages, Python prints) goes to stderr."""

  def __init__(self):
    sys.stdout.flush()
    self.fd = os.dup(1)
    os.dup2(2, 1)
    sys.stdout = sys.stderr

  def emit(self, obj):
    os.write(self.fd, (json.dumps(obj) + "\n").encode())


def main():
  ap = argparse.ArgumentParser()
  ap.add_argument("--gpus", type=int, default=1)
  ap.add_argument("--steps", type=int, default=200)
  ap.add_argument("--warmup", type=int, default=10)
  ap.add_argument("--batch", type=int, default=1)
  ap.add_argument("--model", default="llama3-8b", choices=sorted(MODELS))
  ap.add_argument("--tp", action="store_true",
                  help="(the default with --gpus N > 1) shard one model over the N ranks: tensor parallel")
  ap.add_argument("--replicas", action="store_true",
                  help="with --gpus N > 1: N independent replicas (weak scaling) instead of tensor parallel")
  ap.add_argument("--gen-tokens", type=int, default=128,
                  help="tokens of the end-to-end LlamaPrefill.generate figure (0: skip)")
  ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
  ap.add_argument("--no-cpu-baseline", action="store_true")
  ap.add_argument("--kernel", default=None,
                  help="time one kernel alone: gemv_gu | gemv_qkv | gemv_o | gemv_down | gemv_cfg1 | attn | lm_head "
                       "| gemv_i4_gu | gemv_i4_qkv | gemv_i4_o | gemv_i4_down | gemv_i4_moe_gu | gemm_gu | gemm_i4_gu "
                       "| gemm_qkv | gemm_o | gemm_down "
                       "| rmsnorm | moe_gate | prefill (the whole prefill program of --model) | prefill_1layer | chain")
  ap.add_argument("--reps", type=int, default=50)
  ap.add_argument("--timeline", action="store_true",
                  help="print the kernel timeline of decode-step graph replays (CUPTI through torch.profiler)")
  ap.add_argument("--profile-region", action="store_true",
                  help="bracket the timed steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
  args = ap.parse_args()
  select_model(args.model)
  ws, rank, _ = _dist()
  out = _JsonOut()
  if args.timeline:
    out.emit(timeline(args))
    return
  if args.kernel:
    for name in args.kernel.split(","):
      out.emit(kernel_bench(name, args.reps, max(args.warmup, 3), args.batch))
    return
  if args.impl == "reference":
    if rank != 0:
      return
    v, how, per_step = cpu_reference(args.steps, args.warmup)
    tp_on = ws > 1 and not args.replicas
    info = host_info()
    out.emit({"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tokens/s",
                      "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                      "scaling": "strong" if tp_on else "weak", "vs_baseline": None,
                      "dtype": MODELS[MODEL]["dtype"] + " (numpy fp32 on the host)", "data": "synthetic",
                      "config": workload_config(args, ws, tp_on),
                      "ms_per_step": round(per_step * 1e3, 2),
                      "cpu_baseline": {"value": round(v, 4), "unit": "tokens/s", "cores": info["blas_threads"],
                                       "kind": "port", "sample": how, **info},
                      "e2e": {"value": round(v, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}})
    return
  res = run_b200(args)
  if rank == 0 and res is not None:
    if not args.no_cpu_baseline and ws == 1:
      v, how, _ = cpu_reference(3, 1)
      info = host_info()
      res["cpu_baseline"] = {"value": round(v, 4), "unit": "tokens/s", "cores": info["blas_threads"], "kind": "port",
                             "sample": how, **info}
    out.emit(res)


if __name__ == "__main__":
  main()
