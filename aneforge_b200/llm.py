"""LLM decode/prefill on B200: the drop-in for the reference's `aneforge/llm.py` runner.

Same surface: `LlamaConfig`, `LayerSpec`, `rope_tables`, the builder registries
(`PREFILL_MIXERS`, `PREFILL_MLPS`, `DECODE_MIXERS`, `DECODE_MLPS`), `ADAPTERS`, `from_pretrained`
(re-exported as `load_llm`), and `LlamaPrefill` with `compile/prefill/warmup/generate/release`.

What changes underneath (B200-first):
  * Weights are quantized on the GPU (bit-exact to the reference encoders) and packed into fused
    projections (q|k|v rows concatenated, gate/up rows interleaved) that stay resident in HBM.
  * A decode step is ONE program (all layers + final norm + lm_head + greedy argmax) replayed as a
    CUDA graph; registry values are plan emitters that append fused kernel launches.
  * The KV cache is device-resident per layer ([NB, KV, M, dh] fp16); a step writes only slot `pos`.
  * The greedy token and the position stay on the device (the token output port is aliased onto
    the token input port with `share_buffer`, the reference's own resident-state mechanism), so
    steps run back to back with no host round trip; the host reads the token history at the end.
  * Batched prefill writes K/V in the decode cache layout, then seeds the cache with one device copy.
"""
from __future__ import annotations

import os
import time
import warnings
from dataclasses import dataclass, field
from enum import Enum

import numpy as np

from . import _blob
from . import _runtime as R
from .plan import PlanBuilder, at
from .weights import DevLinear, encode_linear, rms_weights, to_device, fp16_bits_exact
from .blocks import is_graph_builder

F16, F32 = np.float16, np.float32


class ModelType(str, Enum):
  GPT2 = "gpt2"
  GEMMA = "gemma"
  GEMMA2 = "gemma2"
  GEMMA3 = "gemma3"
  GEMMA3_TEXT = "gemma3_text"
  MISTRAL = "mistral"
  LLAMA = "llama"
  QWEN = "qwen"


@dataclass
class LayerSpec:
  """Per-layer plan (reference `aneforge/llm.py:36-42`)."""
  mixer: str = "attention"
  mlp: str = "swiglu"
  qk_norm: bool = False


@dataclass
class LlamaConfig:
  """Decoder config (reference `aneforge/llm.py:45-59`)."""
  dim: int; n_layers: int; n_heads: int; n_kv_heads: int; ffn_dim: int; vocab: int
  rope_base: float = 10000.0; norm_eps: float = 1e-5; head_dim: int = 0
  rotary_dim: int = 0; rope_interleaved: bool = False
  rope_scaling: dict | None = None
  layers: list = field(default_factory=list)
  extra: dict = field(default_factory=dict)
  norm_type: str = "rms"
  rope: bool = True

  @property
  def dh(self) -> int:
    return self.head_dim or self.dim // self.n_heads


def _rope_frequencies(rd: int, base: float, scaling: dict | None):
  """float64 angular frequency of each rotated pair: theta_i = base^(-2i/rd). With a "llama3"
  `rope_scaling` (Llama 3.1) the frequencies are remapped by wavelength (what the reference's
  `aneforge/llm.py:62-73` does, following the Hugging Face formula):
    * wavelength 2*pi/theta longer than original_max_positions / low_freq_factor -> theta / factor;
    * shorter than original_max_positions / high_freq_factor                      -> unchanged;
    * in between: a linear blend of the two, weighted by how far into the band the pair sits."""
  freqs = 1.0 / (base ** (np.arange(0, rd, 2) / rd))
  if not (scaling and scaling.get("rope_type") == "llama3"):
    return freqs
  factor = float(scaling["factor"])
  lo, hi = float(scaling["low_freq_factor"]), float(scaling["high_freq_factor"])
  ctx = float(scaling["original_max_position_embeddings"])
  wavelen = 2.0 * np.pi / freqs
  long_edge, short_edge = ctx / lo, ctx / hi
  out = freqs.copy()
  slow = wavelen > long_edge
  out[slow] = freqs[slow] / factor
  band = (wavelen >= short_edge) & (wavelen <= long_edge)
  t = (ctx / wavelen[band] - lo) / (hi - lo)             # 0 at the long edge, 1 at the short edge
  out[band] = (1.0 - t) * freqs[band] / factor + t * freqs[band]
  return out


def rope_tables(seq: int, dh: int, base: float = 10000.0, rotary_dim: int = 0, interleaved: bool = False,
                scaling: dict | None = None):
  """cos / sin tables [seq, dh] for positions 0..seq-1, computed in float64 and rounded to fp16 once
  (the reference's tables, `aneforge/llm.py:76-94`). Neox layout: the first and second halves of a
  head share frequencies; `interleaved` pairs adjacent lanes instead. With a partial rotary
  dimension the unrotated lanes get cos 1, sin 0."""
  rd = rotary_dim or dh
  angle = np.outer(np.arange(seq, dtype=np.float64), _rope_frequencies(rd, base, scaling))   # [seq, rd/2]
  lay = (lambda a: np.repeat(a, 2, axis=1)) if interleaved else (lambda a: np.concatenate([a, a], axis=1))
  cos_t = np.ones((seq, dh), np.float64)
  sin_t = np.zeros((seq, dh), np.float64)
  cos_t[:, :rd] = lay(np.cos(angle))
  sin_t[:, :rd] = lay(np.sin(angle))
  return cos_t.astype(F16), sin_t.astype(F16)


def sample_token(logits, temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0) -> int:
  """One token id from a row of logits (see `LlamaPrefill._sample`)."""
  z = np.asarray(logits, np.float64).ravel()
  if temperature <= 0.0:
    return int(np.argmax(z))
  z = z / temperature
  n = z.size
  if top_k and 0 < top_k < n:
    kth = np.partition(z, n - top_k)[n - top_k]            # the k-th largest logit; ties with it stay
    z = np.where(z >= kth, z, -np.inf)
  prob = np.exp(z - z.max())
  prob /= prob.sum()
  if 0.0 < top_p < 1.0:
    desc = np.argsort(prob)[::-1]                           # most probable first
    mass = np.cumsum(prob[desc])
    n_keep = int(np.count_nonzero(mass < top_p)) + 1        # up to and including the token crossing top_p
    nucleus = np.zeros_like(prob)
    nucleus[desc[:n_keep]] = prob[desc[:n_keep]]
    prob = nucleus / nucleus.sum()
  return int(np.random.choice(n, p=prob))


# ------------------------------------------------------------------------------ plan emitters
#
# A registry value appends the fused launches of one block to a plan. `ctx` carries the program's
# activation buffers and shapes: h (fp32 residual [NB, D]), xn (fp16 [NB, D]), qkv, att, act, pos,
# NB, M; `lw` is the layer's packed device weights (names of bound buffers, see _bind_layer).

# Row counts from which a tiled projection runs as the tensor-core GEMM instead of the GEMV: the GEMV
# streams the weights once per 16 rows, the GEMM once per 128 (or 256) but walks its k slices at a
# fixed pace whatever the rows. Prefill programs switch at 32 rows; decode programs (batches of
# sequences) keep the GEMV below 128: measured on Mixtral at batch 32, the attention projections took
# ~60 µs a launch on the GEMM against ~15 on two 16-row GEMV passes.
GEMM_MIN_ROWS = 32
DECODE_GEMM_MIN_ROWS = 128


def _emit_linear(pb, ctx, name, lin: DevLinear, x, y, epi, nb=None):
  nb = nb or ctx["NB"]
  kv = dict(wf=lin.wf, epi=epi, x=x, w=f"{name}.w", y=y, nb=nb, n=lin.N, k=lin.K)
  if lin.kind == "int8":
    kv["s"] = f"{name}.s"
  if lin.kind in ("int8", "int4_g32") and lin.tiled:
    if nb >= ctx.get("gemm_min", GEMM_MIN_ROWS):
      kv["gemm"] = 1                                 # prompt rows: the tcgen05 GEMM
    else:
      nbytes = R.load_library().af_gemv_tc_scratch_bytes(lin.N, lin.K, nb)
      if nbytes:
        pb.buf("gemv.scr", nbytes, "scratch")        # one split-K scratch shared by every GEMV
        kv["scr"] = "gemv.scr"
  elif lin.kind in ("int4_g32", "lut4", "blockwise", "sparse") and not lin.tiled:
    kv["gs"] = f"{name}.s"                             # group scales / per-row codebooks / kept values
    if lin.kind == "blockwise":
      kv["grp"] = lin.group
    if lin.kind == "sparse":
      kv.update(ro=f"{name}.ro", nnz=lin.s.numel())
  if lin.bias is not None:
    kv["bias"] = f"{name}.b"
  pb.op("gemv", **kv)


def _emit_row_parallel(pb, ctx, name, lin: DevLinear, x):
  """A projection whose output is added to the fp32 residual `h`. Under tensor parallelism each rank
  holds a slice of its input columns: the partial goes to `tp.part`, is all-reduced over the ranks
  and then added to the (replicated) residual."""
  if ctx.get("tp"):
    n = ctx["NB"] * ctx["D"]
    _emit_linear(pb, ctx, name, lin, x, "tp.part", "f32")
    pb.op("allreduce", src="tp.part", dst="tp.part", n=n, addto="h")
  else:
    _emit_linear(pb, ctx, name, lin, x, "h", "resid")


def _emit_attn_norm(pb, cfg, pre, lw, nb):
  """The attention input norm of `nb` residual rows into `xn`: RMSNorm, or LayerNorm (GPT-2,
  `cfg.norm_type == "layer"`, eps rounded to fp16 as the reference bakes it)."""
  if cfg.norm_type == "layer":
    pb.op("layernorm", x="h", g=f"{pre}.attn_lw", b=f"{pre}.attn_lb", eps=float(np.float16(cfg.norm_eps)), out="xn",
          nb=nb, d=cfg.dim)
  else:
    pb.op("rmsnorm", x="h", g=f"{pre}.attn_g", out="xn", nb=nb, d=cfg.dim, floor=lw["attn_floor"])


def _emit_final_norm(pb, cfg, d, nb):
  if cfg.norm_type == "layer":
    pb.op("layernorm", x="h", g="final_g", b="final_b", eps=float(np.float16(cfg.norm_eps)), out="hid", nb=nb,
          d=cfg.dim)
  else:
    pb.op("rmsnorm", x="h", g="final_g", out="hid", nb=nb, d=cfg.dim, floor=d["final_floor"])


def _emit_embedding(pb, cfg, d, nb, pos):
  """Embedding rows into the fp32 residual, plus GPT-2's learned position rows (`wpe`) at `pos`
  (a per-row position buffer) or at the row index (a prompt)."""
  pb.op("embed", tok="tok" if pos else "ids", table="embed", h="h", vocab=cfg.vocab, d=cfg.dim, nb=nb)
  if "wpe" in d:
    P = int(d["wpe"].shape[0])
    pb.buf("wpe", 2 * P * cfg.dim, "weight")
    pb.op("add_pos", h="h", table="wpe", npos=P, pos=pos, nb=nb, d=cfg.dim)


def emit_attention_decode(pb, ctx, li, lw, cfg, ls):
  """`_attn_decode` (reference `llm.py:214-237`): norm -> fused QKV GEMV -> RoPE + cache write at
  pos + GQA split-K attention -> o_proj GEMV with the residual add fused."""
  D, H, KV, dh, NB, M = cfg.dim, cfg.n_heads, cfg.n_kv_heads, cfg.dh, ctx["NB"], ctx["M"]
  pre = f"L{li}"
  _emit_attn_norm(pb, cfg, pre, lw, NB)
  _emit_linear(pb, ctx, f"{pre}.qkv", lw["qkv"], "xn", "qkv", "f32")
  # prefetch=1: the step's position is only advanced by its last kernel (the head), so attention may
  # stage its first cache rows before the qkv projection finishes
  kv = dict(qkv="qkv", kc=f"{pre}.K", vc=f"{pre}.V", pos="pos", out="att", nb=NB, h=H, kv=KV, dh=dh, m=M,
            nsplit=ctx["nsplit"], scale=ctx["scale"], kvc=ctx["kvc"], expand=int(ctx["expand"]), prefetch=1)
  if cfg.rope:
    kv.update(cos="rope.cos", sin="rope.sin")
  if ls.qk_norm:
    kv.update(qn=f"{pre}.qn", kn=f"{pre}.kn", qnf=lw["qn_floor"], knf=lw["kn_floor"])
  if ctx["nsplit"] > 1:
    kv.update(part="attn.part", cnt="attn.cnt")
  if ctx.get("verify"):
    # speculative verify: the NB rows are consecutive tokens of ONE sequence sharing one cache; their
    # K / V rows are appended first, then each row attends up to its own position
    kv.update(seqrows=0, wkv=0, prefetch=0)
    pb.op("kv_append", **{k: v for k, v in kv.items() if k in ("qkv", "kc", "vc", "pos", "nb", "h", "kv", "dh", "m",
                                                              "cos", "sin", "kn", "knf", "seqrows")})
  pb.op("attn_decode", **kv)
  _emit_row_parallel(pb, ctx, f"{pre}.o", lw["o"], "att")


def emit_attention_prefill(pb, ctx, li, lw, cfg, ls):
  """`_attn_prefill_kv` (reference `llm.py:149-169`): K (roped) and V land in cache layout."""
  D, H, KV, dh, S = cfg.dim, cfg.n_heads, cfg.n_kv_heads, cfg.dh, ctx["NB"]
  pre = f"L{li}"
  _emit_attn_norm(pb, cfg, pre, lw, S)
  _emit_linear(pb, ctx, f"{pre}.qkv", lw["qkv"], "xn", "qkv", "f32")
  kv = dict(qkv="qkv", kc=f"{pre}.K", vc=f"{pre}.V", out="att", qbuf="qbuf", s=S, h=H, kv=KV, dh=dh, ldm=S,
            scale=ctx["scale"], kvc=ctx["kvc"], expand=int(ctx["expand"]))
  if ctx["expand"]:
    # K and V times the GQA factor, written once by the rope kernel for the tensor-core attention
    kv.update(kvx=pb.buf("kvx", 2 * 2 * KV * S * dh, "tmp"))
  if cfg.rope:
    kv.update(cos="rope.cos", sin="rope.sin")
  if ls.qk_norm:
    kv.update(qn=f"{pre}.qn", kn=f"{pre}.kn", qnf=lw["qn_floor"], knf=lw["kn_floor"])
  pb.op("attn_prefill", **kv)
  _emit_row_parallel(pb, ctx, f"{pre}.o", lw["o"], "att")


def emit_swiglu(pb, ctx, li, lw, cfg, ls):
  """`_swiglu` (reference `llm.py:171-175`): norm -> fused gate|up GEMV with silu(g)*u epilogue ->
  down GEMV with the residual add fused."""
  pre = f"L{li}"
  pb.op("rmsnorm", x="h", g=f"{pre}.mlp_g", out="xn", nb=ctx["NB"], d=cfg.dim, floor=lw["mlp_floor"])
  _emit_linear(pb, ctx, f"{pre}.gu", lw["gu"], "xn", "act", "swiglu")
  _emit_row_parallel(pb, ctx, f"{pre}.down", lw["down"], "act")


# Registry values are either fused plan emitters f(pb, ctx, li, lw, cfg, ls) - the hot path - or
# graph builders in the reference's form (`aneforge/llm.py:240-245`; see `blocks`), which the
# programs lower through `_compile.Lowering`: a plugin written for the reference registers here
# unchanged. GeGLU and the GPT-2 GELU MLP run as graph builders.
from . import blocks as _blocks  # noqa: E402

PREFILL_MIXERS = {"attention": emit_attention_prefill}
PREFILL_MLPS = {"swiglu": emit_swiglu, "geglu": _blocks.geglu, "gelu_new": _blocks.gelu_mlp}
DECODE_MIXERS = {"attention": emit_attention_decode}
DECODE_MLPS = {"swiglu": emit_swiglu, "geglu": _blocks.geglu, "gelu_new": _blocks.gelu_mlp}
_DECODE_CTX = ("pos",)


def decode_nsplit(M, KV, NB=1):
  """Split count of decode attention over a cache of M rows (see `_ctx`)."""
  cap = max(1, (2 * 148) // max(1, KV * NB))
  nsplit = max(1, min(64, cap, -(-M // 64)))
  if nsplit > 12 and -(-M // 12) <= 512:
    nsplit = 12
  elif nsplit > 16 and -(-M // 16) <= 512:
    nsplit = 16
  return int(os.environ.get("AF_ATTN_NSPLIT", nsplit))


def plan_gemv_chains(pb, enable=None):
  """Fuse runs of consecutive tensor-core GEMVs - each optionally followed by an RMSNorm - into
  `gemv_chain` ops: one persistent launch per run whose CTAs stream every job's weights back to
  back (csrc/gemv_chain.cu). In a decode step the runs are o -> norm -> gate|up -> down -> norm ->
  next qkv, broken by each attention. Same results as the separate launches up to the fp32
  summation order of split row blocks. Off by default (env AF_GEMV_CHAIN=1 turns it on): on B200
  the chain's split-K reductions through L2 and its per-job barrier make a layer's chain slower
  than the separate cluster-reduced launches (91 against ~60 us at Llama-3-8B shapes)."""
  import ctypes
  if enable is None:
    enable = os.environ.get("AF_GEMV_CHAIN", "0") == "1"
  if not enable:
    return
  lib = R.load_library()

  def chainable(kind, kv):
    return (kind == "gemv" and kv.get("wf") in ("i8t", "i4t") and kv.get("epi") in ("f32", "f16", "resid", "swiglu")
            and kv.get("experts", "-") == "-" and not kv.get("gemm") and kv.get("rw", "-") == "-"
            and kv.get("sel", "-") == "-" and int(kv["nb"]) <= 16 and "pf" not in kv)

  def norm_tail(kind, kv):
    return kind == "rmsnorm" and not int(kv.get("xf16", 0)) and "pf" not in kv

  out, run = [], []
  keys = {"w": "w", "s": "s", "bias": "b", "x": "x", "ldx": "ldx", "y": "y", "ldy": "ldy", "n": "n", "k": "k",
          "epi": "epi"}

  def flush():
    for s in range(0, len(run), 8):
      emit(run[s:s + 8])
    run.clear()

  def emit(jobs):
    if len(jobs) < 2:
      for g, n in jobs:                                  # a lone GEMV stays a plain launch
        out.append(("gemv", g))
        if n is not None:
          out.append(("rmsnorm", n))
      return
    nb, wf = int(jobs[0][0]["nb"]), jobs[0][0]["wf"]
    Ns = (ctypes.c_int * len(jobs))(*[int(g["n"]) for g, _ in jobs])
    Ks = (ctypes.c_int * len(jobs))(*[int(g["k"]) for g, _ in jobs])
    nbytes = lib.af_gemv_chain_scratch_bytes(len(jobs), Ns, Ks, nb, 2 if wf == "i4t" else 0)
    if not nbytes:
      raise RuntimeError("gemv_chain: no scratch size for these shapes")
    kv = dict(jobs=len(jobs), nb=nb, wf=wf, scr=pb.buf("chain.scr", nbytes, "scratch"))
    for j, (g, n) in enumerate(jobs):
      p = f"j{j}."
      kv.update({p + ck: g[gk] for gk, ck in keys.items() if g.get(gk, "-") != "-"})
      if n is not None:
        kv.update({p + "nx": n["x"], p + "ng": n["g"], p + "nf": n["floor"], p + "nout": n["out"], p + "nd": n["d"]})
        if "ldx" in n:
          kv[p + "ldnx"] = n["ldx"]
        if "ldo" in n:
          kv[p + "ldno"] = n["ldo"]
    out.append(("gemv_chain", kv))

  for kind, kv in pb.ops:
    if chainable(kind, kv):
      if run and (run[0][0]["wf"] != kv["wf"] or int(run[0][0]["nb"]) != int(kv["nb"])):
        flush()
      run.append((kv, None))
    elif norm_tail(kind, kv) and run and run[-1][1] is None and int(kv["nb"]) == int(run[0][0]["nb"]):
      run[-1] = (run[-1][0], kv)
    else:
      flush()
      out.append((kind, kv))
  flush()
  pb.ops[:] = out


def plan_fuse_allreduce_norm(pb, enable=None):
  """Tensor parallel: each residual all-reduce followed by the RMSNorm of the same residual becomes
  one `allreduce_rms` op (csrc/comm.cu): h += the ranks' sum, then the norm, in one launch. Env
  AF_TP_FUSED_NORM=1 turns it on; off by default: at TP2 on the 8B shape the single-CTA fused launch
  measured 460.8 against 465.7 tok/s for the all-reduce and the rmsnorm kernel apart."""
  if enable is None:
    enable = os.environ.get("AF_TP_FUSED_NORM", "0") == "1"
  if not enable:
    return
  out = []
  ops = pb.ops
  i = 0
  while i < len(ops):
    kind, kv = ops[i]
    if (kind == "allreduce" and i + 1 < len(ops) and ops[i + 1][0] == "rmsnorm" and kv.get("addto", "-") != "-"):
      nk = ops[i + 1][1]
      nb, d = int(nk["nb"]), int(nk["d"])
      if (nk["x"] == kv["addto"] and nb * d == int(kv["n"]) and not int(nk.get("xf16", 0))
          and int(nk.get("ldx", d)) == d and int(nk.get("ldo", d)) == d and "pf" not in nk):
        out.append(("allreduce_rms", dict(src=kv["src"], dst=kv["dst"], h=kv["addto"], nb=nb, d=d, g=nk["g"],
                                          out=nk["out"], floor=nk["floor"])))
        i += 2
        continue
    out.append((kind, kv))
    i += 1
  pb.ops[:] = out


def plan_l2_prefetch(pb, budget=None, mode=None):
  """Attach L2 prefetch keys to a decode plan: each tensor-core GEMV's weights are (partly) fetched
  into L2 by the kernel that runs before it - the previous GEMV once its own weight copies are all
  requested, or an attention / norm kernel at its start - so HBM keeps streaming through the
  dependent-launch gaps (kernel drain, attention, norms). Up to `budget` bytes per target (env
  AF_L2_PF_MB, default 0: off), the first share of each of the target's CTA ranges. Off by default:
  on B200 bulk prefetches queue on the issuing SM's copy engine, so beyond a few MB they slow the
  issuing kernel more than they save.
  mode "first": only the earliest kernel before the target issues; "all": every kernel in between."""
  import ctypes
  if budget is None:
    budget = int(float(os.environ.get("AF_L2_PF_MB", "0")) * (1 << 20))
  mode = mode or os.environ.get("AF_L2_PF_MODE", "first")
  if budget <= 0:
    return
  lib = R.load_library()
  ops = pb.ops

  def tc_gemv(kind, kv):
    return (kind == "gemv" and kv.get("wf") in ("i8t", "i4t") and "experts" not in kv and not kv.get("gemm"))

  epis = {"f32": 0, "f16": 1, "resid": 2, "swiglu": 3}

  def attach(kv, t, keep):
    total = pb.bufs[t["w"]].nbytes
    grid, cs = ctypes.c_int(), ctypes.c_int()
    if lib.af_gemv_tc_grid(int(t["n"]), int(t["k"]), int(t["nb"]), epis[t["epi"]], 2 if t["wf"] == "i4t" else 0,
                           ctypes.byref(grid), ctypes.byref(cs)) != 0:
      return False
    kv.update(pf=t["w"], pfs=total, pfn=min(total, budget), pfg=max(1, grid.value), pfk=int(keep))
    return True

  if mode == "ahead":
    # each layer's attention (latency-bound: HBM nearly idle) prefetches the NEXT layer's fused qkv
    # weights with the evict-last priority, so that they survive the layer's MLP stream
    attn = [i for i, (kind, _) in enumerate(ops) if kind == "attn_decode"]
    for i, j2 in zip(attn, attn[1:]):
      q = max((j for j in range(i + 1, j2) if tc_gemv(*ops[j])), default=None)
      if q is not None:
        attach(ops[i][1], ops[q][1], keep=True)
    return
  issued = set()
  for i, (kind, kv) in enumerate(ops):
    if not (tc_gemv(kind, kv) or kind in ("attn_decode", "rmsnorm")):
      continue
    j = next((j for j in range(i + 1, len(ops)) if tc_gemv(*ops[j])), None)
    if j is None or (mode == "first" and j in issued):
      continue
    t = ops[j][1]
    total = pb.bufs[t["w"]].nbytes
    grid, cs = ctypes.c_int(), ctypes.c_int()
    rc = lib.af_gemv_tc_grid(int(t["n"]), int(t["k"]), int(t["nb"]), epis[t["epi"]], 2 if t["wf"] == "i4t" else 0,
                             ctypes.byref(grid), ctypes.byref(cs))
    if rc != 0:
      continue
    kv.update(pf=t["w"], pfs=total, pfn=min(total, budget), pfg=max(1, grid.value))
    issued.add(j)


# ------------------------------------------------------------------------------ the runner

class LlamaPrefill:
  """A decoder resident on one B200. `prefill(ids)` returns next-token logits; `generate(...)` runs
  greedy / sampled decode over a device-resident KV cache. Weights: the reference's dict layout
  (`aneforge/llm.py:636-654`) of numpy arrays or torch tensors (host or device)."""

  def __init__(self, cfg: LlamaConfig, weights: dict, compress: str | None = None, ane_lm_head: bool = True,
               device: int = 0, compress_atol: float = 0.05, block_size: int = 32, tp=None, moe_compress="same"):
    # expert weights may use their own format (e.g. int4_g32 experts with int8 attention)
    self.moe_compress = compress if moe_compress == "same" else moe_compress
    self.tp = tp if tp is not None and tp.world > 1 else None
    self.full_cfg, self._w_full = cfg, weights
    if self.tp is not None:
      # this rank's shard (aneforge_b200.tp): local heads / FFN rows / vocabulary rows
      from .tp import plan_shard, shard_model
      self.shard = plan_shard(cfg, self.tp.rank, self.tp.world)
      cfg, weights = shard_model(cfg, weights, self.shard)
    self.cfg = cfg; self.w = weights; self.compress = compress
    self.compress_atol, self.block_size = compress_atol, block_size
    self.device = int(device)
    self.ane_lm_head = ane_lm_head          # kept for API parity: the head always runs on the device
    self.lmhead_tie_margin = 3e-3
    self._chunk_bytes = 1e15                # one program holds every layer on a 180 GB device
    self._chunk_max_layers = 1 << 30
    self._dev = None
    self._dec = None
    self._ver = None
    self._pre = None
    self._head = None
    self._lmT = None
    self.eos_check_every = 16               # greedy device loop: steps between EOS checks

  # -- weights
  def _spec(self, i: int) -> LayerSpec:
    if self.cfg.layers:
      return self.cfg.layers[i]
    lw = self.w["layers"][i]
    return LayerSpec(qk_norm="q_norm" in lw, mlp="moe" if "router" in lw else "swiglu")

  def _layer_chunks(self):
    """Reference chunk plan (`llm.py:425-433`); on B200 decode always runs as one program, which
    is output-invariant to the chunking (there is no ~2 GB per-program ceiling to respect)."""
    per = sum(int(np.prod(np.shape(v))) for v in self.w["layers"][0].values()) * 2
    if self.compress in ("int8", "blockwise"):
      per //= 2
    elif self.compress in ("int4", "int4_g32"):
      per //= 4
    n = max(1, min(self.cfg.n_layers, self._chunk_max_layers, int(self._chunk_bytes // max(per, 1))))
    return [range(i, min(i + n, self.cfg.n_layers)) for i in range(0, self.cfg.n_layers, n)]

  def _load(self):
    """Quantize + pack every weight onto the device once (the reference bakes them per compile)."""
    if self._dev is not None:
      return self._dev
    import torch
    R.lib()
    cfg, dev = self.cfg, torch.device("cuda", self.device)
    c, atol, bs = self.compress, self.compress_atol, self.block_size
    layers = []
    for i in range(cfg.n_layers):
      lw = self.w["layers"][i]
      ls = self._spec(i)
      if ls.mixer not in DECODE_MIXERS:
        raise NotImplementedError(f"mixer {ls.mixer!r} has no B200 emitter or graph builder")
      if ls.mlp not in DECODE_MLPS:
        raise NotImplementedError(f"mlp {ls.mlp!r} has no B200 emitter or graph builder")
      d = {}
      if not is_graph_builder(DECODE_MIXERS[ls.mixer]):
        # the fused attention mixer; a graph-builder mixer is lowered from the host weights instead
        d["qkv"] = encode_linear([lw["wq"], lw["wk"], lw["wv"]], c, dev,
                                 biases=[lw.get("q_bias"), lw.get("k_bias"), lw.get("v_bias")], atol=atol,
                                 block_size=bs)
        d["o"] = encode_linear([lw["wo"]], c, dev, biases=[lw.get("o_bias")], atol=atol, block_size=bs)
        if cfg.norm_type == "layer":
          d["attn_lw"] = to_device(lw["attn_norm_w"], dev, torch.float16)
          d["attn_lb"] = to_device(lw["attn_norm_b"], dev, torch.float16)
        else:
          d["attn_g"], d["attn_floor"] = rms_weights(lw["attn_norm"], cfg.norm_eps, dev)
        if ls.qk_norm:
          d["qn"], d["qn_floor"] = rms_weights(lw["q_norm"], cfg.norm_eps, dev)
          d["kn"], d["kn_floor"] = rms_weights(lw["k_norm"], cfg.norm_eps, dev)
      if is_graph_builder(DECODE_MLPS[ls.mlp]):
        layers.append(d)
        continue
      d["mlp_g"], d["mlp_floor"] = rms_weights(lw["mlp_norm"], cfg.norm_eps, dev)
      if ls.mlp == "swiglu":
        d["gu"] = encode_linear([lw["wgate"], lw["wup"]], c, dev, swiglu=True, atol=atol, block_size=bs)
        d["down"] = encode_linear([lw["wdown"]], c, dev, atol=atol, block_size=bs)
      else:
        d.update(DECODE_MLP_LOADERS[ls.mlp](self, lw, dev))
      layers.append(d)
      free = getattr(self.w["layers"], "free", None)
      if free is not None:
        free(i)                              # a lazily read checkpoint layer is on the device now
    extra = {}
    if cfg.norm_type == "layer":
      fg, ff = to_device(self.w["final_norm_w"], dev, torch.float16), None
      extra["final_b"] = to_device(self.w["final_norm_b"], dev, torch.float16)
    else:
      fg, ff = rms_weights(self.w["final_norm"], cfg.norm_eps, dev)
    if self.w.get("wpe") is not None:
      extra["wpe"] = to_device(self.w["wpe"], dev, torch.float16)       # learned positions (GPT-2)
    lm = self.w["lm_head"]
    self._head_exact = fp16_bits_exact(lm)
    self._dev = {"layers": layers, "final_g": fg, "final_floor": ff, **extra,
                 "embed": to_device(self.w["embed"], dev, torch.float16),
                 "lm_head": to_device(lm, dev, torch.float16),
                 "kvc": _blob.gqa_expand_factor(cfg.n_kv_heads, cfg.n_heads // cfg.n_kv_heads, c, atol, bs),
                 "scale": float(np.float16(1.0 / cfg.dh ** 0.5))}
    return self._dev

  def weight_bytes(self) -> dict:
    """Device bytes by role (for roofline accounting)."""
    d = self._load()
    proj = sum(l[k].nbytes for l in d["layers"] for k in ("qkv", "o", "gu", "down") if k in l)
    return {"projections": proj, "lm_head": d["lm_head"].numel() * 2,
            "norms": sum(l[k].numel() * 2 for l in d["layers"] for k in ("attn_g", "mlp_g", "attn_lw", "attn_lb")
                         if k in l)}

  def _bind_globals(self, prog):
    """The final norm's weights and GPT-2's position table."""
    d = self._load()
    prog.bind("final_g", d["final_g"])
    if "final_b" in d:
      prog.bind("final_b", d["final_b"])
    if "wpe" in d:
      prog.bind("wpe", d["wpe"])

  def _bind_layer(self, prog, li, d, with_kv_state=True):
    if "experts" in d:
      ex = d["experts"]
      prog.bind(f"L{li}.egu.w", ex.gu_w); prog.bind(f"L{li}.edown.w", ex.down_w)
      if ex.gu_s is not None:
        prog.bind(f"L{li}.egu.s", ex.gu_s); prog.bind(f"L{li}.edown.s", ex.down_s)
    for key in ("qkv", "o", "gu", "down", "router", "shgu", "shdown", "shg"):
      if key not in d:
        continue
      lin = d[key]
      prog.bind(f"L{li}.{key}.w", lin.w)
      if lin.s is not None:
        prog.bind(f"L{li}.{key}.s", lin.s)
      if lin.bias is not None:
        prog.bind(f"L{li}.{key}.b", lin.bias)
      if lin.rowoff is not None:
        prog.bind(f"L{li}.{key}.ro", lin.rowoff)
    for key in ("attn_g", "mlp_g", "qn", "kn", "attn_lw", "attn_lb"):
      if key in d:
        prog.bind(f"L{li}.{key}", d[key])

  def _declare_layer_weights(self, pb, li, d):
    if "experts" in d:
      ex = d["experts"]
      pb.buf(f"L{li}.egu.w", ex.gu_w.numel(), "weight"); pb.buf(f"L{li}.edown.w", ex.down_w.numel(), "weight")
      if ex.gu_s is not None:
        pb.buf(f"L{li}.egu.s", ex.gu_s.numel() * 2, "weight"); pb.buf(f"L{li}.edown.s", ex.down_s.numel() * 2, "weight")
    for key in ("qkv", "o", "gu", "down", "router", "shgu", "shdown", "shg"):
      if key not in d:
        continue
      lin = d[key]
      pb.buf(f"L{li}.{key}.w", lin.w.numel() * lin.w.element_size(), "weight")
      if lin.s is not None:
        pb.buf(f"L{li}.{key}.s", lin.s.numel() * 2, "weight")
      if lin.bias is not None:
        pb.buf(f"L{li}.{key}.b", lin.bias.numel() * 2, "weight")
      if lin.rowoff is not None:
        pb.buf(f"L{li}.{key}.ro", lin.rowoff.numel() * 4, "weight")
    for key in ("attn_g", "mlp_g", "qn", "kn", "attn_lw", "attn_lb"):
      if key in d:
        pb.buf(f"L{li}.{key}", d[key].numel() * 2, "weight")

  def _ctx(self, NB, M, decode=True):
    cfg, d = self.cfg, self._load()
    G = cfg.n_heads // cfg.n_kv_heads
    # split-K over the cache: one split per 64 cache rows (the kernel also keeps >= 64 keys per
    # busy split at shorter positions), but all CTAs in one wave (2 CTAs of 8 warps per SM) and at
    # most 64 splits. Up to 16 splits of a head run as one thread-block cluster and merge in its
    # shared memory; at most 12 (then 16) while each split then holds at most 512 keys (on B200,
    # decoding at positions 512-830, clusters of 10-12 beat 8 and 16); past that the splits merge
    # through scratch (the last CTA of each head merges them).
    nsplit = decode_nsplit(M, cfg.n_kv_heads, NB)
    return {"NB": NB, "M": M, "nsplit": nsplit, "scale": d["scale"], "kvc": d["kvc"], "expand": G > 1 and d["kvc"] != 1.0,
            "tp": self.tp is not None, "tp_rank": self.tp.rank if self.tp is not None else 0, "D": cfg.dim,
            "gemm_min": DECODE_GEMM_MIN_ROWS if decode else GEMM_MIN_ROWS}

  # -- programs
  def _decoder(self, M, NB=1):
    """Build (once, cached by (M, NB)) the decode-step program: embedding gather -> all layers ->
    final norm -> lm_head + greedy argmax; KV caches and the token/position are resident state."""
    M, NB = int(M), int(NB)
    if self._dec is not None and self._dec["M"] == M and self._dec["NB"] == NB:
      return self._dec
    if self._dec is not None:
      self._dec["prog"].release()
      self._dec = None
    self._dec = self._build_decoder(M, NB, verify=False)
    return self._dec

  def _verifier(self, M, Kq):
    """The speculative-verify program (cached by (M, Kq)): the decode step over Kq consecutive tokens
    of one sequence at positions pos[0..Kq) sharing one resident cache - each row appends its K / V
    and attends up to its own position; the head's greedy argmax gives the target's next token after
    each of them (the reference's multi-token verify, `aneforge/speculative.py:21-106`)."""
    M, Kq = int(M), int(Kq)
    if self._ver is not None and self._ver["M"] == M and self._ver["NB"] == Kq:
      return self._ver
    if self._ver is not None:
      self._ver["prog"].release()
      self._ver = None
    if any(self._spec(i).mixer != "attention" or is_graph_builder(DECODE_MIXERS["attention"])
           for i in range(self.cfg.n_layers)) or self.tp is not None:
      raise NotImplementedError("speculative verify needs the fused attention mixer on one GPU")
    self._ver = self._build_decoder(M, Kq, verify=True)
    return self._ver

  def _check_positions(self, n):
    """A learned position table bounds the sequence (reference `aneforge/llm.py:298-303`)."""
    wpe = self.w.get("wpe")
    if wpe is not None and n > np.shape(wpe)[0]:
      raise ValueError(f"sequence length {n} exceeds this model's {np.shape(wpe)[0]} max positions")

  def _build_decoder(self, M, NB, verify):
    self._check_positions(M)
    cfg, d = self.cfg, self._load()
    D, H, KV, dh, V = cfg.dim, cfg.n_heads, cfg.n_kv_heads, cfg.dh, cfg.vocab
    Q = (H + 2 * KV) * dh
    ctx = self._ctx(NB, M)
    ctx["verify"] = verify
    CB = 1 if verify else NB                                # sequences with a cache of their own
    pb = PlanBuilder()
    pb.buf("tok", 4 * NB, "state"); pb.buf("pos", 4 * NB, "state")
    pb.buf("tok_out", 4 * NB, "out"); pb.buf("hist", 4 * NB * M, "out")
    pb.buf("hid", 2 * NB * D, "out"); pb.buf("logits", 4 * NB * V, "out")
    pb.buf("h", 4 * NB * D, "tmp"); pb.buf("xn", 2 * NB * D, "tmp"); pb.buf("qkv", 4 * NB * Q, "tmp")
    pb.buf("att", 2 * NB * H * dh, "tmp")
    F = max([l["gu"].N // 2 for l in d["layers"] if "gu" in l] + [l["experts"].F for l in d["layers"] if "experts" in l]
            + [l["shgu"].N // 2 for l in d["layers"] if "shgu" in l] + [1])
    pb.buf("act", 2 * NB * F, "tmp")
    VL = int(d["lm_head"].shape[0])                       # local vocabulary rows (all of them without TP)
    pb.buf("embed", 2 * V * D, "weight"); pb.buf("lm_head", 2 * VL * D, "weight"); pb.buf("final_g", 2 * D, "weight")
    if cfg.norm_type == "layer":
      pb.buf("final_b", 2 * D, "weight")
    if cfg.rope:
      pb.buf("rope.cos", 2 * M * dh, "weight"); pb.buf("rope.sin", 2 * M * dh, "weight")
    if self.tp is not None:
      pb.buf("tp.part", 4 * NB * D, "tmp")
      pb.buf("tp.cand", 8 * NB, "tmp"); pb.buf("tp.gath", 8 * NB * self.tp.world, "tmp")
      pb.buf("logits", 4 * NB * VL, "out")
    from . import kernels
    if ctx["nsplit"] > 1:
      pb.buf("attn.part", kernels.attn_decode_scratch_bytes(NB, KV, ctx["nsplit"], H // KV, dh), "scratch")
      pb.buf("attn.cnt", 4 * NB * KV, "scratch")
    import ctypes
    nb = ctypes.c_size_t()
    R.check(R.load_library().af_lm_head_argmax_scratch(R.W_F16, VL, D, NB, ctypes.byref(nb)), "scratch")
    pb.buf("am.val", nb.value, "scratch"); pb.buf("am.idx", nb.value, "scratch")
    pb.buf("am.cnt", 4 * ((NB + 3) // 4), "scratch")
    for li in range(cfg.n_layers):
      self._declare_layer_weights(pb, li, d["layers"][li])
      pb.buf(f"L{li}.K", 2 * CB * KV * M * dh, "state"); pb.buf(f"L{li}.V", 2 * CB * KV * M * dh, "state")
    _emit_embedding(pb, cfg, d, NB, "pos")
    lows, gstates = [], []
    graph_mix = [is_graph_builder(DECODE_MIXERS[self._spec(i).mixer]) for i in range(cfg.n_layers)]
    graph_mlp = [is_graph_builder(DECODE_MLPS[self._spec(i).mlp]) for i in range(cfg.n_layers)]
    if (any(graph_mix) or any(graph_mlp)) and (NB != 1 or self.tp is not None):
      raise NotImplementedError("graph-builder layers decode one sequence on one GPU (the reference's runner)")
    if any(graph_mix):
      # the reference's per-step decode inputs, built on the device from the resident position
      for k, n in (("oh", M), ("inv", M), ("mask", M), ("cosp", dh), ("sinp", dh)):
        pb.buf(f"dctx.{k}", 4 * n, "tmp")
      pb.op("g_decode_ctx", pos="pos", cos="rope.cos" if cfg.rope else None, sin="rope.sin" if cfg.rope else None,
            m=M, dh=dh, oh="dctx.oh", inv="dctx.inv", mask="dctx.mask", cosp="dctx.cosp", sinp="dctx.sinp")
    for li in range(cfg.n_layers):
      ls = self._spec(li)
      if graph_mix[li]:
        gstates += self._lower_graph_mixer(pb, li, DECODE_MIXERS[ls.mixer], M, lows)
      else:
        DECODE_MIXERS[ls.mixer](pb, ctx, li, d["layers"][li], cfg, ls)
      if graph_mlp[li]:
        self._lower_graph_mlp(pb, li, DECODE_MLPS[ls.mlp], NB, lows, "dec")
      else:
        DECODE_MLPS[ls.mlp](pb, ctx, li, d["layers"][li], cfg, ls)
    _emit_final_norm(pb, cfg, d, NB)
    if self.tp is None:
      pb.op("gemv", wf="f16", epi="argmax", x="hid", w="lm_head", y="logits", nb=NB, n=V, k=D, amv="am.val",
            ami="am.idx", amc="am.cnt", tok="tok_out", pos="pos", hist="hist", histld=M)
    else:
      # vocabulary shard: local (best logit, global index) -> all-gather -> cross-rank argmax
      pb.op("gemv", wf="f16", epi="argmax", x="hid", w="lm_head", y="logits", nb=NB, n=VL, k=D, amv="am.val",
            ami="am.idx", amc="am.cnt", tok=at("tp.cand", 4 * NB), val="tp.cand", ibase=self.shard.vocab[0])
      pb.op("allgather", src="tp.cand", dst="tp.gath", n=2 * NB, ranks=self.tp.world)
      pb.op("tp_argmax", src="tp.gath", ranks=self.tp.world, nb=NB, tok="tok_out", pos="pos", hist="hist", histld=M)
    plan_gemv_chains(pb)
    plan_fuse_allreduce_norm(pb)
    plan_l2_prefetch(pb)
    ins = {"tok": (NB,), "pos": (NB,)}
    for li in range(cfg.n_layers):
      ins[f"L{li}.K"] = (CB, KV, M, dh); ins[f"L{li}.V"] = (CB, KV, M, dh)
    outs = {"tok_out": (NB,), "hist": (NB, M), "hid": (NB, D), "logits": (NB, VL)}
    dt = {"tok": "int32", "pos": "int32", "tok_out": "int32", "hist": "int32", "logits": "fp32"}
    prog = R.Program.from_text(pb.text(), ins, outs, self.device, dt)
    if self.tp is not None:
      prog.set_comm(self.tp.handle)
    prog.share_buffer(0, "tok_out", 0, "tok")              # device-resident token feedback
    prog.bind("embed", d["embed"]); prog.bind("lm_head", d["lm_head"])
    self._bind_globals(prog)
    if cfg.rope:
      cos_t, sin_t = rope_tables(M, dh, cfg.rope_base, cfg.rotary_dim, cfg.rope_interleaved, cfg.rope_scaling)
      prog.upload("rope.cos", cos_t); prog.upload("rope.sin", sin_t)
    for li in range(cfg.n_layers):
      self._bind_layer(prog, li, d["layers"][li])
    for low in lows:
      low.finish(prog)
    return {"M": M, "NB": NB, "CB": CB, "prog": prog, "plan": pb, "graphs": lows, "gstates": gstates}

  # -- graph-builder registry entries (the reference's form; lowered by `_compile.Lowering`)
  def _lower_graph_mlp(self, pb, li, fn, rows, lows, tag):
    """An MLP graph builder h -> h' over `rows` residual rows: its input is the program's fp32
    residual `h`, its result is copied back into it."""
    from ._compile import Lowering
    from .graph import input as ginput, topo_order
    cfg = self.cfg
    x = ginput((rows, cfg.dim))
    out = fn(x, self.w["layers"][li], cfg, self._spec(li))
    low = Lowering(pb, self.compress, self.compress_atol, self.block_size, self.device, prefix=f"L{li}.{tag}.mlp")
    low.set_value(x, "h")
    order = topo_order(out)
    stray = [t for t in order if t.op == "input" and t is not x]
    if stray:
      raise ValueError(f"layer {li}: an MLP graph builder may only read its input (found {len(stray)} more)")
    low.lower(order, {id(t): f"n{i}" for i, t in enumerate(order)})
    if low.value(out) != "h":
      pb.op("copy", dst="h", src=low.value(out), bytes=4 * rows * cfg.dim)
    lows.append(low)

  def _lower_graph_mixer(self, pb, li, fn, M, lows):
    """A decode-mixer graph builder (x, w, cfg, ls, ctx, M) -> (h, state pairs): x is the residual,
    ctx the per-step inputs the program builds from the position, and every (out, in) state pair a
    resident fp16 state buffer (the reference aliases it with `share_buffer`) that the step reads
    at its start and writes back at its end. Returns [(state buffer, elements)]."""
    from . import blocks
    from ._compile import Lowering
    from .graph import input as ginput, topo_order
    cfg = self.cfg
    x = ginput((1, cfg.dim))
    ctx = blocks.decode_inputs(M, cfg.dh)
    out, pairs = fn(x, self.w["layers"][li], cfg, self._spec(li), ctx, M)
    low = Lowering(pb, self.compress, self.compress_atol, self.block_size, self.device, prefix=f"L{li}.mix")
    low.set_value(x, "h")
    for k, t in ctx.items():
      low.set_value(t, f"dctx.{k}")
    states = []
    for j, (o, i) in enumerate(pairs):
      if o.shape != i.shape:
        raise ValueError(f"layer {li}: state pair {j} changes shape {i.shape} -> {o.shape}")
      sb = pb.buf(f"L{li}.gs{j}", 2 * i.size, "state")
      v = low._buf(f"gs{j}.v", 4 * i.size)
      pb.op("cast", src=sb, dst=v, n=i.size, mode=0)
      low.set_value(i, v)
      states.append((sb, i.size))
    order = topo_order(out, *[o for o, _ in pairs])
    known = {id(x), *(id(t) for t in ctx.values()), *(id(i) for _, i in pairs)}
    stray = [t for t in order if t.op == "input" and id(t) not in known]
    if stray:
      raise ValueError(f"layer {li}: a mixer graph reads {len(stray)} input(s) that are neither ctx nor state")
    low.lower(order, {id(t): f"n{i}" for i, t in enumerate(order)})
    for j, (o, _) in enumerate(pairs):
      pb.op("cast", src=low.value(o), dst=f"L{li}.gs{j}", n=o.size, mode=1)
    pb.op("copy", dst="h", src=low.value(out), bytes=4 * cfg.dim)
    lows.append(low)
    return states

  def _batched_prefill_ok(self) -> bool:
    """Batched prefill needs the fused attention mixer in every layer (the reference's rule:
    batched prefill supports attention layers only)."""
    return all(self._spec(i).mixer == "attention" and not is_graph_builder(DECODE_MIXERS["attention"])
               for i in range(self.cfg.n_layers))

  def _prefiller(self, seq):
    """Build (once, cached by seq) the batched-prefill program: all layers over `seq` rows, each
    attention layer's K (roped) / V written as [KV, seq, dh] outputs, final norm -> hidden."""
    seq = int(seq)
    if self._pre is not None and self._pre["seq"] == seq:
      return self._pre
    if self._pre is not None:
      self._pre["prog"].release()
      self._pre = None
    self._check_positions(seq)
    cfg, d = self.cfg, self._load()
    D, H, KV, dh, V = cfg.dim, cfg.n_heads, cfg.n_kv_heads, cfg.dh, cfg.vocab
    Q = (H + 2 * KV) * dh
    ctx = self._ctx(seq, seq, decode=False)
    pb = PlanBuilder()
    pb.buf("ids", 4 * seq, "in"); pb.buf("hid", 2 * seq * D, "out")
    pb.buf("h", 4 * seq * D, "tmp"); pb.buf("xn", 2 * seq * D, "tmp"); pb.buf("qkv", 4 * seq * Q, "tmp")
    pb.buf("att", 2 * seq * H * dh, "tmp"); pb.buf("qbuf", 2 * seq * H * dh, "tmp")
    F = max([l["gu"].N // 2 for l in d["layers"] if "gu" in l] + [l["experts"].F for l in d["layers"] if "experts" in l]
            + [l["shgu"].N // 2 for l in d["layers"] if "shgu" in l] + [1])
    pb.buf("act", 2 * seq * F, "tmp")
    if self.tp is not None:
      pb.buf("tp.part", 4 * seq * D, "tmp")
    pb.buf("embed", 2 * V * D, "weight"); pb.buf("final_g", 2 * D, "weight")
    if cfg.norm_type == "layer":
      pb.buf("final_b", 2 * D, "weight")
    if cfg.rope:
      pb.buf("rope.cos", 2 * seq * dh, "weight"); pb.buf("rope.sin", 2 * seq * dh, "weight")
    for li in range(cfg.n_layers):
      self._declare_layer_weights(pb, li, d["layers"][li])
      pb.buf(f"L{li}.K", 2 * KV * seq * dh, "out"); pb.buf(f"L{li}.V", 2 * KV * seq * dh, "out")
    _emit_embedding(pb, cfg, d, seq, None)
    lows = []
    for li in range(cfg.n_layers):
      ls = self._spec(li)
      if ls.mixer != "attention" or is_graph_builder(PREFILL_MIXERS[ls.mixer]):
        raise NotImplementedError("batched prefill supports attention layers only")
      PREFILL_MIXERS[ls.mixer](pb, ctx, li, d["layers"][li], cfg, ls)
      mlp = PREFILL_MLPS.get(ls.mlp)
      if mlp is None:
        raise NotImplementedError(f"mlp {ls.mlp!r} has no prefill emitter or graph builder")
      if is_graph_builder(mlp):
        self._lower_graph_mlp(pb, li, mlp, seq, lows, "pre")
      else:
        mlp(pb, ctx, li, d["layers"][li], cfg, ls)
    _emit_final_norm(pb, cfg, d, seq)
    outs = {"hid": (seq, D)}
    for li in range(cfg.n_layers):
      outs[f"L{li}.K"] = (KV, seq, dh); outs[f"L{li}.V"] = (KV, seq, dh)
    prog = R.Program.from_text(pb.text(), {"ids": (seq,)}, outs, self.device, {"ids": "int32"})
    if self.tp is not None:
      prog.set_comm(self.tp.handle)
    prog.bind("embed", d["embed"])
    self._bind_globals(prog)
    if cfg.rope:
      cos_t, sin_t = rope_tables(seq, dh, cfg.rope_base, cfg.rotary_dim, cfg.rope_interleaved, cfg.rope_scaling)
      prog.upload("rope.cos", cos_t); prog.upload("rope.sin", sin_t)
    for li in range(cfg.n_layers):
      self._bind_layer(prog, li, d["layers"][li])
    for low in lows:
      low.finish(prog)
    self._pre = {"seq": seq, "prog": prog, "graphs": lows}
    return self._pre

  def _head_program(self, NB=1):
    """lm_head + argmax over NB fp16 hidden rows (the reference's `_lm_head_program`, `llm.py:357-385`)."""
    if self._head is not None and self._head["NB"] == NB:
      return self._head
    if self._head is not None:
      self._head["prog"].release()
    cfg, d = self.cfg, self._load()
    D, V = cfg.dim, cfg.vocab
    import ctypes
    nb = ctypes.c_size_t()
    R.check(R.load_library().af_lm_head_argmax_scratch(R.W_F16, V, D, NB, ctypes.byref(nb)), "scratch")
    pb = PlanBuilder()
    pb.buf("x", 2 * NB * D, "in"); pb.buf("logits", 4 * NB * V, "out"); pb.buf("tok", 4 * NB, "out")
    pb.buf("lm_head", 2 * V * D, "weight")
    pb.buf("am.val", nb.value, "scratch"); pb.buf("am.idx", nb.value, "scratch")
    pb.buf("am.cnt", 4 * ((NB + 3) // 4), "scratch")
    pb.op("gemv", wf="f16", epi="argmax", x="x", w="lm_head", y="logits", nb=NB, n=V, k=D, amv="am.val",
          ami="am.idx", amc="am.cnt", tok="tok")
    prog = R.Program.from_text(pb.text(), {"x": (NB, D)}, {"logits": (NB, V), "tok": (NB,)}, self.device,
                               {"logits": "fp32", "tok": "int32"})
    prog.bind("lm_head", d["lm_head"])
    self._head = {"NB": NB, "prog": prog}
    return self._head

  # -- reference API
  def compile(self, seq: int):
    self._prefiller(seq)
    return self

  def warmup(self, max_len):
    self._decoder(int(max_len))
    self._head_program()
    return self

  def release(self) -> None:
    for k in ("_dec", "_ver", "_pre", "_head"):
      v = getattr(self, k)
      if v is not None:
        v["prog"].release()
      setattr(self, k, None)
    self._dev = None
    self._lmT = None

  def _host_logits(self, hidden_row):
    if self._lmT is None:
      lm = self._w_full["lm_head"]                       # the whole head, also under tensor parallelism
      self._lmT = np.ascontiguousarray(np.asarray(
        lm.detach().float().cpu().numpy() if hasattr(lm, "detach") else lm).T, F32)
    return np.asarray(hidden_row, F32) @ self._lmT

  def _logits(self, hidden_row, ane=None):
    """Device lm_head (fp16 weights, fp32 accumulation) for one fp16 hidden row [D]; under tensor
    parallelism each rank holds only a vocabulary shard, so the full-row logits come from the host."""
    if self.tp is not None:
      return self._host_logits(np.asarray(hidden_row, F16).astype(F32))
    hp = self._head_program()["prog"]
    hp.set_input("x", np.asarray(hidden_row).astype(F16)[None])
    hp.execute()
    return hp.read_output("logits")[0]

  def _decode_logits(self, hidden_row, use_ane, greedy):
    """Logits with the reference's greedy tie-margin protocol (`llm.py:395-404`): only a head whose
    weights are not exactly fp16 can differ from the host fp32 head, and then a near tie is
    recomputed on the host."""
    logits = self._logits(hidden_row)
    if greedy and not self._head_exact:
      p = np.partition(logits, -2)
      if p[-1] - p[-2] < self.lmhead_tie_margin * (float(np.abs(logits).max()) + 1e-9):
        logits = self._host_logits(np.asarray(hidden_row, F16).astype(F32))
    return logits

  @staticmethod
  def _sample(logits, temperature, top_p, top_k):
    """Next token from host logits, with the reference's sampling rules (`aneforge/llm.py:407-419`):
    greedy argmax at temperature <= 0; otherwise softmax(logits / temperature) restricted to the
    logits >= the k-th largest (top_k > 0) and to the most probable tokens whose probability mass
    first reaches top_p (the token that crosses top_p included), renormalised, one draw from
    numpy's global generator."""
    return sample_token(logits, temperature, top_p, top_k)

  def _prefill_hidden(self, token_ids, pad_to=None):
    real = len(token_ids)
    seq = max(int(pad_to), real) if pad_to else real
    pre = self._prefiller(seq)
    ids = np.asarray(list(token_ids) + [0] * (seq - real), np.int32)
    self._check_ids(ids)
    pre["prog"].set_input("ids", ids)
    pre["prog"].execute()
    return pre, real, seq

  def _check_ids(self, ids):
    ids = np.asarray(ids)
    if ids.size and (ids.min() < 0 or ids.max() >= self.cfg.vocab):
      raise ValueError(f"token id out of range [0, {self.cfg.vocab})")

  def prefill(self, token_ids):
    """Prefill and return next-token logits [1, vocab] (reference `llm.py:421-423`)."""
    pre, real, _ = self._prefill_hidden(token_ids)
    hid = pre["prog"].read_output("hid")
    return self._logits(hid[real - 1])[None]

  def _seed_cache(self, dec, pre, real, slot=0):
    """Copy the prefill K/V [KV, real, dh] into decode cache slot `slot`, positions [0, real)
    (reference `_seed_cache`, `llm.py:546-558`) - device to device."""
    cfg = self.cfg
    KV, dh, M, NB = cfg.n_kv_heads, cfg.dh, dec["M"], dec.get("CB", dec["NB"])
    seq = pre["seq"]
    for li in range(cfg.n_layers):
      for nm in ("K", "V"):
        src = pre["prog"].tensor(f"L{li}.{nm}", (KV, seq, dh))
        dst = dec["prog"].tensor(f"L{li}.{nm}", (NB, KV, M, dh))
        dst[slot, :, :real].copy_(src[:, :real])

  def _reset_state(self, dec):
    for li in range(self.cfg.n_layers):
      if is_graph_builder(DECODE_MIXERS[self._spec(li).mixer]):
        continue
      for nm in ("K", "V"):
        dec["prog"].tensor(f"L{li}.{nm}", (dec.get("CB", dec["NB"]), self.cfg.n_kv_heads, dec["M"], self.cfg.dh)).zero_()
    for name, n in dec.get("gstates", ()):
      dec["prog"].tensor(name, (n,)).zero_()

  def generate(self, token_ids, max_new_tokens=40, eos_id=None, max_len=None, on_token=None,
               temperature=0.0, top_p=1.0, top_k=0, batched_prefill=True, prefill_pad=None, on_stage=None,
               ane_lm_head=None):
    """Autoregressive generation over the device-resident KV cache (reference `llm.py:560-633`)."""
    import torch
    cfg = self.cfg
    prompt = [int(t) for t in token_ids]
    self._check_ids(prompt)
    M = int(max_len or len(prompt) + max_new_tokens)
    eos = {int(eos_id)} if isinstance(eos_id, int) else {int(e) for e in (eos_id or ())}
    greedy = temperature <= 0.0
    dec = self._decoder(M, 1)
    prog = dec["prog"]
    with torch.cuda.device(self.device):
      torch.cuda.synchronize()
      self._reset_state(dec)
      torch.cuda.synchronize()
    out = []
    t0 = time.perf_counter()
    if batched_prefill and len(prompt) > 1 and self._batched_prefill_ok():
      pre, real, seq = self._prefill_hidden(prompt, prefill_pad)
      hid = pre["prog"].read_output("hid")
      logits0 = self._decode_logits(hid[real - 1], None, greedy)
      with torch.cuda.device(self.device):
        self._seed_cache(dec, pre, real)
        torch.cuda.synchronize()
      cur = self._sample(logits0, temperature, top_p, top_k)
      out.append(cur)
      if on_stage is not None:
        on_stage("prefill", time.perf_counter() - t0)
      if cur in eos:
        return out
      if on_token is not None:
        on_token(cur)
      pos = real
    else:
      for p, tok in enumerate(prompt[:-1]):
        prog.set_input("tok", np.array([tok], np.int32)); prog.set_input("pos", np.array([p], np.int32))
        prog.execute()
      cur, pos = prompt[-1], len(prompt) - 1
    prog.set_input("tok", np.array([cur], np.int32)); prog.set_input("pos", np.array([pos], np.int32))
    n_steps = min(max_new_tokens - len(out), M - 1 - pos)
    if n_steps <= 0:
      return out
    exact_head = greedy and self._head_exact
    if self.tp is not None and not (exact_head and on_token is None and on_stage is None):
      raise NotImplementedError("tensor-parallel generate runs greedy decode with the on-device head only")
    if exact_head and on_token is None and on_stage is None:
      # greedy with an exact head: every step's token stays on the device; run the steps back to
      # back and read the token history once. With a stop set the steps go in groups of
      # `eos_check_every`, so an early EOS wastes at most one group.
      group = n_steps if not eos else max(1, int(self.eos_check_every))
      done = 0
      while done < n_steps:
        k = min(group, n_steps - done)
        for _ in range(k):
          prog.execute_async()
        prog.sync()
        hist = prog.read_output("hist")[0]
        for t in hist[pos + done:pos + done + k]:
          out.append(int(t))
          if int(t) in eos:
            return out
        done += k
      return out
    # stage names follow the reference's profiling hooks (`aneforge/llm.py:568-575`): the embedding
    # gather, every layer, the head and the greedy argmax all run inside one graph replay here, so
    # `embedding` times the host's token hand-off, `layers` the replay, `lm_head` the host-side
    # logits work (tie-margin recheck or reading the sampled-path logits) and `sample` the draw
    pending = None                             # a host-sampled token still to hand to the device
    for _ in range(n_steps):
      ts = time.perf_counter()
      if pending is not None:
        prog.set_input("tok", np.array([pending], np.int32))
      if on_stage is not None:
        on_stage("embedding", time.perf_counter() - ts)
      t1 = time.perf_counter()
      prog.execute()
      if on_stage is not None:
        on_stage("layers", time.perf_counter() - t1)
        on_stage("step", time.perf_counter() - ts)
      t2 = time.perf_counter()
      if exact_head:
        nxt = int(prog.read_output("tok_out")[0])
        t3 = time.perf_counter()
      else:
        hid = prog.read_output("hid")[0]
        logits = self._decode_logits(hid, None, greedy) if greedy else prog.read_output("logits")[0]
        t3 = time.perf_counter()
        nxt = pending = self._sample(logits, temperature, top_p, top_k)
      if on_stage is not None:
        on_stage("lm_head", t3 - t2)
        on_stage("sample", time.perf_counter() - t3)
      out.append(nxt)
      if nxt in eos:
        break
      if on_token is not None:
        on_token(nxt)
    return out

  def generate_batch(self, prompts, max_new_tokens=40, max_len=None):
    """Greedy decode of NB independent prompts in one batched program (B200 extension; the
    reference runner is batch 1). Each sequence has its own cache slot and position."""
    import torch
    NB = len(prompts)
    prompts = [[int(t) for t in p] for p in prompts]
    for p in prompts:
      self._check_ids(p)
    M = int(max_len or max(len(p) for p in prompts) + max_new_tokens)
    dec = self._decoder(M, NB)
    prog = dec["prog"]
    with torch.cuda.device(self.device):
      torch.cuda.synchronize()
      self._reset_state(dec)
    first, pos = [], []
    for b, p in enumerate(prompts):
      pre, real, _ = self._prefill_hidden(p)
      hid = pre["prog"].read_output("hid")
      first.append(int(np.argmax(self._decode_logits(hid[real - 1], None, True))))
      with torch.cuda.device(self.device):
        self._seed_cache(dec, pre, real, slot=b)
      pos.append(real)
    with torch.cuda.device(self.device):
      torch.cuda.synchronize()
    prog.set_input("tok", np.array(first, np.int32)); prog.set_input("pos", np.array(pos, np.int32))
    n_steps = min(max_new_tokens - 1, M - 1 - max(pos))
    for _ in range(max(0, n_steps)):
      prog.execute_async()
    prog.sync()
    hist = prog.read_output("hist")
    return [[first[b]] + [int(t) for t in hist[b, pos[b]:pos[b] + max(0, n_steps)]] for b in range(NB)]


DECODE_MLP_LOADERS: dict = {}


def decoder_block_step(cfg: LlamaConfig, lw: dict, h, Kc, Vc, pos: int, compress="int8", device: int = 0):
  """One decode step of ONE block (no embedding, final norm or head) through a program: the
  single-block decode workload (d 2048, GQA 16/4, FFN 8192 at pos 1024 is the benchmarked case). h [1, D] fp16; Kc/Vc [KV, M, dh] fp16 prior cache. Returns (fp16 block
  output [1, D], updated K, updated V)."""
  M = int(Kc.shape[1])
  w = {"embed": np.zeros((1, cfg.dim), F16), "lm_head": np.zeros((1, cfg.dim), F16),
       "final_norm": np.ones(cfg.dim, F32), "layers": [lw]}
  c1 = LlamaConfig(**{**cfg.__dict__, "n_layers": 1, "layers": [cfg.layers[0] if cfg.layers else LayerSpec()]})
  m = LlamaPrefill(c1, w, compress=compress, device=device)
  d = m._load()
  D, H, KV, dh = c1.dim, c1.n_heads, c1.n_kv_heads, c1.dh
  ctx = m._ctx(1, M)
  pb = PlanBuilder()
  pb.buf("x", 2 * D, "in"); pb.buf("pos", 4, "state"); pb.buf("out", 2 * D, "out")
  pb.buf("h", 4 * D, "tmp"); pb.buf("xn", 2 * D, "tmp"); pb.buf("qkv", 4 * (H + 2 * KV) * dh, "tmp")
  pb.buf("att", 2 * H * dh, "tmp"); pb.buf("act", 2 * d["layers"][0]["gu"].N // 2, "tmp")
  pb.buf("rope.cos", 2 * M * dh, "weight"); pb.buf("rope.sin", 2 * M * dh, "weight")
  from . import kernels
  if ctx["nsplit"] > 1:
    pb.buf("attn.part", kernels.attn_decode_scratch_bytes(1, KV, ctx["nsplit"], H // KV, dh), "scratch")
    pb.buf("attn.cnt", 4 * KV, "scratch")
  m._declare_layer_weights(pb, 0, d["layers"][0])
  pb.buf("L0.K", 2 * KV * M * dh, "state"); pb.buf("L0.V", 2 * KV * M * dh, "state")
  pb.op("cast", src="x", dst="h", n=D, mode=0)
  ls = c1.layers[0]
  DECODE_MIXERS[ls.mixer](pb, ctx, 0, d["layers"][0], c1, ls)
  DECODE_MLPS[ls.mlp](pb, ctx, 0, d["layers"][0], c1, ls)
  pb.op("cast", src="h", dst="out", n=D, mode=1)
  prog = R.Program.from_text(pb.text(), {"x": (1, D), "pos": (1,), "L0.K": (1, KV, M, dh), "L0.V": (1, KV, M, dh)},
                             {"out": (1, D)}, device, {"pos": "int32"})
  cos_t, sin_t = rope_tables(M, dh, c1.rope_base, c1.rotary_dim, c1.rope_interleaved, c1.rope_scaling)
  prog.upload("rope.cos", cos_t); prog.upload("rope.sin", sin_t)
  m._bind_layer(prog, 0, d["layers"][0])
  prog.set_input("x", np.asarray(h, F16).reshape(1, D))
  prog.set_input("pos", np.array([pos], np.int32))
  prog.set_input("L0.K", np.asarray(Kc, F16)[None]); prog.set_input("L0.V", np.asarray(Vc, F16)[None])
  prog.execute()
  out = prog.read_output("out")
  K = prog.download("L0.K", (KV, M, dh)); V = prog.download("L0.V", (KV, M, dh))
  prog.release(); m.release()
  return out, K, V


# ------------------------------------------------------------------------------ loaders

# Hugging Face checkpoint -> the reference's weight dict (`aneforge/llm.py:636-654` layout). The key
# names are the checkpoint format's; every other detail of the mapping is table-driven here.
_HF_LAYER_REQUIRED = {
  "wq": "self_attn.q_proj.weight", "wk": "self_attn.k_proj.weight", "wv": "self_attn.v_proj.weight",
  "wo": "self_attn.o_proj.weight", "wgate": "mlp.gate_proj.weight", "wup": "mlp.up_proj.weight",
  "wdown": "mlp.down_proj.weight", "attn_norm": "input_layernorm.weight",
  "mlp_norm": "post_attention_layernorm.weight",
}
_HF_LAYER_OPTIONAL = {
  "q_norm": "self_attn.q_norm.weight", "k_norm": "self_attn.k_norm.weight",          # Qwen3 QK-norm
  "q_bias": "self_attn.q_proj.bias", "k_bias": "self_attn.k_proj.bias",              # Qwen2 biases
  "v_bias": "self_attn.v_proj.bias", "o_bias": "self_attn.o_proj.bias",
}
# architectures whose semantics the dense loader does not implement (logit soft-capping, GELU MLPs,
# LayerNorm, sandwich norms): refused rather than silently run as Llama
_HF_REFUSED = {"gemma2", "gemma3", "gemma3_text"}


def hf_weights(sd: dict, n_layers: int) -> dict:
  """Reference weight dict from a Hugging Face Llama / Qwen2 / Qwen3 / Mistral state dict; a model
  without a separate `lm_head.weight` ties its head to the embedding."""
  embed = sd["model.embed_tokens.weight"]
  layers = []
  for i in range(n_layers):
    pre = f"model.layers.{i}."
    lw = {ours: sd[pre + theirs] for ours, theirs in _HF_LAYER_REQUIRED.items()}
    lw.update({ours: sd[pre + theirs] for ours, theirs in _HF_LAYER_OPTIONAL.items() if pre + theirs in sd})
    if ("q_norm" in lw) != ("k_norm" in lw):
      raise ValueError(f"layer {i}: a checkpoint with QK-norm needs both q_norm and k_norm")
    layers.append(lw)
  return {"embed": embed, "final_norm": sd["model.norm.weight"], "lm_head": sd.get("lm_head.weight", embed),
          "layers": layers}


def hf_config(c, sd: dict) -> LlamaConfig:
  """`LlamaConfig` from a Hugging Face config object. The RoPE base is read from `rope_parameters`
  (transformers >= 5) or `rope_theta`; only the "llama3" scaling type changes the tables."""
  rp = getattr(c, "rope_parameters", None)
  theta = rp.get("rope_theta") if isinstance(rp, dict) else None
  theta = float(theta if theta is not None else getattr(c, "rope_theta", 10000.0))
  sc = getattr(c, "rope_scaling", None)
  if not (isinstance(sc, dict) and sc.get("rope_type") == "llama3"):
    sc = rp if isinstance(rp, dict) and rp.get("rope_type") == "llama3" else None
  n = int(c.num_hidden_layers)
  qk = "model.layers.0.self_attn.q_norm.weight" in sd
  return LlamaConfig(dim=int(c.hidden_size), n_layers=n, n_heads=int(c.num_attention_heads),
                     n_kv_heads=int(getattr(c, "num_key_value_heads", None) or c.num_attention_heads),
                     ffn_dim=int(c.intermediate_size), vocab=int(c.vocab_size), rope_base=theta,
                     norm_eps=float(c.rms_norm_eps), head_dim=int(getattr(c, "head_dim", 0) or 0),
                     rope_scaling=sc, layers=[LayerSpec(qk_norm=qk) for _ in range(n)])


def _dense_adapter(c, sd):
  """Llama / Qwen2 / Qwen3 adapter (the reference's default, `aneforge/llm.py:657-668`)."""
  return hf_config(c, sd), hf_weights(sd, int(c.num_hidden_layers))


def _mistral_adapter(c, sd):
  """Mistral (reference `aneforge/llm.py:705-718`): no RoPE scaling; the sliding window, which the
  decode kernels do not apply, is recorded in `cfg.extra` for callers to check."""
  cfg, w = _dense_adapter(c, sd)
  cfg.rope_scaling = None
  win = getattr(c, "sliding_window", None)
  if win:
    cfg.extra["sliding_window"] = int(win)
  return cfg, w


def _gemma_adapter(c, sd):
  """Gemma (reference `aneforge/llm.py:685-702`): Llama-shaped attention, the GeGLU MLP (tanh GELU,
  the "geglu" graph builder) and two conventions baked into the weights - the input embedding is
  scaled by sqrt(hidden) (the head keeps the unscaled, tied rows) and the RMSNorm weights are
  stored as w with the model applying (1 + w)."""
  cfg, w = _dense_adapter(c, sd)
  cfg.rope_scaling = None
  cfg.layers = [LayerSpec(mixer="attention", mlp="geglu") for _ in range(cfg.n_layers)]
  w["embed"] = np.asarray(w["embed"]) * np.sqrt(c.hidden_size)      # float64: rounded once, at the port
  for lw in w["layers"]:
    lw["attn_norm"] = lw["attn_norm"] + 1.0
    lw["mlp_norm"] = lw["mlp_norm"] + 1.0
  w["final_norm"] = w["final_norm"] + 1.0
  return cfg, w


def _gpt2_adapter(c, sd):
  """GPT-2 (reference `aneforge/llm.py:730-767`): LayerNorm with bias, learned positions (`wpe`,
  added to the embedding) instead of RoPE, biases on every projection, the tanh-GELU MLP
  ("gelu_new", a graph builder) and the head tied to the token embedding. HF stores the
  projections as Conv1D [in, out]; they are transposed to [out, in]. Checkpoints that rescale the
  attention per layer or upcast it are refused (their logits would differ)."""
  for flag in ("scale_attn_by_inverse_layer_idx", "reorder_and_upcast_attn"):
    if getattr(c, flag, False):
      raise ValueError(f"load_gpt2: {flag} is set, which this GPT-2 adapter does not implement")
  g = lambda *names: next(getattr(c, n) for n in names if getattr(c, n, None) is not None)
  n, D, H = int(g("n_layer", "num_hidden_layers")), int(g("n_embd", "hidden_size")), int(g("n_head", "num_attention_heads"))
  F = int(getattr(c, "n_inner", None) or getattr(c, "intermediate_size", None) or 4 * D)
  cfg = LlamaConfig(dim=D, n_layers=n, n_heads=H, n_kv_heads=H, ffn_dim=F, vocab=int(c.vocab_size),
                    norm_eps=float(g("layer_norm_epsilon", "layer_norm_eps")), norm_type="layer", rope=False,
                    layers=[LayerSpec(mixer="attention", mlp="gelu_new") for _ in range(n)])
  T = lambda a: np.ascontiguousarray(np.asarray(a).T)
  wte = sd["transformer.wte.weight"]
  w = {"embed": wte, "wpe": sd["transformer.wpe.weight"], "final_norm_w": sd["transformer.ln_f.weight"],
       "final_norm_b": sd["transformer.ln_f.bias"], "lm_head": sd.get("lm_head.weight", wte), "layers": []}
  for i in range(n):
    p = f"transformer.h.{i}."
    qkv, bqkv = T(sd[p + "attn.c_attn.weight"]), np.asarray(sd[p + "attn.c_attn.bias"])
    lw = {"attn_norm_w": sd[p + "ln_1.weight"], "attn_norm_b": sd[p + "ln_1.bias"],
          "wo": T(sd[p + "attn.c_proj.weight"]), "o_bias": sd[p + "attn.c_proj.bias"],
          "mlp_norm_w": sd[p + "ln_2.weight"], "mlp_norm_b": sd[p + "ln_2.bias"],
          "wfc": T(sd[p + "mlp.c_fc.weight"]), "fc_bias": sd[p + "mlp.c_fc.bias"],
          "wproj": T(sd[p + "mlp.c_proj.weight"]), "proj_bias": sd[p + "mlp.c_proj.bias"]}
    for j, (wk, bk) in enumerate((("wq", "q_bias"), ("wk", "k_bias"), ("wv", "v_bias"))):
      lw[wk], lw[bk] = np.ascontiguousarray(qkv[j * D:(j + 1) * D]), bqkv[j * D:(j + 1) * D]
    w["layers"].append(lw)
  return cfg, w


ADAPTERS: list = [
  (lambda c: getattr(c, "model_type", None) == ModelType.GPT2, _gpt2_adapter),
  (lambda c: getattr(c, "model_type", None) == ModelType.GEMMA, _gemma_adapter),
  (lambda c: getattr(c, "model_type", None) == ModelType.MISTRAL, _mistral_adapter),
]


def _assert_dense_compatible(c) -> None:
  """Refuse configs the dense loader would run with the wrong semantics (the reference's guard,
  `aneforge/llm.py:776-788`)."""
  kind = str(getattr(c, "model_type", "?"))
  softcap = getattr(c, "attn_logit_softcapping", None) or getattr(c, "final_logit_softcapping", None)
  if softcap:
    raise ValueError(f"load_llm: {kind!r} uses logit soft-capping, which the B200 dense loader does not implement")
  if kind in _HF_REFUSED:
    raise ValueError(f"load_llm: {kind!r} has architecture-specific semantics the B200 dense loader does not implement")


def from_pretrained(name: str, compress: str | None = None, ane_lm_head: bool = True, device: int = 0) -> LlamaPrefill:
  """Load a Hugging Face decoder (a hub name or a local checkpoint directory; reference
  `aneforge/llm.py:791-806`) onto one B200: the first matching `ADAPTERS` entry maps it, else the
  dense Llama/Qwen adapter."""
  import torch
  from transformers import AutoModelForCausalLM
  hf = AutoModelForCausalLM.from_pretrained(name)
  adapt = next((fn for pred, fn in ADAPTERS if pred(hf.config)), None)
  if adapt is None:
    _assert_dense_compatible(hf.config)
    adapt = _dense_adapter
  # fp16 numpy state dict: the weights are baked to fp16 (or quantized) anyway, and the adapters'
  # weight arithmetic (Gemma's scaled embedding and 1 + w norms) follows numpy's fp16 rules
  sd = {k: v.detach().to(torch.float16).numpy() for k, v in hf.state_dict().items()}
  cfg, weights = adapt(hf.config, sd)
  return LlamaPrefill(cfg, weights, compress=compress, ane_lm_head=ane_lm_head, device=device)
