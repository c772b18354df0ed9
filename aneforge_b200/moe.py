"""Mixture-of-experts SwiGLU layers on the device (reference `aneforge/moe.py:40-67`), registered as
the "moe" MLP of the Llama runner the way the reference registers its `_moe` builder.

Per token row: RMSNorm -> router GEMV (the graph's compress=, int8 per row under int8) -> device
gate kernel (fp32 softmax, top-k by row-max peel with the lowest index winning ties, renormalised
when `norm_topk_prob`) -> experts. The reference evaluates every expert densely and weights the
unselected ones by exactly 0; on the device:
  * one sequence (decode at batch 1): only the k selected experts run - their index is read by the
    expert GEMVs from device memory, so the graph is static and 1/4 of Mixtral's expert bytes move;
  * a decode batch (2-64 rows): a routing kernel lists each expert's rows; each expert's GEMVs
    gather only those rows (16 a launch) and scatter the routing-weighted results back, so every
    expert's weights stream about once per step and carry only its share of the rows;
  * prefill (longer row counts): every expert runs densely over all rows with the per-row routing
    weight applied in the down projection's residual epilogue (0 for unselected rows).
Either way each selected expert's contribution is added to the fp32 residual, scaled by its weight.
"""
from __future__ import annotations

from . import _runtime as R
from . import llm
from .weights import encode_experts, encode_linear


def load_moe(runner, lw, dev):
  """Router (graph compress=) and experts (`moe_compress`) of one layer, plus Qwen2-MoE's shared
  expert and its gate when the layer has them (graph compress=, like the router)."""
  c, kw = runner.compress, dict(atol=runner.compress_atol, block_size=runner.block_size)
  d = {"router": encode_linear([lw["router"]], c, dev, **kw),
       "experts": encode_experts(lw["wgate_exps"], lw["wup_exps"], lw["wdown_exps"], runner.moe_compress, dev)}
  if "wgate_sh" in lw:
    d["shgu"] = encode_linear([lw["wgate_sh"], lw["wup_sh"]], c, dev, swiglu=True, **kw)
    d["shdown"] = encode_linear([lw["wdown_sh"]], c, dev, **kw)
    d["shg"] = encode_linear([lw["shared_gate"]], c, dev, **kw)
  return d


def _shared_expert(pb, ctx, pre, lw, y):
  """Qwen2-MoE's always-on shared expert (`aneforge/moe.py:60-62`): y += sigmoid(xn . g) *
  down(silu(gate(xn)) * up(xn)) per row; the sigmoid gate scales the down projection's residual
  epilogue like a routing weight."""
  NB = ctx["NB"]
  pb.buf("moe.shg", 4 * NB, "tmp")
  llm._emit_linear(pb, ctx, f"{pre}.shg", lw["shg"], "xn", "moe.shg", "f32")
  pb.op("g_un", op=2, x="moe.shg", y="moe.shg", n=NB)                 # sigmoid, in place
  llm._emit_linear(pb, ctx, f"{pre}.shgu", lw["shgu"], "xn", "act", "swiglu")
  down = lw["shdown"]
  kv = dict(wf=down.wf, epi="resid", x="act", w=f"{pre}.shdown.w", y=y, nb=NB, n=down.N, k=down.K, rw="moe.shg", rwe=1)
  if down.kind == "int8":
    kv["s"] = f"{pre}.shdown.s"
  if not down.tiled:
    raise NotImplementedError("the shared expert runs on the tensor-core GEMV: compress='int8' (K % 32 == 0) "
                              "or 'int4_g32'")
  nbytes = R.load_library().af_gemv_tc_scratch_bytes(down.N, down.K, NB)
  if nbytes:
    kv["scr"] = pb.buf("gemv.scr", nbytes, "scratch")
  pb.op("gemv", **kv)                                     # per-row gate applied in the residual epilogue


ROUTED_MAX_ROWS = 64           # batches up to this many rows take the routed expert GEMVs


def _expert_gemvs(pb, pre, ex, NB, E, k, sparse, y="h", e_base=0):
  """The expert projections of one layer: `ex` holds experts [e_base, e_base + ex.E) of E; each
  selected expert's down projection adds its routing-weighted output into `y`."""
  lib = R.load_library()
  scr = max(lib.af_gemv_tc_scratch_bytes(2 * ex.F, ex.D, NB), lib.af_gemv_tc_scratch_bytes(ex.D, ex.F, NB))
  if scr:
    pb.buf("gemv.scr", scr, "scratch")
  gu = dict(wf=ex.wf, epi="swiglu", x="xn", w=f"{pre}.egu.w", y="act", nb=NB, n=2 * ex.F, k=ex.D, experts=ex.E,
            ebase=e_base, scr="gemv.scr" if scr else None)
  dn = dict(wf=ex.wf, epi="resid", x="act", w=f"{pre}.edown.w", y=y, nb=NB, n=ex.D, k=ex.F, experts=ex.E,
            ebase=e_base, rw="moe.gw", rwe=E, scr="gemv.scr" if scr else None)
  if ex.gu_s is not None:
    gu["s"] = f"{pre}.egu.s"; dn["s"] = f"{pre}.edown.s"
  # one sequence: the k selected experts, read on the device (a launch whose expert another GPU
  # holds does nothing)
  if sparse:
    for s in range(k):
      pb.op("gemv", **gu, sel="moe.sel", slot=s)
      pb.op("gemv", **dn, sel="moe.sel", slot=s)
    return
  if NB > ROUTED_MAX_ROWS:
    for e in range(ex.E):                    # every expert densely over all rows
      pb.op("gemv", **gu, fixe=e)
      pb.op("gemv", **dn, fixe=e)
    return
  # several rows: per local expert, only the rows routed to it (`moe_route` lists), up to 16 a
  # launch; gate|up gathers those rows of xn into a compact act, down scatters its routing-weighted
  # rows back into y. A list shorter than a launch's share leaves that launch empty (a no-op), so
  # the batch's weights stream about once per expert instead of once per 16 rows.
  R16 = min(16, NB)
  gu.update(nb=R16, xrows=NB, route=1, rows="moe.rows", rcnt="moe.rcnt", rld=NB, eg=E)
  dn.update(nb=R16, yrows=NB, route=2, rows="moe.rows", rcnt="moe.rcnt", rld=NB, eg=E)
  for e in range(ex.E):
    for r0 in range(0, NB, R16):
      pb.op("gemv", **gu, fixe=e, r0=r0)
      pb.op("gemv", **dn, fixe=e, r0=r0)


def emit_moe(pb, ctx, li, lw, cfg, ls):
  """`_moe` (reference `moe.py:48-63`) for NB rows of the program's residual `h`.

  Expert parallel (a tensor-parallel program over a MoE model): every rank routes the same rows
  with the replicated router and gate, runs the experts it holds (`cfg.extra["ep_experts"]`) into a
  zeroed partial, and the partials' all-reduce adds the combined expert output into the residual.
  The hidden rows are replicated on every rank, so dispatch needs no exchange; the combine is the
  one collective (the dense layers' row-parallel all-reduce, same size)."""
  pre, NB = f"L{li}", ctx["NB"]
  ex = lw["experts"]
  E = int(cfg.extra.get("n_experts", ex.E))
  k = int(cfg.extra.get("n_experts_per_tok", 2))
  renorm = bool(cfg.extra.get("norm_topk_prob", True))
  ep = ctx.get("tp")
  e0, e1 = cfg.extra.get("ep_experts", (0, E)) if ep else (0, E)
  if e1 - e0 != ex.E:
    raise ValueError(f"layer {li}: {ex.E} local experts for the range [{e0}, {e1})")
  pb.buf("moe.logits", 4 * NB * E, "tmp"); pb.buf("moe.gw", 4 * NB * E, "tmp"); pb.buf("moe.sel", 4 * NB * k, "tmp")
  pb.op("rmsnorm", x="h", g=f"{pre}.mlp_g", out="xn", nb=NB, d=cfg.dim, floor=lw["mlp_floor"])
  llm._emit_linear(pb, ctx, f"{pre}.router", lw["router"], "xn", "moe.logits", "f32")
  pb.op("moe_gate", logits="moe.logits", nb=NB, e=E, k=k, renorm=int(renorm), gw="moe.gw", sel="moe.sel")
  if 1 < NB <= ROUTED_MAX_ROWS:
    pb.buf("moe.rows", 4 * E * NB, "tmp"); pb.buf("moe.rcnt", 4 * E, "tmp")
    pb.op("moe_route", sel="moe.sel", nb=NB, e=E, k=k, rld=NB, rows="moe.rows", cnt="moe.rcnt")
  if not ep:
    _expert_gemvs(pb, pre, ex, NB, E, k, sparse=NB == 1)
    if "shgu" in lw:
      _shared_expert(pb, ctx, pre, lw, "h")
    return
  n = NB * cfg.dim
  pb.op("fill", dst="tp.part", bytes=4 * n, value=0)
  _expert_gemvs(pb, pre, ex, NB, E, k, sparse=NB == 1, y="tp.part", e_base=e0)
  if "shgu" in lw and ctx.get("tp_rank", 0) == 0:
    _shared_expert(pb, ctx, pre, lw, "tp.part")        # replicated weights: added once, by rank 0
  pb.op("allreduce", src="tp.part", dst="tp.part", n=n, addto="h")


def hf_moe_adapter(c, sd):
  """Qwen3-MoE Hugging Face checkpoints (reference `aneforge/moe.py:70-107`): attention as in the
  dense adapter; a sparse layer's router is `mlp.gate`, its experts the fused
  `mlp.experts.gate_up_proj` [E, 2 ffn, dim] (gate rows first) and `mlp.experts.down_proj`
  [E, dim, ffn], re-laid as the MoE layer's [E, ffn, dim] matrices. `decoder_sparse_step` and
  `mlp_only_layers` choose which layers are sparse; the others are SwiGLU layers."""
  import numpy as np
  cfg = llm.hf_config(c, sd)
  n = cfg.n_layers
  step = int(getattr(c, "decoder_sparse_step", 1) or 1)
  dense_only = set(getattr(c, "mlp_only_layers", None) or [])
  sparse = [li not in dense_only and (li + 1) % step == 0 for li in range(n)]
  qk = cfg.layers[0].qk_norm if cfg.layers else False
  cfg.layers = [llm.LayerSpec(mixer="attention", mlp="moe" if s else "swiglu", qk_norm=qk) for s in sparse]
  cfg.extra.update(n_experts=int(c.num_experts), n_experts_per_tok=int(c.num_experts_per_tok),
                   norm_topk_prob=bool(getattr(c, "norm_topk_prob", True)))
  embed = sd["model.embed_tokens.weight"]
  w = {"embed": embed, "final_norm": sd["model.norm.weight"], "lm_head": sd.get("lm_head.weight", embed), "layers": []}
  for li in range(n):
    pre = f"model.layers.{li}."
    lw = {ours: sd[pre + theirs] for ours, theirs in llm._HF_LAYER_REQUIRED.items()
          if not (sparse[li] and theirs.startswith("mlp."))}
    lw.update({ours: sd[pre + theirs] for ours, theirs in llm._HF_LAYER_OPTIONAL.items() if pre + theirs in sd})
    if sparse[li]:
      gu = np.asarray(sd[pre + "mlp.experts.gate_up_proj"])
      F = gu.shape[1] // 2
      lw["router"] = sd[pre + "mlp.gate.weight"]
      lw["wgate_exps"] = np.ascontiguousarray(gu[:, :F])
      lw["wup_exps"] = np.ascontiguousarray(gu[:, F:])
      lw["wdown_exps"] = np.ascontiguousarray(np.asarray(sd[pre + "mlp.experts.down_proj"]).transpose(0, 2, 1))
    w["layers"].append(lw)
  return cfg, w


llm.ADAPTERS.append((lambda c: bool(getattr(c, "num_experts", 0)), hf_moe_adapter))


def load_gguf(path: str, n_layers: int | None = None, compress: str | None = None, **runner_kw) -> "llm.LlamaPrefill":
  """A Qwen-MoE GGUF checkpoint as a runner (reference `aneforge/moe.py:129-173`): Qwen3-MoE
  (QK-norm) or Qwen2-MoE / Qwen1.5-MoE (QKV biases, the sigmoid-gated shared expert, no top-k
  renormalisation). The architecture's features are read off the tensors present; `n_layers`
  keeps the first layers only. Layer weights are dequantized to fp16 when the runner encodes them
  and dropped right after, so the host never holds the whole model; the embedding and lm_head are
  kept fp32 as the reference keeps them."""
  from .gguf_file import GGUFFile, LazyLayers
  import numpy as np
  g = GGUFFile(path)
  total = int(g.scalar("block_count", 0))
  n = total if n_layers is None else min(int(n_layers), total)
  dim, heads = int(g.scalar("embedding_length", 0)), int(g.scalar("attention.head_count", 0))
  ffn = g.shape("blk.0.ffn_gate_exps.weight")[1]      # [dim, ffn, E]: Qwen1.5 has no ffn length key
  qk_norm = g.has("blk.0.attn_q_norm.weight")
  shared = g.has("blk.0.ffn_gate_shexp.weight")
  cfg = llm.LlamaConfig(
    dim=dim, n_layers=n, n_heads=heads, n_kv_heads=int(g.scalar("attention.head_count_kv", heads)),
    ffn_dim=int(ffn), vocab=g.rows("token_embd.weight"), rope_base=float(g.scalar("rope.freq_base", 10000.0)),
    norm_eps=float(g.scalar("attention.layer_norm_rms_epsilon", 1e-6)),
    head_dim=int(g.scalar("attention.key_length", 0) or dim // heads),
    layers=[llm.LayerSpec(mixer="attention", mlp="moe", qk_norm=qk_norm) for _ in range(n)],
    extra={"n_experts": int(g.scalar("expert_count", 0)), "n_experts_per_tok": int(g.scalar("expert_used_count", 0)),
           "norm_topk_prob": g.arch != "qwen2moe"})

  def layer(i):
    b = f"blk.{i}."
    lw = {"wq": g.get(b + "attn_q.weight"), "wk": g.get(b + "attn_k.weight"), "wv": g.get(b + "attn_v.weight"),
          "wo": g.get(b + "attn_output.weight"), "attn_norm": g.get(b + "attn_norm.weight"),
          "mlp_norm": g.get(b + "ffn_norm.weight"), "router": g.get(b + "ffn_gate_inp.weight"),
          "wgate_exps": g.get(b + "ffn_gate_exps.weight"), "wup_exps": g.get(b + "ffn_up_exps.weight"),
          # stored [E, dim, ffn]; the MoE layer takes [E, ffn, dim]
          "wdown_exps": np.ascontiguousarray(g.get(b + "ffn_down_exps.weight").transpose(0, 2, 1))}
    for key, t in (("q_norm", "attn_q_norm.weight"), ("k_norm", "attn_k_norm.weight"),
                   ("q_bias", "attn_q.bias"), ("k_bias", "attn_k.bias"), ("v_bias", "attn_v.bias")):
      if g.has(b + t):
        lw[key] = g.get(b + t)
    if shared:
      lw.update(wgate_sh=g.get(b + "ffn_gate_shexp.weight"), wup_sh=g.get(b + "ffn_up_shexp.weight"),
                wdown_sh=g.get(b + "ffn_down_shexp.weight"),
                shared_gate=g.get(b + "ffn_gate_inp_shexp.weight").reshape(1, dim))
    g.release_pages()
    return lw

  head = "output.weight" if g.has("output.weight") else "token_embd.weight"     # tied embeddings
  w = {"embed": g.get("token_embd.weight", np.float32), "final_norm": g.get("output_norm.weight"),
       "lm_head": g.get(head, np.float32), "layers": LazyLayers(layer, n)}
  return llm.LlamaPrefill(cfg, w, compress=compress, **runner_kw)


llm.DECODE_MLP_LOADERS["moe"] = load_moe
llm.DECODE_MLPS["moe"] = emit_moe
llm.PREFILL_MLPS["moe"] = emit_moe
