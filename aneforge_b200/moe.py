"""Mixture-of-experts SwiGLU layers on the device (reference `aneforge/moe.py:40-67`), registered as
the "moe" MLP of the Llama runner the way the reference registers its `_moe` builder.

Per token row: RMSNorm -> router GEMV (the graph's compress=, int8 per row under int8) -> device
gate kernel (fp32 softmax, top-k by row-max peel with the lowest index winning ties, renormalised
when `norm_topk_prob`) -> experts. The reference evaluates every expert densely and weights the
unselected ones by exactly 0; on the device:
  * one sequence (decode at batch 1): only the k selected experts run - their index is read by the
    expert GEMVs from device memory, so the graph is static and 1/4 of Mixtral's expert bytes move;
  * several rows (batched decode, prefill): every expert runs densely over all rows with the
    per-row routing weight applied in the down projection's residual epilogue (0 for unselected
    rows), which at batch >= 32 reads the same bytes a sparse gather would.
Either way each selected expert's contribution is added to the fp32 residual, scaled by its weight.
"""
from __future__ import annotations

from . import _runtime as R
from . import llm
from .weights import encode_experts, encode_linear


def load_moe(runner, lw, dev):
  """Router (graph compress=) and experts (`moe_compress`) of one layer."""
  c = runner.compress
  return {"router": encode_linear([lw["router"]], c, dev, atol=runner.compress_atol, block_size=runner.block_size),
          "experts": encode_experts(lw["wgate_exps"], lw["wup_exps"], lw["wdown_exps"], runner.moe_compress, dev)}


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
  # holds does nothing); several rows: every local expert densely with per-row weights
  picks = [dict(sel="moe.sel", slot=s) for s in range(k)] if sparse else [dict(fixe=e) for e in range(ex.E)]
  for p in picks:
    pb.op("gemv", **gu, **p)
    pb.op("gemv", **dn, **p)


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
  if not ep:
    _expert_gemvs(pb, pre, ex, NB, E, k, sparse=NB == 1)
    return
  n = NB * cfg.dim
  pb.op("fill", dst="tp.part", bytes=4 * n, value=0)
  _expert_gemvs(pb, pre, ex, NB, E, k, sparse=NB == 1, y="tp.part", e_base=e0)
  pb.op("allreduce", src="tp.part", dst="tp.part", n=n, addto="h")


llm.DECODE_MLP_LOADERS["moe"] = load_moe
llm.DECODE_MLPS["moe"] = emit_moe
llm.PREFILL_MLPS["moe"] = emit_moe
