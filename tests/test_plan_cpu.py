"""Plan emission and rewrites on the host (no GPU): the chained-GEMV pass and the tensor-parallel
all-reduce + RMSNorm fusion rewrite a decode plan's op list without changing what it computes; the
MoE expert launches per batch size (selected, routed, dense) and the GEMM / GEMV choice per program."""
from aneforge_b200.llm import plan_fuse_allreduce_norm, plan_gemv_chains
from aneforge_b200.plan import PlanBuilder


def _layer_ops(pb, tp):
  """One decode layer's ops after the attention, as the emitters write them."""
  if tp:
    pb.op("gemv", wf="i8t", epi="f32", x="att", w="o.w", s="o.s", y="tp.part", nb=1, n=4096, k=4096)
    pb.op("allreduce", src="tp.part", dst="tp.part", n=4096, addto="h")
  else:
    pb.op("gemv", wf="i8t", epi="resid", x="att", w="o.w", s="o.s", y="h", nb=1, n=4096, k=4096)
  pb.op("rmsnorm", x="h", g="mg", out="xn", nb=1, d=4096, floor=0.1)
  pb.op("gemv", wf="i8t", epi="swiglu", x="xn", w="gu.w", s="gu.s", y="act", nb=1, n=28672, k=4096)
  if tp:
    pb.op("gemv", wf="i8t", epi="f32", x="act", w="dn.w", s="dn.s", y="tp.part", nb=1, n=4096, k=14336)
    pb.op("allreduce", src="tp.part", dst="tp.part", n=4096, addto="h")
  else:
    pb.op("gemv", wf="i8t", epi="resid", x="act", w="dn.w", s="dn.s", y="h", nb=1, n=4096, k=14336)
  pb.op("rmsnorm", x="h", g="ag", out="xn", nb=1, d=4096, floor=0.1)
  pb.op("gemv", wf="i8t", epi="f32", x="xn", w="qkv.w", s="qkv.s", bias="qkv.b", y="qkv", nb=1, n=6144, k=4096)


def _plan(tp):
  pb = PlanBuilder()
  for nm in ("h", "xn", "att", "act", "qkv", "tp.part"):
    pb.buf(nm, 1 << 20, "tmp")
  pb.op("attn_decode", qkv="qkv")
  _layer_ops(pb, tp)
  pb.op("attn_decode", qkv="qkv")
  return pb


def test_chain_pass_groups_a_layer():
  pb = _plan(False)
  plan_gemv_chains(pb, enable=True)
  kinds = [k for k, _ in pb.ops]
  assert kinds == ["attn_decode", "gemv_chain", "attn_decode"]
  kv = pb.ops[1][1]
  assert kv["jobs"] == 4 and kv["j0.x"] == "att" and kv["j0.nout"] == "xn" and kv["j1.epi"] == "swiglu"
  assert kv["j2.nx"] == "h" and kv["j3.b"] == "qkv.b" and "j1.nx" not in kv and "j3.nx" not in kv
  assert "chain.scr" in pb.bufs


def test_chain_pass_off_leaves_the_plan():
  pb = _plan(False)
  before = list(pb.ops)
  plan_gemv_chains(pb, enable=False)
  assert pb.ops == before


def test_allreduce_norm_fusion():
  pb = _plan(True)
  plan_fuse_allreduce_norm(pb, enable=True)
  kinds = [k for k, _ in pb.ops]
  assert kinds == ["attn_decode", "gemv", "allreduce_rms", "gemv", "gemv", "allreduce_rms", "gemv", "attn_decode"]
  fused = [kv for k, kv in pb.ops if k == "allreduce_rms"]
  assert fused[0] == dict(src="tp.part", dst="tp.part", h="h", nb=1, d=4096, g="mg", out="xn", floor=0.1)
  assert fused[1]["g"] == "ag"
  # an all-reduce not followed by a norm of its residual stays
  pb2 = PlanBuilder()
  pb2.op("allreduce", src="p", dst="p", n=8, addto="h")
  pb2.op("rmsnorm", x="other", g="g", out="xn", nb=1, d=8, floor=0.1)
  plan_fuse_allreduce_norm(pb2, enable=True)
  assert [k for k, _ in pb2.ops] == ["allreduce", "rmsnorm"]


def _experts(E=8, F=512, D=256, kind="int8"):
  from aneforge_b200.weights import DevExperts
  return DevExperts(kind=kind, gu_w=None, gu_s=object() if kind == "int8" else None, down_w=None,
                    down_s=object() if kind == "int8" else None, E=E, F=F, D=D)


def test_routed_expert_gemvs_for_decode_batches():
  """Decode batches of 2-64 rows: per expert, 16-row launches over the routed rows (gate|up gathers
  x rows, down scatters y rows with their routing weights), ceil(NB / 16) launches each."""
  from aneforge_b200 import moe
  pb = PlanBuilder()
  moe._expert_gemvs(pb, "L0", _experts(), 24, 8, 2, sparse=False)
  gemvs = [kv for k, kv in pb.ops if k == "gemv"]
  assert len(gemvs) == 8 * 2 * 2
  for i, kv in enumerate(gemvs):
    e, r0, down = i // 4, 16 * ((i // 2) % 2), i % 2 == 1
    assert kv["fixe"] == e and kv["r0"] == r0 and kv["nb"] == 16 and kv["rld"] == 24 and kv["eg"] == 8
    assert kv["rows"] == "moe.rows" and kv["rcnt"] == "moe.rcnt"
    if down:
      assert kv["route"] == 2 and kv["yrows"] == 24 and kv["rw"] == "moe.gw" and kv["x"] == "act"
    else:
      assert kv["route"] == 1 and kv["xrows"] == 24 and kv["x"] == "xn" and kv["y"] == "act"


def test_expert_gemvs_batch_one_and_prefill():
  """One row: the k selected experts read from device memory; prefill-sized row counts: every expert
  densely with per-row weights (no routing lists)."""
  from aneforge_b200 import moe
  pb = PlanBuilder()
  moe._expert_gemvs(pb, "L0", _experts(), 1, 8, 2, sparse=True)
  assert [(kv.get("sel"), kv.get("slot")) for _, kv in pb.ops] == [("moe.sel", 0)] * 2 + [("moe.sel", 1)] * 2
  pb = PlanBuilder()
  moe._expert_gemvs(pb, "L0", _experts(), moe.ROUTED_MAX_ROWS + 1, 8, 2, sparse=False)
  ops = [kv for _, kv in pb.ops]
  assert len(ops) == 16 and all("route" not in kv and kv["nb"] == moe.ROUTED_MAX_ROWS + 1 for kv in ops)
  assert [kv["fixe"] for kv in ops] == [e for e in range(8) for _ in range(2)]


def test_decode_batches_keep_the_gemv():
  """Tiled projections over prompt rows (>= 32) run as the tcgen05 GEMM; decode programs keep the
  GEMV below 128 rows."""
  from aneforge_b200 import llm
  from aneforge_b200.weights import DevLinear
  lin = DevLinear(kind="int8", w=None, s=object(), bias=None, N=4096, K=4096, tiled=True)
  for ctx, want in (({"NB": 32, "gemm_min": llm.GEMM_MIN_ROWS}, True),
                    ({"NB": 32, "gemm_min": llm.DECODE_GEMM_MIN_ROWS}, False),
                    ({"NB": 128, "gemm_min": llm.DECODE_GEMM_MIN_ROWS}, True),
                    ({"NB": 16}, False)):
    pb = PlanBuilder()
    llm._emit_linear(pb, ctx, "L0.o", lin, "att", "h", "resid")
    (kind, kv), = pb.ops
    assert kind == "gemv" and bool(kv.get("gemm")) == want, ctx
    assert ("scr" in kv) == (not want)


def test_prefill_attention_stages_expanded_kv_only_under_the_gqa_factor():
  """Under int8 the reference's GQA expansion multiplies K and V by c = 127 * f16(1/127): the prefill
  attention op then names a `kvx` buffer of [2][KV][S][dh] fp16 that the rope kernel fills with
  f16(c * f16(x)) for the tensor-core attention; with c = 1 (or no grouping) it names none."""
  from aneforge_b200 import llm
  from aneforge_b200.weights import DevLinear
  cfg = llm.LlamaConfig(dim=1024, n_layers=1, n_heads=8, n_kv_heads=2, ffn_dim=2048, vocab=4096)
  lin = lambda n, k: DevLinear(kind="int8", w=None, s=object(), bias=None, N=n, K=k, tiled=True)
  lw = {"qkv": lin((8 + 4) * 128, 1024), "o": lin(1024, 1024), "attn_floor": 0.1}
  for expand in (True, False):
    pb = PlanBuilder()
    ctx = {"NB": 300, "scale": 128 ** -0.5, "kvc": 0.99993896484375 if expand else 1.0, "expand": expand,
           "gemm_min": llm.GEMM_MIN_ROWS}
    llm.emit_attention_prefill(pb, ctx, 0, lw, cfg, llm.LayerSpec())
    (kv,) = [kv for k, kv in pb.ops if k == "attn_prefill"]
    assert kv["expand"] == int(expand) and kv["s"] == 300 and kv["dh"] == 128
    assert ("kvx" in kv) == expand
    if expand:
      assert pb.bufs["kvx"].nbytes == 2 * 2 * 2 * 300 * 128 and pb.bufs["kvx"].role == "tmp"
