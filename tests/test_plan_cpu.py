"""Plan rewrites on the host (no GPU): the chained-GEMV pass and the tensor-parallel all-reduce +
RMSNorm fusion rewrite a decode plan's op list without changing what it computes."""
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
