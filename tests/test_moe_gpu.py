"""Mixture-of-experts on the device against the oracle: the router tail (softmax + top-k peel with
lowest-index ties + renormalisation), expert selection inside the tensor-core GEMV (index read from
device memory, routing-weighted residual epilogue), the routed batch GEMVs against the dense ones, and
whole MoE decoders (sparse top-k at batch 1, routed at batch 2-3) with int8 and group-32 int4 experts."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from aneforge_b200 import _runtime as R                                          # noqa: E402
from oracle import quant as Q                                                   # noqa: E402
from oracle.model import Config, OracleModel, random_llama_weights, softmax, topk_gate   # noqa: E402

F16, F32 = np.float16, np.float32


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")


def cuda(a):
  return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("E,k", [(8, 2), (16, 4), (60, 8), (4, 1)])
def test_moe_gate_matches_reference_rule(E, k):
  from aneforge_b200 import kernels as K
  rng = np.random.default_rng(E + k)
  lg = rng.standard_normal((37, E)).astype(F32)
  lg[0, :] = 0.5                                   # a full tie: the lowest indices win
  lg[1, 3:] = lg[1, 2]                             # partial ties
  gw, sel = K.moe_gate(cuda(lg), k)
  gw, sel = gw.cpu().numpy(), sel.cpu().numpy()
  probs = softmax(lg)
  ref = topk_gate(probs, k)
  ref = ref / ref.sum(axis=1, keepdims=True)
  chosen = ref > 0
  assert np.array_equal(gw > 0, chosen)
  np.testing.assert_allclose(gw, ref, rtol=1e-5, atol=1e-7)
  assert list(sel[0]) == list(range(k))
  for b in range(37):
    assert set(sel[b]) == set(np.nonzero(chosen[b])[0])


@pytest.mark.parametrize("fmt", ["int8", "int4_g32"])
@pytest.mark.parametrize("NB", [1, 3])
def test_expert_gemv_selection_and_weighting(fmt, NB):
  from aneforge_b200 import kernels as K, _runtime as R
  rng = np.random.default_rng(5 + NB)
  E, N, Kd = 4, 192, 512
  Ws = [(rng.standard_normal((N, Kd)) * 0.02).astype(F16) for _ in range(E)]
  x = rng.standard_normal((NB, Kd)).astype(F16)
  if fmt == "int8":
    enc = [Q.quantize_per_row(W) for W in Ws]
    deq = [q.astype(F32) * s.astype(F32)[:, None] for q, s in enc]
    tiles = torch.cat([K.pack_i8_tiles(cuda(q)) for q, _ in enc])
    scales = cuda(np.concatenate([s for _, s in enc]))
    wf = R.W_I8
  else:
    enc = [Q.quantize_g32_int4(W) for W in Ws]
    deq = [Q.dequant_g32_int4(p, s) for p, s in enc]
    tiles = torch.cat([K.pack_i4_tiles(cuda(p), cuda(s), N, Kd) for p, s in enc])
    scales, wf = None, R.W_I4G32
  sel = cuda(np.array([2, 1], np.int32))
  for slot, e in ((0, 2), (1, 1)):
    y = K.gemv_tc_expert(cuda(x), tiles, scales, N, Kd, E, wf=wf, sel=sel, slot=slot).cpu().numpy()
    ref = x.astype(F32) @ deq[e].T
    assert np.abs(y - ref).max() <= 1e-4 * np.abs(ref).max() + 1e-5
  rw = rng.random((NB, E)).astype(F32)
  y0 = rng.standard_normal((NB, N)).astype(F32)
  yr = cuda(y0.copy())
  K.gemv_tc_expert(cuda(x), tiles, scales, N, Kd, E, wf=wf, epi=R.EPI_RESID, y=yr, fixed_e=3, rw=cuda(rw))
  ref = y0 + rw[:, 3:4] * (x.astype(F32) @ deq[3].T)
  assert np.abs(yr.cpu().numpy() - ref).max() <= 1e-4 * np.abs(ref).max() + 1e-5


def _moe_cfg():
  return Config(dim=512, n_layers=2, n_heads=8, n_kv_heads=2, ffn_dim=384, vocab=2048, rope_base=10000.0,
                head_dim=64, extra={"n_experts": 8, "n_experts_per_tok": 2, "norm_topk_prob": True})


def _b200_cfg(cfg):
  from aneforge_b200.llm import LlamaConfig, LayerSpec
  return LlamaConfig(dim=cfg.dim, n_layers=cfg.n_layers, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
                     ffn_dim=cfg.ffn_dim, vocab=cfg.vocab, rope_base=cfg.rope_base, norm_eps=cfg.norm_eps,
                     head_dim=cfg.head_dim, extra=dict(cfg.extra),
                     layers=[LayerSpec(mlp="moe") for _ in range(cfg.n_layers)])


@pytest.mark.parametrize("experts", ["int8", "int4_g32"])
def test_moe_decoder_matches_oracle(experts):
  from aneforge_b200.llm import LlamaPrefill
  from tests.test_llm_gpu import teacher_forced_check
  cfg = _moe_cfg()
  w = random_llama_weights(cfg, seed=31, std=0.05, moe=True)
  # a well-separated router (logit spread ~10): the top-k choice never sits on a near tie, which the
  # token-level tie margin below would not cover (a flipped expert changes the whole layer output)
  for lw in w["layers"]:
    lw["router"] = (lw["router"].astype(np.float32) * 10).astype(F16)
  m = LlamaPrefill(_b200_cfg(cfg), w, compress="int8", moe_compress=experts)
  prompt = list(np.random.default_rng(32).integers(0, cfg.vocab, 21))
  toks = m.generate(prompt, 24, max_len=64)
  om = OracleModel(cfg, w, "int8", precision="device", moe_compress=experts)
  assert teacher_forced_check(om, prompt, toks, 64, n_check=24) <= 2
  # batch 3 runs the routed expert GEMVs: the same tokens as batch 1 for each sequence
  prompts = [prompt, list(np.random.default_rng(33).integers(0, cfg.vocab, 9)),
             list(np.random.default_rng(34).integers(0, cfg.vocab, 14))]
  batch = m.generate_batch(prompts, 12, max_len=48)
  for p, b in zip(prompts, batch):
    assert m.generate(p, 12, max_len=48) == b
  m.release()


@pytest.mark.parametrize("compress", ["int8", "int4_g32"])
def test_moe_shared_expert_matches_oracle(compress):
  """Qwen2-MoE layers: routed experts plus the sigmoid-gated shared expert (`aneforge/moe.py:60-62`),
  decode at batch 1 and 3 and the prefill GEMM rows, against the oracle's teacher-forced pass."""
  from aneforge_b200.llm import LlamaPrefill
  from tests.test_llm_gpu import teacher_forced_check
  cfg = _moe_cfg()
  cfg.extra["norm_topk_prob"] = False                     # Qwen1.5-MoE does not renormalise the top-k
  w = random_llama_weights(cfg, seed=41, std=0.05, moe=True, shared_expert=640)
  for lw in w["layers"]:
    lw["router"] = (lw["router"].astype(np.float32) * 10).astype(F16)
    lw["shared_gate"] = (lw["shared_gate"].astype(np.float32) * 20).astype(F16)   # gates away from 0.5
  m = LlamaPrefill(_b200_cfg(cfg), w, compress=compress, moe_compress=compress)
  prompt = list(np.random.default_rng(42).integers(0, cfg.vocab, 37))       # >= 32 rows: prefill GEMM
  toks = m.generate(prompt, 20, max_len=96)
  om = OracleModel(cfg, w, compress, precision="device", moe_compress=compress)
  assert teacher_forced_check(om, prompt, toks, 96, n_check=20) <= 2
  # the shared expert changes the output: the same model without it decodes another sequence
  w2 = {**w, "layers": [{k: v for k, v in lw.items() if not k.endswith("_sh") and k != "shared_gate"}
                        for lw in w["layers"]]}
  m2 = LlamaPrefill(_b200_cfg(cfg), w2, compress=compress, moe_compress=compress)
  assert m2.generate(prompt, 20, max_len=96) != toks
  m2.release()
  prompts = [prompt, list(np.random.default_rng(43).integers(0, cfg.vocab, 11))]
  batch = m.generate_batch(prompts, 10, max_len=64)
  for p, b in zip(prompts, batch):
    assert m.generate(p, 10, max_len=64) == b
  m.release()


@pytest.mark.parametrize("arch", ["qwen2moe", "qwen3moe"])
def test_load_gguf_decodes_like_the_oracle(tmp_path, arch):
  """A Qwen-MoE GGUF (Q8_0 experts) through `moe.load_gguf` onto the device, against the oracle
  on the same host weights."""
  pytest.importorskip("gguf")
  from aneforge_b200.moe import load_gguf
  from tests.test_llm_gpu import teacher_forced_check
  from tests.test_moe_cpu import _write_qwen_moe_gguf
  path = tmp_path / "m.gguf"
  _write_qwen_moe_gguf(path, arch, np.random.default_rng(8), dim=256, heads=4, kv=2, ffn=128, E=4, vocab=512,
                        router_scale=10.0)          # expert choices well clear of ties
  m = load_gguf(str(path), compress="int8")
  c = m.cfg
  oc = Config(dim=c.dim, n_layers=c.n_layers, n_heads=c.n_heads, n_kv_heads=c.n_kv_heads, ffn_dim=c.ffn_dim,
              vocab=c.vocab, rope_base=c.rope_base, norm_eps=c.norm_eps, head_dim=c.head_dim, extra=dict(c.extra))
  ow = {"embed": m.w["embed"], "final_norm": m.w["final_norm"], "lm_head": m.w["lm_head"],
        "layers": [m.w["layers"][i] for i in range(c.n_layers)]}
  prompt = list(np.random.default_rng(9).integers(0, c.vocab, 13))
  toks = m.generate(prompt, 16, max_len=48)
  om = OracleModel(oc, ow, "int8", precision="device")
  assert teacher_forced_check(om, prompt, toks, 48, n_check=16) <= 2
  m.release()


def _expert_plan(NB, E, k, ex, routed_max, monkeypatch):
  """moe_gate -> (moe_route) -> the layer's expert GEMVs over NB rows of xn, adding into h."""
  from aneforge_b200 import moe
  from aneforge_b200.plan import PlanBuilder
  monkeypatch.setattr(moe, "ROUTED_MAX_ROWS", routed_max)
  D, F = ex.D, ex.F
  pb = PlanBuilder()
  pb.buf("moe.logits", 4 * NB * E, "in"); pb.buf("xn", 2 * NB * D, "in"); pb.buf("h", 4 * NB * D, "state")
  pb.buf("moe.gw", 4 * NB * E, "tmp"); pb.buf("moe.sel", 4 * NB * k, "tmp"); pb.buf("act", 2 * NB * F, "tmp")
  pb.buf("L0.egu.w", ex.gu_w.numel(), "weight"); pb.buf("L0.edown.w", ex.down_w.numel(), "weight")
  if ex.gu_s is not None:
    pb.buf("L0.egu.s", ex.gu_s.numel() * 2, "weight"); pb.buf("L0.edown.s", ex.down_s.numel() * 2, "weight")
  pb.op("moe_gate", logits="moe.logits", nb=NB, e=E, k=k, renorm=1, gw="moe.gw", sel="moe.sel")
  if 1 < NB <= routed_max:
    pb.buf("moe.rows", 4 * E * NB, "tmp"); pb.buf("moe.rcnt", 4 * E, "tmp")
    pb.op("moe_route", sel="moe.sel", nb=NB, e=E, k=k, rld=NB, rows="moe.rows", cnt="moe.rcnt")
  moe._expert_gemvs(pb, "L0", ex, NB, E, k, sparse=False)
  prog = R.Program.from_text(pb.text(), {"moe.logits": (NB, E), "xn": (NB, D), "h": (NB, D)}, {}, 0,
                             {"moe.logits": "fp32", "h": "fp32"})
  prog.bind("L0.egu.w", ex.gu_w); prog.bind("L0.edown.w", ex.down_w)
  if ex.gu_s is not None:
    prog.bind("L0.egu.s", ex.gu_s); prog.bind("L0.edown.s", ex.down_s)
  return prog


@pytest.mark.parametrize("experts", ["int8", "int4_g32"])
@pytest.mark.parametrize("NB,hot", [(5, False), (24, False), (24, True), (64, True)])
def test_routed_expert_gemvs_match_dense(experts, NB, hot, monkeypatch):
  """Decode batches run each expert over the rows routed to it (`moe_route` lists; gate|up gathers
  them, down scatters the routing-weighted rows back) instead of every expert over every row with
  zero weights: the same residual, to fp32 rounding. `hot` sends every row to expert 0 first, so
  its list spans several 16-row launches while other experts' lists are empty."""
  import torch
  from aneforge_b200 import weights
  E, k, D, F = 8, 2, 256, 512
  rng = np.random.default_rng(NB + 100 * hot)
  wg = (rng.standard_normal((E, F, D)) * 0.05).astype(F16)
  wu = (rng.standard_normal((E, F, D)) * 0.05).astype(F16)
  wd = (rng.standard_normal((E, F, D)) * 0.05).astype(F16)
  ex = weights.encode_experts(wg, wu, wd, experts, torch.device("cuda", 0))
  logits = (rng.standard_normal((NB, E)) * 3).astype(F32)
  if hot:
    logits[:, 0] += 50.0
  x = rng.standard_normal((NB, D)).astype(F16)
  h0 = rng.standard_normal((NB, D)).astype(F32)
  out = {}
  for name, routed_max in (("routed", 64), ("dense", 0)):
    prog = _expert_plan(NB, E, k, ex, routed_max, monkeypatch)
    prog.set_input("moe.logits", logits); prog.set_input("xn", x); prog.set_input("h", h0)
    prog.execute()
    out[name] = prog.tensor("h", (NB, D), "fp32").cpu().numpy().copy()
    prog.release()
  d_r, d_d = out["routed"] - h0, out["dense"] - h0
  assert np.abs(d_r - d_d).max() <= 1e-4 * np.abs(d_d).max(), np.abs(d_r - d_d).max()
  assert np.abs(d_d).max() > 0.1                              # the experts did add something
