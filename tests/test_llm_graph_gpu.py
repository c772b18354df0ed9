"""Graph-builder registry entries inside `LlamaPrefill` (the reference's registry form,
`aneforge/llm.py:240-245`): a mixer / MLP written over graph Tensors is lowered into the decode and
prefill programs and must decode like the oracle.

Bars: greedy tokens equal the oracle's along the GPU's own tokens (teacher-forced) except at a step
inside the reference's tie margin, at most 1 such step in 12 (`teacher_forced_check`); prompt logits
within rel-err 1e-2 and cosine >= 0.999.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from oracle.model import Config, OracleModel, random_llama_weights               # noqa: E402
from tests.test_llm_gpu import teacher_forced_check, to_b200_cfg, cosine          # noqa: E402

F32 = np.float32


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")


@pytest.fixture
def registries():
  from aneforge_b200 import llm, blocks
  llm.DECODE_MIXERS["attention_graph"] = blocks.attn_decode
  llm.DECODE_MLPS["swiglu_graph"] = blocks.swiglu
  llm.PREFILL_MLPS["swiglu_graph"] = blocks.swiglu
  yield llm
  for reg, key in ((llm.DECODE_MIXERS, "attention_graph"), (llm.DECODE_MLPS, "swiglu_graph"),
                   (llm.PREFILL_MLPS, "swiglu_graph")):
    reg.pop(key, None)


@pytest.mark.parametrize("compress", ["int8", None])
def test_graph_mixer_and_mlp_decode_match_oracle(registries, compress):
  """Every layer's mixer and MLP are graph builders (`blocks.attn_decode` / `blocks.swiglu`): the
  program keeps their K / V as resident state, builds the per-step inputs from the device position,
  and prefills token by token (batched prefill is for the fused attention mixer only)."""
  llm = registries
  cfg = Config(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=512, vocab=512, rope_base=10000.0,
               head_dim=64)
  w = random_llama_weights(cfg, seed=41, std=0.05)
  bcfg = to_b200_cfg(cfg)
  bcfg.layers = [llm.LayerSpec(mixer="attention_graph", mlp="swiglu_graph") for _ in range(2)]
  m = llm.LlamaPrefill(bcfg, w, compress=compress)
  prompt = list(np.random.default_rng(42).integers(0, cfg.vocab, 20))
  toks = m.generate(prompt, 12, max_len=40)
  assert len(toks) == 12
  om = OracleModel(cfg, w, compress, precision="device")
  assert teacher_forced_check(om, prompt, toks, 40, n_check=12) <= 1
  # the same model through the fused kernels
  fused = llm.LlamaPrefill(to_b200_cfg(cfg), w, compress=compress)
  ftoks = fused.generate(prompt, 12, max_len=40)
  agree = sum(a == b for a, b in zip(toks, ftoks))
  print(f"\ngraph-builder layers vs fused layers: {agree}/12 tokens equal")
  m.release(); fused.release()


def test_geglu_mlp_graph_builder_matches_oracle():
  """GeGLU (the reference's Gemma MLP, `aneforge/llm.py:189-196`) registered as a graph builder:
  lowered into the batched-prefill program (40 rows: tcgen05 GEMM projections) and into the decode
  program next to the fused attention."""
  from aneforge_b200 import llm
  cfg = Config(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=512, vocab=512, rope_base=10000.0,
               head_dim=64, mlp="geglu")
  w = random_llama_weights(cfg, seed=43, std=0.05)
  bcfg = to_b200_cfg(cfg)
  bcfg.layers = [llm.LayerSpec(mlp="geglu") for _ in range(2)]
  m = llm.LlamaPrefill(bcfg, w, compress="int8")
  prompt = list(np.random.default_rng(44).integers(0, cfg.vocab, 40))
  toks = m.generate(prompt, 12, max_len=64)
  om = OracleModel(cfg, w, "int8", precision="device")
  assert teacher_forced_check(om, prompt, toks, 64, n_check=12) <= 1
  pl = m.prefill(prompt)[0]
  hid, _ = om.prefill_hidden(prompt)
  ol = om.logits(hid[-1].astype(F32))
  assert np.abs(pl - ol).max() <= 1e-2 * np.abs(ol).max()
  assert cosine(pl, ol) > 0.999
  m.release()
