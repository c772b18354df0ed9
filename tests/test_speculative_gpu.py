"""Speculative decoding (reference `aneforge/speculative.py:131-165`) on the device. The reference's
invariants (`tests/test_speculative.py:7-29`): greedy speculative decoding emits exactly the target's
greedy tokens for any draft, and a draft equal to the target has every proposal accepted, so the
target verifies far fewer times than it emits tokens."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from oracle.model import Config, random_llama_weights                      # noqa: E402
from tests.test_llm_gpu import to_b200_cfg                                # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")


def _models(draft_seed, compress="int8", cfg=None):
  from aneforge_b200.llm import LlamaPrefill
  cfg = cfg or Config(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=512, vocab=512, rope_base=10000.0,
                      head_dim=64)
  tgt = LlamaPrefill(to_b200_cfg(cfg), random_llama_weights(cfg, seed=0, std=0.05), compress=compress)
  drf = LlamaPrefill(to_b200_cfg(cfg), random_llama_weights(cfg, seed=draft_seed, std=0.05), compress=compress)
  return cfg, tgt, drf


@pytest.mark.parametrize("n_draft", [1, 3, 6])
def test_spec_generate_matches_greedy(n_draft):
  from aneforge_b200.speculative import spec_generate
  cfg, tgt, drf = _models(draft_seed=1)
  prompt = list(np.random.default_rng(3).integers(0, cfg.vocab, 17))
  g = tgt.generate(prompt, 24, max_len=64)
  st = {}
  s = spec_generate(tgt, drf, prompt, max_new_tokens=24, max_len=64, n_draft=n_draft, stats=st)
  assert s == g, f"spec {s}\ngreedy {g}"
  assert st["verify_steps"] >= 1
  tgt.release(); drf.release()


def test_spec_accepts_every_draft_when_draft_equals_target():
  from aneforge_b200.speculative import spec_generate
  cfg, tgt, drf = _models(draft_seed=0)
  prompt = list(np.random.default_rng(4).integers(0, cfg.vocab, 9))
  st = {}
  out = spec_generate(tgt, drf, prompt, max_new_tokens=25, max_len=64, n_draft=4, stats=st)
  assert out == tgt.generate(prompt, 25, max_len=64)
  assert st["verify_steps"] < len(out) // 3, st
  assert st["accepted"] >= 4 * (st["verify_steps"] - 1), st
  tgt.release(); drf.release()


def test_spec_generate_llama_shaped_gqa_and_eos():
  """Llama-3-shaped heads (GQA 4:1, head dim 128) with a smaller draft of the same vocabulary;
  EOS stops both paths at the same token."""
  from aneforge_b200.llm import LlamaPrefill
  from aneforge_b200.speculative import spec_generate
  cfg = Config(dim=1024, n_layers=2, n_heads=8, n_kv_heads=2, ffn_dim=2048, vocab=2048, rope_base=500000.0)
  dcfg = Config(dim=512, n_layers=1, n_heads=4, n_kv_heads=1, ffn_dim=1024, vocab=2048, rope_base=500000.0)
  tgt = LlamaPrefill(to_b200_cfg(cfg), random_llama_weights(cfg, seed=5), compress="int8")
  drf = LlamaPrefill(to_b200_cfg(dcfg), random_llama_weights(dcfg, seed=6), compress="int8")
  prompt = list(np.random.default_rng(7).integers(0, cfg.vocab, 40))
  g = tgt.generate(prompt, 20, max_len=96)
  assert spec_generate(tgt, drf, prompt, max_new_tokens=20, max_len=96, n_draft=4) == g
  eos = g[7]
  assert spec_generate(tgt, drf, prompt, max_new_tokens=20, max_len=96, n_draft=4, eos_id=eos) == \
    tgt.generate(prompt, 20, max_len=96, eos_id=eos)
  tgt.release(); drf.release()
