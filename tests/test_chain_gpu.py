"""The chained decode GEMVs (one persistent launch for o -> norm -> gate|up -> down -> norm -> next
qkv, csrc/gemv_chain.cu) against the same plan run as separate launches and against the oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from oracle.model import Config, OracleModel, random_llama_weights               # noqa: E402
from tests.test_llm_gpu import cosine, teacher_forced_check, to_b200_cfg          # noqa: E402

F32 = np.float32


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")


def _run(cfg, w, compress, chain, prompts, steps, max_len, monkeypatch):
  from aneforge_b200.llm import LlamaPrefill
  monkeypatch.setenv("AF_GEMV_CHAIN", "1" if chain else "0")
  m = LlamaPrefill(to_b200_cfg(cfg), w, compress=compress)
  if len(prompts) == 1:
    toks = [m.generate(prompts[0], steps, max_len=max_len)]
  else:
    toks = m.generate_batch(prompts, steps, max_len=max_len)
  dec = m._dec
  kinds = [k for k, _ in dec["plan"].ops]
  logits = dec["prog"].read_output("logits").astype(F32)
  m.release()
  return toks, kinds, logits


@pytest.mark.parametrize("compress,NB,bias", [("int8", 1, False), ("int8", 1, True), ("int4_g32", 1, True),
                                              ("int8", 3, False), ("int8", 11, False), ("int4_g32", 5, False)])
def test_chain_matches_separate_launches_and_oracle(compress, NB, bias, monkeypatch):
  cfg = Config(dim=1024, n_layers=3, n_heads=8, n_kv_heads=2, ffn_dim=2816, vocab=4096, rope_base=500000.0)
  w = random_llama_weights(cfg, seed=61 + NB, std=0.03, qkv_bias=bias)
  rng = np.random.default_rng(62)
  prompts = [list(rng.integers(0, cfg.vocab, int(n))) for n in rng.integers(5, 40, NB)]
  # the first decode step from the same prefix (the first token comes from the prefill): the same
  # logits up to the fp32 order of split row blocks and of the norms' sums of squares
  t1, kinds, lg_chain = _run(cfg, w, compress, True, prompts, 2, 72, monkeypatch)
  # one chain per layer boundary: [o, norm, gate|up, down, norm, next qkv] x (L - 1) + the last layer's
  assert kinds.count("gemv_chain") == cfg.n_layers and "rmsnorm" in kinds    # the first layer's norm stays
  s1, kinds_sep, lg_sep = _run(cfg, w, compress, False, prompts, 2, 72, monkeypatch)
  assert [t[0] for t in t1] == [t[0] for t in s1]
  assert "gemv_chain" not in kinds_sep
  for a, b in zip(lg_chain, lg_sep):
    assert cosine(a, b) > 0.99999
    assert np.abs(a - b).max() <= 2e-3 * np.abs(b).max()
  # 16 greedy steps through the chain: every token the oracle's argmax on the same prefix (near
  # ties excepted), each sequence of a batch as when decoded alone
  toks, _, _ = _run(cfg, w, compress, True, prompts, 16, 72, monkeypatch)
  om = OracleModel(cfg, w, compress, precision="device")
  for p, t in zip(prompts, toks):
    assert teacher_forced_check(om, p, t, 72, n_check=16) <= 2


def test_chain_replays_many_steps(monkeypatch):
  """The chain's counters and flags are reset by the launch itself: a long greedy run (hundreds of
  replays of every chain) is the same run to run and follows the oracle."""
  cfg = Config(dim=512, n_layers=2, n_heads=8, n_kv_heads=2, ffn_dim=1024, vocab=2048, rope_base=10000.0,
               head_dim=64)
  w = random_llama_weights(cfg, seed=71, std=0.05)
  prompt = [list(np.random.default_rng(72).integers(0, cfg.vocab, 9))]
  a, _, _ = _run(cfg, w, "int8", True, prompt, 200, 256, monkeypatch)
  b, _, _ = _run(cfg, w, "int8", True, prompt, 200, 256, monkeypatch)
  assert a == b                                            # deterministic run to run
  om = OracleModel(cfg, w, "int8", precision="device")
  assert teacher_forced_check(om, prompt[0], a[0], 256, n_check=40) <= 2
