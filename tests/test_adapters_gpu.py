"""Hugging Face checkpoints through the adapters onto the device (Gemma's GeGLU graph-builder MLP,
Qwen3-MoE's sparse and dense layers), greedy decode against the oracle on the adapted weights."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
pytest.importorskip("transformers")

from oracle.model import OracleModel                                           # noqa: E402
from tests.test_llm_gpu import teacher_forced_check                             # noqa: E402
from tests.test_loaders_cpu import _oracle_cfg, _tiny                           # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")


@pytest.mark.parametrize("kind", ["gemma", "qwen3_moe", "qwen2", "gpt2"])
def test_hf_checkpoint_decodes_like_the_oracle(kind, tmp_path):
  from aneforge_b200 import llm
  d, _ = _tiny(kind, tmp_path, hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2,
               head_dim=64, vocab_size=512, initializer_range=0.08)
  m = llm.from_pretrained(str(d), compress="int8")
  prompt = list(np.random.default_rng(3).integers(0, 512, 19))
  toks = m.generate(prompt, 16, max_len=48)
  assert m.generate(prompt[:5], 16, max_len=48, batched_prefill=False) == m.generate(prompt[:5], 16, max_len=48)
  om = OracleModel(_oracle_cfg(m.cfg), m.w, "int8", precision="device")
  assert teacher_forced_check(om, prompt, toks, 48, n_check=16) <= 2
  m.release()
