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


_HYBRID_LINEARS = ("in_proj_qkv", "in_proj_z", "in_proj_a", "in_proj_b", "out_proj", "wq", "wk", "wv", "wo", "wgate",
                   "wup", "wdown")


def _oracle_hybrid_logits(cfg, w, seq, M):
  """The reference's numerics for a hybrid decoder, token by token: every layer's graph builders
  (mixer + SwiGLU) and the final norm through the oracle's graph interpreter, with the mixers'
  states carried as fp16 between steps (fp16 ports), then the fp16 hidden row times the fp16 head."""
  from aneforge_b200 import blocks, llm
  from aneforge_b200 import graph as G
  from oracle.graph import GraphInterp
  x = G.input((1, cfg.dim))
  ctx = blocks.decode_inputs(M, cfg.dh)
  h, pairs = x, []
  for li, ls in enumerate(cfg.layers):
    h, p = llm.DECODE_MIXERS[ls.mixer](h, w["layers"][li], cfg, ls, ctx, M)
    pairs += p
    h = blocks.swiglu(h, w["layers"][li], cfg, ls)
  interp = GraphInterp([h.rms_norm(w["final_norm"], cfg.norm_eps)] + [o for o, _ in pairs])
  state = [np.zeros(i.shape, np.float16) for _, i in pairs]
  cos_t, sin_t = llm.rope_tables(M, cfg.dh, cfg.rope_base, cfg.rotary_dim)
  head = np.asarray(w["lm_head"], np.float32)
  out = []
  for t, tok in enumerate(seq):
    feeds = {x: np.asarray(w["embed"][tok], np.float16)[None]}
    feeds.update({i: s for (_, i), s in zip(pairs, state)})
    feeds.update({ctx[k]: v for k, v in blocks.decode_values(t, M, cos_t, sin_t).items()})
    r = interp.run(feeds)
    out.append(np.asarray(r[0], np.float32).reshape(-1).astype(np.float16).astype(np.float32) @ head.T)
    state = [np.asarray(v, np.float16) for v in r[1:]]
  return np.stack(out)


def _cos(a, b):
  return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


@pytest.mark.parametrize("compress", [None, "int8"])
def test_qwen35_hybrid_decodes_like_transformers(compress, monkeypatch):
  """A Qwen3.5 hybrid (three gated-DeltaNet layers, one gated-attention layer; reference
  `aneforge/qwen35.py`, `tests/test_qwen35.py:87-117`) through `hybrid.adapt` onto the device: the
  graph-builder mixers keep their conv / recurrent / K-V states resident. Every step's device logits
  against (1) the reference's own numerics - the same graph builders through the oracle's graph
  interpreter, fp16 states between steps, under int8 the projections as they decode - to a cosine of
  0.999 with the greedy tokens under the tie protocol, and (2) the checkpoint in transformers (fp32
  states), to the tolerance the reference's own checks give that comparison (`tests/test_qwen35.py`:
  a cosine of 0.96 for a gated-DeltaNet layer, 0.99 for the hybrid model's hidden states; the fp16
  recurrent state drifts from the fp32 one, so single steps of the logits dip to ~0.92)."""
  from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
  from transformers.models.qwen3_5 import modeling_qwen3_5 as q35
  from aneforge_b200 import _blob, hybrid, llm
  # The reference model runs on the host: its constructor must pick transformers' torch kernels,
  # not the Triton / CUDA ones it selects when those libraries are importable.
  for name in ("FusedRMSNormGated", "chunk_gated_delta_rule", "fused_recurrent_gated_delta_rule",
               "causal_conv1d_fn", "causal_conv1d_update"):
    if hasattr(q35, name):
      monkeypatch.setattr(q35, name, None)
  torch.manual_seed(0)
  ct = Qwen3_5TextConfig(hidden_size=256, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                         head_dim=64, partial_rotary_factor=0.25, linear_num_key_heads=2, linear_num_value_heads=4,
                         linear_key_head_dim=64, linear_value_head_dim=64, linear_conv_kernel_dim=4, vocab_size=512,
                         intermediate_size=512, rms_norm_eps=1e-6, initializer_range=0.08)
  with torch.device("cpu"):                                # the reference model runs on the host
    hf = q35.Qwen3_5ForCausalLM(ct).eval().cpu()
  sd = {k: v.detach().cpu().half().numpy() for k, v in hf.state_dict().items()}
  cfg, w = hybrid.adapt(ct, sd, prefix="model.")
  m = llm.LlamaPrefill(cfg, w, compress=compress)
  prompt = list(np.random.default_rng(5).integers(0, 512, 12))
  logs = []                                  # the device's fp32 logits of every step
  toks = m.generate(prompt, 10, max_len=32,
                    on_token=lambda t: logs.append(m._dec["prog"].read_output("logits")[0].astype(np.float32)))
  m.release()
  seq = prompt + toks
  w_ref = w
  if compress:
    # what the device multiplies by: each decoder-layer projection as its `compress` encoding decodes
    # (embedding and lm_head stay fp16)
    w_ref = {**w, "layers": [{k: (_blob.dense_of(np.asarray(v, np.float16), compress) if k in _HYBRID_LINEARS else v)
                              for k, v in lw.items()} for lw in w["layers"]]}
    with torch.no_grad():
      for mod in hf.model.layers.modules():
        if isinstance(mod, torch.nn.Linear):
          mod.weight.copy_(torch.from_numpy(_blob.dense_of(mod.weight.half().numpy(), compress)))
  ol = _oracle_hybrid_logits(cfg, w_ref, seq, 32)
  with torch.no_grad():
    lg = hf(torch.tensor([seq], device="cpu")).logits[0].float().cpu().numpy()
  ties, hf_cos = 0, []
  for i, t in enumerate(toks):
    dl, ref, ref_hf = logs[i], ol[len(prompt) - 1 + i], lg[len(prompt) - 1 + i]
    assert int(np.argmax(dl)) == t
    assert _cos(dl, ref) > 0.999, f"step {i}: cosine to the reference numerics {_cos(dl, ref)}"
    if int(np.argmax(ref)) != t:
      assert np.sort(ref)[-1] - ref[t] < 0.05 * np.abs(ref).max(), f"step {i}: {t} vs {int(np.argmax(ref))}"
      ties += 1
    hf_cos.append(_cos(dl, ref_hf))
  assert ties <= 2
  assert min(hf_cos) > 0.9 and float(np.mean(hf_cos)) > 0.95, hf_cos
