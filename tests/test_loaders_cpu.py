"""Host-side loader and sampling logic, no GPU: the Hugging Face adapters (reference
`aneforge/llm.py:636-806`) on tiny random `transformers` checkpoints written to a temporary
directory, the RoPE tables and the sampling rules against the oracle's restatement."""
import numpy as np
import pytest

from oracle.model import OracleModel, rope_tables as oracle_rope_tables

torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")


def _tiny(kind, tmp_path, **extra):
  """A tiny random HF model saved with save_pretrained (offline; weights from a fixed seed)."""
  torch.manual_seed(0)
  common = dict(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                num_key_value_heads=2, vocab_size=97, max_position_embeddings=256, rms_norm_eps=1e-6)
  hd = extra.pop("head_dim", 16)
  common.update(extra)
  if kind == "llama":
    cfg = transformers.LlamaConfig(**common)
    model = transformers.LlamaForCausalLM(cfg)
  elif kind == "qwen2":
    cfg = transformers.Qwen2Config(**common)
    model = transformers.Qwen2ForCausalLM(cfg)
  elif kind == "qwen3":
    cfg = transformers.Qwen3Config(head_dim=hd, **common)
    model = transformers.Qwen3ForCausalLM(cfg)
  elif kind == "mistral":
    cfg = transformers.MistralConfig(sliding_window=64, **common)
    model = transformers.MistralForCausalLM(cfg)
  elif kind == "gpt2":
    cfg = transformers.GPT2Config(n_embd=common["hidden_size"], n_layer=common["num_hidden_layers"],
                                  n_head=common["num_attention_heads"], n_inner=common["intermediate_size"],
                                  vocab_size=common["vocab_size"], n_positions=common["max_position_embeddings"],
                                  initializer_range=common.get("initializer_range", 0.02))
    model = transformers.GPT2LMHeadModel(cfg)
  elif kind == "gemma":
    cfg = transformers.GemmaConfig(head_dim=hd, hidden_act="gelu_pytorch_tanh", **common)
    model = transformers.GemmaForCausalLM(cfg)
  elif kind == "qwen3_moe":
    cfg = transformers.Qwen3MoeConfig(head_dim=hd, moe_intermediate_size=32, num_experts=4, num_experts_per_tok=2,
                                      mlp_only_layers=[1], norm_topk_prob=False, **common)
    model = transformers.Qwen3MoeForCausalLM(cfg)
  else:
    raise ValueError(kind)
  d = tmp_path / kind
  model.save_pretrained(str(d))
  return d, model


@pytest.mark.parametrize("kind", ["llama", "qwen2", "qwen3", "mistral"])
def test_from_pretrained_maps_checkpoint(kind, tmp_path):
  from aneforge_b200 import llm
  d, model = _tiny(kind, tmp_path)
  m = llm.from_pretrained(str(d), compress="int8")          # no device work until the first program
  c = model.config
  cfg = m.cfg
  assert (cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.ffn_dim, cfg.vocab) == (
    c.hidden_size, c.num_hidden_layers, c.num_attention_heads, c.num_key_value_heads, c.intermediate_size, c.vocab_size)
  assert cfg.norm_eps == pytest.approx(c.rms_norm_eps)
  sd = model.state_dict()
  w = m.w
  np.testing.assert_array_equal(np.asarray(w["embed"], np.float32), sd["model.embed_tokens.weight"].half().float().numpy())
  for i in range(cfg.n_layers):
    lw = w["layers"][i]
    pre = f"model.layers.{i}."
    np.testing.assert_array_equal(np.asarray(lw["wq"], np.float32), sd[pre + "self_attn.q_proj.weight"].half().float().numpy())
    np.testing.assert_array_equal(np.asarray(lw["wdown"], np.float32), sd[pre + "mlp.down_proj.weight"].half().float().numpy())
    assert ("q_bias" in lw) == (kind == "qwen2")
    assert ("q_norm" in lw) == (kind == "qwen3")
    assert cfg.layers[i].qk_norm == (kind == "qwen3")
  if kind == "qwen3":
    assert cfg.dh == 16
  if kind == "mistral":
    assert cfg.extra["sliding_window"] == 64 and cfg.rope_scaling is None
  if kind == "llama":
    # untied head: its own rows
    np.testing.assert_array_equal(np.asarray(w["lm_head"], np.float32), sd["lm_head.weight"].half().float().numpy())


def _oracle_cfg(cfg):
  from oracle.model import Config
  return Config(dim=cfg.dim, n_layers=cfg.n_layers, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
                ffn_dim=cfg.ffn_dim, vocab=cfg.vocab, rope_base=cfg.rope_base, norm_eps=cfg.norm_eps,
                head_dim=cfg.head_dim, rope_scaling=cfg.rope_scaling, extra=dict(cfg.extra),
                qk_norm=cfg.layers[0].qk_norm, norm_type=cfg.norm_type, rope=cfg.rope,
                mlp=cfg.layers[0].mlp if cfg.layers[0].mlp in ("geglu", "gelu_new") else "swiglu")


def _hf_last_logits(model, prompt):
  model.eval()                                             # GPT-2 has dropout
  with torch.no_grad():
    return model(torch.tensor([prompt])).logits[0, -1].float().numpy()


@pytest.mark.parametrize("kind", ["gemma", "qwen3_moe", "gpt2"])
def test_adapter_runs_like_transformers(kind, tmp_path):
  """Gemma (GeGLU, sqrt(hidden)-scaled embedding, 1 + w norms) and Qwen3-MoE (fused expert tensors,
  dense layers from `mlp_only_layers`, QK-norm, no top-k renormalisation): the adapted weights run
  through the oracle give the checkpoint's own next-token logits (transformers on the CPU)."""
  from aneforge_b200 import llm
  d, model = _tiny(kind, tmp_path)
  m = llm.from_pretrained(str(d))
  cfg, w = m.cfg, m.w
  if kind == "gemma":
    assert [ls.mlp for ls in cfg.layers] == ["geglu", "geglu"]
    sd = model.state_dict()
    e = sd["model.embed_tokens.weight"].half().numpy()
    np.testing.assert_array_equal(np.asarray(w["lm_head"]), e)                  # tied, unscaled
    np.testing.assert_allclose(w["embed"], e.astype(np.float64) * np.sqrt(64))
    np.testing.assert_array_equal(w["layers"][0]["attn_norm"],
                                  sd["model.layers.0.input_layernorm.weight"].half().numpy() + np.float16(1))
  elif kind == "gpt2":
    assert cfg.norm_type == "layer" and not cfg.rope and [ls.mlp for ls in cfg.layers] == ["gelu_new", "gelu_new"]
    sd = model.state_dict()
    np.testing.assert_array_equal(w["layers"][1]["wk"], sd["transformer.h.1.attn.c_attn.weight"].half().numpy()[:, 64:128].T)
    np.testing.assert_array_equal(w["wpe"], sd["transformer.wpe.weight"].half().numpy())
  else:
    assert [ls.mlp for ls in cfg.layers] == ["moe", "swiglu"]
    assert cfg.extra == {"n_experts": 4, "n_experts_per_tok": 2, "norm_topk_prob": False}
    assert w["layers"][0]["wgate_exps"].shape == (4, 32, 64) and w["layers"][0]["wdown_exps"].shape == (4, 32, 64)
    assert "wgate" in w["layers"][1] and "router" not in w["layers"][1]
  om = OracleModel(_oracle_cfg(cfg), w, None, precision="fp32")
  prompt = [3, 17, 42, 5, 88, 1, 60]
  hid, _ = om.prefill_hidden(prompt)
  got = om.logits(hid[-1].astype(np.float32))
  ref = _hf_last_logits(model.float(), prompt)
  cos = float(got @ ref / (np.linalg.norm(got) * np.linalg.norm(ref)))
  assert cos > 0.999, cos
  assert np.abs(got - ref).max() < 0.02 * np.abs(ref).max()


def test_llama3_rope_scaling_read_from_checkpoint(tmp_path):
  from aneforge_b200 import llm
  rs = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
        "original_max_position_embeddings": 64}
  d, _ = _tiny("llama", tmp_path, rope_scaling=rs, rope_theta=500000.0)
  m = llm.from_pretrained(str(d))
  assert m.cfg.rope_base == 500000.0
  assert m.cfg.rope_scaling and m.cfg.rope_scaling["rope_type"] == "llama3"
  got = llm.rope_tables(200, m.cfg.dh, m.cfg.rope_base, scaling=m.cfg.rope_scaling)
  ref = oracle_rope_tables(200, m.cfg.dh, m.cfg.rope_base, scaling=m.cfg.rope_scaling)
  for a, b in zip(got, ref):
    np.testing.assert_array_equal(a.view(np.uint16), b.view(np.uint16))


def test_dense_loader_refuses_unsupported_architectures():
  from aneforge_b200 import llm

  class C:
    model_type = "gemma3_text"
  with pytest.raises(ValueError):
    llm._assert_dense_compatible(C())

  class D:
    model_type = "llama"
    final_logit_softcapping = 30.0
  with pytest.raises(ValueError):
    llm._assert_dense_compatible(D())


@pytest.mark.parametrize("args", [(600, 128, 5e5, 0), (64, 64, 1e4, 32), (33, 80, 1e6, 0)])
def test_rope_tables_match_oracle(args):
  from aneforge_b200.llm import rope_tables
  got = rope_tables(*args)
  ref = oracle_rope_tables(*args)
  for a, b in zip(got, ref):
    np.testing.assert_array_equal(a.view(np.uint16), b.view(np.uint16))


def test_sampling_rules_match_oracle_draws():
  """Temperature / top-k / top-p sampling draws the same tokens as the oracle's restatement of the
  reference's `_sample` (`aneforge/llm.py:407-419`) from the same seeded global generator."""
  from aneforge_b200.llm import sample_token
  rng = np.random.default_rng(3)
  for trial in range(200):
    lg = rng.standard_normal(257).astype(np.float32) * 3
    if trial % 7 == 0:
      lg[rng.integers(0, 257, 5)] = lg.max()              # exact ties at the top
    t, p, k = [(0.0, 1.0, 0), (0.7, 1.0, 0), (1.0, 0.9, 0), (0.8, 1.0, 5), (1.3, 0.5, 40)][trial % 5]
    np.random.seed(trial)
    a = sample_token(lg, t, p, k)
    np.random.seed(trial)
    b = OracleModel.sample(lg, t, p, k)
    assert a == b, (trial, t, p, k)
