"""CPU checks of the mixture-of-experts pieces: the oracle's Qwen2-MoE shared expert against the
reference formula (`aneforge/moe.py:60-62`) and the GGUF loader (`aneforge/moe.py:129-173`)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle.model import F16, F32, Config, OracleModel, random_llama_weights, rms_norm, silu


def _cfg(renorm=False):
  return Config(dim=256, n_layers=1, n_heads=4, n_kv_heads=2, ffn_dim=128, vocab=512, rope_base=10000.0,
                head_dim=64, extra={"n_experts": 4, "n_experts_per_tok": 2, "norm_topk_prob": renorm})


def test_oracle_shared_expert_is_the_reference_formula():
  cfg = _cfg()
  w = random_llama_weights(cfg, seed=3, std=0.05, moe=True, shared_expert=192)
  plain = {**w, "layers": [{k: v for k, v in w["layers"][0].items()
                            if not k.endswith("_sh") and k != "shared_gate"}]}
  with_sh = OracleModel(cfg, w, None, precision="fp32")
  without = OracleModel(cfg, plain, None, precision="fp32")
  h = np.random.default_rng(4).standard_normal((5, cfg.dim)).astype(F32)
  d = with_sh._mlp(with_sh.layers[0], h) - without._mlp(without.layers[0], h)
  lw = w["layers"][0]
  f = lambda a: np.asarray(a, F32)
  hn = rms_norm(h, *with_sh.layers[0]["mlp_norm"])
  sh = (silu(hn @ f(lw["wgate_sh"]).T) * (hn @ f(lw["wup_sh"]).T)) @ f(lw["wdown_sh"]).T
  gate = 1.0 / (1.0 + np.exp(-(hn @ f(lw["shared_gate"]).T)))
  np.testing.assert_allclose(d, sh * gate, rtol=1e-4, atol=1e-5 * np.abs(sh).max())
  assert np.abs(sh * gate).max() > 1e-3                  # the term is not vanishing


def _write_qwen_moe_gguf(path, arch, rng, n_layers=2, dim=128, heads=4, kv=2, ffn=64, E=4, k=2, vocab=96,
                         q8_experts=True, router_scale=1.0):
  """A small Qwen-MoE GGUF in llama.cpp's tensor naming; returns the arrays written (numpy order)."""
  import gguf
  from gguf.quants import dequantize, quantize
  Q8 = gguf.GGMLQuantizationType.Q8_0
  wr = gguf.GGUFWriter(str(path), arch)
  for key, v in (("block_count", n_layers), ("embedding_length", dim), ("attention.head_count", heads),
                 ("attention.head_count_kv", kv), ("expert_count", E), ("expert_used_count", k)):
    wr.add_uint32(f"{arch}.{key}", v)
  wr.add_float32(f"{arch}.rope.freq_base", 1000000.0)
  wr.add_float32(f"{arch}.attention.layer_norm_rms_epsilon", 1e-6)
  dh = dim // heads
  arrays = {}

  def put(name, a, q8=False):
    a = a.astype(np.float32)
    if q8:
      qa = quantize(a.reshape(-1, a.shape[-1]), Q8)
      wr.add_tensor(name, qa.reshape(*a.shape[:-1], qa.shape[-1]), raw_dtype=Q8)
      arrays[name] = dequantize(qa, Q8).reshape(a.shape).astype(np.float16)
    else:
      wr.add_tensor(name, a.astype(np.float16) if a.ndim > 1 else a)
      arrays[name] = a.astype(np.float16)

  R = lambda *s: rng.standard_normal(s).astype(np.float32) * 0.05
  put("token_embd.weight", R(vocab, dim)); put("output_norm.weight", 1 + R(dim)); put("output.weight", R(vocab, dim))
  for L in range(n_layers):
    b = f"blk.{L}."
    put(b + "attn_q.weight", R(heads * dh, dim)); put(b + "attn_k.weight", R(kv * dh, dim))
    put(b + "attn_v.weight", R(kv * dh, dim)); put(b + "attn_output.weight", R(dim, heads * dh))
    put(b + "attn_norm.weight", 1 + R(dim)); put(b + "ffn_norm.weight", 1 + R(dim))
    put(b + "ffn_gate_inp.weight", R(E, dim) * router_scale)
    put(b + "ffn_gate_exps.weight", R(E, ffn, dim), q8_experts); put(b + "ffn_up_exps.weight", R(E, ffn, dim), q8_experts)
    put(b + "ffn_down_exps.weight", R(E, dim, ffn), q8_experts)
    if arch == "qwen3moe":
      put(b + "attn_q_norm.weight", 1 + R(dh)); put(b + "attn_k_norm.weight", 1 + R(dh))
    else:
      put(b + "attn_q.bias", R(heads * dh)); put(b + "attn_k.bias", R(kv * dh)); put(b + "attn_v.bias", R(kv * dh))
      put(b + "ffn_gate_shexp.weight", R(2 * ffn, dim)); put(b + "ffn_up_shexp.weight", R(2 * ffn, dim))
      put(b + "ffn_down_shexp.weight", R(dim, 2 * ffn)); put(b + "ffn_gate_inp_shexp.weight", R(dim))
  wr.write_header_to_file(); wr.write_kv_data_to_file(); wr.write_tensors_to_file(); wr.close()
  return arrays


@pytest.mark.parametrize("arch", ["qwen2moe", "qwen3moe"])
def test_load_gguf_config_and_weights(tmp_path, arch):
  pytest.importorskip("gguf")
  from aneforge_b200.moe import load_gguf
  path = tmp_path / "m.gguf"
  src = _write_qwen_moe_gguf(path, arch, np.random.default_rng(7))
  m = load_gguf(str(path), n_layers=1, compress="int8")
  c = m.cfg
  assert (c.dim, c.n_layers, c.n_heads, c.n_kv_heads, c.ffn_dim, c.vocab, c.dh) == (128, 1, 4, 2, 64, 96, 32)
  assert c.rope_base == 1000000.0 and abs(c.norm_eps - 1e-6) < 1e-12
  assert c.extra == {"n_experts": 4, "n_experts_per_tok": 2, "norm_topk_prob": arch != "qwen2moe"}
  assert [ls.mlp for ls in c.layers] == ["moe"] and c.layers[0].qk_norm == (arch == "qwen3moe")
  assert m.w["embed"].dtype == np.float32 and m.w["lm_head"].dtype == np.float32
  lw = m.w["layers"][0]
  np.testing.assert_array_equal(lw["wq"], src["blk.0.attn_q.weight"])
  np.testing.assert_array_equal(lw["router"], src["blk.0.ffn_gate_inp.weight"])
  np.testing.assert_array_equal(lw["wgate_exps"], src["blk.0.ffn_gate_exps.weight"])   # Q8_0, dequantized
  np.testing.assert_array_equal(lw["wdown_exps"], src["blk.0.ffn_down_exps.weight"].transpose(0, 2, 1))
  assert lw["wdown_exps"].shape == (4, 64, 128)
  if arch == "qwen2moe":
    assert lw["shared_gate"].shape == (1, 128) and "q_bias" in lw and "q_norm" not in lw
    np.testing.assert_array_equal(lw["wdown_sh"], src["blk.0.ffn_down_shexp.weight"])
  else:
    assert "wgate_sh" not in lw and "q_bias" not in lw
    np.testing.assert_array_equal(lw["k_norm"], src["blk.0.attn_k_norm.weight"])
  # the lazily read layer is made again after the runner drops it
  m.w["layers"].free(0)
  np.testing.assert_array_equal(m.w["layers"][0]["wk"], src["blk.0.attn_k.weight"])
  # the loaded layers run through the oracle's MoE layer (shared expert included for Qwen2-MoE)
  from oracle.model import Config, OracleModel
  oc = Config(dim=c.dim, n_layers=1, n_heads=c.n_heads, n_kv_heads=c.n_kv_heads, ffn_dim=c.ffn_dim,
              vocab=c.vocab, rope_base=c.rope_base, norm_eps=c.norm_eps, head_dim=c.head_dim, extra=dict(c.extra))
  ow = {"embed": m.w["embed"], "final_norm": m.w["final_norm"], "lm_head": m.w["lm_head"], "layers": [lw]}
  om = OracleModel(oc, ow, "int8")
  assert len(om.generate([1, 2, 3], 4, max_len=16)) == 4
