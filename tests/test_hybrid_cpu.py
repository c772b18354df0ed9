"""The Qwen3.5 hybrid mixers (gated DeltaNet, gated attention; reference `aneforge/qwen35.py`, its
tests `tests/test_qwen35.py`) as graph builders, run token by token through the oracle's graph
interpreter (fp16 states carried between steps, as the device keeps them) against the transformers
modules, and the Hugging Face adapter's layer plan."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
q35 = pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")
from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig   # noqa: E402

from aneforge_b200 import blocks, hybrid, llm                                    # noqa: E402
from aneforge_b200 import graph as G                                             # noqa: E402
from oracle.graph import GraphInterp                                             # noqa: E402

F16, F32 = np.float16, np.float32


def _cos(a, b):
  a, b = np.ravel(a).astype(np.float64), np.ravel(b).astype(np.float64)
  return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def _unit_rows(T, D, seed):
  torch.manual_seed(seed)
  x = torch.randn(1, T, D)
  return x / x.pow(2).mean(-1, keepdim=True).sqrt()          # unit RMS: the unit-gamma norm is identity


def _step_mixer(fn, w, cfg, xs, ctx_values=None, M=1):
  """Run a decode-mixer builder token by token; states start at zero and carry over (fp16)."""
  x = G.input((1, cfg.dim))
  ctx = blocks.decode_inputs(M, cfg.dh) if ctx_values else {}
  h, pairs = fn(x, w, cfg, llm.LayerSpec(), ctx, M)
  interp = GraphInterp([h] + [o for o, _ in pairs])
  state = [np.zeros(i.shape, F16) for _, i in pairs]
  outs = []
  for t, row in enumerate(xs):
    feeds = {x: row[None].astype(F16)}
    feeds.update({i: s for (_, i), s in zip(pairs, state)})
    if ctx_values:
      feeds.update({ctx[k]: v for k, v in ctx_values(t).items()})
    r = interp.run(feeds)
    outs.append(np.asarray(r[0], F32).reshape(-1))
    state = [np.asarray(s, F16) for s in r[1:]]
  return np.stack(outs)


def test_gated_deltanet_matches_transformers():
  nk, nv, dk, dv, K, D, T = 2, 6, 16, 16, 4, 64, 8
  ct = Qwen3_5TextConfig(hidden_size=D, linear_num_key_heads=nk, linear_num_value_heads=nv, linear_key_head_dim=dk,
                         linear_value_head_dim=dv, linear_conv_kernel_dim=K, hidden_act="silu", rms_norm_eps=1e-6)
  m = q35.Qwen3_5GatedDeltaNet(ct, layer_idx=0).eval()
  x = _unit_rows(T, D, 0)
  with torch.no_grad():
    o = m(x)
  ref = (o[0] if isinstance(o, tuple) else o)[0].numpy()
  P = {n: p.detach().numpy().astype(F32) for n, p in m.named_parameters()}
  w = {"in_norm": np.ones(D, F32), "in_proj_qkv": P["in_proj_qkv.weight"], "in_proj_z": P["in_proj_z.weight"],
       "in_proj_a": P["in_proj_a.weight"], "in_proj_b": P["in_proj_b.weight"], "conv1d": np.squeeze(P["conv1d.weight"]),
       "neg_exp_A": -np.exp(P["A_log"]), "dt_bias": P["dt_bias"], "ssm_norm": P["norm.weight"],
       "out_proj": P["out_proj.weight"]}
  cfg = llm.LlamaConfig(dim=D, n_layers=1, n_heads=1, n_kv_heads=1, ffn_dim=1, vocab=1, norm_eps=1e-6,
                        extra={"nk": nk, "nv": nv, "dk": dk, "dv": dv, "conv_k": K})
  xs = x[0].numpy()
  out = _step_mixer(hybrid.gated_deltanet_decode, w, cfg, xs) - xs.astype(F16).astype(F32)   # strip the residual
  assert _cos(out, ref) > 0.96, _cos(out, ref)               # fp16 states at a tiny T (reference: ~0.97)


def test_gated_attention_matches_transformers():
  H, KV, dh, D, T = 4, 2, 32, 128, 6
  ct = Qwen3_5TextConfig(hidden_size=D, num_attention_heads=H, num_key_value_heads=KV, head_dim=dh,
                         partial_rotary_factor=0.5, rms_norm_eps=1e-6, rope_theta=1e4, max_position_embeddings=64)
  att = q35.Qwen3_5Attention(ct, layer_idx=0).eval()
  rot = q35.Qwen3_5TextRotaryEmbedding(ct)
  x = _unit_rows(T, D, 1)
  cos, sin = rot(x, torch.arange(T)[None])
  rd = cos.shape[-1]
  mask = torch.full((T, T), float("-inf")).triu(1)[None, None]
  with torch.no_grad():
    ref = att(x, (cos, sin), mask)[0][0].numpy()
  P = {n: p.detach().numpy().astype(F32) for n, p in att.named_parameters()}
  w = {"in_norm": np.ones(D, F32), "wq": P["q_proj.weight"], "wk": P["k_proj.weight"], "wv": P["v_proj.weight"],
       "wo": P["o_proj.weight"], "q_norm": 1.0 + P["q_norm.weight"], "k_norm": 1.0 + P["k_norm.weight"]}
  cfg = llm.LlamaConfig(dim=D, n_layers=1, n_heads=H, n_kv_heads=KV, ffn_dim=1, vocab=1, head_dim=dh, rotary_dim=rd,
                        norm_eps=1e-6, rope_base=1e4)
  cos_t, sin_t = llm.rope_tables(T, dh, 1e4, rd)
  out = _step_mixer(hybrid.gated_attention_decode, w, cfg, x[0].numpy(),
                    lambda t: blocks.decode_values(t, T, cos_t, sin_t), M=T) - x[0].numpy().astype(F16).astype(F32)
  assert _cos(out, ref) > 0.99, _cos(out, ref)


def test_adapter_layer_plan_and_weights():
  ct = Qwen3_5TextConfig(hidden_size=64, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                         partial_rotary_factor=0.5, linear_num_key_heads=2, linear_num_value_heads=6,
                         linear_key_head_dim=16, linear_value_head_dim=16, linear_conv_kernel_dim=4, vocab_size=32,
                         intermediate_size=128, rms_norm_eps=1e-6)
  m = q35.Qwen3_5TextModel(ct).eval()
  sd = {k: v.detach().float().numpy() for k, v in m.state_dict().items()}
  cfg, w = hybrid.adapt(ct, sd)
  assert [ls.mixer for ls in cfg.layers] == ["gated_deltanet"] * 3 + ["gated_attention"]
  assert cfg.rotary_dim == 8 and cfg.extra == {"nk": 2, "nv": 6, "dk": 16, "dv": 16, "conv_k": 4}
  np.testing.assert_allclose(w["layers"][0]["neg_exp_A"], -np.exp(sd["layers.0.linear_attn.A_log"]))
  np.testing.assert_allclose(w["layers"][3]["q_norm"], 1.0 + sd["layers.3.self_attn.q_norm.weight"])
  assert w["layers"][0]["conv1d"].shape == (2 * 32 + 96, 4)
