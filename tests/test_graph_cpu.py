"""The graph IR and the graph-form decoder blocks, on the host: shape rules, and the blocks'
numerics (interpreted by `oracle.graph.GraphInterp`) against the oracle decoder (`OracleModel`, pinned
to the reference's golden vectors). The GPU side - `compile` / `compile_multi` of the same graphs -
is `tests/test_graph_gpu.py`."""
import numpy as np
import pytest

from aneforge_b200 import graph as G
from aneforge_b200 import blocks
from aneforge_b200.llm import LlamaConfig, LayerSpec
from oracle.graph import GraphInterp
from oracle.model import Config, OracleModel, random_llama_weights

F16, F32 = np.float16, np.float32


def cos(a, b):
  a = np.asarray(a, np.float64).ravel(); b = np.asarray(b, np.float64).ravel()
  return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def small(qkv_bias=False, qk_norm=False, n_kv=2):
  ocfg = Config(dim=256, n_layers=1, n_heads=4, n_kv_heads=n_kv, ffn_dim=512, vocab=64, rope_base=10000.0,
                head_dim=64, qk_norm=qk_norm)
  w = random_llama_weights(ocfg, seed=3, std=0.05, qkv_bias=qkv_bias)
  if qk_norm:
    rng = np.random.default_rng(4)
    w["layers"][0]["q_norm"] = (1 + 0.1 * rng.standard_normal(64)).astype(F32)
    w["layers"][0]["k_norm"] = (1 + 0.1 * rng.standard_normal(64)).astype(F32)
  bcfg = LlamaConfig(dim=256, n_layers=1, n_heads=4, n_kv_heads=n_kv, ffn_dim=512, vocab=64, rope_base=10000.0,
                     head_dim=64, layers=[LayerSpec(qk_norm=qk_norm)])
  return ocfg, bcfg, w


def test_shape_rules():
  x = G.input((3, 1, 8))
  y = G.input((4, 8))
  assert (x + y).shape == (3, 4, 8)
  with pytest.raises(ValueError):
    _ = x + G.input((5, 7))
  w = np.zeros((16, 8), F32)
  assert x.linear(w).shape == (3, 1, 16)
  assert (x @ w.T).shape == (3, 1, 16)
  assert (G.input((2, 5, 8)) @ G.input((2, 8, 3))).shape == (2, 5, 3)
  assert x.transpose([2, 0, 1]).shape == (8, 3, 1)
  assert x.reshape(-1, 8).shape == (3, 8)
  assert x.sum([0, 2]).shape == (1, 1, 1)
  with pytest.raises(ValueError):
    x.slice_by_size([0, 0, 4], [3, 1, 5])
  assert G.concat([x, x], axis=2).shape == (3, 1, 16)
  assert len(G.split(y, 2, axis=1)) == 2 and G.split(y, 2, axis=1)[1].shape == (4, 4)
  with pytest.raises(ValueError):
    G.Tensor((1, 1, 1, 1, 1, 1), "input")
  assert blocks.is_graph_builder(blocks.swiglu) and not blocks.is_graph_builder(lambda pb, ctx, li, lw, cfg, ls: 0)


def test_elementwise_and_reductions_interpreted():
  rng = np.random.default_rng(0)
  a = rng.standard_normal((2, 3, 4)).astype(F16)
  b = rng.standard_normal((3, 1)).astype(F16)
  x, y = G.input(a.shape), G.input(b.shape)
  out = ((x * y + x.exp().sum(2)) / G.maximum(x.abs(), y.abs().adds(0.5))).softmax(1)
  got = GraphInterp([out]).run({x: a, y: b})[0].astype(F32)
  A, B = a.astype(F32), b.astype(F32)
  ref = (A * B + np.exp(A).sum(2, keepdims=True)) / np.maximum(np.abs(A), np.abs(B) + 0.5)
  ref = np.exp(ref - ref.max(1, keepdims=True)); ref /= ref.sum(1, keepdims=True)
  np.testing.assert_allclose(got, ref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("compress,qkv_bias,qk_norm,n_kv", [("int8", False, False, 2), (None, True, True, 4),
                                                            ("int8", True, False, 1)])
def test_decode_block_graph_matches_oracle(compress, qkv_bias, qk_norm, n_kv):
  """`blocks.attn_decode` + `blocks.swiglu` (the reference's `_attn_decode` / `_swiglu` in graph
  form) at a decode position against `OracleModel.decode_layer`."""
  ocfg, bcfg, w = small(qkv_bias, qk_norm, n_kv)
  M, pos = 48, 29
  rng = np.random.default_rng(5)
  Kc = rng.standard_normal((n_kv, M, 64)).astype(F16)
  Vc = rng.standard_normal((n_kv, M, 64)).astype(F16)
  h = rng.standard_normal((1, 256)).astype(F16)
  from aneforge_b200.llm import rope_tables
  cos_t, sin_t = rope_tables(M, 64, 10000.0)
  x = G.input((1, 256))
  ctx = blocks.decode_inputs(M, 64)
  lw, ls = w["layers"][0], bcfg.layers[0]
  hm, pairs = blocks.attn_decode(x, lw, bcfg, ls, ctx, M)
  out = blocks.swiglu(hm, lw, bcfg, ls)
  (k_out, k_in), (v_out, v_in) = pairs
  vals = blocks.decode_values(pos, M, cos_t, sin_t)
  feeds = {x: h, k_in: Kc, v_in: Vc, **{ctx[k]: vals[k] for k in blocks.DECODE_CTX}}
  got, gk, gv = GraphInterp([out, k_out, v_out], compress).run(feeds)
  om = OracleModel(ocfg, w, compress, precision="device")
  om._tables(M)
  Ko, Vo = Kc.copy(), Vc.copy()
  ref = om.decode_layer(om.layers[0], h.astype(F32), Ko, Vo, pos).astype(F16)
  assert cos(got, ref) > 0.9999
  assert np.linalg.norm(got.astype(F32) - ref.astype(F32)) / np.linalg.norm(ref.astype(F32)) < 1e-2
  # the cache: only slot pos changes, to the step's (roped) k / v
  np.testing.assert_array_equal(np.delete(gk, pos, axis=1), np.delete(Kc, pos, axis=1))
  np.testing.assert_allclose(gk[:, pos].astype(F32), Ko[:, pos].astype(F32), rtol=2e-3, atol=2e-3)
  np.testing.assert_allclose(gv[:, pos].astype(F32), Vo[:, pos].astype(F32), rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("compress", ["int8", None])
def test_prefill_block_graph_matches_oracle(compress):
  """`blocks.attn_prefill_kv` + `blocks.swiglu` over a prompt against the oracle's batched prefill."""
  ocfg, bcfg, w = small()
  S = 21
  rng = np.random.default_rng(6)
  rows = (rng.standard_normal((S, 256)) * 0.5).astype(F16)
  from aneforge_b200.llm import rope_tables
  cos_t, sin_t = rope_tables(S, 64, 10000.0)
  x = G.input((S, 256))
  lw, ls = w["layers"][0], bcfg.layers[0]
  h, (kc, vc) = blocks.attn_prefill_kv(x, lw, bcfg, ls, cos_t, sin_t)
  out = blocks.swiglu(h, lw, bcfg, ls)
  got, gk, gv = GraphInterp([out, kc, vc], compress).run({x: rows})
  om = OracleModel(ocfg, {**w, "final_norm": np.ones(256, F32)}, compress, precision="device")
  # the oracle's prefill without its final norm: run its layer loop on the same rows
  om._tables(S)
  hid, kv = om.causal_pass(rows, om.layers)
  # causal_pass applies the final norm; compare K / V and the normed hidden of the graph output
  from oracle.model import rms_norm, rms_consts
  normed = rms_norm(got.astype(F32), *rms_consts(np.ones(256, F32), ocfg.norm_eps)).astype(F16)
  assert cos(normed, hid) > 0.9999
  np.testing.assert_allclose(gk.astype(F32), kv[0][0].astype(F32), rtol=5e-3, atol=5e-3)
  np.testing.assert_allclose(gv.astype(F32), kv[0][1].astype(F32), rtol=5e-3, atol=5e-3)
