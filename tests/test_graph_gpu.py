"""`compile(graph, compress=...)` and `compile_multi` (reference `aneforge/_compile.py:1360-1404`,
`:987-1037`) on the B200, against the host interpreter of the same graph (`oracle.graph`) and the
oracle decoder.

Bars: outputs within rel-err 1e-2 and cosine >= 0.999 of the interpreter (the graph path's own
kernels differ from the interpreter only in fp32 summation order); the one-block decode graph run
for several steps through `compile_multi` with its K / V state aliased onto its inputs
(`share_buffer`, as `LlamaPrefill._decoder` does) matches the oracle decoder at every step.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from aneforge_b200 import graph as G                                           # noqa: E402
from aneforge_b200 import blocks                                              # noqa: E402
from oracle.graph import GraphInterp                                          # noqa: E402
from oracle.model import Config, OracleModel, random_llama_weights            # noqa: E402

F16, F32 = np.float16, np.float32


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")


def close(got, ref, rel=1e-2, cmin=0.999):
  g = np.asarray(got, np.float64).ravel(); r = np.asarray(ref, np.float64).ravel()
  c = float(g @ r / (np.linalg.norm(g) * np.linalg.norm(r) + 1e-30))
  e = float(np.linalg.norm(g - r) / (np.linalg.norm(r) + 1e-30))
  assert e <= rel and c >= cmin, (e, c)


def test_compile_generic_ops_match_interpreter():
  from aneforge_b200 import compile as afc
  rng = np.random.default_rng(1)
  a = rng.standard_normal((2, 6, 8)).astype(F16)
  b = rng.standard_normal((6, 1)).astype(F16)
  x, y = G.input(a.shape), G.input(b.shape)
  t = (x * y + x.exp().sum(2)) / G.maximum(x.abs(), y.abs().adds(0.5))
  t = t.softmax(1).transpose([0, 2, 1])                                          # [2, 8, 6]
  u = G.concat([t.slice_by_size([0, 0, 0], [2, 8, 3]), (t.slice_by_size([0, 0, 3], [2, 8, 3]) * -2.0)], axis=2)
  s = G.select(u.greater(G.const(np.zeros((1, 1, 6), F16))), u, u.square())
  m = (s @ x).amax([1]) + s.mean([1, 2]).reshape(2, 1, 1)                        # bmm [2, 8, 8] -> [2, 1, 8]
  out = m.linear(rng.standard_normal((5, 8)).astype(F32) * 0.3, bias=np.arange(5, dtype=F32)).tanh().rsqrt(2.0)
  model = afc(out)
  got = model(a, b)
  ref = GraphInterp([out]).run({x: a, y: b})[0]
  assert got.shape == out.shape and got.dtype == F32
  close(got, ref, rel=2e-3, cmin=0.99999)
  with pytest.raises(ValueError):
    model(a[:1], b)
  assert model.n_ops > 15
  model.release()


@pytest.mark.parametrize("compress", ["int8", None, "int4_g32", "blockwise"])
@pytest.mark.parametrize("rows,K", [(1, 256), (20, 256), (40, 256), (3, 24)])
def test_compile_linear_paths(compress, rows, K):
  """A `linear` on each path: tensor-core GEMV (<= 16 rows, 16-row slices above), tcgen05 GEMM
  (>= 32 rows), the packed blockwise GEMV, and the generic matmul (contraction not a multiple of 32)."""
  from aneforge_b200 import compile as afc
  if compress == "int4_g32" and K % 32:
    pytest.skip("group-32 int4 needs K % 32 == 0 (falls back to fp16, covered by compress=None)")
  rng = np.random.default_rng(rows + K)
  W = (rng.standard_normal((96, K)) * 0.05).astype(F32)
  bias = (rng.standard_normal(96) * 0.1).astype(F32)
  xv = rng.standard_normal((rows, K)).astype(F16)
  x = G.input((rows, K))
  out = x.linear(W, bias)
  got = afc(out, compress=compress)(xv)
  ref = GraphInterp([out], compress).run({x: xv})[0]
  close(got, ref, rel=3e-3, cmin=0.99999)


def _block_case(n_kv=2, qk_norm=False, qkv_bias=False):
  from aneforge_b200.llm import LlamaConfig, LayerSpec
  ocfg = Config(dim=256, n_layers=1, n_heads=4, n_kv_heads=n_kv, ffn_dim=512, vocab=64, rope_base=10000.0,
                head_dim=64, qk_norm=qk_norm)
  w = random_llama_weights(ocfg, seed=3, std=0.05, qkv_bias=qkv_bias)
  bcfg = LlamaConfig(dim=256, n_layers=1, n_heads=4, n_kv_heads=n_kv, ffn_dim=512, vocab=64, rope_base=10000.0,
                     head_dim=64, layers=[LayerSpec(qk_norm=qk_norm)])
  return ocfg, bcfg, w


@pytest.mark.parametrize("compress,n_kv,qkv_bias", [("int8", 2, False), (None, 4, True), ("int8", 1, True)])
def test_compile_multi_decode_block_resident_state(compress, n_kv, qkv_bias):
  """The reference's decode-step construction (`aneforge/llm.py:435-478`): one block's decode graph,
  compiled with its K / V state outputs aliased onto the state inputs, stepped 4 times."""
  from aneforge_b200 import compile_multi
  from aneforge_b200.llm import rope_tables
  ocfg, bcfg, w = _block_case(n_kv, qkv_bias=qkv_bias)
  M = 40
  cos_t, sin_t = rope_tables(M, 64, 10000.0)
  x = G.input((1, 256))
  ctx = blocks.decode_inputs(M, 64)
  lw, ls = w["layers"][0], bcfg.layers[0]
  hm, pairs = blocks.attn_decode(x, lw, bcfg, ls, ctx, M)
  h = blocks.swiglu(hm, lw, bcfg, ls)
  net = compile_multi([h] + [o for o, _ in pairs], compress=compress)
  inm = {id(t): n for t, n in net.input_ports}
  om = dict((id(t), n) for t, n in net.output_ports)
  for o, i in pairs:
    net.prog.share_buffer(0, om[id(o)], 0, inm[id(i)])
  om_ = OracleModel(ocfg, w, compress, precision="device")
  om_._tables(M)
  Ko, Vo = om_.new_caches(M)[0]
  rng = np.random.default_rng(9)
  pre = 30
  Kc = rng.standard_normal((n_kv, M, 64)).astype(F16); Kc[:, pre:] = 0
  Vc = rng.standard_normal((n_kv, M, 64)).astype(F16); Vc[:, pre:] = 0
  Ko[:] = Kc; Vo[:] = Vc
  (k_out, k_in), (v_out, v_in) = pairs
  net.prog.set_input(inm[id(k_in)], Kc); net.prog.set_input(inm[id(v_in)], Vc)
  for step in range(4):
    pos = pre + step
    hv = rng.standard_normal((1, 256)).astype(F16)
    vals = blocks.decode_values(pos, M, cos_t, sin_t)
    net.prog.set_input(inm[id(x)], hv)
    for k in blocks.DECODE_CTX:
      net.prog.set_input(inm[id(ctx[k])], vals[k])
    net.prog.execute()
    got = net.prog.read_output(om[id(h)])
    ref = om_.decode_layer(om_.layers[0], hv.astype(F32), Ko, Vo, pos).astype(F16)
    close(got, ref)
    kd = net.prog.read_output(om[id(k_out)])
    np.testing.assert_allclose(kd[:, pos].astype(F32), Ko[:, pos].astype(F32), rtol=4e-3, atol=4e-3)
  net.release()


@pytest.mark.parametrize("S,compress", [(21, "int8"), (40, "int8"), (40, None)])
def test_compile_multi_prefill_block(S, compress):
  """The reference's prefill construction (`aneforge/llm.py:489-519`): a prompt block emitting its
  cache K / V; 40 rows run the projections on the tcgen05 GEMM."""
  from aneforge_b200 import compile_multi
  from aneforge_b200.llm import rope_tables
  ocfg, bcfg, w = _block_case()
  cos_t, sin_t = rope_tables(S, 64, 10000.0)
  x = G.input((S, 256))
  lw, ls = w["layers"][0], bcfg.layers[0]
  h, (kc, vc) = blocks.attn_prefill_kv(x, lw, bcfg, ls, cos_t, sin_t)
  h = blocks.swiglu(h, lw, bcfg, ls)
  net = compile_multi([h, kc, vc], compress=compress)
  rows = (np.random.default_rng(2).standard_normal((S, 256)) * 0.5).astype(F16)
  out = net(rows)
  ref = GraphInterp([h, kc, vc], compress).run({x: rows})
  for (t, name), r in zip(net.output_ports, ref):
    close(out[name], r)
  net.release()


def test_model_zero_copy_views():
  """`input_view` / `output_view` / `execute`: the reference's hot-loop API, device views here."""
  from aneforge_b200 import compile as afc
  x = G.input((4, 32))
  m = afc((x * 2.0).adds(1.0))
  xv = m.input_view()
  assert xv.is_cuda and tuple(xv.shape) == (4, 32) and xv.dtype == torch.float16
  xv.copy_(torch.arange(128, device=xv.device, dtype=torch.float16).reshape(4, 32) / 64)
  torch.cuda.synchronize()
  m.execute()
  got = m.output_view().float().cpu().numpy()
  ref = (np.arange(128, dtype=F32).reshape(4, 32) / 64) * 2 + 1
  np.testing.assert_allclose(got, ref, rtol=1e-3)
  m.release()
