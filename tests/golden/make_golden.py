"""Generate the golden fixtures that pin the oracle to the reference (sbryngelson/ANEForge).

Run ONLY where the reference is mounted (it imports the reference package read-only):

    ANEFORGE_REF=/path/to/ANEForge python tests/golden/make_golden.py

Nothing at test time imports the reference; the tests read the `.npz` files written here.

What is captured, all from the reference's own code on seeded inputs:
  * quant.npz   - bytes of `_blob.quantize_per_row`, `palettize_lut4`, `quantize_blockwise`
                  (divisible and indivisible IN), `sparsify`; the encoding `_Emitter.weight`
                  picks per compress mode; the RMSNorm constants `_e_rms_norm` bakes.
  * llm_*.npz   - tokens and per-step logits of the reference `LlamaPrefill.generate`
                  (and `prefill`) on tiny random models. The device is replaced by a numpy
                  interpreter of the reference graph IR, patched in at
                  `aneforge._compile.compile` / `compile_multi` - the seam the reference's own
                  off-device tests use (`tests/test_lm_head.py:15-36`). The interpreter runs every
                  internal node in fp32 and rounds ports to fp16; matmul weights are decoded from
                  the blobs the reference's `_Emitter.weight` writes.
  * moe.npz     - the reference `moe._moe` layer and `_topk_gate` through the same interpreter.
"""
from __future__ import annotations

import os
import re
import sys
from pathlib import Path
from unittest import mock

import numpy as np

HERE = Path(__file__).resolve().parent
REF = os.environ.get("ANEFORGE_REF", "")
if not REF or not os.path.isdir(os.path.join(REF, "aneforge")):
  sys.exit("set ANEFORGE_REF to a checkout of the reference (the directory holding aneforge/)")
sys.path.insert(0, REF)

import aneforge as af                               # noqa: E402  (reference package)
from aneforge import _blob, _compile               # noqa: E402
from aneforge import llm as rllm                    # noqa: E402
from aneforge import moe as rmoe                    # noqa: E402

F16, F32 = np.float16, np.float32


# ----------------------------------------------------------------------------- weight decoding

def _decode_last_weight(em, W, start_items: int, line: str):
  """Decode the blobs `_Emitter.weight` just appended into the fp32 matrix the device uses."""
  items = em.blob._items[start_items:]
  W2 = np.asarray(W).reshape(W.shape[0], -1)
  if "constexpr_affine_dequantize" in line:
    q = np.frombuffer(items[0][0], np.int8).reshape(W2.shape).astype(F32)
    s = np.frombuffer(items[1][0], F16).astype(F32)
    return "int8", (q * s[:, None]).reshape(W.shape)
  if "constexpr_lut_to_dense" in line:
    raw = np.frombuffer(items[0][0], np.uint8)
    lut = np.frombuffer(items[1][0], F16).astype(F32)
    idx = np.empty(raw.size * 2, np.uint8); idx[0::2], idx[1::2] = raw & 15, raw >> 4
    return "lut4", lut[idx][: W2.size].reshape(W.shape)
  if "constexpr_blockwise_shift_scale" in line or re.search(r"_bw\b", line):
    OUT, IN = W2.shape
    q = np.frombuffer(items[0][0], np.int8).astype(F32)
    s = np.frombuffer(items[1][0], F16).astype(F32)
    nb = s.size // OUT
    return "blockwise", (q.reshape(OUT, nb, IN // nb) * s.reshape(OUT, nb)[:, :, None]).reshape(W.shape)
  if "constexpr_sparse_to_dense" in line:
    mask = np.unpackbits(np.frombuffer(items[0][0], np.uint8), bitorder="little")[: W2.size].astype(bool)
    nz = np.frombuffer(items[1][0], F16).astype(F32)
    out = np.zeros(W2.size, F32); out[mask] = nz
    return "sparse", out.reshape(W.shape)
  return "fp16", np.frombuffer(items[0][0], F16).astype(F32).reshape(W.shape)


def encode_with_reference(W, compress, atol=0.05, block_size=32, **kw):
  """Run the reference `_Emitter.weight` and decode what it wrote."""
  em = _compile._Emitter(False, compress=compress, compress_atol=atol, block_size=block_size)
  n0, l0 = len(em.blob._items), len(em.lines)
  em.weight("w", np.asarray(W), **kw)
  line = "\n".join(em.lines[l0:])
  return _decode_last_weight(em, np.asarray(W), n0, line)


def rms_constants_with_reference(gamma, eps):
  """Run the reference `_e_rms_norm` emitter and read back g_eff and the floor it baked."""
  D = gamma.shape[0]
  em = _compile._Emitter(False)
  t = af.input((2, D)).rms_norm(gamma, eps)
  _compile._EMIT["rms_norm"](em, t, "n", ["x"])
  g = np.frombuffer(em.blob._items[-1][0], F16).copy()
  m = re.search(r"n_ep = const\(\)\[name=string\(\"n_ep\"\), val=fp16\(([^)]*)\)", "\n".join(em.lines))
  return g, np.float16(float.fromhex(m.group(1)))


# ----------------------------------------------------------------------------- IR interpreter

class Interp:
  """fp32 numpy evaluation of a reference graph; ports are fp16."""

  def __init__(self, outs, compress, atol=0.05, block_size=32):
    self.order = _compile._topo_multi(*outs)
    for i, t in enumerate(self.order):
      t._name = f"t{i}"
    self.inputs = sorted((t for t in self.order if t.op == "input"), key=lambda t: t.attrs.get("idx", 0))
    self.outs = list(outs)
    self.compress, self.atol, self.bs = compress, atol, block_size
    self.wcache: dict = {}
    self.ports = {t._name: np.zeros(t.shape, F16) for t in self.inputs}
    self.results: dict = {}
    self.alias: list = []

  def _w(self, t, key="wt", **kw):
    if id(t) not in self.wcache:
      self.wcache[id(t)] = encode_with_reference(t.attrs[key], self.compress, self.atol, self.bs, **kw)[1]
    return self.wcache[id(t)]

  def run(self):
    v: dict = {}
    for t in self.order:
      s = [v[id(x)] for x in t.srcs]
      op, a = t.op, t.attrs
      if op == "input":
        r = self.ports[t._name].astype(F32)
      elif op == "const_array":
        r = np.asarray(a["value"], F16).astype(F32)
      elif op == "matmul":
        W = self._w(t, allow_int8=True, int8=a.get("int8"), allow_int4=True, allow_sparse=True)
        r = s[0] @ W.reshape(W.shape[0], -1).T
        if "bias" in a:
          r = r + np.asarray(a["bias"]).astype(F16).astype(F32).reshape(1, -1)
      elif op == "bmm":
        r = np.matmul(s[0], s[1])
      elif op == "bmm_w":
        W = self._w(t, allow_int8=True, int8=a.get("int8"), allow_int4=True)
        r = np.matmul(s[0], W)
      elif op == "rms_norm":
        g, floor = rms_constants_with_reference(np.asarray(a["gamma"]).reshape(-1), a["eps"])
        x = s[0]
        nrm = np.sqrt(np.sum(x * x, axis=-1, keepdims=True, dtype=F32))
        r = (x / np.maximum(nrm, F32(floor))) * g.astype(F32)
      elif op == "muls":
        r = s[0] * F32(np.float16(a["k"]))
      elif op == "adds":
        r = s[0] + F32(np.float16(a["k"]))
      elif op == "add": r = s[0] + s[1]
      elif op == "sub": r = s[0] - s[1]
      elif op == "mul": r = s[0] * s[1]
      elif op == "real_div": r = s[0] / s[1]
      elif op == "maximum": r = np.maximum(s[0], s[1])
      elif op == "minimum": r = np.minimum(s[0], s[1])
      elif op == "pow": r = np.power(s[0], s[1])
      elif op == "reshape": r = s[0].reshape(t.shape)
      elif op == "transpose": r = np.transpose(s[0], a["perm"])
      elif op == "slice_by_size":
        sl = tuple(slice(b, b + z) for b, z in zip(a["begin"], a["size"]))
        r = s[0][sl]
      elif op == "concat": r = np.concatenate(s, axis=a["axis"])
      elif op == "softmax":
        x = s[0]; m = x.max(axis=a["axis"], keepdims=True); e = np.exp(x - m)
        r = e / e.sum(axis=a["axis"], keepdims=True)
      elif op == "silu": r = s[0] / (F32(1.0) + np.exp(-s[0]))
      elif op == "sigmoid": r = F32(1.0) / (F32(1.0) + np.exp(-s[0]))
      elif op == "tanh": r = np.tanh(s[0])
      elif op == "exp": r = np.exp(s[0])
      elif op == "reduce_max": r = s[0].max(axis=tuple(a["axes"]), keepdims=True)
      elif op == "reduce_sum": r = s[0].sum(axis=tuple(a["axes"]), keepdims=True)
      elif op == "greater_equal": r = s[0] >= s[1]
      elif op == "equal": r = s[0] == s[1]
      elif op == "select": r = np.where(s[0], s[1], s[2])
      else:
        raise NotImplementedError(op)
      if r.dtype != bool:
        r = np.asarray(r, F32)
      v[id(t)] = r
    self.results = {o._name: v[id(o)].astype(F16) for o in self.outs}
    for out_name, in_name in self.alias:                     # resident state: output buffer IS the input
      self.ports[in_name] = self.results[out_name].copy()


class NumpyProgram:
  """The `Program` surface `llm.py` drives (`_runtime.py:138-248`)."""

  def __init__(self, interp: Interp):
    self.it = interp

  def set_input(self, name, arr):
    if name not in self.it.ports:
      raise KeyError(name)
    self.it.ports[name] = np.asarray(arr).astype(F16).reshape(self.it.ports[name].shape)

  def execute(self):
    self.it.run()

  def read_output(self, name):
    return self.it.results[name].copy()

  def share_buffer(self, src_op, src_out, dst_op, dst_in):
    self.it.alias.append((src_out, dst_in))

  def release(self):
    pass

  def eval(self, feed):
    for k, a in feed.items():
      self.set_input(k, a)
    self.execute()
    return dict(self.it.results)


class NumpyMultiModel:
  def __init__(self, outs, compress=None, compress_atol=0.05, block_size=32, **_):
    it = Interp(outs, compress, compress_atol, block_size)
    self.prog = NumpyProgram(it)
    self.input_ports = [(t, t._name) for t in it.inputs]
    self.output_ports = [(t, t._name) for t in it.outs]

  def release(self):
    pass


class NumpyModel:
  def __init__(self, out, compress=None, compress_atol=0.05, block_size=32, **_):
    self.it = Interp([out], compress, compress_atol, block_size)
    self.out = out

  def __call__(self, *arrays):
    for t, a in zip(self.it.inputs, arrays):
      self.it.ports[t._name] = np.asarray(a).astype(F16)
    self.it.run()
    return self.it.results[self.out._name].astype(F32)

  def release(self):
    pass


def fake_compile(out, int8=False, build_dir=None, opt="routes", compress=None, compress_atol=0.05,
                 block_size=32, validate=False, target=None, **_):
  if out.op == "input":
    out = out * 1.0
  return NumpyModel(out, compress, compress_atol, block_size)


def fake_compile_multi(outs, build_dir=None, int8=False, compress=None, compress_atol=0.05, block_size=32):
  return NumpyMultiModel(outs, compress, compress_atol, block_size)


def patched():
  return mock.patch.multiple(_compile, compile=fake_compile, compile_multi=fake_compile_multi)


# ----------------------------------------------------------------------------- fixtures

def random_weights(cfg, seed, std=0.02, bias=False, qk_norm=False, moe=None):
  """Seeded N(0, std) fp16 weights in the reference layout, unit norms."""
  rng = np.random.default_rng(seed)
  R = lambda *s: (rng.standard_normal(s, dtype=F32) * F32(std)).astype(F16)
  D, dh = cfg.dim, cfg.dh
  w = {"embed": R(cfg.vocab, D), "final_norm": np.ones(D, F32), "lm_head": R(cfg.vocab, D), "layers": []}
  for _ in range(cfg.n_layers):
    lw = {"wq": R(cfg.n_heads * dh, D), "wk": R(cfg.n_kv_heads * dh, D), "wv": R(cfg.n_kv_heads * dh, D),
          "wo": R(D, cfg.n_heads * dh), "attn_norm": (1.0 + 0.1 * rng.standard_normal(D)).astype(F32),
          "mlp_norm": (1.0 + 0.1 * rng.standard_normal(D)).astype(F32)}
    if bias:
      lw["q_bias"] = R(cfg.n_heads * dh); lw["k_bias"] = R(cfg.n_kv_heads * dh); lw["v_bias"] = R(cfg.n_kv_heads * dh)
    if qk_norm:
      lw["q_norm"] = (1.0 + 0.1 * rng.standard_normal(dh)).astype(F32)
      lw["k_norm"] = (1.0 + 0.1 * rng.standard_normal(dh)).astype(F32)
    if moe:
      E, ffn = moe
      lw["router"] = R(E, D); lw["wgate_exps"] = R(E, ffn, D); lw["wup_exps"] = R(E, ffn, D)
      lw["wdown_exps"] = R(E, ffn, D)
    else:
      lw["wgate"] = R(cfg.ffn_dim, D); lw["wup"] = R(cfg.ffn_dim, D); lw["wdown"] = R(D, cfg.ffn_dim)
    w["layers"].append(lw)
  return w


def flatten_weights(w):
  flat = {k: np.asarray(v) for k, v in w.items() if k != "layers"}
  for i, lw in enumerate(w["layers"]):
    for k, v in lw.items():
      flat[f"L{i}.{k}"] = np.asarray(v)
  return flat


def quant_fixtures():
  out = {}
  rng = np.random.default_rng(1234)
  W = (rng.standard_normal((48, 96)) * 0.02).astype(F32)
  W[3] = 0.0                                              # an all-zero row: scale clips at 1e-8
  W[5, :7] = [0.5, -0.5, 1.5, 2.5, -2.5, 127.0, -127.0]   # exact ties for round-half-even
  W16 = W.astype(F16)
  out["W"] = W; out["W16"] = W16
  q, s = _blob.quantize_per_row(W)
  out["per_row_q"] = np.frombuffer(q, np.int8).copy(); out["per_row_s"] = np.frombuffer(s, F16).copy()
  q, s = _blob.quantize_per_row(W16)
  out["per_row16_q"] = np.frombuffer(q, np.int8).copy(); out["per_row16_s"] = np.frombuffer(s, F16).copy()
  Wl = (rng.standard_normal((32, 64)) * 0.02).astype(F32)
  out["Wl"] = Wl
  p, lut = _blob.palettize_lut4(Wl)
  out["lut4_packed"] = np.frombuffer(p, np.uint8).copy(); out["lut4_lut"] = np.frombuffer(lut, F16).copy()
  Wo = (rng.standard_normal((8, 33)) * 0.5).astype(F32)        # odd IN: padded row packing
  out["Wo"] = Wo
  p, lut = _blob.palettize_lut4(Wo)
  out["lut4o_packed"] = np.frombuffer(p, np.uint8).copy(); out["lut4o_lut"] = np.frombuffer(lut, F16).copy()
  d, s, nb = _blob.quantize_blockwise(W, 32)
  out["bw_q"] = np.frombuffer(d, np.int8).copy(); out["bw_s"] = np.frombuffer(s, F16).copy(); out["bw_nb"] = np.int64(nb)
  Wi = (rng.standard_normal((8, 90)) * 0.02).astype(F32)       # 90 % 32 != 0: block clamps to 30
  out["Wi"] = Wi
  d, s, nb = _blob.quantize_blockwise(Wi, 32)
  out["bwi_q"] = np.frombuffer(d, np.int8).copy(); out["bwi_s"] = np.frombuffer(s, F16).copy(); out["bwi_nb"] = np.int64(nb)
  Ws = W.copy(); Ws[np.abs(Ws) < 0.02] = 0.0
  out["Ws"] = Ws
  m, v = _blob.sparsify(Ws)
  out["sp_mask"] = np.frombuffer(m, np.uint8).copy(); out["sp_vals"] = np.frombuffer(v, F16).copy()
  # encoding decisions of _Emitter.weight, per compress mode
  modes = [None, "int8", "int4", "blockwise", "sparse", "auto"]
  Mx = np.repeat(np.eye(4, dtype=F16), 2, axis=0)              # the GQA 0/1 expansion matrix
  for name, M in (("W", W), ("Ws", Ws), ("Mx", Mx), ("Wl", Wl)):
    for mode in modes:
      kind, deq = encode_with_reference(M, mode, allow_int8=True, allow_int4=True, allow_sparse=True)
      out[f"enc_{name}_{mode}_kind"] = np.array(kind)
      out[f"enc_{name}_{mode}_deq"] = deq.astype(F32)
  for D, eps in ((64, 1e-5), (4096, 1e-5), (128, 1e-6)):
    gamma = (1.0 + 0.1 * rng.standard_normal(D)).astype(F32)
    g, floor = rms_constants_with_reference(gamma, eps)
    out[f"rms_{D}_{eps}_gamma"] = gamma; out[f"rms_{D}_{eps}_g"] = g; out[f"rms_{D}_{eps}_floor"] = floor
  np.savez_compressed(HERE / "quant.npz", **out)


def llm_fixture(tag, cfg, w, compress, prompt, n_new, max_len=None, batched=True, pad=None, qk=False):
  specs = [rllm.LayerSpec(mixer="attention", mlp="swiglu", qk_norm=qk) for _ in range(cfg.n_layers)]
  cfg.layers = specs
  steps = []
  with patched():
    m = rllm.LlamaPrefill(cfg, w, compress=compress, ane_lm_head=False)
    orig = m._logits
    def spy(h, ane=None):
      lg = orig(h, ane); steps.append(np.asarray(lg, F32).copy()); return lg
    m._logits = spy
    toks = m.generate(prompt, max_new_tokens=n_new, max_len=max_len, batched_prefill=batched,
                      prefill_pad=pad)
    m._logits = orig
    m2 = rllm.LlamaPrefill(cfg, w, compress=compress, ane_lm_head=False)
    pre = np.asarray(m2.prefill(prompt), F32)
  out = flatten_weights(w)
  out.update(tokens=np.array(toks, np.int64), logits=np.stack(steps), prefill_logits=pre,
             prompt=np.array(prompt, np.int64), n_new=np.int64(n_new),
             max_len=np.int64(max_len or 0), batched=np.bool_(batched), pad=np.int64(pad or 0),
             compress=np.array(str(compress)),
             cfg=np.array([cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.ffn_dim, cfg.vocab,
                           cfg.head_dim], np.int64),
             rope_base=np.float64(cfg.rope_base), norm_eps=np.float64(cfg.norm_eps), qk_norm=np.bool_(qk))
  np.savez_compressed(HERE / f"llm_{tag}.npz", **out)
  print(tag, toks)


def moe_fixture():
  cfg = rllm.LlamaConfig(dim=64, n_layers=1, n_heads=4, n_kv_heads=2, ffn_dim=32, vocab=16,
                         extra={"n_experts": 8, "n_experts_per_tok": 2, "norm_topk_prob": True})
  w = random_weights(cfg, 7, std=0.1, moe=(8, 32))["layers"][0]
  out = {k: np.asarray(v) for k, v in w.items()}
  rng = np.random.default_rng(9)
  for compress in (None, "int8"):
    for T in (1, 5):
      h = (rng.standard_normal((T, cfg.dim)) * 0.5).astype(F16)
      with patched():
        net = _compile.compile(rmoe._moe(af.input((T, cfg.dim)), w, cfg, rllm.LayerSpec(mlp="moe")),
                               compress=compress)
        y = net(h)
      out[f"h_{compress}_{T}"] = h; out[f"y_{compress}_{T}"] = y
  rows = np.array([[0.2, 0.2, 0.2, 0.1, 0.1, 0.1, 0.05, 0.05],
                   [0.3, 0.2, 0.2, 0.2, 0.05, 0.03, 0.01, 0.01],
                   [0.1, 0.1, 0.1, 0.1, 0.1, 0.1, 0.2, 0.2],
                   [0.4, 0.3, 0.1, 0.1, 0.05, 0.03, 0.01, 0.01]], F16)
  with patched():
    g = _compile.compile(rmoe._topk_gate(af.input((4, 8)), 2, 8, 4))(rows)
  out["topk_rows"] = rows; out["topk_out"] = g
  np.savez_compressed(HERE / "moe.npz", **out)


def main():
  quant_fixtures()
  C = rllm.LlamaConfig
  cfg = C(dim=64, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=128, vocab=48)
  w = random_weights(cfg, 0, std=0.1)
  llm_fixture("int8", cfg, w, "int8", list(range(1, 9)), 8)
  llm_fixture("int8_tbt", cfg, w, "int8", list(range(1, 9)), 8, batched=False)
  llm_fixture("fp16", cfg, w, None, list(range(1, 9)), 8)
  llm_fixture("int4", cfg, w, "int4", [5, 3, 9, 1], 6, max_len=16, pad=8)
  cfgb = C(dim=64, n_layers=2, n_heads=4, n_kv_heads=1, ffn_dim=96, vocab=40, rope_base=500000.0, head_dim=32)
  wb = random_weights(cfgb, 3, std=0.1, bias=True, qk_norm=True)
  llm_fixture("bias_qknorm", cfgb, wb, "int8", [7, 2, 2, 11, 30], 6, qk=True)
  cfgm = C(dim=64, n_layers=2, n_heads=4, n_kv_heads=4, ffn_dim=64, vocab=32)
  wm = random_weights(cfgm, 5, std=0.1)
  llm_fixture("mha", cfgm, wm, "int8", [1, 2, 3], 5, batched=False)
  moe_fixture()


if __name__ == "__main__":
  main()
