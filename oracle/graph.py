"""Numpy interpreter of the graph IR (`aneforge_b200.graph`, the reference's `aneforge/graph.py`
ops): what a graph computes under the reference's lowering, as the oracle states it.

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`): the GPU tests compare `compile(graph)` with
this interpreter, and the CPU tests compare graphs built by the block builders with
`oracle.model.OracleModel` (whose decoder numerics are pinned to the reference's golden vectors).

Semantics (the oracle's device precision, `oracle/model.py` header):
  * every value is fp32; input ports and output ports are fp16;
  * a `matmul` weight is encoded by the reference policy (`quant.encode_weight`, i.e.
    `aneforge/_compile.py:112-188`) and applied as `oracle.model.Linear` does: int8 as
    (x . codes^T) * scale, others as x . decoded^T, plus the fp16 bias; the activation operand is
    rounded to fp16 first, as are both operands of an activation x activation `bmm`;
  * `bmm_weight` decodes its weight as one row per batch entry (`aneforge/_compile.py:393-399`) and
    multiplies the fp16-rounded activation by the decoded fp32 values;
  * `rms_norm` uses the reference's baked constants (`aneforge/_compile.py:738-755`).
"""
from __future__ import annotations

import numpy as np

from . import quant
from .model import Linear, layer_norm, rms_consts, rms_norm, softmax

F16, F32 = np.float16, np.float32


def _f16(x):
  return np.asarray(x, F32).astype(F16).astype(F32)


def _topo(outs):
  seen, order = set(), []

  def visit(t):
    stack = [(t, False)]
    while stack:
      n, done = stack.pop()
      if done:
        order.append(n)
        continue
      if id(n) in seen:
        continue
      seen.add(id(n))
      stack.append((n, True))
      for s in reversed(n.srcs):
        if id(s) not in seen:
          stack.append((s, False))
  for o in outs:
    visit(o)
  return order


_UNARY = {
  "relu": lambda x, a: np.maximum(x, 0), "silu": lambda x, a: x / (1 + np.exp(-x)),
  "sigmoid": lambda x, a: 1 / (1 + np.exp(-x)), "tanh": lambda x, a: np.tanh(x), "exp": lambda x, a: np.exp(x),
  "sqrt": lambda x, a: np.sqrt(x), "abs": lambda x, a: np.abs(x), "square": lambda x, a: x * x,
  "sin": lambda x, a: np.sin(x), "cos": lambda x, a: np.cos(x),
  "log": lambda x, a: np.log(x + a["eps"]), "rsqrt": lambda x, a: 1 / np.sqrt(x + a["eps"]),
  "inverse": lambda x, a: 1 / (x + a["eps"]),
  # scalar constants are baked fp16 like every constant of the reference program (`_compile.py:334-346`)
  "muls": lambda x, a: x * F32(np.float16(a["k"])), "adds": lambda x, a: x + F32(np.float16(a["k"])), "clip": lambda x, a: np.clip(x, a["lo"], a["hi"]),
  "logical_not": lambda x, a: (x == 0).astype(F32), "floor": lambda x, a: np.floor(x),
  "ceil": lambda x, a: np.ceil(x), "round": lambda x, a: np.rint(x), "sign": lambda x, a: np.sign(x),
  "softplus": lambda x, a: np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))),
}
_BINARY = {
  "add": np.add, "sub": np.subtract, "mul": np.multiply, "real_div": np.divide, "maximum": np.maximum,
  "minimum": np.minimum, "pow": np.power,
  "greater": lambda a, b: (a > b).astype(F32), "greater_equal": lambda a, b: (a >= b).astype(F32),
  "less": lambda a, b: (a < b).astype(F32), "less_equal": lambda a, b: (a <= b).astype(F32),
  "equal": lambda a, b: (a == b).astype(F32), "not_equal": lambda a, b: (a != b).astype(F32),
}
_REDUCE = {"reduce_sum": np.sum, "reduce_mean": np.mean, "reduce_max": np.max, "reduce_min": np.min}


class GraphInterp:
  """Evaluate a multi-output graph: `run({input tensor: array})` -> [fp16 output arrays]."""

  def __init__(self, outs, compress=None, compress_atol=0.05, block_size=32):
    self.outs = list(outs)
    self.order = _topo(self.outs)
    self.compress, self.atol, self.bs = compress, compress_atol, block_size
    self._lin: dict = {}

  def _linear(self, t):
    if id(t) not in self._lin:
      self._lin[id(t)] = Linear(np.asarray(t.attrs["wt"]), t.attrs.get("bias"), self.compress, self.atol, self.bs)
    return self._lin[id(t)]

  def run(self, feeds: dict) -> list:
    v: dict = {}
    for t in self.order:
      s = [v[id(x)] for x in t.srcs]
      op, a = t.op, t.attrs
      if op == "input":
        r = _f16(np.asarray(feeds[t]).reshape(t.shape))
      elif op == "const_array":
        r = np.asarray(a["value"], F16).astype(F32)
      elif op == "reshape":
        r = s[0].reshape(t.shape)
      elif op in _UNARY:
        r = _UNARY[op](s[0], a)
      elif op == "gelu":
        from math import erf
        r = 0.5 * s[0] * (1 + np.vectorize(erf)(s[0] / np.sqrt(2.0)).astype(F32))
      elif op == "erf":
        from math import erf
        r = np.vectorize(erf)(s[0]).astype(F32)
      elif op in _BINARY:
        r = _BINARY[op](s[0], s[1])
      elif op == "select":
        r = np.where(s[0] != 0, s[1], s[2])
      elif op == "transpose":
        r = np.transpose(s[0], a["perm"])
      elif op == "slice_by_size":
        r = s[0][tuple(slice(b, b + n) for b, n in zip(a["begin"], a["size"]))]
      elif op == "concat":
        r = np.concatenate(s, axis=a["axis"])
      elif op in _REDUCE:
        r = _REDUCE[op](s[0], axis=a["axes"], keepdims=True)
      elif op == "reduce_sum_square":
        r = np.sum(s[0] * s[0], axis=a["axes"], keepdims=True)
      elif op == "reduce_l1_norm":
        r = np.sum(np.abs(s[0]), axis=a["axes"], keepdims=True)
      elif op == "softmax":
        r = softmax(s[0], axis=a["axis"])
      elif op == "rms_norm":
        g, floor = rms_consts(a["gamma"], a["eps"])
        r = rms_norm(s[0], g, floor)
      elif op == "layer_norm":
        beta = a.get("beta")
        r = layer_norm(s[0], np.asarray(a["gamma"], F16),
                       np.zeros(t.shape[-1], F16) if beta is None else np.asarray(beta, F16), a["eps"])
      elif op == "matmul":
        x = s[0]
        r = self._linear(t)(_f16(x).reshape(-1, x.shape[-1])).reshape(t.shape)
      elif op == "bmm":
        r = np.matmul(_f16(s[0]), _f16(s[1]))
      elif op == "bmm_w":
        W = np.asarray(a["wt"])
        enc = quant.encode_weight(W, self.compress, self.atol, self.bs, allow_int8=True, allow_int4=True,
                                  allow_sparse=False)
        r = np.matmul(_f16(s[0]), enc.deq.reshape(W.shape).astype(F32))
      else:
        raise NotImplementedError(op)
      v[id(t)] = np.asarray(r, F32)
    return [v[id(o)].astype(F16) for o in self.outs]
