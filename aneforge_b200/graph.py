"""Device-free graph IR: the lazy `Tensor` DAG the reference's model code builds
(`aneforge/graph.py:29-436`), kept so that graph-building code written for the reference - the
decoder block builders of `aneforge/llm.py:96-237`, a plugin's mixer or MLP - runs here unchanged and
is lowered by `aneforge_b200.compile` / `compile_multi` onto this package's CUDA kernels.

A `Tensor` is (shape, op, srcs, attrs); nothing is computed when it is built. The op names, the
shape rules (numpy broadcasting, `linear` weights stored [out, in], `@` with a weight array stored
transposed, reductions keeping their axes) and the constructor signatures follow the reference, so
a graph means the same thing on both sides; which ops exist is this module's own list (the ones a
decoder needs, plus the common elementwise and shape ops).
"""
from __future__ import annotations

import itertools
from typing import Any, Sequence

import numpy as np

MAX_RANK = 5                      # the reference's device limit, kept so graphs port both ways

_input_order = itertools.count()


def _weight_array(a, what: str) -> np.ndarray:
  a = np.asarray(a.detach().float().cpu().numpy() if hasattr(a, "detach") else a)
  if a.dtype not in (np.float16, np.float32, np.float64):
    raise TypeError(f"{what}: weights must be floating point (got {a.dtype})")
  return a


def broadcast_shape(sa: Sequence[int], sb: Sequence[int]) -> tuple:
  """numpy broadcasting of two shapes (ValueError when they do not broadcast)."""
  n = max(len(sa), len(sb))
  a = (1,) * (n - len(sa)) + tuple(sa)
  b = (1,) * (n - len(sb)) + tuple(sb)
  out = []
  for x, y in zip(a, b):
    if x != y and x != 1 and y != 1:
      raise ValueError(f"shapes {tuple(sa)} and {tuple(sb)} do not broadcast")
    out.append(max(x, y))
  return tuple(out)


class Tensor:
  """One node of a graph: its output shape, the op that makes it, its source nodes and attributes."""

  __slots__ = ("shape", "op", "srcs", "attrs", "_name")

  def __init__(self, shape: Sequence[int], op: str, srcs: Sequence["Tensor"] = (), attrs: dict | None = None):
    self.shape = tuple(int(d) for d in shape)
    if len(self.shape) > MAX_RANK:
      raise ValueError(f"rank {len(self.shape)} > {MAX_RANK} (op {op!r}, shape {self.shape})")
    if any(d <= 0 for d in self.shape):
      raise ValueError(f"op {op!r}: every dimension must be positive, got {self.shape}")
    self.op = op
    self.srcs = list(srcs)
    self.attrs = dict(attrs or {})
    self._name = ""

  def __repr__(self) -> str:
    return f"Tensor({self.op}, shape={self.shape})"

  @property
  def size(self) -> int:
    return int(np.prod(self.shape))

  # -- elementwise, one operand
  def _unary(self, op: str, **attrs) -> "Tensor":
    return Tensor(self.shape, op, [self], attrs)

  def relu(self): return self._unary("relu")
  def gelu(self): return self._unary("gelu")
  def silu(self): return self._unary("silu")
  def sigmoid(self): return self._unary("sigmoid")
  def tanh(self): return self._unary("tanh")
  def exp(self): return self._unary("exp")
  def sqrt(self): return self._unary("sqrt")
  def abs(self): return self._unary("abs")
  def square(self): return self._unary("square")
  def sin(self): return self._unary("sin")
  def cos(self): return self._unary("cos")
  def erf(self): return self._unary("erf")
  def softplus(self): return self._unary("softplus")
  def floor(self): return self._unary("floor")
  def ceil(self): return self._unary("ceil")
  def round(self): return self._unary("round")
  def sign(self): return self._unary("sign")
  def logical_not(self): return self._unary("logical_not")
  def log(self, eps: float = 0.0): return self._unary("log", eps=float(eps))
  def rsqrt(self, eps: float = 0.0): return self._unary("rsqrt", eps=float(eps))
  def inverse(self, eps: float = 0.0): return self._unary("inverse", eps=float(eps))
  def clip(self, lo: float, hi: float): return self._unary("clip", lo=float(lo), hi=float(hi))
  clamp = clip

  def adds(self, k: float) -> "Tensor":
    """`x + k` for a scalar k."""
    return self._unary("adds", k=float(k))

  # -- elementwise, two operands (numpy broadcasting; a non-Tensor operand becomes a constant)
  def __add__(self, o): return _binary(self, o, "add")
  def __sub__(self, o): return _binary(self, o, "sub")
  def __truediv__(self, o): return _binary(self, o, "real_div")
  def __pow__(self, o): return _binary(self, o, "pow")
  pow = __pow__

  def __mul__(self, o):
    if isinstance(o, (int, float)):
      return self._unary("muls", k=float(o))
    return _binary(self, o, "mul")
  __rmul__ = __mul__

  def __neg__(self): return self._unary("muls", k=-1.0)

  def greater(self, o): return _binary(self, o, "greater")
  def less(self, o): return _binary(self, o, "less")
  def equal(self, o): return _binary(self, o, "equal")
  def not_equal(self, o): return _binary(self, o, "not_equal")
  def less_equal(self, o): return _binary(self, o, "less_equal")
  def greater_equal(self, o): return _binary(self, o, "greater_equal")

  # -- matrix products
  def __matmul__(self, W) -> "Tensor":
    """`x @ W`: a weight array W [K, N] (quantizable under compress=), or a Tensor for an
    activation x activation product (batched over the leading axes, numpy broadcasting)."""
    if isinstance(W, Tensor):
      if len(self.shape) < 2 or len(W.shape) < 2 or self.shape[-1] != W.shape[-2]:
        raise ValueError(f"matmul: {self.shape} @ {W.shape}")
      batch = broadcast_shape(self.shape[:-2], W.shape[:-2])
      return Tensor(batch + (self.shape[-2], W.shape[-1]), "bmm", [self, W])
    W = _weight_array(W, "matmul weight")
    if W.ndim != 2 or self.shape[-1] != W.shape[0]:
      raise ValueError(f"matmul: x{self.shape} @ W{W.shape}")
    return Tensor(self.shape[:-1] + (W.shape[1],), "matmul", [self], {"wt": np.ascontiguousarray(W.T)})

  def linear(self, W, bias=None) -> "Tensor":
    """`x @ W.T + bias` with W [out, in] (the PyTorch layout)."""
    W = _weight_array(W, "linear weight")
    if W.ndim != 2 or self.shape[-1] != W.shape[1]:
      raise ValueError(f"linear: x{self.shape} W{W.shape}")
    attrs: dict[str, Any] = {"wt": np.ascontiguousarray(W)}
    if bias is not None:
      attrs["bias"] = _weight_array(bias, "linear bias").astype(np.float32).reshape(-1)
    return Tensor(self.shape[:-1] + (W.shape[0],), "matmul", [self], attrs)

  def bmm_weight(self, W) -> "Tensor":
    """`x [B, M, K] @ W [B, K, N]` with W a quantizable baked weight (per-expert projections)."""
    W = _weight_array(W, "bmm_weight")
    if W.ndim != 3 or len(self.shape) != 3 or self.shape[-1] != W.shape[1] or self.shape[0] not in (1, W.shape[0]):
      raise ValueError(f"bmm_weight: x{self.shape} @ W{W.shape}")
    return Tensor((W.shape[0], self.shape[1], W.shape[2]), "bmm_w", [self], {"wt": np.ascontiguousarray(W)})

  # -- shape
  def transpose(self, perm) -> "Tensor":
    perm = tuple(int(p) % len(self.shape) for p in perm)
    if sorted(perm) != list(range(len(self.shape))):
      raise ValueError(f"transpose: {perm} is not a permutation of rank {len(self.shape)}")
    return Tensor(tuple(self.shape[p] for p in perm), "transpose", [self], {"perm": perm})

  def reshape(self, *shape) -> "Tensor":
    if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
      shape = tuple(shape[0])
    shape = tuple(int(d) for d in shape)
    if -1 in shape:
      known = int(np.prod([d for d in shape if d != -1]))
      shape = tuple(self.size // known if d == -1 else d for d in shape)
    if int(np.prod(shape)) != self.size:
      raise ValueError(f"reshape: {self.shape} -> {shape} changes the element count")
    return Tensor(shape, "reshape", [self])

  def squeeze(self, axes) -> "Tensor":
    axes = {int(a) % len(self.shape) for a in (axes if isinstance(axes, (tuple, list)) else (axes,))}
    if any(self.shape[a] != 1 for a in axes):
      raise ValueError(f"squeeze: an axis of {sorted(axes)} is not of size 1 in {self.shape}")
    return Tensor(tuple(d for i, d in enumerate(self.shape) if i not in axes), "reshape", [self])

  def expand_dims(self, axes) -> "Tensor":
    axes = axes if isinstance(axes, (tuple, list)) else (axes,)
    rank = len(self.shape) + len(axes)
    ax = {int(a) % rank for a in axes}
    it = iter(self.shape)
    return Tensor(tuple(1 if i in ax else next(it) for i in range(rank)), "reshape", [self])

  def flatten2d(self, axis: int = 1) -> "Tensor":
    ax = axis % len(self.shape)
    rows = int(np.prod(self.shape[:ax])) if ax else 1
    return Tensor((rows, self.size // rows), "reshape", [self])

  def slice_by_size(self, begin, size) -> "Tensor":
    begin, size = [int(b) for b in begin], [int(s) for s in size]
    if len(begin) != len(self.shape) or len(size) != len(self.shape):
      raise ValueError(f"slice_by_size: begin/size need rank {len(self.shape)}")
    for d, (b, s) in enumerate(zip(begin, size)):
      if b < 0 or s <= 0 or b + s > self.shape[d]:
        raise ValueError(f"slice_by_size: axis {d} window [{b}, {b + s}) outside {self.shape[d]}")
    return Tensor(tuple(size), "slice_by_size", [self], {"begin": begin, "size": size})

  # -- reductions (axes kept with size 1) and normalisation
  def _reduce(self, op: str, axes) -> "Tensor":
    axes = tuple(sorted({int(a) % len(self.shape) for a in (axes if isinstance(axes, (tuple, list)) else (axes,))}))
    return Tensor(tuple(1 if i in axes else d for i, d in enumerate(self.shape)), op, [self], {"axes": axes})

  def sum(self, axes): return self._reduce("reduce_sum", axes)
  def mean(self, axes): return self._reduce("reduce_mean", axes)
  def amax(self, axes): return self._reduce("reduce_max", axes)
  def amin(self, axes): return self._reduce("reduce_min", axes)
  def sum_square(self, axes): return self._reduce("reduce_sum_square", axes)
  def l1_norm(self, axes): return self._reduce("reduce_l1_norm", axes)

  def softmax(self, axis: int = -1) -> "Tensor":
    return Tensor(self.shape, "softmax", [self], {"axis": axis % len(self.shape)})

  def l2_norm(self, axis: int = -1, eps: float = 1e-12) -> "Tensor":
    """x / sqrt(sum(x^2, axis) + eps)."""
    n = self.sum_square(axis).adds(eps).sqrt()
    return self / n

  def rms_norm(self, gamma, eps: float = 1e-5) -> "Tensor":
    """RMSNorm over the last axis with the reference's lowering (`aneforge/_compile.py:738-755`):
    x / max(||x||_2, f16(sqrt(D * eps))) * f16(gamma * sqrt(D)). `gamma` a [D] array, or a Tensor
    (then a unit-gamma norm times it)."""
    if isinstance(gamma, Tensor):
      return self.rms_norm(np.ones(self.shape[-1], np.float32), eps) * gamma
    gamma = _weight_array(gamma, "rms_norm gamma").reshape(-1)
    if gamma.shape != (self.shape[-1],):
      raise ValueError(f"rms_norm: gamma {gamma.shape} for rows of {self.shape[-1]}")
    return Tensor(self.shape, "rms_norm", [self], {"gamma": gamma.astype(np.float32), "eps": float(eps)})

  def layer_norm(self, gamma, beta, eps: float = 1e-5) -> "Tensor":
    """LayerNorm over the last axis: (x - mean) / sqrt(var + eps) * gamma + beta."""
    gamma = _weight_array(gamma, "layer_norm gamma").reshape(-1).astype(np.float32)
    beta = None if beta is None else _weight_array(beta, "layer_norm beta").reshape(-1).astype(np.float32)
    return Tensor(self.shape, "layer_norm", [self], {"gamma": gamma, "beta": beta, "eps": float(eps)})


def input(shape: Sequence[int], dtype: str = "fp16", max_abs: float | None = None) -> Tensor:  # noqa: A001
  """A graph input (a program port), fed to the compiled model in creation order."""
  if dtype != "fp16":
    raise ValueError(f"input: only fp16 ports exist on this path (got {dtype!r})")
  t = Tensor(tuple(shape), "input")
  t.attrs["idx"] = next(_input_order)
  if max_abs is not None:
    t.attrs["max_abs"] = float(max_abs)
  return t


def const(value) -> Tensor:
  """A baked constant (stored fp16, as the reference bakes `const_array`)."""
  v = np.asarray(value, np.float16)
  if v.ndim == 0:
    v = v.reshape(1)
  return Tensor(v.shape, "const_array", [], {"value": v})


_const = const                                  # the reference's private name, used by model code


def _binary(a: Tensor, b, op: str) -> Tensor:
  if not isinstance(b, Tensor):
    b = const(b)
  return Tensor(broadcast_shape(a.shape, b.shape), op, [a, b])


def maximum(a: Tensor, b) -> Tensor:
  return _binary(a, b, "maximum")


def minimum(a: Tensor, b) -> Tensor:
  return _binary(a, b, "minimum")


def concat(tensors: Sequence[Tensor], axis: int = 1) -> Tensor:
  ts = list(tensors)
  ax = axis % len(ts[0].shape)
  for t in ts[1:]:
    if len(t.shape) != len(ts[0].shape) or any(d != e for i, (d, e) in enumerate(zip(t.shape, ts[0].shape)) if i != ax):
      raise ValueError(f"concat: {t.shape} vs {ts[0].shape} on axis {ax}")
  shape = list(ts[0].shape)
  shape[ax] = sum(t.shape[ax] for t in ts)
  return Tensor(tuple(shape), "concat", ts, {"axis": ax})


_concat = concat


def stack(tensors: Sequence[Tensor], axis: int = 0) -> Tensor:
  ts = list(tensors)
  ax = axis % (len(ts[0].shape) + 1)
  return concat([t.expand_dims(ax) for t in ts], axis=ax)


def split(x: Tensor, num_splits: int, axis: int = 0) -> list[Tensor]:
  ax = axis % len(x.shape)
  if x.shape[ax] % num_splits:
    raise ValueError(f"split: axis {ax} of {x.shape} does not divide into {num_splits}")
  part = x.shape[ax] // num_splits
  out = []
  for i in range(num_splits):
    begin = [0] * len(x.shape); begin[ax] = i * part
    size = list(x.shape); size[ax] = part
    out.append(x.slice_by_size(begin, size))
  return out


def gather(x: Tensor, indices, axis: int = 0) -> Tensor:
  """Rows of `x` at STATIC integer indices along `axis`."""
  ax = axis % len(x.shape)
  rows = []
  for i in (int(i) for i in indices):
    if not 0 <= i < x.shape[ax]:
      raise ValueError(f"gather: index {i} outside axis {ax} of size {x.shape[ax]}")
    begin = [0] * len(x.shape); begin[ax] = i
    size = list(x.shape); size[ax] = 1
    rows.append(x.slice_by_size(begin, size))
  return concat(rows, axis=ax)


def select(cond: Tensor, a: Tensor, b: Tensor) -> Tensor:
  """Elementwise `cond ? a : b` (cond nonzero = true), numpy broadcasting over all three."""
  if not all(isinstance(t, Tensor) for t in (cond, a, b)):
    raise TypeError("select takes three graph Tensors")
  return Tensor(broadcast_shape(cond.shape, broadcast_shape(a.shape, b.shape)), "select", [cond, a, b])


where = select


def topo_order(*outs: Tensor) -> list[Tensor]:
  """Every node reachable from `outs`, each after its sources (iterative post-order)."""
  seen, order = set(), []
  for root in outs:
    stack_ = [(root, False)]
    while stack_:
      t, done = stack_.pop()
      if done:
        order.append(t)
        continue
      if id(t) in seen:
        continue
      seen.add(id(t))
      stack_.append((t, True))
      for s in reversed(t.srcs):
        if id(s) not in seen:
          stack_.append((s, False))
  return order
