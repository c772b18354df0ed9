"""`compile(graph, compress=...)` -> callable and `compile_multi`: the reference's compile API
(`aneforge/_compile.py:1360-1404`, `:987-1037`) over this package's graph IR, lowered onto a program
of CUDA kernels instead of an ANE program.

Lowering. The graph is visited in topological order (ports named `t<i>` by that order, as the
reference names them) and every node becomes plan ops over device buffers:

  * values are fp32 buffers; a reshape / squeeze / expand_dims aliases its source;
  * inputs and outputs are fp16 ports (cast in / cast out), so `share_buffer` can alias a state
    output onto its input for resident state, as `LlamaPrefill` does with the KV cache;
  * a `linear` / `@` weight is encoded by the reference's policy (`compress`, `compress_atol`,
    `block_size`; `weights.encode_linear`): int8 per-row and group-32 int4 weights whose contraction
    is a multiple of 32 run on the tensor-core GEMV (<= 16 rows at a time) or the tcgen05 GEMM
    (>= 32 rows); anything else runs the generic matmul kernel;
  * the remaining ops run the generic kernels of `csrc/graph_ops.cu`.

Numerics are the reference graph's as the oracle states them (`oracle/graph.py` interprets the same
IR on the host): fp32 values, fp16 ports, fp16-rounded activation operands of every matmul, the
reference's RMSNorm constants. There is no CPU path: compiling needs the built library and a GPU.
"""
from __future__ import annotations

import numpy as np

from . import _blob
from . import _runtime as R
from .graph import Tensor, topo_order
from .plan import PlanBuilder, at

F16, F32 = np.float16, np.float32

_UNARY = {"relu": 0, "silu": 1, "sigmoid": 2, "tanh": 3, "exp": 4, "sqrt": 5, "abs": 6, "square": 7, "sin": 8,
          "cos": 9, "erf": 10, "log": 11, "rsqrt": 12, "inverse": 13, "muls": 14, "adds": 15, "clip": 16,
          "logical_not": 17, "floor": 18, "ceil": 19, "round": 20, "sign": 21, "gelu": 23, "softplus": 24}
_BINARY = {"add": 0, "sub": 1, "mul": 2, "real_div": 3, "maximum": 4, "minimum": 5, "pow": 6, "greater": 7,
           "greater_equal": 8, "less": 9, "less_equal": 10, "equal": 11, "not_equal": 12}
_SELECT = 13
_REDUCE = {"reduce_sum": 0, "reduce_mean": 1, "reduce_max": 2, "reduce_min": 3, "reduce_sum_square": 4,
           "reduce_l1_norm": 6}
_ALIASES = ("reshape",)
SUPPORTED_OPS = (set(_UNARY) | set(_BINARY) | set(_REDUCE) | set(_ALIASES) |
                 {"input", "const_array", "select", "transpose", "slice_by_size", "concat", "softmax", "rms_norm",
                  "layer_norm", "matmul", "bmm", "bmm_w"})
GEMM_MIN_ROWS = 32


def contiguous_strides(shape) -> list:
  st, s = [], 1
  for d in reversed(shape):
    st.append(s)
    s *= int(d)
  return st[::-1]


def broadcast_strides(shape, out_shape) -> list:
  """Element strides of a contiguous operand of `shape` read at every index of `out_shape` (numpy
  broadcasting: 0 along an axis the operand repeats)."""
  pad = len(out_shape) - len(shape)
  full = [1] * pad + list(shape)
  cs = contiguous_strides(full)
  return [0 if full[d] == 1 and out_shape[d] != 1 else cs[d] for d in range(len(out_shape))]


def _csv(v) -> str:
  return ",".join(str(int(x)) for x in v)


def rms_constants(gamma, eps):
  """The two constants the reference bakes for `rms_norm` (`aneforge/_compile.py:738-748`):
  g_eff = f16(f32(gamma) * sqrt(D)) and floor = f16(sqrt(D * eps))."""
  g = np.asarray(gamma, F32).reshape(-1)
  D = g.shape[0]
  return (g * np.float32(np.sqrt(D))).astype(F16), float(np.float16((D * float(eps)) ** 0.5))


class Lowering:
  """Plan ops for a graph, appended to `pb` (a fresh plan, or a decode program being built:
  `inputs` then maps graph inputs to existing fp32 value buffers and no ports are made for them).
  Buffer names carry `prefix` so several graphs can share one plan."""

  def __init__(self, pb: PlanBuilder, compress=None, atol=0.05, block_size=32, device=0, prefix="g"):
    self.pb, self.compress, self.atol, self.bs, self.device, self.prefix = pb, compress, atol, block_size, device, prefix
    self.val: dict = {}              # id(tensor) -> fp32 value buffer (contiguous)
    self.binds: list = []            # (buffer, torch CUDA tensor) bound after the program exists
    self.uploads: list = []          # (buffer, host array) uploaded after the program exists
    self.n_ops = 0

  def _buf(self, name, nbytes, role="tmp"):
    return self.pb.buf(f"{self.prefix}.{name}", nbytes, role)

  def value(self, t: Tensor) -> str:
    return self.val[id(t)]

  def set_value(self, t: Tensor, buf: str) -> None:
    self.val[id(t)] = buf

  def _weight(self, name, arr: np.ndarray) -> str:
    a = np.ascontiguousarray(arr)
    b = self._buf(name, max(a.nbytes, 1), "weight")
    self.uploads.append((b, a))
    return b

  def lower(self, order, names) -> None:
    for t in order:
      if id(t) in self.val:
        continue
      self._node(t, names[id(t)])

  # -- one node
  def _node(self, t: Tensor, nm: str) -> None:
    pb, op, a = self.pb, t.op, t.attrs
    n = t.size
    if op in _ALIASES:
      self.val[id(t)] = self.value(t.srcs[0])
      return
    self.n_ops += op not in ("input", "const_array")
    if op == "const_array":
      self.val[id(t)] = self._weight(f"{nm}.c", np.asarray(a["value"], F16).astype(F32))
      return
    if op == "input":
      raise ValueError(f"graph input {nm} has no port or binding")
    y = self._buf(f"{nm}.v", 4 * n)
    self.val[id(t)] = y
    if op in _UNARY:
      k = a.get("k", a.get("eps", a.get("lo", 0.0)))
      if op in ("muls", "adds"):
        k = float(np.float16(k))            # scalar constants are baked fp16, as in the reference program
      k2 = a.get("hi", 0.0)
      pb.op("g_un", op=_UNARY[op], x=self.value(t.srcs[0]), y=y, n=n, k=float(k), k2=float(k2))
    elif op in _BINARY or op == "select":
      srcs = t.srcs
      kv = dict(op=_SELECT if op == "select" else _BINARY[op], shape=_csv(t.shape), y=y)
      for key, s in zip(("a", "b", "c"), srcs):
        kv[key] = self.value(s)
        kv["s" + key] = _csv(broadcast_strides(s.shape, t.shape))
      pb.op("g_ew", **kv)
    elif op == "transpose":
      src = t.srcs[0]
      ist = contiguous_strides(src.shape)
      pb.op("g_copy", x=self.value(src), y=y, shape=_csv(t.shape), sx=_csv([ist[p] for p in a["perm"]]),
            sy=_csv(contiguous_strides(t.shape)))
    elif op == "slice_by_size":
      src = t.srcs[0]
      ist = contiguous_strides(src.shape)
      off = sum(b * s for b, s in zip(a["begin"], ist))
      pb.op("g_copy", x=at(self.value(src), 4 * off), y=y, shape=_csv(t.shape), sx=_csv(ist),
            sy=_csv(contiguous_strides(t.shape)))
    elif op == "concat":
      ax, ost, off = a["axis"], contiguous_strides(t.shape), 0
      for s in t.srcs:
        pb.op("g_copy", x=self.value(s), y=at(y, 4 * off * ost[ax]), shape=_csv(s.shape),
              sx=_csv(contiguous_strides(s.shape)), sy=_csv(ost))
        off += s.shape[ax]
    elif op in _REDUCE:
      src = t.srcs[0]
      mask = sum(1 << d for d in a["axes"])
      pb.op("g_reduce", op=_REDUCE[op], x=self.value(src), y=y, shape=_csv(src.shape), mask=mask)
    elif op == "softmax":
      ax = a["axis"]
      outer = int(np.prod(t.shape[:ax])) if ax else 1
      inner = int(np.prod(t.shape[ax + 1:])) if ax + 1 < len(t.shape) else 1
      pb.op("g_softmax", x=self.value(t.srcs[0]), y=y, outer=outer, n=t.shape[ax], inner=inner)
    elif op == "rms_norm":
      g, floor = rms_constants(a["gamma"], a["eps"])
      D = t.shape[-1]
      pb.op("g_rms", x=self.value(t.srcs[0]), y=y, g=self._weight(f"{nm}.g", g), floor=floor, rows=n // D, d=D)
    elif op == "layer_norm":
      D = t.shape[-1]
      # eps rounded to fp16, as the reference's emitter bakes it (`_compile.py:762`)
      kv = dict(x=self.value(t.srcs[0]), y=y, g=self._weight(f"{nm}.g", a["gamma"].astype(F16)),
                eps=float(np.float16(a["eps"])), rows=n // D, d=D)
      if a.get("beta") is not None:
        kv["b"] = self._weight(f"{nm}.b", a["beta"].astype(F16))
      pb.op("g_ln", **kv)
    elif op == "matmul":
      self._linear(t, nm, y)
    elif op == "bmm":
      self._bmm(t, y)
    elif op == "bmm_w":
      self._bmm_weight(t, nm, y)
    else:
      raise NotImplementedError(f"graph op {op!r} has no B200 lowering")

  def _linear(self, t: Tensor, nm: str, y: str) -> None:
    from .weights import encode_linear
    import torch
    W = np.asarray(t.attrs["wt"])
    N, K = W.shape
    bias = t.attrs.get("bias")
    rows = t.size // N
    x = self.value(t.srcs[0])
    lin = encode_linear([W], self.compress, torch.device("cuda", self.device),
                        biases=[None if bias is None else np.asarray(bias, F32)], atol=self.atol,
                        block_size=self.bs)
    wb = self._buf(f"{nm}.w", lin.w.numel() * lin.w.element_size(), "weight")
    self.binds.append((wb, lin.w))
    kv = dict(n=N, k=K)
    if lin.s is not None:
      sb = self._buf(f"{nm}.s", lin.s.numel() * 2, "weight")
      self.binds.append((sb, lin.s))
      kv["s"] = sb
    if lin.bias is not None:
      bb = self._buf(f"{nm}.b", lin.bias.numel() * 2, "weight")
      self.binds.append((bb, lin.bias))
      kv["bias"] = bb
    if lin.tiled and K % 32 == 0:
      # tensor-core path: fp16 operand rows, fp32 result
      xh = self._buf(f"{nm}.xh", 2 * rows * K)
      self.pb.op("cast", src=x, dst=xh, n=rows * K, mode=1)
      kv.update(wf=lin.wf, epi="f32", x=xh, w=wb, y=y, nb=rows)
      if rows >= GEMM_MIN_ROWS:
        kv["gemm"] = 1
      else:
        nbytes = R.load_library().af_gemv_tc_scratch_bytes(N, K, min(rows, 16))
        kv["scr"] = self.pb.buf("gemv.scr", nbytes, "scratch")
      self.pb.op("gemv", **kv)
    elif lin.kind in ("lut4", "blockwise", "sparse"):
      # packed palette / blockwise codes / sparse bitmask: the CUDA-core GEMVs stream them as they are
      xh = self._buf(f"{nm}.xh", 2 * rows * K)
      self.pb.op("cast", src=x, dst=xh, n=rows * K, mode=1)
      kv["gs"] = kv.pop("s")
      if lin.kind == "blockwise":
        kv["grp"] = lin.group
      if lin.kind == "sparse":
        rb = self._buf(f"{nm}.ro", lin.rowoff.numel() * 4, "weight")
        self.binds.append((rb, lin.rowoff))
        kv.update(ro=rb, nnz=lin.s.numel())
      kv.update(wf=lin.wf, epi="f32", x=xh, w=wb, y=y, nb=rows)
      self.pb.op("gemv", **kv)
    else:
      if lin.kind not in ("int8", "fp16"):
        raise NotImplementedError(f"generic matmul over {lin.kind} weights")
      kv.update(x=x, w=wb, y=y, rows=rows, i8=int(lin.kind == "int8"))
      self.pb.op("g_linear", **kv)

  def _bmm(self, t: Tensor, y: str) -> None:
    A, B = t.srcs
    M, K, N = A.shape[-2], A.shape[-1], B.shape[-1]
    batch = list(t.shape[:-2]) or [1]
    sa = broadcast_strides(list(A.shape[:-2]) or [1], batch) if len(A.shape) > 2 else [0] * len(batch)
    sb = broadcast_strides(list(B.shape[:-2]) or [1], batch) if len(B.shape) > 2 else [0] * len(batch)
    # batch strides above are in units of matrices: scale to elements
    sa = [s * M * K for s in sa]
    sb = [s * K * N for s in sb]
    self.pb.op("g_bmm", a=self.value(A), b=self.value(B), y=y, bshape=_csv(batch), sa=_csv(sa), sb=_csv(sb), m=M,
               n=N, k=K, sam=K, sak=1, sbk=N, sbn=1, rb=1)

  def _bmm_weight(self, t: Tensor, nm: str, y: str) -> None:
    """x [B or 1, M, K] @ W [B, K, N]: W encoded as the reference encodes a `bmm_weight` (one row per
    batch entry of [B, K*N]: per-expert int8 scale under compress="int8"), multiplied by its decoded
    fp32 values (not rounded again); x rounded to fp16 like every matmul operand."""
    W = np.asarray(t.attrs["wt"])
    Bn, K, N = W.shape
    comp = self.compress
    if comp == "int4_g32":
      raise NotImplementedError("bmm_weight under int4_g32 (the expert GEMVs carry that format)")
    dense = _blob.dense_of(W.astype(F32), comp, compress_atol=self.atol, block_size=self.bs, allow_sparse=False)
    wv = self._weight(f"{nm}.wd", dense.astype(F32).reshape(Bn, K, N))
    A = t.srcs[0]
    M = A.shape[1]
    sa = [0 if A.shape[0] == 1 else M * K]
    self.pb.op("g_bmm", a=self.value(A), b=wv, y=y, bshape=str(Bn), sa=_csv(sa), sb=str(K * N), m=M, n=N, k=K,
               sam=K, sak=1, sbk=N, sbn=1, rb=0)

  def finish(self, prog) -> None:
    """Bind / upload every weight this lowering declared into `prog`."""
    for b, tensor in self.binds:
      prog.bind(b, tensor)
    for b, arr in self.uploads:
      prog.upload(b, arr)


def _check_ops(order):
  bad = sorted({t.op for t in order if t.op not in SUPPORTED_OPS})
  if bad:
    raise NotImplementedError(f"aneforge_b200: graph ops with no B200 lowering: {bad}")


def _program(outs, compress, atol, block_size, device):
  """(Program, inputs ordered by creation, {id: port}, lowering) for a multi-output graph."""
  outs = [o if o.op != "input" else o * 1.0 for o in outs]
  order = topo_order(*outs)
  _check_ops(order)
  inputs = sorted((t for t in order if t.op == "input"), key=lambda t: t.attrs.get("idx", 0))
  if not inputs:
    raise ValueError("aneforge_b200.compile: graph has no inputs")
  names = {}
  for i, t in enumerate(order):
    t._name = f"t{i}"
    names[id(t)] = t._name
  pb = PlanBuilder()
  low = Lowering(pb, compress, atol, block_size, device, prefix="g")
  for t in inputs:
    port = pb.buf(t._name, 2 * t.size, "in")
    v = low._buf(f"{t._name}.v", 4 * t.size)
    pb.op("cast", src=port, dst=v, n=t.size, mode=0)
    low.set_value(t, v)
  low.lower(order, names)
  out_ports = {}
  for o in outs:
    if o._name in out_ports:
      continue
    port = pb.buf(o._name, 2 * o.size, "out")
    pb.op("cast", src=low.value(o), dst=port, n=o.size, mode=1)
    out_ports[o._name] = o.shape
  prog = R.Program.from_text(pb.text(), {t._name: t.shape for t in inputs}, out_ports, device)
  low.finish(prog)
  return prog, inputs, outs, low


def _policy(int8, compress):
  if compress is None and int8:
    return "int8"
  return compress


class Model:
  """One compiled graph with one output (the reference's `Model`, `aneforge/_compile.py:837-879`):
  call it with one array per graph input, in `input()` creation order; returns the fp32 output."""

  def __init__(self, prog, inputs, out: Tensor, n_ops: int, keep=None):
    self._prog = prog
    self._inputs = [(t._name, t.shape) for t in inputs]
    self._input_tensors = list(inputs)
    self._out_name, self._out_shape = out._name, out.shape
    self.n_ops = n_ops
    self._keep = keep                   # device weights the program reads

  @property
  def prog(self):
    return self._prog

  def __call__(self, *arrays):
    if len(arrays) != len(self._inputs):
      raise ValueError(f"expected {len(self._inputs)} input(s), got {len(arrays)}")
    feed = {}
    for (name, shape), a in zip(self._inputs, arrays):
      a = np.asarray(a)
      if tuple(a.shape) != tuple(shape):
        raise ValueError(f"input '{name}' shape {a.shape} != compiled {shape}")
      feed[name] = a.astype(F16)
    return self._prog.eval(feed)[self._out_name].astype(F32)

  def input_view(self, name: str | None = None):
    """Writable fp16 device view of an input port (torch CUDA tensor; the sole input by default)."""
    return self._prog.input_view(name or self._inputs[0][0])

  def output_view(self):
    """fp16 device view of the output port, valid after `execute()`."""
    return self._prog.output_view(self._out_name)

  def execute(self) -> None:
    self._prog.execute()

  def release(self) -> None:
    self._prog.release()
    self._keep = None


class MultiModel:
  """One compiled graph with several named outputs (the reference's `MultiModel`,
  `aneforge/_compile.py:987-1010`): `input_ports` / `output_ports` pair each graph tensor with its
  port name; `prog` exposes `set_input / execute / read_output / share_buffer`."""

  def __init__(self, prog, inputs, outputs, keep=None):
    self.prog = prog
    self.input_tensors = list(inputs)
    self.output_tensors = list(outputs)
    self.input_ports = [(t, t._name) for t in inputs]
    self.output_ports = [(t, t._name) for t in outputs]
    self._keep = keep

  def __call__(self, *arrays) -> dict:
    if len(arrays) != len(self.input_ports):
      raise ValueError(f"expected {len(self.input_ports)} input(s), got {len(arrays)}")
    feed = {name: np.asarray(a).astype(F16) for (_, name), a in zip(self.input_ports, arrays)}
    out = self.prog.eval(feed)
    return {name: out[name].astype(F32) for _, name in self.output_ports}

  def release(self) -> None:
    self.prog.release()
    self._keep = None


def compile(out: Tensor, int8: bool = False, build_dir=None, opt="routes", compress: str | None = None,  # noqa: A001
            compress_atol: float = 0.05, block_size: int = 32, validate: bool = False, target=None,
            device: int = 0) -> Model:
  """Lower `out` into one program of CUDA kernels (reference signature, `aneforge/_compile.py:1360`).
  `compress` / `compress_atol` / `block_size` / `int8` pick each weight's encoding exactly as the
  reference's policy does; `opt`, `build_dir`, `validate` and `target` select ANE compiler passes
  and have no effect here."""
  prog, inputs, outs, low = _program([out], _policy(int8, compress), compress_atol, block_size, device)
  return Model(prog, inputs, outs[0], low.n_ops, keep=low.binds)


def compile_multi(outs, build_dir=None, int8: bool = False, compress: str | None = None, compress_atol: float = 0.05,
                  block_size: int = 32, device: int = 0) -> MultiModel:
  """Lower a multi-output graph into one program with one fp16 port per output (reference
  signature, `aneforge/_compile.py:1013`)."""
  outs = list(outs)
  prog, inputs, outs, low = _program(outs, _policy(int8, compress), compress_atol, block_size, device)
  return MultiModel(prog, inputs, outs, keep=low.binds)
