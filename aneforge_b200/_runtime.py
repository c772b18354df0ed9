"""ctypes binding of libaf_cuda.so: the CUDA invoker that replaces the reference's e5rt dispatch
(`aneforge/_runtime.py`, whose `Program` class this module's `Program` mirrors: same methods, same
errors - KeyError for an unknown port, ValueError for a shape mismatch, RuntimeError("... rc=...")
for a native failure).

There is no CPU fallback: if the library is missing or no CUDA device is present, `lib()` raises.
Buffers handed out by `input_view` / `output_view` are device memory, wrapped as torch CUDA tensors.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Any

import numpy as np

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libaf_cuda.so"
_lib = None

c_void_p, c_size_t, c_int, c_float = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_float
c_char_p, c_uint64 = ctypes.c_char_p, ctypes.c_uint64

# (name, restype, argtypes): every symbol include/af_cuda.h declares
SIGNATURES = [
  ("af_last_error", c_char_p, []),
  ("af_abi_version", c_int, []),
  ("af_program_compile", c_void_p, [c_char_p, c_char_p, c_uint64, ctypes.POINTER(c_char_p), ctypes.POINTER(c_size_t),
                                    c_size_t, ctypes.POINTER(c_char_p), ctypes.POINTER(c_size_t), c_size_t]),
  ("af_program_compile_text", c_void_p, [c_char_p, c_char_p, c_uint64]),
  ("af_compile_check", c_int, [c_char_p, c_char_p, c_uint64, c_char_p]),
  ("af_program_set_input_fp16", c_int, [c_void_p, c_char_p, c_void_p, c_size_t]),
  ("af_program_get_output_fp16", c_int, [c_void_p, c_char_p, c_void_p, c_size_t]),
  ("af_program_set_input_bytes", c_int, [c_void_p, c_char_p, c_void_p, c_size_t]),
  ("af_program_get_output_bytes", c_int, [c_void_p, c_char_p, c_void_p, c_size_t]),
  ("af_program_input_buffer", c_int, [c_void_p, c_char_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_size_t)]),
  ("af_program_output_buffer", c_int, [c_void_p, c_char_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_size_t)]),
  ("af_program_buffer", c_int, [c_void_p, c_char_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_size_t)]),
  ("af_program_upload", c_int, [c_void_p, c_char_p, c_void_p, c_size_t, c_size_t]),
  ("af_program_download", c_int, [c_void_p, c_char_p, c_void_p, c_size_t]),
  ("af_program_bind_buffer", c_int, [c_void_p, c_char_p, c_void_p, c_size_t]),
  ("af_program_execute", c_int, [c_void_p]),
  ("af_program_execute_async", c_int, [c_void_p]),
  ("af_program_sync", c_int, [c_void_p]),
  ("af_program_stream", c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
  ("af_program_set_options", c_int, [c_void_p, c_int, c_int]),
  ("af_program_share_buffer", c_int, [c_void_p, c_size_t, c_char_p, c_size_t, c_char_p]),
  ("af_program_release", None, [c_void_p]),
  ("af_quantize_per_row_i8", c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
  ("af_quantize_g32_i4", c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
  ("af_gemv", c_int, [c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                      c_int, c_void_p]),
  ("af_lm_head_argmax_scratch", c_int, [c_int, c_int, c_int, c_int, ctypes.POINTER(c_size_t)]),
  ("af_lm_head_argmax", c_int, [c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p,
                                c_void_p, c_void_p, c_size_t, c_void_p]),
  ("af_pack_i8_tiles_bytes", c_size_t, [c_int, c_int]),
  ("af_pack_i8_tiles", c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
  ("af_gemv_tc_scratch_bytes", c_size_t, [c_int, c_int, c_int]),
  ("af_gemv_chain_scratch_bytes", c_size_t, [c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int), c_int, c_int]),
  ("af_gemv_tc_grid", c_int, [c_int, c_int, c_int, c_int, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
  ("af_gemv_tc", c_int, [c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                         c_void_p, c_size_t, c_void_p]),
  ("af_pack_i4_tiles_bytes", c_size_t, [c_int, c_int]),
  ("af_pack_i4_tiles", c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
  ("af_gemv_tc_i4", c_int, [c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                            c_void_p, c_size_t, c_void_p]),
  ("af_comm_unique_id", c_int, [c_void_p, c_size_t]),
  ("af_comm_init", c_int, [c_void_p, c_int, c_int, c_int, ctypes.POINTER(c_void_p)]),
  ("af_comm_destroy", None, [c_void_p]),
  ("af_comm_p2p_handle", c_int, [c_void_p, c_size_t, c_void_p, c_size_t]),
  ("af_comm_p2p_open", c_int, [c_void_p, c_void_p, c_size_t]),
  ("af_comm_p2p_disable", None, [c_void_p]),
  ("af_program_set_comm", c_int, [c_void_p, c_void_p]),
  ("af_moe_gate", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
  ("af_gemv_tc_expert", c_int, [c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                c_void_p, c_int, c_int, ctypes.c_longlong, c_int, c_void_p, c_int, c_void_p, c_size_t,
                                c_void_p]),
  ("af_gemm_tc", c_int, [c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                         c_int, c_void_p]),
  ("af_rmsnorm", c_int, [c_void_p, c_int, c_int, c_void_p, c_float, c_void_p, c_int, c_int, c_int, c_void_p]),
  ("af_attn_decode_scratch", c_int, [c_int, c_int, c_int, c_int, c_int, ctypes.POINTER(c_size_t)]),
  ("af_attn_decode", c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                             c_int, c_int, c_int, c_int, c_int, c_float, c_float, c_int, c_void_p, c_size_t, c_void_p,
                             c_void_p]),
  ("af_attn_decode_noalloc_max_bytes", c_size_t, []),
  ("af_attn_decode_noalloc", c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                     c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_float, c_int, c_void_p,
                                     c_void_p]),
]

W_I8, W_F16, W_I4G32 = 0, 1, 2
EPI_F32, EPI_F16, EPI_RESID, EPI_SWIGLU = 0, 1, 2, 3


def lib_path() -> Path:
  return Path(os.environ.get("AF_CUDA_LIB", str(_LIB_PATH)))


def load_library():
  """Load libaf_cuda.so and bind every exported symbol (no device needed)."""
  global _lib
  if _lib is not None:
    return _lib
  p = lib_path()
  if not p.exists():
    raise RuntimeError(f"aneforge_b200: {p} is not built; run `python -m aneforge_b200.build` "
                       "(there is no CPU fallback)")
  L = ctypes.CDLL(str(p))
  for name, res, args in SIGNATURES:
    fn = getattr(L, name)
    fn.restype = res
    fn.argtypes = args
  _lib = L
  return L


def lib():
  """The bound library, after checking a CUDA device is usable (no CPU fallback)."""
  import torch
  if not torch.cuda.is_available():
    raise RuntimeError("aneforge_b200 needs a CUDA device (B200); no CPU fallback exists")
  return load_library()


def last_error() -> str:
  L = load_library()
  return (L.af_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str) -> None:
  if rc != 0:
    raise RuntimeError(f"{what} failed rc={rc}: {last_error()}")


def _numel(shape) -> int:
  n = 1
  for d in shape:
    n *= int(d)
  return n


_DT_BYTES = {"fp16": 2, "int32": 4, "fp32": 4}
_TORCH_DT = {"fp16": "float16", "int32": "int32", "fp32": "float32"}


class Program:
  """A compiled CUDA program (the B200 counterpart of the reference's `aneforge._runtime.Program`).

  `inputs` / `outputs`: {port: shape}; `dtypes`: {port: "fp16" | "int32" | "fp32"} (fp16 default).
  """

  def __init__(self, handle: int, inputs: dict, outputs: dict, device: int = 0, dtypes: dict | None = None):
    self._handle = handle
    self._inputs = {k: tuple(v) for k, v in inputs.items()}
    self._outputs = {k: tuple(v) for k, v in outputs.items()}
    self._dtypes = dict(dtypes or {})
    self.device = device
    self._L = load_library()

  # -- construction
  @classmethod
  def from_text(cls, plan_text: str, inputs: dict, outputs: dict, device: int = 0, dtypes=None,
                weights_dir: str | None = None) -> "Program":
    L = lib()
    h = L.af_program_compile_text(plan_text.encode(), (weights_dir or ".").encode(), c_uint64(1 << device))
    if not h:
      raise RuntimeError(f"af_program_compile_text failed: {last_error()}")
    return cls(h, inputs, outputs, device, dtypes)

  @classmethod
  def from_dir(cls, plan_dir: str, inputs: dict, outputs: dict, device: int = 0, dtypes=None) -> "Program":
    L = lib()
    dtypes = dict(dtypes or {})
    in_names, out_names = list(inputs), list(outputs)
    in_n = (c_char_p * len(in_names))(*[n.encode() for n in in_names])
    in_s = (c_size_t * len(in_names))(*[_numel(inputs[n]) * _DT_BYTES[dtypes.get(n, "fp16")] for n in in_names])
    out_n = (c_char_p * len(out_names))(*[n.encode() for n in out_names])
    out_s = (c_size_t * len(out_names))(*[_numel(outputs[n]) * _DT_BYTES[dtypes.get(n, "fp16")] for n in out_names])
    h = L.af_program_compile(str(plan_dir).encode(), str(plan_dir).encode(), c_uint64(1 << device),
                             in_n, in_s, c_size_t(len(in_names)), out_n, out_s, c_size_t(len(out_names)))
    if not h:
      raise RuntimeError(f"af_program_compile failed (plan={plan_dir}): {last_error()}")
    return cls(h, inputs, outputs, device, dtypes)

  # -- ports
  def _np_dtype(self, name):
    return {"fp16": np.float16, "int32": np.int32, "fp32": np.float32}[self._dtypes.get(name, "fp16")]

  def set_input(self, name: str, arr) -> None:
    """Write one input/state port (host -> device copy, synchronous)."""
    if name not in self._inputs:
      raise KeyError(f"unknown input port: {name!r}")
    a = np.asarray(arr)
    if tuple(a.shape) != self._inputs[name]:
      raise ValueError(f"input {name!r}: expected {self._inputs[name]}, got {tuple(a.shape)}")
    a = np.ascontiguousarray(a.astype(self._np_dtype(name), copy=False))
    rc = self._L.af_program_set_input_bytes(self._handle, name.encode(), a.ctypes.data, a.nbytes)
    if rc != 0:
      raise RuntimeError(f"set_input({name}) failed rc={rc}: {last_error()}")

  def read_output(self, name: str) -> np.ndarray:
    """Read one output port into a fresh host array."""
    if name not in self._outputs:
      raise KeyError(f"unknown output port: {name!r}")
    out = np.empty(self._outputs[name], self._np_dtype(name))
    rc = self._L.af_program_get_output_bytes(self._handle, name.encode(), out.ctypes.data, out.nbytes)
    if rc != 0:
      raise RuntimeError(f"get_output({name}) failed rc={rc}: {last_error()}")
    return out

  def eval(self, inputs: dict) -> dict:
    for name, arr in inputs.items():
      self.set_input(name, arr)
    self.execute()
    return {name: self.read_output(name) for name in self._outputs}

  def execute(self) -> None:
    rc = self._L.af_program_execute(self._handle)
    if rc != 0:
      raise RuntimeError(f"execute failed rc={rc}: {last_error()}")

  def execute_async(self) -> None:
    rc = self._L.af_program_execute_async(self._handle)
    if rc != 0:
      raise RuntimeError(f"execute_async failed rc={rc}: {last_error()}")

  def sync(self) -> None:
    rc = self._L.af_program_sync(self._handle)
    if rc != 0:
      raise RuntimeError(f"sync failed rc={rc}: {last_error()}")

  def share_buffer(self, src_op_idx: int, src_out_port: str, dst_op_idx: int, dst_in_port: str) -> None:
    """Alias input `dst_in_port` onto output `src_out_port` (resident state across executes)."""
    rc = self._L.af_program_share_buffer(self._handle, c_size_t(src_op_idx), src_out_port.encode(),
                                         c_size_t(dst_op_idx), dst_in_port.encode())
    if rc != 0:
      raise RuntimeError(f"share_buffer(op{src_op_idx}.{src_out_port}->op{dst_op_idx}.{dst_in_port}) "
                         f"failed rc={rc}: {last_error()}")

  # -- device buffers
  def buffer_ptr(self, name: str) -> tuple[int, int]:
    ptr, nbytes = c_void_p(), c_size_t()
    rc = self._L.af_program_buffer(self._handle, name.encode(), ctypes.byref(ptr), ctypes.byref(nbytes))
    if rc != 0 or not ptr.value:
      raise RuntimeError(f"no device buffer {name!r} (rc={rc}): {last_error()}")
    return ptr.value, nbytes.value

  def tensor(self, name: str, shape, dtype: str = "fp16"):
    """A torch CUDA tensor viewing a program buffer (zero copy)."""
    import torch
    ptr, nbytes = self.buffer_ptr(name)
    n = _numel(shape)
    tdt = getattr(torch, _TORCH_DT[dtype])
    if n * _DT_BYTES[dtype] > nbytes:
      raise RuntimeError(f"buffer {name!r} too small for {shape} {dtype}")
    return _wrap_device_ptr(ptr, n, tdt, self.device).view(*shape)

  def input_view(self, name: str):
    if name not in self._inputs:
      raise KeyError(f"unknown input port: {name!r}")
    return self.tensor(name, self._inputs[name], self._dtypes.get(name, "fp16"))

  def output_view(self, name: str):
    if name not in self._outputs:
      raise KeyError(f"unknown output port: {name!r}")
    return self.tensor(name, self._outputs[name], self._dtypes.get(name, "fp16"))

  def upload(self, name: str, arr: np.ndarray, offset: int = 0) -> None:
    a = np.ascontiguousarray(arr)
    rc = self._L.af_program_upload(self._handle, name.encode(), a.ctypes.data, a.nbytes, offset)
    if rc != 0:
      raise RuntimeError(f"upload({name}) failed rc={rc}: {last_error()}")

  def download(self, name: str, shape, dtype=np.float16) -> np.ndarray:
    out = np.empty(shape, dtype)
    rc = self._L.af_program_download(self._handle, name.encode(), out.ctypes.data, out.nbytes)
    if rc != 0:
      raise RuntimeError(f"download({name}) failed rc={rc}: {last_error()}")
    return out

  def bind(self, name: str, tensor) -> None:
    """Use a caller-owned CUDA tensor as the program buffer `name` (the caller keeps it alive)."""
    rc = self._L.af_program_bind_buffer(self._handle, name.encode(), c_void_p(tensor.data_ptr()),
                                        c_size_t(tensor.numel() * tensor.element_size()))
    if rc != 0:
      raise RuntimeError(f"bind({name}) failed rc={rc}: {last_error()}")

  def stream(self) -> int:
    s = c_void_p()
    check(self._L.af_program_stream(self._handle, ctypes.byref(s)), "af_program_stream")
    return s.value or 0

  def set_comm(self, comm) -> None:
    """Attach a tensor-parallel communicator (before the first execute; it must outlive the program)."""
    rc = self._L.af_program_set_comm(self._handle, comm)
    if rc != 0:
      raise RuntimeError(f"set_comm failed rc={rc}: {last_error()}")

  def set_options(self, use_graph: bool = True, use_pdl: bool = True) -> None:
    check(self._L.af_program_set_options(self._handle, int(use_graph), int(use_pdl)), "set_options")

  def release(self) -> None:
    if self._handle:
      self._L.af_program_release(self._handle)
      self._handle = 0

  def __enter__(self) -> "Program":
    return self

  def __exit__(self, *args: Any) -> None:
    self.release()

  def __del__(self) -> None:
    try:
      self.release()
    except Exception:
      pass


def _wrap_device_ptr(ptr: int, numel: int, dtype, device: int):
  """Zero-copy torch CUDA tensor over raw device memory owned elsewhere."""
  import torch

  class _CudaArray:
    def __init__(self):
      self.__cuda_array_interface__ = {
        "shape": (numel,), "typestr": _TYPESTR[dtype], "data": (ptr, False), "version": 3, "strides": None}

  with torch.cuda.device(device):
    return torch.as_tensor(_CudaArray(), device=f"cuda:{device}")


def _typestr():
  import torch
  return {torch.float16: "<f2", torch.float32: "<f4", torch.int32: "<i4", torch.int8: "|i1", torch.uint8: "|u1"}


class _LazyTypestr(dict):
  def __missing__(self, k):
    self.update(_typestr())
    return dict.__getitem__(self, k)


_TYPESTR = _LazyTypestr()
