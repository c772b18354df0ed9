"""The drop-in boundary exactly as a reference maintainer binds it: the e5rt-shaped C ABI
(`aneforge/_lib/ane_e5rt_dispatch.mm:416-725`, bound at `aneforge/_runtime.py:61-92`), through a
ctypes table written the way a reference maintainer would add it on the reference side (not this
package's own binding).

Contract under test (the shim's documented behaviour, kept by libaf_cuda.so):
  * `af_program_compile(dir, cache, mask, in_names, in_bytes, n_in, out_names, out_bytes, n_out)`
    returns NULL when the plan is missing or a declared port is absent / larger than the plan's;
  * ports are zero-initialised;
  * `af_program_set_input_fp16` returns -1 for an unknown port or more bytes than the port holds;
  * `af_program_get_output_fp16` copies min(2 n, port bytes) and leaves the rest of `dst` alone;
  * `af_program_share_buffer` aliases an input onto an output (resident state across executes)
    before the first execute, and fails after it;
  * `af_program_input_buffer` / `output_buffer` hand out persistent (device) pointers;
  * `af_compile_check` returns 0 for a plan that validates, -1 otherwise (no device needed).
"""
import ctypes as C
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "aneforge_b200", "_lib", "libaf_cuda.so")

# x (32 fp16) is an input; s (32 fp16) is state; y = x; s_out = s + x. With s_out shared onto s,
# every execute adds x into the resident state.
PLAN = """AFPLAN 1
buf x 64 in
buf s 64 state
buf y 64 out
buf s_out 64 out
buf t 128 tmp
buf a 128 tmp
op cast src=x dst=t n=32 mode=0
op cast src=s dst=a n=32 mode=0
op add y=a x=t n=32
op cast src=a dst=s_out n=32 mode=1
op cast src=t dst=y n=32 mode=1
"""


def bind():
  """The reference-side ctypes table: one entry per e5rt-shaped call, the reference's argument types."""
  if not os.path.exists(LIB):
    pytest.skip("libaf_cuda.so is not built")
  lib = C.CDLL(LIB)
  lib.af_program_compile.restype = C.c_void_p
  lib.af_program_compile.argtypes = [C.c_char_p, C.c_char_p, C.c_uint64, C.POINTER(C.c_char_p), C.POINTER(C.c_size_t),
                                     C.c_size_t, C.POINTER(C.c_char_p), C.POINTER(C.c_size_t), C.c_size_t]
  for fn in ("af_program_set_input_fp16", "af_program_get_output_fp16"):
    getattr(lib, fn).restype = C.c_int
    getattr(lib, fn).argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_uint16), C.c_size_t]
  lib.af_program_execute.restype = C.c_int
  lib.af_program_execute.argtypes = [C.c_void_p]
  for fn in ("af_program_input_buffer", "af_program_output_buffer"):
    getattr(lib, fn).restype = C.c_int
    getattr(lib, fn).argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
  lib.af_program_release.restype = None
  lib.af_program_release.argtypes = [C.c_void_p]
  lib.af_program_share_buffer.restype = C.c_int
  lib.af_program_share_buffer.argtypes = [C.c_void_p, C.c_size_t, C.c_char_p, C.c_size_t, C.c_char_p]
  lib.af_compile_check.restype = C.c_int
  lib.af_compile_check.argtypes = [C.c_char_p, C.c_char_p, C.c_uint64, C.c_char_p]
  lib.af_last_error.restype = C.c_char_p
  lib.af_last_error.argtypes = []
  return lib


def plan_dir(tmp_path, text=PLAN, name="prog"):
  d = tmp_path / name
  d.mkdir()
  (d / "plan.txt").write_text(text)
  return str(d)


def names(*ns):
  return (C.c_char_p * len(ns))(*[n.encode() for n in ns])


def sizes(*bs):
  return (C.c_size_t * len(bs))(*bs)


def f16_ptr(a):
  return a.ctypes.data_as(C.POINTER(C.c_uint16))


# ------------------------------------------------------------------------------------ no device

def test_compile_check_validates_plans_without_a_device(tmp_path):
  lib = bind()
  assert lib.af_compile_check(plan_dir(tmp_path).encode(), b"", 1, None) == 0
  bad_ref = PLAN.replace("src=x dst=t", "src=nope dst=t")
  assert lib.af_compile_check(plan_dir(tmp_path, bad_ref, "bad_ref").encode(), b"", 1, None) == -1
  assert b"nope" in lib.af_last_error()
  too_small = PLAN.replace("buf t 128 tmp", "buf t 64 tmp")          # cast of 32 fp32 needs 128 bytes
  assert lib.af_compile_check(plan_dir(tmp_path, too_small, "small").encode(), b"", 1, None) == -1
  assert lib.af_compile_check(plan_dir(tmp_path, "AFPLAN 2\n", "ver").encode(), b"", 1, None) == -1
  assert lib.af_compile_check(str(tmp_path / "missing").encode(), b"", 1, None) == -1


def test_compile_fails_cleanly_without_plan(tmp_path):
  lib = bind()
  h = lib.af_program_compile(str(tmp_path / "missing").encode(), b"", 1, names("x"), sizes(64), 1, names("y"),
                             sizes(64), 1)
  assert not h
  assert b"plan.txt" in lib.af_last_error()


# ------------------------------------------------------------------------------------ on the GPU

@pytest.fixture
def gpu():
  torch = pytest.importorskip("torch")
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  return torch


@pytest.mark.gpu
def test_e5rt_shaped_program_lifecycle(tmp_path, gpu):
  lib = bind()
  d = plan_dir(tmp_path).encode()
  # a declared port larger than the plan's, or one the plan lacks: NULL
  assert not lib.af_program_compile(d, d, 1, names("x", "s"), sizes(64, 128), 2, names("y", "s_out"), sizes(64, 64), 2)
  assert not lib.af_program_compile(d, d, 1, names("x"), sizes(64), 1, names("nope"), sizes(8), 1)
  h = lib.af_program_compile(d, d, 1, names("x", "s"), sizes(64, 64), 2, names("y", "s_out"), sizes(64, 64), 2)
  assert h, lib.af_last_error()
  try:
    # zero-initialised ports
    got = np.full(32, 7, np.float16)
    assert lib.af_program_get_output_fp16(h, b"y", f16_ptr(got), 32) == 0
    assert np.all(got == 0)
    # persistent device pointers with the port sizes
    p, n = C.c_void_p(), C.c_size_t()
    assert lib.af_program_input_buffer(h, b"x", C.byref(p), C.byref(n)) == 0 and p.value and n.value == 64
    assert lib.af_program_output_buffer(h, b"s_out", C.byref(p), C.byref(n)) == 0 and p.value and n.value == 64
    assert lib.af_program_input_buffer(h, b"y", C.byref(p), C.byref(n)) == -1     # an output, not an input
    # set_input: oversize and unknown ports refused
    x = (np.arange(32) + 1).astype(np.float16)
    big = np.zeros(33, np.float16)
    assert lib.af_program_set_input_fp16(h, b"x", f16_ptr(big), 33) == -1
    assert lib.af_program_set_input_fp16(h, b"nope", f16_ptr(x), 32) == -1
    assert lib.af_program_set_input_fp16(h, b"x", f16_ptr(x), 32) == 0
    # resident state: s reads s_out's buffer from now on
    assert lib.af_program_share_buffer(h, 0, b"s_out", 0, b"s") == 0
    for _ in range(3):
      assert lib.af_program_execute(h) == 0
    y = np.zeros(32, np.float16)
    assert lib.af_program_get_output_fp16(h, b"y", f16_ptr(y), 32) == 0
    np.testing.assert_array_equal(y, x)
    s = np.zeros(32, np.float16)
    assert lib.af_program_get_output_fp16(h, b"s_out", f16_ptr(s), 32) == 0
    np.testing.assert_array_equal(s, 3 * x)
    # get_output copies min(2 n, port bytes): a short read, and an over-long one that stops at 64 B
    short = np.full(32, -1, np.float16)
    assert lib.af_program_get_output_fp16(h, b"y", f16_ptr(short), 10) == 0
    np.testing.assert_array_equal(short[:10], x[:10])
    assert np.all(short[10:] == -1)
    longer = np.full(40, -1, np.float16)
    assert lib.af_program_get_output_fp16(h, b"y", f16_ptr(longer), 40) == 0
    np.testing.assert_array_equal(longer[:32], x)
    assert np.all(longer[32:] == -1)
    # the program is finalised by its first execute: no more aliasing
    assert lib.af_program_share_buffer(h, 0, b"y", 0, b"x") == -1
    assert b"after the first execute" in lib.af_last_error()
  finally:
    lib.af_program_release(h)


@pytest.mark.gpu
def test_program_from_dir_python_mirror(tmp_path, gpu):
  """The package's `Program.from_dir` (the mirror of the reference's `_runtime.Program`) over the same
  plan: KeyError for unknown ports, ValueError for a shape mismatch, eval() returning every output."""
  from aneforge_b200._runtime import Program
  d = plan_dir(tmp_path)
  with Program.from_dir(d, {"x": (32,), "s": (32,)}, {"y": (32,), "s_out": (32,)}) as prog:
    with pytest.raises(KeyError):
      prog.set_input("nope", np.zeros(32, np.float16))
    with pytest.raises(ValueError):
      prog.set_input("x", np.zeros(31, np.float16))
    prog.share_buffer(0, "s_out", 0, "s")
    x = np.linspace(-2, 2, 32).astype(np.float16)
    out = prog.eval({"x": x})
    out = prog.eval({"x": x})
    np.testing.assert_array_equal(out["y"], x)
    np.testing.assert_array_equal(out["s_out"], (x.astype(np.float32) * 2).astype(np.float16))
    with pytest.raises(RuntimeError):
      prog.share_buffer(0, "y", 0, "x")
