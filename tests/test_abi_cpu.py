"""CPU checks of the C-ABI boundary and the host-side logic (no kernel is launched).

* libaf_cuda.so loads and exports every function include/af_cuda.h declares, and the ctypes
  signature table of the Python runtime names exactly those functions.
* The package's weight-encoding policy (`aneforge_b200._blob`, the device-side restatement of the
  reference's `_compile.py:112-188`) picks the same encoding and the same dequantized matrix as the
  reference did on the golden inputs.
* RoPE tables, RMSNorm constants and the gate/up interleave are the ones the oracle uses.
"""
import ctypes
import os
import re

import numpy as np
import pytest

from oracle import quant as Q
from tests._golden import load

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
F16, F32 = np.float16, np.float32


def declared_functions():
  src = open(os.path.join(ROOT, "include", "af_cuda.h")).read()
  src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
  return sorted(set(re.findall(r"\b(af_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
  from aneforge_b200 import build
  return ctypes.CDLL(str(build.build()))


def test_library_exports_every_declared_symbol(lib):
  names = declared_functions()
  assert len(names) >= 30
  missing = [n for n in names if not hasattr(lib, n)]
  assert not missing, missing


def test_runtime_signature_table_matches_header():
  from aneforge_b200 import _runtime as R
  table = sorted(n for n, _, _ in R.SIGNATURES)
  assert table == declared_functions()


def test_abi_version_and_error_channel(lib):
  lib.af_abi_version.restype = ctypes.c_int
  assert lib.af_abi_version() == 1
  lib.af_last_error.restype = ctypes.c_char_p
  lib.af_attn_decode_noalloc_max_bytes.restype = ctypes.c_size_t
  assert lib.af_attn_decode_noalloc_max_bytes() == 2 << 20


def test_pack_tile_and_scratch_sizes(lib):
  """Host-side size helpers: fragment tiles are [ceil(n/64)][ceil(k/32)][4][512 B]."""
  lib.af_pack_i8_tiles_bytes.restype = ctypes.c_size_t
  for n, k in ((16, 32), (37, 64), (4096, 4096), (28672, 4096)):
    assert lib.af_pack_i8_tiles_bytes(n, k) == (-(-n // 64)) * (-(-k // 32)) * 4 * 512


@pytest.mark.parametrize("name", ["W", "Ws", "Mx", "Wl"])
@pytest.mark.parametrize("mode", ["None", "int8", "int4", "blockwise", "sparse", "auto"])
def test_package_encoding_policy_matches_reference(name, mode):
  from aneforge_b200 import _blob
  qz = load("quant.npz")
  M = {"W": qz["W"], "Ws": qz["Ws"], "Wl": qz["Wl"], "Mx": np.repeat(np.eye(4, dtype=F16), 2, axis=0)}[name]
  comp = None if mode == "None" else mode
  kind, _ = _blob.decide(M, comp)
  ref_kind = str(qz[f"enc_{name}_{mode}_kind"])
  assert {"lut4": "lut4", "int8": "int8", "fp16": "fp16", "blockwise": "blockwise",
          "sparse": "sparse"}.get(kind, kind) == ref_kind
  np.testing.assert_array_equal(_blob.dense_of(M, comp).astype(F32), qz[f"enc_{name}_{mode}_deq"])


@pytest.mark.parametrize("mode", ["int4", "blockwise", "sparse"])
def test_decoded_encodings_match_oracle_values(mode):
  """Encodings with no packed device format (an accepted LUT4, blockwise, sparse) run as fp16
  matrices of their decoded values: those values must be the oracle's dequantized matrix
  (exactly for LUT4 and sparse; blockwise within one fp16 rounding)."""
  from aneforge_b200 import weights as W
  from oracle.quant import encode_weight
  rng = np.random.default_rng(5)
  if mode == "int4":
    lut = np.linspace(-0.05, 0.05, 16).astype(np.float16)
    A = lut[rng.integers(0, 16, (48, 96))].astype(np.float32)
  elif mode == "sparse":
    A = rng.normal(0, 0.02, (48, 96)).astype(np.float32) * (rng.random((48, 96)) < 0.3)
  else:
    A = rng.normal(0, 0.02, (48, 96)).astype(np.float32)
  kind, dense = W._decoded_fp16(A, mode, 0.05, 32)
  ref = encode_weight(A, mode, 0.05, 32)
  assert kind == ref.kind == {"int4": "lut4", "blockwise": "blockwise", "sparse": "sparse"}[mode]
  if mode == "blockwise":
    assert np.allclose(dense, ref.deq, rtol=2 ** -10, atol=0)
  else:
    assert np.array_equal(dense, ref.deq) and np.array_equal(dense.astype(np.float16).astype(np.float32), dense)
  # a near-Gaussian weight under "int4" is rejected by the LUT gate and stays per-row int8
  g = rng.normal(0, 0.02, (48, 96)).astype(np.float32)
  assert W._decoded_fp16(g, "int4", 0.05, 32) == ("int8", None)


def test_gqa_expand_factor():
  from aneforge_b200 import _blob
  assert _blob.gqa_expand_factor(8, 4, "int8") == 127 * float(np.float16(1 / 127))
  assert _blob.gqa_expand_factor(8, 4, None) == 1.0
  assert _blob.gqa_expand_factor(8, 1, "int8") == 1.0


@pytest.mark.parametrize("M,dh,base", [(64, 128, 500000.0), (300, 64, 10000.0)])
def test_rope_tables_match_oracle(M, dh, base):
  from aneforge_b200.llm import rope_tables
  from oracle.model import rope_tables as orope
  c, s = rope_tables(M, dh, base)
  oc, os_ = orope(M, dh, base)
  assert np.array_equal(c.view(np.uint16), oc.view(np.uint16))
  assert np.array_equal(s.view(np.uint16), os_.view(np.uint16))


def test_swiglu_interleave_layout():
  torch = pytest.importorskip("torch")
  from aneforge_b200 import layout
  g = torch.arange(32).reshape(16, 2)
  u = 100 + torch.arange(32).reshape(16, 2)
  w = layout.interleave_blocks(g, u, 8)
  assert w.shape == (32, 2)
  assert torch.equal(w[:8], g[:8]) and torch.equal(w[8:16], u[:8])
  assert torch.equal(w[16:24], g[8:]) and torch.equal(w[24:], u[8:])


def test_sparse_device_encoding_round_trips():
  """The sparse projection's device payload (keep-mask words, kept values, row offsets) decodes to
  the fused fp16 matrix - gate/up interleaved in blocks of 4 rows - with the reference's LSB-first
  bit order (`aneforge/_blob.py:59-64`)."""
  import torch
  from aneforge_b200 import layout
  from aneforge_b200.weights import _encode_sparse
  rng = np.random.default_rng(0)
  g, u = (np.where(rng.random((16, 96)) < 0.7, 0, rng.standard_normal((16, 96))).astype(np.float16) for _ in range(2))
  for mats, swiglu in (([g], False), ([g, u], True), ([g, u], False)):
    mask, vals, ro = _encode_sparse(mats, torch.device("cpu"), swiglu)
    W = layout.interleave_blocks(g, u, layout.SWIGLU_HALF) if swiglu else np.concatenate(mats, 0)
    m, v, r = mask.numpy().view(np.uint32), vals.numpy(), ro.numpy()
    D = np.zeros_like(W)
    for i in range(W.shape[0]):
      cols = [c for c in range(W.shape[1]) if (m[i, c // 32] >> (c % 32)) & 1]
      D[i, cols] = v[r[i]:r[i + 1]]
    np.testing.assert_array_equal(D, W)
    ref_mask, ref_vals = Q.sparsify(W)                   # the oracle's restatement of the encoder
    np.testing.assert_array_equal(np.frombuffer(mask.numpy().tobytes(), np.uint8), np.asarray(ref_mask, np.uint8))
    np.testing.assert_array_equal(v[:r[-1]], np.asarray(ref_vals, np.float16))


@pytest.mark.parametrize("compress", ["blockwise", "sparse"])
def test_packed_projection_cache_round_trips(tmp_path, monkeypatch, compress):
  """The content-addressed packed-projection cache: a second encode of the same weights loads the
  stored payload (no host encoding runs), equal tensors; other weights or settings miss."""
  import torch
  from aneforge_b200 import weights as Wm
  rng = np.random.default_rng(1)
  g = (rng.standard_normal((64, 128)) * 0.05).astype(np.float16)
  u = (rng.standard_normal((64, 128)) * 0.05).astype(np.float16)
  if compress == "sparse":
    g, u = (np.where(rng.random(x.shape) < 0.7, 0, x).astype(np.float16) for x in (g, u))
  Wm.set_weight_cache(tmp_path)
  try:
    cpu = torch.device("cpu")
    a = Wm.encode_linear([g, u], compress, cpu, swiglu=True)
    assert a.kind == compress and len(list(tmp_path.rglob("*.pt"))) == 1
    calls = []
    monkeypatch.setattr(Wm, "_encode_linear", lambda *args, **kw: calls.append(1))
    b = Wm.encode_linear([g, u], compress, cpu, swiglu=True)
    assert not calls
    assert (b.kind, b.N, b.K, b.group) == (a.kind, a.N, a.K, a.group)
    for k in ("w", "s", "bias", "rowoff"):
      ta, tb = getattr(a, k), getattr(b, k)
      assert (ta is None) == (tb is None)
      if ta is not None:
        assert torch.equal(ta, tb)
    monkeypatch.undo()
    Wm.set_weight_cache(tmp_path)
    Wm.encode_linear([g, u], compress, cpu, swiglu=False)   # another layout: a second entry
    assert len(list(tmp_path.rglob("*.pt"))) == 2
  finally:
    Wm.set_weight_cache(None)
