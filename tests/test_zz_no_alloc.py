"""af_attn_decode_noalloc (split-K decode attention with the library's built-in scratch) against
af_attn_decode with caller scratch, through the C ABI.

The entry point allocates nothing; the test allocates its own inputs with torch. Two calls in a row
must each match the caller-scratch entry point (the tickets left by the first call are cleared
before the second), and a shape larger than the built-in scratch is rejected before any launch.
Tolerance: the attention bar of the kernel tests (max abs diff <= 2^-9 * max|ref| + 1e-3); both
entry points run the same kernel with the same split, so the outputs are in practice identical.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from oracle import model as OM                                       # noqa: E402

F16, F32 = np.float16, np.float32


@pytest.fixture(scope="module")
def K():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")
  from aneforge_b200 import kernels
  return kernels


def cuda(a):
  return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _case(dh, H, KV, NB, M, seed):
  rng = np.random.default_rng(seed)
  pos = rng.integers(0, M, NB).astype(np.int32)
  Kc = rng.standard_normal((NB, KV, M, dh), dtype=F32).astype(F16)
  Vc = rng.standard_normal((NB, KV, M, dh), dtype=F32).astype(F16)
  qkv = rng.standard_normal((NB, (H + 2 * KV) * dh), dtype=F32)
  cos, sin = OM.rope_tables(M, dh, 10000.0)
  return pos, Kc, Vc, qkv, cos, sin


# n_split 37 and 24 merge through the library's array (the second with several sequences and GQA
# 4:1, so the tickets of many (sequence, kv head) pairs must be cleared between the two calls); 9 and
# 16 merge inside a thread-block cluster and touch none of it; the 16-sequence, 16-split cluster
# shape would need 4.3 MB of partials through scratch, more than the array holds, and must still run
@pytest.mark.parametrize("dh,H,KV,NB,n_split", [(128, 32, 8, 1, 37), (128, 32, 8, 4, 24), (128, 32, 8, 4, 9),
                                                (64, 16, 2, 3, 16), (128, 16, 4, 2, 1), (128, 32, 8, 16, 16)])
def test_noalloc_matches_caller_scratch_twice(K, dh, H, KV, NB, n_split):
  M = 1200
  pos, Kc, Vc, qkv, cos, sin = _case(dh, H, KV, NB, M, dh + H + NB)
  scale = float(np.float16(1 / np.sqrt(dh)))
  kv_c = 127 * float(np.float16(1 / 127))
  q, p, c, s = cuda(qkv), cuda(pos), cuda(cos), cuda(sin)
  kr, vr = cuda(Kc), cuda(Vc)
  ref = K.attn_decode(q, kr, vr, p, c, s, H, KV, dh, scale, kv_c, H != KV, n_split).cpu().numpy().astype(F32)
  kn, vn = cuda(Kc), cuda(Vc)
  for call in range(2):
    rc, out = K.attn_decode_noalloc(q, kn, vn, p, c, s, H, KV, dh, scale, kv_c, H != KV, n_split)
    assert rc == 0, K.R.last_error()
    got = out.cpu().numpy().astype(F32)
    d = np.abs(got - ref)
    assert d.max() <= 2 ** -9 * np.abs(ref).max() + 1e-3, (call, d.max())
  assert torch.equal(kn, kr) and torch.equal(vn, vr)          # same cache slot written by both


def test_noalloc_rejects_shapes_beyond_builtin_scratch(K):
  """16 sequences x 8 kv heads x 64 splits x 4 q heads x 130 floats = 17 MB > 2 MiB: refused up front,
  nothing launched (the inputs are never read, so tiny placeholders suffice)."""
  R = K.R
  cap = R.lib().af_attn_decode_noalloc_max_bytes()
  assert cap == 2 << 20
  dummy = torch.zeros((1, 1, 1, 1), device="cuda")
  rc, _ = K.attn_decode_noalloc(torch.zeros((16, 48 * 128), device="cuda"), dummy, dummy, dummy, dummy, dummy,
                                32, 8, 128, 0.088, 1.0, True, 64)
  assert rc != 0
  assert "built-in maximum" in R.last_error()


def test_noalloc_on_every_visible_device(K):
  """Kernel attributes and the array's address are per device: a 16-split cluster call (over 48 KB
  of dynamic shared memory) on each visible GPU in turn matches the caller-scratch entry point."""
  n = torch.cuda.device_count()
  dh, H, KV, NB, n_split, M = 128, 64, 8, 1, 16, 1100
  pos, Kc, Vc, qkv, cos, sin = _case(dh, H, KV, NB, M, 5)
  scale = float(np.float16(1 / np.sqrt(dh)))
  kv_c = 127 * float(np.float16(1 / 127))
  for d in range(n):
    with torch.cuda.device(d):
      dev = f"cuda:{d}"
      t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
      q, p, c, s = t(qkv), t(pos), t(cos), t(sin)
      ref = K.attn_decode(q, t(Kc), t(Vc), p, c, s, H, KV, dh, scale, kv_c, True, n_split).cpu().numpy().astype(F32)
      rc, out = K.attn_decode_noalloc(q, t(Kc), t(Vc), p, c, s, H, KV, dh, scale, kv_c, True, n_split)
      assert rc == 0, K.R.last_error()
      got = out.cpu().numpy().astype(F32)
      assert np.abs(got - ref).max() <= 2 ** -9 * np.abs(ref).max() + 1e-3, d
