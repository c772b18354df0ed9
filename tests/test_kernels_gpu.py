"""GPU parity of the individual sm_100a kernels against the CPU oracle, through the C ABI.

Bars: quantizer codes/scales bit-exact; GEMV outputs within rel-err 1e-2 (fp16) and cosine >= 0.999
(measured errors are far below: same fp32 math, different summation order); greedy argmax exact.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from oracle import quant as Q                                        # noqa: E402
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


def relerr(a, b):
  a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
  return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30))


def cosine(a, b):
  a = np.asarray(a, np.float64).ravel(); b = np.asarray(b, np.float64).ravel()
  return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


@pytest.mark.parametrize("shape", [(48, 96), (7, 33), (256, 4096), (4096, 4096)])
@pytest.mark.parametrize("src", ["f32", "f16"])
def test_quantize_per_row_bit_exact(K, shape, src):
  rng = np.random.default_rng(shape[0] * 7 + shape[1])
  W = (rng.standard_normal(shape, dtype=F32) * F32(0.02))
  W[0] = 0.0
  if shape[1] >= 8:
    W[1, :6] = [0.5, -0.5, 1.5, 2.5, -2.5, 127.0]
  W = W.astype(F16) if src == "f16" else W
  q, s = K.quantize_per_row_i8(cuda(W))
  qr, sr = Q.quantize_per_row(W)
  assert np.array_equal(q.cpu().numpy(), qr)
  assert np.array_equal(s.cpu().numpy().view(np.uint16), sr.view(np.uint16))


@pytest.mark.parametrize("shape", [(16, 128), (1024, 4096)])
def test_quantize_g32_int4_bit_exact(K, shape):
  rng = np.random.default_rng(3)
  W = (rng.standard_normal(shape, dtype=F32) * F32(0.02)).astype(F16)
  p, s = K.quantize_g32_i4(cuda(W))
  pr, sr = Q.quantize_g32_int4(W)
  assert np.array_equal(p.cpu().numpy(), pr)
  assert np.array_equal(s.cpu().numpy().view(np.uint16), sr.view(np.uint16))


def test_gemv_config1_int8_4096(K):
  """Benchmark config 1: W 4096x4096 ~ N(0,0.02) int8 per row, x 1x4096 ~ N(0,1) fp16, y fp16."""
  rng = np.random.default_rng(0)
  W = rng.standard_normal((4096, 4096), dtype=F32) * F32(0.02)
  x = rng.standard_normal((1, 4096), dtype=F32).astype(F16)
  q, s = K.quantize_per_row_i8(cuda(W))
  qr, sr = Q.quantize_per_row(W)
  assert np.array_equal(q.cpu().numpy(), qr)
  from aneforge_b200 import _runtime as R
  y = K.gemv(cuda(x), q, s, wf=R.W_I8, epi=R.EPI_F16).cpu().numpy()
  ref = OM.gemv_int8(x, qr, sr)
  assert relerr(y, ref) < 1e-2 and cosine(y, ref) > 0.999
  assert relerr(y, ref) < 2e-3


@pytest.mark.parametrize("NB", [1, 2, 3, 4, 5, 16])
@pytest.mark.parametrize("N,Kd", [(37, 64), (520, 2048), (300, 3584), (1024, 14336)])
@pytest.mark.parametrize("wfmt", ["i8", "f16", "i4"])
def test_gemv_formats_and_batches(K, NB, N, Kd, wfmt):
  from aneforge_b200 import _runtime as R
  rng = np.random.default_rng(NB * 1000 + N)
  W = (rng.standard_normal((N, Kd), dtype=F32) * F32(0.02)).astype(F16)
  x = rng.standard_normal((NB, Kd), dtype=F32).astype(F16)
  bias = (rng.standard_normal(N, dtype=F32) * F32(0.1)).astype(F16)
  xf = x.astype(F32)
  if wfmt == "i8":
    qr, sr = Q.quantize_per_row(W)
    w, s, wf = cuda(qr), cuda(sr), R.W_I8
    ref = (xf @ qr.astype(F32).T) * sr.astype(F32)
  elif wfmt == "f16":
    w, s, wf = cuda(W), None, R.W_F16
    ref = xf @ W.astype(F32).T
  else:
    if Kd % 32:
      pytest.skip("int4 needs K % 32 == 0")
    pr, sr = Q.quantize_g32_int4(W)
    w, s, wf = cuda(pr), cuda(sr), R.W_I4G32
    ref = xf @ Q.dequant_g32_int4(pr, sr).T
  ref = ref + bias.astype(F32)
  y = K.gemv(cuda(x), w, s, bias=cuda(bias), wf=wf, epi=R.EPI_F32).cpu().numpy()
  assert np.abs(y - ref).max() <= 1e-4 * np.abs(ref).max() + 1e-5
  # residual epilogue accumulates into y
  y0 = rng.standard_normal((NB, N), dtype=F32)
  yr = torch.from_numpy(y0.copy()).cuda()
  K.gemv(cuda(x), w, s, bias=cuda(bias), wf=wf, epi=R.EPI_RESID, y=yr)
  assert np.abs(yr.cpu().numpy() - (y0 + ref)).max() <= 1e-4 * np.abs(y0 + ref).max()


@pytest.mark.parametrize("NB", [1, 2, 4, 16])
def test_gemv_swiglu_epilogue(K, NB):
  from aneforge_b200 import _runtime as R
  from aneforge_b200.layout import pack_gate_up
  rng = np.random.default_rng(5)
  F, Kd = 96, 256
  Wg = (rng.standard_normal((F, Kd), dtype=F32) * F32(0.05)).astype(F16)
  Wu = (rng.standard_normal((F, Kd), dtype=F32) * F32(0.05)).astype(F16)
  x = rng.standard_normal((NB, Kd), dtype=F32).astype(F16)
  qg, sg = Q.quantize_per_row(Wg); qu, su = Q.quantize_per_row(Wu)
  qp, sp = pack_gate_up(qg, qu, sg, su)
  y = K.gemv(cuda(x), cuda(qp), cuda(sp), wf=R.W_I8, epi=R.EPI_SWIGLU).cpu().numpy().astype(F32)
  xf = x.astype(F32)
  g = (xf @ qg.astype(F32).T) * sg.astype(F32); u = (xf @ qu.astype(F32).T) * su.astype(F32)
  ref = OM.silu(g) * u
  assert relerr(y, ref) < 2e-3 and cosine(y, ref) > 0.9999


@pytest.mark.parametrize("NB", [1, 2, 3, 4, 6, 16])
def test_lm_head_argmax(K, NB):
  rng = np.random.default_rng(11)
  V, D = 1000, 256
  W = (rng.standard_normal((V, D), dtype=F32) * F32(0.02)).astype(F16)
  x = rng.standard_normal((NB, D), dtype=F32).astype(F16)
  W[17] = W[3]                                  # an exact tie: lowest index must win
  x[0] = 0
  x[0, :4] = 1.0
  tok, lg = K.lm_head_argmax(cuda(x), cuda(W))
  ref = x.astype(F32) @ W.astype(F32).T
  assert np.abs(lg.cpu().numpy() - ref).max() <= 1e-4 * np.abs(ref).max() + 1e-6
  assert list(tok.cpu().numpy()) == [int(np.argmax(lg.cpu().numpy()[b])) for b in range(NB)]
  assert list(tok.cpu().numpy()) == [int(np.argmax(ref[b])) for b in range(NB)]


def test_lm_head_argmax_large_vocab_and_pos_advance(K):
  rng = np.random.default_rng(12)
  V, D = 128256, 512
  W = (rng.standard_normal((V, D), dtype=F32) * F32(0.02)).astype(F16)
  x = rng.standard_normal((1, D), dtype=F32).astype(F16)
  pos = torch.tensor([41], dtype=torch.int32, device="cuda")
  tok, lg = K.lm_head_argmax(cuda(x), cuda(W), pos=pos)
  ref = x.astype(F32) @ W.astype(F32).T
  assert int(tok.item()) == int(np.argmax(lg.cpu().numpy()[0]))
  assert int(tok.item()) == int(np.argmax(ref[0]))
  assert int(pos.item()) == 42


@pytest.mark.parametrize("NB", [2, 9, 16])
def test_lm_head_argmax_batched_large_vocab(K, NB):
  """Batches of 2-16 rows take the tensor-core head (one pass over the weights): logits within fp32
  summation-order noise of the reference, tokens equal to the kernel's own logits' argmax and to the
  reference's wherever its top-2 gap is above that noise; positions advance."""
  rng = np.random.default_rng(13 + NB)
  V, D = 128256, 4096
  W = (rng.standard_normal((V, D), dtype=F32) * F32(0.02)).astype(F16)
  x = rng.standard_normal((NB, D), dtype=F32).astype(F16)
  pos = torch.tensor([3 + b % 4 for b in range(NB)], dtype=torch.int32, device="cuda")
  tok, lg = K.lm_head_argmax(cuda(x), cuda(W), pos=pos)
  ref = x.astype(F32) @ W.astype(F32).T
  lgn = lg.cpu().numpy()
  assert np.abs(lgn - ref).max() <= 1e-4 * np.abs(ref).max()
  t = tok.cpu().numpy()
  for b in range(NB):
    assert t[b] == int(np.argmax(lgn[b]))
    top2 = np.sort(ref[b])[-2:]
    if top2[1] - top2[0] > 1e-4 * np.abs(ref).max():
      assert t[b] == int(np.argmax(ref[b]))
    assert int(pos[b].item()) == 4 + b % 4


@pytest.mark.parametrize("D", [64, 2048, 4096])
@pytest.mark.parametrize("xf16", [False, True])
def test_rmsnorm_matches_reference_lowering(K, D, xf16):
  rng = np.random.default_rng(D)
  x = rng.standard_normal((3, D), dtype=F32)
  x[2] = 1e-6                                   # below the floor: max(||x||, floor) engages
  if xf16:
    x = x.astype(F16)
  gamma = (1 + 0.1 * rng.standard_normal(D)).astype(F32)
  g, floor = OM.rms_consts(gamma, 1e-5)
  y = K.rmsnorm(cuda(x), cuda(g), float(floor)).cpu().numpy()
  ref = OM.rms_norm(x.astype(F32), g, floor).astype(F16)
  diff = np.abs(y.astype(F32) - ref.astype(F32))
  assert diff.max() <= 2 ** -10 * np.abs(ref.astype(F32)).max()      # at most one fp16 ulp apart
  assert (y != ref).mean() < 0.01


def _attn_ref(qkv, Kc, Vc, pos, cos, sin, H, KV, dh, kv_c, expand):
  """Oracle decode attention for one sequence (device precision): returns fp16 [H*dh] + new k/v."""
  q = qkv[: H * dh].reshape(H, dh)
  k = qkv[H * dh:(H + KV) * dh].reshape(KV, dh)
  v = qkv[(H + KV) * dh:].reshape(KV, dh)
  q = OM.rope(q, cos[pos], sin[pos]); k = OM.rope(k, cos[pos], sin[pos])
  Kw = Kc[:, : pos + 1].astype(F32); Vw = Vc[:, : pos + 1].astype(F32)
  Kw[:, pos] = k.astype(F16); Vw[:, pos] = v.astype(F16)
  G = H // KV
  Kr = np.repeat(Kw, G, axis=0); Vr = np.repeat(Vw, G, axis=0)
  if expand:
    Kr = (F32(kv_c) * Kr).astype(F16).astype(F32); Vr = (F32(kv_c) * Vr).astype(F16).astype(F32)
  q16 = q.astype(F16).astype(F32)
  sc = np.einsum("hd,hkd->hk", q16, Kr) * F32(np.float16(1 / np.sqrt(dh)))
  p = OM.softmax(sc)
  return np.einsum("hk,hkd->hd", p, Vr).reshape(-1).astype(F16), k.astype(F16), v.astype(F16)


@pytest.mark.parametrize("dh,H,KV", [(128, 32, 8), (128, 16, 4), (64, 8, 8), (64, 8, 2), (64, 16, 2), (32, 4, 1),
                                     (16, 4, 2)])
@pytest.mark.parametrize("n_split", [1, 2, 4, 12, 16, 24])
@pytest.mark.parametrize("expand", [False, True])
def test_attn_decode(K, dh, H, KV, n_split, expand):
  rng = np.random.default_rng(dh + H + n_split)
  NB, M = 3, 300
  pos_h = np.array([257, 3, 16], np.int32)
  Kc = rng.standard_normal((NB, KV, M, dh), dtype=F32).astype(F16)
  Vc = rng.standard_normal((NB, KV, M, dh), dtype=F32).astype(F16)
  qkv = rng.standard_normal((NB, (H + 2 * KV) * dh), dtype=F32)
  cos, sin = OM.rope_tables(M, dh, 10000.0)
  kv_c = 127 * float(np.float16(1 / 127)) if expand else 1.0
  kc, vc = cuda(Kc), cuda(Vc)
  out = K.attn_decode(cuda(qkv), kc, vc, cuda(pos_h), cuda(cos), cuda(sin), H, KV, dh,
                      float(np.float16(1 / np.sqrt(dh))), kv_c, expand and H != KV, n_split).cpu().numpy()
  kc_h, vc_h = kc.cpu().numpy(), vc.cpu().numpy()
  for b in range(NB):
    ref, kn, vn = _attn_ref(qkv[b], Kc[b], Vc[b], int(pos_h[b]), cos, sin, H, KV, dh, kv_c, expand and H != KV)
    d = np.abs(out[b].astype(F32) - ref.astype(F32))
    assert d.max() <= 2 ** -9 * np.abs(ref.astype(F32)).max() + 1e-3, d.max()
    assert cosine(out[b], ref) > 0.99999
    p = int(pos_h[b])
    assert np.array_equal(kc_h[b][:, p], kn) and np.array_equal(vc_h[b][:, p], vn)
    untouched = np.ones(M, bool); untouched[p] = False
    assert np.array_equal(kc_h[b][:, untouched], Kc[b][:, untouched])


@pytest.mark.parametrize("NB", [1, 2, 3, 8, 9, 16, 40])
@pytest.mark.parametrize("N,Kd", [(16, 32), (37, 64), (520, 2048), (300, 3584), (6144, 4096), (4096, 14336)])
def test_gemv_tensor_core_int8(K, NB, N, Kd):
  from aneforge_b200 import _runtime as R
  rng = np.random.default_rng(NB * 7 + N)
  W = (rng.standard_normal((N, Kd), dtype=F32) * F32(0.02)).astype(F16)
  x = rng.standard_normal((NB, Kd), dtype=F32).astype(F16)
  bias = (rng.standard_normal(N, dtype=F32) * F32(0.1)).astype(F16)
  qr, sr = Q.quantize_per_row(W)
  tiles = K.pack_i8_tiles(cuda(qr))
  ref = (x.astype(F32) @ qr.astype(F32).T) * sr.astype(F32) + bias.astype(F32)
  y = K.gemv_tc(cuda(x), tiles, cuda(sr), N, Kd, bias=cuda(bias), epi=R.EPI_F32).cpu().numpy()
  assert np.abs(y - ref).max() <= 1e-4 * np.abs(ref).max() + 1e-5
  y0 = rng.standard_normal((NB, N), dtype=F32)
  yr = torch.from_numpy(y0.copy()).cuda()
  K.gemv_tc(cuda(x), tiles, cuda(sr), N, Kd, bias=cuda(bias), epi=R.EPI_RESID, y=yr)
  assert np.abs(yr.cpu().numpy() - (y0 + ref)).max() <= 1e-4 * np.abs(y0 + ref).max()
  y16 = K.gemv_tc(cuda(x), tiles, cuda(sr), N, Kd, bias=cuda(bias), epi=R.EPI_F16).cpu().numpy()
  assert np.abs(y16.astype(F32) - ref).max() <= 2 ** -10 * np.abs(ref).max() + 1e-4


@pytest.mark.parametrize("NB", [1, 5, 16])
def test_gemv_tensor_core_swiglu(K, NB):
  from aneforge_b200 import _runtime as R
  from aneforge_b200.layout import interleave_blocks, SWIGLU_HALF_TC
  rng = np.random.default_rng(15)
  F, Kd = 96, 512
  Wg = (rng.standard_normal((F, Kd), dtype=F32) * F32(0.05)).astype(F16)
  Wu = (rng.standard_normal((F, Kd), dtype=F32) * F32(0.05)).astype(F16)
  x = rng.standard_normal((NB, Kd), dtype=F32).astype(F16)
  qg, sg = Q.quantize_per_row(Wg); qu, su = Q.quantize_per_row(Wu)
  qp = interleave_blocks(qg, qu, SWIGLU_HALF_TC); sp = interleave_blocks(sg, su, SWIGLU_HALF_TC)
  y = K.gemv_tc(cuda(x), K.pack_i8_tiles(cuda(qp)), cuda(sp), 2 * F, Kd, epi=R.EPI_SWIGLU).cpu().numpy()
  xf = x.astype(F32)
  g = (xf @ qg.astype(F32).T) * sg.astype(F32); u = (xf @ qu.astype(F32).T) * su.astype(F32)
  ref = OM.silu(g) * u
  assert relerr(y.astype(F32), ref) < 2e-3 and cosine(y, ref) > 0.9999


def test_gemv_tensor_core_shared_scratch_across_shapes(K):
  """One scratch buffer serves GEMVs of different shapes back to back (as in a program)."""
  from aneforge_b200 import _runtime as R
  rng = np.random.default_rng(21)
  shapes = [(1536, 1024), (7168, 1024), (1024, 3584), (1536, 1024)]
  need = max(R.load_library().af_gemv_tc_scratch_bytes(n, k, 4) for n, k in shapes)
  scratch = torch.zeros((need,), dtype=torch.uint8, device="cuda")
  for N, Kd in shapes * 2:
    W = (rng.standard_normal((N, Kd), dtype=F32) * F32(0.02)).astype(F16)
    x = rng.standard_normal((4, Kd), dtype=F32).astype(F16)
    qr, sr = Q.quantize_per_row(W)
    y = K.gemv_tc(cuda(x), K.pack_i8_tiles(cuda(qr)), cuda(sr), N, Kd, scratch=scratch).cpu().numpy()
    ref = (x.astype(F32) @ qr.astype(F32).T) * sr.astype(F32)
    assert np.abs(y - ref).max() <= 1e-4 * np.abs(ref).max()


@pytest.mark.parametrize("NB", [1, 3, 8, 9, 16, 20])
@pytest.mark.parametrize("N,Kd", [(16, 32), (37, 64), (520, 2048), (300, 3584), (7392, 8192), (8192, 3712)])
def test_gemv_tensor_core_int4_g32(K, NB, N, Kd):
  """Group-32 int4 tiles: y = sum_g s_g (x . codes_g) against the oracle's fp32 dequantised matrix."""
  from aneforge_b200 import _runtime as R
  rng = np.random.default_rng(NB * 11 + N)
  W = (rng.standard_normal((N, Kd), dtype=F32) * F32(0.02)).astype(F16)
  x = rng.standard_normal((NB, Kd), dtype=F32).astype(F16)
  bias = (rng.standard_normal(N, dtype=F32) * F32(0.1)).astype(F16)
  p, s = Q.quantize_g32_int4(W)
  Wd = Q.dequant_g32_int4(p, s)
  tiles = K.pack_i4_tiles(cuda(p), cuda(s), N, Kd)
  assert tiles.numel() == (-(-N // 64)) * (Kd // 32) * 1152
  ref = x.astype(F32) @ Wd.T + bias.astype(F32)
  y = K.gemv_tc_i4(cuda(x), tiles, N, Kd, bias=cuda(bias), epi=R.EPI_F32).cpu().numpy()
  assert np.abs(y - ref).max() <= 1e-4 * np.abs(ref).max() + 1e-5
  y0 = rng.standard_normal((NB, N), dtype=F32)
  yr = torch.from_numpy(y0.copy()).cuda()
  K.gemv_tc_i4(cuda(x), tiles, N, Kd, bias=cuda(bias), epi=R.EPI_RESID, y=yr)
  assert np.abs(yr.cpu().numpy() - (y0 + ref)).max() <= 1e-4 * np.abs(y0 + ref).max()
  y16 = K.gemv_tc_i4(cuda(x), tiles, N, Kd, bias=cuda(bias), epi=R.EPI_F16).cpu().numpy()
  assert np.abs(y16.astype(F32) - ref).max() <= 2 ** -10 * np.abs(ref).max() + 1e-4


@pytest.mark.parametrize("NB", [1, 4, 16])
def test_gemv_tensor_core_int4_swiglu(K, NB):
  from aneforge_b200 import _runtime as R
  from aneforge_b200.layout import interleave_blocks, SWIGLU_HALF_TC
  rng = np.random.default_rng(25)
  F, Kd = 160, 1024
  Wg = (rng.standard_normal((F, Kd), dtype=F32) * F32(0.05)).astype(F16)
  Wu = (rng.standard_normal((F, Kd), dtype=F32) * F32(0.05)).astype(F16)
  x = rng.standard_normal((NB, Kd), dtype=F32).astype(F16)
  pg, sg = Q.quantize_g32_int4(Wg); pu, su = Q.quantize_g32_int4(Wu)
  pp = interleave_blocks(pg, pu, SWIGLU_HALF_TC); sp = interleave_blocks(sg, su, SWIGLU_HALF_TC)
  y = K.gemv_tc_i4(cuda(x), K.pack_i4_tiles(cuda(pp), cuda(sp), 2 * F, Kd), 2 * F, Kd,
                   epi=R.EPI_SWIGLU).cpu().numpy()
  xf = x.astype(F32)
  g = xf @ Q.dequant_g32_int4(pg, sg).T; u = xf @ Q.dequant_g32_int4(pu, su).T
  ref = OM.silu(g) * u
  assert relerr(y.astype(F32), ref) < 2e-3 and cosine(y, ref) > 0.9999
