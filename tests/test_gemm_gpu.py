"""Prefill GEMM on tcgen05 (fp16 operands from the packed int8 / int4 tiles, fp32 accumulation in
tensor memory) against numpy on the same dequantised weights: int8 exact per-row scales applied to the
fp32 sums (rel-err 1e-4 bar), int4 dequantised to fp16 code * scale before the MMA (the fp16 rounding of
each dequantised weight bounds the error: 2^-10 relative per weight, bar 2e-3)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from oracle import quant as Q                                                    # noqa: E402

F16, F32 = np.float16, np.float32


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
  if not torch.cuda.is_available():
    pytest.skip("no CUDA device")


def cuda(a):
  return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _weights(fmt, N, Kd, rng):
  from aneforge_b200 import kernels as K, _runtime as R
  W = (rng.standard_normal((N, Kd)) * 0.02).astype(F16)
  if fmt == "int8":
    q, s = Q.quantize_per_row(W)
    return K.pack_i8_tiles(cuda(q)), cuda(s), q.astype(F32) * s.astype(F32)[:, None], R.W_I8
  p, s = Q.quantize_g32_int4(W)
  nib = np.stack([p & 15, p >> 4], -1).reshape(N, Kd).astype(F32) - 8
  deq = (nib.reshape(N, -1, 32) * s.astype(F32)[:, :, None]).reshape(N, Kd).astype(F16).astype(F32)
  return K.pack_i4_tiles(cuda(p), cuda(s), N, Kd), None, deq, R.W_I4G32


@pytest.mark.parametrize("fmt", ["int8", "int4"])
@pytest.mark.parametrize("M,N,Kd", [(128, 256, 64), (7, 256, 64), (300, 640, 2048), (512, 6144, 4096), (129, 4096, 14336),
                                    (64, 512, 96)])
def test_gemm_tc_matches_numpy(fmt, M, N, Kd):
  from aneforge_b200 import kernels as K, _runtime as R
  rng = np.random.default_rng(M + N + Kd)
  tiles, scales, deq, wf = _weights(fmt, N, Kd, rng)
  x = rng.standard_normal((M, Kd)).astype(F16)
  bias = (rng.standard_normal(N) * 0.1).astype(F16)
  ref = x.astype(F32) @ deq.T + bias.astype(F32)
  y = K.gemm_tc(cuda(x), tiles, scales, N, Kd, wf=wf, bias=cuda(bias)).cpu().numpy()
  tol = 1e-4 if fmt == "int8" else 2e-3
  assert np.abs(y - ref).max() <= tol * np.abs(ref).max() + 1e-4, np.abs(y - ref).max()
  y0 = rng.standard_normal((M, N)).astype(F32)
  yr = cuda(y0.copy())
  K.gemm_tc(cuda(x), tiles, scales, N, Kd, wf=wf, bias=cuda(bias), epi=R.EPI_RESID, y=yr)
  assert np.abs(yr.cpu().numpy() - (y0 + ref)).max() <= tol * np.abs(y0 + ref).max() + 1e-4


@pytest.mark.parametrize("fmt", ["int8", "int4"])
def test_gemm_tc_swiglu_matches_gemv(fmt):
  """The SWIGLU epilogue over gate/up rows interleaved in blocks of 8, against the decode GEMV."""
  from aneforge_b200 import kernels as K, _runtime as R
  from aneforge_b200.layout import interleave_blocks, SWIGLU_HALF_TC
  rng = np.random.default_rng(9)
  F, Kd, M = 384, 1024, 200
  Wg = (rng.standard_normal((F, Kd)) * 0.05).astype(F16)
  Wu = (rng.standard_normal((F, Kd)) * 0.05).astype(F16)
  x = rng.standard_normal((M, Kd)).astype(F16)
  if fmt == "int8":
    (qg, sg), (qu, su) = Q.quantize_per_row(Wg), Q.quantize_per_row(Wu)
    tiles = K.pack_i8_tiles(cuda(interleave_blocks(qg, qu, SWIGLU_HALF_TC)))
    sc = cuda(interleave_blocks(sg, su, SWIGLU_HALF_TC))
    y = K.gemm_tc(cuda(x), tiles, sc, 2 * F, Kd, wf=R.W_I8, epi=R.EPI_SWIGLU).cpu().numpy().astype(F32)
    ref = K.gemv_tc(cuda(x), tiles, sc, 2 * F, Kd, epi=R.EPI_SWIGLU).cpu().numpy().astype(F32)
    assert np.abs(y - ref).max() <= 2e-3 * np.abs(ref).max()
  else:
    (pg, sg), (pu, su) = Q.quantize_g32_int4(Wg), Q.quantize_g32_int4(Wu)
    pp, sp = interleave_blocks(pg, pu, SWIGLU_HALF_TC), interleave_blocks(sg, su, SWIGLU_HALF_TC)
    tiles = K.pack_i4_tiles(cuda(pp), cuda(sp), 2 * F, Kd)
    y = K.gemm_tc(cuda(x), tiles, None, 2 * F, Kd, wf=R.W_I4G32, epi=R.EPI_SWIGLU).cpu().numpy().astype(F32)
    ref = K.gemv_tc_i4(cuda(x), tiles, 2 * F, Kd, epi=R.EPI_SWIGLU).cpu().numpy().astype(F32)
    assert np.abs(y - ref).max() <= 1e-2 * np.abs(ref).max()
