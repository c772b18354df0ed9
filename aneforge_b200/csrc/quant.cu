// Device weight quantizers.
//
// quantize_rows_i8 restates the reference's per-output-row int8 encoder (aneforge/_blob.py:20-25)
// with the same IEEE-f32 operations so the codes and fp16 scales are bit-identical to numpy:
//   scale = max(max|row| / 127, 1e-8)   (f32 divide, round to nearest)
//   code  = clip(rint(w / scale), -127, 127)   (round half to even)
//   stored scale = f16(scale)            (round to nearest even)
// quantize_g32_i4 is this build's group-32 4-bit format (no reference counterpart): per 32 columns
// scale = max(max|g| / 7, 1e-8); code = clip(rint(w / scale), -7, 7) + 8, two codes per byte with
// element 2i in the low nibble; stored scale f16.
#include "af_common.cuh"
#include "af_kernels.h"

namespace af {

template <bool F16SRC>
AF_DEV float load_w(const void* src, size_t i) {
  if (F16SRC) return __half2float(reinterpret_cast<const __half*>(src)[i]);
  return reinterpret_cast<const float*>(src)[i];
}

template <bool F16SRC>
__global__ void __launch_bounds__(256) quant_rows_i8_kernel(const void* src, int N, int K, int8_t* codes,
                                                            __half* scales) {
  const int row = blockIdx.x;
  if (row >= N) return;
  const size_t base = (size_t)row * K;
  float m = 0.f;
  for (int i = threadIdx.x; i < K; i += blockDim.x) m = fmaxf(m, fabsf(load_w<F16SRC>(src, base + i)));
  m = warp_max(m);
  __shared__ float sm[8];
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = sm[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, sm[w]);
    sm[0] = fmaxf(__fdiv_rn(t, 127.0f), 1e-8f);
  }
  __syncthreads();
  const float s = sm[0];
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    float q = rintf(__fdiv_rn(load_w<F16SRC>(src, base + i), s));
    q = fminf(fmaxf(q, -127.f), 127.f);
    codes[base + i] = (int8_t)(int)q;
  }
  if (threadIdx.x == 0) scales[row] = __float2half_rn(s);
}

template <bool F16SRC>
__global__ void __launch_bounds__(256) quant_g32_i4_kernel(const void* src, int N, int K, uint8_t* packed,
                                                           __half* scales) {
  const int ng = K / 32;
  const size_t gid = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gid >= (size_t)N * ng) return;
  const int lane = threadIdx.x & 31;
  const size_t row = gid / ng, g = gid % ng;
  const float w = load_w<F16SRC>(src, row * K + g * 32 + lane);
  const float m = warp_max(fabsf(w));
  const float s = fmaxf(__fdiv_rn(m, 7.0f), 1e-8f);
  float q = rintf(__fdiv_rn(w, s));
  q = fminf(fmaxf(q, -7.f), 7.f);
  const uint32_t nib = (uint32_t)((int)q + 8);
  const uint32_t hi = __shfl_down_sync(0xffffffffu, nib, 1);
  if ((lane & 1) == 0) packed[row * (K / 2) + g * 16 + lane / 2] = (uint8_t)(nib | (hi << 4));
  if (lane == 0) scales[row * ng + g] = __float2half_rn(s);
}

cudaError_t quantize_rows_i8(const void* src, int src_f16, int N, int K, int8_t* codes, __half* scales,
                             cudaStream_t st) {
  if (N <= 0 || K <= 0) return cudaErrorInvalidValue;
  if (src_f16) quant_rows_i8_kernel<true><<<N, 256, 0, st>>>(src, N, K, codes, scales);
  else quant_rows_i8_kernel<false><<<N, 256, 0, st>>>(src, N, K, codes, scales);
  return cudaGetLastError();
}

cudaError_t quantize_g32_i4(const void* src, int src_f16, int N, int K, uint8_t* packed, __half* scales,
                            cudaStream_t st) {
  if (N <= 0 || K <= 0 || K % 32) return cudaErrorInvalidValue;
  const size_t groups = (size_t)N * (K / 32);
  const unsigned blocks = (unsigned)((groups + 7) / 8);
  if (src_f16) quant_g32_i4_kernel<true><<<blocks, 256, 0, st>>>(src, N, K, packed, scales);
  else quant_g32_i4_kernel<false><<<blocks, 256, 0, st>>>(src, N, K, packed, scales);
  return cudaGetLastError();
}

}  // namespace af
