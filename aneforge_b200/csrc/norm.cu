// RMSNorm (the reference lowering, aneforge/_compile.py:738-755) and the embedding gather.
//
// The reference bakes RMSNorm as reduce_l2_norm -> maximum(floor) -> real_div -> mul(g_eff) with
// g_eff = f16(gamma * sqrt(D)) and floor = f16(sqrt(D * eps)); this kernel evaluates exactly that
// chain in fp32 (IEEE sqrt and divide) and writes the fp16 operand the next matmul consumes.
#include "af_common.cuh"
#include "af_kernels.h"

namespace af {

template <bool XF16>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const void* x, int ldx, const __half* g, float floor,
                                                      __half* out, int ldo, int D) {
  const int b = blockIdx.x;
  pdl_wait();
  const float* xf = reinterpret_cast<const float*>(x) + (size_t)b * ldx;
  const __half* xh = reinterpret_cast<const __half*>(x) + (size_t)b * ldx;
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float v = XF16 ? __half2float(__ldcg(xh + i)) : __ldcg(xf + i);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  __shared__ float sm[32];
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += sm[w];
    sm[0] = fmaxf(sqrtf(t), floor);
  }
  __syncthreads();
  const float sn = sm[0];
  pdl_trigger();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float v = XF16 ? __half2float(__ldcg(xh + i)) : __ldcg(xf + i);
    out[(size_t)b * ldo + i] = __float2half_rn(__fdiv_rn(v, sn) * __half2float(g[i]));
  }
}

__global__ void __launch_bounds__(256) embed_kernel(const int* tok, const __half* table, int vocab, float* h,
                                                    int ldh, int D, int* err) {
  const int b = blockIdx.x;
  pdl_wait();
  const int t = __ldcg(tok + b);
  const bool ok = t >= 0 && t < vocab;
  if (!ok && threadIdx.x == 0) af_set_err(err, AF_DEV_BAD_TOKEN);
  pdl_trigger();
  for (int i = threadIdx.x; i < D; i += blockDim.x)
    h[(size_t)b * ldh + i] = ok ? __half2float(table[(size_t)t * D + i]) : 0.f;
}

// dtype conversion: mode 0 = fp16 -> fp32, 1 = fp32 -> fp16 (round to nearest even)
__global__ void __launch_bounds__(256) cast_kernel(const void* src, void* dst, size_t n, int mode) {
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    if (mode == 0) reinterpret_cast<float*>(dst)[i] = __half2float(__ldcg(reinterpret_cast<const __half*>(src) + i));
    else reinterpret_cast<__half*>(dst)[i] = __float2half_rn(__ldcg(reinterpret_cast<const float*>(src) + i));
  }
}

static cudaLaunchConfig_t mkcfg(dim3 g, dim3 b, size_t smem, cudaStream_t st, bool pdl, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g;
  cfg.blockDim = b;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

cudaError_t rmsnorm_launch(const void* x, int x_f16, int ldx, const __half* g, float floor, __half* out, int ldo,
                           int NB, int D, cudaStream_t st, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = mkcfg(dim3(NB), dim3(256), 0, st, pdl, attr);
  if (x_f16) return cudaLaunchKernelEx(&cfg, rmsnorm_kernel<true>, x, ldx, g, floor, out, ldo, D);
  return cudaLaunchKernelEx(&cfg, rmsnorm_kernel<false>, x, ldx, g, floor, out, ldo, D);
}

cudaError_t embed_launch(const int* tok, const __half* table, int vocab, float* h, int ldh, int NB, int D, int* err,
                         cudaStream_t st, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = mkcfg(dim3(NB), dim3(256), 0, st, pdl, attr);
  return cudaLaunchKernelEx(&cfg, embed_kernel, tok, table, vocab, h, ldh, D, err);
}

cudaError_t cast_launch(const void* src, void* dst, size_t n, int mode, cudaStream_t st, bool pdl) {
  cudaLaunchAttribute attr[1];
  unsigned blocks = (unsigned)((n + 255) / 256);
  if (blocks > 4096) blocks = 4096;
  if (blocks == 0) blocks = 1;
  cudaLaunchConfig_t cfg = mkcfg(dim3(blocks), dim3(256), 0, st, pdl, attr);
  return cudaLaunchKernelEx(&cfg, cast_kernel, src, dst, n, mode);
}

}  // namespace af
