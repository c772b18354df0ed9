// RMSNorm (the reference lowering, aneforge/_compile.py:738-755) and the embedding gather.
//
// The reference bakes RMSNorm as reduce_l2_norm -> maximum(floor) -> real_div -> mul(g_eff) with
// g_eff = f16(gamma * sqrt(D)) and floor = f16(sqrt(D * eps)); this kernel evaluates exactly that
// chain in fp32 (IEEE sqrt and divide) and writes the fp16 operand the next matmul consumes.
#include "af_common.cuh"
#include "af_kernels.h"

namespace af {

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


// One CTA per row, 1024 threads; the row stays in registers between the sum of squares and the
// scaling (one read of x). Vector path: D % 4 == 0 (fp32) or D % 8 == 0 (fp16) with aligned rows.
template <bool XF16, int PER>
__global__ void __launch_bounds__(1024) rmsnorm_kernel(const void* x, int ldx, const __half* g, float floor,
                                                       __half* out, int ldo, int D, L2Pf pf) {
  const int b = blockIdx.x;
  constexpr int VW = XF16 ? 8 : 4;                   // elements per vector load
  float v[PER * VW];
  const int nvec = D / VW;
  // γ is a weight: this thread's γ values are read before the programmatic-launch wait, so only the
  // row read remains after it
  __half gh[PER * VW];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int vi = threadIdx.x + k * blockDim.x;
    if (vi < nvec) {
      if (VW == 8) *reinterpret_cast<uint4*>(gh + k * VW) = __ldg(reinterpret_cast<const uint4*>(g) + vi);
      else *reinterpret_cast<uint2*>(gh + k * VW) = __ldg(reinterpret_cast<const uint2*>(g) + vi);
    }
  }
  l2_prefetch_lines(pf, blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x);
  pdl_wait();
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int vi = threadIdx.x + k * blockDim.x;
    if (vi < nvec) {
      if (XF16) {
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(x) + (size_t)b * ldx) + vi);
        h8_to_f32(u, v + k * VW);
      } else {
        const float4 f = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + (size_t)b * ldx) + vi);
        v[k * VW] = f.x; v[k * VW + 1] = f.y; v[k * VW + 2] = f.z; v[k * VW + 3] = f.w;
      }
#pragma unroll
      for (int e = 0; e < VW; ++e) ss = fmaf(v[k * VW + e], v[k * VW + e], ss);
    }
  }
  ss = warp_sum(ss);
  __shared__ float sm[32];
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? sm[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) sm[0] = fmaxf(sqrtf(t), floor);
  }
  __syncthreads();
  const float sn = sm[0];
  pdl_trigger();
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int vi = threadIdx.x + k * blockDim.x;
    if (vi < nvec) {
      __half o[VW];
#pragma unroll
      for (int e = 0; e < VW; ++e) o[e] = __float2half_rn(__fdiv_rn(v[k * VW + e], sn) * __half2float(gh[k * VW + e]));
      __half* dst = out + (size_t)b * ldo + (size_t)vi * VW;
      if (VW == 8) *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(o);
      else *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(o);
    }
  }
}

// scalar fallback for odd sizes / alignment
template <bool XF16>
__global__ void __launch_bounds__(256) rmsnorm_scalar_kernel(const void* x, int ldx, const __half* g, float floor,
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

// One CTA per row; each thread moves 8 fp16 (one 16-byte load) into 8 fp32 of the residual stream.
__global__ void __launch_bounds__(512) embed_kernel(const int* tok, const __half* table, int vocab, float* h,
                                                    int ldh, int D, int* err) {
  const int b = blockIdx.x;
  pdl_wait();
  const int t = __ldcg(tok + b);
  const bool ok = t >= 0 && t < vocab;
  if (!ok && threadIdx.x == 0) af_set_err(err, AF_DEV_BAD_TOKEN);
  pdl_trigger();
  const bool vec = (D % 8) == 0 && (ldh % 4) == 0;
  if (vec) {
    for (int i = threadIdx.x; i < D / 8; i += blockDim.x) {
      float f[8];
      if (ok) h8_to_f32(__ldg(reinterpret_cast<const uint4*>(table + (size_t)t * D) + i), f);
      else for (int e = 0; e < 8; ++e) f[e] = 0.f;
      float4* dst = reinterpret_cast<float4*>(h + (size_t)b * ldh) + 2 * i;
      dst[0] = make_float4(f[0], f[1], f[2], f[3]);
      dst[1] = make_float4(f[4], f[5], f[6], f[7]);
    }
  } else {
    for (int i = threadIdx.x; i < D; i += blockDim.x)
      h[(size_t)b * ldh + i] = ok ? __half2float(table[(size_t)t * D + i]) : 0.f;
  }
}

// dtype conversion: mode 0 = fp16 -> fp32, 1 = fp32 -> fp16 (round to nearest even)
__global__ void __launch_bounds__(256) cast_kernel(const void* src, void* dst, size_t n, int mode) {
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    if (mode == 0) reinterpret_cast<float*>(dst)[i] = __half2float(__ldcg(reinterpret_cast<const __half*>(src) + i));
    else reinterpret_cast<__half*>(dst)[i] = __float2half_rn(__ldcg(reinterpret_cast<const float*>(src) + i));
  }
}


cudaError_t rmsnorm_launch(const void* x, int x_f16, int ldx, const __half* g, float floor, __half* out, int ldo,
                           int NB, int D, cudaStream_t st, bool pdl, const L2Pf& pf) {
  cudaLaunchAttribute attr[1];
  const int VW = x_f16 ? 8 : 4;
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(g) % 16 == 0) &&
                       (ldx % VW == 0) && (ldo % 8 == 0) && (D % 8 == 0);
  const int nvec = D / VW;
  const int per = (nvec + 1023) / 1024;
  if (aligned && per <= 8) {
    const int threads = nvec < 1024 ? ((nvec + 31) / 32) * 32 : 1024;
    cudaLaunchConfig_t cfg = mkcfg(dim3(NB), dim3(threads), 0, st, pdl, attr);
#define AF_RMS(XF, P) if (per <= P) return cudaLaunchKernelEx(&cfg, rmsnorm_kernel<XF, P>, x, ldx, g, floor, out, ldo, D, pf);
    if (x_f16) { AF_RMS(true, 1) AF_RMS(true, 2) AF_RMS(true, 4) AF_RMS(true, 8) }
    else { AF_RMS(false, 1) AF_RMS(false, 2) AF_RMS(false, 4) AF_RMS(false, 8) }
#undef AF_RMS
  }
  cudaLaunchConfig_t cfg = mkcfg(dim3(NB), dim3(256), 0, st, pdl, attr);
  if (x_f16) return cudaLaunchKernelEx(&cfg, rmsnorm_scalar_kernel<true>, x, ldx, g, floor, out, ldo, D);
  return cudaLaunchKernelEx(&cfg, rmsnorm_scalar_kernel<false>, x, ldx, g, floor, out, ldo, D);
}

// Block-wide sum (blockDim a multiple of 32, at most 1024); `red` holds 32 floats.
static __device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];
  __syncthreads();                          // red is reused by the next call
  return t;
}

// LayerNorm of fp32 rows into fp16 (reference `_e_layer_norm`, `aneforge/_compile.py:758-776`):
// xc = x - mean(x); out = xc * (1 / sqrt(mean(xc^2) + eps)) * g + b, each step rounded in fp32.
__global__ void __launch_bounds__(256) layernorm_kernel(const float* x, int ldx, const __half* g, const __half* bta,
                                                        float eps, __half* out, int ldo, int D) {
  __shared__ float red[32];
  const float* xr = x + (size_t)blockIdx.x * ldx;
  pdl_wait();
  float s = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) s += __ldcg(xr + i);
  const float mu = __fdiv_rn(block_sum(s, red), (float)D);
  float v = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float c = __fsub_rn(__ldcg(xr + i), mu);
    v = fmaf(c, c, v);
  }
  const float var = __fdiv_rn(block_sum(v, red), (float)D);
  const float rr = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, eps)));
  pdl_trigger();
  __half* o = out + (size_t)blockIdx.x * ldo;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float xn = __fmul_rn(__fsub_rn(__ldcg(xr + i), mu), rr);
    o[i] = f2h(__fadd_rn(__fmul_rn(xn, h2f(g[i])), bta ? h2f(bta[i]) : 0.f));
  }
}

cudaError_t layernorm_launch(const float* x, int ldx, const __half* g, const __half* b, float eps, __half* out, int ldo,
                             int NB, int D, cudaStream_t st, bool pdl) {
  if (NB < 1 || D < 1) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = mkcfg(dim3(NB), dim3(256), 0, st, pdl, attr);
  return cudaLaunchKernelEx(&cfg, layernorm_kernel, x, ldx, g, b, eps, out, ldo, D);
}

// Learned positional embedding (GPT-2's wpe): h[b] += table[p] with p = pos[b] (decode) or b (the
// rows of a prompt), a position outside the table recorded as AF_DEV_BAD_POS.
__global__ void __launch_bounds__(256) add_pos_kernel(float* h, int ldh, const __half* table, int npos, const int* pos,
                                                      int D, int* err) {
  const int b = blockIdx.x;
  pdl_wait();
  const int p = pos ? __ldcg(pos + b) : b;
  if (p < 0 || p >= npos) {
    if (threadIdx.x == 0) af_set_err(err, AF_DEV_BAD_POS);
    return;
  }
  pdl_trigger();
  float* hr = h + (size_t)b * ldh;
  for (int i = threadIdx.x; i < D; i += blockDim.x) hr[i] = __fadd_rn(hr[i], h2f(table[(size_t)p * D + i]));
}

cudaError_t add_pos_launch(float* h, int ldh, const __half* table, int npos, const int* pos, int NB, int D, int* err,
                           cudaStream_t st, bool pdl) {
  if (NB < 1 || D < 1) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = mkcfg(dim3(NB), dim3(256), 0, st, pdl, attr);
  return cudaLaunchKernelEx(&cfg, add_pos_kernel, h, ldh, table, npos, pos, D, err);
}

cudaError_t embed_launch(const int* tok, const __half* table, int vocab, float* h, int ldh, int NB, int D, int* err,
                         cudaStream_t st, bool pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = mkcfg(dim3(NB), dim3(512), 0, st, pdl, attr);
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
