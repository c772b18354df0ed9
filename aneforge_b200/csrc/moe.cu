// Mixture-of-experts router tail: the reference's `_moe` gate (aneforge/moe.py:48-56 with
// `_topk_gate`, moe.py:21-37) on the device, one warp per token row:
//   probs = softmax(router logits) in fp32;
//   k rounds of: take the row max of the remaining probabilities, choose the lowest index holding
//   it, overwrite that entry with f16(-3e4) (the reference's peel value);
//   gw = probs on the chosen experts (0 elsewhere), divided by their sum when norm_topk_prob.
// sel[b][i] is the expert chosen in round i; the expert GEMVs read it from device memory.
#include "af_common.cuh"
#include "af_kernels.h"

namespace af {

constexpr int MOE_EMAX = 64;

__global__ void __launch_bounds__(32) moe_gate_kernel(const float* logits, int ld, int E, int k, int renorm, float* gw,
                                                      int* sel) {
  const int b = blockIdx.x, lane = threadIdx.x;
  pdl_wait();
  // each lane holds experts lane and lane + 32
  float v[2], p[2];
  for (int j = 0; j < 2; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < E ? __ldcg(logits + (size_t)b * ld + e) : -INFINITY;
  }
  const float mx = warp_max(fmaxf(v[0], v[1]));
  float s = 0.f;
  for (int j = 0; j < 2; ++j) {
    p[j] = (lane + 32 * j) < E ? expf(v[j] - mx) : 0.f;
    s += p[j];
  }
  s = warp_sum(s);
  for (int j = 0; j < 2; ++j) p[j] = p[j] / s;
  float rem[2] = {p[0], p[1]};
  bool chosen[2] = {false, false};
  const float peel = __half2float(__float2half_rn(-3.0e4f));
  for (int r = 0; r < k; ++r) {
    float m = -INFINITY;
    for (int j = 0; j < 2; ++j) if (lane + 32 * j < E) m = fmaxf(m, rem[j]);
    m = warp_max(m);
    int first = 0x7fffffff;
    for (int j = 0; j < 2; ++j) if (lane + 32 * j < E && rem[j] >= m) first = min(first, lane + 32 * j);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
    for (int j = 0; j < 2; ++j)
      if (lane + 32 * j == first) { chosen[j] = true; rem[j] = peel; }
    if (lane == 0) sel[(size_t)b * k + r] = first;
  }
  float g[2], gs = 0.f;
  for (int j = 0; j < 2; ++j) { g[j] = chosen[j] ? p[j] : 0.f; gs += g[j]; }
  gs = warp_sum(gs);
  for (int j = 0; j < 2; ++j) {
    const int e = lane + 32 * j;
    if (e < E) gw[(size_t)b * E + e] = renorm ? g[j] / gs : g[j];
  }
  pdl_trigger();
}

cudaError_t moe_gate_launch(const float* logits, int ld, int NB, int E, int k, int renorm, float* gw, int* sel,
                            cudaStream_t st, bool pdl) {
  if (NB < 1 || E < 1 || E > MOE_EMAX || k < 1 || k > E) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(NB);
  cfg.blockDim = dim3(32);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, moe_gate_kernel, logits, ld, E, k, renorm, gw, sel);
}

// Per-expert row lists of a batch (the routed expert GEMVs gather their rows through them): thread
// e walks the rows in order and lists each row that selected expert e; rows[e * rld + i], i < cnt[e].
__global__ void __launch_bounds__(MOE_EMAX) moe_route_kernel(const int* sel, int NB, int k, int E, int rld, int* rows,
                                                             int* cnt) {
  const int e = threadIdx.x;
  pdl_wait();
  if (e < E) {
    int n = 0;
    for (int b = 0; b < NB; ++b)
      for (int j = 0; j < k; ++j)
        if (__ldcg(sel + (size_t)b * k + j) == e) {
          if (n < rld) rows[(size_t)e * rld + n] = b;
          ++n;
          break;
        }
    cnt[e] = n < rld ? n : rld;
  }
  pdl_trigger();
}

cudaError_t moe_route_launch(const int* sel, int NB, int k, int E, int rld, int* rows, int* cnt, cudaStream_t st,
                             bool pdl) {
  if (NB < 1 || E < 1 || E > MOE_EMAX || k < 1 || k > E || rld < 1) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(MOE_EMAX);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, moe_route_kernel, sel, NB, k, E, rld, rows, cnt);
}

}  // namespace af

extern "C" int af_moe_gate(const float* logits, int ld, int nb, int e, int k, int renorm, float* gw, int* sel,
                           void* stream) {
  const cudaError_t r = af::moe_gate_launch(logits, ld, nb, e, k, renorm, gw, sel, static_cast<cudaStream_t>(stream),
                                            false);
  if (r != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return 0;
}
