// Decode GEMV over bitmask-sparse fp16 weights (the reference's `sparsify`, `aneforge/_blob.py:59-64`,
// accepted for a weight at most half nonzero): per row a K-bit keep mask and the kept values in
// column order, so a row streams K/8 + 2 nnz bytes instead of 2 K.
//
// One warp per output (two rows - gate and up - for the SWIGLU epilogue). A round covers 32 mask
// words (1024 columns), one per lane: each lane counts its word's bits, an inclusive warp scan turns
// the counts into the offsets of the lanes' first values, and each lane then walks its set bits,
// reading its run of values and the matching x columns. x rows are read through L1 (every warp of a
// CTA reads the same x).
#include "af_common.cuh"
#include "af_kernels.h"

namespace af {

namespace {

constexpr int SP_WARPS = 8;

template <int NB>
AF_DEV void sparse_row(const GemvArgs& a, int row, int lane, float (&acc)[NB]) {
  const int KW = a.K / 32;
  const uint32_t* m = static_cast<const uint32_t*>(a.w) + (size_t)row * KW;
  int base = __ldg(a.rowoff + row);
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.f;
  for (int w0 = 0; w0 < KW; w0 += 32) {
    const int w = w0 + lane;
    uint32_t bits = w < KW ? __ldg(m + w) : 0u;
    const int c = __popc(bits);
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int off = base + incl - c;
    while (bits) {
      const int j = __ffs(bits) - 1;
      bits &= bits - 1;
      const float v = h2f(__ldg(a.gscale + off));
      ++off;
      const int col = 32 * w + j;
#pragma unroll
      for (int b = 0; b < NB; ++b)
        if (b < a.NB) acc[b] = fmaf(v, h2f(__ldg(a.x + (size_t)b * a.ldx + col)), acc[b]);
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = warp_sum(acc[b]);
}

template <int NB>
__global__ void __launch_bounds__(SP_WARPS * 32) gemv_sparse_kernel(GemvArgs a) {
  const int lane = threadIdx.x & 31;
  const int u = blockIdx.x * SP_WARPS + (threadIdx.x >> 5);      // output column
  const bool swiglu = a.epi == EPI_SWIGLU;
  const int units = swiglu ? a.N / 2 : a.N;
  pdl_wait();
  pdl_trigger();
  if (u >= units) return;
  if (swiglu) {
    // gate / up rows in blocks of 4 (the fused layout): unit u = block u / 4, row u % 4 of each half
    const int gr = (u / 4) * 8 + (u % 4), ur = gr + 4;
    float g[NB], up[NB];
    sparse_row<NB>(a, gr, lane, g);
    sparse_row<NB>(a, ur, lane, up);
    if (lane < NB && lane < a.NB) {
      float gv = g[0], uv = up[0];
#pragma unroll
      for (int b = 1; b < NB; ++b)
        if (lane == b) { gv = g[b]; uv = up[b]; }
      if (a.bias) { gv = __fadd_rn(gv, h2f(a.bias[gr])); uv = __fadd_rn(uv, h2f(a.bias[ur])); }
      reinterpret_cast<__half*>(a.y)[(size_t)lane * a.ldy + u] = f2h(silu_f(gv) * uv);
    }
    return;
  }
  float acc[NB];
  sparse_row<NB>(a, u, lane, acc);
  if (lane < NB && lane < a.NB) {
    float v = acc[0];
#pragma unroll
    for (int b = 1; b < NB; ++b)
      if (lane == b) v = acc[b];
    if (a.bias) v = __fadd_rn(v, h2f(a.bias[u]));
    const size_t o = (size_t)lane * a.ldy + u;
    if (a.epi == EPI_F32) reinterpret_cast<float*>(a.y)[o] = v;
    else if (a.epi == EPI_F16) reinterpret_cast<__half*>(a.y)[o] = f2h(v);
    else reinterpret_cast<float*>(a.y)[o] += v;
  }
}

}  // namespace

cudaError_t gemv_sparse_launch(const GemvArgs& a0, cudaStream_t st, bool pdl) {
  if (a0.NB < 1 || a0.N < 1 || a0.K < 32 || a0.K % 32 || !a0.w || !a0.gscale || !a0.rowoff || !a0.x || !a0.y)
    return cudaErrorInvalidValue;
  if (a0.epi == EPI_ARGMAX || (a0.epi == EPI_SWIGLU && a0.N % 8)) return cudaErrorInvalidValue;
  const int units = a0.epi == EPI_SWIGLU ? a0.N / 2 : a0.N;
  for (int b0 = 0; b0 < a0.NB; b0 += 8) {
    GemvArgs a = a0;
    a.NB = a0.NB - b0 < 8 ? a0.NB - b0 : 8;
    a.x = a0.x + (size_t)b0 * a0.ldx;
    const size_t esz = (a0.epi == EPI_F16 || a0.epi == EPI_SWIGLU) ? 2 : 4;
    a.y = static_cast<char*>(a0.y) + (size_t)b0 * a0.ldy * esz;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((units + SP_WARPS - 1) / SP_WARPS);
    cfg.blockDim = dim3(SP_WARPS * 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl && b0 == 0) ? 1 : 0;
    cudaError_t e = a.NB == 1 ? cudaLaunchKernelEx(&cfg, gemv_sparse_kernel<1>, a)
                  : a.NB <= 4 ? cudaLaunchKernelEx(&cfg, gemv_sparse_kernel<4>, a)
                              : cudaLaunchKernelEx(&cfg, gemv_sparse_kernel<8>, a);
    if (e != cudaSuccess) return e;
  }
  return cudaGetLastError();
}

}  // namespace af
