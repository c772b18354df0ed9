// Bandwidth-bound dequant GEMV for decode (K1 int8 per-row, K2 int4 group-32, fp16 weights for the
// lm_head and uncompressed projections), with fused epilogues:
//   F32 / F16  : y = scale (.) (x . W^T) + bias
//   RESID      : y += scale (.) (x . W^T) + bias          (o_proj / down_proj residual add, fp32 stream)
//   SWIGLU     : y = silu(g) * u over gate/up rows packed in blocks of R (gate rows, then up rows)
//   ARGMAX     : logits (optional) + per-row-block (max, index) partials, reduced by the last CTA
//                to the greedy token (lowest index on exact ties, numpy argmax semantics)
//
// Layout: weights are row-major [N][K] codes (int8: K bytes per row; int4: K/2 bytes per row,
// element 2i in the low nibble; fp16: 2K bytes per row) so every thread issues 16-byte loads that a
// warp coalesces into 512 contiguous bytes of one row. Scales are fp16, per row (int8) or per
// 32-element group [N][K/32] (int4). Activations x are fp16 [NB][ldx].
//
// Mapping: a CTA of 256 threads is split into G groups of TG threads; each group owns R rows and
// strides over the row's 16-byte chunks; partial dots are reduced with warp shuffles, then across the
// group's warps in shared memory. All weight loads of a chunk are issued before the math so each
// thread keeps R x 16 bytes in flight.
#include "af_common.cuh"
#include "af_kernels.h"
#include "tc_common.cuh"

namespace af {

template <int WF>
struct WTraits;
template <>
struct WTraits<W_I8> { static constexpr int EPC = 16; };   // elements per 16-byte chunk
template <>
struct WTraits<W_F16> { static constexpr int EPC = 8; };
template <>
struct WTraits<W_I4G32> { static constexpr int EPC = 32; };
template <>
struct WTraits<W_LUT4> { static constexpr int EPC = 32; };
template <>
struct WTraits<W_I8G> { static constexpr int EPC = 16; };

// elements per 16-byte chunk of a weight format (host side)
static int chunk_elems(int wf) {
  return wf == W_I8 || wf == W_I8G ? 16 : wf == W_F16 ? 8 : 32;
}

// Rows per thread group: 8 for one sequence (128 B of weights in flight per thread), fewer as the
// batch grows; the SWIGLU epilogue always works on blocks of 8 packed rows (4 gate + 4 up), the
// granularity of the packed gate/up layout.
__host__ __device__ constexpr int rows_per_group(int nb, int epi) {
  return epi == EPI_SWIGLU ? 8 : (nb == 1 ? 8 : (nb == 2 ? 4 : 2));
}

template <int WF, int NB, int R, int EPI>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs a) {
  constexpr int EPC = WTraits<WF>::EPC;
  const int TG = a.tg;                         // threads per group (multiple of 32)
  const int G = blockDim.x / TG;
  const int grp = threadIdx.x / TG;
  const int tid = threadIdx.x - grp * TG;
  const int row0 = (blockIdx.x * G + grp) * R;
  const int nch = a.K / EPC;
  const size_t row_bytes = (size_t)nch * 16;
  const char* Wb = reinterpret_cast<const char*>(a.w);
  const int nbr = a.NB;                        // rows of x in this launch (<= NB)

  float acc[R][NB];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[r][b] = 0.f;

  // LUT4: the codebooks of this CTA's rows (at most 8 groups x 8 rows), decoded to fp32 once
  __shared__ float lut_s[WF == W_LUT4 ? 64 * 16 : 1];
  if (WF == W_LUT4) {
    const int cta_row0 = blockIdx.x * G * R;
    for (int i = threadIdx.x; i < G * R * 16; i += blockDim.x) {
      const int row = cta_row0 + i / 16;
      lut_s[i] = row < a.N ? h2f(a.gscale[(size_t)row * 16 + (i & 15)]) : 0.f;
    }
    __syncthreads();
  }
  const int ngroups = WF == W_I8G ? a.K / a.group : 0;

  bool waited = false;
  for (int c = tid; c < nch; c += TG) {
    uint4 wv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int row = row0 + r;
      wv[r] = row < a.N ? ldg_stream(Wb + (size_t)row * row_bytes + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
    }
    float gs[R];
    if (WF == W_I4G32) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int row = row0 + r;
        gs[r] = row < a.N ? h2f(a.gscale[(size_t)row * nch + c]) : 0.f;
      }
    }
    if (WF == W_I8G) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int row = row0 + r;
        gs[r] = row < a.N ? h2f(a.gscale[(size_t)row * ngroups + (c * EPC) / a.group]) : 0.f;
      }
    }
    if (!waited) { pdl_wait(); waited = true; }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b >= nbr) break;
      const __half* xp = a.x + (size_t)b * a.ldx + (size_t)c * EPC;
      float xf[EPC];
#pragma unroll
      for (int i = 0; i < EPC / 8; ++i) h8_to_f32(ld_act_v4(xp + 8 * i), xf + 8 * i);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t* wu = reinterpret_cast<const uint32_t*>(&wv[r]);
        float s = 0.f;
        if (WF == W_I8 || WF == W_I8G) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float f0, f1, f2, f3;
            i8x4_to_f32(wu[q], f0, f1, f2, f3);
            s = fmaf(f0, xf[4 * q + 0], s);
            s = fmaf(f1, xf[4 * q + 1], s);
            s = fmaf(f2, xf[4 * q + 2], s);
            s = fmaf(f3, xf[4 * q + 3], s);
          }
          if (WF == W_I8) acc[r][b] += s;
          else acc[r][b] = fmaf(gs[r], s, acc[r][b]);
        } else if (WF == W_LUT4) {
          const float* lut = lut_s + (grp * R + r) * 16;
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int i = 0; i < 8; ++i) s = fmaf(lut[(wu[q] >> (4 * i)) & 15u], xf[8 * q + i], s);
          acc[r][b] += s;
        } else if (WF == W_F16) {
          float wf[8];
          h8_to_f32(wv[r], wf);
#pragma unroll
          for (int i = 0; i < 8; ++i) s = fmaf(wf[i], xf[i], s);
          acc[r][b] += s;
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float f[8];
            u4x8_to_f32(wu[q], f);
#pragma unroll
            for (int i = 0; i < 8; ++i) s = fmaf(f[i], xf[8 * q + i], s);
          }
          acc[r][b] = fmaf(gs[r], s, acc[r][b]);
        }
      }
    }
  }
  if (!waited) pdl_wait();
  pdl_trigger();

  // ---- reduction: warp shuffles, then across the group's warps in shared memory
  extern __shared__ float red[];                  // [G][TG/32][R*NB]
  const int lane = threadIdx.x & 31;
  const int wig = tid >> 5;
  const int nw = TG >> 5;
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float v = warp_sum(acc[r][b]);
      if (lane == 0) red[(grp * nw + wig) * R * NB + r * NB + b] = v;
    }
  __syncthreads();

  if (EPI == EPI_ARGMAX) {
    // every (row, batch) value of this CTA -> logits + CTA-local argmax, then the last CTA reduces
    float* vals = red + G * nw * R * NB;            // [G*R][NB]
    for (int i = threadIdx.x; i < G * R * NB; i += blockDim.x) {
      const int g = i / (R * NB), rb = i - g * (R * NB);
      const int r = rb / NB, b = rb - r * NB;
      float v = 0.f;
      for (int w = 0; w < nw; ++w) v += red[(g * nw + w) * R * NB + rb];
      const int row = (blockIdx.x * G + g) * R + r;
      if (row < a.N && b < nbr) {
        if (WF == W_I8) v *= h2f(a.scale[row]);
        if (a.bias) v += h2f(a.bias[row]);
        if (a.y) reinterpret_cast<float*>(a.y)[(size_t)b * a.ldy + row] = v;
      } else {
        v = -INFINITY;
      }
      vals[(g * R + r) * NB + b] = v;
    }
    __syncthreads();
    if (threadIdx.x < nbr) {
      const int b = threadIdx.x;
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int j = 0; j < G * R; ++j) {
        const int row = (blockIdx.x * G + j / R) * R + (j % R);
        const float v = vals[j * NB + b];
        if (row < a.N && (bi == 0x7fffffff || v > best)) { best = v; bi = row; }   // rows ascend: ties keep the lowest
      }
      a.am_val[(size_t)blockIdx.x * NB + b] = best;
      a.am_idx[(size_t)blockIdx.x * NB + b] = bi;
    }
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) last = (atomicAdd(a.am_count, 1) == (int)gridDim.x - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int b = 0; b < nbr; ++b) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int j = threadIdx.x; j < (int)gridDim.x; j += blockDim.x) {
        const float v = __ldcg(a.am_val + (size_t)j * NB + b);
        const int ix = __ldcg(a.am_idx + (size_t)j * NB + b);
        if (v > best || (v == best && ix < bi)) { best = v; bi = ix; }
      }
      // block argmax, ties -> lowest index
      __shared__ float sv[32];
      __shared__ int si[32];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
      }
      if (lane == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
          if (sv[w] > best || (sv[w] == best && si[w] < bi)) { best = sv[w]; bi = si[w]; }
        a.tok_out[b] = bi + a.idx_base;
        if (a.val_out) a.val_out[b] = best;
        if (a.pos_adv) {
          const int p = __ldcg(a.pos_adv + b);
          if (a.hist && p >= 0 && p < a.hist_ld) a.hist[(size_t)b * a.hist_ld + p] = bi;
          a.pos_adv[b] = p + 1;
        }
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) *a.am_count = 0;
    return;
  }

  if (EPI == EPI_SWIGLU) {
    constexpr int H2 = R / 2;
    for (int i = tid; i < H2 * NB; i += TG) {
      const int r = i / NB, b = i - r * NB;
      if (b >= nbr) continue;
      float g = 0.f, u = 0.f;
      for (int w = 0; w < nw; ++w) {
        g += red[(grp * nw + w) * R * NB + r * NB + b];
        u += red[(grp * nw + w) * R * NB + (r + H2) * NB + b];
      }
      const int rg = row0 + r, ru = row0 + H2 + r;
      if (ru < a.N) {
        if (WF == W_I8) { g *= h2f(a.scale[rg]); u *= h2f(a.scale[ru]); }
        if (a.bias) { g += h2f(a.bias[rg]); u += h2f(a.bias[ru]); }
        const int out = row0 / 2 + r;
        reinterpret_cast<__half*>(a.y)[(size_t)b * a.ldy + out] = f2h(silu_f(g) * u);
      }
    }
    return;
  }

  for (int i = tid; i < R * NB; i += TG) {
    const int r = i / NB, b = i - r * NB;
    const int row = row0 + r;
    if (row >= a.N || b >= nbr) continue;
    float v = 0.f;
    for (int w = 0; w < nw; ++w) v += red[(grp * nw + w) * R * NB + i];
    if (WF == W_I8) v *= h2f(a.scale[row]);
    if (a.bias) v += h2f(a.bias[row]);
    const size_t o = (size_t)b * a.ldy + row;
    if (EPI == EPI_F32) reinterpret_cast<float*>(a.y)[o] = v;
    else if (EPI == EPI_F16) reinterpret_cast<__half*>(a.y)[o] = f2h(v);
    else if (EPI == EPI_RESID) reinterpret_cast<float*>(a.y)[o] = __ldcg(reinterpret_cast<const float*>(a.y) + o) + v;
  }
}

// ---- the fp16 lm_head for 2..16 sequences on the tensor pipe (mma.sync m16n8k16, fp32 accumulate)
// The CUDA-core kernel above is bandwidth-bound for one sequence but compute-bound from about four:
// it re-streams the head per 4-row tile at ~4x the single-row time. Here one launch reads the head
// once: each warp owns 16 vocabulary rows and walks K in 32-wide chunks with 16-byte loads (rows g and
// g + 8 of the fragment from lanes 4g..4g+3, x from the same k positions: the k order inside a chunk
// is permuted identically for both operands, so the dot products are unchanged); the batch is the
// MMA's N (8 per n-tile). Epilogue: optional fp32 logits, then the argmax of the CUDA-core kernel
// (per-CTA candidates, ties to the lowest index, the last CTA merges and advances pos / history).
template <int NT>
__global__ void __launch_bounds__(256) lm_head_tc_kernel(GemvArgs a) {
  constexpr int NW = 8, U = 4;                       // warps per CTA, 32-wide chunks per load batch
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int row0 = (blockIdx.x * NW + warp) * 16;
  const int K = a.K, NB = a.NB;
  const __half* W = static_cast<const __half*>(a.w);
  const int ra = row0 + g, rb = row0 + g + 8;
  const __half* wa = W + (size_t)(ra < a.N ? ra : 0) * K + 8 * t;
  const __half* wb = W + (size_t)(rb < a.N ? rb : 0) * K + 8 * t;
  const __half* xr[NT];
  bool xv[NT];
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int b = n * 8 + g;
    xv[n] = b < NB;
    xr[n] = a.x + (size_t)(xv[n] ? b : 0) * a.ldx + 8 * t;
  }
  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[n][q] = 0.f;
  pdl_wait();
  const int nchunk = K / 32;
  for (int c0 = 0; c0 < nchunk; c0 += U) {
    uint4 A0[U], A1[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u;
      A0[u] = c < nchunk ? ldg_stream(wa + (size_t)c * 32) : make_uint4(0u, 0u, 0u, 0u);
      A1[u] = c < nchunk ? ldg_stream(wb + (size_t)c * 32) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u;
      if (c >= nchunk) break;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint4 xq = xv[n] ? *reinterpret_cast<const uint4*>(xr[n] + (size_t)c * 32) : make_uint4(0u, 0u, 0u, 0u);
        // k-step 0: elements 0..3 of each lane's 8; k-step 1: elements 4..7
        const uint32_t f0[4] = {A0[u].x, A1[u].x, A0[u].y, A1[u].y};
        const uint32_t f1[4] = {A0[u].z, A1[u].z, A0[u].w, A1[u].w};
        mma_16816(acc[n], f0, xq.x, xq.y);
        mma_16816(acc[n], f1, xq.z, xq.w);
      }
    }
  }
  pdl_trigger();
  // ---- this warp's rows: logits, then the best (value, row) per batch column over its 16 rows
  __shared__ float cv[NW][16];
  __shared__ int ci[NW][16];
#pragma unroll
  for (int n = 0; n < NT; ++n) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int b = n * 8 + 2 * t + h;
      float v0 = acc[n][h], v1 = acc[n][2 + h];           // rows ra, rb
      if (a.y && b < NB) {
        if (ra < a.N) reinterpret_cast<float*>(a.y)[(size_t)b * a.ldy + ra] = v0;
        if (rb < a.N) reinterpret_cast<float*>(a.y)[(size_t)b * a.ldy + rb] = v1;
      }
      float best = ra < a.N ? v0 : -INFINITY;
      int bi = ra < a.N ? ra : 0x7fffffff;
      if (rb < a.N && (v1 > best || bi == 0x7fffffff)) { best = v1; bi = rb; }
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {                  // over g: lanes with the same t
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
      }
      if (g == 0 && b < 16) { cv[warp][b] = best; ci[warp][b] = bi; }
    }
  }
  __syncthreads();
  if (threadIdx.x < NB) {
    const int b = threadIdx.x;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int w = 0; w < NW; ++w)
      if (cv[w][b] > best || (cv[w][b] == best && ci[w][b] < bi)) { best = cv[w][b]; bi = ci[w][b]; }
    a.am_val[(size_t)blockIdx.x * NB + b] = best;
    a.am_idx[(size_t)blockIdx.x * NB + b] = bi;
  }
  __threadfence();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = (atomicAdd(a.am_count, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  // the last CTA: one warp per batch column merges the CTAs' candidates in index order
  for (int b = warp; b < NB; b += NW) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = lane; j < (int)gridDim.x; j += 32) {
      const float v = __ldcg(a.am_val + (size_t)j * NB + b);
      const int ix = __ldcg(a.am_idx + (size_t)j * NB + b);
      if (v > best || (v == best && ix < bi)) { best = v; bi = ix; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) {
      a.tok_out[b] = bi + a.idx_base;
      if (a.val_out) a.val_out[b] = best;
      if (a.pos_adv) {
        const int p = __ldcg(a.pos_adv + b);
        if (a.hist && p >= 0 && p < a.hist_ld) a.hist[(size_t)b * a.hist_ld + p] = bi;
        a.pos_adv[b] = p + 1;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *a.am_count = 0;
}

static int lm_head_tc_ctas(int N) { return (N + 127) / 128; }

static bool lm_head_tc_ok(const GemvArgs& a) {
  static const int on = env_int("AF_LM_HEAD_TC", 1);
  return on && a.wf == W_F16 && a.epi == EPI_ARGMAX && a.NB >= 2 && a.NB <= 16 && a.K % 32 == 0 && a.ldx % 8 == 0 &&
         !a.scale && !a.bias && (reinterpret_cast<uintptr_t>(a.w) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
}

static cudaError_t lm_head_tc_launch(const GemvArgs& a, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(lm_head_tc_ctas(a.N));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = a.NB <= 8 ? cudaLaunchKernelEx(&cfg, lm_head_tc_kernel<1>, a) : cudaLaunchKernelEx(&cfg, lm_head_tc_kernel<2>, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <int WF, int NB, int R, int EPI>
static cudaError_t launch_one(const GemvArgs& a, int ctas, size_t smem, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<WF, NB, R, EPI>, a);
}

// Threads per row group: the power of two in [32, 256] covering a row's chunks, so that groups tile
// the 256-thread CTA exactly (a group size that does not divide 256 would leave a partial group).
static int pick_tg(int nch) {
  int tg = 32;
  while (tg < 256 && tg < nch) tg *= 2;
  return tg;
}

template <int WF, int NB, int EPI>
static cudaError_t dispatch_r(GemvArgs a, cudaStream_t st, bool pdl) {
  constexpr int EPC = WTraits<WF>::EPC;
  const int nch = a.K / EPC;
  const int tg = pick_tg(nch);
  a.tg = tg;
  const int G = 256 / tg;
  constexpr int R = rows_per_group(NB, EPI);
  const int rows_per_cta = G * R;
  const int ctas = (a.N + rows_per_cta - 1) / rows_per_cta;
  size_t smem = (size_t)G * (tg / 32) * R * NB * sizeof(float);
  if (EPI == EPI_ARGMAX) smem += (size_t)G * R * NB * sizeof(float);
  if (EPI == EPI_ARGMAX && a.am_grid_cap && ctas > a.am_grid_cap) return cudaErrorInvalidValue;
  return launch_one<WF, NB, R, EPI>(a, ctas, smem, st, pdl);
}

template <int WF, int EPI>
static cudaError_t dispatch_nb(const GemvArgs& a, int tmpl, cudaStream_t st, bool pdl) {
  switch (tmpl) {
    case 1: return dispatch_r<WF, 1, EPI>(a, st, pdl);
    case 2: return dispatch_r<WF, 2, EPI>(a, st, pdl);
    case 4: return dispatch_r<WF, 4, EPI>(a, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

// Compile-time batch width used for a tile of `nb_tile` rows of a launch over `nb_total` rows.
// The argmax path keeps one width for every tile so all tiles share one partial-slot layout.
static int tile_template(int epi, int nb_tile, int nb_total) {
  if (epi == EPI_ARGMAX) return nb_total == 1 ? 1 : 4;
  return nb_tile == 1 ? 1 : (nb_tile == 2 ? 2 : 4);
}

// Host entry: the batch is processed in tiles of up to 4 rows of x (weights re-streamed per tile).
// Argmax tiles each own a counter and a partial region of the scratch (see gemv_argmax_scratch).
cudaError_t gemv_launch(const GemvArgs& a0, cudaStream_t st, bool pdl) {
  if (a0.wf == W_SPARSE) return gemv_sparse_launch(a0, st, pdl);
  if (a0.K % chunk_elems(a0.wf)) return cudaErrorInvalidValue;
  if (a0.wf == W_I8G && (a0.group < 16 || a0.group % 16 || a0.K % a0.group)) return cudaErrorInvalidValue;
  if ((a0.wf == W_LUT4 || a0.wf == W_I8G) && (!a0.gscale || a0.epi == EPI_ARGMAX)) return cudaErrorInvalidValue;
  if (a0.NB < 1) return cudaErrorInvalidValue;
  // one launch over every row (gemv_argmax_scratch sizes the partial slots for it too)
  if (lm_head_tc_ok(a0)) return lm_head_tc_launch(a0, st, pdl);
  const int ctas_am = a0.epi == EPI_ARGMAX ? gemv_argmax_ctas(a0.wf, a0.N, a0.K, a0.NB) : 0;
  for (int b0 = 0, t = 0; b0 < a0.NB; b0 += 4, ++t) {
    GemvArgs a = a0;
    a.NB = a0.NB - b0 < 4 ? a0.NB - b0 : 4;
    a.x = a0.x + (size_t)b0 * a0.ldx;
    const size_t esz = (a0.epi == EPI_F16 || a0.epi == EPI_SWIGLU) ? 2 : 4;
    if (a0.y) a.y = (char*)a0.y + (size_t)b0 * a0.ldy * esz;
    if (a0.epi == EPI_ARGMAX) {
      a.am_count = a0.am_count + t;
      a.am_val = a0.am_val + (size_t)t * ctas_am * 4;
      a.am_idx = a0.am_idx + (size_t)t * ctas_am * 4;
      a.tok_out = a0.tok_out + b0;
      if (a0.val_out) a.val_out = a0.val_out + b0;
      if (a0.pos_adv) a.pos_adv = a0.pos_adv + b0;
      if (a0.hist) a.hist = a0.hist + (size_t)b0 * a0.hist_ld;
    }
    const int tmpl = tile_template(a0.epi, a.NB, a0.NB);
    cudaError_t e = cudaSuccess;
#define AF_GEMV_CASE(WFV, EPIV) \
  if (a.wf == WFV && a.epi == EPIV) e = dispatch_nb<WFV, EPIV>(a, tmpl, st, pdl && b0 == 0);
    AF_GEMV_CASE(W_I8, EPI_F32)
    AF_GEMV_CASE(W_I8, EPI_F16)
    AF_GEMV_CASE(W_I8, EPI_RESID)
    AF_GEMV_CASE(W_I8, EPI_SWIGLU)
    AF_GEMV_CASE(W_I8, EPI_ARGMAX)
    AF_GEMV_CASE(W_F16, EPI_F32)
    AF_GEMV_CASE(W_F16, EPI_F16)
    AF_GEMV_CASE(W_F16, EPI_RESID)
    AF_GEMV_CASE(W_F16, EPI_SWIGLU)
    AF_GEMV_CASE(W_F16, EPI_ARGMAX)
    AF_GEMV_CASE(W_I4G32, EPI_F32)
    AF_GEMV_CASE(W_I4G32, EPI_F16)
    AF_GEMV_CASE(W_I4G32, EPI_RESID)
    AF_GEMV_CASE(W_I4G32, EPI_SWIGLU)
    AF_GEMV_CASE(W_LUT4, EPI_F32)
    AF_GEMV_CASE(W_LUT4, EPI_F16)
    AF_GEMV_CASE(W_LUT4, EPI_RESID)
    AF_GEMV_CASE(W_LUT4, EPI_SWIGLU)
    AF_GEMV_CASE(W_I8G, EPI_F32)
    AF_GEMV_CASE(W_I8G, EPI_F16)
    AF_GEMV_CASE(W_I8G, EPI_RESID)
    AF_GEMV_CASE(W_I8G, EPI_SWIGLU)
#undef AF_GEMV_CASE
    if (e != cudaSuccess) return e;
  }
  return cudaGetLastError();
}

// Number of CTAs of one argmax tile launch (every tile of a launch uses the same width).
int gemv_argmax_ctas(int wf, int N, int K, int NB) {
  const int tg = pick_tg(K / chunk_elems(wf));
  const int G = 256 / tg;
  const int R = rows_per_group(tile_template(EPI_ARGMAX, NB < 4 ? NB : 4, NB), EPI_ARGMAX);
  return (N + G * R - 1) / (G * R);
}

// Scratch an argmax launch over NB rows needs: partial (value, index) slots per tile and a counter
// per tile. Counters must be zero before the first launch; the kernel leaves them at zero.
void gemv_argmax_scratch(int wf, int N, int K, int NB, size_t* slot_floats, size_t* counters) {
  const int tiles = (NB + 3) / 4;
  *slot_floats = (size_t)tiles * gemv_argmax_ctas(wf, N, K, NB) * 4;
  const size_t tc = (size_t)lm_head_tc_ctas(N) * NB;       // the tensor-core head's slots
  if (tc > *slot_floats) *slot_floats = tc;
  *counters = (size_t)tiles;
}

}  // namespace af
