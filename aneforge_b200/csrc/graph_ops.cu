// Generic graph ops: the kernels `compile(graph)` lowers an arbitrary graph of the reference's IR
// (aneforge/graph.py) onto when no fused kernel covers a node. They keep the reference graph's
// value semantics as the oracle states them: every value is fp32 in device memory, ports are fp16,
// and the activation operands of a matmul (x of `linear`, both operands of `bmm`) are rounded to
// fp16 first - what the fp16 operand ports of the fused kernels (and of the ANE) see.
//
// Shapes are at most rank 5 (the reference's limit, graph.py:37-41). An N-d operand is described by
// the output shape plus one element stride per axis (0 on a broadcast axis), so one kernel serves
// broadcasting, transposes, slices and concatenation (a copy into a strided window of the output).
// These kernels are correctness-first: one thread per output element (a warp per row for the row
// reductions, a warp per output column group for `linear`), grid-stride loops, no shared state
// between threads beyond warp shuffles; the decode / prefill hot path never runs them (its graphs
// lower onto the fused kernels).
#include <cmath>

#include "af_common.cuh"
#include "af_kernels.h"

namespace af {

namespace {

constexpr int R = GRAPH_MAX_RANK;

struct Nd {
  int rank;
  long long shape[R];
};

// element offset of flat output index i under per-axis strides
AF_DEV long long nd_offset(long long i, const long long (&shape)[R], const long long (&stride)[R], int rank) {
  long long off = 0;
  for (int d = rank - 1; d >= 0; --d) {
    const long long c = i % shape[d];
    i /= shape[d];
    off += c * stride[d];
  }
  return off;
}

AF_DEV float f16_round(float x) { return __half2float(__float2half_rn(x)); }

AF_DEV float apply_binary(int op, float a, float b) {
  switch (op) {
    case G_ADD: return a + b;
    case G_SUB: return a - b;
    case G_MUL: return a * b;
    case G_DIV: return a / b;
    case G_MAX: return fmaxf(a, b);
    case G_MIN: return fminf(a, b);
    case G_POW: return powf(a, b);
    case G_GT: return a > b ? 1.f : 0.f;
    case G_GE: return a >= b ? 1.f : 0.f;
    case G_LT: return a < b ? 1.f : 0.f;
    case G_LE: return a <= b ? 1.f : 0.f;
    case G_EQ: return a == b ? 1.f : 0.f;
    case G_NE: return a != b ? 1.f : 0.f;
    default: return 0.f;
  }
}

AF_DEV float apply_unary(int op, float x, float k, float k2) {
  switch (op) {
    case U_RELU: return fmaxf(x, 0.f);
    case U_SILU: return x / (1.f + expf(-x));
    case U_SIGMOID: return 1.f / (1.f + expf(-x));
    case U_TANH: return tanhf(x);
    case U_EXP: return expf(x);
    case U_SQRT: return sqrtf(x);
    case U_ABS: return fabsf(x);
    case U_SQUARE: return x * x;
    case U_SIN: return sinf(x);
    case U_COS: return cosf(x);
    case U_ERF: return erff(x);
    case U_LOG: return logf(x + k);
    case U_RSQRT: return rsqrtf(x + k);
    case U_INV: return 1.f / (x + k);
    case U_MULS: return x * k;
    case U_ADDS: return x + k;
    case U_CLIP: return fminf(fmaxf(x, k), k2);
    case U_NOT: return x == 0.f ? 1.f : 0.f;
    case U_FLOOR: return floorf(x);
    case U_CEIL: return ceilf(x);
    case U_ROUND: return rintf(x);
    case U_SIGN: return x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
    case U_GELU_TANH: {
      const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
      return 0.5f * x * (1.f + tanhf(u));
    }
    case U_GELU: return 0.5f * x * (1.f + erff(x * 0.7071067811865476f));
    case U_SOFTPLUS: return x > 20.f ? x : log1pf(expf(x));
    default: return x;
  }
}

__global__ void ew_kernel(GraphEwArgs a) {
  const long long n = a.n;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float va = a.a[nd_offset(i, a.shape, a.sa, a.rank)];
    const float vb = a.b ? a.b[nd_offset(i, a.shape, a.sb, a.rank)] : 0.f;
    float r;
    if (a.op == G_SELECT) {
      const float vc = a.c[nd_offset(i, a.shape, a.sc, a.rank)];
      r = va != 0.f ? vb : vc;
    } else {
      r = apply_binary(a.op, va, vb);
    }
    a.y[i] = r;
  }
}

__global__ void unary_kernel(const float* x, float* y, long long n, int op, float k, float k2) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = apply_unary(op, x[i], k, k2);
}

// y[dst window] = x[src view]: both described by the copied shape and per-axis strides
__global__ void copy_kernel(GraphCopyArgs a) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += (long long)gridDim.x * blockDim.x)
    a.y[nd_offset(i, a.shape, a.sy, a.rank)] = a.x[nd_offset(i, a.shape, a.sx, a.rank)];
}

// reduce over the axes in `mask` of a contiguous input of shape a.shape; output contiguous with those
// axes of size 1. One thread per output element walks the reduced index space in order.
__global__ void reduce_kernel(GraphReduceArgs a) {
  long long in_stride[R];
  long long s = 1;
  for (int d = a.rank - 1; d >= 0; --d) { in_stride[d] = s; s *= a.shape[d]; }
  long long oshape[R], red_count = 1;
  for (int d = 0; d < a.rank; ++d) {
    const bool r = (a.mask >> d) & 1;
    oshape[d] = r ? 1 : a.shape[d];
    if (r) red_count *= a.shape[d];
  }
  for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < a.n_out; o += (long long)gridDim.x * blockDim.x) {
    long long base = 0, t = o;
    for (int d = a.rank - 1; d >= 0; --d) {
      const long long c = t % oshape[d];
      t /= oshape[d];
      base += c * in_stride[d];
    }
    float acc = a.op == RD_MAX ? -INFINITY : (a.op == RD_MIN ? INFINITY : 0.f);
    for (long long j = 0; j < red_count; ++j) {
      long long off = base, u = j;
      for (int d = a.rank - 1; d >= 0; --d) {
        if (!((a.mask >> d) & 1)) continue;
        const long long c = u % a.shape[d];
        u /= a.shape[d];
        off += c * in_stride[d];
      }
      const float v = a.x[off];
      switch (a.op) {
        case RD_SUM: case RD_MEAN: acc += v; break;
        case RD_MAX: acc = fmaxf(acc, v); break;
        case RD_MIN: acc = fminf(acc, v); break;
        case RD_SUMSQ: case RD_L2: acc = fmaf(v, v, acc); break;
        case RD_L1: acc += fabsf(v); break;
        default: break;
      }
    }
    if (a.op == RD_MEAN) acc /= (float)red_count;
    if (a.op == RD_L2) acc = sqrtf(acc);
    a.y[o] = acc;
  }
}

// softmax over the middle axis of [outer][n][inner]: one thread per (outer, inner) column
__global__ void softmax_kernel(const float* x, float* y, long long outer, long long n, long long inner) {
  const long long cols = outer * inner;
  for (long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += (long long)gridDim.x * blockDim.x) {
    const long long o = c / inner, in = c - o * inner;
    const float* xp = x + o * n * inner + in;
    float* yp = y + o * n * inner + in;
    float m = -INFINITY;
    for (long long j = 0; j < n; ++j) m = fmaxf(m, xp[j * inner]);
    float sum = 0.f;
    for (long long j = 0; j < n; ++j) sum += expf(xp[j * inner] - m);
    const float inv = 1.f / sum;
    for (long long j = 0; j < n; ++j) yp[j * inner] = expf(xp[j * inner] - m) * inv;
  }
}

// the reference RMSNorm over the last axis: x / max(||x||_2, floor) * g_eff (one warp per row)
__global__ void rms_kernel(const float* x, float* y, const __half* g, float floor, long long rows, int d) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const float* xr = x + r * d;
    float ss = 0.f;
    for (int j = lane; j < d; j += 32) ss = fmaf(xr[j], xr[j], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float den = fmaxf(sqrtf(ss), floor);
    for (int j = lane; j < d; j += 32) y[r * d + j] = __fdiv_rn(xr[j], den) * __half2float(g[j]);
  }
}

// layer norm over the last axis: (x - mean) / sqrt(var + eps) * gamma + beta (one warp per row)
__global__ void layernorm_kernel(const float* x, float* y, const __half* g, const __half* b, float eps, long long rows,
                                 int d) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const float* xr = x + r * d;
    float s = 0.f;
    for (int j = lane; j < d; j += 32) s += xr[j];
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)d;
    float v = 0.f;
    for (int j = lane; j < d; j += 32) { const float t = xr[j] - mean; v = fmaf(t, t, v); }
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const float inv = rsqrtf(v / (float)d + eps);
    for (int j = lane; j < d; j += 32) {
      float t = (xr[j] - mean) * inv * __half2float(g[j]);
      if (b) t += __half2float(b[j]);
      y[r * d + j] = t;
    }
  }
}

// y[r][n] = (sum_k f16(x[r][k]) * W[n][k]) * scale[n] + bias[n]; W int8 codes with per-row fp16 scales,
// or fp16. One warp per (group of 4 rows, output column): the lanes split k, a shuffle reduces.
template <bool I8>
__global__ void linear_kernel(GraphLinearArgs a) {
  const int lane = threadIdx.x & 31;
  const long long rgroups = (a.rows + 3) / 4;
  const long long items = rgroups * a.N;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long it = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += warps) {
    const long long n = it % a.N, rg = it / a.N;
    const long long r0 = rg * 4;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (long long k = lane; k < a.K; k += 32) {
      const float w = I8 ? (float)reinterpret_cast<const int8_t*>(a.w)[n * a.K + k]
                         : __half2float(reinterpret_cast<const __half*>(a.w)[n * a.K + k]);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (r0 + j < a.rows) acc[j] = fmaf(f16_round(a.x[(r0 + j) * a.ldx + k]), w, acc[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int o = 16; o; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    }
    if (lane == 0) {
      const float s = a.scale ? __half2float(a.scale[n]) : 1.f;
      const float bb = a.bias ? __half2float(a.bias[n]) : 0.f;
      for (int j = 0; j < 4; ++j)
        if (r0 + j < a.rows) a.y[(r0 + j) * a.ldy + n] = (I8 ? acc[j] * s : acc[j]) + bb;
    }
  }
}

// batched matmul y[b][m][n] = sum_k f16(A[b][m][k]) * f16(B[b][k][n]); A and B addressed by per-axis
// strides over the output's batch axes (broadcast = stride 0) plus their own matrix strides
__global__ void bmm_kernel(GraphBmmArgs a) {
  const long long total = a.batch * a.M * a.N;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long n = i % a.N, m = (i / a.N) % a.M, bi = i / (a.N * a.M);
    const long long offa = nd_offset(bi, a.bshape, a.sa, a.brank) + m * a.sam;
    const long long offb = nd_offset(bi, a.bshape, a.sb, a.brank) + n * a.sbn;
    float acc = 0.f;
    for (long long k = 0; k < a.K; ++k)
      acc = fmaf(f16_round(a.a[offa + k * a.sak]), a.round_b ? f16_round(a.b[offb + k * a.sbk]) : a.b[offb + k * a.sbk],
                 acc);
    a.y[i] = acc;
  }
}

// The reference's per-step decode inputs (`aneforge/llm.py:585-590`) built on the device from the
// resident position: oh / inv (one-hot of pos over the M cache rows and its complement), the additive
// mask (0 up to pos, f16(-1e4) beyond) and the position's RoPE row (cos 1 / sin 0 without tables).
__global__ void decode_ctx_kernel(const int* pos, const __half* cos_t, const __half* sin_t, int M, int dh, float* oh,
                                  float* inv, float* mask, float* cosp, float* sinp) {
  const int p = *pos;
  const bool ok = p >= 0 && p < M;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < M; j += gridDim.x * blockDim.x) {
    const bool hit = ok && j == p;
    oh[j] = hit ? 1.f : 0.f;
    inv[j] = hit ? 0.f : 1.f;
    mask[j] = (ok && j <= p) ? 0.f : -10000.f;
  }
  if (blockIdx.x == 0)
    for (int d = threadIdx.x; d < dh; d += blockDim.x) {
      cosp[d] = (ok && cos_t) ? __half2float(cos_t[(size_t)p * dh + d]) : 1.f;
      sinp[d] = (ok && sin_t) ? __half2float(sin_t[(size_t)p * dh + d]) : 0.f;
    }
}

int grid_for(long long work, int per_block) {
  long long g = (work + per_block - 1) / per_block;
  if (g < 1) g = 1;
  if (g > 148 * 32) g = 148 * 32;
  return (int)g;
}

}  // namespace

cudaError_t graph_ew_launch(const GraphEwArgs& a, cudaStream_t st) {
  if (a.n <= 0) return cudaSuccess;
  ew_kernel<<<grid_for(a.n, 256), 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t graph_unary_launch(const float* x, float* y, long long n, int op, float k, float k2, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  unary_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, y, n, op, k, k2);
  return cudaGetLastError();
}

cudaError_t graph_copy_launch(const GraphCopyArgs& a, cudaStream_t st) {
  if (a.n <= 0) return cudaSuccess;
  copy_kernel<<<grid_for(a.n, 256), 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t graph_reduce_launch(const GraphReduceArgs& a, cudaStream_t st) {
  if (a.n_out <= 0) return cudaSuccess;
  reduce_kernel<<<grid_for(a.n_out, 128), 128, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t graph_softmax_launch(const float* x, float* y, long long outer, long long n, long long inner,
                                 cudaStream_t st) {
  if (outer * inner <= 0 || n <= 0) return cudaSuccess;
  softmax_kernel<<<grid_for(outer * inner, 128), 128, 0, st>>>(x, y, outer, n, inner);
  return cudaGetLastError();
}

cudaError_t graph_rms_launch(const float* x, float* y, const __half* g, float floor, long long rows, int d,
                             cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  rms_kernel<<<grid_for(rows * 32, 256), 256, 0, st>>>(x, y, g, floor, rows, d);
  return cudaGetLastError();
}

cudaError_t graph_layernorm_launch(const float* x, float* y, const __half* g, const __half* b, float eps, long long rows,
                                   int d, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  layernorm_kernel<<<grid_for(rows * 32, 256), 256, 0, st>>>(x, y, g, b, eps, rows, d);
  return cudaGetLastError();
}

cudaError_t graph_linear_launch(const GraphLinearArgs& a, cudaStream_t st) {
  if (a.rows <= 0 || a.N <= 0) return cudaSuccess;
  const long long warps = (a.rows + 3) / 4 * a.N;
  if (a.int8) linear_kernel<true><<<grid_for(warps * 32, 256), 256, 0, st>>>(a);
  else linear_kernel<false><<<grid_for(warps * 32, 256), 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t graph_decode_ctx_launch(const int* pos, const __half* cos_t, const __half* sin_t, int M, int dh, float* oh,
                                    float* inv, float* mask, float* cosp, float* sinp, cudaStream_t st) {
  if (M <= 0 || dh <= 0) return cudaErrorInvalidValue;
  decode_ctx_kernel<<<grid_for(M, 256), 256, 0, st>>>(pos, cos_t, sin_t, M, dh, oh, inv, mask, cosp, sinp);
  return cudaGetLastError();
}

cudaError_t graph_bmm_launch(const GraphBmmArgs& a, cudaStream_t st) {
  const long long total = a.batch * a.M * a.N;
  if (total <= 0) return cudaSuccess;
  bmm_kernel<<<grid_for(total, 128), 128, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace af
