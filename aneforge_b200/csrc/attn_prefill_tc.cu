// Prefill causal attention on the 5th-generation tensor cores (head dim 128), flash-attention style:
// one CTA per (query head, 128 query rows), the head's kv group streamed in 128-key blocks.
//
//   S_j  = Q K_j^T        tcgen05.mma M=128 N=128 K=16 x 8, Q and K K-major in shared memory, S in
//                         tensor memory (fp32, two 128-column buffers)
//   P_j  = exp(S_j - m)   four softmax warps, one thread per query row (its TMEM lane): the row
//                         maximum, the exponentials (rounded to fp16, the MMA operand) written into
//                         a K-major 128-byte-swizzled tile, the row sum
//   O   += P_j V_j        tcgen05.mma with V as an MN-major operand: the TMA copy of a {64 dh, 128
//                         keys} box of the cache IS the MN-major swizzled layout, so V needs no
//                         transpose; O accumulates in tensor memory (fp32, 128 columns)
//   before O += P_j V_j   the softmax thread rescales its O row in tensor memory by
//                         exp(m_old - m_new) once the previous block's MMAs are done (skipped when
//                         no row of the warp moved its maximum); at the end O / l is stored as fp16
//                         [S][H * dh].
//
// Roles (192 threads): warps 0-3 softmax + output; warp 4 owns the tensor memory (all 512 columns)
// and one thread issues the MMAs; warp 5 one thread issues the TMA copies (Q once, K and V per block
// into a two-stage ring). Blocks past the diagonal are never visited; the diagonal block masks keys
// above the row. Rows past the prompt read zeros (tensor-map bounds), so masked keys meet finite V.
// Every wait is bounded (iterations and ~2 s of wall clock); on a timeout the CTA records
// AF_DEV_WAIT_TIMEOUT, waits (bounded) for the MMAs and copies it issued, frees its tensor memory and
// returns. Every copy lands in this CTA's own shared memory (no multicast).
#include <cuda.h>

#include "af_common.cuh"
#include "af_kernels.h"
#include "tcgen05.cuh"

namespace af {

namespace fa5 {
constexpr int BQ = 128, BK = 128, DH = 128;
constexpr int SLICE = 128 * 64 * 2;           // 16 KB: 128 rows x 64 fp16, 128-byte swizzled
constexpr int TILE = 2 * SLICE;               // a 128 x 128 operand (two slices along the 128)
constexpr int Q_OFF = 0;
constexpr int K_OFF = Q_OFF + TILE;           // two stages
constexpr int V_OFF = K_OFF + 2 * TILE;       // two stages
constexpr int P_OFF = V_OFF + 2 * TILE;       // two buffers
constexpr int BAR_OFF = P_OFF + 2 * TILE;     // 224 KB of operands, then the barriers
constexpr int THREADS = 192;
constexpr int MMA_WARP = 4, TMA_WARP = 5;
constexpr uint32_t S_COL = 0, O_COL = 256;    // TMEM columns: S buffers 0 / 128, the O accumulator 256
constexpr long long LIMIT = 1ll << 26;
// kind::f16, fp16 A and B, fp32 accumulate, M = 128, N = 128; PV: B (V) MN-major
constexpr uint32_t IDESC_S = (1u << 4) | ((uint32_t)(128 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
constexpr uint32_t IDESC_PV = IDESC_S | (1u << 16);
}  // namespace fa5

struct Fa5Shared {
  uint64_t q_full;
  uint64_t k_full[2], v_full[2];    // TMA bytes landed
  uint64_t kv_empty[2];             // the block's PV MMAs (its last reader) finished
  uint64_t s_full[2];               // S_j in tensor memory
  uint64_t p_full[2];               // P_j in shared memory (softmax threads, 128 arrivals)
  uint64_t o_full;                  // O += P_j V_j finished (once per block)
  uint64_t done;                    // every MMA issued has finished
  uint32_t tmem;
  int abort;
};
constexpr size_t FA5_SMEM = fa5::BAR_OFF + sizeof(Fa5Shared) + 1024;   // + alignment slack

AF_DEV bool fa5_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  SpinBudget budget;
  for (long long i = 0; i < fa5::LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 255 && (*abort || budget.spent())) return false;
  }
  return false;
}

// the same wait in every lane of a warp, with one outcome for all of them (the tensor-memory loads
// and stores that follow are warp-collective)
AF_DEV bool fa5_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort) {
  return __all_sync(0xffffffffu, fa5_wait(bar, parity, abort));
}

AF_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// qmap: q [H][S][128] fp16; kmap / vmap: K / V [KV][rows][128] fp16 (rows past S read as zeros)
__global__ void __launch_bounds__(fa5::THREADS, 1)
    attn_prefill_tc_kernel(AttnPrefillArgs a, const __grid_constant__ CUtensorMap qmap,
                           const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
  using namespace fa5;
  extern __shared__ unsigned char fa5_raw[];
  const uint32_t raw = smem_u32(fa5_raw);
  unsigned char* smem = fa5_raw + ((1024u - (raw & 1023u)) & 1023u);
  Fa5Shared* sh = reinterpret_cast<Fa5Shared*>(smem + BAR_OFF);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the last query tiles see the most keys: they take the lowest block indices, so they start first
  const int h = blockIdx.x, qt = gridDim.y - 1 - blockIdx.y, q0 = qt * BQ;
  const int G = a.H / a.KV, kvh = h / G;
  const int nblk = qt + 1;                                   // key blocks 0..qt (BK == BQ)

  if (threadIdx.x == 0) {
    mbar_init(&sh->q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sh->k_full[s], 1);
      mbar_init(&sh->v_full[s], 1);
      mbar_init(&sh->kv_empty[s], 1);
      mbar_init(&sh->s_full[s], 1);
      mbar_init(&sh->p_full[s], 128);
    }
    mbar_init(&sh->o_full, 1);
    mbar_init(&sh->done, 1);
    sh->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&sh->tmem)), "r"(512) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = sh->tmem;
  volatile int* abort = &sh->abort;

  if (warp == TMA_WARP) {
    // ------------------------------------------------------------- TMA copies (one thread)
    if (lane == 0) {
      pdl_wait();                                            // q, K, V come from the rope kernel
      mbar_arrive_expect_tx(&sh->q_full, TILE);
      tma_load_3d(smem + Q_OFF, &qmap, 0, q0, h, &sh->q_full);
      tma_load_3d(smem + Q_OFF + SLICE, &qmap, 64, q0, h, &sh->q_full);
      int issued = 0;
      for (int j = 0; j < nblk; ++j) {
        const int st = j & 1;
        if (j >= 2 && !fa5_wait(&sh->kv_empty[st], (uint32_t)(((j >> 1) - 1) & 1), abort)) {
          *abort = 1;
          break;
        }
        unsigned char* kd = smem + K_OFF + st * TILE;
        unsigned char* vd = smem + V_OFF + st * TILE;
        mbar_arrive_expect_tx(&sh->k_full[st], TILE);
        tma_load_3d(kd, &kmap, 0, j * BK, kvh, &sh->k_full[st]);
        tma_load_3d(kd + SLICE, &kmap, 64, j * BK, kvh, &sh->k_full[st]);
        mbar_arrive_expect_tx(&sh->v_full[st], TILE);
        tma_load_3d(vd, &vmap, 0, j * BK, kvh, &sh->v_full[st]);
        tma_load_3d(vd + SLICE, &vmap, 64, j * BK, kvh, &sh->v_full[st]);
        issued = j + 1;
      }
      // shared memory must outlive every copy issued: wait (time-bounded only) for the last ones
      SpinBudget b;
      while (!mbar_try_wait(&sh->q_full, 0) && !b.spent()) {
      }
      for (int j = issued - 1; j >= 0 && j >= issued - 2; --j) {
        const uint32_t par = (uint32_t)((j >> 1) & 1);
        SpinBudget b2;
        while (!(mbar_try_wait(&sh->k_full[j & 1], par) && mbar_try_wait(&sh->v_full[j & 1], par)) && !b2.spent()) {
        }
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------- MMA issuer (one thread)
    if (lane == 0) {
      const uint32_t qa = smem_u32(smem + Q_OFF);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!fa5_wait(&sh->k_full[st], (uint32_t)((j >> 1) & 1), abort)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t kb = smem_u32(smem + K_OFF + st * TILE);
#pragma unroll
        for (int ks = 0; ks < DH / 16; ++ks) {
          const uint32_t off = (uint32_t)((ks >> 2) * SLICE + (ks & 3) * 32);
          mma_f16(tmem + S_COL + (uint32_t)(st * 128), smem_desc(qa + off), smem_desc(kb + off), IDESC_S, ks != 0);
        }
        mma_commit(&sh->s_full[st]);
        return true;
      };
      bool ok = fa5_wait(&sh->q_full, 0, abort) && issue_s(0) && (nblk < 2 || issue_s(1));
      for (int j = 0; ok && j < nblk; ++j) {
        const int b = j & 1;
        const uint32_t par = (uint32_t)((j >> 1) & 1);
        if (!fa5_wait(&sh->v_full[b], par, abort) || !fa5_wait(&sh->p_full[b], par, abort)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t pa = smem_u32(smem + P_OFF + b * TILE);
        const uint32_t vb = smem_u32(smem + V_OFF + b * TILE);
#pragma unroll
        for (int ks = 0; ks < BK / 16; ++ks)
          mma_f16(tmem + O_COL, smem_desc(pa + (uint32_t)((ks >> 2) * SLICE + (ks & 3) * 32)),
                  smem_desc_mn(vb + (uint32_t)(ks * 2048), SLICE, 1024), IDESC_PV, (j | ks) != 0);
        mma_commit(&sh->o_full);
        mma_commit(&sh->kv_empty[b]);
        if (j + 2 < nblk && !issue_s(j + 2)) ok = false;   // S buffer b: P_j is written, S_j read
      }
      if (!ok) *abort = 1;
      // completes once every MMA issued so far has finished (also on abort, so that the tensor
      // memory is idle before it is freed)
      mma_commit(&sh->done);
    }
  } else {
    // ------------------------------------------------------------- softmax + output (warps 0-3)
    const int r = warp * 32 + lane;                          // query row in the tile = TMEM lane
    const int row = q0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const float sl2 = a.scale * 1.4426950408889634f;         // scores in the exp2 domain
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int b = j & 1;
      if (!fa5_wait_warp(&sh->s_full[b], (uint32_t)((j >> 1) & 1), abort)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t sbase = lane_base + S_COL + (uint32_t)(b * 128);
      const int klim = j == nblk - 1 ? row - j * BK : BK;    // keys 0..klim of the block are visible
      float bm = -INFINITY;
#pragma unroll
      for (int c0 = 0; c0 < BK; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(sbase + (uint32_t)c0, v);
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (c0 + e <= klim) bm = fmaxf(bm, __uint_as_float(v[e]) * sl2);
      }
      const float mn = fmaxf(m, bm);                         // finite: key j * BK <= row is visible
      const float corr = ex2_approx(m - mn);                 // 0 on the first block (m = -inf)
      unsigned char* pt = smem + P_OFF + b * TILE;
      float ps = 0.f;
#pragma unroll
      for (int c0 = 0; c0 < BK; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(sbase + (uint32_t)c0, v);
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float p0 = c0 + e <= klim ? ex2_approx(fmaf(__uint_as_float(v[e]), sl2, -mn)) : 0.f;
          const float p1 = c0 + e + 1 <= klim ? ex2_approx(fmaf(__uint_as_float(v[e + 1]), sl2, -mn)) : 0.f;
          ps += p0 + p1;
          const __half2 hp = __floats2half2_rn(p0, p1);
          pk[e >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = (c0 >> 3) + q;                   // 8 keys per 16-byte chunk
          *reinterpret_cast<uint4*>(pt + (chunk >> 3) * SLICE + sw128(r, chunk & 7)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      l = l * corr + ps;
      m = mn;
      if (j >= 1) {
        // O holds blocks 0..j-1 against the old maximum: once their MMAs are done, rescale the rows
        // whose maximum moved (skipped for a warp whose 32 rows all kept theirs)
        if (!fa5_wait_warp(&sh->o_full, (uint32_t)((j - 1) & 1), abort)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (!__all_sync(0xffffffffu, corr == 1.f)) {
#pragma unroll
          for (int c0 = 0; c0 < DH; c0 += 32) {
            uint32_t v[32];
            tmem_ld32(lane_base + O_COL + (uint32_t)c0, v);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * corr);
            tmem_st32(lane_base + O_COL + (uint32_t)c0, v);
          }
        }
      }
      // generic-proxy P stores -> visible to the tensor core's async proxy; this thread's tensor
      // memory reads and writes ordered before the MMAs the barrier releases
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&sh->p_full[b]);
    }
    if (ok) {
      ok = fa5_wait_warp(&sh->o_full, (uint32_t)((nblk - 1) & 1), abort);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    }
    if (!ok) {
      *abort = 1;
      af_set_err(a.err, AF_DEV_WAIT_TIMEOUT);
    } else {
      const float il = l > 0.f ? 1.f / l : 0.f;
      __half* dst = a.out + (size_t)row * a.H * DH + (size_t)h * DH;
#pragma unroll
      for (int c0 = 0; c0 < DH; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(lane_base + O_COL + (uint32_t)c0, v);      // warp-collective: every lane loads
        if (row < a.S) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const __half2 hv = __floats2half2_rn(__uint_as_float(v[8 * q + 2 * i]) * il,
                                                   __uint_as_float(v[8 * q + 2 * i + 1]) * il);
              w[i] = *reinterpret_cast<const uint32_t*>(&hv);
            }
            *reinterpret_cast<uint4*>(dst + c0 + 8 * q) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
  }
  // the tensor memory is freed only once the MMAs are idle
  if (warp == MMA_WARP) {
    SpinBudget b;
    if (lane == 0)
      while (!mbar_try_wait(&sh->done, 0) && !b.spent()) {
      }
    __syncwarp();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

// fp16 [planes][rows][128] with row stride 256 bytes and plane stride `plane_rows` rows: 64 x 128 x 1
// boxes, 128-byte swizzle, rows past `rows` read as zeros
static bool make_map3(CUtensorMap* map, const __half* base, int rows, size_t plane_rows, int planes) {
  const EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  const cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)planes};
  const cuuint64_t strides[2] = {256, (cuuint64_t)plane_rows * 256};
  const cuuint32_t box[3] = {64, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool attn_prefill_tc_ok(const AttnPrefillArgs& a) {
  return a.dh == 128 && a.S >= 1 && a.KV > 0 && a.H % a.KV == 0 && (!a.expand || a.kvx) &&
         (reinterpret_cast<uintptr_t>(a.kc) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.vc) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.kvx) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0;
}

cudaError_t attn_prefill_tc_launch(const AttnPrefillArgs& a, const __half* qbuf, cudaStream_t st) {
  if (!attn_prefill_tc_ok(a) || (reinterpret_cast<uintptr_t>(qbuf) & 15)) return cudaErrorInvalidValue;
  CUtensorMap qmap, kmap, vmap;
  // expanded copies ([2][KV][S][128], written by the rope kernel) when the GQA factor applies
  const __half* kb = a.expand ? a.kvx : a.kc;
  const __half* vb = a.expand ? a.kvx + (size_t)a.KV * a.S * 128 : a.vc;
  const size_t plane = a.expand ? (size_t)a.S : (size_t)a.ldm;
  if (!make_map3(&qmap, qbuf, a.S, a.S, a.H) || !make_map3(&kmap, kb, a.S, plane, a.KV) ||
      !make_map3(&vmap, vb, a.S, plane, a.KV))
    return cudaErrorInvalidValue;
  static PerDeviceOnce attrs;
  const cudaError_t ae = attrs.run([] {
    return cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FA5_SMEM);
  });
  if (ae != cudaSuccess) return ae;
  attn_prefill_tc_kernel<<<dim3(a.H, (a.S + fa5::BQ - 1) / fa5::BQ), fa5::THREADS, FA5_SMEM, st>>>(a, qmap, kmap,
                                                                                                 vmap);
  return cudaGetLastError();
}

}  // namespace af
