// Prefill GEMM on the 5th-generation tensor cores: C[M, N] = X[M, K] . W[N, K]^T for the prompt rows
// of a prefill (M = prompt length), W the same packed int8 / group-32 int4 fragment tiles the decode
// GEMV streams, X fp16 activations.
//
// One CTA per 128 x 256 output tile (tcgen05.mma M=128, N=256, K=16 per instruction, fp32
// accumulators in tensor memory: 256 TMEM columns x 128 lanes). A 3-stage shared-memory ring holds
// 64-deep K slices of A (16 KB) and B (32 KB), both in the canonical K-major 128-byte-swizzled layout
// the MMA reads through shared-memory descriptors:
//   row r, 16-byte chunk c (8 fp16 along K) of a slice lives at (r / 8) * 1024 + (r % 8) * 128 +
//   ((c ^ (r % 8)) * 16)  - eight-row atoms 1024 bytes apart (the descriptor's stride offset).
// The raw packed weights have a ring of their own (4 x 16 KB), so their copies run ahead of the MMAs
// instead of waiting for a whole operand stage to free up.
// Roles: warp 13 (one thread) bulk-copies the raw packed weight units of each slice (4 row blocks x 2
// k tiles) into the raw ring, starting before the programmatic-launch wait; warp 14 (one thread)
// issues per slice a TMA tensor copy of the A tile (the copy engine applies the 128-byte swizzle;
// rows past M read as zeros); warps 0-11 turn the raw units into the fp16 B slice
// (a weight tile lane's 16 bytes are 2 rows x 8 consecutive columns - the GEMV's column permutation;
// int8 codes become exact fp16 by a byte permute under the exponent of 1024 and one subtract, the
// per-row scale is applied to the fp32 result; group-32 int4 codes become fp16 code * scale since
// the scale changes along K inside a slice); warp 12 owns the tensor memory and one of its threads
// issues the MMAs, committing each slice to its "empty" barrier and the last to the accumulator
// barrier. Warps 0-3 then read the accumulators (tcgen05.ld, 32 lanes each: one output row per
// lane) and run the GEMV's epilogues (F32 / F16 / RESID / SWIGLU); F32 / F16 / RESID stage each
// 32-column chunk in the idle operand ring so that their global loads and stores run along rows.
// Every wait is bounded; on a timeout the CTA records AF_DEV_WAIT_TIMEOUT, waits (bounded) for the
// MMAs it issued, frees its tensor memory and returns. Every copy lands in the issuing CTA's own
// shared memory.
#include <cuda.h>

#include "af_common.cuh"
#include "af_kernels.h"
#include "tc_common.cuh"
#include "tcgen05.cuh"

namespace af {

namespace gm {
constexpr int BM = 128, BN = 256, BK = 64;
constexpr int STAGES = 3;
constexpr int A_BYTES = BM * BK * 2;          // 16 KB
constexpr int B_BYTES = BN * BK * 2;          // 32 KB
constexpr int RAW_BYTES = (BN / 64) * 2 * tc::UNIT;   // 16 KB: raw int8 units of one slice (int4: less)
constexpr int STAGE = A_BYTES + B_BYTES;      // one slice's MMA operands
constexpr int RSTAGES = 4;                    // raw weight ring, ahead of the operand ring
constexpr int MAX_STAGES = 6, MAX_RSTAGES = 8;  // ring depths a kernel variant may use (below)
constexpr int CONV = 384;                     // warps 0-11 convert (three per SM sub-partition, to hide
                                              // each other's latency); warps 0-3 then run the epilogue
constexpr int MMA_WARP = CONV / 32;           // TMEM owner, MMA issuer
constexpr int RAW_WARP = MMA_WARP + 1;        // raw weight copies
constexpr int A_WARP = MMA_WARP + 2;          // A tiles
constexpr int THREADS = CONV + 96;
constexpr int TMEM_COLS = 256;
constexpr long long LIMIT = 1ll << 26;
}  // namespace gm

// per output-tile width: 256 columns (the default) or 128 (prompt-sized shapes with few tiles, so
// that more SMs get one)
template <int BNV>
struct Gt {
  static constexpr int BN = BNV;
  static constexpr int B_BYTES = BN * gm::BK * 2;
  static constexpr int RAW_BYTES = (BN / 64) * 2 * tc::UNIT;
  static constexpr int STAGE = gm::A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = BN;
  // kind::f16, fp16 A and B (K-major), fp32 accumulate, M = 128, N = BN
  static constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(gm::BM >> 4) << 24);
};

struct GemmShared {
  uint64_t raw_full[gm::MAX_RSTAGES];         // raw weight units landed (copy bytes)
  uint64_t raw_empty[gm::MAX_RSTAGES];        // the converters are done with them
  uint64_t a_full[gm::MAX_STAGES];            // A tile landed (TMA bytes)
  uint64_t full[gm::MAX_STAGES];              // fp16 B slice written (converters)
  uint64_t empty[gm::MAX_STAGES];             // the slice's MMAs finished reading (tcgen05.commit)
  uint64_t accum;
  uint32_t tmem;
  int abort;
};

AF_DEV bool gm_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  for (long long i = 0; i < gm::LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023) == 1023 && *abort) return false;
  }
  return false;
}

// group-32 int4: 8 nibbles of one k-step (fragment slot order of pack_i4_tiles) -> the lane's two
// rows' 4 values each, as code * scale in fp16
AF_DEV void i4_rows(uint32_t w, __half2 s_lo, __half2 s_hi, uint32_t& row_lo0, uint32_t& row_lo1, uint32_t& row_hi0,
                    uint32_t& row_hi1) {
  uint32_t A[4];
  i4x8_to_frag(w, A);                       // A0 = row g (c0, c1), A1 = row g+8 (c0, c1), A2 = row g (c2, c3), A3 = row g+8 (c2, c3)
  __half2 a0 = __hmul2(*reinterpret_cast<__half2*>(&A[0]), s_lo);
  __half2 a2 = __hmul2(*reinterpret_cast<__half2*>(&A[2]), s_lo);
  __half2 a1 = __hmul2(*reinterpret_cast<__half2*>(&A[1]), s_hi);
  __half2 a3 = __hmul2(*reinterpret_cast<__half2*>(&A[3]), s_hi);
  row_lo0 = *reinterpret_cast<uint32_t*>(&a0);
  row_lo1 = *reinterpret_cast<uint32_t*>(&a2);
  row_hi0 = *reinterpret_cast<uint32_t*>(&a1);
  row_hi1 = *reinterpret_cast<uint32_t*>(&a3);
}

// NS = operand ring depth (A + converted B slices), NR = raw weight ring depth. One k-slice takes
// about the same time (~1 µs on the 8B prompt shapes) whatever the tile width, so 128-column tiles
// run far below the tensor pipe's rate; deeper rings recover 10-15 % of that: 128-column tiles fit
// four operand and eight raw slices in shared memory, 256-column tiles three and four.
// MM = 128-row M tiles per CTA: with MM = 2 each converted B slice feeds two M tiles (two TMEM
// accumulators side by side), so every weight byte is dequantised once per 256 prompt rows.
template <bool I4, int BNV, int NS, int NR, int MM>
__global__ void __launch_bounds__(gm::THREADS, 1) gemm_tc_kernel(GemvTcArgs a, const __grid_constant__ CUtensorMap amap) {
  static_assert(NS <= gm::MAX_STAGES && NR <= gm::MAX_RSTAGES, "ring deeper than the barrier arrays");
  static_assert(MM * BNV <= 512, "accumulators beyond the 512 TMEM columns");
  using T = Gt<BNV>;
  constexpr int STG = MM * gm::A_BYTES + T::B_BYTES;        // one slice: MM A tiles, then B
  constexpr uint32_t TCOLS = (uint32_t)(MM * T::TMEM_COLS);
  extern __shared__ unsigned char smem_raw[];
  // the swizzled slices need 1024-byte aligned bases
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  unsigned char* rawring = smem + NS * STG;
  GemmShared* sh = reinterpret_cast<GemmShared*>(rawring + NR * T::RAW_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int MT = (a.NB + gm::BM * MM - 1) / (gm::BM * MM);
  const int tiles = MT * ((a.N + T::BN - 1) / T::BN);
  const int ksp = blockIdx.x / tiles, tile = blockIdx.x % tiles;  // k split of this CTA (split-K: RESID only)
  const int mt = tile % MT, nt = tile / MT;                 // M fastest: CTAs sharing a weight tile run together
  const int m0 = mt * gm::BM * MM, n0 = nt * T::BN;
  const int mlive = min(MM, (a.NB - m0 + gm::BM - 1) / gm::BM);   // M tiles of this CTA holding prompt rows
  const int KT = a.K / 32, RB = a.Np / 64;
  const int KBT = (a.K + gm::BK - 1) / gm::BK;
  const int kb0 = ksp * KBT / a.ksplit;                    // this CTA's slices [kb0, kb0 + KB)
  const int KB = (ksp + 1) * KBT / a.ksplit - kb0;
  constexpr int UNIT = I4 ? tc::UNIT4 : tc::UNIT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NR; ++s) {
      mbar_init(&sh->raw_full[s], 1);
      mbar_init(&sh->raw_empty[s], gm::CONV);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(&sh->a_full[s], 1);
      mbar_init(&sh->full[s], gm::CONV);
      mbar_init(&sh->empty[s], 1);
    }
    mbar_init(&sh->accum, 1);
    sh->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == gm::MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&sh->tmem)), "r"(TCOLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = sh->tmem;
  volatile int* abort = &sh->abort;

  if (warp == gm::RAW_WARP) {
    // ------------------------------------------------- raw weight copies (one thread, no launch wait:
    // the weights never change, so the ring fills while the preceding kernel still runs)
    if (lane == 0) {
      const char* W = reinterpret_cast<const char*>(a.w);
      int issued = 0;
      for (int kb = 0; kb < KB; ++kb) {
        const int r = kb % NR;
        if (kb >= NR &&
            !gm_wait(&sh->raw_empty[r], (uint32_t)(((kb / NR) - 1) & 1), abort)) {
          *abort = 1;
          break;
        }
        unsigned char* rs = rawring + r * T::RAW_BYTES;
        const int kt = (kb0 + kb) * 2, nk = min(2, KT - kt);
        uint32_t bytes = 0;
        for (int rbi = 0; rbi < T::BN / 64; ++rbi)
          if (n0 / 64 + rbi < RB) bytes += (uint32_t)nk * UNIT;
        mbar_arrive_expect_tx(&sh->raw_full[r], bytes);
        for (int rbi = 0; rbi < T::BN / 64; ++rbi) {
          const int rb = n0 / 64 + rbi;
          if (rb < RB)
            bulk_g2s(rs + rbi * 2 * UNIT, W + ((size_t)rb * KT + kt) * UNIT, nk * UNIT, &sh->raw_full[r]);
        }
        issued = kb + 1;
      }
      // shared memory must outlive every copy issued: wait (time-bounded only) for the last ones
      for (int kb = issued - 1; kb >= 0 && kb >= issued - NR; --kb) {
        const int r = kb % NR;
        for (long long i = 0;
             i < gm::LIMIT && !mbar_try_wait(&sh->raw_full[r], (uint32_t)((kb / NR) & 1)); ++i) {
        }
      }
    }
  } else if (warp == gm::A_WARP) {
    // ---------------------------------------------------------------- A tiles (one thread)
    if (lane == 0) {
      pdl_wait();                                     // A is the preceding kernel's output
      int issued = 0;
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % NS;
        if (kb >= NS && !gm_wait(&sh->empty[s], (uint32_t)(((kb / NS) - 1) & 1), abort)) {
          *abort = 1;
          break;
        }
        mbar_arrive_expect_tx(&sh->a_full[s], (uint32_t)(mlive * gm::A_BYTES));
        for (int i = 0; i < mlive; ++i)
          tma_load_2d(smem + s * STG + i * gm::A_BYTES, &amap, (kb0 + kb) * gm::BK, m0 + i * gm::BM, &sh->a_full[s]);
        issued = kb + 1;
      }
      for (int kb = issued - 1; kb >= 0 && kb >= issued - NS; --kb) {
        const int s = kb % NS;
        for (long long i = 0; i < gm::LIMIT && !mbar_try_wait(&sh->a_full[s], (uint32_t)((kb / NS) & 1)); ++i) {
        }
      }
    }
  } else if (warp == gm::MMA_WARP) {
    // ---------------------------------------------------------------- MMA issuer (one thread)
    if (lane == 0) {
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % NS;
        if (!gm_wait(&sh->a_full[s], (uint32_t)((kb / NS) & 1), abort) ||
            !gm_wait(&sh->full[s], (uint32_t)((kb / NS) & 1), abort)) {
          *abort = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t abase = smem_u32(smem + s * STG);
        const uint32_t bbase = abase + MM * gm::A_BYTES;
        for (int i = 0; i < mlive; ++i)
#pragma unroll
          for (int ks = 0; ks < gm::BK / 16; ++ks)
            mma_f16(tmem + (uint32_t)(i * T::BN), smem_desc(abase + i * gm::A_BYTES + ks * 32),
                    smem_desc(bbase + ks * 32), T::IDESC, (kb | ks) != 0);
        mma_commit(&sh->empty[s]);
      }
      // completes once every MMA issued so far has finished (also on abort, so that the tensor
      // memory is idle before it is freed)
      mma_commit(&sh->accum);
    }
  } else {
    // ---------------------------------------------------------------- converters (warps 0-3)
    const int t = threadIdx.x;
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % NS, r = kb % NR;
      // the raw units landed, and the MMAs of the slice that last used this B slot are done
      if (!gm_wait(&sh->raw_full[r], (uint32_t)((kb / NR) & 1), abort) ||
          (kb >= NS && !gm_wait(&sh->empty[s], (uint32_t)(((kb / NS) - 1) & 1), abort))) {
        *abort = 1;
        break;
      }
      unsigned char* st = smem + s * STG;
      unsigned char* Bs = st + MM * gm::A_BYTES;
      const unsigned char* Rw = rawring + r * T::RAW_BYTES;
      const int kt0 = (kb0 + kb) * 2;
#pragma unroll 4
      for (int q = t; q < T::BN / 64 * 2 * 128; q += gm::CONV) {
        const int u = q >> 7, rbi = u >> 1, kti = u & 1;
        // fragment lane of this thread: the 8 threads of each quarter warp take rows g and g ^ 5
        // (g < 4) with their 4 chunks each, so their 16-byte stores cover the 8 swizzled positions of
        // a 128-byte line exactly once (and their int8 loads 8 distinct 16-byte columns)
        const int qi = q & 7, qp = (q >> 3) & 3;
        const int g = qp ^ (5 * (qi >> 2)), t4 = qi & 3, ln = g * 4 + t4;
        const int w = (q >> 5) & 3;
        const int nb = rbi * 64 + w * 16 + g;                 // row of the B slice (and nb + 8)
        const int kc = kti * 4 + t4;                          // 16-byte chunk of the slice's K
        uint32_t lo[4] = {0u, 0u, 0u, 0u}, hi[4] = {0u, 0u, 0u, 0u};
        if (n0 / 64 + rbi < RB && kt0 + kti < KT) {
          const unsigned char* unit = Rw + (rbi * 2 + kti) * UNIT;
          if constexpr (I4) {
            const uint2 wv = *reinterpret_cast<const uint2*>(unit + w * tc::TILE4 + ln * 8);
            const __half2 sc = *reinterpret_cast<const __half2*>(unit + tc::WARPS * tc::TILE4 + (w * 16 + 2 * g) * 2);
            const __half2 s_lo = __half2half2(__low2half(sc)), s_hi = __half2half2(__high2half(sc));
            i4_rows(wv.x, s_lo, s_hi, lo[0], lo[1], hi[0], hi[1]);
            i4_rows(wv.y, s_lo, s_hi, lo[2], lo[3], hi[2], hi[3]);
          } else {
            const uint4 wv = *reinterpret_cast<const uint4*>(unit + w * tc::TILE + ln * 16);
            i8x4_to_h2x2(wv.x, lo[0], hi[0]);
            i8x4_to_h2x2(wv.y, lo[1], hi[1]);
            i8x4_to_h2x2(wv.z, lo[2], hi[2]);
            i8x4_to_h2x2(wv.w, lo[3], hi[3]);
          }
        }
        *reinterpret_cast<uint4*>(Bs + sw128(nb, kc)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4*>(Bs + sw128(nb + 8, kc)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      }
      // generic-proxy stores -> visible to the tensor core's async proxy, then signal the slice
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&sh->full[s]);
      mbar_arrive(&sh->raw_empty[r]);
    }
  }

  // ---------------------------------------------------------------- epilogue (warps 0-3)
  if (warp < 4) {
    const bool ok = gm_wait(&sh->accum, 0, abort) && !*abort;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ok) {
      af_set_err(a.err, AF_DEV_WAIT_TIMEOUT);
    } else {
      // A warp's 32 TMEM lanes are 32 output rows. SwiGLU stores each row's 8-output groups as
      // 16-byte vectors; the other epilogues stage each 32-column chunk in shared memory (the operand
      // ring is idle once the accumulators are final; rows 144 bytes apart) and write it back as
      // float4s with 8 consecutive lanes on one row's 128 bytes, so global loads and stores coalesce.
      float* stage = reinterpret_cast<float*>(smem) + warp * (32 * 36);
      const bool vec = a.N % 4 == 0 && a.ldy % 4 == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0;
      for (int mi = 0; mi < mlive; ++mi) {
      const int rowbase = m0 + mi * gm::BM + warp * 32;
      const int m = rowbase + lane;
#pragma unroll 1
      for (int c0 = 0; c0 < T::BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(mi * T::BN + c0), v);
        const int nbase = n0 + c0;
        float f[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int n = nbase + j;
          float x = __uint_as_float(v[j]);
          if (n < a.N) {
            if (!I4) x = __fmul_rn(x, h2f(a.scale[n]));
            if (a.bias && ksp == 0) x = __fadd_rn(x, h2f(a.bias[n]));
          }
          f[j] = x;
        }
        if (a.epi == EPI_SWIGLU) {
          // rows 16i..16i+7 gate, 16i+8..16i+15 up -> 8 outputs per 16 rows
          if (m >= a.NB) continue;
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int r0 = nbase + 16 * i;
            if (r0 + 16 > a.N) continue;
            __half o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = f2h(silu_f(f[16 * i + j]) * f[16 * i + 8 + j]);
            *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(a.y) + (size_t)m * a.ldy + r0 / 2) =
                *reinterpret_cast<const uint4*>(o);
          }
          continue;
        }
        if (!vec) {
          if (m >= a.NB) continue;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = nbase + j;
            if (n >= a.N) break;
            const size_t o = (size_t)m * a.ldy + n;
            if (a.epi == EPI_F32) reinterpret_cast<float*>(a.y)[o] = f[j];
            else if (a.epi == EPI_F16) reinterpret_cast<__half*>(a.y)[o] = f2h(f[j]);
            else if (a.ksplit > 1) atomicAdd(reinterpret_cast<float*>(a.y) + o, f[j]);   // k splits meet in y
            else reinterpret_cast<float*>(a.y)[o] = __ldcg(reinterpret_cast<const float*>(a.y) + o) + f[j];
          }
          continue;
        }
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4)
          *reinterpret_cast<float4*>(stage + lane * 36 + 4 * q4) =
              make_float4(f[4 * q4], f[4 * q4 + 1], f[4 * q4 + 2], f[4 * q4 + 3]);
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int q = 4 * k + (lane >> 3), jj = lane & 7;       // row q of the chunk, its float4 jj
          const int mr = rowbase + q, n = nbase + 4 * jj;
          if (mr >= a.NB || n >= a.N) continue;
          const float4 val = *reinterpret_cast<const float4*>(stage + q * 36 + 4 * jj);
          const size_t o = (size_t)mr * a.ldy + n;
          if (a.epi == EPI_F32) {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.y) + o) = val;
          } else if (a.epi == EPI_F16) {
            const __half2 lo = __floats2half2_rn(val.x, val.y), hi = __floats2half2_rn(val.z, val.w);
            *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(a.y) + o) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
          } else if (a.ksplit > 1) {
            float* yp = reinterpret_cast<float*>(a.y) + o;           // k splits meet in y
            atomicAdd(yp, val.x); atomicAdd(yp + 1, val.y); atomicAdd(yp + 2, val.z); atomicAdd(yp + 3, val.w);
          } else {
            float4* yp = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.y) + o);
            const float4 old = __ldcg(yp);
            *yp = make_float4(old.x + val.x, old.y + val.y, old.z + val.z, old.w + val.w);
          }
        }
        __syncwarp();
      }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == gm::MMA_WARP) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS) : "memory");
  }
}

template <int BNV, int NS, int NR, int MM = 1>
static size_t smem_for() {
  using T = Gt<BNV>;
  return (size_t)NS * (MM * gm::A_BYTES + T::B_BYTES) + (size_t)NR * T::RAW_BYTES + sizeof(GemmShared) + 1024;
}

size_t gemm_tc_smem_bytes() { return smem_for<256, gm::STAGES, gm::RSTAGES>(); }

// The A operand's tensor map: fp16 [M rows][K] with row stride ldx, 64 x 128 boxes, 128-byte swizzle.
static bool make_amap(const GemvTcArgs& a, CUtensorMap* map) {
  const EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.NB};
  const cuuint64_t strides[1] = {(cuuint64_t)a.ldx * 2};
  const cuuint32_t box[2] = {(cuuint32_t)gm::BK, (cuuint32_t)gm::BM};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(a.x), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// x [M][ldx] fp16 (M = a.NB rows), weights as for gemv_tc, y per epilogue (ldy); M >= 1, K % 32 == 0.
cudaError_t gemm_tc_launch(GemvTcArgs a, cudaStream_t st, bool pdl) {
  if (a.NB < 1 || a.N <= 0 || a.K <= 0 || a.K % 32 || a.ldx % 8) return cudaErrorInvalidValue;
  if (a.epi != EPI_F32 && a.epi != EPI_F16 && a.epi != EPI_RESID && a.epi != EPI_SWIGLU) return cudaErrorInvalidValue;
  if (a.epi == EPI_SWIGLU && a.N % 16) return cudaErrorInvalidValue;
  if (a.sel || a.rw) return cudaErrorInvalidValue;            // experts run through the GEMV
  const bool i4 = a.wf == W_I4G32;
  if (!i4 && (a.wf != W_I8 || !a.scale)) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.x) & 15) || (reinterpret_cast<uintptr_t>(a.w) & 15)) return cudaErrorInvalidValue;
  a.Np = (a.N + 63) / 64 * 64;
  CUtensorMap amap;
  if (!make_amap(a, &amap)) return cudaErrorInvalidValue;
  // 128-column tiles when 256-column ones would leave SMs idle (few output tiles: the prompt-sized
  // qkv / o / down shapes), 256 otherwise (half the A re-reads per output)
  const int sms = device_attr(cudaDevAttrMultiProcessorCount, 148);
  static const int narrow_ok = env_int("AF_GEMM_NARROW", 1);
  // two 128-row M tiles per CTA (one dequantisation of each weight slice per 256 prompt rows) when
  // that still gives every SM a 256-column tile: measured on the 8B 512-row prompt, gate|up 285.7 ->
  // 203.6 µs and the 72B 2048-row int4 gate|up 2333 -> 1752 µs, while the narrow o / down shapes
  // (64 CTAs) got slower (64 -> 93, 136 -> 182 µs). AF_GEMM_MM: 0 this rule, 1 never, 2 always.
  static const int mm_env = env_int("AF_GEMM_MM", 0);
  const int tiles2 = ((a.NB + 2 * gm::BM - 1) / (2 * gm::BM)) * ((a.N + 255) / 256);
  // (AF_GEMM_MM=4, measurement: four M tiles on 128-column tiles, each weight slice dequantised once
  // per 512 prompt rows)
  const int MM = (mm_env == 4 && a.NB > 3 * gm::BM) ? 4
                 : a.NB > gm::BM && (mm_env == 2 || (mm_env == 0 && tiles2 >= sms)) ? 2 : 1;
  const int MT = (a.NB + gm::BM * MM - 1) / (gm::BM * MM);
  // 128-column tiles only where they add no wave: twice the tiles must fit in as many waves of
  // `sms` CTAs as the 256-column tiles (AF_GEMM_NARROW: 0 never, 2 always, 1 this rule)
  const int wide_tiles = MT * ((a.N + 255) / 256), narrow_tiles = MT * ((a.N + 127) / 128);
  const bool narrow = MM == 4 || narrow_ok == 2 || (narrow_ok == 1 && wide_tiles < sms &&
                                         (narrow_tiles + sms - 1) / sms == (wide_tiles + sms - 1) / sms);
  const int BNV = narrow ? 128 : 256;
  const int NT = (a.N + BNV - 1) / BNV;
  // ring depths: 128-column tiles run four operand and eight raw slices (AF_GEMM_DEEP=0: three and
  // four, as 256-column tiles do). Measured on the 8B prompt shapes (qkv / o / down, µs): 3+4 143 /
  // 69 / 162, 6+4 130 / 62 / 138, 4+8 128 / 62 / 134; for 256-column tiles 4+2 was slower than 3+4.
  static const int deep = env_int("AF_GEMM_DEEP", 1);
  // MM = 2: 128-column tiles with three operand and eight raw slices, 256-column with two and four
  // (the second A tile per slice takes the shared memory of one operand stage)
  int var = MM == 4 ? 8 : MM == 2 ? (narrow ? 3 : 4) : (narrow ? (deep >= 1 ? 1 : 0) : 2);
  // deeper operand rings at the same shared memory (measurement variants, AF_GEMM_RING=1): 128-column
  // tiles with six operand and four raw slices, two-tile 256-column with three and two
  static const int ring = env_int("AF_GEMM_RING", 0);
  if (ring == 1 && var == 1) var = 5;
  if (ring == 1 && var == 4) var = 6;
  // split-K for the residual epilogue (o / down prompt shapes, fewer tiles than SMs): AF_GEMM_SPLITK=S
  // runs S CTAs per 128-column tile over disjoint k ranges on the half-size rings (two CTAs per SM),
  // each adding its partial into the fp32 residual atomically (summation order then varies by run).
  // Off by default: with the coalesced epilogue it measured slower (8B prompt o 50.8 -> 66.3 µs).
  static const int splitk = env_int("AF_GEMM_SPLITK", 0);
  a.ksplit = 1;
  const int KBT = (a.K + gm::BK - 1) / gm::BK;
  if (splitk >= 2 && a.epi == EPI_RESID && !a.bias && MM == 1 && BNV == 128 &&
      MT * ((a.N + 127) / 128) * splitk <= 2 * sms && KBT >= 8 * splitk) {
    var = 7;
    a.ksplit = splitk;
  }
  constexpr int NV = 9;
  static const size_t smems[NV] = {smem_for<128, 3, 4>(), smem_for<128, 4, 8>(), smem_for<256, 3, 4>(),
                                   smem_for<128, 3, 8, 2>(), smem_for<256, 2, 4, 2>(), smem_for<128, 6, 4>(),
                                   smem_for<256, 3, 2, 2>(), smem_for<128, 2, 4>(), smem_for<128, 2, 4, 4>()};
  void* const fns[2][NV] = {
      {(void*)gemm_tc_kernel<false, 128, 3, 4, 1>, (void*)gemm_tc_kernel<false, 128, 4, 8, 1>,
       (void*)gemm_tc_kernel<false, 256, 3, 4, 1>, (void*)gemm_tc_kernel<false, 128, 3, 8, 2>,
       (void*)gemm_tc_kernel<false, 256, 2, 4, 2>, (void*)gemm_tc_kernel<false, 128, 6, 4, 1>,
       (void*)gemm_tc_kernel<false, 256, 3, 2, 2>, (void*)gemm_tc_kernel<false, 128, 2, 4, 1>,
       (void*)gemm_tc_kernel<false, 128, 2, 4, 4>},
      {(void*)gemm_tc_kernel<true, 128, 3, 4, 1>, (void*)gemm_tc_kernel<true, 128, 4, 8, 1>,
       (void*)gemm_tc_kernel<true, 256, 3, 4, 1>, (void*)gemm_tc_kernel<true, 128, 3, 8, 2>,
       (void*)gemm_tc_kernel<true, 256, 2, 4, 2>, (void*)gemm_tc_kernel<true, 128, 6, 4, 1>,
       (void*)gemm_tc_kernel<true, 256, 3, 2, 2>, (void*)gemm_tc_kernel<true, 128, 2, 4, 1>,
       (void*)gemm_tc_kernel<true, 128, 2, 4, 4>}};
  const size_t smem = smems[var];
  void* fn = fns[i4 ? 1 : 0][var];
  static PerDeviceOnce attr[2][NV];
  const cudaError_t ae = attr[i4 ? 1 : 0][var].run(
      [fn, smem] { return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); });
  if (ae != cudaSuccess) return ae;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(MT * NT * a.ksplit));
  cfg.blockDim = dim3(gm::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  void* args[] = {&a, &amap};
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace af
