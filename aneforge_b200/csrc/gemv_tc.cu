// K1: int8 per-row dequant GEMV for decode on B200 - a persistent, stream-K kernel that streams the
// weights through a TMA (cp.async.bulk) shared-memory ring and multiplies on the tensor cores.
//
// Why this shape. The GEMV is bound by HBM: every weight byte is read once per decode step. Keeping
// ~6.5 TB/s in flight needs tens of KB of outstanding loads per SM, more than registers can hold at
// useful occupancy, so one producer thread per CTA issues 8 KB bulk copies into a 6-stage ring
// (tracked by mbarriers, 4 CTAs per SM: ~190 KB in flight per SM); four consumer warps per CTA read
// their 16-byte A fragments from shared memory,
// dequantise them (a byte permute places each int8 code under the fp16 exponent of 1024, one half2
// subtract removes the bias - exact for every code) and run mma.sync m16n8k16 (fp16 x fp16 ->
// fp32). The batch (1..16 sequences) is the MMA's N dimension, so batching adds no weight traffic.
//
// Weight layout (pack_i8_tiles): a 16-row x 32-column tile is 512 bytes; lane l owns bytes
// [16l, 16l+16) = its A fragment for the tile's two k-steps:
//   bytes [8s .. 8s+7] (k-step s): (g,2t) (g,2t+1) (g+8,2t) (g+8,2t+1) (g,2t+8) (g,2t+9) (g+8,2t+8) (g+8,2t+9)
// with g = l/4, t = l%4. Tiles are grouped [row block of 64 rows][k tile][4 row tiles][512 B].
//
// Work split (stream-K): the RB x KT "units" (one k tile of one row block = 2 KB) are cut into one
// contiguous range per CTA of a persistent grid, so every CTA streams the same number of bytes from
// one contiguous address range. A row block covered by a single CTA gets its epilogue directly; a
// row block shared by n CTAs (at most two per CTA: its first and last) is finished by the CTA that
// takes the last ticket, which adds the n fp32 partials in CTA order - deterministic. x is
// bulk-copied per chunk (<= 16 k tiles) into a 2-slot ring by the producer, after the programmatic
// launch wait; the first chunk's weights are requested before that wait.
//
// Group-32 int4 weights (I4 = true) use the same tiling at half the bytes: a 16x32 tile is 256 bytes
// (lane l owns bytes [8l, 8l+8), one 32-bit word per k-step whose nibbles at bit offsets
// (0,16) (4,20) (8,24) (12,28) are the fragment pairs a0a1, a2a3, a4a5, a6a7), and each unit ends
// with the 64 fp16 group scales of its rows for that k tile (unit = 4 x 256 + 128 = 1152 bytes). A
// nibble n (= code + 8) becomes fp16 1024 + n with one mask-or, minus 1032 exactly; each k tile's
// product is accumulated fresh and added to the running sum times its group scale, so the scale is
// applied in fp32 as the dequantised weight s * code would be.
//
// Epilogues: F32 / F16 / RESID (y += ..) / SWIGLU (tiles hold 8 gate rows then the matching 8 up).
// Every mbarrier wait is bounded: on timeout the kernel records AF_DEV_WAIT_TIMEOUT in the error
// word, consumers leave together after a barrier, and the producer waits (bounded) for the copies
// it issued before its thread exits.
#include <cstdlib>

#include "af_common.cuh"
#include "af_kernels.h"
#include "tc_common.cuh"

namespace af {

template <int NT, int EPI, bool I4>
AF_DEV void epilogue(const GemvTcArgs& a, float (&acc)[NT][4], int rt, int g, int t) {
  const int r0 = rt * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int b = n * 8 + 2 * t + h;
      if (b >= a.nlive) continue;
      const int yb = (a.route & 2) ? __ldcg(a.rows + a.rbase + b) : b;   // output row (scattered when routed)
      const float v0 = acc[n][h], v1 = acc[n][2 + h];
      if (EPI == EPI_SWIGLU) {
        if (r1 >= a.N) continue;
        float gv = I4 ? v0 : __fmul_rn(v0, h2f(a.scale[r0]));
        float uv = I4 ? v1 : __fmul_rn(v1, h2f(a.scale[r1]));
        if (a.bias) { gv = __fadd_rn(gv, h2f(a.bias[r0])); uv = __fadd_rn(uv, h2f(a.bias[r1])); }
        reinterpret_cast<__half*>(a.y)[(size_t)yb * a.ldy + rt * 8 + g] = f2h(silu_f(gv) * uv);
      } else {
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int row = rr ? r1 : r0;
          if (row >= a.N) continue;
          float v = I4 ? (rr ? v1 : v0) : __fmul_rn(rr ? v1 : v0, h2f(a.scale[row]));
          if (a.bias) v = __fadd_rn(v, h2f(a.bias[row]));
          const size_t o = (size_t)yb * a.ldy + row;
          if (EPI == EPI_F32) reinterpret_cast<float*>(a.y)[o] = v;
          else if (EPI == EPI_F16) reinterpret_cast<__half*>(a.y)[o] = f2h(v);
          else if (EPI == EPI_RESID) {
            if (a.rw) v *= __ldcg(a.rw + (size_t)yb * a.rw_e + a.e_base + a.fixed_e);
            reinterpret_cast<float*>(a.y)[o] = __ldcg(reinterpret_cast<const float*>(a.y) + o) + v;
          }
        }
      }
    }
  }
}

template <int NT, int EPI, bool I4>
__global__ void __launch_bounds__((Cw<I4>::n + 1) * 32) gemv_tc_kernel(GemvTcArgs a) {
  constexpr int CW = Cw<I4>::n;
  // expert selection (MoE): the expert index may be produced by the preceding kernel, so with `sel`
  // the weights are addressed only after the programmatic-launch wait
  int expert = a.fixed_e;
  if (a.sel) {
    pdl_wait();
    expert = __ldcg(a.sel + a.slot) - a.e_base;
    // expert parallel: an expert held by another GPU contributes nothing here (uniform over the grid:
    // every thread of every CTA leaves before any barrier)
    if (a.n_exp > 0 && (expert < 0 || expert >= a.n_exp)) return;
  }
  if (a.sel || a.fixed_e) {
    a.w = static_cast<const char*>(a.w) + (size_t)expert * a.w_stride;
    if (a.scale) a.scale += (size_t)expert * a.s_stride;
  }
  a.fixed_e = expert;
  a.nlive = a.NB;
  if (a.route) {
    // routed batch: the row list comes from the preceding kernel; an empty share is a no-op (uniform
    // over the grid, before any barrier)
    pdl_wait();
    a.rbase = (a.e_base + expert) * a.rld + a.r0;
    a.nlive = min(a.NB, __ldcg(a.rcnt + a.e_base + expert) - a.r0);
    if (a.nlive <= 0) return;
  }
  using F = tc::Fmt<I4>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int NS = a.nst;                                                    // weight ring depth (<= STAGES)
  unsigned char* ring = smem_raw;                                          // [NS][F::stage]
  TcShared* sh = reinterpret_cast<TcShared*>(smem_raw + NS * F::stage);
  __half* xring = reinterpret_cast<__half*>(smem_raw + NS * F::stage + SH_BYTES);
  const int xslot_halves = a.NB * tc::XSTRIDE;                             // one x chunk

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = a.Kp / 32;
  const int RB = a.Np / 64;
  const long long U = (long long)RB * KT;
  const int G = gridDim.x, c = blockIdx.x;
  long long u0 = unit_begin(c, U, G), u1 = unit_begin(c + 1, U, G);
  if (a.csize > 1) {
    // one thread-block cluster per row block: rank r takes k tiles [r KT / d, (r + 1) KT / d)
    const long long rb0 = c / a.csize, r = c % a.csize;
    u0 = rb0 * KT + r * KT / a.csize;
    u1 = rb0 * KT + (r + 1) * KT / a.csize;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], CW);
    }
    for (int s = 0; s < tc::XSLOTS; ++s) {
      mbar_init(&sh->xfull[s], 1);
      mbar_init(&sh->xempty[s], CW);
    }
    sh->cabort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == CW) {
    // -------------------------------------------------------------- producer (one thread)
    // (with clusters every thread still takes part in the two cluster barriers of the reduction)
    if (lane != 0) {
      if (a.csize > 1) { cluster_sync_any(); cluster_sync_any(); }
      return;
    }
    const char* W = reinterpret_cast<const char*>(a.w);
    const uint64_t pol = a.evict_first ? l2_evict_first_policy() : 0;
    int stage = 0, xs = 0;
    uint32_t phase = 0, xphase = 0;
    int in_flight = 0;
    bool ok = true, waited = false;
    // the first chunk's weights go out before the programmatic-launch wait (weights never change)
    long long u = u0;
    while (u < u1 && ok) {
      const int rb = (int)(u / KT), kta = (int)(u % KT);
      const int ktb = (int)min((long long)KT, kta + (u1 - u));
      for (int kc = kta; kc < ktb && ok; kc += tc::XKT) {
        const int kce = min(kc + tc::XKT, ktb);
        int kt = kc;
        if (!waited) {
          // chunk 0: weights first, then wait for the producer kernel of x, then x
          for (; kt < kce && in_flight < NS; kt += F::ks) {
            const int nk = min(F::ks, kce - kt);
            mbar_arrive_expect_tx(&sh->full[stage], (uint32_t)nk * F::unit);
            bulk_w(ring + (size_t)stage * F::stage, W + ((size_t)rb * KT + kt) * F::unit, nk * F::unit,
                   &sh->full[stage], a.evict_first, pol);
            ++in_flight;
            if (++stage == NS) { stage = 0; phase ^= 1; }
          }
          pdl_wait();
          waited = true;
        }
        // x chunk [kc, kce) for every real batch row
        if (!mbar_wait(&sh->xempty[xs], xphase ^ 1)) { ok = false; break; }
        const uint32_t xbytes = (uint32_t)(kce - kc) * 32 * 2;
        mbar_arrive_expect_tx(&sh->xfull[xs], xbytes * a.NB);
        for (int b = 0; b < a.NB; ++b) {
          // routed: row b of the list (rows past the list repeat its first row: finite, never stored)
          const int xb = (a.route & 1) ? __ldcg(a.rows + a.rbase + (b < a.nlive ? b : 0)) : b;
          bulk_g2s(xring + (size_t)xs * xslot_halves + (size_t)b * tc::XSTRIDE, a.x + (size_t)xb * a.ldx + (size_t)kc * 32,
                   xbytes, &sh->xfull[xs]);
        }
        if (++xs == tc::XSLOTS) { xs = 0; xphase ^= 1; }
        for (; kt < kce; kt += F::ks) {
          const int nk = min(F::ks, kce - kt);
          if (!mbar_wait(&sh->empty[stage], phase ^ 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&sh->full[stage], (uint32_t)nk * F::unit);
          bulk_w(ring + (size_t)stage * F::stage, W + ((size_t)rb * KT + kt) * F::unit, nk * F::unit,
                 &sh->full[stage], a.evict_first, pol);
          in_flight = min(in_flight + 1, NS);
          if (++stage == NS) { stage = 0; phase ^= 1; }
        }
      }
      u += ktb - kta;
    }
    if (!waited) pdl_wait();
    if (!ok) af_set_err(a.err, AF_DEV_WAIT_TIMEOUT);
    // shared memory must outlive every copy this thread issued: wait (bounded) for the last use of
    // each weight stage and x slot to land before the thread exits
    for (int i = 0; i < in_flight; ++i) {
      if (--stage < 0) { stage = NS - 1; phase ^= 1; }
      mbar_wait(&sh->full[stage], phase);
    }
    for (int i = 0; i < tc::XSLOTS; ++i) {
      if (--xs < 0) { xs = tc::XSLOTS - 1; xphase ^= 1; }
      mbar_wait(&sh->xfull[xs], xphase);
    }
    if (a.csize > 1) { cluster_sync_any(); cluster_sync_any(); }
    return;
  }

  // ---------------------------------------------------------------- consumers (4 or 8 warps)
  // Warps w and w + 4 share row tile w of the row block: within every stage the first multiplies the
  // even k tiles, the second the odd ones; their sums meet in shared memory at the end of each
  // row-block range. The tiles' columns are permuted so that a lane's B fragments for both k-steps
  // of a k tile are 8 consecutive x values: one 16-byte shared load per k tile.
  const int g = lane >> 2, t = lane & 3;
  const int rtw = warp & 3, par = warp >> 2;          // par: 0 with 4 consumer warps
  float* red = reinterpret_cast<float*>(smem_raw + NS * F::stage + SH_BYTES +
                                        (size_t)tc::XSLOTS * xslot_halves * 2);       // [4][32][NT*4]
  pdl_wait();
  pdl_trigger();
  int stage = 0, xs = 0;
  uint32_t phase = 0, xphase = 0;
  long long u = u0;
  while (u < u1) {
    const int rb = (int)(u / KT), kta = (int)(u % KT);
    const int ktb = (int)min((long long)KT, kta + (u1 - u));
    float acc[NT][4], acc2[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int q = 0; q < 4; ++q) { acc[n][q] = 0.f; acc2[n][q] = 0.f; }
    bool stuck = false;
    for (int kc = kta; kc < ktb && !stuck; kc += tc::XKT) {
      const int kce = min(kc + tc::XKT, ktb);
      if (!mbar_wait(&sh->xfull[xs], xphase)) { stuck = true; break; }
      const __half* xsl = xring + (size_t)xs * xslot_halves;
      for (int kt = kc; kt < kce; kt += F::ks) {
        const int nk = min(F::ks, kce - kt);
        if (!mbar_wait(&sh->full[stage], phase)) { stuck = true; break; }
        consume_stage<I4, NT, CW / 4>(ring + (size_t)stage * F::stage, nk, xsl + (kt - kc) * 32, tc::XSTRIDE, a.nlive, lane,
                                      rtw, par, acc, acc2);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh->empty[stage]);
        if (++stage == NS) { stage = 0; phase ^= 1; }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->xempty[xs]);
      if (++xs == tc::XSLOTS) { xs = 0; xphase ^= 1; }
    }
    if (stuck) {
      af_set_err(a.err, AF_DEV_WAIT_TIMEOUT);
      *reinterpret_cast<volatile int*>(&sh->cabort) = 1;
    }
    // this CTA's stream is done: its share of a later kernel's weights into L2 meanwhile
    if (u + (ktb - kta) >= u1) l2_prefetch_lines(a.pf, c * (CW * 32) + threadIdx.x, G * (CW * 32));
    // odd-tile warps hand their sums to the even-tile warps of the same row tile
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[n][q] += acc2[n][q];
    float* rw = red + ((size_t)rtw * 32 + lane) * (NT * 4);
    if (CW == 8 && par) {
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int q = 0; q < 4; ++q) rw[n * 4 + q] = acc[n][q];
    }
    consumer_sync_n<CW>();
    if (*reinterpret_cast<volatile int*>(&sh->cabort)) break;
    if (CW == 8 && !par) {
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[n][q] += rw[n * 4 + q];
    }
    const int rt = rb * tc::WARPS + rtw;
    if (kta == 0 && ktb == KT) {
      // this CTA owns the whole row block
      if (!par) epilogue<NT, EPI, I4>(a, acc, rt, g, t);
    } else if (a.csize > 1) {
      // cluster rank: the partial waits at the start of this CTA's weight ring (every stage has
      // been consumed) until rank 0 reads it after the cluster barrier below
      if (!par) {
        float* slot = reinterpret_cast<float*>(ring) + (size_t)(rtw * 32 + lane) * (NT * 4);
#pragma unroll
        for (int n = 0; n < NT; ++n)
          *reinterpret_cast<float4*>(slot + n * 4) = make_float4(acc[n][0], acc[n][1], acc[n][2], acc[n][3]);
      }
    } else {
      // stream-K row block shared by CTAs cf..cl: the owner cf holds its first k tiles and reaches
      // them last (they end its range), the others start with theirs. Those publish a partial in
      // slot j = c - cf and count it on the row block's counter; the owner waits (bounded) until
      // all nc - 1 are in and sums them in CTA order onto its own, so the result is deterministic
      const int cf = owner_of((long long)rb * KT, U, G), cl = owner_of((long long)rb * KT + KT - 1, U, G);
      const int nc = cl - cf + 1, j = c - cf;
      constexpr int NBP = NT * 8;
      const int r0 = rtw * 16 + g, r1 = r0 + 8;
      if (j > 0) {
        float* slot = a.part + (((size_t)rb * a.maxc + j) * 64) * NBP;
        if (!par) {
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            const int c0 = n * 8 + 2 * t;
            if (c0 >= a.NB) continue;
            __stcg(reinterpret_cast<float2*>(slot + (size_t)r0 * NBP + c0), make_float2(acc[n][0], acc[n][1]));
            __stcg(reinterpret_cast<float2*>(slot + (size_t)r1 * NBP + c0), make_float2(acc[n][2], acc[n][3]));
          }
          __threadfence();
        }
        consumer_sync_n<CW>();
        if (threadIdx.x == 0) atomicAdd(a.counters + rb, 1);
      } else {
        if (threadIdx.x == 0) {
          bool in = false;
          SpinBudget budget;
          for (long long i = 0; i < tc::WAIT_LIMIT && !in && !budget.spent(); ++i) {
            int v;
            asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(a.counters + rb) : "memory");
            in = v >= nc - 1;
          }
          if (!in) {
            af_set_err(a.err, AF_DEV_WAIT_TIMEOUT);
            sh->cabort = 1;
          }
        }
        consumer_sync_n<CW>();
        if (!par) {
          __threadfence();
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            const int c0 = n * 8 + 2 * t;
            if (c0 >= a.NB) continue;
            for (int jj = 1; jj < nc; ++jj) {
              const float* sp = a.part + (((size_t)rb * a.maxc + jj) * 64) * NBP;
              const float2 p = __ldcg(reinterpret_cast<const float2*>(sp + (size_t)r0 * NBP + c0));
              const float2 q = __ldcg(reinterpret_cast<const float2*>(sp + (size_t)r1 * NBP + c0));
              acc[n][0] += p.x; acc[n][1] += p.y; acc[n][2] += q.x; acc[n][3] += q.y;
            }
          }
          epilogue<NT, EPI, I4>(a, acc, rt, g, t);
        }
        if (threadIdx.x == 0) a.counters[rb] = 0;
      }
    }
    consumer_sync_n<CW>();          // the reduction slots in shared memory are free for the next range
    u += ktb - kta;
  }
  if (a.csize > 1) {
    // rank 0 sums the ranks' partials in rank order (deterministic) straight from their shared
    // memory and runs the epilogue; no global scratch, fence or ticket
    cluster_sync_any();
    if (c % a.csize == 0 && !par) {
      float acc[NT][4];
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[n][q] = 0.f;
      const float* mine = reinterpret_cast<const float*>(ring) + (size_t)(rtw * 32 + lane) * (NT * 4);
      for (int r = 0; r < a.csize; ++r) {
        const uint32_t src = cluster_addr(mine, r);
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const float4 v = ld_cluster_v4(src + n * 16);
          acc[n][0] += v.x; acc[n][1] += v.y; acc[n][2] += v.z; acc[n][3] += v.w;
        }
      }
      epilogue<NT, EPI, I4>(a, acc, (c / a.csize) * tc::WARPS + rtw, g, t);
    }
    cluster_sync_any();             // no rank leaves while rank 0 may still read its shared memory
  }
}

// ------------------------------------------------------------------------------------ host side

// Shared memory to request so that at most k CTAs fit on one SM: the grid is sized for k per SM,
// and a programmatic launch places CTAs on whichever SMs free up first, so without the cap an SM
// that frees early takes one CTA more than the others and finishes last.
static size_t smem_for_ctas_per_sm(size_t need, int k) {
  static const int cap = env_int("AF_TC_OCC_CAP", 0);     // measured slower on B200: off by default
  if (!cap || k < 1) return need;
  const int per_sm = device_attr(cudaDevAttrMaxSharedMemoryPerMultiprocessor, 1);
  const int reserved = device_attr(cudaDevAttrReservedSharedMemoryPerBlock, 1024);
  const int per_block = device_attr(cudaDevAttrMaxSharedMemoryPerBlockOptin, 0);
  if (per_sm <= 1) return need;
  const long long floor_k = (long long)per_sm / (k + 1) - reserved + 16;   // k + 1 CTAs no longer fit
  size_t want = floor_k > (long long)need ? (size_t)((floor_k + 127) / 128 * 128) : need;
  if (per_block > 0 && want > (size_t)per_block) want = need;
  return want;
}

static int sm_count() { return device_attr(cudaDevAttrMultiProcessorCount, 148); }

// weight ring depth per format (AF_TC_STAGES / AF_TC_STAGES_I4, 2..6)
static int ring_stages(bool i4) {
  static const int s8 = env_int("AF_TC_STAGES", tc::STAGES), s4 = env_int("AF_TC_STAGES_I4", tc::STAGES);
  const int s = i4 ? s4 : s8;
  return s < 2 ? 2 : (s > tc::STAGES ? tc::STAGES : s);
}

static size_t smem_bytes(int NB, bool i4) {
  // weight ring | barriers | x ring | odd-warp sums [4 row tiles][32 lanes][8 floats]
  return (size_t)ring_stages(i4) * (i4 ? tc::STAGE_BYTES4 : tc::STAGE_BYTES) + SH_BYTES +
         (size_t)tc::XSLOTS * NB * tc::XSTRIDE * 2 + tc::WARPS * 32 * 8 * 4;
}

// the kernel's shared-memory limit and cluster permission, set once per device
template <int NT, int EPI, bool I4>
static cudaError_t set_attrs() {
  static PerDeviceOnce once;
  return once.run([] {
    const int optin = device_attr(cudaDevAttrMaxSharedMemoryPerBlockOptin, 0);
    cudaError_t e = cudaFuncSetAttribute(gemv_tc_kernel<NT, EPI, I4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         optin > (int)smem_bytes(16, I4) ? optin : (int)smem_bytes(16, I4));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemv_tc_kernel<NT, EPI, I4>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    return e;
  });
}

// CTAs of this instantiation resident at once on the current device (per SM x SMs)
template <int NT, int EPI, bool I4>
static int grid_for(int NB) {
  static PerDeviceInt<17> occ;
  const int per_sm = occ.get(NB, [NB] {
    if (set_attrs<NT, EPI, I4>() != cudaSuccess) { cudaGetLastError(); return 1; }
    int o = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, gemv_tc_kernel<NT, EPI, I4>, (Cw<I4>::n + 1) * 32,
                                                      smem_bytes(NB, I4)) != cudaSuccess || o < 1) {
      cudaGetLastError();
      o = 1;
    }
    const int cap = env_int("AF_TC_CTAS_PER_SM", 4);
    return o < cap ? o : cap;
  });
  return per_sm * sm_count();
}

// clusters of d CTAs that can be resident at once on the current device (0 if the query fails)
template <int NT, int EPI, bool I4>
static int clusters_for(int NB, int d) {
  static PerDeviceInt<17 * 17> cache;
  const int n = cache.get(NB * 17 + d, [NB, d] {
    if (set_attrs<NT, EPI, I4>() != cudaSuccess) { cudaGetLastError(); return -1; }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(d * 64);
    cfg.blockDim = dim3((Cw<I4>::n + 1) * 32);
    cfg.dynamicSmemBytes = smem_bytes(NB, I4);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = d;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int m = 0;
    if (cudaOccupancyMaxActiveClusters(&m, gemv_tc_kernel<NT, EPI, I4>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      m = 0;
    }
    return m > 0 ? m : -1;
  });
  return n > 0 ? n : 0;
}

template <bool I4>
static int clusters_any(int NB, int epi, int d) {
  const bool two = NB > 8;
  switch (epi) {
    case EPI_F32: return two ? clusters_for<2, EPI_F32, I4>(NB, d) : clusters_for<1, EPI_F32, I4>(NB, d);
    case EPI_F16: return two ? clusters_for<2, EPI_F16, I4>(NB, d) : clusters_for<1, EPI_F16, I4>(NB, d);
    case EPI_RESID: return two ? clusters_for<2, EPI_RESID, I4>(NB, d) : clusters_for<1, EPI_RESID, I4>(NB, d);
    default: return two ? clusters_for<2, EPI_SWIGLU, I4>(NB, d) : clusters_for<1, EPI_SWIGLU, I4>(NB, d);
  }
}

template <bool I4>
static int grid_any(int NB, int epi) {
  const bool two = NB > 8;
  switch (epi) {
    case EPI_F32: return two ? grid_for<2, EPI_F32, I4>(NB) : grid_for<1, EPI_F32, I4>(NB);
    case EPI_F16: return two ? grid_for<2, EPI_F16, I4>(NB) : grid_for<1, EPI_F16, I4>(NB);
    case EPI_RESID: return two ? grid_for<2, EPI_RESID, I4>(NB) : grid_for<1, EPI_RESID, I4>(NB);
    default: return two ? grid_for<2, EPI_SWIGLU, I4>(NB) : grid_for<1, EPI_SWIGLU, I4>(NB);
  }
}

// Grid geometry on the host. The bytes a CTA streams should be the same on every SM: a CTA is bound
// to one SM, and an SM hosting one more CTA than the others finishes last (at 4 CTAs against 3,
// a third later). Two layouts:
//  * more row blocks than resident CTAs: stream-K over all G = resident CTAs, U = RB * KT units split
//    evenly, so every CTA range spans at least one row block and a row block is shared by at most
//    two CTAs (owner fixup in the kernel);
//  * otherwise thread-block clusters: each row block gets a cluster of d CTAs (csize = d <= 16)
//    splitting its k range, the partials meeting in rank 0's shared memory. d maximises
//    balance * fill, balance = G / (SMs * ceil(G / SMs)) (how evenly the G = RB * d CTAs spread over
//    the SMs), fill = min(1, G / min_ctas) (enough bytes in flight), with G within the resident
//    capacity and the row blocks' clusters within `cfrac` percent of the clusters of d CTAs the GPU
//    holds at once (a cluster is placed whole within a GPC).
// `allow_cluster` false (scratch sizing) always describes the stream-K
// layout at the resident capacity; `maxc` is then the most CTAs sharing one row block.
static void plan_geometry(int N, int K, int NB, int epi, bool i4, int* G, int* maxc, int* csize,
                          bool allow_cluster = true) {
  static const int min_ctas = env_int("AF_TC_MIN_CTAS", 450);
  static const int use_cluster = env_int("AF_TC_CLUSTER", 1);
  static const int cfrac = env_int("AF_TC_CFRAC", 100);
  static const int max_d = env_int("AF_TC_MAX_CLUSTER", 16);
  const long long RB = (N + 63) / 64, KT = (K + 31) / 32;
  const long long slots = i4 ? grid_any<true>(NB, epi) : grid_any<false>(NB, epi);
  const long long sms = sm_count(), occ = slots / sms > 0 ? slots / sms : 1;
  *csize = 0;
  *maxc = 1;
  if (allow_cluster && use_cluster && RB <= slots) {
    long long best_d = 1;
    double best = -1.0;
    for (long long d = 1; d <= max_d && d <= KT; ++d) {
      const long long g = RB * d;
      if (g > slots) break;
      if (d > 1) {
        const long long fit = i4 ? clusters_any<true>(NB, epi, (int)d) : clusters_any<false>(NB, epi, (int)d);
        if (env_int("AF_TC_DEBUG", 0) > 1)
          fprintf(stderr, "[gemv_tc]   RB=%lld d=%lld: %lld clusters fit\n", RB, d, fit);
        if (RB * 100 > fit * cfrac) continue;
      }
      const double balance = (double)g / (double)(sms * ((g + sms - 1) / sms));
      const double fill = g >= min_ctas ? 1.0 : (double)g / min_ctas;
      const double score = balance * fill;
      if (score > best + 1e-9) { best = score; best_d = d; }
    }
    if (env_int("AF_TC_DEBUG", 0))
      fprintf(stderr, "[gemv_tc] N=%d K=%d NB=%d epi=%d i4=%d: RB=%lld slots=%lld cluster d=%lld (score %.3f)\n", N, K,
              NB, epi, (int)i4, RB, slots, best_d, best);
    *G = (int)(RB * best_d);
    *csize = (int)best_d;
    return;
  }
  long long g = occ * sms;
  if (g > RB * KT) g = RB * KT;
  *G = (int)g;
  const long long U = RB * KT;
  const long long per = U / g;
  *maxc = (int)((KT + per - 1) / (per > 0 ? per : 1)) + 1;
  if (allow_cluster && env_int("AF_TC_DEBUG", 0))
    fprintf(stderr, "[gemv_tc] N=%d K=%d NB=%d epi=%d i4=%d: RB=%lld stream-K G=%lld\n", N, K, NB, epi, (int)i4, RB, g);
}

void gemv_tc_grid(int N, int K, int NB, int epi, bool i4, int* G, int* csize) {
  int maxc = 0;
  plan_geometry(N, K, NB, epi, i4, G, &maxc, csize);
}

void gemv_tc_plan(int N, int K, int NB, int* S_out, int* nt_out) {
  int G, maxc, cs;
  plan_geometry(N, K, NB > 16 ? 16 : NB, EPI_F32, false, &G, &maxc, &cs, false);
  *S_out = maxc;
  *nt_out = NB <= 8 ? 1 : 2;
}

static size_t scratch_for_slice(int N, int K, int nb) {
  int G = 0, maxc = 0, maxc4 = 0, cs = 0;
  plan_geometry(N, K, nb, EPI_F32, false, &G, &maxc, &cs, false);
  plan_geometry(N, K, nb, EPI_F32, true, &G, &maxc4, &cs, false);
  if (maxc4 > maxc) maxc = maxc4;
  const int NT = nb <= 8 ? 1 : 2;
  const size_t RB = (N + 63) / 64;
  return tc::CNT_BYTES + RB * maxc * 64 * NT * 8 * 4;
}

size_t gemv_tc_scratch_bytes(int N, int K, int NB) {
  // enough for either weight format and every epilogue (the grid may differ with shared memory);
  // a batch above 16 runs as 16-row slices and a remainder, whose grid (and so its split) differs
  if (NB <= 16) return scratch_for_slice(N, K, NB);
  const size_t full = scratch_for_slice(N, K, 16);
  const size_t rest = NB % 16 ? scratch_for_slice(N, K, NB % 16) : 0;
  return full > rest ? full : rest;
}

template <int NT, int EPI, bool I4>
static cudaError_t launch_tc(GemvTcArgs a, cudaStream_t st, bool pdl) {
  const cudaError_t ae = set_attrs<NT, EPI, I4>();
  if (ae != cudaSuccess) return ae;
  int G = 0, maxc = 0, cs = 0;
  plan_geometry(a.N, a.K, a.NB, EPI, I4, &G, &maxc, &cs);
  a.maxc = maxc;
  a.csize = cs;
  a.nst = ring_stages(I4);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3((Cw<I4>::n + 1) * 32);
  cfg.dynamicSmemBytes = smem_for_ctas_per_sm(smem_bytes(a.NB, I4), (G + sm_count() - 1) / sm_count());
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cs > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cs;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemv_tc_kernel<NT, EPI, I4>, a);
}

static cudaError_t gemv_tc_launch16(GemvTcArgs a, cudaStream_t st, bool pdl);

// Batches above 16 run as 16-row slices of x (the weights stream once per slice).
cudaError_t gemv_tc_launch(const GemvTcArgs& a0, cudaStream_t st, bool pdl) {
  if (a0.NB < 1 || (a0.route && (a0.NB > 16 || !a0.rows || !a0.rcnt || a0.sel))) return cudaErrorInvalidValue;
  for (int b0 = 0; b0 < a0.NB; b0 += 16) {
    GemvTcArgs a = a0;
    a.NB = a0.NB - b0 < 16 ? a0.NB - b0 : 16;
    a.x = a0.x + (size_t)b0 * a0.ldx;
    const size_t esz = (a0.epi == EPI_F16 || a0.epi == EPI_SWIGLU) ? 2 : 4;
    a.y = static_cast<char*>(a0.y) + (size_t)b0 * a0.ldy * esz;
    if (a0.rw) a.rw = a0.rw + (size_t)b0 * a0.rw_e;           // routing weights follow the rows
    cudaError_t e = gemv_tc_launch16(a, st, pdl && b0 == 0);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

static cudaError_t gemv_tc_launch16(GemvTcArgs a, cudaStream_t st, bool pdl) {
  if (a.NB < 1 || a.NB > 16 || a.N <= 0 || a.K <= 0) return cudaErrorInvalidValue;
  if (a.K % 32 || a.ldx % 8) return cudaErrorInvalidValue;            // whole x chunks, 16-byte rows
  if (a.epi == EPI_SWIGLU && a.N % 16) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.w) & 15) || (reinterpret_cast<uintptr_t>(a.x) & 15)) return cudaErrorInvalidValue;
  a.Np = (a.N + 63) / 64 * 64;
  a.Kp = a.K;
  const size_t RB = a.Np / 64;
  if (RB * 4 > tc::CNT_BYTES) return cudaErrorInvalidValue;
  if (!a.scratch || a.scratch_bytes < gemv_tc_scratch_bytes(a.N, a.K, a.NB)) return cudaErrorInvalidValue;
  a.counters = reinterpret_cast<int*>(a.scratch);
  a.part = reinterpret_cast<float*>(static_cast<char*>(a.scratch) + tc::CNT_BYTES);
  cudaError_t e = cudaErrorInvalidValue;
  const bool two = a.NB > 8;
  if (a.wf != W_I8 && a.wf != W_I4G32) return cudaErrorInvalidValue;
  const bool i4 = a.wf == W_I4G32;
  if (!i4 && !a.scale) return cudaErrorInvalidValue;
#define AF_TC_CASE(EPIV)                                                                            \
  if (a.epi == EPIV)                                                                               \
    e = i4 ? (two ? launch_tc<2, EPIV, true>(a, st, pdl) : launch_tc<1, EPIV, true>(a, st, pdl))  \
           : (two ? launch_tc<2, EPIV, false>(a, st, pdl) : launch_tc<1, EPIV, false>(a, st, pdl));
  AF_TC_CASE(EPI_F32)
  AF_TC_CASE(EPI_F16)
  AF_TC_CASE(EPI_RESID)
  AF_TC_CASE(EPI_SWIGLU)
#undef AF_TC_CASE
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// Column of the k tile that mma k-index j of k-step s multiplies: lane t's B fragments (k 2t, 2t+1,
// 2t+8, 2t+9 of both k-steps) become the 8 consecutive x values [8t, 8t + 8) of the k tile.
AF_HD int tile_col(int s, int j) { return 8 * ((j & 7) >> 1) + 4 * s + 2 * (j >> 3) + (j & 1); }

// row-major int8 codes [N][K] -> [Np/64][Kp/32][4 row tiles][32 lanes][16 B], zero padded
__global__ void pack_i8_tiles_kernel(const int8_t* src, int N, int K, uint8_t* dst, int Np, int Kp) {
  const size_t total = (size_t)(Np / 16) * (Kp / 32) * 32;
  const int KT = Kp / 32;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
    const int lane = (int)(idx & 31);
    const size_t q = idx >> 5;                    // (rb, kt, w) flattened
    const int w = (int)(q % tc::WARPS);
    const size_t rk = q / tc::WARPS;
    const int kt = (int)(rk % KT);
    const int rb = (int)(rk / KT);
    const int rt = rb * tc::WARPS + w;
    const int g = lane >> 2, t = lane & 3;
    uint8_t out[16];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int rows[8] = {g, g, g + 8, g + 8, g, g, g + 8, g + 8};
      const int js[8] = {2 * t, 2 * t + 1, 2 * t, 2 * t + 1, 2 * t + 8, 2 * t + 9, 2 * t + 8, 2 * t + 9};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = rt * 16 + rows[j], c = kt * 32 + tile_col(s, js[j]);
        out[8 * s + j] = (r < N && c < K) ? (uint8_t)src[(size_t)r * K + c] : 0;
      }
    }
    uint4 v;
    memcpy(&v, out, 16);
    reinterpret_cast<uint4*>(dst)[idx] = v;
  }
}

cudaError_t pack_i8_tiles(const int8_t* src, int N, int K, uint8_t* dst, cudaStream_t st) {
  const int Np = (N + 63) / 64 * 64, Kp = (K + 31) / 32 * 32;
  const size_t total = (size_t)(Np / 16) * (Kp / 32) * 32;
  unsigned blocks = (unsigned)((total + 255) / 256);
  if (blocks > 65535u * 8) blocks = 65535u * 8;
  pack_i8_tiles_kernel<<<blocks, 256, 0, st>>>(src, N, K, dst, Np, Kp);
  return cudaGetLastError();
}

size_t pack_i8_tiles_bytes(int N, int K) {
  return (size_t)((N + 63) / 64 * 64) * ((K + 31) / 32 * 32);
}

// group-32 int4 [N][K/2] (low nibble first, nibble = code + 8) + scales [N][K/32] ->
// [Np/64][K/32][4 row tiles x 32 lanes x 8 B | 64 fp16 scales]. Padding rows hold nibble 8 (code 0)
// and scale 0. One thread per (row block, k tile, 16-byte piece of the unit).
__global__ void pack_i4_tiles_kernel(const uint8_t* src, const __half* sc, int N, int K, uint8_t* dst, int Np) {
  const int KT = K / 32;
  constexpr int PIECES = tc::UNIT4 / 16;                   // 72: 64 weight pieces + 8 scale pieces
  const size_t total = (size_t)(Np / 64) * KT * PIECES;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
    const int piece = (int)(idx % PIECES);
    const size_t u = idx / PIECES;
    const int kt = (int)(u % KT), rb = (int)(u / KT);
    uint8_t out[16];
    if (piece < 64) {
      // pieces 0..63: two lanes (8 bytes each) of row tile piece / 16
      const int w = piece / 16;
      for (int half = 0; half < 2; ++half) {
        const int lane = (piece % 16) * 2 + half;
        const int g = lane >> 2, t = lane & 3;
        const int rt = rb * tc::WARPS + w;
        for (int s = 0; s < 2; ++s) {
          uint32_t word = 0;
          const int rows[8] = {g, g + 8, g, g + 8, g, g + 8, g, g + 8};
          const int js[8] = {2 * t, 2 * t, 2 * t + 8, 2 * t + 8, 2 * t + 1, 2 * t + 1, 2 * t + 9, 2 * t + 9};
          for (int j = 0; j < 8; ++j) {                     // nibble slot j sits at bit 4j
            const int r = rt * 16 + rows[j], c = kt * 32 + tile_col(s, js[j]);
            uint32_t nib = 8;
            if (r < N) {
              const uint8_t b = src[(size_t)r * (K / 2) + c / 2];
              nib = (c & 1) ? (b >> 4) : (b & 15);
            }
            word |= nib << (4 * j);
          }
          memcpy(out + half * 8 + s * 4, &word, 4);
        }
      }
    } else {
      // scales of row tile w in the order (g, g + 8) for g = 0..7: one 32-bit load per lane
      const int i0 = (piece - 64) * 8;
      for (int i = 0; i < 8; ++i) {
        const int idx = i0 + i, w = idx / 16, gg = (idx % 16) / 2, hi = idx & 1;
        const int r = rb * 64 + w * 16 + gg + 8 * hi;
        const __half v = r < N ? sc[(size_t)r * KT + kt] : __float2half(0.f);
        memcpy(out + 2 * i, &v, 2);
      }
    }
    uint4 v;
    memcpy(&v, out, 16);
    reinterpret_cast<uint4*>(dst)[idx] = v;
  }
}

cudaError_t pack_i4_tiles(const uint8_t* src, const __half* scales, int N, int K, uint8_t* dst, cudaStream_t st) {
  if (K % 32) return cudaErrorInvalidValue;
  const int Np = (N + 63) / 64 * 64;
  const size_t total = (size_t)(Np / 64) * (K / 32) * (tc::UNIT4 / 16);
  unsigned blocks = (unsigned)((total + 255) / 256);
  if (blocks > 65535u * 8) blocks = 65535u * 8;
  pack_i4_tiles_kernel<<<blocks, 256, 0, st>>>(src, scales, N, K, dst, Np);
  return cudaGetLastError();
}

size_t pack_i4_tiles_bytes(int N, int K) { return (size_t)((N + 63) / 64) * (K / 32) * tc::UNIT4; }

}  // namespace af
