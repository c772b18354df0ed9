// A chain of decode GEMVs in one persistent launch - e.g. o_proj (+ the MLP RMSNorm), gate|up,
// down (+ the next layer's attention RMSNorm), the next layer's qkv - on the tensor-core GEMV's
// tiles, ring and fragment math (tc_common.cuh).
//
// Why. A decode step is a sequence of weight streams, each a few tens of MB, with a data dependency
// between consecutive ones. Run as separate launches, each GEMV pays a ramp (its CTAs only become
// resident once the previous kernel's leave, then every CTA waits for its first weight stage while
// the DRAM serves the whole wave) and a drain (the last CTAs' reduction and epilogue while the rest
// of the GPU idles). The weights do not depend on the data, so here every CTA's producer thread
// streams the weights of ALL its jobs back to back into one ring; only the consumers wait at a job
// boundary, and while they do the ring keeps filling with the next job's weights (up to ~190 KB
// per SM, a few microseconds of HBM time), so the stream does not stop at the boundary.
//
// Work split. Every job is cut stream-K style: its RB x KT units (one k tile of one 64-row block)
// in G contiguous equal ranges, one per CTA, so each CTA streams the same bytes of every job. A row
// block split over several CTAs is finished by the LAST of them to arrive (a ticket per row
// block): each piece writes its fp32 partial to its slot, and the last sums the slots in piece order
// (deterministic) and runs the epilogue. Nobody waits for a partial.
//
// Job boundaries. The CTA that finishes a job's last row block runs the job's RMSNorm (if any) and
// then publishes the job as ready (release); a second producer thread per CTA (its own warp) waits (bounded, with
// acquire) for the previous job to be ready before it copies the next job's x chunks into the x
// ring. Counters are reset by the CTA that last uses them, so the launch can be replayed.
//
// Residency. All G CTAs must be resident at once (a CTA waiting for a job boundary holds its SM):
// G = resident CTAs of this kernel per SM x SMs, and a programmatic dependent launch of the next
// kernel cannot start before every CTA here has started. Every wait is bounded; on a timeout the
// error word gets AF_DEV_WAIT_TIMEOUT, the CTA's consumers leave together and each producer waits
// (bounded) for the copies it issued.
#include <cstdlib>

#include "af_common.cuh"
#include "af_kernels.h"
#include "tc_common.cuh"

namespace af {

namespace {

constexpr int CHAIN_MAX_STAGES = 12;          // weight ring depth: 6 at 4 CTAs per SM, 12 at 2
constexpr long long FLAG_LIMIT = 1ll << 21;     // ~1 s of L2 polls with 32 ns sleeps

struct ChainShared {
  uint64_t full[CHAIN_MAX_STAGES];
  uint64_t empty[CHAIN_MAX_STAGES];
  uint64_t xfull[tc::XSLOTS];
  uint64_t xempty[tc::XSLOTS];
  int cabort;        // a consumer gave up (written by consumers, read after a consumer barrier)
  int bcast;         // thread 0's ticket result for the other consumer threads
  float nsum[8];     // per-warp partial sums of the RMSNorm tail
};
constexpr int CHAIN_SH_BYTES = 512;
static_assert(sizeof(ChainShared) <= CHAIN_SH_BYTES, "ChainShared grew past its slot");

// the epilogue of one 16-row tile of job J (rows rt*16 + g and + 8, batch columns of this lane)
template <int NT, bool I4>
AF_DEV void chain_epilogue(const ChainJob& J, int NB, const float (&acc)[NT][4], int rt, int g, int t) {
  const int r0 = rt * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int b = n * 8 + 2 * t + h;
      if (b >= NB) continue;
      const float v0 = acc[n][h], v1 = acc[n][2 + h];
      if (J.epi == EPI_SWIGLU) {
        if (r1 >= J.N) continue;
        float gv = I4 ? v0 : __fmul_rn(v0, h2f(J.scale[r0]));
        float uv = I4 ? v1 : __fmul_rn(v1, h2f(J.scale[r1]));
        if (J.bias) { gv = __fadd_rn(gv, h2f(J.bias[r0])); uv = __fadd_rn(uv, h2f(J.bias[r1])); }
        reinterpret_cast<__half*>(J.y)[(size_t)b * J.ldy + rt * 8 + g] = f2h(silu_f(gv) * uv);
      } else {
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int row = rr ? r1 : r0;
          if (row >= J.N) continue;
          float v = I4 ? (rr ? v1 : v0) : __fmul_rn(rr ? v1 : v0, h2f(J.scale[row]));
          if (J.bias) v = __fadd_rn(v, h2f(J.bias[row]));
          const size_t o = (size_t)b * J.ldy + row;
          if (J.epi == EPI_F32) reinterpret_cast<float*>(J.y)[o] = v;
          else if (J.epi == EPI_F16) reinterpret_cast<__half*>(J.y)[o] = f2h(v);
          else reinterpret_cast<float*>(J.y)[o] = __ldcg(reinterpret_cast<const float*>(J.y) + o) + v;
        }
      }
    }
  }
}

// the job's RMSNorm on this CTA's consumer threads (the rmsnorm kernel's formula:
// x / max(|x|, floor) * g). It sits on the chain's critical path (every CTA waits for it), so each
// thread keeps NL independent 16-byte loads in flight instead of one L2 round trip per element.
template <int CW>
AF_DEV void chain_norm(const ChainJob& J, int NB, ChainShared* sh) {
  constexpr int NL = 4;
  const int tid = threadIdx.x, nthr = CW * 32, warp = tid >> 5, lane = tid & 31;
  const bool vec = (J.nd % 4) == 0 && (J.ldnx % 4) == 0 && (J.ldno % 4) == 0 &&
                   (reinterpret_cast<uintptr_t>(J.nx) & 15) == 0 && (reinterpret_cast<uintptr_t>(J.nout) & 7) == 0 &&
                   (reinterpret_cast<uintptr_t>(J.ng) & 7) == 0;
  const int n4 = J.nd / 4;
  for (int b = 0; b < NB; ++b) {
    const float* x = J.nx + (size_t)b * J.ldnx;
    __half* out = J.nout + (size_t)b * J.ldno;
    float ss = 0.f;
    if (vec) {
      const float4* x4 = reinterpret_cast<const float4*>(x);
      for (int i0 = tid; i0 < n4; i0 += nthr * NL) {
        float4 v[NL];
#pragma unroll
        for (int u = 0; u < NL; ++u) {
          const int i = i0 + u * nthr;
          v[u] = i < n4 ? __ldcg(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < NL; ++u) {
          ss = fmaf(v[u].x, v[u].x, ss); ss = fmaf(v[u].y, v[u].y, ss);
          ss = fmaf(v[u].z, v[u].z, ss); ss = fmaf(v[u].w, v[u].w, ss);
        }
      }
    } else {
      for (int i = tid; i < J.nd; i += nthr) {
        const float v = __ldcg(x + i);
        ss = fmaf(v, v, ss);
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) sh->nsum[warp] = ss;
    consumer_sync_n<CW>();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < CW; ++w) tot += sh->nsum[w];
    const float sn = fmaxf(sqrtf(tot), J.nfloor);
    if (vec) {
      const float4* x4 = reinterpret_cast<const float4*>(x);
      const uint2* g4 = reinterpret_cast<const uint2*>(J.ng);
      uint2* o4 = reinterpret_cast<uint2*>(out);
      for (int i0 = tid; i0 < n4; i0 += nthr * NL) {
        float4 v[NL];
        uint2 gv[NL];
#pragma unroll
        for (int u = 0; u < NL; ++u) {
          const int i = i0 + u * nthr;
          if (i < n4) { v[u] = __ldcg(x4 + i); gv[u] = __ldg(g4 + i); }
        }
#pragma unroll
        for (int u = 0; u < NL; ++u) {
          const int i = i0 + u * nthr;
          if (i >= n4) continue;
          const __half2* g2 = reinterpret_cast<const __half2*>(&gv[u]);
          const float2 ga = __half22float2(g2[0]), gb = __half22float2(g2[1]);
          __half2 r[2];
          r[0] = __halves2half2(f2h(__fdiv_rn(v[u].x, sn) * ga.x), f2h(__fdiv_rn(v[u].y, sn) * ga.y));
          r[1] = __halves2half2(f2h(__fdiv_rn(v[u].z, sn) * gb.x), f2h(__fdiv_rn(v[u].w, sn) * gb.y));
          o4[i] = *reinterpret_cast<const uint2*>(r);
        }
      }
    } else {
      for (int i = tid; i < J.nd; i += nthr) out[i] = f2h(__fdiv_rn(__ldcg(x + i), sn) * h2f(J.ng[i]));
    }
    consumer_sync_n<CW>();           // nsum is reused by the next row
  }
}

// CTAs that work on job J: all G, or one per unit when the job has fewer units than CTAs (every
// working CTA then has a non-empty range, so a row block's pieces are exactly CTAs cf..cl)
AF_HD int job_grid(const ChainJob& J, int G) { return J.U < (long long)G ? (int)J.U : G; }

// a ticket: release orders this CTA's earlier writes (made CTA-wide by the barrier before it) ahead of
// the count, acquire makes the writes of the CTAs counted before visible (to the CTA after the
// barrier that follows); no full memory barrier per thread
AF_DEV int ticket(int* p) {
  int r;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(r) : "l"(p) : "memory");
  return r;
}

AF_DEV bool wait_flag(const int* f) {
  SpinBudget budget;
  for (long long i = 0; i < FLAG_LIMIT && !budget.spent(); ++i) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (v) return true;
    __nanosleep(32);
  }
  return false;
}

}  // namespace

// consumer warps, then the weight producer's warp, then the x producer's warp (each producer is one
// thread of a warp of its own, so that neither waits behind the other's spins)
template <bool I4> struct ChainThreads {
  static constexpr int n = (Cw<I4>::n + 2) * 32;
  static constexpr int min_ctas = I4 ? 3 : 4;     // resident CTAs per SM the register budget keeps
};

template <int NT, bool I4>
__global__ void __launch_bounds__(ChainThreads<I4>::n, ChainThreads<I4>::min_ctas) gemv_chain_kernel(const __grid_constant__ GemvChainArgs a) {
  constexpr int CW = Cw<I4>::n;
  using F = tc::Fmt<I4>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char* ring = smem_raw;                                          // [STAGES][F::stage]
  const int NS = a.nstages;                                               // weight ring depth
  ChainShared* sh = reinterpret_cast<ChainShared*>(smem_raw + NS * F::stage);
  __half* xring = reinterpret_cast<__half*>(smem_raw + NS * F::stage + CHAIN_SH_BYTES);
  const int NB = a.NB;
  const int xslot_halves = NB * tc::XSTRIDE;
  float* red = reinterpret_cast<float*>(smem_raw + NS * F::stage + CHAIN_SH_BYTES +
                                        (size_t)tc::XSLOTS * xslot_halves * 2);   // [4][32][NT*4]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, c = blockIdx.x;

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

  if (warp >= CW) {
    if (warp == CW && lane == 0) {
      // ---------------------------------------------------------- weight producer: every job's
      // weights back to back, never waiting for data (the weights are constant)
      const uint64_t pol = a.evict_first ? l2_evict_first_policy() : 0;
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int j = 0; j < a.njobs && ok; ++j) {
        const ChainJob& J = a.job[j];
        const char* W = static_cast<const char*>(J.w);
        const int Gj = job_grid(J, G);
        if (c >= Gj) continue;
        const long long u1 = unit_begin(c + 1, J.U, Gj);
        for (long long u = unit_begin(c, J.U, Gj); u < u1 && ok;) {
          const int rb = (int)(u / J.KT), kta = (int)(u % J.KT);
          const int ktb = (int)min((long long)J.KT, kta + (u1 - u));
          for (int kc = kta; kc < ktb && ok; kc += tc::XKT) {
            const int kce = min(kc + tc::XKT, ktb);
            for (int kt = kc; kt < kce; kt += F::ks) {
              const int nk = min(F::ks, kce - kt);
              if (!mbar_wait(&sh->empty[stage], phase ^ 1)) { ok = false; break; }
              mbar_arrive_expect_tx(&sh->full[stage], (uint32_t)nk * F::unit);
              bulk_w(ring + (size_t)stage * F::stage, W + ((size_t)rb * J.KT + kt) * F::unit, nk * F::unit,
                     &sh->full[stage], a.evict_first, pol);
              ++issued;
              if (++stage == NS) { stage = 0; phase ^= 1; }
            }
          }
          u += ktb - kta;
        }
      }
      if (!ok) af_set_err(a.err, AF_DEV_WAIT_TIMEOUT);
      // the ring must outlive every copy issued: wait (bounded) for the last ones to land
      const int tail = issued < NS ? issued : NS;
      for (int i = 0; i < tail; ++i) {
        if (--stage < 0) { stage = NS - 1; phase ^= 1; }
        mbar_wait(&sh->full[stage], phase);
      }
    } else if (warp == CW + 1 && lane == 0) {
      // ---------------------------------------------------------- x producer: a job's input rows
      // once the previous job (and its norm) is complete
      int xs = 0, issued = 0;
      uint32_t xphase = 0;
      bool ok = true;
      for (int j = 0; j < a.njobs && ok; ++j) {
        const ChainJob& J = a.job[j];
        if (j == 0) {
          pdl_wait();
        } else {
          if (!wait_flag(a.ready + j - 1)) { ok = false; break; }
          asm volatile("fence.proxy.async.global;" ::: "memory");   // generic writes -> bulk-copy reads
        }
        const int Gj = job_grid(J, G);
        if (c >= Gj) continue;
        const long long u1 = unit_begin(c + 1, J.U, Gj);
        for (long long u = unit_begin(c, J.U, Gj); u < u1 && ok;) {
          const int kta = (int)(u % J.KT);
          const int ktb = (int)min((long long)J.KT, kta + (u1 - u));
          for (int kc = kta; kc < ktb; kc += tc::XKT) {
            const int kce = min(kc + tc::XKT, ktb);
            if (!mbar_wait(&sh->xempty[xs], xphase ^ 1)) { ok = false; break; }
            const uint32_t xbytes = (uint32_t)(kce - kc) * 32 * 2;
            mbar_arrive_expect_tx(&sh->xfull[xs], xbytes * NB);
            for (int b = 0; b < NB; ++b)
              bulk_g2s(xring + (size_t)xs * xslot_halves + (size_t)b * tc::XSTRIDE,
                       J.x + (size_t)b * J.ldx + (size_t)kc * 32, xbytes, &sh->xfull[xs]);
            ++issued;
            if (++xs == tc::XSLOTS) { xs = 0; xphase ^= 1; }
          }
          u += ktb - kta;
        }
      }
      if (!ok) af_set_err(a.err, AF_DEV_WAIT_TIMEOUT);
      // this CTA reads no more job flags: the last CTA to get here resets them for the next launch
      // (the last job publishes no flag, nobody waits for it)
      __threadfence();
      if (atomicAdd(a.exits, 1) == G - 1) {
        __threadfence();
        for (int j = 0; j + 1 < a.njobs; ++j) a.ready[j] = 0;
        *a.exits = 0;
        __threadfence();
      }
      const int tail = issued < tc::XSLOTS ? issued : tc::XSLOTS;
      for (int i = 0; i < tail; ++i) {
        if (--xs < 0) { xs = tc::XSLOTS - 1; xphase ^= 1; }
        mbar_wait(&sh->xfull[xs], xphase);
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumers (4 or 8 warps)
  const int g = lane >> 2, t = lane & 3;
  const int rtw = warp & 3, par = warp >> 2;          // par: 0 with 4 consumer warps
  constexpr int NBP = NT * 8;
  pdl_wait();
  pdl_trigger();
  int stage = 0, xs = 0;
  uint32_t phase = 0, xphase = 0;
  bool quit = false;
  for (int j = 0; j < a.njobs && !quit; ++j) {
    const ChainJob& J = a.job[j];
    const int KT = J.KT;
    const int Gj = job_grid(J, G);
    if (c >= Gj) continue;
    const long long U = J.U, u1 = unit_begin(c + 1, U, Gj);
    for (long long u = unit_begin(c, U, Gj); u < u1;) {
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
        if (*reinterpret_cast<volatile int*>(&sh->cabort) || !mbar_wait(&sh->xfull[xs], xphase)) {
          stuck = true;
          break;
        }
        const __half* xsl = xring + (size_t)xs * xslot_halves;
        for (int kt = kc; kt < kce; kt += F::ks) {
          const int nk = min(F::ks, kce - kt);
          if (!mbar_wait(&sh->full[stage], phase)) { stuck = true; break; }
          consume_stage<I4, NT, CW / 4>(ring + (size_t)stage * F::stage, nk, xsl + (kt - kc) * 32, tc::XSTRIDE, NB,
                                        lane, rtw, par, acc, acc2);
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
      if (*reinterpret_cast<volatile int*>(&sh->cabort)) { quit = true; break; }
      if (CW == 8 && !par) {
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[n][q] += rw[n * 4 + q];
      }
      const int rt = rb * tc::WARPS + rtw;
      bool finished = false;                 // this CTA completed row block rb (uniform in the CTA)
      if (kta == 0 && ktb == KT) {
        if (!par) chain_epilogue<NT, I4>(J, NB, acc, rt, g, t);
        finished = true;
      } else {
        // a piece of a shared row block: publish it; the last piece to arrive sums them all
        const int cf = owner_of((long long)rb * KT, U, Gj), cl = owner_of((long long)rb * KT + KT - 1, U, Gj);
        const int nc = cl - cf + 1, jj = c - cf;
        const int r0 = rtw * 16 + g, r1 = r0 + 8;
        if (!par) {
          float* slot = J.part + (((size_t)rb * J.maxc + jj) * 64) * NBP;
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            const int c0 = n * 8 + 2 * t;
            if (c0 >= NB) continue;
            __stcg(reinterpret_cast<float2*>(slot + (size_t)r0 * NBP + c0), make_float2(acc[n][0], acc[n][1]));
            __stcg(reinterpret_cast<float2*>(slot + (size_t)r1 * NBP + c0), make_float2(acc[n][2], acc[n][3]));
          }
        }
        consumer_sync_n<CW>();
        if (threadIdx.x == 0) sh->bcast = ticket(J.cnt + rb);
        consumer_sync_n<CW>();
        if (sh->bcast == nc - 1) {
          if (!par) {
            float s[NT][4];
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
              for (int q = 0; q < 4; ++q) s[n][q] = 0.f;
            // the pieces in order (deterministic), two pieces' loads in flight at a time
            for (int p0 = 0; p0 < nc; p0 += 2) {
#pragma unroll
              for (int n = 0; n < NT; ++n) {
                const int c0 = n * 8 + 2 * t;
                if (c0 >= NB) continue;
                float2 q0[2], q1[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                  if (p0 + u >= nc) break;
                  const float* sp = J.part + (((size_t)rb * J.maxc + p0 + u) * 64) * NBP;
                  q0[u] = __ldcg(reinterpret_cast<const float2*>(sp + (size_t)r0 * NBP + c0));
                  q1[u] = __ldcg(reinterpret_cast<const float2*>(sp + (size_t)r1 * NBP + c0));
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                  if (p0 + u >= nc) break;
                  s[n][0] += q0[u].x; s[n][1] += q0[u].y; s[n][2] += q1[u].x; s[n][3] += q1[u].y;
                }
              }
            }
            chain_epilogue<NT, I4>(J, NB, s, rt, g, t);
          }
          if (threadIdx.x == 0) J.cnt[rb] = 0;
          finished = true;
        }
      }
      if (finished) {
        consumer_sync_n<CW>();               // this row block's outputs before its count
        if (threadIdx.x == 0) sh->bcast = ticket(a.done + j);
        consumer_sync_n<CW>();
        if (sh->bcast == J.RB - 1) {
          // the job's last row block: its norm, then the job is ready for the next one
          if (J.nd) chain_norm<CW>(J, NB, sh);
          consumer_sync_n<CW>();
          if (threadIdx.x == 0) {
            a.done[j] = 0;
            if (j + 1 < a.njobs) asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(a.ready + j), "r"(1) : "memory");
          }
        }
      }
      consumer_sync_n<CW>();                 // red / bcast are reused by the next range
      u += ktb - kta;
    }
  }
}

// ------------------------------------------------------------------------------------ host side

namespace {

constexpr size_t CHAIN_HDR = 256;                // done[8] | ready[8] | exits
// Every chain op of a program shares one scratch buffer, so the counters (which must read zero at
// the start of every launch) live at the same place for every job slot whatever the chain's shapes:
// CHAIN_CNT_CAP row-block tickets per job slot, then the partial sums (rewritten before each read)
constexpr int CHAIN_CNT_CAP = 4096;
constexpr size_t CHAIN_CNT_BYTES = (size_t)CHAIN_MAX_JOBS * CHAIN_CNT_CAP * 4;

// CTAs per SM the chain is sized for (env AF_CHAIN_CTAS_PER_SM: 4 with a 6-stage ring, or 2 with 12)
int chain_ctas_per_sm() {
  static const int v = env_int("AF_CHAIN_CTAS_PER_SM", 4) <= 2 ? 2 : 4;
  return v;
}
int chain_stages() { return chain_ctas_per_sm() == 2 ? CHAIN_MAX_STAGES : 6; }

size_t chain_smem(int NB, bool i4) {
  return (size_t)chain_stages() * (i4 ? tc::STAGE_BYTES4 : tc::STAGE_BYTES) + CHAIN_SH_BYTES +
         (size_t)tc::XSLOTS * NB * tc::XSTRIDE * 2 + tc::WARPS * 32 * 8 * 4;
}

template <int NT, bool I4>
cudaError_t chain_attrs() {
  static PerDeviceOnce once;
  return once.run([] {
    return cudaFuncSetAttribute(gemv_chain_kernel<NT, I4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)chain_smem(16, I4));
  });
}

// CTAs of the chain kernel resident at once on the current device: the whole grid must be
template <int NT, bool I4>
int chain_grid(int NB) {
  static PerDeviceInt<17> occ;
  const int per_sm = occ.get(NB, [NB] {
    if (chain_attrs<NT, I4>() != cudaSuccess) { cudaGetLastError(); return 0; }
    int o = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, gemv_chain_kernel<NT, I4>, ChainThreads<I4>::n,
                                                      chain_smem(NB, I4)) != cudaSuccess) {
      cudaGetLastError();
      o = 0;
    }
    const int cap = chain_ctas_per_sm();
    return o < cap ? o : cap;
  });
  return per_sm * device_attr(cudaDevAttrMultiProcessorCount, 148);
}

int chain_grid_any(int NB, bool i4) {
  const bool two = NB > 8;
  return i4 ? (two ? chain_grid<2, true>(NB) : chain_grid<1, true>(NB))
            : (two ? chain_grid<2, false>(NB) : chain_grid<1, false>(NB));
}

long long unit_begin_h(int c, long long U, int G) { return (long long)c * U / G; }
int owner_h(long long u, long long U, int G) {
  int c = (int)((u * G) / U);
  while (c + 1 < G && unit_begin_h(c + 1, U, G) <= u) ++c;
  while (c > 0 && unit_begin_h(c, U, G) > u) --c;
  return c;
}

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

// per-job geometry and the scratch layout for a grid of G CTAs; returns the scratch bytes
size_t chain_layout(GemvChainArgs& a, int G) {
  const int NT = a.NB > 8 ? 2 : 1;
  size_t off = CHAIN_HDR + CHAIN_CNT_BYTES;
  for (int j = 0; j < a.njobs; ++j) {
    ChainJob& J = a.job[j];
    J.RB = (J.N + 63) / 64;
    J.KT = J.K / 32;
    J.U = (long long)J.RB * J.KT;
    int maxc = 1;
    const int Gj = job_grid(J, G);
    for (int rb = 0; rb < J.RB; ++rb) {
      const int n = owner_h((long long)rb * J.KT + J.KT - 1, J.U, Gj) - owner_h((long long)rb * J.KT, J.U, Gj) + 1;
      if (n > maxc) maxc = n;
    }
    J.maxc = maxc;
  }
  for (int j = 0; j < a.njobs; ++j) {
    const ChainJob& J = a.job[j];
    off += align256((size_t)J.RB * J.maxc * 64 * NT * 8 * 4);
  }
  return off;
}

void chain_bind(GemvChainArgs& a) {
  const int NT = a.NB > 8 ? 2 : 1;
  char* base = static_cast<char*>(a.scratch);
  a.done = reinterpret_cast<int*>(base);
  a.ready = a.done + CHAIN_MAX_JOBS;
  a.exits = a.ready + CHAIN_MAX_JOBS;
  for (int j = 0; j < a.njobs; ++j) a.job[j].cnt = reinterpret_cast<int*>(base + CHAIN_HDR) + (size_t)j * CHAIN_CNT_CAP;
  size_t off = CHAIN_HDR + CHAIN_CNT_BYTES;
  for (int j = 0; j < a.njobs; ++j) {
    ChainJob& J = a.job[j];
    J.part = reinterpret_cast<float*>(base + off);
    off += align256((size_t)J.RB * J.maxc * 64 * NT * 8 * 4);
  }
}

bool chain_valid(const GemvChainArgs& a) {
  if (a.njobs < 1 || a.njobs > CHAIN_MAX_JOBS || a.NB < 1 || a.NB > 16) return false;
  if (a.wf != W_I8 && a.wf != W_I4G32) return false;
  for (int j = 0; j < a.njobs; ++j) {
    const ChainJob& J = a.job[j];
    if (J.N <= 0 || J.K <= 0 || J.K % 32 || J.ldx % 8 || J.ldx < J.K || !J.w || !J.x || !J.y) return false;
    if ((J.N + 63) / 64 > CHAIN_CNT_CAP) return false;
    if ((reinterpret_cast<uintptr_t>(J.w) & 15) || (reinterpret_cast<uintptr_t>(J.x) & 15)) return false;
    if (J.epi < EPI_F32 || J.epi > EPI_SWIGLU) return false;
    if (J.epi == EPI_SWIGLU && J.N % 16) return false;
    if (a.wf == W_I8 && !J.scale) return false;
    if (J.nd && (!J.nx || !J.ng || !J.nout || J.ldnx < J.nd || J.ldno < J.nd)) return false;
  }
  return true;
}

template <int NT, bool I4>
cudaError_t launch_chain(const GemvChainArgs& a, int G, cudaStream_t st, bool pdl) {
  const cudaError_t ae = chain_attrs<NT, I4>();
  if (ae != cudaSuccess) return ae;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(ChainThreads<I4>::n);
  cfg.dynamicSmemBytes = chain_smem(a.NB, I4);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_chain_kernel<NT, I4>, a);
}

}  // namespace

size_t gemv_chain_scratch_bytes(const GemvChainArgs& a0) {
  if (a0.njobs < 1 || a0.njobs > CHAIN_MAX_JOBS || a0.NB < 1 || a0.NB > 16) return 0;
  GemvChainArgs a = a0;
  const int G = chain_grid_any(a.NB, a.wf == W_I4G32);
  return chain_layout(a, G > 0 ? G : 4 * 148);
}

cudaError_t gemv_chain_launch(GemvChainArgs a, cudaStream_t st, bool pdl) {
  if (!chain_valid(a)) return cudaErrorInvalidValue;
  const bool i4 = a.wf == W_I4G32;
  const int G = chain_grid_any(a.NB, i4);
  if (G < 1) return cudaErrorInvalidConfiguration;
  const size_t need = chain_layout(a, G);
  if (!a.scratch || a.scratch_bytes < need) return cudaErrorInvalidValue;
  chain_bind(a);
  a.nstages = chain_stages();
  const bool two = a.NB > 8;
  cudaError_t e = i4 ? (two ? launch_chain<2, true>(a, G, st, pdl) : launch_chain<1, true>(a, G, st, pdl))
                     : (two ? launch_chain<2, false>(a, G, st, pdl) : launch_chain<1, false>(a, G, st, pdl));
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace af
