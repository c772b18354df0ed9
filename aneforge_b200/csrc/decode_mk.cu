// Decode megakernel: ONE persistent, cooperatively launched grid runs a whole decode step — the
// embedding gather, every decoder layer and the final norm — for 1..8 sequences. It replaces the
// 7 launches per layer of the per-op path (rmsnorm, qkv GEMV, attention, o GEMV, rmsnorm, gate|up
// GEMV, down GEMV), whose fixed costs (launch, pipeline fill, split-K tail, per kernel) dominate a
// batch-1 step, with grid-wide barriers between the phases that depend on each other.
//
// Layout of a CTA (2 per SM when shared memory allows): one producer warp + 8 consumer warps.
//  * The producer (one thread) walks the WHOLE step's weight stream — layer by layer, qkv, o,
//    gate|up, down, each split stream-K over the grid exactly as the consumers will walk it — and
//    bulk-copies (cp.async.bulk into its own shared memory) 8-9 KB stages into an mbarrier ring. Weights do not
//    depend on activations, so it runs ahead across phase boundaries and keeps HBM busy while the
//    consumers wait at a grid barrier, compute attention or stage the next input.
//  * The consumers run the phases in order. GEMV phase: stage the CTA's slice of x in shared
//    memory (normalising the fp32 residual on the fly for the qkv and gate|up inputs: the reference
//    RMSNorm, computed redundantly by every CTA from the same row), then multiply the ring stages
//    exactly as the stand-alone tensor-core GEMV does (two warps per row tile split the k tiles by
//    parity; split row blocks are finished by the last ticket holder, deterministically). Attention
//    phase: (sequence, kv head, split) tasks over the CTAs, each the split-K flash-decode step of the
//    stand-alone kernel, merged by the last split. Every phase ends with a grid barrier.
// Every wait (ring, grid barrier) is bounded in time and gives up when any CTA recorded an error;
// the producer always waits (time-bounded) for its copies in flight before it exits.
#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "af_common.cuh"
#include "af_kernels.h"
#include "tc_common.cuh"
#include "attn_common.cuh"

namespace af {

namespace mk {
constexpr int CW = 8;                          // consumer warps
constexpr int NTHR = (CW + 1) * 32;
constexpr int MAXST = 16;                      // ring stages (runtime count <= this)
constexpr int XPAD = 32;                       // halves of padding per staged x row
constexpr int NBMAX = 8;
constexpr unsigned long long SPIN_NS = 2000000000ull;   // 2 s
constexpr int SH_BYTES = 1024;
constexpr int RED_BYTES = tc::WARPS * 32 * 8 * 4;
}  // namespace mk

struct MkSmem {                      // shared-memory layout of one launch (bytes / halves)
  int nst;                           // ring stages
  int xsn, xsp;                      // staged-x row strides (halves): norm phases, plain phases
  int red_off;                       // odd-warp sums, after the x region
};

struct MkShared {
  uint64_t full[mk::MAXST];
  uint64_t empty[mk::MAXST];
  int ticket, cabort, abort, last;
  float sn[mk::NBMAX];
  float wsum[mk::CW][mk::NBMAX];
};
static_assert(sizeof(MkShared) <= mk::SH_BYTES, "MkShared grew past its slot");

AF_DEV unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

AF_DEV int ld_err(const int* err) { return *reinterpret_cast<const volatile int*>(err); }

AF_DEV void csync() { asm volatile("bar.sync 1, %0;" ::"n"(mk::CW * 32) : "memory"); }

// ring wait: bounded in time, gives up early once any CTA recorded an error (unless `drain`)
AF_DEV bool mk_wait(uint64_t* bar, uint32_t parity, const int* err, bool drain = false) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = gtimer();
  for (unsigned i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      if (!drain && ld_err(err)) return false;
      if (gtimer() - t0 > mk::SPIN_NS) return false;
    }
  }
}

// Grid barrier over all CTAs (consumers call it together). `target` = barriers so far x grid size.
AF_DEV bool grid_barrier(const MkArgs& a, MkShared* sh, unsigned target) {
  csync();
  if (threadIdx.x == 0) {
    const size_t pslot = ((size_t)blockIdx.x * (1 + 5 * a.L) + (target / gridDim.x - 1)) * 4;
    if (a.prof) a.prof[pslot] = gtimer();
    __threadfence();
    atomicAdd(a.bar, 1u);
    bool ok = false;
    const unsigned long long t0 = gtimer();
    for (unsigned i = 0;; ++i) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.bar) : "memory");
      if (v >= target) { ok = true; break; }
      if ((i & 15u) == 15u) {
        if (ld_err(a.err)) break;
        if (gtimer() - t0 > mk::SPIN_NS) { af_set_err(a.err, AF_DEV_WAIT_TIMEOUT); break; }
      }
    }
    __threadfence();
    if (a.prof) a.prof[pslot + 1] = gtimer();
    *reinterpret_cast<volatile int*>(&sh->abort) = ok ? 0 : 1;
  }
  csync();
  return *reinterpret_cast<volatile int*>(&sh->abort) == 0;
}

// ----------------------------------------------------------------------------------- GEMV phase

// CTAs in [c0, c1) whose stream-K range is not empty (all of them when U >= G)
AF_DEV int busy_between(int c0, int c1, long long U, int G) {
  if (U >= G) return c1 - c0;
  int n = 0;
  for (int c = c0; c < c1; ++c) n += unit_begin(c + 1, U, G) > unit_begin(c, U, G);
  return n;
}

struct XPlan {
  bool full;          // stage x[0, K) (else the CTA's one or two k segments, back to back)
  int kta[2], ktb[2];
};

AF_DEV XPlan x_plan(long long u0, long long u1, int KT) {
  XPlan p;
  p.full = false;
  int nseg = 0;
  for (long long u = u0; u < u1;) {
    const int kta = (int)(u % KT);
    const int ktb = (int)min((long long)KT, kta + (u1 - u));
    if (kta == 0 && ktb == KT) p.full = true;
    if (nseg < 2) { p.kta[nseg] = kta; p.ktb[nseg] = ktb; }
    ++nseg;
    u += ktb - kta;
  }
  if (nseg > 2) p.full = true;
  if (nseg == 1) { p.kta[1] = p.ktb[1] = 0; }
  if (nseg == 0) { p.kta[0] = p.ktb[0] = p.kta[1] = p.ktb[1] = 0; }
  if (!p.full && (p.ktb[0] - p.kta[0]) + (p.ktb[1] - p.kta[1]) >= KT) p.full = true;
  return p;
}

// x offset (halves) of k tile 0 for segment `si` of the staged slice
AF_DEV int x_base(const XPlan& p, int si) {
  if (p.full) return 0;
  return si == 0 ? -p.kta[0] * 32 : (p.ktb[0] - p.kta[0]) * 32 - p.kta[1] * 32;
}

// Stage the x slice of this CTA into shared memory [NB][xstride] (consumer threads 0..255) with
// plain L2 loads. The norm phases first reduce the sum of squares of each fp32 row (same thread
// mapping, so the same fp32 sum, in every CTA), then write the normalised fp16 operand.
AF_DEV void stage_x(const MkGemv& gd, int NB, const XPlan& p, __half* xs, int xstride, MkShared* sh) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (gd.xnorm) {
    const float* h = reinterpret_cast<const float*>(gd.x);
    for (int b = 0; b < NB; ++b) {
      float ss = 0.f;
      for (int i = tid; i < gd.K / 4; i += mk::CW * 32) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(h + (size_t)b * gd.ldx) + i);
        ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss); ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
      }
      ss = warp_sum(ss);
      if (lane == 0) sh->wsum[warp][b] = ss;
    }
    csync();
    if (tid < NB) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < mk::CW; ++w) s += sh->wsum[w][tid];
      sh->sn[tid] = fmaxf(sqrtf(s), gd.floor);
    }
    csync();
  }
  const int nr = p.full ? 1 : 2;
  int base = 0;
  for (int r = 0; r < nr; ++r) {
    const int k0 = p.full ? 0 : p.kta[r], k1 = p.full ? gd.K / 32 : p.ktb[r];
    const int n8 = (k1 - k0) * 4;                          // 8-half vectors per row
    for (int idx = tid; idx < NB * n8; idx += mk::CW * 32) {
      const int b = idx / n8, v = idx - b * n8;
      const int k = k0 * 32 + v * 8;
      uint4 out;
      if (gd.xnorm) {
        const float* hr = reinterpret_cast<const float*>(gd.x) + (size_t)b * gd.ldx + k;
        const float4 f0 = __ldcg(reinterpret_cast<const float4*>(hr));
        const float4 f1 = __ldcg(reinterpret_cast<const float4*>(hr) + 1);
        float g8[8];
        h8_to_f32(__ldg(reinterpret_cast<const uint4*>(gd.g + k)), g8);
        const float f[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
        const float sn = sh->sn[b];
        __half o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = __float2half_rn(__fdiv_rn(f[e], sn) * g8[e]);
        out = *reinterpret_cast<const uint4*>(o);
      } else {
        out = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(gd.x) + (size_t)b * gd.ldx + k));
      }
      *reinterpret_cast<uint4*>(xs + (size_t)b * xstride + base + v * 8) = out;
    }
    base += n8 * 8;
  }
}

template <int NT>
AF_DEV void mk_epilogue(const MkGemv& gd, int NB, bool i4, float (&acc)[NT][4], int rt, int g, int t) {
  const int r0 = rt * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int b = n * 8 + 2 * t + hh;
      if (b >= NB) continue;
      const float v0 = acc[n][hh], v1 = acc[n][2 + hh];
      if (gd.epi == EPI_SWIGLU) {
        if (r1 >= gd.N) continue;
        float gv = i4 ? v0 : __fmul_rn(v0, h2f(gd.scale[r0]));
        float uv = i4 ? v1 : __fmul_rn(v1, h2f(gd.scale[r1]));
        if (gd.bias) { gv = __fadd_rn(gv, h2f(gd.bias[r0])); uv = __fadd_rn(uv, h2f(gd.bias[r1])); }
        reinterpret_cast<__half*>(gd.y)[(size_t)b * gd.ldy + rt * 8 + g] = f2h(silu_f(gv) * uv);
      } else {
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int row = rr ? r1 : r0;
          if (row >= gd.N) continue;
          float v = i4 ? (rr ? v1 : v0) : __fmul_rn(rr ? v1 : v0, h2f(gd.scale[row]));
          if (gd.bias) v = __fadd_rn(v, h2f(gd.bias[row]));
          const size_t o = (size_t)b * gd.ldy + row;
          if (gd.epi == EPI_F32) reinterpret_cast<float*>(gd.y)[o] = v;
          else if (gd.epi == EPI_F16) reinterpret_cast<__half*>(gd.y)[o] = f2h(v);
          else reinterpret_cast<float*>(gd.y)[o] = __ldcg(reinterpret_cast<const float*>(gd.y) + o) + v;
        }
      }
    }
  }
}

// One GEMV phase on the consumer side. Returns false when the CTA must stop (a ring wait gave up).
template <bool I4, int NT>
AF_DEV bool gemv_phase(const MkArgs& a, const MkGemv& gd, MkShared* sh, unsigned char* ring, const MkSmem& L,
                       unsigned char* xreg, float* red, int& stage, uint32_t& phase, unsigned pk) {
  const int nst = L.nst;
  const int xstride = gd.xnorm ? L.xsn : L.xsp;
  __half* xs = reinterpret_cast<__half*>(xreg);
  using F = tc::Fmt<I4>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3, rtw = warp & 3, par = warp >> 2;
  const int G = gridDim.x, c = blockIdx.x;
  const int RB = (gd.N + 63) / 64, KT = gd.K / 32;
  const long long U = (long long)RB * KT;
  const long long u0 = unit_begin(c, U, G), u1 = unit_begin(c + 1, U, G);
  const XPlan xp = x_plan(u0, u1, KT);
  stage_x(gd, a.NB, xp, xs, xstride, sh);
  csync();
  unsigned long long* prof = a.prof ? a.prof + ((size_t)c * (1 + 5 * a.L) + pk) * 4 : nullptr;
  if (prof && threadIdx.x == 0) prof[2] = gtimer();
  int si = 0;
  for (long long u = u0; u < u1; ++si) {
    const int rb = (int)(u / KT), kta = (int)(u % KT);
    const int ktb = (int)min((long long)KT, kta + (u1 - u));
    const int xb = x_base(xp, si);
    float acc[NT][4], acc2[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int q = 0; q < 4; ++q) { acc[n][q] = 0.f; acc2[n][q] = 0.f; }
    bool stuck = false;
    for (int kt = kta; kt < ktb; kt += F::ks) {
      const int nk = min(F::ks, ktb - kt);
      if (!mk_wait(&sh->full[stage], phase, a.err)) { stuck = true; break; }
      consume_stage<I4, NT, 2>(ring + (size_t)stage * F::stage, nk, xs + xb + kt * 32, xstride, a.NB, lane, rtw, par, acc,
                               acc2);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty[stage]);
      if (++stage == nst) { stage = 0; phase ^= 1; }
    }
    if (stuck) {
      af_set_err(a.err, AF_DEV_WAIT_TIMEOUT);
      *reinterpret_cast<volatile int*>(&sh->cabort) = 1;
    }
    if (prof && threadIdx.x == 0) prof[3] = gtimer();
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[n][q] += acc2[n][q];
    float* rw = red + ((size_t)rtw * 32 + lane) * (NT * 4);
    if (par) {
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int q = 0; q < 4; ++q) rw[n * 4 + q] = acc[n][q];
    }
    csync();
    if (*reinterpret_cast<volatile int*>(&sh->cabort)) return false;
    if (!par) {
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[n][q] += rw[n * 4 + q];
    }
    const int rt = rb * tc::WARPS + rtw;
    if (kta == 0 && ktb == KT) {
      if (!par) mk_epilogue<NT>(gd, a.NB, I4, acc, rt, g, t);
    } else {
      // CTAs sharing the row block: with fewer units than CTAs some ranges are empty and take no ticket
      const int cf = owner_of((long long)rb * KT, U, G), cl = owner_of((long long)rb * KT + KT - 1, U, G);
      const int nc = busy_between(cf, cl + 1, U, G), j = busy_between(cf, c, U, G);
      constexpr int NBP = NT * 8;
      float* slot = a.part + (((size_t)rb * a.maxc + j) * 64) * NBP;
      const int r0 = rtw * 16 + g, r1 = r0 + 8;
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
      csync();
      if (threadIdx.x == 0) sh->ticket = atomicAdd(a.counters + rb, 1) == nc - 1;
      csync();
      if (sh->ticket && !par) {
        __threadfence();
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const int c0 = n * 8 + 2 * t;
          if (c0 >= a.NB) continue;
          float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
          for (int jj = 0; jj < nc; ++jj) {
            const float* sp = a.part + (((size_t)rb * a.maxc + jj) * 64) * NBP;
            const float2 p = __ldcg(reinterpret_cast<const float2*>(sp + (size_t)r0 * NBP + c0));
            const float2 q = __ldcg(reinterpret_cast<const float2*>(sp + (size_t)r1 * NBP + c0));
            s0 += p.x; s1 += p.y; s2 += q.x; s3 += q.y;
          }
          acc[n][0] = s0; acc[n][1] = s1; acc[n][2] = s2; acc[n][3] = s3;
        }
        mk_epilogue<NT>(gd, a.NB, I4, acc, rt, g, t);
        if (threadIdx.x == 0) a.counters[rb] = 0;
      }
    }
    csync();
    u += ktb - kta;
  }
  return true;
}

// ------------------------------------------------------------------------------ attention phase

template <int DH, int G>
struct AttnSmem {
  float q[G][DH];
  float kn[DH], vn[DH];
  float wm[mk::CW][G], wl[mk::CW][G];
  float wacc[mk::CW][G][DH];
  float fw[64][G], lw[64][G];
  float den[G];
};

// One (sequence b, kv head, split) task of the split-K decode attention on the 8 consumer warps:
// the stand-alone attn_decode_kernel's algorithm (QK-norm, RoPE, cache write at pos by the split
// that holds it, online softmax over the split's keys, last split merges) on named barriers.
template <int DH, int G>
AF_DEV void attn_task(const MkArgs& a, const MkLayer& ly, int split, int kvh, int b, AttnSmem<DH, G>& S,
                      MkShared* sh) {
  using HL = HeadLayout<DH>;
  using DB = DecodeBatch<DH, G, (G >= 8 ? 2 : 4)>;   // short batches: fit the megakernel register cap
  constexpr int EPL = HL::EPL;
  constexpr int NW = mk::CW;
  constexpr int PB = DB::PB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool active = lane < HL::LANES;
  const int pos = __ldcg(a.pos + b);
  if (pos < 0 || pos >= a.M) {
    if (threadIdx.x == 0 && split == 0 && kvh == 0) af_set_err(a.err, AF_DEV_BAD_POS);
    return;
  }
  const int ns = a.nsplit;
  const int len = (pos + ns) / ns;
  const int j0 = split * len;
  const int j1 = min(j0 + len, pos + 1);
  const bool owns_pos = j0 <= pos && pos < j1;
  const float* qkv = a.qkv + (size_t)b * a.ldq;
  const int H = a.H, KV = a.KV;

  for (int gg = warp; gg < G; gg += NW) {
    float v[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) v[e] = active ? __ldcg(qkv + (size_t)(kvh * G + gg) * DH + lane * EPL + e) : 0.f;
    norm_rope_head<DH>(v, lane, ly.qn, ly.qnf, a.cos_t, a.sin_t, pos);
    if (active)
#pragma unroll
      for (int e = 0; e < EPL; ++e) S.q[gg][lane * EPL + e] = round_f16(v[e]);
  }
  if (owns_pos && warp == NW - 1) {
    float k[EPL], vv[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      k[e] = active ? __ldcg(qkv + (size_t)H * DH + (size_t)kvh * DH + lane * EPL + e) : 0.f;
      vv[e] = active ? __ldcg(qkv + (size_t)(H + KV) * DH + (size_t)kvh * DH + lane * EPL + e) : 0.f;
    }
    norm_rope_head<DH>(k, lane, ly.kn, ly.knf, a.cos_t, a.sin_t, pos);
    const size_t slot = (((size_t)b * KV + kvh) * a.M + pos) * DH;
    if (active)
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const __half kh = f2h(k[e]), vh = f2h(vv[e]);
        ly.kc[slot + lane * EPL + e] = kh;
        ly.vc[slot + lane * EPL + e] = vh;
        S.kn[lane * EPL + e] = h2f(kh);
        S.vn[lane * EPL + e] = h2f(vh);
      }
  }
  csync();

  float qr[G][EPL];
#pragma unroll
  for (int gg = 0; gg < G; ++gg)
#pragma unroll
    for (int e = 0; e < EPL; ++e) qr[gg][e] = active ? S.q[gg][lane * EPL + e] : 0.f;
  float m[G], l[G], acc[G][EPL];
#pragma unroll
  for (int gg = 0; gg < G; ++gg) {
    m[gg] = -INFINITY; l[gg] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[gg][e] = 0.f;
  }
  const __half* kbase = ly.kc + ((size_t)b * KV + kvh) * a.M * DH;
  const __half* vbase = ly.vc + ((size_t)b * KV + kvh) * a.M * DH;
  const float cexp = a.kv_c;
  const int my_idx = lane >> DB::SHIFT;
  const int my_g = my_idx / PB, my_p = my_idx % PB;
  const bool rep0 = (lane & ((1 << DB::SHIFT) - 1)) == 0;
  for (int base = j0 + warp * PB; base < j1; base += NW * PB) {
    float kf[PB][EPL], vf[PB][EPL];
#pragma unroll
    for (int p = 0; p < PB; ++p) {
      const int j = base + p;
      const bool in_range = j < j1;
      if (in_range && j != pos) {
        load_row_f16<DH>(kbase + (size_t)j * DH, lane, kf[p]);
        load_row_f16<DH>(vbase + (size_t)j * DH, lane, vf[p]);
      } else {
        const bool nw = in_range && active;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          kf[p][e] = nw ? S.kn[lane * EPL + e] : 0.f;
          vf[p][e] = nw ? S.vn[lane * EPL + e] : 0.f;
        }
      }
    }
    if (a.expand) {
#pragma unroll
      for (int p = 0; p < PB; ++p)
#pragma unroll
        for (int e = 0; e < EPL; ++e) { kf[p][e] = round_f16(cexp * kf[p][e]); vf[p][e] = round_f16(cexp * vf[p][e]); }
    }
    float d[DB::NV];
#pragma unroll
    for (int gg = 0; gg < G; ++gg)
#pragma unroll
      for (int p = 0; p < PB; ++p) {
        float sdot = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) sdot = fmaf(qr[gg][e], kf[p][e], sdot);
        d[gg * PB + p] = sdot;
      }
    const float sc = transpose_reduce<DB::NV>(d, lane) * a.scale;
    const bool valid = base + my_p < j1;
    const float s = valid ? sc : -INFINITY;
    float tmax = s;
#pragma unroll
    for (int off = DB::GS / 2; off >= 1; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
    float mnew_mine = fmaxf(m[0], tmax);
#pragma unroll
    for (int gg = 1; gg < G; ++gg) if (gg == my_g) mnew_mine = fmaxf(m[gg], tmax);
    const float pe = valid ? expf(s - mnew_mine) : 0.f;
    float tsum = rep0 ? pe : 0.f;
#pragma unroll
    for (int off = DB::GS / 2; off >= 1; off >>= 1) tsum += __shfl_xor_sync(0xffffffffu, tsum, off);
#pragma unroll
    for (int gg = 0; gg < G; ++gg) {
      const float mg = __shfl_sync(0xffffffffu, tmax, gg * DB::GS);
      const float sg = __shfl_sync(0xffffffffu, tsum, gg * DB::GS);
      const float mn = fmaxf(m[gg], mg);
      const float corr = expf(m[gg] - mn);
      l[gg] = l[gg] * corr + sg;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[gg][e] *= corr;
#pragma unroll
      for (int p = 0; p < PB; ++p) {
        const float pp = __shfl_sync(0xffffffffu, pe, (gg * PB + p) << DB::SHIFT);
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[gg][e] = fmaf(pp, vf[p][e], acc[gg][e]);
      }
      m[gg] = mn;
    }
  }
#pragma unroll
  for (int gg = 0; gg < G; ++gg) {
    if (lane == 0) { S.wm[warp][gg] = m[gg]; S.wl[warp][gg] = l[gg]; }
    if (active)
#pragma unroll
      for (int e = 0; e < EPL; ++e) S.wacc[warp][gg][lane * EPL + e] = acc[gg][e];
  }
  csync();
  const size_t pair = (size_t)b * KV + kvh;
  float* part = a.apart + (pair * ns + split) * G * (DH + 2);
  for (int i = threadIdx.x; i < G * DH; i += NW * 32) {
    const int gg = i / DH, dd = i - gg * DH;
    float Mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) Mx = fmaxf(Mx, S.wm[w][gg]);
    float num = 0.f, den = 0.f;
    if (Mx != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float f = expf(S.wm[w][gg] - Mx);
        num = fmaf(f, S.wacc[w][gg][dd], num);
        den = fmaf(f, S.wl[w][gg], den);
      }
    }
    if (ns == 1) {
      a.att[(size_t)b * H * DH + (size_t)(kvh * G + gg) * DH + dd] = f2h(num / den);
    } else {
      __stcg(part + gg * (DH + 2) + dd, num);
      if (dd == 0) { __stcg(part + gg * (DH + 2) + DH, Mx); __stcg(part + gg * (DH + 2) + DH + 1, den); }
    }
  }
  if (ns == 1) { csync(); return; }
  __threadfence();
  csync();
  if (threadIdx.x == 0) sh->last = atomicAdd(a.acount + pair, 1) == ns - 1;
  csync();
  if (!sh->last) return;
  __threadfence();
  const float* pp = a.apart + pair * ns * G * (DH + 2);
  for (int i = threadIdx.x; i < ns * G; i += NW * 32) {
    const int sp = i / G, gg = i - sp * G;
    S.fw[sp][gg] = __ldcg(pp + (sp * G + gg) * (DH + 2) + DH);
    S.lw[sp][gg] = __ldcg(pp + (sp * G + gg) * (DH + 2) + DH + 1);
  }
  csync();
  if (threadIdx.x < G) {
    const int gg = threadIdx.x;
    float Mx = -INFINITY;
    for (int sp = 0; sp < ns; ++sp) Mx = fmaxf(Mx, S.fw[sp][gg]);
    float den = 0.f;
    for (int sp = 0; sp < ns; ++sp) {
      const float f = S.fw[sp][gg] == -INFINITY ? 0.f : expf(S.fw[sp][gg] - Mx);
      den = fmaf(f, S.lw[sp][gg], den);
      S.fw[sp][gg] = f;
    }
    S.den[gg] = den;
  }
  csync();
  for (int i = threadIdx.x; i < G * DH; i += NW * 32) {
    const int gg = i / DH, dd = i - gg * DH;
    float num = 0.f;
#pragma unroll 8
    for (int sp = 0; sp < ns; ++sp) num = fmaf(S.fw[sp][gg], __ldcg(pp + (sp * G + gg) * (DH + 2) + dd), num);
    a.att[(size_t)b * H * DH + (size_t)(kvh * G + gg) * DH + dd] = f2h(num / S.den[gg]);
  }
  if (threadIdx.x == 0) a.acount[pair] = 0;
}

// ------------------------------------------------------------------------------------ the kernel

template <bool I4, int NT, int DH, int G>
__global__ void __maxnreg__(96) decode_mk_kernel(MkArgs a, MkSmem L) {
  using F = tc::Fmt<I4>;
  extern __shared__ __align__(128) unsigned char smem[];
  const int nst = L.nst;
  unsigned char* ring = smem;
  MkShared* sh = reinterpret_cast<MkShared*>(smem + (size_t)nst * F::stage);
  unsigned char* xreg = smem + (size_t)nst * F::stage + mk::SH_BYTES;
  AttnSmem<DH, G>& S = *reinterpret_cast<AttnSmem<DH, G>*>(xreg);      // aliases the x region (phases differ)
  float* red = reinterpret_cast<float*>(xreg + L.red_off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Gd = gridDim.x, c = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], mk::CW);
    }
    sh->cabort = 0; sh->abort = 0; sh->last = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == mk::CW) {
    // ------------------------------------------------------------ producer: the step's weight stream
    if (lane != 0) return;
    int stage = 0, inflight = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int l = 0; l < a.L && ok; ++l) {
      const MkLayer& ly = a.layers[l];
      for (int p = 0; p < 4 && ok; ++p) {
        const MkGemv& gd = p == 0 ? ly.qkv : p == 1 ? ly.o : p == 2 ? ly.gu : ly.down;
        const char* W = reinterpret_cast<const char*>(gd.w);
        const int RB = (gd.N + 63) / 64, KT = gd.K / 32;
        const long long U = (long long)RB * KT;
        const long long u1 = unit_begin(c + 1, U, Gd);
        for (long long u = unit_begin(c, U, Gd); u < u1 && ok;) {
          const int rb = (int)(u / KT), kta = (int)(u % KT);
          const int ktb = (int)min((long long)KT, kta + (u1 - u));
          for (int kt = kta; kt < ktb; kt += F::ks) {
            const int nk = min(F::ks, ktb - kt);
            if (!mk_wait(&sh->empty[stage], ph ^ 1, a.err)) { ok = false; break; }
            mbar_arrive_expect_tx(&sh->full[stage], (uint32_t)nk * F::unit);
            bulk_g2s(ring + (size_t)stage * F::stage, W + ((size_t)rb * KT + kt) * F::unit, nk * F::unit,
                     &sh->full[stage]);
            inflight = min(inflight + 1, nst);
            if (++stage == nst) { stage = 0; ph ^= 1; }
          }
          u += ktb - kta;
        }
      }
    }
    if (!ok && !ld_err(a.err)) af_set_err(a.err, AF_DEV_WAIT_TIMEOUT);
    // the ring must outlive every copy issued: wait (time-bounded only) for the last ones to land
    for (int i = 0; i < inflight; ++i) {
      if (--stage < 0) { stage = nst - 1; ph ^= 1; }
      mk_wait(&sh->full[stage], ph, a.err, true);
    }
    return;
  }

  // -------------------------------------------------------------------------------- consumers
  int stage = 0;
  uint32_t phase = 0;
  unsigned nbar = 0;
  // embedding gather (the token ids were written by the previous step's head kernel)
  {
    const int nvec = a.NB * a.D / 8;
    for (int i = c * (mk::CW * 32) + threadIdx.x; i < nvec; i += Gd * mk::CW * 32) {
      const int b = i / (a.D / 8), v = i - b * (a.D / 8);
      const int tk = __ldcg(a.tok + b);
      const bool okt = tk >= 0 && tk < a.vocab;
      if (!okt && v == 0) af_set_err(a.err, AF_DEV_BAD_TOKEN);
      float f[8];
      if (okt) h8_to_f32(__ldg(reinterpret_cast<const uint4*>(a.embed + (size_t)tk * a.D) + v), f);
      else for (int e = 0; e < 8; ++e) f[e] = 0.f;
      float4* dst = reinterpret_cast<float4*>(a.h + (size_t)b * a.D) + 2 * v;
      dst[0] = make_float4(f[0], f[1], f[2], f[3]);
      dst[1] = make_float4(f[4], f[5], f[6], f[7]);
    }
  }
  if (!grid_barrier(a, sh, ++nbar * Gd)) return;
  for (int l = 0; l < a.L; ++l) {
    const MkLayer& ly = a.layers[l];
    if (!gemv_phase<I4, NT>(a, ly.qkv, sh, ring, L, xreg, red, stage, phase, nbar)) return;
    if (!grid_barrier(a, sh, ++nbar * Gd)) return;
    const int T = a.NB * a.KV * a.nsplit;
    for (int task = c; task < T; task += Gd) {
      const int split = task % a.nsplit, rest = task / a.nsplit;
      attn_task<DH, G>(a, ly, split, rest % a.KV, rest / a.KV, S, sh);
      csync();
    }
    if (!grid_barrier(a, sh, ++nbar * Gd)) return;
    if (!gemv_phase<I4, NT>(a, ly.o, sh, ring, L, xreg, red, stage, phase, nbar)) return;
    if (!grid_barrier(a, sh, ++nbar * Gd)) return;
    if (!gemv_phase<I4, NT>(a, ly.gu, sh, ring, L, xreg, red, stage, phase, nbar)) return;
    if (!grid_barrier(a, sh, ++nbar * Gd)) return;
    if (!gemv_phase<I4, NT>(a, ly.down, sh, ring, L, xreg, red, stage, phase, nbar)) return;
    if (!grid_barrier(a, sh, ++nbar * Gd)) return;
  }
  // final norm of the residual rows (CTA 0) for the head kernel
  if (c == 0) {
    MkGemv fin;
    fin.x = a.h; fin.ldx = a.D; fin.K = a.D; fin.xnorm = 1; fin.g = a.final_g; fin.floor = a.final_floor;
    const int tid = threadIdx.x;
    for (int b = 0; b < a.NB; ++b) {
      float ss = 0.f;
      for (int i = tid; i < a.D / 4; i += mk::CW * 32) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(a.h + (size_t)b * a.D) + i);
        ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss); ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
      }
      ss = warp_sum(ss);
      if (lane == 0) sh->wsum[warp][b] = ss;
    }
    csync();
    if (tid < a.NB) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < mk::CW; ++w) s += sh->wsum[w][tid];
      sh->sn[tid] = fmaxf(sqrtf(s), a.final_floor);
    }
    csync();
    for (int i = tid; i < a.NB * a.D; i += mk::CW * 32) {
      const int b = i / a.D, d = i - b * a.D;
      a.hid[i] = __float2half_rn(__fdiv_rn(__ldcg(a.h + i), sh->sn[b]) * h2f(a.final_g[d]));
    }
  }
}

// ------------------------------------------------------------------------------------ host side

static int mk_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

static size_t attn_smem_bytes(int dh, int G) {
  return sizeof(float) * ((size_t)G * dh + 2 * dh + 2 * mk::CW * G + (size_t)mk::CW * G * dh + 2 * 64 * G + G);
}

// staged-x halves one CTA needs for a GEMV of K columns split over `grid` CTAs (host copy of x_plan)
static int x_halves_needed(int N, int K, int grid) {
  const long long RB = (N + 63) / 64, KT = K / 32, U = RB * KT;
  int need = 0;
  for (int c = 0; c < grid; ++c) {
    const long long u0 = (long long)c * U / grid, u1 = (long long)(c + 1) * U / grid;
    bool full = false;
    int nseg = 0, tiles = 0;
    for (long long u = u0; u < u1;) {
      const long long kta = u % KT, ktb = std::min(KT, kta + (u1 - u));
      if (kta == 0 && ktb == KT) full = true;
      if (nseg < 2) tiles += (int)(ktb - kta);
      ++nseg;
      u += ktb - kta;
    }
    if (nseg > 2 || tiles >= KT) full = true;
    need = std::max(need, (full ? (int)KT : tiles) * 32);
  }
  return need;
}

static int max_ctas_sharing(int N, int K, int grid) {
  const long long RB = (N + 63) / 64, KT = K / 32, U = RB * KT;
  const long long per = U / grid;
  return (int)((KT + (per > 0 ? per : 1) - 1) / (per > 0 ? per : 1)) + 1;
}

template <bool I4, int NT, int DH, int G>
static void* mk_kernel_ptr() { return (void*)decode_mk_kernel<I4, NT, DH, G>; }

static void* mk_pick(bool i4, int dh, int G) {
#define AF_MK_G(I4V, DHV)                                            \
  switch (G) {                                                       \
    case 1: return mk_kernel_ptr<I4V, 1, DHV, 1>();                  \
    case 2: return mk_kernel_ptr<I4V, 1, DHV, 2>();                  \
    case 4: return mk_kernel_ptr<I4V, 1, DHV, 4>();                  \
    case 8: return mk_kernel_ptr<I4V, 1, DHV, 8>();                  \
    default: return nullptr;                                         \
  }
  if (i4) {
    if (dh == 64) { AF_MK_G(true, 64) }
    if (dh == 128) { AF_MK_G(true, 128) }
  } else {
    if (dh == 64) { AF_MK_G(false, 64) }
    if (dh == 128) { AF_MK_G(false, 128) }
  }
#undef AF_MK_G
  return nullptr;
}

bool decode_mk_plan(const MkLayer& sh, int wf, int NB, int H, int KV, int dh, int nsplit, MkPlan* plan) {
  if (NB < 1 || NB > mk::NBMAX || KV <= 0 || H % KV || nsplit < 1 || nsplit > 64) return false;
  if (wf != W_I8 && wf != W_I4G32) return false;
  const bool i4 = wf == W_I4G32;
  void* fn = mk_pick(i4, dh, H / KV);
  if (!fn) return false;
  const MkGemv* gs[4] = {&sh.qkv, &sh.o, &sh.gu, &sh.down};
  for (const MkGemv* g : gs)
    if (g->K % 32 || (g->epi == EPI_SWIGLU && g->N % 16)) return false;
  const int stage = i4 ? tc::STAGE_BYTES4 : tc::STAGE_BYTES;
  const int sms = mk_sms();
  auto al = [](size_t v) { return (v + 127) / 128 * 128; };
  for (int cps = 2; cps >= 1; --cps) {
    const int grid = cps * sms;
    int xn = 0, xp = 0, maxc = 0;
    for (int q = 0; q < 4; ++q) {
      const int need = x_halves_needed(gs[q]->N, gs[q]->K, grid);
      if (q == 0 || q == 2) xn = std::max(xn, need);        // qkv, gate|up: normalised residual rows
      else xp = std::max(xp, need);
      maxc = std::max(maxc, max_ctas_sharing(gs[q]->N, gs[q]->K, grid));
    }
    const int xsn = xn + mk::XPAD, xsp = xp + mk::XPAD;
    const size_t region =
        al(std::max(attn_smem_bytes(dh, H / KV), std::max((size_t)NB * xsn * 2, (size_t)NB * xsp * 2)));
    const size_t fixed = mk::SH_BYTES + region + mk::RED_BYTES;
    const size_t budget = (size_t)(cps == 2 ? 113 : 227) * 1024 - 1024;
    if (fixed + 4 * (size_t)stage > budget) continue;
    int nst = (int)((budget - fixed) / stage);
    if (nst > mk::MAXST) nst = mk::MAXST;
    plan->grid = grid;
    plan->maxc = maxc;
    plan->xs_halves = std::max(xsn, xsp);
    plan->nst = nst;
    plan->xsn = xsn;
    plan->xsp = xsp;
    plan->hs_off = -1;
    plan->region = (int)region;
    plan->smem = (size_t)nst * stage + fixed;
    size_t rbmax = 0;
    for (const MkGemv* g : gs) rbmax = std::max(rbmax, (size_t)(g->N + 63) / 64);
    plan->part_floats = rbmax * maxc * 64 * 8;
    plan->counters = rbmax;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan->smem) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    int occ = 0;
    const cudaError_t oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, mk::NTHR, plan->smem);
    if (getenv("AF_MK_DEBUG")) {
      cudaFuncAttributes fa;
      cudaFuncGetAttributes(&fa, fn);
      fprintf(stderr, "[decode_mk] cps %d grid %d stages %d smem %zu xsn %d xsp %d region %zu occ %d (%s) regs %d\n",
              cps, grid, nst, plan->smem, xsn, xsp, region, occ, cudaGetErrorString(oe), fa.numRegs);
    }
    if (oe != cudaSuccess || occ < cps) {
      cudaGetLastError();
      continue;
    }
    return true;
  }
  return false;
}

cudaError_t decode_mk_launch(const MkArgs& a0, const MkPlan& plan, cudaStream_t st) {
  const bool i4 = a0.wf == W_I4G32;
  void* fn = mk_pick(i4, a0.dh, a0.H / a0.KV);
  if (!fn || !a0.layers || !a0.bar || !a0.part || !a0.counters || plan.grid <= 0 || plan.nst < 2) return cudaErrorInvalidValue;
  if (a0.nsplit > 1 && (!a0.apart || !a0.acount)) return cudaErrorInvalidValue;
  MkArgs a = a0;
  a.maxc = plan.maxc;
  a.xs_halves = plan.xs_halves;
  MkSmem L;
  L.nst = plan.nst;
  L.xsn = plan.xsn;
  L.xsp = plan.xsp;
  L.red_off = plan.region;
  cudaError_t e = cudaMemsetAsync(a.bar, 0, sizeof(unsigned), st);
  if (e != cudaSuccess) return e;
  void* args[] = {&a, &L};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(mk::NTHR);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace af
