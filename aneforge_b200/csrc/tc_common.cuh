// Shared pieces of the tensor-core dequant GEMVs: tile geometry, mbarrier / bulk-copy wrappers, the
// mma.sync wrappers and the exact int8 / int4 -> fp16 fragment conversions.
#pragma once
#include "af_common.cuh"

namespace af {

namespace tc {
constexpr int WARPS = 4;                   // row tiles per row block
constexpr int CWARPS = 8;                  // consumer warps: two per row tile (even / odd k tiles)
constexpr int KS = 4;                      // k tiles per weight stage (int8)
constexpr int TILE = 512;                  // bytes per 16x32 int8 tile
constexpr int UNIT = WARPS * TILE;         // one k tile of one row block
constexpr int STAGE_BYTES = KS * UNIT;     // 8 KB
constexpr int KS4 = 8;                     // int4: k tiles per stage
constexpr int TILE4 = 256;                 // bytes per 16x32 int4 tile
constexpr int UNIT4 = WARPS * TILE4 + 64 * 2;   // 4 tiles + 64 fp16 group scales
constexpr int STAGE_BYTES4 = KS4 * UNIT4;  // 9 KB
constexpr int STAGE_MAX = STAGE_BYTES4 > STAGE_BYTES ? STAGE_BYTES4 : STAGE_BYTES;
constexpr int STAGES = 6;
constexpr int XKT = 16;                    // k tiles per x chunk
constexpr int XSTRIDE = XKT * 32 + 32;     // halves per staged x row (+32: rows 16 banks apart)
constexpr int XSLOTS = 2;
constexpr size_t CNT_BYTES = 16384;        // scratch: per-row-block tickets, then partial slots
constexpr long long WAIT_LIMIT = 1ll << 26;
template <bool I4> struct Fmt {
  static constexpr int ks = I4 ? KS4 : KS;
  static constexpr int unit = I4 ? UNIT4 : UNIT;
  static constexpr int tile = I4 ? TILE4 : TILE;
  static constexpr int stage = ks * unit;
};
}  // namespace tc

AF_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

AF_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

AF_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

AF_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {   // bounded: iterations and ~2 s
  SpinBudget budget;
  for (long long i = 0; i < tc::WAIT_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (budget.spent()) return false;
  }
  return false;
}

AF_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

AF_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// 1-D bulk copy global -> this CTA's own shared memory, completion counted on `bar`
AF_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// An L2 policy that evicts the lines it touches first: for data read once per step (the weights),
// so the stream does not push out lines that are still to be used.
AF_DEV uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// bulk_g2s with an L2 cache-policy hint
AF_DEV void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol) : "memory");
}

// weight stage copy: evict-first when `hint`
AF_DEV void bulk_w(void* dst, const void* src, uint32_t bytes, uint64_t* bar, bool hint, uint64_t pol) {
  if (hint) bulk_g2s_hint(dst, src, bytes, bar, pol);
  else bulk_g2s(dst, src, bytes, bar);
}

AF_DEV void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(tc::CWARPS * 32) : "memory"); }

// consumer warps per CTA: one per row tile (int8), or two splitting the k tiles (int4, whose
// conversion costs more instructions per byte)
template <bool I4> struct Cw { static constexpr int n = I4 ? 8 : 4; };

template <int CW>
AF_DEV void consumer_sync_n() { asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory"); }

// (not volatile: the MMA has no effect beyond its outputs, so the compiler may interleave independent
// MMAs of neighbouring tiles; measured 1-2 % faster on the decode GEMVs)
AF_DEV void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// d = a . b (a fresh accumulation: the C operand is zero)
AF_DEV void mma_16816_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}

// 4 int8 codes (bytes of w) -> two half2: (byte0, byte1) and (byte2, byte3), exact.
AF_DEV void i8x4_to_h2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;                        // b + 128 as an unsigned byte
  const uint32_t blo = __byte_perm(u, 0x64646464u, 0x5140);  // fp16 bits 0x64uu = 1024 + u
  const uint32_t bhi = __byte_perm(u, 0x64646464u, 0x7362);
  const __half2 bias = __half2half2(__ushort_as_half(0x6480));  // 1152 = 1024 + 128
  __half2 l = __hsub2(*reinterpret_cast<const __half2*>(&blo), bias);
  __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&bhi), bias);
  lo = *reinterpret_cast<uint32_t*>(&l);
  hi = *reinterpret_cast<uint32_t*>(&h);
}

// 8 int4 nibbles (code + 8) of one k-step -> the four A-fragment registers, exact. A nibble in bits
// 0-3 of a half becomes fp16 1024 + n (minus 1032 = code); one in bits 4-7 becomes 1024 + 16 n
// (times 1/16 minus 72 = code); the second pair of slots is reached through w >> 8.
AF_DEV uint32_t lop_or(uint32_t w, uint32_t mask) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w), "r"(mask), "r"(0x64006400u));   // (w & mask) | magic
  return r;
}
AF_DEV void i4x8_to_frag(uint32_t w, uint32_t (&A)[4]) {
  const __half2 b_lo = __half2half2(__ushort_as_half(0x6408));   // 1032
  const __half2 m_hi = __half2half2(__ushort_as_half(0x2C00));   // 1/16
  const __half2 b_hi = __half2half2(__ushort_as_half(0xD480));   // -72
  const uint32_t w8 = w >> 8;
  uint32_t v0 = lop_or(w, 0x000F000Fu), v1 = lop_or(w, 0x00F000F0u);
  uint32_t v2 = lop_or(w8, 0x000F000Fu), v3 = lop_or(w8, 0x00F000F0u);
  __half2 h0 = __hsub2(*reinterpret_cast<const __half2*>(&v0), b_lo);
  __half2 h1 = __hfma2(*reinterpret_cast<const __half2*>(&v1), m_hi, b_hi);
  __half2 h2 = __hsub2(*reinterpret_cast<const __half2*>(&v2), b_lo);
  __half2 h3 = __hfma2(*reinterpret_cast<const __half2*>(&v3), m_hi, b_hi);
  A[0] = *reinterpret_cast<uint32_t*>(&h0);
  A[1] = *reinterpret_cast<uint32_t*>(&h1);
  A[2] = *reinterpret_cast<uint32_t*>(&h2);
  A[3] = *reinterpret_cast<uint32_t*>(&h3);
}

// One ring stage on one consumer warp: the warp owns row tile `rtw` and the k tiles par, par + PSTEP,
// ... of the stage (with PSTEP = 2 a partner warp takes the others). Consecutive tiles of the warp
// alternate between two accumulator sets (acc, acc2) so that two MMA chains are in flight. `xk`
// points at the staged x of the stage's first k tile (row stride `xstride` halves); the tiles' column
// permutation makes a lane's B fragments for both k-steps of a tile one 16-byte load. int4 products
// are formed fresh per tile and added times the tile's group scale.
template <bool I4, int NT, int PSTEP>
AF_DEV void consume_stage(const unsigned char* sb, int nk, const __half* xk, int xstride, int NB, int lane, int rtw,
                          int par, float (&acc)[NT][4], float (&acc2)[NT][4]) {
  using F = tc::Fmt<I4>;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int i = 0; i < F::ks / PSTEP; ++i) {
    const int k2 = par + PSTEP * i;
    if (k2 >= nk) break;
    float (&ac)[NT][4] = (i & 1) ? acc2 : acc;
    uint4 xv[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int row = n * 8 + g;
      xv[n] = row < NB ? *reinterpret_cast<const uint4*>(xk + (size_t)row * xstride + k2 * 32 + 8 * t)
                       : make_uint4(0u, 0u, 0u, 0u);
    }
    if constexpr (I4) {
      const unsigned char* ub = sb + k2 * F::unit;
      const uint2 w = *reinterpret_cast<const uint2*>(ub + rtw * F::tile + lane * 8);
      const float2 sc = __half22float2(
          *reinterpret_cast<const __half2*>(ub + tc::WARPS * F::tile + (rtw * 16 + 2 * g) * 2));
      uint32_t A[4];
      float tmp[NT][4];
      i4x8_to_frag(w.x, A);
#pragma unroll
      for (int n = 0; n < NT; ++n)
        if (n * 8 < NB) mma_16816_z(tmp[n], A, xv[n].x, xv[n].y);   // n-tiles past the live rows: skipped
      i4x8_to_frag(w.y, A);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        if (n * 8 >= NB) continue;
        mma_16816(tmp[n], A, xv[n].z, xv[n].w);
        ac[n][0] = fmaf(sc.x, tmp[n][0], ac[n][0]);
        ac[n][1] = fmaf(sc.x, tmp[n][1], ac[n][1]);
        ac[n][2] = fmaf(sc.y, tmp[n][2], ac[n][2]);
        ac[n][3] = fmaf(sc.y, tmp[n][3], ac[n][3]);
      }
    } else {
      const uint4 w = *reinterpret_cast<const uint4*>(sb + k2 * F::unit + rtw * F::tile + lane * 16);
      uint32_t A[4];
      i8x4_to_h2x2(w.x, A[0], A[1]);
      i8x4_to_h2x2(w.y, A[2], A[3]);
#pragma unroll
      for (int n = 0; n < NT; ++n)
        if (n * 8 < NB) mma_16816(ac[n], A, xv[n].x, xv[n].y);
      i8x4_to_h2x2(w.z, A[0], A[1]);
      i8x4_to_h2x2(w.w, A[2], A[3]);
#pragma unroll
      for (int n = 0; n < NT; ++n)
        if (n * 8 < NB) mma_16816(ac[n], A, xv[n].z, xv[n].w);
    }
  }
}

struct TcShared {
  uint64_t full[tc::STAGES];
  uint64_t empty[tc::STAGES];
  uint64_t xfull[tc::XSLOTS];
  uint64_t xempty[tc::XSLOTS];
  int ticket;
  int cabort;   // a consumer gave up: written by consumers only, read after a consumer barrier
};
constexpr int SH_BYTES = 256;
static_assert(sizeof(TcShared) <= SH_BYTES, "TcShared grew past its slot");

// ---- stream-K geometry (identical on host and device)
AF_DEV long long unit_begin(int c, long long U, int G) { return (long long)c * U / G; }

// the CTA whose range holds unit u
AF_DEV int owner_of(long long u, long long U, int G) {
  int c = (int)((u * G) / U);
  while (c + 1 < G && unit_begin(c + 1, U, G) <= u) ++c;
  while (c > 0 && unit_begin(c, U, G) > u) --c;
  return c;
}

}  // namespace af
