// Decode-attention building blocks shared by the decode and prefill attention kernels: the
// per-lane head layout, QK-norm + RoPE on one head vector, fp16 row loads and the
// batched transpose-reduce of G x PB dot products.
#pragma once
#include "af_common.cuh"

namespace af {

template <int DH>
struct HeadLayout {
  static constexpr int EPL = DH >= 32 ? DH / 32 : 1;   // elements per lane
  static constexpr int LANES = DH >= 32 ? 32 : DH;     // lanes holding the head vector
  static constexpr int PARTNER = LANES / 2;            // xor distance of the rotate-half partner
};

// This lane's RoPE factors of row `p` (cos, sin of its EPL elements); zeros without RoPE.
template <int DH>
AF_DEV void load_rope_row(const __half* cos_t, const __half* sin_t, int p, int lane, float (&cs)[HeadLayout<DH>::EPL],
                          float (&sn)[HeadLayout<DH>::EPL]) {
  using HL = HeadLayout<DH>;
#pragma unroll
  for (int e = 0; e < HL::EPL; ++e) {
    const int d = lane * HL::EPL + e;
    const bool ok = cos_t && lane < HL::LANES;
    cs[e] = ok ? h2f(cos_t[(size_t)p * DH + d]) : 0.f;
    sn[e] = ok ? h2f(sin_t[(size_t)p * DH + d]) : 0.f;
  }
}

// One head vector held as EPL contiguous elements per lane: optional RMSNorm, then RoPE with this
// lane's factors (`rope` false: none).
template <int DH>
AF_DEV void norm_rope_head_pre(float (&v)[HeadLayout<DH>::EPL], int lane, const __half* ng, float nfloor, bool rope,
                               const float (&cs)[HeadLayout<DH>::EPL], const float (&sn)[HeadLayout<DH>::EPL]) {
  using HL = HeadLayout<DH>;
  const bool active = lane < HL::LANES;
  if (ng) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < HL::EPL; ++e) ss = fmaf(v[e], v[e], ss);
    ss = active ? ss : 0.f;
    ss = warp_sum(ss);
    const float sq = fmaxf(sqrtf(ss), nfloor);
#pragma unroll
    for (int e = 0; e < HL::EPL; ++e) {
      const int d = lane * HL::EPL + e;
      v[e] = active ? __fmul_rn(__fdiv_rn(v[e], sq), h2f(ng[d])) : 0.f;
    }
  }
  if (rope) {
#pragma unroll
    for (int e = 0; e < HL::EPL; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, v[e], HL::PARTNER);
      if (active) {
        const int d = lane * HL::EPL + e;
        const float rot = d < DH / 2 ? -other : other;
        v[e] = __fadd_rn(__fmul_rn(v[e], cs[e]), __fmul_rn(rot, sn[e]));
      }
    }
  }
}

// One head vector held as EPL contiguous elements per lane: optional RMSNorm, RoPE at row `p`.
template <int DH>
AF_DEV void norm_rope_head(float (&v)[HeadLayout<DH>::EPL], int lane, const __half* ng, float nfloor,
                           const __half* cos_t, const __half* sin_t, int p) {
  float cs[HeadLayout<DH>::EPL], sn[HeadLayout<DH>::EPL];
  load_rope_row<DH>(cos_t, sin_t, p, lane, cs, sn);
  norm_rope_head_pre<DH>(v, lane, ng, nfloor, cos_t != nullptr, cs, sn);
}

template <int DH>
AF_DEV void load_row_f16(const __half* p, int lane, float (&f)[HeadLayout<DH>::EPL]) {
  using HL = HeadLayout<DH>;
  if (lane >= HL::LANES) {
#pragma unroll
    for (int e = 0; e < HL::EPL; ++e) f[e] = 0.f;
    return;
  }
  const __half* q = p + lane * HL::EPL;
  if constexpr (HL::EPL == 4) {
    const uint2 u = __ldcg(reinterpret_cast<const uint2*>(q));
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    const float2 x = __half22float2(h[0]), y = __half22float2(h[1]);
    f[0] = x.x; f[1] = x.y; f[2] = y.x; f[3] = y.y;
  } else if constexpr (HL::EPL == 2) {
    const float2 x = __half22float2(__ldcg(reinterpret_cast<const __half2*>(q)));
    f[0] = x.x; f[1] = x.y;
  } else {
#pragma unroll
    for (int e = 0; e < HL::EPL; ++e) f[e] = h2f(__ldcg(q + e));
  }
}

// Each warp walks its keys in batches of PB positions: all PB K rows and PB V rows of a batch are
// loaded before any math (2*PB loads in flight per lane), the G*PB partial dot products are summed
// across the warp with a transpose-reduce (each shuffle level halves the values a lane keeps, so 32
// sums cost 31 shuffles instead of 160) and the online softmax then runs once per batch.
template <int DH, int G, int PBMAX = 8>
struct DecodeBatch {
  static constexpr int PB = (32 / G) < PBMAX ? (32 / G) : PBMAX;   // positions per batch
  static constexpr int NV = G * PB;                         // dot products per batch (power of 2)
  static constexpr int LOGNV = NV == 32 ? 5 : NV == 16 ? 4 : NV == 8 ? 3 : NV == 4 ? 2 : 1;
  static constexpr int SHIFT = 5 - LOGNV;                   // lane L holds value index L >> SHIFT
  static constexpr int GS = 32 / G;                         // lanes per head after the reduce
};

template <int NV>
AF_DEV float transpose_reduce(float (&v)[NV], int lane) {
  // level `off` keeps the lower or upper half of the remaining values and adds the partner's copy
  int n = NV;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    if (n > 1) {
      const bool upper = lane & off;
#pragma unroll
      for (int i = 0; i < NV / 2; ++i) {
        if (i < n / 2) {
          const float send = upper ? v[i] : v[i + n / 2];
          const float keep = upper ? v[i + n / 2] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      n >>= 1;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
  return v[0];
}

}  // namespace af
