// GQA attention over the resident fp16 KV cache.
//
// K5 decode (one new token per sequence): one CTA per (split, kv head, sequence). The CTA
//   1. takes the G = H/KV query heads of its kv head from the fused QKV output, applies the optional
//      per-head RMSNorm (QK-norm) and RoPE (neox half split: the partner of lane l is lane l^16), and
//      rounds q to fp16 (the bmm operand);
//   2. if its key range holds `pos`, ropes the new k, writes k and v into the cache slot `pos`
//      (the reference's `Kin*inv + k*oh` write of llm.py:232, without touching the other M-1 slots);
//   3. runs an online softmax over its keys (split-K / flash-decode), each key expanded as the
//      reference's 0/1 GQA matmul does (f16(c * k), c = 1 without expansion, llm.py:205-211);
//   4. merges the splits of its (sequence, kv head): with up to 16 splits they form one thread-block
//      cluster and rank 0 reads every split's (m, l, acc) from the others' shared memory (no global
//      round trips); otherwise each writes its partial to scratch and the last CTA to finish
//      (atomic ticket) merges them. Either way the merge runs in split order, so it is deterministic.
// Keys after `pos` carry the reference's additive -1e4 mask, whose exp underflows to exactly 0 in
// fp32, so they are skipped. Probabilities stay fp32.
//
// Prefill (S prompt rows): rope_kv_prefill ropes q/k for every row, writes the roped K and raw V
// straight into cache rows 0..S-1 (the decode layout, so no seeding copy), and attn_prefill runs a
// causal online softmax with one warp per query row.
#include "af_common.cuh"
#include "af_kernels.h"
#include "attn_common.cuh"
#include "tc_common.cuh"

namespace af {

constexpr int DEC_WARPS = 8;
constexpr int DEC_PRE_MAX = 128;               // cache rows per CTA staged in shared memory up front (max)
constexpr int DEC_CLUSTER_MAX = 16;            // splits merged inside one cluster
// keys per CTA for the three-phase path (its score table must fit the static shared memory)
template <int G> struct DirectMax { static constexpr int n = G <= 4 ? 128 : 64; };

// Keys per split at position pos: the first ns splits share the pos + 1 keys evenly, where ns is
// n_split but at most one split per `min_keys` keys (short prefixes leave the other splits idle).
AF_DEV int split_len(int pos, int n_split, int min_keys) {
  const int ns = min(n_split, max(1, (pos + min_keys) / min_keys));
  return (pos + ns) / ns;                      // ceil((pos + 1) / ns)
}


AF_DEV void load_row_f16_sh(const __half* p, int lane, float* f, int epl, int lanes) {
  if (lane >= lanes) {
    for (int e = 0; e < epl; ++e) f[e] = 0.f;
    return;
  }
  if (epl == 4) {                                  // one 8-byte shared load
    const uint2 u = *reinterpret_cast<const uint2*>(p + lane * 4);
    const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    f[0] = x.x; f[1] = x.y; f[2] = y.x; f[3] = y.y;
    return;
  }
  for (int e = 0; e < epl; ++e) f[e] = __half2float(p[lane * epl + e]);
}

template <int DH, int G, bool DIRECT>
__global__ void __launch_bounds__(DEC_WARPS * 32, 2) attn_decode_kernel(AttnDecodeArgs a) {
  using HL = HeadLayout<DH>;
  using DB = DecodeBatch<DH, G>;
  constexpr int EPL = HL::EPL;
  constexpr int NW = DEC_WARPS;
  constexpr int PB = DB::PB;
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool active = lane < HL::LANES;

  __shared__ float q_s[G][DH];
  __shared__ float kn_s[DH], vn_s[DH];
  __shared__ float wm[NW][G], wl[NW][G];
  __shared__ float wacc[NW][G][DH];
  __shared__ int last_s;
  __shared__ uint64_t kv_bar;
  extern __shared__ __align__(16) unsigned char kv_pre[];     // [K rows | V rows] x pre_rows x DH fp16

  // with `prefetch`, the first pre_rows cache rows of this CTA's key range (all before pos, so
  // written in earlier steps) and the RoPE factors of row pos are requested before waiting for the
  // qkv projection
  int n_pre = 0;
  int pos = 0;
  float rc[EPL], rs[EPL];
  const size_t seq_rows = a.kv_seq_rows < 0 ? (size_t)a.KV * a.M : (size_t)a.kv_seq_rows;
  l2_prefetch_lines(a.pf, ((blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) * blockDim.x + threadIdx.x,
                    gridDim.x * gridDim.y * gridDim.z * blockDim.x);
  if (a.prefetch) {
    pos = __ldcg(a.pos + b);
    if (pos >= 0 && pos < a.M) {
      load_rope_row<DH>(a.cos_t, a.sin_t, pos, lane, rc, rs);
      const int len0 = split_len(pos, a.n_split, a.min_keys);
      const int j00 = split * len0;
      n_pre = max(0, min(min(j00 + len0, pos), j00 + a.pre_rows) - j00);
      if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"((uint32_t)__cvta_generic_to_shared(&kv_bar)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (n_pre > 0) {
          const uint32_t bytes = (uint32_t)n_pre * DH * 2;
          const __half* kb0 = a.kc + ((size_t)b * seq_rows + (size_t)kvh * a.M + j00) * DH;
          const __half* vb0 = a.vc + ((size_t)b * seq_rows + (size_t)kvh * a.M + j00) * DH;
          const uint32_t bar = (uint32_t)__cvta_generic_to_shared(&kv_bar);
          asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(2 * bytes) : "memory");
          asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                       ::"r"((uint32_t)__cvta_generic_to_shared(kv_pre)), "l"(kb0), "r"(bytes), "r"(bar) : "memory");
          asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                       ::"r"((uint32_t)__cvta_generic_to_shared(kv_pre + (size_t)a.pre_rows * DH * 2)), "l"(vb0),
                         "r"(bytes), "r"(bar)
                       : "memory");
        }
      }
    }
  }
  pdl_wait();
  if (!a.prefetch) pos = __ldcg(a.pos + b);
  if (pos < 0 || pos >= a.M) {
    // every CTA of a cluster holds the same sequence, so the whole cluster leaves here together
    if (threadIdx.x == 0 && split == 0 && kvh == 0) af_set_err(a.err, AF_DEV_BAD_POS);
    return;
  }
  if (!a.prefetch) load_rope_row<DH>(a.cos_t, a.sin_t, pos, lane, rc, rs);
  const bool rope = a.cos_t != nullptr;
  const int len = split_len(pos, a.n_split, a.min_keys);
  const int j0 = split * len;
  const int j1 = min(j0 + len, pos + 1);
  const bool owns_pos = j0 <= pos && pos < j1;
  const float* qkv = a.qkv + (size_t)b * a.ld_qkv;
  const int H = a.H, KV = a.KV;

  // ---- q heads (and the new k/v in the CTA that owns pos)
  for (int g = warp; g < G; g += NW) {
    float v[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) v[e] = active ? __ldcg(qkv + (size_t)(kvh * G + g) * DH + lane * EPL + e) : 0.f;
    norm_rope_head_pre<DH>(v, lane, a.qn_g, a.qn_floor, rope, rc, rs);
    if (active)
#pragma unroll
      for (int e = 0; e < EPL; ++e) q_s[g][lane * EPL + e] = round_f16(v[e]);
  }
  if (owns_pos && warp == NW - 1) {
    float k[EPL], vv[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      k[e] = active ? __ldcg(qkv + (size_t)H * DH + (size_t)kvh * DH + lane * EPL + e) : 0.f;
      vv[e] = active ? __ldcg(qkv + (size_t)(H + KV) * DH + (size_t)kvh * DH + lane * EPL + e) : 0.f;
    }
    norm_rope_head_pre<DH>(k, lane, a.kn_g, a.kn_floor, rope, rc, rs);
    const size_t slot = ((size_t)b * seq_rows + (size_t)kvh * a.M + pos) * DH;
    if (active)
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const __half kh = f2h(k[e]), vh = f2h(vv[e]);
        if (a.write_kv) {
          a.kc[slot + lane * EPL + e] = kh;
          a.vc[slot + lane * EPL + e] = vh;
        }
        kn_s[lane * EPL + e] = h2f(kh);
        vn_s[lane * EPL + e] = h2f(vh);
      }
  }
  __syncthreads();
  pdl_trigger();

  float qr[G][EPL];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < EPL; ++e) qr[g][e] = active ? q_s[g][lane * EPL + e] : 0.f;

  float m[G], l[G], acc[G][EPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY; l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[g][e] = 0.f;
  }
  const __half* kbase = a.kc + ((size_t)b * seq_rows + (size_t)kvh * a.M) * DH;
  const __half* vbase = a.vc + ((size_t)b * seq_rows + (size_t)kvh * a.M) * DH;
  const float c = a.kv_c;
  const int my_idx = lane >> DB::SHIFT;                 // value index this lane ends up holding
  const int my_g = my_idx / PB, my_p = my_idx % PB;
  const bool rep0 = (lane & ((1 << DB::SHIFT) - 1)) == 0;
  if (n_pre > 0) {
    // bounded wait for the staged rows; on a timeout they are read from global memory instead
    const uint32_t bar = (uint32_t)__cvta_generic_to_shared(&kv_bar);
    bool ok = false;
    for (long long i = 0; i < (1ll << 24) && !ok; ++i) {
      uint32_t r;
      asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n selp.u32 %0, 1, 0, p;\n}\n"
                   : "=r"(r) : "r"(bar) : "memory");
      ok = r != 0;
    }
    if (!ok) {
      if (threadIdx.x == 0) af_set_err(a.err, AF_DEV_WAIT_TIMEOUT);
      n_pre = 0;
    }
  }
  const __half* kpre = reinterpret_cast<const __half*>(kv_pre);
  const __half* vpre = kpre + (size_t)a.pre_rows * DH;
  // DIRECT (every split holds at most DirectMax keys): the split runs as three short phases
  // instead of one long per-warp online softmax: scores (each warp a batch of PB keys: dot products
  // + transpose-reduce) -> per-head max, exp and sum (one warp per head) -> P.V with the keys dealt
  // over the warps, partial sums per warp. Rows come from the staged copy when it holds them.
  constexpr bool direct = DIRECT;
  const int n_keys = j1 > j0 ? j1 - j0 : 0;
  __shared__ float s_s[G][DIRECT ? DirectMax<G>::n : 1];        // scores, then exp(s - m)
  __shared__ float dm[G], dl[G];
  if constexpr (DIRECT) {
    for (int base = j0 + warp * PB; base < j1; base += NW * PB) {
      float kf[PB][EPL];
#pragma unroll
      for (int p = 0; p < PB; ++p) {
        const int j = base + p;
        if (j < j1 && j != pos && j - j0 < n_pre) {
          load_row_f16_sh(kpre + (size_t)(j - j0) * DH, lane, kf[p], EPL, HL::LANES);
        } else if (j < j1 && j != pos) {
          load_row_f16<DH>(kbase + (size_t)j * DH, lane, kf[p]);
        } else {
          const bool nw = j < j1 && active;
#pragma unroll
          for (int e = 0; e < EPL; ++e) kf[p][e] = nw ? kn_s[lane * EPL + e] : 0.f;
        }
      }
      if (a.expand) {
#pragma unroll
        for (int p = 0; p < PB; ++p)
#pragma unroll
          for (int e = 0; e < EPL; ++e) kf[p][e] = round_f16(c * kf[p][e]);
      }
      float d[DB::NV];
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int p = 0; p < PB; ++p) {
          float sdot = 0.f;
#pragma unroll
          for (int e = 0; e < EPL; ++e) sdot = fmaf(qr[g][e], kf[p][e], sdot);
          d[g * PB + p] = sdot;
        }
      const float sc = transpose_reduce<DB::NV>(d, lane) * a.scale;
      if (rep0 && base + my_p < j1) s_s[my_g][base + my_p - j0] = sc;
    }
    __syncthreads();
    if (warp < G) {
      float mx = -INFINITY;
      for (int k = lane; k < n_keys; k += 32) mx = fmaxf(mx, s_s[warp][k]);
      mx = warp_max(mx);
      float sum = 0.f;
      for (int k = lane; k < n_keys; k += 32) {
        const float pe = expf(s_s[warp][k] - mx);
        s_s[warp][k] = pe;
        sum += pe;
      }
      sum = warp_sum(sum);
      if (lane == 0) { dm[warp] = mx; dl[warp] = sum; }
    }
    __syncthreads();
    float pacc[G][EPL];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int e = 0; e < EPL; ++e) pacc[g][e] = 0.f;
    for (int k = warp; k < n_keys; k += NW) {
      float vf[EPL];
      if (j0 + k != pos && k < n_pre) {
        load_row_f16_sh(vpre + (size_t)k * DH, lane, vf, EPL, HL::LANES);
      } else if (j0 + k != pos) {
        load_row_f16<DH>(vbase + (size_t)(j0 + k) * DH, lane, vf);
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) vf[e] = active ? vn_s[lane * EPL + e] : 0.f;
      }
      if (a.expand) {
#pragma unroll
        for (int e = 0; e < EPL; ++e) vf[e] = round_f16(c * vf[e]);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pg = s_s[g][k];
#pragma unroll
        for (int e = 0; e < EPL; ++e) pacc[g][e] = fmaf(pg, vf[e], pacc[g][e]);
      }
    }
    if (active)
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < EPL; ++e) wacc[warp][g][lane * EPL + e] = pacc[g][e];
  }
  if constexpr (!DIRECT)
  for (int base = j0 + warp * PB; base < j1; base += NW * PB) {
    float kf[PB][EPL], vf[PB][EPL];
#pragma unroll
    for (int p = 0; p < PB; ++p) {
      const int j = base + p;
      const bool in_range = j < j1;                // keys past this CTA's range are zeros
      if (in_range && j != pos && j - j0 < n_pre) {
        load_row_f16_sh(kpre + (size_t)(j - j0) * DH, lane, kf[p], EPL, HL::LANES);
        load_row_f16_sh(vpre + (size_t)(j - j0) * DH, lane, vf[p], EPL, HL::LANES);
      } else if (in_range && j != pos) {
        load_row_f16<DH>(kbase + (size_t)j * DH, lane, kf[p]);
        load_row_f16<DH>(vbase + (size_t)j * DH, lane, vf[p]);
      } else {
        // the new key/value live in shared memory, written only by the CTA whose range holds pos
        const bool nw = in_range && active;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          kf[p][e] = nw ? kn_s[lane * EPL + e] : 0.f;
          vf[p][e] = nw ? vn_s[lane * EPL + e] : 0.f;
        }
      }
    }
    if (a.expand) {
#pragma unroll
      for (int p = 0; p < PB; ++p)
#pragma unroll
        for (int e = 0; e < EPL; ++e) { kf[p][e] = round_f16(c * kf[p][e]); vf[p][e] = round_f16(c * vf[p][e]); }
    }
    float d[DB::NV];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int p = 0; p < PB; ++p) {
        float sdot = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) sdot = fmaf(qr[g][e], kf[p][e], sdot);
        d[g * PB + p] = sdot;
      }
    const float sc = transpose_reduce<DB::NV>(d, lane) * a.scale;
    const bool valid = base + my_p < j1;
    const float s = valid ? sc : -INFINITY;
    // per-head tile max / sum over the head's lane group
    float tmax = s;
#pragma unroll
    for (int off = DB::GS / 2; off >= 1; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
    float mnew_mine = fmaxf(m[0], tmax);
#pragma unroll
    for (int g = 1; g < G; ++g) if (g == my_g) mnew_mine = fmaxf(m[g], tmax);
    const float pe = valid ? expf(s - mnew_mine) : 0.f;
    float tsum = rep0 ? pe : 0.f;
#pragma unroll
    for (int off = DB::GS / 2; off >= 1; off >>= 1) tsum += __shfl_xor_sync(0xffffffffu, tsum, off);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mg = __shfl_sync(0xffffffffu, tmax, g * DB::GS);
      const float sg = __shfl_sync(0xffffffffu, tsum, g * DB::GS);
      const float mn = fmaxf(m[g], mg);
      const float corr = expf(m[g] - mn);
      l[g] = l[g] * corr + sg;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[g][e] *= corr;
#pragma unroll
      for (int p = 0; p < PB; ++p) {
        const float pp = __shfl_sync(0xffffffffu, pe, (g * PB + p) << DB::SHIFT);
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[g][e] = fmaf(pp, vf[p][e], acc[g][e]);
      }
      m[g] = mn;
    }
  }
  // ---- merge the warps of this CTA: (num, M, den) of head g, element dd
  if constexpr (!DIRECT) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (lane == 0) { wm[warp][g] = m[g]; wl[warp][g] = l[g]; }
      if (active)
#pragma unroll
        for (int e = 0; e < EPL; ++e) wacc[warp][g][lane * EPL + e] = acc[g][e];
    }
  }
  __syncthreads();
  auto merge_warps = [&](int g, int dd, float& num, float& M, float& den) {
    num = 0.f;
    if constexpr (DIRECT) {
      M = dm[g];
      den = dl[g];
#pragma unroll
      for (int w = 0; w < NW; ++w) num += wacc[w][g][dd];
      return;
    }
    M = -INFINITY;
    den = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w][g]);
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float f = expf(wm[w][g] - M);
        num = fmaf(f, wacc[w][g][dd], num);
        den = fmaf(f, wl[w][g], den);
      }
    }
  };
  const size_t pair = (size_t)b * KV + kvh;
  __shared__ float fw[64][G];      // per split: m_s, then the weight exp(m_s - M)
  __shared__ float lw[64][G];      // per split: l_s
  __shared__ float den_s[G];
  if (a.cluster) {
    // ---- cluster merge: every split stores its (acc, m, l) straight into rank 0's merge area
    // (dynamic shared memory after the staged rows, [n_split][G][DH + 2]); after one cluster barrier
    // rank 0 (split 0) merges them from its own shared memory and the other CTAs leave
    float* mrg = reinterpret_cast<float*>(kv_pre + (size_t)2 * a.pre_rows * DH * 2);
    const uint32_t dst = cluster_addr(mrg, 0) + (uint32_t)split * G * (DH + 2) * 4;
    for (int i = threadIdx.x; i < G * DH; i += blockDim.x) {
      const int g = i / DH, dd = i - g * DH;
      float num, M, den;
      merge_warps(g, dd, num, M, den);
      const uint32_t at = dst + (uint32_t)(g * (DH + 2)) * 4;
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(at + dd * 4), "f"(num) : "memory");
      if (dd == 0) {
        asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(at + DH * 4), "f"(M) : "memory");
        asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(at + (DH + 1) * 4), "f"(den) : "memory");
      }
    }
    cluster_sync_all();
    if (split != 0) return;
    for (int i = threadIdx.x; i < a.n_split * G; i += blockDim.x) {
      const int sp = i / G, g = i - sp * G;
      fw[sp][g] = mrg[(sp * G + g) * (DH + 2) + DH];
      lw[sp][g] = mrg[(sp * G + g) * (DH + 2) + DH + 1];
    }
    __syncthreads();
    if (threadIdx.x < G) {
      const int g = threadIdx.x;
      float M = -INFINITY;
      for (int sp = 0; sp < a.n_split; ++sp) M = fmaxf(M, fw[sp][g]);
      float den = 0.f;
      for (int sp = 0; sp < a.n_split; ++sp) {
        const float f = fw[sp][g] == -INFINITY ? 0.f : expf(fw[sp][g] - M);
        den = fmaf(f, lw[sp][g], den);
        fw[sp][g] = f;
      }
      den_s[g] = den;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * DH; i += blockDim.x) {
      const int g = i / DH, dd = i - g * DH;
      float num = 0.f;
#pragma unroll 4
      for (int sp = 0; sp < a.n_split; ++sp) num = fmaf(fw[sp][g], mrg[(sp * G + g) * (DH + 2) + dd], num);
      a.out[(size_t)b * a.ld_out + (size_t)(kvh * G + g) * DH + dd] = f2h(num / den_s[g]);
    }
    return;
  }
  float* part = a.part + (pair * a.n_split + split) * G * (DH + 2);
  for (int i = threadIdx.x; i < G * DH; i += blockDim.x) {
    const int g = i / DH, dd = i - g * DH;
    float num, M, den;
    merge_warps(g, dd, num, M, den);
    if (a.n_split == 1) {
      a.out[(size_t)b * a.ld_out + (size_t)(kvh * G + g) * DH + dd] = f2h(num / den);
    } else {
      __stcg(part + g * (DH + 2) + dd, num);
      if (dd == 0) { __stcg(part + g * (DH + 2) + DH, M); __stcg(part + g * (DH + 2) + DH + 1, den); }
    }
  }
  if (a.n_split == 1) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last_s = atomicAdd(a.counters + pair, 1) == a.n_split - 1;
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  // ---- merge the splits: (m_s, l_s) of every split land in shared memory in one parallel pass, the
  // per-head weights exp(m_s - M) are formed once, then each output issues its n_split loads together
  const float* pp = a.part + pair * a.n_split * G * (DH + 2);
  for (int i = threadIdx.x; i < a.n_split * G; i += blockDim.x) {
    const int sp = i / G, g = i - sp * G;
    fw[sp][g] = __ldcg(pp + (sp * G + g) * (DH + 2) + DH);
    lw[sp][g] = __ldcg(pp + (sp * G + g) * (DH + 2) + DH + 1);
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    float M = -INFINITY;
    for (int sp = 0; sp < a.n_split; ++sp) M = fmaxf(M, fw[sp][g]);
    float den = 0.f;
    for (int sp = 0; sp < a.n_split; ++sp) {
      const float f = fw[sp][g] == -INFINITY ? 0.f : expf(fw[sp][g] - M);
      den = fmaf(f, lw[sp][g], den);
      fw[sp][g] = f;
    }
    den_s[g] = den;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * DH; i += blockDim.x) {
    const int g = i / DH, dd = i - g * DH;
    float num = 0.f;
#pragma unroll 8
    for (int sp = 0; sp < a.n_split; ++sp) num = fmaf(fw[sp][g], __ldcg(pp + (sp * G + g) * (DH + 2) + dd), num);
    a.out[(size_t)b * a.ld_out + (size_t)(kvh * G + g) * DH + dd] = f2h(num / den_s[g]);
  }
  if (threadIdx.x == 0) a.counters[pair] = 0;
}

size_t attn_decode_scratch_floats(int NB, int KV, int n_split, int G, int dh) {
  return (size_t)NB * KV * n_split * G * (dh + 2);
}

template <int DH, int G, bool DIRECT>
static cudaError_t launch_decode(const AttnDecodeArgs& a, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_split, a.KV, a.NB);
  cfg.blockDim = dim3(DEC_WARPS * 32);
  // staged cache rows, then (clusters) rank 0's merge area [n_split][G][DH + 2] fp32
  cfg.dynamicSmemBytes = (a.prefetch ? 2 * (size_t)a.pre_rows * DH * 2 : 0) +
                         (a.cluster ? (size_t)a.n_split * G * (DH + 2) * 4 : 0);
  static PerDeviceOnce attrs;                  // static + dynamic shared memory may pass 48 KB
  const cudaError_t ae = attrs.run([] {
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<DH, G, DIRECT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         2 * DEC_PRE_MAX * DH * 2 + DEC_CLUSTER_MAX * G * (DH + 2) * 4);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attn_decode_kernel<DH, G, DIRECT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    return e;
  });
  if (ae != cudaSuccess) return ae;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (a.cluster) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = a.n_split;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, attn_decode_kernel<DH, G, DIRECT>, a);
}

// the three-phase kernel when no split can hold more than DirectMax keys: at most
// max(min_keys, ceil(M / n_split)) keys per split
template <int DH, int G>
static cudaError_t decode_d(const AttnDecodeArgs& a, cudaStream_t st, bool pdl) {
  static const int use_direct = env_int("AF_ATTN_DIRECT", 1);
  const int most = max((a.M + a.n_split - 1) / a.n_split, a.min_keys);
  if (use_direct && most <= DirectMax<G>::n) return launch_decode<DH, G, true>(a, st, pdl);
  return launch_decode<DH, G, false>(a, st, pdl);
}

template <int DH>
static cudaError_t decode_g(const AttnDecodeArgs& a, cudaStream_t st, bool pdl) {
  switch (a.H / a.KV) {
    case 1: return decode_d<DH, 1>(a, st, pdl);
    case 2: return decode_d<DH, 2>(a, st, pdl);
    case 4: return decode_d<DH, 4>(a, st, pdl);
    case 8: return decode_d<DH, 8>(a, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

// splits merge inside a cluster when they fit one (AF_ATTN_CLUSTER=0: always through scratch)
static bool merge_in_cluster(const AttnDecodeArgs& a) {
  static const int use_cluster = env_int("AF_ATTN_CLUSTER", 1);
  return use_cluster && a.n_split > 1 && a.n_split <= DEC_CLUSTER_MAX;
}

bool attn_decode_uses_scratch(const AttnDecodeArgs& a) { return a.n_split > 1 && !merge_in_cluster(a); }

cudaError_t attn_decode_launch(const AttnDecodeArgs& a0, cudaStream_t st, bool pdl) {
  AttnDecodeArgs a = a0;
  if (a.KV <= 0 || a.H % a.KV || a.n_split < 1 || a.n_split > 64) return cudaErrorInvalidValue;
  a.cluster = merge_in_cluster(a) ? 1 : 0;
  if (!a.cluster && a.n_split > 1 && (!a.part || !a.counters)) return cudaErrorInvalidValue;
  static const int min_keys = env_int("AF_ATTN_MIN_KEYS", 64);
  a.min_keys = a.min_keys > 0 ? a.min_keys : min_keys;
  // staged rows: a CTA's whole key range when it fits, else its first DEC_PRE_MAX rows
  const int per_split = max((a.M + a.n_split - 1) / a.n_split, a.min_keys);
  a.pre_rows = a.prefetch ? (per_split < DEC_PRE_MAX ? (per_split + 1) / 2 * 2 : DEC_PRE_MAX) : 0;
  switch (a.dh) {
    case 16: return decode_g<16>(a, st, pdl);
    case 32: return decode_g<32>(a, st, pdl);
    case 64: return decode_g<64>(a, st, pdl);
    case 128: return decode_g<128>(a, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

// ----------------------------------------------------------------------------------- K/V append

// grid (NB, KV), one warp: the k of batch row b, kv head kvh (QK-norm, RoPE at pos[b]) and its v,
// written to cache row pos[b] - the same values the decode kernel forms for its own row
template <int DH>
__global__ void __launch_bounds__(32) kv_append_kernel(AttnDecodeArgs a) {
  using HL = HeadLayout<DH>;
  constexpr int EPL = HL::EPL;
  const int b = blockIdx.x, kvh = blockIdx.y, lane = threadIdx.x;
  const bool active = lane < HL::LANES;
  pdl_wait();
  const int pos = __ldcg(a.pos + b);
  if (pos < 0 || pos >= a.M) {
    if (lane == 0 && kvh == 0) af_set_err(a.err, AF_DEV_BAD_POS);
    return;
  }
  float rc[EPL], rs[EPL];
  load_rope_row<DH>(a.cos_t, a.sin_t, pos, lane, rc, rs);
  const float* qkv = a.qkv + (size_t)b * a.ld_qkv;
  float k[EPL], vv[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    k[e] = active ? __ldcg(qkv + (size_t)a.H * DH + (size_t)kvh * DH + lane * EPL + e) : 0.f;
    vv[e] = active ? __ldcg(qkv + (size_t)(a.H + a.KV) * DH + (size_t)kvh * DH + lane * EPL + e) : 0.f;
  }
  norm_rope_head_pre<DH>(k, lane, a.kn_g, a.kn_floor, a.cos_t != nullptr, rc, rs);
  const size_t seq_rows = a.kv_seq_rows < 0 ? (size_t)a.KV * a.M : (size_t)a.kv_seq_rows;
  const size_t slot = ((size_t)b * seq_rows + (size_t)kvh * a.M + pos) * DH;
  if (active)
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      a.kc[slot + lane * EPL + e] = f2h(k[e]);
      a.vc[slot + lane * EPL + e] = f2h(vv[e]);
    }
  pdl_trigger();
}

cudaError_t kv_append_launch(const AttnDecodeArgs& a, cudaStream_t st, bool pdl) {
  if (a.NB < 1 || a.KV <= 0 || a.M <= 0) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.NB, a.KV);
  cfg.blockDim = dim3(32);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  switch (a.dh) {
    case 16: return cudaLaunchKernelEx(&cfg, kv_append_kernel<16>, a);
    case 32: return cudaLaunchKernelEx(&cfg, kv_append_kernel<32>, a);
    case 64: return cudaLaunchKernelEx(&cfg, kv_append_kernel<64>, a);
    case 128: return cudaLaunchKernelEx(&cfg, kv_append_kernel<128>, a);
    default: return cudaErrorInvalidValue;
  }
}

// ----------------------------------------------------------------------------------- prefill

// grid (S, H + KV): block y < H ropes query head y of row x into qbuf [H][S][DH]; the others rope
// key head (y - H) and write K (roped) and V into cache rows.
template <int DH>
__global__ void __launch_bounds__(32) rope_kv_prefill_kernel(AttnPrefillArgs a, __half* qbuf) {
  using HL = HeadLayout<DH>;
  constexpr int EPL = HL::EPL;
  const int s = blockIdx.x, y = blockIdx.y, lane = threadIdx.x;
  const bool active = lane < HL::LANES;
  const float* row = a.qkv + (size_t)s * a.ld_qkv;
  float v[EPL];
  if (y < a.H) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) v[e] = active ? row[(size_t)y * DH + lane * EPL + e] : 0.f;
    norm_rope_head<DH>(v, lane, a.qn_g, a.qn_floor, a.cos_t, a.sin_t, s);
    if (active)
#pragma unroll
      for (int e = 0; e < EPL; ++e) qbuf[((size_t)y * a.S + s) * DH + lane * EPL + e] = f2h(v[e]);
  } else {
    const int kvh = y - a.H;
#pragma unroll
    for (int e = 0; e < EPL; ++e) v[e] = active ? row[(size_t)(a.H + kvh) * DH + lane * EPL + e] : 0.f;
    norm_rope_head<DH>(v, lane, a.kn_g, a.kn_floor, a.cos_t, a.sin_t, s);
    if (active)
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const size_t o = ((size_t)kvh * a.ldm + s) * DH + lane * EPL + e;
        const __half kh = f2h(v[e]), vh = f2h(row[(size_t)(a.H + a.KV + kvh) * DH + lane * EPL + e]);
        a.kc[o] = kh;
        a.vc[o] = vh;
        if (a.expand && a.kvx) {                           // f16(c * f16(k)), as the attention reads them
          const size_t x = ((size_t)kvh * a.S + s) * DH + lane * EPL + e;
          a.kvx[x] = f2h(a.kv_c * h2f(kh));
          a.kvx[(size_t)a.KV * a.S * DH + x] = f2h(a.kv_c * h2f(vh));
        }
      }
  }
}

// grid (H, ceil(S/4)), 4 warps: warp w handles query row i = blockIdx.y*4 + w over keys 0..i.
template <int DH>
__global__ void __launch_bounds__(128) attn_prefill_kernel(AttnPrefillArgs a, const __half* qbuf) {
  using HL = HeadLayout<DH>;
  constexpr int EPL = HL::EPL;
  const int h = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.y * 4 + warp;
  if (i >= a.S) return;
  const int G = a.H / a.KV, kvh = h / G;
  float q[EPL];
  load_row_f16<DH>(qbuf + ((size_t)h * a.S + i) * DH, lane, q);
  const __half* kb = a.kc + (size_t)kvh * a.ldm * DH;
  const __half* vb = a.vc + (size_t)kvh * a.ldm * DH;
  float m = -INFINITY, l = 0.f, acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) acc[e] = 0.f;
  for (int j = 0; j <= i; ++j) {
    float kf[EPL], vf[EPL];
    load_row_f16<DH>(kb + (size_t)j * DH, lane, kf);
    load_row_f16<DH>(vb + (size_t)j * DH, lane, vf);
    if (a.expand) {
#pragma unroll
      for (int e = 0; e < EPL; ++e) { kf[e] = round_f16(a.kv_c * kf[e]); vf[e] = round_f16(a.kv_c * vf[e]); }
    }
    float sc = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) sc = fmaf(q[e], kf[e], sc);
    sc = warp_sum(sc) * a.scale;
    const float mn = fmaxf(m, sc);
    const float corr = expf(m - mn), p = expf(sc - mn);
    l = l * corr + p;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = fmaf(p, vf[e], acc[e] * corr);
    m = mn;
  }
  if (lane < HL::LANES)
#pragma unroll
    for (int e = 0; e < EPL; ++e) a.out[(size_t)i * a.H * DH + (size_t)h * DH + lane * EPL + e] = f2h(acc[e] / l);
}

// ---- prefill causal attention on the tensor pipe (head dim 128): flash-attention style, mma.sync
// m16n8k16 with fp32 accumulators. CTA = (head, 64 query rows), 4 warps of 16 rows. Per 64-key block
// of the head's kv group: K and V rows staged in shared memory (rows padded to 136 halves so the
// fragment loads hit 32 distinct banks; the GQA expansion factor applied while staging), S = Q K^T
// (Q fragments held in registers), causal and length masks, online softmax in fp32 per row, then
// P (rounded to fp16, the MMA operand) times V through ldmatrix.trans fragments into the fp32 output
// accumulators.
constexpr int FA_BQ = 64, FA_BK = 64, FA_LD = 136;

AF_DEV void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

AF_DEV uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 16-byte global -> shared copy that bypasses registers; src_bytes 0 writes zeros (rows past the
// prompt: V must be 0 there, since a masked key's P of 0 times a non-finite V would not vanish)
AF_DEV void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
AF_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
AF_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int FA_SMEM = 2 * 2 * FA_BK * FA_LD * 2;   // K and V, two 64-key blocks in flight: 68 KB

__global__ void __launch_bounds__(128) attn_prefill_fa_kernel(AttnPrefillArgs a, const __half* qbuf) {
  constexpr int DH = 128;
  extern __shared__ __align__(16) unsigned char fa_smem[];
  __half (*Kb)[FA_BK][FA_LD] = reinterpret_cast<__half (*)[FA_BK][FA_LD]>(fa_smem);   // [2][64][136]
  __half (*Vb)[FA_BK][FA_LD] = Kb + 2;
  // the last query tiles see the most keys: they take the lowest block indices, so they start first
  const int h = blockIdx.x, q0 = (gridDim.y - 1 - blockIdx.y) * FA_BQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int G = a.H / a.KV, kvh = h / G;
  const int r0 = q0 + warp * 16 + g, r1 = r0 + 8;           // this lane's two query rows
  // Q fragments for the 8 k-steps of the head dimension
  uint32_t qf[8][4];
  const __half* qb = qbuf + (size_t)h * a.S * DH;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int c = ks * 16 + 2 * t;
    qf[ks][0] = r0 < a.S ? *reinterpret_cast<const uint32_t*>(qb + (size_t)r0 * DH + c) : 0u;
    qf[ks][1] = r1 < a.S ? *reinterpret_cast<const uint32_t*>(qb + (size_t)r1 * DH + c) : 0u;
    qf[ks][2] = r0 < a.S ? *reinterpret_cast<const uint32_t*>(qb + (size_t)r0 * DH + c + 8) : 0u;
    qf[ks][3] = r1 < a.S ? *reinterpret_cast<const uint32_t*>(qb + (size_t)r1 * DH + c + 8) : 0u;
  }
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n)
#pragma unroll
    for (int q = 0; q < 4; ++q) o[n][q] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const __half* kb = a.kc + (size_t)kvh * a.ldm * DH;
  const __half* vb = a.vc + (size_t)kvh * a.ldm * DH;
  const int last_q = min(q0 + FA_BQ, a.S) - 1;
  const int nblk = last_q / FA_BK + 1;
  // each thread copies the same 16-byte chunks of every block (i = tid + 128 k), so it can apply
  // the expansion factor to its own chunks once they land, before the block-wide barrier
  auto stage = [&](int blk) {
    const int j0 = blk * FA_BK, buf = blk & 1;
#pragma unroll
    for (int i = threadIdx.x; i < FA_BK * (DH / 8); i += 128) {
      const int r = i / (DH / 8), c = (i % (DH / 8)) * 8;
      const bool ok = j0 + r < a.S;
      const size_t row = ok ? (size_t)(j0 + r) : 0;
      cp_async16(&Kb[buf][r][c], kb + row * DH + c, ok ? 16 : 0);
      cp_async16(&Vb[buf][r][c], vb + row * DH + c, ok ? 16 : 0);
    }
    cp_async_commit();
  };
  stage(0);
  for (int blk = 0; blk < nblk; ++blk) {
    const int j0 = blk * FA_BK, buf = blk & 1;
    if (blk + 1 < nblk) {
      stage(blk + 1);                                    // its buffer was released at the end of blk - 1
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    if (a.expand) {
#pragma unroll
      for (int i = threadIdx.x; i < FA_BK * (DH / 8); i += 128) {
        const int r = i / (DH / 8), c = (i % (DH / 8)) * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          Kb[buf][r][c + e] = f2h(round_f16(a.kv_c * h2f(Kb[buf][r][c + e])));
          Vb[buf][r][c + e] = f2h(round_f16(a.kv_c * h2f(Vb[buf][r][c + e])));
        }
      }
    }
    __syncthreads();
    __half (*Ks)[FA_LD] = Kb[buf];
    __half (*Vs)[FA_LD] = Vb[buf];
    // S = Q K^T for this warp's 16 rows x 64 keys
    float sc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int q = 0; q < 4; ++q) sc[n][q] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&Ks[n * 8 + g][ks * 16 + 2 * t]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&Ks[n * 8 + g][ks * 16 + 8 + 2 * t]);
        mma_16816(sc[n], qf[ks], b0, b1);
      }
    }
    // scale, causal / length mask, block row maxima
    float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = j0 + n * 8 + 2 * t + e;
        const float s0 = (j <= r0 && j < a.S) ? sc[n][e] * a.scale : -INFINITY;
        const float s1 = (j <= r1 && j < a.S) ? sc[n][2 + e] * a.scale : -INFINITY;
        sc[n][e] = s0; sc[n][2 + e] = s1;
        bm0 = fmaxf(bm0, s0); bm1 = fmaxf(bm1, s1);
      }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
      bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
    }
    const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
    const float c0 = mn0 == -INFINITY ? 1.f : expf(m0 - mn0);
    const float c1 = mn1 == -INFINITY ? 1.f : expf(m1 - mn1);
    float ps0 = 0.f, ps1 = 0.f;
    uint32_t pf[4][4];                                   // P as fp16 A fragments, 4 k-steps of 16 keys
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p00 = sc[n][0] == -INFINITY ? 0.f : expf(sc[n][0] - mn0);
      const float p01 = sc[n][1] == -INFINITY ? 0.f : expf(sc[n][1] - mn0);
      const float p10 = sc[n][2] == -INFINITY ? 0.f : expf(sc[n][2] - mn1);
      const float p11 = sc[n][3] == -INFINITY ? 0.f : expf(sc[n][3] - mn1);
      ps0 += p00 + p01; ps1 += p10 + p11;
      pf[n >> 1][(n & 1) * 2 + 0] = pack_h2(p00, p01);
      pf[n >> 1][(n & 1) * 2 + 1] = pack_h2(p10, p11);
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      ps0 += __shfl_xor_sync(0xffffffffu, ps0, off);
      ps1 += __shfl_xor_sync(0xffffffffu, ps1, off);
    }
    l0 = l0 * c0 + ps0; l1 = l1 * c1 + ps1;
    m0 = mn0; m1 = mn1;
#pragma unroll
    for (int n = 0; n < 16; ++n) { o[n][0] *= c0; o[n][1] *= c0; o[n][2] *= c1; o[n][3] *= c1; }
    // O += P V: for key step ks, dh tiles n (8 columns each) via ldmatrix.trans of V rows
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int n = 0; n < 16; n += 2) {
        // matrices: (keys ks*16 + 0..7, dh n*8..), (keys +8..15, dh n*8..), (keys 0..7, dh (n+1)*8..), (keys 8..15, dh (n+1)*8..)
        const int mi = lane >> 3, rr = lane & 7;
        const int key = ks * 16 + (mi & 1) * 8 + rr;
        const int col = (n + (mi >> 1)) * 8;
        uint32_t b00, b01, b10, b11;
        ldsm_x4_trans((uint32_t)__cvta_generic_to_shared(&Vs[key][col]), b00, b01, b10, b11);
        // a k-step's A fragment: {a0, a1, a2, a3} = {P[g][2t..], P[g+8][2t..], P[g][8+2t..], P[g+8][8+2t..]}
        const uint32_t A[4] = {pf[ks][0], pf[ks][1], pf[ks][2], pf[ks][3]};
        mma_16816(o[n], A, b00, b01);
        mma_16816(o[n + 1], A, b10, b11);
      }
    }
    __syncthreads();                                     // every warp is done with this buffer
  }
  // normalise and store [S][H * DH] fp16
  const float il0 = l0 > 0.f ? 1.f / l0 : 0.f, il1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int c = h * DH + n * 8 + 2 * t;
    if (r0 < a.S)
      *reinterpret_cast<__half2*>(a.out + (size_t)r0 * a.H * DH + c) = __floats2half2_rn(o[n][0] * il0, o[n][1] * il0);
    if (r1 < a.S)
      *reinterpret_cast<__half2*>(a.out + (size_t)r1 * a.H * DH + c) = __floats2half2_rn(o[n][2] * il1, o[n][3] * il1);
  }
}

cudaError_t rope_kv_prefill_launch(const AttnPrefillArgs& a, __half* qbuf, cudaStream_t st) {
  if (a.S <= 0 || a.KV <= 0 || a.H % a.KV) return cudaErrorInvalidValue;
  dim3 grid(a.S, a.H + a.KV);
  switch (a.dh) {
    case 16: rope_kv_prefill_kernel<16><<<grid, 32, 0, st>>>(a, qbuf); break;
    case 32: rope_kv_prefill_kernel<32><<<grid, 32, 0, st>>>(a, qbuf); break;
    case 64: rope_kv_prefill_kernel<64><<<grid, 32, 0, st>>>(a, qbuf); break;
    case 128: rope_kv_prefill_kernel<128><<<grid, 32, 0, st>>>(a, qbuf); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t attn_prefill_with_q(const AttnPrefillArgs& a, const __half* qbuf, cudaStream_t st) {
  // AF_PREFILL_FA: 2 (default) the tcgen05 kernel where it applies, 1 the mma.sync kernel, 0 neither
  static const int fa = env_int("AF_PREFILL_FA", 2);
  if (fa >= 2 && attn_prefill_tc_ok(a)) return attn_prefill_tc_launch(a, qbuf, st);
  if (fa && a.dh == 128 && a.S >= 16) {
    static PerDeviceOnce attrs;
    const cudaError_t attr = attrs.run(
        [] { return cudaFuncSetAttribute(attn_prefill_fa_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM); });
    if (attr != cudaSuccess) return attr;
    attn_prefill_fa_kernel<<<dim3(a.H, (a.S + FA_BQ - 1) / FA_BQ), 128, FA_SMEM, st>>>(a, qbuf);
    return cudaGetLastError();
  }
  dim3 grid(a.H, (a.S + 3) / 4);
  switch (a.dh) {
    case 16: attn_prefill_kernel<16><<<grid, 128, 0, st>>>(a, qbuf); break;
    case 32: attn_prefill_kernel<32><<<grid, 128, 0, st>>>(a, qbuf); break;
    case 64: attn_prefill_kernel<64><<<grid, 128, 0, st>>>(a, qbuf); break;
    case 128: attn_prefill_kernel<128><<<grid, 128, 0, st>>>(a, qbuf); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace af
