// Shared device helpers for the B200 (sm_100a) decode/prefill kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define AF_DEV __device__ __forceinline__
#define AF_HD __host__ __device__ __forceinline__

// Error codes a kernel may record in the program's device error word (first error wins).
enum AfDevErr : int {
  AF_DEV_OK = 0,
  AF_DEV_BAD_TOKEN = 1,     // embedding index outside [0, vocab)
  AF_DEV_BAD_POS = 2,       // decode position outside [0, max_len)
  AF_DEV_WAIT_TIMEOUT = 3,  // a bounded spin-wait gave up
};

AF_DEV void af_set_err(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// Wall-clock bound of a device-side wait, on top of its iteration limit (a suspended
// `mbarrier.try_wait` or a slow poll can make an iteration limit minutes long): `spent()` turns
// true once the wait has lasted `limit_ns` (checked every 64 calls).
AF_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
struct SpinBudget {
  uint64_t t0 = 0;
  uint32_t n = 0;
  AF_DEV bool spent(uint64_t limit_ns = 2000000000ull) {
    if ((++n & 63) != 0) return false;
    const uint64_t t = global_ns();
    if (t0 == 0) { t0 = t; return false; }
    return t - t0 > limit_ns;
  }
};

// ---- host: per-device caches. Kernel attributes (cudaFuncSetAttribute) belong to the current
// device's context, and occupancy answers are per device too, so every cache of them is keyed by
// the device ordinal; one mutex per cache makes concurrent first calls from several host threads
// safe (later calls read the value behind an acquire load, without the lock).
#ifndef __CUDACC_RTC__
#include <atomic>
#include <mutex>
namespace af {
constexpr int kMaxDevices = 64;

inline int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) d = 0;
  return d;
}

// `fn()` (returning cudaError_t) runs once per device until it succeeds; a failure is returned and
// retried on the next call.
struct PerDeviceOnce {
  std::atomic<int> done[kMaxDevices] = {};
  std::mutex mu;
  template <class F> cudaError_t run(F&& fn) {
    const int d = current_device();
    if (done[d].load(std::memory_order_acquire)) return cudaSuccess;
    std::lock_guard<std::mutex> g(mu);
    if (done[d].load(std::memory_order_relaxed)) return cudaSuccess;
    const cudaError_t e = fn();
    if (e == cudaSuccess) done[d].store(1, std::memory_order_release);
    return e;
  }
};

// A value computed once per device and key slot (`fn()` returns it; 0 means "not computed").
template <int SLOTS> struct PerDeviceInt {
  std::atomic<int> v[kMaxDevices][SLOTS] = {};
  std::mutex mu;
  template <class F> int get(int slot, F&& fn) {
    const int d = current_device();
    int x = v[d][slot].load(std::memory_order_acquire);
    if (x) return x;
    std::lock_guard<std::mutex> g(mu);
    x = v[d][slot].load(std::memory_order_relaxed);
    if (!x) {
      x = fn();
      v[d][slot].store(x, std::memory_order_release);
    }
    return x;
  }
};

inline int device_attr(cudaDeviceAttr what, int fallback) {
  static PerDeviceInt<1> cache_sm, cache_smem_sm, cache_res, cache_optin;
  PerDeviceInt<1>* c = what == cudaDevAttrMultiProcessorCount ? &cache_sm
                     : what == cudaDevAttrMaxSharedMemoryPerMultiprocessor ? &cache_smem_sm
                     : what == cudaDevAttrReservedSharedMemoryPerBlock ? &cache_res
                     : what == cudaDevAttrMaxSharedMemoryPerBlockOptin ? &cache_optin : nullptr;
  auto q = [&] {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, what, current_device()) != cudaSuccess) { cudaGetLastError(); n = 0; }
    return n > 0 ? n : fallback;
  };
  return c ? c->get(0, q) : q();
}
}  // namespace af
#endif

// Programmatic dependent launch (sm_90+): wait for the preceding grid's memory to be visible /
// allow the next grid in the stream to start its prologue.
AF_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
AF_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Issue this thread's share (pieces idx, idx + n, ...) of an L2 prefetch spec; fire and forget.
template <class PF>
AF_DEV void l2_prefetch(const PF& pf, unsigned idx, unsigned n) {
  if (!pf.base) return;
  for (size_t j = idx; j * pf.stride < pf.bytes; j += n) {
    const size_t off = j * pf.stride;
    const size_t left = pf.bytes - off;
    const unsigned len = (unsigned)((left < pf.piece ? left : pf.piece) & ~(size_t)15);
    if (len)
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(pf.base + off), "r"(len) : "memory");
  }
}

// The same spec through the load/store units: one `prefetch.global.L2` per 128-byte line, lines
// idx, idx + n, ... of the spec's pieces (keeps the copy engine free for the issuing kernel's own
// bulk copies).
template <class PF>
AF_DEV void l2_prefetch_lines(const PF& pf, unsigned idx, unsigned n) {
  if (!pf.base) return;
  const size_t lines_per_piece = (pf.piece + 127) / 128;
  const size_t pieces = (pf.bytes + pf.stride - 1) / pf.stride;
  const size_t total = pieces * lines_per_piece;
  for (size_t i = idx; i < total; i += n) {
    const size_t off = (i / lines_per_piece) * pf.stride + (i % lines_per_piece) * 128;
    if (off >= pf.bytes) continue;
    if (pf.keep) asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(pf.base + off));
    else asm volatile("prefetch.global.L2 [%0];" ::"l"(pf.base + off));
  }
}

// ---- thread-block clusters: another CTA's shared memory, and the cluster-wide barrier
// address of `p` (this CTA's shared memory) in the shared window of cluster rank `rank`
AF_DEV uint32_t cluster_addr(const void* p, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"((uint32_t)__cvta_generic_to_shared(p)), "r"(rank));
  return r;
}

AF_DEV float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

AF_DEV float4 ld_cluster_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr)
               : "memory");
  return v;
}

// every thread of every CTA in the cluster, warps converged; release/acquire orders the
// shared-memory writes before it against the remote reads after it
AF_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// the same barrier for threads that may arrive from divergent code
AF_DEV void cluster_sync_any() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// 16-byte streaming load that bypasses L1 (weights are read once per decode step).
AF_DEV uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// Activations written by the preceding kernel. With programmatic dependent launch a kernel starts
// while its producer is still writing, so its data must not come through the non-coherent
// (read-only) path, whose L1 lines may predate the producer's stores: load at L2 (.cg) instead.
AF_DEV uint4 ld_act_v4(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}

// Four signed int8 lanes of `w` -> four exact floats. Each byte b is biased to b+128, placed in
// the low mantissa byte of 2^23 (0x4B000000) with a byte permute, and the bias 2^23+128 is
// subtracted: exact for every int8 value, two integer/float ops per element and no I2F.
AF_DEV void i8x4_to_f32(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
  const uint32_t u = w ^ 0x80808080u;
  const float bias = 8388736.0f;  // 2^23 + 128
  f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - bias;
  f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - bias;
  f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - bias;
  f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - bias;
}

// Eight unsigned 4-bit codes (low nibble first) minus 8 -> eight exact floats.
AF_DEV void u4x8_to_f32(uint32_t w, float* f) {
  // nibble k of w holds code for element k; value = code - 8
#pragma unroll
  for (int k = 0; k < 8; ++k) f[k] = (float)((int)((w >> (4 * k)) & 0xFu) - 8);
}

AF_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

AF_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

AF_DEV float h2f(__half h) { return __half2float(h); }
AF_DEV __half f2h(float f) { return __float2half_rn(f); }
AF_DEV float round_f16(float f) { return __half2float(__float2half_rn(f)); }

// Eight fp16 packed in a uint4 -> floats.
AF_DEV void h8_to_f32(const uint4& v, float* f) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

AF_DEV float silu_f(float g) { return g / (1.0f + expf(-g)); }
