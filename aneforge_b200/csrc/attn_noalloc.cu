// af_attn_decode_noalloc: the decode-attention entry point for callers that cannot allocate device
// memory.
//
// af_attn_decode needs a scratch buffer from its caller (split-K partial sums + one ticket counter
// per (sequence, kv head)). Some callers have no way to provide one: code running inside a host
// framework that owns every device allocation and hands out only tensor pointers, hooks that run
// while a memory pool is locked, or plug-ins loaded into a process whose allocator must not be
// touched. This variant takes the scratch from a fixed array that lives in the library itself, so a
// call needs nothing but its inputs and outputs.
//
// Limits and sharing rules:
//  * the array is AF_ATTN_NOALLOC_SCRATCH_BYTES (2 MiB) per GPU and stays resident on every GPU that
//    loads the library until the process exits; a shape whose splits merge through global scratch
//    and need more is rejected (rc -1, reason in af_last_error()) before anything is launched.
//    Shapes whose splits merge inside a thread-block cluster (at most 16 splits) touch no scratch
//    and have no size limit here;
//  * every call on a GPU uses the same array and leaves its contents behind; when a call merges
//    through the array its ticket counters are cleared on the caller's stream before the launch,
//    the partial sums need no clearing;
//  * two calls whose kernels overlap on the GPU (different streams without ordering) race on the
//    array and produce wrong results - order them on one stream or with events;
//  * the first call on each device looks the array's device address up (cudaGetSymbolAddress with
//    that device current) and caches it: make that first call before any stream capture begins;
//  * the cached address is not refreshed after cudaDeviceReset (which may reload the library's
//    module at another address): do not use this entry point across a device reset.
#include <mutex>
#include <string>

#include "af_common.cuh"
#include "af_kernels.h"
#include "../../include/af_cuda.h"

namespace af {
void set_error_public(const std::string& msg);
}

namespace {

constexpr size_t kScratchBytes = AF_ATTN_NOALLOC_SCRATCH_BYTES;
constexpr size_t kCounterBytes = 16384;   // ticket counters first, then the partial sums
constexpr int kMaxDevices = af::kMaxDevices;

// The scratch itself. In host code this name is only a stand-in for the symbol: its device address
// comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

// Device address of g_attn_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    af::set_error_public("af_attn_decode_noalloc: no usable current CUDA device");
    return -1;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || !p) {
      af::set_error_public(std::string("af_attn_decode_noalloc: cudaGetSymbolAddress failed: ") +
                           cudaGetErrorString(e));
      cudaGetLastError();
      return -1;
    }
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return 0;
}

}  // namespace

extern "C" {

size_t af_attn_decode_noalloc_max_bytes(void) { return kScratchBytes; }

int af_attn_decode_noalloc(const float* qkv, int ld_qkv, uint16_t* kc, uint16_t* vc, const int* pos,
                           const uint16_t* cos_t, const uint16_t* sin_t, uint16_t* out, int ld_out, int nb, int h,
                           int kv, int dh, int m, int n_split, float scale, float kv_c, int expand, int* err,
                           void* stream) {
  if (nb < 1 || kv <= 0 || h % kv || n_split < 1) {
    af::set_error_public("af_attn_decode_noalloc: bad shape (need nb >= 1, kv > 0, h % kv == 0, n_split >= 1)");
    return -1;
  }
  af::AttnDecodeArgs a;
  a.qkv = qkv; a.ld_qkv = ld_qkv;
  a.kc = reinterpret_cast<__half*>(kc); a.vc = reinterpret_cast<__half*>(vc);
  a.pos = pos;
  a.cos_t = reinterpret_cast<const __half*>(cos_t); a.sin_t = reinterpret_cast<const __half*>(sin_t);
  a.out = reinterpret_cast<__half*>(out); a.ld_out = ld_out;
  a.NB = nb; a.H = h; a.KV = kv; a.dh = dh; a.M = m; a.n_split = n_split;
  a.scale = scale; a.kv_c = kv_c; a.expand = expand; a.err = err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool merges_in_scratch = af::attn_decode_uses_scratch(a);
  const size_t counters = (size_t)nb * kv * sizeof(int);
  const size_t partial = 4 * af::attn_decode_scratch_floats(nb, kv, n_split, h / kv, dh);
  if (merges_in_scratch && (counters > kCounterBytes || kCounterBytes + partial > kScratchBytes)) {
    af::set_error_public("af_attn_decode_noalloc: this shape needs " + std::to_string(kCounterBytes + partial) +
                         " bytes of scratch; the built-in maximum is " + std::to_string(kScratchBytes) +
                         " (use af_attn_decode with caller scratch, or fewer splits / sequences)");
    return -1;
  }
  if (n_split > 1) {
    void* base = nullptr;
    if (scratch_address(&base) != 0) return -1;
    if (merges_in_scratch) {
      // the tickets must start at zero whatever an earlier call left behind
      cudaError_t e = cudaMemsetAsync(base, 0, counters, st);
      if (e != cudaSuccess) {
        af::set_error_public(std::string("af_attn_decode_noalloc: clearing the tickets failed: ") +
                             cudaGetErrorString(e));
        cudaGetLastError();
        return -1;
      }
    }
    a.counters = static_cast<int*>(base);
    a.part = reinterpret_cast<float*>(static_cast<char*>(base) + kCounterBytes);
  }
  const cudaError_t e = af::attn_decode_launch(a, st, false);
  if (e != cudaSuccess) {
    af::set_error_public(std::string("af_attn_decode_noalloc: ") + cudaGetErrorString(e));
    cudaGetLastError();
    return -1;
  }
  return 0;
}

}  // extern "C"
