// Tensor-parallel plumbing: an NCCL communicator per rank (NCCL is opened at run time, so a
// single-GPU process never needs it), the collectives a sharded decode/prefill plan issues on the
// program's stream (captured into its CUDA graph), and the cross-rank greedy argmax of a
// vocabulary-parallel lm_head.
//
// Sharding (column-parallel qkv and gate|up, row-parallel o and down, vocab-parallel head) follows
// the Megatron layout; the only exchanges per layer are two all-reduces of the fp32 residual
// update [NB, D] and, per token, an all-gather of each rank's (best logit, index) pair.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>

#include "af_common.cuh"
#include "af_kernels.h"
#include "../../include/af_cuda.h"

namespace af {
void set_error_public(const std::string& msg);

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

// Bind the NCCL entry points, preferring a library the process already loaded (e.g. the one torch
// brought in) so that one NCCL serves everything in the process.
bool nccl_load(std::string& why) {
  std::lock_guard<std::mutex> lock(g_nccl_mu);
  if (g_nccl.ok) return true;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) { why = std::string("cannot load NCCL: ") + dlerror(); return false; }
  g_nccl.get_unique_id = reinterpret_cast<decltype(g_nccl.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
  g_nccl.comm_init_rank = reinterpret_cast<decltype(g_nccl.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
  g_nccl.comm_destroy = reinterpret_cast<decltype(g_nccl.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
  g_nccl.all_reduce = reinterpret_cast<decltype(g_nccl.all_reduce)>(dlsym(h, "ncclAllReduce"));
  g_nccl.all_gather = reinterpret_cast<decltype(g_nccl.all_gather)>(dlsym(h, "ncclAllGather"));
  g_nccl.error_string = reinterpret_cast<decltype(g_nccl.error_string)>(dlsym(h, "ncclGetErrorString"));
  g_nccl.ok = g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.comm_destroy && g_nccl.all_reduce &&
              g_nccl.all_gather && g_nccl.error_string;
  if (!g_nccl.ok) why = "NCCL library lacks an expected entry point";
  return g_nccl.ok;
}

}  // namespace

cudaError_t add_f32_launch(float* y, const float* x, size_t n, cudaStream_t st);

// ---- one-shot all-reduce over NVLink peer memory (optional; set up by af_comm_p2p_open)
//
// Every rank owns one exchange buffer, mapped into every peer's address space through CUDA IPC:
//   [2 sets][T source slots][cap] u64 words   value bits (low 32) | call epoch (high 32)
//   u32                                       this rank's epoch counter
// Call e (all ranks issue the same sequence of all-reduces) uses set e & 1. Each rank stores word
// i = (partial[i], e) into slot `rank` of every rank's buffer (its own included) with plain 8-byte
// peer stores, then polls its own buffer until every slot's word i carries epoch e and sums the T
// values in rank order, so every rank computes the same bits. A word is one aligned 8-byte store,
// so its value and epoch become visible together: no fence and no separate flag round trip (the
// low-latency protocol of NCCL's LL transport). Two sets make reuse safe: a rank writes set s again
// (call e + 2) only after it has read every peer's call e + 1 words, which each peer stores only
// after finishing its reads of call e. Every poll is bounded; a timeout is recorded in the error word.
constexpr int P2P_MAX_RANKS = 8;
constexpr long long P2P_SPIN = 1ll << 22;             // bounded polls per word (well above any wait)

struct P2pPeers {
  char* base[P2P_MAX_RANKS];                          // every rank's exchange buffer (own included)
};

struct Comm {
  ncclComm_t nccl = nullptr;
  int nranks = 1, rank = 0, device = 0;
  // peer-memory all-reduce
  char* xbuf = nullptr;                               // this rank's exchange buffer
  size_t cap = 0;                                     // words per slot
  size_t xbytes = 0;
  char* peer[P2P_MAX_RANKS] = {};                     // opened IPC mappings (peer[rank] = xbuf)
  bool p2p = false;
};

AF_HD size_t p2p_data_off(int set, int src, int T, size_t cap) { return ((size_t)set * T + src) * cap * 8; }
AF_HD size_t p2p_epoch_off(int T, size_t cap) { return (size_t)2 * T * cap * 8; }
AF_HD size_t p2p_bytes(int T, size_t cap) { return p2p_epoch_off(T, cap) + 16; }

// The words are split over the grid's CTAs (each CTA pushes and polls its own share); every CTA reads
// the epoch when it starts, and the last CTA to finish (a ticket next to the epoch) stores the new one,
// so no CTA of this call can see it early.
__global__ void __launch_bounds__(256) p2p_all_reduce_kernel(P2pPeers peers, int T, int rank, size_t cap,
                                                              const float* src, float* dst, float* addto, int n,
                                                              int* err) {
  char* mine = peers.base[rank];
  unsigned* epoch = reinterpret_cast<unsigned*>(mine + p2p_epoch_off(T, cap));
  unsigned* ticket = epoch + 1;
  pdl_wait();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(epoch) + 1u;
  const int set = (int)(e & 1u);
  const int i0 = blockIdx.x * blockDim.x + threadIdx.x, step = gridDim.x * blockDim.x;
  // push: word i of this rank's slot on every rank
  for (int i = i0; i < n; i += step) {
    const unsigned long long w = ((unsigned long long)e << 32) | __float_as_uint(__ldcg(src + i));
    for (int p = 0; p < T; ++p) {
      unsigned long long* d = reinterpret_cast<unsigned long long*>(peers.base[p] + p2p_data_off(set, rank, T, cap)) + i;
      asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(d), "l"(w) : "memory");
    }
  }
  // reduce: every rank's word i, in rank order, once it carries this call's epoch
  bool late = false;
  for (int i = i0; i < n; i += step) {
    float acc = 0.f;
    for (int s = 0; s < T; ++s) {
      const unsigned long long* w = reinterpret_cast<const unsigned long long*>(mine + p2p_data_off(set, s, T, cap)) + i;
      unsigned long long v = 0;
      bool in = false;
      for (long long k = 0; k < P2P_SPIN && !in; ++k) {
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(w) : "memory");
        in = (unsigned)(v >> 32) == e;
      }
      late |= !in;
      acc += __uint_as_float((unsigned)(v & 0xffffffffull));
    }
    if (addto) addto[i] += acc;        // the residual update, as the separate add would do it
    else dst[i] = acc;
  }
  if (late) af_set_err(err, AF_DEV_WAIT_TIMEOUT);
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(ticket, 1u) == gridDim.x - 1) {
    *ticket = 0u;                      // every CTA of this call has read the epoch: the last one moves it
    *reinterpret_cast<volatile unsigned*>(epoch) = e;
  }
  pdl_trigger();
}

// CTAs of the peer all-reduce for n words: 256 threads each, up to 32 (one word per thread below that)
static int p2p_ctas(size_t n) {
  const size_t c = (n + 255) / 256;
  return c < 1 ? 1 : (c > 32 ? 32 : (int)c);
}

cudaError_t comm_all_reduce_f32(void* comm, const float* src, float* dst, size_t n, cudaStream_t st, std::string& why,
                                int* err, float* addto, bool pdl) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) { why = "no communicator"; return cudaErrorInvalidValue; }
  if (c->p2p && n <= c->cap) {
    P2pPeers peers;
    for (int r = 0; r < P2P_MAX_RANKS; ++r) peers.base[r] = r < c->nranks ? c->peer[r] : nullptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p2p_ctas(n));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, p2p_all_reduce_kernel, peers, c->nranks, c->rank, c->cap, src, dst, addto, (int)n,
                              err);
  }
  if (!g_nccl.ok || !c->nccl) { why = "no communicator"; return cudaErrorInvalidValue; }
  const ncclResult_t r = g_nccl.all_reduce(src, dst, n, ncclFloat32, ncclSum, c->nccl, st);
  if (r != ncclSuccess) { why = std::string("ncclAllReduce: ") + g_nccl.error_string(r); return cudaErrorUnknown; }
  return addto ? add_f32_launch(addto, dst, n, st) : cudaSuccess;
}

// The residual all-reduce fused with the RMSNorm that reads the residual next (a tensor-parallel
// decode step's o / down projections): h += the ranks' partials summed in rank order (the protocol
// of p2p_all_reduce_kernel), then out = fp16(h / max(|h|, floor) * g) per row with the rmsnorm
// kernel's formula. One launch and one boundary instead of two; every rank computes the same bits.
__global__ void __launch_bounds__(1024) p2p_all_reduce_rms_kernel(P2pPeers peers, int T, int rank, size_t cap,
                                                                   const float* src, float* h, int NB, int D,
                                                                   const __half* g, float floor, __half* out, int* err) {
  char* mine = peers.base[rank];
  unsigned* epoch = reinterpret_cast<unsigned*>(mine + p2p_epoch_off(T, cap));
  __shared__ float red[32];
  pdl_wait();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(epoch) + 1u;
  const int set = (int)(e & 1u);
  const int n = NB * D;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long w = ((unsigned long long)e << 32) | __float_as_uint(__ldcg(src + i));
    for (int p = 0; p < T; ++p) {
      unsigned long long* d = reinterpret_cast<unsigned long long*>(peers.base[p] + p2p_data_off(set, rank, T, cap)) + i;
      asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(d), "l"(w) : "memory");
    }
  }
  bool late = false;
  for (int b = 0; b < NB; ++b) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      const int idx = b * D + i;
      float acc = 0.f;
      for (int s = 0; s < T; ++s) {
        const unsigned long long* w = reinterpret_cast<const unsigned long long*>(mine + p2p_data_off(set, s, T, cap)) + idx;
        unsigned long long v = 0;
        bool in = false;
        for (long long k = 0; k < P2P_SPIN && !in; ++k) {
          asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(w) : "memory");
          in = (unsigned)(v >> 32) == e;
        }
        late |= !in;
        acc += __uint_as_float((unsigned)(v & 0xffffffffull));
      }
      const float hv = h[idx] + acc;
      h[idx] = hv;
      ss = fmaf(hv, hv, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int wv = 0; wv < (int)(blockDim.x >> 5); ++wv) tot += red[wv];
    const float sn = fmaxf(sqrtf(tot), floor);
    for (int i = threadIdx.x; i < D; i += blockDim.x)      // the h values this thread just wrote
      out[(size_t)b * D + i] = f2h(__fdiv_rn(h[(size_t)b * D + i], sn) * h2f(g[i]));
    __syncthreads();                                       // red is reused by the next row
  }
  if (late) af_set_err(err, AF_DEV_WAIT_TIMEOUT);
  __syncthreads();
  if (threadIdx.x == 0) *reinterpret_cast<volatile unsigned*>(epoch) = e;
  pdl_trigger();
}

cudaError_t comm_all_reduce_rms_f32(void* comm, const float* src, float* tmp, float* h, int NB, int D, const __half* g,
                                    float floor, __half* out, cudaStream_t st, std::string& why, int* err, bool pdl) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c) { why = "no communicator"; return cudaErrorInvalidValue; }
  const size_t n = (size_t)NB * D;
  if (c->p2p && n <= c->cap) {
    P2pPeers peers;
    for (int r = 0; r < P2P_MAX_RANKS; ++r) peers.base[r] = r < c->nranks ? c->peer[r] : nullptr;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(D >= 1024 ? 1024 : (D + 31) / 32 * 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, p2p_all_reduce_rms_kernel, peers, c->nranks, c->rank, c->cap, src, h, NB, D, g,
                              floor, out, err);
  }
  // NCCL: the all-reduce (added into h), then the norm
  cudaError_t e = comm_all_reduce_f32(comm, src, tmp, n, st, why, err, h, false);
  if (e != cudaSuccess) return e;
  return rmsnorm_launch(h, 0, D, g, floor, out, D, NB, D, st, false, L2Pf());
}

cudaError_t comm_all_gather_i32(void* comm, const int* src, int* dst, size_t n, cudaStream_t st, std::string& why) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || !g_nccl.ok) { why = "no communicator"; return cudaErrorInvalidValue; }
  const ncclResult_t r = g_nccl.all_gather(src, dst, n, ncclInt32, c->nccl, st);
  if (r != ncclSuccess) { why = std::string("ncclAllGather: ") + g_nccl.error_string(r); return cudaErrorUnknown; }
  return cudaSuccess;
}

int comm_size(void* comm) { return comm ? static_cast<Comm*>(comm)->nranks : 1; }
int comm_rank(void* comm) { return comm ? static_cast<Comm*>(comm)->rank : 0; }

// gathered[r] = [NB values (fp32 bits) | NB vocabulary indices] of rank r: the greedy token is the
// best value over ranks, ties to the lowest index (as the single-device argmax); then the position
// advance and token history of the single-device head.
__global__ void tp_argmax_kernel(const int* gathered, int T, int NB, int* tok_out, int* pos_adv, int* hist,
                                 int hist_ld) {
  const int b = threadIdx.x;
  if (b >= NB) return;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int r = 0; r < T; ++r) {
    const float v = __int_as_float(__ldcg(gathered + (size_t)r * 2 * NB + b));
    const int ix = __ldcg(gathered + (size_t)r * 2 * NB + NB + b);
    if (v > best || (v == best && ix < bi) || bi == 0x7fffffff) { best = v; bi = ix; }
  }
  tok_out[b] = bi;
  if (pos_adv) {
    const int p = pos_adv[b];
    if (hist && p >= 0 && p < hist_ld) hist[(size_t)b * hist_ld + p] = bi;
    pos_adv[b] = p + 1;
  }
}

cudaError_t tp_argmax_launch(const int* gathered, int T, int NB, int* tok_out, int* pos_adv, int* hist, int hist_ld,
                             cudaStream_t st) {
  if (NB < 1 || NB > 1024 || T < 1) return cudaErrorInvalidValue;
  tp_argmax_kernel<<<1, NB <= 32 ? 32 : (NB + 31) / 32 * 32, 0, st>>>(gathered, T, NB, tok_out, pos_adv, hist, hist_ld);
  return cudaGetLastError();
}

// y[i] += x[i] (the residual update of ranks that keep a separate partial)
__global__ void add_f32_kernel(float* y, const float* x, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    y[i] += __ldcg(x + i);
}

cudaError_t add_f32_launch(float* y, const float* x, size_t n, cudaStream_t st) {
  unsigned blocks = (unsigned)((n + 255) / 256);
  if (blocks > 1024) blocks = 1024;
  if (!blocks) return cudaSuccess;
  add_f32_kernel<<<blocks, 256, 0, st>>>(y, x, n);
  return cudaGetLastError();
}

}  // namespace af

extern "C" {

int af_comm_unique_id(void* out, size_t bytes) {
  std::string why;
  if (!out || bytes < NCCL_UNIQUE_ID_BYTES) { af::set_error_public("af_comm_unique_id: buffer too small"); return -1; }
  if (!af::nccl_load(why)) { af::set_error_public(why); return -1; }
  ncclUniqueId id;
  const ncclResult_t r = af::g_nccl.get_unique_id(&id);
  if (r != ncclSuccess) { af::set_error_public(std::string("ncclGetUniqueId: ") + af::g_nccl.error_string(r)); return -1; }
  memcpy(out, &id, NCCL_UNIQUE_ID_BYTES);
  return 0;
}

int af_comm_init(const void* id, int nranks, int rank, int device, void** comm) {
  std::string why;
  if (!id || !comm || nranks < 1 || rank < 0 || rank >= nranks) { af::set_error_public("af_comm_init: bad arguments"); return -1; }
  if (!af::nccl_load(why)) { af::set_error_public(why); return -1; }
  int prev = 0;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) { af::set_error_public("af_comm_init: bad device"); return -1; }
  af::Comm* c = new af::Comm();
  c->nranks = nranks; c->rank = rank; c->device = device;
  ncclUniqueId uid;
  memcpy(&uid, id, NCCL_UNIQUE_ID_BYTES);
  const ncclResult_t r = af::g_nccl.comm_init_rank(&c->nccl, nranks, uid, rank);
  cudaSetDevice(prev);
  if (r != ncclSuccess) {
    af::set_error_public(std::string("ncclCommInitRank: ") + af::g_nccl.error_string(r));
    delete c;
    return -1;
  }
  *comm = c;
  return 0;
}

void af_comm_destroy(void* comm) {
  af::Comm* c = static_cast<af::Comm*>(comm);
  if (!c) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < c->nranks && r < af::P2P_MAX_RANKS; ++r)
    if (c->peer[r] && r != c->rank) cudaIpcCloseMemHandle(c->peer[r]);
  if (c->xbuf) cudaFree(c->xbuf);
  cudaSetDevice(prev);
  if (c->nccl && af::g_nccl.ok) af::g_nccl.comm_destroy(c->nccl);
  delete c;
}

int af_comm_p2p_handle(void* comm, size_t cap_floats, void* handle, size_t bytes) {
  af::Comm* c = static_cast<af::Comm*>(comm);
  if (!c || !handle || bytes < sizeof(cudaIpcMemHandle_t) || cap_floats == 0 || c->nranks > af::P2P_MAX_RANKS ||
      c->xbuf) {
    af::set_error_public("af_comm_p2p_handle: bad arguments");
    return -1;
  }
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  c->cap = (cap_floats + 3) / 4 * 4;                 // words per slot
  c->xbytes = af::p2p_bytes(c->nranks, c->cap);
  cudaError_t e = cudaMalloc(&c->xbuf, c->xbytes);
  if (e == cudaSuccess) e = cudaMemset(c->xbuf, 0, c->xbytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), c->xbuf);
  cudaDeviceSynchronize();
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    af::set_error_public(std::string("af_comm_p2p_handle: ") + cudaGetErrorString(e));
    if (c->xbuf) cudaFree(c->xbuf);
    c->xbuf = nullptr;
    return -1;
  }
  return 0;
}

void af_comm_p2p_disable(void* comm) {
  af::Comm* c = static_cast<af::Comm*>(comm);
  if (c) c->p2p = false;
}

int af_comm_p2p_open(void* comm, const void* handles, size_t bytes_each) {
  af::Comm* c = static_cast<af::Comm*>(comm);
  if (!c || !handles || bytes_each < sizeof(cudaIpcMemHandle_t) || !c->xbuf) {
    af::set_error_public("af_comm_p2p_open: bad arguments (call af_comm_p2p_handle first)");
    return -1;
  }
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  for (int r = 0; r < c->nranks; ++r) {
    if (r == c->rank) { c->peer[r] = c->xbuf; continue; }
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const char*>(handles) + (size_t)r * bytes_each, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      cudaGetLastError();
      for (int q = 0; q < r; ++q)
        if (q != c->rank && c->peer[q]) { cudaIpcCloseMemHandle(c->peer[q]); c->peer[q] = nullptr; }
      cudaSetDevice(prev);
      af::set_error_public(std::string("af_comm_p2p_open: ") + cudaGetErrorString(e));
      return -1;
    }
    c->peer[r] = static_cast<char*>(p);
  }
  c->p2p = true;
  cudaSetDevice(prev);
  return 0;
}

}  // extern "C"
