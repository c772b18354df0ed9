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

struct Comm {
  ncclComm_t nccl = nullptr;
  int nranks = 1, rank = 0, device = 0;
};

cudaError_t comm_all_reduce_f32(void* comm, const float* src, float* dst, size_t n, cudaStream_t st, std::string& why) {
  Comm* c = static_cast<Comm*>(comm);
  if (!c || !g_nccl.ok) { why = "no communicator"; return cudaErrorInvalidValue; }
  const ncclResult_t r = g_nccl.all_reduce(src, dst, n, ncclFloat32, ncclSum, c->nccl, st);
  if (r != ncclSuccess) { why = std::string("ncclAllReduce: ") + g_nccl.error_string(r); return cudaErrorUnknown; }
  return cudaSuccess;
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
  if (c->nccl && af::g_nccl.ok) af::g_nccl.comm_destroy(c->nccl);
  delete c;
}

}  // extern "C"
