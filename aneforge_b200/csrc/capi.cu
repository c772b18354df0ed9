// Kernel-level C ABI: each entry takes device pointers and a cudaStream_t (as void*), launches one
// fused kernel and returns 0, or -1 with the reason in af_last_error(). These are the building
// blocks the program plans sequence; tests and the model loader call them directly.
#include <string>

#include "af_common.cuh"
#include "af_kernels.h"
#include "../../include/af_cuda.h"

namespace af {
void set_error_public(const std::string& msg);
}

static int rc_of(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return 0;
  std::string m = std::string(what) + ": " + cudaGetErrorString(e);
  af::set_error_public(m);
  cudaGetLastError();
  return -1;
}

extern "C" {

int af_quantize_per_row_i8(const void* src, int src_f16, int n, int k, int8_t* codes, uint16_t* scales,
                           void* stream) {
  return rc_of(af::quantize_rows_i8(src, src_f16, n, k, codes, reinterpret_cast<__half*>(scales),
                                    static_cast<cudaStream_t>(stream)),
               "quantize_per_row_i8");
}

int af_quantize_g32_i4(const void* src, int src_f16, int n, int k, uint8_t* packed, uint16_t* scales,
                       void* stream) {
  return rc_of(af::quantize_g32_i4(src, src_f16, n, k, packed, reinterpret_cast<__half*>(scales),
                                   static_cast<cudaStream_t>(stream)),
               "quantize_g32_i4");
}

int af_gemv(int wf, int epi, const uint16_t* x, int ldx, const void* w, const uint16_t* scales,
            const uint16_t* bias, void* y, int ldy, int nb, int n, int k, void* stream) {
  if (epi == af::EPI_ARGMAX) return rc_of(cudaErrorInvalidValue, "af_gemv: use af_lm_head_argmax");
  af::GemvArgs a;
  a.wf = wf; a.epi = epi;
  a.x = reinterpret_cast<const __half*>(x); a.ldx = ldx;
  a.w = w;
  if (wf == af::W_I8) a.scale = reinterpret_cast<const __half*>(scales);
  if (wf == af::W_I4G32) a.gscale = reinterpret_cast<const __half*>(scales);
  a.bias = reinterpret_cast<const __half*>(bias);
  a.y = y; a.ldy = ldy; a.NB = nb; a.N = n; a.K = k;
  return rc_of(af::gemv_launch(a, static_cast<cudaStream_t>(stream), false), "af_gemv");
}

// scratch layout: [counters, padded to 256 B][values: slots floats][indices: slots ints]
static void argmax_layout(int wf, int n, int k, int nb, size_t* slots, size_t* cnt_bytes) {
  size_t counters = 0;
  af::gemv_argmax_scratch(wf, n, k, nb, slots, &counters);
  *cnt_bytes = ((4 * counters + 255) / 256) * 256;
}

int af_lm_head_argmax_scratch(int wf, int n, int k, int nb, size_t* bytes) {
  if (!bytes) return -1;
  size_t slots = 0, cb = 0;
  argmax_layout(wf, n, k, nb, &slots, &cb);
  *bytes = cb + 8 * slots;
  return 0;
}

int af_lm_head_argmax(int wf, const uint16_t* x, int ldx, const void* w, const uint16_t* scales, float* logits,
                      int nb, int n, int k, int* tok_out, int* pos_advance, void* scratch, size_t scratch_bytes,
                      void* stream) {
  size_t need = 0;
  af_lm_head_argmax_scratch(wf, n, k, nb, &need);
  if (!scratch || scratch_bytes < need) return rc_of(cudaErrorInvalidValue, "af_lm_head_argmax: scratch too small");
  size_t slots = 0, cb = 0;
  argmax_layout(wf, n, k, nb, &slots, &cb);
  af::GemvArgs a;
  a.wf = wf; a.epi = af::EPI_ARGMAX;
  a.x = reinterpret_cast<const __half*>(x); a.ldx = ldx;
  a.w = w;
  if (wf == af::W_I8) a.scale = reinterpret_cast<const __half*>(scales);
  if (wf == af::W_I4G32) return rc_of(cudaErrorInvalidValue, "af_lm_head_argmax: int4 head unsupported");
  a.y = logits; a.ldy = n; a.NB = nb; a.N = n; a.K = k;
  char* s = static_cast<char*>(scratch);
  a.am_count = reinterpret_cast<int*>(s);
  a.am_val = reinterpret_cast<float*>(s + cb);
  a.am_idx = reinterpret_cast<int*>(s + cb + 4 * slots);
  a.am_grid_cap = af::gemv_argmax_ctas(wf, n, k, nb);
  a.tok_out = tok_out;
  a.pos_adv = pos_advance;
  return rc_of(af::gemv_launch(a, static_cast<cudaStream_t>(stream), false), "af_lm_head_argmax");
}

int af_pack_i8_tiles(const int8_t* codes, int n, int k, uint8_t* tiles, void* stream) {
  return rc_of(af::pack_i8_tiles(codes, n, k, tiles, static_cast<cudaStream_t>(stream)), "af_pack_i8_tiles");
}

size_t af_pack_i8_tiles_bytes(int n, int k) { return af::pack_i8_tiles_bytes(n, k); }

size_t af_gemv_tc_scratch_bytes(int n, int k, int nb) { return af::gemv_tc_scratch_bytes(n, k, nb); }
size_t af_gemv_chain_scratch_bytes(int njobs, const int* n, const int* k, int nb, int wf) {
  if (njobs < 1 || njobs > af::CHAIN_MAX_JOBS || !n || !k || nb < 1 || nb > 16 ||
      (wf != af::W_I8 && wf != af::W_I4G32))
    return 0;
  af::GemvChainArgs a;
  a.njobs = njobs;
  a.NB = nb;
  a.wf = wf;
  for (int j = 0; j < njobs; ++j) {
    if (n[j] <= 0 || k[j] <= 0 || k[j] % 32) return 0;
    a.job[j].N = n[j];
    a.job[j].K = k[j];
  }
  return af::gemv_chain_scratch_bytes(a);
}
int af_gemv_tc_grid(int n, int k, int nb, int epi, int wf, int* grid, int* csize) {
  if (!grid || !csize || n <= 0 || k <= 0 || nb < 1 || (wf != af::W_I8 && wf != af::W_I4G32) || epi < 0 ||
      epi > af::EPI_SWIGLU)
    return -1;
  af::gemv_tc_grid(n, k, nb > 16 ? 16 : nb, epi, wf == af::W_I4G32, grid, csize);
  return 0;
}

int af_gemv_tc(int epi, const uint16_t* x, int ldx, const void* tiles, const uint16_t* scales, const uint16_t* bias,
               void* y, int ldy, int nb, int n, int k, void* scratch, size_t scratch_bytes, void* stream) {
  af::GemvTcArgs a;
  a.epi = epi;
  a.x = reinterpret_cast<const __half*>(x); a.ldx = ldx;
  a.w = tiles; a.scale = reinterpret_cast<const __half*>(scales); a.bias = reinterpret_cast<const __half*>(bias);
  a.y = y; a.ldy = ldy; a.NB = nb; a.N = n; a.K = k;
  a.scratch = scratch; a.scratch_bytes = scratch_bytes;
  return rc_of(af::gemv_tc_launch(a, static_cast<cudaStream_t>(stream), false), "af_gemv_tc");
}

size_t af_pack_i4_tiles_bytes(int n, int k) { return k % 32 ? 0 : af::pack_i4_tiles_bytes(n, k); }

int af_pack_i4_tiles(const uint8_t* packed, const uint16_t* scales, int n, int k, uint8_t* tiles, void* stream) {
  return rc_of(af::pack_i4_tiles(packed, reinterpret_cast<const __half*>(scales), n, k, tiles,
                                 static_cast<cudaStream_t>(stream)), "af_pack_i4_tiles");
}

int af_gemv_tc_i4(int epi, const uint16_t* x, int ldx, const void* tiles, const uint16_t* bias, void* y, int ldy,
                  int nb, int n, int k, void* scratch, size_t scratch_bytes, void* stream) {
  af::GemvTcArgs a;
  a.wf = af::W_I4G32;
  a.epi = epi;
  a.x = reinterpret_cast<const __half*>(x); a.ldx = ldx;
  a.w = tiles; a.bias = reinterpret_cast<const __half*>(bias);
  a.y = y; a.ldy = ldy; a.NB = nb; a.N = n; a.K = k;
  a.scratch = scratch; a.scratch_bytes = scratch_bytes;
  return rc_of(af::gemv_tc_launch(a, static_cast<cudaStream_t>(stream), false), "af_gemv_tc_i4");
}


int af_gemv_tc_expert(int wf, int epi, const uint16_t* x, int ldx, const void* tiles, const uint16_t* scales,
                      void* y, int ldy, int nb, int n, int k, const int* sel, int slot, int fixed_e, long long w_stride,
                      int s_stride, const float* rw, int rw_e, void* scratch, size_t scratch_bytes, void* stream) {
  af::GemvTcArgs a;
  a.wf = wf; a.epi = epi;
  a.x = reinterpret_cast<const __half*>(x); a.ldx = ldx;
  a.w = tiles; a.scale = reinterpret_cast<const __half*>(scales);
  a.y = y; a.ldy = ldy; a.NB = nb; a.N = n; a.K = k;
  a.sel = sel; a.slot = slot; a.fixed_e = fixed_e; a.w_stride = w_stride; a.s_stride = s_stride;
  a.rw = rw; a.rw_e = rw_e;
  a.scratch = scratch; a.scratch_bytes = scratch_bytes;
  return rc_of(af::gemv_tc_launch(a, static_cast<cudaStream_t>(stream), false), "af_gemv_tc_expert");
}

int af_gemm_tc(int wf, int epi, const uint16_t* x, int ldx, const void* tiles, const uint16_t* scales,
               const uint16_t* bias, void* y, int ldy, int m, int n, int k, void* stream) {
  af::GemvTcArgs a;
  a.wf = wf; a.epi = epi;
  a.x = reinterpret_cast<const __half*>(x); a.ldx = ldx;
  a.w = tiles; a.scale = reinterpret_cast<const __half*>(scales); a.bias = reinterpret_cast<const __half*>(bias);
  a.y = y; a.ldy = ldy; a.NB = m; a.N = n; a.K = k;
  return rc_of(af::gemm_tc_launch(a, static_cast<cudaStream_t>(stream), false), "af_gemm_tc");
}

int af_rmsnorm(const void* x, int x_f16, int ldx, const uint16_t* g, float floor, uint16_t* out, int ldo, int nb,
               int d, void* stream) {
  return rc_of(af::rmsnorm_launch(x, x_f16, ldx, reinterpret_cast<const __half*>(g), floor,
                                  reinterpret_cast<__half*>(out), ldo, nb, d, static_cast<cudaStream_t>(stream), false),
               "af_rmsnorm");
}

int af_attn_decode_scratch(int nb, int kv, int n_split, int g, int dh, size_t* bytes) {
  if (!bytes) return -1;
  *bytes = 4 * af::attn_decode_scratch_floats(nb, kv, n_split, g, dh) + 4 * (size_t)nb * kv;
  return 0;
}

int af_attn_decode(const float* qkv, int ld_qkv, uint16_t* kc, uint16_t* vc, const int* pos, const uint16_t* cos_t,
                   const uint16_t* sin_t, uint16_t* out, int ld_out, int nb, int h, int kv, int dh, int m,
                   int n_split, float scale, float kv_c, int expand, void* scratch, size_t scratch_bytes,
                   int* err, void* stream) {
  af::AttnDecodeArgs a;
  a.qkv = qkv; a.ld_qkv = ld_qkv;
  a.kc = reinterpret_cast<__half*>(kc); a.vc = reinterpret_cast<__half*>(vc);
  a.pos = pos;
  a.cos_t = reinterpret_cast<const __half*>(cos_t); a.sin_t = reinterpret_cast<const __half*>(sin_t);
  a.out = reinterpret_cast<__half*>(out); a.ld_out = ld_out;
  a.NB = nb; a.H = h; a.KV = kv; a.dh = dh; a.M = m; a.n_split = n_split;
  a.scale = scale; a.kv_c = kv_c; a.expand = expand; a.err = err;
  if (kv <= 0 || h % kv) return rc_of(cudaErrorInvalidValue, "af_attn_decode: H % KV");
  size_t need = 0;
  af_attn_decode_scratch(nb, kv, n_split, h / kv, dh, &need);
  if (n_split > 1) {
    if (!scratch || scratch_bytes < need) return rc_of(cudaErrorInvalidValue, "af_attn_decode: scratch too small");
    a.counters = static_cast<int*>(scratch);
    a.part = reinterpret_cast<float*>(static_cast<char*>(scratch) + 4 * (size_t)nb * kv);
  }
  return rc_of(af::attn_decode_launch(a, static_cast<cudaStream_t>(stream), false), "af_attn_decode");
}

}  // extern "C"
