// Internal C++ interface between the program runtime and the sm_100a kernels.
#pragma once
#include <string>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

namespace af {

// integer tuning knob from the environment (read once by each caller)
inline int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}

// W_LUT4: 4-bit indices (two per byte, low nibble first) into a 16-entry fp16 codebook per row
// (gscale [N][16]); W_I8G: int8 codes with one fp16 scale per `group` consecutive elements of a row
// (gscale [N][K / group]); W_SPARSE: a K-bit keep mask per row (w = [N][K/32] 32-bit words, bit j of
// word i = column 32 i + j) with the row's kept fp16 values in column order (gscale, the row's first
// at rowoff[row]) - the reference's palettized, blockwise and bitmask-sparse encodings, streamed packed
enum WFormat : int { W_I8 = 0, W_F16 = 1, W_I4G32 = 2, W_LUT4 = 3, W_I8G = 4, W_SPARSE = 5 };

// L2 prefetch of (part of) a later kernel's weights, issued by a kernel whose own phase leaves HBM
// idle: pieces of `piece` bytes every `stride` bytes of [base, base + bytes), spread evenly over the
// issuing threads, so every CTA of the consuming kernel finds the same share of its range in L2.
struct L2Pf {
  const char* base = nullptr;
  size_t bytes = 0, piece = 0, stride = 0;
  int keep = 0;                // prefetch with the evict-last L2 priority (survives evict-first streams)
};
enum Epilogue : int { EPI_F32 = 0, EPI_F16 = 1, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_ARGMAX = 4 };

struct GemvArgs {
  int wf = W_I8, epi = EPI_F32;
  const __half* x = nullptr;   // [NB][ldx] fp16
  int ldx = 0;
  const void* w = nullptr;     // codes / fp16 weights, [N] rows
  const __half* scale = nullptr;   // int8: [N] per-row scale
  const __half* gscale = nullptr;  // int4: [N][K/32] group scales; LUT4: [N][16] codebooks; I8G: [N][K/group]
  int group = 32;                  // I8G: elements per scale (a multiple of 16)
  const int* rowoff = nullptr;     // SPARSE: [N + 1] offsets of each row's values in gscale
  const __half* bias = nullptr;    // [N] or null
  void* y = nullptr;           // output (see Epilogue); ARGMAX: optional fp32 logits
  int ldy = 0;
  int N = 0, K = 0, NB = 1;
  int tg = 256;                // set by the dispatcher
  // ARGMAX scratch: [ctas][NB] partials + one launch counter (must start at 0; reset by the kernel)
  float* am_val = nullptr;
  int* am_idx = nullptr;
  int* am_count = nullptr;
  int am_grid_cap = 0;         // partial slots available (0 = unchecked)
  int* tok_out = nullptr;      // [NB] greedy token
  int* pos_adv = nullptr;      // [NB] decode position, advanced by one when non-null
  int* hist = nullptr;         // [NB][hist_ld] token history: hist[b][pos[b]] = token (needs pos_adv)
  int hist_ld = 0;
  float* val_out = nullptr;    // [NB] best logit (optional; a vocabulary shard's candidate)
  int idx_base = 0;            // added to the row index written to tok_out (vocabulary shard offset)
};

cudaError_t gemv_launch(const GemvArgs& a, cudaStream_t st, bool pdl);
cudaError_t gemv_sparse_launch(const GemvArgs& a, cudaStream_t st, bool pdl);

// Tensor-core int8 GEMV over fragment-tile packed weights (gemv_tc.cu). Epilogues F32/F16/RESID/SWIGLU.
struct GemvTcArgs {
  int wf = W_I8;               // W_I8: pack_i8_tiles layout + per-row scales; W_I4G32: pack_i4_tiles (scales inside)
  int epi = EPI_F32;
  const __half* x = nullptr;   // [NB][ldx] fp16, ldx % 8 == 0
  int ldx = 0;
  const void* w = nullptr;     // pack_i8_tiles layout
  const __half* scale = nullptr;   // [N] per-row
  const __half* bias = nullptr;
  void* y = nullptr;
  int ldy = 0;
  int N = 0, K = 0, NB = 1;
  void* scratch = nullptr;     // split-K partials + counters (gemv_tc_scratch_bytes); zero before first use
  size_t scratch_bytes = 0;
  int* err = nullptr;          // device error word (AF_DEV_WAIT_TIMEOUT if a pipeline wait gives up)
  // mixture of experts: the weights are E experts' tiles back to back; the expert is `sel[slot]`
  // (device memory, written by the gate kernel) or `fixed_e`; the RESID epilogue scales each batch
  // row's contribution by rw[b * rw_e + expert] when rw is given
  const int* sel = nullptr;
  int slot = 0, fixed_e = 0;
  long long w_stride = 0;      // bytes between experts' tiles
  int s_stride = 0;            // halves between experts' per-row scales
  const float* rw = nullptr;
  int rw_e = 0;
  // expert parallel: this GPU holds experts [e_base, e_base + n_exp) of the model; `sel` holds global
  // expert ids (a selected expert held elsewhere makes the whole launch a no-op here) and the
  // routing-weight column of local expert e is e_base + e
  int e_base = 0, n_exp = 0;
  // routed batch (with fixed_e): this launch serves the rows rows[(e_base + fixed_e) * rld + r0 + b]
  // for b < min(NB, rcnt[e_base + fixed_e] - r0) (none: the launch does nothing); route bit 0 gathers
  // the x rows through that list, bit 1 scatters the output rows (and their routing weights)
  const int* rows = nullptr;
  const int* rcnt = nullptr;
  int rld = 0, r0 = 0, route = 0;
  int evict_first = 0;         // weight stages with the evict-first L2 policy (read once per step)
  // set by the launcher
  int Np = 0, Kp = 0, S = 1, maxc = 1;
  int nst = 6;                 // set by the launcher: weight ring stages (<= tc::STAGES)
  int ksplit = 1;              // set by the launcher: prefill GEMM k splits per output tile (RESID only)
  int nlive = 0;               // set in the kernel: batch rows this launch computes (NB unless routed)
  int rbase = 0;               // set in the kernel: offset of this launch's first row in `rows`
  int csize = 0;               // > 1: thread-block clusters of csize CTAs split each row block's k range
  L2Pf pf;                     // issued by each CTA once its own weight copies are all requested
  float* part = nullptr;
  int* counters = nullptr;
};
cudaError_t gemv_tc_launch(const GemvTcArgs& a, cudaStream_t st, bool pdl);

// A chain of tiled GEMVs run by one persistent launch (gemv_chain.cu): job j + 1 reads what job j
// (and the RMSNorm attached to it) wrote, while every CTA keeps streaming the weights of its later
// jobs into its ring. All jobs share the weight format and the batch (1..16 rows).
constexpr int CHAIN_MAX_JOBS = 8;
struct ChainJob {
  const void* w = nullptr;          // pack_i8_tiles / pack_i4_tiles layout
  const __half* scale = nullptr;    // int8: [N] per-row scales
  const __half* bias = nullptr;
  const __half* x = nullptr;        // [NB][ldx] fp16
  int ldx = 0;
  void* y = nullptr;                // EPI_F32 / EPI_F16 / EPI_RESID (fp32 y += ..) / EPI_SWIGLU (fp16)
  int ldy = 0;
  int N = 0, K = 0, epi = EPI_F32;
  // optional RMSNorm run once the job is complete (before the next job starts):
  // nout[b] = fp16(nx[b] / max(|nx[b]|, nfloor) * ng) over nd columns, nx fp32
  const float* nx = nullptr;
  int ldnx = 0;
  const __half* ng = nullptr;
  float nfloor = 0.f;
  __half* nout = nullptr;
  int ldno = 0, nd = 0;
  // set by the launcher
  int RB = 0, KT = 0, maxc = 1;
  long long U = 0;
  int* cnt = nullptr;               // [RB] arrival tickets
  float* part = nullptr;            // [RB][maxc][64][NT * 8] partial sums
};
struct GemvChainArgs {
  ChainJob job[CHAIN_MAX_JOBS];
  int njobs = 0, NB = 1, wf = W_I8;
  void* scratch = nullptr;          // gemv_chain_scratch_bytes; zero before the first launch
  size_t scratch_bytes = 0;
  int* err = nullptr;
  int evict_first = 0;
  // set by the launcher
  int* done = nullptr;              // [njobs] row blocks finished
  int* ready = nullptr;             // [njobs] job (and its norm) complete
  int* exits = nullptr;             // CTAs finished
  int nstages = 6;                  // weight ring depth
};
cudaError_t gemv_chain_launch(GemvChainArgs a, cudaStream_t st, bool pdl);
size_t gemv_chain_scratch_bytes(const GemvChainArgs& a);
// Prefill GEMM on tcgen05 (gemm_tc.cu): same arguments as the tiled GEMV with NB = M prompt rows.
cudaError_t gemm_tc_launch(GemvTcArgs a, cudaStream_t st, bool pdl);
size_t gemv_tc_scratch_bytes(int N, int K, int NB);
void gemv_tc_plan(int N, int K, int NB, int* S, int* NT);
void gemv_tc_grid(int N, int K, int NB, int epi, bool i4, int* G, int* csize);
cudaError_t pack_i8_tiles(const int8_t* src, int N, int K, uint8_t* dst, cudaStream_t st);
size_t pack_i8_tiles_bytes(int N, int K);
cudaError_t pack_i4_tiles(const uint8_t* src, const __half* scales, int N, int K, uint8_t* dst, cudaStream_t st);
size_t pack_i4_tiles_bytes(int N, int K);
int gemv_argmax_ctas(int wf, int N, int K, int NB);
void gemv_argmax_scratch(int wf, int N, int K, int NB, size_t* slot_floats, size_t* counters);

// Per-row int8 quantizer, bit-exact to the reference's numpy `quantize_per_row`.
// src: [N][K] fp32 (src_f16 = 0) or fp16 (src_f16 = 1); codes [N][K] int8; scales [N] fp16.
cudaError_t quantize_rows_i8(const void* src, int src_f16, int N, int K, int8_t* codes, __half* scales,
                             cudaStream_t st);
// Group-32 int4 quantizer (this build's format): packed [N][K/2] bytes, scales [N][K/32] fp16.
cudaError_t quantize_g32_i4(const void* src, int src_f16, int N, int K, uint8_t* packed, __half* scales,
                            cudaStream_t st);

// out[b] = f16( x[b] / max(||x[b]||_2, floor) * g )  (the reference's RMSNorm lowering)
cudaError_t rmsnorm_launch(const void* x, int x_f16, int ldx, const __half* g, float floor, __half* out,
                           int ldo, int NB, int D, cudaStream_t st, bool pdl,
                           const L2Pf& pf = L2Pf());

// h[b][:] = f32(table[tok[b]][:]); records AF_DEV_BAD_TOKEN and writes zeros on an out-of-range id.
cudaError_t layernorm_launch(const float* x, int ldx, const __half* g, const __half* b, float eps, __half* out, int ldo,
                             int NB, int D, cudaStream_t st, bool pdl);
cudaError_t add_pos_launch(float* h, int ldh, const __half* table, int npos, const int* pos, int NB, int D, int* err,
                           cudaStream_t st, bool pdl);
cudaError_t embed_launch(const int* tok, const __half* table, int vocab, float* h, int ldh, int NB, int D,
                         int* err, cudaStream_t st, bool pdl);

// elementwise dtype conversion: mode 0 fp16 -> fp32, mode 1 fp32 -> fp16
cudaError_t cast_launch(const void* src, void* dst, size_t n, int mode, cudaStream_t st, bool pdl);

struct AttnDecodeArgs {
  const float* qkv = nullptr;  // [NB][ld_qkv] fp32: q (H*dh) | k (KV*dh) | v (KV*dh)
  int ld_qkv = 0;
  __half* kc = nullptr;        // [NB][KV][M][dh]
  __half* vc = nullptr;
  const int* pos = nullptr;    // [NB]
  const __half* cos_t = nullptr;  // [M][dh] (null: no RoPE)
  const __half* sin_t = nullptr;
  const __half* qn_g = nullptr;   // optional per-head RMSNorm (QK-norm) g_eff [dh]
  const __half* kn_g = nullptr;
  float qn_floor = 0.f, kn_floor = 0.f;
  __half* out = nullptr;       // [NB][ld_out] fp16, head-major (h*dh + d)
  int ld_out = 0;
  float* part = nullptr;       // scratch [NB][KV][n_split][G][dh + 2]
  int* counters = nullptr;     // scratch [NB][KV], zero at first launch, reset by the kernel
  int* err = nullptr;
  int NB = 1, H = 0, KV = 0, dh = 0, M = 0, n_split = 1;
  float scale = 0.f;           // fp16-rounded 1/sqrt(dh)
  float kv_c = 1.f;            // GQA expansion factor (applied as f16(c * f16(k)))
  int expand = 0;
  // 1: `pos` was written before the preceding kernel started (a decode step's position is advanced
  // by the step's last kernel), so each CTA may read it and bulk-copy its first cache rows into
  // shared memory before the programmatic-launch wait, overlapping the qkv projection's tail
  int prefetch = 0;
  // set by attn_decode_launch: cache rows staged per CTA with `prefetch`; 1 when the splits of a
  // (sequence, kv head) run as one thread-block cluster and merge through its shared memory
  int pre_rows = 0;
  int cluster = 0;
  // fewest keys per split: at short positions only ceil((pos + 1) / min_keys) splits hold keys
  // (0: the launcher's default)
  int min_keys = 0;
  L2Pf pf;                     // issued at kernel start (the attention phase reads little from HBM)
  // cache rows between consecutive sequences' caches (-1: KV * M, one cache per sequence). 0: every
  // row b of the batch is a query of ONE sequence at its own position pos[b], all reading the same
  // cache (speculative verify); the new K / V rows are then written beforehand by
  // kv_append_launch and write_kv is 0
  int kv_seq_rows = -1;
  int write_kv = 1;
};
cudaError_t attn_decode_launch(const AttnDecodeArgs& a, cudaStream_t st, bool pdl);
// QK-norm + RoPE of each batch row's k at pos[b], written with its v into cache row pos[b] (the
// cache addressing of AttnDecodeArgs: kv_seq_rows 0 = one shared cache); grid (NB, KV)
cudaError_t kv_append_launch(const AttnDecodeArgs& a, cudaStream_t st, bool pdl);
// true when a launch with these arguments merges its splits through a.part / a.counters (false
// when there is one split, or the splits of a kv head merge inside a thread-block cluster)
bool attn_decode_uses_scratch(const AttnDecodeArgs& a);
size_t attn_decode_scratch_floats(int NB, int KV, int n_split, int G, int dh);

// MoE router tail (moe.cu): softmax over E, top-k by repeated row-max peel (lowest index on ties),
// optional renormalisation -> gw [NB][E] (zeros off the top k) and sel [NB][k] (peel order)
cudaError_t moe_gate_launch(const float* logits, int ld, int NB, int E, int k, int renorm, float* gw, int* sel,
                            cudaStream_t st, bool pdl);
// per-expert row lists of a batch from the gate's selections: rows[e * rld + i] for i < cnt[e]
cudaError_t moe_route_launch(const int* sel, int NB, int k, int E, int rld, int* rows, int* cnt, cudaStream_t st,
                             bool pdl);

// ---- tensor parallel (comm.cu): collectives on a program's stream, cross-rank argmax, residual add
// dst = sum over the ranks of src; with `addto`, addto += that sum instead (dst then scratch)
cudaError_t comm_all_reduce_rms_f32(void* comm, const float* src, float* tmp, float* h, int NB, int D, const __half* g,
                                    float floor, __half* out, cudaStream_t st, std::string& why, int* err, bool pdl);
cudaError_t comm_all_reduce_f32(void* comm, const float* src, float* dst, size_t n, cudaStream_t st, std::string& why,
                                int* err = nullptr, float* addto = nullptr, bool pdl = false);
cudaError_t comm_all_gather_i32(void* comm, const int* src, int* dst, size_t n, cudaStream_t st, std::string& why);
int comm_size(void* comm);
int comm_rank(void* comm);
cudaError_t tp_argmax_launch(const int* gathered, int T, int NB, int* tok_out, int* pos_adv, int* hist, int hist_ld,
                             cudaStream_t st);
cudaError_t add_f32_launch(float* y, const float* x, size_t n, cudaStream_t st);

// Prefill causal attention over S prompt rows (CUDA-core flash form, fp16 q/K/V operands).
struct AttnPrefillArgs {
  const float* qkv = nullptr;  // [S][ld_qkv] fp32 (q | k | v), bias included
  int ld_qkv = 0;
  const __half* cos_t = nullptr;
  const __half* sin_t = nullptr;
  const __half* qn_g = nullptr;
  const __half* kn_g = nullptr;
  float qn_floor = 0.f, kn_floor = 0.f;
  __half* kc = nullptr;        // [KV][ldm][dh]: roped K written at rows 0..S-1 (cache layout)
  __half* vc = nullptr;
  int ldm = 0;
  __half* out = nullptr;       // [S][H*dh]
  int S = 0, H = 0, KV = 0, dh = 0;
  float scale = 0.f, kv_c = 1.f;
  int expand = 0;
  __half* kvx = nullptr;       // optional [2][KV][S][dh]: K and V times the GQA factor (expand), for the
                               // tensor-core attention
  int* err = nullptr;          // device error word (AF_DEV_WAIT_TIMEOUT if a pipeline wait gives up)
};
// rope q (-> qbuf [H][S][dh] fp16) and k, write roped K / raw V into cache rows 0..S-1 (and, with
// expand and kvx, the expanded copies)
cudaError_t rope_kv_prefill_launch(const AttnPrefillArgs& a, __half* qbuf, cudaStream_t st);
// causal attention of the staged q rows against cache rows 0..i
cudaError_t attn_prefill_with_q(const AttnPrefillArgs& a, const __half* qbuf, cudaStream_t st);
// the tcgen05 form (attn_prefill_tc.cu): head dim 128; with expand it reads kvx
bool attn_prefill_tc_ok(const AttnPrefillArgs& a);
cudaError_t attn_prefill_tc_launch(const AttnPrefillArgs& a, const __half* qbuf, cudaStream_t st);

// ---- generic graph ops (graph_ops.cu): what `compile(graph)` lowers nodes onto when no fused kernel
// covers them. fp32 values, fp16-rounded matmul operands, rank <= GRAPH_MAX_RANK.
constexpr int GRAPH_MAX_RANK = 5;
enum GraphBinary : int { G_ADD = 0, G_SUB, G_MUL, G_DIV, G_MAX, G_MIN, G_POW, G_GT, G_GE, G_LT, G_LE, G_EQ, G_NE,
                         G_SELECT };
enum GraphUnary : int { U_RELU = 0, U_SILU, U_SIGMOID, U_TANH, U_EXP, U_SQRT, U_ABS, U_SQUARE, U_SIN, U_COS, U_ERF,
                        U_LOG, U_RSQRT, U_INV, U_MULS, U_ADDS, U_CLIP, U_NOT, U_FLOOR, U_CEIL, U_ROUND, U_SIGN,
                        U_GELU_TANH, U_GELU, U_SOFTPLUS };
enum GraphReduce : int { RD_SUM = 0, RD_MEAN, RD_MAX, RD_MIN, RD_SUMSQ, RD_L2, RD_L1 };
struct GraphEwArgs {          // y[i] = op(a[.], b[.]) (select: a ? b : c) over the output shape
  const float* a = nullptr;
  const float* b = nullptr;
  const float* c = nullptr;
  float* y = nullptr;
  int op = 0, rank = 0;
  long long n = 0;
  long long shape[GRAPH_MAX_RANK] = {};
  long long sa[GRAPH_MAX_RANK] = {}, sb[GRAPH_MAX_RANK] = {}, sc[GRAPH_MAX_RANK] = {};
};
struct GraphCopyArgs {        // y at strides sy <- x at strides sx, over `shape`
  const float* x = nullptr;
  float* y = nullptr;
  int rank = 0;
  long long n = 0;
  long long shape[GRAPH_MAX_RANK] = {};
  long long sx[GRAPH_MAX_RANK] = {}, sy[GRAPH_MAX_RANK] = {};
};
struct GraphReduceArgs {      // contiguous x of `shape`; reduce the axes whose bit is set in mask
  const float* x = nullptr;
  float* y = nullptr;
  int op = 0, rank = 0, mask = 0;
  long long n_out = 0;
  long long shape[GRAPH_MAX_RANK] = {};
};
struct GraphLinearArgs {      // y[r][n] = (sum_k f16(x[r][k]) w[n][k]) * scale[n] + bias[n]
  const float* x = nullptr;
  const void* w = nullptr;    // int8 [N][K] codes (int8 != 0) or fp16 [N][K]
  const __half* scale = nullptr;
  const __half* bias = nullptr;
  float* y = nullptr;
  long long rows = 0, ldx = 0, ldy = 0, N = 0, K = 0;
  int int8 = 0;
};
struct GraphBmmArgs {         // y[b][m][n] = sum_k f16(a) f16(b)
  const float* a = nullptr;
  const float* b = nullptr;
  float* y = nullptr;
  long long batch = 1, M = 0, N = 0, K = 0;
  int brank = 0;
  long long bshape[GRAPH_MAX_RANK] = {};
  long long sa[GRAPH_MAX_RANK] = {}, sb[GRAPH_MAX_RANK] = {};
  long long sam = 0, sak = 0, sbk = 0, sbn = 0;
  int round_b = 1;            // 0: b is a baked weight used at full fp32 (bmm_weight)
};
cudaError_t graph_ew_launch(const GraphEwArgs& a, cudaStream_t st);
cudaError_t graph_unary_launch(const float* x, float* y, long long n, int op, float k, float k2, cudaStream_t st);
cudaError_t graph_copy_launch(const GraphCopyArgs& a, cudaStream_t st);
cudaError_t graph_reduce_launch(const GraphReduceArgs& a, cudaStream_t st);
cudaError_t graph_softmax_launch(const float* x, float* y, long long outer, long long n, long long inner, cudaStream_t st);
cudaError_t graph_rms_launch(const float* x, float* y, const __half* g, float floor, long long rows, int d,
                             cudaStream_t st);
cudaError_t graph_layernorm_launch(const float* x, float* y, const __half* g, const __half* b, float eps,
                                   long long rows, int d, cudaStream_t st);
cudaError_t graph_linear_launch(const GraphLinearArgs& a, cudaStream_t st);
cudaError_t graph_bmm_launch(const GraphBmmArgs& a, cudaStream_t st);
cudaError_t graph_decode_ctx_launch(const int* pos, const __half* cos_t, const __half* sin_t, int M, int dh, float* oh,
                                    float* inv, float* mask, float* cosp, float* sinp, cudaStream_t st);

}  // namespace af
