/* C ABI of libaf_cuda.so, the B200 (sm_100a) invoker for ANEForge's quantized LLM hot path.
 *
 * Two layers:
 *  1. The program API (af_program_*): a drop-in for the reference's e5rt dispatch shim
 *     (aneforge/_lib/ane_e5rt_dispatch.mm, bound by aneforge/_runtime.py:61-92). Same shapes: a
 *     program is compiled from a path, owns named zero-initialised ports, copies fp16 in/out,
 *     hands out persistent zero-copy buffer pointers (here: DEVICE pointers), aliases an output
 *     port onto an input port for resident state, and executes synchronously; the first execute
 *     finalises the program (captures one CUDA graph), after which aliasing and binding fail.
 *     Return codes: 0 ok, -1 error (reason in af_last_error() and on stderr), -2 a kernel
 *     recorded an error (bad token id / position) during execute.
 *  2. Kernel entry points (af_quantize_*, af_gemv, af_lm_head_argmax, af_rmsnorm, af_attn_decode):
 *     plain device pointers + a cudaStream_t passed as void*, one fused kernel each.
 *
 * No torch types cross this boundary; fp16 values travel as uint16_t bit patterns.
 */
#ifndef AF_CUDA_H
#define AF_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AF_CUDA_ABI_VERSION 1

/* Weight formats / GEMV epilogues (af_gemv, af_lm_head_argmax). */
#define AF_W_I8 0    /* per-row int8 codes [N][K] + fp16 scales [N] (reference _blob.quantize_per_row) */
#define AF_W_F16 1   /* fp16 weights [N][K] */
#define AF_W_I4G32 2 /* group-32 int4: packed [N][K/2] (low nibble first) + fp16 scales [N][K/32] */
#define AF_EPI_F32 0    /* y (fp32) = s*(x.W^T) + bias */
#define AF_EPI_F16 1    /* y (fp16) = s*(x.W^T) + bias */
#define AF_EPI_RESID 2  /* y (fp32) += s*(x.W^T) + bias */
#define AF_EPI_SWIGLU 3 /* y (fp16) = silu(gate)*up, gate/up rows packed in blocks of R */

/* Last error message of this thread (valid until the next failing call). */
const char* af_last_error(void);
int af_abi_version(void);

/* ---------------------------------------------------------------- program API (e5rt replacement) */

/* Replaces ane_e5rt_program_compile (aneforge/_lib/ane_e5rt_dispatch.mm:528-608; bound at
 * aneforge/_runtime.py:61-66, called from E5RT.compile, _runtime.py:251-280). `program_path` is a
 * directory holding plan.txt (+ optional weights.bin) written by aneforge_b200._compile;
 * `device_mask` bit i selects GPU i (0 = current device). The declared ports must exist in the
 * plan with at least the declared byte sizes. Returns NULL on failure. */
void* af_program_compile(const char* program_path, const char* cache_dir, uint64_t device_mask,
                         const char* const* in_names, const size_t* in_bytes, size_t n_in,
                         const char* const* out_names, const size_t* out_bytes, size_t n_out);

/* Same, from plan text in memory (weights only by upload/bind). No reference counterpart: the e5rt
 * shim always compiles from a file. */
void* af_program_compile_text(const char* plan_text, const char* weights_dir, uint64_t device_mask);

/* Replaces ane_e5rt_compile_check (ane_e5rt_dispatch.mm:416-469): validate a plan without
 * allocating device memory. 0 = valid. */
int af_compile_check(const char* program_path, const char* cache_dir, uint64_t device_mask,
                     const char* custom_options);

/* Replaces ane_e5rt_program_set_input_fp16 (ane_e5rt_dispatch.mm:617-630): copy n fp16 elements
 * into an input/state port; -1 if 2n exceeds the port or the port is unknown. */
int af_program_set_input_fp16(void* prog, const char* port, const uint16_t* src, size_t n_elems);

/* Replaces ane_e5rt_program_get_output_fp16 (ane_e5rt_dispatch.mm:632-645): copy min(2n, port
 * bytes) out of an output port. */
int af_program_get_output_fp16(void* prog, const char* port, uint16_t* dst, size_t n_elems);

/* Raw-byte variants for non-fp16 ports (token ids, positions). Extends the fp16-only e5rt ports. */
int af_program_set_input_bytes(void* prog, const char* port, const void* src, size_t nbytes);
int af_program_get_output_bytes(void* prog, const char* port, void* dst, size_t nbytes);

/* Replace ane_e5rt_program_input_buffer / output_buffer (ane_e5rt_dispatch.mm:647-665): persistent
 * zero-copy pointers valid for the program's lifetime. Here they are device pointers. */
int af_program_input_buffer(void* prog, const char* port, void** ptr, size_t* bytes);
int af_program_output_buffer(void* prog, const char* port, void** ptr, size_t* bytes);

/* Any named buffer of the plan (weights, activations): device pointer + size. Used by the loader
 * to fill packed weights in place. No e5rt counterpart (its weights live in the compiled bundle). */
int af_program_buffer(void* prog, const char* name, void** ptr, size_t* bytes);
/* Host -> device copy into any named buffer at a byte offset. */
int af_program_upload(void* prog, const char* name, const void* src, size_t nbytes, size_t offset);
/* Device -> host copy of any named buffer. */
int af_program_download(void* prog, const char* name, void* dst, size_t nbytes);
/* Make a named buffer use caller-owned device memory (16-byte aligned, >= the declared size).
 * Before the first execute only; the program never frees bound memory. */
int af_program_bind_buffer(void* prog, const char* name, void* device_ptr, size_t bytes);

/* Replaces ane_e5rt_program_execute (ane_e5rt_dispatch.mm:667-673): synchronous; the first call
 * finalises the program (CUDA graph capture). */
int af_program_execute(void* prog);
/* Asynchronous execute on the program's stream, and the matching wait + device error check.
 * The e5rt shim's unbound async surface (ane_e5rt_dispatch.mm:905-1012) is the counterpart. */
int af_program_execute_async(void* prog);
int af_program_sync(void* prog);
/* The program's CUDA stream (cudaStream_t) for callers that interoperate with other work. */
int af_program_stream(void* prog, void** stream);
/* Before the first execute: disable CUDA-graph replay / programmatic dependent launch. */
int af_program_set_options(void* prog, int use_graph, int use_pdl);

/* Tensor parallel (no reference counterpart: the ANE runtime is single-device). One communicator per
 * rank over NCCL (loaded at run time): rank 0 makes the unique id, every rank passes it to
 * af_comm_init with its GPU. A program whose plan holds collective ops (allreduce / allgather) gets
 * the communicator before its first execute; the communicator must outlive the program. */
int af_comm_unique_id(void* out, size_t bytes);
int af_comm_init(const void* id, int nranks, int rank, int device, void** comm);
void af_comm_destroy(void* comm);
/* Optional one-shot all-reduce over NVLink peer memory for small fp32 all-reduces (the decode
 * residual updates), replacing NCCL for them: every rank calls af_comm_p2p_handle (allocates its
 * exchange buffer for up to cap_floats per call and writes its CUDA IPC handle, 64 bytes), the
 * handles are exchanged between the ranks (rank order), then every rank calls af_comm_p2p_open with
 * all of them. Each call waits (bounded, ~1 s) for the peers and records AF_DEV_WAIT_TIMEOUT in the
 * program's error word if one never arrives. Up to 8 ranks, one process per GPU. */
int af_comm_p2p_handle(void* comm, size_t cap_floats, void* handle, size_t bytes);
int af_comm_p2p_open(void* comm, const void* handles, size_t bytes_each);
/* Back to NCCL for every all-reduce (when another rank could not open the peer buffers). */
void af_comm_p2p_disable(void* comm);
int af_program_set_comm(void* prog, void* comm);

/* Replaces ane_e5rt_program_share_buffer (ane_e5rt_dispatch.mm:687-714): rebind input `dst_in` to
 * output `src_out`'s buffer (resident state). Op indices must be 0. Before the first execute only;
 * the destination's own buffer is freed exactly once. */
int af_program_share_buffer(void* prog, size_t src_op_idx, const char* src_out, size_t dst_op_idx,
                            const char* dst_in);

/* Replaces ane_e5rt_program_release (ane_e5rt_dispatch.mm:716-725). */
void af_program_release(void* prog);

/* ---------------------------------------------------------------- kernel entry points */

/* Per-row int8 quantizer on the device, bit-exact to the reference's numpy encoder
 * (aneforge/_blob.py:20-25, applied by _compile.py:173-179). src [n][k] fp32 (src_f16=0) or
 * fp16 (src_f16=1); codes [n][k]; scales [n] fp16 bits. */
int af_quantize_per_row_i8(const void* src, int src_f16, int n, int k, int8_t* codes, uint16_t* scales,
                           void* stream);

/* Group-32 int4 quantizer (no reference counterpart; modelled on _blob.quantize_blockwise,
 * aneforge/_blob.py:46-56): packed [n][k/2], scales [n][k/32]. */
int af_quantize_g32_i4(const void* src, int src_f16, int n, int k, uint8_t* packed, uint16_t* scales,
                       void* stream);

/* Dequant GEMV (decode matmul): replaces the `matmul` of _compile.py:375-385 over a
 * constexpr_affine_dequantize weight (int8) / fp16 const. x [nb][ldx] fp16; y per `epi`. */
int af_gemv(int wf, int epi, const uint16_t* x, int ldx, const void* w, const uint16_t* scales,
            const uint16_t* bias, void* y, int ldy, int nb, int n, int k, void* stream);

/* Tensor-core int8 GEMV (the decode K1 kernel): weights re-packed once into 16x32 fragment tiles
 * (af_pack_i8_tiles, [ceil(n/64)][ceil(k/32)][4 row tiles of 16][512 B]: 16 rows x 32 codes per tile) from per-row int8 codes [n][k]; same epilogues as
 * af_gemv (AF_EPI_SWIGLU tiles hold 8 gate rows then the 8 matching up rows). Replaces the same
 * reference `matmul` (_compile.py:375-385). Scratch (split-K partials + counters):
 * af_gemv_tc_scratch_bytes, zero before the first call, left zeroed; 0 bytes needs no scratch. */
size_t af_pack_i8_tiles_bytes(int n, int k);
int af_pack_i8_tiles(const int8_t* codes, int n, int k, uint8_t* tiles, void* stream);
size_t af_gemv_tc_scratch_bytes(int n, int k, int nb);
/* Scratch of a plan's `gemv_chain` op (no counterpart in the reference: several tensor-core GEMVs,
 * each with an optional RMSNorm after it, in one persistent launch) for njobs jobs of shapes
 * n[j] x k[j] at batch nb; wf 0 int8 tiles, 2 group-32 int4 tiles. 0 on bad arguments. */
size_t af_gemv_chain_scratch_bytes(int njobs, const int* n, const int* k, int nb, int wf);
/* Grid of the tensor-core GEMV for one shape on the current device (no counterpart in the
 * reference): CTAs per 16-row slice (*grid) and the thread-block cluster size splitting each
 * 64-row block (*csize; 0: stream-K). The CTAs' k ranges cover the packed weights in grid equal,
 * contiguous, ordered pieces, which is what a plan's L2 prefetch of those weights follows.
 * wf: 0 int8 tiles, 2 group-32 int4 tiles; epi as af_gemv_tc. Returns 0, or -1 on bad arguments. */
int af_gemv_tc_grid(int n, int k, int nb, int epi, int wf, int* grid, int* csize);
int af_gemv_tc(int epi, const uint16_t* x, int ldx, const void* tiles, const uint16_t* scales, const uint16_t* bias,
               void* y, int ldy, int nb, int n, int k, void* scratch, size_t scratch_bytes, void* stream);

/* Prefill GEMM on the 5th-generation tensor cores (tcgen05.mma, fp32 accumulators in tensor memory):
 * y[m][n] = epilogue(sum_k x[m][k] * w[n][k]) for m prompt rows, over the same packed tiles as the
 * decode GEMVs (wf AF_W_I8: af_pack_i8_tiles + per-row scales applied to the fp32 sums; AF_W_I4G32:
 * af_pack_i4_tiles, dequantised to fp16 code * scale before the MMA). Epilogues AF_EPI_F32 / F16 /
 * RESID / SWIGLU as af_gemv_tc; k % 32 == 0. Replaces the reference's prefill `matmul`
 * (_compile.py:375-385 inside the prefill graph, llm.py:118-169). */
int af_gemm_tc(int wf, int epi, const uint16_t* x, int ldx, const void* tiles, const uint16_t* scales,
               const uint16_t* bias, void* y, int ldy, int m, int n, int k, void* stream);

/* Group-32 int4 on the tensor pipe: codes from af_quantize_g32_i4 (packed [n][k/2] + scales [n][k/32])
 * re-packed once into 16x32 fragment tiles with each k tile's 64 row scales appended
 * ([ceil(n/64)][k/32][4 x 256 B | 64 fp16], k % 32 == 0). y = sum over groups of s_g * (x . codes_g),
 * fp32 accumulation, same epilogues and scratch rule as af_gemv_tc. Replaces the reference `matmul`
 * (_compile.py:375-385) for this build's int4_g32 weights (no reference counterpart for the format). */
size_t af_pack_i4_tiles_bytes(int n, int k);
int af_pack_i4_tiles(const uint8_t* packed, const uint16_t* scales, int n, int k, uint8_t* tiles, void* stream);
int af_gemv_tc_i4(int epi, const uint16_t* x, int ldx, const void* tiles, const uint16_t* bias, void* y, int ldy,
                  int nb, int n, int k, void* scratch, size_t scratch_bytes, void* stream);

/* Mixture of experts (reference aneforge/moe.py:21-63). af_moe_gate: router logits [nb][ld] fp32 ->
 * softmax, top-k by k row-max peels (lowest index on ties, peel value f16(-3e4)), renormalised when
 * renorm -> gw [nb][e] (0 off the top k) and sel [nb][k]. af_gemv_tc_expert: the tensor-core GEMV
 * (wf AF_W_I8 tiles + scales, or AF_W_I4G32 tiles) over E experts stored back to back
 * (`w_stride` bytes, `s_stride` scale halves apart), expert = sel[slot] (sel non-NULL, read on the
 * device) or fixed_e; with epi AF_EPI_RESID and rw non-NULL each batch row's contribution is scaled
 * by rw[b * rw_e + expert]. */
int af_moe_gate(const float* logits, int ld, int nb, int e, int k, int renorm, float* gw, int* sel, void* stream);
int af_gemv_tc_expert(int wf, int epi, const uint16_t* x, int ldx, const void* tiles, const uint16_t* scales,
                      void* y, int ldy, int nb, int n, int k, const int* sel, int slot, int fixed_e, long long w_stride,
                      int s_stride, const float* rw, int rw_e, void* scratch, size_t scratch_bytes, void* stream);

/* lm_head GEMV + greedy argmax (lowest index on ties): replaces the host `hidden @ lm_head.T` and
 * np.argmax of LlamaPrefill._logits/_sample (aneforge/llm.py:349-355, :407-410). `logits` [nb][n]
 * may be NULL; `pos_advance` (may be NULL) is incremented per row. Scratch: see _scratch; it must be
 * zero before the first call and is left zeroed. */
int af_lm_head_argmax_scratch(int wf, int n, int k, int nb, size_t* bytes);
int af_lm_head_argmax(int wf, const uint16_t* x, int ldx, const void* w, const uint16_t* scales, float* logits,
                      int nb, int n, int k, int* tok_out, int* pos_advance, void* scratch, size_t scratch_bytes,
                      void* stream);

/* RMSNorm as the reference lowers it (aneforge/_compile.py:738-755):
 * out = f16(x / max(||x||, floor) * g), x fp32 (x_f16=0) or fp16. */
int af_rmsnorm(const void* x, int x_f16, int ldx, const uint16_t* g, float floor, uint16_t* out, int ldo, int nb,
               int d, void* stream);

/* GQA decode attention with RoPE and the resident-cache write at pos: replaces the attention part of
 * _attn_decode (aneforge/llm.py:214-237). Caches [nb][kv][m][dh] fp16; qkv [nb][ld_qkv] fp32.
 * Scratch (n_split > 1): af_attn_decode_scratch bytes, zero before the first call, left zeroed. */
int af_attn_decode_scratch(int nb, int kv, int n_split, int g, int dh, size_t* bytes);
int af_attn_decode(const float* qkv, int ld_qkv, uint16_t* kc, uint16_t* vc, const int* pos, const uint16_t* cos_t,
                   const uint16_t* sin_t, uint16_t* out, int ld_out, int nb, int h, int kv, int dh, int m,
                   int n_split, float scale, float kv_c, int expand, void* scratch, size_t scratch_bytes,
                   int* err, void* stream);

/* af_attn_decode without caller scratch, for callers that cannot allocate device memory (a host
 * framework that owns every allocation, code running while a memory pool is locked, plug-ins that
 * must not touch the process allocator). No counterpart in the reference: the ANE runtime had no
 * split-K scratch. The scratch is a fixed AF_ATTN_NOALLOC_SCRATCH_BYTES array inside the library,
 * resident on every GPU that loads it until exit; shapes that merge their splits through it and
 * need more return -1 before launching (shapes whose splits merge inside a thread-block cluster,
 * at most 16 splits, use none of it). All calls on a GPU share that array: calls that overlap on
 * the GPU race (order them on one stream). The first call on a device looks the array's address up
 * and caches it; make it before any stream capture, and do not use the entry point across a
 * cudaDeviceReset. Same arguments as af_attn_decode minus the scratch pair; the current device must
 * be the stream's device. */
#define AF_ATTN_NOALLOC_SCRATCH_BYTES (2u << 20)
size_t af_attn_decode_noalloc_max_bytes(void);
int af_attn_decode_noalloc(const float* qkv, int ld_qkv, uint16_t* kc, uint16_t* vc, const int* pos,
                           const uint16_t* cos_t, const uint16_t* sin_t, uint16_t* out, int ld_out, int nb, int h,
                           int kv, int dh, int m, int n_split, float scale, float kv_c, int expand, int* err,
                           void* stream);

#ifdef __cplusplus
}
#endif
#endif /* AF_CUDA_H */
