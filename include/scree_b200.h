/*
 * scree_b200.h — C ABI of libscree_b200.so, the B200 (sm_100a) implementation of
 * scree's varlen hot path.
 *
 * Conventions
 *  - Every function returns a scree_status; on failure scree_last_error() gives a
 *    message (thread-local).  Nothing here allocates device memory: callers pass
 *    outputs and, where a kernel needs scratch, a workspace whose size the
 *    matching *_workspace_size() function reports.
 *  - Pointers are device pointers unless the name says host.  `stream` is a
 *    cudaStream_t (pass 0 for the legacy default stream).  All work is enqueued
 *    asynchronously on that stream; no function synchronises.
 *  - Packed ("varlen") tensors follow scree.Array: `values` of shape (T, ...)
 *    with sequence b occupying rows [offsets[b], offsets[b+1]).  `offsets` is a
 *    device array of B+1 int32 (offs_is_i64 = 0) or int64 (offs_is_i64 = 1).
 *  - Row strides are in ELEMENTS.  The innermost (feature / head_dim) stride is 1.
 */
#ifndef SCREE_B200_H_
#define SCREE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SCREE_ABI_VERSION 1

typedef enum {
  SCREE_OK = 0,
  SCREE_ERR_INVALID = 1,     /* bad argument: maps to AssertionError / ValueError */
  SCREE_ERR_UNSUPPORTED = 2, /* valid but not implemented (e.g. head_dim 96)   */
  SCREE_ERR_CUDA = 3         /* a CUDA runtime call failed                       */
} scree_status;

typedef enum { SCREE_F16 = 0, SCREE_BF16 = 1, SCREE_F32 = 2 } scree_dtype;

/* Codes of the device status word (scree_device_status). */
#define SCREE_DEVERR_WAIT_TIMEOUT 1
#define SCREE_DEVERR_BAD_INPUT 2

/* Copies the calling thread's last error message into buf (NUL-terminated). */
int scree_last_error(char* buf, size_t n);
/* Returns SCREE_ABI_VERSION. */
int scree_version(void);
/* Reads (and optionally clears) the device status word that kernels set when a
 * bounded wait gave up or an input was out of range.  0 = no error, otherwise
 * (code << 16) | site with code SCREE_DEVERR_WAIT_TIMEOUT (1) or
 * SCREE_DEVERR_BAD_INPUT (2).  This call synchronises with the device. */
int scree_device_status(int* status_out, int reset);
/* Number of kernels this library has launched in the process so far. */
long long scree_launch_count(void);
/* Per-kernel timing for benchmarks: when enabled, each main kernel launch is
 * bracketed by CUDA events on its stream.  scree_profile_read() waits for the
 * recorded events, returns the summed milliseconds and launch count of one
 * kernel kind (0 attention fwd, 1 attention bwd, 2 norm fwd, 3 norm bwd,
 * 4 gathers) and
 * clears them.  Neither call has a reference counterpart. */
int scree_profile_enable(int on);
int scree_profile_read(int kernel, double* total_ms, long long* launches);

/* Device-side check of an offsets array (B+1 entries, int32 or int64):
 * offsets[0] == 0, non-decreasing, offsets[B] == T.  Enqueued on `stream`; a
 * violation sets the device status word to (SCREE_DEVERR_BAD_INPUT << 16) | 40,
 * read with scree_device_status.  The attention entry points run the same check
 * in their schedule kernel and then do no work at all on invalid offsets; the
 * softmax and gather kernels skip (and report) any sequence whose range falls
 * outside [0, T).  Replaces the invariant checks of scree/_core.py:44-62, which
 * cover only offsets[0] and offsets[-1], with a full check on the device (no
 * host synchronisation). */
int scree_validate_offsets(const void* offsets, int offs_is_i64, int64_t B, int64_t T,
                           void* stream);

/* Self-test of failure detection (no reference counterpart): one GPU thread
 * waits on an mbarrier that nothing arrives on, bounded by limit_ns (at most
 * 1 s), exactly as every pipeline wait of the library is bounded.  When the
 * limit expires the kernel writes 0 to *result_dev (device int; 1 if the wait
 * had completed), sets the status word to (SCREE_DEVERR_WAIT_TIMEOUT << 16) | 99
 * and returns, leaving the context usable.  Reset the status word before and
 * after (scree_device_status with reset = 1): kernels skip their work while it
 * holds an error. */
int scree_selftest_wait_timeout(long long limit_ns, int* result_dev, void* stream);

/* ------------------------------------------------------------------ attention
 * Varlen self-attention forward.
 * Replaces: scree/kernels/triton/varlen_attention.py:165-268
 *   varlen_attention_triton(q, k, v, cu_seqlens, causal, block_m, block_n,
 *                           return_lse, out, lse_buffer)
 * and the kernel it launches (varlen_attention.py:36-162).
 * q, k, v, o: (T, H, D) fp16/bf16 with strides (row_stride, head_stride, 1)
 * in elements; o may alias nothing else.  lse: (T, H) fp32 contiguous, natural
 * log of the softmax denominator (m + ln l), or NULL.  scale is the softmax
 * scale (scree uses 1/sqrt(D)).  max_seqlen is accepted for signature
 * compatibility and ignored: the work list is built on the device from the
 * offsets, with no host synchronisation.  Invalid offsets (see
 * scree_validate_offsets) make the call do no work and set the status word.
 * D must be 32, 64 or 128.  workspace: scree_attn_fwd_workspace_size() bytes. */
size_t scree_attn_fwd_workspace_size(int64_t B, int64_t T, int64_t H, int D);
int scree_attn_fwd(const void* q, const void* k, const void* v, int64_t q_row_stride,
                   int64_t q_head_stride, int64_t k_row_stride, int64_t k_head_stride,
                   int64_t v_row_stride, int64_t v_head_stride, const void* offsets,
                   int offs_is_i64, int64_t B, int64_t T, int64_t H, int D, int dtype,
                   int causal, float scale, int64_t max_seqlen, void* o, int64_t o_row_stride,
                   int64_t o_head_stride, float* lse, void* workspace, size_t workspace_bytes,
                   void* stream);

/* Grouped-query attention forward: q (T, H, D) with H = H_kv * G query heads,
 * k and v (T, H_kv, D); query head h reads K / V head h / G.  Otherwise as
 * scree_attn_fwd (which is this call with H_kv = H).  The reference lists GQA
 * as not yet supported (docs/kernels.md:177); no reference counterpart. */
int scree_attn_fwd_gqa(const void* q, const void* k, const void* v, int64_t q_row_stride,
                       int64_t q_head_stride, int64_t k_row_stride, int64_t k_head_stride,
                       int64_t v_row_stride, int64_t v_head_stride, const void* offsets,
                       int offs_is_i64, int64_t B, int64_t T, int64_t H, int64_t H_kv, int D,
                       int dtype, int causal, float scale, int64_t max_seqlen, void* o,
                       int64_t o_row_stride, int64_t o_head_stride, float* lse, void* workspace,
                       size_t workspace_bytes, void* stream);

/* KV-cache attention forward (no reference counterpart; docs/kernels.md:178
 * lists KV-cache support as planned): queries and keys have offsets of their
 * own.  q / o: (Tq, H, D) with offsets_q; k / v: (Tk, H_kv, D) with offsets_k;
 * both arrays hold B + 1 entries of the same integer type.  Causal masking is
 * aligned at the end of each sequence: query i of a sequence with Lq queries
 * and Lk keys sees keys j <= i + (Lk - Lq) (decode and chunked prefill against
 * a cache that already holds the earlier tokens).  A query with no key gets
 * O = 0 and LSE = -inf.  Workspace: scree_attn_fwd_workspace_size(B, Tq, H, D).
 * Both offsets arrays are validated on the device. */
int scree_attn_fwd_kv(const void* q, const void* k, const void* v, int64_t q_row_stride,
                      int64_t q_head_stride, int64_t k_row_stride, int64_t k_head_stride,
                      int64_t v_row_stride, int64_t v_head_stride, const void* offsets_q,
                      const void* offsets_k, int offs_is_i64, int64_t B, int64_t Tq, int64_t Tk,
                      int64_t H, int64_t H_kv, int D, int dtype, int causal, float scale, void* o,
                      int64_t o_row_stride, int64_t o_head_stride, float* lse, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Allocation-free variant of scree_attn_fwd (no counterpart in the reference).
 * For callers that cannot allocate device memory when they run attention (an
 * engine with a fixed pre-planned memory arena, or a binding that only holds
 * raw input/output pointers): same arguments and results as scree_attn_fwd
 * minus the workspace, which comes from a 64 KiB array built into the library
 * (one per GPU, held until process exit).  Limit: B <= 4095 sequences, larger
 * batches return SCREE_ERR_INVALID.  All calls on a device share that array:
 * calls that overlap on the GPU race, so order them (one stream).  The first
 * call on a device resolves the array's address; make it before any stream
 * capture.  That address is cached per device: after a cudaDeviceReset of a
 * device, do not call this entry point on it again in the same process.
 * Allocates nothing. */
int scree_attn_fwd_noalloc(const void* q, const void* k, const void* v, int64_t q_row_stride,
                           int64_t q_head_stride, int64_t k_row_stride, int64_t k_head_stride,
                           int64_t v_row_stride, int64_t v_head_stride, const void* offsets,
                           int offs_is_i64, int64_t B, int64_t T, int64_t H, int D, int dtype,
                           int causal, float scale, int64_t max_seqlen, void* o,
                           int64_t o_row_stride, int64_t o_head_stride, float* lse, void* stream);

/* Varlen self-attention backward: dq, dk, dv from do, q, k, v, o, lse.
 * Replaces: scree/kernels/triton/_backward.py:288-396
 *   varlen_attention_triton_backward(do, q, k, v, o, lse, cu_seqlens, causal,
 *                                    block_m, block_n) -> (dq, dk, dv)
 * and its three kernels (_backward.py:37-69, :73-187, :191-285).
 * All (T, H, D) tensors here must be contiguous (row stride H*D, head stride D).
 * lse: (T, H) fp32 from scree_attn_fwd.  workspace: see the size function
 * (fp32 dQ accumulator + per-row Delta + the tile schedule). */
size_t scree_attn_bwd_workspace_size(int64_t B, int64_t T, int64_t H, int D);
int scree_attn_bwd(const void* dout, const void* q, const void* k, const void* v, const void* o,
                   const float* lse, const void* offsets, int offs_is_i64, int64_t B, int64_t T,
                   int64_t H, int D, int dtype, int causal, float scale, int64_t max_seqlen,
                   void* dq, void* dk, void* dv, void* workspace, size_t workspace_bytes,
                   void* stream);

/* Grouped-query attention backward: dq (T, H, D); dk, dv (T, H_kv, D) summed
 * over the G query heads that share each K / V head.  Contiguous tensors as in
 * scree_attn_bwd (= this call with H_kv = H); same workspace size (H = query
 * heads).  No reference counterpart (docs/kernels.md:177). */
int scree_attn_bwd_gqa(const void* dout, const void* q, const void* k, const void* v,
                       const void* o, const float* lse, const void* offsets, int offs_is_i64,
                       int64_t B, int64_t T, int64_t H, int64_t H_kv, int D, int dtype, int causal,
                       float scale, int64_t max_seqlen, void* dq, void* dk, void* dv,
                       void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ norms
 * RMSNorm forward over the last dim of a (rows, C) row-major buffer.
 * Replaces: scree/kernels/triton/varlen_rmsnorm.py:49-99 varlen_rmsnorm_triton
 * (kernel :17-46); numerics follow scree/kernels/reference/varlen_rmsnorm.py:58-65
 * (fp32 math, weight applied in its own precision).
 * x, y: dtype; weight: w_dtype or NULL; rstd: (rows,) fp32 or NULL (saved for
 * the backward).  x_row_stride / y_row_stride in elements. */
int scree_rmsnorm_fwd(const void* x, int64_t x_row_stride, const void* weight, int w_dtype,
                      void* y, int64_t y_row_stride, float* rstd, int64_t rows, int64_t C,
                      int dtype, float eps, void* stream);
/* RMSNorm backward (no reference counterpart: the reference has only the torch
 * autograd of reference/varlen_rmsnorm.py:50-57).  dx (rows, C) dtype; dweight
 * (C,) fp32 or NULL.  Needs scree_norm_bwd_workspace_size() bytes of workspace
 * when dweight != NULL. */
size_t scree_norm_bwd_workspace_size(int64_t rows, int64_t C);
int scree_rmsnorm_bwd(const void* dy, const void* x, const void* weight, int w_dtype,
                      const float* rstd, void* dx, float* dweight, int64_t rows, int64_t C,
                      int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* LayerNorm forward (biased variance).
 * Replaces: scree/kernels/triton/varlen_layernorm.py:52-109 varlen_layernorm_triton
 * (kernel :14-49); numerics follow reference/varlen_layernorm.py:64-74.
 * mean, rstd: (rows,) fp32 or NULL. */
int scree_layernorm_fwd(const void* x, int64_t x_row_stride, const void* weight,
                        const void* bias, int w_dtype, void* y, int64_t y_row_stride,
                        float* mean, float* rstd, int64_t rows, int64_t C, int dtype, float eps,
                        void* stream);
/* LayerNorm backward (new: reference relies on torch autograd of
 * reference/varlen_layernorm.py:53-63).  dweight / dbias (C,) fp32 or NULL. */
int scree_layernorm_bwd(const void* dy, const void* x, const void* weight, int w_dtype,
                        const float* mean, const float* rstd, void* dx, float* dweight,
                        float* dbias, int64_t rows, int64_t C, int dtype, void* workspace,
                        size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ fused pre-norm QKV
 * y = (rmsnorm(x) * gamma) @ weight in one tcgen05 GEMM: x (T, C) with row
 * stride x_row_stride (elements), weight (C, N) row-major (the reference's
 * Wqkv, used as h @ Wqkv), y (T, N) contiguous in x's dtype (fp16 / bf16), so
 * y viewed as (T, 3, H, D) gives the packed q / k / v of the attention call.
 * rstd (T,) fp32 or NULL (then kept in the workspace).  gamma (C,) in g_dtype
 * or NULL (no weight).  workspace: scree_rmsnorm_qkv_workspace_size bytes
 * (the gamma-scaled weight rows and the rstd scratch).  A row-statistics pass
 * precedes the GEMM.  C must be a multiple of 64 and N of 128.
 * Replaces the caller-side sequence of scree/examples/03_train_step.py:36-41
 * (varlen_rmsnorm then a matmul), which has no kernel of its own in the
 * reference. */
size_t scree_rmsnorm_qkv_workspace_size(int64_t T, int64_t C, int64_t N);
int scree_rmsnorm_qkv_fwd(const void* x, int64_t x_row_stride, const void* gamma, int g_dtype,
                          const void* weight, void* y, float* rstd, int64_t T, int64_t C,
                          int64_t N, int dtype, float eps, void* workspace,
                          size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ softmax
 * Varlen softmax along the ragged dimension: within each sequence, independently
 * for every feature column of the (T, F) row-major values.
 * Replaces: scree/kernels/reference/varlen_softmax.py:13-63 varlen_softmax (the
 * reference ships no GPU kernel for it).  fp32 statistics; y same dtype as x. */
int scree_softmax_fwd(const void* x, const void* offsets, int offs_is_i64, int64_t B, int64_t T,
                      int64_t F, int dtype, void* y, void* stream);
/* Its backward: dx = y * (dy - sum over the sequence's rows of dy * y), per column
 * (torch autograd of reference/varlen_softmax.py:41-48 computes the same). */
int scree_softmax_bwd(const void* dy, const void* y, const void* offsets, int offs_is_i64,
                      int64_t B, int64_t T, int64_t F, int dtype, void* dx, void* stream);

/* ------------------------------------------------------------------ gathers
 * pack: concatenate B contiguous row-major sources along rows.
 * Replaces: scree/_core.py:97-141 pack (torch branch :108-113, torch.cat).
 * src_ptrs: device array of B source pointers; offsets: device (B+1,) row
 * offsets (int64 when offs_is_i64); row_bytes = bytes of one row (prod of the
 * feature dims x element size).  src_align: a power of two dividing every
 * source address (e.g. 16 when all are 16-byte aligned).  max_rows: the longest
 * sequence (sizes the grid; <= 0 means unknown and T is used).  dst: (T, ...)
 * contiguous. */
int scree_pack(const void* const* src_ptrs, const void* offsets, int offs_is_i64, int64_t B,
               int64_t T, int64_t max_rows, int64_t row_bytes, int64_t src_align, void* dst,
               void* stream);

/* to_padded: (T, ...) packed -> (B, max_len, ...) padded + (B, max_len) mask.
 * Replaces: scree/_core.py:161-250 to_padded (torch branch :224-250).
 * side_left = 0 pads on the right, 1 on the left.  fill_pattern: host pointer
 * to elem_bytes bytes holding fill_value in the values' dtype.  mask: bool
 * (1 byte per entry) or NULL. */
int scree_to_padded(const void* values, const void* offsets, int offs_is_i64, int64_t B,
                    int64_t max_len, int64_t row_bytes, int64_t elem_bytes,
                    const void* fill_pattern_host, int side_left, void* padded, uint8_t* mask,
                    void* stream);

/* to_padded with the mask written in an integer width of 1, 2, 4 or 8 bytes
 * (1 / 0 per position): the HF attention_mask convention is int64.
 * Replaces: scree/bridges/_hf_padded.py:32-46 to_hf_padded (to_padded, then a
 * mask dtype conversion) with one kernel.  Otherwise as scree_to_padded. */
int scree_to_padded_ex(const void* values, const void* offsets, int offs_is_i64, int64_t B,
                       int64_t max_len, int64_t row_bytes, int64_t elem_bytes,
                       const void* fill_pattern_host, int side_left, void* padded, void* mask,
                       int mask_elem_bytes, void* stream);

/* KV-cache append (no reference counterpart; docs/kernels.md:178): out holds,
 * for each sequence b, its Tc-buffer rows cache[cache_offsets[b] ..
 * cache_offsets[b+1]) followed by its new rows fresh[fresh_offsets[b] ..
 * fresh_offsets[b+1]); out_offsets (B+1, int64) = cache_offsets + fresh_offsets
 * is written on the device.  out: (Tc + Tn, ...) rows of row_bytes bytes.
 * max_rows: the longest output sequence (sizes the grid; <= 0 for unknown). */
int scree_kv_append(const void* cache, const void* cache_offsets, const void* fresh,
                    const void* fresh_offsets, int offs_is_i64, int64_t B, int64_t Tc, int64_t Tn,
                    int64_t max_rows, int64_t row_bytes, void* out, int64_t* out_offsets,
                    void* stream);

/* from_padded, step 1: per-row lengths = mask.sum(1) and int32 offsets (B+1,).
 * Replaces: scree/_core.py:253-301 from_padded (torch branch :260-267), which
 * assumes right padding. */
int scree_padded_lengths(const uint8_t* mask, int64_t B, int64_t max_len, int32_t* offsets_out,
                         void* stream);
/* Step 1 for a mask of 1-, 2-, 4- or 8-byte integers (nonzero = valid), read
 * as is: the HF attention_mask is int64.
 * Replaces: scree/bridges/_hf_padded.py:15-29 from_hf_padded (mask cast to bool,
 * then from_padded). */
int scree_padded_lengths_ex(const void* mask, int mask_elem_bytes, int64_t B, int64_t max_len,
                            int32_t* offsets_out, void* stream);
/* from_padded, step 2: gather the first lengths[b] rows of each padded row into
 * the packed (T, ...) buffer, using the offsets from step 1. */
int scree_from_padded(const void* padded, const int32_t* offsets, int64_t B, int64_t max_len,
                      int64_t T, int64_t row_bytes, void* values, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SCREE_B200_H_ */
