/*
 * fk_b200.h — C ABI of the B200 (sm_100a) decode-step kernels.
 *
 * Plain pointers and sizes only; no torch or TVM types cross this boundary.
 * Every function is asynchronous on `stream` (a cudaStream_t; NULL = legacy
 * default stream), validates its arguments before launching, and returns 0 on
 * success or a negative status:
 *   -1  invalid argument (shape, alignment, null pointer)
 *   -2  unsupported configuration
 *   -3  CUDA runtime / driver error
 *   -4  a device-side bounded wait ran out (see fk_get_device_error)
 * The message of the last failure on the calling thread is fk_last_error().
 *
 * Ownership follows the reference: the caller allocates every tensor,
 * including outputs and split-KV partial buffers; kernels write in place and
 * allocate nothing (reference: python/cdsl_helpers/cdsl_fn_utils.py:38-44,
 * demo/gemm_run.py:56-59).
 *
 * Layouts are dense row-major (last dimension contiguous) unless stated.
 */
#ifndef FK_B200_H_
#define FK_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FK_B200_ABI_VERSION 1

#if defined(__GNUC__)
#define FK_API __attribute__((visibility("default")))
#else
#define FK_API
#endif

/* ---- library plumbing --------------------------------------------------- */

/* Message of the last failing call on this thread ("" if none). */
FK_API const char* fk_last_error(void);
/* FK_B200_ABI_VERSION of the loaded library. */
FK_API int fk_version(void);
/* SM count of the current device. */
FK_API int fk_num_sms(void);
/* Makes `device` current for this library on the calling thread (the library
 * links its own CUDA runtime, so a caller's cudaSetDevice in another runtime
 * instance is not assumed to carry over). */
FK_API int fk_use_device(int device);
/* Reads (and optionally clears) the device error word of the current device:
 * 0 = no error, 1/2 = a pipeline stage wait ran out, 3 = a tensor-core commit
 * wait ran out, 4 = a global-flag wait ran out. Synchronous. */
FK_API int fk_get_device_error(int* code_out, int clear);

/* ---- split-KV decode attention ------------------------------------------
 * Replaces the reference's decode attention kernel DAttn1
 * (python/cutedsl_kernels/decoding_attention/attn1.py:89-141, called as
 * DAttn1(...)(Q, K, V, O, softmax_scale)) with softmax attention over a
 * KV cache, the semantics of the reference's attention check paths
 * (attn/attempt6_epi_pipeline/attn.py:778-784, tests.py:85).
 *
 *   q            [batch, 1, num_heads_q, 128]            bf16
 *   k_cache      [batch, max_seqlen, num_heads_kv, 128]  bf16
 *   v_cache      [batch, max_seqlen, num_heads_kv, 128]  bf16
 *   cache_seqlens[batch]                                 int32 (clamped to [0, max_seqlen])
 *   o_partial    [num_splits, batch, num_heads_q, 128]   fp32  (caller scratch)
 *   lse_partial  [num_splits, batch, num_heads_q]        fp32  (caller scratch)
 *   out          [batch, 1, num_heads_q, 128]            bf16
 *   lse          [batch, num_heads_q]                    fp32, natural log
 *
 * Query head h attends kv head h / (num_heads_q / num_heads_kv); the group
 * size must be <= 8. Split s of row b covers tokens
 * [s*chunk, min((s+1)*chunk, cache_seqlens[b])) with
 * chunk = fk_dec_attn_chunk_tokens(max_seqlen, num_splits); only the first
 * ceil(len/chunk) splits of a row are written and read. A row of length 0
 * yields out = 0 and lse = -inf.
 */
FK_API int fk_dec_attn_chunk_tokens(int max_seqlen, int num_splits);

/* Pass 1: partial O (normalised per split) and natural-log LSE per split. */
FK_API int fk_dec_attn_splitkv_fwd(const void* q, const void* k_cache, const void* v_cache,
                            const int32_t* cache_seqlens, float* o_partial, float* lse_partial,
                            int batch, int max_seqlen, int num_heads_q, int num_heads_kv,
                            int head_dim, int num_splits, float softmax_scale, void* stream);

/* Pass 2: LSE-weighted merge of the splits into bf16 out and fp32 lse. */
FK_API int fk_dec_attn_combine(const float* o_partial, const float* lse_partial,
                        const int32_t* cache_seqlens, void* out, float* lse, int batch,
                        int max_seqlen, int num_heads_q, int head_dim, int num_splits,
                        void* stream);

/* Pass 1 followed by pass 2 on the same stream. */
FK_API int fk_dec_attn_fwd(const void* q, const void* k_cache, const void* v_cache,
                    const int32_t* cache_seqlens, void* out, float* lse, float* o_partial,
                    float* lse_partial, int batch, int max_seqlen, int num_heads_q,
                    int num_heads_kv, int head_dim, int num_splits, float softmax_scale,
                    void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* FK_B200_H_ */
