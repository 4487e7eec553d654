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

#include <stddef.h>
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
/* Sets the bound on every device-side wait of this library's kernels on the
 * current device, in ns (0 restores the built-in 1 s). Synchronous. Tests
 * shorten it so that a deliberately starved pipeline times out quickly. */
FK_API int fk_set_wait_limit_ns(unsigned long long ns);

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

/* Both passes with q read at a row stride: row b of q starts q_batch_stride
 * elements after row b-1 (its Hq x 128 values contiguous). Lets attention read
 * q straight out of a fused QKV projection output [B, (Hq + 2 Hkv) * 128]. */
FK_API int fk_dec_attn_fwd_ex(const void* q, long long q_batch_stride, const void* k_cache,
                              const void* v_cache, const int32_t* cache_seqlens, void* out, float* lse,
                              float* o_partial, float* lse_partial, int batch, int max_seqlen,
                              int num_heads_q, int num_heads_kv, int head_dim, int num_splits,
                              float softmax_scale, void* stream);

/* Paged KV cache: k_pool / v_pool [num_blocks, block_size, Hkv, 128] bf16 and
 * block_table [batch, max_blocks_per_seq] int32 (logical block j of row b is
 * physical block block_table[b][j]); block_size must be a multiple of 64 and
 * splits follow max_seqlen = max_blocks_per_seq * block_size. Entries past a
 * row's length are never read. Otherwise as fk_dec_attn_fwd. (The reference
 * has only a contiguous cache, decoding_attention/attn1.py:92-94.) */
FK_API int fk_dec_attn_fwd_paged(const void* q, const void* k_pool, const void* v_pool,
                                 const int32_t* block_table, const int32_t* cache_seqlens, void* out, float* lse,
                                 float* o_partial, float* lse_partial, int batch, int max_blocks_per_seq,
                                 int block_size, int num_blocks, int num_heads_q, int num_heads_kv, int head_dim,
                                 int num_splits, float softmax_scale, void* stream);

/* Both passes (contiguous cache, or paged when block_table is non-null:
 * max_seqlen = max_blocks_per_seq * block_size, num_blocks in the pool), q at
 * a row stride, and pass 2 also writes the lengths it used to
 * seqlens_commit[b] (a different array from cache_seqlens). Used after
 * fk_linear_kv_append advanced the lengths into a scratch array: attention
 * reads the scratch and publishes it to the caller's length array, so the
 * decode step needs no separate append or copy kernel. */
FK_API int fk_dec_attn_fwd_commit(const void* q, long long q_batch_stride, const void* k_cache,
                                  const void* v_cache, const int32_t* block_table, const int32_t* cache_seqlens,
                                  int32_t* seqlens_commit, void* out, float* lse, float* o_partial,
                                  float* lse_partial, int batch, int max_seqlen, int block_size, int num_blocks,
                                  int num_heads_q, int num_heads_kv, int head_dim, int num_splits,
                                  float softmax_scale, void* stream);

/* Single-launch decode attention: pass 2 folded into pass 1. Every unit
 * (row, kv head, split) writes its partial; the last unit of a (row, kv head)
 * to finish, found by an atomic count per pair, merges that pair's splits in
 * split order and writes out / lse (the same bits as fk_dec_attn_fwd). Rows
 * with one split write out / lse directly and touch no partials. No unit waits
 * on another. Covers every variant of the two-pass entries: q at a row stride
 * (q_batch_stride, elements); a paged cache when block_table is non-null
 * (max_seqlen = max_blocks_per_seq * block_size); seqlens_commit (optional,
 * receives cache_seqlens[b] once row b is done); npeers <= 7 copies of each
 * out row at peer_out[i] (other GPUs' buffers, same offsets).
 *   counters  [batch * num_heads_kv] int32, zero before the first call; each
 *             call leaves them zero again. Calls that may overlap on the GPU
 *             need their own counters.
 * Replaces the reference's decode-attention pair dec_attn_run /
 * dec_attn_second_part (demo/dec_attn_run.py:45-46,
 * demo/dec_attn_second_part.py:17-43) in one launch. */
FK_API int fk_dec_attn_fwd_fused(const void* q, long long q_batch_stride, const void* k_cache,
                                 const void* v_cache, const int32_t* block_table, const int32_t* cache_seqlens,
                                 int32_t* seqlens_commit, void* out, void* const* peer_out, int npeers, float* lse,
                                 float* o_partial, float* lse_partial, int32_t* counters, int batch,
                                 int max_seqlen, int block_size, int num_blocks, int num_heads_q,
                                 int num_heads_kv, int head_dim, int num_splits, float softmax_scale,
                                 void* stream);

/* Test hook: CTA 0 of every later decode-attention launch skips issuing its
 * tile number `tile` (a stage that never fills), so its consumers' bounded
 * waits run out; -1 turns it off. Host-side setting, no GPU work. */
FK_API int fk_debug_attn_withhold_tile(int tile);

/* Paged form of fk_kv_append: the new row of b goes to block
 * block_table[b][len / block_size], row len % block_size (any block_size >= 1). */
FK_API int fk_kv_append_paged(const void* src, long long src_row_stride, int k_col, int v_col, void* k_pool,
                              void* v_pool, const int32_t* block_table, const int32_t* cache_seqlens,
                              int32_t* seqlens_out, int batch, int max_blocks_per_seq, int block_size,
                              int num_heads_kv, int head_dim, void* stream);

/* KV-cache append: for each row b with 0 <= cache_seqlens[b] < max_seqlen,
 * copy the new K row (src + b*src_row_stride + k_col, num_heads_kv*head_dim
 * bf16) and V row (… + v_col) into k_cache/v_cache[b, cache_seqlens[b]] and
 * write seqlens_out[b] = cache_seqlens[b] + 1 (rows already full are left
 * alone and keep their length). seqlens_out may alias cache_seqlens or be
 * null. Counterpart of the cache write of the reference's DAttn2
 * (python/cutedsl_kernels/decoding_attention/attempt2.py:276-286). */
FK_API int fk_kv_append(const void* src, long long src_row_stride, int k_col, int v_col, void* k_cache,
                        void* v_cache, const int32_t* cache_seqlens, int32_t* seqlens_out, int batch,
                        int max_seqlen, int num_heads_kv, int head_dim, void* stream);

/* Reference-semantics decode attention of DAttn1
 * (python/cutedsl_kernels/decoding_attention/attn1.py:89-141, called as
 * DAttn1(qk_mnk, stages, p_stages, is_persistent)(Q, K, V, O, softmax_scale)):
 *   O[h] = bf16( bf16(Q[h] K[h]^T) V[h]^T ), no softmax, no scale
 * Q [H, seq_q <= 16, 128], K [H, P, 128], v_t = V stored transposed [H, 128, P],
 * O [H, seq_q, 128], all bf16; P % 8 == 0. */
FK_API int fk_dattn1(const void* q, const void* k, const void* v_t, void* out, int num_heads, int seq_q,
                     int seqlen_kv, int head_dim, void* stream);

/* Head-major scatter of the three outputs of a QKV projection, the layout step
 * of the reference's DAttn2 (python/cutedsl_kernels/decoding_attention/attempt2.py:270-286;
 * check demo/dec_attn_run.py:51-63): with q/k/v_src [M, H*D],
 *   q_out[h][m][d] = q_src[m][h*D + d],
 *   k_cache[h][cache_len - M + m][d] = k_src[m][h*D + d] (and v likewise),
 * q_out [H, M, D], caches [H, cache_len, D]; all bf16, 16-byte aligned. */
FK_API int fk_qkv_head_scatter(const void* q_src, const void* k_src, const void* v_src, void* q_out,
                               void* k_cache, void* v_cache, int M, int num_heads, int head_dim, int cache_len,
                               void* stream);

/* ---- linear family: y[M, N] = epilogue(x[M, K] . W[N, K]^T) ---------------
 * x bf16 [M, K] (K % 8 == 0, 16-byte aligned), W bf16 [N, K] (row = output
 * feature), y bf16 [M, N], fp32 accumulation. M <= 16 runs the persistent
 * stream-K weight-streaming kernel (mma.sync, W as the M side); M > 16 runs
 * the tcgen05/TMEM kernel (token tiles of up to 256).
 *
 * `workspace` is caller scratch for the stream-K split partials and per-row-
 * block counters: at least fk_linear_workspace_bytes(...) bytes, 256-byte
 * aligned, ZERO-FILLED before its first use. Every call leaves the counters
 * at zero again, so one workspace serves any number of calls in stream
 * order; calls that overlap on the GPU need separate workspaces.
 */
#define FK_LINEAR_SWIGLU 1

FK_API int fk_linear_workspace_bytes(int M, int N, int K, int flags, size_t* bytes_out);

/* General form. gamma (bf16 [K]) non-null => RMSNorm of x (with eps) fused in;
 * w_up non-null => SwiGLU: y = silu(x.W[n]) * (x.W_up[up_row_offset + n]);
 * residual (bf16 [M, N]) non-null => added in the epilogue (may alias y). */
FK_API int fk_linear(const void* x, const void* gamma, const void* w, const void* w_up,
                     int up_row_offset, const void* residual, void* y, int M, int N, int K,
                     float eps, void* workspace, size_t workspace_bytes, void* stream);

/* y = x W^T. Replaces Gemm4SM90(...)(a, b, c)
 * (python/cutedsl_kernels/gemm/kernel/attempt4.py:133-168; check demo/gemm_run.py:29). */
FK_API int fk_skinny_gemm(const void* x, const void* w, void* y, int M, int N, int K,
                          void* workspace, size_t workspace_bytes, void* stream);

/* y = rms_norm(x, gamma, eps) W^T. Replaces RMSNormLinear1SM90(...)(a, b, c, stream)
 * (python/cutedsl_kernels/rmsnorm_linear/attempt1/gemm.py:136-170, check :721-722),
 * adding the gain gamma. */
FK_API int fk_rmsnorm_linear(const void* x, const void* gamma, const void* w, void* y, int M,
                             int N, int K, float eps, void* workspace, size_t workspace_bytes,
                             void* stream);

/* y[M, N] = silu(x Wg^T) * (x Wu^T) with w_gate_up = [Wg; Wu] of shape [2N, K]
 * (demo/swiglu.py:47-49 `(a @ bb1.t()).chunk(2)`). */
FK_API int fk_swiglu_gemm(const void* x, const void* w_gate_up, void* y, int M, int N, int K,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Two-weight form: replaces Swiglu2SM90(...)(a, b, b1, c)
 * (python/cutedsl_kernels/swiglu/attempt1/gemm2.py:145-187, check :714-717). */
FK_API int fk_swiglu_gemm2(const void* x, const void* w_gate, const void* w_up, void* y, int M,
                           int N, int K, void* workspace, size_t workspace_bytes, void* stream);

/* RMSNorm -> gate/up projection -> SwiGLU in one kernel (the FFN input of the
 * decode layer). */
FK_API int fk_rmsnorm_swiglu(const void* x, const void* gamma, const void* w_gate_up, void* y,
                             int M, int N, int K, float eps, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Prefill attention O = softmax(Q K^T * softmax_scale) V on the tensor cores:
 * q / out [batch, num_heads_q, seqlen_q, head_dim], k / v [batch, num_heads_kv,
 * seqlen_kv, head_dim] bf16 contiguous (q head h reads kv head
 * h / (num_heads_q / num_heads_kv)), head_dim 64 or 128, no mask. lse (may be
 * null) [batch, num_heads_q, seqlen_q] fp32 natural-log logsumexp of the
 * scaled scores. Replaces FlashSM90(...)(mQ, mK, mV, mO, softmax_scale, stream)
 * of python/cutedsl_kernels/attn/attempt6_epi_pipeline/attn.py:73-175
 * (checked against F.scaled_dot_product_attention, tests.py:85). */
FK_API int fk_prefill_attn_fwd(const void* q, const void* k, const void* v, void* out, float* lse, int batch,
                               int num_heads_q, int num_heads_kv, int seqlen_q, int seqlen_kv, int head_dim,
                               float softmax_scale, void* stream);

/* LoRA linear: y[M, N] = x W^T + xA B^T (+ residual when non-null), with
 * xA = x A^T given as [M, rank] and B as [N, rank] (rank a multiple of 8).
 * Replaces GemmSM90(...)(a, b, lora_xA, lora_B, c, stream) of
 * python/cutedsl_kernels/lora/attempt1/gemm.py:136-178 (check :672-675:
 * (a @ b.t()) + (a @ lA.t() @ lB.t())). The low-rank term is extra k blocks
 * of the same accumulation, rounded to bf16 once. Workspace as fk_linear. */
FK_API int fk_lora_linear(const void* x, const void* w, const void* lora_xa, const void* lora_b,
                          const void* residual, void* y, int M, int N, int K, int rank, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Projection (RMSNorm -> linear when gamma is non-null, else plain) whose
 * epilogue also appends the new K/V rows to the cache: output columns
 * [k_col, k_col + num_heads_kv*head_dim) of token m go to the K cache at
 * position cache_seqlens[m], [v_col, ...) to the V cache, and seqlens_next[m]
 * (a different array from cache_seqlens, may be null) receives the advanced
 * length; rows already at max_seqlen keep their length and are not written.
 * block_table null: caches [M, max_seqlen, Hkv, D]; else block pools
 * [*, block_size, Hkv, D] with max_seqlen = max_blocks_per_seq * block_size.
 * The fused form of DAttn2's projection + cache write
 * (python/cutedsl_kernels/decoding_attention/attempt2.py:98-302, write :276-286). */
FK_API int fk_linear_kv_append(const void* x, const void* gamma, const void* w, void* y, int M, int N, int K,
                               float eps, void* k_cache, void* v_cache, const int32_t* block_table,
                               const int32_t* cache_seqlens, int32_t* seqlens_next, int k_col, int v_col,
                               int num_heads_kv, int head_dim, int max_seqlen, int block_size, void* workspace,
                               size_t workspace_bytes, void* stream);

/* ---- tensor-parallel decode step over peer memory (one process per GPU) ----
 * A column-parallel GEMM writes its output block into the full activation
 * buffer of every rank from its epilogue (plain stores through CUDA IPC
 * mappings), and fk_peer_barrier orders the ranks between stages: together they
 * replace the all-gather + re-layout of an NCCL layer. */

/* fk_linear with output placement: y rows ldy (0: N) elements apart, residual
 * rows ldr (0: N) apart, and npeers (<= 7) more copies of y at peer_y[i] (other
 * GPUs' buffers, same offsets). */
FK_API int fk_linear_ex(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
                        const void* residual, int ldr, void* y, int ldy, void* const* peer_y, int npeers, int M,
                        int N, int K, float eps, void* workspace, size_t workspace_bytes, void* stream);

/* fk_dec_attn_fwd_ex whose pass 2 also writes each output row to peer_out[i]
 * (npeers <= 7 other GPUs' buffers, same offsets): the all-gather of a
 * batch-sharded attention output. */
FK_API int fk_dec_attn_fwd_peers(const void* q, long long q_batch_stride, const void* k_cache, const void* v_cache,
                                 const int32_t* cache_seqlens, void* out, void* const* peer_out, int npeers,
                                 float* lse, float* o_partial, float* lse_partial, int batch, int max_seqlen,
                                 int num_heads_q, int num_heads_kv, int head_dim, int num_splits,
                                 float softmax_scale, void* stream);

/* Zero-filled device buffer that can be shared through CUDA IPC, and its release. */
FK_API int fk_peer_alloc(size_t bytes, void** ptr_out);
FK_API int fk_peer_free(void* ptr);
/* Size of an IPC handle; export a buffer's handle; map / unmap a peer's buffer. */
FK_API int fk_ipc_handle_bytes(void);
FK_API int fk_ipc_get_handle(void* ptr, void* handle_out);
FK_API int fk_ipc_open(const void* handle, void** ptr_out);
FK_API int fk_ipc_close(void* ptr);

/* Stage barrier among nranks GPUs: one thread advances *counter to seq, fences
 * at system scope (ordering every earlier write of this stream, peer stores
 * included), stores seq into peer_flags[r][rank] for every r != rank and waits
 * (at most 1 s, then the device error word is set) until local_flags[r] >= seq
 * for every r != rank. counter and local_flags live in this GPU's memory;
 * peer_flags[r] is rank r's flags array mapped here. */
FK_API int fk_peer_barrier(int32_t* counter, int32_t* local_flags, int32_t* const* peer_flags, int rank,
                           int nranks, void* stream);

/* The two halves of fk_peer_barrier, for a barrier whose wait is done by the
 * kernel that consumes the stage. fk_peer_signal: one thread advances *counter
 * to seq, fences at system scope and stores seq into peer_flags[r][rank] for
 * every r != rank; it does not wait. The next launch on the stream then waits
 * (bounded, 1 s) until local flags[r] >= *counter for every peer before it
 * reads data the peers wrote: fk_linear_ex_wait (in the kernel that loads x:
 * the GEMM's token-load warp, or the RMSNorm prologue) and fk_kv_append_wait.
 * Otherwise as fk_linear_ex / fk_kv_append. Removes the separate waiting kernel
 * between stages: the wait overlaps the next GEMM's weight prefetch. */
FK_API int fk_peer_signal(int32_t* counter, int32_t* const* peer_flags, int rank, int nranks, void* stream);
FK_API int fk_linear_ex_wait(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
                             const void* residual, int ldr, void* y, int ldy, void* const* peer_y, int npeers, int M,
                             int N, int K, float eps, void* workspace, size_t workspace_bytes,
                             const int32_t* wait_counter, const int32_t* wait_flags, int rank, int nranks,
                             void* stream);
FK_API int fk_kv_append_wait(const void* src, long long src_row_stride, int k_col, int v_col, void* k_cache,
                             void* v_cache, const int32_t* cache_seqlens, int32_t* seqlens_out, int batch,
                             int max_seqlen, int num_heads_kv, int head_dim, const int32_t* wait_counter,
                             const int32_t* wait_flags, int rank, int nranks, void* stream);

/* Skinny GEMM y = x W^T (1 <= M <= 16, N <= 524288) that allocates nothing:
 * its stream-K scratch is a fixed ~2.7 MB device array inside this library
 * (one per GPU, kept until process exit) instead of a caller workspace. For
 * callers that cannot allocate GPU memory while they run (a runtime that owns
 * every allocation, plain-C callers without an allocator). No counterpart in
 * the reference. The first call on a device looks up the array's address; make
 * it before any stream capture. All calls share the array: calls that may
 * overlap on the GPU race, so order them on one stream. */
FK_API int fk_skinny_gemm_noalloc(const void* x, const void* w, void* y, int M, int N, int K,
                                  void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* FK_B200_H_ */
