// TVM-FFI entry points over the C ABI of libfk_b200 (include/fk_b200.h).
//
// The reference requires its kernels to be TVM-FFI functions taking torch
// tensors (README.md:1; compiled with `--enable-tvm-ffi`,
// python/cdsl_helpers/cdsl_fn_utils.py:38-44). This module provides that
// surface for the sm_100a kernels: every function takes DLPack tensor views
// (torch tensors pass straight through tvm_ffi), launches on the environment
// stream of the tensors' device (TVMFFIEnvGetStream, the current torch stream
// when called from torch) and raises ValueError / RuntimeError with the
// library's message on a bad status. Outputs and scratch are caller-allocated.
#include <tvm/ffi/container/tensor.h>
#include <tvm/ffi/error.h>
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/function.h>

#include <cmath>
#include <string>

#include "fk_b200.h"

namespace {

using tvm::ffi::TensorView;

void* stream_of(const TensorView& t) {
  return TVMFFIEnvGetStream(t.device().device_type, t.device().device_id);
}

void check(int rc) {
  if (rc == 0) return;
  const std::string msg = fk_last_error();
  if (rc == -1) TVM_FFI_THROW(ValueError) << msg;
  TVM_FFI_THROW(RuntimeError) << "libfk_b200 status " << rc << ": " << msg;
}

void use(const TensorView& t) { check(fk_use_device(t.device().device_id)); }

size_t nbytes(const TensorView& t) {
  size_t n = (t.dtype().bits + 7) / 8;
  for (int i = 0; i < t.ndim(); ++i) n *= static_cast<size_t>(t.size(i));
  return n;
}

void require(bool ok, const char* msg) {
  if (!ok) TVM_FFI_THROW(ValueError) << msg;
}

// ---- split-KV decode attention -------------------------------------------
void dec_attn_splitkv_fwd(TensorView q, TensorView k_cache, TensorView v_cache, TensorView cache_seqlens,
                          TensorView out, TensorView lse, TensorView o_partial, TensorView lse_partial,
                          int64_t num_splits, double softmax_scale) {
  require(k_cache.ndim() == 4, "k_cache must be [B, Lmax, Hkv, D]");
  use(q);
  const int B = (int)k_cache.size(0), L = (int)k_cache.size(1), Hkv = (int)k_cache.size(2);
  const int D = (int)k_cache.size(3);
  const int Hq = (int)(q.ndim() == 4 ? q.size(2) : q.size(1));
  const float scale = softmax_scale > 0 ? (float)softmax_scale : 1.0f / std::sqrt((float)D);
  check(fk_dec_attn_fwd(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                        static_cast<const int32_t*>(cache_seqlens.data_ptr()), out.data_ptr(),
                        static_cast<float*>(lse.data_ptr()), static_cast<float*>(o_partial.data_ptr()),
                        static_cast<float*>(lse_partial.data_ptr()), B, L, Hq, Hkv, D, (int)num_splits, scale,
                        stream_of(q)));
}

void dec_attn_combine(TensorView o_partial, TensorView lse_partial, TensorView cache_seqlens, TensorView out,
                      TensorView lse, int64_t max_seqlen) {
  require(o_partial.ndim() == 4, "o_partial must be [S, B, Hq, D]");
  use(o_partial);
  check(fk_dec_attn_combine(static_cast<const float*>(o_partial.data_ptr()),
                            static_cast<const float*>(lse_partial.data_ptr()),
                            static_cast<const int32_t*>(cache_seqlens.data_ptr()), out.data_ptr(),
                            static_cast<float*>(lse.data_ptr()), (int)o_partial.size(1), (int)max_seqlen,
                            (int)o_partial.size(2), (int)o_partial.size(3), (int)o_partial.size(0),
                            stream_of(o_partial)));
}

void dattn1(TensorView Q, TensorView K, TensorView V, TensorView O, double softmax_scale) {
  (void)softmax_scale;  // unused, as in the reference kernel
  use(Q);
  check(fk_dattn1(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), (int)Q.size(0), (int)Q.size(1),
                  (int)K.size(1), (int)Q.size(2), stream_of(Q)));
}

// Prefill attention with FlashSM90's call shape (mQ, mK, mV, mO, softmax_scale):
// [b, h, seqlen, d] tensors, d 64 or 128, k/v may have fewer heads than q.
void prefill_attn(TensorView q, TensorView k, TensorView v, TensorView o, double softmax_scale) {
  require(q.ndim() == 4 && k.ndim() == 4 && v.ndim() == 4 && o.ndim() == 4, "tensors must be [b, h, seqlen, d]");
  use(q);
  check(fk_prefill_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), nullptr, (int)q.size(0),
                            (int)q.size(1), (int)k.size(1), (int)q.size(2), (int)k.size(2), (int)q.size(3),
                            (float)softmax_scale, stream_of(q)));
}

// DAttn2's call (X, Wq, Wk, Wv, Q_out, K_cache, V_cache) plus caller scratch:
// tmp [3, M, H*D] bf16 for the three projections and a linear-family workspace.
// Q_out [H, M, D] gets the head-major queries, K/V_cache [H, P, D] the new rows
// at [P - M, P) (decoding_attention/attempt2.py:77-99, 276-286).
void dattn2(TensorView x, TensorView wq, TensorView wk, TensorView wv, TensorView q_out, TensorView k_cache,
            TensorView v_cache, TensorView tmp, TensorView workspace) {
  require(x.ndim() == 2 && q_out.ndim() == 3 && k_cache.ndim() == 3 && v_cache.ndim() == 3 && tmp.ndim() == 3,
          "X [M, H*D], Q_out [H, M, D], caches [H, P, D], tmp [3, M, H*D]");
  use(x);
  const int M = (int)x.size(0), HD = (int)x.size(1);
  const int H = (int)q_out.size(0), D = (int)q_out.size(2), P = (int)k_cache.size(1);
  require(H * D == HD && (int)q_out.size(1) == M, "Q_out must be [H, M, D] with H * D = X's features");
  require((int)tmp.size(0) == 3 && (int)tmp.size(1) == M && (int)tmp.size(2) == HD, "tmp must be [3, M, H*D]");
  void* st = stream_of(x);
  char* t = static_cast<char*>(tmp.data_ptr());
  const size_t plane = (size_t)M * HD * 2;
  const TensorView* ws[3] = {&wq, &wk, &wv};
  for (int i = 0; i < 3; ++i)
    check(fk_skinny_gemm(x.data_ptr(), ws[i]->data_ptr(), t + i * plane, M, HD, HD, workspace.data_ptr(),
                         nbytes(workspace), st));
  check(fk_qkv_head_scatter(t, t + plane, t + 2 * plane, q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), M,
                            H, D, P, st));
}

// ---- linear family (x [M, K], w [N, K], y [M, N]; workspace zero-filled) ---
void skinny_gemm(TensorView x, TensorView w, TensorView y, TensorView workspace) {
  use(x);
  check(fk_skinny_gemm(x.data_ptr(), w.data_ptr(), y.data_ptr(), (int)x.size(0), (int)w.size(0), (int)x.size(1),
                       workspace.data_ptr(), nbytes(workspace), stream_of(x)));
}

void rmsnorm_linear(TensorView x, TensorView gamma, TensorView w, TensorView y, double eps, TensorView workspace) {
  use(x);
  check(fk_rmsnorm_linear(x.data_ptr(), gamma.data_ptr(), w.data_ptr(), y.data_ptr(), (int)x.size(0),
                          (int)w.size(0), (int)x.size(1), (float)eps, workspace.data_ptr(), nbytes(workspace),
                          stream_of(x)));
}

void swiglu_gemm(TensorView x, TensorView w_gate_up, TensorView y, TensorView workspace) {
  use(x);
  check(fk_swiglu_gemm(x.data_ptr(), w_gate_up.data_ptr(), y.data_ptr(), (int)x.size(0),
                       (int)(w_gate_up.size(0) / 2), (int)x.size(1), workspace.data_ptr(), nbytes(workspace),
                       stream_of(x)));
}

void swiglu_gemm2(TensorView x, TensorView b, TensorView b1, TensorView y, TensorView workspace) {
  use(x);
  check(fk_swiglu_gemm2(x.data_ptr(), b.data_ptr(), b1.data_ptr(), y.data_ptr(), (int)x.size(0), (int)b.size(0),
                        (int)x.size(1), workspace.data_ptr(), nbytes(workspace), stream_of(x)));
}

// LoRA GEMM with the reference's call shape (a, b, lora_xA, lora_B, c): c = a b^T + lora_xA lora_B^T.
void lora_gemm(TensorView x, TensorView w, TensorView lora_xa, TensorView lora_b, TensorView y, TensorView workspace) {
  use(x);
  check(fk_lora_linear(x.data_ptr(), w.data_ptr(), lora_xa.data_ptr(), lora_b.data_ptr(), nullptr, y.data_ptr(),
                       (int)x.size(0), (int)w.size(0), (int)x.size(1), (int)lora_b.size(1), workspace.data_ptr(),
                       nbytes(workspace), stream_of(x)));
}

// ---- reference call shapes without a workspace argument ---------------------
// The reference's compiled kernels take only their operands (Gemm4SM90(...)(a, b, c),
// Swiglu2SM90(...)(a, b, b1, c)); their split-K scratch lives here instead: one
// zeroed buffer per device from fk_peer_alloc, grown when a call needs more and
// kept until exit. Every call leaves the buffer's counters zero again, so
// calls ordered on one stream share it; calls on concurrent streams must use
// the explicit-workspace functions.
void* module_workspace(int device, size_t need, size_t* have) {
  static void* bufs[64] = {};
  static size_t sizes[64] = {};
  require(device >= 0 && device < 64, "device index out of range");
  if (sizes[device] < need) {
    if (bufs[device]) check(fk_peer_free(bufs[device]));
    bufs[device] = nullptr;
    sizes[device] = 0;
    void* p = nullptr;
    const size_t n = need < ((size_t)16 << 20) ? ((size_t)16 << 20) : need;
    check(fk_peer_alloc(n, &p));
    bufs[device] = p;
    sizes[device] = n;
  }
  *have = sizes[device];
  return bufs[device];
}

void gemm(TensorView a, TensorView b, TensorView c) {
  use(a);
  const int M = (int)a.size(0), N = (int)b.size(0), K = (int)a.size(1);
  size_t need = 0, have = 0;
  check(fk_linear_workspace_bytes(M, N, K, 0, &need));
  void* ws = module_workspace(a.device().device_id, need, &have);
  check(fk_linear(a.data_ptr(), nullptr, b.data_ptr(), nullptr, 0, nullptr, c.data_ptr(), M, N, K, 0.f, ws, have,
                  stream_of(a)));
}

// The tcgen05 path by name (M > 16 tokens), explicit workspace.
void gemm_tc(TensorView x, TensorView w, TensorView y, TensorView workspace) {
  require(x.size(0) > 16, "gemm_tc takes M > 16 tokens (M <= 16 runs the weight-streaming path: skinny_gemm)");
  use(x);
  check(fk_linear(x.data_ptr(), nullptr, w.data_ptr(), nullptr, 0, nullptr, y.data_ptr(), (int)x.size(0),
                  (int)w.size(0), (int)x.size(1), 0.f, workspace.data_ptr(), nbytes(workspace), stream_of(x)));
}

void swiglu2(TensorView a, TensorView b, TensorView b1, TensorView c) {
  use(a);
  const int M = (int)a.size(0), N = (int)b.size(0), K = (int)a.size(1);
  size_t need = 0, have = 0;
  check(fk_linear_workspace_bytes(M, N, K, FK_LINEAR_SWIGLU, &need));
  void* ws = module_workspace(a.device().device_id, need, &have);
  check(fk_swiglu_gemm2(a.data_ptr(), b.data_ptr(), b1.data_ptr(), c.data_ptr(), M, N, K, ws, have, stream_of(a)));
}

// Single-launch decode attention: partial slots = o_partial.size(0) (>= 2);
// counters int32 [B * Hkv], zero, left zero.
void dec_attn_fused(TensorView q, TensorView k_cache, TensorView v_cache, TensorView cache_seqlens, TensorView out,
                    TensorView lse, TensorView o_partial, TensorView lse_partial, TensorView counters,
                    double softmax_scale) {
  require(k_cache.ndim() == 4, "k_cache must be [B, Lmax, Hkv, D]");
  use(q);
  const int B = (int)k_cache.size(0), L = (int)k_cache.size(1), Hkv = (int)k_cache.size(2);
  const int D = (int)k_cache.size(3);
  const int Hq = (int)(q.ndim() == 4 ? q.size(2) : q.size(1));
  const float scale = softmax_scale > 0 ? (float)softmax_scale : 1.0f / std::sqrt((float)D);
  check(fk_dec_attn_fwd_fused(q.data_ptr(), (long long)Hq * D, k_cache.data_ptr(), v_cache.data_ptr(), nullptr,
                              static_cast<const int32_t*>(cache_seqlens.data_ptr()), nullptr, out.data_ptr(), nullptr,
                              0, static_cast<float*>(lse.data_ptr()), static_cast<float*>(o_partial.data_ptr()),
                              static_cast<float*>(lse_partial.data_ptr()), static_cast<int32_t*>(counters.data_ptr()),
                              B, L, 0, 0, Hq, Hkv, D, (int)o_partial.size(0), scale, stream_of(q)));
}

// Paged single-launch decode attention: k_pool / v_pool [num_blocks, block_size, Hkv, D],
// block_table [B, max_blocks] int32.
void dec_attn_paged(TensorView q, TensorView k_pool, TensorView v_pool, TensorView block_table,
                    TensorView cache_seqlens, TensorView out, TensorView lse, TensorView o_partial,
                    TensorView lse_partial, TensorView counters, double softmax_scale) {
  require(k_pool.ndim() == 4 && block_table.ndim() == 2, "k_pool [NB, BS, Hkv, D], block_table [B, max_blocks]");
  use(q);
  const int NB = (int)k_pool.size(0), BS = (int)k_pool.size(1), Hkv = (int)k_pool.size(2), D = (int)k_pool.size(3);
  const int B = (int)block_table.size(0), MB = (int)block_table.size(1);
  const int Hq = (int)(q.ndim() == 4 ? q.size(2) : q.size(1));
  const float scale = softmax_scale > 0 ? (float)softmax_scale : 1.0f / std::sqrt((float)D);
  check(fk_dec_attn_fwd_fused(q.data_ptr(), (long long)Hq * D, k_pool.data_ptr(), v_pool.data_ptr(),
                              static_cast<const int32_t*>(block_table.data_ptr()),
                              static_cast<const int32_t*>(cache_seqlens.data_ptr()), nullptr, out.data_ptr(), nullptr,
                              0, static_cast<float*>(lse.data_ptr()), static_cast<float*>(o_partial.data_ptr()),
                              static_cast<float*>(lse_partial.data_ptr()), static_cast<int32_t*>(counters.data_ptr()),
                              B, MB * BS, BS, NB, Hq, Hkv, D, (int)o_partial.size(0), scale, stream_of(q)));
}

// RMSNorm -> QKV projection whose epilogue appends the new K/V rows at
// cache_seqlens[m] (contiguous caches [M, Lmax, Hkv, D]) and writes the advanced
// lengths to seqlens_next. y [M, (Hq + 2 Hkv) * D]: q columns, then k, then v.
void linear_kv_append(TensorView x, TensorView gamma, TensorView w, TensorView y, TensorView k_cache,
                      TensorView v_cache, TensorView cache_seqlens, TensorView seqlens_next, int64_t num_heads_q,
                      double eps, TensorView workspace) {
  require(k_cache.ndim() == 4, "k_cache must be [M, Lmax, Hkv, D]");
  use(x);
  const int Hkv = (int)k_cache.size(2), D = (int)k_cache.size(3);
  check(fk_linear_kv_append(x.data_ptr(), gamma.data_ptr(), w.data_ptr(), y.data_ptr(), (int)x.size(0),
                            (int)w.size(0), (int)x.size(1), (float)eps, k_cache.data_ptr(), v_cache.data_ptr(),
                            nullptr, static_cast<const int32_t*>(cache_seqlens.data_ptr()),
                            static_cast<int32_t*>(seqlens_next.data_ptr()), (int)num_heads_q * D,
                            (int)(num_heads_q + Hkv) * D, Hkv, D, (int)k_cache.size(1), 0, workspace.data_ptr(),
                            nbytes(workspace), stream_of(x)));
}

int64_t linear_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t swiglu) {
  size_t b = 0;
  check(fk_linear_workspace_bytes((int)M, (int)N, (int)K, swiglu ? FK_LINEAR_SWIGLU : 0, &b));
  return (int64_t)b;
}

}  // namespace

TVM_FFI_DLL_EXPORT_TYPED_FUNC(dec_attn_splitkv_fwd, dec_attn_splitkv_fwd);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(dec_attn_combine, dec_attn_combine);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(dattn1, dattn1);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(prefill_attn, prefill_attn);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(dattn2, dattn2);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(skinny_gemm, skinny_gemm);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(rmsnorm_linear, rmsnorm_linear);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(swiglu_gemm, swiglu_gemm);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(swiglu_gemm2, swiglu_gemm2);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(lora_gemm, lora_gemm);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(linear_workspace_bytes, linear_workspace_bytes);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(gemm, gemm);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(gemm_tc, gemm_tc);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(swiglu2, swiglu2);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(dec_attn_fused, dec_attn_fused);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(dec_attn_paged, dec_attn_paged);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(linear_kv_append, linear_kv_append);
