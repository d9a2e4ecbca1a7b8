// extern "C" entry points: argument checks and dispatch to the kernels.
#include "common.cuh"
#include "kernels.h"

using namespace ck;

namespace {
inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }
}  // namespace

namespace ck {

int linear_dispatch(const void* A, int dtype, int64_t M, int64_t K, int64_t lda, const void* W,
                    int w_dtype, int w_layout, int64_t N, int64_t ldw, const float* w_scale,
                    int epi, const void* aux, int64_t ld_aux, int64_t aux_row_mod, void* Y,
                    int64_t ldy, cudaStream_t st, bool w_static) {
  if (M < 0 || N < 0 || K < 0) return CK_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return CK_OK;
  if (!A || !W || !Y) return CK_ERR_INVALID_ARG;
  if (epi < CK_EPI_STORE || epi > CK_EPI_BIAS) return CK_ERR_INVALID_ARG;
  if ((epi == CK_EPI_RESID || epi == CK_EPI_BIAS) && aux == nullptr) return CK_ERR_INVALID_ARG;
  if (w_layout != CK_W_NK && w_layout != CK_W_KN) return CK_ERR_INVALID_ARG;
  if (w_dtype != dtype && w_dtype != CK_I8) return CK_ERR_UNSUPPORTED;
  if (w_dtype == CK_I8 && (w_scale == nullptr || w_layout != CK_W_NK)) return CK_ERR_INVALID_ARG;
  if (dtype == CK_BF16 && gemm_tc_supported(M, K, lda, w_dtype, w_layout, N, ldw, A, W, ldy, Y,
                                            epi, aux, ld_aux)) {
    GemmFusion fz;
    fz.w_static = w_static;
    return gemm_tc(A, M, K, lda, W, w_dtype, w_layout, N, ldw, w_scale, epi, aux, ld_aux,
                   aux_row_mod, Y, ldy, st, w_static ? &fz : nullptr);
  }
  return gemm_simt(A, dtype, M, K, lda, W, w_dtype, w_layout, N, ldw, w_scale, epi, aux, ld_aux,
                   aux_row_mod, Y, ldy, st);
}

bool norm_linear_fused(int dtype, int64_t M, int64_t K, int64_t ldx, const void* x,
                       const void* gamma, int norm_mode, const void* W, int w_dtype,
                       int w_layout, int64_t N, int64_t ldw, int epi, const void* aux,
                       int64_t ld_aux, const void* Y, int64_t ldy) {
  return norm_mode == CK_NORM_RMS && dtype == CK_BF16 && gamma != nullptr && K % 8 == 0 &&
         (reinterpret_cast<uintptr_t>(gamma) & 15u) == 0 &&
         (epi == CK_EPI_STORE || epi == CK_EPI_BIAS) && (w_dtype == CK_BF16 || w_dtype == CK_I8) &&
         gemm_tc_supported(M, K, ldx, w_dtype, w_layout, N, ldw, x, W, ldy, Y, epi, aux, ld_aux);
}

int norm_linear(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx, const void* gamma,
                const void* beta, float eps, int norm_mode, const void* W, int w_dtype,
                int w_layout, int64_t N, int64_t ldw, const float* w_scale, int epi,
                const void* aux, int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy,
                void* workspace, size_t workspace_bytes, cudaStream_t st) {
  if (norm_mode == CK_NORM_NONE)
    return linear_dispatch(x, dtype, M, K, ldx, W, w_dtype, w_layout, N, ldw, w_scale, epi, aux,
                           ld_aux, aux_row_mod, Y, ldy, st);
  if (norm_mode != CK_NORM_LAYER && norm_mode != CK_NORM_RMS) return CK_ERR_INVALID_ARG;
  if (M < 0 || N < 0 || K <= 0) return CK_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return CK_OK;
  if (!x || !gamma || !W || !Y) return CK_ERR_INVALID_ARG;
  if (epi < CK_EPI_STORE || epi > CK_EPI_BIAS) return CK_ERR_INVALID_ARG;
  if ((epi == CK_EPI_RESID || epi == CK_EPI_BIAS) && aux == nullptr) return CK_ERR_INVALID_ARG;
  if (w_dtype == CK_I8 && (w_scale == nullptr || w_layout != CK_W_NK)) return CK_ERR_INVALID_ARG;
  // RMSNorm with bf16 activations: one launch, the norm inside the tcgen05 GEMM
  if (norm_linear_fused(dtype, M, K, ldx, x, gamma, norm_mode, W, w_dtype, w_layout, N, ldw, epi,
                        aux, ld_aux, Y, ldy)) {
    GemmFusion fz;
    fz.rms_gamma = gamma;
    fz.eps = eps;
    return gemm_tc(x, M, K, ldx, W, w_dtype, w_layout, N, ldw, w_scale, epi, aux, ld_aux,
                   aux_row_mod, Y, ldy, st, &fz);
  }
  // otherwise the normalised rows go through the workspace to a second launch
  if (workspace == nullptr || workspace_bytes < (size_t)M * (size_t)K * (dtype == CK_F32 ? 4 : 2))
    return CK_ERR_WORKSPACE;
  int rc = row_norm(x, dtype, M, (int32_t)K, ldx, gamma, beta, eps, norm_mode, workspace, K, st);
  if (rc != CK_OK) return rc;
  return linear_dispatch(workspace, dtype, M, K, K, W, w_dtype, w_layout, N, ldw, w_scale, epi,
                         aux, ld_aux, aux_row_mod, Y, ldy, st);
}

int attention_dispatch(const ck_attention_args& a, cudaStream_t st) {
  if (a.B < 0 || a.H <= 0 || a.Dh <= 0 || a.Lq < 0) return CK_ERR_INVALID_ARG;
  if (a.B == 0 || a.Lq == 0) return CK_OK;
  if (!a.q || !a.k || !a.v || !a.o) return CK_ERR_INVALID_ARG;
  if (a.key_offsets == nullptr && a.n_keys < 0) return CK_ERR_INVALID_ARG;
  if (a.block_mask != nullptr && (a.block_l <= 0 || a.block_e <= 0 || a.n_k_tiles < 0))
    return CK_ERR_INVALID_ARG;
  if (attention_ws_supported(a)) return attention_ws(a, st);
  if (attention_tc_supported(a)) return attention_tc(a, st);
  return attention_simt(a, st);
}

}  // namespace ck

extern "C" {

size_t ck_pack_workspace_bytes(int64_t E, int32_t B) { return pack_workspace_bytes(E, B); }

size_t ck_collate_bins_workspace_bytes(int32_t B, int32_t window_bins) {
  return collate_bins_workspace_bytes(B, window_bins);
}

int ck_collate_bins(const ck_bin_window* windows, int32_t B, int32_t window_bins,
                    int32_t n_buckets, int32_t max_neurons, int32_t* batch, int64_t capacity,
                    void* workspace, size_t workspace_bytes, int32_t* n_total, void* stream) {
  return collate_bins(windows, B, window_bins, n_buckets, max_neurons, batch, capacity, workspace,
                      workspace_bytes, n_total, S(stream));
}

int ck_pack_events(const void* batch_indices, int idx_dtype, int64_t idx_stride, int64_t E,
                   int32_t B, int32_t* counts, int32_t* offsets, int32_t* dest, int32_t* e_max,
                   void* workspace, size_t workspace_bytes, void* stream) {
  return pack_events(batch_indices, idx_dtype, idx_stride, E, B, nullptr, counts, offsets, dest,
                     e_max, workspace, workspace_bytes, S(stream));
}

int ck_pack_scatter(const void* flat, int dtype, int64_t E, int32_t D, int64_t flat_stride,
                    const void* batch_indices, int idx_dtype, int64_t idx_stride,
                    const int32_t* dest, const int32_t* offsets, int32_t e_max, void* out,
                    uint8_t* mask, void* stream) {
  return pack_scatter(flat, dtype, E, D, flat_stride, batch_indices, idx_dtype, idx_stride, dest,
                      offsets, e_max, out, mask, S(stream));
}

int ck_tokenize(const void* n_emb, const void* t_emb, const void* v_emb, int dtype, int32_t D,
                int64_t n_vocab, int64_t t_vocab, int64_t v_vocab, int64_t n_ld, int64_t t_ld,
                int64_t v_ld, const void* nid, const void* tb, const void* val, int idx_dtype,
                int64_t s_nid, int64_t s_tb, int64_t s_val, int64_t E, const int32_t* dest,
                const void* gamma, const void* beta, float eps, void* out, int64_t out_ld,
                void* stream) {
  return tokenize(n_emb, t_emb, v_emb, dtype, D, n_vocab, t_vocab, v_vocab, n_ld, t_ld, v_ld, nid,
                  tb, val, idx_dtype, s_nid, s_tb, s_val, E, dest, gamma, beta, eps, out, out_ld,
                  S(stream));
}

size_t ck_tokenize_packed_workspace_bytes(void) { return tokenize_packed_slots() * 4; }

int ck_tokenize_packed(const void* n_emb, const void* t_emb, const void* v_emb, int dtype,
                       int32_t D, int64_t n_vocab, int64_t t_vocab, int64_t v_vocab,
                       const void* nid, const void* tb, const void* val, const void* batch_indices,
                       int idx_dtype, int64_t E, int32_t B, const void* gamma, const void* beta,
                       float eps, void* out, int64_t out_ld, int32_t* offsets, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (E < 0 || B <= 0 || offsets == nullptr) return CK_ERR_INVALID_ARG;
  if (E > kTokPackMaxE || B > kTokPackMaxB) return CK_ERR_UNSUPPORTED;
  if (E == 0)  // no events: every window is empty
    return cudaMemsetAsync(offsets, 0, (size_t)(B + 1) * 4, S(stream)) == cudaSuccess
               ? CK_OK
               : record_cuda_error();
  if (workspace == nullptr || workspace_bytes < tokenize_packed_slots() * 4)
    return CK_ERR_WORKSPACE;
  return tokenize_packed(n_emb, t_emb, v_emb, dtype, D, n_vocab, t_vocab, v_vocab, nid, tb, val,
                         batch_indices, idx_dtype, E, B, gamma, beta, eps, out, out_ld, offsets,
                         reinterpret_cast<int32_t*>(workspace), S(stream), nullptr);
}

int ck_dequantize_int8(const void* w_int8, const float* scale, int64_t N, int64_t K, int64_t ldw,
                       void* out, int64_t ldo, void* stream) {
  if (N == 0) return CK_OK;
  DequantSeg g{reinterpret_cast<const int8_t*>(w_int8), scale, out, N, K, ldw, ldo};
  if (!dequant_seg_ok(g)) return CK_ERR_INVALID_ARG;
  return dequant_int8(&g, 1, S(stream));
}

int ck_row_norm(const void* x, int dtype, int64_t M, int32_t D, int64_t ldx, const void* gamma,
                const void* beta, float eps, int mode, void* y, int64_t ldy, void* stream) {
  return row_norm(x, dtype, M, D, ldx, gamma, beta, eps, mode, y, ldy, S(stream));
}

int ck_linear(const void* A, int dtype, int64_t M, int64_t K, int64_t lda, const void* W,
              int w_dtype, int w_layout, int64_t N, int64_t ldw, const float* w_scale, int epi,
              const void* aux, int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy,
              void* stream) {
  return linear_dispatch(A, dtype, M, K, lda, W, w_dtype, w_layout, N, ldw, w_scale, epi, aux,
                         ld_aux, aux_row_mod, Y, ldy, S(stream));
}

size_t ck_norm_linear_workspace_bytes(int dtype, int64_t M, int64_t K) {
  return (size_t)M * (size_t)K * (dtype == CK_F32 ? 4 : 2);
}

int ck_norm_linear(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx, const void* gamma,
                   const void* beta, float eps, int norm_mode, const void* W, int w_dtype,
                   int w_layout, int64_t N, int64_t ldw, const float* w_scale, int epi,
                   const void* aux, int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy,
                   void* workspace, size_t workspace_bytes, void* stream) {
  return norm_linear(x, dtype, M, K, ldx, gamma, beta, eps, norm_mode, W, w_dtype, w_layout, N,
                     ldw, w_scale, epi, aux, ld_aux, aux_row_mod, Y, ldy, workspace,
                     workspace_bytes, S(stream));
}

int ck_attention(const ck_attention_args* args, void* stream) {
  if (args == nullptr) return CK_ERR_INVALID_ARG;
  return attention_dispatch(*args, S(stream));
}

}  // extern "C"
