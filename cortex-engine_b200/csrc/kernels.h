// Internal host-side interface between the kernel files and the C ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "cortex_b200.h"

namespace ck {

// runtime helpers (status.cu)
int num_sms();
int record_cuda_error();  // stores cudaGetLastError() and returns CK_ERR_CUDA
int check_launch();       // CK_OK or record_cuda_error()
bool smem_attr_ready(const void* kernel, int bytes);  // per device, once

bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                  uint64_t inner, uint64_t outer, uint64_t ld_elems, uint32_t box_inner,
                  uint32_t box_outer, int swizzle_bytes /* 0, 64 or 128 */);

// tcgen05 GEMM (gemm_tc.cu)
bool gemm_tc_supported(int64_t M, int64_t K, int64_t lda, int w_dtype, int w_layout, int64_t N,
                       int64_t ldw, const void* A, const void* W, int64_t ldy, const void* Y,
                       int epi, const void* aux, int64_t ld_aux);
int gemm_tc(const void* A, int64_t M, int64_t K, int64_t lda, const void* W, int w_dtype,
            int w_layout, int64_t N, int64_t ldw, const float* w_scale, int epi, const void* aux,
            int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy, cudaStream_t st);

// CUDA-core GEMM, fp32 accumulate (gemm_simt.cu)
int gemm_simt(const void* A, int dtype, int64_t M, int64_t K, int64_t lda, const void* W,
              int w_dtype, int w_layout, int64_t N, int64_t ldw, const float* w_scale, int epi,
              const void* aux, int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy,
              cudaStream_t st);

// attention (attention_tc.cu, attention_simt.cu)
bool attention_tc_supported(const ck_attention_args& a);
int attention_tc(const ck_attention_args& a, cudaStream_t st);
int attention_simt(const ck_attention_args& a, cudaStream_t st);

// row norm (norm.cu)
int row_norm(const void* x, int dtype, int64_t M, int32_t D, int64_t ldx, const void* gamma,
             const void* beta, float eps, int mode, void* y, int64_t ldy, cudaStream_t st);
// two LayerNorms in a row (final_norm then the head's norm), one pass
int row_norm2(const void* x, int dtype, int64_t M, int32_t D, int64_t ldx, const void* g1,
              const void* b1, const void* g2, const void* b2, float eps, void* y, int64_t ldy,
              cudaStream_t st);

// packing and tokenizer (pack.cu, tokenizer.cu)
size_t pack_workspace_bytes(int64_t E, int32_t B);
int pack_events(const void* bidx, int idx_dtype, int64_t idx_stride, int64_t E, int32_t B,
                int32_t* counts, int32_t* offsets, int32_t* dest, int32_t* e_max, void* ws,
                size_t ws_bytes, cudaStream_t st);
int pack_scatter(const void* flat, int dtype, int64_t E, int32_t D, int64_t flat_stride,
                 const void* bidx, int idx_dtype, int64_t idx_stride, const int32_t* dest,
                 const int32_t* offsets, int32_t e_max, void* out, uint8_t* mask,
                 cudaStream_t st);
int tokenize(const void* n_emb, const void* t_emb, const void* v_emb, int dtype, int32_t D,
             int64_t n_vocab, int64_t t_vocab, int64_t v_vocab, int64_t n_ld, int64_t t_ld,
             int64_t v_ld, const void* nid, const void* tb, const void* val, int idx_dtype,
             int64_t s_nid, int64_t s_tb, int64_t s_val, int64_t E, const int32_t* dest,
             const void* gamma, const void* beta, float eps, void* out, int64_t out_ld,
             cudaStream_t st);

// behaviour head tail: attention of `nq` learned queries over L latents per
// sample followed by out_proj (D -> 1) (head.cu)
int head_attention_out(const void* q, const void* kv, int dtype, int32_t B, int32_t L, int32_t nq,
                       int32_t H, int32_t Dh, const void* w_out, int w_dtype,
                       const float* w_scale, const void* bias, void* y, cudaStream_t st);

}  // namespace ck
