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
bool pdl_enabled();       // CK_PDL=0 in the environment turns programmatic launch off
int finish_launch(cudaError_t e);  // counts the launch; CK_OK or CK_ERR_CUDA

// Launch trace (trace.cpp): while ck_trace_begin is active, every launch of
// this library outside a stream capture is bracketed by two CUDA events on its
// stream, so that the host can read each kernel's device time afterwards.
extern int g_trace_on;
void trace_before(cudaStream_t st);
void trace_after(cudaStream_t st, const void* func);

// Every kernel of the library goes through this launch: trace events when
// tracing is on, then the launch itself and its status.
template <typename... KArgs, typename... Args>
int launch_cfg(const cudaLaunchConfig_t& cfg, void (*kernel)(KArgs...), Args&&... args) {
  if (g_trace_on) trace_before(cfg.stream);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
  if (g_trace_on) trace_after(cfg.stream, reinterpret_cast<const void*>(kernel));
  return finish_launch(e);
}

// Launch a kernel with programmatic stream serialisation: the grid may be
// scheduled while the previous kernel in the stream is finishing, and waits
// for it inside the kernel (grid_dep_wait in common.cuh). Captured into a CUDA
// graph this becomes a programmatic edge.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return launch_cfg(cfg, kernel, static_cast<Args&&>(args)...);
}

bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                  uint64_t inner, uint64_t outer, uint64_t ld_elems, uint32_t box_inner,
                  uint32_t box_outer, int swizzle_bytes /* 0, 64 or 128 */);

// tcgen05 GEMM (gemm_tc.cu)
bool gemm_tc_supported(int64_t M, int64_t K, int64_t lda, int w_dtype, int w_layout, int64_t N,
                       int64_t ldw, const void* A, const void* W, int64_t ldy, const void* Y,
                       int epi, const void* aux, int64_t ld_aux);
// Optional fusions of the tcgen05 GEMM (see gemm_common.cuh):
//   ln_out     residual epilogue also writes LayerNorm(Y) (gamma ln_gamma, beta
//              ln_beta or none, eps) to ln_out (row stride ln_ld): bf16, N = 512
//   rms_gamma  RMSNorm of the A rows (gamma rms_gamma, eps) applied inside the GEMM
struct GemmFusion {
  float eps = 0.f;
  void* ln_out = nullptr;
  int64_t ln_ld = 0;
  const void* ln_gamma = nullptr;
  const void* ln_beta = nullptr;
  // the weight is not written by the kernel launched just before on the stream
  // (model weights inside the forward): its first tiles may load before the
  // GEMM's dependency wait
  bool w_static = false;
  // RMSNorm of A fused into the GEMM (bf16 A, K a multiple of 8, gamma 16-byte
  // aligned, store or bias epilogue): y = epi((x * gamma) W^T / sqrt(mean_k(x^2) + eps))
  const void* rms_gamma = nullptr;
};
// Tensor-core GEMM when supported, else the CUDA-core one (capi.cu).
// w_static: the weight is not written by the kernel launched just before on
// the stream, so the tcgen05 GEMM may start loading it before its dependency
// wait.
int linear_dispatch(const void* A, int dtype, int64_t M, int64_t K, int64_t lda, const void* W,
                    int w_dtype, int w_layout, int64_t N, int64_t ldw, const float* w_scale,
                    int epi, const void* aux, int64_t ld_aux, int64_t aux_row_mod, void* Y,
                    int64_t ldy, cudaStream_t st, bool w_static = false);
// Norm then linear (capi.cu). RMSNorm over bf16 rows that the tcgen05 GEMM
// takes (K a multiple of 8, store or bias epilogue) runs as one launch with the norm
// inside the GEMM (norm_linear_fused); every other case writes the normalised
// rows to the workspace (M * K elements of dtype) and runs the linear after
// it, and returns CK_ERR_WORKSPACE without launching when that is too small.
bool norm_linear_fused(int dtype, int64_t M, int64_t K, int64_t ldx, const void* x,
                       const void* gamma, int norm_mode, const void* W, int w_dtype,
                       int w_layout, int64_t N, int64_t ldw, int epi, const void* aux,
                       int64_t ld_aux, const void* Y, int64_t ldy);
int norm_linear(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx, const void* gamma,
                const void* beta, float eps, int norm_mode, const void* W, int w_dtype,
                int w_layout, int64_t N, int64_t ldw, const float* w_scale, int epi,
                const void* aux, int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy,
                void* workspace, size_t workspace_bytes, cudaStream_t st);
int gemm_tc_block_n(int64_t N);
int gemm_tc(const void* A, int64_t M, int64_t K, int64_t lda, const void* W, int w_dtype,
            int w_layout, int64_t N, int64_t ldw, const float* w_scale, int epi, const void* aux,
            int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy, cudaStream_t st,
            const GemmFusion* fz = nullptr);

// CUDA-core GEMM, fp32 accumulate (gemm_simt.cu)
int gemm_simt(const void* A, int dtype, int64_t M, int64_t K, int64_t lda, const void* W,
              int w_dtype, int w_layout, int64_t N, int64_t ldw, const float* w_scale, int epi,
              const void* aux, int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy,
              cudaStream_t st);

// attention (attention_tc.cu, attention_simt.cu)
bool attention_tc_supported(const ck_attention_args& a);
int attention_tc(const ck_attention_args& a, cudaStream_t st);
int attention_simt(const ck_attention_args& a, cudaStream_t st);
// warp-specialised persistent variant for unmasked bf16 head_dim 64 (attention_ws.cu)
bool attention_ws_supported(const ck_attention_args& a);
int attention_ws(const ck_attention_args& a, cudaStream_t st);

// row norm (norm.cu)
int row_norm(const void* x, int dtype, int64_t M, int32_t D, int64_t ldx, const void* gamma,
             const void* beta, float eps, int mode, void* y, int64_t ldy, cudaStream_t st);
// two LayerNorms in a row (final_norm then the head's norm), one pass
int row_norm2(const void* x, int dtype, int64_t M, int32_t D, int64_t ldx, const void* g1,
              const void* b1, const void* g2, const void* b2, float eps, void* y, int64_t ldy,
              cudaStream_t st);

// INT8 weight dequantisation (dequant.cu): out[n, k] = bf16(float(w[n, k]) *
// scale[n]) for a list of (N, K) matrices; K a multiple of 16, rows 16-byte
// aligned.
struct DequantSeg {
  const int8_t* w;     // (N, K) int8, row stride ldw
  const float* scale;  // (N,)
  void* out;           // (N, K) bf16, row stride ldo
  int64_t N, K, ldw, ldo;
};
bool dequant_seg_ok(const DequantSeg& g);
int dequant_int8(const DequantSeg* segs, int n, cudaStream_t st);

// packing and tokenizer (pack.cu, tokenizer.cu)
size_t pack_workspace_bytes(int64_t E, int32_t B);
// n_valid (device, may be NULL): events n_valid..E-1 are padding (pack.cu)
int pack_events(const void* bidx, int idx_dtype, int64_t idx_stride, int64_t E, int32_t B,
                const int32_t* n_valid, int32_t* counts, int32_t* offsets, int32_t* dest,
                int32_t* e_max, void* ws, size_t ws_bytes, cudaStream_t st);
int pack_scatter(const void* flat, int dtype, int64_t E, int32_t D, int64_t flat_stride,
                 const void* bidx, int idx_dtype, int64_t idx_stride, const int32_t* dest,
                 const int32_t* offsets, int32_t e_max, void* out, uint8_t* mask,
                 cudaStream_t st);
int tokenize(const void* n_emb, const void* t_emb, const void* v_emb, int dtype, int32_t D,
             int64_t n_vocab, int64_t t_vocab, int64_t v_vocab, int64_t n_ld, int64_t t_ld,
             int64_t v_ld, const void* nid, const void* tb, const void* val, int idx_dtype,
             int64_t s_nid, int64_t s_tb, int64_t s_val, int64_t E, const int32_t* dest,
             const void* gamma, const void* beta, float eps, void* out, int64_t out_ld,
             cudaStream_t st, const int32_t* n_valid = nullptr);

// Packing inside the tokenizer for the forward (tokenizer.cu): tokens of event
// e go to row e and the window offsets come from the batch boundaries, which
// is _pack_events' result when batch_indices is sorted (collate_events'
// layout). A second launch checks the tokenizer blocks' flags (slots, at least
// tokenize_packed_slots() words) and, for unsorted or out-of-range batch
// indices, redoes the packing as a stable counting sort and tokenizes every
// event into its packed row. dest is not produced. E <= kTokPackMaxE and
// B <= kTokPackMaxB; larger batches use pack_events + tokenize.
constexpr int64_t kTokPackMaxE = int64_t(1) << 20;
constexpr int32_t kTokPackMaxB = 4096;
size_t tokenize_packed_slots();
int tokenize_packed(const void* n_emb, const void* t_emb, const void* v_emb, int dtype, int32_t D,
                    int64_t n_vocab, int64_t t_vocab, int64_t v_vocab, const void* nid,
                    const void* tb, const void* val, const void* bidx, int idx_dtype, int64_t E,
                    int32_t B, const void* gamma, const void* beta, float eps, void* out,
                    int64_t out_ld, int32_t* offsets, int32_t* slots, cudaStream_t st,
                    const int32_t* n_valid);

// event ingest from bin-count matrices (ingest.cu)
size_t collate_bins_workspace_bytes(int32_t B, int32_t W);
int collate_bins(const ck_bin_window* wins, int32_t B, int32_t W, int32_t n_buckets,
                 int32_t max_neurons, int32_t* batch, int64_t capacity, void* ws, size_t ws_bytes,
                 int32_t* n_total, cudaStream_t st);

// row-segment copies (rows.cu)
int copy_rows(const void* src, int64_t src_rows, void* dst, int64_t dst_rows, int64_t row_bytes,
              const int32_t* segments, int32_t n_segments, cudaStream_t st);

// behaviour head in algebraic form (head.cu): head_prep builds the weight-only
// (NT, D) matrix once per forward, head_fused runs both LayerNorms, the
// projection against it, the per-head softmax and out_proj in one kernel.
bool head_fused_supported(const ck_model* m);
size_t head_qall_bytes(const ck_model* m);
int head_prep(const ck_model* m, void* qall, cudaStream_t st);
int head_fused(const ck_model* m, const void* lat, int32_t B, const void* qall, void* out,
               cudaStream_t st);

}  // namespace ck
