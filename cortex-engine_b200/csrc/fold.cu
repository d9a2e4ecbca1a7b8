// LayerNorm folding for the linears that consume a normalised residual
// (SelfAttentionBlock.norm_attn -> qkv_proj, norm_mlp -> mlp.0;
// cortex/models/perceiver.py:97-126):
//
//   LN(x) W^T = rstd * (x (W * gamma)^T - mean * colsum) + bias
//   colsum[n] = sum_k bf16(W[n,k] * gamma[k]),   bias[n] = sum_k W[n,k] * beta[k]
//
// One warp per output row n, 16-byte vectors along K. The GEMM epilogue
// (gemm_common.cuh, FUSE_NORM) applies the right-hand side per row.
#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

__global__ void __launch_bounds__(256) norm_fold_kernel(const __nv_bfloat16* W, int64_t N,
                                                        int64_t K, int64_t ldw,
                                                        const __nv_bfloat16* gamma,
                                                        const __nv_bfloat16* beta,
                                                        __nv_bfloat16* w_out, float* colsum,
                                                        float* bias) {
  grid_dep_wait();
  // no early signal: the kernel after this one may read the weights written
  // here before its own dependency wait (the tcgen05 GEMM's weight prefetch)
  const int lane = threadIdx.x & 31;
  const int64_t n = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (n >= N) return;
  float cs = 0.f, bw = 0.f;
  for (int64_t c = lane; c < K / 8; c += 32) {
    float w[8], g[8], b[8], o[8];
    unpack8(reinterpret_cast<const uint4*>(W + n * ldw)[c], w);
    unpack8(reinterpret_cast<const uint4*>(gamma)[c], g);
    if (beta != nullptr) {
      unpack8(reinterpret_cast<const uint4*>(beta)[c], b);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) b[k] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      o[k] = rbf(w[k] * g[k]);
      cs += o[k];
      bw = fmaf(w[k], b[k], bw);
    }
    reinterpret_cast<uint4*>(w_out + n * K)[c] = pack8(o);
  }
  cs = warp_sum(cs);
  bw = warp_sum(bw);
  if (lane == 0) {
    colsum[n] = cs;
    bias[n] = bw;
  }
}

}  // namespace

}  // namespace ck

extern "C" int ck_norm_fold_weights(const void* W, int64_t N, int64_t K, int64_t ldw,
                                    const void* gamma, const void* beta, void* w_out,
                                    float* colsum, float* bias, void* stream) {
  using namespace ck;
  if (N < 0 || K < 0) return CK_ERR_INVALID_ARG;
  if (N == 0) return CK_OK;
  if (!W || !gamma || !w_out || !colsum || !bias) return CK_ERR_INVALID_ARG;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (K % 8 != 0 || ldw % 8 != 0 || ldw < K || !al16(W) || !al16(gamma) || !al16(w_out) ||
      (beta != nullptr && !al16(beta)))
    return CK_ERR_INVALID_ARG;
  const int64_t blocks = (N * 32 + 255) / 256;
  if (blocks > INT32_MAX) return CK_ERR_INVALID_ARG;
  return launch_pdl(norm_fold_kernel, dim3((unsigned)blocks), dim3(256), 0,
                    reinterpret_cast<cudaStream_t>(stream),
                    reinterpret_cast<const __nv_bfloat16*>(W), N, K, ldw,
                    reinterpret_cast<const __nv_bfloat16*>(gamma),
                    reinterpret_cast<const __nv_bfloat16*>(beta),
                    reinterpret_cast<__nv_bfloat16*>(w_out), colsum, bias);
}
