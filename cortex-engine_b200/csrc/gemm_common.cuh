// Pieces shared by the 1-SM and 2-SM tcgen05 GEMM kernels: the argument block
// and the epilogue arithmetic (per-channel INT8 scale, rounding of the linear
// output to bf16 as torch's F.linear returns it, then GELU / residual / bias).
#pragma once

#include "common.cuh"

namespace ck {
namespace gemm {

struct GemmArgs {
  int M, N, K;
  int num_m_tiles, num_n_tiles, num_k_blocks;
  const __nv_bfloat16* aux;
  int64_t ld_aux;
  int64_t aux_row_mod;
  const float* w_scale;
  int scale_vec;  // w_scale is 16-byte aligned: vector loads
};

// Epilogue math for 32 consecutive columns n0.. of row m (v: fp32 accumulators).
template <int EPI>
__device__ __forceinline__ void epilogue_math(const GemmArgs& p, int m, int n0, float* v) {
  const bool full = (n0 + 32 <= p.N);
  if (p.w_scale != nullptr) {
    if (full && p.scale_vec) {
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 s = __ldg(reinterpret_cast<const float4*>(p.w_scale + n0) + c);
        v[4 * c] *= s.x;
        v[4 * c + 1] *= s.y;
        v[4 * c + 2] *= s.z;
        v[4 * c + 3] *= s.w;
      }
    } else {
      for (int i = 0; i < 32; ++i) v[i] *= (n0 + i < p.N) ? __ldg(p.w_scale + n0 + i) : 0.f;
    }
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = rbf(v[i]);  // linear output in bf16, as F.linear returns it
  if (EPI == CK_EPI_GELU) {
    gelu32(v);
  } else if (EPI == CK_EPI_RESID || EPI == CK_EPI_BIAS) {
    if (m >= p.M) return;
    const __nv_bfloat16* src;
    if (EPI == CK_EPI_RESID) {
      const int64_t r = p.aux_row_mod > 0 ? (m % p.aux_row_mod) : m;
      src = p.aux + r * p.ld_aux + n0;
    } else {
      src = p.aux + n0;
    }
    if (full) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float f[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(src) + c), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[8 * c + j] = f[j] + v[8 * c + j];
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (n0 + i < p.N) v[i] = bf2f(src[i]) + v[i];
    }
  }
}

}  // namespace gemm
}  // namespace ck
