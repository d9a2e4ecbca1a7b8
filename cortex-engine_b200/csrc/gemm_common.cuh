// Pieces of the tcgen05 GEMM: the argument block and the epilogue arithmetic
// (per-channel INT8 scale, rounding of the linear output to
// bf16 as torch's F.linear returns it, then GELU / residual / bias).
#pragma once

#include "common.cuh"

namespace ck {
namespace gemm {

struct GemmArgs {
  int M, N, K;
  int num_m_tiles, num_n_tiles, num_k_blocks;
  // Tiles [split_from, num_tiles) of the persistent schedule are half tiles:
  // the last round's full tiles split into their two BN/2-column halves, so
  // that a short last wave keeps twice as many SMs busy for half as long.
  int split_from, num_tiles;
  const __nv_bfloat16* aux;
  int64_t ld_aux;
  int64_t aux_row_mod;
  const float* w_scale;
  int scale_vec;  // w_scale is 16-byte aligned: vector loads
  float norm_eps;
  // LayerNorm of the residual output (FUSE_LN): a second output
  //   y2 = (y - mean) * rstd * ln_gamma + ln_beta   over each full row of y,
  // where the row's two BN-column halves belong to the two CTAs of a cluster.
  const __nv_bfloat16* ln_gamma;
  const __nv_bfloat16* ln_beta;  // may be NULL
  // FUSE_LN: the residual tile comes in by TMA (the kernel's residual map)
  // ahead of the accumulator, else by per-row loads
  int res_tma;
  int pre_b;  // B (the weight) may be prefetched before the dependency wait
  // RMSNorm of A fused into the GEMM (FUSE_RMS): the norm warps scale every
  // A tile by rms_gamma in shared memory and sum x^2 per row; the epilogue
  // multiplies each row by 1 / sqrt(sum / K + norm_eps).
  const __nv_bfloat16* rms_gamma;
};

enum Fuse { FUSE_NONE = 0, FUSE_LN = 3, FUSE_RMS = 4 };

__device__ __forceinline__ int64_t residual_row(const GemmArgs& p, int m) {
  return p.aux_row_mod > 0 ? (m % p.aux_row_mod) : m;
}

// Epilogue math for 32 consecutive columns n0.. of row m (v: fp32 accumulators),
// result packed as 16 bf16 pairs in out.
// res: the residual row's 32 columns (RESID) when the caller prefetched them
// (whole chunks), else NULL and the residual is read here.
// The linear output is rounded to bf16 as F.linear returns it; for STORE that
// rounding is the final pack itself.
template <int EPI>
__device__ __forceinline__ void epilogue_math(const GemmArgs& p, int m, int n0, float* v,
                                              const uint4* res, uint32_t* out) {
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
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= (n0 + i < p.N) ? __ldg(p.w_scale + n0 + i) : 0.f;
    }
  }
  if ((EPI == CK_EPI_RESID || EPI == CK_EPI_BIAS) && full && m < p.M) {
    // bf16(bf16(acc) + r) as torch's bf16 add computes it, one bf16x2 add per pair
    const __nv_bfloat16* src =
        EPI == CK_EPI_RESID ? p.aux + residual_row(p, m) * p.ld_aux + n0 : p.aux + n0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 u = res != nullptr ? res[c] : __ldg(reinterpret_cast<const uint4*>(src) + c);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        out[4 * c + j] = add_bf16x2(cvt_bf16x2(v[8 * c + 2 * j], v[8 * c + 2 * j + 1]), w[j]);
    }
    return;
  }
  if (EPI != CK_EPI_STORE) {
#pragma unroll
    for (int i = 0; i < 32; i += 2) rbf2(v[i], v[i + 1]);
  }
  if (EPI == CK_EPI_GELU) {
    gelu32(v);
  } else if ((EPI == CK_EPI_RESID || EPI == CK_EPI_BIAS) && m < p.M) {
    const __nv_bfloat16* src;
    if (EPI == CK_EPI_RESID) {
      src = p.aux + residual_row(p, m) * p.ld_aux + n0;
    } else {
      src = p.aux + n0;
    }
    if (full) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 u = res != nullptr ? res[c] : __ldg(reinterpret_cast<const uint4*>(src) + c);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float lo = v[8 * c + 2 * j], hi = v[8 * c + 2 * j + 1];
          f2up(fadd2(f2pk(bf16_lo(w[j]), bf16_hi(w[j])), f2pk(lo, hi)), lo, hi);
          v[8 * c + 2 * j] = lo;
          v[8 * c + 2 * j + 1] = hi;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (n0 + i < p.N) v[i] = bf2f(src[i]) + v[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) out[i] = cvt_bf16x2(v[2 * i], v[2 * i + 1]);
}

}  // namespace gemm
}  // namespace ck
