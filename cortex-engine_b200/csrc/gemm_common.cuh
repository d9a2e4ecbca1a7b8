// Pieces of the tcgen05 GEMM: the argument block and the epilogue arithmetic
// (folded LayerNorm, per-channel INT8 scale, rounding of the linear output to
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
  // Row statistics written by a residual epilogue (FUSE_STATS): for every row m
  // and every stats_sw-wide column segment s, stats_out[s * M + m] = (mean,
  // sum of squared deviations) of the segment's bf16 outputs.
  float2* stats_out;
  int stats_sw;
  // LayerNorm folded into this GEMM (FUSE_NORM): A holds the raw rows, the
  // weight is W * gamma, and the epilogue applies
  //   y = rstd * (acc - mean * fold_cs[n]) + fold_bw[n]
  // with mean / rstd combined from the producer's segment statistics.
  const float2* stats_in;
  int stats_in_sw, stats_in_nseg;
  float norm_eps;
  const float* fold_cs;
  const float* fold_bw;
  // LayerNorm of the residual output (FUSE_LN): a second output
  //   y2 = (y - mean) * rstd * ln_gamma + ln_beta   over each full row of y,
  // where the row's two BN-column halves belong to the two CTAs of a cluster.
  const __nv_bfloat16* ln_gamma;
  const __nv_bfloat16* ln_beta;  // may be NULL
  // FUSE_LN: the residual tile comes in by TMA (the kernel's residual map)
  // ahead of the accumulator, else by per-row loads
  int res_tma;
  int pre_b;  // B (the weight) may be prefetched before the dependency wait
};

enum Fuse { FUSE_NONE = 0, FUSE_NORM = 1, FUSE_STATS = 2, FUSE_LN = 3 };

__device__ __forceinline__ int64_t residual_row(const GemmArgs& p, int m) {
  return p.aux_row_mod > 0 ? (m % p.aux_row_mod) : m;
}

// Producer statistics of one row (up to 8 segments), fetched ahead of use.
struct StatsRow {
  float2 seg[8];
};

__device__ __forceinline__ StatsRow load_stats(const GemmArgs& p, int m) {
  StatsRow r;
#pragma unroll
  for (int s = 0; s < 8; ++s)
    r.seg[s] = (m < p.M && s < p.stats_in_nseg) ? p.stats_in[(int64_t)s * p.M + m]
                                                : make_float2(0.f, 0.f);
  return r;
}

// Mean and rstd of the row from its per-segment (mean, M2) pairs (Chan et
// al.'s pairwise combination).
__device__ __forceinline__ void combine_stats(const GemmArgs& p, const StatsRow& r, float& mean,
                                              float& rstd) {
  float mu = 0.f;
#pragma unroll
  for (int s = 0; s < 8; ++s)
    if (s < p.stats_in_nseg) mu += (float)min(p.stats_in_sw, p.K - s * p.stats_in_sw) * r.seg[s].x;
  mu /= (float)p.K;
  float m2 = 0.f;
#pragma unroll
  for (int s = 0; s < 8; ++s)
    if (s < p.stats_in_nseg) {
      const float d = r.seg[s].x - mu;
      m2 += r.seg[s].y + (float)min(p.stats_in_sw, p.K - s * p.stats_in_sw) * d * d;
    }
  mean = mu;
  rstd = 1.0f / sqrtf(m2 / (float)p.K + p.norm_eps);
}

// Epilogue math for 32 consecutive columns n0.. of row m (v: fp32 accumulators),
// result packed as 16 bf16 pairs in out.
// FUSE_NORM applies the folded LayerNorm with the row's (mean, rstd) first.
// fold: the (colsum, bias) pairs of columns n0..n0+31 in shared memory.
// res: the residual row's 32 columns (RESID) when the caller prefetched them
// (whole chunks), else NULL and the residual is read here.
// The linear output is rounded to bf16 as F.linear returns it; for STORE that
// rounding is the final pack itself.
template <int EPI, int FUSE = FUSE_NONE>
__device__ __forceinline__ void epilogue_math(const GemmArgs& p, int m, int n0, float* v,
                                              float mean, float rstd, const float2* fold,
                                              const uint4* res, uint32_t* out) {
  const bool full = (n0 + 32 <= p.N);
  if (FUSE == FUSE_NORM) {
#pragma unroll
    for (int c = 0; c < 16; ++c) {  // columns beyond N hold (0, 0)
      const float4 f = reinterpret_cast<const float4*>(fold)[c];
      v[2 * c + 0] = fmaf(rstd, fmaf(-mean, f.x, v[2 * c + 0]), f.y);
      v[2 * c + 1] = fmaf(rstd, fmaf(-mean, f.z, v[2 * c + 1]), f.w);
    }
  }
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
