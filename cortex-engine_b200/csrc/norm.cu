// Row norms with fp32 statistics, one warp per row, the row held in registers.
//   LayerNorm: y = (x - mean) / sqrt(var + eps) * gamma + beta     (nn.LayerNorm,
//              cortex/models/perceiver.py:51-52,97-98,143; cortex/models/cortex.py:25)
//   RMSNorm:   y = x / sqrt(mean(x^2) + eps) * gamma               (rms_norm_linear_reference,
//              cortex/kernels/fused_rmsnorm.py:101-103)
// Output is rounded to the input dtype, as the reference's .to(x.dtype) / bf16
// LayerNorm output is. row_norm2 applies two LayerNorms back to back (the
// encoder's final_norm, then the behaviour head's norm), rounding in between.
#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

template <typename T>
__device__ __forceinline__ void ld_vec(const T* p, float* f, int n);
template <>
__device__ __forceinline__ void ld_vec<__nv_bfloat16>(const __nv_bfloat16* p, float* f, int n) {
  if (n == 8) {
    unpack8(*reinterpret_cast<const uint4*>(p), f);
  } else {
    for (int k = 0; k < n; ++k) f[k] = bf2f(p[k]);
  }
}
template <>
__device__ __forceinline__ void ld_vec<float>(const float* p, float* f, int n) {
  if (n == 4) {
    float4 v = *reinterpret_cast<const float4*>(p);
    f[0] = v.x, f[1] = v.y, f[2] = v.z, f[3] = v.w;
  } else {
    for (int k = 0; k < n; ++k) f[k] = p[k];
  }
}
template <typename T>
__device__ __forceinline__ void st_vec(T* p, const float* f, int n);
template <>
__device__ __forceinline__ void st_vec<__nv_bfloat16>(__nv_bfloat16* p, const float* f, int n) {
  if (n == 8) {
    *reinterpret_cast<uint4*>(p) = pack8(f);
  } else {
    for (int k = 0; k < n; ++k) p[k] = f2bf(f[k]);
  }
}
template <>
__device__ __forceinline__ void st_vec<float>(float* p, const float* f, int n) {
  if (n == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  } else {
    for (int k = 0; k < n; ++k) p[k] = f[k];
  }
}

template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return x;
}
template <>
__device__ __forceinline__ float rnd<__nv_bfloat16>(float x) {
  return rbf(x);
}

template <int VEC, int MAXV>
__device__ __forceinline__ void layer_norm_regs(float (&x)[MAXV][VEC], int lane, int nvec, int D,
                                                float eps) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i)
    if (lane + 32 * i < nvec)
#pragma unroll
      for (int k = 0; k < VEC; ++k) s += x[i][k];
  const float mean = warp_sum(s) / (float)D;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i)
    if (lane + 32 * i < nvec)
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        const float d = x[i][k] - mean;
        q += d * d;
      }
  const float rstd = 1.0f / sqrtf(warp_sum(q) / (float)D + eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i)
    if (lane + 32 * i < nvec)
#pragma unroll
      for (int k = 0; k < VEC; ++k) x[i][k] = (x[i][k] - mean) * rstd;
}

template <typename T, int VEC, int MAXV>
__global__ void row_norm_kernel(const T* x, int64_t M, int D, int64_t ldx, const T* g1,
                                const T* b1, const T* g2, const T* b2, float eps, int mode,
                                int two, T* y, int64_t ldy) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int nvec = D / VEC;
  for (int64_t r = warp; r < M; r += nwarps) {
    float v[MAXV][VEC];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) ld_vec<T>(x + r * ldx + c * VEC, v[i], VEC);
    }
    if (mode == CK_NORM_RMS) {
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < MAXV; ++i)
        if (lane + 32 * i < nvec)
#pragma unroll
          for (int k = 0; k < VEC; ++k) q += v[i][k] * v[i][k];
      const float rms = sqrtf(warp_sum(q) / (float)D + eps);
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int c = lane + 32 * i;
        if (c < nvec)
#pragma unroll
          for (int k = 0; k < VEC; ++k) v[i][k] = (v[i][k] / rms) * (float)g1[c * VEC + k];
      }
    } else {
      layer_norm_regs<VEC, MAXV>(v, lane, nvec, D, eps);
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int c = lane + 32 * i;
        if (c < nvec)
#pragma unroll
          for (int k = 0; k < VEC; ++k)
            v[i][k] = v[i][k] * (float)g1[c * VEC + k] + (b1 ? (float)b1[c * VEC + k] : 0.f);
      }
      if (two) {
#pragma unroll
        for (int i = 0; i < MAXV; ++i)
#pragma unroll
          for (int k = 0; k < VEC; ++k) v[i][k] = rnd<T>(v[i][k]);
        layer_norm_regs<VEC, MAXV>(v, lane, nvec, D, eps);
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
          const int c = lane + 32 * i;
          if (c < nvec)
#pragma unroll
            for (int k = 0; k < VEC; ++k)
              v[i][k] = v[i][k] * (float)g2[c * VEC + k] + (b2 ? (float)b2[c * VEC + k] : 0.f);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) st_vec<T>(y + r * ldy + c * VEC, v[i], VEC);
    }
  }
}

// bf16 LayerNorm fast path: G lanes per row (32 / G rows per warp), MAXV
// 16-byte vectors per lane, gamma / beta as 16-byte vectors. Same two-pass
// statistics as row_norm_kernel; TWO applies a second LayerNorm after rounding.
template <int MAXV, int G, bool TWO>
__global__ void __launch_bounds__(256, MAXV <= 6 ? 3 : 2) layer_norm_bf16_kernel(
    const __nv_bfloat16* x, int64_t M, int D, int64_t ldx, const __nv_bfloat16* g1,
    const __nv_bfloat16* b1, const __nv_bfloat16* g2, const __nv_bfloat16* b2, float eps,
    __nv_bfloat16* y, int64_t ldy) {
  grid_dep_wait();
  grid_dep_launch();
  constexpr int RPW = 32 / G;
  const int lane = threadIdx.x & 31;
  const int sub = lane % G;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int nvec = D / 8;
  for (int64_t base = warp * RPW; base < M; base += nwarps * RPW) {
    const int64_t r = base + lane / G;
    const bool live = r < M;
    float v[MAXV][8];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = sub + G * i;
      if (live && c < nvec) {
        unpack8(reinterpret_cast<const uint4*>(x + r * ldx)[c], v[i]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[i][k] = 0.f;
      }
    }
#pragma unroll
    for (int pass = 0; pass < (TWO ? 2 : 1); ++pass) {
      const __nv_bfloat16* g = pass == 0 ? g1 : g2;
      const __nv_bfloat16* b = pass == 0 ? b1 : b2;
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < MAXV; ++i)
#pragma unroll
        for (int k = 0; k < 8; ++k) s += v[i][k];
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const float mean = s / (float)D;
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < MAXV; ++i)
        if (sub + G * i < nvec)
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float d = v[i][k] - mean;
            q += d * d;
          }
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
      const float rstd = 1.0f / sqrtf(q / (float)D + eps);
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int c = sub + G * i;
        if (c < nvec) {
          float gf[8], bf[8];
          unpack8(reinterpret_cast<const uint4*>(g)[c], gf);
          if (b != nullptr) {
            unpack8(reinterpret_cast<const uint4*>(b)[c], bf);
          } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) bf[k] = 0.f;
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            v[i][k] = (v[i][k] - mean) * rstd;
            v[i][k] = v[i][k] * gf[k] + bf[k];
            if (TWO && pass == 0) v[i][k] = rbf(v[i][k]);
          }
        }
      }
    }
    if (live) {
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int c = sub + G * i;
        if (c < nvec) reinterpret_cast<uint4*>(y + r * ldy)[c] = pack8(v[i]);
      }
    }
  }
}

template <int MAXV, int G>
int launch_ln_fast(const void* x, int64_t M, int D, int64_t ldx, const void* g1, const void* b1,
                   const void* g2, const void* b2, float eps, int two, void* y, int64_t ldy,
                   cudaStream_t st) {
  constexpr int rows_per_block = 8 * (32 / G);
  int64_t blocks = (M + rows_per_block - 1) / rows_per_block;
  const int64_t cap = 16 * (int64_t)num_sms();
  if (blocks > cap) blocks = cap;
  using B = __nv_bfloat16;
  auto X = reinterpret_cast<const B*>(x);
  auto Y = reinterpret_cast<B*>(y);
  if (two)
    return launch_pdl(layer_norm_bf16_kernel<MAXV, G, true>, dim3((unsigned)blocks), dim3(256), 0,
                      st, X, M, D, ldx, reinterpret_cast<const B*>(g1),
                      reinterpret_cast<const B*>(b1), reinterpret_cast<const B*>(g2),
                      reinterpret_cast<const B*>(b2), eps, Y, ldy);
  return launch_pdl(layer_norm_bf16_kernel<MAXV, G, false>, dim3((unsigned)blocks), dim3(256), 0,
                    st, X, M, D, ldx, reinterpret_cast<const B*>(g1),
                    reinterpret_cast<const B*>(b1), reinterpret_cast<const B*>(g2),
                    reinterpret_cast<const B*>(b2), eps, Y, ldy);
}

template <typename T, int VEC, int MAXV>
int launch_norm(const void* x, int64_t M, int D, int64_t ldx, const void* g1, const void* b1,
                const void* g2, const void* b2, float eps, int mode, int two, void* y,
                int64_t ldy, cudaStream_t st) {
  int64_t blocks = (M * 32 + 255) / 256;
  const int cap = 32 * num_sms();
  if (blocks > cap) blocks = cap;
  return launch_pdl(row_norm_kernel<T, VEC, MAXV>, dim3((unsigned)blocks), dim3(256), 0, st,
      reinterpret_cast<const T*>(x), M, D, ldx, reinterpret_cast<const T*>(g1),
      reinterpret_cast<const T*>(b1), reinterpret_cast<const T*>(g2),
      reinterpret_cast<const T*>(b2), eps, mode, two, reinterpret_cast<T*>(y), ldy);
}

template <typename T>
int dispatch_norm(const void* x, int64_t M, int D, int64_t ldx, const void* g1, const void* b1,
                  const void* g2, const void* b2, float eps, int mode, int two, void* y,
                  int64_t ldy, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec = (D % V == 0) && ((ldx * (int64_t)sizeof(T)) % 16 == 0) &&
                   ((ldy * (int64_t)sizeof(T)) % 16 == 0) && al16(x) && al16(y);
  if constexpr (sizeof(T) == 2) {
    const bool params16 = al16(g1) && (b1 == nullptr || al16(b1)) &&
                          (!two || (al16(g2) && (b2 == nullptr || al16(b2))));
    if (vec && params16 && mode == CK_NORM_LAYER) {
      const int nvec = D / 8;
      // 8 lanes per row (4 rows per warp) and up to 8 vectors per lane: all rows
      // of a Cortex-S latent batch are loaded in a single wave of the grid
      if (nvec <= 64) return launch_ln_fast<8, 8>(x, M, D, ldx, g1, b1, g2, b2, eps, two, y, ldy, st);
      // D = 768 (Cortex-M): 16 lanes x 6 vectors, two rows per warp, three CTAs
      // per SM, so that more rows are in flight than with a warp per row
      if (nvec <= 96) return launch_ln_fast<6, 16>(x, M, D, ldx, g1, b1, g2, b2, eps, two, y, ldy, st);
      if (nvec <= 128) return launch_ln_fast<4, 32>(x, M, D, ldx, g1, b1, g2, b2, eps, two, y, ldy, st);
    }
  }
  if (vec) {
    const int per = (D / V + 31) / 32;
    if (per <= 1) return launch_norm<T, V, 1>(x, M, D, ldx, g1, b1, g2, b2, eps, mode, two, y, ldy, st);
    if (per <= 2) return launch_norm<T, V, 2>(x, M, D, ldx, g1, b1, g2, b2, eps, mode, two, y, ldy, st);
    if (per <= 4) return launch_norm<T, V, 4>(x, M, D, ldx, g1, b1, g2, b2, eps, mode, two, y, ldy, st);
    if (per <= 8) return launch_norm<T, V, 8>(x, M, D, ldx, g1, b1, g2, b2, eps, mode, two, y, ldy, st);
    return CK_ERR_UNSUPPORTED;
  }
  const int per = (D + 31) / 32;
  if (per <= 8) return launch_norm<T, 1, 8>(x, M, D, ldx, g1, b1, g2, b2, eps, mode, two, y, ldy, st);
  if (per <= 32) return launch_norm<T, 1, 32>(x, M, D, ldx, g1, b1, g2, b2, eps, mode, two, y, ldy, st);
  return CK_ERR_UNSUPPORTED;
}

}  // namespace

int row_norm(const void* x, int dtype, int64_t M, int32_t D, int64_t ldx, const void* gamma,
             const void* beta, float eps, int mode, void* y, int64_t ldy, cudaStream_t st) {
  if (M == 0) return CK_OK;
  if (M < 0 || D <= 0 || !x || !y || !gamma) return CK_ERR_INVALID_ARG;
  if (mode != CK_NORM_LAYER && mode != CK_NORM_RMS) return CK_ERR_INVALID_ARG;
  if (dtype == CK_BF16)
    return dispatch_norm<__nv_bfloat16>(x, M, D, ldx, gamma, beta, nullptr, nullptr, eps, mode, 0, y, ldy, st);
  if (dtype == CK_F32)
    return dispatch_norm<float>(x, M, D, ldx, gamma, beta, nullptr, nullptr, eps, mode, 0, y, ldy, st);
  return CK_ERR_UNSUPPORTED;
}

int row_norm2(const void* x, int dtype, int64_t M, int32_t D, int64_t ldx, const void* g1,
              const void* b1, const void* g2, const void* b2, float eps, void* y, int64_t ldy,
              cudaStream_t st) {
  if (M == 0) return CK_OK;
  if (M < 0 || D <= 0 || !x || !y || !g1 || !g2) return CK_ERR_INVALID_ARG;
  if (dtype == CK_BF16)
    return dispatch_norm<__nv_bfloat16>(x, M, D, ldx, g1, b1, g2, b2, eps, CK_NORM_LAYER, 1, y, ldy, st);
  if (dtype == CK_F32)
    return dispatch_norm<float>(x, M, D, ldx, g1, b1, g2, b2, eps, CK_NORM_LAYER, 1, y, ldy, st);
  return CK_ERR_UNSUPPORTED;
}

}  // namespace ck
