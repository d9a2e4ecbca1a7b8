// CUDA-core GEMM with fp32 accumulation for the cases the tcgen05 kernel does
// not take: fp32 activations (the fp32 configurations must match the reference
// to 1e-4, which TF32 tensor-core products cannot), and bf16 problems whose
// strides break TMA's 16-byte rules (e.g. K = 70). Same epilogue semantics as
// the tensor-core kernel (the linear output is rounded to the activation dtype
// before GELU / residual / bias, as torch eager does).
//
// 64x64 output tile per 256-thread CTA, 4x4 per thread, K staged 16 at a time
// through shared memory.
#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

constexpr int TM = 64, TN = 64, TK = 16;

template <typename T>
__device__ __forceinline__ float tof(T v) {
  return (float)v;
}
template <>
__device__ __forceinline__ float tof<int8_t>(int8_t v) {
  return (float)(int)v;
}

template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return x;
}
template <>
__device__ __forceinline__ float rnd<__nv_bfloat16>(float x) {
  return rbf(x);
}

template <typename T, typename WT>
__global__ void __launch_bounds__(256) gemm_simt_kernel(
    const T* A, int64_t M, int64_t K, int64_t lda, const WT* W, int w_layout, int64_t N,
    int64_t ldw, const float* w_scale, int epi, const T* aux, int64_t ld_aux, int64_t aux_row_mod,
    T* Y, int64_t ldy) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ float As[TK][TM + 4];
  __shared__ float Ws[TK][TN + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t m0 = (int64_t)blockIdx.y * TM, n0 = (int64_t)blockIdx.x * TN;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += TK) {
    for (int i = threadIdx.x; i < TM * TK; i += 256) {
      const int mm = i / TK, kk = i % TK;
      const int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? tof<T>(A[gm * lda + gk]) : 0.f;
    }
    for (int i = threadIdx.x; i < TN * TK; i += 256) {
      int nn, kk;
      if (w_layout == CK_W_NK) {
        nn = i / TK;
        kk = i % TK;
      } else {
        kk = i / TN;
        nn = i % TN;
      }
      const int64_t gn = n0 + nn, gk = k0 + kk;
      float w = 0.f;
      if (gn < N && gk < K) w = tof<WT>(w_layout == CK_W_NK ? W[gn * ldw + gk] : W[gk * ldw + gn]);
      Ws[kk][nn] = w;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Ws[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx + 16 * j;
      if (n >= N) continue;
      float v = acc[i][j];
      if (w_scale != nullptr) v *= w_scale[n];
      v = rnd<T>(v);
      if (epi == CK_EPI_GELU) {
        v = gelu_erf(v);
      } else if (epi == CK_EPI_RESID) {
        const int64_t r = aux_row_mod > 0 ? m % aux_row_mod : m;
        v = tof<T>(aux[r * ld_aux + n]) + v;
      } else if (epi == CK_EPI_BIAS) {
        v = v + tof<T>(aux[n]);
      }
      Y[m * ldy + n] = (T)v;
    }
  }
}

// Skinny outputs (N <= 8, e.g. the behaviour head's D -> 1 projection): one warp
// per row, lanes split K, N dot products reduced with shuffles.
template <typename T, typename WT, int NMAX>
__global__ void __launch_bounds__(256) gemv_rows_kernel(
    const T* A, int64_t M, int64_t K, int64_t lda, const WT* W, int w_layout, int64_t N,
    int64_t ldw, const float* w_scale, int epi, const T* aux, int64_t ld_aux, int64_t aux_row_mod,
    T* Y, int64_t ldy) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t m = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (m >= M) return;
  float acc[NMAX];
#pragma unroll
  for (int n = 0; n < NMAX; ++n) acc[n] = 0.f;
  for (int64_t k = lane; k < K; k += 32) {
    const float a = tof<T>(A[m * lda + k]);
#pragma unroll
    for (int n = 0; n < NMAX; ++n)
      if (n < N)
        acc[n] = fmaf(a, tof<WT>(w_layout == CK_W_NK ? W[n * ldw + k] : W[k * ldw + n]), acc[n]);
  }
#pragma unroll
  for (int n = 0; n < NMAX; ++n) acc[n] = warp_sum(acc[n]);
  if (lane < N) {
    float v = 0.f;
#pragma unroll
    for (int n = 0; n < NMAX; ++n)
      if (n == lane) v = acc[n];
    const int n = lane;
    if (w_scale != nullptr) v *= w_scale[n];
    v = rnd<T>(v);
    if (epi == CK_EPI_GELU) {
      v = gelu_erf(v);
    } else if (epi == CK_EPI_RESID) {
      const int64_t r = aux_row_mod > 0 ? m % aux_row_mod : m;
      v = tof<T>(aux[r * ld_aux + n]) + v;
    } else if (epi == CK_EPI_BIAS) {
      v = v + tof<T>(aux[n]);
    }
    Y[m * ldy + n] = (T)v;
  }
}

template <typename T, typename WT>
int launch(const void* A, int64_t M, int64_t K, int64_t lda, const void* W, int w_layout,
           int64_t N, int64_t ldw, const float* w_scale, int epi, const void* aux, int64_t ld_aux,
           int64_t mod, void* Y, int64_t ldy, cudaStream_t st) {
  if (N <= 8) {
    const int64_t blocks = (M * 32 + 255) / 256;
    if (blocks > INT32_MAX) return CK_ERR_INVALID_ARG;
    return launch_pdl(gemv_rows_kernel<T, WT, 8>, dim3((unsigned)blocks), dim3(256), 0, st,
        reinterpret_cast<const T*>(A), M, K, lda, reinterpret_cast<const WT*>(W), w_layout, N,
        ldw, w_scale, epi, reinterpret_cast<const T*>(aux), ld_aux, mod, reinterpret_cast<T*>(Y),
        ldy);
  }
  dim3 grid((unsigned)((N + TN - 1) / TN), (unsigned)((M + TM - 1) / TM));
  if (grid.y > 65535) return CK_ERR_INVALID_ARG;
  return launch_pdl(gemm_simt_kernel<T, WT>, dim3(grid), dim3(256), 0, st,
      reinterpret_cast<const T*>(A), M, K, lda, reinterpret_cast<const WT*>(W), w_layout, N, ldw,
      w_scale, epi, reinterpret_cast<const T*>(aux), ld_aux, mod, reinterpret_cast<T*>(Y), ldy);
}

}  // namespace

int gemm_simt(const void* A, int dtype, int64_t M, int64_t K, int64_t lda, const void* W,
              int w_dtype, int w_layout, int64_t N, int64_t ldw, const float* w_scale, int epi,
              const void* aux, int64_t ld_aux, int64_t mod, void* Y, int64_t ldy,
              cudaStream_t st) {
  if (M == 0 || N == 0) return CK_OK;
  if (w_dtype == CK_I8 && w_scale == nullptr) return CK_ERR_INVALID_ARG;
  const float* sc = (w_dtype == CK_I8) ? w_scale : nullptr;
  if (dtype == CK_F32) {
    if (w_dtype == CK_F32) return launch<float, float>(A, M, K, lda, W, w_layout, N, ldw, sc, epi, aux, ld_aux, mod, Y, ldy, st);
    if (w_dtype == CK_I8) return launch<float, int8_t>(A, M, K, lda, W, w_layout, N, ldw, sc, epi, aux, ld_aux, mod, Y, ldy, st);
  } else if (dtype == CK_BF16) {
    if (w_dtype == CK_BF16) return launch<__nv_bfloat16, __nv_bfloat16>(A, M, K, lda, W, w_layout, N, ldw, sc, epi, aux, ld_aux, mod, Y, ldy, st);
    if (w_dtype == CK_I8) return launch<__nv_bfloat16, int8_t>(A, M, K, lda, W, w_layout, N, ldw, sc, epi, aux, ld_aux, mod, Y, ldy, st);
  }
  return CK_ERR_UNSUPPORTED;
}

}  // namespace ck
