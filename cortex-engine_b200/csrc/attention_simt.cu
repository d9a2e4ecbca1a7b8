// CUDA-core attention with fp32 arithmetic: the fp32 configurations (which must
// match the reference to 1e-4), head dims other than 64, unaligned layouts, and
// the behaviour head's 2-query attention (cortex/models/cortex.py:44-49).
// Same addressing, masking and empty-row semantics as attention_tc.cu.
//
// One CTA (8 warps) per (batch, head, 32-query tile); each warp owns 4 query
// rows. Keys and values stream through shared memory 32 at a time; within a
// chunk lane i scores key i, and the output accumulates with the probability
// broadcast by shuffles (online softmax, expf).
#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

constexpr int QROWS = 32;
constexpr int KCH = 32;

template <typename T>
__device__ __forceinline__ float tof(T v) {
  return (float)v;
}

template <typename T, int DHMAX>
__global__ void __launch_bounds__(256) attn_simt_kernel(const ck_attention_args p, int num_q_tiles) {
  grid_dep_wait();
  grid_dep_launch();
  extern __shared__ float sm[];
  constexpr int LD = DHMAX + 1;
  float* Qs = sm;
  float* Ks = Qs + QROWS * LD;
  float* Vs = Ks + KCH * LD;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int work = blockIdx.x;
  const int qt = work % num_q_tiles;
  work /= num_q_tiles;
  const int h = work % p.H;
  const int b = work / p.H;
  const int Dh = p.Dh;

  int64_t krow0, vrow0;
  int nk;
  if (p.key_offsets != nullptr) {
    krow0 = vrow0 = p.key_offsets[b];
    nk = p.key_offsets[b + 1] - p.key_offsets[b];
  } else {
    krow0 = (int64_t)b * p.k_rows_per_b;
    vrow0 = (int64_t)b * p.v_rows_per_b;
    nk = p.n_keys;
  }
  krow0 += (int64_t)h * p.k_rows_per_h;
  vrow0 += (int64_t)h * p.v_rows_per_h;
  const T* Q = reinterpret_cast<const T*>(p.q);
  const T* K = reinterpret_cast<const T*>(p.k);
  const T* V = reinterpret_cast<const T*>(p.v);
  T* O = reinterpret_cast<T*>(p.o);
  const int l0 = qt * QROWS;

  for (int i = tid; i < QROWS * Dh; i += 256) {
    const int r = i / Dh, d = i % Dh;
    const int l = l0 + r;
    float v = 0.f;
    if (l < p.Lq)
      v = tof<T>(Q[((int64_t)b * p.q_rows_per_b + (int64_t)h * p.q_rows_per_h + l) * p.q_ld +
                   (int64_t)h * p.q_col_per_h + d]);
    Qs[r * LD + d] = v;
  }

  constexpr int NJ = DHMAX / 32;
  float m[4], lsum[4], o[4][NJ];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    lsum[i] = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) o[i][j] = 0.f;
  }

  for (int e0 = 0; e0 < nk; e0 += KCH) {
    __syncthreads();
    for (int i = tid; i < KCH * Dh; i += 256) {
      const int r = i / Dh, d = i % Dh;
      const int e = e0 + r;
      float kv = 0.f, vv = 0.f;
      if (e < nk) {
        kv = tof<T>(K[(krow0 + e) * p.k_ld + (int64_t)h * p.k_col_per_h + d]);
        vv = tof<T>(V[(vrow0 + e) * p.v_ld + (int64_t)h * p.v_col_per_h + d]);
      }
      Ks[r * LD + d] = kv;
      Vs[r * LD + d] = vv;
    }
    __syncthreads();
    const int e = e0 + lane;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = warp * 4 + i;
      const int l = l0 + r;
      if (l >= p.Lq) continue;  // warp-uniform
      bool valid = e < nk;
      if (valid && p.block_mask != nullptr)
        valid = p.block_mask[(int64_t)(l / p.block_l) * p.n_k_tiles + e / p.block_e] != 0;
      if (valid && p.key_mask != nullptr) valid = p.key_mask[(int64_t)b * p.key_mask_ld + e] != 0;
      float s = -INFINITY;
      if (valid) {
        float acc = 0.f;
        for (int d = 0; d < Dh; ++d) acc = fmaf(Qs[r * LD + d], Ks[lane * LD + d], acc);
        s = acc * p.scale;
      }
      const float cmax = warp_max(s);
      const float m_new = fmaxf(m[i], cmax);
      if (m_new == -INFINITY) continue;  // nothing valid yet for this row (warp-uniform)
      const float alpha = (m[i] == -INFINITY) ? 0.f : expf(m[i] - m_new);
      const float pr = valid ? expf(s - m_new) : 0.f;
      lsum[i] = lsum[i] * alpha + warp_sum(pr);
#pragma unroll
      for (int j = 0; j < NJ; ++j) o[i][j] *= alpha;
      for (int kk = 0; kk < KCH; ++kk) {
        const float pk = __shfl_sync(0xffffffffu, pr, kk);
        if (pk != 0.f) {
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            const int d = lane + 32 * j;
            if (d < Dh) o[i][j] = fmaf(pk, Vs[kk * LD + d], o[i][j]);
          }
        }
      }
      m[i] = m_new;
    }
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = warp * 4 + i;
    const int l = l0 + r;
    if (l >= p.Lq) continue;
    const float inv = lsum[i] > 0.f ? 1.f / lsum[i] : 0.f;
    T* dst = O + ((int64_t)b * p.o_rows_per_b + (int64_t)h * p.o_rows_per_h + l) * p.o_ld +
             (int64_t)h * p.o_col_per_h;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int d = lane + 32 * j;
      if (d < Dh) dst[d] = (T)(o[i][j] * inv);
    }
  }
}

template <typename T, int DHMAX>
int launch(const ck_attention_args& a, cudaStream_t st) {
  const int nqt = (a.Lq + QROWS - 1) / QROWS;
  const int64_t blocks = (int64_t)nqt * a.H * a.B;
  if (blocks == 0) return CK_OK;
  if (blocks > INT32_MAX) return CK_ERR_INVALID_ARG;
  const int smem = (QROWS + 2 * KCH) * (DHMAX + 1) * (int)sizeof(float);
  if (!smem_attr_ready(reinterpret_cast<const void*>(attn_simt_kernel<T, DHMAX>), smem))
    return record_cuda_error();
  return launch_pdl(attn_simt_kernel<T, DHMAX>, dim3((unsigned)blocks), dim3(256), smem, st, a, nqt);
}

}  // namespace

int attention_simt(const ck_attention_args& a, cudaStream_t st) {
  if (a.Dh <= 0 || a.Dh > 256) return CK_ERR_UNSUPPORTED;
  if (a.dtype == CK_F32) {
    if (a.Dh <= 64) return launch<float, 64>(a, st);
    if (a.Dh <= 128) return launch<float, 128>(a, st);
    return launch<float, 256>(a, st);
  }
  if (a.dtype == CK_BF16) {
    if (a.Dh <= 64) return launch<__nv_bfloat16, 64>(a, st);
    if (a.Dh <= 128) return launch<__nv_bfloat16, 128>(a, st);
    return launch<__nv_bfloat16, 256>(a, st);
  }
  return CK_ERR_UNSUPPORTED;
}

}  // namespace ck
