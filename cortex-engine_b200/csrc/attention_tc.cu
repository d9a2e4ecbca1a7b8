// tcgen05 attention for head_dim 64, bf16 (B200, sm_100a).
//
// One CTA (128 threads, two CTAs per SM) per (batch b, head h, 128-query tile).
// The query tile is loaded once by TMA; keys and values stream in 128-key chunks
// through two K and two V buffers with separate barriers, so a K buffer is
// refilled as soon as its S = Q K^T product is done and a V buffer as soon as
// its P V product is done. Per chunk k:
//   S_k = Q K_k^T     tcgen05.mma M=128 N=128 K=64   -> TMEM cols [0,128)
//   softmax           thread r owns query row r (its TMEM lane): the 128 scores
//                     are loaded with four tcgen05.ld and one wait, masked,
//                     reduced with short independent chains (max, sum),
//                     exponentiated with ex2, rounded to bf16 and written as P
//                     into smem (128B-swizzled K-major operand layout)
//   O_k = P_k V_k     tcgen05.mma M=128 N=64 K=128  -> TMEM cols [128,192)
//   o = o * alpha + O  in registers, one chunk late: O_{k-1} is read back after
//                     the softmax of chunk k, so the P V product overlaps it.
// Chunks with no unmasked (query, key) pair for this tile are never loaded.
// Keys of a packed varlen batch start at key_offsets[b]; rows past the last
// event are masked, and the tensor map ends at the last real row so that TMA
// fills anything beyond it with zeros.
//
// This covers the Perceiver cross-attention (latent queries over packed spike
// keys, cortex/models/perceiver.py:54-82), the latent self-attention
// (cortex/models/perceiver.py:107-126), the behaviour head's query attention
// (cortex/models/cortex.py:44-49) and the block-sparse kernel API
// (cortex/kernels/sparse_xattn.py:205-334).
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

constexpr int QT = 128;  // queries per CTA
constexpr int KC = 128;  // keys per chunk
constexpr int DH = 64;
constexpr int TILE_BYTES = QT * DH * 2;  // 16 KB (also one K or V chunk)
constexpr int P_BYTES = QT * KC * 2;     // 32 KB
// Two CTAs per SM: 2 x (SMEM_BYTES + 1 KB reserved) <= 228 KB. The dynamic smem
// base is 1024-byte aligned (no static smem in this kernel); the kernel checks it.
constexpr int SMEM_BYTES = TILE_BYTES * 5 + P_BYTES + 128;
constexpr uint32_t IDESC_S = idesc_bf16(128, 128, 0);
constexpr uint32_t IDESC_O = idesc_bf16(128, 64, 1);

struct TcAttnArgs {
  int B, H, Lq, n_keys, num_q_tiles;
  const int32_t* key_offsets;
  int64_t q_rows_per_b, q_rows_per_h, q_col_per_h;
  int64_t k_rows_per_b, k_rows_per_h, k_col_per_h;
  int64_t v_rows_per_b, v_rows_per_h, v_col_per_h;
  __nv_bfloat16* o;
  int64_t o_ld, o_rows_per_b, o_rows_per_h, o_col_per_h;
  const uint8_t* block_mask;
  int n_q_tiles, n_k_tiles, block_l, block_e;
  const uint8_t* key_mask;  // (B, key_mask_ld) per-key validity, or NULL
  int64_t key_mask_ld;
  float scale_log2;
};

// 2^x with the hardware approximation (ex2.approx(-inf) = +0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool chunk_active(const TcAttnArgs& p, int l0, int l1, int j, int nk) {
  const int e0 = j * KC;
  if (e0 >= nk) return false;
  if (p.block_mask == nullptr) return true;
  const int e1 = min(e0 + KC, nk);
  for (int lt = l0 / p.block_l; lt <= (l1 - 1) / p.block_l; ++lt)
    for (int et = e0 / p.block_e; et <= (e1 - 1) / p.block_e; ++et)
      if (p.block_mask[(int64_t)lt * p.n_k_tiles + et]) return true;
  return false;
}

__device__ __forceinline__ int next_active(const TcAttnArgs& p, int l0, int l1, int j, int nk) {
  const int nch = (nk + KC - 1) / KC;
  for (; j < nch; ++j)
    if (chunk_active(p, l0, l1, j, nk)) return j;
  return -1;
}

// 128 validity bits of this thread's query row for keys e0 .. e0+127.
__device__ __forceinline__ void key_bits(const TcAttnArgs& p, const uint8_t* mask_row,
                                         const uint8_t* kmask, int e0, int nk, uint32_t* vb) {
  const int lim = nk - e0;  // keys past the sample are invalid
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int lo = w * 32;
    vb[w] = (lim <= lo) ? 0u : (lim >= lo + 32 ? 0xffffffffu : ((1u << (lim - lo)) - 1u));
  }
  if (mask_row != nullptr) {
    const int t0 = e0 / p.block_e;
    const int t1 = (min(e0 + KC, nk) - 1) / p.block_e;
    for (int t = t0; t <= t1; ++t) {
      if (mask_row[t]) continue;
      const int a = max(t * p.block_e - e0, 0);
      const int b = min((t + 1) * p.block_e - e0, KC);
      for (int c = a; c < b; ++c) vb[c >> 5] &= ~(1u << (c & 31));
    }
  }
  if (kmask != nullptr) {
    for (int c = 0; c < KC && c < lim; ++c)
      if (!kmask[e0 + c]) vb[c >> 5] &= ~(1u << (c & 31));
  }
}

template <bool MASKED>
__global__ void __launch_bounds__(128, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const TcAttnArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {  // swizzled operand tiles need 1 KB alignment
    grid_dep_wait();
    if (threadIdx.x == 0) set_status(CK_ERR_INVALID_ARG, 1024, (int)(smem_u32(smem_raw) & 1023u));
    return;
  }
  uint8_t* sQ = smem_raw;
  uint8_t* sK = sQ + TILE_BYTES;      // 2 buffers
  uint8_t* sV = sK + 2 * TILE_BYTES;  // 2 buffers
  uint8_t* sP = sV + 2 * TILE_BYTES;  // 2 x 16 KB atoms (keys 0..63, 64..127)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + P_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;  // [2]
  uint64_t* v_full = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* o_full = bars + 6;
  uint64_t* drain = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid / 32;
  const int lane = tid % 32;

  int work = blockIdx.x;
  const int qt = work % p.num_q_tiles;
  work /= p.num_q_tiles;
  const int h = work % p.H;
  const int b = work / p.H;

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_wait();
  grid_dep_launch();
  int64_t key_row0;
  int nk;
  if (p.key_offsets != nullptr) {
    key_row0 = p.key_offsets[b];
    nk = p.key_offsets[b + 1] - p.key_offsets[b];
  } else {
    key_row0 = (int64_t)b * p.k_rows_per_b;
    nk = p.n_keys;
  }
  const int64_t v_row0 = (p.key_offsets != nullptr) ? key_row0 : (int64_t)b * p.v_rows_per_b;
  const int l0 = qt * QT;
  const int l1 = min(l0 + QT, p.Lq);
  const int q_row = (int)((int64_t)b * p.q_rows_per_b + (int64_t)h * p.q_rows_per_h + l0);
  const int q_col = (int)((int64_t)h * p.q_col_per_h);
  const int k_row_h = (int)(key_row0 + (int64_t)h * p.k_rows_per_h);
  const int k_col = (int)((int64_t)h * p.k_col_per_h);
  const int v_row_h = (int)(v_row0 + (int64_t)h * p.v_rows_per_h);
  const int v_col = (int)((int64_t)h * p.v_col_per_h);

  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_s = tmem_base;
  const uint32_t tmem_o = tmem_base + 128;

  const int row = warp * 32 + lane;  // query row within the tile == TMEM lane
  const int l = l0 + row;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const uint8_t* mask_row = nullptr;
  const uint8_t* kmask = nullptr;
  if (MASKED) {
    if (p.block_mask != nullptr && l < p.Lq)
      mask_row = p.block_mask + (int64_t)(l / p.block_l) * p.n_k_tiles;
    if (p.key_mask != nullptr) kmask = p.key_mask + (int64_t)b * p.key_mask_ld;
  }

  float o_acc[DH];
#pragma unroll
  for (int i = 0; i < DH; ++i) o_acc[i] = 0.f;
  float m_i = -INFINITY;
  float l_i = 0.f;
  float alpha_pend = 0.f;  // rescale factor that goes with the O not yet added
  int k_loads0 = 0, k_loads1 = 0, v_loads0 = 0, v_loads1 = 0;  // thread 0 only

  // chunk schedule: current, next and the one after (active chunks only)
  int c_cur = next_active(p, l0, l1, 0, nk);
  int c_next = c_cur >= 0 ? next_active(p, l0, l1, c_cur + 1, nk) : -1;
  int c_next2 = c_next >= 0 ? next_active(p, l0, l1, c_next + 1, nk) : -1;

  if (tid == 0 && c_cur >= 0) {
    mbar_arrive_expect_tx(q_full, TILE_BYTES);
    tma_load_2d(sQ, &tmQ, q_full, q_col, q_row);
    mbar_arrive_expect_tx(&k_full[0], TILE_BYTES);
    tma_load_2d(sK, &tmK, &k_full[0], k_col, k_row_h + c_cur * KC);
    mbar_arrive_expect_tx(&v_full[0], TILE_BYTES);
    tma_load_2d(sV, &tmV, &v_full[0], v_col, v_row_h + c_cur * KC);
    k_loads0 = v_loads0 = 1;
    if (c_next >= 0) {
      mbar_arrive_expect_tx(&k_full[1], TILE_BYTES);
      tma_load_2d(sK + TILE_BYTES, &tmK, &k_full[1], k_col, k_row_h + c_next * KC);
      mbar_arrive_expect_tx(&v_full[1], TILE_BYTES);
      tma_load_2d(sV + TILE_BYTES, &tmV, &v_full[1], v_col, v_row_h + c_next * KC);
      k_loads1 = v_loads1 = 1;
    }
    if (mbar_wait(q_full, 0, abort_flag, 20) && mbar_wait(&k_full[0], 0, abort_flag, 21)) {
      tc_fence_after();
      const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK);
#pragma unroll
      for (int k = 0; k < DH / 16; ++k)
        tc_mma_ss(tmem_s, sw128_desc(qa + k * 32, 16, 1024), sw128_desc(ka + k * 32, 16, 1024),
                  IDESC_S, k != 0);
      tc_commit(s_full);
    }
  }

  int it = 0;
  bool ok = true;
  while (c_cur >= 0) {
    const int buf = it & 1;
    if (!mbar_wait(s_full, (uint32_t)(it & 1), abort_flag, 22)) {
      ok = false;
      break;
    }
    tc_fence_after();
    // K buffer `buf` is free once S_it is done: prefetch the chunk two ahead
    if (tid == 0 && c_next2 >= 0) {
      mbar_arrive_expect_tx(&k_full[buf], TILE_BYTES);
      tma_load_2d(sK + buf * TILE_BYTES, &tmK, &k_full[buf], k_col, k_row_h + c_next2 * KC);
      if (buf) ++k_loads1; else ++k_loads0;
    }
    float s[KC];
#pragma unroll
    for (int g = 0; g < 4; ++g) tmem_ld32(tmem_s + lane_off + g * 32, s + 32 * g);
    tc_wait_ld();
    const int e0 = c_cur * KC;
    if (MASKED) {
      uint32_t vb[4];
      key_bits(p, mask_row, kmask, e0, nk, vb);
#pragma unroll
      for (int c = 0; c < KC; ++c)
        if (!((vb[c >> 5] >> (c & 31)) & 1u)) s[c] = -INFINITY;
    } else if (e0 + KC > nk) {
      const int lim = nk - e0;
#pragma unroll
      for (int c = 0; c < KC; ++c)
        if (c >= lim) s[c] = -INFINITY;
    }
    // row max over 8 independent chains, new running max, rescale factor
    float t[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) t[c] = s[c];
#pragma unroll
    for (int c = 8; c < KC; ++c) t[c & 7] = fmaxf(t[c & 7], s[c]);
    const float cmax = fmaxf(fmaxf(fmaxf(t[0], t[1]), fmaxf(t[2], t[3])),
                             fmaxf(fmaxf(t[4], t[5]), fmaxf(t[6], t[7]))) *
                       p.scale_log2;  // scale > 0: max commutes with it
    const float m_new = fmaxf(m_i, cmax);
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = (m_i == -INFINITY) ? 0.f : ex2(m_i - m_use);
    // probabilities and their sum
#pragma unroll
    for (int c = 0; c < KC; ++c) s[c] = ex2(fmaf(s[c], p.scale_log2, -m_use));
#pragma unroll
    for (int c = 0; c < 8; ++c) t[c] = s[c];
#pragma unroll
    for (int c = 8; c < KC; ++c) t[c & 7] += s[c];
    l_i = l_i * alpha + (((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7])));
    m_i = m_new;

    // P_{it-1} and V of chunk it-1 are released once the previous P V is done
    if (it > 0 && !mbar_wait(o_full, (uint32_t)((it - 1) & 1), abort_flag, 24)) {
      ok = false;
      break;
    }
    // P_it -> smem (bf16, 128B swizzle, keys 0..63 in atom 0, 64..127 in atom 1)
#pragma unroll
    for (int g = 0; g < 16; ++g) {
      uint8_t* atom = sP + (g >> 3) * (QT * 128);
      *reinterpret_cast<uint4*>(atom + sw128_off(row, g & 7)) = pack8(s + 8 * g);
    }
    fence_proxy_async_smem();
    if (it > 0) {
      // add the previous chunk's O (TMEM is rewritten only after the barrier below)
      tc_fence_after();
      float ov[DH];
      tmem_ld32(tmem_o + lane_off, ov);
      tmem_ld32(tmem_o + lane_off + 32, ov + 32);
      tc_wait_ld();
#pragma unroll
      for (int i = 0; i < DH; ++i) o_acc[i] = fmaf(o_acc[i], alpha_pend, ov[i]);
      // V buffer of chunk it-1 is free: load the next chunk's V into it
      if (tid == 0 && c_next >= 0) {
        const int vb_ = buf ^ 1;
        mbar_arrive_expect_tx(&v_full[vb_], TILE_BYTES);
        tma_load_2d(sV + vb_ * TILE_BYTES, &tmV, &v_full[vb_], v_col, v_row_h + c_next * KC);
        if (vb_) ++v_loads1; else ++v_loads0;
      }
    }
    alpha_pend = alpha;
    tc_fence_before();
    __syncthreads();

    if (tid == 0) {
      tc_fence_after();
      // O_it = P_it V_it
      if (mbar_wait(&v_full[buf], (uint32_t)((it >> 1) & 1), abort_flag, 25)) {
        const uint32_t pa = smem_u32(sP), va = smem_u32(sV + buf * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < KC / 16; ++k) {
          const uint64_t adesc = sw128_desc(pa + (k >> 2) * (QT * 128) + (k & 3) * 32, 16, 1024);
          const uint64_t bdesc = sw128_desc(va + k * 16 * 128, 8192, 1024);
          tc_mma_ss(tmem_o, adesc, bdesc, IDESC_O, k != 0);
        }
        tc_commit(o_full);
      }
      // S_{it+1} = Q K_{it+1}^T
      if (c_next >= 0 &&
          mbar_wait(&k_full[buf ^ 1], (uint32_t)(((it + 1) >> 1) & 1), abort_flag, 23)) {
        tc_fence_after();
        const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK + (buf ^ 1) * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < DH / 16; ++k)
          tc_mma_ss(tmem_s, sw128_desc(qa + k * 32, 16, 1024), sw128_desc(ka + k * 32, 16, 1024),
                    IDESC_S, k != 0);
        tc_commit(s_full);
      }
    }
    c_cur = c_next;
    c_next = c_next2;
    c_next2 = c_next2 >= 0 ? next_active(p, l0, l1, c_next2 + 1, nk) : -1;
    ++it;
    if (*abort_flag) {
      ok = false;
      break;
    }
  }

  // the last chunk's O
  if (ok && it > 0 && mbar_wait(o_full, (uint32_t)((it - 1) & 1), abort_flag, 26)) {
    tc_fence_after();
    float ov[DH];
    tmem_ld32(tmem_o + lane_off, ov);
    tmem_ld32(tmem_o + lane_off + 32, ov + 32);
    tc_wait_ld();
#pragma unroll
    for (int i = 0; i < DH; ++i) o_acc[i] = fmaf(o_acc[i], alpha_pend, ov[i]);
  }

  // store the normalised output row
  if (l < p.Lq) {
    const float inv = (l_i > 0.f) ? 1.f / l_i : 0.f;
    __nv_bfloat16* dst = p.o + ((int64_t)b * p.o_rows_per_b + (int64_t)h * p.o_rows_per_h + l) *
                                   p.o_ld +
                         (int64_t)h * p.o_col_per_h;
#pragma unroll
    for (int c = 0; c < DH / 8; ++c) {
      float f[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = o_acc[c * 8 + i] * inv;
      *reinterpret_cast<uint4*>(dst + c * 8) = pack8(f);
    }
  }

  // drain: outstanding MMAs and TMA loads must finish before TMEM/smem go away
  if (tid == 0) {
    tc_commit(drain);
    mbar_wait(drain, 0, nullptr, 28);
    if (k_loads0 > 0) mbar_wait(q_full, 0, nullptr, 29);
    if (k_loads0 > 0) mbar_wait(&k_full[0], (uint32_t)((k_loads0 - 1) & 1), nullptr, 30);
    if (k_loads1 > 0) mbar_wait(&k_full[1], (uint32_t)((k_loads1 - 1) & 1), nullptr, 30);
    if (v_loads0 > 0) mbar_wait(&v_full[0], (uint32_t)((v_loads0 - 1) & 1), nullptr, 31);
    if (v_loads1 > 0) mbar_wait(&v_full[1], (uint32_t)((v_loads1 - 1) & 1), nullptr, 31);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 256);
  }
}

}  // namespace

bool attention_tc_supported(const ck_attention_args& a) {
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (a.dtype != CK_BF16 || a.Dh != DH) return false;
  if (!al16(a.q) || !al16(a.k) || !al16(a.v) || !al16(a.o)) return false;
  if ((a.q_ld * 2) % 16 || (a.k_ld * 2) % 16 || (a.v_ld * 2) % 16 || (a.o_ld * 2) % 16) return false;
  if ((a.q_col_per_h * 2) % 16 || (a.k_col_per_h * 2) % 16 || (a.v_col_per_h * 2) % 16 ||
      (a.o_col_per_h * 2) % 16)
    return false;
  if (a.q_rows > INT32_MAX || a.k_rows > INT32_MAX || a.v_rows > INT32_MAX) return false;
  if (a.block_mask != nullptr && (a.block_l <= 0 || a.block_e <= 0)) return false;
  return true;
}

int attention_tc(const ck_attention_args& a, cudaStream_t st) {
  TcAttnArgs p;
  p.B = a.B;
  p.H = a.H;
  p.Lq = a.Lq;
  p.n_keys = a.n_keys;
  p.num_q_tiles = (a.Lq + QT - 1) / QT;
  p.key_offsets = a.key_offsets;
  p.q_rows_per_b = a.q_rows_per_b;
  p.q_rows_per_h = a.q_rows_per_h;
  p.q_col_per_h = a.q_col_per_h;
  p.k_rows_per_b = a.k_rows_per_b;
  p.k_rows_per_h = a.k_rows_per_h;
  p.k_col_per_h = a.k_col_per_h;
  p.v_rows_per_b = a.v_rows_per_b;
  p.v_rows_per_h = a.v_rows_per_h;
  p.v_col_per_h = a.v_col_per_h;
  p.o = reinterpret_cast<__nv_bfloat16*>(a.o);
  p.o_ld = a.o_ld;
  p.o_rows_per_b = a.o_rows_per_b;
  p.o_rows_per_h = a.o_rows_per_h;
  p.o_col_per_h = a.o_col_per_h;
  p.block_mask = a.block_mask;
  p.n_q_tiles = a.n_q_tiles;
  p.n_k_tiles = a.n_k_tiles;
  p.block_l = a.block_l > 0 ? a.block_l : 1;
  p.block_e = a.block_e > 0 ? a.block_e : 1;
  p.key_mask = a.key_mask;
  p.key_mask_ld = a.key_mask_ld;
  p.scale_log2 = a.scale * 1.4426950408889634f;

  CUtensorMap tq, tk, tv;
  if (!make_tmap_2d(&tq, a.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.q_ld, a.q_rows, a.q_ld, 64,
                    QT, 128) ||
      !make_tmap_2d(&tk, a.k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.k_ld, a.k_rows, a.k_ld, 64,
                    KC, 128) ||
      !make_tmap_2d(&tv, a.v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.v_ld, a.v_rows, a.v_ld, 64,
                    KC, 128))
    return CK_ERR_INVALID_ARG;

  const bool masked = a.block_mask != nullptr || a.key_mask != nullptr;
  const void* kern = masked ? reinterpret_cast<const void*>(attn_tc_kernel<true>)
                            : reinterpret_cast<const void*>(attn_tc_kernel<false>);
  if (!smem_attr_ready(kern, SMEM_BYTES)) return record_cuda_error();
  const int64_t blocks = (int64_t)p.num_q_tiles * a.H * a.B;
  if (blocks <= 0) return CK_OK;
  if (blocks > INT32_MAX) return CK_ERR_INVALID_ARG;
  if (masked)
    return launch_pdl(attn_tc_kernel<true>, dim3((unsigned)blocks), dim3(128), SMEM_BYTES, st, tq,
                      tk, tv, p);
  return launch_pdl(attn_tc_kernel<false>, dim3((unsigned)blocks), dim3(128), SMEM_BYTES, st, tq,
                    tk, tv, p);
}

}  // namespace ck
