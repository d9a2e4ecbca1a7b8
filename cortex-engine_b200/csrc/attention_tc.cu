// tcgen05 attention for head_dim 64, bf16 (B200, sm_100a).
//
// One CTA (128 threads) per (batch b, head h, 128-query tile). The query tile
// is loaded once by TMA; keys and values stream in 128-key chunks through a
// double-buffered TMA ring. Per chunk:
//   S  = Q K^T        tcgen05.mma M=128 N=128 K=64   -> TMEM cols [0,128)
//   softmax           each thread owns one query row (its TMEM lane): scores
//                     are masked (key count, optional tile mask), the running
//                     max/sum updated in fp32 and P = exp2(s - m) written to
//                     smem as bf16 in the 128B-swizzled K-major layout
//   O_j = P V         tcgen05.mma M=128 N=64 K=128  -> TMEM cols [128,192)
//   o  = o*alpha + O_j   in registers (fp32)
// Chunks with no unmasked (query, key) pair for this tile are never loaded.
// Keys of a packed varlen batch start at key_offsets[b]; rows past the last
// event are masked, and the tensor map ends at the last real row so that TMA
// fills anything beyond it with zeros.
//
// This covers the Perceiver cross-attention (latent queries over packed spike
// keys, cortex/models/perceiver.py:54-82), the latent self-attention
// (cortex/models/perceiver.py:107-126) and the block-sparse kernel API
// (cortex/kernels/sparse_xattn.py:205-334).
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

constexpr int QT = 128;  // queries per CTA
constexpr int KC = 128;  // keys per chunk
constexpr int DH = 64;
constexpr int TILE_BYTES = QT * DH * 2;  // 16 KB (also K/V chunk size)
constexpr int P_BYTES = QT * KC * 2;     // 32 KB
// Two CTAs per SM: 2 x (114816 + 1024 reserved) <= 228 KB. The dynamic smem base
// is 1024-byte aligned (no static smem in this kernel); the kernel checks it.
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

__global__ void __launch_bounds__(128, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const TcAttnArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {  // swizzled operand tiles need 1 KB alignment
    if (threadIdx.x == 0) set_status(CK_ERR_INVALID_ARG, 1024, (int)(smem_u32(smem_raw) & 1023u));
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + TILE_BYTES;            // 2 buffers
  uint8_t* sV = sK + 2 * TILE_BYTES;        // 2 buffers
  uint8_t* sP = sV + 2 * TILE_BYTES;        // 2 x 16 KB atoms (keys 0..63, 64..127)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + P_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;  // [2]
  uint64_t* s_full = bars + 3;
  uint64_t* o_full = bars + 4;
  uint64_t* drain = bars + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid / 32;
  const int lane = tid % 32;

  int work = blockIdx.x;
  const int qt = work % p.num_q_tiles;
  work /= p.num_q_tiles;
  const int h = work % p.H;
  const int b = work / p.H;

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

  if (tid == 0) {
    mbar_init(q_full, 1);
    mbar_init(&kv_full[0], 1);
    mbar_init(&kv_full[1], 1);
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
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_s = tmem_base;
  const uint32_t tmem_o = tmem_base + 128;

  const int row = warp * 32 + lane;  // query row within the tile == TMEM lane
  const int l = l0 + row;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;

  float o_acc[DH];
#pragma unroll
  for (int i = 0; i < DH; ++i) o_acc[i] = 0.f;
  float m_i = -INFINITY;
  float l_i = 0.f;
  int tma_issued[2] = {0, 0};  // loads issued per K/V buffer (thread 0 only)
  bool q_issued = false;

  int j = next_active(p, l0, l1, 0, nk);
  if (tid == 0 && j >= 0) {
    mbar_arrive_expect_tx(q_full, TILE_BYTES);
    tma_load_2d(sQ, &tmQ, q_full, q_col, q_row);
    q_issued = true;
    mbar_arrive_expect_tx(&kv_full[0], 2 * TILE_BYTES);
    tma_load_2d(sK, &tmK, &kv_full[0], k_col, k_row_h + j * KC);
    tma_load_2d(sV, &tmV, &kv_full[0], v_col, v_row_h + j * KC);
    tma_issued[0] = 1;
    int j1 = next_active(p, l0, l1, j + 1, nk);
    if (j1 >= 0) {
      mbar_arrive_expect_tx(&kv_full[1], 2 * TILE_BYTES);
      tma_load_2d(sK + TILE_BYTES, &tmK, &kv_full[1], k_col, k_row_h + j1 * KC);
      tma_load_2d(sV + TILE_BYTES, &tmV, &kv_full[1], v_col, v_row_h + j1 * KC);
      tma_issued[1] = 1;
    }
    bool ok = mbar_wait(q_full, 0, abort_flag, 20) && mbar_wait(&kv_full[0], 0, abort_flag, 21);
    if (ok) {
      tc_fence_after();
      const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK);
#pragma unroll
      for (int k = 0; k < DH / 16; ++k)
        tc_mma_ss(tmem_s, sw128_desc(qa + k * 32, 16, 1024), sw128_desc(ka + k * 32, 16, 1024),
                  IDESC_S, k != 0);
      tc_commit(s_full);
    }
  }

  const uint8_t* mask_row = nullptr;
  if (p.block_mask != nullptr && l < p.Lq)
    mask_row = p.block_mask + (int64_t)(l / p.block_l) * p.n_k_tiles;
  const uint8_t* kmask = (p.key_mask != nullptr) ? p.key_mask + (int64_t)b * p.key_mask_ld : nullptr;

  int it = 0;
  while (j >= 0) {
    const int buf = it & 1;
    if (!mbar_wait(s_full, (uint32_t)(it & 1), abort_flag, 22)) break;
    tc_fence_after();
    const int e0 = j * KC;
    // pass 1: masked row max of this chunk
    float cmax = -INFINITY;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      float s[32];
      tmem_ld32(tmem_s + lane_off + g * 32, s);
      tc_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int e = e0 + g * 32 + c;
        bool valid = e < nk;
        if (mask_row != nullptr && valid) valid = mask_row[e / p.block_e] != 0;
        if (kmask != nullptr && valid) valid = kmask[e] != 0;
        if (valid) cmax = fmaxf(cmax, s[c] * p.scale_log2);
      }
    }
    const float m_new = fmaxf(m_i, cmax);
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = (m_i == -INFINITY) ? 0.f : exp2f(m_i - m_use);
    // pass 2: probabilities -> bf16 P tile, row sum
    float psum = 0.f;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
      float s[32];
      tmem_ld32(tmem_s + lane_off + g * 32, s);
      tc_wait_ld();
      float pr[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int e = e0 + g * 32 + c;
        bool valid = e < nk;
        if (mask_row != nullptr && valid) valid = mask_row[e / p.block_e] != 0;
        if (kmask != nullptr && valid) valid = kmask[e] != 0;
        pr[c] = valid ? exp2f(s[c] * p.scale_log2 - m_use) : 0.f;
        psum += pr[c];
      }
      uint8_t* atom = sP + (g >> 1) * (QT * 128);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4)
        *reinterpret_cast<uint4*>(atom + sw128_off(row, (g & 1) * 4 + q4)) = pack8(pr + 8 * q4);
    }
    l_i = l_i * alpha + psum;
    m_i = m_new;
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    int jn = -1;
    if (tid == 0) {
      tc_fence_after();
      // O_j = P V_j
      const uint32_t pa = smem_u32(sP), va = smem_u32(sV + buf * TILE_BYTES);
#pragma unroll
      for (int k = 0; k < KC / 16; ++k) {
        uint64_t adesc = sw128_desc(pa + (k >> 2) * (QT * 128) + (k & 3) * 32, 16, 1024);
        uint64_t bdesc = sw128_desc(va + k * 16 * 128, 8192, 1024);
        tc_mma_ss(tmem_o, adesc, bdesc, IDESC_O, k != 0);
      }
      tc_commit(o_full);
      // S_{next} = Q K_next (next chunk already in the other buffer)
      jn = next_active(p, l0, l1, j + 1, nk);
      if (jn >= 0) {
        const int nb = buf ^ 1;
        if (mbar_wait(&kv_full[nb], (uint32_t)(((it + 1) >> 1) & 1), abort_flag, 23)) {
          tc_fence_after();
          const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK + nb * TILE_BYTES);
#pragma unroll
          for (int k = 0; k < DH / 16; ++k)
            tc_mma_ss(tmem_s, sw128_desc(qa + k * 32, 16, 1024),
                      sw128_desc(ka + k * 32, 16, 1024), IDESC_S, k != 0);
          tc_commit(s_full);
        }
      }
    }
    if (!mbar_wait(o_full, (uint32_t)(it & 1), abort_flag, 24)) break;
    tc_fence_after();
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      float ov[32];
      tmem_ld32(tmem_o + lane_off + g * 32, ov);
      tc_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c) o_acc[g * 32 + c] = o_acc[g * 32 + c] * alpha + ov[c];
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && jn >= 0) {
      // prefetch the chunk after next into the buffer PV_j has finished with
      const int j2 = next_active(p, l0, l1, jn + 1, nk);
      if (j2 >= 0) {
        mbar_arrive_expect_tx(&kv_full[buf], 2 * TILE_BYTES);
        tma_load_2d(sK + buf * TILE_BYTES, &tmK, &kv_full[buf], k_col, k_row_h + j2 * KC);
        tma_load_2d(sV + buf * TILE_BYTES, &tmV, &kv_full[buf], v_col, v_row_h + j2 * KC);
        tma_issued[buf] += 1;
      }
    }
    // all threads agree on the next chunk (same deterministic scan)
    j = next_active(p, l0, l1, j + 1, nk);
    ++it;
    if (*abort_flag) break;
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
    if (q_issued) mbar_wait(q_full, 0, nullptr, 29);
    for (int bb = 0; bb < 2; ++bb)
      if (tma_issued[bb] > 0) mbar_wait(&kv_full[bb], (uint32_t)((tma_issued[bb] - 1) & 1), nullptr, 30);
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

  if (!smem_attr_ready(reinterpret_cast<const void*>(attn_tc_kernel), SMEM_BYTES))
    return record_cuda_error();
  const int64_t blocks = (int64_t)p.num_q_tiles * a.H * a.B;
  if (blocks <= 0) return CK_OK;
  if (blocks > INT32_MAX) return CK_ERR_INVALID_ARG;
  attn_tc_kernel<<<(unsigned)blocks, 128, SMEM_BYTES, st>>>(tq, tk, tv, p);
  return check_launch();
}

}  // namespace ck
