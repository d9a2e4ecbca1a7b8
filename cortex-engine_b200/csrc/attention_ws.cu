// Warp-specialised tcgen05 attention for head_dim 64, bf16, without block or
// key masks: the Perceiver cross-attention over packed varlen keys
// (cortex/models/perceiver.py:54-82) and the latent self-attention
// (cortex/models/perceiver.py:107-126).
//
// Two persistent CTAs per SM walk the (batch, head, 128-query tile) work items
// with a stride of the grid. Each CTA runs one in-order pipeline over the
// 128-key chunks of its items:
//   warp 8   TMA producer: the item's Q tile, then K and V of every chunk into
//            a two-stage ring (the next item's loads start while the current
//            item is still in its softmax)
//   warp 9   TMEM owner and MMA issuer:
//              S_g   = Q K_g^T          M=128 N=128 K=64 -> TMEM cols [0,128)
//              O_h  += P_g,h V_g,h      M=128 N=64  K=64 -> TMEM cols [128+64h, +64)
//            for the two key halves h (keys 64h .. 64h+63 of the chunk).
//            S_{g+1} is issued as soon as the softmax has read S_g, so the next
//            product runs under the current chunk's softmax
//   warps 0-7 softmax, two warps per TMEM lane quarter: warp w takes query
//            row r = 32 (w % 4) + lane and key half h = w / 4 of every chunk:
//            its 64 scores from TMEM, its own running max and row sum, exp2,
//            and the 64-key atom h of P (bf16, 128B-swizzled smem operand).
//            The halves are two independent online softmaxes with their own
//            accumulators O_0, O_1, so the two warps of a row never wait for
//            each other inside an item. Two warps per row halve each thread's
//            dependent chain and give every scheduler four softmax warps (two
//            CTAs per SM) to hide its latencies with.
// An item's output is written once the next item's first chunk has been
// exponentiated (or at the end): half 1 divides O_1 by its row sum in TMEM and
// publishes its log2-sum-exp c_1 = m_1 + log2 l_1; half 0 combines
//   O = (O_0 / l_0) w_0 + (O_1 / l_1) w_1,  w_h = 2^c_h / (2^c_0 + 2^c_1),
// and writes the row. Each half keeps a running base m and rescales its O_h
// (in TMEM) only when a chunk's maximum exceeds m by more than 2^8; otherwise
// P = exp2(s - m) <= 256 is used as is, which is exact in real arithmetic after
// the final division. All waits are bounded.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

constexpr int QT = 128;  // queries per work item
constexpr int KC = 128;  // keys per chunk
constexpr int DH = 64;
constexpr int Q_BYTES = QT * DH * 2;    // 16 KB
constexpr int KV_BYTES = KC * DH * 2;   // 16 KB: one K or one V chunk
constexpr int P_BYTES = QT * KC * 2;    // 32 KB: two 128B-swizzled atoms
constexpr int STAGES = 2;               // K/V ring
constexpr int NTHREADS = 320;           // softmax warps 0-7, producer warp 8, MMA warp 9
constexpr int NSOFT = 256;              // softmax threads: two per query row
constexpr int BAR_BYTES = 256;
constexpr int XCH_BYTES = QT * 4;       // c_1 of every row, from key half 1 to half 0
constexpr int CTAS_PER_SM = 2;          // 2 x (SMEM_BYTES + 1 KB) <= 228 KB; 2 x 256 TMEM cols
constexpr int SMEM_BYTES = Q_BYTES + STAGES * 2 * KV_BYTES + P_BYTES + XCH_BYTES + BAR_BYTES;
constexpr uint32_t TMEM_COLS = 256;     // S [0, 128), O_0 [128, 192), O_1 [192, 256)
constexpr int KH = KC / 2;              // keys per half chunk
constexpr uint32_t IDESC_S = idesc_bf16(128, KC, 0);
constexpr uint32_t IDESC_O = idesc_bf16(128, DH, 1);
constexpr float kRescaleLog2 = 8.f;
static_assert(2 * (SMEM_BYTES + 1024) <= 228 * 1024, "two CTAs per SM");

struct WsArgs {
  int B, H, Lq, n_keys, num_q_tiles, num_items;
  const int32_t* key_offsets;
  int64_t q_rows_per_b, q_rows_per_h, q_col_per_h;
  int64_t k_rows_per_b, k_rows_per_h, k_col_per_h;
  int64_t v_rows_per_b, v_rows_per_h, v_col_per_h;
  __nv_bfloat16* o;
  int64_t o_ld, o_rows_per_b, o_rows_per_h, o_col_per_h;
  float scale_log2;
};

struct Item {
  int b, h, l0, nk, nch;
  int q_row, q_col, k_row, k_col, v_row, v_col;
};

// Work item w = ((b * H) + h) * num_q_tiles + q tile. Every role derives the
// same chunk count from it, so they agree on the pipeline's sequence.
__device__ __forceinline__ Item make_item(const WsArgs& p, int w) {
  Item it;
  const int qt = w % p.num_q_tiles;
  w /= p.num_q_tiles;
  it.h = w % p.H;
  it.b = w / p.H;
  int64_t key_row0;
  if (p.key_offsets != nullptr) {
    key_row0 = p.key_offsets[it.b];
    it.nk = p.key_offsets[it.b + 1] - p.key_offsets[it.b];
  } else {
    key_row0 = (int64_t)it.b * p.k_rows_per_b;
    it.nk = p.n_keys;
  }
  const int64_t v_row0 = (p.key_offsets != nullptr) ? key_row0 : (int64_t)it.b * p.v_rows_per_b;
  it.l0 = qt * QT;
  it.nch = it.nk > 0 ? (it.nk + KC - 1) / KC : 0;
  it.q_row = (int)((int64_t)it.b * p.q_rows_per_b + (int64_t)it.h * p.q_rows_per_h + it.l0);
  it.q_col = (int)((int64_t)it.h * p.q_col_per_h);
  it.k_row = (int)(key_row0 + (int64_t)it.h * p.k_rows_per_h);
  it.k_col = (int)((int64_t)it.h * p.k_col_per_h);
  it.v_row = (int)(v_row0 + (int64_t)it.h * p.v_rows_per_h);
  it.v_col = (int)((int64_t)it.h * p.v_col_per_h);
  return it;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 16 consecutive fp32 TMEM columns of this thread's lane, and the store back.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

__device__ __forceinline__ void tc_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(NTHREADS, CTAS_PER_SM)
    attn_ws_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const WsArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {  // swizzled operand tiles need 1 KB alignment
    grid_dep_wait();
    if (threadIdx.x == 0) set_status(CK_ERR_INVALID_ARG, 1024, (int)(smem_u32(smem_raw) & 1023u));
    return;
  }
  uint8_t* sQ = smem_raw;
  uint8_t* sKV = sQ + Q_BYTES;  // [STAGES][K chunk | V chunk]
  uint8_t* sP = sKV + STAGES * 2 * KV_BYTES;
  float* xlse = reinterpret_cast<float*>(sP + P_BYTES);  // [QT]: c_1 per row
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + P_BYTES + XCH_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;    // [STAGES]
  uint64_t* v_full = bars + 4;    // [STAGES]
  uint64_t* k_empty = bars + 6;   // [STAGES] the stage's K was read by its QK^T
  uint64_t* s_full = bars + 8;
  uint64_t* s_free = bars + 9;
  uint64_t* p_full = bars + 10;   // [2 key halves]
  uint64_t* o_full = bars + 12;   // [2 key halves]
  uint64_t* o_free = bars + 14;
  uint64_t* drain = bars + 15;
  uint64_t* x_ready = bars + 16;  // [4 lane quarters]: half 1 published c_1, O_1 / l_1
  uint64_t* v_empty = bars + 20;  // [STAGES] the stage's V was read by its two P V products
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid / 32;
  const int lane = tid % 32;

  if (tid == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, NSOFT);
    for (int h = 0; h < 2; ++h) {
      mbar_init(&p_full[h], NSOFT / 2);
      mbar_init(&o_full[h], 1);
    }
    mbar_init(o_free, NSOFT);
    mbar_init(drain, 1);
    for (int q = 0; q < 4; ++q) mbar_init(&x_ready[q], 32);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_wait();
  grid_dep_launch();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_s = tmem_base;
  const uint32_t tmem_o = tmem_base + 128;

  if (warp == 8) {
    // ── TMA producer ──
    if (lane == 0) {
      int g = 0, nq = 0;
      int kv_loads[STAGES] = {0, 0};
      bool ok = true;
      for (int w = blockIdx.x; w < p.num_items && ok; w += gridDim.x) {
        const Item it = make_item(p, w);
        if (it.nch == 0) continue;
        if (!mbar_wait(q_empty, (uint32_t)((nq & 1) ^ 1), abort_flag, 40)) break;
        mbar_arrive_expect_tx(q_full, Q_BYTES);
        tma_load_2d(sQ, &tmQ, q_full, it.q_col, it.q_row);
        ++nq;
        for (int j = 0; j < it.nch; ++j, ++g) {
          const int st = g & 1;
          // K and V of a stage are released separately: the next K can load
          // as soon as the QK^T that read this one is done
          uint8_t* kv = sKV + st * 2 * KV_BYTES;
          if (!mbar_wait(&k_empty[st], (uint32_t)(((g >> 1) & 1) ^ 1), abort_flag, 41)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[st], KV_BYTES);
          tma_load_2d(kv, &tmK, &k_full[st], it.k_col, it.k_row + j * KC);
          if (!mbar_wait(&v_empty[st], (uint32_t)(((g >> 1) & 1) ^ 1), abort_flag, 41)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[st], KV_BYTES);
          tma_load_2d(kv + KV_BYTES, &tmV, &v_full[st], it.v_col, it.v_row + j * KC);
          ++kv_loads[st];
        }
      }
      // every issued copy has landed before the CTA can exit
      if (nq > 0) mbar_wait(q_full, (uint32_t)((nq - 1) & 1), nullptr, 42);
      for (int st = 0; st < STAGES; ++st)
        if (kv_loads[st] > 0) {
          mbar_wait(&k_full[st], (uint32_t)((kv_loads[st] - 1) & 1), nullptr, 43);
          mbar_wait(&v_full[st], (uint32_t)((kv_loads[st] - 1) & 1), nullptr, 43);
        }
    }
  } else if (warp == 9) {
    // ── MMA issuer ──
    if (lane == 0) {
      int g = 0, nq = 0;
      // the P V product still to issue: global chunk index, chunk within its
      // item, and the item's index among this CTA's non-empty items
      int pv_g = -1, pv_j = 0, pv_item = 0;
      bool ok = true;
      auto issue_pv = [&]() -> bool {
        const int st = pv_g & 1;
        if (!mbar_wait(&v_full[st], (uint32_t)((pv_g >> 1) & 1), abort_flag, 45)) return false;
        // the item's first products overwrite O_0, O_1: the previous item's are read
        if (pv_j == 0 && pv_item > 0 &&
            !mbar_wait(o_free, (uint32_t)((pv_item - 1) & 1), abort_flag, 46))
          return false;
        const uint32_t pa = smem_u32(sP), va = smem_u32(sKV + st * 2 * KV_BYTES + KV_BYTES);
        for (int h = 0; h < 2; ++h) {  // each half's product once its P atom is in
          if (!mbar_wait(&p_full[h], (uint32_t)(pv_g & 1), abort_flag, 44)) return false;
          tc_fence_after();
#pragma unroll
          for (int k = 4 * h; k < 4 * h + 4; ++k) {
            const uint64_t adesc = sw128_desc(pa + h * (QT * 128) + (k & 3) * 32, 16, 1024);
            const uint64_t bdesc = sw128_desc(va + k * 16 * 128, 8192, 1024);
            tc_mma_ss(tmem_o + 64 * h, adesc, bdesc, IDESC_O, (pv_j > 0 || k > 4 * h) ? 1u : 0u);
          }
          tc_commit(&o_full[h]);
        }
        tc_commit(&v_empty[st]);
        return true;
      };
      for (int w = blockIdx.x; w < p.num_items && ok; w += gridDim.x) {
        const Item it = make_item(p, w);
        if (it.nch == 0) continue;
        if (!mbar_wait(q_full, (uint32_t)(nq & 1), abort_flag, 47)) break;
        for (int j = 0; j < it.nch; ++j, ++g) {
          const int st = g & 1;
          if (!mbar_wait(&k_full[st], (uint32_t)((g >> 1) & 1), abort_flag, 48) ||
              (g > 0 && !mbar_wait(s_free, (uint32_t)((g - 1) & 1), abort_flag, 49))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t qa = smem_u32(sQ), ka = smem_u32(sKV + st * 2 * KV_BYTES);
#pragma unroll
          for (int k = 0; k < DH / 16; ++k)
            tc_mma_ss(tmem_s, sw128_desc(qa + k * 32, 16, 1024),
                      sw128_desc(ka + k * 32, 16, 1024), IDESC_S, k != 0);
          tc_commit(s_full);
          tc_commit(&k_empty[st]);
          if (j == it.nch - 1) tc_commit(q_empty);
          if (pv_g >= 0 && !issue_pv()) {
            ok = false;
            break;
          }
          pv_g = g;
          pv_j = j;
          pv_item = nq;
        }
        ++nq;
      }
      if (ok && pv_g >= 0) issue_pv();
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 50);
    }
  } else {
    // ── softmax: two warps per query row, each one key half of every chunk ──
    // An item's output is written after the next item's first chunk has been
    // exponentiated, so the last P V products of the item complete under that
    // softmax instead of stalling the warps.
    const int quarter = warp & 3;  // TMEM lane quarter
    const int kh = warp >> 2;      // key half
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tmem_oh = tmem_o + lane_off + 64 * kh;
    int g = 0, nout = 0;
    bool ok = true;
    bool pend = false;  // an item whose output has not been written yet
    float pend_m = 0.f, pend_l = 0.f;
    __nv_bfloat16* pend_dst = nullptr;
    // Runs after o_full[kh] of the item's last chunk. Half 1 normalises O_1
    // in TMEM and publishes c_1; half 0 waits for that and writes the row.
    auto epilogue = [&]() -> bool {
      __syncwarp();
      tc_fence_after();
      const float inv = (pend_l > 0.f) ? 1.f / pend_l : 0.f;
      const float c = (pend_l > 0.f) ? pend_m + lg2(pend_l) : -INFINITY;
      if (kh == 1) {  // the whole row in one TMEM round trip
        float ov[DH];
        tmem_ld32(tmem_oh, ov);
        tmem_ld32(tmem_oh + 32, ov + 32);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < DH; ++i) ov[i] *= inv;
#pragma unroll
        for (int q = 0; q < DH / 16; ++q) tmem_st16(tmem_oh + q * 16, ov + 16 * q);
        tc_wait_st();
        xlse[row] = c;
        tc_fence_before();
        mbar_arrive(&x_ready[quarter]);
      } else {
        if (!mbar_wait(&x_ready[quarter], (uint32_t)(nout & 1), abort_flag, 54)) return false;
        tc_fence_after();
        const float c1 = xlse[row];
        const float mx = fmaxf(c, c1);  // c (half 0) is finite: the item has keys
        const float e0 = ex2(c - mx), e1 = ex2(c1 - mx);
        const float rt = 1.f / (e0 + e1);
        const float f0 = e0 * rt * inv, f1 = e1 * rt;
#pragma unroll
        for (int q = 0; q < DH / 32; ++q) {  // 32 columns of O_0 and O_1 per round trip
          float o0[32], o1[32];
          tmem_ld32(tmem_oh + q * 32, o0);
          tmem_ld32(tmem_oh + 64 + q * 32, o1);
          tc_wait_ld();
          if (q + 1 == DH / 32) {  // all of O read: the next item's products may start
            tc_fence_before();
            mbar_arrive(o_free);
          }
          if (pend_dst != nullptr) {
#pragma unroll
            for (int i = 0; i < 32; ++i) o0[i] = fmaf(o0[i], f0, o1[i] * f1);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              reinterpret_cast<uint4*>(pend_dst)[4 * q + c] = pack8(o0 + 8 * c);
          }
        }
      }
      if (kh == 1) mbar_arrive(o_free);  // O_0, O_1 may be overwritten by the next item
      ++nout;
      pend = false;
      return true;
    };
    for (int w = blockIdx.x; w < p.num_items && ok; w += gridDim.x) {
      const Item it = make_item(p, w);
      const int l = it.l0 + row;
      __nv_bfloat16* dst = p.o +
                           ((int64_t)it.b * p.o_rows_per_b + (int64_t)it.h * p.o_rows_per_h + l) *
                               p.o_ld +
                           (int64_t)it.h * p.o_col_per_h;
      if (it.nch == 0) {  // no keys: attention over nothing is 0
        if (l < p.Lq)
#pragma unroll
          for (int c = 0; c < DH / 16; ++c)
            reinterpret_cast<uint4*>(dst + kh * (DH / 2))[c] = make_uint4(0, 0, 0, 0);
        continue;
      }
      float m_run = 0.f, l_run = 0.f;
      bool have = false;  // a valid key of this half seen in this item
      for (int j = 0; j < it.nch; ++j, ++g) {
        if (!mbar_wait(s_full, (uint32_t)(g & 1), abort_flag, 51)) {
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after();
        float s[KH];
#pragma unroll
        for (int q = 0; q < KH / 32; ++q)
          tmem_ld32(tmem_s + lane_off + kh * KH + q * 32, s + 32 * q);
        tc_wait_ld();
        tc_fence_before();
        mbar_arrive(s_free);  // S may be overwritten by the next product
        const int lim = it.nk - j * KC - kh * KH;  // valid keys in this half
        if (lim < KH) {
#pragma unroll
          for (int c = 0; c < KH; ++c)
            if (c >= lim) s[c] = -INFINITY;
        }
        float u[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) u[c] = s[c];
#pragma unroll
        for (int c = 8; c < KH; ++c) u[c & 7] = fmaxf(u[c & 7], s[c]);
        const float cmax = fmaxf(fmaxf(fmaxf(u[0], u[1]), fmaxf(u[2], u[3])),
                                 fmaxf(fmaxf(u[4], u[5]), fmaxf(u[6], u[7]))) *
                           p.scale_log2;  // scale > 0: max commutes with it
        float alpha = 1.f;
        bool rescale = false;
        if (!have) {
          // O_h and l hold zeros so far (every earlier P of this half was 0):
          // the base can start here without a rescale
          if (cmax > -INFINITY) {
            m_run = cmax;
            have = true;
          } else {
            m_run = 0.f;  // no key in this half yet: P = 0
          }
        } else if (cmax > m_run + kRescaleLog2) {
          alpha = ex2(m_run - cmax);
          m_run = cmax;
          rescale = true;
        }
        // P_h V_h of the previous chunk is done: atom h of P is free and O_h holds it
        if (g > 0 && !mbar_wait(&o_full[kh], (uint32_t)((g - 1) & 1), abort_flag, 52)) {
          ok = false;
          break;
        }
        // exp2 straight into atom h of P (bf16, 128B swizzle), and the row sum
        uint8_t* patom = sP + kh * (QT * 128);
        float t[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) t[c] = 0.f;
#pragma unroll
        for (int gq = 0; gq < KH / 8; ++gq) {
          float e[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            e[i] = ex2(fmaf(s[8 * gq + i], p.scale_log2, -m_run));
            t[i] += e[i];
          }
          sts128(smem_u32(patom + sw128_off(row, gq)),
                 make_uint4(cvt_bf16x2(e[0], e[1]), cvt_bf16x2(e[2], e[3]),
                            cvt_bf16x2(e[4], e[5]), cvt_bf16x2(e[6], e[7])));
        }
        l_run = l_run * alpha + (((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7])));
        if (__any_sync(0xffffffffu, rescale)) {  // rare: bring O_h to the new base
          __syncwarp();
          tc_fence_after();
#pragma unroll
          for (int q = 0; q < DH / 16; ++q) {
            float ov[16];
            tmem_ld16(tmem_oh + q * 16, ov);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) ov[i] *= alpha;
            tmem_st16(tmem_oh + q * 16, ov);
          }
          tc_wait_st();
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&p_full[kh]);
        // the previous item, whose last products completed before this chunk's
        // P V could start (that product waits for o_free from here)
        if (pend && !epilogue()) {
          ok = false;
          break;
        }
      }
      if (!ok) break;
      pend = true;
      pend_m = m_run;
      pend_l = l_run;
      pend_dst = (l < p.Lq) ? dst : nullptr;
    }
    // the last item's output, once its last products are done
    if (ok && pend && mbar_wait(&o_full[kh], (uint32_t)((g - 1) & 1), abort_flag, 53))
      epilogue();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace

bool attention_ws_supported(const ck_attention_args& a) {
  return a.block_mask == nullptr && a.key_mask == nullptr && attention_tc_supported(a);
}

int attention_ws(const ck_attention_args& a, cudaStream_t st) {
  WsArgs p;
  p.B = a.B;
  p.H = a.H;
  p.Lq = a.Lq;
  p.n_keys = a.n_keys;
  p.num_q_tiles = (a.Lq + QT - 1) / QT;
  const int64_t items = (int64_t)p.num_q_tiles * a.H * a.B;
  if (items <= 0) return CK_OK;
  if (items > INT32_MAX) return CK_ERR_INVALID_ARG;
  p.num_items = (int)items;
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
  p.scale_log2 = a.scale * 1.4426950408889634f;

  CUtensorMap tq, tk, tv;
  if (!make_tmap_2d(&tq, a.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.q_ld, a.q_rows, a.q_ld, 64,
                    QT, 128) ||
      !make_tmap_2d(&tk, a.k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.k_ld, a.k_rows, a.k_ld, 64,
                    KC, 128) ||
      !make_tmap_2d(&tv, a.v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.v_ld, a.v_rows, a.v_ld, 64,
                    KC, 128))
    return CK_ERR_INVALID_ARG;
  if (!smem_attr_ready(reinterpret_cast<const void*>(attn_ws_kernel), SMEM_BYTES))
    return record_cuda_error();
  int64_t grid = CTAS_PER_SM * (int64_t)num_sms();
  if (grid > items) grid = items;
  return launch_pdl(attn_ws_kernel, dim3((unsigned)grid), dim3(NTHREADS), SMEM_BYTES, st, tq, tk,
                    tv, p);
}

}  // namespace ck
