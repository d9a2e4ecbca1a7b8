// Behaviour head in algebraic form (BehaviorDecoder.forward,
// cortex/models/cortex.py:29-53), bf16 models.
//
// The reference computes, per sample b with x = head_norm(final_norm(latents_b)):
//   q = q_proj(query)            (nq, D), batch-invariant
//   K | V = kv_proj(x)           (L, 2D)
//   o_h = softmax(q_h K_h^T / sqrt(Dh)) V_h     per head h
//   y[j] = out_proj(concat_h o_h[j])            (nq,)
// Because K_h = x W_k,h^T and V_h = x W_v,h^T, the same result is
//   s_{h,j}(l) = x_l . qt_{h,j}          qt_{h,j} = W_k,h^T q_h[j] / sqrt(Dh)
//   c_h(l)     = x_l . vt_h              vt_h     = W_v,h^T w_out,h
//   y[j]       = sum_h  sum_l softmax_l(s_{h,j}) c_h(l)
// so the (B*L, D) x (D, 2D) kv_proj GEMM collapses into a (B*L, D) x (D, 2*H*nq)
// product against a matrix that depends only on the weights.
//
//   head_prep_kernel  builds that matrix, Qall (NT, D) bf16, per forward: rows
//                     [0, PH) hold qt_{h,j} (pair p = h*nq + j, pre-multiplied
//                     by log2(e) so the softmax runs on exp2), rows [PH, 2PH)
//                     hold vt_{h(p)} for the same pairs, and rows [NC, 2NC) hold
//                     the bf16 remainders (value - bf16(value)) of rows [0, NC),
//                     so hi + lo carries the fp32 weights into the bf16 MMA.
//   head_kernel       one CTA per R-latent tile (R = 64 while ceil(L/64) <= 8,
//                     else 128), a cluster of ceil(L/R) CTAs per sample; the MMA
//                     runs M = 128 with zero rows. Each CTA applies the two LayerNorms to its rows
//                     exactly as row_norm2 does (bf16 rounding after each), writes
//                     them as the 128B-swizzled MMA A operand, multiplies by Qall
//                     with tcgen05 into TMEM, then reduces the tile to per-pair
//                     (max, sum exp2, sum exp2 * c). The cluster's rank 0 merges
//                     the tiles over distributed shared memory and writes y.
#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

// 16 warps: the two LayerNorms run a row per warp with warp-wide reductions,
// so more warps shorten that latency chain (4 rows per warp at 64 rows per
// CTA; measured 2.5 us per forward against 8 warps)
constexpr int HEAD_THREADS = 512;
constexpr int TILE_L = 128;
constexpr int HEAD_SMEM_LIMIT = 232448;
constexpr int MISC_BYTES = 1024;  // barriers, TMEM slot, cluster partials
constexpr float kLog2e = 1.4426950408889634f;

struct HeadPrepArgs {
  const __nv_bfloat16* query;  // (nq, D)
  const __nv_bfloat16* wq;     // head q_proj (D, D)
  const __nv_bfloat16* wkv;    // head kv_proj (2D, D)
  const __nv_bfloat16* wout;   // head out_proj (1, D)
  int D, H, Dh, nq, PH, NC;
  float qscale;  // softmax scale * log2(e)
  __nv_bfloat16* qall;  // (2 * NC, D)
};

// grid (ceil(D / 256), NC): blockIdx.y is the Qall row n in [0, NC); thread k
// writes row n's hi value at column k and its lo value in row NC + n.
template <int MAXV>
__global__ void __launch_bounds__(256) head_prep_kernel(const HeadPrepArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ float qh[128];
  const int n = blockIdx.y;
  const int k = blockIdx.x * 256 + threadIdx.x;
  const int HQ = a.H * a.nq;
  const int pr = n < a.PH ? n : n - a.PH;  // pair index of this row
  float val = 0.f;
  if (pr < HQ) {
    const int h = pr / a.nq, j = pr % a.nq;
    const int64_t D = a.D;
    if (n < a.PH) {
      // q[j, h*Dh + d] = bf16(W_q[h*Dh + d, :] . query[j, :])   (F.linear output rounding)
      const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
      float qf[MAXV][8];
#pragma unroll
      for (int i = 0; i < MAXV; ++i)
        unpack8(reinterpret_cast<const uint4*>(a.query + j * D)[lane + 32 * i], qf[i]);
      for (int d0 = warp; d0 < a.Dh; d0 += 32) {
        float s[4];
        uint4 w[4][MAXV];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int i = 0; i < MAXV; ++i) {
            const int d = min(d0 + 8 * u, a.Dh - 1);
            w[u][i] = reinterpret_cast<const uint4*>(a.wq + ((int64_t)h * a.Dh + d) * D)[lane + 32 * i];
          }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          s[u] = 0.f;
#pragma unroll
          for (int i = 0; i < MAXV; ++i) {
            float wf[8];
            unpack8(w[u][i], wf);
#pragma unroll
            for (int e = 0; e < 8; ++e) s[u] = fmaf(wf[e], qf[i][e], s[u]);
          }
          s[u] = warp_sum(s[u]);
          if (lane == 0 && d0 + 8 * u < a.Dh) qh[d0 + 8 * u] = rbf(s[u]);
        }
      }
      __syncthreads();
      if (k < a.D) {
        float acc = 0.f;
        const __nv_bfloat16* wk = a.wkv + (int64_t)h * a.Dh * D + k;
#pragma unroll 16
        for (int d = 0; d < a.Dh; ++d) acc = fmaf(qh[d], bf2f(wk[d * D]), acc);
        val = acc * a.qscale;
      }
    } else if (k < a.D) {
      float acc = 0.f;
      const __nv_bfloat16* wv = a.wkv + (D + (int64_t)h * a.Dh) * D + k;
      const __nv_bfloat16* wo = a.wout + (int64_t)h * a.Dh;
#pragma unroll 16
      for (int d = 0; d < a.Dh; ++d) acc = fmaf(bf2f(wo[d]), bf2f(wv[d * D]), acc);
      val = acc;
    }
  }
  if (k < a.D) {
    const __nv_bfloat16 hi = f2bf(val);
    a.qall[(int64_t)n * a.D + k] = hi;
    a.qall[(int64_t)(a.NC + n) * a.D + k] = f2bf(val - bf2f(hi));
  }
}

struct HeadArgs {
  const __nv_bfloat16 *g1, *b1, *g2, *b2;
  float eps;
  int L, R, H, nq, n_stages, C;  // R: latent rows per CTA (64 or 128)
  void* out;  // (B, nq), bf16
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_index() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ float ld_peer_f32(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void merge3(float& m, float& s, float& w, float m2, float s2, float w2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  const float a = ex2(m - mn), b = ex2(m2 - mn);
  s = s * a + s2 * b;
  w = w * a + w2 * b;
  m = mn;
}

// LayerNorms of NR rows held as MAXV 8-wide vectors per lane, one warp (per
// row the arithmetic of row_norm_kernel's layer_norm_regs followed by the
// gamma/beta step), the rows' reductions interleaved so that one row's
// shuffle latency covers the others'.
template <int MAXV, int NR>
__device__ __forceinline__ void ln_lane_rows(float (&v)[NR][MAXV][8], const uint4 (&g)[MAXV],
                                             const uint4 (&bt)[MAXV], bool has_b, int D,
                                             float eps) {
  float s[NR], mean[NR], q[NR], rstd[NR];
#pragma unroll
  for (int j = 0; j < NR; ++j) {
    s[j] = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
#pragma unroll
      for (int k = 0; k < 8; ++k) s[j] += v[j][i][k];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int j = 0; j < NR; ++j) s[j] += __shfl_xor_sync(0xffffffffu, s[j], o);
#pragma unroll
  for (int j = 0; j < NR; ++j) {
    mean[j] = s[j] / (float)D;
    q[j] = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float d = v[j][i][k] - mean[j];
        q[j] += d * d;
      }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int j = 0; j < NR; ++j) q[j] += __shfl_xor_sync(0xffffffffu, q[j], o);
#pragma unroll
  for (int j = 0; j < NR; ++j) rstd[j] = 1.0f / sqrtf(q[j] / (float)D + eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    float gf[8], bf[8];
    unpack8(g[i], gf);
    unpack8(bt[i], bf);
#pragma unroll
    for (int j = 0; j < NR; ++j)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        v[j][i][k] = (v[j][i][k] - mean[j]) * rstd[j];
        v[j][i][k] = v[j][i][k] * gf[k] + (has_b ? bf[k] : 0.f);
      }
  }
}

// MAXV = D / 256 (16-byte vectors per lane); PH = score/value pairs per half
// (16 or 32): NC = 2 * PH Qall rows, NT = 2 * NC MMA columns.
template <int MAXV, int PH>
__global__ void __launch_bounds__(HEAD_THREADS, 1)
    head_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmB,
                const HeadArgs p) {
  constexpr int NC = 2 * PH;
  constexpr int NT = 2 * NC;
  constexpr int D = MAXV * 256;
  constexpr int NKB = D / 64;
  constexpr int A_KB_BYTES = TILE_L * 128;
  constexpr int B_STAGE_BYTES = NT * 128;
  constexpr uint32_t TMEM_COLS = NT < 32 ? 32 : NT;
  constexpr uint32_t IDESC = idesc_bf16(TILE_L, NT, 0);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + NKB * A_KB_BYTES;
  uint8_t* misc = sB + p.n_stages * B_STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(misc);  // [n_stages <= 12]
  uint64_t* empty = full + 12;
  uint64_t* done = empty + 12;
  uint64_t* xfull = done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* mma_ok = reinterpret_cast<int*>(tmem_slot + 2);  // the MMAs completed
  float* part = reinterpret_cast<float*>(misc + 256);  // [PH][3] this CTA's partials
  float* ofin = part + PH * 3;                         // [PH]
  // [4 lane quarters][PH][3] partials; the A tile is dead once the MMAs are done
  float* red = reinterpret_cast<float*>(sA);

  const int tid = threadIdx.x;
  const int warp = tid / 32, lane = tid % 32;
  const int S = p.n_stages;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_init(xfull, 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmX);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dep_wait();
  grid_dep_launch();

  const int rank = (int)cluster_rank();
  const int64_t b = (int64_t)cluster_index();
  const int l0 = rank * p.R;
  const int rows = min(p.R, p.L - l0);

  // Raw latent rows land in the A tile (128B-swizzled K-blocks, the MMA
  // layout), then the first S K-blocks of Qall; both under one thread.
  if (tid == 0) {
    mbar_arrive_expect_tx(xfull, (uint32_t)(NKB * p.R * 128));
    for (int kb = 0; kb < NKB; ++kb)
      tma_load_2d(sA + kb * A_KB_BYTES, &tmX, xfull, kb * 64, (int)(b * p.L + l0));
    for (int kb = 0; kb < S && kb < NKB; ++kb) {
      mbar_arrive_expect_tx(&full[kb], B_STAGE_BYTES);
      tma_load_2d(sB + kb * B_STAGE_BYTES, &tmB, &full[kb], kb * 64, 0);
    }
  }
  const uint4 z = make_uint4(0, 0, 0, 0);
  if (p.R < TILE_L) {  // MMA rows the CTA does not own are zero
    for (int i = tid; i < NKB * (TILE_L - p.R) * 8; i += HEAD_THREADS) {
      const int kb = i / ((TILE_L - p.R) * 8), rem = i % ((TILE_L - p.R) * 8);
      *reinterpret_cast<uint4*>(sA + kb * A_KB_BYTES + (p.R + rem / 8) * 128 + (rem % 8) * 16) = z;
    }
  }

  // A operand: both LayerNorms per latent row, in place in the swizzled tile.
  {
    uint4 g1[MAXV], b1[MAXV], g2[MAXV], b2[MAXV];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = lane + 32 * i;
      g1[i] = reinterpret_cast<const uint4*>(p.g1)[c];
      g2[i] = reinterpret_cast<const uint4*>(p.g2)[c];
      b1[i] = p.b1 ? reinterpret_cast<const uint4*>(p.b1)[c] : z;
      b2[i] = p.b2 ? reinterpret_cast<const uint4*>(p.b2)[c] : z;
    }
    const bool landed = mbar_wait(xfull, 0, abort_flag, 20);
    // rows r0 + j * NW, j < NRP, per pass (R is 64 or 128, so all are below
    // R; D = 768 keeps one row per pass inside the register budget); a row
    // past the sample's end is normalised as zeros and stored as zeros
    constexpr int NW = HEAD_THREADS / 32;
    constexpr int NRP = MAXV <= 2 ? 2 : 1;
    for (int r0 = warp; r0 < p.R; r0 += NRP * NW) {
      uint4* slot[NRP][MAXV];
      bool live[NRP];
      float v[NRP][MAXV][8];
#pragma unroll
      for (int j = 0; j < NRP; ++j) {
        const int r = r0 + j * NW;
        live[j] = landed && r < rows;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
          const int c = lane + 32 * i;  // 16-byte chunk of the row
          slot[j][i] = reinterpret_cast<uint4*>(sA + (c >> 3) * A_KB_BYTES + sw128_off(r, c & 7));
          if (live[j]) {
            unpack8(*slot[j][i], v[j][i]);
          } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) v[j][i][k] = 0.f;
          }
        }
      }
      ln_lane_rows<MAXV, NRP>(v, g1, b1, p.b1 != nullptr, D, p.eps);
#pragma unroll
      for (int j = 0; j < NRP; ++j)
#pragma unroll
        for (int i = 0; i < MAXV; ++i)
#pragma unroll
          for (int k = 0; k < 8; ++k) v[j][i][k] = rbf(v[j][i][k]);
      ln_lane_rows<MAXV, NRP>(v, g2, b2, p.b2 != nullptr, D, p.eps);
#pragma unroll
      for (int j = 0; j < NRP; ++j)
#pragma unroll
        for (int i = 0; i < MAXV; ++i) *slot[j][i] = live[j] ? pack8(v[j][i]) : z;
    }
  }
  fence_proxy_async_smem();
  __syncthreads();

  // MMA: (128 x D) x (D x NT) -> TMEM, refilling the B ring when it is short.
  // Issued from warp 4, so no lane of the epilogue warps 0-3 spins beside it.
  if (tid == 128) {
    const uint32_t a_addr = smem_u32(sA);
    const uint32_t b_addr = smem_u32(sB);
    int issued = S < NKB ? S : NKB;
    bool ok = true;
    for (int kb = 0; kb < NKB && ok; ++kb) {
      const int s = kb % S;
      const uint32_t ph = (uint32_t)((kb / S) & 1);
      if (!mbar_wait(&full[s], ph, abort_flag, 21)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < 4; ++k)
        tc_mma_ss(tmem_base, sw128_desc(a_addr + kb * A_KB_BYTES + k * 32, 16, 1024),
                  sw128_desc(b_addr + s * B_STAGE_BYTES + k * 32, 16, 1024), IDESC,
                  (kb | k) != 0 ? 1u : 0u);
      tc_commit(&empty[s]);
      if (kb + S < NKB) {
        if (!mbar_wait(&empty[s], ph, abort_flag, 22)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], B_STAGE_BYTES);
        tma_load_2d(sB + s * B_STAGE_BYTES, &tmB, &full[s], (kb + S) * 64, 0);
        ++issued;
      }
    }
    tc_commit(done);
    if (!ok) {
      // Let the last copy issued into each stage land before the CTA can exit.
      mbar_wait(xfull, 0, nullptr, 25);
      for (int s = 0; s < S && s < issued; ++s) {
        const int last = issued - 1 - ((issued - 1 - s) % S);
        mbar_wait(&full[s], (uint32_t)((last / S) & 1), nullptr, 23);
      }
    }
  }

  // Epilogue (one latent row per thread): per-pair tile partials. The four
  // warps of a TMEM lane quarter (warp % 4) share its rows and take every
  // fourth pair each.
  // Only the MMA thread waits on `done`; the other warps wait at the barrier
  // instead of polling the mbarrier beside the MMAs' shared-memory reads.
  if (tid == 128) *mma_ok = mbar_wait(done, 0, abort_flag, 24) ? 1 : 0;
  __syncthreads();
  {
    const int quarter = warp & 3, slice = warp >> 2;
    const bool got = *mma_ok != 0;
    tc_fence_after();
    const int r = quarter * 32 + lane;
    const bool valid = got && r < rows;
    const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    float val[NC];
#pragma unroll
    for (int c0 = 0; c0 < NC; c0 += 32) {
      float hi[32], lo[32];
      tmem_ld32(taddr + c0, hi);
      tmem_ld32(taddr + NC + c0, lo);
      tc_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) val[c0 + i] = hi[i] + lo[i];
    }
    const int HQ = p.H * p.nq;
    static_assert(HEAD_THREADS / 32 == 16, "four warps per TMEM lane quarter");
#pragma unroll
    for (int q = 0; q < PH; ++q) {
      if (q < HQ && (q & 3) == slice) {
        const float s = valid ? val[q] : -INFINITY;
        const float m = warp_max(s);
        const float e = valid ? ex2(s - m) : 0.f;
        const float se = warp_sum(e);
        const float we = warp_sum(e * val[PH + q]);
        if (lane == 0) {
          red[(quarter * PH + q) * 3 + 0] = m;
          red[(quarter * PH + q) * 3 + 1] = se;
          red[(quarter * PH + q) * 3 + 2] = we;
        }
      }
    }
  }
  __syncthreads();
  const int HQ = p.H * p.nq;
  if (tid < HQ) {
    float m = -INFINITY, s = 0.f, w = 0.f;
    for (int wi = 0; wi < 4; ++wi)
      merge3(m, s, w, red[(wi * PH + tid) * 3 + 0], red[(wi * PH + tid) * 3 + 1],
             red[(wi * PH + tid) * 3 + 2]);
    part[tid * 3 + 0] = m;
    part[tid * 3 + 1] = s;
    part[tid * 3 + 2] = w;
  }
  cluster_sync_all();
  if (rank == 0) {
    if (tid < HQ) {
      float m = -INFINITY, s = 0.f, w = 0.f;
      for (int rr = 0; rr < p.C; ++rr)
        merge3(m, s, w, ld_peer_f32(&part[tid * 3 + 0], rr), ld_peer_f32(&part[tid * 3 + 1], rr),
               ld_peer_f32(&part[tid * 3 + 2], rr));
      ofin[tid] = s > 0.f ? w / s : 0.f;
    }
    __syncthreads();
    if (tid < p.nq) {
      float y = 0.f;
      for (int h = 0; h < p.H; ++h) y += ofin[h * p.nq + tid];
      reinterpret_cast<__nv_bfloat16*>(p.out)[b * p.nq + tid] = f2bf(y);
    }
  }
  cluster_sync_all();  // peers keep their partials alive until rank 0 has read them
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

struct HeadGeom {
  int D, L, H, Dh, nq, HQ, PH, NC, NT, R, C, maxv, stages, smem;
};

bool head_geom(const ck_model* m, HeadGeom* g) {
  g->D = m->latent_dim;
  g->L = m->num_latents;
  g->H = m->num_heads;
  g->Dh = m->head_dim;
  g->nq = m->behavior_dim;
  g->HQ = g->H * g->nq;
  if (m->dtype != CK_BF16) return false;
  if (g->D % 256 != 0 || g->D / 256 > 3) return false;
  if (g->Dh > 128 || g->HQ > 32 || g->HQ <= 0) return false;
  if (g->L <= 0 || g->L > 8 * TILE_L) return false;
  g->PH = g->HQ <= 16 ? 16 : 32;
  g->NC = 2 * g->PH;
  g->NT = 2 * g->NC;
  // 64 latent rows per CTA while a cluster of <= 8 covers the sample (twice the
  // CTAs for the norms; the MMA still runs M = 128 with zero rows), else 128.
  g->R = (g->L + 63) / 64 <= 8 ? 64 : TILE_L;
  g->C = (g->L + g->R - 1) / g->R;
  g->maxv = g->D / 256;
  const int nkb = g->D / 64;
  const int fixed = 1024 + nkb * TILE_L * 128 + MISC_BYTES;
  int stages = (HEAD_SMEM_LIMIT - fixed) / (g->NT * 128);
  if (stages > nkb) stages = nkb;
  if (stages > 12) stages = 12;
  if (stages < 1) return false;
  g->stages = stages;
  g->smem = fixed + stages * g->NT * 128;
  auto lin_ok = [](const ck_linear_weight& w) {
    return w.w != nullptr && w.bias == nullptr && w.dtype == CK_BF16;
  };
  if (!lin_ok(m->head_q) || !lin_ok(m->head_kv) || !lin_ok(m->head_out)) return false;
  if (m->head_query == nullptr || m->final_norm_w == nullptr || m->head_norm_w == nullptr)
    return false;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (!al16(m->final_norm_w) || !al16(m->head_norm_w) || !al16(m->head_query) ||
      !al16(m->head_q.w) || (m->final_norm_b && !al16(m->final_norm_b)) ||
      (m->head_norm_b && !al16(m->head_norm_b)))
    return false;
  return true;
}

template <int MAXV, int PH>
int launch_head(const CUtensorMap& tx, const CUtensorMap& tb, const HeadArgs& a, int B, int smem,
                cudaStream_t st) {
  auto kern = head_kernel<MAXV, PH>;
  if (!smem_attr_ready(reinterpret_cast<const void*>(kern), smem)) return record_cuda_error();
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)a.C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(B * a.C));
  cfg.blockDim = dim3(HEAD_THREADS);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return launch_cfg(cfg, kern, tx, tb, a);
}

}  // namespace

size_t head_qall_bytes(const ck_model* m) {
  HeadGeom g;
  if (!head_geom(m, &g)) return 0;
  return (size_t)g.NT * g.D * 2;
}

bool head_fused_supported(const ck_model* m) {
  HeadGeom g;
  return head_geom(m, &g);
}

int head_prep(const ck_model* m, void* qall, cudaStream_t st) {
  HeadGeom g;
  if (!head_geom(m, &g) || qall == nullptr) return CK_ERR_UNSUPPORTED;
  HeadPrepArgs a;
  a.query = reinterpret_cast<const __nv_bfloat16*>(m->head_query);
  a.wq = reinterpret_cast<const __nv_bfloat16*>(m->head_q.w);
  a.wkv = reinterpret_cast<const __nv_bfloat16*>(m->head_kv.w);
  a.wout = reinterpret_cast<const __nv_bfloat16*>(m->head_out.w);
  a.D = g.D;
  a.H = g.H;
  a.Dh = g.Dh;
  a.nq = g.nq;
  a.PH = g.PH;
  a.NC = g.NC;
  a.qscale = kLog2e / sqrtf((float)g.Dh);
  a.qall = reinterpret_cast<__nv_bfloat16*>(qall);
  const dim3 grid((unsigned)((g.D + 255) / 256), (unsigned)g.NC);
  if (g.maxv == 1) return launch_pdl(head_prep_kernel<1>, grid, dim3(256), 0, st, a);
  if (g.maxv == 2) return launch_pdl(head_prep_kernel<2>, grid, dim3(256), 0, st, a);
  return launch_pdl(head_prep_kernel<3>, grid, dim3(256), 0, st, a);
}

int head_fused(const ck_model* m, const void* lat, int32_t B, const void* qall, void* out,
               cudaStream_t st) {
  HeadGeom g;
  if (!head_geom(m, &g)) return CK_ERR_UNSUPPORTED;
  if (B <= 0) return CK_OK;
  if ((reinterpret_cast<uintptr_t>(lat) & 15u) != 0) return CK_ERR_INVALID_ARG;
  CUtensorMap tx, tb;
  if (!make_tmap_2d(&tx, lat, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.D, (uint64_t)B * g.L, g.D,
                    64, g.R, 128) ||
      !make_tmap_2d(&tb, qall, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.D, g.NT, g.D, 64, g.NT, 128))
    return CK_ERR_INVALID_ARG;
  HeadArgs a;
  a.g1 = reinterpret_cast<const __nv_bfloat16*>(m->final_norm_w);
  a.b1 = reinterpret_cast<const __nv_bfloat16*>(m->final_norm_b);
  a.g2 = reinterpret_cast<const __nv_bfloat16*>(m->head_norm_w);
  a.b2 = reinterpret_cast<const __nv_bfloat16*>(m->head_norm_b);
  a.eps = 1e-5f;
  a.L = g.L;
  a.R = g.R;
  a.H = g.H;
  a.nq = g.nq;
  a.n_stages = g.stages;
  a.C = g.C;
  a.out = out;
  if (g.maxv == 1)
    return g.PH == 16 ? launch_head<1, 16>(tx, tb, a, B, g.smem, st)
                      : launch_head<1, 32>(tx, tb, a, B, g.smem, st);
  if (g.maxv == 2)
    return g.PH == 16 ? launch_head<2, 16>(tx, tb, a, B, g.smem, st)
                      : launch_head<2, 32>(tx, tb, a, B, g.smem, st);
  return g.PH == 16 ? launch_head<3, 16>(tx, tb, a, B, g.smem, st)
                    : launch_head<3, 32>(tx, tb, a, B, g.smem, st);
}

}  // namespace ck
