// Chained tcgen05 GEMMs: the linears of one decoder block in one launch.
//
// A chain is up to four bf16 linears, each reading the previous one's output
// as its A operand. In the Cortex latent stack (cortex/models/perceiver.py:
// 107-141) the linears after a self-attention are
//   out_proj + residual (+ LayerNorm norm_mlp)    -> lat, x
//   mlp.0 + GELU                                  -> h
//   mlp.2 + residual (+ the next block's norm_attn) -> lat, x
//   the next block's qkv_proj                     -> qkv
// and as separate launches each of them ends in a partly idle wave, a pipeline
// drain and an epilogue that nothing overlaps. Here every linear is cut into
// 128-row x 256-column tiles, and a tile of linear i reads only the 128-row
// block of linear i-1's output that has the same rows. One persistent launch
// of two-CTA clusters walks a single list of cluster jobs, linear by linear
// (a job is two tiles, one per CTA of the cluster; for a LayerNorm linear, the
// two 256-column halves of one row block), with the cluster count as stride.
// Before loading a tile's A, the producer waits until linear i-1 has finished
// the tile's row block: a per-(linear, row block) counter in global memory,
// raised by each epilogue warp once its stores of a tile are complete.
//
// Progress: the launch never has more clusters than the device keeps resident
// at once, and a job only waits on jobs earlier in the list, so the earliest
// unfinished job always has what it needs. Every wait is bounded; a timeout
// records CK_ERR_TIMEOUT, raises a global abort word that the other CTAs'
// waits poll, and every role drains.
//
// Warp roles of a CTA (576 threads, one CTA per SM):
//   warp 0        TMA producer: A and B tiles into a 3-deep shared-memory ring
//   warp 1        TMEM allocator + tcgen05.mma issuer (128 x 256 x 16 bf16)
//   warps 2..17   epilogue: four warps per TMEM lane quarter, 64 columns each,
//                 in two 32-column chunks: bias-free linear output rounded to
//                 bf16 as F.linear returns it, then GELU or residual, TMA store
//                 through a 64B-swizzled 32 x 32 box. LayerNorm linears put
//                 the stored values back into TMEM, exchange per-warp
//                 (mean, M2) partials of the 512-column row with the partner
//                 CTA through distributed shared memory, and store LN(y) too.
// The accumulator is double-buffered in TMEM (2 x 256 columns) so a tile's
// epilogue overlaps the next tile's main loop, across linears as well.
#include <cuda.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int MAX_LINKS = 4;
constexpr int EPI_WARPS = 16;
constexpr int SLICE = BN / 4;      // columns per epilogue warp
constexpr int NCH = SLICE / 32;    // 32-column chunks per warp and tile
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int STG_BOX = 32 * 32 * 2;           // one 32 x 32 bf16 store box
constexpr int EPI_SMEM = EPI_WARPS * 2 * STG_BOX;
constexpr int XCH_SMEM = 2 * 8 * BM * 8;       // [2][8 partials][BM rows] float2
constexpr int BAR_BYTES = 256;
constexpr int RING = (232448 - 1024 - EPI_SMEM - XCH_SMEM - BAR_BYTES) / STAGE_BYTES;
constexpr int SMEM_BYTES = 1024 + RING * STAGE_BYTES + EPI_SMEM + XCH_SMEM + BAR_BYTES;
constexpr int NUM_THREADS = 32 * (2 + EPI_WARPS);
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr uint32_t IDESC = idesc_bf16(BM, BN, 0u);
static_assert(RING >= 3, "chain GEMM: at least three pipeline stages");
static_assert(SMEM_BYTES <= 232448, "chain GEMM smem budget");

struct Link {
  int kind;         // CK_CHAIN_STORE / GELU / RESID / RESID_LN
  int n_tiles;      // N / BN (even)
  int k_blocks;     // ceil(K / BK)
  int job0, jobs;   // this linear's cluster jobs [job0, job0 + jobs)
  int wait_target;  // epilogue-warp completions of the previous linear per row block (0: none)
  int signal;       // a later linear waits on this one's row blocks
  const __nv_bfloat16* aux;  // residual (RESID kinds)
  int64_t ld_aux, aux_row_mod;
  int aux_link, aux_target;  // the earlier linear of this launch that writes aux (-1: none)
  int aux_tma;               // the residual comes in by TMA (maps.r), else by coherent loads
  const __nv_bfloat16* ln_gamma;  // RESID_LN
  const __nv_bfloat16* ln_beta;   // may be NULL
  float eps;
};

struct ChainArgs {
  int M, num_m_tiles, num_links, total_jobs;
  int* done;   // [num_links][num_m_tiles] epilogue-warp completions, zero at launch
  int* abort;  // zero at launch
  Link l[MAX_LINKS];
};

struct ChainMaps {
  CUtensorMap a[MAX_LINKS], b[MAX_LINKS], y[MAX_LINKS], y2[MAX_LINKS], r[MAX_LINKS];
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Order this thread's generic-proxy view of global memory with its
// async-proxy (TMA) accesses, in both directions.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait for *ctr >= target (acquire at GPU scope). Polls the global
// abort word and the CTA's abort flag; on a timeout records CK_ERR_TIMEOUT and
// raises both.
__device__ __forceinline__ bool wait_count(const int* ctr, int target, int* abort_g,
                                           volatile int* abort_flag, int site) {
  const long long t0 = clock64();
  for (uint32_t n = 0;; ++n) {
    if (ld_acquire_gpu(ctr) >= target) return true;
    if ((n & 15u) == 15u) {
      if (*abort_flag) return false;
      if (*reinterpret_cast<volatile int*>(abort_g) != 0) {
        *abort_flag = 1;
        return false;
      }
      if (clock64() - t0 > kWaitCycles) {
        set_status(CK_ERR_TIMEOUT, site, target);
        atomicExch(abort_g, 1);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Cluster job -> (linear, row block, column tile) of this CTA.
__device__ __forceinline__ void decode(const ChainArgs& p, int job, uint32_t crank, int& li,
                                       int& r, int& n) {
  li = 0;
#pragma unroll
  for (int i = 1; i < MAX_LINKS; ++i)
    if (i < p.num_links && job >= p.l[i].job0) li = i;
  const int t = 2 * (job - p.l[li].job0) + (int)crank;
  r = t / p.l[li].n_tiles;
  n = t - r * p.l[li].n_tiles;
}

// 16 packed bf16 pairs into a 64B-swizzled 32 x 32 box (row = lane), then one
// TMA store of the box; the box was last read by the store issued two boxes
// ago by this warp.
__device__ __forceinline__ void store_box(uint8_t* box, const uint32_t* w, const CUtensorMap* map,
                                          int n0, int m0, bool issue, int lane) {
  if (lane == 0) bulk_wait_read<1>();
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4*>(box + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) =
        make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && issue) {
    tma_store_2d(map, box, n0, m0);
    bulk_commit();
  }
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_chain_kernel(const __grid_constant__ ChainMaps maps, const __grid_constant__ ChainArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + RING * A_BYTES;
  uint8_t* sStg = sB + RING * B_BYTES;
  float2* sXch = reinterpret_cast<float2*>(sStg + EPI_SMEM);
  uint8_t* sBar = reinterpret_cast<uint8_t*>(sXch) + XCH_SMEM;
  uint64_t* full = reinterpret_cast<uint64_t*>(sBar);
  uint64_t* empty = full + RING;
  uint64_t* tfull = empty + RING;
  uint64_t* tempty = tfull + 2;
  uint64_t* sready = tempty + 2;  // [2]: a LayerNorm tile's row partials of both CTAs are in
  uint64_t* drain = sready + 2;
  uint64_t* rbar = drain + 1;  // [EPI_WARPS]: a warp's residual boxes have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t crank = cl_rank();
  const int cl_id = (int)(blockIdx.x >> 1);
  const int n_cl = (int)(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < RING; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], EPI_WARPS * 32);
      mbar_init(&sready[a], 2 * EPI_WARPS * 32);  // local and partner arrivals
    }
    mbar_init(drain, 1);
    for (int w = 0; w < EPI_WARPS; ++w) mbar_init(&rbar[w], 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane < p.num_links) {
    prefetch_tmap(&maps.a[lane]);
    prefetch_tmap(&maps.b[lane]);
    prefetch_tmap(&maps.y[lane]);
    if (p.l[lane].kind == CK_CHAIN_RESID_LN) prefetch_tmap(&maps.y2[lane]);
    if (p.l[lane].aux_tma) prefetch_tmap(&maps.r[lane]);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cl_sync();  // the partner's barriers are initialised before any remote arrival
  const uint32_t tmem_base = *tmem_slot;
  grid_dep_wait();
  grid_dep_launch();

  if (warp == 0) {
    // ── TMA producer ──
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int job = cl_id; job < p.total_jobs && !*abort_flag; job += n_cl) {
        int li, r, n;
        decode(p, job, crank, li, r, n);
        const Link& L = p.l[li];
        if (L.wait_target > 0) {
          // the previous linear's row block r is complete; its stores are
          // visible to the TMA loads below
          if (!wait_count(p.done + (int64_t)(li - 1) * p.num_m_tiles + r, L.wait_target, p.abort,
                          abort_flag, 20))
            break;
          fence_proxy_async_global();
        }
        bool ok = true;
        for (int kb = 0; kb < L.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, 21)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &maps.a[li], &full[stage], kb * BK, r * BM);
          tma_load_2d(sB + stage * B_BYTES, &maps.b[li], &full[stage], kb * BK, n * BN);
          ++issued;
          if (++stage == RING) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
      // every issued copy has landed before the CTA can exit
      for (int s = 0; s < RING && s < issued; ++s) {
        const int last = issued - 1 - ((issued - 1 - s) % RING);
        mbar_wait(&full[s], (uint32_t)((last / RING) & 1), nullptr, 22);
      }
    }
  } else if (warp == 1) {
    // ── MMA issuer ──
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int job = cl_id; job < p.total_jobs && ok; job += n_cl) {
        int li, r, n;
        decode(p, job, crank, li, r, n);
        const int k_blocks = p.l[li].k_blocks;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, 23)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, 24)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc_mma_ss(d_tmem, sw128_desc(a_addr + k * 32, 16, 1024),
                      sw128_desc(b_addr + k * 32, 16, 1024), IDESC, (kb | k) != 0 ? 1u : 0u);
          tc_commit(&empty[stage]);
          if (++stage == RING) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 25);
    }
  } else {
    // ── epilogue: (lane quarter, 64-column slice) per warp ──
    const int e = warp - 2;
    const int quarter = warp & 3;  // the TMEM lane quarter this warp may access
    const int slice = e >> 2;
    const int row = quarter * 32 + lane;
    uint8_t* stg = sStg + e * 2 * STG_BOX;
    int acc = 0;
    uint32_t acc_phase = 0;
    int ln_count = 0;  // LayerNorm tiles so far: selects the exchange buffer and phase
    uint32_t rph = 0;  // phase of this warp's residual barrier
    bool res_pending = false;
    // A job's residual (this warp's 32 rows x 64 columns) into the warp's two
    // store boxes by TMA, issued before the job's accumulator is ready. A
    // residual written by an earlier linear of this launch is read only after
    // that linear's row-block count has been acquired.
    auto prefetch_res = [&](int job) -> bool {
      int li, r, n;
      decode(p, job, crank, li, r, n);
      const Link& L = p.l[li];
      if (!L.aux_tma) return true;
      bool ok = true;
      if (lane == 0) {
        if (L.aux_link >= 0) {
          ok = wait_count(p.done + (int64_t)L.aux_link * p.num_m_tiles + r, L.aux_target, p.abort,
                          abort_flag, 28);
          if (ok) fence_proxy_async_global();
        }
        if (ok) {
          bulk_wait_read<0>();  // the boxes' last stores have read them
          const int m0 = r * BM + quarter * 32;
          const int row0 = L.aux_row_mod > 0 ? (int)((int64_t)m0 % L.aux_row_mod) : m0;
          mbar_arrive_expect_tx(&rbar[e], 2 * STG_BOX);
#pragma unroll
          for (int c = 0; c < NCH; ++c)
            tma_load_2d(stg + c * STG_BOX, &maps.r[li], &rbar[e], n * BN + slice * SLICE + c * 32,
                        row0);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      res_pending = ok;
      return ok;
    };
    if (cl_id < p.total_jobs && !prefetch_res(cl_id)) goto epi_done;
    for (int job = cl_id; job < p.total_jobs; job += n_cl) {
      int li, r, n;
      decode(p, job, crank, li, r, n);
      const Link& L = p.l[li];
      const int kind = L.kind;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, 26)) break;
      __syncwarp();
      tc_fence_after();
      const int m = r * BM + row;
      const bool row_ok = m < p.M;
      const int m0 = r * BM + quarter * 32;
      const int nbase = n * BN + slice * SLICE;
      const uint32_t tbase =
          tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN + slice * SLICE);
      if (L.aux_tma) {
        if (!mbar_wait(&rbar[e], rph, abort_flag, 29)) break;
        rph ^= 1;
        res_pending = false;
      } else if (L.aux_link >= 0) {
        // the residual rows were written by an earlier linear of this launch:
        // acquire its row-block count before reading them (coherent loads)
        bool got = true;
        if (lane == 0)
          got = wait_count(p.done + (int64_t)L.aux_link * p.num_m_tiles + r, L.aux_target, p.abort,
                           abort_flag, 28);
        if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) break;
      }
      const bool res_box = L.aux_tma != 0;
      const __nv_bfloat16* rrow =
          (kind >= CK_CHAIN_RESID && !res_box && row_ok)
              ? L.aux + (L.aux_row_mod > 0 ? (int64_t)m % L.aux_row_mod : (int64_t)m) * L.ld_aux
              : nullptr;
      float st_shift = 0.f, st_s1 = 0.f, st_s2 = 0.f;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int n0 = nbase + c * 32;
        uint4 res[4];
        if (res_box) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            res[q] = *reinterpret_cast<const uint4*>(stg + c * STG_BOX + lane * 64 +
                                                     ((q ^ ((lane >> 1) & 3)) << 4));
        } else if (rrow != nullptr) {
#pragma unroll
          for (int q = 0; q < 4; ++q) res[q] = __ldcg(reinterpret_cast<const uint4*>(rrow + n0) + q);
        }
        float v[32];
        tmem_ld32(tbase + (uint32_t)(c * 32), v);
        tc_wait_ld();
        if (c + 1 == NCH && kind != CK_CHAIN_RESID_LN) {  // the accumulator goes back
          tc_fence_before();
          mbar_arrive(&tempty[acc]);
        }
        if (kind != CK_CHAIN_STORE) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) rbf2(v[i], v[i + 1]);
        }
        if (kind == CK_CHAIN_GELU) {
          gelu32(v);
        } else if (res_box || rrow != nullptr) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t w[4] = {res[q].x, res[q].y, res[q].z, res[q].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float lo = v[8 * q + 2 * j], hi = v[8 * q + 2 * j + 1];
              f2up(fadd2(f2pk(bf16_lo(w[j]), bf16_hi(w[j])), f2pk(lo, hi)), lo, hi);
              v[8 * q + 2 * j] = lo;
              v[8 * q + 2 * j + 1] = hi;
            }
          }
        }
        uint32_t y[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) y[i] = cvt_bf16x2(v[2 * i], v[2 * i + 1]);
        if (kind == CK_CHAIN_RESID_LN) {
          // Y (bf16) goes back into the accumulator's columns for the norm pass
          tmem_st16w(tbase + (uint32_t)(c * 32), y);
          // statistics of the values as stored (bf16), shifted by the slice's
          // first value so the sum of squares does not cancel
          if (c == 0) st_shift = bf16_lo(y[0]);
          float s1a = 0.f, s1b = 0.f, s2a = 0.f, s2b = 0.f;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float d0 = bf16_lo(y[i]) - st_shift, d1 = bf16_hi(y[i]) - st_shift;
            s1a += d0;
            s1b += d1;
            s2a = fmaf(d0, d0, s2a);
            s2b = fmaf(d1, d1, s2b);
          }
          st_s1 += s1a + s1b;
          st_s2 += s2a + s2b;
        }
        store_box(stg + c * STG_BOX, y, &maps.y[li], n0, m0, m0 < p.M, lane);
      }
      if (kind == CK_CHAIN_RESID_LN) {
        // Row statistics: this warp's (mean, M2) over its 64 columns goes to
        // its slot in both CTAs' shared memory (local store, DSMEM store), with
        // one arrival on each CTA's barrier; the eight slots of a row then
        // cover the 512 columns of both CTAs. The buffer alternates per
        // LayerNorm tile: a CTA writes buffer b again only after passing the
        // next tile's exchange, which needs the partner's arrivals for it, made
        // after the partner has read buffer b.
        const int lb = ln_count & 1;
        const uint32_t lph = (uint32_t)((ln_count >> 1) & 1);
        ++ln_count;
        const float mu = st_s1 / (float)SLICE;
        const float2 part = make_float2(st_shift + mu, fmaxf(st_s2 - st_s1 * mu, 0.f));
        float2* xb = sXch + lb * (8 * BM);
        float2* mine = xb + (int)(crank * 4 + slice) * BM + row;
        *mine = part;
        cl_store_f2(cl_map(mine, crank ^ 1u), part);
        mbar_arrive(&sready[lb]);
        cl_mbar_arrive(cl_map(&sready[lb], crank ^ 1u));
        if (!mbar_wait_cl(&sready[lb], lph, abort_flag, 27)) break;
        float2 q[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) q[k] = xb[k * BM + row];
        const float mean =
            0.125f * (((q[0].x + q[1].x) + (q[2].x + q[3].x)) + ((q[4].x + q[5].x) + (q[6].x + q[7].x)));
        float m2 = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float d = q[k].x - mean;
          m2 += q[k].y + (float)SLICE * d * d;
        }
        const float rstd = 1.0f / sqrtf(m2 / (float)(8 * SLICE) + L.eps);
        tc_wait_store();
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          const int n0 = nbase + c * 32;
          uint32_t y[16], normed[16];
          tmem_ld16w(tbase + (uint32_t)(c * 32), y);
          tc_wait_ld();
          if (c + 1 == NCH) {  // the accumulator goes back to the MMA warp
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
          }
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const uint4 g = __ldg(reinterpret_cast<const uint4*>(L.ln_gamma + n0) + q4);
            const uint4 b = L.ln_beta != nullptr
                                ? __ldg(reinterpret_cast<const uint4*>(L.ln_beta + n0) + q4)
                                : make_uint4(0u, 0u, 0u, 0u);
            const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
            const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int i = 4 * q4 + j;
              float y0 = (bf16_lo(y[i]) - mean) * rstd;
              float y1 = (bf16_hi(y[i]) - mean) * rstd;
              y0 = y0 * bf16_lo(gw[j]) + bf16_lo(bw[j]);
              y1 = y1 * bf16_hi(gw[j]) + bf16_hi(bw[j]);
              normed[i] = cvt_bf16x2(y0, y1);
            }
          }
          store_box(stg + c * STG_BOX, normed, &maps.y2[li], n0, m0, m0 < p.M, lane);
        }
      }
      if (L.signal) {
        // this warp's stores of the tile are complete and ordered before the
        // count that releases the row block to the next linear
        if (lane == 0) {
          bulk_wait<0>();
          fence_proxy_async_global();
          red_release_gpu_add(p.done + (int64_t)li * p.num_m_tiles + r, 1);
        }
        __syncwarp();
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
      if (job + n_cl < p.total_jobs && !prefetch_res(job + n_cl)) break;
    }
  epi_done:
    // a residual load still in flight (abort paths) lands before the CTA exits
    if (res_pending) mbar_wait(&rbar[e], rph, nullptr, 30);
    if (lane == 0) bulk_wait<0>();  // stores complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  // neither CTA leaves while its partner may still write its shared memory
  cl_sync();
}

// Clusters of two that the device keeps resident at once for this kernel.
int max_active_clusters() {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] > 0) return cached[dev];
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(num_sms() & ~1));
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = (size_t)SMEM_BYTES;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_chain_kernel, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  cached[dev] = n;
  return n;
}

bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace

// Opt-in (CK_CHAIN=1). Measured on B200 (Cortex-S, B = 32, CUDA graph of
// the forward): 821 us chained against 790 us with one launch per linear. The
// row blocks of a chain advance in lockstep, so every linear's epilogue
// latency (about 9 us for a LayerNorm tile: residual, row-statistics
// exchange, second pass, store completion before the count) lies on the
// chain's critical path, while the separate launches overlap it with other
// tiles.
bool gemm_chain_enabled() {
  const char* v = std::getenv("CK_CHAIN");
  return v != nullptr && std::strcmp(v, "1") == 0;
}

bool gemm_chain_supported(const ChainLinear* l, int n_links, int64_t M) {
  if (l == nullptr || n_links < 1 || n_links > MAX_LINKS || M <= 0 || M > INT32_MAX) return false;
  for (int i = 0; i < n_links; ++i) {
    const ChainLinear& c = l[i];
    if (c.A == nullptr || c.W == nullptr || c.Y == nullptr) return false;
    if (c.N <= 0 || c.K <= 0 || c.N % (2 * BN) != 0 || c.N > INT32_MAX || c.K > INT32_MAX)
      return false;
    if (!al16(c.A) || !al16(c.W) || !al16(c.Y) || (c.lda * 2) % 16 != 0 || (c.K * 2) % 16 != 0 ||
        (c.ldy * 2) % 16 != 0)
      return false;
    if (c.kind < CK_CHAIN_STORE || c.kind > CK_CHAIN_RESID_LN) return false;
    if (c.kind >= CK_CHAIN_RESID &&
        (c.aux == nullptr || !al16(c.aux) || (c.ld_aux * 2) % 16 != 0 || c.aux_link >= i))
      return false;
    if (c.kind == CK_CHAIN_RESID_LN &&
        (c.N != 2 * BN || c.Y2 == nullptr || !al16(c.Y2) || (c.ldy2 * 2) % 16 != 0 ||
         c.ln_gamma == nullptr || !al16(c.ln_gamma) || (c.ln_beta != nullptr && !al16(c.ln_beta))))
      return false;
  }
  return true;
}

size_t gemm_chain_counter_bytes(int64_t M, int n_links) {
  const int64_t mt = (M + BM - 1) / BM;
  return (size_t)(n_links * mt + 1) * sizeof(int);
}

int gemm_chain(const ChainLinear* l, int n_links, int64_t M, int* counters, cudaStream_t st) {
  if (!gemm_chain_supported(l, n_links, M) || counters == nullptr) return CK_ERR_INVALID_ARG;
  ChainArgs a;
  memset(&a, 0, sizeof(a));
  a.M = (int)M;
  a.num_m_tiles = (int)((M + BM - 1) / BM);
  a.num_links = n_links;
  a.done = counters;
  a.abort = counters + (int64_t)n_links * a.num_m_tiles;
  ChainMaps maps;
  memset(&maps, 0, sizeof(maps));
  int job = 0;
  for (int i = 0; i < n_links; ++i) {
    const ChainLinear& c = l[i];
    Link& L = a.l[i];
    L.kind = c.kind;
    L.n_tiles = (int)(c.N / BN);
    L.k_blocks = (int)((c.K + BK - 1) / BK);
    L.job0 = job;
    L.jobs = a.num_m_tiles * L.n_tiles / 2;
    job += L.jobs;
    L.wait_target = i > 0 ? a.l[i - 1].n_tiles * EPI_WARPS : 0;
    L.signal = i + 1 < n_links;
    L.aux = reinterpret_cast<const __nv_bfloat16*>(c.aux);
    L.ld_aux = c.ld_aux;
    L.aux_row_mod = c.aux_row_mod;
    L.aux_link = c.kind >= CK_CHAIN_RESID ? c.aux_link : -1;
    L.aux_target = L.aux_link >= 0 ? a.l[L.aux_link].n_tiles * EPI_WARPS : 0;
    // a 32-row residual box is contiguous unless a broadcast period cuts it
    L.aux_tma = c.kind >= CK_CHAIN_RESID && (c.aux_row_mod <= 0 || c.aux_row_mod % 32 == 0);
    if (L.aux_tma &&
        !make_tmap_2d(&maps.r[i], c.aux, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, c.N,
                      c.aux_row_mod > 0 ? (uint64_t)c.aux_row_mod : (uint64_t)M, c.ld_aux, 32, 32,
                      64))
      return CK_ERR_INVALID_ARG;
    L.ln_gamma = reinterpret_cast<const __nv_bfloat16*>(c.ln_gamma);
    L.ln_beta = reinterpret_cast<const __nv_bfloat16*>(c.ln_beta);
    L.eps = c.eps;
    if (!make_tmap_2d(&maps.a[i], c.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, c.K, M, c.lda, BK, BM,
                      128) ||
        !make_tmap_2d(&maps.b[i], c.W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, c.K, c.N, c.K, BK, BN,
                      128) ||
        !make_tmap_2d(&maps.y[i], c.Y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, c.N, M, c.ldy, 32, 32,
                      64))
      return CK_ERR_INVALID_ARG;
    if (c.kind == CK_CHAIN_RESID_LN) {
      if (!make_tmap_2d(&maps.y2[i], c.Y2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, c.N, M, c.ldy2, 32,
                        32, 64))
        return CK_ERR_INVALID_ARG;
    } else {
      maps.y2[i] = maps.y[i];
    }
  }
  a.total_jobs = job;
  if (!smem_attr_ready(reinterpret_cast<const void*>(gemm_chain_kernel), SMEM_BYTES))
    return record_cuda_error();
  const int resident = max_active_clusters();
  if (resident <= 0) return CK_ERR_UNSUPPORTED;
  const int clusters = a.total_jobs < resident ? a.total_jobs : resident;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * clusters));
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = (size_t)SMEM_BYTES;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return finish_launch(cudaLaunchKernelEx(&cfg, gemm_chain_kernel, maps, a));
}

}  // namespace ck
