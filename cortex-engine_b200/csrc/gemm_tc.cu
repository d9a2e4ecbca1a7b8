// tcgen05 GEMM for the Cortex linears on B200 (sm_100a).
//
//   Y[M, N] = epilogue( A[M, K] (bf16, K-major) x B^T )
//
// B is the weight: (N, K) bf16 K-major (nn.Linear), (K, N) bf16 N-major
// (rms_norm_linear's w), or (N, K) int8 K-major with per-output-channel fp32
// scales (QuantizedLinear, cortex/quantization/calibrate.py:170-228). The int8
// tile is widened to bf16 in shared memory by a converter warpgroup (exact for
// |w| <= 127) and the scale is applied to the fp32 accumulator.
//
// Structure (one persistent CTA per SM, warp-specialised):
//   warp 0       TMA producer: A and B tiles into a STAGES-deep smem ring
//   warp 1       TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..17  epilogue (2..9 in int8 mode): four (two) warps per TMEM lane
//                quarter, each taking a quarter (half) of the tile's columns in
//                32-column chunks: tcgen05.ld of the fp32
//                accumulator (the next chunk's read and residual load in flight
//                while the current one is finished), the epilogue op (scale,
//                bf16 rounding, GELU / residual / bias), a 64B-swizzled
//                32 x 32 smem box per chunk and one TMA tile store per chunk
//   warps 18..21 (int8 only: 10..13) int8 -> bf16 converter
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile i overlaps the main loop of tile i+1. All mbarrier waits are bounded
// (common.cuh); a timeout raises a CTA-wide abort flag and every role drains.
//
// FUSE_LN (residual epilogue, N == 2 * BN): the two column halves of a row
// block go to the two CTAs of a cluster. Each epilogue warp has one store box
// per 32-column chunk of its slice; the tile's residual arrives in them by
// TMA before the accumulator is ready. The regular epilogue pass writes the
// residual output Y through the boxes (each lane replaces its row's residual
// with Y), forms per-row (mean, M2) of its columns and leaves Y (bf16) in the
// TMEM accumulator; the partials go to both CTAs' shared memory (local store +
// DSMEM store, mbarrier arrivals local and remote). Once a row's four partials
// are in, a second pass reads Y back from TMEM and writes its LayerNorm Y2
// (the next block's normalised input), with gamma and beta staged in shared
// memory.
#include <cuda.h>

#include <cstdlib>
#include <cstring>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemm_common.cuh"
#include "kernels.h"

namespace ck {

namespace {

using gemm::GemmArgs;
using gemm::epilogue_math;

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int STG_BOX = 32 * 32 * 2;  // one 32-row x 32-col bf16 store box (64B rows)
// FUSE_LN: each warp's columns in 32-row x 64-col boxes (128B rows, 128B
// swizzle), two 32-column chunks per box, so that the residual loads and the
// two output stores take half as many TMA commands
constexpr int LN_BOX = 32 * 64 * 2;

enum WMode { W_BF16_NK = 0, W_BF16_KN = 1, W_I8_NK = 2 };

template <int BN, int WMODE, int FUSE = 0, int EPI = CK_EPI_STORE, bool PAIR_ = false>
struct GemmCfg {
  // PAIR: 2-SM MMA. A cluster of two CTAs computes a 256-row tile: each CTA
  // holds its 128 rows of A and of the accumulator and half of B's BN rows;
  // the even CTA issues the cta_group::2 MMAs for both.
  static constexpr bool PAIR = PAIR_;
  // epilogue warps: four per TMEM lane quarter for the GELU epilogue with bf16
  // weights, whose arithmetic per element is heavy enough that two warps per
  // scheduler cannot keep up with the tensor cores, and for the fused
  // LayerNorm with bf16 weights, whose two-pass epilogue is latency-bound and
  // lies on the critical path (one tile per CTA); two per quarter otherwise
  // (and always in int8 mode, whose converter warps need the registers)
  static constexpr bool LN = FUSE == 3;   // gemm::FUSE_LN
  static constexpr bool RMS = FUSE == 4;  // gemm::FUSE_RMS: a norm warpgroup scales the A tiles
  static constexpr int EPI_WARPS =
      (WMODE != W_I8_NK && (EPI == CK_EPI_GELU || LN)) ? 16 : 8;
  static constexpr int EPI_GROUPS = EPI_WARPS / 4;  // column slices of a tile
  static constexpr int EPI_COLS = BN / EPI_GROUPS;  // columns per epilogue warp per tile
  static constexpr int A_BYTES = BM * BK * 2;                        // 16 KB
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;     // bf16 operand (this CTA's)
  static constexpr int B8_BYTES = (WMODE == W_I8_NK) ? BN * BK : 0;  // int8 staging
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + B8_BYTES;
  // per epilogue warp: 32-row x 32-column bf16 store boxes (64B-swizzled): one
  // per chunk of its columns for FUSE_LN (they take the residual tile first),
  // else two (one with four warps per lane quarter)
  static constexpr int STG_WARP = (LN ? EPI_COLS / 32 : (EPI_WARPS == 8 ? 2 : 1)) * STG_BOX;
  static constexpr int EPI_SMEM = EPI_WARPS * STG_WARP;
  static constexpr int BAR_BYTES = (LN || RMS) ? 512 : 256;
  // FUSE_LN: per accumulator buffer, the (mean, M2) partials of the 4 column
  // quarters (2 CTAs x 2 warp column slices) of every row
  static constexpr int XCH_SMEM = LN ? 2 * (2 * EPI_GROUPS) * BM * 8 : 0;
  // FUSE_LN: each epilogue warp's gamma | beta columns (bf16), staged once
  // (two warps per lane quarter only: with four, the pipeline ring needs the room
  // and the norm pass reads them through the read-only cache)
  static constexpr int GB_SMEM = (LN && EPI_WARPS == 8) ? EPI_WARPS * 2 * EPI_COLS * 2 : 0;
  // FUSE_RMS: the per-row 1 / rms of each TMEM accumulator buffer (gamma
  // comes through the read-only cache, so that the ring keeps its stages)
  // FUSE_RMS norm warps: eight (two per scheduler, each thread half a row of a
  // stage) with bf16 weights, four (a whole row each) beside the int8
  // converter warps, whose registers they would otherwise take
  static constexpr int RMS_WARPS = !RMS ? 0 : (WMODE == W_I8_NK ? 4 : 8);
  static constexpr int RMS_SPLIT = RMS ? RMS_WARPS / 4 : 1;  // threads per row
  static constexpr int RSTD_SMEM = RMS ? 2 * RMS_SPLIT * BM * 4 : 0;
  static constexpr int BUDGET =
      232448 - 1024 - BAR_BYTES - EPI_SMEM - XCH_SMEM - GB_SMEM - RSTD_SMEM;
  static constexpr int STAGES = BUDGET / STAGE_BYTES > 8 ? 8 : BUDGET / STAGE_BYTES;
  // bytes completing one stage's barrier (PAIR: both CTAs' loads, on the even CTA's)
  static constexpr int TX_BYTES = (PAIR ? 2 : 1) * (A_BYTES + (WMODE == W_I8_NK ? B8_BYTES : B_BYTES));
  static constexpr int CONV_WARP0 = 2 + EPI_WARPS;
  static constexpr int NORM_WARP0 = CONV_WARP0 + (WMODE == W_I8_NK ? 4 : 0);
  static constexpr int NUM_THREADS = 32 * (NORM_WARP0 + RMS_WARPS);
  // arrivals that make a stage's operands ready for the MMA after the TMA:
  // the int8 converter and / or the norm warpgroup, 128 threads each
  static constexpr int CONV_COUNT = 128 * (WMODE == W_I8_NK ? 1 : 0) + 32 * RMS_WARPS;
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // double-buffered accumulator
  static constexpr int SMEM_BYTES =
      1024 + STAGES * STAGE_BYTES + EPI_SMEM + XCH_SMEM + GB_SMEM + RSTD_SMEM + BAR_BYTES;
  static constexpr uint32_t IDESC = idesc_bf16(BM, BN, WMODE == W_BF16_KN ? 1u : 0u);
  static constexpr uint32_t IDESC_HALF = idesc_bf16(BM, BN / 2, 0u);  // split tiles (NK only)
  static constexpr uint32_t IDESC_PAIR = idesc_bf16(2 * BM, BN, 0u);   // PAIR (NK only)
};

template <int BN, int WMODE, int EPI, int FUSE, bool PAIR = false>
__global__ void __launch_bounds__(GemmCfg<BN, WMODE, FUSE, EPI, PAIR>::NUM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmY2,
                   const __grid_constant__ CUtensorMap tmR, const GemmArgs p) {
  using C = GemmCfg<BN, WMODE, FUSE, EPI, PAIR>;
  static_assert(!PAIR || (WMODE == W_BF16_NK && FUSE == 0), "PAIR: bf16 (N, K) weights, no fusion");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + C::STAGES * C::A_BYTES;
  uint8_t* sB8 = sB + C::STAGES * C::B_BYTES;
  uint8_t* sStg = sB8 + C::STAGES * C::B8_BYTES;  // 1 KB aligned (all sizes above are)
  float2* sXch = reinterpret_cast<float2*>(sStg + C::EPI_SMEM);
  uint8_t* sGB = reinterpret_cast<uint8_t*>(sXch) + C::XCH_SMEM;  // [EPI_WARPS][gamma | beta]
  // FUSE_RMS: per accumulator buffer, each row's sum of squares in RMS_SPLIT parts
  float* sRstd = reinterpret_cast<float*>(sGB + C::GB_SMEM);  // [2][RMS_SPLIT][BM]
  uint8_t* sBar = reinterpret_cast<uint8_t*>(sRstd) + C::RSTD_SMEM;
  uint64_t* full = reinterpret_cast<uint64_t*>(sBar);
  uint64_t* empty = full + C::STAGES;
  uint64_t* conv = empty + C::STAGES;
  uint64_t* tfull = conv + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* sready = drain + 1;  // FUSE_LN: row partials of both CTAs' warps are in sXch[acc]
  uint64_t* rbar = sready + 2;   // FUSE_LN: [EPI_WARPS] a warp's residual boxes have landed
  uint64_t* rfull = rbar + (C::LN ? C::EPI_WARPS : 0);  // FUSE_RMS: sRstd[acc] is written
  uint64_t* rempty = rfull + 2;                          // FUSE_RMS: sRstd[acc] was read
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rempty + (C::RMS ? 2 : 0));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_tiles = p.num_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], C::CONV_COUNT > 0 ? C::CONV_COUNT : 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      // PAIR: the even CTA's copy collects both CTAs' epilogue threads
      mbar_init(&tempty[a], (PAIR ? 2 : 1) * C::EPI_WARPS * 32);
    }
    mbar_init(drain, 1);
    if (C::LN) {
      for (int a = 0; a < 2; ++a) mbar_init(&sready[a], 2 * C::EPI_WARPS);  // a warp arrives once
      for (int w = 0; w < C::EPI_WARPS; ++w) mbar_init(&rbar[w], 1);
    }
    if (C::RMS) {
      for (int a = 0; a < 2; ++a) {
        mbar_init(&rfull[a], 32 * C::RMS_WARPS);
        mbar_init(&rempty[a], C::EPI_WARPS * 32);
      }
    }
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmY);
    if (C::LN) {
      prefetch_tmap(&tmY2);
      if (p.res_tma) prefetch_tmap(&tmR);
    }
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // FUSE_LN / PAIR: the partner CTA's barriers are initialised before any
  // remote arrival or load completion
  if (C::LN || PAIR) cl_sync();
  const uint32_t crank = PAIR ? cl_rank() : 0u;  // PAIR: 0 issues the MMAs
  // the tile loop of a PAIR cluster: both CTAs walk the same 256-row tiles
  const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tstep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const uint32_t tmem_base = *tmem_slot;
  // Tile -> (row block, column block). FUSE_LN pairs the two column blocks of a
  // row block on the two CTAs of a cluster (consecutive tiles, even stride).
  // part: -1 for a whole tile, 0 / 1 for the first / second BN/2 columns of a
  // split tile (tiles from p.split_from on).
  auto tile_mn = [&](int tile, int& mt, int& nt, int& part) {
    part = -1;
    if (C::LN) {
      mt = tile >> 1;
      nt = tile & 1;
      return;
    }
    if (tile >= p.split_from) {
      part = (tile - p.split_from) & 1;
      tile = p.split_from + ((tile - p.split_from) >> 1);
    }
    mt = tile % p.num_m_tiles;  // PAIR: 256-row tiles, this CTA's half
    nt = tile / p.num_m_tiles;
    if (PAIR) mt = 2 * mt + (int)crank;
  };

  // When the caller vouches that the weight (B) is not written by the kernel
  // this one may overlap (p.pre_b: model weights inside the forward), the
  // producer issues the first ring stages' B loads before the dependency wait
  // (one-CTA tiles with bf16 weights); their A loads follow the wait. The
  // weights' HBM latency then runs under the previous kernel's tail.
  int pre_b = 0;
  if (p.pre_b && !PAIR && WMODE != W_I8_NK && warp == 0 && lane == 0 && tile0 < num_tiles) {
    int mt, nt, part;
    tile_mn(tile0, mt, nt, part);
    pre_b = p.num_k_blocks < C::STAGES ? p.num_k_blocks : C::STAGES;
    for (int kb = 0; kb < pre_b; ++kb) {
      mbar_arrive_expect_tx(&full[kb], C::TX_BYTES);
      if (WMODE == W_BF16_NK) {
        tma_load_2d(sB + kb * C::B_BYTES, &tmB, &full[kb], kb * BK,
                    nt * BN + (part > 0 ? BN / 2 : 0));
      } else {
#pragma unroll
        for (int j = 0; j < BN / 64; ++j)
          tma_load_2d(sB + kb * C::B_BYTES + j * (64 * BK * 2), &tmB, &full[kb], nt * BN + j * 64,
                      kb * BK);
      }
    }
  }
  grid_dep_wait();
  // Dependent grids may launch at once; FUSE_LN signals them only when its
  // epilogue is done (measured on B200: the early signal made the Cortex
  // forward 1.5-2 % slower with the fused LayerNorm, 1 % faster without it).
  if (!C::LN) grid_dep_launch();

  if (warp == 0) {
    // ── TMA producer ──
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int tile = tile0; tile < num_tiles && !*abort_flag; tile += tstep) {
        int mt, nt, part;
        tile_mn(tile, mt, nt, part);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait_park(&empty[stage], phase ^ 1, abort_flag, 1)) break;
          if (PAIR) {
            // both CTAs' bytes complete on the even CTA's barrier, which alone
            // announces them
            if (crank == 0) mbar_arrive_expect_tx(&full[stage], C::TX_BYTES);
            const uint32_t fb = cl_map(&full[stage], 0);
            tma_load_2d_pair(sA + stage * C::A_BYTES, &tmA, fb, kb * BK, mt * BM);
            tma_load_2d_pair(sB + stage * C::B_BYTES, &tmB, fb, kb * BK,
                             nt * BN + (int)crank * (BN / 2));
            ++issued;
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          const bool pre = tile == tile0 && kb < pre_b;  // B already in flight
          if (!pre) mbar_arrive_expect_tx(&full[stage], C::TX_BYTES);
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * BK, mt * BM);
          if (pre) {
          } else if (WMODE == W_BF16_NK) {
            // (a split tile's second half starts BN/2 rows further; the box
            // stays BN rows, of which its N = BN/2 MMA reads the first half)
            tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * BK,
                        nt * BN + (part > 0 ? BN / 2 : 0));
          } else if (WMODE == W_BF16_KN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sB + stage * C::B_BYTES + j * (64 * BK * 2), &tmB, &full[stage],
                          nt * BN + j * 64, kb * BK);
          } else {
            tma_load_2d(sB8 + stage * C::B8_BYTES, &tmB, &full[stage], kb * BK, nt * BN);
          }
          ++issued;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: make sure every issued copy has landed before the CTA can exit
      // (PAIR: the even CTA's barriers count both CTAs' copies; the odd CTA is
      // held by the cluster barrier before exit).
      for (int s = 0; s < C::STAGES && s < issued && crank == 0; ++s) {
        const int last = issued - 1 - ((issued - 1 - s) % C::STAGES);
        mbar_wait(&full[s], (uint32_t)((last / C::STAGES) & 1), nullptr, 9);
      }
    }
  } else if (warp == 1) {
    // ── MMA issuer (PAIR: the even CTA only) ──
    if (lane == 0 && crank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = tile0; tile < num_tiles && ok; tile += tstep) {
        int mt_, nt_, part;
        tile_mn(tile, mt_, nt_, part);
        const uint32_t idesc = PAIR ? C::IDESC_PAIR : (part >= 0 ? C::IDESC_HALF : C::IDESC);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          uint64_t* ready = C::CONV_COUNT > 0 ? &conv[stage] : &full[stage];
          if (!mbar_wait(ready, phase, abort_flag, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = sw128_desc(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = (WMODE == W_BF16_KN)
                                       ? sw128_desc(b_addr + k * 16 * 128, 64 * BK * 2, 1024)
                                       : sw128_desc(b_addr + k * 32, 16, 1024);
            if (PAIR)
              tc_mma_ss_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
            else
              tc_mma_ss(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          if (PAIR)
            tc_commit_pair(&empty[stage], 3);  // both CTAs' stage is free
          else
            tc_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (PAIR)
          tc_commit_pair(&tfull[acc], 3);  // both CTAs' accumulators are ready
        else
          tc_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // Drain all issued MMAs before TMEM / smem can be released.
      if (PAIR)
        tc_commit_pair(drain, 1);
      else
        tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 8);
    }
  } else if (warp < C::CONV_WARP0) {
    // ── epilogue: (lane quarter, column slice) per warp ──
    const int e = warp - 2;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int half = e >> 2;       // column slice
    const int row = quarter * 32 + lane;
    constexpr int COLS = C::EPI_COLS;
    constexpr int NCH = COLS / 32;  // 32-column chunks per warp per tile
    constexpr int NBOX = C::STG_WARP / STG_BOX;
    uint8_t* stg = sStg + e * C::STG_WARP;
    // FUSE_LN: byte offset of 16-byte piece q of chunk c of this lane's row
    auto ln_off = [&](int c, int q) -> uint32_t {
      return (uint32_t)((c >> 1) * LN_BOX + lane * 128 + ((((c & 1) * 4 + q) ^ (lane & 7)) << 4));
    };
    int acc = 0;
    uint32_t acc_phase = 0;
    // FUSE_LN: this warp's gamma | beta columns into shared memory (a CTA
    // keeps one column half: tiles alternate halves and the stride is even),
    // and the residual tile of each row block by TMA into the warp's boxes,
    // issued before the tile's accumulator is ready.
    uint8_t* wgb = sGB + e * (2 * COLS * 2);
    constexpr bool res_box = C::LN;  // (the host only fuses residuals it can box)
    uint32_t rph = 0;
    bool res_pending = false;
    auto prefetch_res = [&](int tile) {
      int mt, nt, part;
      tile_mn(tile, mt, nt, part);
      if (lane == 0) {
        bulk_wait_read<0>();  // the boxes' last stores have read them
        const int m0 = mt * BM + quarter * 32;
        const int row0 = p.aux_row_mod > 0 ? (int)((int64_t)m0 % p.aux_row_mod) : m0;
        mbar_arrive_expect_tx(&rbar[e], C::STG_WARP);
#pragma unroll
        for (int c = 0; c < NCH; c += 2)
          tma_load_2d(stg + (c >> 1) * LN_BOX, &tmR, &rbar[e], nt * BN + half * COLS + c * 32, row0);
      }
      res_pending = true;
    };
    if constexpr (C::LN) {
      if (tile0 < num_tiles) {
        if constexpr (C::GB_SMEM > 0) {
          static_assert(2 * COLS * 2 == 32 * 16, "FUSE_LN: one 16-byte piece of gamma | beta per lane");
          int mt, nt, part;
          tile_mn(tile0, mt, nt, part);
          const int n0 = nt * BN + half * COLS;
          const int k = lane & 15;
          const __nv_bfloat16* src = lane < 16 ? p.ln_gamma : p.ln_beta;
          *reinterpret_cast<uint4*>(wgb + lane * 16) =
              src != nullptr ? __ldg(reinterpret_cast<const uint4*>(src + n0) + k)
                             : make_uint4(0u, 0u, 0u, 0u);
          __syncwarp();
        } else {
          // gamma / beta go through the read-only cache in the second pass:
          // bring this warp's 64 columns of each into L1 now, so that the
          // second pass does not wait on L2 right after the row exchange
          int mt, nt, part;
          tile_mn(tile0, mt, nt, part);
          const int n0 = nt * BN + half * COLS;
          const __nv_bfloat16* src = lane == 0 ? p.ln_gamma : (lane == 1 ? p.ln_beta : nullptr);
          if (src != nullptr)
            for (int b = 0; b < COLS * 2; b += 128)
              asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<const uint8_t*>(src + n0) + b));
        }
        if (res_box) prefetch_res(tile0);
      }
    }
    for (int tile = tile0; tile < num_tiles; tile += tstep) {
      int mt, nt, part;
      tile_mn(tile, mt, nt, part);
      if (!mbar_wait_park(&tfull[acc], acc_phase, abort_flag, 4)) break;
      if (res_box) {
        if (!mbar_wait_park(&rbar[e], rph, abort_flag, 10)) break;
        rph ^= 1;
        res_pending = false;
      }
      float row_rstd = 1.f;  // FUSE_RMS: 1 / rms of this row
      if constexpr (C::RMS) {
        if (!mbar_wait_park(&rfull[acc], acc_phase, abort_flag, 12)) break;
        float ss = 0.f;
#pragma unroll
        for (int h = 0; h < C::RMS_SPLIT; ++h) ss += sRstd[(acc * C::RMS_SPLIT + h) * BM + row];
        row_rstd = 1.0f / sqrtf(ss / (float)p.K + p.norm_eps);
        mbar_arrive(&rempty[acc]);
      }
      __syncwarp();
      tc_fence_after();
      const int m = mt * BM + row;
      float st_shift = 0.f, st_s1 = 0.f, st_s2 = 0.f;  // row statistics (FUSE_LN)
      // a split tile's BN/2 columns are spread over all column slices
      const int col0 = part >= 0 ? half * (COLS / 2) : half * COLS;
      const int nch = part >= 0 ? NCH / 2 : NCH;
      const int nbase = nt * BN + (part > 0 ? BN / 2 : 0) + col0;
      const uint32_t tbase =
          tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN + col0);
      const bool row_ok = m < p.M;
      const int m0 = mt * BM + quarter * 32;
      const __nv_bfloat16* rrow =
          (EPI == CK_EPI_RESID && row_ok) ? p.aux + gemm::residual_row(p, m) * p.ld_aux : nullptr;
      // 32-column chunks, TMEM reads double-buffered: chunk c + 1 (and its
      // residual) is in flight while chunk c is finished and handed to a TMA
      // store; TMEM goes back to the MMA warp as soon as the last chunk has
      // been read.
      float va[32], vb[32];
      uint4 ra[4], rb[4];
      // (only the bf16 mode with two warps per lane quarter prefetches: with
      // four warps the other warps hide the load, and the registers are short)
      constexpr bool kPrefetch =
          EPI == CK_EPI_RESID && WMODE != W_I8_NK && C::EPI_WARPS == 8 && !res_box;
      auto fetch_res = [&](int c, uint4* dst) {
        if (kPrefetch && !res_box && row_ok && nbase + c * 32 + 32 <= p.N) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = __ldg(reinterpret_cast<const uint4*>(rrow + nbase + c * 32) + q);
        }
      };
      // Two warps per lane quarter read ahead (double-buffered chunks); with
      // four, each warp reads a chunk when it needs it and the other warps of
      // its scheduler cover the latency, which keeps it inside 96 registers.
      constexpr bool kAhead = C::EPI_WARPS == 8;
      tmem_ld32(tbase, va);
      fetch_res(0, ra);
      tc_wait_ld();
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        if (c >= nch) break;
        float* cur = (kAhead && (c & 1)) ? vb : va;
        float* nxt = (c & 1) ? va : vb;
        uint4* rcur = (c & 1) ? rb : ra;
        uint4* rnxt = (c & 1) ? ra : rb;
        if (!kAhead && c > 0) {
          tmem_ld32(tbase + (uint32_t)(c * 32), va);
          tc_wait_ld();
        }
        if (kAhead && c + 1 < nch) {
          tmem_ld32(tbase + (uint32_t)((c + 1) * 32), nxt);
          fetch_res(c + 1, rnxt);
        } else if (c + 1 == nch && !C::LN) {  // (FUSE_LN reads the tile again below)
          tc_fence_before();
          if (PAIR && crank != 0)
            cl_mbar_arrive(cl_map(&tempty[acc], 0));  // the even CTA issues the MMAs
          else
            mbar_arrive(&tempty[acc]);
        }
        const int n0 = nbase + c * 32;
        if (n0 < p.N) {
          if (res_box) {  // the residual chunk from its box (this lane's row)
#pragma unroll
            for (int q = 0; q < 4; ++q)
              rcur[q] = lds128(smem_u32(stg + ln_off(c, q)));
          }
          uint32_t packed[16];
          if constexpr (C::RMS) {
#pragma unroll
            for (int i = 0; i < 32; ++i) cur[i] *= row_rstd;
          }
          epilogue_math<EPI>(p, m, n0, cur,
                             ((kPrefetch || res_box) && n0 + 32 <= p.N) ? rcur : nullptr, packed);
          if (C::LN) tmem_st16w(tbase + (uint32_t)(c * 32), packed);  // Y, for the norm pass
          if (C::LN) {
            // statistics of the values as stored (bf16), shifted by the
            // segment's first value so the sum of squares does not cancel
            if (c == 0) st_shift = bf16_lo(packed[0]);
            // (even, odd) columns in the two lanes of paired fp32 sums
            const unsigned long long nshift = f2pk(-st_shift, -st_shift);
            unsigned long long s1 = f2pk(0.f, 0.f), s2 = f2pk(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const bool ok0 = n0 + 2 * i < p.N, ok1 = n0 + 2 * i + 1 < p.N;
              const unsigned long long d =
                  fadd2(f2pk(ok0 ? bf16_lo(packed[i]) : st_shift, ok1 ? bf16_hi(packed[i]) : st_shift),
                        nshift);
              s1 = fadd2(s1, d);
              s2 = ffma2(d, d, s2);
            }
            float s1a, s1b, s2a, s2b;
            f2up(s1, s1a, s1b);
            f2up(s2, s2a, s2b);
            st_s1 += s1a + s1b;
            st_s2 += s2a + s2b;
          }
          // 64B-swizzled 32 x 32 box, then one TMA store per chunk; the box was
          // last read by the store issued two chunks ago
          // the box is free once the store that last used it has read it
          // (FUSE_LN: one box per chunk, all free since the tile began; the
          // chunks' stores go out together after the last one)
          uint8_t* box = stg + (NBOX == 2 ? (c & 1) : NBOX == 1 ? 0 : c) * STG_BOX;
          if (lane == 0) {
            if (NBOX == 2)
              bulk_wait_read<1>();
            else if (NBOX == 1)
              bulk_wait_read<0>();
          }
          if (!C::LN) __syncwarp();
#pragma unroll
          for (int q = 0; q < 4; ++q)
            sts128(smem_u32(C::LN ? stg + ln_off(c, q)
                                  : box + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)),
                   make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]));
          if (!C::LN) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && m0 < p.M) {
              tma_store_2d(&tmY, box, n0, m0);
              bulk_commit();
            }
          }
        }
        if (kAhead && c + 1 < nch) tc_wait_ld();
      }
      if constexpr (C::LN) {
        // Row statistics: this warp's (mean, M2) over its COLS columns goes to
        // its slot in both CTAs' shared memory, with one arrival per warp on
        // each CTA's barrier; the NP slots of a row then hold both CTAs' column
        // slices. The lanes store their rows' partials locally (32 contiguous
        // rows per warp); lane 0 copies the warp's 256 bytes to the partner
        // (DSMEM) and arrives on both barriers, whose release at cluster scope
        // covers its copies and, through the warp barrier, the lanes' stores.
        // Lane 0 alone polls the barrier (acquire at cluster scope) and the
        // warp barrier passes the partials on to the other lanes.
        constexpr int NP = 2 * C::EPI_GROUPS;
        const float mu = st_s1 / (float)COLS;
        const float2 part = make_float2(st_shift + mu, fmaxf(st_s2 - st_s1 * mu, 0.f));
        const uint32_t self = cl_rank();
        const uint32_t peer = self ^ 1u;
        float2* xb = sXch + acc * (NP * BM);
        float2* mine = xb + ((int)self * C::EPI_GROUPS + half) * BM + quarter * 32;  // 32 rows
        mine[lane] = part;
        __syncwarp();
        int xok = 1;
        if (lane == 0) {
          const uint32_t src = smem_u32(mine);
          const uint32_t dst = cl_map(mine, peer);
#pragma unroll
          for (int i = 0; i < 16; ++i) cl_store_v4(dst + 16 * i, lds128(src + 16 * i));
          mbar_arrive(&sready[acc]);
          cl_mbar_arrive(cl_map(&sready[acc], peer));
        }
        // the first pass's boxes (Y) go out while the partials cross over
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (m0 < p.M) {
#pragma unroll
            for (int c = 0; c < NCH; c += 2)
              tma_store_2d(&tmY, stg + (c >> 1) * LN_BOX, nbase + c * 32, m0);
            bulk_commit();
          }
          xok = mbar_wait_cl(&sready[acc], acc_phase, abort_flag, 6) ? 1 : 0;
        }
        xok = __shfl_sync(0xffffffffu, xok, 0);
        __syncwarp();
        if (!xok) break;
        float2 q[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) q[k] = xb[k * BM + row];
        float msum = 0.f;
#pragma unroll
        for (int k = 0; k < NP; ++k) msum += q[k].x;
        const float mean = msum / (float)NP;
        float m2 = 0.f;
#pragma unroll
        for (int k = 0; k < NP; ++k) {
          const float d = q[k].x - mean;
          m2 += q[k].y + (float)COLS * d * d;
        }
        const float rstd = 1.0f / sqrtf(m2 / (float)(NP * COLS) + p.norm_eps);
        // LN(Y): Y comes back from TMEM, where the first pass left it as bf16;
        // the boxes are reused once the first pass's stores have read them
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        tc_wait_store();
#pragma unroll 1
        for (int c = 0; c < NCH; ++c) {
          uint32_t yk[16], normed[16];
          tmem_ld16w(tbase + (uint32_t)(c * 32), yk);
          tc_wait_ld();
          if (c + 1 == NCH) {
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
          }
          const int n0 = nbase + c * 32;
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 g, b;
            if constexpr (C::GB_SMEM > 0) {
              g = lds128(smem_u32(wgb + (c * 32 + q4 * 8) * 2));
              b = lds128(smem_u32(wgb + (COLS + c * 32 + q4 * 8) * 2));
            } else {
              g = __ldg(reinterpret_cast<const uint4*>(p.ln_gamma + n0) + q4);
              b = p.ln_beta != nullptr ? __ldg(reinterpret_cast<const uint4*>(p.ln_beta + n0) + q4)
                                       : make_uint4(0u, 0u, 0u, 0u);
            }
            const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
            const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int i = 4 * q4 + j;
              float y0 = (bf16_lo(yk[i]) - mean) * rstd;
              float y1 = (bf16_hi(yk[i]) - mean) * rstd;
              y0 = y0 * bf16_lo(gw[j]) + bf16_lo(bw[j]);
              y1 = y1 * bf16_hi(gw[j]) + bf16_hi(bw[j]);
              normed[i] = cvt_bf16x2(y0, y1);
            }
          }
          // the boxes were read by the first pass's stores (waited for above)
#pragma unroll
          for (int q = 0; q < 4; ++q)
            sts128(smem_u32(stg + ln_off(c, q)),
                   make_uint4(normed[4 * q], normed[4 * q + 1], normed[4 * q + 2], normed[4 * q + 3]));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && m0 < p.M) {
#pragma unroll
          for (int c = 0; c < NCH; c += 2) tma_store_2d(&tmY2, stg + (c >> 1) * LN_BOX, nbase + c * 32, m0);
          bulk_commit();
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
      if (res_box && tile + tstep < num_tiles) prefetch_res(tile + tstep);
    }
    // a residual load still in flight (abort paths) lands before the CTA exits
    if (res_pending) mbar_wait(&rbar[e], rph, nullptr, 11);
    if (C::LN) grid_dep_launch();
    if (lane == 0) bulk_wait<0>();  // stores complete before the CTA exits
  } else if (WMODE == W_I8_NK && warp < C::NORM_WARP0) {
    // ── int8 -> bf16 converter (4 warps) ──
    const int t = threadIdx.x - 32 * C::CONV_WARP0;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = tile0; tile < num_tiles && ok; tile += tstep) {
      for (int kb = 0; kb < p.num_k_blocks; ++kb) {
        if (!mbar_wait_park(&full[stage], phase, abort_flag, 5)) {
          ok = false;
          break;
        }
        const uint8_t* src = sB8 + stage * C::B8_BYTES;
        uint8_t* dst = sB + stage * C::B_BYTES;
        // BN rows x 64 int8: thread t takes 16-byte chunk c = t & 3 (k = 16c ..
        // 16c + 15) of rows t / 4 + 32 j; all loads first, then the stores
        constexpr int NJ = BN * 4 / 128;
        const int c = t & 3;
        uint4 raw[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j)
          raw[j] = lds128(smem_u32(src + ((t >> 2) + 32 * j) * 64 + c * 16));
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          const int n = (t >> 2) + 32 * j;
          uint4 o0, o1;
          i8x4_to_bf16x4(raw[j].x, o0.x, o0.y);
          i8x4_to_bf16x4(raw[j].y, o0.z, o0.w);
          i8x4_to_bf16x4(raw[j].z, o1.x, o1.y);
          i8x4_to_bf16x4(raw[j].w, o1.z, o1.w);
          sts128(smem_u32(dst + sw128_off(n, 2 * c)), o0);
          sts128(smem_u32(dst + sw128_off(n, 2 * c + 1)), o1);
        }
        fence_proxy_async_smem();
        mbar_arrive(&conv[stage]);
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (C::RMS) {
    // ── RMSNorm of A (RMS_WARPS warps): RMS_SPLIT threads per row of the A
    // tile, each taking 8 / RMS_SPLIT of the row's 16-byte chunks in every
    // stage. A thread scales its values by gamma in place (bf16, the layout
    // the MMA reads) and sums their squares; at the end of the tile's K loop
    // the parts go to the epilogue, which forms 1 / sqrt(sum / K + eps). ──
    constexpr int CPT = 8 / C::RMS_SPLIT;  // chunks per thread per stage
    const int tt = threadIdx.x - 32 * C::NORM_WARP0;
    const int t = tt % BM;         // row
    const int c0 = (tt / BM) * CPT;  // first chunk
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int tile = tile0; tile < num_tiles && ok; tile += tstep) {
      unsigned long long ss = f2pk(0.f, 0.f);
      for (int kb = 0; kb < p.num_k_blocks; ++kb) {
        if (!mbar_wait_park(&full[stage], phase, abort_flag, 13)) {
          ok = false;
          break;
        }
        const uint32_t rowp = smem_u32(sA + stage * C::A_BYTES + t * 128);
        const int k0 = kb * BK;
        uint4 xs[CPT], gs[CPT];
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
          const int c = c0 + i;
          xs[i] = lds128(rowp + ((c ^ (t & 7)) << 4));
          // gamma of these 8 columns (one address for every lane); past K (a
          // multiple of 8) the tile holds zeros and stays zero
          gs[i] = k0 + c * 8 < p.K
                      ? __ldg(reinterpret_cast<const uint4*>(p.rms_gamma + k0 + c * 8))
                      : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
          const int c = c0 + i;
          const uint32_t xw[4] = {xs[i].x, xs[i].y, xs[i].z, xs[i].w};
          const uint32_t gw[4] = {gs[i].x, gs[i].y, gs[i].z, gs[i].w};
          uint32_t yw[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const unsigned long long a = f2pk(bf16_lo(xw[j]), bf16_hi(xw[j]));
            ss = ffma2(a, a, ss);
            float y0, y1;
            f2up(fmul2(a, f2pk(bf16_lo(gw[j]), bf16_hi(gw[j]))), y0, y1);
            yw[j] = cvt_bf16x2(y0, y1);
          }
          sts128(rowp + ((c ^ (t & 7)) << 4), make_uint4(yw[0], yw[1], yw[2], yw[3]));
        }
        fence_proxy_async_smem();
        mbar_arrive(&conv[stage]);
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (!mbar_wait_park(&rempty[acc], acc_phase ^ 1, abort_flag, 14)) break;
      float s0, s1;
      f2up(ss, s0, s1);
      sRstd[(acc * C::RMS_SPLIT + tt / BM) * BM + t] = s0 + s1;
      mbar_arrive(&rfull[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  // PAIR: the even CTA's MMAs (into both CTAs' TMEM, from both CTAs' shared
  // memory) are drained before either CTA frees its columns or exits
  if (PAIR) cl_sync();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  // FUSE_LN: neither CTA leaves while its partner may still write its shared memory
  if (C::LN) cl_sync();
}

template <int BN, int WMODE, int EPI, int FUSE, bool PAIR = false>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ty,
                const CUtensorMap& ty2, const CUtensorMap& tr, const GemmArgs& a, cudaStream_t st) {
  using C = GemmCfg<BN, WMODE, FUSE, EPI, PAIR>;
  static_assert(C::SMEM_BYTES <= 232448, "GEMM smem budget");
  static_assert(!C::LN || C::EPI_COLS % 64 == 0, "FUSE_LN: whole 64-column boxes per warp");
  static_assert(!C::LN || C::EPI_GROUPS == 2 || C::EPI_GROUPS == 4,
                "FUSE_LN: two or four column slices per CTA");
  auto kern = gemm_tc_kernel<BN, WMODE, EPI, FUSE, PAIR>;
  if (!smem_attr_ready(reinterpret_cast<const void*>(kern), C::SMEM_BYTES))
    return record_cuda_error();
  const int tiles = a.num_tiles;
  if (!C::LN && !PAIR) {
    const int grid = tiles < num_sms() ? tiles : num_sms();
    return launch_pdl(kern, dim3(grid), dim3(C::NUM_THREADS), C::SMEM_BYTES, st, ta, tb, ty, ty2,
                      tr, a);
  }
  // clusters of two CTAs, an even grid: FUSE_LN, the two column halves of a
  // row block (one tile each); PAIR, the two row halves of a 256-row tile (one
  // tile per cluster)
  const int sms = num_sms() & ~1;
  const int grid = PAIR ? 2 * (tiles < sms / 2 ? tiles : sms / 2) : (tiles < sms ? tiles : sms);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(C::NUM_THREADS);
  cfg.dynamicSmemBytes = (size_t)C::SMEM_BYTES;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return launch_cfg(cfg, kern, ta, tb, ty, ty2, tr, a);
}

// (dispatch value for a 2-SM pair launch, beside the gemm::Fuse modes)
constexpr int FUSE_PAIR = 100;

template <int BN, int WMODE>
int dispatch_epi(int epi, int fuse, const CUtensorMap& ta, const CUtensorMap& tb,
                 const CUtensorMap& ty0, const CUtensorMap& ty2, const CUtensorMap& tr,
                 const GemmArgs& a, cudaStream_t st) {
  using gemm::FUSE_LN;
  using gemm::FUSE_NONE;
  using gemm::FUSE_RMS;
  // every instantiation takes the second output map; only FUSE_LN writes it
  if (fuse == FUSE_PAIR) {
    if constexpr (BN == 256 && WMODE == W_BF16_NK) {
      if (epi == CK_EPI_STORE) return launch_gemm<BN, WMODE, CK_EPI_STORE, FUSE_NONE, true>(ta, tb, ty0, ty2, tr, a, st);
      if (epi == CK_EPI_GELU) return launch_gemm<BN, WMODE, CK_EPI_GELU, FUSE_NONE, true>(ta, tb, ty0, ty2, tr, a, st);
      if (epi == CK_EPI_RESID) return launch_gemm<BN, WMODE, CK_EPI_RESID, FUSE_NONE, true>(ta, tb, ty0, ty2, tr, a, st);
    }
    return CK_ERR_UNSUPPORTED;
  }
  if (fuse == FUSE_RMS) {
    if (epi == CK_EPI_STORE) return launch_gemm<BN, WMODE, CK_EPI_STORE, FUSE_RMS>(ta, tb, ty0, ty2, tr, a, st);
    if (epi == CK_EPI_BIAS) return launch_gemm<BN, WMODE, CK_EPI_BIAS, FUSE_RMS>(ta, tb, ty0, ty2, tr, a, st);
    return CK_ERR_UNSUPPORTED;
  }
  if (fuse == FUSE_LN) {
    if constexpr (BN == 256) {
      if (epi == CK_EPI_RESID) return launch_gemm<BN, WMODE, CK_EPI_RESID, FUSE_LN>(ta, tb, ty0, ty2, tr, a, st);
    }
    return CK_ERR_UNSUPPORTED;
  }
  switch (epi) {
    case CK_EPI_STORE: return launch_gemm<BN, WMODE, CK_EPI_STORE, FUSE_NONE>(ta, tb, ty0, ty2, tr, a, st);
    case CK_EPI_GELU: return launch_gemm<BN, WMODE, CK_EPI_GELU, FUSE_NONE>(ta, tb, ty0, ty2, tr, a, st);
    case CK_EPI_RESID: return launch_gemm<BN, WMODE, CK_EPI_RESID, FUSE_NONE>(ta, tb, ty0, ty2, tr, a, st);
    case CK_EPI_BIAS: return launch_gemm<BN, WMODE, CK_EPI_BIAS, FUSE_NONE>(ta, tb, ty0, ty2, tr, a, st);
  }
  return CK_ERR_INVALID_ARG;
}

}  // namespace

bool gemm_tc_supported(int64_t M, int64_t K, int64_t lda, int w_dtype, int w_layout, int64_t N,
                       int64_t ldw, const void* A, const void* W, int64_t ldy, const void* Y,
                       int epi, const void* aux, int64_t ld_aux) {
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (M <= 0 || N <= 0 || K <= 0) return false;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return false;
  if (!al16(A) || !al16(W) || !al16(Y)) return false;
  if ((lda * 2) % 16 != 0 || (ldy * 2) % 16 != 0) return false;
  if (w_dtype == CK_I8) {
    if (w_layout != CK_W_NK || ldw % 16 != 0) return false;
  } else if (w_dtype == CK_BF16) {
    if ((ldw * 2) % 16 != 0) return false;
  } else {
    return false;
  }
  if (epi == CK_EPI_RESID || epi == CK_EPI_BIAS) {
    if (!al16(aux)) return false;
    if (epi == CK_EPI_RESID && (ld_aux * 2) % 16 != 0) return false;
  }
  return true;
}

// 2-SM pairs by default for long K, and for K >= 768 on tall A: measured on
// B200 (bf16, 256-wide N tiles) they take 8 % off 16384 x 2048 x 2048, 2 % off
// 8192 x 2048 x 1024, and 4-7 % off the Cortex-M forward from 16384 rows up
// (K = 768 and 3072; at 8192 rows they cost 0.6 %), but nothing off K = 512
// shapes (the Cortex-S forwards at 8192 and 65536 rows), where the weight
// prefetch and the split last round are the better tools. CK_GEMM_PAIR=1 / 0
// forces them on / off.
bool gemm_pair_enabled(int64_t M, int64_t K) {
  const char* v = std::getenv("CK_GEMM_PAIR");
  if (v != nullptr) return std::strcmp(v, "0") != 0;
  return K >= 2048 || (K >= 768 && M >= 16384);
}

bool gemm_split_enabled() {
  const char* v = std::getenv("CK_GEMM_SPLIT");
  return v == nullptr || std::strcmp(v, "0") != 0;
}

int gemm_tc_block_n(int64_t N) { return (N % 256 == 0 || N > 256) ? 256 : 128; }

int gemm_tc(const void* A, int64_t M, int64_t K, int64_t lda, const void* W, int w_dtype,
            int w_layout, int64_t N, int64_t ldw, const float* w_scale, int epi, const void* aux,
            int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy, cudaStream_t st,
            const GemmFusion* fz) {
  const int BN = gemm_tc_block_n(N);
  GemmArgs a;
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.num_m_tiles = (int)((M + BM - 1) / BM);
  a.num_n_tiles = (int)((N + BN - 1) / BN);
  a.num_k_blocks = (int)((K + BK - 1) / BK);
  a.num_tiles = a.num_m_tiles * a.num_n_tiles;
  a.split_from = a.num_tiles;
  a.aux = reinterpret_cast<const __nv_bfloat16*>(aux);
  a.ld_aux = ld_aux;
  a.aux_row_mod = aux_row_mod;
  a.w_scale = (w_dtype == CK_I8) ? w_scale : nullptr;
  if (w_dtype == CK_I8 && w_scale == nullptr) return CK_ERR_INVALID_ARG;
  a.scale_vec = (reinterpret_cast<uintptr_t>(w_scale) & 15u) == 0;
  a.norm_eps = 0.f;
  a.rms_gamma = nullptr;
  a.ln_gamma = nullptr;
  a.ln_beta = nullptr;
  a.res_tma = 0;
  a.pre_b = (fz != nullptr && fz->w_static) ? 1 : 0;
  int fuse = gemm::FUSE_NONE;
  if (fz != nullptr && fz->ln_out != nullptr) {
    // LayerNorm of the residual output as a second output: whole rows of
    // N = 2 * 256 columns, one row block per cluster of two CTAs
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    if (epi != CK_EPI_RESID || BN != 256 || N != 2 * BN || fz->ln_gamma == nullptr ||
        (aux_row_mod > 0 && aux_row_mod % 32 != 0) ||  // residual boxes of 32 rows
        !al16(fz->ln_gamma) || (fz->ln_beta != nullptr && !al16(fz->ln_beta)) ||
        !al16(fz->ln_out) || (fz->ln_ld * 2) % 16 != 0)
      return CK_ERR_UNSUPPORTED;
    a.ln_gamma = reinterpret_cast<const __nv_bfloat16*>(fz->ln_gamma);

    a.ln_beta = reinterpret_cast<const __nv_bfloat16*>(fz->ln_beta);
    a.norm_eps = fz->eps;
    fuse = gemm::FUSE_LN;
  } else if (fz != nullptr && fz->rms_gamma != nullptr) {
    // RMSNorm of A in the GEMM: gamma read 16 bytes at a time
    if (K % 8 != 0 || (reinterpret_cast<uintptr_t>(fz->rms_gamma) & 15u) != 0 ||
        (epi != CK_EPI_STORE && epi != CK_EPI_BIAS))
      return CK_ERR_UNSUPPORTED;
    a.rms_gamma = reinterpret_cast<const __nv_bfloat16*>(fz->rms_gamma);
    a.norm_eps = fz->eps;
    fuse = gemm::FUSE_RMS;
  }

  // 2-SM pairs (256-row tiles, B split over the pair): bf16 (N, K) weights, a
  // store, GELU or residual epilogue, no fusion, 256-wide N tiles (see
  // gemm_pair_enabled for the shapes). The schedule then walks 256-row tiles.
  bool pair = false;
  if (fuse == gemm::FUSE_NONE && w_dtype == CK_BF16 && w_layout == CK_W_NK && BN == 256 &&
      (epi == CK_EPI_STORE || epi == CK_EPI_GELU || epi == CK_EPI_RESID) && a.num_m_tiles >= 2 &&
      gemm_pair_enabled(M, K)) {
    pair = true;
    a.num_m_tiles = (a.num_m_tiles + 1) / 2;
    a.num_tiles = a.num_m_tiles * a.num_n_tiles;
    a.split_from = a.num_tiles;
  }
  // Split the last round's tiles in two when that keeps the round to one wave
  // (bf16 (N, K) weights without epilogue fusions; CK_GEMM_SPLIT=0 disables).
  if (!pair && fuse == gemm::FUSE_NONE && w_dtype == CK_BF16 && w_layout == CK_W_NK &&
      BN == 256 && (int64_t)a.num_n_tiles * BN == N && gemm_split_enabled()) {
    const int sms = num_sms();
    const int rem = a.num_tiles > sms ? a.num_tiles % sms : 0;
    if (rem > 0 && 2 * rem <= sms) {
      a.split_from = a.num_tiles - rem;
      a.num_tiles += rem;
    }
  }
  CUtensorMap ta, tb, ty, ty2, tr;
  if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, lda, BK, BM, 128))
    return CK_ERR_INVALID_ARG;
  // output boxes: 32 x 32 (64B swizzle); FUSE_LN 64 x 32 (128B swizzle)
  const bool ln = fuse == gemm::FUSE_LN;
  if (!make_tmap_2d(&ty, Y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, ldy, ln ? 64 : 32, 32,
                    ln ? 128 : 64))
    return CK_ERR_INVALID_ARG;
  if (ln) {
    if (!make_tmap_2d(&ty2, fz->ln_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, fz->ln_ld, 64,
                      32, 128))
      return CK_ERR_INVALID_ARG;
  } else {
    ty2 = ty;
  }
  // FUSE_LN residual tiles by TMA: 32-row boxes (a broadcast period is a
  // multiple of 32, checked above)
  a.res_tma = fuse == gemm::FUSE_LN;
  if (a.res_tma) {
    if (!make_tmap_2d(&tr, aux, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N,
                      aux_row_mod > 0 ? (uint64_t)aux_row_mod : (uint64_t)M, ld_aux, 64, 32, 128))
      return CK_ERR_INVALID_ARG;
  } else {
    tr = ty;
  }
  bool ok;
  if (w_dtype == CK_I8) {
    ok = make_tmap_2d(&tb, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, ldw, BK, BN, 0);
  } else if (w_layout == CK_W_NK) {
    ok = make_tmap_2d(&tb, W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, ldw, BK,
                      pair ? BN / 2 : BN, 128);
  } else {
    ok = make_tmap_2d(&tb, W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, ldw, 64, BK, 128);
  }
  if (!ok) return CK_ERR_INVALID_ARG;

  if (pair) return dispatch_epi<256, W_BF16_NK>(epi, FUSE_PAIR, ta, tb, ty, ty2, tr, a, st);
  if (BN == 256) {
    if (w_dtype == CK_I8) return dispatch_epi<256, W_I8_NK>(epi, fuse, ta, tb, ty, ty2, tr, a, st);
    if (w_layout == CK_W_NK) return dispatch_epi<256, W_BF16_NK>(epi, fuse, ta, tb, ty, ty2, tr, a, st);
    return dispatch_epi<256, W_BF16_KN>(epi, fuse, ta, tb, ty, ty2, tr, a, st);
  }
  if (w_dtype == CK_I8) return dispatch_epi<128, W_I8_NK>(epi, fuse, ta, tb, ty, ty2, tr, a, st);
  if (w_layout == CK_W_NK) return dispatch_epi<128, W_BF16_NK>(epi, fuse, ta, tb, ty, ty2, tr, a, st);
  return dispatch_epi<128, W_BF16_KN>(epi, fuse, ta, tb, ty, ty2, tr, a, st);
}

}  // namespace ck
