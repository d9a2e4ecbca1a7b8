// Fused spike tokenizer (cortex/kernels/tokenizer.py:68-81 and :177-249;
// cortex/models/tokenizer.py:90-93):
//
//   out[dest[e], :] = n_emb[nid[e], :] + t_emb[tb[e], :] + v_emb[val[e], :]
//
// evaluated left to right in the table dtype, so bf16 tables give
// bf16(bf16(n + t) + v) exactly as torch eager does. A group of lanes per
// event (16 for D = 512 bf16, two events per warp); each lane moves 16-byte
// vectors of the three rows (4 vectors per lane per table at D = 512). With gamma != NULL the finished row is LayerNorm-ed in
// registers before the store, which fuses CrossAttentionBlock.norm_kv
// (cortex/models/perceiver.py:68) into the gather: the raw tokens never reach HBM.
// Out-of-range indices set CK_ERR_INDEX and write a zero row. With n_valid set
// (device count, padded batches) events n_valid..E-1 are padding: their ids
// are not read and their rows are written as zeros, which keeps every row a
// later kernel may touch finite.
//
// tokenize_packed also does _pack_events' index work (cortex/models/cortex.py:
// 125-165) for the forward: with the batch indices sorted, the packed row of
// event e is e and window b starts at its first event, so each event's group
// writes the offsets of the windows that begin at it and its token to row e,
// and each block records whether it saw an index out of order or out of
// [0, B). tok_fixup_kernel, launched after it, reads those flags and, only
// when one is set, redoes the packing as a stable counting sort and tokenizes
// every event again into its packed row.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

// bf16x2 add, round to nearest even (sm_90+)
__device__ __forceinline__ uint32_t badd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ int64_t load_idx(const void* p, int dt, int64_t i, int64_t stride) {
  if (dt == CK_I64) return reinterpret_cast<const int64_t*>(p)[i * stride];
  return (int64_t) reinterpret_cast<const int32_t*>(p)[i * stride];
}

template <typename T>
struct Vec;
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float* f) {
    unpack8(*reinterpret_cast<const uint4*>(p), f);
  }
  __device__ static void store(__nv_bfloat16* p, const float* f) {
    *reinterpret_cast<uint4*>(p) = pack8(f);
  }
  __device__ static float round(float x) { return rbf(x); }
};
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float* f) {
    float4 v = *reinterpret_cast<const float4*>(p);
    f[0] = v.x;
    f[1] = v.y;
    f[2] = v.z;
    f[3] = v.w;
  }
  __device__ static void store(float* p, const float* f) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
  __device__ static float round(float x) { return x; }
};

struct TokArgs {
  const void *n_emb, *t_emb, *v_emb;
  int64_t n_vocab, t_vocab, v_vocab, n_ld, t_ld, v_ld;
  const void *nid, *tb, *val;
  int idx_dt;
  int64_t s_nid, s_tb, s_val, E;
  const int32_t* dest;
  const void *gamma, *beta;
  float eps;
  void* out;
  int64_t out_ld;
  int D;
  const int32_t* n_valid;
  // Packing inside the tokenizer (tokenize_packed): the batch index of every
  // event. Tokens go to row e (the packed row of sorted input), the window
  // offsets come from the batch boundaries, and slots[block] records whether
  // the block saw an event out of batch order or out of [0, B).
  const void* bidx;
  int64_t s_bidx;
  int32_t B;
  int32_t* offsets;
  int32_t* slots;
};

// G lanes share one event row (G in {8, 16, 32}, so a warp handles 32 / G
// events at once); each lane holds MAXV vectors of VEC elements. Index loads,
// the three table gathers and the output store of the 32 / G rows are all
// independent, so a warp keeps 3 * MAXV * (32 / G) 16-byte loads in flight.
// One event row for the G lanes of a group: the three table rows summed, the
// optional LayerNorm, the store to row dst_row (all 32 lanes of the warp call
// it together: the row reductions shuffle across the whole warp).
// tokenize_packed limits: the fix-up kernel keeps two B-sized histograms and
// the destinations of E / kFixupCtas events in shared memory.
constexpr int64_t kFixupCtas = 128;
constexpr int kFixupMaxSmem =
    (int)((2 * kTokPackMaxB + (kTokPackMaxE + kFixupCtas - 1) / kFixupCtas) * 4);

template <typename T, int VEC, int MAXV, bool LN, int G>
__device__ __forceinline__ void tok_event(const TokArgs& a, int64_t e, int64_t dst_row, bool live,
                                          bool real, int sub) {
  constexpr bool kPair = std::is_same<T, __nv_bfloat16>::value && VEC == 8;
  const T* ne = reinterpret_cast<const T*>(a.n_emb);
  const T* te = reinterpret_cast<const T*>(a.t_emb);
  const T* ve = reinterpret_cast<const T*>(a.v_emb);
  T* out = reinterpret_cast<T*>(a.out);
  const int nvec = a.D / VEC;
  {
    int64_t n = 0, t = 0, v = 0;
    if (real) {
      n = load_idx(a.nid, a.idx_dt, e, a.s_nid);
      t = load_idx(a.tb, a.idx_dt, e, a.s_tb);
      v = load_idx(a.val, a.idx_dt, e, a.s_val);
    }
    const bool in_range =
        n >= 0 && n < a.n_vocab && t >= 0 && t < a.t_vocab && v >= 0 && v < a.v_vocab;
    const bool store = live && dst_row >= 0;
    const bool ok = store && real && in_range;
    if (store && real && !in_range && sub == 0)
      set_status(CK_ERR_INDEX, (int)e,
                 (int)(n < 0 || n >= a.n_vocab ? n : (t < 0 || t >= a.t_vocab ? t : v)));
    float x[MAXV][VEC];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = sub + G * i;
#pragma unroll
      for (int k = 0; k < VEC; ++k) x[i][k] = 0.f;
      if (ok && c < nvec) {
        if constexpr (kPair) {
          // bf16(bf16(n + t) + v) on the bf16x2 adder: a correctly rounded bf16
          // sum equals torch's fp32 add then bf16 round (fp32's 24 bits are at
          // least 2 * 8 + 2, so the double rounding is innocuous)
          const uint4 rn = *reinterpret_cast<const uint4*>(ne + n * a.n_ld + c * VEC);
          const uint4 rt = *reinterpret_cast<const uint4*>(te + t * a.t_ld + c * VEC);
          const uint4 rv = *reinterpret_cast<const uint4*>(ve + v * a.v_ld + c * VEC);
          uint4 r;
          r.x = badd2(badd2(rn.x, rt.x), rv.x);
          r.y = badd2(badd2(rn.y, rt.y), rv.y);
          r.z = badd2(badd2(rn.z, rt.z), rv.z);
          r.w = badd2(badd2(rn.w, rt.w), rv.w);
          unpack8(r, x[i]);
        } else {
          float fn[VEC], ft[VEC], fv[VEC];
          if constexpr (VEC == 1) {
            fn[0] = (float)ne[n * a.n_ld + c];
            ft[0] = (float)te[t * a.t_ld + c];
            fv[0] = (float)ve[v * a.v_ld + c];
          } else {
            Vec<T>::load(ne + n * a.n_ld + c * VEC, fn);
            Vec<T>::load(te + t * a.t_ld + c * VEC, ft);
            Vec<T>::load(ve + v * a.v_ld + c * VEC, fv);
          }
#pragma unroll
          for (int k = 0; k < VEC; ++k)
            x[i][k] = Vec<T>::round(Vec<T>::round(fn[k] + ft[k]) + fv[k]);
        }
      }
    }
    if (LN) {
      // Two-pass mean / biased variance over the G lanes of the row (all 32
      // lanes take part in the shuffles; rows that are not stored discard it).
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < MAXV; ++i)
#pragma unroll
        for (int k = 0; k < VEC; ++k) s += x[i][k];
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const float mean = s / (float)a.D;
      float q = 0.f;
      const unsigned long long nmean2 = f2pk(-mean, -mean);
      if constexpr (kPair) {  // even and odd columns on the paired fp32 pipe
        unsigned long long q2 = f2pk(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < MAXV; ++i)
          if (sub + G * i < nvec)
#pragma unroll
            for (int k = 0; k < VEC; k += 2) {
              const unsigned long long d = fadd2(f2pk(x[i][k], x[i][k + 1]), nmean2);
              q2 = ffma2(d, d, q2);
            }
        float q0, q1;
        f2up(q2, q0, q1);
        q = q0 + q1;
      } else {
#pragma unroll
        for (int i = 0; i < MAXV; ++i)
          if (sub + G * i < nvec)
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
              const float d = x[i][k] - mean;
              q += d * d;
            }
      }
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
      const float rstd = 1.0f / sqrtf(q / (float)a.D + a.eps);
      if (ok) {
        const T* g = reinterpret_cast<const T*>(a.gamma);
        const T* bt = reinterpret_cast<const T*>(a.beta);
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
          const int c = sub + G * i;
          if (c < nvec && kPair) {
            // ((x - mean) * rstd) * gamma + beta, two columns per instruction
            // (the same operations and order as the scalar form below)
            const uint4 gw = *reinterpret_cast<const uint4*>(g + c * VEC);
            const uint4 bw = bt ? *reinterpret_cast<const uint4*>(bt + c * VEC)
                                : make_uint4(0u, 0u, 0u, 0u);
            const uint32_t gv[4] = {gw.x, gw.y, gw.z, gw.w};
            const uint32_t bv[4] = {bw.x, bw.y, bw.z, bw.w};
            const unsigned long long rstd2 = f2pk(rstd, rstd);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              unsigned long long y = fadd2(f2pk(x[i][2 * k], x[i][2 * k + 1]), nmean2);
              y = fmul2(y, rstd2);
              y = ffma2(y, f2pk(bf16_lo(gv[k]), bf16_hi(gv[k])),
                        f2pk(bf16_lo(bv[k]), bf16_hi(bv[k])));
              f2up(y, x[i][2 * k], x[i][2 * k + 1]);
            }
          } else if (c < nvec) {
            float gk[VEC], bk[VEC];
            if constexpr (VEC == 1) {
              gk[0] = (float)g[c];
              bk[0] = bt ? (float)bt[c] : 0.f;
            } else {
              Vec<T>::load(g + c * VEC, gk);
              if (bt) {
                Vec<T>::load(bt + c * VEC, bk);
              } else {
#pragma unroll
                for (int k = 0; k < VEC; ++k) bk[k] = 0.f;
              }
            }
#pragma unroll
            for (int k = 0; k < VEC; ++k) x[i][k] = (x[i][k] - mean) * rstd * gk[k] + bk[k];
          }
        }
      }
    }
    if (store) {
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int c = sub + G * i;
        if (c < nvec) {
          if constexpr (VEC == 1) {
            out[dst_row * a.out_ld + c] = (T)x[i][0];
          } else {
            Vec<T>::store(out + dst_row * a.out_ld + c * VEC, x[i]);
          }
        }
      }
    }
  }
}

template <typename T, int VEC, int MAXV, bool LN, int G>
__global__ void __launch_bounds__(256, MAXV <= 4 ? 3 : 1) tokenize_kernel(const TokArgs a) {
  grid_dep_wait();
  grid_dep_launch();
  constexpr int RPW = 32 / G;
  const int lane = threadIdx.x & 31;
  const int sub = lane % G;
  const int slot = lane / G;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t nv = a.n_valid ? min((int64_t)max(*a.n_valid, 0), a.E) : a.E;
  int viol = 0;
  if (a.bidx != nullptr && nv == 0 && blockIdx.x == 0)
    for (int64_t bb = threadIdx.x; bb <= a.B; bb += blockDim.x) a.offsets[bb] = 0;
  for (int64_t base = warp * RPW; base < a.E; base += nwarps * RPW) {
    const int64_t e = base + slot;
    const bool live = e < a.E;
    const bool real = e < nv;
    int64_t dst_row = -1;
    if (live) dst_row = a.dest ? (int64_t)a.dest[e] : e;
    if (a.bidx != nullptr && real && sub == 0) {
      // sorted input: the window offsets are the batch boundaries
      const int64_t b = load_idx(a.bidx, a.idx_dt, e, a.s_bidx);
      const int64_t bp = e > 0 ? load_idx(a.bidx, a.idx_dt, e - 1, a.s_bidx) : -1;
      if (b < 0 || b >= a.B || bp > b) {
        viol = 1;
      } else {
        for (int64_t bb = max(bp + 1, (int64_t)0); bb <= b; ++bb) a.offsets[bb] = (int32_t)e;
        if (e == nv - 1)
          for (int64_t bb = b + 1; bb <= a.B; ++bb) a.offsets[bb] = (int32_t)nv;
      }
    }
    tok_event<T, VEC, MAXV, LN, G>(a, e, dst_row, live, real, sub);
  }
  if (a.slots != nullptr) {
    const int any = __syncthreads_or(viol);
    if (threadIdx.x == 0) a.slots[blockIdx.x] = any;
  }
}

// Exclusive scan of v[0..n) in place by one CTA of 256 threads (each a
// contiguous run); returns the total to every thread.
__device__ int32_t block_scan_runs(int32_t* v, int64_t n) {
  __shared__ int32_t wtot[8];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int64_t per = (n + 255) / 256;
  const int64_t lo = min(n, t * per), hi = min(n, lo + per);
  int32_t sum = 0;
  for (int64_t i = lo; i < hi; ++i) sum += v[i];
  int32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) wtot[w] = incl;
  __syncthreads();
  int32_t before = 0, total = 0;
  for (int k = 0; k < 8; ++k) {
    if (k < w) before += wtot[k];
    total += wtot[k];
  }
  int32_t run = before + incl - sum;
  for (int64_t i = lo; i < hi; ++i) {
    const int32_t c = v[i];
    v[i] = run;
    run += c;
  }
  __syncthreads();
  return total;
}

// The general packing for tokenize_packed, one launch after the tokenizer:
// nothing to do unless a tokenizer block saw an event out of batch order or
// out of [0, B). Otherwise every CTA counts the events of each window over
// the whole batch and before its own segment of `chunk` events (dynamic
// shared memory: two B-sized histograms and the segment's destinations),
// rebuilds the window offsets (CTA 0 stores them), gives each event of its
// segment its packed row (offset + rank among earlier events of its window,
// the stable order of _pack_events) and tokenizes it into that row again.
template <typename T, int VEC, int MAXV, bool LN, int G>
__global__ void __launch_bounds__(256) tok_fixup_kernel(const TokArgs a, const int32_t n_slots,
                                                        const int64_t chunk) {
  grid_dep_wait();
  grid_dep_launch();
  int viol = 0;
  for (int i = threadIdx.x; i < n_slots; i += blockDim.x) viol |= a.slots[i];
  if (!__syncthreads_or(viol)) return;
  extern __shared__ int32_t fx[];
  int32_t* hist = fx;           // [B] events per window, then the window offsets
  int32_t* cur = fx + a.B;      // [B] events before this segment, then the row cursor
  int32_t* dst = fx + 2 * a.B;  // [chunk] packed rows of the segment's events
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t nv = a.n_valid ? min((int64_t)max(*a.n_valid, 0), a.E) : a.E;
  const int64_t s0 = blockIdx.x * chunk, s1 = min(s0 + chunk, a.E);
  for (int64_t i = tid; i < a.B; i += blockDim.x) hist[i] = cur[i] = 0;
  __syncthreads();
  for (int64_t e = tid; e < nv; e += blockDim.x) {
    const int64_t b = load_idx(a.bidx, a.idx_dt, e, a.s_bidx);
    if (b >= 0 && b < a.B) {
      atomicAdd(&hist[b], 1);
      if (e < s0) atomicAdd(&cur[b], 1);
    }
  }
  __syncthreads();
  const int32_t total = block_scan_runs(hist, a.B);
  if (blockIdx.x == 0) {
    for (int64_t i = tid; i < a.B; i += blockDim.x) a.offsets[i] = hist[i];
    if (tid == 0) a.offsets[a.B] = total;
  }
  for (int64_t i = tid; i < a.B; i += blockDim.x) cur[i] += hist[i];
  __syncthreads();
  if (wid == 0) {  // in event order, 32 at a time
    for (int64_t base = s0; base < s1; base += 32) {
      const int64_t e = base + lane;
      const bool in = e < s1;
      int64_t b = -1;  // padding or past the segment
      if (in && e < nv) {
        b = load_idx(a.bidx, a.idx_dt, e, a.s_bidx);
        if (b < 0 || b >= a.B) {
          set_status(CK_ERR_INDEX, (int)e, (int)b);
          b = -2;  // dropped, as _pack_events' index check would reject it
        }
      }
      const unsigned peers = __match_any_sync(0xffffffffu, (long long)b);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      int32_t d = (in && e >= nv) ? (int32_t)e : -1;  // padding keeps its own (zero) row
      if (b >= 0) d = cur[b] + rank;
      __syncwarp();
      if (b >= 0 && rank == 0) cur[b] += __popc(peers);
      __syncwarp();
      if (in) dst[e - s0] = d;
    }
  }
  __syncthreads();
  constexpr int RPW = 32 / G;
  const int sub = lane % G, slot = lane / G;
  for (int64_t base = s0 + wid * RPW; base < s1; base += (blockDim.x / 32) * RPW) {
    const int64_t e = base + slot;
    const bool live = e < s1;
    tok_event<T, VEC, MAXV, LN, G>(a, e, live ? (int64_t)dst[e - s0] : -1, live, live && e < nv,
                                   sub);
  }
}

template <typename T, int VEC, int MAXV, bool LN, int G>
int launch_tok(const TokArgs& a, cudaStream_t st) {
  constexpr int rows_per_block = 8 * (32 / G);
  int64_t blocks = (a.E + rows_per_block - 1) / rows_per_block;
  const int64_t cap = 16 * (int64_t)num_sms();
  if (blocks > cap) blocks = cap;
  const int rc = launch_pdl(tokenize_kernel<T, VEC, MAXV, LN, G>, dim3((unsigned)blocks),
                            dim3(256), 0, st, a);
  if (rc != CK_OK || a.bidx == nullptr) return rc;
  // the general packing, for input that turns out not to be sorted
  int64_t chunk = (a.E + kFixupCtas - 1) / kFixupCtas;
  if (chunk < 1024) chunk = 1024;
  chunk = (chunk + 31) & ~int64_t(31);
  const int64_t fblocks = (a.E + chunk - 1) / chunk;
  const size_t smem = (size_t)(2 * (int64_t)a.B + chunk) * 4;
  auto fk = tok_fixup_kernel<T, VEC, MAXV, LN, G>;
  if (smem > (size_t)kFixupMaxSmem) return CK_ERR_INVALID_ARG;
  if (!smem_attr_ready(reinterpret_cast<const void*>(fk), kFixupMaxSmem))
    return record_cuda_error();
  return launch_pdl(fk, dim3((unsigned)fblocks), dim3(256), smem, st, a, (int32_t)blocks, chunk);
}

template <typename T, int VEC, int MAXV, int G>
int launch_tok_ln(const TokArgs& a, cudaStream_t st) {
  return a.gamma != nullptr ? launch_tok<T, VEC, MAXV, true, G>(a, st)
                            : launch_tok<T, VEC, MAXV, false, G>(a, st);
}

template <typename T>
int dispatch_tok(const TokArgs& a, bool vec_ok, cudaStream_t st) {
  constexpr int V = Vec<T>::N;
  if (vec_ok) {
    const int nvec = a.D / V;
    if (nvec <= 32) return launch_tok_ln<T, V, 4, 8>(a, st);
    if (nvec <= 64) return launch_tok_ln<T, V, 4, 16>(a, st);
    if (nvec <= 128) return launch_tok_ln<T, V, 4, 32>(a, st);
    if (nvec <= 256) return launch_tok_ln<T, V, 8, 32>(a, st);
    return CK_ERR_UNSUPPORTED;
  }
  if (a.D <= 256) return launch_tok_ln<T, 1, 8, 32>(a, st);
  if (a.D <= 1024) return launch_tok_ln<T, 1, 32, 32>(a, st);
  return CK_ERR_UNSUPPORTED;
}

}  // namespace

int tokenize(const void* n_emb, const void* t_emb, const void* v_emb, int dtype, int32_t D,
             int64_t n_vocab, int64_t t_vocab, int64_t v_vocab, int64_t n_ld, int64_t t_ld,
             int64_t v_ld, const void* nid, const void* tb, const void* val, int idx_dtype,
             int64_t s_nid, int64_t s_tb, int64_t s_val, int64_t E, const int32_t* dest,
             const void* gamma, const void* beta, float eps, void* out, int64_t out_ld,
             cudaStream_t st, const int32_t* n_valid) {
  if (E == 0) return CK_OK;
  if (E < 0 || D <= 0 || !n_emb || !t_emb || !v_emb || !nid || !tb || !val || !out)
    return CK_ERR_INVALID_ARG;
  if (idx_dtype != CK_I64 && idx_dtype != CK_I32) return CK_ERR_UNSUPPORTED;
  TokArgs a{n_emb, t_emb, v_emb, n_vocab, t_vocab, v_vocab, n_ld, t_ld, v_ld, nid, tb, val,
            idx_dtype, s_nid, s_tb, s_val, E, dest, gamma, beta, eps, out, out_ld, D, n_valid};
  const int es = dtype == CK_F32 ? 4 : 2;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec_ok = ((int64_t)D * es) % 16 == 0 && (n_ld * es) % 16 == 0 &&
                      (t_ld * es) % 16 == 0 && (v_ld * es) % 16 == 0 && (out_ld * es) % 16 == 0 &&
                      al16(n_emb) && al16(t_emb) && al16(v_emb) && al16(out) &&
                      (gamma == nullptr || al16(gamma)) && (beta == nullptr || al16(beta));
  if (dtype == CK_BF16) return dispatch_tok<__nv_bfloat16>(a, vec_ok, st);
  if (dtype == CK_F32) return dispatch_tok<float>(a, vec_ok, st);
  return CK_ERR_UNSUPPORTED;
}

size_t tokenize_packed_slots() { return (size_t)16 * num_sms(); }

int tokenize_packed(const void* n_emb, const void* t_emb, const void* v_emb, int dtype, int32_t D,
                    int64_t n_vocab, int64_t t_vocab, int64_t v_vocab, const void* nid,
                    const void* tb, const void* val, const void* bidx, int idx_dtype, int64_t E,
                    int32_t B, const void* gamma, const void* beta, float eps, void* out,
                    int64_t out_ld, int32_t* offsets, int32_t* slots, cudaStream_t st,
                    const int32_t* n_valid) {
  if (E <= 0 || E > kTokPackMaxE || B <= 0 || B > kTokPackMaxB || bidx == nullptr ||
      offsets == nullptr || slots == nullptr)
    return CK_ERR_INVALID_ARG;
  if (idx_dtype != CK_I64 && idx_dtype != CK_I32) return CK_ERR_UNSUPPORTED;
  if (!n_emb || !t_emb || !v_emb || !nid || !tb || !val || !out) return CK_ERR_INVALID_ARG;
  TokArgs a{n_emb, t_emb, v_emb, n_vocab, t_vocab, v_vocab, D, D, D, nid, tb, val, idx_dtype,
            1, 1, 1, E, nullptr, gamma, beta, eps, out, out_ld, D, n_valid,
            bidx, 1, B, offsets, slots};
  const int es = dtype == CK_F32 ? 4 : 2;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec_ok = ((int64_t)D * es) % 16 == 0 && (out_ld * es) % 16 == 0 && al16(n_emb) &&
                      al16(t_emb) && al16(v_emb) && al16(out) &&
                      (gamma == nullptr || al16(gamma)) && (beta == nullptr || al16(beta));
  if (dtype == CK_BF16) return dispatch_tok<__nv_bfloat16>(a, vec_ok, st);
  if (dtype == CK_F32) return dispatch_tok<float>(a, vec_ok, st);
  return CK_ERR_UNSUPPORTED;
}

}  // namespace ck
