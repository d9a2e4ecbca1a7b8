// Event packing: the index half of _pack_events (cortex/models/cortex.py:125-165).
//
// Output for a flat event list with batch indices b[e] in [0, B):
//   counts[b]     bincount (:141)
//   offsets[b]    exclusive prefix sum, offsets[B] = number of valid events (:155-160)
//   e_max         max(counts) (:142)
//   dest[e]       packed row of event e = offsets[b] + pos_within, where pos_within
//                 is e's rank among earlier events of the same batch (the stable
//                 argsort of :149 followed by :161)
//
// Device pipeline, no host synchronisation:
//   0. zero     counts, flags and the rank matrix (one kernel, not memsets)
//   1. count    warp-aggregated histogram (match_any) + sortedness flag
//   2. scan     one CTA: exclusive scan of counts, e_max
//   3. rank     (unsorted input only) per 256-event chunk: rank within the chunk
//               and per-(batch, chunk) counts
//   4. colscan  (unsorted input only) per batch: exclusive scan over chunks
//   5. dest     dest[e] = e for sorted input, else offsets + chunk prefix + rank
// Sorted input -- what collate_events produces (cortex/data/nlb.py:492-512) --
// skips steps 3-4 on the device (they exit on the flag).
//
// Padded batches: with n_valid != NULL only events 0..*n_valid-1 are real (the
// count is read on the device, so one captured launch sequence serves every
// batch of a capacity bucket). Padding events are not counted, and dest[e] = e
// for them, which is a row no real event occupies.
#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

constexpr int CHUNK = 256;
// The unsorted path keeps a (B x chunks) int32 matrix; larger problems are
// rejected for unsorted input (CK_ERR_UNSUPPORTED) instead of allocating more.
constexpr int64_t MAX_RANK_MATRIX = 16ll << 20;

__device__ __forceinline__ int64_t load_idx(const void* p, int dt, int64_t i, int64_t stride) {
  if (dt == CK_I64) return reinterpret_cast<const int64_t*>(p)[i * stride];
  return (int64_t) reinterpret_cast<const int32_t*>(p)[i * stride];
}

// Number of real events: *n_valid clamped to [0, E], or E without a count.
__device__ __forceinline__ int64_t real_events(const int32_t* n_valid, int64_t E) {
  if (n_valid == nullptr) return E;
  const int64_t nv = *n_valid;
  return nv < 0 ? 0 : (nv > E ? E : nv);
}

struct PackWs {
  int32_t* flag;    // [0] unsorted, [1] matrix-too-small
  int32_t* matrix;  // B x nchunks (only when it fits)
  int32_t* rank;    // E
  int64_t nchunks;
  bool has_matrix;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

PackWs carve(void* ws, int64_t E, int32_t B) {
  PackWs w;
  uint8_t* p = reinterpret_cast<uint8_t*>(ws);
  w.nchunks = (E + CHUNK - 1) / CHUNK;
  w.has_matrix = (int64_t)B * w.nchunks <= MAX_RANK_MATRIX;
  w.flag = reinterpret_cast<int32_t*>(p);
  p += 256;
  w.rank = reinterpret_cast<int32_t*>(p);
  p += align256((size_t)E * 4);
  w.matrix = reinterpret_cast<int32_t*>(p);
  return w;
}

// The counts, the flags and the rank matrix start at zero: one launch in
// the stream's programmatic chain instead of three memsets.
__global__ void pack_zero_kernel(int32_t* counts, int32_t B, int32_t* flag, int32_t* matrix,
                                 int64_t matrix_words) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = i0; i < B; i += step) counts[i] = 0;
  if (i0 < 64) flag[i0] = 0;
  for (int64_t i = i0; i < matrix_words; i += step) matrix[i] = 0;
}

__global__ void pack_count_kernel(const void* bidx, int dt, int64_t stride, int64_t E, int32_t B,
                                  const int32_t* n_valid, int32_t* counts, int32_t* flag) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t nv = real_events(n_valid, E);
  if (n_valid != nullptr && blockIdx.x == 0 && threadIdx.x == 0 && (*n_valid < 0 || *n_valid > E))
    set_status(CK_ERR_INVALID_ARG, *n_valid, (int)E);
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e - lane < E;
       e += (int64_t)gridDim.x * blockDim.x) {
    const bool in = e < nv;
    int64_t b = in ? load_idx(bidx, dt, e, stride) : -1;
    if (in && (b < 0 || b >= B)) {
      set_status(CK_ERR_INDEX, (int)e, (int)b);
      b = -1;
    }
    if (in && e > 0) {
      int64_t prev = load_idx(bidx, dt, e - 1, stride);
      if (prev > b && b >= 0) atomicOr(&flag[0], 1);
    }
    const unsigned active = __activemask();
    const unsigned peers = __match_any_sync(active, (long long)b);
    const int leader = __ffs(peers) - 1;
    if (b >= 0 && lane == leader) atomicAdd(&counts[b], __popc(peers));
  }
}

__global__ void pack_scan_kernel(const int32_t* counts, int32_t B, int32_t* offsets,
                                 int32_t* e_max) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t warp_max[32];
  const int t = threadIdx.x;
  const int nt = blockDim.x;  // 1024
  const int64_t per = (B + nt - 1) / nt;
  const int64_t lo = t * per;
  const int64_t hi = min((int64_t)B, lo + per);
  int32_t sum = 0, mx = 0;
  for (int64_t i = lo; i < hi; ++i) {
    sum += counts[i];
    mx = max(mx, counts[i]);
  }
  // block exclusive scan of per-thread sums
  const int lane = t & 31, w = t >> 5;
  int32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int32_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  int32_t wm = mx;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wm = max(wm, __shfl_xor_sync(0xffffffffu, wm, o));
  if (lane == 31) warp_tot[w] = incl;
  if (lane == 0) warp_max[w] = wm;
  __syncthreads();
  if (w == 0) {
    int32_t v = (lane < nt / 32) ? warp_tot[lane] : 0;
    int32_t m = (lane < nt / 32) ? warp_max[lane] : 0;
    int32_t vi = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int32_t u = __shfl_up_sync(0xffffffffu, vi, o);
      if (lane >= o) vi += u;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    warp_tot[lane] = vi - v;  // exclusive warp prefix
    if (lane == 0) *e_max = m;
    if (lane == 31) offsets[B] = vi;
  }
  __syncthreads();
  int32_t run = warp_tot[w] + incl - sum;
  for (int64_t i = lo; i < hi; ++i) {
    offsets[i] = run;
    run += counts[i];
  }
}

__global__ void pack_rank_kernel(const void* bidx, int dt, int64_t stride, int64_t E, int32_t B,
                                 const int32_t* n_valid, PackWs w) {
  grid_dep_wait();
  grid_dep_launch();
  if (w.flag[0] == 0) return;  // sorted: ranks are not needed
  if (!w.has_matrix) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_status(CK_ERR_UNSUPPORTED, 1, 0);
    return;
  }
  __shared__ int32_t sb[CHUNK];
  const int t = threadIdx.x;
  const int64_t c = blockIdx.x;
  const int64_t e = c * CHUNK + t;
  int32_t b = -1;
  if (e < real_events(n_valid, E)) {
    int64_t v = load_idx(bidx, dt, e, stride);
    b = (v >= 0 && v < B) ? (int32_t)v : -1;
  }
  sb[t] = b;
  __syncthreads();
  if (b < 0) return;
  int32_t r = 0;
  bool later = false;
  for (int j = 0; j < CHUNK; ++j) {
    const int32_t o = sb[j];
    if (j < t) r += (o == b);
    if (j > t && o == b) later = true;
  }
  w.rank[e] = r;
  if (!later) w.matrix[(int64_t)b * w.nchunks + c] = r + 1;
}

__global__ void pack_colscan_kernel(PackWs w) {
  grid_dep_wait();
  grid_dep_launch();
  if (w.flag[0] == 0 || !w.has_matrix) return;
  __shared__ int32_t carry_s;
  __shared__ int32_t wt[8];
  const int64_t b = blockIdx.x;
  int32_t* row = w.matrix + b * w.nchunks;
  const int t = threadIdx.x, lane = t & 31, wi = t >> 5;  // 256 threads
  if (t == 0) carry_s = 0;
  __syncthreads();
  for (int64_t base = 0; base < w.nchunks; base += 256) {
    const int64_t i = base + t;
    const int32_t v = (i < w.nchunks) ? row[i] : 0;
    int32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int32_t u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    if (lane == 31) wt[wi] = incl;
    __syncthreads();
    int32_t woff = 0, tot = 0;
    for (int k = 0; k < 8; ++k) {
      if (k < wi) woff += wt[k];
      tot += wt[k];
    }
    const int32_t carry = carry_s;
    if (i < w.nchunks) row[i] = carry + woff + incl - v;
    __syncthreads();
    if (t == 0) carry_s = carry + tot;
    __syncthreads();
  }
}

__global__ void pack_dest_kernel(const void* bidx, int dt, int64_t stride, int64_t E, int32_t B,
                                 const int32_t* n_valid, const int32_t* offsets, PackWs w,
                                 int32_t* dest) {
  grid_dep_wait();
  grid_dep_launch();
  const bool unsorted = w.flag[0] != 0;
  const int64_t nv = real_events(n_valid, E);
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < E;
       e += (int64_t)gridDim.x * blockDim.x) {
    if (e >= nv) {  // padding: real events fill rows 0..nv-1
      dest[e] = (int32_t)e;
      continue;
    }
    const int64_t v = load_idx(bidx, dt, e, stride);
    if (v < 0 || v >= B) {
      dest[e] = -1;
      continue;
    }
    if (!unsorted) {
      dest[e] = (int32_t)e;
    } else if (w.has_matrix) {
      dest[e] = offsets[v] + w.matrix[v * w.nchunks + e / CHUNK] + w.rank[e];
    } else {
      dest[e] = -1;
    }
  }
}

template <typename VT>
__global__ void pack_scatter_kernel(const uint8_t* flat, int64_t row_bytes, int64_t flat_stride_b,
                                    const void* bidx, int dt, int64_t stride, int64_t E,
                                    const int32_t* dest, const int32_t* offsets, int32_t e_max,
                                    uint8_t* out, uint8_t* mask) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t e = warp; e < E; e += nwarps) {
    const int32_t d = dest[e];
    if (d < 0) continue;
    const int64_t b = load_idx(bidx, dt, e, stride);
    const int64_t pos = d - offsets[b];
    const VT* src = reinterpret_cast<const VT*>(flat + e * flat_stride_b);
    VT* dst = reinterpret_cast<VT*>(out + (b * e_max + pos) * row_bytes);
    for (int64_t i = lane; i < row_bytes / (int64_t)sizeof(VT); i += 32) dst[i] = src[i];
    if (lane == 0) mask[b * e_max + pos] = 1;
  }
}

}  // namespace

size_t pack_workspace_bytes(int64_t E, int32_t B) {
  const int64_t nchunks = (E + CHUNK - 1) / CHUNK;
  size_t bytes = 256 + align256((size_t)E * 4);
  if ((int64_t)B * nchunks <= MAX_RANK_MATRIX) bytes += align256((size_t)B * nchunks * 4);
  return bytes;
}

int pack_events(const void* bidx, int dt, int64_t stride, int64_t E, int32_t B,
                const int32_t* n_valid, int32_t* counts, int32_t* offsets, int32_t* dest,
                int32_t* e_max, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (E < 0 || B <= 0 || counts == nullptr || offsets == nullptr || e_max == nullptr)
    return CK_ERR_INVALID_ARG;
  if (E > 0 && (bidx == nullptr || dest == nullptr)) return CK_ERR_INVALID_ARG;
  if (E > INT32_MAX - 1) return CK_ERR_INVALID_ARG;
  if (dt != CK_I64 && dt != CK_I32) return CK_ERR_UNSUPPORTED;
  if (ws_bytes < pack_workspace_bytes(E, B) || ws == nullptr) return CK_ERR_WORKSPACE;
  PackWs w = carve(ws, E, B);
  const int sms = num_sms();
  {
    const int64_t mwords = (w.has_matrix && E > 0) ? (int64_t)B * w.nchunks : 0;
    int64_t blocks = ((B > mwords ? (int64_t)B : mwords) + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > 4 * sms) blocks = 4 * sms;
    if (launch_pdl(pack_zero_kernel, dim3((unsigned)blocks), dim3(256), 0, st, counts, B, w.flag,
                   w.matrix, mwords))
      return CK_ERR_CUDA;
  }
  if (E > 0) {
    int64_t blocks = (E + 255) / 256;
    if (blocks > 8 * sms) blocks = 8 * sms;
    if (launch_pdl(pack_count_kernel, dim3((unsigned)blocks), dim3(256), 0, st, bidx, dt, stride, E, B, n_valid, counts, w.flag)) return CK_ERR_CUDA;
  }
  if (launch_pdl(pack_scan_kernel, dim3(1), dim3(1024), 0, st, counts, B, offsets, e_max)) return CK_ERR_CUDA;
  if (E > 0) {
    if (launch_pdl(pack_rank_kernel, dim3((unsigned)w.nchunks), dim3(CHUNK), 0, st, bidx, dt, stride, E, B, n_valid, w)) return CK_ERR_CUDA;
    if (launch_pdl(pack_colscan_kernel, dim3((unsigned)B), dim3(256), 0, st, w)) return CK_ERR_CUDA;
    int64_t blocks = (E + 255) / 256;
    if (blocks > 8 * sms) blocks = 8 * sms;
    if (launch_pdl(pack_dest_kernel, dim3((unsigned)blocks), dim3(256), 0, st, bidx, dt, stride, E, B, n_valid, offsets, w, dest)) return CK_ERR_CUDA;
  }
  return CK_OK;
}

int pack_scatter(const void* flat, int dtype, int64_t E, int32_t D, int64_t flat_stride,
                 const void* bidx, int dt, int64_t stride, const int32_t* dest,
                 const int32_t* offsets, int32_t e_max, void* out, uint8_t* mask,
                 cudaStream_t st) {
  if (E == 0) return CK_OK;
  if (E < 0 || D <= 0 || flat == nullptr || out == nullptr || mask == nullptr) return CK_ERR_INVALID_ARG;
  const int es = (dtype == CK_F32) ? 4 : (dtype == CK_BF16 ? 2 : 0);
  if (es == 0) return CK_ERR_UNSUPPORTED;
  const int64_t row_bytes = (int64_t)D * es;
  const int64_t fs_b = flat_stride * es;
  int64_t blocks = (E * 32 + 255) / 256;
  const int sms = num_sms();
  if (blocks > 16 * sms) blocks = 16 * sms;
  const bool v16 = (row_bytes % 16 == 0) && (fs_b % 16 == 0) &&
                   ((reinterpret_cast<uintptr_t>(flat) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  if (v16)
    return launch_pdl(pack_scatter_kernel<uint4>, dim3((unsigned)blocks), dim3(256), 0, st,
        reinterpret_cast<const uint8_t*>(flat), row_bytes, fs_b, bidx, dt, stride, E, dest,
        offsets, e_max, reinterpret_cast<uint8_t*>(out), mask);
  if (es == 4)
    return launch_pdl(pack_scatter_kernel<uint32_t>, dim3((unsigned)blocks), dim3(256), 0, st,
        reinterpret_cast<const uint8_t*>(flat), row_bytes, fs_b, bidx, dt, stride, E, dest,
        offsets, e_max, reinterpret_cast<uint8_t*>(out), mask);
  return launch_pdl(pack_scatter_kernel<uint16_t>, dim3((unsigned)blocks), dim3(256), 0, st,
      reinterpret_cast<const uint8_t*>(flat), row_bytes, fs_b, bidx, dt, stride, E, dest,
      offsets, e_max, reinterpret_cast<uint8_t*>(out), mask);
}

}  // namespace ck
