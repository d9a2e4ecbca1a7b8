// Event ingest on the device: events_from_bin_matrix + bucket_values +
// collate_events (cortex/data/nlb.py:74-114, 492-512) from bin-count matrices
// resident in HBM straight into a packed event batch (CK_BATCH layout).
//
// Window b covers rows start..start+window_bins-1 of its session's (T, N)
// int32 count matrix. Every nonzero bin is one event, in the order np.nonzero
// gives on the window slice (row-major: time bin, then neuron) and windows in
// batch order, which is the order collate_events concatenates them:
//   neuron_ids    = n + neuron_offset        (NLBDataset.__getitem__, :258)
//   time_bins     = r (window-relative row)
//   values        = clamp(count, 0, n_buckets - 1)      (bucket_values, :83)
//   batch_indices = b
// A neuron id >= max_neurons sets CK_ERR_INDEX (the reference raises, :259).
//
// Three launches, no host synchronisation:
//   1. window_count  one CTA per window: nonzeros per row (a warp per row,
//                    ballot over 32 neurons at a time), CTA scan -> row offsets
//                    within the window and the window's total
//   2. window_scan   one CTA: exclusive scan of the window totals, n_valid
//   3. emit          a warp per (window, row): ballot compaction of the row's
//                    nonzeros into the four arrays (rows past capacity are
//                    dropped and CK_ERR_INVALID_ARG records the shortfall)
// capacity == 0 counts only: launches 1-2 run, *n_total receives the count.
#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

constexpr int WC_THREADS = 512;

struct IngestWs {
  int32_t* row_off;   // B * W: offset of each row within its window
  int32_t* win_tot;   // B: events per window
  int32_t* win_off;   // B + 1: exclusive scan of win_tot
};

size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

IngestWs carve(void* ws, int32_t B, int32_t W) {
  uint8_t* p = reinterpret_cast<uint8_t*>(ws);
  IngestWs w;
  w.row_off = reinterpret_cast<int32_t*>(p);
  p += al256((size_t)B * W * 4);
  w.win_tot = reinterpret_cast<int32_t*>(p);
  p += al256((size_t)B * 4);
  w.win_off = reinterpret_cast<int32_t*>(p);
  return w;
}

// A window whose rows or columns fall outside its matrix is reported and
// treated as empty, so no kernel reads outside the matrix.
__device__ __forceinline__ bool window_ok(const ck_bin_window& w, int32_t W) {
  return w.counts != nullptr && w.start >= 0 && w.start + W <= w.n_rows && w.n_neurons >= 0 &&
         w.n_neurons <= w.ld;
}

__device__ __forceinline__ int row_nonzeros(const int32_t* row, int n, int lane) {
  int c = 0;
  for (int j = lane; j - lane < n; j += 32) {
    const bool nz = j < n && row[j] != 0;
    c += __popc(__ballot_sync(0xffffffffu, nz));
  }
  return c;
}

__global__ void __launch_bounds__(WC_THREADS) window_count_kernel(const ck_bin_window* wins,
                                                                  int32_t W, IngestWs w) {
  grid_dep_wait();
  grid_dep_launch();
  extern __shared__ int32_t cnt[];  // W row counts
  __shared__ int32_t warp_sum[WC_THREADS / 32];
  const int b = blockIdx.x;
  const ck_bin_window win = wins[b];
  const bool ok = window_ok(win, W);
  if (!ok && threadIdx.x == 0) set_status(CK_ERR_INDEX, b, (int)win.start);
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  for (int r = wp; r < W; r += WC_THREADS / 32) {
    const int c = ok ? row_nonzeros(win.counts + (win.start + r) * win.ld, win.n_neurons, lane) : 0;
    if (lane == 0) cnt[r] = c;
  }
  __syncthreads();
  // exclusive scan of cnt[0..W): each thread owns a contiguous run
  const int per = (W + WC_THREADS - 1) / WC_THREADS;
  const int lo = threadIdx.x * per, hi = min(W, lo + per);
  int32_t s = 0;
  for (int i = lo; i < hi; ++i) s += cnt[i];
  int32_t incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_sum[wp] = incl;
  __syncthreads();
  int32_t base = 0, total = 0;
  for (int k = 0; k < WC_THREADS / 32; ++k) {
    if (k < wp) base += warp_sum[k];
    total += warp_sum[k];
  }
  int32_t run = base + incl - s;
  for (int i = lo; i < hi; ++i) {
    w.row_off[(int64_t)b * W + i] = run;
    run += cnt[i];
  }
  if (threadIdx.x == 0) w.win_tot[b] = total;
}

__global__ void window_scan_kernel(int32_t B, IngestWs w, int64_t capacity, int32_t* batch) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ int32_t warp_sum[32];
  __shared__ int64_t carry_s;
  const int t = threadIdx.x, lane = t & 31, wp = t >> 5;  // 1024 threads
  if (t == 0) carry_s = 0;
  __syncthreads();
  for (int64_t base = 0; base < B; base += 1024) {
    const int64_t i = base + t;
    const int32_t v = i < B ? w.win_tot[i] : 0;
    int32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    if (lane == 31) warp_sum[wp] = incl;
    __syncthreads();
    int32_t woff = 0, tot = 0;
    for (int k = 0; k < 32; ++k) {
      if (k < wp) woff += warp_sum[k];
      tot += warp_sum[k];
    }
    const int64_t carry = carry_s;
    if (i < B) w.win_off[i] = (int32_t)min(carry + woff + incl - v, (int64_t)INT32_MAX);
    __syncthreads();
    if (t == 0) carry_s = carry + tot;
    __syncthreads();
  }
  if (t == 0) {
    const int64_t total = carry_s;
    w.win_off[B] = (int32_t)min(total, (int64_t)INT32_MAX);
    batch[0] = (int32_t)min(total, capacity);
    batch[1] = batch[2] = batch[3] = 0;
    if (capacity > 0 && total > capacity) set_status(CK_ERR_INVALID_ARG, (int)min(total, (int64_t)INT32_MAX),
                                     (int)capacity);
  }
}

__global__ void emit_kernel(const ck_bin_window* wins, int32_t B, int32_t W, int32_t n_buckets,
                            int32_t max_neurons, IngestWs w, int64_t capacity, int32_t* arr) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  int32_t* nid = arr;
  int32_t* tb = arr + capacity;
  int32_t* val = arr + 2 * capacity;
  int32_t* bix = arr + 3 * capacity;
  const unsigned below = (1u << lane) - 1u;
  for (int64_t row = warp; row < (int64_t)B * W; row += nwarps) {
    const int b = (int)(row / W), r = (int)(row % W);
    const ck_bin_window win = wins[b];
    if (!window_ok(win, W)) continue;
    const int32_t* src = win.counts + (win.start + r) * win.ld;
    int64_t pos = (int64_t)w.win_off[b] + w.row_off[row];
    for (int j = lane; j - lane < win.n_neurons; j += 32) {
      const int32_t c = j < win.n_neurons ? src[j] : 0;
      const unsigned m = __ballot_sync(0xffffffffu, c != 0);
      if (c != 0) {
        const int64_t at = pos + __popc(m & below);
        const int32_t id = j + win.neuron_offset;
        if (id >= max_neurons) set_status(CK_ERR_INDEX, (int)row, id);
        if (at < capacity) {
          nid[at] = id;
          tb[at] = r;
          val[at] = c < 0 ? 0 : (c > n_buckets - 1 ? n_buckets - 1 : c);
          bix[at] = b;
        }
      }
      pos += __popc(m);
    }
  }
}

}  // namespace

size_t collate_bins_workspace_bytes(int32_t B, int32_t W) {
  if (B <= 0 || W <= 0) return 0;
  return al256((size_t)B * W * 4) + al256((size_t)B * 4) + al256((size_t)(B + 1) * 4);
}

int collate_bins(const ck_bin_window* wins, int32_t B, int32_t W, int32_t n_buckets,
                 int32_t max_neurons, int32_t* batch, int64_t capacity, void* ws, size_t ws_bytes,
                 int32_t* n_total, cudaStream_t st) {
  if (wins == nullptr || batch == nullptr || B <= 0 || W <= 0 || n_buckets <= 0 ||
      capacity < 0 || capacity % 4 != 0 || (reinterpret_cast<uintptr_t>(batch) & 15u) != 0)
    return CK_ERR_INVALID_ARG;
  if ((int64_t)B * W > INT32_MAX) return CK_ERR_INVALID_ARG;
  if (ws == nullptr || ws_bytes < collate_bins_workspace_bytes(B, W)) return CK_ERR_WORKSPACE;
  const size_t smem = (size_t)W * 4;
  if (smem > 200 * 1024) return CK_ERR_UNSUPPORTED;
  if (smem > 48 * 1024 &&
      !smem_attr_ready(reinterpret_cast<const void*>(window_count_kernel), 200 * 1024))
    return record_cuda_error();
  IngestWs w = carve(ws, B, W);
  if (launch_pdl(window_count_kernel, dim3((unsigned)B), dim3(WC_THREADS), smem, st, wins, W, w))
    return CK_ERR_CUDA;
  if (launch_pdl(window_scan_kernel, dim3(1), dim3(1024), 0, st, B, w, capacity, batch))
    return CK_ERR_CUDA;
  if (n_total != nullptr &&
      cudaMemcpyAsync(n_total, w.win_off + B, 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return record_cuda_error();
  if (capacity > 0) {
    int64_t blocks = ((int64_t)B * W * 32 + 255) / 256;
    const int64_t cap = 16 * (int64_t)num_sms();
    if (blocks > cap) blocks = cap;
    if (launch_pdl(emit_kernel, dim3((unsigned)blocks), dim3(256), 0, st, wins, B, W, n_buckets,
                   max_neurons, w, capacity, batch + CK_BATCH_HEADER_WORDS))
      return CK_ERR_CUDA;
  }
  return CK_OK;
}

}  // namespace ck
