// Row-segment copies between row buffers: the data path of the streaming K|V
// cache (cortex/cache/streaming.py:79-236), which keeps kv_proj rows of whole
// windows in fixed-size pages of one HBM pool. Gathering a cached window into
// the packed K|V rows of a batch, and writing a computed window into its pages,
// are both lists of (src_row, dst_row, rows) segments: one launch per list,
// a CTA per segment, 16-byte vectors.
#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

__global__ void __launch_bounds__(256) copy_rows_kernel(const uint4* src, int64_t src_rows,
                                                        uint4* dst, int64_t dst_rows,
                                                        int64_t row_vecs, const int32_t* seg,
                                                        int32_t n_seg) {
  grid_dep_wait();
  grid_dep_launch();
  for (int64_t s = blockIdx.x; s < n_seg; s += gridDim.x) {
    const int64_t sr = seg[3 * s], dr = seg[3 * s + 1], n = seg[3 * s + 2];
    if (sr < 0 || dr < 0 || n < 0 || sr + n > src_rows || dr + n > dst_rows) {
      if (threadIdx.x == 0) set_status(CK_ERR_INDEX, (int)s, (int)n);
      continue;
    }
    const uint4* a = src + sr * row_vecs;
    uint4* b = dst + dr * row_vecs;
    const int64_t total = n * row_vecs;
    for (int64_t i = threadIdx.x; i < total; i += blockDim.x) b[i] = a[i];
  }
}

}  // namespace

int copy_rows(const void* src, int64_t src_rows, void* dst, int64_t dst_rows, int64_t row_bytes,
              const int32_t* segments, int32_t n_segments, cudaStream_t st) {
  if (n_segments == 0) return CK_OK;
  if (src == nullptr || dst == nullptr || segments == nullptr || n_segments < 0 ||
      row_bytes <= 0 || row_bytes % 16 != 0 || src_rows < 0 || dst_rows < 0)
    return CK_ERR_INVALID_ARG;
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) != 0)
    return CK_ERR_INVALID_ARG;
  int64_t blocks = n_segments;
  const int64_t cap = 8 * (int64_t)num_sms();
  if (blocks > cap) blocks = cap;
  return launch_pdl(copy_rows_kernel, dim3((unsigned)blocks), dim3(256), 0, st,
                    reinterpret_cast<const uint4*>(src), src_rows, reinterpret_cast<uint4*>(dst),
                    dst_rows, row_bytes / 16, segments, n_segments);
}

}  // namespace ck

extern "C" int ck_copy_rows(const void* src, int64_t src_rows, void* dst, int64_t dst_rows,
                            int64_t row_bytes, const int32_t* segments, int32_t n_segments,
                            void* stream) {
  return ck::copy_rows(src, src_rows, dst, dst_rows, row_bytes, segments, n_segments,
                       reinterpret_cast<cudaStream_t>(stream));
}
