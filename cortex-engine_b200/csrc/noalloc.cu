// ck_norm_linear_static: the norm-then-linear entry point for callers that
// cannot allocate device memory.
//
// ck_norm_linear needs a scratch buffer for the normalised activations and
// asks the caller to pass one. Some callers have no device allocator to get it
// from: a service binding this C ABI from Go, Java or another host runtime
// without CUDA memory management of its own, or a serving loop that must not
// allocate once it is running. For them this entry point keeps the scratch in a
// fixed array in device memory that the library itself defines; the caller
// still passes inputs and outputs.
//
// Limits and sharing:
//  * the array holds kScratchBytes (8 MiB) -- M*K elements of the activation
//    dtype must fit (e.g. 8192 x 512 bf16); larger problems are rejected with
//    CK_ERR_INVALID_ARG before anything is launched;
//  * every GPU that loads the library holds those 8 MiB until the process exits;
//  * all calls on a device share the one array, so calls whose kernels overlap
//    on that device (different streams, other host threads) race on it and
//    must be serialised by the caller. The array keeps the last call's data;
//    nothing needs clearing, because the norm kernel writes every element the
//    GEMM then reads;
//  * the first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current) and caches it; make that
//    first call before any stream capture.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace ck {
int linear_dispatch(const void* A, int dtype, int64_t M, int64_t K, int64_t lda, const void* W,
                    int w_dtype, int w_layout, int64_t N, int64_t ldw, const float* w_scale,
                    int epi, const void* aux, int64_t ld_aux, int64_t aux_row_mod, void* Y,
                    int64_t ldy, cudaStream_t st, bool w_static);
}  // namespace ck

namespace {

constexpr size_t kScratchBytes = CK_NORM_LINEAR_STATIC_SCRATCH_BYTES;

static __device__ __align__(256) uint8_t g_norm_scratch[kScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {nullptr};

// Device address of g_norm_scratch on the current device (looked up once per
// device). Host code must not pass g_norm_scratch itself: on the host that name
// is only a stand-in, not a device address.
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ck::record_cuda_error();
  if (dev < 0 || dev >= 64) return CK_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> g(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_norm_scratch) != cudaSuccess || p == nullptr)
      return ck::record_cuda_error();
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return CK_OK;
}

}  // namespace

extern "C" int ck_norm_linear_static(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                                     const void* gamma, const void* beta, float eps, int norm_mode,
                                     const void* W, int w_dtype, int w_layout, int64_t N,
                                     int64_t ldw, const float* w_scale, int epi, const void* aux,
                                     int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy,
                                     void* stream) {
  if (M < 0 || K <= 0) return CK_ERR_INVALID_ARG;
  if (dtype != CK_F32 && dtype != CK_BF16) return CK_ERR_UNSUPPORTED;
  if (norm_mode != CK_NORM_LAYER && norm_mode != CK_NORM_RMS) return CK_ERR_INVALID_ARG;
  const size_t es = dtype == CK_F32 ? 4 : 2;
  if ((size_t)M > kScratchBytes / es / (size_t)K) return CK_ERR_INVALID_ARG;  // over the limit
  if (M == 0) return CK_OK;
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc != CK_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = ck::row_norm(x, dtype, M, (int32_t)K, ldx, gamma, beta, eps, norm_mode, scratch, K, st);
  if (rc != CK_OK) return rc;
  return ck::linear_dispatch(scratch, dtype, M, K, K, W, w_dtype, w_layout, N, ldw, w_scale, epi,
                             aux, ld_aux, aux_row_mod, Y, ldy, st);
}
