// ck_norm_linear_static: the norm-then-linear entry point for callers that
// cannot allocate device memory.
//
// ck_norm_linear asks its caller for a scratch buffer whenever the call takes
// the two-launch path (a LayerNorm, fp32 rows, K not a multiple of 8, or a GELU / residual
// epilogue: the normalised rows go to the buffer, then the linear reads them).
// Some callers have no device allocator to get that buffer from: a service
// binding this C ABI from Go, Java or another host runtime without CUDA memory
// management of its own, or a serving loop that must not allocate once it is
// running. For them this entry point keeps the scratch in a fixed array in
// device memory that the library itself defines; the caller still passes
// inputs and outputs. Calls that ck_norm_linear runs as one launch (RMSNorm of
// bf16 rows inside the tensor-core GEMM) need no scratch here either.
//
// Limits and sharing:
//  * the array holds kScratchBytes (8 MiB): on the two-launch path M*K elements
//    of the activation dtype must fit (e.g. 8192 x 512 bf16); larger problems
//    are rejected with CK_ERR_INVALID_ARG before anything is launched;
//  * every GPU that loads the library holds those 8 MiB until the process exits;
//  * all calls on a device share the one array, so calls whose kernels overlap
//    on that device (different streams, other host threads) race on it and
//    must be serialised by the caller. The array keeps the last call's data;
//    nothing needs clearing, because the norm kernel writes every element the
//    GEMM then reads;
//  * each call looks up the array's device address on the current device
//    (cudaGetSymbolAddress); the first call on a device also loads the
//    library's device code there, so make it before any stream capture.
#include "common.cuh"
#include "kernels.h"

namespace {

constexpr size_t kScratchBytes = CK_NORM_LINEAR_STATIC_SCRATCH_BYTES;

static __device__ __align__(256) uint8_t g_norm_scratch[kScratchBytes];

// Device address of g_norm_scratch in the current device's context. Host code
// must not pass g_norm_scratch itself: on the host that name is only a
// stand-in, not a device address. Looked up on every call, so that a device
// reset or another context never leaves a stale address behind.
int scratch_for_current_device(void** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_norm_scratch) != cudaSuccess || p == nullptr)
    return ck::record_cuda_error();
  *out = p;
  return CK_OK;
}

}  // namespace

extern "C" int ck_norm_linear_static(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                                     const void* gamma, const void* beta, float eps, int norm_mode,
                                     const void* W, int w_dtype, int w_layout, int64_t N,
                                     int64_t ldw, const float* w_scale, int epi, const void* aux,
                                     int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy,
                                     void* stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (M < 0 || K <= 0) return CK_ERR_INVALID_ARG;
  if (dtype != CK_F32 && dtype != CK_BF16) return CK_ERR_UNSUPPORTED;
  if (norm_mode == CK_NORM_NONE || M == 0 ||
      ck::norm_linear_fused(dtype, M, K, ldx, x, gamma, norm_mode, W, w_dtype, w_layout, N, ldw,
                            epi, aux, ld_aux, Y, ldy))  // no scratch on these paths
    return ck::norm_linear(x, dtype, M, K, ldx, gamma, beta, eps, norm_mode, W, w_dtype,
                           w_layout, N, ldw, w_scale, epi, aux, ld_aux, aux_row_mod, Y, ldy,
                           nullptr, 0, st);
  const size_t es = dtype == CK_F32 ? 4 : 2;
  if ((size_t)M > kScratchBytes / es / (size_t)K) return CK_ERR_INVALID_ARG;  // over the limit
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != CK_OK) return rc;
  return ck::norm_linear(x, dtype, M, K, ldx, gamma, beta, eps, norm_mode, W, w_dtype, w_layout,
                         N, ldw, w_scale, epi, aux, ld_aux, aux_row_mod, Y, ldy, scratch,
                         kScratchBytes, st);
}
