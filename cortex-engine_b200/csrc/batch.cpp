// Host side of the packed event batch (CK_BATCH_* layout in cortex_b200.h):
// the per-batch work InferenceWorker._run_batch_sync does in Python lists and
// four torch.tensor(..., int64) constructions (cortex/serve/worker.py:166-200),
// done as one pass per array in native code into a (pinned) int32 buffer that
// then crosses to the device in one copy.
#include <cstdint>
#include <cstring>

#include "cortex_b200.h"

namespace {

// The two loops below are written for the compiler's vectoriser; the clones
// give an AVX-512 and an AVX2 build picked at load time (gcc ifunc), with the
// baseline x86-64 one as the fallback.
#define CK_SIMD_CLONES __attribute__((target_clones("avx512f", "avx2", "default")))

// Saturating int64 -> int32 narrowing, plus the min / max of the input.
CK_SIMD_CLONES void narrow(const int64_t* src, int64_t n, int32_t* dst, int64_t* mn_out, int64_t* mx_out) {
  int64_t mn = INT64_MAX, mx = INT64_MIN;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t v = src[i];
    mn = v < mn ? v : mn;
    mx = v > mx ? v : mx;
    const int64_t c = v < INT32_MIN ? INT32_MIN : (v > INT32_MAX ? INT32_MAX : v);
    dst[i] = (int32_t)c;
  }
  *mn_out = mn;
  *mx_out = mx;
}

// Saturating int64 -> int32 narrowing alone (the arrays whose range the
// caller does not need).
CK_SIMD_CLONES void narrow_only(const int64_t* src, int64_t n, int32_t* dst) {
  for (int64_t i = 0; i < n; ++i) {
    const int64_t v = src[i];
    dst[i] = (int32_t)(v < INT32_MIN ? INT32_MIN : (v > INT32_MAX ? INT32_MAX : v));
  }
}

CK_SIMD_CLONES void minmax32(const int32_t* src, int64_t n, int64_t* mn_out, int64_t* mx_out) {
  int32_t mn = INT32_MAX, mx = INT32_MIN;
  for (int64_t i = 0; i < n; ++i) {
    mn = src[i] < mn ? src[i] : mn;
    mx = src[i] > mx ? src[i] : mx;
  }
  *mn_out = mn;
  *mx_out = mx;
}

}  // namespace

extern "C" int ck_batch_stage(const void* nid, const void* tb, const void* val, const void* bidx,
                              int idx_dtype, int64_t E, int32_t* batch, int64_t capacity,
                              int32_t* batch_size) {
  if (batch == nullptr || batch_size == nullptr || E < 0 || capacity < E || capacity % 4 != 0 ||
      E > INT32_MAX)
    return CK_ERR_INVALID_ARG;
  if (idx_dtype != CK_I32 && idx_dtype != CK_I64) return CK_ERR_UNSUPPORTED;
  if (E > 0 && (nid == nullptr || tb == nullptr || val == nullptr || bidx == nullptr))
    return CK_ERR_INVALID_ARG;
  int32_t* arr = batch + CK_BATCH_HEADER_WORDS;
  const void* src[4] = {nid, tb, val, bidx};
  int64_t bmin = 0, bmax = -1;
  for (int k = 0; k < 4 && E > 0; ++k) {
    int64_t mn, mx;
    if (idx_dtype == CK_I64) {
      if (k == 3)  // only the batch indices' range is needed (B, validity)
        narrow(static_cast<const int64_t*>(src[k]), E, arr + k * capacity, &mn, &mx);
      else
        narrow_only(static_cast<const int64_t*>(src[k]), E, arr + k * capacity);
    } else {
      std::memcpy(arr + k * capacity, src[k], (size_t)E * 4);
      if (k == 3) minmax32(static_cast<const int32_t*>(src[k]), E, &mn, &mx);
    }
    if (k == 3) {
      bmin = mn;
      bmax = mx;
    }
  }
  if (E > 0 && (bmin < 0 || bmax >= INT32_MAX)) return CK_ERR_INDEX;
  batch[0] = (int32_t)E;
  batch[1] = batch[2] = batch[3] = 0;
  *batch_size = E > 0 ? (int32_t)(bmax + 1) : 1;
  return CK_OK;
}
