// Per-device status word and small runtime helpers shared by every entry point.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_set>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"

namespace ck {

__device__ int g_status = 0;
__device__ int g_status_info[4] = {0, 0, 0, 0};

namespace {
thread_local int t_last_cuda_error = 0;
std::mutex g_attr_mu;
std::atomic<long long> g_launches{0};
}  // namespace

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  static int cache[64] = {0};
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

int record_cuda_error() {
  cudaError_t e = cudaGetLastError();
  t_last_cuda_error = (int)e;
  return CK_ERR_CUDA;
}

namespace {
int check_launch_noc() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    t_last_cuda_error = (int)e;
    return CK_ERR_CUDA;
  }
  return CK_OK;
}
}  // namespace

int check_launch() {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return check_launch_noc();
}

int finish_launch(cudaError_t e) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (e != cudaSuccess) {
    cudaGetLastError();
    t_last_cuda_error = (int)e;
    return CK_ERR_CUDA;
  }
  return check_launch_noc();
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("CK_PDL");
    return v == nullptr || std::strcmp(v, "0") != 0;
  }();
  return on;
}

bool smem_attr_ready(const void* kernel, int bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  static std::unordered_set<uint64_t> done;
  const uint64_t key = (reinterpret_cast<uint64_t>(kernel) << 8) ^ (uint64_t)dev;
  std::lock_guard<std::mutex> g(g_attr_mu);
  if (done.count(key)) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess)
    return false;
  done.insert(key);
  return true;
}

int last_cuda_error() { return t_last_cuda_error; }

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}
}  // namespace

// 2-D tiled tensor map (innermost dimension first). Host-only; the driver
// entry point is resolved through the runtime so nothing links libcuda.
bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                  uint64_t inner, uint64_t outer, uint64_t ld_elems, uint32_t box_inner,
                  uint32_t box_outer, int swizzle_bytes) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace ck

extern "C" int ck_get_last_status(int* info4) {
  if (cudaDeviceSynchronize() != cudaSuccess) return ck::record_cuda_error();
  int code = 0;
  int info[4] = {0, 0, 0, 0};
  if (cudaMemcpyFromSymbol(&code, ck::g_status, sizeof(int)) != cudaSuccess)
    return ck::record_cuda_error();
  if (cudaMemcpyFromSymbol(info, ck::g_status_info, sizeof(info)) != cudaSuccess)
    return ck::record_cuda_error();
  const int zero[4] = {0, 0, 0, 0};
  if (cudaMemcpyToSymbol(ck::g_status, zero, sizeof(int)) != cudaSuccess)
    return ck::record_cuda_error();
  if (info4 != nullptr)
    for (int i = 0; i < 4; ++i) info4[i] = info[i];
  return code;
}

extern "C" int ck_last_cuda_error(void) { return ck::last_cuda_error(); }

extern "C" const char* ck_status_string(int code) {
  switch (code) {
    case CK_OK: return "ok";
    case CK_ERR_INVALID_ARG: return "invalid argument (shape, stride, alignment or pointer)";
    case CK_ERR_UNSUPPORTED: return "unsupported dtype/layout combination";
    case CK_ERR_CUDA: return "CUDA runtime error";
    case CK_ERR_INDEX: return "event index out of range";
    case CK_ERR_TIMEOUT: return "bounded device wait timed out";
    case CK_ERR_WORKSPACE: return "workspace too small";
  }
  return "unknown status";
}

extern "C" int ck_num_sms(void) { return ck::num_sms(); }

extern "C" long long ck_launch_count(void) {
  return ck::g_launches.load(std::memory_order_relaxed);
}
