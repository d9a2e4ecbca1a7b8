// Per-device status word and small runtime helpers shared by every entry point.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <unordered_set>

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

int check_launch() {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    t_last_cuda_error = (int)e;
    return CK_ERR_CUDA;
  }
  return CK_OK;
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
