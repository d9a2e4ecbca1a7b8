// Launch trace: per-kernel device times of the library's own launches.
//
// Between ck_trace_begin and ck_trace_end every kernel this library launches
// outside a stream capture gets a CUDA event recorded on its stream just before
// the launch and one just after. The pair times the kernel on the device as
// the stream runs it: with the events between launches, a kernel no longer
// overlaps its predecessor's tail (programmatic launch), so each figure is the
// kernel's own duration from the moment its stream reaches it. Events are
// created up front (ck_trace_begin) and recorded into a fixed pool; launches
// past the pool's capacity are counted but not timed. Host-side only: no
// device memory is allocated.
#include <cuda_runtime.h>

#include <cxxabi.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "cortex_b200.h"
#include "kernels.h"

namespace ck {

int g_trace_on = 0;

namespace {

struct Rec {
  cudaStream_t stream;
  const void* func;
  int ev0, ev1;
};

std::mutex g_mu;
std::vector<cudaEvent_t> g_events;
std::vector<Rec> g_recs;
int g_next_event = 0;
long long g_dropped = 0;
// the event recorded by trace_before of the launch in flight on this thread
thread_local int t_pending = -1;

bool capturing(cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) {
    (void)cudaGetLastError();
    return true;  // unknown: do not touch the stream
  }
  return cs != cudaStreamCaptureStatusNone;
}

// "void ck::(anonymous namespace)::gemm_tc_kernel<256, 0, 2, 3, false>(CUtensorMap, ...)"
// -> "gemm_tc_kernel<256, 0, 2, 3, false>"
std::string short_name(const char* mangled) {
  if (mangled == nullptr) return "?";
  // kernels with internal linkage come back as "__nv_static_<n>__<hash>_<file>__Z...":
  // demangle from the Itanium "_Z" on
  if (std::strncmp(mangled, "_Z", 2) != 0) {
    const char* z = std::strstr(mangled, "__Z");
    if (z != nullptr) mangled = z + 1;
  }
  int st = 0;
  char* dem = abi::__cxa_demangle(mangled, nullptr, nullptr, &st);
  std::string s = (st == 0 && dem != nullptr) ? std::string(dem) : std::string(mangled);
  std::free(dem);
  const std::string anon = "(anonymous namespace)::";
  for (size_t i = s.find(anon); i != std::string::npos; i = s.find(anon)) s.erase(i, anon.size());
  // cut the parameter list: the first '(' outside the template argument list
  int depth = 0;
  for (size_t i = 0; i < s.size(); ++i) {
    if (s[i] == '<') ++depth;
    if (s[i] == '>') --depth;
    if (s[i] == '(' && depth == 0) {
      s.resize(i);
      break;
    }
  }
  // drop the return type and the namespaces before the name
  size_t lt = s.find('<');
  if (lt == std::string::npos) lt = s.size();
  const size_t ns = s.rfind("::", lt);
  const size_t sp = s.rfind(' ', lt);
  size_t from = 0;
  if (ns != std::string::npos) from = ns + 2;
  if (sp != std::string::npos && sp + 1 > from) from = sp + 1;
  return s.substr(from);
}

}  // namespace

void trace_before(cudaStream_t st) {
  t_pending = -1;
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_trace_on || capturing(st)) return;
  if (g_next_event + 2 > (int)g_events.size()) {
    ++g_dropped;
    return;
  }
  const int e = g_next_event;
  g_next_event += 2;
  if (cudaEventRecord(g_events[e], st) != cudaSuccess) {
    (void)cudaGetLastError();
    return;
  }
  t_pending = e;
}

void trace_after(cudaStream_t st, const void* func) {
  const int e = t_pending;
  t_pending = -1;
  if (e < 0) return;
  std::lock_guard<std::mutex> g(g_mu);
  if (cudaEventRecord(g_events[e + 1], st) != cudaSuccess) {
    (void)cudaGetLastError();
    return;
  }
  g_recs.push_back(Rec{st, func, e, e + 1});
}

}  // namespace ck

using namespace ck;

extern "C" int ck_trace_begin(int32_t capacity) {
  if (capacity <= 0) return CK_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> g(g_mu);
  for (cudaEvent_t e : g_events) cudaEventDestroy(e);
  g_events.clear();
  g_recs.clear();
  g_next_event = 0;
  g_dropped = 0;
  g_events.reserve(2 * (size_t)capacity);
  for (int i = 0; i < 2 * capacity; ++i) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) {
      for (cudaEvent_t x : g_events) cudaEventDestroy(x);
      g_events.clear();
      return record_cuda_error();
    }
    g_events.push_back(e);
  }
  g_trace_on = 1;
  return CK_OK;
}

extern "C" int ck_trace_end(ck_trace_record* out, int32_t capacity, int32_t* n) {
  std::lock_guard<std::mutex> g(g_mu);
  g_trace_on = 0;
  int rc = CK_OK;
  int w = 0;
  for (const Rec& r : g_recs) {
    if (out != nullptr && w < capacity) {
      ck_trace_record& o = out[w];
      std::memset(&o, 0, sizeof(o));
      const char* nm = nullptr;
      if (cudaFuncGetName(&nm, r.func) != cudaSuccess) {
        (void)cudaGetLastError();
        nm = nullptr;
      }
      const std::string s = short_name(nm);
      std::strncpy(o.name, s.c_str(), sizeof(o.name) - 1);
      o.stream = reinterpret_cast<void*>(r.stream);
      float ms = -1.f;
      if (cudaEventSynchronize(g_events[r.ev1]) != cudaSuccess ||
          cudaEventElapsedTime(&ms, g_events[r.ev0], g_events[r.ev1]) != cudaSuccess) {
        rc = record_cuda_error();
        ms = -1.f;
      }
      o.ms = ms;
    }
    ++w;
  }
  if (n != nullptr) *n = w;
  for (cudaEvent_t e : g_events) cudaEventDestroy(e);
  g_events.clear();
  g_recs.clear();
  g_next_event = 0;
  return rc;
}
