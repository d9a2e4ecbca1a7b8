// Native serving runner: host event arrays in, behaviour out, with one
// host-to-device copy and one CUDA-graph launch per batch.
//
// The per-batch work of InferenceWorker._run_batch_sync and CortexModel.forward
// (cortex/serve/worker.py:166-214, cortex/models/cortex.py:90-122) is split in
// two calls so that the caller can size its output between them:
//   ck_runner_stage   narrows the four host index arrays into a pinned int32
//                     packed batch (ck_batch_stage) and returns B
//   ck_runner_launch  copies that batch to the device, launches the CUDA graph
//                     of ck_forward_batch captured for its (B, capacity)
//                     bucket (captured on first use, after an eager run), and
//                     copies the bucket's output into the caller's buffer.
// Two pinned staging slots alternate, each guarded by the event of the copy
// that last read it. The device batch buffer, the workspace and the graphs'
// outputs belong to the runner; when the batch buffer or the workspace has to
// grow, the runner waits for the device, reallocates and drops its graphs.
// A runner serves one device; calls are serialised by a mutex, and all launches
// of one runner must use one stream (graphs share its buffers).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <utility>
#include <vector>

#include "cortex_b200.h"

namespace ck {
int record_cuda_error();  // status.cu
}

namespace {

struct Graph {
  cudaGraphExec_t exec = nullptr;
  void* out = nullptr;
  uint64_t used = 0;
};

int cuda_fail() { return ck::record_cuda_error(); }

// Event slots of the bucket that holds n events (a multiple of 256, at most
// 1/16 padding past the first bucket); cortex/batching.py uses the same rule.
int64_t bucket(int64_t n) {
  if (n <= 256) return 256;
  int bits = 0;
  for (int64_t v = n; v > 0; v >>= 1) ++bits;
  const int64_t g = int64_t(1) << (bits - 5 > 8 ? bits - 5 : 8);
  return (n + g - 1) / g * g;
}

}  // namespace

struct ck_runner {
  ck_model model;
  std::vector<ck_block_weights> blocks;
  int device = 0;
  size_t max_graphs = 64;
  int64_t capacity = 0;        // event slots of the device batch buffer and pinned slots
  int32_t* dbatch = nullptr;   // device batch buffer
  int32_t* host[2] = {nullptr, nullptr};
  cudaEvent_t copied[2] = {nullptr, nullptr};
  bool used[2] = {false, false};
  int next = 0;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  std::map<std::pair<int32_t, int64_t>, Graph> graphs;
  uint64_t tick = 0;
  cudaStream_t cap_stream = nullptr;
  std::mutex mu;
  // the staged batch waiting for ck_runner_launch
  int staged_slot = -1;
  int64_t staged_cap = 0;
  int32_t staged_b = 0;
  long long captures = 0, replays = 0;
};

namespace {

void drop_graphs(ck_runner* r) {
  for (auto& kv : r->graphs) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (kv.second.out) cudaFree(kv.second.out);
  }
  r->graphs.clear();
}

int reserve(ck_runner* r, int64_t cap) {
  if (cap <= r->capacity) return CK_OK;
  const int64_t want = cap > bucket(r->capacity + r->capacity / 4) ? cap
                                                                   : bucket(r->capacity + r->capacity / 4);
  if (cudaDeviceSynchronize() != cudaSuccess) return cuda_fail();
  drop_graphs(r);
  if (r->dbatch) cudaFree(r->dbatch);
  for (int s = 0; s < 2; ++s)
    if (r->host[s]) cudaFreeHost(r->host[s]);
  r->dbatch = nullptr;
  r->host[0] = r->host[1] = nullptr;
  r->capacity = 0;
  const size_t bytes = (size_t)CK_BATCH_WORDS(want) * 4;
  if (cudaMalloc(&r->dbatch, bytes) != cudaSuccess) return cuda_fail();
  for (int s = 0; s < 2; ++s) {
    if (cudaHostAlloc(&r->host[s], bytes, cudaHostAllocDefault) != cudaSuccess) return cuda_fail();
    r->used[s] = false;
  }
  r->capacity = want;
  return CK_OK;
}

int ensure_ws(ck_runner* r, int64_t cap, int32_t B) {
  const size_t need = ck_forward_workspace_bytes(&r->model, cap, B);
  if (need == 0) return CK_ERR_INVALID_ARG;
  if (need <= r->ws_bytes) return CK_OK;
  if (cudaDeviceSynchronize() != cudaSuccess) return cuda_fail();
  drop_graphs(r);
  if (r->ws) cudaFree(r->ws);
  r->ws = nullptr;
  r->ws_bytes = 0;
  const size_t bytes = need + need / 4 + 4096;
  if (cudaMalloc(&r->ws, bytes) != cudaSuccess) return cuda_fail();
  r->ws_bytes = bytes;
  return CK_OK;
}

size_t elem_bytes(const ck_model& m) { return m.dtype == CK_F32 ? 4 : 2; }

}  // namespace

extern "C" int ck_runner_create(const ck_model* m, int32_t max_graphs, ck_runner** out) {
  if (m == nullptr || out == nullptr || (m->num_layers > 0 && m->blocks == nullptr))
    return CK_ERR_INVALID_ARG;
  ck_runner* r = new (std::nothrow) ck_runner();
  if (r == nullptr) return CK_ERR_INVALID_ARG;
  r->model = *m;
  if (m->num_layers > 0) {
    r->blocks.assign(m->blocks, m->blocks + m->num_layers);
    r->model.blocks = r->blocks.data();
  }
  if (max_graphs > 0) r->max_graphs = (size_t)max_graphs;
  if (cudaGetDevice(&r->device) != cudaSuccess ||
      cudaStreamCreateWithFlags(&r->cap_stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete r;
    return cuda_fail();
  }
  for (int s = 0; s < 2; ++s)
    if (cudaEventCreateWithFlags(&r->copied[s], cudaEventDisableTiming) != cudaSuccess) {
      ck_runner_destroy(r);
      return cuda_fail();
    }
  *out = r;
  return CK_OK;
}

extern "C" void ck_runner_destroy(ck_runner* r) {
  if (r == nullptr) return;
  int prev = 0;
  const bool restore = cudaGetDevice(&prev) == cudaSuccess;
  cudaSetDevice(r->device);
  cudaDeviceSynchronize();
  drop_graphs(r);
  if (r->dbatch) cudaFree(r->dbatch);
  if (r->ws) cudaFree(r->ws);
  for (int s = 0; s < 2; ++s) {
    if (r->host[s]) cudaFreeHost(r->host[s]);
    if (r->copied[s]) cudaEventDestroy(r->copied[s]);
  }
  if (r->cap_stream) cudaStreamDestroy(r->cap_stream);
  delete r;
  if (restore) cudaSetDevice(prev);
}

extern "C" int ck_runner_stage(ck_runner* r, const void* nid, const void* tb, const void* val,
                               const void* bidx, int idx_dtype, int64_t E, int32_t batch_size,
                               int32_t* B_out) {
  if (r == nullptr || B_out == nullptr || E < 0) return CK_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> g(r->mu);
  if (cudaSetDevice(r->device) != cudaSuccess) return cuda_fail();
  const int64_t cap = bucket(E);
  int rc = reserve(r, cap);
  if (rc != CK_OK) return rc;
  const int s = r->next;
  if (r->used[s] && cudaEventSynchronize(r->copied[s]) != cudaSuccess) return cuda_fail();
  int32_t bmax = 0;
  rc = ck_batch_stage(nid, tb, val, bidx, idx_dtype, E, r->host[s], cap, &bmax);
  if (rc != CK_OK) return rc;
  r->staged_slot = s;
  r->staged_cap = cap;
  r->staged_b = batch_size > 0 ? batch_size : bmax;
  *B_out = r->staged_b;
  return CK_OK;
}

namespace {

// The forward of the batch in r->dbatch (capacity cap) through the graph of its
// bucket, output copied to behavior_out. Called with r->mu held.
int run_bucket(ck_runner* r, int64_t cap, int32_t B, void* behavior_out, cudaStream_t st) {
  int rc;
  const size_t out_bytes = (size_t)B * r->model.behavior_dim * elem_bytes(r->model);
  const auto key = std::make_pair(B, cap);
  auto it = r->graphs.find(key);
  if (it != r->graphs.end()) {
    it->second.used = ++r->tick;
    if (cudaGraphLaunch(it->second.exec, st) != cudaSuccess ||
        cudaMemcpyAsync(behavior_out, it->second.out, out_bytes, cudaMemcpyDeviceToDevice, st) !=
            cudaSuccess)
      return cuda_fail();
    ++r->replays;
    return CK_OK;
  }
  // First batch of this bucket: run it eagerly (its result, and any first-use
  // setup outside capture), then capture the same launches on the runner's
  // stream. A bucket whose capture fails keeps running eagerly.
  Graph gr;
  if (cudaMalloc(&gr.out, out_bytes) != cudaSuccess) return cuda_fail();
  rc = ck_forward_batch(&r->model, r->dbatch, cap, B, gr.out, r->ws, r->ws_bytes, st);
  if (rc != CK_OK) {
    cudaFree(gr.out);
    return rc;
  }
  if (cudaMemcpyAsync(behavior_out, gr.out, out_bytes, cudaMemcpyDeviceToDevice, st) !=
      cudaSuccess) {
    cudaFree(gr.out);
    return cuda_fail();
  }
  cudaGraph_t graph = nullptr;
  if (cudaStreamBeginCapture(r->cap_stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
    const int crc = ck_forward_batch(&r->model, r->dbatch, cap, B, gr.out, r->ws, r->ws_bytes,
                                     r->cap_stream);
    const cudaError_t e = cudaStreamEndCapture(r->cap_stream, &graph);
    if (crc == CK_OK && e == cudaSuccess && graph != nullptr &&
        cudaGraphInstantiate(&gr.exec, graph, 0) == cudaSuccess) {
      gr.used = ++r->tick;
      r->graphs[key] = gr;
      ++r->captures;
      gr.out = nullptr;
    }
    if (graph) cudaGraphDestroy(graph);
  }
  cudaGetLastError();  // a failed capture leaves no sticky state behind
  if (gr.out) {
    // the eager result is in flight on the caller's stream: free after it
    cudaStreamSynchronize(st);
    cudaFree(gr.out);
  }
  while (r->graphs.size() > r->max_graphs) {
    auto lru = r->graphs.begin();
    for (auto i = r->graphs.begin(); i != r->graphs.end(); ++i)
      if (i->second.used < lru->second.used) lru = i;
    cudaStreamSynchronize(st);
    cudaGraphExecDestroy(lru->second.exec);
    cudaFree(lru->second.out);
    r->graphs.erase(lru);
  }
  return CK_OK;
}

}  // namespace

extern "C" int ck_runner_launch(ck_runner* r, void* behavior_out, void* stream) {
  if (r == nullptr || behavior_out == nullptr) return CK_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> g(r->mu);
  if (r->staged_slot < 0) return CK_ERR_INVALID_ARG;
  if (cudaSetDevice(r->device) != cudaSuccess) return cuda_fail();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int s = r->staged_slot;
  const int64_t cap = r->staged_cap;
  const int32_t B = r->staged_b;
  r->staged_slot = -1;
  int rc = ensure_ws(r, cap, B);
  if (rc != CK_OK) return rc;
  const size_t words = (size_t)CK_BATCH_WORDS(cap);
  if (cudaMemcpyAsync(r->dbatch, r->host[s], words * 4, cudaMemcpyHostToDevice, st) !=
          cudaSuccess ||
      cudaEventRecord(r->copied[s], st) != cudaSuccess)
    return cuda_fail();
  r->used[s] = true;
  r->next = s ^ 1;
  return run_bucket(r, cap, B, behavior_out, st);
}

extern "C" int ck_runner_launch_batch(ck_runner* r, const int32_t* batch, int64_t capacity,
                                      int32_t B, void* behavior_out, void* stream) {
  if (r == nullptr || batch == nullptr || behavior_out == nullptr || B <= 0 || capacity < 0 ||
      capacity % 4 != 0)
    return CK_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> g(r->mu);
  if (cudaSetDevice(r->device) != cudaSuccess) return cuda_fail();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc = reserve(r, capacity);
  if (rc != CK_OK) return rc;
  rc = ensure_ws(r, capacity, B);
  if (rc != CK_OK) return rc;
  if (cudaMemcpyAsync(r->dbatch, batch, (size_t)CK_BATCH_WORDS(capacity) * 4,
                      cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return cuda_fail();
  return run_bucket(r, capacity, B, behavior_out, st);
}

extern "C" int ck_runner_invalidate(ck_runner* r, const ck_model* m) {
  if (r == nullptr) return CK_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> g(r->mu);
  if (cudaSetDevice(r->device) != cudaSuccess) return cuda_fail();
  if (cudaDeviceSynchronize() != cudaSuccess) return cuda_fail();
  drop_graphs(r);
  if (m != nullptr) {
    if (m->num_layers > 0 && m->blocks == nullptr) return CK_ERR_INVALID_ARG;
    r->model = *m;
    r->blocks.assign(m->blocks, m->blocks + (m->num_layers > 0 ? m->num_layers : 0));
    r->model.blocks = r->blocks.empty() ? nullptr : r->blocks.data();
  }
  return CK_OK;
}

extern "C" int ck_runner_counters(ck_runner* r, long long* captures, long long* replays) {
  if (r == nullptr || captures == nullptr || replays == nullptr) return CK_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> g(r->mu);
  *captures = r->captures;
  *replays = r->replays;
  return CK_OK;
}
