// Per-channel INT8 weight dequantisation, QuantizedLinear.forward's weight
// expression (cortex/quantization/calibrate.py:225-228):
//
//   W[n, k] = bf16(float(w_int8[n, k]) * scale[n])
//
// one fp32 product rounded once to bf16, as torch's (w.float() * s[:, None])
// .to(bfloat16) is. The forward dequantises every INT8 linear of the
// self-attention blocks once per call, on the side stream beside the packing
// and the tokenizer, and runs bf16 GEMMs on the result: each weight is widened
// once per forward instead of once per 128-row tile of activations inside the
// GEMM, and the GEMMs see the reference's own rounded weights.
//
// One launch covers up to kMaxSeg weight matrices (segments), walked as one
// flat space of 16-value chunks (one 16-byte load each). The work is HBM / L2
// bound: K bytes read and 2K bytes written per row.
#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

constexpr int kMaxSeg = 40;

struct DeqLaunch {
  DequantSeg seg[kMaxSeg];
  int64_t chunk_end[kMaxSeg];  // inclusive prefix of the segments' 16-byte chunks
  int nseg;
};

// int8 x 16 (one uint4) -> 16 fp32 values, exactly: the bf16 bit trick of
// i8x4_to_bf16x4 on the integer and half pipes, then bf16 -> fp32 by a shift,
// which keeps the conversion unit free for the final rounding.
__device__ __forceinline__ void i8x16(const uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t lo, hi;
    i8x4_to_bf16x4(w[i], lo, hi);
    f[4 * i] = __uint_as_float(lo << 16);
    f[4 * i + 1] = __uint_as_float(lo & 0xFFFF0000u);
    f[4 * i + 2] = __uint_as_float(hi << 16);
    f[4 * i + 3] = __uint_as_float(hi & 0xFFFF0000u);
  }
}

// The segments' 16-value chunks as one flat index space, kUnroll chunks per
// thread and step (independent loads in flight), consecutive threads on
// consecutive chunks of a row.
constexpr int kUnroll = 4;

__global__ void __launch_bounds__(256) dequant_kernel(const __grid_constant__ DeqLaunch a) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  const int64_t total = a.chunk_end[a.nseg - 1];
  int s = 0;  // a thread's chunks only grow
  for (int64_t c0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c0 < total;
       c0 += kUnroll * nthreads) {
    uint4 v[kUnroll];
    float sc[kUnroll];
    __nv_bfloat16* dst[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t c = c0 + u * nthreads;
      dst[u] = nullptr;
      if (c < total) {
        while (c >= a.chunk_end[s]) ++s;
        const DequantSeg& g = a.seg[s];
        const uint32_t q = (uint32_t)(c - (s > 0 ? a.chunk_end[s - 1] : 0));
        const uint32_t kc = (uint32_t)(g.K / 16);
        const uint32_t row = q / kc, col = q - row * kc;
        v[u] = __ldg(reinterpret_cast<const uint4*>(g.w + (int64_t)row * g.ldw) + col);
        sc[u] = __ldg(g.scale + row);
        dst[u] = reinterpret_cast<__nv_bfloat16*>(g.out) + (int64_t)row * g.ldo + 16 * col;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (dst[u] == nullptr) continue;
      float f[16];
      i8x16(v[u], f);
      const float k = sc[u];
      uint4* o = reinterpret_cast<uint4*>(dst[u]);
      o[0] = make_uint4(cvt_bf16x2(f[0] * k, f[1] * k), cvt_bf16x2(f[2] * k, f[3] * k),
                        cvt_bf16x2(f[4] * k, f[5] * k), cvt_bf16x2(f[6] * k, f[7] * k));
      o[1] = make_uint4(cvt_bf16x2(f[8] * k, f[9] * k), cvt_bf16x2(f[10] * k, f[11] * k),
                        cvt_bf16x2(f[12] * k, f[13] * k), cvt_bf16x2(f[14] * k, f[15] * k));
    }
  }
}

}  // namespace

bool dequant_seg_ok(const DequantSeg& g) {
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return g.w != nullptr && g.scale != nullptr && g.out != nullptr && g.N > 0 && g.K > 0 &&
         g.K % 16 == 0 && g.ldw >= g.K && g.ldo >= g.K && g.ldw % 16 == 0 && g.ldo % 8 == 0 &&
         al16(g.w) && al16(g.out) && g.N * (g.K / 16) < (int64_t(1) << 32);
}

int dequant_int8(const DequantSeg* segs, int n, cudaStream_t st) {
  for (int i0 = 0; i0 < n; i0 += kMaxSeg) {
    DeqLaunch a;
    a.nseg = n - i0 < kMaxSeg ? n - i0 : kMaxSeg;
    int64_t chunks = 0;
    for (int i = 0; i < a.nseg; ++i) {
      const DequantSeg& g = segs[i0 + i];
      if (!dequant_seg_ok(g)) return CK_ERR_INVALID_ARG;
      a.seg[i] = g;
      chunks += g.N * (g.K / 16);
      a.chunk_end[i] = chunks;
    }
    // a resident grid (8 CTAs of 256 threads per SM), fewer for small jobs
    int64_t blocks = (chunks + 256 * kUnroll - 1) / (256 * kUnroll);
    const int64_t cap = 8 * (int64_t)num_sms();
    if (blocks > cap) blocks = cap;
    const int rc = launch_pdl(dequant_kernel, dim3((unsigned)blocks), dim3(256), 0, st, a);
    if (rc != CK_OK) return rc;
  }
  return CK_OK;
}

}  // namespace ck
