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
// One launch covers up to kMaxSeg weight matrices (segments); a warp walks a
// row at a time, 16 int8 values (one 16-byte load) per lane and step. The
// work is HBM / L2 bound: K bytes read and 2K bytes written per row.
#include "common.cuh"
#include "kernels.h"

namespace ck {

namespace {

constexpr int kMaxSeg = 40;

struct DeqLaunch {
  DequantSeg seg[kMaxSeg];
  int64_t row_end[kMaxSeg];  // exclusive prefix of the segments' rows
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

__global__ void __launch_bounds__(256) dequant_kernel(const __grid_constant__ DeqLaunch a) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t rows = a.row_end[a.nseg - 1];
  int s = 0;
  for (int64_t r = warp; r < rows; r += nwarps) {
    while (r >= a.row_end[s]) ++s;  // rows only grow for a warp
    const DequantSeg& g = a.seg[s];
    const int64_t n = r - (s > 0 ? a.row_end[s - 1] : 0);
    const float sc = g.scale[n];
    const uint4* src = reinterpret_cast<const uint4*>(g.w + n * g.ldw);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(g.out) + n * g.ldo);
    for (int64_t c = lane; c < g.K / 16; c += 32) {
      float f[16];
      i8x16(__ldg(src + c), f);
      dst[2 * c] = make_uint4(cvt_bf16x2(f[0] * sc, f[1] * sc), cvt_bf16x2(f[2] * sc, f[3] * sc),
                              cvt_bf16x2(f[4] * sc, f[5] * sc), cvt_bf16x2(f[6] * sc, f[7] * sc));
      dst[2 * c + 1] =
          make_uint4(cvt_bf16x2(f[8] * sc, f[9] * sc), cvt_bf16x2(f[10] * sc, f[11] * sc),
                     cvt_bf16x2(f[12] * sc, f[13] * sc), cvt_bf16x2(f[14] * sc, f[15] * sc));
    }
  }
}

}  // namespace

bool dequant_seg_ok(const DequantSeg& g) {
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return g.w != nullptr && g.scale != nullptr && g.out != nullptr && g.N > 0 && g.K > 0 &&
         g.K % 16 == 0 && g.ldw >= g.K && g.ldo >= g.K && g.ldw % 16 == 0 && g.ldo % 8 == 0 &&
         al16(g.w) && al16(g.out);
}

int dequant_int8(const DequantSeg* segs, int n, cudaStream_t st) {
  for (int i0 = 0; i0 < n; i0 += kMaxSeg) {
    DeqLaunch a;
    a.nseg = n - i0 < kMaxSeg ? n - i0 : kMaxSeg;
    int64_t rows = 0;
    for (int i = 0; i < a.nseg; ++i) {
      const DequantSeg& g = segs[i0 + i];
      if (!dequant_seg_ok(g)) return CK_ERR_INVALID_ARG;
      a.seg[i] = g;
      rows += g.N;
      a.row_end[i] = rows;
    }
    // a resident grid (8 CTAs of 8 warps per SM), fewer for small jobs
    int64_t blocks = (rows + 7) / 8;
    const int64_t cap = 8 * (int64_t)num_sms();
    if (blocks > cap) blocks = cap;
    const int rc = launch_pdl(dequant_kernel, dim3((unsigned)blocks), dim3(256), 0, st, a);
    if (rc != CK_OK) return rc;
  }
  return CK_OK;
}

}  // namespace ck
