// Row-wise e4m3 quantisation for the 8-bit expert GEMM.
//
// Each row r of x [rows, cols] (f16/bf16/f32) becomes q[r, :] = rn_satfinite(x[r, :] / s[r]) in
// e4m3 with s[r] = amax(|x[r, :]|) / 448 (448 = the largest finite e4m3), s[r] = 1 for an
// all-zero row.  q's rows are q_ld bytes apart and the scales scale_ld floats apart, so a row
// and its scale can share one record (d codes, then the scale: the receive rows of an 8-bit
// exchange window).  Rows of activations give per-token scales; rows of an expert's gate or
// up weight [E, I, d] viewed as [E * I, d] give per-output-channel scales.  The reference's
// benchmark casts the whole layer to an 8-bit float with no scale (precision "fp8",
// src/python/MoE/benchmarks/bench.py:184-185); per-row scales keep the 8-bit storage and the
// 8-bit tensor-core kind while the products stay within a few percent of 16-bit ones.
//
// One warp per row, 16-byte loads: the first pass finds amax, the second (an L1/L2 hit)
// converts.  HBM-bound: (input bytes + 1) per element.

#include <cuda_fp8.h>

#include "dmoe_common.cuh"

namespace dmoe {
namespace {

constexpr int kQuantWarps = 8;

template <int DT>
__device__ __forceinline__ void load8(const void* base, int64_t i, float* f) {
  if constexpr (DT == DMOE_F32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i);
    const float4 a = __ldg(p), b = __ldg(p + 1);
    f[0] = a.x;
    f[1] = a.y;
    f[2] = a.z;
    f[3] = a.w;
    f[4] = b.x;
    f[5] = b.y;
    f[6] = b.z;
    f[7] = b.w;
  } else {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(base) + i * 2));
    unpack8<DT>(v, f);
  }
}

template <int DT>
__global__ void __launch_bounds__(kQuantWarps * 32)
    quantize_rows_e4m3_kernel(const void* __restrict__ x, int64_t rows, int cols, uint8_t* __restrict__ q,
                              int64_t q_ld, float* __restrict__ scale, int64_t scale_ld) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kQuantWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t base = row * cols;
  float amax = 0.f;
  for (int c = lane * 8; c < cols; c += 256) {
    float f[8];
    load8<DT>(x, base + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  // fmaxf prefers a number to NaN: a row of NaN gets scale 1 and NaN codes.
  const float s = amax > 0.f ? amax / 448.f : 1.f;
  if (lane == 0) scale[row * scale_ld] = s;
  for (int c = lane * 8; c < cols; c += 256) {
    float f[8];
    load8<DT>(x, base + c, f);
    uint32_t w[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
          make_float2(__fdiv_rn(f[4 * h], s), __fdiv_rn(f[4 * h + 1], s)), __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
          make_float2(__fdiv_rn(f[4 * h + 2], s), __fdiv_rn(f[4 * h + 3], s)), __NV_SATFINITE, __NV_E4M3);
      w[h] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint2*>(q + row * q_ld + c) = make_uint2(w[0], w[1]);
  }
}

}  // namespace
}  // namespace dmoe

using namespace dmoe;

extern "C" int dmoe_quantize_rows_e4m3(const void* x, int dtype, int64_t rows, int cols, void* q, int64_t q_ld,
                                       float* scale, int64_t scale_ld, void* stream) {
  clear_error();
  DMOE_REQUIRE(dtype_ok(dtype), "dmoe_quantize_rows_e4m3: dtype must be f32, f16 or bf16");
  DMOE_REQUIRE(rows >= 0 && cols > 0 && cols % 16 == 0, "dmoe_quantize_rows_e4m3: cols=%d must be a multiple of 16",
               cols);
  if (rows == 0) return DMOE_OK;
  DMOE_REQUIRE(x && q && scale, "dmoe_quantize_rows_e4m3: null pointer");
  DMOE_REQUIRE(aligned16(x) && aligned16(q), "dmoe_quantize_rows_e4m3: x and q must be 16-byte aligned");
  DMOE_REQUIRE(q_ld >= cols && q_ld % 16 == 0 && scale_ld >= 1,
               "dmoe_quantize_rows_e4m3: q_ld=%lld must be >= cols and a multiple of 16, scale_ld=%lld >= 1",
               (long long)q_ld, (long long)scale_ld);
  DMOE_REQUIRE((reinterpret_cast<uintptr_t>(scale) & 3u) == 0, "dmoe_quantize_rows_e4m3: scale must be 4-byte aligned");
  DMOE_REQUIRE(rows <= (int64_t)INT32_MAX * kQuantWarps, "dmoe_quantize_rows_e4m3: %lld rows", (long long)rows);
  const unsigned grid = (unsigned)((rows + kQuantWarps - 1) / kQuantWarps);
  cudaStream_t s = as_stream(stream);
  uint8_t* qb = reinterpret_cast<uint8_t*>(q);
  if (dtype == DMOE_BF16)
    quantize_rows_e4m3_kernel<DMOE_BF16><<<grid, kQuantWarps * 32, 0, s>>>(x, rows, cols, qb, q_ld, scale, scale_ld);
  else if (dtype == DMOE_F16)
    quantize_rows_e4m3_kernel<DMOE_F16><<<grid, kQuantWarps * 32, 0, s>>>(x, rows, cols, qb, q_ld, scale, scale_ld);
  else
    quantize_rows_e4m3_kernel<DMOE_F32><<<grid, kQuantWarps * 32, 0, s>>>(x, rows, cols, qb, q_ld, scale, scale_ld);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}
