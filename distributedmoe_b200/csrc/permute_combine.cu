// Bandwidth-bound row movers of the MoE layer: the segmented gather that fills an input
// buffer (dispatch) and the weighted un-permute that combines expert outputs per token.
//
// dispatch: HostPipelineTask.dispatch gathers input_batch[token_indexes] into
//           Buffer.data[offset : offset + n] per expert (MoE/PipelineTask.py:231-249).
// combine : HostPipelineTask.combine scatter-adds out_buf rows * weights into the output
//           batch per expert (MoE/PipelineTask.py:326-346).  Here each token gathers its k
//           expert rows instead, accumulates in fp32 and stores once: no atomics, and the
//           output is written exactly once.
// Both move 16-byte vectors, one warp per row (dispatch) or per token (combine).
#include "dmoe_common.cuh"

namespace dmoe {
namespace {

constexpr int kMaxSegs = 1024;

struct SegParams {
  int n_seg;
  int32_t row_start[kMaxSegs + 1];  // prefix of seg_len: first output row of each segment
  int32_t src[kMaxSegs];
  int32_t dst[kMaxSegs];
};

__global__ void __launch_bounds__(256) permute_rows_kernel(const char* __restrict__ src, char* __restrict__ dst,
                                                           int64_t row_vecs, const int32_t* __restrict__ row_map,
                                                           const __grid_constant__ SegParams p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int total = p.row_start[p.n_seg];
  for (int r = warp; r < total; r += nwarps) {
    // segment of row r: last s with row_start[s] <= r
    int lo = 0, hi = p.n_seg - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.row_start[mid] <= r) lo = mid; else hi = mid - 1;
    }
    const int off = r - p.row_start[lo];
    const int64_t srow = row_map ? (int64_t)row_map[p.src[lo] + off] : (int64_t)p.src[lo] + off;
    const int64_t drow = (int64_t)p.dst[lo] + off;
    const uint4* s = reinterpret_cast<const uint4*>(src) + srow * row_vecs;
    uint4* d = reinterpret_cast<uint4*>(dst) + drow * row_vecs;
    // Eight 16-byte loads in flight per lane before the stores (a 4096-wide bf16 row is
    // 16 vectors per lane).
    int64_t c = lane;
    for (; c + 224 < row_vecs; c += 256) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = s[c + 32 * u];
#pragma unroll
      for (int u = 0; u < 8; ++u) d[c + 32 * u] = v[u];
    }
    for (; c < row_vecs; c += 32) d[c] = s[c];
  }
}

template <int DT>
__device__ __forceinline__ void load8(const void* base, int64_t elem, float* f) {
  if constexpr (DT == DMOE_F32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + elem);
    const float4 a = p[0], b = p[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(base) + elem * 2);
    unpack8<DT>(v, f);
  }
}

template <int DT>
__device__ __forceinline__ void store8(void* base, int64_t elem, const float* f) {
  if constexpr (DT == DMOE_F32) {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + elem);
    p[0] = make_float4(f[0], f[1], f[2], f[3]);
    p[1] = make_float4(f[4], f[5], f[6], f[7]);
  } else {
    uint4 v;
    v.x = pack2<DT>(f[0], f[1]);
    v.y = pack2<DT>(f[2], f[3]);
    v.z = pack2<DT>(f[4], f[5]);
    v.w = pack2<DT>(f[6], f[7]);
    *reinterpret_cast<uint4*>(reinterpret_cast<char*>(base) + elem * 2) = v;
  }
}

constexpr int kCombineMaxK = 16;

// One 16-byte chunk (8 elements) of a row, raw: one uint4 for 16-bit types, two for fp32.
template <int DT>
struct Chunk {
  uint4 v[DT == DMOE_F32 ? 2 : 1];
};

template <int DT>
__device__ __forceinline__ Chunk<DT> load_chunk(const void* base, int64_t elem) {
  Chunk<DT> c;
  const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(base) + elem * (DT == DMOE_F32 ? 4 : 2));
  c.v[0] = p[0];
  if constexpr (DT == DMOE_F32) c.v[1] = p[1];
  return c;
}

template <int DT>
__device__ __forceinline__ void chunk_to_float(const Chunk<DT>& c, float* f) {
  if constexpr (DT == DMOE_F32) {
    f[0] = __uint_as_float(c.v[0].x); f[1] = __uint_as_float(c.v[0].y);
    f[2] = __uint_as_float(c.v[0].z); f[3] = __uint_as_float(c.v[0].w);
    f[4] = __uint_as_float(c.v[1].x); f[5] = __uint_as_float(c.v[1].y);
    f[6] = __uint_as_float(c.v[1].z); f[7] = __uint_as_float(c.v[1].w);
  } else {
    unpack8<DT>(c.v[0], f);
  }
}

// One warp per token.  KU bounds k at compile time; CU chunks per lane are in flight at once,
// with all k source rows of each loaded before any arithmetic, so a lane keeps KU x CU
// 16-byte loads outstanding (HBM wants many bytes in flight per SM, and a token's rows are
// only k x d x 2 bytes).
template <int DT, int KU, int CU>
__global__ void __launch_bounds__(256) combine_kernel(const void* __restrict__ rows, const int32_t* __restrict__ inverse,
                                                      const void* __restrict__ w, int w_dtype, int T, int k, int d,
                                                      int accumulate, void* __restrict__ out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int nchunk = d / 8;
  for (int t = warp; t < T; t += nwarps) {
    int64_t src[KU];
    float wt[KU];
#pragma unroll
    for (int s = 0; s < KU; ++s) {
      if (s < k) {
        // A negative position marks an activation without an expert row (an invalid expert
        // index in the plan): it is neither loaded nor added.
        const int32_t pos = inverse[(int64_t)t * k + s];
        src[s] = pos < 0 ? -1 : (int64_t)pos * d;
        wt[s] = pos < 0 ? 0.f : load_as_float(w, (int64_t)t * k + s, w_dtype);
      }
    }
    for (int c0 = lane; c0 < nchunk; c0 += 32 * CU) {
      Chunk<DT> raw[CU][KU];
#pragma unroll
      for (int u = 0; u < CU; ++u) {
        const int c = c0 + u * 32;
#pragma unroll
        for (int s = 0; s < KU; ++s)
          if (s < k && c < nchunk && src[s] >= 0) raw[u][s] = load_chunk<DT>(rows, src[s] + (int64_t)c * 8);
      }
#pragma unroll
      for (int u = 0; u < CU; ++u) {
        const int c = c0 + u * 32;
        if (c >= nchunk) break;
        float acc[8];
        if (accumulate) {
          load8<DT>(out, (int64_t)t * d + c * 8, acc);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        }
#pragma unroll
        for (int s = 0; s < KU; ++s) {
          if (s < k && src[s] >= 0) {
            float v[8];
            chunk_to_float<DT>(raw[u][s], v);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = fmaf(wt[s], v[j], acc[j]);
          }
        }
        store8<DT>(out, (int64_t)t * d + c * 8, acc);
      }
    }
  }
}

template <int DT>
void launch_combine(int blocks, cudaStream_t s, const void* rows, const int32_t* inverse, const void* w, int w_dtype,
                    int T, int k, int d, int accumulate, void* out) {
  if (k <= 2)
    combine_kernel<DT, 2, 4><<<blocks, 256, 0, s>>>(rows, inverse, w, w_dtype, T, k, d, accumulate, out);
  else if (k <= 4)
    combine_kernel<DT, 4, 2><<<blocks, 256, 0, s>>>(rows, inverse, w, w_dtype, T, k, d, accumulate, out);
  else if (k <= 8)
    combine_kernel<DT, 8, 1><<<blocks, 256, 0, s>>>(rows, inverse, w, w_dtype, T, k, d, accumulate, out);
  else
    combine_kernel<DT, 16, 1><<<blocks, 256, 0, s>>>(rows, inverse, w, w_dtype, T, k, d, accumulate, out);
}

}  // namespace
}  // namespace dmoe

using namespace dmoe;

extern "C" int dmoe_permute_rows(const void* src, void* dst, int64_t row_bytes, const int32_t* row_map,
                                 const int32_t* seg_src, const int32_t* seg_dst, const int32_t* seg_len, int n_seg,
                                 void* stream) {
  clear_error();
  DMOE_REQUIRE(n_seg >= 0 && n_seg <= kMaxSegs, "dmoe_permute_rows: n_seg=%d not in [0, %d]", n_seg, kMaxSegs);
  if (n_seg == 0) return DMOE_OK;
  DMOE_REQUIRE(src && dst && seg_src && seg_dst && seg_len, "dmoe_permute_rows: null pointer");
  DMOE_REQUIRE(row_bytes > 0 && row_bytes % 16 == 0, "dmoe_permute_rows: row_bytes=%lld must be a multiple of 16",
               (long long)row_bytes);
  DMOE_REQUIRE(aligned16(src) && aligned16(dst), "dmoe_permute_rows: src/dst must be 16-byte aligned");
  static thread_local SegParams p;
  p.n_seg = n_seg;
  int64_t total = 0;
  for (int i = 0; i < n_seg; ++i) {
    DMOE_REQUIRE(seg_len[i] >= 0 && seg_src[i] >= 0 && seg_dst[i] >= 0, "dmoe_permute_rows: negative segment %d", i);
    p.row_start[i] = (int32_t)total;
    p.src[i] = seg_src[i];
    p.dst[i] = seg_dst[i];
    total += seg_len[i];
  }
  DMOE_REQUIRE(total < (1ll << 31), "dmoe_permute_rows: too many rows");
  p.row_start[n_seg] = (int32_t)total;
  if (total == 0) return DMOE_OK;
  const int64_t warps_needed = total;
  int blocks = (int)((warps_needed + 7) / 8);
  if (blocks > 148 * 8) blocks = 148 * 8;
  permute_rows_kernel<<<blocks, 256, 0, as_stream(stream)>>>(reinterpret_cast<const char*>(src),
                                                             reinterpret_cast<char*>(dst), row_bytes / 16, row_map, p);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

extern "C" int dmoe_combine(const void* rows, const int32_t* inverse, const void* w, int w_dtype, int T, int k, int d,
                            int dtype, int accumulate, void* out, void* stream) {
  clear_error();
  DMOE_REQUIRE(T >= 0 && k >= 1 && k <= kCombineMaxK, "dmoe_combine: bad T=%d k=%d", T, k);
  DMOE_REQUIRE(d > 0 && d % 8 == 0, "dmoe_combine: d=%d must be a multiple of 8", d);
  DMOE_REQUIRE(dtype_ok(dtype) && dtype_ok(w_dtype), "dmoe_combine: bad dtype");
  if (T == 0) return DMOE_OK;
  DMOE_REQUIRE(rows && inverse && w && out, "dmoe_combine: null pointer");
  DMOE_REQUIRE(aligned16(rows) && aligned16(out), "dmoe_combine: rows/out must be 16-byte aligned");
  int blocks = (T + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  cudaStream_t s = as_stream(stream);
  if (dtype == DMOE_BF16)
    launch_combine<DMOE_BF16>(blocks, s, rows, inverse, w, w_dtype, T, k, d, accumulate, out);
  else if (dtype == DMOE_F16)
    launch_combine<DMOE_F16>(blocks, s, rows, inverse, w, w_dtype, T, k, d, accumulate, out);
  else
    launch_combine<DMOE_F32>(blocks, s, rows, inverse, w, w_dtype, T, k, d, accumulate, out);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}
