// Shared helpers of the sm_100a MoE-layer kernels: error reporting, dtype conversion,
// vector types.  Every .cu file of the library includes this header.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <mutex>
#include <cstdio>
#include <string>

#include "../../include/dmoe_b200.h"

namespace dmoe {

// ----------------------------------------------------------------------------- errors
void set_error(const char* fmt, ...);
void clear_error();
extern std::atomic<uint64_t> g_launches;

inline void count_launch(uint64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

#define DMOE_REQUIRE(cond, ...)                \
  do {                                         \
    if (!(cond)) {                             \
      ::dmoe::set_error(__VA_ARGS__);          \
      return DMOE_ERR_INVALID;                 \
    }                                          \
  } while (0)

#define DMOE_CUDA(call)                                                                         \
  do {                                                                                          \
    cudaError_t e_ = (call);                                                                    \
    if (e_ != cudaSuccess) {                                                                    \
      ::dmoe::set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
      return DMOE_ERR_CUDA;                                                                     \
    }                                                                                           \
  } while (0)

#define DMOE_LAUNCH_CHECK()                                                                      \
  do {                                                                                           \
    cudaError_t e_ = cudaGetLastError();                                                         \
    if (e_ != cudaSuccess) {                                                                     \
      ::dmoe::set_error("kernel launch failed: %s (%s:%d)", cudaGetErrorString(e_), __FILE__, __LINE__); \
      return DMOE_ERR_CUDA;                                                                      \
    }                                                                                            \
    ::dmoe::count_launch();                                                                      \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Per-device one-time set-up of a launch site (kernel attributes, occupancy queries), safe
// when several host threads make their first launch on a device at the same time: `init`
// runs once per device (< 64) and later calls see its effects.
struct PerDeviceOnce {
  std::mutex m;
  std::atomic<uint64_t> done{0};
};

template <class F>
int once_per_device(PerDeviceOnce& o, int dev, F&& init) {
  const uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0;
  if (bit && (o.done.load(std::memory_order_acquire) & bit)) return DMOE_OK;
  std::lock_guard<std::mutex> g(o.m);
  if (bit && (o.done.load(std::memory_order_relaxed) & bit)) return DMOE_OK;
  const int r = init();
  if (r == DMOE_OK && bit) o.done.fetch_or(bit, std::memory_order_release);
  return r;
}

// SMs the grouped-MLP launches leave free (dmoe_grouped_mlp_set_sm_reserve); short kernels that
// run beside them size their grids for those SMs.
int gemm_sm_reserve();

// Router logits for few tokens on the CUDA cores (router.cu); dmoe_router_logits uses it when
// T is small, where the tensor-core logits GEMM would run on one or two CTAs.
bool logits_few_tokens_eligible(int T, int d, int E);
int run_logits_few_tokens(const void* x, const void* w, int dtype, int T, int d, int E, float* out, cudaStream_t s);

inline int dtype_bytes(int dt) { return dt == DMOE_F32 ? 4 : 2; }
inline bool dtype_ok(int dt) { return dt == DMOE_F32 || dt == DMOE_F16 || dt == DMOE_BF16; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ----------------------------------------------------------------------------- device
__device__ __forceinline__ float load_as_float(const void* p, int64_t i, int dt) {
  if (dt == DMOE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == DMOE_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_from_float(void* p, int64_t i, float v, int dt) {
  if (dt == DMOE_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dt == DMOE_F16)
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}

// 8 x 16-bit values in one 16-byte vector -> 8 floats
template <int DT>
__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (DT == DMOE_BF16) {
      __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
      float2 t = __bfloat1622float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    } else {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 t = __half22float2(h);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
}

template <int DT>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (DT == DMOE_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// ----------------------------------------------------------------------------- async copies
// mbarrier + bulk async copy (global -> this CTA's shared memory) for kernels that stream
// contiguous rows through a shared-memory ring.  All waits are bounded by the caller.
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void bar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make barrier initialisation and earlier shared-memory accesses of this thread visible to
// the async proxy (bulk copies) before the next copy is issued.
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void bar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool bar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global memory
// into shared memory; completes on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_load(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace dmoe
