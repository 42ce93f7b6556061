// Routing plan: stable counting sort of the T*k activations by expert.
//
// Replaces the one-hot mask and the per-expert torch.where loop of
// MoE/DistMoEBlock.py:568-605.  torch.where(expert_mask[e]) on the [k, T] slice lists an
// expert's activations slot-major, then by ascending token.  Walking the activations in
// that flattened order f = s*T + t and sorting stably by expert reproduces it exactly, for
// all experts at once, without a host synchronisation per expert.
//
// Three launches:
//   1. plan_hist    : chunk c of the flattened order -> hist[c][e]        (smem atomics)
//   2. plan_scan    : counts, offsets, and base[c][e] = offsets[e] + sum_{c'<c} hist[c'][e]
//   3. plan_scatter : each chunk ranks its activations stably (warp match + per-warp
//                     prefix) and writes perm_token / perm_slot / inverse / perm_weight.
#include <cstdlib>
#include <mutex>

#include "dmoe_common.cuh"

namespace dmoe {
namespace {

constexpr int kChunk = 2048;       // activations per CTA
constexpr int kPlanThreads = 256;  // 8 warps
constexpr int kMaxPlanExperts = 1024;

__global__ void __launch_bounds__(kPlanThreads) plan_hist(const int64_t* idx, int T, int k, int E, int32_t* hist) {
  extern __shared__ int32_t s_hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_hist[e] = 0;
  __syncthreads();
  const int64_t n = (int64_t)T * k;
  const int64_t f0 = (int64_t)blockIdx.x * kChunk;
  for (int64_t f = f0 + threadIdx.x; f < f0 + kChunk && f < n; f += blockDim.x) {
    const int s = (int)(f / T), t = (int)(f % T);
    const int e = (int)idx[(int64_t)t * k + s];
    if (e >= 0 && e < E) atomicAdd(&s_hist[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[(int64_t)blockIdx.x * E + e] = s_hist[e];
}

// One CTA of up to 1024 threads; thread e owns expert e (loops if E > blockDim).
__global__ void plan_scan(int32_t* hist, int n_chunks, int E, int32_t* counts, int32_t* offsets) {
  __shared__ int32_t s_cnt[kMaxPlanExperts];
  __shared__ int32_t s_warp[32];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int32_t c = 0;
    for (int j = 0; j < n_chunks; ++j) c += hist[(int64_t)j * E + e];
    s_cnt[e] = c;
    counts[e] = c;
  }
  __syncthreads();
  // exclusive scan of s_cnt over E (E <= 1024 = blockDim): one value per thread
  const int e = threadIdx.x;
  int32_t v = e < E ? s_cnt[e] : 0;
  const int lane = e & 31, warp = e >> 5;
  int32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) / 32;
    int32_t w = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t u = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += u;
    }
    if (lane < nw) s_warp[lane] = w;
  }
  __syncthreads();
  const int32_t excl = incl - v + (warp > 0 ? s_warp[warp - 1] : 0);
  if (e < E) offsets[e] = excl;
  if (e == E - 1) offsets[E] = excl + v;
  __syncthreads();
  // base[c][e] = offsets[e] + sum_{c' < c} hist[c'][e]  (in place)
  for (int ee = threadIdx.x; ee < E; ee += blockDim.x) {
    int32_t run = offsets[ee];
    for (int j = 0; j < n_chunks; ++j) {
      const int32_t h = hist[(int64_t)j * E + ee];
      hist[(int64_t)j * E + ee] = run;
      run += h;
    }
  }
}

__global__ void __launch_bounds__(kPlanThreads) plan_scatter(const int64_t* idx, const void* w, int w_dtype, int T,
                                                             int k, int E, const int32_t* base, int32_t* perm_token,
                                                             int32_t* perm_slot, int32_t* inverse, void* perm_weight) {
  extern __shared__ int32_t smem[];
  int32_t* s_run = smem;                 // [E] running position of each expert in this chunk
  int32_t* s_wcnt = smem + E;            // [8][E] per-warp counts of the current round
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = kPlanThreads / 32;
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_run[e] = base[(int64_t)blockIdx.x * E + e];
  const int64_t n = (int64_t)T * k;
  const int64_t f0 = (int64_t)blockIdx.x * kChunk;
  for (int64_t r0 = f0; r0 < f0 + kChunk && r0 < n; r0 += kPlanThreads) {
    for (int i = threadIdx.x; i < nwarps * E; i += blockDim.x) s_wcnt[i] = 0;
    __syncthreads();
    const int64_t f = r0 + threadIdx.x;
    const bool valid = f < f0 + kChunk && f < n;
    int s = 0, t = 0, e = -1;
    if (valid) {
      s = (int)(f / T);
      t = (int)(f % T);
      e = (int)idx[(int64_t)t * k + s];
      if (e < 0 || e >= E) e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_in_warp = __popc(peers & ((1u << lane) - 1u));
    const int leader = __ffs(peers) - 1;
    if (e >= 0 && lane == leader) s_wcnt[warp * E + e] = __popc(peers);
    __syncthreads();
    if (valid && e < 0 && inverse) inverse[(int64_t)t * k + s] = -1;  // no expert: the combine skips it
    if (e >= 0) {
      int pos = s_run[e] + rank_in_warp;
      for (int w2 = 0; w2 < warp; ++w2) pos += s_wcnt[w2 * E + e];
      perm_token[pos] = t;
      if (perm_slot) perm_slot[pos] = s;
      if (inverse) inverse[(int64_t)t * k + s] = pos;
      if (perm_weight) {
        const float wv = load_as_float(w, (int64_t)t * k + s, w_dtype);
        store_from_float(perm_weight, pos, wv, w_dtype);
      }
    }
    __syncthreads();
    for (int ee = threadIdx.x; ee < E; ee += blockDim.x) {
      int32_t add = 0;
      for (int w2 = 0; w2 < nwarps; ++w2) add += s_wcnt[w2 * E + ee];
      s_run[ee] += add;
    }
    __syncthreads();
  }
}

// Small plans (T*k <= kSingleMax / 2 with E <= 64, T*k <= kSingleMax / 4 with E <= kSingleMaxE)
// in one CTA of 1024 threads, one launch instead of three: the expert of every activation is
// read once into shared memory (int16) while the histogram builds; one block-wide scan gives counts and offsets; then rounds of
// 1024 consecutive activations (in the slot-major order f = s*T + t) are ranked stably:
// within a warp by __match_any_sync, across the round's warps by a per-expert scan of the
// per-warp counts, and across rounds by a running position per expert.  The order is the
// multi-CTA path's, element for element.
constexpr int kSingleMax = 32768;
constexpr int kSingleMaxE = 256;
constexpr int kSingleThreads = 1024;

__global__ void __launch_bounds__(kSingleThreads, 1)
    plan_single(const int64_t* idx, const void* w, int w_dtype, int T, int k, int E, int32_t* counts,
                int32_t* offsets, int32_t* perm_token, int32_t* perm_slot, int32_t* inverse, void* perm_weight) {
  extern __shared__ __align__(16) int32_t sm[];
  int32_t* s_run = sm;                          // [E] running position of each expert
  const int ws = E + 1;                         // row stride of s_wc: a column walk hits 32 banks
  int32_t* s_wc = sm + kSingleMaxE;             // [32][E + 1] per-warp counts, then their prefixes
  const int n = T * k;
  const int na = (n + 15) & ~15;
  int16_t* s_e = reinterpret_cast<int16_t*>(s_wc + 32 * ws);  // [n] expert of each activation (-1: none)
  int16_t* s_pos = s_e + na;                                  // [n] position of activation f (-1: none)
  int16_t* s_tok = s_pos + na;                                // [n] token of position p
  int8_t* s_slot = reinterpret_cast<int8_t*>(s_tok + na);     // [n] slot of position p
  __shared__ int32_t s_warp[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E; e += kSingleThreads) s_run[e] = 0;
  __syncthreads();
  // 1. experts of all activations (eight loads in flight per thread) and the histogram
  for (int f0 = tid; f0 < n; f0 += 8 * kSingleThreads) {
    int64_t v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int f = f0 + u * kSingleThreads;
      v[u] = -1;
      if (f < n) {
        const int s = f / T, t = f - (f / T) * T;
        v[u] = idx[(int64_t)t * k + s];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int f = f0 + u * kSingleThreads;
      if (f < n) {
        const int e = (v[u] >= 0 && v[u] < E) ? (int)v[u] : -1;
        s_e[f] = (int16_t)e;
        if (e >= 0) atomicAdd(&s_run[e], 1);
      }
    }
  }
  __syncthreads();
  // 2. counts and exclusive offsets (E <= 1024: one expert per thread)
  const int32_t c = tid < E ? s_run[tid] : 0;
  int32_t incl = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int32_t wv = s_warp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t u = __shfl_up_sync(0xffffffffu, wv, o);
      if (lane >= o) wv += u;
    }
    s_warp[lane] = wv;
  }
  __syncthreads();
  const int32_t excl = incl - c + (warp > 0 ? s_warp[warp - 1] : 0);
  if (tid < E) {
    counts[tid] = c;
    offsets[tid] = excl;
    s_run[tid] = excl;
    if (tid == E - 1) offsets[E] = excl + c;
  }
  // 3. stable ranks, one round of 1024 consecutive activations at a time
  for (int r0 = 0; r0 < n; r0 += kSingleThreads) {
    for (int i = tid; i < 32 * ws; i += kSingleThreads) s_wc[i] = 0;
    __syncthreads();
    const int f = r0 + tid;
    const int e = f < n ? (int)s_e[f] : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_in_warp = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && lane == __ffs(peers) - 1) s_wc[warp * ws + e] = __popc(peers);
    __syncthreads();
    // per expert: exclusive scan of the 32 warps' counts, offset by the running position
    for (int ee = warp; ee < E; ee += 32) {
      const int32_t wc = s_wc[lane * ws + ee];
      int32_t in = wc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t u = __shfl_up_sync(0xffffffffu, in, o);
        if (lane >= o) in += u;
      }
      const int32_t run = s_run[ee];
      s_wc[lane * ws + ee] = run + in - wc;
      __syncwarp();
      if (lane == 31) s_run[ee] = run + in;
    }
    __syncthreads();
    if (f < n) {
      const int s = f / T, t = f - (f / T) * T;
      int pos = -1;
      if (e >= 0) {
        pos = s_wc[warp * ws + e] + rank_in_warp;
        s_tok[pos] = (int16_t)t;
        s_slot[pos] = (int8_t)s;
      }
      s_pos[f] = (int16_t)pos;
    }
    __syncthreads();
  }
  // 4. in-order (coalesced) stores from shared memory: by position, then by (token, slot)
  const int n_valid = s_run[E - 1];  // the last expert's running position is the end
  for (int p = tid; p < n_valid; p += kSingleThreads) {
    const int t = s_tok[p], s = s_slot[p];
    perm_token[p] = t;
    if (perm_slot) perm_slot[p] = s;
    if (perm_weight) store_from_float(perm_weight, p, load_as_float(w, (int64_t)t * k + s, w_dtype), w_dtype);
  }
  if (inverse) {
    for (int i = tid; i < n; i += kSingleThreads) {
      const int t = i / k, s = i - t * k;
      inverse[i] = s_pos[s * T + t];
    }
  }
}

size_t plan_single_smem(int T, int k, int E) {
  const size_t na = (size_t)(((int64_t)T * k + 15) & ~int64_t(15));
  return (size_t)(kSingleMaxE + 32 * (E + 1)) * sizeof(int32_t) + 7 * na;  // expert, position, token, slot
}

bool plan_single_eligible(int T, int k, int E) {
  const char* v = getenv("DMOE_PLAN_SINGLE");
  if (v && v[0] == '0') return false;
  // One CTA ranks 1024 activations per round and scans E experts per round: many experts
  // and many rounds (DeepSeek's 256 experts at 32768 activations) cost more than the three
  // grid-wide launches of the multi-CTA path.
  const int64_t n = (int64_t)T * k;
  return E <= kSingleMaxE && n <= (E <= 64 ? kSingleMax / 2 : kSingleMax / 4);
}

// Few experts (E <= 16, T*k <= 32768: Mixtral-style routing) in one CTA with one ranking
// pass instead of rounds: thread j owns the contiguous activations [j*c, (j+1)*c) of the
// slot-major order (c = ceil(T*k / 1024)).  Each thread counts its activations per expert
// in 16-bit fields packed four to a 64-bit word (no field can exceed T*k <= 32768), one
// block-wide exclusive scan of the four words gives every thread the number of earlier
// activations of each expert, and the thread walks its activations again assigning
// positions offset[e] + earlier[e] + running count.  Same order as the other paths.  The
// results are assembled in shared memory (token and slot by position, position by
// activation) and written out in order at the end: one SM's scattered 4-byte stores to
// global memory, not its arithmetic, bound the one-CTA plans.
constexpr int kFewMaxE = 16;
constexpr int kFewMax = 32768;
constexpr int kFewThreads = 1024;

// NW 64-bit words of four 16-bit fields each (experts 4q .. 4q+3 in word q).
template <int NW>
__device__ __forceinline__ uint64_t pick4(const uint64_t (&v)[NW], int q) {
  uint64_t r = v[0];
#pragma unroll
  for (int i = 1; i < NW; ++i) r = (q == i) ? v[i] : r;
  return r;
}

template <int NW>
__device__ __forceinline__ void add4(uint64_t (&v)[NW], int e, uint64_t amount) {
  const int q = e >> 2;
  const uint64_t inc = amount << ((e & 3) * 16);
#pragma unroll
  for (int i = 0; i < NW; ++i) v[i] += (q == i) ? inc : 0ull;
}

template <int NW>
__device__ __forceinline__ int field4(const uint64_t (&v)[NW], int e) {
  return (int)((pick4<NW>(v, e >> 2) >> ((e & 3) * 16)) & 0xffffu);
}

// floor(f / T) for 0 <= f, T <= 32768 without a division: m = ceil(2^32 / T) makes
// f * m / 2^32 = (f / T)(1 + eps) with eps < T / 2^32, so the error stays below 2^-17 while
// the fractional part of f / T is at most 1 - 1/T <= 1 - 2^-15.
// T = 1 (m would be 2^32) is marked by m = 0.
__device__ __forceinline__ uint32_t div_magic(uint32_t T) {
  return T <= 1 ? 0u : (uint32_t)((0x100000000ull + T - 1) / T);
}
__device__ __forceinline__ int div_small(int f, uint32_t m) { return m ? (int)__umulhi((uint32_t)f, m) : f; }

size_t plan_few_smem(int64_t n) {
  const size_t na = (size_t)((n + 15) & ~int64_t(15));
  return 6 * na;  // expert and slot (int8), position and token (int16) per activation
}

template <int NW>
__global__ void __launch_bounds__(kFewThreads, 1)
    plan_few_experts(const int64_t* __restrict__ idx, const void* __restrict__ w, int w_dtype, int T, int k, int E,
                     int32_t* __restrict__ counts, int32_t* __restrict__ offsets, int32_t* __restrict__ perm_token,
                     int32_t* __restrict__ perm_slot, int32_t* __restrict__ inverse, void* __restrict__ perm_weight) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  __shared__ uint64_t s_warp[32][NW];
  __shared__ uint64_t s_total[NW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = T * k;
  const int na = (n + 15) & ~15;
  int8_t* s_ex = reinterpret_cast<int8_t*>(sm_raw);             // [n] expert of activation f (-1: none)
  int8_t* s_slot = s_ex + na;                                    // [n] slot of position p
  int16_t* s_pos = reinterpret_cast<int16_t*>(s_slot + na);      // [n] position of activation f (-1: none)
  int16_t* s_tok = s_pos + na;                                   // [n] token of position p
  const uint32_t mT = div_magic((uint32_t)T), mk = div_magic((uint32_t)k);
  // 1. experts of all activations, coalesced over tokens (eight loads in flight per thread)
  for (int f0 = tid; f0 < n; f0 += 8 * kFewThreads) {
    int64_t v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int f = f0 + u * kFewThreads;
      v[u] = -1;
      if (f < n) {
        const int s = div_small(f, mT), t = f - s * T;
        v[u] = idx[(int64_t)t * k + s];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int f = f0 + u * kFewThreads;
      if (f < n) s_ex[f] = (int8_t)((v[u] >= 0 && v[u] < E) ? (int)v[u] : -1);
    }
  }
  __syncthreads();
  // 2. counts of this thread's chunk, then a block-wide exclusive scan of the packed words
  const int c = (n + kFewThreads - 1) / kFewThreads;
  const int lo = min(n, tid * c), hi = min(n, lo + c);
  uint64_t cnt[NW];
#pragma unroll
  for (int q = 0; q < NW; ++q) cnt[q] = 0;
  for (int f = lo; f < hi; ++f) {
    const int e = s_ex[f];
    if (e >= 0) add4<NW>(cnt, e, 1);
  }
  uint64_t incl[NW];
#pragma unroll
  for (int q = 0; q < NW; ++q) {
    incl[q] = cnt[q];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t u = __shfl_up_sync(0xffffffffu, incl[q], o);
      if (lane >= o) incl[q] += u;
    }
  }
  if (lane == 31)
#pragma unroll
    for (int q = 0; q < NW; ++q) s_warp[warp][q] = incl[q];
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int q = 0; q < NW; ++q) {
      uint64_t wv = s_warp[lane][q];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint64_t u = __shfl_up_sync(0xffffffffu, wv, o);
        if (lane >= o) wv += u;
      }
      s_warp[lane][q] = wv;  // inclusive over warps
      if (lane == 31) s_total[q] = wv;
    }
  }
  __syncthreads();
  uint64_t base[NW], tot[NW];
#pragma unroll
  for (int q = 0; q < NW; ++q) {
    base[q] = incl[q] - cnt[q] + (warp > 0 ? s_warp[warp - 1][q] : 0ull);
    tot[q] = s_total[q];
  }
  int run = 0;
  for (int e = 0; e < E; ++e) {
    const int ce = field4<NW>(tot, e);
    add4<NW>(base, e, (uint64_t)run);  // base[e] = offsets[e] + earlier activations of e
    if (tid == e) {
      counts[e] = ce;
      offsets[e] = run;
    }
    run += ce;
  }
  if (tid == 0) offsets[E] = run;
  // 3. positions, in order within the chunk, into shared memory
  int cs = div_small(lo, mT), ct = lo - cs * T;  // (slot, token) of activation f, stepped with f
  for (int f = lo; f < hi; ++f) {
    const int e = s_ex[f];
    int pos = -1;
    if (e >= 0) {
      pos = field4<NW>(base, e);
      add4<NW>(base, e, 1);
      s_tok[pos] = (int16_t)ct;
      s_slot[pos] = (int8_t)cs;
    }
    s_pos[f] = (int16_t)pos;
    if (++ct == T) {
      ct = 0;
      ++cs;
    }
  }
  __syncthreads();
  // 4. in-order (coalesced) stores: by position, then by (token, slot)
  for (int p = tid; p < run; p += kFewThreads) {
    const int t = s_tok[p], s = s_slot[p];
    perm_token[p] = t;
    if (perm_slot) perm_slot[p] = s;
    if (perm_weight) store_from_float(perm_weight, p, load_as_float(w, (int64_t)t * k + s, w_dtype), w_dtype);
  }
  if (inverse) {
    for (int i = tid; i < n; i += kFewThreads) {
      const int t = div_small(i, mk), s = i - t * k;
      inverse[i] = s_pos[s * T + t];
    }
  }
}

template <int NW>
int launch_plan_few(cudaStream_t s, const int64_t* idx, const void* w, int w_dtype, int T, int k, int E,
                    int32_t* counts, int32_t* offsets, int32_t* perm_token, int32_t* perm_slot, int32_t* inverse,
                    void* perm_weight) {
  static PerDeviceOnce once;
  int dev = 0;
  DMOE_CUDA(cudaGetDevice(&dev));
  const int r = once_per_device(once, dev, [] {
    DMOE_CUDA(cudaFuncSetAttribute(plan_few_experts<NW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)plan_few_smem(kFewMax)));
    return DMOE_OK;
  });
  if (r) return r;
  plan_few_experts<NW><<<1, kFewThreads, plan_few_smem((int64_t)T * k), s>>>(idx, w, w_dtype, T, k, E, counts, offsets,
                                                                              perm_token, perm_slot, inverse,
                                                                              perm_weight);
  return DMOE_OK;
}

bool plan_few_eligible(int T, int k, int E) {
  const char* v = getenv("DMOE_PLAN_FEW");
  if (v && v[0] == '0') return false;
  return E <= kFewMaxE && (int64_t)T * k <= kFewMax;
}

// Scratch of dmoe_route_plan_noalloc: the per-chunk histogram matrix lives in this
// library-owned device array instead of caller memory.  Every GPU that loads the library
// holds it until the process exits.
constexpr size_t kNoAllocScratchBytes = 512 * 1024;
static __device__ __align__(256) int32_t g_plan_scratch[kNoAllocScratchBytes / sizeof(int32_t)];

// The array's name in host code is a host-side stand-in, not a device address; the device
// address comes from cudaGetSymbolAddress, once per device, with that device current.
int32_t* plan_scratch_address(int* rc) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static int32_t* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("dmoe_route_plan_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
    *rc = DMOE_ERR_CUDA;
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("dmoe_route_plan_noalloc: device index %d is outside the %d devices this entry point serves", dev,
              kMaxDevices);
    *rc = DMOE_ERR_INVALID;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_plan_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("dmoe_route_plan_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev, cudaGetErrorString(e));
      *rc = DMOE_ERR_CUDA;
      return nullptr;
    }
    addr[dev] = reinterpret_cast<int32_t*>(p);
  }
  return addr[dev];
}

}  // namespace
}  // namespace dmoe

using namespace dmoe;

extern "C" size_t dmoe_route_plan_workspace_size(int T, int k, int E) {
  const int64_t n = (int64_t)T * k;
  const int64_t chunks = n > 0 ? (n + kChunk - 1) / kChunk : 1;
  return (size_t)(chunks * (int64_t)E * sizeof(int32_t));
}

extern "C" int dmoe_route_plan(const int64_t* idx, const void* w, int w_dtype, int T, int k, int E, int32_t* counts,
                               int32_t* offsets, int32_t* perm_token, int32_t* perm_slot, int32_t* inverse,
                               void* perm_weight, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  DMOE_REQUIRE(E >= 1 && E <= kMaxPlanExperts, "dmoe_route_plan: need 1 <= E <= %d (E=%d)", kMaxPlanExperts, E);
  DMOE_REQUIRE(T >= 0 && k >= 1 && (int64_t)T * k < (1ll << 31), "dmoe_route_plan: bad T=%d k=%d", T, k);
  DMOE_REQUIRE(counts && offsets && perm_token && workspace, "dmoe_route_plan: null pointer");
  DMOE_REQUIRE(perm_weight == nullptr || (w != nullptr && dtype_ok(w_dtype)), "dmoe_route_plan: perm_weight needs w");
  DMOE_REQUIRE(workspace_bytes >= dmoe_route_plan_workspace_size(T, k, E), "dmoe_route_plan: workspace too small");
  cudaStream_t s = as_stream(stream);
  const int64_t n = (int64_t)T * k;
  if (n > 0 && plan_few_eligible(T, k, E)) {
    const int nw = (E + 3) / 4;
    int r = DMOE_OK;
    if (nw == 1) r = launch_plan_few<1>(s, idx, w, w_dtype, T, k, E, counts, offsets, perm_token, perm_slot, inverse,
                                        perm_weight);
    else if (nw == 2) r = launch_plan_few<2>(s, idx, w, w_dtype, T, k, E, counts, offsets, perm_token, perm_slot,
                                             inverse, perm_weight);
    else r = launch_plan_few<4>(s, idx, w, w_dtype, T, k, E, counts, offsets, perm_token, perm_slot, inverse,
                                perm_weight);
    if (r) return r;
    DMOE_LAUNCH_CHECK();
    return DMOE_OK;
  }
  if (plan_single_eligible(T, k, E)) {
    static PerDeviceOnce once;
    int dev = 0;
    DMOE_CUDA(cudaGetDevice(&dev));
    const int r = once_per_device(once, dev, [] {
      DMOE_CUDA(cudaFuncSetAttribute(plan_single, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)plan_single_smem(kSingleMax / 2, 1, 64)));
      return DMOE_OK;
    });
    if (r) return r;
    plan_single<<<1, kSingleThreads, plan_single_smem(T, k, E), s>>>(idx, w, w_dtype, T, k, E, counts, offsets,
                                                                      perm_token, perm_slot, inverse, perm_weight);
    DMOE_LAUNCH_CHECK();
    return DMOE_OK;
  }
  const int chunks = n > 0 ? (int)((n + kChunk - 1) / kChunk) : 0;
  int32_t* hist = reinterpret_cast<int32_t*>(workspace);
  if (chunks > 0) {
    plan_hist<<<chunks, kPlanThreads, E * sizeof(int32_t), s>>>(idx, T, k, E, hist);
    DMOE_LAUNCH_CHECK();
  }
  const int scan_threads = E <= 32 ? 32 : ((E + 31) / 32) * 32;
  plan_scan<<<1, scan_threads, 0, s>>>(hist, chunks, E, counts, offsets);
  DMOE_LAUNCH_CHECK();
  if (chunks > 0) {
    const size_t smem = (size_t)E * sizeof(int32_t) * (1 + kPlanThreads / 32);
    if (smem > 48 * 1024)
      DMOE_CUDA(cudaFuncSetAttribute(plan_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    plan_scatter<<<chunks, kPlanThreads, smem, s>>>(idx, w, w_dtype, T, k, E, hist, perm_token, perm_slot, inverse,
                                                    perm_weight);
    DMOE_LAUNCH_CHECK();
  }
  return DMOE_OK;
}

extern "C" int dmoe_route_plan_noalloc(const int64_t* idx, const void* w, int w_dtype, int T, int k, int E,
                                       int32_t* counts, int32_t* offsets, int32_t* perm_token, int32_t* perm_slot,
                                       int32_t* inverse, void* perm_weight, void* stream) {
  clear_error();
  DMOE_REQUIRE(E >= 1 && E <= kMaxPlanExperts, "dmoe_route_plan_noalloc: need 1 <= E <= %d (E=%d)", kMaxPlanExperts, E);
  DMOE_REQUIRE(T >= 0 && k >= 1 && (int64_t)T * k < (1ll << 31), "dmoe_route_plan_noalloc: bad T=%d k=%d", T, k);
  const size_t need = dmoe_route_plan_workspace_size(T, k, E);
  DMOE_REQUIRE(need <= kNoAllocScratchBytes,
               "dmoe_route_plan_noalloc: T*k=%lld with E=%d needs %zu bytes of scratch, more than the library's "
               "static %zu bytes; use dmoe_route_plan with a caller workspace",
               (long long)T * k, E, need, kNoAllocScratchBytes);
  int rc = DMOE_OK;
  int32_t* scratch = plan_scratch_address(&rc);
  if (scratch == nullptr) return rc;
  // plan_hist writes every histogram entry it later reads, so the shared scratch needs no clearing.
  return dmoe_route_plan(idx, w, w_dtype, T, k, E, counts, offsets, perm_token, perm_slot, inverse, perm_weight,
                         scratch, kNoAllocScratchBytes, stream);
}
