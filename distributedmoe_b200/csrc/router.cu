// Router: fp32 logits, softmax (or sigmoid + group-limited) top-k, routing weights.
//
// Replaces MoE/DistMoEBlock.py:556-562 of the reference:
//   router_logits = self.gate(x); routing_weights = softmax(logits, dim=1, dtype=float)
//   routing_weights, selected = torch.topk(routing_weights, top_k); .to(dtype)
// One warp owns one token: the dot products with the E router rows are split over the
// lanes in 16-byte chunks of the token's row and reduced with shuffles; selection is k
// rounds of a warp arg-max (ties resolve to the lower expert index).
#include <cstdlib>

#include "dmoe_common.cuh"

namespace dmoe {
namespace {

constexpr int kRouterWarps = 8;
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 16;
constexpr int kExpertGroup = 8;  // experts whose dot products one pass over the row computes
constexpr int kRowBatch = 4;     // row vectors a lane loads at once

template <int DT>
struct VecTraits {
  static constexpr int kElems = 8;
};
template <>
struct VecTraits<DMOE_F32> {
  static constexpr int kElems = 4;
};

template <int DT>
__device__ __forceinline__ void load_vec(const void* base, int64_t elem_off, float* f) {
  const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(base) + elem_off * (DT == DMOE_F32 ? 4 : 2));
  if constexpr (DT == DMOE_F32) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  } else {
    unpack8<DT>(v, f);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Selection order of (value, index): NaN ranks above every number (torch.topk treats NaN
// as the largest value), then larger values, then the lower index.  Every available expert
// beats the empty candidate (-inf, 0x7fffffff), so each pick is an index in [0, E).
__device__ __forceinline__ bool ranks_before(float v, int i, float ov, int oi) {
  const bool n = v != v, on = ov != ov;
  if (n != on) return n;
  if (!n && v != ov) return v > ov;
  return i < oi;
}

// Arg-max over the warp of (value, index) in the order of ranks_before.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ranks_before(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
}

struct RouterArgs {
  const void* x;
  const void* w_r;
  const float* logit_bias;
  const float* score_bias;
  const float* logits_in;
  float* logits_out;
  int64_t* idx_out;
  void* w_out;
  int T, d, E, k, mode, renormalize, n_group, topk_group, w_dtype;
  float scale;
};

// With W_SMEM the block first copies the router weights (E x d, at most kWSmemMax bytes) into
// shared memory: every warp then reads them from there instead of re-fetching the whole
// matrix through L1/L2 for each of its tokens, and the kernel streams only x from HBM.
constexpr int kWSmemMax = 96 * 1024;

template <int DT, bool W_SMEM>
__global__ void __launch_bounds__(kRouterWarps * 32) router_kernel(RouterArgs a) {
  __shared__ float s_logit[kRouterWarps][kMaxExperts];
  __shared__ float s_gscore[kRouterWarps][32];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = a.E;
  constexpr int VE = VecTraits<DT>::kElems;
  const int nvec = a.d / VE;
  const void* wsrc = a.w_r;
  if constexpr (W_SMEM) {
    extern __shared__ uint4 s_w[];
    const int n16 = (int)((int64_t)a.E * a.d * (DT == DMOE_F32 ? 4 : 2) / 16);
    const uint4* g = reinterpret_cast<const uint4*>(a.w_r);
    int i = threadIdx.x;
    for (; i + 7 * (int)blockDim.x < n16; i += 8 * blockDim.x) {  // eight loads in flight per thread
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = g[i + u * blockDim.x];
#pragma unroll
      for (int u = 0; u < 8; ++u) s_w[i + u * blockDim.x] = v[u];
    }
    for (; i < n16; i += blockDim.x) s_w[i] = g[i];
    __syncthreads();
    wsrc = s_w;
  }

  for (int t = blockIdx.x * kRouterWarps + warp; t < a.T; t += gridDim.x * kRouterWarps) {
    // ---------------------------------------------------------------- logits
    if (a.logits_in != nullptr) {
      for (int e = lane; e < E; e += 32) s_logit[warp][e] = a.logits_in[(int64_t)t * E + e];
    } else {
      for (int e0 = 0; e0 < E; e0 += kExpertGroup) {
        float acc[kExpertGroup];
#pragma unroll
        for (int i = 0; i < kExpertGroup; ++i) acc[i] = 0.f;
        // kRowBatch vectors of the token's row per lane are loaded before any arithmetic, so
        // a lane keeps that many HBM reads in flight instead of one.
        for (int c0 = lane; c0 < nvec; c0 += 32 * kRowBatch) {
          float xv[kRowBatch][VE];
#pragma unroll
          for (int u = 0; u < kRowBatch; ++u) {
            const int c = c0 + 32 * u;
            if (c < nvec) {
              load_vec<DT>(a.x, (int64_t)t * a.d + (int64_t)c * VE, xv[u]);
            } else {
#pragma unroll
              for (int j = 0; j < VE; ++j) xv[u][j] = 0.f;
            }
          }
#pragma unroll
          for (int u = 0; u < kRowBatch; ++u) {
            const int c = c0 + 32 * u;
            if (c >= nvec) break;
#pragma unroll
            for (int i = 0; i < kExpertGroup; ++i) {
              if (e0 + i < E) {
                float wv[VE];
                load_vec<DT>(wsrc, (int64_t)(e0 + i) * a.d + (int64_t)c * VE, wv);
#pragma unroll
                for (int j = 0; j < VE; ++j) acc[i] = fmaf(xv[u][j], wv[j], acc[i]);
              }
            }
          }
        }
#pragma unroll
        for (int i = 0; i < kExpertGroup; ++i) acc[i] = warp_sum(acc[i]);
        if (lane < kExpertGroup && e0 + lane < E) {
          float v = acc[0];
#pragma unroll
          for (int i = 1; i < kExpertGroup; ++i)
            if (lane == i) v = acc[i];
          if (a.logit_bias) v += a.logit_bias[e0 + lane];
          s_logit[warp][e0 + lane] = v;
        }
      }
      __syncwarp();
      if (a.logits_out)
        for (int e = lane; e < E; e += 32) a.logits_out[(int64_t)t * E + e] = s_logit[warp][e];
    }
    __syncwarp();

    // ---------------------------------------------------------------- selection
    constexpr int NJ = kMaxExperts / 32;
    float sel_val[NJ];   // value used for ranking
    float wgt[NJ];       // value reported as the routing weight
    uint32_t avail = 0;  // bit j: expert lane + 32 j is selectable
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int e = lane + 32 * j;
      sel_val[j] = -INFINITY;
      wgt[j] = 0.f;
      if (e < E) {
        sel_val[j] = s_logit[warp][e];
        avail |= 1u << j;
      }
    }
    if (a.mode == DMOE_ROUTER_SOFTMAX) {
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < NJ; ++j) m = fmaxf(m, sel_val[j]);
      m = warp_max(m);
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        wgt[j] = (avail >> j & 1u) ? expf(sel_val[j] - m) : 0.f;
        s += wgt[j];
      }
      s = warp_sum(s);
#pragma unroll
      for (int j = 0; j < NJ; ++j) wgt[j] = wgt[j] / s;
      // softmax is monotone in the logits: rank by the logits themselves
    } else {
      // sigmoid scores; ranking uses score + selection bias; weights use the score
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int e = lane + 32 * j;
        if (avail >> j & 1u) {
          const float sc = 1.f / (1.f + expf(-sel_val[j]));
          wgt[j] = sc;
          sel_val[j] = sc + (a.score_bias ? a.score_bias[e] : 0.f);
          s_logit[warp][e] = sel_val[j];
        }
      }
      __syncwarp();
      const int per_group = E / a.n_group;
      if (lane < a.n_group) {
        // The two best scores of the group in torch.topk's order (NaN above every number),
        // so a group holding a NaN score ranks first, as the group top-k does.
        float b1 = -INFINITY, b2 = -INFINITY;
        for (int e = lane * per_group; e < (lane + 1) * per_group; ++e) {
          const float v = s_logit[warp][e];
          if (ranks_before(v, 0, b1, 1)) {
            b2 = b1;
            b1 = v;
          } else if (ranks_before(v, 0, b2, 1)) {
            b2 = v;
          }
        }
        s_gscore[warp][lane] = (per_group >= 2) ? b1 + b2 : b1;
      }
      __syncwarp();
      float gv = lane < a.n_group ? s_gscore[warp][lane] : -INFINITY;
      uint32_t kept = 0;
      for (int r = 0; r < a.topk_group; ++r) {
        float v = gv;
        int i = lane < a.n_group ? lane : 0x7fffffff;
        warp_argmax(v, i);
        if (i < 32) kept |= 1u << i;
        if (lane == i) gv = -INFINITY;
      }
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int e = lane + 32 * j;
        if ((avail >> j & 1u) && !(kept >> (e / per_group) & 1u)) avail &= ~(1u << j);
      }
      __syncwarp();
    }

    float picked_w = 0.f;  // lane r keeps the weight of the r-th pick
    int picked_e = 0;
    float wsum = 0.f;
    for (int r = 0; r < a.k; ++r) {
      float v = -INFINITY;
      int idx = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int e = lane + 32 * j;
        if ((avail >> j & 1u) && ranks_before(sel_val[j], e, v, idx)) {
          v = sel_val[j];
          idx = e;
        }
      }
      warp_argmax(v, idx);
      float w = 0.f;
#pragma unroll
      for (int j = 0; j < NJ; ++j)
        if (lane + 32 * j == idx) {
          w = wgt[j];
          avail &= ~(1u << j);
        }
      w = warp_sum(w);  // exactly one lane contributed
      wsum += w;
      if (lane == r) {
        picked_w = w;
        picked_e = idx;
      }
    }
    if (lane < a.k) {
      float w = picked_w;
      if (a.renormalize) w = w / wsum;
      w *= a.scale;
      a.idx_out[(int64_t)t * a.k + lane] = picked_e;
      store_from_float(a.w_out, (int64_t)t * a.k + lane, w, a.w_dtype);
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------------- few experts
// Softmax router for E <= 8 experts and 16-bit inputs (the Mixtral-style router).  One
// persistent CTA per SM with nw compute warps and one selection warp.  The compute warps
// split the hidden dimension (warp w owns V runs of 512 contiguous bytes of every row) and
// each lane keeps its columns of all router rows in registers as fp32 for the whole kernel,
// so the weights are read once per CTA.  Tiles of consecutive tokens (contiguous in x)
// stream into a 4-stage shared-memory ring through bulk async copies that complete on
// mbarriers.  Per token, a warp's EP partial dot products are reduced with a butterfly
// reduce-scatter (EP/2 + ... + 1 + 2 shuffles) that leaves each lane one expert's warp sum,
// written to a double-buffered partials array.  No CTA-wide barrier: each compute warp
// arrives on the tile's "partials written" mbarrier; the selection warp waits for it, refills
// the consumed stage with the tile STAGES ahead, sums the warps' partials in a fixed order
// (one lane per token and expert), does each token's softmax and top-k with shuffles (same
// order as the warp kernel: NaN first, then larger, then lower index) and arrives on the
// buffer's "partials read" mbarrier, which the compute warps wait for two tiles later.
// Every wait is bounded; on expiry the warp raises a shared abort flag that ends every
// other warp's waits, and the refilling thread drains its copies still in flight.
constexpr int kSmallStages = 4;
constexpr int kSmallStageBytes = 32 * 1024;
constexpr int kSmallMaxTile = 16;
constexpr uint64_t kSmallWaitNs = 2000000000ull;

__device__ __forceinline__ void bar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Bounded wait on an mbarrier phase; false (and the abort flag raised) on expiry or when
// another warp has raised it.
__device__ __forceinline__ bool bar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (bar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!bar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > kSmallWaitNs) {
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

// Butterfly reduce-scatter of EP values per lane over the 32 lanes of a warp: returns the
// full warp sum of value number `expert_of_lane(lane)`.
template <int EP>
__device__ __forceinline__ float warp_reduce_scatter(float (&v)[EP], int lane) {
  float cur[EP];
#pragma unroll
  for (int e = 0; e < EP; ++e) cur[e] = v[e];
  int n = EP;
#pragma unroll
  for (int o = 16; n > 1; o >>= 1) {
    const bool hi = lane & o;
    const int h = n / 2;
#pragma unroll
    for (int q = 0; q < EP / 2; ++q) {
      if (q < h) {
        const float send = hi ? cur[q] : cur[q + h];
        const float keep = hi ? cur[q + h] : cur[q];
        cur[q] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    n = h;
  }
  // n == 1: lanes that differ only in the low bits hold partial sums of the same value
  float r = cur[0];
  constexpr int used = EP == 8 ? 3 : (EP == 4 ? 2 : (EP == 2 ? 1 : 0));
#pragma unroll
  for (int o = 1 << (4 - used); o >= 1; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}

// Which value a lane holds after warp_reduce_scatter: its bits 4, 3, 2 (EP = 8) select the
// upper halves of the successive splits.
template <int EP>
__device__ __forceinline__ int expert_of_lane(int lane) {
  constexpr int used = EP == 8 ? 3 : (EP == 4 ? 2 : (EP == 2 ? 1 : 0));
  return (lane >> (5 - used)) & (EP - 1);
}

// Softmax + top-k of the tokens of one tile from the compute warps' partials (selection warp).
template <int EP>
__device__ __forceinline__ void select_tile(const RouterArgs& a, const float* part, int nw, int t0, int nt,
                                            int lane) {
  // lane = token-in-chunk * EP + expert; groups of EP lanes hold one token's logits
  const int e = lane % EP;
  const float bias = (a.logit_bias && e < a.E) ? a.logit_bias[e] : 0.f;  // one load, before the tokens
  for (int r0 = 0; r0 < nt; r0 += 32 / EP) {
    const int r = r0 + lane / EP;
    const bool live = r < nt && e < a.E;
    float l = -INFINITY;
    if (live) {
      float v = 0.f;
      for (int w = 0; w < nw; ++w) v += part[(r * nw + w) * EP + e];
      if (a.logit_bias) v += bias;
      if (a.logits_out) a.logits_out[(int64_t)(t0 + r) * a.E + e] = v;
      l = v;
    }
    float m = l;
#pragma unroll
    for (int o = 1; o < EP; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o, EP));
    float p = live ? expf(l - m) : 0.f;
    float ps = p;
#pragma unroll
    for (int o = 1; o < EP; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o, EP);
    p = p / ps;
    bool avail = live;
    float wsum = 0.f, mine_w = 0.f;
    int mine_e = 0;
    for (int q = 0; q < a.k; ++q) {
      float bv = avail ? l : -INFINITY;
      int bi = avail ? e : 0x7fffffff;
#pragma unroll
      for (int o = 1; o < EP; o <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o, EP);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o, EP);
        if (ranks_before(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      const float pw = __shfl_sync(0xffffffffu, p, (lane & ~(EP - 1)) | (bi & (EP - 1)), 32);
      if (e == bi) avail = false;
      wsum += pw;
      if (e == q) {
        mine_w = pw;
        mine_e = bi;
      }
    }
    if (r < nt && e < a.k) {
      float w = a.renormalize ? mine_w / wsum : mine_w;
      w *= a.scale;
      a.idx_out[(int64_t)(t0 + r) * a.k + e] = mine_e;
      store_from_float(a.w_out, (int64_t)(t0 + r) * a.k + e, w, a.w_dtype);
    }
  }
}

template <int DT, int EP, int V>
__global__ void __launch_bounds__(544, 1) router_small_kernel(const RouterArgs a, int tile_t, int n_tiles) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int nw = (blockDim.x >> 5) - 1;  // compute warps; warp nw selects
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row_bytes = (int64_t)a.d * 2;
  uint8_t* ring = smem_raw;
  float* s_part = reinterpret_cast<float*>(smem_raw + kSmallStages * kSmallStageBytes);  // [2][tile][nw][EP]
  uint64_t* full = reinterpret_cast<uint64_t*>(s_part + 2 * tile_t * nw * EP);
  uint64_t* pfull = full + kSmallStages;  // [2]: every compute warp wrote its partials
  uint64_t* pempty = pfull + 2;           // [2]: the selection warp read them
  volatile int* abort_flag = reinterpret_cast<volatile int*>(pempty + 2);
  const int my_tiles = blockIdx.x < n_tiles ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSmallStages; ++s) bar_init(&full[s], 1);
    for (int b = 0; b < 2; ++b) {
      bar_init(&pfull[b], (uint32_t)nw);
      bar_init(&pempty[b], 1);
    }
    *abort_flag = 0;
    fence_async_shared();
  }
  __syncthreads();

  auto issue = [&](int i) {
    const int t0 = ((int)blockIdx.x + i * (int)gridDim.x) * tile_t;
    const int nt = min(tile_t, a.T - t0);
    const int s = i % kSmallStages;
    const uint32_t bytes = (uint32_t)(nt * row_bytes);
    bar_expect_tx(&full[s], bytes);
    bulk_load(ring + s * kSmallStageBytes, reinterpret_cast<const char*>(a.x) + t0 * row_bytes, bytes, &full[s]);
  };

  if (warp == nw) {
    // ---------------------------------------------------------------- selection + refills
    int issued = 0;
    if (lane == 0)
      for (; issued < kSmallStages && issued < my_tiles; ++issued) issue(issued);
    int done = 0;
    for (int i = 0; i < my_tiles; ++i) {
      const bool ok = bar_wait_bounded(&pfull[i & 1], (uint32_t)(i >> 1) & 1u, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      // every compute warp has consumed stage i % STAGES: refill it
      if (lane == 0 && i + kSmallStages < my_tiles) {
        fence_async_shared();
        issue(i + kSmallStages);
        issued = i + kSmallStages + 1;
      }
      const int t0 = ((int)blockIdx.x + i * (int)gridDim.x) * tile_t;
      select_tile<EP>(a, s_part + (i & 1) * tile_t * nw * EP, nw, t0, min(tile_t, a.T - t0), lane);
      __syncwarp();
      if (lane == 0) bar_arrive(&pempty[i & 1]);
      done = i + 1;
    }
    // After an abort, wait (bounded) for this thread's copies still in flight.
    if (lane == 0) {
      for (int j = done; j < issued; ++j) {
        const uint32_t ph = (uint32_t)(j / kSmallStages) & 1u;
        const uint64_t t0 = global_timer_ns();
        while (!bar_try_wait(&full[j % kSmallStages], ph))
          if (global_timer_ns() - t0 > kSmallWaitNs) break;
      }
    }
    return;
  }

  // ------------------------------------------------------------------ compute warps
  float wf[EP][V * 8];
#pragma unroll
  for (int e = 0; e < EP; ++e)
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int64_t col = ((int64_t)(warp * V + j) * 32 + lane) * 8;
      uint4 raw = make_uint4(0, 0, 0, 0);
      if (e < a.E) raw = *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(a.w_r) + ((int64_t)e * a.d + col) * 2);
      unpack8<DT>(raw, &wf[e][j * 8]);
    }
  constexpr int used = EP == 8 ? 3 : (EP == 4 ? 2 : (EP == 2 ? 1 : 0));
  constexpr uint32_t low_mask = (1u << (5 - used)) - 1u;  // lanes sharing one reduced value
  const int my_e = expert_of_lane<EP>(lane);
  for (int i = 0; i < my_tiles; ++i) {
    const int t0 = ((int)blockIdx.x + i * (int)gridDim.x) * tile_t;
    const int nt = min(tile_t, a.T - t0);
    bool ok = bar_wait_bounded(&full[i % kSmallStages], (uint32_t)(i / kSmallStages) & 1u, abort_flag);
    if (ok && i >= 2) ok = bar_wait_bounded(&pempty[i & 1], ((uint32_t)(i >> 1) & 1u) ^ 1u, abort_flag);
    if (!__all_sync(0xffffffffu, ok)) break;
    const uint8_t* st = ring + (i % kSmallStages) * kSmallStageBytes;
    float* part = s_part + (i & 1) * tile_t * nw * EP;
    for (int r = 0; r < nt; ++r) {
      float acc[EP];
#pragma unroll
      for (int e = 0; e < EP; ++e) acc[e] = 0.f;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const int64_t col = ((int64_t)(warp * V + j) * 32 + lane) * 8;
        float xf[8];
        unpack8<DT>(*reinterpret_cast<const uint4*>(st + r * row_bytes + col * 2), xf);
#pragma unroll
        for (int e = 0; e < EP; ++e)
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[e] = fmaf(xf[q], wf[e][j * 8 + q], acc[e]);
      }
      const float sum = warp_reduce_scatter<EP>(acc, lane);
      if ((lane & low_mask) == 0) part[(r * nw + warp) * EP + my_e] = sum;
    }
    __syncwarp();
    if (lane == 0) bar_arrive(&pfull[i & 1]);
  }
}

// ------------------------------------------------------------------------- few experts, MMA
// The same router with the dot products on the tensor cores (16x8x16 bf16/f16 MMAs with fp32
// accumulation), for E <= 8 and d a multiple of 1024 up to 5120: a 16-token group is one MMA
// row block and the (up to) 8 experts one column block, so a warp's 16 x 16 slice of x costs
// one MMA instead of 64 FMAs per lane.  Per CTA: a producer warp streams each group's rows in
// K-chunks of 1024 elements (16 bulk copies of 2 KB, one per token, into rows padded by 16
// bytes so that 8x8 matrix loads hit 32 banks) through a 4-stage ring; 4 compute warps each
// take 256 columns of every chunk and keep a 16 x 8 fp32 accumulator over the group's chunks;
// the selection warp sums the 4 partials in a fixed order and selects as router_small_kernel.
// The router rows sit in shared memory (padded the same way) for the whole kernel.
constexpr int kMmaChunk = 1024;        // K elements per stage
constexpr int kMmaWarps = 4;           // compute warps: 256 columns of a chunk each
constexpr int kMmaStages = 4;
constexpr int kMmaRowPad = 16;         // bytes after each 2 KB row (bank spread for ldmatrix)
constexpr int kMmaRowStride = kMmaChunk * 2 + kMmaRowPad;
constexpr int kMmaStageBytes = 16 * kMmaRowStride;
constexpr int kMmaMaxD = 5120;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

template <int DT>
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  if constexpr (DT == DMOE_BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

template <int DT>
__global__ void __launch_bounds__((kMmaWarps + 2) * 32, 1) router_mma_kernel(const RouterArgs a, int n_groups) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = a.d / kMmaChunk;
  const int w_stride = a.d * 2 + kMmaRowPad;  // bytes between router rows in shared memory
  uint8_t* ring = smem_raw;
  uint8_t* s_w = ring + kMmaStages * kMmaStageBytes;                       // [8][d] padded
  float* s_part = reinterpret_cast<float*>(s_w + 8 * w_stride);            // [2][16][4][8]
  uint64_t* full = reinterpret_cast<uint64_t*>(s_part + 2 * 16 * kMmaWarps * 8);
  uint64_t* empty = full + kMmaStages;
  uint64_t* pfull = empty + kMmaStages;  // [2]: the compute warps wrote a group's partials
  uint64_t* pempty = pfull + 2;          // [2]: the selection warp read them
  uint64_t* wbar = pempty + 2;           // the router rows landed
  volatile int* abort_flag = reinterpret_cast<volatile int*>(wbar + 1);
  const int my_groups = (int)blockIdx.x < n_groups ? (n_groups - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int64_t row_bytes = (int64_t)a.d * 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMmaStages; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], kMmaWarps);
    }
    for (int b = 0; b < 2; ++b) {
      bar_init(&pfull[b], kMmaWarps);
      bar_init(&pempty[b], 1);
    }
    bar_init(wbar, 1);
    *abort_flag = 0;
    fence_async_shared();
    // The router rows arrive by bulk copies, like the tokens; rows past E are zeroed below.
    bar_expect_tx(wbar, (uint32_t)(a.E * row_bytes));
    for (int e = 0; e < a.E; ++e)
      bulk_load(s_w + e * w_stride, reinterpret_cast<const char*>(a.w_r) + (int64_t)e * row_bytes, (uint32_t)row_bytes,
                wbar);
  }
  for (int i = threadIdx.x; i < (8 - a.E) * (a.d / 8); i += blockDim.x) {
    const int e = a.E + i / (a.d / 8), c = i - (e - a.E) * (a.d / 8);
    *reinterpret_cast<uint4*>(s_w + e * w_stride + c * 16) = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();

  const int total = my_groups * nch;  // stages this CTA streams
  if (warp == kMmaWarps + 1) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int j = 0;
      for (; j < total; ++j) {
        const int s = j % kMmaStages;
        if (j >= kMmaStages && !bar_wait_bounded(&empty[s], ((uint32_t)(j / kMmaStages) & 1u) ^ 1u, abort_flag)) break;
        const int g = (int)blockIdx.x + (j / nch) * (int)gridDim.x, c = j % nch;
        const int t0 = g * 16, nt = min(16, a.T - t0);
        bar_expect_tx(&full[s], (uint32_t)(nt * kMmaChunk * 2));
        uint8_t* dst = ring + s * kMmaStageBytes;
        const char* src = reinterpret_cast<const char*>(a.x) + (int64_t)t0 * row_bytes + (int64_t)c * kMmaChunk * 2;
        for (int r = 0; r < nt; ++r) bulk_load(dst + r * kMmaRowStride, src + r * row_bytes, kMmaChunk * 2, &full[s]);
      }
      // After an abort, wait (bounded) for the copies still in flight.
      if (j < total) {
        const uint64_t tw = global_timer_ns();
        while (!bar_try_wait(wbar, 0))
          if (global_timer_ns() - tw > kSmallWaitNs) break;
        for (int q = j - kMmaStages > 0 ? j - kMmaStages : 0; q < j; ++q) {
          const uint64_t t0 = global_timer_ns();
          while (!bar_try_wait(&full[q % kMmaStages], (uint32_t)(q / kMmaStages) & 1u))
            if (global_timer_ns() - t0 > kSmallWaitNs) break;
        }
      }
    }
    return;
  }
  if (warp == kMmaWarps) {
    // ---------------------------------------------------------------- selection
    for (int i = 0; i < my_groups; ++i) {
      const bool ok = bar_wait_bounded(&pfull[i & 1], (uint32_t)(i >> 1) & 1u, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      const int t0 = ((int)blockIdx.x + i * (int)gridDim.x) * 16;
      select_tile<8>(a, s_part + (i & 1) * 16 * kMmaWarps * 8, kMmaWarps, t0, min(16, a.T - t0), lane);
      __syncwarp();
      if (lane == 0) bar_arrive(&pempty[i & 1]);
    }
    return;
  }
  // ------------------------------------------------------------------ compute warps
  // ldmatrix addresses: A rows lane % 16, 8-column block lane / 16; B (router rows) lane % 8,
  // 8-column block (lane / 8) % 2.
  const uint32_t a_off = (uint32_t)((lane & 15) * kMmaRowStride + (lane >> 4) * 16 + warp * 512);
  const uint32_t b_base = smem_addr(s_w) + (uint32_t)((lane & 7) * w_stride + ((lane >> 3) & 1) * 16);
  if (!__all_sync(0xffffffffu, bar_wait_bounded(wbar, 0, abort_flag))) return;
  int j = 0;
  for (int i = 0; i < my_groups; ++i) {
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    bool ok = true;
    for (int c = 0; c < nch && ok; ++c, ++j) {
      const int s = j % kMmaStages;
      ok = bar_wait_bounded(&full[s], (uint32_t)(j / kMmaStages) & 1u, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      const uint32_t a_base = smem_addr(ring + s * kMmaStageBytes) + a_off;
      const uint32_t kb = (uint32_t)(c * kMmaChunk + warp * 256) * 2;  // byte column of this warp's slice
#pragma unroll
      for (int q = 0; q < 16; ++q) {  // 16 steps of 16 columns
        uint32_t a0, a1, a2, a3, b0, b1;
        ldsm_x4(a_base + q * 32, a0, a1, a2, a3);
        ldsm_x2(b_base + kb + q * 32, b0, b1);
        mma_16816<DT>(acc[q & 1], a0, a1, a2, a3, b0, b1);
      }
      __syncwarp();
      if (lane == 0) bar_arrive(&empty[s]);
    }
    if (!ok) break;
    if (i >= 2 && !__all_sync(0xffffffffu, bar_wait_bounded(&pempty[i & 1], ((uint32_t)(i >> 1) & 1u) ^ 1u, abort_flag)))
      break;
    // D fragment: rows lane / 4 and lane / 4 + 8, experts 2 * (lane % 4) and + 1
    float* part = s_part + (i & 1) * 16 * kMmaWarps * 8;
    const int r = lane >> 2, e = 2 * (lane & 3);
    part[(r * kMmaWarps + warp) * 8 + e] = acc[0][0] + acc[1][0];
    part[(r * kMmaWarps + warp) * 8 + e + 1] = acc[0][1] + acc[1][1];
    part[((r + 8) * kMmaWarps + warp) * 8 + e] = acc[0][2] + acc[1][2];
    part[((r + 8) * kMmaWarps + warp) * 8 + e + 1] = acc[0][3] + acc[1][3];
    __syncwarp();
    if (lane == 0) bar_arrive(&pfull[i & 1]);
  }
}

bool router_mma_eligible(int x_dtype, int mode, const float* logits_in, int E, int d) {
  if (logits_in != nullptr || mode != DMOE_ROUTER_SOFTMAX || E > 8) return false;
  if (x_dtype != DMOE_BF16 && x_dtype != DMOE_F16) return false;
  if (d % kMmaChunk != 0 || d > kMmaMaxD) return false;
  const char* v = getenv("DMOE_ROUTER_MMA");
  return !(v && v[0] == '0');
}

template <int DT>
int run_router_mma(const RouterArgs& a, cudaStream_t s) {
  const int n_groups = (a.T + 15) / 16;
  const int grid = n_groups < 148 ? n_groups : 148;
  const size_t smem = (size_t)kMmaStages * kMmaStageBytes + (size_t)8 * (a.d * 2 + kMmaRowPad) +
                      (size_t)2 * 16 * kMmaWarps * 8 * sizeof(float) + (2 * kMmaStages + 5) * sizeof(uint64_t) + 16;
  static PerDeviceOnce once;
  int dev = 0;
  DMOE_CUDA(cudaGetDevice(&dev));
  const int r = once_per_device(once, dev, [] {
    DMOE_CUDA(cudaFuncSetAttribute(router_mma_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    return DMOE_OK;
  });
  if (r) return r;
  router_mma_kernel<DT><<<grid, (kMmaWarps + 2) * 32, smem, s>>>(a, n_groups);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

// Router logits for few tokens (decode): the tensor-core logits GEMM would give the whole
// reduction to one or two CTAs when T is small, so here eight experts go to each CTA: their
// weight rows land in shared memory with one bulk copy, each warp takes tokens in turn and
// streams the token's row (L2-resident: a decode batch is small), and the 9-shuffle
// reduce-scatter leaves lane groups holding one expert's sum each.
constexpr int kFewTokensMax = 256;
constexpr int kFewTokensSmemMax = 200 * 1024;

template <int DT>
__global__ void __launch_bounds__(256) logits_few_tokens_kernel(const void* x, const void* w, int T, int d, int E,
                                                                float* out) {
  extern __shared__ __align__(128) uint8_t s_wrows[];
  __shared__ uint64_t bar;
  const int e0 = blockIdx.x * 8;
  const uint32_t bytes = (uint32_t)(8 * d * 2);
  if (threadIdx.x == 0) {
    bar_init(&bar, 1);
    fence_async_shared();
    bar_expect_tx(&bar, bytes);
    const char* src = reinterpret_cast<const char*>(w) + (int64_t)e0 * d * 2;
    for (uint32_t off = 0; off < bytes; off += 16384u) {  // 16 KB pieces, one completion count
      const uint32_t n = bytes - off < 16384u ? bytes - off : 16384u;
      bulk_load(s_wrows + off, src + off, n, &bar);
    }
  }
  __syncthreads();
  bool ok = bar_try_wait(&bar, 0);
  if (!ok) {
    const uint64_t w0 = global_timer_ns();
    while (!(ok = bar_try_wait(&bar, 0)))
      if (global_timer_ns() - w0 > kSmallWaitNs) break;
  }
  if (__syncthreads_or(!ok)) return;  // never wait forever for a copy from valid memory
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = d / 8;
  for (int t = warp; t < T; t += blockDim.x >> 5) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    const uint4* xr = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(x) + (int64_t)t * d * 2);
    for (int c = lane; c < nvec; c += 32) {
      float xf[8];
      unpack8<DT>(xr[c], xf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float wf[8];
        unpack8<DT>(reinterpret_cast<const uint4*>(s_wrows + (int64_t)e * d * 2)[c], wf);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[e] = fmaf(xf[q], wf[q], acc[e]);
      }
    }
    const float v = warp_reduce_scatter<8>(acc, lane);
    if ((lane & 3) == 0) out[(int64_t)t * E + e0 + expert_of_lane<8>(lane)] = v;
  }
}

template <int DT, int EP, int V>
int launch_router_small(int grid, int threads, size_t smem, cudaStream_t s, const RouterArgs& a, int tile_t,
                        int n_tiles) {
  static PerDeviceOnce once;
  int dev = 0;
  DMOE_CUDA(cudaGetDevice(&dev));
  // The attribute is set once per device, so to the most any call can ask for: the ring, and
  // partials for tile_t * nw <= 64 (tile_t = 32 KB / row bytes, nw = row bytes / 512), plus
  // the barriers.  A first call with a small row must not cap later calls with larger rows.
  constexpr size_t kMaxSmem = (size_t)kSmallStages * kSmallStageBytes + 2 * 64 * 8 * sizeof(float) +
                              (kSmallStages + 4) * sizeof(uint64_t) + 16;
  DMOE_REQUIRE(smem <= kMaxSmem, "router: %zu bytes of shared memory exceed %zu", smem, kMaxSmem);
  const int r = once_per_device(once, dev, [&] {
    DMOE_CUDA(cudaFuncSetAttribute(router_small_kernel<DT, EP, V>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kMaxSmem));
    return DMOE_OK;
  });
  if (r) return r;
  router_small_kernel<DT, EP, V><<<grid, threads, smem, s>>>(a, tile_t, n_tiles);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

// The few-expert kernel applies when the softmax router computes its own logits from 16-bit
// x, d is a multiple of 256, and the lane's weight registers (E x V vectors) stay within what
// a 512-thread CTA holds without spilling: E <= 8 with d <= 4096, or E <= 4 with d <= 8192.
bool router_small_eligible(int x_dtype, int mode, const float* logits_in, int E, int d) {
  if (logits_in != nullptr || mode != DMOE_ROUTER_SOFTMAX) return false;
  if (x_dtype != DMOE_BF16 && x_dtype != DMOE_F16) return false;
  if (d % 256 != 0 || !((E <= 8 && d <= 4096) || (E <= 4 && d <= 8192 && d % 512 == 0))) return false;
  const char* v = getenv("DMOE_ROUTER_SMALL");
  return !(v && v[0] == '0');
}

template <int DT>
int run_router_small_dt(const RouterArgs& a, cudaStream_t s) {
  const int V = a.d <= 4096 ? 1 : 2;
  const int nw = a.d / (256 * V);
  const int64_t row_bytes = (int64_t)a.d * 2;
  int tile_t = (int)(kSmallStageBytes / row_bytes);
  if (tile_t > kSmallMaxTile) tile_t = kSmallMaxTile;
  const int n_tiles = (a.T + tile_t - 1) / tile_t;
  const int EP = a.E <= 4 ? 4 : 8;
  const int grid = n_tiles < 148 ? n_tiles : 148;
  const size_t smem = (size_t)kSmallStages * kSmallStageBytes + (size_t)2 * tile_t * nw * EP * sizeof(float) +
                      (kSmallStages + 4) * sizeof(uint64_t) + 16;
  const int threads = (nw + 1) * 32;
  if (EP == 8) return launch_router_small<DT, 8, 1>(grid, threads, smem, s, a, tile_t, n_tiles);
  if (V == 1) return launch_router_small<DT, 4, 1>(grid, threads, smem, s, a, tile_t, n_tiles);
  return launch_router_small<DT, 4, 2>(grid, threads, smem, s, a, tile_t, n_tiles);
}

int run_router_small(int x_dtype, const RouterArgs& a, cudaStream_t s) {
  return x_dtype == DMOE_BF16 ? run_router_small_dt<DMOE_BF16>(a, s) : run_router_small_dt<DMOE_F16>(a, s);
}

template <int DT, bool W_SMEM>
int launch_router(dim3 grid, dim3 block, size_t smem, cudaStream_t s, const RouterArgs& a) {
  if (W_SMEM) {
    static PerDeviceOnce once;
    int dev = 0;
    DMOE_CUDA(cudaGetDevice(&dev));
    const int r = once_per_device(once, dev, [] {
      DMOE_CUDA(cudaFuncSetAttribute(router_kernel<DT, W_SMEM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kWSmemMax));
      return DMOE_OK;
    });
    if (r) return r;
  }
  router_kernel<DT, W_SMEM><<<grid, block, smem, s>>>(a);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

template <int DT>
int launch_logits_few_tokens(const void* x, const void* w, int T, int d, int E, float* out, cudaStream_t s) {
  static PerDeviceOnce once;
  int dev = 0;
  DMOE_CUDA(cudaGetDevice(&dev));
  const int r = once_per_device(once, dev, [] {
    DMOE_CUDA(cudaFuncSetAttribute(logits_few_tokens_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kFewTokensSmemMax));
    return DMOE_OK;
  });
  if (r) return r;
  logits_few_tokens_kernel<DT><<<E / 8, 256, (size_t)8 * d * 2, s>>>(x, w, T, d, E, out);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

}  // namespace

bool logits_few_tokens_eligible(int T, int d, int E) {
  const char* v = getenv("DMOE_LOGITS_FEW_TOKENS");
  if (v && v[0] == '0') return false;
  return T <= kFewTokensMax && E % 8 == 0 && (int64_t)8 * d * 2 <= kFewTokensSmemMax;
}

int run_logits_few_tokens(const void* x, const void* w, int dtype, int T, int d, int E, float* out, cudaStream_t s) {
  if (dtype == DMOE_BF16) return launch_logits_few_tokens<DMOE_BF16>(x, w, T, d, E, out, s);
  return launch_logits_few_tokens<DMOE_F16>(x, w, T, d, E, out, s);
}

}  // namespace dmoe

using namespace dmoe;

extern "C" int dmoe_router(const void* x, const void* w_r, int x_dtype, const float* logit_bias,
                           const float* score_bias, const float* logits_in, int T, int d, int E, int k, int mode,
                           int renormalize, float scale, int n_group, int topk_group, float* logits_out,
                           int64_t* idx_out, void* w_out, int w_dtype, void* stream) {
  clear_error();
  DMOE_REQUIRE(T >= 0 && E >= 1 && E <= kMaxExperts, "dmoe_router: need 1 <= E <= %d (E=%d)", kMaxExperts, E);
  DMOE_REQUIRE(k >= 1 && k <= E && k <= kMaxTopK && k <= 32, "dmoe_router: bad top_k %d", k);
  DMOE_REQUIRE(dtype_ok(x_dtype) && dtype_ok(w_dtype), "dmoe_router: bad dtype");
  DMOE_REQUIRE(idx_out && w_out, "dmoe_router: null output");
  DMOE_REQUIRE(mode == DMOE_ROUTER_SOFTMAX || mode == DMOE_ROUTER_SIGMOID_GROUP, "dmoe_router: bad mode %d", mode);
  if (mode == DMOE_ROUTER_SIGMOID_GROUP) {
    DMOE_REQUIRE(n_group >= 1 && n_group <= 32 && E % n_group == 0, "dmoe_router: bad n_group %d", n_group);
    DMOE_REQUIRE(topk_group >= 1 && topk_group <= n_group, "dmoe_router: bad topk_group %d", topk_group);
    DMOE_REQUIRE((E / n_group) * topk_group >= k, "dmoe_router: kept groups hold fewer than k experts");
  }
  if (logits_in == nullptr) {
    DMOE_REQUIRE(x && w_r, "dmoe_router: null input");
    DMOE_REQUIRE(d > 0 && d % 8 == 0, "dmoe_router: d=%d must be a multiple of 8", d);
    DMOE_REQUIRE(aligned16(x) && aligned16(w_r), "dmoe_router: x and w_r must be 16-byte aligned");
  }
  if (T == 0) return DMOE_OK;
  RouterArgs a{x, w_r, logit_bias, score_bias, logits_in, logits_out, idx_out, w_out, T, d, E, k, mode,
               renormalize, mode == DMOE_ROUTER_SIGMOID_GROUP ? n_group : 1, topk_group, w_dtype, scale};
  if (router_mma_eligible(x_dtype, mode, logits_in, E, d))
    return x_dtype == DMOE_BF16 ? run_router_mma<DMOE_BF16>(a, as_stream(stream))
                                : run_router_mma<DMOE_F16>(a, as_stream(stream));
  if (router_small_eligible(x_dtype, mode, logits_in, E, d)) return run_router_small(x_dtype, a, as_stream(stream));
  int blocks = (T + kRouterWarps - 1) / kRouterWarps;
  cudaStream_t s = as_stream(stream);
  const int64_t w_bytes = logits_in ? 0 : (int64_t)E * d * (x_dtype == DMOE_F32 ? 4 : 2);
  if (logits_in == nullptr && w_bytes <= kWSmemMax) {
    // Router weights in shared memory: enough blocks for every SM, each reused over tokens.
    const int per_sm = (int)((227 * 1024) / (w_bytes + 10 * 1024));
    // Each block first stages the weights: with an SM reserve set, the grouped MLP holds the
    // other SMs, so size the grid for the reserved ones instead of queueing waves of copies.
    const int reserve = gemm_sm_reserve();
    const int cap = (reserve > 0 ? reserve : 148) * (per_sm < 1 ? 1 : per_sm);
    if (blocks > cap) blocks = cap;
    const dim3 grid(blocks), block(kRouterWarps * 32);
    if (x_dtype == DMOE_BF16) return launch_router<DMOE_BF16, true>(grid, block, (size_t)w_bytes, s, a);
    if (x_dtype == DMOE_F16) return launch_router<DMOE_F16, true>(grid, block, (size_t)w_bytes, s, a);
    return launch_router<DMOE_F32, true>(grid, block, (size_t)w_bytes, s, a);
  }
  if (blocks > 148 * 16) blocks = 148 * 16;
  const dim3 grid(blocks), block(kRouterWarps * 32);
  if (x_dtype == DMOE_BF16) return launch_router<DMOE_BF16, false>(grid, block, 0, s, a);
  if (x_dtype == DMOE_F16) return launch_router<DMOE_F16, false>(grid, block, 0, s, a);
  return launch_router<DMOE_F32, false>(grid, block, 0, s, a);
}
