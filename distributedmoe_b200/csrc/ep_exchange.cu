// Expert-parallel exchange over NVLink peer memory: the device-driven data plane of the
// NVLinkDirect transfer backend.
//
// Replaces, for hosts and expert blocks that run in lockstep (one forward per step on
// every GPU), the task protocol of the reference:
//   DispatchSubmit metadata over ZeroMQ  (MoE/PipelineTask.py:262-270)
//   READ of the host's input buffer       (MoE/pools/BuffersPool.py:55-71, PipelineTask.py:459)
//   WRITE of the expert output            (MoE/pools/BuffersPool.py:73-90, PipelineTask.py:555)
//   HostOutputBufferUnlocked + combine    (MoE/PipelineTask.py:306-370, 558-565)
// with these kernels around one grouped-MLP launch per GPU:
//   ep_plan      exchange per-instance row counts with every rank (peer stores + an epoch
//                flag), then derive where this rank's rows land in each receiver's buffer
//                and this GPU's grouped-MLP segment table.
//   ep_dispatch  gather this rank's rows straight into the receivers' registered buffers
//                (peer stores over NVLink) with each row's return address (this rank,
//                token * k + slot) in the receiver's back map, remember each row's (rank,
//                row), and raise the data flag on every rank once the last CTA is done.
//   ep_wait      bounded wait until every rank's flag of a kind reached the epoch.
//   ep_signal    raise this rank's result flag on every rank after the grouped MLP.
//   ep_combine   per token, sum its k expert rows, which the owners' down-projection
//                epilogues stored into this rank's return rows (peer stores during the
//                GEMM, dmoe_ep_expert_mlp), weighted in fp32, and store once.
//
// An expert "instance" is one copy of an expert's weights on one rank (replicas give an
// expert several instances).  Instances are numbered rank-major and, within a rank, in the
// order of that rank's weight stack, so a rank's instances are the contiguous range
// [inst_first[r], inst_first[r+1]).  A receiver lays its rows out instance by instance and,
// inside an instance, sender rank by sender rank; each instance's rows are therefore one
// contiguous grouped-MLP segment holding every host's tokens for that expert.
//
// Flags are monotonic 64-bit epochs (one per forward, equal on every rank).  A rank's flag
// array holds [kind][sender] for three kinds (counts, data, results) and, after them, the
// rank's own epoch counter: ep_plan advances it at the start of every forward and the later
// kernels of the forward read it, so a forward takes no per-step argument from the host (a
// captured CUDA graph replays correctly).  All waits are bounded by time and report through
// the status word; nothing traps.
#include "dmoe_common.cuh"

namespace dmoe {
namespace {

constexpr int kMaxRanks = DMOE_EP_MAX_RANKS;
constexpr int kMaxReplicas = DMOE_EP_MAX_REPLICAS;
constexpr int kMaxInstances = DMOE_EP_MAX_INSTANCES;
constexpr int kFlagKinds = 3;
constexpr int kEpochSlot = kFlagKinds * kMaxRanks;  // index of the epoch counter in a flag array

__device__ __forceinline__ uint64_t current_epoch(const uint64_t* my_flags) { return my_flags[kEpochSlot]; }

struct EpPeers {
  int world, rank;
  uint64_t* flags[kMaxRanks];   // [kFlagKinds][kMaxRanks] epochs of each rank
  int32_t* counts[kMaxRanks];   // [2][kMaxRanks][n_inst] count matrix of each rank
  char* recv[kMaxRanks];        // receive rows of each rank
  int32_t* back[kMaxRanks];     // back map of each rank's receive rows
  char* rows[kMaxRanks];        // return rows of each rank, (token, slot) order
};

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ int32_t ld_uncached(const int32_t* p) {
  int32_t v;
  asm volatile("ld.relaxed.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded acquire-wait for flag >= epoch; false on expiry.
__device__ bool wait_flag(const uint64_t* flag, uint64_t epoch, uint64_t timeout_ns) {
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (ld_acquire_sys(flag) < epoch) {
    if ((++spins & 63u) == 0 && global_timer_ns() - t0 > timeout_ns) return false;
    __nanosleep(100);
  }
  return true;
}

// ------------------------------------------------------------------------- ep_plan
struct EpPlanArgs {
  EpPeers peers;
  const int32_t* counts_e;   // [E] this rank's rows per expert (NULL: none)
  int E, n_inst, policy;
  const int32_t* alive_n;    // [E] alive instances of each expert (for this sender)
  const int32_t* alive_inst; // [E][kMaxReplicas] those instances
  const int32_t* inst_rank;  // [n_inst]
  const int32_t* inst_slot;  // [n_inst] position in the owner's weight stack
  const int32_t* inst_first; // [world + 1]
  int64_t cap;               // receive rows of every rank
  uint64_t timeout_ns;
  int32_t* status;
  // outputs (this rank's device scratch)
  int32_t* part_n;           // [E] parts the expert's rows are split into this step (0: dropped)
  int32_t* part_inst;        // [E][kMaxReplicas] instance of each part
  int32_t* part_start;       // [E][kMaxReplicas + 1] first row (within the expert) of each part
  int32_t* dest_off;         // [n_inst] first receive row of this rank's rows of each instance
  int32_t* seg_expert;       // [local instances] weight-stack position of each local segment
  int32_t* seg_end;          // [local instances] segment ends in the receive buffer
};

__global__ void __launch_bounds__(1024) ep_plan_kernel(const EpPlanArgs a) {
  __shared__ int32_t s_mine[kMaxInstances];
  __shared__ int32_t s_tot[kMaxInstances];
  __shared__ int32_t s_scan[kMaxInstances];
  __shared__ int32_t s_warp[32];
  __shared__ int s_arrived[kMaxRanks];
  __shared__ uint64_t s_epoch;
  const int tid = threadIdx.x;
  const int G = a.peers.world, me = a.peers.rank, n_inst = a.n_inst;
  if (tid == 0) {
    uint64_t* counter = a.peers.flags[me] + kEpochSlot;
    s_epoch = *counter + 1;
    *counter = s_epoch;  // this forward's epoch; the later kernels of the forward read it
  }
  __syncthreads();
  const uint64_t epoch = s_epoch;
  const int parity = (int)(epoch & 1ull);

  for (int i = tid; i < n_inst; i += blockDim.x) s_mine[i] = 0;
  __syncthreads();
  // 1. Split each expert's rows over its alive instances.  "rotate": all rows to one
  //    instance, a different one each step and rank; "split": near-equal contiguous parts.
  for (int e = tid; e < a.E; e += blockDim.x) {
    const int n = a.counts_e ? a.counts_e[e] : 0;
    int na = a.alive_n[e];
    if (na > kMaxReplicas) na = kMaxReplicas;
    int32_t* ps = a.part_start + (int64_t)e * (kMaxReplicas + 1);
    int32_t* pi = a.part_inst + (int64_t)e * kMaxReplicas;
    int np = 0;
    if (na > 0) {
      if (a.policy == DMOE_EP_POLICY_SPLIT) {
        np = na;
        for (int q = 0; q < np; ++q) {
          const int lo = (int)((int64_t)q * n / np), hi = (int)((int64_t)(q + 1) * n / np);
          const int inst = a.alive_inst[e * kMaxReplicas + q];
          ps[q] = lo;
          pi[q] = inst;
          if (inst >= 0 && inst < n_inst) s_mine[inst] = hi - lo;  // an instance belongs to one expert
        }
        ps[np] = n;
      } else {
        np = 1;
        const int inst = a.alive_inst[e * kMaxReplicas + (int)((epoch + (uint64_t)me) % (uint64_t)na)];
        ps[0] = 0;
        ps[1] = n;
        pi[0] = inst;
        if (inst >= 0 && inst < n_inst) s_mine[inst] = n;
      }
    }
    a.part_n[e] = np;
  }
  __syncthreads();

  // 2. Exchange: this rank's row of every rank's count matrix, then the count flags.
  if (G > 1) {
    for (int idx = tid; idx < G * n_inst; idx += blockDim.x) {
      const int g = idx / n_inst, i = idx - g * n_inst;
      a.peers.counts[g][((int64_t)parity * kMaxRanks + me) * n_inst + i] = s_mine[i];
    }
    __threadfence_system();
    __syncthreads();
    if (tid < G) st_release_sys(a.peers.flags[tid] + 0 * kMaxRanks + me, epoch);
    if (tid < G) {
      const bool ok = tid == me || wait_flag(a.peers.flags[me] + 0 * kMaxRanks + tid, epoch, a.timeout_ns);
      s_arrived[tid] = ok ? 1 : 0;
      if (!ok) atomicOr(a.status, DMOE_DEVERR_EP_TIMEOUT);
    }
    __syncthreads();
  }

  // 3. Totals per instance and this rank's rows ahead of it (senders of lower rank).
  const int32_t* M = a.peers.counts[me] + (int64_t)parity * kMaxRanks * n_inst;
  for (int i = tid; i < n_inst; i += blockDim.x) {
    int32_t tot = 0, before = 0;
    if (G == 1) {
      tot = s_mine[i];
    } else {
      for (int g = 0; g < G; ++g) {
        const int32_t c = g == me ? s_mine[i] : (s_arrived[g] ? ld_uncached(M + (int64_t)g * n_inst + i) : 0);
        tot += c;
        if (g < me) before += c;
      }
    }
    s_tot[i] = tot;
    s_scan[i] = before;  // kept here until the scan below needs the slot
  }
  __syncthreads();
  // Inclusive scan of s_tot over all instances (n_inst <= 1024 = one value per thread).
  int32_t before_i = 0, v = 0;
  if (tid < n_inst) {
    before_i = s_scan[tid];
    v = s_tot[tid];
  }
  int32_t incl = v;
  const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) / 32;
    int32_t wv = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t u = __shfl_up_sync(0xffffffffu, wv, o);
      if (lane >= o) wv += u;
    }
    if (lane < nw) s_warp[lane] = wv;
  }
  __syncthreads();
  incl += warp > 0 ? s_warp[warp - 1] : 0;
  __syncthreads();
  if (tid < n_inst) s_scan[tid] = incl;
  __syncthreads();
  // 4. Receive offsets: an instance's rows start after the rows of its rank's earlier
  //    instances; this rank's share of them after the shares of lower ranks.
  if (tid < n_inst) {
    const int r = a.inst_rank[tid];
    const int first = a.inst_first[r];
    const int64_t base = (int64_t)incl - v - (first > 0 ? s_scan[first - 1] : 0);
    int64_t off = base + before_i;
    if (base + v > a.cap) atomicOr(a.status, DMOE_DEVERR_EP_OVERFLOW);
    a.dest_off[tid] = (int32_t)(off < a.cap ? off : a.cap);
    if (r == me) {
      const int j = tid - first;
      const int64_t end = base + v;
      a.seg_expert[j] = a.inst_slot[tid];
      a.seg_end[j] = (int32_t)(end < a.cap ? end : a.cap);
    }
  }
}

// ------------------------------------------------------------------------- ep_dispatch
struct EpDispatchArgs {
  EpPeers peers;
  const char* x;             // [T, row_bytes]
  int64_t row_vecs;          // 16-byte vectors per row
  int64_t n;                 // T * k activations in permuted order
  int E;
  const int32_t* offsets;    // [E + 1] permuted-order start of each expert
  const int32_t* perm_token; // [n]
  const int32_t* perm_slot;  // [n]
  int k;
  const int32_t* part_n;
  const int32_t* part_inst;
  const int32_t* part_start;
  const int32_t* inst_rank;
  const int32_t* dest_off;
  int64_t cap;
  int32_t* ret;              // [n] (rank << 27 | row) of each activation, -1 when dropped
  uint32_t* done;            // CTA completion counter (zero between launches)
  int32_t* status;
};

constexpr int kRowShift = 27;

// Per-expert placement as the gather reads it: where the expert's rows start in the
// permuted order, how its rows split into parts, and each part's (rank, receive row of the
// expert's row 0 of that part).  Kept in shared memory when E <= kTableMaxE, so a row's
// destination costs a few shared-memory reads instead of a chain of dependent global loads.
constexpr int kTableMaxE = 256;

struct ExpertPlacement {
  int32_t start[kMaxReplicas + 1];  // part q holds the expert's rows [start[q], start[q+1])
  int32_t rank[kMaxReplicas];
  int32_t base[kMaxReplicas];       // receive row = base[q] + row index within the expert
  int32_t np;
};

__device__ __forceinline__ void load_placement(const EpDispatchArgs& a, int e, ExpertPlacement& pl) {
  int np = a.part_n[e];
  if (np > kMaxReplicas) np = kMaxReplicas;
  pl.np = 0;
  for (int q = 0; q <= np; ++q) pl.start[q] = a.part_start[e * (kMaxReplicas + 1) + q];
  for (int q = 0; q < np; ++q) {
    const int inst = a.part_inst[e * kMaxReplicas + q];
    const int r = a.inst_rank[inst];
    if (r < 0 || r >= a.peers.world) return;  // a malformed table: the expert's rows are dropped
    pl.rank[q] = r;
    pl.base[q] = a.dest_off[inst] - pl.start[q];
  }
  pl.np = np;
}

template <bool TABLE>
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const EpDispatchArgs a) {
  __shared__ int32_t s_off[TABLE ? kTableMaxE + 1 : 1];
  __shared__ ExpertPlacement s_pl[TABLE ? kTableMaxE : 1];
  if constexpr (TABLE) {
    // An empty batch has no plan (offsets may be NULL): nothing to look up, only the flags.
    if (a.n > 0) {
      for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
        s_off[e] = a.offsets[e];
        load_placement(a, e, s_pl[e]);
      }
    }
    __syncthreads();
  }
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int64_t p = warp; p < a.n; p += nwarps) {
    int lo = 0, hi = a.E - 1;  // expert of permuted position p: last e with offsets[e] <= p
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((TABLE ? s_off[mid] : a.offsets[mid]) <= p) lo = mid; else hi = mid - 1;
    }
    const int e = lo;
    const int i = (int)(p - (TABLE ? s_off[e] : a.offsets[e]));
    ExpertPlacement local;
    const ExpertPlacement* pl = &local;
    if constexpr (TABLE) {
      pl = &s_pl[e];
    } else {
      load_placement(a, e, local);
    }
    const int np = pl->np;
    int q = -1;
    for (int t = 0; t < np; ++t)
      if (pl->start[t] <= i) q = t;
    // Positions past the plan's last expert row (activations without a valid expert) and
    // experts without an alive instance are dropped.
    if (np > 0 && i >= pl->start[np]) q = -1;
    int32_t code = -1;
    if (q >= 0) {
      const int r = pl->rank[q];
      const int64_t row = (int64_t)pl->base[q] + i;
      if (row < a.cap) {
        code = (int32_t)(((uint32_t)r << kRowShift) | (uint32_t)row);
        const int tok = a.perm_token[p];
        if (lane == 0)
          a.peers.back[r][row] =
              (int32_t)(((uint32_t)a.peers.rank << kRowShift) | (uint32_t)(tok * a.k + a.perm_slot[p]));
        const uint4* src = reinterpret_cast<const uint4*>(a.x) + (int64_t)tok * a.row_vecs;
        uint4* d = reinterpret_cast<uint4*>(a.peers.recv[r]) + row * a.row_vecs;
        int64_t c = lane;
        for (; c + 224 < a.row_vecs; c += 256) {
          uint4 v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) v[u] = src[c + 32 * u];
#pragma unroll
          for (int u = 0; u < 8; ++u) d[c + 32 * u] = v[u];
        }
        for (; c < a.row_vecs; c += 32) d[c] = src[c];
      } else if (lane == 0) {
        atomicOr(a.status, DMOE_DEVERR_EP_OVERFLOW);
      }
    }
    if (lane == 0) a.ret[p] = code;
  }
  // Last CTA out raises the data flag on every rank: each thread's stores are made visible
  // system-wide before its CTA counts itself done.  One rank waits on no flag: the GEMM
  // that reads the rows follows on the same stream.
  if (a.peers.world == 1) return;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(a.done, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      *a.done = 0;
      if (a.peers.world > 1) {
        const uint64_t epoch = current_epoch(a.peers.flags[a.peers.rank]);
        for (int g = 0; g < a.peers.world; ++g) st_release_sys(a.peers.flags[g] + 1 * kMaxRanks + a.peers.rank, epoch);
      }
    }
  }
}

// ------------------------------------------------------------------------- ep_wait / ep_signal
__global__ void ep_wait_kernel(const uint64_t* flags, int kind, int world, int me, uint64_t timeout_ns,
                               int32_t* status) {
  const uint64_t epoch = current_epoch(flags);
  const int g = threadIdx.x;
  if (g < world && g != me) {
    if (!wait_flag(flags + kind * kMaxRanks + g, epoch, timeout_ns)) atomicOr(status, DMOE_DEVERR_EP_TIMEOUT);
  }
}

__global__ void ep_signal_kernel(EpPeers peers, int kind) {
  const uint64_t epoch = current_epoch(peers.flags[peers.rank]);
  __threadfence_system();
  const int g = threadIdx.x;
  if (g < peers.world) st_release_sys(peers.flags[g] + kind * kMaxRanks + peers.rank, epoch);
}

// ------------------------------------------------------------------------- ep_combine
// One 16-byte vector <-> its elements as floats: 8 of a 16-bit type, 4 of fp32.
template <int DT>
__device__ __forceinline__ void unpack_vec(const uint4& v, float* f) {
  if constexpr (DT == DMOE_F32) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  } else {
    unpack8<DT>(v, f);
  }
}

template <int DT>
__device__ __forceinline__ uint4 pack_vec(const float* f) {
  if constexpr (DT == DMOE_F32) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  } else {
    return make_uint4(pack2<DT>(f[0], f[1]), pack2<DT>(f[2], f[3]), pack2<DT>(f[4], f[5]), pack2<DT>(f[6], f[7]));
  }
}

template <int DT, int KU, int CU>
__global__ void __launch_bounds__(256) ep_combine_kernel(const char* __restrict__ rows, const int32_t* __restrict__ inverse,
                                                         const int32_t* __restrict__ ret, const void* __restrict__ w,
                                                         int w_dtype, int T, int k, int d, int accumulate,
                                                         void* __restrict__ out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  constexpr int EV = DT == DMOE_F32 ? 4 : 8;  // elements per 16-byte vector
  const int nchunk = d / EV;
  const int64_t row_vecs = d / EV;  // 16-byte vectors per row
  for (int t = warp; t < T; t += nwarps) {
    const uint4* src[KU];
    float wt[KU];
#pragma unroll
    for (int s = 0; s < KU; ++s) {
      src[s] = nullptr;
      wt[s] = 0.f;
      if (s < k) {
        // The owner's epilogue wrote slot (t, s) at row t*k + s unless the activation was
        // dropped (no alive instance, or past a receive buffer's capacity).
        const int32_t pos = inverse[(int64_t)t * k + s];
        const int32_t code = pos < 0 ? -1 : ret[pos];
        if (code >= 0) {
          src[s] = reinterpret_cast<const uint4*>(rows) + ((int64_t)t * k + s) * row_vecs;
          wt[s] = load_as_float(w, (int64_t)t * k + s, w_dtype);
        }
      }
    }
    for (int c0 = lane; c0 < nchunk; c0 += 32 * CU) {
      uint4 raw[CU][KU];
#pragma unroll
      for (int u = 0; u < CU; ++u) {
        const int c = c0 + u * 32;
#pragma unroll
        for (int s = 0; s < KU; ++s)
          if (s < k && c < nchunk && src[s] != nullptr) raw[u][s] = __ldcg(src[s] + c);
      }
#pragma unroll
      for (int u = 0; u < CU; ++u) {
        const int c = c0 + u * 32;
        if (c >= nchunk) break;
        float acc[EV];
        uint4* o = reinterpret_cast<uint4*>(out) + (int64_t)t * row_vecs + c;
        if (accumulate) {
          unpack_vec<DT>(*o, acc);
        } else {
#pragma unroll
          for (int j = 0; j < EV; ++j) acc[j] = 0.f;
        }
#pragma unroll
        for (int s = 0; s < KU; ++s) {
          if (s < k && src[s] != nullptr) {
            float v[EV];
            unpack_vec<DT>(raw[u][s], v);
#pragma unroll
            for (int j = 0; j < EV; ++j) acc[j] = fmaf(wt[s], v[j], acc[j]);
          }
        }
        *o = pack_vec<DT>(acc);
      }
    }
  }
}

template <int DT>
void launch_ep_combine(int blocks, cudaStream_t s, const char* rows, const int32_t* inverse, const int32_t* ret,
                       const void* w, int w_dtype, int T, int k, int d, int accumulate, void* out) {
  if (k <= 2)
    ep_combine_kernel<DT, 2, 4><<<blocks, 256, 0, s>>>(rows, inverse, ret, w, w_dtype, T, k, d, accumulate, out);
  else if (k <= 4)
    ep_combine_kernel<DT, 4, 2><<<blocks, 256, 0, s>>>(rows, inverse, ret, w, w_dtype, T, k, d, accumulate, out);
  else if (k <= 8)
    ep_combine_kernel<DT, 8, 1><<<blocks, 256, 0, s>>>(rows, inverse, ret, w, w_dtype, T, k, d, accumulate, out);
  else
    ep_combine_kernel<DT, 16, 1><<<blocks, 256, 0, s>>>(rows, inverse, ret, w, w_dtype, T, k, d, accumulate, out);
}

int fill_peers(EpPeers* p, const dmoe_ep_window* w) {
  DMOE_REQUIRE(w != nullptr, "dmoe_ep: null window table");
  DMOE_REQUIRE(w->world >= 1 && w->world <= kMaxRanks, "dmoe_ep: world %d not in [1, %d]", w->world, kMaxRanks);
  DMOE_REQUIRE(w->rank >= 0 && w->rank < w->world, "dmoe_ep: rank %d not in [0, %d)", w->rank, w->world);
  p->world = w->world;
  p->rank = w->rank;
  for (int g = 0; g < kMaxRanks; ++g) {
    const bool in = g < w->world;
    p->flags[g] = in ? reinterpret_cast<uint64_t*>(w->flags[g]) : nullptr;
    p->counts[g] = in ? reinterpret_cast<int32_t*>(w->counts[g]) : nullptr;
    p->recv[g] = in ? reinterpret_cast<char*>(w->recv[g]) : nullptr;
    p->back[g] = in ? reinterpret_cast<int32_t*>(w->back[g]) : nullptr;
    p->rows[g] = in ? reinterpret_cast<char*>(w->rows[g]) : nullptr;
    if (in) {
      DMOE_REQUIRE(w->recv[g] && w->rows[g] && w->back[g] && aligned16(w->recv[g]) && aligned16(w->rows[g]),
                   "dmoe_ep: rank %d's receive rows, back map and return rows must be device pointers (rows "
                   "16-byte aligned)", g);
      DMOE_REQUIRE(w->flags[g] != nullptr, "dmoe_ep: rank %d has no flag array", g);
      if (w->world > 1) DMOE_REQUIRE(w->counts[g] != nullptr, "dmoe_ep: rank %d has no count matrix", g);
    }
  }
  return DMOE_OK;
}

}  // namespace
}  // namespace dmoe

using namespace dmoe;

extern "C" size_t dmoe_ep_flags_bytes(void) { return (size_t)(kEpochSlot + 1) * sizeof(uint64_t); }

extern "C" size_t dmoe_ep_counts_bytes(int n_inst) {
  return (size_t)2 * kMaxRanks * (size_t)(n_inst > 0 ? n_inst : 0) * sizeof(int32_t);
}

extern "C" int dmoe_ep_plan(const dmoe_ep_window* win, const int32_t* counts_e, int E, int n_inst, int policy,
                            const int32_t* alive_n, const int32_t* alive_inst, const int32_t* inst_rank,
                            const int32_t* inst_slot, const int32_t* inst_first, int64_t cap, uint64_t timeout_ns, int32_t* part_n, int32_t* part_inst, int32_t* part_start,
                            int32_t* dest_off, int32_t* seg_expert, int32_t* seg_end, int32_t* dev_status,
                            void* stream) {
  clear_error();
  EpPlanArgs a{};
  int r = fill_peers(&a.peers, win);
  if (r) return r;
  DMOE_REQUIRE(E >= 1 && E <= 1024, "dmoe_ep_plan: E=%d not in [1, 1024]", E);
  DMOE_REQUIRE(n_inst >= 1 && n_inst <= kMaxInstances, "dmoe_ep_plan: %d instances not in [1, %d]", n_inst,
               kMaxInstances);
  DMOE_REQUIRE(policy == DMOE_EP_POLICY_ROTATE || policy == DMOE_EP_POLICY_SPLIT, "dmoe_ep_plan: bad policy %d",
               policy);
  DMOE_REQUIRE(cap >= 0 && cap < (1ll << kRowShift), "dmoe_ep_plan: capacity %lld rows not in [0, 2^27)",
               (long long)cap);
  DMOE_REQUIRE(alive_n && alive_inst && inst_rank && inst_slot && inst_first && part_n && part_inst && part_start &&
                   dest_off && seg_expert && seg_end && dev_status,
               "dmoe_ep_plan: null pointer");
  a.counts_e = counts_e;
  a.E = E;
  a.n_inst = n_inst;
  a.policy = policy;
  a.alive_n = alive_n;
  a.alive_inst = alive_inst;
  a.inst_rank = inst_rank;
  a.inst_slot = inst_slot;
  a.inst_first = inst_first;
  a.cap = cap;
  a.timeout_ns = timeout_ns;
  a.status = dev_status;
  a.part_n = part_n;
  a.part_inst = part_inst;
  a.part_start = part_start;
  a.dest_off = dest_off;
  a.seg_expert = seg_expert;
  a.seg_end = seg_end;
  ep_plan_kernel<<<1, 1024, 0, as_stream(stream)>>>(a);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

extern "C" int dmoe_ep_dispatch(const dmoe_ep_window* win, const void* x, int64_t row_bytes, int T, int k, int E,
                                const int32_t* offsets, const int32_t* perm_token, const int32_t* perm_slot,
                                const int32_t* part_n, const int32_t* part_inst, const int32_t* part_start,
                                const int32_t* inst_rank, const int32_t* dest_off, int64_t cap, int32_t* ret,
                                uint32_t* done, int32_t* dev_status, void* stream) {
  clear_error();
  EpDispatchArgs a{};
  int r = fill_peers(&a.peers, win);
  if (r) return r;
  DMOE_REQUIRE(T >= 0 && k >= 1 && (int64_t)T * k < (1ll << 31), "dmoe_ep_dispatch: bad T=%d k=%d", T, k);
  DMOE_REQUIRE(E >= 1 && E <= 1024, "dmoe_ep_dispatch: E=%d not in [1, 1024]", E);
  DMOE_REQUIRE(row_bytes > 0 && row_bytes % 16 == 0, "dmoe_ep_dispatch: row_bytes=%lld must be a multiple of 16",
               (long long)row_bytes);
  DMOE_REQUIRE(cap >= 0 && cap < (1ll << kRowShift), "dmoe_ep_dispatch: capacity %lld rows", (long long)cap);
  DMOE_REQUIRE(done && dev_status && part_n && part_inst && part_start && inst_rank && dest_off,
               "dmoe_ep_dispatch: null pointer");
  if (T > 0)
    DMOE_REQUIRE(x && aligned16(x) && offsets && perm_token && perm_slot && ret,
                 "dmoe_ep_dispatch: null or unaligned x, or a missing plan array");
  DMOE_REQUIRE((int64_t)T * k < (1ll << kRowShift), "dmoe_ep_dispatch: T*k=%lld exceeds 2^27 return rows",
               (long long)T * k);
  a.x = reinterpret_cast<const char*>(x);
  a.row_vecs = row_bytes / 16;
  a.n = (int64_t)T * k;
  a.E = E;
  a.offsets = offsets;
  a.perm_token = perm_token;
  a.perm_slot = perm_slot;
  a.k = k;
  a.part_n = part_n;
  a.part_inst = part_inst;
  a.part_start = part_start;
  a.inst_rank = inst_rank;
  a.dest_off = dest_off;
  a.cap = cap;
  a.ret = ret;
  a.done = done;
  a.status = dev_status;
  int64_t blocks = (a.n + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;  // an empty batch still raises the data flags
  if (E <= kTableMaxE)
    ep_dispatch_kernel<true><<<(int)blocks, 256, 0, as_stream(stream)>>>(a);
  else
    ep_dispatch_kernel<false><<<(int)blocks, 256, 0, as_stream(stream)>>>(a);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

extern "C" int dmoe_ep_wait(const dmoe_ep_window* win, int kind, uint64_t timeout_ns, int32_t* dev_status,
                            void* stream) {
  clear_error();
  EpPeers p{};
  int r = fill_peers(&p, win);
  if (r) return r;
  DMOE_REQUIRE(kind >= 0 && kind < kFlagKinds, "dmoe_ep_wait: bad flag kind %d", kind);
  DMOE_REQUIRE(dev_status, "dmoe_ep_wait: null status");
  if (p.world == 1) return DMOE_OK;
  ep_wait_kernel<<<1, 32, 0, as_stream(stream)>>>(p.flags[p.rank], kind, p.world, p.rank, timeout_ns, dev_status);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

extern "C" int dmoe_ep_signal(const dmoe_ep_window* win, int kind, void* stream) {
  clear_error();
  EpPeers p{};
  int r = fill_peers(&p, win);
  if (r) return r;
  DMOE_REQUIRE(kind >= 0 && kind < kFlagKinds, "dmoe_ep_signal: bad flag kind %d", kind);
  if (p.world == 1) return DMOE_OK;
  ep_signal_kernel<<<1, 32, 0, as_stream(stream)>>>(p, kind);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

extern "C" int dmoe_ep_combine(const dmoe_ep_window* win, const int32_t* inverse, const int32_t* ret, const void* w,
                               int w_dtype, int T, int k, int d, int dtype, int accumulate, void* out, void* stream) {
  clear_error();
  EpPeers p{};
  int r = fill_peers(&p, win);
  if (r) return r;
  DMOE_REQUIRE(T >= 0 && k >= 1 && k <= 16, "dmoe_ep_combine: bad T=%d k=%d", T, k);
  DMOE_REQUIRE(d > 0 && d % 8 == 0, "dmoe_ep_combine: d=%d must be a multiple of 8", d);
  DMOE_REQUIRE(dtype == DMOE_BF16 || dtype == DMOE_F16 || dtype == DMOE_F32,
               "dmoe_ep_combine: rows must be f16, bf16 or f32");
  DMOE_REQUIRE(dtype_ok(w_dtype), "dmoe_ep_combine: bad weight dtype");
  if (T == 0) return DMOE_OK;
  DMOE_REQUIRE(inverse && ret && w && out && aligned16(out), "dmoe_ep_combine: null or unaligned pointer");
  int blocks = (T + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  cudaStream_t s = as_stream(stream);
  const char* rows = p.rows[p.rank];
  if (dtype == DMOE_BF16)
    launch_ep_combine<DMOE_BF16>(blocks, s, rows, inverse, ret, w, w_dtype, T, k, d, accumulate, out);
  else if (dtype == DMOE_F32)
    launch_ep_combine<DMOE_F32>(blocks, s, rows, inverse, ret, w, w_dtype, T, k, d, accumulate, out);
  else
    launch_ep_combine<DMOE_F16>(blocks, s, rows, inverse, ret, w, w_dtype, T, k, d, accumulate, out);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}
