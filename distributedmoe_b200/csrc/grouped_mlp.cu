// Grouped expert gated MLP on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the grouped path of ExpertsBlockPipelineTask.run (MoE/PipelineTask.py:478-520):
//   gate_out = grouped_mm(X, Wg^T, offs); up_out = grouped_mm(X, Wu^T, offs)
//   h = relu(gate_out) * up_out;           Y = grouped_mm(h, Wd^T, offs)
// where offs are the cumulative (padded) ends of the per-expert row segments of one buffer.
// The reference also copies the active experts' weights each run (:511-513); here the
// kernels index the stacked weights by expert id through a 3-D TMA descriptor instead.
//
// Two launches of one persistent, warp-specialised kernel template:
//   GEMM1 (gated): tile = 128 rows x (128 gate + 128 up) columns, K = d.  The MMA is
//                  M=128, N=256: the B tile stacks the gate rows and the matching up rows,
//                  so one accumulator holds both halves and the epilogue writes
//                  h = act(gate) * up (128 columns) straight from TMEM.
//   GEMM2 (plain): tile = 128 rows x 256 columns of Y, K = I.
// Roles per CTA (192 threads, one CTA per SM):
//   warp 0      TMA producer: A tile [128 x 64] and B tile [256 x 64] per stage, SW128
//   warp 1      TMEM allocator + MMA issuer: 4 x tcgen05.mma (K=16) per stage
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, activation, 16-byte stores
// Smem ring of 4 stages (48 KB each); TMEM holds two 256-column fp32 accumulators so the
// epilogue of tile i overlaps the MMAs of tile i+1.  Every mbarrier wait is bounded by time
// and reports through the caller's device status word instead of hanging.
#include <cuda.h>

#include <cstdlib>
#include <cstring>

#include "dmoe_common.cuh"

namespace dmoe {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;    // one 128-byte swizzle atom of 16-bit elements

// Elements in one 128-byte swizzle row: 64 of a 16-bit type, 128 of e4m3, 32 of fp32.
// Shared-memory tiles, barriers and MMA counts are byte-based and the same for all; only the
// K extent of a box and the MMA kind change (one kind::f16 MMA takes K=16, one kind::f8f6f4
// MMA K=32, one kind::tf32 MMA K=8: 32 bytes of a row each).
template <int DT>
__host__ __device__ constexpr int row_elems() {
  return DT == DMOE_E4M3 ? 128 : (DT == DMOE_F32 ? 32 : 64);
}

// Type a GEMM on DT operands stores: e4m3 products are stored as bf16.
template <int DT>
__host__ __device__ constexpr int out_dtype() {
  return DT == DMOE_E4M3 ? DMOE_BF16 : DT;
}
constexpr int BN = 256;   // MMA N
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;
constexpr int kThreads = 192;
constexpr int kMaxSegDev = 1024;
constexpr int kMaxSegParam = 512;  // host tables hold up to 256 segments; the pair/single split doubles that
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

constexpr int kBarBytes = 256;
constexpr int kSegBytes = 4 * (kMaxSegDev + 1) * 4;
constexpr int kSmemBytes = 1024 /*align slack*/ + STAGES * STAGE_BYTES + kBarBytes + kSegBytes;

struct GemmSegs {
  int n_seg;
  int m_rows;
  int e_stack;
  // Which rows of each segment a launch computes: 0 all; 1 the pair kernel's part of a
  // split (the whole 256-row blocks, plus the remainder when it exceeds 128 rows); 2 the
  // single-SM kernel's part (a remainder of at most 128 rows, one 128-row tile).
  int split;
  const int32_t* dev_expert;
  const int32_t* dev_end;
  int32_t expert[kMaxSegParam];
  int32_t end[kMaxSegParam];
};

struct GemmArgs {
  void* out;
  int64_t ldo;      // elements between output rows
  int n_out;        // valid output columns
  int K;            // reduction length
  int n_tiles_n;    // output column tiles
  int raster_n_fast;  // tile order: 0 M fastest over all segments, 1 N fastest, 2 segment by segment, M fastest
  int act;
  int prefetch;     // k-blocks of L2 prefetch ahead of the TMA loads (0: off)
  int32_t* status;
  int out_f32;      // plain GEMM only: store the fp32 accumulators instead of rounding to DT
  // plain GEMM only: instead of row r of `out`, store row r at scatter_base[code >> 27] +
  // (code & 0x7ffffff) rows, code = scatter_map[r] (code < 0: the row is not stored).  The
  // bases may be other GPUs' memory (peer stores over NVLink).
  int scatter;
  const int32_t* scatter_map;
  char* scatter_base[DMOE_EP_MAX_RANKS];
  // e4m3 gated GEMM only: the fp32 scale of each A row (a_scale_ld floats apart) and of each
  // B row of the gate / up stacks ([E_stack][n_out]); the epilogue multiplies every
  // accumulator by its row's and its column's scale.
  const float* a_scale;
  int a_scale_ld;
  const float* b0_scale;
  const float* b1_scale;
};

// Destination of output row `row` of a plain GEMM with ESZ-byte elements (nullptr: not stored).
template <int ESZ>
__device__ __forceinline__ char* out_row(const GemmArgs& args, int row, bool valid) {
  if (!valid) return nullptr;
  if (!args.scatter) return reinterpret_cast<char*>(args.out) + (int64_t)row * args.ldo * ESZ;
  const int32_t code = args.scatter_map[row];
  if (code < 0) return nullptr;
  char* base = args.scatter_base[(uint32_t)code >> 27];  // index <= 15: code is non-negative
  if (base == nullptr) return nullptr;                    // no such rank: never stored
  return base + (int64_t)(code & 0x7ffffff) * args.ldo * ESZ;
}

// ------------------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: true once the phase of `parity` completed; false on timeout or when another
// role of this CTA already gave up (abort flag).
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int32_t* status,
                                            int code) {
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1;
      atomicOr(status, code);
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int32_t* status,
                                          int code) {
  return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity, abort_flag, status, code);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// L2 prefetch of a tile (no shared memory, no barrier): hides the DRAM latency of the
// weight tiles that several CTAs request at the same time.
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

template <int DT>
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  if constexpr (DT == DMOE_E4M3) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (DT == DMOE_F32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

#define DMOE_R8(b) "=r"(r[b + 0]), "=r"(r[b + 1]), "=r"(r[b + 2]), "=r"(r[b + 3]), "=r"(r[b + 4]), "=r"(r[b + 5]), \
                   "=r"(r[b + 6]), "=r"(r[b + 7])
#define DMOE_S8(b) "=r"(s[b + 0]), "=r"(s[b + 1]), "=r"(s[b + 2]), "=r"(s[b + 3]), "=r"(s[b + 4]), "=r"(s[b + 5]), \
                   "=r"(s[b + 6]), "=r"(s[b + 7])

// 32 lanes x 32 consecutive fp32 columns, then wait: the outputs exist only after the wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : DMOE_R8(0), DMOE_R8(8), DMOE_R8(16), DMOE_R8(24)
      : "r"(taddr)
      : "memory");
}

// Two 32-column loads (gate part and up part of the accumulator) and one wait.
__device__ __forceinline__ void tmem_ld32x2(uint32_t ta, uint32_t tb, uint32_t (&r)[32], uint32_t (&s)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, "
      "%46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : DMOE_R8(0), DMOE_R8(8), DMOE_R8(16), DMOE_R8(24), DMOE_S8(0), DMOE_S8(8), DMOE_S8(16), DMOE_S8(24)
      : "r"(ta), "r"(tb)
      : "memory");
}

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle layout written by
// TMA (rows of 128 bytes, 8-row groups 1024 bytes apart): LBO = 16 B (unused), SBO = 1024 B,
// descriptor version 1 (sm_100), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: D fp32 (bit 4), A and B formats at bits 7 and 10 (kind::f16: f16 0,
// bf16 1; kind::tf32: tf32 2; kind::f8f6f4: e4m3 0), both K-major, N >> 3 at bit 17, M >> 4
// at bit 24; M=128, N=256.
template <int DT>
__host__ __device__ constexpr uint32_t operand_format() {
  return DT == DMOE_BF16 ? 1u : (DT == DMOE_F32 ? 2u : 0u);
}

template <int DT>
__host__ __device__ constexpr uint32_t make_idesc() {
  return (1u << 4) | (operand_format<DT>() << 7) | (operand_format<DT>() << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ float act_fn(float g, int act) {
  return act == DMOE_ACT_SILU ? g / (1.f + __expf(-g)) : fmaxf(g, 0.f);
}

struct TileInfo {
  int row0, row_end, expert, nt;
};

// The part of a segment [first, first + len) that a launch with split mode `split` computes
// (see GemmSegs::split); updates len and returns the first row.
__device__ __forceinline__ int split_rows(int split, int first, int& len) {
  if (split == 0) return first;
  int full = (len / 256) * 256;
  if (len - full > 128) full = len;
  if (split == 1) {
    len = full;
    return first;
  }
  len -= full;
  return first + full;
}

template <int TILE_M>
__device__ __forceinline__ TileInfo decode_tile(int tile, int total_m, int n_tiles_n, int raster_n_fast, int n_seg,
                                                const int32_t* s_start, const int32_t* s_end,
                                                const int32_t* s_expert, const int32_t* s_tile) {
  int mt, nt;
  if (raster_n_fast == 2) {
    // Segment by segment, M fastest inside one: the tiles in flight together share one
    // expert's weight columns (read from DRAM once, then from L2) and its few row tiles.
    int lo = 0, hi = n_seg - 1;  // last segment whose first tile is <= tile (skips empty segments)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((int64_t)s_tile[mid] * n_tiles_n <= tile) lo = mid; else hi = mid - 1;
    }
    const int mt_seg = s_tile[lo + 1] - s_tile[lo];
    const int local = tile - s_tile[lo] * n_tiles_n;
    nt = local / mt_seg;
    const int m_in = local - nt * mt_seg;
    TileInfo ti;
    ti.row0 = s_start[lo] + m_in * TILE_M;
    ti.row_end = s_end[lo];
    ti.expert = s_expert[lo];
    ti.nt = nt;
    return ti;
  }
  if (raster_n_fast) {
    mt = tile / n_tiles_n;
    nt = tile - mt * n_tiles_n;
  } else {
    nt = tile / total_m;
    mt = tile - nt * total_m;
  }
  int lo = 0, hi = n_seg - 1;  // last segment whose first tile is <= mt (skips empty segments)
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_tile[mid] <= mt) lo = mid; else hi = mid - 1;
  }
  TileInfo ti;
  ti.row0 = s_start[lo] + (mt - s_tile[lo]) * TILE_M;
  ti.row_end = s_end[lo];
  ti.expert = s_expert[lo];
  ti.nt = nt;
  return ti;
}

template <bool GATED, int DT>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b0,
                        const __grid_constant__ CUtensorMap tm_b1, const __grid_constant__ GemmSegs segs,
                        const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint64_t* acce = accf + 2;
  uint64_t* fin = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* s_start = reinterpret_cast<int32_t*>(smem + STAGES * STAGE_BYTES + kBarBytes);
  int32_t* s_end = s_start + (kMaxSegDev + 1);
  int32_t* s_expert = s_end + (kMaxSegDev + 1);
  int32_t* s_tile = s_expert + (kMaxSegDev + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_seg = segs.n_seg;

  for (int i = threadIdx.x; i < n_seg; i += blockDim.x) {
    s_expert[i] = segs.dev_expert ? segs.dev_expert[i] : segs.expert[i];
    s_end[i] = segs.dev_end ? segs.dev_end[i] : segs.end[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int prev = 0, tiles = 0, bad = 0;
    for (int i = 0; i < n_seg; ++i) {
      int en = s_end[i];
      if (en < prev || en > segs.m_rows) {
        bad = 1;
        en = en < prev ? prev : segs.m_rows;
      }
      int e = s_expert[i];
      int len = en - prev;
      if (e == -1) {  // rows another launch computes
        len = 0;
        s_expert[i] = 0;
      } else if (e < 0 || e >= segs.e_stack) {
        bad = 1;
        len = 0;
        s_expert[i] = 0;
      }
      const int first = split_rows(segs.split, prev, len);
      s_start[i] = first;
      s_end[i] = first + len;
      s_tile[i] = tiles;
      tiles += (len + BM - 1) / BM;
      prev = en;
    }
    s_tile[n_seg] = tiles;
    if (bad && blockIdx.x == 0) atomicOr(args.status, DMOE_DEVERR_BAD_SEGMENT);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 4);
    }
    mbar_init(fin, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_m = s_tile[n_seg];
  const int total = total_m * args.n_tiles_n;
  constexpr int RE = row_elems<DT>();
  const int nk = (args.K + RE - 1) / RE;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      uint32_t armed = 0, armed_ph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const TileInfo ti = decode_tile<BM>(tile, total_m, args.n_tiles_n, args.raster_n_fast, n_seg, s_start, s_end,
                                        s_expert, s_tile);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], ph ^ 1u, abort_flag, args.status, DMOE_DEVERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sa, &tm_a, &full[stage], kb * RE, ti.row0);
          if constexpr (GATED) {
            tma_load_3d(sb, &tm_b0, &full[stage], kb * RE, ti.nt * (BN / 2), ti.expert);
            tma_load_3d(sb + B_BYTES / 2, &tm_b1, &full[stage], kb * RE, ti.nt * (BN / 2), ti.expert);
          } else {
            tma_load_3d(sb, &tm_b0, &full[stage], kb * RE, ti.nt * BN, ti.expert);
          }
          const int kp = kb + args.prefetch;
          if (args.prefetch > 0 && kp < nk) {
            tma_prefetch_2d(&tm_a, kp * RE, ti.row0);
            if constexpr (GATED) {
              tma_prefetch_3d(&tm_b0, kp * RE, ti.nt * (BN / 2), ti.expert);
              tma_prefetch_3d(&tm_b1, kp * RE, ti.nt * (BN / 2), ti.expert);
            } else {
              tma_prefetch_3d(&tm_b0, kp * RE, ti.nt * BN, ti.expert);
            }
          }
          armed |= 1u << stage;
          armed_ph = (armed_ph & ~(1u << stage)) | (ph << stage);
          if (++stage == STAGES) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
      // Every copy this thread started must land before the CTA exits.
      for (int s = 0; s < STAGES; ++s) {
        if (armed >> s & 1u) {
          const uint64_t t0 = global_timer_ns();
          while (!mbar_try_wait(&full[s], armed_ph >> s & 1u)) {
            if (global_timer_ns() - t0 > kWaitTimeoutNs) {
              atomicOr(args.status, DMOE_DEVERR_TIMEOUT_TEARDOWN);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc<DT>();
      int stage = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        if (!mbar_wait(&acce[acc], acc_ph ^ 1u, abort_flag, args.status, DMOE_DEVERR_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], ph, abort_flag, args.status, DMOE_DEVERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sdesc_sw128(smem_u32(smem + stage * STAGE_BYTES));
          const uint64_t bd = sdesc_sw128(smem_u32(smem + stage * STAGE_BYTES + A_BYTES));
#pragma unroll
          for (int k = 0; k < 4; ++k)  // 32 bytes of K per MMA: +2 in the address field
            umma_f16<DT>(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&accf[acc]);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1u;
      }
      // All MMAs issued by this thread complete before TMEM is released.
      umma_commit(fin);
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(fin, 0)) {
        if (global_timer_ns() - t0 > kWaitTimeoutNs) {
          atomicOr(args.status, DMOE_DEVERR_TIMEOUT_TEARDOWN);
          break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      const TileInfo ti = decode_tile<BM>(tile, total_m, args.n_tiles_n, args.raster_n_fast, n_seg, s_start, s_end,
                                      s_expert, s_tile);
      const bool got = mbar_wait(&accf[acc], acc_ph, abort_flag, args.status, DMOE_DEVERR_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const int row = ti.row0 + q * 32 + lane;
      const bool valid = row < ti.row_end;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      if constexpr (GATED) {
#pragma unroll 1
        for (int j = 0; j < 4; ++j) {
          uint32_t g[32], u[32];
          __syncwarp();
          tmem_ld32x2(tbase + j * 32, tbase + BN / 2 + j * 32, g, u);
          const int col0 = ti.nt * (BN / 2) + j * 32;
          if (valid && DT == DMOE_F32) {
            // fp32 operands (tf32 MMAs): h is stored in fp32, eight 16-byte vectors per 32 columns
            float* dst = reinterpret_cast<float*>(args.out) + (int64_t)row * args.ldo + col0;
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              float h[4];
#pragma unroll
              for (int i = 0; i < 4; ++i)
                h[i] = act_fn(__uint_as_float(g[4 * v + i]), args.act) * __uint_as_float(u[4 * v + i]);
              if (col0 + v * 4 < args.n_out) *reinterpret_cast<float4*>(dst + v * 4) = make_float4(h[0], h[1], h[2], h[3]);
            }
          } else if (valid) {
            uint32_t pk[16];
            if constexpr (DT == DMOE_E4M3) {
              // e4m3 operands: back to scale by the row's and each column's quantisation scale.
              const float sa = args.a_scale[(int64_t)row * args.a_scale_ld];
              const float* sg = args.b0_scale + (int64_t)ti.expert * args.n_out;
              const float* su = args.b1_scale + (int64_t)ti.expert * args.n_out;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int c = col0 + 2 * i;
                const float g0 = c < args.n_out ? __uint_as_float(g[2 * i]) * sa * sg[c] : 0.f;
                const float u0 = c < args.n_out ? __uint_as_float(u[2 * i]) * sa * su[c] : 0.f;
                const float g1 = c + 1 < args.n_out ? __uint_as_float(g[2 * i + 1]) * sa * sg[c + 1] : 0.f;
                const float u1 = c + 1 < args.n_out ? __uint_as_float(u[2 * i + 1]) * sa * su[c + 1] : 0.f;
                pk[i] = pack2<out_dtype<DT>()>(act_fn(g0, args.act) * u0, act_fn(g1, args.act) * u1);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float h0 = act_fn(__uint_as_float(g[2 * i]), args.act) * __uint_as_float(u[2 * i]);
                const float h1 = act_fn(__uint_as_float(g[2 * i + 1]), args.act) * __uint_as_float(u[2 * i + 1]);
                pk[i] = pack2<DT>(h0, h1);
              }
            }
            char* dst = reinterpret_cast<char*>(args.out) + ((int64_t)row * args.ldo + col0) * 2;
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col0 + v * 8 < args.n_out)
                *reinterpret_cast<uint4*>(dst + v * 16) = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
          }
        }
      } else {
        char* const drow = args.out_f32 ? nullptr : out_row<DT == DMOE_F32 ? 4 : 2>(args, row, valid);
#pragma unroll 1
        for (int j = 0; j < BN / 32; ++j) {
          uint32_t y[32];
          __syncwarp();
          tmem_ld32(tbase + j * 32, y);
          const int col0 = ti.nt * BN + j * 32;
          if (valid && args.out_f32) {
            float* dst = reinterpret_cast<float*>(args.out) + (int64_t)row * args.ldo + col0;
#pragma unroll
            for (int v = 0; v < 8; ++v)
              if (col0 + v * 4 < args.n_out)
                *reinterpret_cast<uint4*>(dst + v * 4) = make_uint4(y[4 * v], y[4 * v + 1], y[4 * v + 2], y[4 * v + 3]);
          } else if (drow != nullptr && DT == DMOE_F32) {
            float* dst = reinterpret_cast<float*>(drow) + col0;
#pragma unroll
            for (int v = 0; v < 8; ++v)
              if (col0 + v * 4 < args.n_out)
                *reinterpret_cast<uint4*>(dst + v * 4) = make_uint4(y[4 * v], y[4 * v + 1], y[4 * v + 2], y[4 * v + 3]);
          } else if (drow != nullptr) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) pk[i] = pack2<DT>(__uint_as_float(y[2 * i]), __uint_as_float(y[2 * i + 1]));
            char* dst = drow + (int64_t)col0 * 2;
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col0 + v * 8 < args.n_out)
                *reinterpret_cast<uint4*>(dst + v * 16) = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[acc]);
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1u;
    }
  }

  // Scattered rows may live in other GPUs' memory: make them visible system-wide before the
  // kernel ends (the caller raises a flag the other GPUs act on after this launch).
  if (args.scatter) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------- 2-SM variant
// A CTA pair (cluster of 2) computes a 256-row x 256-column tile with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=16).  Each CTA loads its own 128 rows of A and
// its own half of B (128 of the 256 B rows), which
// halves the B traffic per SM.  A stage spans K=128 (two 64-wide TMA boxes per operand,
// 8 MMAs per barrier round): 3 stages of 64 KB.  Each CTA's TMEM holds its 128 rows x 256
// fp32 columns; each CTA's epilogue drains its own TMEM.  For the gated GEMM, CTA 0's B
// half is the gate tile and CTA 1's the up tile, so each accumulator again holds gate in
// columns 0..127 and up in 128..255.
// Synchronisation (all waits bounded):
//   full[s]   (leader only) count 1: the leader's producer arms expect_tx with both CTAs'
//             bytes; both CTAs' TMA loads (.cta_group::2) complete on the leader's barrier.
//   empty[s]  (both) count 1: the leader's MMA commit arrives on both CTAs.
//   accf[a]   (both) count 1: the leader's commit after a tile arrives on both CTAs.
//   acce[a]   (leader) count 8: 4 epilogue warps of each CTA (the peer's remotely).
//   bye       (both) count 1: exit handshake, so no CTA leaves while the peer may still
//             touch its shared memory.
constexpr int BM2 = 256;
constexpr int STAGES2 = 3;                    // a stage: two 128-byte swizzle rows of K, 8 MMAs per barrier round
constexpr int SUB2_BYTES = 128 * BK * 2;      // one box: 128 rows x 128 bytes
constexpr int A2_BYTES = 2 * SUB2_BYTES;
constexpr int B2_BYTES = 2 * SUB2_BYTES;
constexpr int STAGE2_BYTES = A2_BYTES + B2_BYTES;
constexpr int kSmemBytes2 = 1024 + STAGES2 * STAGE2_BYTES + kBarBytes + kSegBytes;

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t map_to_cta(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                                 int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

template <int DT>
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  if constexpr (DT == DMOE_E4M3) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (DT == DMOE_F32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Arrive on the barrier at this offset in both CTAs of the pair once the MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_both(uint64_t* bar) {
  const uint16_t both = 0x3;
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                   "r"(smem_u32(bar)),
               "h"(both)
               : "memory");
}

template <int DT>
__host__ __device__ constexpr uint32_t make_idesc_pair() {
  return (1u << 4) | (operand_format<DT>() << 7) | (operand_format<DT>() << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM2 >> 4) << 24);
}

template <bool GATED, int DT>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_2sm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b0,
                            const __grid_constant__ CUtensorMap tm_b1, const __grid_constant__ GemmSegs segs,
                            const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES2 * STAGE2_BYTES);
  uint64_t* empty = full + STAGES2;
  uint64_t* accf = empty + STAGES2;
  uint64_t* acce = accf + 2;
  uint64_t* fin = acce + 2;
  uint64_t* bye = fin + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bye + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* s_start = reinterpret_cast<int32_t*>(smem + STAGES2 * STAGE2_BYTES + kBarBytes);
  int32_t* s_end = s_start + (kMaxSegDev + 1);
  int32_t* s_expert = s_end + (kMaxSegDev + 1);
  int32_t* s_tile = s_expert + (kMaxSegDev + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int n_seg = segs.n_seg;
  const int pair = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;

  for (int i = threadIdx.x; i < n_seg; i += blockDim.x) {
    s_expert[i] = segs.dev_expert ? segs.dev_expert[i] : segs.expert[i];
    s_end[i] = segs.dev_end ? segs.dev_end[i] : segs.end[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int prev = 0, tiles = 0, bad = 0;
    for (int i = 0; i < n_seg; ++i) {
      int en = s_end[i];
      if (en < prev || en > segs.m_rows) {
        bad = 1;
        en = en < prev ? prev : segs.m_rows;
      }
      int len = en - prev;
      if (s_expert[i] == -1) {  // rows another launch computes
        len = 0;
        s_expert[i] = 0;
      } else if (s_expert[i] < 0 || s_expert[i] >= segs.e_stack) {
        bad = 1;
        len = 0;
        s_expert[i] = 0;
      }
      const int first = split_rows(segs.split, prev, len);
      s_start[i] = first;
      s_end[i] = first + len;
      s_tile[i] = tiles;
      tiles += (len + BM2 - 1) / BM2;
      prev = en;
    }
    s_tile[n_seg] = tiles;
    if (bad && blockIdx.x == 0) atomicOr(args.status, DMOE_DEVERR_BAD_SEGMENT);
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 8);
    }
    mbar_init(fin, 1);
    mbar_init(bye, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrive or TMA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_m = s_tile[n_seg];
  const int total = total_m * args.n_tiles_n;
  constexpr int RE = row_elems<DT>();  // one swizzle row; a stage holds two
  const int nk = (args.K + 2 * RE - 1) / (2 * RE);
  const uint32_t full_leader0 = map_to_cta(smem_u32(&full[0]), 0);

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      uint32_t armed = 0, armed_ph = 0;
      bool ok = true;
      for (int tile = pair; tile < total && ok; tile += n_pairs) {
        const TileInfo ti = decode_tile<BM2>(tile, total_m, args.n_tiles_n, args.raster_n_fast, n_seg, s_start, s_end,
                                        s_expert, s_tile);
        const int arow = ti.row0 + (int)rank * 128;
        const int brow = GATED ? ti.nt * 128 : ti.nt * BN + (int)rank * 128;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], ph ^ 1u, abort_flag, args.status, DMOE_DEVERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * STAGE2_BYTES;
          uint8_t* sb = sa + A2_BYTES;
          const uint32_t fbar = full_leader0 + (uint32_t)(stage * sizeof(uint64_t));
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * STAGE2_BYTES);
          const CUtensorMap* tb = (GATED && rank == 1) ? &tm_b1 : &tm_b0;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int k0 = kb * 2 * RE + h * RE;  // a box past K reads zeros and still counts its bytes
            tma_load_2d_pair(sa + h * SUB2_BYTES, &tm_a, fbar, k0, arow);
            tma_load_3d_pair(sb + h * SUB2_BYTES, tb, fbar, k0, brow, ti.expert);
          }
          const int kp = kb + args.prefetch;
          if (args.prefetch > 0 && kp < nk) {
            tma_prefetch_2d(&tm_a, kp * 2 * RE, arow);
            tma_prefetch_3d(tb, kp * 2 * RE, brow, ti.expert);
          }
          armed |= 1u << stage;
          armed_ph = (armed_ph & ~(1u << stage)) | (ph << stage);
          if (++stage == STAGES2) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
      // The leader's full barriers count both CTAs' bytes: wait for every phase it armed.
      if (leader) {
        for (int s = 0; s < STAGES2; ++s) {
          if (armed >> s & 1u) {
            const uint64_t t0 = global_timer_ns();
            while (!mbar_try_wait(&full[s], armed_ph >> s & 1u)) {
              if (global_timer_ns() - t0 > kWaitTimeoutNs) {
                atomicOr(args.status, DMOE_DEVERR_TIMEOUT_TEARDOWN);
                break;
              }
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader CTA)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = make_idesc_pair<DT>();
      int stage = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      bool ok = true;
      for (int tile = pair; tile < total && ok; tile += n_pairs) {
        if (!mbar_wait(&acce[acc], acc_ph ^ 1u, abort_flag, args.status, DMOE_DEVERR_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], ph, abort_flag, args.status, DMOE_DEVERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sdesc_sw128(smem_u32(smem + stage * STAGE2_BYTES));
          const uint64_t bd = sdesc_sw128(smem_u32(smem + stage * STAGE2_BYTES + A2_BYTES));
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            // sub-box k/4 (16 KB = 1024 in the descriptor's 16-byte units), then +32 bytes of K per MMA
            const uint64_t off = (uint64_t)((k >> 2) * (SUB2_BYTES >> 4) + 2 * (k & 3));
            umma_f16_pair<DT>(d_tmem, ad + off, bd + off, idesc, (kb | k) != 0);
          }
          umma_commit_both(&empty[stage]);
          if (++stage == STAGES2) {
            stage = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_both(&accf[acc]);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1u;
      }
      umma_commit_both(fin);
    }
    if (lane == 0) {
      // Every MMA of the pair (issued by the leader) has completed once `fin` fires in this CTA.
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(fin, 0)) {
        if (global_timer_ns() - t0 > kWaitTimeoutNs) {
          atomicOr(args.status, DMOE_DEVERR_TIMEOUT_TEARDOWN);
          break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const uint32_t acce_leader0 = map_to_cta(smem_u32(&acce[0]), 0);
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int tile = pair; tile < total; tile += n_pairs) {
      const TileInfo ti = decode_tile<BM2>(tile, total_m, args.n_tiles_n, args.raster_n_fast, n_seg, s_start, s_end,
                                      s_expert, s_tile);
      const bool got = mbar_wait(&accf[acc], acc_ph, abort_flag, args.status, DMOE_DEVERR_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      const int row = ti.row0 + (int)rank * 128 + q * 32 + lane;
      const bool valid = row < ti.row_end;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      if constexpr (GATED) {
#pragma unroll 1
        for (int j = 0; j < 4; ++j) {
          uint32_t g[32], u[32];
          __syncwarp();
          tmem_ld32x2(tbase + j * 32, tbase + BN / 2 + j * 32, g, u);
          const int col0 = ti.nt * (BN / 2) + j * 32;
          if (valid && DT == DMOE_F32) {
            // fp32 operands (tf32 MMAs): h is stored in fp32, eight 16-byte vectors per 32 columns
            float* dst = reinterpret_cast<float*>(args.out) + (int64_t)row * args.ldo + col0;
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              float h[4];
#pragma unroll
              for (int i = 0; i < 4; ++i)
                h[i] = act_fn(__uint_as_float(g[4 * v + i]), args.act) * __uint_as_float(u[4 * v + i]);
              if (col0 + v * 4 < args.n_out) *reinterpret_cast<float4*>(dst + v * 4) = make_float4(h[0], h[1], h[2], h[3]);
            }
          } else if (valid) {
            uint32_t pk[16];
            if constexpr (DT == DMOE_E4M3) {
              // e4m3 operands: back to scale by the row's and each column's quantisation scale.
              const float sa = args.a_scale[(int64_t)row * args.a_scale_ld];
              const float* sg = args.b0_scale + (int64_t)ti.expert * args.n_out;
              const float* su = args.b1_scale + (int64_t)ti.expert * args.n_out;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int c = col0 + 2 * i;
                const float g0 = c < args.n_out ? __uint_as_float(g[2 * i]) * sa * sg[c] : 0.f;
                const float u0 = c < args.n_out ? __uint_as_float(u[2 * i]) * sa * su[c] : 0.f;
                const float g1 = c + 1 < args.n_out ? __uint_as_float(g[2 * i + 1]) * sa * sg[c + 1] : 0.f;
                const float u1 = c + 1 < args.n_out ? __uint_as_float(u[2 * i + 1]) * sa * su[c + 1] : 0.f;
                pk[i] = pack2<out_dtype<DT>()>(act_fn(g0, args.act) * u0, act_fn(g1, args.act) * u1);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const float h0 = act_fn(__uint_as_float(g[2 * i]), args.act) * __uint_as_float(u[2 * i]);
                const float h1 = act_fn(__uint_as_float(g[2 * i + 1]), args.act) * __uint_as_float(u[2 * i + 1]);
                pk[i] = pack2<DT>(h0, h1);
              }
            }
            char* dst = reinterpret_cast<char*>(args.out) + ((int64_t)row * args.ldo + col0) * 2;
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col0 + v * 8 < args.n_out)
                *reinterpret_cast<uint4*>(dst + v * 16) = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
          }
        }
      } else {
        char* const drow = args.out_f32 ? nullptr : out_row<DT == DMOE_F32 ? 4 : 2>(args, row, valid);
#pragma unroll 1
        for (int j = 0; j < BN / 32; ++j) {
          uint32_t y[32];
          __syncwarp();
          tmem_ld32(tbase + j * 32, y);
          const int col0 = ti.nt * BN + j * 32;
          if (valid && args.out_f32) {
            float* dst = reinterpret_cast<float*>(args.out) + (int64_t)row * args.ldo + col0;
#pragma unroll
            for (int v = 0; v < 8; ++v)
              if (col0 + v * 4 < args.n_out)
                *reinterpret_cast<uint4*>(dst + v * 4) = make_uint4(y[4 * v], y[4 * v + 1], y[4 * v + 2], y[4 * v + 3]);
          } else if (drow != nullptr && DT == DMOE_F32) {
            float* dst = reinterpret_cast<float*>(drow) + col0;
#pragma unroll
            for (int v = 0; v < 8; ++v)
              if (col0 + v * 4 < args.n_out)
                *reinterpret_cast<uint4*>(dst + v * 4) = make_uint4(y[4 * v], y[4 * v + 1], y[4 * v + 2], y[4 * v + 3]);
          } else if (drow != nullptr) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) pk[i] = pack2<DT>(__uint_as_float(y[2 * i]), __uint_as_float(y[2 * i + 1]));
            char* dst = drow + (int64_t)col0 * 2;
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col0 + v * 8 < args.n_out)
                *reinterpret_cast<uint4*>(dst + v * 16) = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce_leader0 + (uint32_t)(acc * sizeof(uint64_t)));
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1u;
    }
  }

  if (args.scatter) __threadfence_system();  // scattered rows may live in other GPUs' memory
  tc_fence_before();
  __syncthreads();
  // Exit handshake: tell the peer this CTA is done with the pair's shared state, then wait
  // (bounded) until the peer says the same.
  if (threadIdx.x == 0) {
    mbar_arrive_cluster(map_to_cta(smem_u32(bye), rank ^ 1u));
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bye, 0)) {
      if (global_timer_ns() - t0 > kWaitTimeoutNs) {
        atomicOr(args.status, DMOE_DEVERR_TIMEOUT_TEARDOWN);
        break;
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------- host side
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}

// Encoded maps are reused: weights and registered buffers keep their addresses across calls.
struct MapCacheEntry {
  const void* base;
  int dt, rank;
  uint64_t ld;
  uint64_t dims[3];
  uint32_t box[3];
  int dev;
  CUtensorMap map;
};
constexpr int kMapCache = 64;

// rank-2 or rank-3 row-major tensor of f16, bf16 or e4m3; dims innermost first; box innermost
// first.  ld: bytes between rows (dimension 1) when they are not packed, 0 for packed rows.
int make_map(CUtensorMap* map, int dt, const void* base, int rank, const uint64_t* dims, const uint32_t* box,
             uint64_t ld = 0) {
  static thread_local MapCacheEntry cache[kMapCache];
  static thread_local int cache_n = 0, cache_next = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  for (int i = 0; i < cache_n; ++i) {
    const MapCacheEntry& c = cache[i];
    if (c.base == base && c.dt == dt && c.rank == rank && c.dev == dev && c.ld == ld && c.dims[0] == dims[0] &&
        c.box[0] == box[0] &&
        c.dims[1] == dims[1] && c.box[1] == box[1] && (rank < 3 || (c.dims[2] == dims[2] && c.box[2] == box[2]))) {
      *map = c.map;
      return DMOE_OK;
    }
  }
  PFN_encodeTiled enc = get_encode_fn();
  DMOE_REQUIRE(enc != nullptr, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t gdim[3], gstride[2];
  cuuint32_t bdim[3], estr[3] = {1, 1, 1};
  uint64_t stride = dt == DMOE_E4M3 ? 1 : (dt == DMOE_F32 ? 4 : 2);  // bytes of one element
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    if (i > 0) gstride[i - 1] = stride;
    stride *= dims[i];
    if (i == 0 && ld != 0) stride = ld;
  }
  const CUtensorMapDataType et = dt == DMOE_BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : dt == DMOE_E4M3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : dt == DMOE_F32  ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, et, (cuuint32_t)rank, const_cast<void*>(base), gdim, gstride, bdim, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return DMOE_ERR_CUDA;
  }
  MapCacheEntry& c = cache[cache_next];
  c.base = base;
  c.dt = dt;
  c.rank = rank;
  c.dev = dev;
  c.ld = ld;
  for (int i = 0; i < 3; ++i) {
    c.dims[i] = i < rank ? dims[i] : 0;
    c.box[i] = i < rank ? box[i] : 0;
  }
  c.map = *map;
  cache_next = (cache_next + 1) % kMapCache;
  if (cache_n < kMapCache) ++cache_n;
  return DMOE_OK;
}

// SMs the persistent GEMM leaves free (dmoe_grouped_mlp_set_sm_reserve).  A persistent launch
// holds every SM it gets until its last tile, so without a reserve the small kernels of other
// streams (gathers, the combine, the router of another host's forward) wait for the whole GEMM.
std::atomic<int> g_sm_reserve{0};

template <bool GATED, int DT>
int launch_gemm(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1, const GemmSegs& segs,
                const GemmArgs& args, int grid, cudaStream_t stream) {
  static PerDeviceOnce once;
  int dev = 0;
  DMOE_CUDA(cudaGetDevice(&dev));
  const int r = once_per_device(once, dev, [] {
    DMOE_CUDA(cudaFuncSetAttribute(grouped_gemm_kernel<GATED, DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmemBytes));
    return DMOE_OK;
  });
  if (r) return r;
  grouped_gemm_kernel<GATED, DT><<<grid, kThreads, kSmemBytes, stream>>>(a, b0, b1, segs, args);
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

template <bool GATED, int DT>
int launch_gemm_2sm(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1, const GemmSegs& segs,
                    const GemmArgs& args, int max_pairs, cudaStream_t stream) {
  static PerDeviceOnce once;
  static int max_clusters[64];
  int dev = 0;
  DMOE_CUDA(cudaGetDevice(&dev));
  DMOE_REQUIRE(dev >= 0 && dev < 64, "grouped MLP: device index %d out of range", dev);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes2;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int r = once_per_device(once, dev, [&] {
    DMOE_CUDA(cudaFuncSetAttribute(grouped_gemm_2sm_kernel<GATED, DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmemBytes2));
    cfg.gridDim = dim3(2 * 74);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, grouped_gemm_2sm_kernel<GATED, DT>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 64;
    }
    max_clusters[dev] = n;
    return DMOE_OK;
  });
  if (r) return r;
  int pairs = max_clusters[dev] - (g_sm_reserve.load(std::memory_order_relaxed) + 1) / 2;
  if (max_pairs >= 0 && max_pairs < pairs) pairs = max_pairs;
  if (pairs < 1) pairs = 1;
  cfg.gridDim = dim3(2 * pairs);
  DMOE_CUDA(cudaLaunchKernelEx(&cfg, grouped_gemm_2sm_kernel<GATED, DT>, a, b0, b1, segs, args));
  DMOE_LAUNCH_CHECK();
  return DMOE_OK;
}

// Kernel variant: DMOE_GEMM_VARIANT=1sm|2sm forces one; otherwise 2-SM tiles are used when the
// segments average at least 128 rows (a 256-row pair tile would otherwise be mostly padding).
// L2 prefetch distance in k-blocks (DMOE_GEMM_PREFETCH; default 0 = off: on B200 the extra TMA
// prefetch requests cost more throughput than the latency they hide for these shapes).
// Tile order of the pair kernels (GemmArgs::raster_n_fast); DMOE_GEMM_RASTER overrides.
int raster_mode(int dflt) {
  const char* v = getenv("DMOE_GEMM_RASTER");
  if (v && (v[0] == '0' || v[0] == '1' || v[0] == '2') && v[1] == 0) return v[0] - '0';
  return dflt;
}

// Tile order of the down-projection GEMM alone (DMOE_GEMM2_RASTER), else raster_mode.
int raster_mode2(int dflt) {
  const char* v = getenv("DMOE_GEMM2_RASTER");
  if (v && (v[0] == '0' || v[0] == '1' || v[0] == '2') && v[1] == 0) return v[0] - '0';
  return raster_mode(dflt);
}

int prefetch_distance() {
  const char* v = getenv("DMOE_GEMM_PREFETCH");
  if (v && *v) return atoi(v);
  return 0;
}

bool use_2sm(int n_seg, int m_rows) {
  const char* v = getenv("DMOE_GEMM_VARIANT");
  if (v && strcmp(v, "1sm") == 0) return false;
  if (v && strcmp(v, "2sm") == 0) return true;
  return n_seg > 0 && m_rows / n_seg >= 128;
}

int sm_count();

int usable_sms() {
  const int n = sm_count() - g_sm_reserve.load(std::memory_order_relaxed);
  return n > 1 ? n : 1;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// Where GEMM2 stores its rows when they are scattered to their hosts (see GemmArgs::scatter).
struct ScatterSpec {
  const int32_t* map;
  char* base[DMOE_EP_MAX_RANKS];
};

void apply_scatter(GemmArgs& a, const ScatterSpec* sc) {
  if (sc == nullptr) return;
  a.scatter = 1;
  a.scatter_map = sc->map;
  for (int g = 0; g < DMOE_EP_MAX_RANKS; ++g) a.scatter_base[g] = sc->base[g];
}

// Quantisation scales of an e4m3 gate/up GEMM (GemmArgs::a_scale) and the A rows' stride.
struct Fp8Scales {
  const float* a;
  int a_ld;       // floats between rows' scales
  const float* gate;
  const float* up;
  uint64_t x_ld;  // bytes between A rows (0: packed)
};

void apply_scales(GemmArgs& a, const Fp8Scales* f) {
  if (f == nullptr) return;
  a.a_scale = f->a;
  a.a_scale_ld = f->a_ld;
  a.b0_scale = f->gate;
  a.b1_scale = f->up;
}

// GEMM1 (gate/up + activation) on DT1 operands, GEMM2 (down) on DT2 operands; h is DT2.
template <int DT1, int DT2>
int run_mlp2(const void* X, const void* w_gate, const void* w_up, const void* w_down, int E_stack, int d, int I,
             GemmSegs& segs, int total_m_host, int m_rows, int act, void* Y, void* H, int32_t* status,
             cudaStream_t stream, int policy, const ScatterSpec* sc = nullptr, const Fp8Scales* f8 = nullptr) {
  static_assert(out_dtype<DT1>() == DT2, "h is written in the down GEMM's operand type");
  constexpr int RE1 = row_elems<DT1>();
  constexpr int RE2 = row_elems<DT2>();
  CUtensorMap ta, tg, tu, th, td;
  {
    const uint64_t dims[2] = {(uint64_t)d, (uint64_t)m_rows};
    const uint32_t box[2] = {RE1, BM};
    int r = make_map(&ta, DT1, X, 2, dims, box, f8 ? f8->x_ld : 0);
    if (r) return r;
  }
  {
    const uint64_t dims[3] = {(uint64_t)d, (uint64_t)I, (uint64_t)E_stack};
    const uint32_t box[3] = {RE1, BN / 2, 1};
    int r = make_map(&tg, DT1, w_gate, 3, dims, box);
    if (r) return r;
    r = make_map(&tu, DT1, w_up, 3, dims, box);
    if (r) return r;
  }
  {
    const uint64_t dims[2] = {(uint64_t)I, (uint64_t)m_rows};
    const uint32_t box[2] = {RE2, BM};
    int r = make_map(&th, DT2, H, 2, dims, box);
    if (r) return r;
  }
  {
    const uint64_t dims[3] = {(uint64_t)I, (uint64_t)d, (uint64_t)E_stack};
    const uint32_t box[3] = {RE2, BN, 1};
    int r = make_map(&td, DT2, w_down, 3, dims, box);
    if (r) return r;
  }
  const int nt1 = (I + BN / 2 - 1) / (BN / 2);
  const int nt2 = (d + BN - 1) / BN;
  bool pair = policy == DMOE_TILES_PAIR || policy == DMOE_TILES_PAIR_SPLIT;
  if (policy == DMOE_TILES_AUTO) pair = use_2sm(segs.n_seg, m_rows);
  const char* hyb = getenv("DMOE_GEMM_HYBRID");
  const bool split = policy == DMOE_TILES_PAIR_SPLIT || (pair && hyb && strcmp(hyb, "1") == 0);
  if (pair && split) {
    // Whole 256-row blocks (and remainders over 128 rows) as pair tiles, remainders of at
    // most 128 rows as one single-SM tile each: a segment of 257-384 rows costs three
    // SM-tile units instead of four.  Both launches read the same segment table.
    CUtensorMap td2;
    const uint64_t dims[3] = {(uint64_t)I, (uint64_t)d, (uint64_t)E_stack};
    const uint32_t box[3] = {RE2, 128, 1};
    int r = make_map(&td2, DT2, w_down, 3, dims, box);
    if (r) return r;
    GemmArgs a1{H, I, I, d, nt1, raster_mode(2), act, prefetch_distance(), status};
    GemmArgs a2{Y, d, d, I, nt2, raster_mode2(2), act, prefetch_distance(), status};
    GemmArgs s1{H, I, I, d, nt1, 0, act, prefetch_distance(), status};
    GemmArgs s2{Y, d, d, I, nt2, 1, act, prefetch_distance(), status};
    apply_scatter(a2, sc);
    apply_scatter(s2, sc);
    apply_scales(a1, f8);
    apply_scales(s1, f8);
    const int sms = usable_sms();
    segs.split = 1;
    r = launch_gemm_2sm<true, DT1>(ta, tg, tu, segs, a1, -1, stream);
    if (r) return r;
    segs.split = 2;
    r = launch_gemm<true, DT1>(ta, tg, tu, segs, s1, sms, stream);
    if (r) return r;
    segs.split = 1;
    r = launch_gemm_2sm<false, DT2>(th, td2, td2, segs, a2, -1, stream);
    if (r) return r;
    segs.split = 2;
    r = launch_gemm<false, DT2>(th, td, td, segs, s2, sms, stream);
    segs.split = 0;
    return r;
  }
  if (pair) {
    CUtensorMap td2;
    const uint64_t dims[3] = {(uint64_t)I, (uint64_t)d, (uint64_t)E_stack};
    const uint32_t box[3] = {RE2, 128, 1};
    int r = make_map(&td2, DT2, w_down, 3, dims, box);
    if (r) return r;
    GemmArgs a1{H, I, I, d, nt1, raster_mode(2), act, prefetch_distance(), status};
    GemmArgs a2{Y, d, d, I, nt2, raster_mode2(2), act, prefetch_distance(), status};
    apply_scatter(a2, sc);
    apply_scales(a1, f8);
    // Pair tiles only.  With the segment-by-segment tile order a remainder's pair tile reads
    // the expert's weights from L2 next to the expert's other tiles, while a separate
    // single-SM launch re-reads them from DRAM after the pair launch (measured on the
    // Mixtral layer, about 1000 rows per expert: 2.22 ms for pair tiles only against 2.26 ms
    // split); the split pays off for ragged experts of a few hundred rows.
    r = launch_gemm_2sm<true, DT1>(ta, tg, tu, segs, a1, -1, stream);
    if (r) return r;
    return launch_gemm_2sm<false, DT2>(th, td2, td2, segs, a2, -1, stream);
  }
  const int sms = usable_sms();
  int g1 = sms, g2 = sms;
  if (total_m_host >= 0) {
    const int64_t t1 = (int64_t)total_m_host * nt1, t2 = (int64_t)total_m_host * nt2;
    if (t1 == 0) return DMOE_OK;
    g1 = (int)(t1 < sms ? t1 : sms);
    g2 = (int)(t2 < sms ? t2 : sms);
  }
  GemmArgs a1{H, I, I, d, nt1, 0, act, prefetch_distance(), status};
  apply_scales(a1, f8);
  int r = launch_gemm<true, DT1>(ta, tg, tu, segs, a1, g1, stream);
  if (r) return r;
  GemmArgs a2{Y, d, d, I, nt2, 1, act, prefetch_distance(), status};
  apply_scatter(a2, sc);
  return launch_gemm<false, DT2>(th, td, td, segs, a2, g2, stream);
}

template <int DT>
int run_mlp(const void* X, const void* w_gate, const void* w_up, const void* w_down, int E_stack, int d, int I,
            GemmSegs& segs, int total_m_host, int m_rows, int act, void* Y, void* H, int32_t* status,
            cudaStream_t stream, int policy, const ScatterSpec* sc = nullptr) {
  return run_mlp2<DT, DT>(X, w_gate, w_up, w_down, E_stack, d, I, segs, total_m_host, m_rows, act, Y, H, status,
                          stream, policy, sc, nullptr);
}

// Router logits on the tensor cores: L[T, E] = X[T, d] · W_r[E, d]^T in fp32 (the plain GEMM
// with one segment and W_r as a one-expert stack; E plays the output width, d the reduction).
template <int DT>
int run_logits(const void* X, const void* W, int T, int d, int E, float* out, int32_t* status, cudaStream_t stream) {
  static thread_local GemmSegs segs;
  segs.n_seg = 1;
  segs.m_rows = T;
  segs.e_stack = 1;
  segs.split = 0;
  segs.dev_expert = nullptr;
  segs.dev_end = nullptr;
  segs.expert[0] = 0;
  segs.end[0] = T;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)d, (uint64_t)T};
    const uint32_t box[2] = {BK, BM};
    int r = make_map(&ta, DT, X, 2, dims, box);
    if (r) return r;
  }
  const int nt = (E + BN - 1) / BN;
  GemmArgs a{out, E, E, d, nt, raster_mode(2), DMOE_ACT_RELU, 0, status, 1};
  if (use_2sm(1, T)) {
    const uint64_t dims[3] = {(uint64_t)d, (uint64_t)E, 1};
    const uint32_t box[3] = {BK, 128, 1};
    int r = make_map(&tb, DT, W, 3, dims, box);
    if (r) return r;
    return launch_gemm_2sm<false, DT>(ta, tb, tb, segs, a, ((T + BM2 - 1) / BM2) * nt, stream);
  }
  const uint64_t dims[3] = {(uint64_t)d, (uint64_t)E, 1};
  const uint32_t box[3] = {BK, BN, 1};
  int r = make_map(&tb, DT, W, 3, dims, box);
  if (r) return r;
  const int64_t tiles = (int64_t)((T + BM - 1) / BM) * nt;
  const int sms = usable_sms();
  return launch_gemm<false, DT>(ta, tb, tb, segs, a, (int)(tiles < sms ? tiles : sms), stream);
}

}  // namespace
}  // namespace dmoe

using namespace dmoe;

namespace dmoe {
int gemm_sm_reserve() { return g_sm_reserve.load(std::memory_order_relaxed); }

// Segment tables of a grouped MLP call: device tables are read by the kernels, host tables
// are checked and copied into the launch parameters.  total_m: M tiles of a host table, -1
// for a device table.
int fill_segs(GemmSegs& segs, const int32_t* seg_expert, const int32_t* seg_end, int n_seg, int seg_on_device,
              int m_rows, int E_stack, int* total_m) {
  segs.n_seg = n_seg;
  segs.m_rows = m_rows;
  segs.e_stack = E_stack;
  segs.split = 0;
  *total_m = -1;
  if (seg_on_device) {
    DMOE_REQUIRE(n_seg <= kMaxSegDev, "dmoe_grouped_gated_mlp: n_seg=%d > %d", n_seg, kMaxSegDev);
    segs.dev_expert = seg_expert;
    segs.dev_end = seg_end;
    return DMOE_OK;
  }
  DMOE_REQUIRE(n_seg <= 256, "dmoe_grouped_gated_mlp: n_seg=%d > 256 for host segment tables", n_seg);
  segs.dev_expert = nullptr;
  segs.dev_end = nullptr;
  int prev = 0, tiles = 0;
  for (int i = 0; i < n_seg; ++i) {
    DMOE_REQUIRE(seg_end[i] >= prev && seg_end[i] <= m_rows, "dmoe_grouped_gated_mlp: segment %d end %d invalid", i,
                 seg_end[i]);
    DMOE_REQUIRE(seg_expert[i] >= 0 && seg_expert[i] < E_stack, "dmoe_grouped_gated_mlp: segment %d expert %d", i,
                 seg_expert[i]);
    segs.expert[i] = seg_expert[i];
    segs.end[i] = seg_end[i];
    tiles += (seg_end[i] - prev + BM - 1) / BM;
    prev = seg_end[i];
  }
  *total_m = tiles;
  return DMOE_OK;
}

}  // namespace dmoe

extern "C" int dmoe_grouped_mlp_set_sm_reserve(int sms) {
  clear_error();
  DMOE_REQUIRE(sms >= 0 && sms <= 64, "dmoe_grouped_mlp_set_sm_reserve: %d SMs (0..64)", sms);
  g_sm_reserve.store(sms, std::memory_order_relaxed);
  return DMOE_OK;
}

extern "C" int dmoe_router_logits(const void* x, const void* w_r, int dtype, int T, int d, int E, float* logits_out,
                                  int32_t* dev_status, void* stream) {
  clear_error();
  DMOE_REQUIRE(dtype == DMOE_BF16 || dtype == DMOE_F16, "dmoe_router_logits: dtype must be f16 or bf16");
  DMOE_REQUIRE(T >= 0 && d > 0 && E > 0 && d % 8 == 0 && E % 8 == 0,
               "dmoe_router_logits: d=%d and E=%d must be multiples of 8", d, E);
  if (T == 0) return DMOE_OK;
  DMOE_REQUIRE(x && w_r && logits_out && dev_status, "dmoe_router_logits: null pointer");
  DMOE_REQUIRE(aligned16(x) && aligned16(w_r) && aligned16(logits_out), "dmoe_router_logits: 16-byte alignment");
  cudaStream_t s = as_stream(stream);
  if (logits_few_tokens_eligible(T, d, E)) return run_logits_few_tokens(x, w_r, dtype, T, d, E, logits_out, s);
  if (dtype == DMOE_BF16) return run_logits<DMOE_BF16>(x, w_r, T, d, E, logits_out, dev_status, s);
  return run_logits<DMOE_F16>(x, w_r, T, d, E, logits_out, dev_status, s);
}

extern "C" size_t dmoe_grouped_mlp_workspace_size(int m_rows, int I, int dtype) {
  return (size_t)m_rows * (size_t)I * (dtype == DMOE_F32 ? 4 : 2) + 256;
}

extern "C" int dmoe_grouped_gated_mlp_ex(const void* X, const void* w_gate, const void* w_up, const void* w_down,
                                         int E_stack, int d, int I, int dtype, const int32_t* seg_expert,
                                         const int32_t* seg_end, int n_seg, int seg_on_device, int m_rows, int act,
                                         void* Y, void* workspace, size_t workspace_bytes, int32_t* dev_status,
                                         int tile_policy, void* stream) {
  clear_error();
  DMOE_REQUIRE(tile_policy >= DMOE_TILES_AUTO && tile_policy <= DMOE_TILES_PAIR_SPLIT,
               "dmoe_grouped_gated_mlp: bad tile policy %d", tile_policy);
  DMOE_REQUIRE(dtype == DMOE_BF16 || dtype == DMOE_F16 || dtype == DMOE_F32,
               "dmoe_grouped_gated_mlp: dtype must be f16, bf16 or f32");
  DMOE_REQUIRE(act == DMOE_ACT_RELU || act == DMOE_ACT_SILU, "dmoe_grouped_gated_mlp: bad activation %d", act);
  DMOE_REQUIRE(d > 0 && I > 0 && d % 8 == 0 && I % 8 == 0, "dmoe_grouped_gated_mlp: d=%d, I=%d must be multiples of 8",
               d, I);
  DMOE_REQUIRE(E_stack >= 1 && m_rows >= 0, "dmoe_grouped_gated_mlp: bad E_stack/m_rows");
  DMOE_REQUIRE(n_seg >= 0, "dmoe_grouped_gated_mlp: bad n_seg");
  if (n_seg == 0 || m_rows == 0) return DMOE_OK;
  DMOE_REQUIRE(X && w_gate && w_up && w_down && Y && workspace && dev_status && seg_expert && seg_end,
               "dmoe_grouped_gated_mlp: null pointer");
  DMOE_REQUIRE(aligned16(X) && aligned16(w_gate) && aligned16(w_up) && aligned16(w_down) && aligned16(Y) &&
                   aligned16(workspace),
               "dmoe_grouped_gated_mlp: tensors must be 16-byte aligned");
  DMOE_REQUIRE(workspace_bytes >= dmoe_grouped_mlp_workspace_size(m_rows, I, dtype),
               "dmoe_grouped_gated_mlp: workspace %zu < %zu bytes", workspace_bytes,
               dmoe_grouped_mlp_workspace_size(m_rows, I, dtype));
  static thread_local GemmSegs segs;
  int total_m = -1;
  if (int r = fill_segs(segs, seg_expert, seg_end, n_seg, seg_on_device, m_rows, E_stack, &total_m)) return r;
  void* H = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  cudaStream_t s = as_stream(stream);
  if (dtype == DMOE_BF16)
    return run_mlp<DMOE_BF16>(X, w_gate, w_up, w_down, E_stack, d, I, segs, total_m, m_rows, act, Y, H, dev_status, s,
                              tile_policy);
  if (dtype == DMOE_F32)
    return run_mlp<DMOE_F32>(X, w_gate, w_up, w_down, E_stack, d, I, segs, total_m, m_rows, act, Y, H, dev_status, s,
                             tile_policy);
  return run_mlp<DMOE_F16>(X, w_gate, w_up, w_down, E_stack, d, I, segs, total_m, m_rows, act, Y, H, dev_status, s,
                           tile_policy);
}

extern "C" int dmoe_grouped_gated_mlp(const void* X, const void* w_gate, const void* w_up, const void* w_down,
                                      int E_stack, int d, int I, int dtype, const int32_t* seg_expert,
                                      const int32_t* seg_end, int n_seg, int seg_on_device, int m_rows, int act,
                                      void* Y, void* workspace, size_t workspace_bytes, int32_t* dev_status,
                                      void* stream) {
  return dmoe_grouped_gated_mlp_ex(X, w_gate, w_up, w_down, E_stack, d, I, dtype, seg_expert, seg_end, n_seg,
                                   seg_on_device, m_rows, act, Y, workspace, workspace_bytes, dev_status,
                                   DMOE_TILES_AUTO, stream);
}

extern "C" int dmoe_grouped_gated_mlp_fp8(const void* Xq, const float* x_scale, const void* wg_q,
                                          const float* wg_scale, const void* wu_q, const float* wu_scale,
                                          const void* w_down, int E_stack, int d, int I, const int32_t* seg_expert,
                                          const int32_t* seg_end, int n_seg, int seg_on_device, int m_rows, int act,
                                          void* Y, void* workspace, size_t workspace_bytes, int32_t* dev_status,
                                          int tile_policy, void* stream) {
  clear_error();
  DMOE_REQUIRE(tile_policy >= DMOE_TILES_AUTO && tile_policy <= DMOE_TILES_PAIR_SPLIT,
               "dmoe_grouped_gated_mlp_fp8: bad tile policy %d", tile_policy);
  DMOE_REQUIRE(act == DMOE_ACT_RELU || act == DMOE_ACT_SILU, "dmoe_grouped_gated_mlp_fp8: bad activation %d", act);
  DMOE_REQUIRE(d > 0 && I > 0 && d % 16 == 0 && I % 8 == 0,
               "dmoe_grouped_gated_mlp_fp8: d=%d must be a multiple of 16, I=%d of 8", d, I);
  DMOE_REQUIRE(E_stack >= 1 && m_rows >= 0 && n_seg >= 0, "dmoe_grouped_gated_mlp_fp8: bad E_stack/m_rows/n_seg");
  if (n_seg == 0 || m_rows == 0) return DMOE_OK;
  DMOE_REQUIRE(Xq && x_scale && wg_q && wg_scale && wu_q && wu_scale && w_down && Y && workspace && dev_status &&
                   seg_expert && seg_end,
               "dmoe_grouped_gated_mlp_fp8: null pointer");
  DMOE_REQUIRE(aligned16(Xq) && aligned16(wg_q) && aligned16(wu_q) && aligned16(w_down) && aligned16(Y) &&
                   aligned16(workspace),
               "dmoe_grouped_gated_mlp_fp8: tensors must be 16-byte aligned");
  DMOE_REQUIRE(workspace_bytes >= dmoe_grouped_mlp_workspace_size(m_rows, I, DMOE_BF16),
               "dmoe_grouped_gated_mlp_fp8: workspace %zu < %zu bytes", workspace_bytes,
               dmoe_grouped_mlp_workspace_size(m_rows, I, DMOE_BF16));
  static thread_local GemmSegs segs;
  int total_m = -1;
  if (int r = fill_segs(segs, seg_expert, seg_end, n_seg, seg_on_device, m_rows, E_stack, &total_m)) return r;
  void* H = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  const Fp8Scales f8{x_scale, 1, wg_scale, wu_scale, 0};
  return run_mlp2<DMOE_E4M3, DMOE_BF16>(Xq, wg_q, wu_q, w_down, E_stack, d, I, segs, total_m, m_rows, act, Y, H,
                                        dev_status, as_stream(stream), tile_policy, nullptr, &f8);
}

namespace dmoe {
namespace {
// Checks shared by the 16-bit and the 8-bit exchange expert steps; fills the segment table
// and the scatter targets (each host's return rows).
int ep_mlp_setup(const char* name, const dmoe_ep_window* win, const void* w_gate, const void* w_up,
                 const void* w_down, int E_stack, int d, int I, int h_dtype, const int32_t* seg_expert,
                 const int32_t* seg_end, int n_seg, int64_t cap, int act, const void* workspace,
                 size_t workspace_bytes, int32_t* dev_status, int tile_policy, GemmSegs& segs, ScatterSpec& sc) {
  DMOE_REQUIRE(win != nullptr && win->world >= 1 && win->world <= DMOE_EP_MAX_RANKS && win->rank >= 0 &&
                   win->rank < win->world,
               "%s: bad window table", name);
  DMOE_REQUIRE(act == DMOE_ACT_RELU || act == DMOE_ACT_SILU, "%s: bad activation %d", name, act);
  DMOE_REQUIRE(d > 0 && I > 0 && d % 8 == 0 && I % 8 == 0, "%s: d=%d, I=%d must be multiples of 8", name, d, I);
  DMOE_REQUIRE(E_stack >= 1 && n_seg >= 0 && n_seg <= kMaxSegDev, "%s: bad E_stack/n_seg", name);
  DMOE_REQUIRE(cap >= 0 && cap < (1ll << 31), "%s: bad capacity", name);
  DMOE_REQUIRE(tile_policy >= DMOE_TILES_AUTO && tile_policy <= DMOE_TILES_PAIR_SPLIT, "%s: bad tile policy %d", name,
               tile_policy);
  if (n_seg == 0 || cap == 0) return DMOE_OK;
  const void* X = win->recv[win->rank];
  DMOE_REQUIRE(X && win->back[win->rank] && w_gate && w_up && w_down && workspace && dev_status && seg_expert &&
                   seg_end,
               "%s: null pointer", name);
  for (int g = 0; g < win->world; ++g)
    DMOE_REQUIRE(win->rows[g] != nullptr && aligned16(win->rows[g]), "%s: rank %d has no return rows", name, g);
  DMOE_REQUIRE(aligned16(X) && aligned16(w_gate) && aligned16(w_up) && aligned16(w_down) && aligned16(workspace),
               "%s: tensors must be 16-byte aligned", name);
  DMOE_REQUIRE(workspace_bytes >= dmoe_grouped_mlp_workspace_size((int)cap, I, h_dtype), "%s: workspace %zu < %zu bytes",
               name, workspace_bytes, dmoe_grouped_mlp_workspace_size((int)cap, I, h_dtype));
  segs.n_seg = n_seg;
  segs.m_rows = (int)cap;
  segs.e_stack = E_stack;
  segs.split = 0;
  segs.dev_expert = seg_expert;
  segs.dev_end = seg_end;
  sc.map = reinterpret_cast<const int32_t*>(win->back[win->rank]);
  for (int g = 0; g < DMOE_EP_MAX_RANKS; ++g) sc.base[g] = g < win->world ? reinterpret_cast<char*>(win->rows[g]) : nullptr;
  return DMOE_OK;
}
}  // namespace
}  // namespace dmoe

extern "C" int dmoe_ep_expert_mlp(const dmoe_ep_window* win, const void* w_gate, const void* w_up, const void* w_down,
                                  int E_stack, int d, int I, int dtype, const int32_t* seg_expert,
                                  const int32_t* seg_end, int n_seg, int64_t cap, int act, void* workspace,
                                  size_t workspace_bytes, int32_t* dev_status, int tile_policy, void* stream) {
  clear_error();
  DMOE_REQUIRE(dtype == DMOE_BF16 || dtype == DMOE_F16 || dtype == DMOE_F32,
               "dmoe_ep_expert_mlp: dtype must be f16, bf16 or f32");
  static thread_local GemmSegs segs;
  ScatterSpec sc{};
  if (int r = ep_mlp_setup("dmoe_ep_expert_mlp", win, w_gate, w_up, w_down, E_stack, d, I, dtype, seg_expert, seg_end,
                           n_seg, cap, act, workspace, workspace_bytes, dev_status, tile_policy, segs, sc))
    return r;
  if (n_seg == 0 || cap == 0) return DMOE_OK;
  const void* X = win->recv[win->rank];
  void* H = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  cudaStream_t s = as_stream(stream);
  if (dtype == DMOE_BF16)
    return run_mlp<DMOE_BF16>(X, w_gate, w_up, w_down, E_stack, d, I, segs, -1, (int)cap, act, nullptr, H, dev_status,
                              s, tile_policy, &sc);
  if (dtype == DMOE_F32)
    return run_mlp<DMOE_F32>(X, w_gate, w_up, w_down, E_stack, d, I, segs, -1, (int)cap, act, nullptr, H, dev_status,
                             s, tile_policy, &sc);
  return run_mlp<DMOE_F16>(X, w_gate, w_up, w_down, E_stack, d, I, segs, -1, (int)cap, act, nullptr, H, dev_status, s,
                           tile_policy, &sc);
}

extern "C" int dmoe_ep_expert_mlp_fp8(const dmoe_ep_window* win, const void* wg_q, const float* wg_scale,
                                      const void* wu_q, const float* wu_scale, const void* w_down, int E_stack, int d,
                                      int I, const int32_t* seg_expert, const int32_t* seg_end, int n_seg, int64_t cap,
                                      int act, void* workspace, size_t workspace_bytes, int32_t* dev_status,
                                      int tile_policy, void* stream) {
  clear_error();
  DMOE_REQUIRE(d % 16 == 0, "dmoe_ep_expert_mlp_fp8: d=%d must be a multiple of 16", d);
  static thread_local GemmSegs segs;
  ScatterSpec sc{};
  if (int r = ep_mlp_setup("dmoe_ep_expert_mlp_fp8", win, wg_q, wu_q, w_down, E_stack, d, I, DMOE_BF16, seg_expert,
                           seg_end, n_seg, cap, act, workspace, workspace_bytes, dev_status, tile_policy, segs, sc))
    return r;
  if (n_seg == 0 || cap == 0) return DMOE_OK;
  DMOE_REQUIRE(wg_scale && wu_scale, "dmoe_ep_expert_mlp_fp8: null scale pointer");
  // Receive records: d e4m3 codes, the row's fp32 scale, padding to d + 16 bytes.
  const char* X = reinterpret_cast<const char*>(win->recv[win->rank]);
  const Fp8Scales f8{reinterpret_cast<const float*>(X + d), (d + 16) / 4, wg_scale, wu_scale, (uint64_t)d + 16};
  void* H = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  return run_mlp2<DMOE_E4M3, DMOE_BF16>(X, wg_q, wu_q, w_down, E_stack, d, I, segs, -1, (int)cap, act, nullptr, H,
                                        dev_status, as_stream(stream), tile_policy, &sc, &f8);
}
