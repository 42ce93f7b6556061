/*
 * dmoe_b200.h -- C ABI of the B200 (sm_100a) MoE-layer hot path.
 *
 * The library (libdmoe_b200.so) replaces the torch-op sequences of the reference
 * (slivanovich/DistributedMoE, paths relative to src/python/) on the path
 *   DistMoEBlock routing -> dispatch into BuffersPool input buffers -> grouped expert
 *   gated MLP -> weighted combine.
 *
 * Conventions
 *  - Plain pointers and sizes; device pointers unless a parameter says "host".
 *  - Every call is stream-ordered on `stream` (a cudaStream_t passed as void*; NULL is the
 *    legacy default stream) and returns 0 on success or a DMOE_ERR_* code.  The message of
 *    the last failure on the calling thread is returned by dmoe_last_error().
 *  - The library never allocates or frees caller memory.  Scratch is passed in as
 *    `workspace` with a size query function.
 *  - Kernels that wait (mbarriers inside the grouped GEMM, dmoe_flag_wait) bound every
 *    wait by time; on expiry they OR a DMOE_DEVERR_* bit into the caller's device word
 *    `dev_status` (int32) and return, never trap.
 *  - dtype codes: DMOE_F32, DMOE_F16, DMOE_BF16.
 */
#ifndef DMOE_B200_H
#define DMOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DMOE_OK 0
#define DMOE_ERR_INVALID 1     /* bad argument, shape or alignment */
#define DMOE_ERR_CUDA 2        /* a CUDA runtime/driver call failed */
#define DMOE_ERR_UNSUPPORTED 3 /* valid request this build does not implement */
#define DMOE_NOT_READY 4       /* dmoe_event_query: work before the event is still pending */

#define DMOE_F32 0
#define DMOE_F16 1
#define DMOE_BF16 2
#define DMOE_E4M3 3 /* 8-bit float (1-4-3): only where an entry point says so, always with fp32 scales */

#define DMOE_ACT_RELU 0 /* reference: relu(gate) * up  (MoE/PipelineTask.py:518, MoE/MoE.py:25) */
#define DMOE_ACT_SILU 1 /* SwiGLU: silu(gate) * up */

#define DMOE_ROUTER_SOFTMAX 0       /* softmax(fp32) -> top-k (MoE/DistMoEBlock.py:557-562) */
#define DMOE_ROUTER_SIGMOID_GROUP 1 /* sigmoid + selection bias + group-limited top-k */

/* device status bits (OR-ed into *dev_status) */
#define DMOE_DEVERR_TIMEOUT_PRODUCER 0x1
#define DMOE_DEVERR_TIMEOUT_MMA 0x2
#define DMOE_DEVERR_TIMEOUT_EPILOGUE 0x4
#define DMOE_DEVERR_TIMEOUT_TEARDOWN 0x8
#define DMOE_DEVERR_FLAG_TIMEOUT 0x10
#define DMOE_DEVERR_BAD_SEGMENT 0x20
#define DMOE_DEVERR_EP_TIMEOUT 0x40  /* an expert-parallel flag wait gave up (a rank fell behind) */
#define DMOE_DEVERR_EP_OVERFLOW 0x80 /* rows beyond a receive buffer's capacity were dropped */

/* Library identity: returns a static version string. */
const char* dmoe_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* dmoe_last_error(void);

/*
 * Router: logits, top-k selection and routing weights, one warp per token.
 * Replaces DistMoEBlock._setup_forward_pass routing, MoE/DistMoEBlock.py:556-562
 * (gate = nn.Linear(d, E, bias=False), :134; softmax in fp32, torch.topk, cast to dtype).
 *
 *  x            [T, d] activations (x_dtype); ignored when logits_in != NULL
 *  w_r          [E, d] router weight (same dtype as x)
 *  logit_bias   [E] fp32 added to the logits, or NULL (the bias=True gate replacement, :133)
 *  score_bias   [E] fp32 selection bias for DMOE_ROUTER_SIGMOID_GROUP, or NULL
 *  logits_in    [T, E] fp32 logits to route from instead of computing them, or NULL
 *  logits_out   [T, E] fp32 logits written when not NULL (and logits_in == NULL)
 *  idx_out      [T, k] int64 selected experts, best first (torch.topk order)
 *  w_out        [T, k] routing weights in w_dtype
 *  renormalize  divide the k weights by their sum (extension; the reference does not)
 *  scale        multiply the weights (1.0 in the reference)
 *  n_group/topk_group  group-limited selection (DMOE_ROUTER_SIGMOID_GROUP)
 *  Limits: E <= 256, k <= min(E, 16), d % 8 == 0.
 */
int dmoe_router(const void* x, const void* w_r, int x_dtype, const float* logit_bias, const float* score_bias,
                const float* logits_in, int T, int d, int E, int k, int mode, int renormalize, float scale,
                int n_group, int topk_group, float* logits_out, int64_t* idx_out, void* w_out, int w_dtype,
                void* stream);

/*
 * Router logits on the tensor cores: logits_out[T, E] = x[T, d] · w_r[E, d]^T in fp32
 * (fp32 accumulation of the bf16/f16 products; no bias).  Replaces the gate Linear of
 * MoE/DistMoEBlock.py:134,556 for large expert counts, where a dot product per (token,
 * expert) on the CUDA cores is the slow part of routing; feed the result to dmoe_router as
 * logits_in.  d % 8 == 0, E % 8 == 0.  Bounded waits report through *dev_status like the
 * grouped MLP.  For T <= 256 (decode) the logits are computed on the CUDA cores instead,
 * eight experts per CTA, so that the reduction is spread over E / 8 CTAs.
 */
int dmoe_router_logits(const void* x, const void* w_r, int dtype, int T, int d, int E, float* logits_out,
                       int32_t* dev_status, void* stream);

/*
 * Routing plan: per-expert counts, offsets and the permutation of the T*k activations.
 * Replaces the one-hot mask + per-expert torch.where loop of MoE/DistMoEBlock.py:568-605:
 * within an expert, activations are ordered slot-major then by ascending token, exactly as
 * torch.where(expert_mask[e]) orders them.  Experts are concatenated in index order.
 *
 *  idx          [T, k] int64 expert of each (token, slot)
 *  w            [T, k] routing weights (w_dtype) or NULL
 *  counts       [E] int32, offsets [E+1] int32 (exclusive prefix of counts)
 *  perm_token   [T*k] int32 token of each permuted activation
 *  perm_slot    [T*k] int32 slot of each permuted activation (may be NULL)
 *  inverse      [T*k] int32 permuted position of (token t, slot s) at t*k+s (may be NULL);
 *               -1 for an activation whose expert index is outside [0, E)
 *  perm_weight  [T*k] weight of each permuted activation in w_dtype (NULL if w is NULL)
 *  workspace    dmoe_route_plan_workspace_size(T, k, E) bytes of device scratch
 *  Limits: 1 <= E <= 1024, T*k < 2^31.
 */
size_t dmoe_route_plan_workspace_size(int T, int k, int E);
int dmoe_route_plan(const int64_t* idx, const void* w, int w_dtype, int T, int k, int E, int32_t* counts,
                    int32_t* offsets, int32_t* perm_token, int32_t* perm_slot, int32_t* inverse,
                    void* perm_weight, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Routing plan without caller scratch.  No counterpart in the reference: it exists for
 * callers that cannot allocate device memory around a call -- an FFI host that is handed
 * only its input and output buffers, or a serving loop whose device memory is owned by
 * another allocator and where cudaMalloc/cudaFree (which can synchronise the device) are
 * not allowed.  Same arguments and results as dmoe_route_plan, minus the workspace; it
 * calls no allocator.
 *  Scratch: a 512 KiB library-owned static device array, held by every GPU that loads the
 *  library until the process exits.  Limit: dmoe_route_plan_workspace_size(T, k, E) must be
 *  <= 512 KiB, i.e. ceil(T*k / 2048) * E <= 131072 (T*k <= 1048576 with E <= 256,
 *  T*k <= 262144 with E <= 1024); larger requests fail with DMOE_ERR_INVALID and a message.
 *  The first call on a device looks up the array's device address (cudaGetSymbolAddress)
 *  with that device current; make that first call before any stream capture.
 *  All calls share the one array: calls whose executions overlap on the GPU (different
 *  streams, or different host threads) race and corrupt each other's plans.  Serialise
 *  them on one stream.
 */
int dmoe_route_plan_noalloc(const int64_t* idx, const void* w, int w_dtype, int T, int k, int E, int32_t* counts,
                            int32_t* offsets, int32_t* perm_token, int32_t* perm_slot, int32_t* inverse,
                            void* perm_weight, void* stream);

/*
 * Segmented row gather/copy: for segment i and r < seg_len[i]
 *     dst[seg_dst[i] + r] = src[ row_map ? row_map[seg_src[i] + r] : seg_src[i] + r ]
 * with rows of row_bytes bytes (multiple of 16, 16-byte aligned bases).
 * With row_map = perm_token this is the gather of HostPipelineTask.dispatch
 * (MoE/PipelineTask.py:231-249) into an input buffer; dst may be a peer GPU's buffer
 * (CUDA IPC / peer pointer).  Without row_map it moves contiguous runs (buffer staging).
 *  seg_src, seg_dst, seg_len: host arrays of n_seg int32 (n_seg <= 1024).
 */
int dmoe_permute_rows(const void* src, void* dst, int64_t row_bytes, const int32_t* row_map,
                      const int32_t* seg_src, const int32_t* seg_dst, const int32_t* seg_len, int n_seg,
                      void* stream);

/*
 * Grouped expert gated MLP over per-expert row segments of one buffer.
 * Replaces the grouped path of ExpertsBlockPipelineTask.run, MoE/PipelineTask.py:478-520:
 *   offs = cumulative (padded) segment ends; gate_out = grouped_mm(X, Wg^T); up_out = ...;
 *   h = act(gate_out) * up_out; Y = grouped_mm(h, Wd^T); copy into the output buffer.
 * Weights are the stacks of DistExpertsBlock.initialize_expert_layers
 * (MoE/DistExpertsBlock.py:163-177) in nn.Linear layout:
 *   w_gate, w_up [E_stack, I, d]; w_down [E_stack, d, I]   (dtype DMOE_F16, DMOE_BF16, or DMOE_F32:
 *   fp32 operands run as tf32 MMAs (10-bit mantissa operands, fp32 accumulation) with h in fp32,
 *   the reference's fp32 precision)
 * Segment i covers rows [seg_end[i-1], seg_end[i]) (seg_end[-1] = 0) and uses stack entry
 * seg_expert[i]; rows outside every segment are not written.  seg_* are host arrays when
 * seg_on_device == 0 (n_seg <= 256), device arrays otherwise (n_seg <= 1024).
 *  X [m_rows, d], Y [m_rows, d]; workspace >= dmoe_grouped_mlp_workspace_size(m_rows, I, dtype)
 *  Computes on tcgen05 tensor cores (fp32 accumulate in TMEM); h is rounded to dtype.
 *  Limits: d % 8 == 0, I % 8 == 0 (K and N tails are zero-filled by TMA and masked).
 */
size_t dmoe_grouped_mlp_workspace_size(int m_rows, int I, int dtype);
int dmoe_grouped_gated_mlp(const void* X, const void* w_gate, const void* w_up, const void* w_down, int E_stack,
                           int d, int I, int dtype, const int32_t* seg_expert, const int32_t* seg_end, int n_seg,
                           int seg_on_device, int m_rows, int act, void* Y, void* workspace, size_t workspace_bytes,
                           int32_t* dev_status, void* stream);

/*
 * dmoe_grouped_gated_mlp with a tile policy (no reference counterpart: how the segments are
 * cut into tensor-core tiles).  DMOE_TILES_AUTO (what dmoe_grouped_gated_mlp uses) takes
 * 256-row two-SM pair tiles when the segments average at least 128 rows of m_rows, else
 * 128-row single-SM tiles; DMOE_TILES_PAIR / DMOE_TILES_SINGLE force one; and
 * DMOE_TILES_PAIR_SPLIT runs every segment's whole 256-row blocks (and remainders over 128
 * rows) as pair tiles and remainders of at most 128 rows as single-SM tiles (two launches
 * per GEMM), for ragged experts of a few hundred rows.  With a device segment table the
 * host cannot see the segment sizes, so a caller that knows the expected rows per expert
 * picks the policy.
 */
#define DMOE_TILES_AUTO 0
#define DMOE_TILES_PAIR 1
#define DMOE_TILES_SINGLE 2
#define DMOE_TILES_PAIR_SPLIT 3
int dmoe_grouped_gated_mlp_ex(const void* X, const void* w_gate, const void* w_up, const void* w_down, int E_stack,
                              int d, int I, int dtype, const int32_t* seg_expert, const int32_t* seg_end, int n_seg,
                              int seg_on_device, int m_rows, int act, void* Y, void* workspace,
                              size_t workspace_bytes, int32_t* dev_status, int tile_policy, void* stream);

/* 8-bit experts.  The reference's benchmark runs the layer on 8-bit float tensors (precision
 * "fp8", src/python/MoE/benchmarks/bench.py:184-185); here the gate/up GEMM takes e4m3
 * operands with fp32 row scales and the down GEMM stays bf16.
 *
 * dmoe_quantize_rows_e4m3: x [rows, cols] (f32/f16/bf16) -> q [rows, cols] e4m3 (rows q_ld
 *   bytes apart) and scale (rows scale_ld floats apart), s = amax(|row|) / 448 (1 for an
 *   all-zero row), q = e4m3_rn_satfinite(x / s).  cols % 16 == 0, q_ld >= cols and % 16 == 0;
 *   x and q 16-byte aligned.  Activations give per-token scales; an expert weight [E, I, d]
 *   viewed as [E * I, d] gives per-output-channel scales.
 *
 * dmoe_grouped_gated_mlp_fp8: as dmoe_grouped_gated_mlp_ex with
 *   Xq [m_rows, d] e4m3, x_scale [m_rows];  wg_q, wu_q [E_stack, I, d] e4m3, wg_scale,
 *   wu_scale [E_stack, I];  w_down [E_stack, d, I] bf16;  Y [m_rows, d] bf16.
 *   gate = (Xq . wg_q^T) * x_scale[row] * wg_scale[e, col] (likewise up), accumulated in fp32
 *   by tcgen05 kind::f8f6f4 MMAs; h = act(gate) * up rounded to bf16.  d % 16 == 0, I % 8 == 0;
 *   workspace >= dmoe_grouped_mlp_workspace_size(m_rows, I, DMOE_BF16).
 */
int dmoe_quantize_rows_e4m3(const void* x, int dtype, int64_t rows, int cols, void* q, int64_t q_ld, float* scale,
                            int64_t scale_ld, void* stream);
int dmoe_grouped_gated_mlp_fp8(const void* Xq, const float* x_scale, const void* wg_q, const float* wg_scale,
                               const void* wu_q, const float* wu_scale, const void* w_down, int E_stack, int d, int I,
                               const int32_t* seg_expert, const int32_t* seg_end, int n_seg, int seg_on_device,
                               int m_rows, int act, void* Y, void* workspace, size_t workspace_bytes,
                               int32_t* dev_status, int tile_policy, void* stream);

/*
 * Number of SMs (0..64, process-wide, default 0) that later dmoe_grouped_gated_mlp launches
 * leave free.  No counterpart in the reference.  The grouped MLP is a persistent kernel that
 * holds each SM it gets until its last tile; where one GPU also serves other streams' short
 * kernels (an expert-parallel GPU gathers and combines for its own host while it computes
 * other hosts' experts), a reserve lets those kernels start at once.
 */
int dmoe_grouped_mlp_set_sm_reserve(int sms);

/*
 * Weighted combine (gather form): for each token t
 *     out[t] = sum_s w[t, s] * rows[inverse[t*k + s]]       (fp32 accumulation, one store)
 * `rows` [T*k, d] holds the expert outputs in permuted order; an activation whose inverse
 * entry is negative adds nothing.  Replaces the per-expert
 * weighted scatter_add_ of HostPipelineTask.combine (MoE/PipelineTask.py:326-346), which
 * accumulates in the model dtype; results agree up to summation order and rounding.
 *  If accumulate != 0, out[t] (dtype) is added to the sum (shared-expert / residual input).
 */
int dmoe_combine(const void* rows, const int32_t* inverse, const void* w, int w_dtype, int T, int k, int d,
                 int dtype, int accumulate, void* out, void* stream);

/*
 * CUDA IPC for the NVLink TensorTransferEngine backend (replaces NIXL/MoonCake memory
 * registration: TensorTransferEngine.register_batch / deserialize_descs / deregister_batch,
 * TensorTransferEngine/TensorTransferEngine.py:146-192).
 *  handle: 64 opaque bytes (cudaIpcMemHandle_t) of the allocation that contains dev_ptr;
 *  *offset_out: byte offset of dev_ptr inside that allocation (caching allocators
 *  sub-allocate).  The importer adds the offset to the pointer dmoe_ipc_open returns.
 */
int dmoe_ipc_export(const void* dev_ptr, uint8_t* handle_out64, uint64_t* offset_out);
int dmoe_ipc_open(const uint8_t* handle64, int device, void** dev_ptr_out);
int dmoe_ipc_close(void* dev_ptr);
int dmoe_enable_peer_access(int device, int peer_device);

/*
 * Byte copy between any two device (or peer-mapped) buffers, stream-ordered.  Replaces the
 * NIXL READ/WRITE of Buffer.read_from / write_to (MoE/pools/BuffersPool.py:55-90).
 */
int dmoe_copy(void* dst, const void* src, size_t bytes, void* stream);

/*
 * Raw CUDA events for stream-ordered completion (replace the transfer handles that the
 * completion monitor polls, TensorTransferEngine/TensorTransferEngine.py:305-344, and the
 * NIXL/MoonCake transfer-state queries, NIXLTensorTransferEngine.py:251-262).  Events have
 * timing disabled; interprocess != 0 makes them exportable.  dmoe_event_query returns
 * DMOE_OK when the work before the last record is done and DMOE_NOT_READY otherwise.
 * dmoe_ipc_event_open opens another process's event in the context of `device`, which must
 * be the GPU the exporter records it on; only streams of that GPU wait on the result.
 */
int dmoe_event_create(int device, int interprocess, void** event_out);
int dmoe_event_destroy(void* event);
int dmoe_event_record(void* event, void* stream);
int dmoe_event_query(void* event);
int dmoe_stream_wait_event(void* stream, void* event);
int dmoe_ipc_event_export(void* event, uint8_t* handle_out64);
int dmoe_ipc_event_open(const uint8_t* handle64, int device, void** event_out);

/*
 * Completion flags (replace the transfer-monitor poll, TensorTransferEngine.py:305-344).
 * dmoe_flag_signal stores `value` to *flag with release semantics (system scope) after the
 * preceding work of `stream`.  dmoe_flag_wait makes `stream` wait until *flag >= value, at
 * most timeout_ns; on expiry it ORs DMOE_DEVERR_FLAG_TIMEOUT into *dev_status and lets the
 * stream continue.  A waiter and its signaller must run on different GPUs: two kernels on
 * one GPU are not guaranteed to run concurrently.
 */
int dmoe_flag_signal(uint64_t* flag, uint64_t value, void* stream);
int dmoe_flag_wait(const uint64_t* flag, uint64_t value, uint64_t timeout_ns, int32_t* dev_status, void* stream);

/*
 * Expert-parallel exchange over NVLink peer memory (the NVLinkDirect transfer backend).
 * No single reference function: these replace, for ranks that run one forward per step in
 * lockstep, the per-task protocol of the reference's NIXL/MoonCake path --
 *   DispatchSubmit metadata (MoE/PipelineTask.py:262-270) -> dmoe_ep_plan (count exchange),
 *   gather + READ of the input buffer (MoE/PipelineTask.py:231-252,459;
 *     MoE/pools/BuffersPool.py:55-71) -> dmoe_ep_dispatch (peer stores into the receiver),
 *   WRITE of the expert output + HostOutputBufferUnlocked (MoE/PipelineTask.py:555-565;
 *     MoE/pools/BuffersPool.py:73-90) -> dmoe_ep_signal / dmoe_ep_wait (epoch flags),
 *   HostPipelineTask.combine (MoE/PipelineTask.py:306-370) -> dmoe_ep_combine (local rows).
 * Between dmoe_ep_wait(DATA) and dmoe_ep_signal(RESULTS) each rank runs ONE
 * dmoe_ep_expert_mlp over its receive buffer with the device segment table that
 * dmoe_ep_plan wrote (seg_expert, seg_end; n_seg = the rank's instance count); its
 * down-projection epilogue stores every row straight into its host's `rows` (the fused
 * return path: the transfer overlaps the GEMM, and the combine reads local rows).
 *
 * Window: per rank, in its own GPU memory and mapped into every rank (CUDA IPC):
 *   flags   dmoe_ep_flags_bytes() of uint64, zero-initialised: epochs [kind][sender], then
 *           the rank's epoch counter (advanced by dmoe_ep_plan, read by the other calls)
 *   counts  dmoe_ep_counts_bytes(n_inst) of int32 [2][DMOE_EP_MAX_RANKS][n_inst]
 *   recv    [cap, d] rows other ranks dispatch to (instance-major, then sender rank)
 *   back    [cap] int32: for each receive row, (sender rank << 27) | (token * k + slot)
 *   rows    [max_tokens * k, d] this rank's expert outputs, written by the owners' grouped
 *           MLP epilogues (peer stores) in (token, slot) order
 * The table passed to every call lists all ranks' windows as this process addresses them.
 * Instances (an expert's weights on one rank) are numbered rank-major; rank r's instances
 * are [inst_first[r], inst_first[r+1]) in the order of its weight stack (inst_slot).
 * Epochs: one per forward, counted on the device (every rank calls dmoe_ep_plan once per
 * forward, so the counters agree), starting at 1; no call takes an epoch from the host, so a
 * forward can be captured in a CUDA graph and replayed.  With world == 1 no flag of another
 * rank is touched.  Every wait is bounded by timeout_ns and reports DMOE_DEVERR_EP_TIMEOUT;
 * the rows of a rank that did not answer are left out.
 * A rank's waits are only ever satisfied by other GPUs: every rank must be its own GPU.
 */
#define DMOE_EP_MAX_RANKS 16
#define DMOE_EP_MAX_REPLICAS 4
#define DMOE_EP_MAX_INSTANCES 1024
#define DMOE_EP_POLICY_ROTATE 0 /* all of an expert's rows to one alive instance, rotating per step and rank */
#define DMOE_EP_POLICY_SPLIT 1  /* an expert's rows split evenly over its alive instances */
#define DMOE_EP_FLAG_COUNTS 0
#define DMOE_EP_FLAG_DATA 1
#define DMOE_EP_FLAG_RESULTS 2

typedef struct dmoe_ep_window {
  int32_t world, rank;
  void* flags[DMOE_EP_MAX_RANKS];
  void* counts[DMOE_EP_MAX_RANKS];
  void* recv[DMOE_EP_MAX_RANKS];
  void* back[DMOE_EP_MAX_RANKS];
  void* rows[DMOE_EP_MAX_RANKS];
} dmoe_ep_window;

size_t dmoe_ep_flags_bytes(void);
size_t dmoe_ep_counts_bytes(int n_inst);

/*
 * Count exchange and placement (one CTA).  counts_e [E]: this rank's rows per expert (the
 * routing plan's counts; NULL for an empty batch).  alive_n [E] / alive_inst
 * [E][DMOE_EP_MAX_REPLICAS]: the instances this sender may use (its ExpertBlocksPool's
 * alive blocks, MoE/pools/ExpertBlocksPool.py:37-71); an expert with none has its rows
 * dropped.  Writes part_n [E], part_inst [E][R], part_start [E][R+1], dest_off [n_inst]
 * (first receive row of this rank's rows of each instance on the owner) and this rank's
 * grouped-MLP table seg_expert / seg_end [its instance count].  Advances the epoch counter.
 */
int dmoe_ep_plan(const dmoe_ep_window* win, const int32_t* counts_e, int E, int n_inst, int policy,
                 const int32_t* alive_n, const int32_t* alive_inst, const int32_t* inst_rank, const int32_t* inst_slot,
                 const int32_t* inst_first, int64_t cap, uint64_t timeout_ns, int32_t* part_n,
                 int32_t* part_inst, int32_t* part_start, int32_t* dest_off, int32_t* seg_expert, int32_t* seg_end,
                 int32_t* dev_status, void* stream);

/*
 * Gather x[perm_token[p]] of every permuted activation p into its receiver's recv buffer and
 * (this rank << 27) | (perm_token[p] * k + perm_slot[p]) into the receiver's back map (peer
 * stores), record ret[p] = (rank << 27) | row (-1: dropped), then raise the DATA flag of
 * this rank on every rank.  done: a zeroed uint32 of this rank's scratch.
 */
int dmoe_ep_dispatch(const dmoe_ep_window* win, const void* x, int64_t row_bytes, int T, int k, int E,
                     const int32_t* offsets, const int32_t* perm_token, const int32_t* perm_slot,
                     const int32_t* part_n, const int32_t* part_inst, const int32_t* part_start,
                     const int32_t* inst_rank, const int32_t* dest_off, int64_t cap, int32_t* ret, uint32_t* done,
                     int32_t* dev_status, void* stream);

/*
 * The expert step of the exchange: the grouped gated MLP over this rank's receive buffer
 * (rows [0, cap), device segment table seg_expert / seg_end of n_seg local instances), whose
 * down-projection stores each row r at rows[back[r] >> 27] + (back[r] & 0x7ffffff) rows --
 * the host's return buffer, over NVLink for other ranks -- instead of an output buffer.
 * Replaces ExpertsBlockPipelineTask.run + the WRITE to the host's output buffer
 * (MoE/PipelineTask.py:478-520,555).  workspace >= dmoe_grouped_mlp_workspace_size(cap, I,
 * dtype); tile_policy as dmoe_grouped_gated_mlp_ex.
 */
int dmoe_ep_expert_mlp(const dmoe_ep_window* win, const void* w_gate, const void* w_up, const void* w_down,
                       int E_stack, int d, int I, int dtype, const int32_t* seg_expert, const int32_t* seg_end,
                       int n_seg, int64_t cap, int act, void* workspace, size_t workspace_bytes, int32_t* dev_status,
                       int tile_policy, void* stream);

/* The exchange's expert step with 8-bit receive rows: each receive record is d e4m3 codes,
 * the row's fp32 scale at byte d, padding to d + 16 bytes (dmoe_quantize_rows_e4m3 with
 * q_ld = d + 16, the scale pointer at q + d and scale_ld = (d + 16) / 4 makes them on the
 * sending side; the gather then moves d + 16 bytes a row, about half the bytes of a bf16
 * row).  Gate/up e4m3 [E_stack, I, d] with fp32 scales [E_stack, I]; down bf16
 * [E_stack, d, I]; the return rows are bf16.  d % 16 == 0; workspace as dmoe_ep_expert_mlp
 * with dtype DMOE_BF16. */
int dmoe_ep_expert_mlp_fp8(const dmoe_ep_window* win, const void* wg_q, const float* wg_scale, const void* wu_q,
                           const float* wu_scale, const void* w_down, int E_stack, int d, int I,
                           const int32_t* seg_expert, const int32_t* seg_end, int n_seg, int64_t cap, int act,
                           void* workspace, size_t workspace_bytes, int32_t* dev_status, int tile_policy,
                           void* stream);

/* Wait (bounded) until every other rank raised its flag of `kind` to this forward's epoch. */
int dmoe_ep_wait(const dmoe_ep_window* win, int kind, uint64_t timeout_ns, int32_t* dev_status, void* stream);

/* Raise this rank's flag of `kind` to this forward's epoch on every rank after the stream's
 * prior work. */
int dmoe_ep_signal(const dmoe_ep_window* win, int kind, void* stream);

/*
 * out[t] = (out[t] if accumulate) + sum_s w[t,s] * rows[t*k + s], over this rank's own return
 * rows (written by the owners' epilogues), skipping slots whose activation was dropped
 * (ret[inverse[t*k+s]] < 0); fp32 accumulation, one store.  dtype: DMOE_BF16, DMOE_F16 or
 * DMOE_F32 (rows and out).
 */
int dmoe_ep_combine(const dmoe_ep_window* win, const int32_t* inverse, const int32_t* ret, const void* w, int w_dtype,
                    int T, int k, int d, int dtype, int accumulate, void* out, void* stream);

/* Number of kernels this library launched in this process (for launch accounting). */
uint64_t dmoe_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* DMOE_B200_H */
