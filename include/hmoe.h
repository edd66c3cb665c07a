/*
 * hmoe.h -- C ABI of the B200 (sm_100a) HyperMoE sparse-expert hot path.
 *
 * Library: hypermoe-engine_b200/lib/libhmoe.so.  Plain pointers and sizes
 * only; every device pointer is CUDA global memory on the current device and
 * every `stream` is a cudaStream_t passed as void* (the reference's
 * StreamHandle, src/backend/Backend.hpp:12).  All launches are
 * stream-ordered and return before completion; no entry point allocates,
 * frees or synchronises unless its comment says so.  Errors are returned as
 * hmoe_status; nothing throws across this boundary.
 *
 * Two groups of entry points:
 *
 *  1. Per-operator drop-ins for the reference's CUDA kernel launchers
 *     hypermoe::backend::cuda::kernels::* (src/backend/cuda/CudaKernels.hpp:
 *     10-46) and planInt8Gemm (src/backend/cuda/Int8GemmPlan.hpp:19-20).
 *     Same arguments, same meaning, FP32 results within the reference's own
 *     CUDA-vs-CPU tolerance (1e-5 + 1e-5*|ref|).  The C++ shim in
 *     hypermoe-engine_b200/host/CudaKernelsShim.cpp defines the reference's
 *     C++ symbols over these.
 *
 *  2. The fused layer path that replaces the per-expert host loop of
 *     MoERuntime::executeBatch (src/core/runtime/MoERuntime.cpp:58-349) when
 *     every expert of the layer is resident: route -> permute -> grouped
 *     INT8 expert MLP (dequantised to BF16 for tensor cores, FP32
 *     accumulation, SwiGLU fused) -> deterministic weighted combine.
 */
#ifndef HMOE_H
#define HMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    HMOE_OK = 0,
    HMOE_INVALID_ARGUMENT = 1,  /* std::invalid_argument in the reference */
    HMOE_NON_FINITE_ROUTER = 2, /* "router produced a non-finite score" */
    HMOE_CUDA_ERROR = 3,        /* launch/runtime error (checkLaunch) */
    HMOE_NCCL_ERROR = 4,
    HMOE_TIMEOUT = 5,
    HMOE_WORKSPACE_TOO_SMALL = 6,
    HMOE_UNSUPPORTED = 7
} hmoe_status;

/* Last CUDA error string seen by this thread (checkLaunch's message). */
const char *hmoe_last_error(void);

/* ------------------------------------------------ 1. per-operator drop-ins */

/* kernels::activation (CudaKernels.hpp:10-11): type 0 = SiLU, 1 = GELU(erf). */
hmoe_status hmoe_activation(int type, const float *input, float *output,
                            size_t elements, void *stream);

/* kernels::int8WeightMatmul (CudaKernels.hpp:12-15):
 * output[r,c] = sum_k left[r,k] * (float(right[k,c] - zero_point) * scale),
 * left [rows,inner] FP32, right [inner,columns] INT8 row-major. */
hmoe_status hmoe_int8_weight_matmul(const float *left, const int8_t *right,
                                    float *output, size_t rows, size_t inner,
                                    size_t columns, float scale,
                                    int32_t zero_point, void *stream);

/* kernels::int8WeightMatmulCooperative (CudaKernels.hpp:16-21).  Validates
 * `partitions` against hmoe_int8_gemm_plan(..., COOPERATIVE) exactly as the
 * reference does (CudaKernels.cu:330-333) and returns
 * HMOE_INVALID_ARGUMENT on a mismatch or a missing `partials` buffer. */
hmoe_status hmoe_int8_weight_matmul_cooperative(
    const float *left, const int8_t *right, float *output, float *partials,
    size_t rows, size_t inner, size_t columns, size_t partitions, float scale,
    int32_t zero_point, void *stream);

/* planInt8Gemm (Int8GemmPlan.hpp:8-20, Int8GemmPlan.cpp:29-53). */
typedef enum {
    HMOE_INT8_GEMM_AUTO = 0,
    HMOE_INT8_GEMM_REFERENCE = 1,
    HMOE_INT8_GEMM_COOPERATIVE = 2
} hmoe_int8_gemm_mode;

typedef struct {
    int32_t implementation; /* hmoe_int8_gemm_mode, never AUTO */
    size_t partitions;
    size_t blocks;
    size_t scratch_elements;
} hmoe_int8_gemm_plan_t;

hmoe_status hmoe_int8_gemm_plan(size_t rows, size_t inner, size_t columns,
                                int32_t mode, hmoe_int8_gemm_plan_t *plan);

/* kernels::routerTopK (CudaKernels.hpp:28-31).  `logits` [tokens,experts]
 * is overwritten with probabilities when softmax != 0, as the reference
 * kernel does.  Selection is (score desc, id asc); renormalisation uses a
 * double sum; a non-finite or zero selected sum writes NaN to the token's
 * first score (CudaKernels.cu:195-203). */
hmoe_status hmoe_router_topk(float *logits, size_t tokens, size_t experts,
                             size_t top_k, int softmax, int renormalize,
                             uint32_t *selected_ids, float *selected_scores,
                             void *stream);

/* kernels::gatherRows (CudaKernels.hpp:40-41): output[r,:] = input[rows[r],:]. */
hmoe_status hmoe_gather_rows(const float *input, float *output,
                             const uint32_t *rows, size_t row_count,
                             size_t width, void *stream);

/* kernels::scatterAddRows (CudaKernels.hpp:42-45):
 * output[rows[r],:] += input[r,:] * weights[r] (atomic, like the reference). */
hmoe_status hmoe_scatter_add_rows(const float *input, float *output,
                                  const uint32_t *rows, const float *weights,
                                  size_t row_count, size_t width,
                                  void *stream);

/* kernels::zero (CudaKernels.hpp:46). */
hmoe_status hmoe_zero(float *output, size_t elements, void *stream);

/* ------------------------------------------------------- 2. fused layer */

/* Quantisation parameters of one expert: gate, up, down
 * (ExpertMlpWeights, src/experts/ExpertExecutor.hpp:18-43; each
 * QuantizationParameters{scale, zeroPoint}, Quantization.hpp:19-25). */
typedef struct {
    float scale[3];
    int32_t zero_point[3];
} hmoe_expert_quant;

/* One MoE layer, all experts resident on this device.
 *
 * Expert weights: one INT8 arena in the ExpertPacker layout
 * (tools/model_convert/ExpertPacker.cpp:150-247): expert e's blob starts at
 * arena + e*expert_stride and holds gate [H,I], up [H,I], down [I,H], each
 * row-major [in,out] (INPUT_OUTPUT), at gate_offset/up_offset/down_offset
 * inside the blob.  ExpertWeightMap::createViews (ExpertWeightMap.cpp:
 * 65-108) slices exactly these views.  expert_stride and the offsets must
 * be multiples of 16 bytes and H, I multiples of 64.  The arena and the
 * router matrix must start on a 16-byte boundary, the quantisation records
 * and the bias on a 4-byte one (cudaMalloc and the reference's memory pool
 * give 256): tensor and bulk copies read them, and a misaligned address
 * would fault, so every layer entry point refuses it with
 * HMOE_INVALID_ARGUMENT.
 *
 * Routed experts are ids [0, experts); `shared_experts` always-on experts
 * follow them in the arena (ids experts..experts+shared-1), see every token
 * with weight 1.0, and are combined after the routed ones.
 *
 * `router_bias` (NULL for none) is added to each logit as the last term of
 * the double accumulation (what the reference computes for a hidden row
 * extended by 1 and a router matrix extended by the bias row).
 *
 * ep_rank/ep_size: expert parallelism (one process per GPU).  The
 * single-GPU entry points need ep_rank = 0, ep_size = 1.  For
 * hmoe_ep_moe_forward this rank owns the routed experts
 * hmoe_ep_expert_range(experts, ep_size, ep_rank) returns, and `arena` /
 * `quant` hold only those (local ids 0..count-1) followed by the shared
 * experts, which every rank holds and applies to its own tokens. */
typedef struct {
    uint32_t hidden;          /* H */
    uint32_t intermediate;    /* I */
    uint32_t experts;         /* E, routed */
    uint32_t top_k;           /* k */
    int32_t softmax;          /* RoutingNormalization::Softmax */
    int32_t renormalize;      /* RouterConfig::renormalizeSelected */
    uint32_t shared_experts;  /* always-on experts after the routed ones */
    uint32_t reserved0;
    const float *router_weight; /* device [H, E] FP32 row-major */
    const float *router_bias;   /* device [E] FP32 or NULL */
    const int8_t *arena;        /* device, see above */
    uint64_t expert_stride;
    uint64_t gate_offset, up_offset, down_offset;
    const hmoe_expert_quant *quant; /* device [experts + shared_experts] */
    int32_t ep_rank, ep_size;
} hmoe_layer_desc;

/* Scratch bytes hmoe_route / hmoe_moe_forward need for up to max_tokens
 * (OR max_tokens with HMOE_WORKSPACE_HOST_IO to include the staging area of
 * hmoe_moe_forward_host). */
#define HMOE_WORKSPACE_HOST_IO ((size_t)1 << 62)
hmoe_status hmoe_workspace_size(const hmoe_layer_desc *desc,
                                size_t max_tokens, size_t *bytes);

/* Router + device-built expert grouping (CudaTensorBackend::routeTopK,
 * CudaTensorBackend.cpp:601-652, plus the grouping of
 * CpuRouterBackend::routeBatch, CpuRouterBackend.cpp:140-158), in one
 * stream-ordered call with no host readback.
 *   ids/scores [T,k]  rank order (score desc, id asc), bit-exact selection
 *                     against the CPU router on the same inputs;
 *   offsets [E+1]     exclusive prefix of tokens per routed expert;
 *   group_tokens [T*k], group_scores [T*k]: expert groups, ascending expert,
 *                     tokens ascending inside a group.
 * Any output pointer may be NULL. */
hmoe_status hmoe_route(const hmoe_layer_desc *desc, const float *x,
                       size_t tokens, uint32_t *ids, float *scores,
                       int32_t *offsets, uint32_t *group_tokens,
                       float *group_scores, void *workspace,
                       size_t workspace_bytes, void *stream);

/* One MoE layer forward: y[T,H] FP32 = sum over the token's experts, in
 * ascending expert id, of routing_weight * expert_mlp(x).  x [T,H] FP32.
 * x, y and the workspace start on 16-byte boundaries (HMOE_INVALID_ARGUMENT
 * otherwise), as do residual and y_bf16 in the entry points that take them. */
hmoe_status hmoe_moe_forward(const hmoe_layer_desc *desc, const float *x,
                             float *y, size_t tokens, void *workspace,
                             size_t workspace_bytes, void *stream);

/* hmoe_moe_forward for callers holding HOST buffers (the reference's CPU
 * backend callers): copies x_host [T,H] into the workspace, runs the layer
 * and copies y back to y_host, all on `stream` (page-locked host memory
 * makes the copies asynchronous).  Returns after enqueueing; y_host is
 * valid once the stream has completed.  Needs hmoe_workspace_size(...,
 * HMOE_WORKSPACE_HOST_IO) bytes. */
hmoe_status hmoe_moe_forward_host(const hmoe_layer_desc *desc,
                                  const float *x_host, float *y_host,
                                  size_t tokens, void *workspace,
                                  size_t workspace_bytes, void *stream);

/* hmoe_moe_forward with the transformer layer's residual add and its
 * activation boundary fused into the combine (MoELayer::execute,
 * src/transformer/MoELayer.cpp:19-48: output = attention + moe.output
 * followed by a host synchronisation; TransformerBlock.cpp:101-104):
 *   y[t]      = residual[t] + moe(x)[t], one FP32 rounding after the
 *               token's expert outputs are summed (the reference's add);
 *   y_bf16[t] = BF16(y[t]) (round to nearest even), for a next layer that
 *               reads BF16 activations; [T, H] of uint16_t bit patterns.
 * residual == NULL gives hmoe_moe_forward's y; y_bf16 may be NULL.
 * residual may alias x or y (in place); y may alias x.  Same workspace and
 * stream rules as hmoe_moe_forward; no host synchronisation. */
hmoe_status hmoe_moe_forward_residual(const hmoe_layer_desc *desc,
                                      const float *x, const float *residual,
                                      float *y, uint16_t *y_bf16,
                                      size_t tokens, void *workspace,
                                      size_t workspace_bytes, void *stream);

/* RMSNorm of `tokens` rows of `hidden` FP32 values (replaces the CUDA
 * branch of RMSNorm::execute, src/transformer/norm/RMSNorm.cpp:53-58, with
 * the CPU branch's arithmetic, :64-77):
 *   output[t][i] = float(double(input[t][i]) * inv_t * double(weight[i])),
 *   inv_t = 1 / sqrt(sum_i double(input[t][i])^2 / hidden + epsilon),
 * the sum taken in double (as a tree, where the reference sums
 * sequentially).  This is the normalisation a transformer block applies
 * before its MoE layer (TransformerBlock.cpp:90-92); a stack of MoE layers
 * calls it before every layer.  output may alias input.  epsilon > 0 and
 * finite (RMSNorm's constructor check); tokens == 0 is a no-op.  Enqueues
 * on `stream`; no host synchronisation, no allocation. */
hmoe_status hmoe_rms_norm(const float *input, const float *weight,
                          float *output, size_t tokens, size_t hidden,
                          float epsilon, void *stream);

/* hmoe_moe_forward with no caller workspace: scratch is a file-scope
 * device array of 16 MiB per device inside libhmoe.so, so the call allocates
 * nothing.  No counterpart in the reference (whose layer path allocates
 * through CudaMemoryPool); it serves callers that cannot allocate device
 * memory at the call site.  Batches whose hmoe_workspace_size exceeds
 * 16 MiB return HMOE_WORKSPACE_TOO_SMALL (C3 layer: up to 185 tokens).
 * Calls that overlap in time on one device race on the shared scratch.
 * The first call on a device looks the array up (cudaGetSymbolAddress);
 * make it before any stream capture on that device.  The looked-up address
 * is kept for the life of the process: it is not valid across
 * cudaDeviceReset. */
hmoe_status hmoe_moe_forward_noalloc(const hmoe_layer_desc *desc,
                                     const float *x, float *y, size_t tokens,
                                     void *stream);

/* hmoe_read_status for hmoe_moe_forward_noalloc: reads (and resets) the
 * device status word the last no-allocation call on the current device left
 * at the start of the static scratch -- HMOE_NON_FINITE_ROUTER for a NaN or
 * Inf router input, HMOE_TIMEOUT from a bounded device wait, the near-tie
 * and sequential-logit counts.  Synchronises `stream`.  Like the forward
 * call it has no counterpart in the reference. */
hmoe_status hmoe_noalloc_read_status(int32_t *status, int32_t *near_ties,
                                     int32_t *sequential_logits, void *stream);

/* Forces the expert-MLP variant for measurement: 0 = automatic (the
 * single-kernel decode layer for batches of at most 2 tokens whose shape it
 * takes, GEMV for launches of at most 8 permuted rows, tensor-core GEMM
 * otherwise, with its narrow-tile kernel when no expert can hold more than
 * 64 rows), 1 = multi-kernel GEMV only, 2 = tensor-core GEMM only, 3 = the
 * decode layer only (HMOE_UNSUPPORTED for a batch or shape it does not
 * take), 4 = tensor-core GEMM with its wide-tile kernel only.  The decode
 * layer gives the multi-kernel GEMV variant's result bit for bit, and the
 * two GEMM kernels give the same bits.  Process-wide. */
hmoe_status hmoe_set_variant(int32_t variant);

/* Forces the router kernel for measurement: 0 = automatic (the tiled kernel
 * for batches of 512 tokens or more when E <= 128, E % 4 == 0 and
 * H % 32 == 0; the decode kernel for 1 or 2 tokens when H % 128 == 0),
 * 1 = the per-8-token cluster kernel, 2 = the tiled kernel (64-token tiles
 * on the FP64 tensor-core path), 3 = the decode kernel (a grid over H and
 * the experts, up to 16 tokens); routing calls whose shape a forced kernel does not take
 * return HMOE_UNSUPPORTED.  All produce bit-identical results.  Process-wide;
 * query hmoe_workspace_size after setting it. */
hmoe_status hmoe_set_route_variant(int32_t variant);

/* Measurement hooks.  hmoe_set_stage_events registers `count` (= 6)
 * cudaEvent_t handles (passed as void*) that every later hmoe_moe_forward
 * records on its stream at the stage boundaries: [0] start, [1] after the
 * router, [2] after the grouping, [3] after gate/up, [4] after down,
 * [5] after the combine.  count = 0 unregisters them.  Stage [2] covers
 * the grouping, the BF16 row permutation and the tile list (for
 * hmoe_ep_moe_forward also the count exchange and the dispatch); [5]
 * after the return transfer and the combine.  Process-wide, for
 * benchmarks; the events are the caller's. */
hmoe_status hmoe_set_stage_events(void *const *events, int32_t count);

/* Number of kernels this library has launched in the process so far. */
int64_t hmoe_launch_count(void);

/* Synchronises `stream` and reads the device status word the last call on
 * `workspace` left: status (hmoe_status), the number of router near-ties the
 * device could not certify against the CPU's expf rounding, and the number
 * of logits it recomputed in sequential order.  Resets the word. */
hmoe_status hmoe_read_status(void *workspace, int32_t *status,
                             int32_t *near_ties, int32_t *sequential_logits,
                             void *stream);

/* ------------------------------------------------ expert parallelism
 *
 * One process per GPU.  Routed experts are split into contiguous ranges,
 * tokens stay data-parallel: each rank routes its own tokens, sends each
 * row (BF16) and its routing weight to the rank owning the expert, runs its
 * experts over what it received, and gets the weighted output rows back for
 * a combine in ascending expert id.  Transfers are NCCL point-to-point
 * operations over NVLink/NVSwitch, loaded with dlopen (HMOE_NCCL_LIBRARY
 * overrides the library name).  The reference is single-process and
 * single-device: these entry points have no counterpart there. */
#define HMOE_EP_MAX_RANKS 64
#define HMOE_EP_UNIQUE_ID_BYTES 128

typedef struct hmoe_ep_comm hmoe_ep_comm;

/* Expert ownership: rank r owns routed experts [first, first + count),
 * first = r*(E/P) + min(r, E%P) (e.g. 60 experts on 8 ranks: 8,8,8,8,7,7,7,7).
 * Host only. */
hmoe_status hmoe_ep_expert_range(uint32_t experts, int32_t ep_size,
                                 int32_t ep_rank, uint32_t *first,
                                 uint32_t *count);

/* Transfer plan of one rank, from the routed row counts of every
 * (source rank, expert) pair, counts[ep_size][experts].  Host only; every
 * rank computes it from the same counts, so a rejection (negative counts,
 * a total that is not a multiple of top_k, a rank with more than max_tokens
 * tokens -> HMOE_WORKSPACE_TOO_SMALL) happens on all ranks alike. */
typedef struct {
    uint32_t first_expert, local_experts;
    int64_t tokens[HMOE_EP_MAX_RANKS];      /* tokens of each rank */
    int64_t send_rows[HMOE_EP_MAX_RANKS];   /* rows to each peer ... */
    int64_t send_offset[HMOE_EP_MAX_RANKS]; /* ... from this permuted row */
    int64_t recv_rows[HMOE_EP_MAX_RANKS];   /* rows from each peer ... */
    int64_t recv_offset[HMOE_EP_MAX_RANKS]; /* ... into this receive row */
    int64_t recv_total;
} hmoe_ep_plan_t;
hmoe_status hmoe_ep_plan(const int32_t *counts, uint32_t experts,
                         uint32_t top_k, int32_t ep_size, int32_t ep_rank,
                         size_t max_tokens, hmoe_ep_plan_t *plan);

/* Transfer plan of one rank on the peer-memory path (a registered
 * workspace), as ep_exchange_kernel builds it on the device from the
 * exchanged per-slot row counts slot_counts[ep_size][experts] (negative
 * counts count as zero).  Owner q holds the slots hmoe_ep_expert_range
 * gives it; every owner's receive rows hold its sources' rows source by
 * source.  Host only (the device kernel runs the same code).  A rank
 * receiving more than capacity_rows rows (ep_size * max_tokens * top_k on
 * the device) gives HMOE_INVALID_ARGUMENT and a plan that moves nothing,
 * on every rank alike.  No counterpart in the reference (single process). */
typedef struct {
    int32_t send_off[HMOE_EP_MAX_RANKS];  /* this rank's rows for owner q start here ... */
    int32_t send_rows[HMOE_EP_MAX_RANKS]; /* ... and are this many */
    int32_t dest_base[HMOE_EP_MAX_RANKS]; /* and land at this row of q's receive rows */
    int32_t recv_base[HMOE_EP_MAX_RANKS]; /* rows from source p start at this receive row ... */
    int32_t recv_rows[HMOE_EP_MAX_RANKS]; /* ... and are this many */
    int32_t ret_off[HMOE_EP_MAX_RANKS];   /* and return to this row of p's permuted rows */
    int32_t recv_total, sent_total;
} hmoe_ep_peer_plan_t;
hmoe_status hmoe_ep_peer_plan(const int32_t *slot_counts, uint32_t experts,
                              int32_t ep_size, int32_t ep_rank,
                              int64_t capacity_rows,
                              hmoe_ep_peer_plan_t *plan);

/* NCCL unique id (HMOE_EP_UNIQUE_ID_BYTES bytes) made on one rank and
 * shared with the others by the caller. */
hmoe_status hmoe_ep_unique_id(void *id, size_t bytes);

/* Collective over ep_size processes: creates this rank's communicator on
 * the current device (allocates pinned host memory and an event; blocks
 * until every rank has joined).  timeout_ms bounds every later host wait
 * for peers; when it expires the communicator is aborted and
 * hmoe_ep_moe_forward returns HMOE_TIMEOUT. */
hmoe_status hmoe_ep_comm_create(const void *unique_id, int32_t rank,
                                int32_t size, int32_t timeout_ms,
                                hmoe_ep_comm **comm);
hmoe_status hmoe_ep_comm_destroy(hmoe_ep_comm *comm);

/* Expert placement of the communicator (all ranks must set the same one):
 * slot_of_expert[e] is a permutation of [0, experts); rank r owns the slots
 * hmoe_ep_expert_range returns, so its arena holds the experts whose slot
 * is in that range, in slot order, followed by the shared experts.
 * NULL / 0 restores the identity (contiguous expert ids).  Results do not
 * depend on the placement: rows are combined in ascending expert id.
 * Set-up call (allocates a small device table). */
hmoe_status hmoe_ep_set_placement(hmoe_ep_comm *comm,
                                  const int32_t *slot_of_expert,
                                  uint32_t experts);

/* Static load balancing of experts over ep_size ranks from an expected load
 * per expert (e.g. a routing-frequency profile): largest load first, each to
 * the least-loaded rank with a free slot.  Host only. */
hmoe_status hmoe_ep_balanced_placement(const double *load, uint32_t experts,
                                       int32_t ep_size,
                                       int32_t *slot_of_expert);

/* The transfer plan of the communicator's last hmoe_ep_moe_forward
 * (observability: received rows, per-peer transfer sizes). */
hmoe_status hmoe_ep_last_plan(const hmoe_ep_comm *comm, hmoe_ep_plan_t *plan);

/* Collective: maps this rank's EP workspace (from cudaMalloc, the size
 * hmoe_ep_workspace_size returns, the same on every rank) into every other
 * rank's process (CUDA IPC over NVLink/NVSwitch) and every other rank's into
 * this one.  hmoe_ep_moe_forward called with exactly this workspace then
 * runs the peer-memory path: the count exchange, the dispatch of rows and
 * the return of expert outputs are stores into the peers' memory ordered by
 * epoch flags, with no host synchronisation and no NCCL; any other
 * workspace takes the NCCL path.  Waits for the device first; NULL
 * unregisters (also collective).  HMOE_UNSUPPORTED on every rank when any
 * rank cannot map every workspace.  Each flag wait gives up after the
 * communicator's timeout and reports HMOE_TIMEOUT in the status word
 * (hmoe_ep_read_status).  A rank that times out (or whose count exchange
 * fails) marks every rank's workspace aborted before it signals anything:
 * the other ranks' waits then fail at once, so every rank reports
 * HMOE_TIMEOUT instead of computing on rows that were never sent, and every
 * later forward on these workspaces fails the same way until the ranks
 * register them again (which clears the mark). */
hmoe_status hmoe_ep_register_workspace(hmoe_ep_comm *comm, void *workspace,
                                       size_t bytes);

/* hmoe_read_status for an EP workspace (its single-GPU part follows the
 * peer path's flag area). */
hmoe_status hmoe_ep_read_status(void *workspace, int32_t *status,
                                int32_t *near_ties, int32_t *sequential_logits,
                                void *stream);

/* Self-test of the peer path's bounded flag wait (registered workspace
 * needed): waits for a flag epoch no rank reaches, with the given limit,
 * and returns the status the wait reported (HMOE_TIMEOUT).  Synchronous. */
hmoe_status hmoe_ep_selftest_flag_wait(hmoe_ep_comm *comm, uint64_t limit_ns,
                                       int32_t *status);

/* Scratch bytes of hmoe_ep_moe_forward for up to max_tokens tokens on
 * every rank (the receive side holds ep_size*max_tokens*top_k rows, the
 * worst case of every token of every rank choosing this rank's experts). */
hmoe_status hmoe_ep_workspace_size(const hmoe_layer_desc *desc,
                                   size_t max_tokens, size_t *bytes);

/* Collective: one MoE layer forward of this rank's `tokens` tokens
 * (0 allowed) with experts spread over the communicator's ranks.  Every
 * rank passes the same desc (except arena/quant/ep_rank) and the same
 * max_tokens.  Enqueues on `stream`; without a registered workspace it
 * synchronises on the host once, to read the exchanged row counts (bounded
 * by the communicator's timeout).
 * The result equals hmoe_moe_forward on the concatenation of all ranks'
 * tokens for the same expert-MLP variant. */
hmoe_status hmoe_ep_moe_forward(const hmoe_layer_desc *desc,
                                hmoe_ep_comm *comm, const float *x, float *y,
                                size_t tokens, size_t max_tokens,
                                void *workspace, size_t workspace_bytes,
                                void *stream);

/* Collective: hmoe_ep_moe_forward with the residual add and the BF16 copy
 * of hmoe_moe_forward_residual fused into this rank's combine
 * (MoELayer::execute, src/transformer/MoELayer.cpp:19-48, plus the residual
 * add of TransformerBlock::forward, TransformerBlock.cpp:101-104, for a
 * layer whose experts are spread over ranks).  residual may be NULL and may
 * alias x or y; y may alias x; y_bf16 may be NULL.  A stack of layers calls
 * it once per layer with the same communicator and workspace. */
hmoe_status hmoe_ep_moe_forward_residual(const hmoe_layer_desc *desc,
                                         hmoe_ep_comm *comm, const float *x,
                                         const float *residual, float *y,
                                         uint16_t *y_bf16, size_t tokens,
                                         size_t max_tokens, void *workspace,
                                         size_t workspace_bytes,
                                         void *stream);

/* Failure-detection self-test (no counterpart in the reference): launches
 * one kernel that waits on an mbarrier nothing arrives on, using the same
 * bounded wait as every kernel of the library.  After limit_us (1..10^6)
 * microseconds the wait gives up, HMOE_TIMEOUT is recorded in the status
 * word at the start of `workspace` (read it with hmoe_read_status) and the
 * kernel returns; the context stays usable. */
hmoe_status hmoe_selftest_bounded_wait(void *workspace, uint32_t limit_us,
                                       void *stream);

/* ----------------------------------------- host-side synthetic inputs */

/* Seeded counter-based normal generator (SplitMix64 + Box-Muller in double),
 * identical on every host: out[i] = sigma * N(0,1) for stream `stream`. */
void hmoe_synth_normal(uint64_t seed, uint64_t stream, float sigma, float *out,
                       size_t n, int threads);

/* Zipf(alpha) per-expert logit bias: bias[e] = -alpha*ln(pi(e)+1) for a
 * seeded permutation pi of [0, E). */
void hmoe_synth_zipf_bias(uint64_t seed, float alpha, float *bias, size_t E);

/* Symmetric per-tensor INT8 quantiser (quantizeInt8,
 * src/tensor/quantization/Quantization.cpp:45-79). */
hmoe_status hmoe_quantize_int8(const float *w, size_t n, int8_t *q,
                               float *scale, int32_t *zero_point,
                               float *max_abs_error);

/* Fills a host INT8 arena (layout as in hmoe_layer_desc) for `count`
 * experts starting at expert id `first`: gate/up/down ~ N(0, sigma^2) from
 * streams derived from (layer, expert, projection), each quantised per
 * projection.  quant[count] receives the parameters. */
void hmoe_synth_arena(uint64_t seed, uint32_t layer, uint32_t first,
                      uint32_t count, uint32_t H, uint32_t I, float sigma,
                      int8_t *arena, uint64_t expert_stride,
                      uint64_t gate_offset, uint64_t up_offset,
                      uint64_t down_offset, hmoe_expert_quant *quant,
                      int threads);

#ifdef __cplusplus
}
#endif

#endif /* HMOE_H */
