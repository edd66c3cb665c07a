// layer.cuh -- internal interfaces between the fused-layer kernels.
#pragma once

#include "common.cuh"

#include <cuda.h>

namespace hmoe {

// Byte offsets of the workspace segments (all 256-byte aligned).
// hmid holds the intermediate rows: FP32 for the GEMV variant, BF16 for the
// GEMM variant (one launch uses one of them).
// Tokens per block of the grouping's counting sort; the router counts the
// selected experts of each block.
constexpr int kGroupBlock = 256;

struct Workspace {
    size_t status, counts, block_counts, route_acc, route_acc_bytes, zero_bytes, offsets, ids, scores, perm_token, perm_weight, inv;
    size_t xperm, xscale, hmid, yrows, tiles, tile_count;
    size_t dl_ctl, dl_ctl_bytes, dl_data, dl_data_bytes; // decode layer kernel (0 bytes when it does not apply)
    int tile_cap;
    size_t total;
};

Workspace plan_workspace(const hmoe_layer_desc& d, size_t T);

// Batches with at most this many (token, expert) assignments use the
// weight-streaming GEMV for every expert; larger ones the tcgen05 GEMM.  On
// the Qwen3-30B-A3B layer (top-8) the GEMM is as fast as the GEMV at one
// token (95 us per layer call) and faster from two tokens on (106 against
// 123 us at T=2, 124 against 172 us at T=8).
constexpr int kGemvMaxAssignments = 8;

// Upper bound of a token's rows (top_k routed + shared experts).
constexpr int kMaxSlots = 96;

// One expert-MLP pass over permuted rows.  Rows of one expert are cut into
// tiles (expert, first row, rows, segment group) of at most kTileRows rows;
// both variants consume the same tile list.  The segment group is the
// source rank under expert parallelism (0 on one GPU).
constexpr int kTileRows = 256;

// Where the down projection's output rows go when they are pushed back to
// their source ranks (expert parallelism, peer-memory path): receive row d
// of a tile from source p is stored at row ret_off[p] + d - recv_base[p] of
// the BF16 rows at byte offset `off` of source p's workspace peer[p], unless
// the abort word is set.  peer == null: rows stay in ExpertRun::yrows.
struct PushRows {
    char* const* peer;
    size_t off;
    const int32_t* ret_off;
    const int32_t* recv_base;
    const uint32_t* abort;
};

// Row d of a pushed tile from source p (or row d of `local`).
__device__ __forceinline__ __nv_bfloat16* pushed_row(const PushRows& p, __nv_bfloat16* local, int src, int d, int N) {
    if (!p.peer) return local + static_cast<size_t>(d) * N;
    return reinterpret_cast<__nv_bfloat16*>(p.peer[src] + p.off) +
           static_cast<size_t>(p.ret_off[src] + d - p.recv_base[src]) * N;
}

struct ExpertRun {
    const __half* xrows;        // [rows_cap, H] permuted input rows, FP16, scaled per token
    const float* xscale;        // [rows_cap] 1 / (power-of-two scale) of each row
    const float* weight;        // [rows_cap] routing weight of each row
    const int4* tiles;          // device tile list
    const int32_t* tile_count;  // device count
    int tile_cap;               // launch capacity (>= count)
    int rows_cap;               // rows allocated in xrows / hmid / yrows
    float* hmid32;              // [rows_cap, I] GEMV intermediate
    __nv_bfloat16* hmid16;      // [rows_cap, I] GEMM intermediate
    __nv_bfloat16* yrows;       // [rows_cap, H] weighted expert outputs
    const int8_t* arena;        // experts indexed by tile expert id
    uint64_t stride, gate_offset, up_offset, down_offset;
    const hmoe_expert_quant* quant;
    int experts;                // experts in the arena
    int H, I;
    int max_group;              // upper bound of rows of one expert
    DeviceStatus* st;
    PushRows push;              // down outputs pushed to their sources (peer == null: yrows)
};

struct GemvArgs {
    const int4* tiles;
    const int32_t* tile_count;
    const __half* act16;        // gate/up input rows (FP16, scaled per token)
    const float* xscale;        // gate/up: 1 / scale of each row
    const float* act32;         // down input rows (FP32 intermediate)
    const float* weight;        // down: routing weight per row
    const hmoe_expert_quant* quant;
    int proj0;                  // 0: gate (and up), 2: down
    float* out32;               // gate/up: FP32 intermediate
    __nv_bfloat16* out16;       // down: BF16 weighted rows
    PushRows push;              // down: rows pushed to their sources instead (peer != null)
    int K, N, KS;
    DeviceStatus* st;
};

// Segments of permuted rows: segment i holds rows of expert
// expert_base + (i mod eps).  Rows come from offsets[i] .. offsets[i+1] or,
// when offsets is null, from an exclusive scan of
// counts[(i / eps) * count_stride + (i mod eps)] starting at row_base.
constexpr int kMaxSegments = 512;

struct SegSpec {
    const int32_t* offsets;
    const int32_t* counts;
    int count_stride;
    int nseg;
    int eps;
    int expert_base;
    int row_base;
};

bool gemm_available();
// The tensor-core GEMM streams K in 128-deep stages.
inline bool gemm_shape_ok(int H, int I) { return H % 128 == 0 && I % 128 == 0; }
int device_sm_count();
// TMA map of one INT8 projection over all experts: dims {N, K, experts},
// box [box_k][box_n] (no swizzle).  False when the driver rejects it.
bool map_weights_box(CUtensorMap* m, const int8_t* base, int N, int K, int experts, uint64_t stride, int box_n,
                     int box_k);
// TMA map of an FP32 row-major matrix [rows][cols] (cols % 4 == 0): box
// [box_rows][box_cols] of 128-byte rows, 128-byte swizzle, zero fill outside.
bool map_f32_rows_sw128(CUtensorMap* m, const float* base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                        uint32_t box_rows);
hmoe_status gemm_gate_up(const ExpertRun& r, cudaStream_t stream);
hmoe_status gemm_down(const ExpertRun& r, cudaStream_t stream);
hmoe_status gemv_gate_up(const ExpertRun& r, cudaStream_t stream);
hmoe_status gemv_down(const ExpertRun& r, cudaStream_t stream);

hmoe_status launch_tile_list(const SegSpec& spec, int4* tiles, int32_t* tile_count, int capacity,
                             cudaStream_t stream);
// xrows[inv[t, s]] = FP16(x[t] * s_t), xscale[inv[t, s]] = 1 / s_t for
// every token t and slot s (s_t: power of two, max |x[t]| s_t in [2^14, 2^15)).
// With `seg`, the same launch also builds the tile list of `seg` (as
// launch_tile_list does).
hmoe_status launch_permute(const float* x, const int32_t* inv, int tokens, int slots, int H, __half* xrows,
                           float* xscale, cudaStream_t stream, const SegSpec* seg = nullptr, int4* tiles = nullptr,
                           int32_t* tile_count = nullptr, int capacity = 0);

// The grouping of a batch of at most kGroupBlock tokens fused with its
// permutation and tile list (one launch instead of the grouping's and the
// permutation's): the same offsets, permutation, inverse map, token rows
// and tiles as launch_group followed by launch_permute with `seg`, for a
// layer without an expert placement.  ids/scores/counts are the router's.
struct SmallGroup {
    const uint32_t* ids;   // [T, k]
    const float* scores;   // [T, k]
    const int32_t* counts; // [E] routed rows per expert
    int T, k, E, S;
    int32_t* offsets;      // [E+S+1]
    uint32_t* perm_token;  // [T*(k+S)]
    float* perm_weight;    // [T*(k+S)]
    int32_t* inv;          // [T*(k+S)]
};
hmoe_status launch_group_permute(const SmallGroup& g, const float* x, int H, __half* xrows, float* xscale,
                                 const SegSpec& seg, int4* tiles, int32_t* tile_count, int capacity,
                                 cudaStream_t stream);

// Upper bound of the tiles of `rows` rows spread over `segments` segments.
int tile_capacity_for(long rows, int segments);

hmoe_status launch_route(const float* x, const float* w, const float* bias, int T, int H, int E, int k,
                         int softmax, int renorm, uint32_t* ids, float* scores, int32_t* counts,
                         int32_t* block_counts, double* decode_scratch, DeviceStatus* st, cudaStream_t stream);
// Zeroed scratch bytes the decode router needs for T tokens (0 when it does
// not take the shape).
size_t route_decode_scratch_bytes(size_t T, int H, int E);
// Expert groups in ascending expert id, or in placement-slot order when
// expert_of_slot is given (then slot_counts[b] = rows of slot b).
hmoe_status launch_group(const uint32_t* ids, const float* scores, const int32_t* counts,
                         const int32_t* block_counts, int T, int k, int E, int S, int32_t* offsets,
                         uint32_t* perm_token, float* perm_weight, int32_t* inv, const int32_t* expert_of_slot,
                         int32_t* slot_counts, cudaStream_t stream);
// out[t] = sum of the token's rows in ascending expert id: routed slot j has
// expert ids[t, j] (when ids is null the row order is the expert order),
// shared expert s counts as expert E + s.
// residual (may be null, may equal out): out[t] = residual[t] + sum, one
// FP32 rounding; out16 (may be null): a BF16 copy of out.
hmoe_status launch_combine(const __nv_bfloat16* yrows, const int32_t* inv, const uint32_t* ids, int k, int E,
                           int tokens, int slots, int H, float* out, cudaStream_t stream,
                           const float* residual = nullptr, __nv_bfloat16* out16 = nullptr);

// Layer driver pieces shared by the single-GPU and expert-parallel paths.
hmoe_status validate_layer(const hmoe_layer_desc* d);
// With group = false only the router runs (the caller groups the rows).
hmoe_status enqueue_route(const hmoe_layer_desc& d, const float* x, size_t T, char* ws, const Workspace& w,
                          bool permute, cudaStream_t s, const int32_t* expert_of_slot = nullptr,
                          int32_t* slot_counts = nullptr, bool group = true);
ExpertRun local_run(const hmoe_layer_desc& d, size_t T, char* ws, const Workspace& w);
// gate/up then down of every tile of `r`; `stages` records stage events 3, 4.
hmoe_status run_experts(const ExpertRun& r, bool gemv, bool stages, cudaStream_t s);
// GEMV or tensor-core GEMM for `rows` permuted rows of an [H, I] expert.
bool use_gemv(long rows, int H, int I);

// The single-kernel decode layer (decode_layer.cu): whether the shape and
// batch qualify, its zeroed control bytes and its scratch bytes (0 when the
// shape does not qualify), and the launch (HMOE_UNSUPPORTED when this device
// cannot hold it; the caller then runs the multi-kernel layer).
bool decode_layer_shape_ok(const hmoe_layer_desc& d, size_t T);
size_t decode_layer_ctl_bytes(const hmoe_layer_desc& d, size_t T);
size_t decode_layer_data_bytes(const hmoe_layer_desc& d, size_t T);
hmoe_status launch_decode_layer(const hmoe_layer_desc& d, const float* x, const float* residual, float* y,
                                __nv_bfloat16* y16, size_t T, char* ws, const Workspace& w, cudaStream_t stream);
// Records stage event i (0..5) when stage events are registered.  Under
// stream capture the record becomes an external event node, so the caller
// can still synchronise on and time the event after each graph launch.
void stage(int i, cudaStream_t s);

} // namespace hmoe
