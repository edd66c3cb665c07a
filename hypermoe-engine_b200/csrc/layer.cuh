// layer.cuh -- internal interfaces between the fused-layer kernels.
#pragma once

#include "common.cuh"

namespace hmoe {

// Byte offsets of the workspace segments (all 256-byte aligned).
struct Workspace {
    size_t status, counts, zero_bytes, offsets, list_sizes, small_list, large_list;
    size_t ids, scores, perm_token, perm_weight, inv, hmid, yrows, xperm;
    size_t hmid16, tiles, tile_count;
    size_t total;
};

Workspace plan_workspace(const hmoe_layer_desc& d, size_t T, int local_experts);

// Batches with at most this many (token, expert) assignments use the
// weight-streaming GEMV for every expert; larger ones the tcgen05 GEMM.
constexpr int kGemvMaxAssignments = 64;

// Upper bound of a token's rows (top_k routed + shared experts).
constexpr int kMaxSlots = 96;

struct GemvArgs {
    const int32_t* list;        // experts to process
    const int32_t* list_size;   // device count
    const int32_t* offsets;     // [E+S+1] first permuted row of each expert
    const uint32_t* perm_token; // gate/up: token of each permuted row
    const float* perm_weight;   // down: routing weight of each permuted row
    const float* act;           // gate/up: x [T,K]; down: hmid [R,K]
    const int8_t* arena;
    uint64_t stride, off0, off1; // expert stride; projection offsets
    const hmoe_expert_quant* quant;
    int proj0;                  // quant index of the first projection
    float* out;                 // gate/up: hmid [R,N]; down: y [R,N]
    int K, N, KS;
};

hmoe_status launch_expert_gemv(bool gate_up, const GemvArgs& args, int list_capacity, int max_tokens,
                               cudaStream_t stream);

bool gemm_available();
hmoe_status launch_expert_gemm_gate_up(const hmoe_layer_desc& d, const float* x, size_t T,
                                       char* ws, const Workspace& w, int list_capacity,
                                       cudaStream_t stream);
hmoe_status launch_expert_gemm_down(const hmoe_layer_desc& d, size_t T, char* ws,
                                    const Workspace& w, int list_capacity, cudaStream_t stream);

} // namespace hmoe
