// layer.cu -- the fused MoE layer: workspace layout, hmoe_route,
// hmoe_moe_forward and the deterministic combine.
//
// Replaces the per-expert host loop of MoERuntime::executeBatch
// (src/core/runtime/MoERuntime.cpp:58-349) for a layer whose experts are all
// resident: instead of one host-driven gather / 3 projections / activation /
// multiply / scatter sequence per expert with a host synchronisation after
// each gather and scatter (CudaTensorBackend.cpp:741, :781), the whole layer
// is a fixed sequence of stream-ordered launches whose grids cover the
// worst case and read the expert lists the router built on the device:
//
//   memset(status, counts)                          (one cudaMemsetAsync)
//   route_kernel     logits, softmax, top-k, renorm, expert histogram
//   group_kernel     offsets, permutation, inverse map
//   permute_kernel   each token row once -> FP16 copies (power-of-two scaled);
//                    one more CTA builds the (expert, first row, rows) tiles
//   gate/up          tcgen05 GEMM (or the weight-streaming GEMV for
//                    decode-sized batches), SwiGLU in the epilogue
//   down             same variant, routing weight in the epilogue, BF16 rows
//   combine_kernel   out[t] = sum of the token's rows in ascending expert id
//
// No host synchronisation, no allocation.  The combine order (ascending
// expert id, starting from zero, `out += w*y`) is the reference's
// (MoERuntime.cpp:311-325), so the result does not depend on how experts
// were split between kernels, launches or GPUs.
#include "common.cuh"
#include "layer.cuh"
#include "rows.cuh"

#include <algorithm>
#include <climits>

namespace hmoe {

int g_variant = 0;
constexpr int kDecodeLayerAutoTokens = 2; // single-kernel decode layer chosen automatically up to here (faster at T <= 2)
extern int g_route_variant; // router.cu
cudaEvent_t g_stage_events[6];
int g_stage_count = 0;

void stage(int i, cudaStream_t s) {
    if (g_stage_count != 6) return;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(s, &cs);
    if (cs == cudaStreamCaptureStatusActive)
        cudaEventRecordWithFlags(g_stage_events[i], s, cudaEventRecordExternal);
    else
        cudaEventRecord(g_stage_events[i], s);
}

Workspace plan_workspace(const hmoe_layer_desc& d, size_t T) {
    Workspace w{};
    const size_t E = d.experts, S = d.shared_experts, k = d.top_k;
    const size_t slots = k + S;
    const size_t R = T * slots; // permuted rows of this batch (exact)
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align_up(off + bytes, 256);
        return at;
    };
    w.status = take(sizeof(DeviceStatus));
    // zeroed together with status: routed counts, then per token block
    w.counts = take((E + S) * 4);
    w.block_counts = take(((T + kGroupBlock - 1) / kGroupBlock) * E * 4);
    w.route_acc_bytes = route_decode_scratch_bytes(T, static_cast<int>(d.hidden), static_cast<int>(E));
    w.route_acc = take(w.route_acc_bytes); // decode router partials (zeroed)
    w.dl_ctl_bytes = decode_layer_ctl_bytes(d, T);
    w.dl_ctl = take(w.dl_ctl_bytes); // decode layer barriers and counters (zeroed)
    w.zero_bytes = off;
    w.offsets = take((E + S + 1) * 4);
    w.ids = take(T * k * 4);
    w.scores = take(T * k * 4);
    w.perm_token = take(R * 4);
    w.perm_weight = take(R * 4);
    w.inv = take(R * 4);
    w.xperm = take(R * static_cast<size_t>(d.hidden) * 2);
    w.xscale = take(R * 4);
    w.hmid = take(R * static_cast<size_t>(d.intermediate) * 4);
    w.yrows = take(R * static_cast<size_t>(d.hidden) * 2);
    w.tile_count = take(16);
    w.tile_cap = tile_capacity_for(static_cast<long>(R), static_cast<int>(E + S));
    w.tiles = take(static_cast<size_t>(w.tile_cap) * 16);
    w.dl_data_bytes = decode_layer_data_bytes(d, T);
    w.dl_data = take(w.dl_data_bytes);
    w.total = off;
    return w;
}

// Checks shared by the single-GPU and expert-parallel entry points.
hmoe_status validate_layer(const hmoe_layer_desc* d) {
    if (!d) return HMOE_INVALID_ARGUMENT;
    if (d->hidden == 0 || d->intermediate == 0 || d->experts == 0 || d->top_k == 0 ||
        d->top_k > d->experts || !d->router_weight || !d->arena || !d->quant)
        return HMOE_INVALID_ARGUMENT; // RouterConfig::validate, RouterConfig.cpp:9-22
    if (d->hidden % 64 || d->intermediate % 64) return HMOE_UNSUPPORTED;
    if (d->expert_stride % 16 || d->gate_offset % 16 || d->up_offset % 16 || d->down_offset % 16)
        return HMOE_INVALID_ARGUMENT;
    if (!aligned(d->router_weight, 16) || !aligned(d->arena, 16) || !aligned(d->quant, 4) ||
        !aligned(d->router_bias, 4))
        return HMOE_INVALID_ARGUMENT;
    if (d->experts > 256 || d->top_k > 32 || d->shared_experts > 64 ||
        d->top_k + d->shared_experts > static_cast<uint32_t>(kMaxSlots))
        return HMOE_UNSUPPORTED;
    return HMOE_OK;
}

hmoe_status validate_desc(const hmoe_layer_desc* d) {
    const hmoe_status v = validate_layer(d);
    if (v != HMOE_OK) return v;
    if (d->ep_size != 1 || d->ep_rank != 0) return HMOE_UNSUPPORTED; // hmoe_ep_moe_forward
    return HMOE_OK;
}

// ------------------------------------------------------------- combine

// One CTA per token (combine_token) over this GPU's rows.
struct LocalOut {
    const __nv_bfloat16* yrows;
    int H;
    __device__ const __nv_bfloat16* operator()(int r) const { return yrows + static_cast<size_t>(r) * H; }
};

__global__ void __launch_bounds__(256) combine_kernel(const __nv_bfloat16* __restrict__ yrows,
                                                      const int32_t* __restrict__ inv,
                                                      const uint32_t* __restrict__ ids, int k, int E, int slots,
                                                      int H, float* out, const float* residual,
                                                      __nv_bfloat16* __restrict__ out16) {
    combine_token(inv, ids, k, E, slots, H, blockIdx.x, out, LocalOut{yrows, H}, residual, out16);
}

hmoe_status launch_combine(const __nv_bfloat16* yrows, const int32_t* inv, const uint32_t* ids, int k, int E,
                           int tokens, int slots, int H, float* out, cudaStream_t s, const float* residual,
                           __nv_bfloat16* out16) {
    if (tokens <= 0) return HMOE_OK;
    combine_kernel<<<static_cast<unsigned>(tokens), 256, 0, s>>>(yrows, inv, ids, k, E, slots, H, out, residual,
                                                                 out16);
    return check_launch("hmoe combine kernel");
}

// ------------------------------------------------------- layer driver

// Router, histogram, grouping and the BF16 row permutation of one batch.
hmoe_status enqueue_route(const hmoe_layer_desc& d, const float* x, size_t T, char* ws, const Workspace& w,
                          bool permute, cudaStream_t s, const int32_t* expert_of_slot, int32_t* slot_counts,
                          bool group) {
    cudaError_t err = cudaMemsetAsync(ws, 0, w.zero_bytes, s);
    if (err != cudaSuccess) {
        set_last_error("hmoe workspace reset", err);
        return HMOE_CUDA_ERROR;
    }
    auto* st = reinterpret_cast<DeviceStatus*>(ws + w.status);
    hmoe_status r = launch_route(x, d.router_weight, d.router_bias, static_cast<int>(T),
                                 static_cast<int>(d.hidden), static_cast<int>(d.experts),
                                 static_cast<int>(d.top_k), d.softmax, d.renormalize,
                                 reinterpret_cast<uint32_t*>(ws + w.ids),
                                 reinterpret_cast<float*>(ws + w.scores),
                                 reinterpret_cast<int32_t*>(ws + w.counts),
                                 reinterpret_cast<int32_t*>(ws + w.block_counts),
                                 w.route_acc_bytes ? reinterpret_cast<double*>(ws + w.route_acc) : nullptr, st, s);
    if (r != HMOE_OK) return r;
    stage(1, s);
    if (!group) return HMOE_OK;
    r = launch_group(reinterpret_cast<uint32_t*>(ws + w.ids), reinterpret_cast<float*>(ws + w.scores),
                     reinterpret_cast<int32_t*>(ws + w.counts), reinterpret_cast<int32_t*>(ws + w.block_counts),
                     static_cast<int>(T), static_cast<int>(d.top_k),
                     static_cast<int>(d.experts), static_cast<int>(d.shared_experts),
                     reinterpret_cast<int32_t*>(ws + w.offsets), reinterpret_cast<uint32_t*>(ws + w.perm_token),
                     reinterpret_cast<float*>(ws + w.perm_weight), reinterpret_cast<int32_t*>(ws + w.inv),
                     expert_of_slot, slot_counts, s);
    if (r != HMOE_OK || !permute) return r;
    return launch_permute(x, reinterpret_cast<int32_t*>(ws + w.inv), static_cast<int>(T),
                          static_cast<int>(d.top_k + d.shared_experts), static_cast<int>(d.hidden),
                          reinterpret_cast<__half*>(ws + w.xperm), reinterpret_cast<float*>(ws + w.xscale), s);
}

// gate/up then down of every tile of `r` with the chosen variant.
hmoe_status run_experts(const ExpertRun& r, bool gemv, bool stages, cudaStream_t s) {
    hmoe_status st = gemv ? gemv_gate_up(r, s) : gemm_gate_up(r, s);
    if (st != HMOE_OK) return st;
    if (stages) stage(3, s);
    st = gemv ? gemv_down(r, s) : gemm_down(r, s);
    if (stages) stage(4, s);
    return st;
}

// The GEMV streams each touched expert's weights once per 4 rows; the
// tensor-core GEMM wins as soon as a launch holds more than one token's rows.
// The choice is made per launch from the number of permuted rows, which the
// host knows without reading the routing.
bool use_gemv(long rows, int H, int I) {
    if (g_variant == 1 || !gemm_available() || !gemm_shape_ok(H, I)) return true;
    if (g_variant == 2 || g_variant == 4) return false;
    return rows <= kGemvMaxAssignments;
}

ExpertRun local_run(const hmoe_layer_desc& d, size_t T, char* ws, const Workspace& w) {
    ExpertRun r{};
    r.xrows = reinterpret_cast<__half*>(ws + w.xperm);
    r.xscale = reinterpret_cast<float*>(ws + w.xscale);
    r.weight = reinterpret_cast<float*>(ws + w.perm_weight);
    r.tiles = reinterpret_cast<int4*>(ws + w.tiles);
    r.tile_count = reinterpret_cast<int32_t*>(ws + w.tile_count);
    r.tile_cap = w.tile_cap;
    r.rows_cap = static_cast<int>(T * (d.top_k + d.shared_experts));
    r.hmid32 = reinterpret_cast<float*>(ws + w.hmid);
    r.hmid16 = reinterpret_cast<__nv_bfloat16*>(ws + w.hmid);
    r.yrows = reinterpret_cast<__nv_bfloat16*>(ws + w.yrows);
    r.arena = d.arena;
    r.stride = d.expert_stride;
    r.gate_offset = d.gate_offset;
    r.up_offset = d.up_offset;
    r.down_offset = d.down_offset;
    r.quant = d.quant;
    r.experts = static_cast<int>(d.experts + d.shared_experts);
    r.H = static_cast<int>(d.hidden);
    r.I = static_cast<int>(d.intermediate);
    r.max_group = static_cast<int>(T);
    r.st = reinterpret_cast<DeviceStatus*>(ws + w.status);
    return r;
}

} // namespace hmoe

using namespace hmoe;

extern "C" {

hmoe_status hmoe_set_variant(int32_t variant) {
    if (variant < 0 || variant > 4) return HMOE_INVALID_ARGUMENT;
    if ((variant == 2 || variant == 4) && !gemm_available()) return HMOE_UNSUPPORTED;
    g_variant = variant;
    return HMOE_OK;
}

hmoe_status hmoe_set_stage_events(void* const* events, int32_t count) {
    if (count == 0) {
        g_stage_count = 0;
        return HMOE_OK;
    }
    if (count != 6 || !events) return HMOE_INVALID_ARGUMENT;
    for (int i = 0; i < 6; ++i) g_stage_events[i] = static_cast<cudaEvent_t>(events[i]);
    g_stage_count = 6;
    return HMOE_OK;
}

hmoe_status hmoe_workspace_size(const hmoe_layer_desc* desc, size_t max_tokens, size_t* bytes) {
    if (!bytes) return HMOE_INVALID_ARGUMENT;
    const hmoe_status v = validate_desc(desc);
    if (v != HMOE_OK) return v;
    const bool host_io = (max_tokens & HMOE_WORKSPACE_HOST_IO) != 0;
    const size_t T = std::max<size_t>(max_tokens & ~HMOE_WORKSPACE_HOST_IO, 1);
    *bytes = plan_workspace(*desc, T).total;
    if (host_io) *bytes += 2 * align_up(T * desc->hidden * sizeof(float), 256);
    return HMOE_OK;
}

hmoe_status hmoe_route(const hmoe_layer_desc* desc, const float* x, size_t tokens, uint32_t* ids,
                       float* scores, int32_t* offsets, uint32_t* group_tokens, float* group_scores,
                       void* workspace, size_t workspace_bytes, void* stream) {
    const hmoe_status v = validate_desc(desc);
    if (v != HMOE_OK) return v;
    if (tokens == 0) return HMOE_OK;
    if (!x || !workspace || tokens > static_cast<size_t>(INT_MAX) / 128) return HMOE_INVALID_ARGUMENT;
    if (!aligned(x, 16) || !aligned(workspace, 16)) return HMOE_INVALID_ARGUMENT;
    const Workspace w = plan_workspace(*desc, tokens);
    if (workspace_bytes < w.total) return HMOE_WORKSPACE_TOO_SMALL;
    char* ws = static_cast<char*>(workspace);
    cudaStream_t s = as_stream(stream);
    hmoe_status r = enqueue_route(*desc, x, tokens, ws, w, false, s);
    if (r != HMOE_OK) return r;
    const size_t tk = tokens * desc->top_k;
    auto copy = [&](void* dst, size_t src_off, size_t bytes) {
        if (!dst) return cudaSuccess;
        return cudaMemcpyAsync(dst, ws + src_off, bytes, cudaMemcpyDeviceToDevice, s);
    };
    cudaError_t err = cudaSuccess;
    if (err == cudaSuccess) err = copy(ids, w.ids, tk * 4);
    if (err == cudaSuccess) err = copy(scores, w.scores, tk * 4);
    if (err == cudaSuccess) err = copy(offsets, w.offsets, (desc->experts + 1) * 4);
    if (err == cudaSuccess) err = copy(group_tokens, w.perm_token, tk * 4);
    if (err == cudaSuccess) err = copy(group_scores, w.perm_weight, tk * 4);
    if (err != cudaSuccess) {
        set_last_error("hmoe route outputs", err);
        return HMOE_CUDA_ERROR;
    }
    return HMOE_OK;
}

} // extern "C"

namespace hmoe {

// The fused layer; residual and y16 are optional (see
// hmoe_moe_forward_residual).
hmoe_status forward_layer(const hmoe_layer_desc* desc, const float* x, const float* residual, float* y,
                          __nv_bfloat16* y16, size_t tokens, void* workspace, size_t workspace_bytes,
                          void* stream) {
    const hmoe_status v = validate_desc(desc);
    if (v != HMOE_OK) return v;
    if (tokens == 0) return HMOE_OK;
    if (!x || !y || !workspace || tokens > static_cast<size_t>(INT_MAX) / 128) return HMOE_INVALID_ARGUMENT;
    if (!aligned(x, 16) || !aligned(y, 16) || !aligned(residual, 16) || !aligned(y16, 16) ||
        !aligned(workspace, 16))
        return HMOE_INVALID_ARGUMENT;
    const Workspace w = plan_workspace(*desc, tokens);
    if (workspace_bytes < w.total) return HMOE_WORKSPACE_TOO_SMALL;
    char* ws = static_cast<char*>(workspace);
    cudaStream_t s = as_stream(stream);
    const int E = static_cast<int>(desc->experts), S = static_cast<int>(desc->shared_experts);
    const int slots = static_cast<int>(desc->top_k) + S;
    stage(0, s);
    // Decode-sized batches: the whole layer in one kernel (the GEMV
    // variant's arithmetic), unless a variant or a router kernel is forced.
    // Automatic up to kDecodeLayerAutoTokens, where it is measured faster.
    const bool dl_forced = g_variant == 3;
    if (dl_forced || (g_variant == 0 && (g_route_variant == 0 || g_route_variant == 3) &&
                      tokens <= static_cast<size_t>(kDecodeLayerAutoTokens) && decode_layer_shape_ok(*desc, tokens))) {
        cudaError_t err = cudaMemsetAsync(ws, 0, w.zero_bytes, s);
        if (err != cudaSuccess) {
            set_last_error("hmoe workspace reset", err);
            return HMOE_CUDA_ERROR;
        }
        const hmoe_status r = launch_decode_layer(*desc, x, residual, y, y16, tokens, ws, w, s);
        if (r == HMOE_OK || dl_forced || r != HMOE_UNSUPPORTED) {
            for (int i = 1; i < 6; ++i) stage(i, s);
            if (dl_forced && r == HMOE_UNSUPPORTED)
                set_last_error_text("hmoe: the decode layer kernel does not take this shape or batch");
            return r;
        }
    }
    // Batches of one group block: the grouping joins the permutation's
    // launch (one launch less on the decode-sized path).
    const bool small = tokens <= static_cast<size_t>(kGroupBlock) && E + S <= 2 * kGroupBlock;
    hmoe_status r = enqueue_route(*desc, x, tokens, ws, w, false, s, nullptr, nullptr, !small);
    if (r != HMOE_OK) return r;
    const ExpertRun run = local_run(*desc, tokens, ws, w);
    // the permutation's launch also builds the tile list (one more CTA)
    const SegSpec seg{reinterpret_cast<int32_t*>(ws + w.offsets), nullptr, 0, E + S, E + S, 0, 0};
    if (small) {
        const SmallGroup g{reinterpret_cast<const uint32_t*>(ws + w.ids), reinterpret_cast<const float*>(ws + w.scores),
                           reinterpret_cast<const int32_t*>(ws + w.counts), static_cast<int>(tokens),
                           static_cast<int>(desc->top_k), E, S, reinterpret_cast<int32_t*>(ws + w.offsets),
                           reinterpret_cast<uint32_t*>(ws + w.perm_token), reinterpret_cast<float*>(ws + w.perm_weight),
                           reinterpret_cast<int32_t*>(ws + w.inv)};
        r = launch_group_permute(g, x, static_cast<int>(desc->hidden), reinterpret_cast<__half*>(ws + w.xperm),
                                 reinterpret_cast<float*>(ws + w.xscale), seg, const_cast<int4*>(run.tiles),
                                 const_cast<int32_t*>(run.tile_count), run.tile_cap, s);
    } else {
        r = launch_permute(x, reinterpret_cast<int32_t*>(ws + w.inv), static_cast<int>(tokens), slots,
                           static_cast<int>(desc->hidden), reinterpret_cast<__half*>(ws + w.xperm),
                           reinterpret_cast<float*>(ws + w.xscale), s, &seg, const_cast<int4*>(run.tiles),
                           const_cast<int32_t*>(run.tile_count), run.tile_cap);
    }
    if (r != HMOE_OK) return r;
    stage(2, s);
    r = run_experts(run, use_gemv(static_cast<long>(tokens) * slots, run.H, run.I), true, s);
    if (r != HMOE_OK) return r;
    r = launch_combine(run.yrows, reinterpret_cast<int32_t*>(ws + w.inv), nullptr, 0, E, static_cast<int>(tokens),
                       slots, static_cast<int>(desc->hidden), y, s, residual, y16);
    stage(5, s);
    return r;
}

} // namespace hmoe

extern "C" {

hmoe_status hmoe_moe_forward(const hmoe_layer_desc* desc, const float* x, float* y, size_t tokens,
                             void* workspace, size_t workspace_bytes, void* stream) {
    return forward_layer(desc, x, nullptr, y, nullptr, tokens, workspace, workspace_bytes, stream);
}

hmoe_status hmoe_moe_forward_residual(const hmoe_layer_desc* desc, const float* x, const float* residual,
                                      float* y, uint16_t* y_bf16, size_t tokens, void* workspace,
                                      size_t workspace_bytes, void* stream) {
    return forward_layer(desc, x, residual, y, reinterpret_cast<__nv_bfloat16*>(y_bf16), tokens, workspace,
                         workspace_bytes, stream);
}

hmoe_status hmoe_moe_forward_host(const hmoe_layer_desc* desc, const float* x_host, float* y_host,
                                  size_t tokens, void* workspace, size_t workspace_bytes, void* stream) {
    const hmoe_status v = validate_desc(desc);
    if (v != HMOE_OK) return v;
    if (tokens == 0) return HMOE_OK;
    if (!x_host || !y_host || !workspace || tokens > static_cast<size_t>(INT_MAX) / 128)
        return HMOE_INVALID_ARGUMENT;
    if (!aligned(workspace, 16)) return HMOE_INVALID_ARGUMENT;
    const Workspace w = plan_workspace(*desc, tokens);
    const size_t io = align_up(tokens * desc->hidden * sizeof(float), 256);
    if (workspace_bytes < w.total + 2 * io) return HMOE_WORKSPACE_TOO_SMALL;
    char* ws = static_cast<char*>(workspace);
    float* dx = reinterpret_cast<float*>(ws + w.total);
    float* dy = reinterpret_cast<float*>(ws + w.total + io);
    cudaStream_t s = as_stream(stream);
    const size_t bytes = tokens * desc->hidden * sizeof(float);
    cudaError_t err = cudaMemcpyAsync(dx, x_host, bytes, cudaMemcpyHostToDevice, s);
    if (err != cudaSuccess) {
        set_last_error("hmoe host input copy", err);
        return HMOE_CUDA_ERROR;
    }
    const hmoe_status r = hmoe_moe_forward(desc, dx, dy, tokens, workspace, w.total, stream);
    if (r != HMOE_OK) return r;
    err = cudaMemcpyAsync(y_host, dy, bytes, cudaMemcpyDeviceToHost, s);
    if (err != cudaSuccess) {
        set_last_error("hmoe host output copy", err);
        return HMOE_CUDA_ERROR;
    }
    return HMOE_OK;
}

hmoe_status hmoe_read_status(void* workspace, int32_t* status, int32_t* near_ties,
                             int32_t* sequential_logits, void* stream) {
    if (!workspace) return HMOE_INVALID_ARGUMENT;
    DeviceStatus host{};
    cudaStream_t s = as_stream(stream);
    cudaError_t err = cudaMemcpyAsync(&host, workspace, sizeof(host), cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err == cudaSuccess) err = cudaMemsetAsync(workspace, 0, sizeof(DeviceStatus), s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) {
        set_last_error("hmoe read status", err);
        return HMOE_CUDA_ERROR;
    }
    if (status) *status = host.status;
    if (near_ties) *near_ties = host.near_ties;
    if (sequential_logits) *sequential_logits = host.sequential_logits;
    return HMOE_OK;
}

} // extern "C"
