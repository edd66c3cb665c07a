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
//   group_kernel     offsets, permutation, inverse map, GEMV/GEMM lists
//   gate/up          GEMV for small groups, tcgen05 GEMM for large groups
//   down             same split, routing weight folded into the epilogue
//   combine_kernel   out[t] = sum of the token's rows in ascending expert id
//
// No host synchronisation, no allocation.  The combine order (ascending
// expert id, starting from zero, `out += w*y`) is the reference's
// (MoERuntime.cpp:311-325), so the result does not depend on how experts
// were split between kernels, launches or GPUs.
#include "common.cuh"
#include "layer.cuh"

#include <algorithm>
#include <climits>

namespace hmoe {

hmoe_status launch_route(const float* x, const float* w, const float* bias, int T, int H, int E,
                         int k, int softmax, int renorm, uint32_t* ids, float* scores,
                         int32_t* counts, DeviceStatus* st, cudaStream_t stream);
hmoe_status launch_group(const uint32_t* ids, const float* scores, const int32_t* counts, int T,
                         int k, int E, int S, int small_max, int32_t* offsets,
                         uint32_t* perm_token, float* perm_weight, int32_t* inv,
                         int32_t* small_list, int32_t* large_list, int32_t* list_sizes,
                         cudaStream_t stream);

int g_variant = 0;
cudaEvent_t g_stage_events[6];
int g_stage_count = 0;

// Records stage event i.  Under stream capture the record becomes an
// external event node, so the caller can still synchronise on and time the
// event after each graph launch.
inline void stage(int i, cudaStream_t s) {
    if (g_stage_count != 6) return;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(s, &cs);
    if (cs == cudaStreamCaptureStatusActive)
        cudaEventRecordWithFlags(g_stage_events[i], s, cudaEventRecordExternal);
    else
        cudaEventRecord(g_stage_events[i], s);
}

Workspace plan_workspace(const hmoe_layer_desc& d, size_t T, int local_experts) {
    Workspace w{};
    const size_t E = d.experts, S = d.shared_experts, k = d.top_k;
    const size_t slots = k + S;
    const size_t R = T * slots; // upper bound of permuted rows on this device
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align_up(off + bytes, 256);
        return at;
    };
    w.status = take(sizeof(DeviceStatus));
    w.counts = take((E + S) * 4); // zeroed together with status
    w.zero_bytes = off;
    w.offsets = take((E + S + 1) * 4);
    w.list_sizes = take(2 * 4);
    w.small_list = take((E + S) * 4);
    w.large_list = take((E + S) * 4);
    w.ids = take(T * k * 4);
    w.scores = take(T * k * 4);
    w.perm_token = take(R * 4);
    w.perm_weight = take(R * 4);
    w.inv = take(T * slots * 4);
    w.hmid = take(R * static_cast<size_t>(d.intermediate) * 4);
    w.yrows = take(R * static_cast<size_t>(d.hidden) * 4);
    w.xperm = take(R * static_cast<size_t>(d.hidden) * 2);
    w.hmid16 = take(R * static_cast<size_t>(d.intermediate) * 2);
    w.tile_count = take(16);
    w.tiles = take((R / 128 + E + S + 2) * 16);
    w.total = off;
    (void)local_experts;
    return w;
}

hmoe_status validate_desc(const hmoe_layer_desc* d) {
    if (!d) return HMOE_INVALID_ARGUMENT;
    if (d->hidden == 0 || d->intermediate == 0 || d->experts == 0 || d->top_k == 0 ||
        d->top_k > d->experts || !d->router_weight || !d->arena || !d->quant)
        return HMOE_INVALID_ARGUMENT; // RouterConfig::validate, RouterConfig.cpp:9-22
    if (d->hidden % 64 || d->intermediate % 64) return HMOE_UNSUPPORTED;
    if (d->expert_stride % 16 || d->gate_offset % 16 || d->up_offset % 16 || d->down_offset % 16)
        return HMOE_INVALID_ARGUMENT;
    if (d->experts > 256 || d->top_k > 32 || d->shared_experts > 64 ||
        d->top_k + d->shared_experts > static_cast<uint32_t>(kMaxSlots))
        return HMOE_UNSUPPORTED;
    if (d->ep_size != 1 || d->ep_rank != 0) return HMOE_UNSUPPORTED; // see hmoe_ep_*
    return HMOE_OK;
}

// ------------------------------------------------------------- combine

// One CTA per token: gather the token's rows (routed slots, then shared),
// order them ascending (rows are laid out in ascending expert id, so row
// order is expert order) and accumulate in that order from zero.
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ yrows,
                                                      const int32_t* __restrict__ inv, int slots,
                                                      int H, float* __restrict__ out) {
    __shared__ int rows_s[kMaxSlots];
    const int t = blockIdx.x;
    if (threadIdx.x == 0) {
        int n = 0;
        for (int s = 0; s < slots; ++s) {
            const int r = inv[static_cast<size_t>(t) * slots + s];
            int j = n++;
            while (j > 0 && rows_s[j - 1] > r) {
                rows_s[j] = rows_s[j - 1];
                --j;
            }
            rows_s[j] = r;
        }
    }
    __syncthreads();
    const int H4 = H / 4;
    for (int c = threadIdx.x; c < H4; c += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < slots; ++s) {
            const float4 v = reinterpret_cast<const float4*>(yrows + static_cast<size_t>(rows_s[s]) * H)[c];
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        reinterpret_cast<float4*>(out + static_cast<size_t>(t) * H)[c] = acc;
    }
}

// ------------------------------------------------------- layer driver

hmoe_status enqueue_route(const hmoe_layer_desc& d, const float* x, size_t T, char* ws,
                          const Workspace& w, int small_max, cudaStream_t s) {
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
                                 reinterpret_cast<int32_t*>(ws + w.counts), st, s);
    if (r != HMOE_OK) return r;
    stage(1, s);
    r = launch_group(reinterpret_cast<uint32_t*>(ws + w.ids), reinterpret_cast<float*>(ws + w.scores),
                        reinterpret_cast<int32_t*>(ws + w.counts), static_cast<int>(T),
                        static_cast<int>(d.top_k), static_cast<int>(d.experts),
                        static_cast<int>(d.shared_experts), small_max,
                        reinterpret_cast<int32_t*>(ws + w.offsets),
                        reinterpret_cast<uint32_t*>(ws + w.perm_token),
                        reinterpret_cast<float*>(ws + w.perm_weight),
                        reinterpret_cast<int32_t*>(ws + w.inv),
                        reinterpret_cast<int32_t*>(ws + w.small_list),
                        reinterpret_cast<int32_t*>(ws + w.large_list),
                        reinterpret_cast<int32_t*>(ws + w.list_sizes), s);
    stage(2, s);
    return r;
}

int choose_split(int capacity, int col_blocks) {
    int ks = 1;
    while (ks < 8 && static_cast<long>(capacity) * col_blocks * ks < 2L * 148) ks *= 2;
    return ks;
}

hmoe_status enqueue_experts(const hmoe_layer_desc& d, const float* x, size_t T, char* ws,
                            const Workspace& w, int small_max, cudaStream_t s) {
    const int E = static_cast<int>(d.experts), S = static_cast<int>(d.shared_experts);
    const int H = static_cast<int>(d.hidden), I = static_cast<int>(d.intermediate);
    const long assignments = static_cast<long>(T) * d.top_k;
    // Worst-case list sizes: experts that can hold >= 1 (GEMV) or > small_max
    // (GEMM) tokens.
    const int shared_small = (static_cast<long>(T) <= small_max) ? S : 0;
    const int small_cap = small_max <= 0 ? 0 : static_cast<int>(std::min<long>(E, assignments)) + shared_small;
    const int large_cap = static_cast<int>(std::min<long>(E, assignments / (small_max + 1))) + (S - shared_small);
    // Largest possible group: T tokens (a shared expert, or one routed expert
    // taking every token).
    const int max_group = static_cast<int>(T);
    GemvArgs g{};
    g.list = reinterpret_cast<int32_t*>(ws + w.small_list);
    g.list_size = reinterpret_cast<int32_t*>(ws + w.list_sizes);
    g.offsets = reinterpret_cast<int32_t*>(ws + w.offsets);
    g.perm_token = reinterpret_cast<uint32_t*>(ws + w.perm_token);
    g.perm_weight = reinterpret_cast<float*>(ws + w.perm_weight);
    g.arena = d.arena;
    g.stride = d.expert_stride;
    g.quant = d.quant;
    hmoe_status r;
    // gate/up
    if (small_cap > 0) {
        g.act = x;
        g.off0 = d.gate_offset;
        g.off1 = d.up_offset;
        g.proj0 = 0;
        g.out = reinterpret_cast<float*>(ws + w.hmid);
        g.K = H;
        g.N = I;
        g.KS = choose_split(small_cap, (I + 255) / 256);
        r = launch_expert_gemv(true, g, small_cap, max_group, s);
        if (r != HMOE_OK) return r;
    }
    if (large_cap > 0) {
        r = launch_expert_gemm_gate_up(d, x, T, ws, w, large_cap, s);
        if (r != HMOE_OK) return r;
    }
    stage(3, s);
    // down
    if (small_cap > 0) {
        g.act = reinterpret_cast<float*>(ws + w.hmid);
        g.off0 = d.down_offset;
        g.off1 = 0;
        g.proj0 = 2;
        g.out = reinterpret_cast<float*>(ws + w.yrows);
        g.K = I;
        g.N = H;
        g.KS = choose_split(small_cap, (H + 255) / 256);
        r = launch_expert_gemv(false, g, small_cap, max_group, s);
        if (r != HMOE_OK) return r;
    }
    if (large_cap > 0) {
        r = launch_expert_gemm_down(d, T, ws, w, large_cap, s);
        if (r != HMOE_OK) return r;
    }
    stage(4, s);
    return HMOE_OK;
}

// Experts with at most this many tokens take the GEMV.  The choice is made
// per launch from the batch size alone (the host never reads the routing):
// decode-sized batches stream every touched expert through the GEMV, larger
// ones run every expert on the tensor-core GEMM.
int small_threshold(size_t T, const hmoe_layer_desc& d) {
    if (g_variant == 1 || !gemm_available()) return INT_MAX / 2;
    if (g_variant == 2) return 0;
    const size_t assignments = T * (d.top_k + d.shared_experts);
    return assignments <= static_cast<size_t>(kGemvMaxAssignments) ? INT_MAX / 2 : 0;
}

} // namespace hmoe

using namespace hmoe;

extern "C" {

hmoe_status hmoe_set_variant(int32_t variant) {
    if (variant < 0 || variant > 2) return HMOE_INVALID_ARGUMENT;
    if (variant == 2 && !gemm_available()) return HMOE_UNSUPPORTED;
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
    *bytes = plan_workspace(*desc, T, static_cast<int>(desc->experts)).total;
    if (host_io) *bytes += 2 * align_up(T * desc->hidden * sizeof(float), 256);
    return HMOE_OK;
}

hmoe_status hmoe_route(const hmoe_layer_desc* desc, const float* x, size_t tokens, uint32_t* ids,
                       float* scores, int32_t* offsets, uint32_t* group_tokens, float* group_scores,
                       void* workspace, size_t workspace_bytes, void* stream) {
    const hmoe_status v = validate_desc(desc);
    if (v != HMOE_OK) return v;
    if (tokens == 0) return HMOE_OK;
    if (!x || !workspace || tokens > static_cast<size_t>(INT_MAX) / 64) return HMOE_INVALID_ARGUMENT;
    const Workspace w = plan_workspace(*desc, tokens, static_cast<int>(desc->experts));
    if (workspace_bytes < w.total) return HMOE_WORKSPACE_TOO_SMALL;
    char* ws = static_cast<char*>(workspace);
    cudaStream_t s = as_stream(stream);
    hmoe_status r = enqueue_route(*desc, x, tokens, ws, w, small_threshold(tokens, *desc), s);
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

hmoe_status hmoe_moe_forward(const hmoe_layer_desc* desc, const float* x, float* y, size_t tokens,
                             void* workspace, size_t workspace_bytes, void* stream) {
    const hmoe_status v = validate_desc(desc);
    if (v != HMOE_OK) return v;
    if (tokens == 0) return HMOE_OK;
    if (!x || !y || !workspace || tokens > static_cast<size_t>(INT_MAX) / 64) return HMOE_INVALID_ARGUMENT;
    const Workspace w = plan_workspace(*desc, tokens, static_cast<int>(desc->experts));
    if (workspace_bytes < w.total) return HMOE_WORKSPACE_TOO_SMALL;
    char* ws = static_cast<char*>(workspace);
    cudaStream_t s = as_stream(stream);
    const int small_max = small_threshold(tokens, *desc);
    stage(0, s);
    hmoe_status r = enqueue_route(*desc, x, tokens, ws, w, small_max, s);
    if (r != HMOE_OK) return r;
    r = enqueue_experts(*desc, x, tokens, ws, w, small_max, s);
    if (r != HMOE_OK) return r;
    const int slots = static_cast<int>(desc->top_k + desc->shared_experts);
    combine_kernel<<<static_cast<unsigned>(tokens), 256, 0, s>>>(
        reinterpret_cast<float*>(ws + w.yrows), reinterpret_cast<int32_t*>(ws + w.inv), slots,
        static_cast<int>(desc->hidden), y);
    r = check_launch("hmoe combine kernel");
    stage(5, s);
    return r;
}

hmoe_status hmoe_moe_forward_host(const hmoe_layer_desc* desc, const float* x_host, float* y_host,
                                  size_t tokens, void* workspace, size_t workspace_bytes, void* stream) {
    const hmoe_status v = validate_desc(desc);
    if (v != HMOE_OK) return v;
    if (tokens == 0) return HMOE_OK;
    if (!x_host || !y_host || !workspace || tokens > static_cast<size_t>(INT_MAX) / 64)
        return HMOE_INVALID_ARGUMENT;
    const Workspace w = plan_workspace(*desc, tokens, static_cast<int>(desc->experts));
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
