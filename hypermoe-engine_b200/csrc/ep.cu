// ep.cu -- expert parallelism: one process per GPU, routed experts split
// into contiguous ranges, tokens data-parallel, NCCL over NVLink/NVSwitch.
//
// Per layer call on every rank (all on the caller's stream):
//   route + group + permute   the rank's own tokens over all E experts; rows
//                             for the experts of rank p are contiguous
//   all-gather of counts      int32 [P][E] routed rows per (source, expert)
//   one host read             the counts size every transfer (NCCL p2p
//                             sizes are host values); bounded wait
//   dispatch                  grouped ncclSend/ncclRecv of FP16 rows, their
//                             scales and routing weights to the expert owners
//   expert MLP                the single-GPU kernels over the received
//                             (source, expert) segments; shared experts run
//                             locally on the rank's own rows
//   return                    grouped ncclSend/ncclRecv of the weighted BF16
//                             output rows back to their source positions
//   combine                   ascending expert id per token, as on one GPU
//
// A row's expert output depends only on the row and the expert, and the
// combine order is fixed, so for a fixed expert-MLP variant the result of
// every rank equals the single-GPU result on the concatenated batch.
//
// NCCL is opened with dlopen on first use, so libhmoe.so loads (and every
// single-GPU entry point works) on hosts without NCCL; the EP entry points
// then return HMOE_NCCL_ERROR.
//
// The reference runs one process on one device and has no multi-device
// path, so these entry points have no reference counterpart; the grouping
// and combine semantics they keep are those of MoERuntime::executeBatch
// (MoERuntime.cpp:58-349).
#include "common.cuh"
#include "layer.cuh"

#include <nccl.h> // types and enums only; the functions are resolved with dlsym

#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

namespace hmoe {
namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) getUniqueId = nullptr;
    decltype(&ncclCommInitRank) commInitRank = nullptr;
    decltype(&ncclCommDestroy) commDestroy = nullptr;
    decltype(&ncclCommAbort) commAbort = nullptr;
    decltype(&ncclCommGetAsyncError) commGetAsyncError = nullptr;
    decltype(&ncclGetErrorString) getErrorString = nullptr;
    decltype(&ncclGroupStart) groupStart = nullptr;
    decltype(&ncclGroupEnd) groupEnd = nullptr;
    decltype(&ncclSend) send = nullptr;
    decltype(&ncclRecv) recv = nullptr;
    decltype(&ncclAllGather) allGather = nullptr;
    bool ok = false;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, []() {
        const char* names[] = {getenv("HMOE_NCCL_LIBRARY"), "libnccl.so.2", "libnccl.so"};
        void* h = nullptr;
        for (const char* n : names)
            if (n && (h = dlopen(n, RTLD_NOW | RTLD_GLOBAL)) != nullptr) break;
        if (!h) return;
        auto sym = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            return fn != nullptr;
        };
        api.ok = sym(api.getUniqueId, "ncclGetUniqueId") && sym(api.commInitRank, "ncclCommInitRank") &&
                 sym(api.commDestroy, "ncclCommDestroy") && sym(api.commAbort, "ncclCommAbort") &&
                 sym(api.commGetAsyncError, "ncclCommGetAsyncError") &&
                 sym(api.getErrorString, "ncclGetErrorString") && sym(api.groupStart, "ncclGroupStart") &&
                 sym(api.groupEnd, "ncclGroupEnd") && sym(api.send, "ncclSend") && sym(api.recv, "ncclRecv") &&
                 sym(api.allGather, "ncclAllGather");
    });
    return api;
}

hmoe_status nccl_fail(const char* what, ncclResult_t r) {
    std::string msg = std::string("hmoe ") + what + ": " +
                      (nccl().getErrorString ? nccl().getErrorString(r) : "NCCL error");
    set_last_error_text(msg.c_str());
    return HMOE_NCCL_ERROR;
}

} // namespace
} // namespace hmoe

struct hmoe_ep_comm {
    ncclComm_t comm = nullptr;
    int rank = 0, size = 1, device = 0;
    int timeout_ms = 0;
    int32_t* host_counts = nullptr; // pinned [size][256]
    cudaEvent_t counts_ready = nullptr;
    bool broken = false;
    hmoe_ep_plan_t last_plan{};
    // Expert placement (slot of each expert; rank r owns a contiguous slot
    // range), or identity when placement_experts == 0.
    uint32_t placement_experts = 0;
    int32_t slot_of_expert[256] = {};
    int32_t* d_expert_of_slot = nullptr; // device [256]
};

namespace hmoe {
namespace {

constexpr int kEpMaxExperts = 256;

// Waits for the count read-back while watching the communicator; aborts it
// when a peer reports an error or the wait exceeds the communicator's
// timeout.
hmoe_status wait_counts(hmoe_ep_comm* c) {
    const auto t0 = std::chrono::steady_clock::now();
    for (int spin = 0;; ++spin) {
        const cudaError_t q = cudaEventQuery(c->counts_ready);
        if (q == cudaSuccess) return HMOE_OK;
        if (q != cudaErrorNotReady) {
            set_last_error("hmoe EP count exchange", q);
            return HMOE_CUDA_ERROR;
        }
        ncclResult_t async = ncclSuccess;
        nccl().commGetAsyncError(c->comm, &async);
        if (async != ncclSuccess && async != ncclInProgress) {
            nccl().commAbort(c->comm);
            c->comm = nullptr;
            c->broken = true;
            return nccl_fail("EP communicator", async);
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0)
                            .count();
        if (ms > c->timeout_ms) {
            nccl().commAbort(c->comm);
            c->comm = nullptr;
            c->broken = true;
            set_last_error_text("hmoe EP count exchange: timed out waiting for peers; communicator aborted");
            return HMOE_TIMEOUT;
        }
        if (spin > 64) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

// Workspace of one EP rank: the single-GPU layout for max_tokens local
// tokens (routing over all E experts, local and shared-expert rows) and the
// receive side for up to P * max_tokens * k rows.
struct EpWorkspace {
    Workspace local;
    size_t slot_counts, counts_all, xin, win, scale_in, hin, yin, tiles_in, count_in;
    int tile_cap_in;
    size_t total;
};

EpWorkspace plan_ep(const hmoe_layer_desc& d, size_t max_tokens) {
    static_assert(sizeof(__half) == 2, "FP16 rows");
    EpWorkspace w{};
    w.local = plan_workspace(d, max_tokens);
    const size_t P = static_cast<size_t>(d.ep_size);
    const size_t rin = P * max_tokens * d.top_k;
    uint32_t first = 0, count = 0;
    hmoe_ep_expert_range(d.experts, d.ep_size, d.ep_rank, &first, &count);
    size_t off = w.local.total;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align_up(off + bytes, 256);
        return at;
    };
    w.slot_counts = take(static_cast<size_t>(d.experts) * 4);
    w.counts_all = take(P * d.experts * 4);
    w.xin = take(rin * d.hidden * 2);
    w.win = take(rin * 4);
    w.scale_in = take(rin * 4);
    w.hin = take(rin * d.intermediate * 4);
    w.yin = take(rin * d.hidden * 2);
    w.count_in = take(16);
    w.tile_cap_in = tile_capacity_for(static_cast<long>(rin), static_cast<int>(P * count));
    w.tiles_in = take(static_cast<size_t>(w.tile_cap_in) * 16);
    w.total = off;
    return w;
}

hmoe_status validate_ep(const hmoe_layer_desc* d) {
    const hmoe_status v = validate_layer(d);
    if (v != HMOE_OK) return v;
    if (d->ep_size < 1 || d->ep_size > HMOE_EP_MAX_RANKS || d->ep_rank < 0 || d->ep_rank >= d->ep_size ||
        static_cast<uint32_t>(d->ep_size) > d->experts)
        return HMOE_INVALID_ARGUMENT;
    const uint32_t per = (d->experts + d->ep_size - 1) / d->ep_size;
    if (static_cast<long>(per) * d->ep_size > kMaxSegments) return HMOE_UNSUPPORTED;
    return HMOE_OK;
}

// Receive rows must index as int (tile rows, tensor-map extents).
bool ep_rows_fit(const hmoe_layer_desc& d, size_t max_tokens) {
    const double rin = static_cast<double>(d.ep_size) * static_cast<double>(max_tokens) * d.top_k;
    return rin * std::max(d.hidden, d.intermediate) < 4e18 && rin <= static_cast<double>(INT_MAX / 2);
}

} // namespace
} // namespace hmoe

using namespace hmoe;

extern "C" {

hmoe_status hmoe_ep_expert_range(uint32_t experts, int32_t ep_size, int32_t ep_rank, uint32_t* first,
                                 uint32_t* count) {
    if (!first || !count || ep_size < 1 || ep_rank < 0 || ep_rank >= ep_size || experts < static_cast<uint32_t>(ep_size))
        return HMOE_INVALID_ARGUMENT;
    const uint32_t base = experts / ep_size, extra = experts % ep_size;
    const uint32_t r = static_cast<uint32_t>(ep_rank);
    *first = r * base + std::min(r, extra);
    *count = base + (r < extra ? 1u : 0u);
    return HMOE_OK;
}

hmoe_status hmoe_ep_plan(const int32_t* counts, uint32_t experts, uint32_t top_k, int32_t ep_size,
                         int32_t ep_rank, size_t max_tokens, hmoe_ep_plan_t* plan) {
    if (!counts || !plan || top_k == 0 || ep_size > HMOE_EP_MAX_RANKS) return HMOE_INVALID_ARGUMENT;
    hmoe_ep_plan_t p{};
    hmoe_status st = hmoe_ep_expert_range(experts, ep_size, ep_rank, &p.first_expert, &p.local_experts);
    if (st != HMOE_OK) return st;
    // Every rank sees the same counts, so every check below fails or passes
    // on all ranks alike.
    for (int s = 0; s < ep_size; ++s) {
        int64_t total = 0;
        for (uint32_t e = 0; e < experts; ++e) {
            const int32_t c = counts[static_cast<size_t>(s) * experts + e];
            if (c < 0) return HMOE_INVALID_ARGUMENT;
            total += c;
        }
        if (total % top_k) return HMOE_INVALID_ARGUMENT;
        p.tokens[s] = total / top_k;
        if (static_cast<uint64_t>(p.tokens[s]) > max_tokens) return HMOE_WORKSPACE_TOO_SMALL;
    }
    const int32_t* mine = counts + static_cast<size_t>(ep_rank) * experts;
    int64_t row = 0;
    for (int q = 0; q < ep_size; ++q) {
        uint32_t f = 0, n = 0;
        hmoe_ep_expert_range(experts, ep_size, q, &f, &n);
        p.send_offset[q] = row;
        for (uint32_t e = f; e < f + n; ++e) row += mine[e];
        p.send_rows[q] = row - p.send_offset[q];
    }
    int64_t in = 0;
    for (int s = 0; s < ep_size; ++s) {
        p.recv_offset[s] = in;
        for (uint32_t e = p.first_expert; e < p.first_expert + p.local_experts; ++e)
            in += counts[static_cast<size_t>(s) * experts + e];
        p.recv_rows[s] = in - p.recv_offset[s];
    }
    p.recv_total = in;
    *plan = p;
    return HMOE_OK;
}

hmoe_status hmoe_ep_unique_id(void* id, size_t bytes) {
    if (!id || bytes < HMOE_EP_UNIQUE_ID_BYTES) return HMOE_INVALID_ARGUMENT;
    static_assert(sizeof(ncclUniqueId) == HMOE_EP_UNIQUE_ID_BYTES, "NCCL unique id size");
    if (!nccl().ok) {
        set_last_error_text("hmoe: NCCL library not found (set HMOE_NCCL_LIBRARY)");
        return HMOE_NCCL_ERROR;
    }
    ncclUniqueId u;
    const ncclResult_t r = nccl().getUniqueId(&u);
    if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
    std::memcpy(id, &u, sizeof(u));
    return HMOE_OK;
}

hmoe_status hmoe_ep_comm_create(const void* id, int32_t rank, int32_t size, int32_t timeout_ms,
                                hmoe_ep_comm** out) {
    if (!id || !out || size < 1 || size > HMOE_EP_MAX_RANKS || rank < 0 || rank >= size || timeout_ms <= 0)
        return HMOE_INVALID_ARGUMENT;
    *out = nullptr;
    if (!nccl().ok) {
        set_last_error_text("hmoe: NCCL library not found (set HMOE_NCCL_LIBRARY)");
        return HMOE_NCCL_ERROR;
    }
    auto* c = new hmoe_ep_comm();
    c->rank = rank;
    c->size = size;
    c->timeout_ms = timeout_ms;
    cudaError_t err = cudaGetDevice(&c->device);
    if (err == cudaSuccess)
        err = cudaHostAlloc(reinterpret_cast<void**>(&c->host_counts),
                            static_cast<size_t>(size) * kEpMaxExperts * sizeof(int32_t), cudaHostAllocDefault);
    if (err == cudaSuccess) err = cudaEventCreateWithFlags(&c->counts_ready, cudaEventDisableTiming);
    if (err != cudaSuccess) {
        set_last_error("hmoe EP communicator set-up", err);
        hmoe_ep_comm_destroy(c);
        return HMOE_CUDA_ERROR;
    }
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    const ncclResult_t r = nccl().commInitRank(&c->comm, size, u, rank);
    if (r != ncclSuccess) {
        c->comm = nullptr;
        hmoe_ep_comm_destroy(c);
        return nccl_fail("ncclCommInitRank", r);
    }
    *out = c;
    return HMOE_OK;
}

hmoe_status hmoe_ep_comm_destroy(hmoe_ep_comm* c) {
    if (!c) return HMOE_OK;
    hmoe_status st = HMOE_OK;
    if (c->comm) {
        const ncclResult_t r = nccl().commDestroy(c->comm);
        if (r != ncclSuccess) st = nccl_fail("ncclCommDestroy", r);
    }
    if (c->counts_ready) cudaEventDestroy(c->counts_ready);
    if (c->d_expert_of_slot) cudaFree(c->d_expert_of_slot);
    if (c->host_counts) cudaFreeHost(c->host_counts);
    delete c;
    return st;
}

hmoe_status hmoe_ep_set_placement(hmoe_ep_comm* comm, const int32_t* slot_of_expert, uint32_t experts) {
    if (!comm) return HMOE_INVALID_ARGUMENT;
    if (experts == 0 || !slot_of_expert) { // back to identity
        comm->placement_experts = 0;
        return HMOE_OK;
    }
    if (experts > 256) return HMOE_UNSUPPORTED;
    int32_t expert_of_slot[256];
    bool seen[256] = {};
    for (uint32_t e = 0; e < experts; ++e) {
        const int32_t sl = slot_of_expert[e];
        if (sl < 0 || static_cast<uint32_t>(sl) >= experts || seen[sl]) return HMOE_INVALID_ARGUMENT;
        seen[sl] = true;
        expert_of_slot[sl] = static_cast<int32_t>(e);
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device) return HMOE_INVALID_ARGUMENT;
    cudaError_t err = cudaSuccess;
    if (!comm->d_expert_of_slot) err = cudaMalloc(&comm->d_expert_of_slot, 256 * sizeof(int32_t));
    if (err == cudaSuccess)
        err = cudaMemcpy(comm->d_expert_of_slot, expert_of_slot, experts * sizeof(int32_t), cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
        set_last_error("hmoe EP placement", err);
        return HMOE_CUDA_ERROR;
    }
    std::memcpy(comm->slot_of_expert, slot_of_expert, experts * sizeof(int32_t));
    comm->placement_experts = experts;
    return HMOE_OK;
}

hmoe_status hmoe_ep_balanced_placement(const double* load, uint32_t experts, int32_t ep_size,
                                       int32_t* slot_of_expert) {
    if (!load || !slot_of_expert || ep_size < 1 || ep_size > HMOE_EP_MAX_RANKS || experts > 256 ||
        experts < static_cast<uint32_t>(ep_size))
        return HMOE_INVALID_ARGUMENT;
    // Largest expected load first (ties by expert id), each to the rank with
    // the least load so far among those with free slots (ties: lowest rank).
    int32_t order[256];
    for (uint32_t e = 0; e < experts; ++e) {
        if (!(load[e] >= 0.0)) return HMOE_INVALID_ARGUMENT;
        order[e] = static_cast<int32_t>(e);
    }
    std::stable_sort(order, order + experts, [&](int32_t a, int32_t b) { return load[a] > load[b]; });
    double rank_load[HMOE_EP_MAX_RANKS] = {};
    uint32_t filled[HMOE_EP_MAX_RANKS] = {};
    for (uint32_t i = 0; i < experts; ++i) {
        int best = -1;
        for (int r = 0; r < ep_size; ++r) {
            uint32_t first = 0, count = 0;
            hmoe_ep_expert_range(experts, ep_size, r, &first, &count);
            if (filled[r] < count && (best < 0 || rank_load[r] < rank_load[best])) best = r;
        }
        uint32_t first = 0, count = 0;
        hmoe_ep_expert_range(experts, ep_size, best, &first, &count);
        slot_of_expert[order[i]] = static_cast<int32_t>(first + filled[best]++);
        rank_load[best] += load[order[i]];
    }
    return HMOE_OK;
}

hmoe_status hmoe_ep_last_plan(const hmoe_ep_comm* comm, hmoe_ep_plan_t* plan) {
    if (!comm || !plan) return HMOE_INVALID_ARGUMENT;
    *plan = comm->last_plan;
    return HMOE_OK;
}

hmoe_status hmoe_ep_workspace_size(const hmoe_layer_desc* desc, size_t max_tokens, size_t* bytes) {
    if (!bytes) return HMOE_INVALID_ARGUMENT;
    const hmoe_status v = validate_ep(desc);
    if (v != HMOE_OK) return v;
    if (!ep_rows_fit(*desc, max_tokens)) return HMOE_UNSUPPORTED;
    *bytes = plan_ep(*desc, std::max<size_t>(max_tokens, 1)).total;
    return HMOE_OK;
}

hmoe_status hmoe_ep_moe_forward(const hmoe_layer_desc* desc, hmoe_ep_comm* comm, const float* x, float* y,
                                size_t tokens, size_t max_tokens, void* workspace, size_t workspace_bytes,
                                void* stream) {
    const hmoe_status v = validate_ep(desc);
    if (v != HMOE_OK) return v;
    if (!comm || comm->broken || !comm->comm) return HMOE_INVALID_ARGUMENT;
    if (desc->ep_size != comm->size || desc->ep_rank != comm->rank) return HMOE_INVALID_ARGUMENT;
    if (tokens > max_tokens || max_tokens == 0 || max_tokens > static_cast<size_t>(INT_MAX) / 128 ||
        !workspace || (tokens > 0 && (!x || !y)))
        return HMOE_INVALID_ARGUMENT;
    if (!ep_rows_fit(*desc, max_tokens)) return HMOE_UNSUPPORTED;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device) return HMOE_INVALID_ARGUMENT;
    const EpWorkspace w = plan_ep(*desc, max_tokens);
    if (workspace_bytes < w.total) return HMOE_WORKSPACE_TOO_SMALL;
    const NcclApi& N = nccl();
    char* ws = static_cast<char*>(workspace);
    cudaStream_t s = as_stream(stream);
    const int E = static_cast<int>(desc->experts), S = static_cast<int>(desc->shared_experts);
    const int k = static_cast<int>(desc->top_k), P = comm->size;
    const size_t H = desc->hidden;
    const int slots = k + S;

    // 1. route, group and permute this rank's tokens (T may be 0); with a
    // placement the expert groups follow slot order, so each rank's slots
    // are contiguous rows
    const bool placed = comm->placement_experts != 0;
    if (placed && comm->placement_experts != desc->experts) return HMOE_INVALID_ARGUMENT;
    auto* slot_counts = reinterpret_cast<int32_t*>(ws + w.slot_counts);
    stage(0, s);
    hmoe_status r = enqueue_route(*desc, x, tokens, ws, w.local, true, s, placed ? comm->d_expert_of_slot : nullptr,
                                  placed ? slot_counts : nullptr);
    if (r != HMOE_OK) return r;

    // 2. counts of every (source, slot), read once on the host
    auto* counts_all = reinterpret_cast<int32_t*>(ws + w.counts_all);
    ncclResult_t nr = N.allGather(placed ? static_cast<void*>(slot_counts) : static_cast<void*>(ws + w.local.counts),
                                  counts_all, static_cast<size_t>(E), ncclInt32, comm->comm, s);
    if (nr != ncclSuccess) return nccl_fail("EP count all-gather", nr);
    cudaError_t err = cudaMemcpyAsync(comm->host_counts, counts_all, static_cast<size_t>(P) * E * 4,
                                      cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaEventRecord(comm->counts_ready, s);
    if (err != cudaSuccess) {
        set_last_error("hmoe EP count read", err);
        return HMOE_CUDA_ERROR;
    }
    r = wait_counts(comm);
    if (r != HMOE_OK) return r;
    hmoe_ep_plan_t plan;
    r = hmoe_ep_plan(comm->host_counts, desc->experts, desc->top_k, P, comm->rank, max_tokens, &plan);
    if (r != HMOE_OK) return r; // identical on every rank: nobody is left waiting
    if (plan.tokens[comm->rank] != static_cast<int64_t>(tokens)) return HMOE_INVALID_ARGUMENT;
    comm->last_plan = plan;

    // 3. dispatch rows and routing weights to the expert owners
    auto* xperm = reinterpret_cast<__half*>(ws + w.local.xperm);
    auto* wperm = reinterpret_cast<float*>(ws + w.local.perm_weight);
    auto* sperm = reinterpret_cast<float*>(ws + w.local.xscale);
    auto* yrows = reinterpret_cast<__nv_bfloat16*>(ws + w.local.yrows);
    auto* xin = reinterpret_cast<__half*>(ws + w.xin);
    auto* win = reinterpret_cast<float*>(ws + w.win);
    auto* scale_in = reinterpret_cast<float*>(ws + w.scale_in);
    auto* yin = reinterpret_cast<__nv_bfloat16*>(ws + w.yin);
    N.groupStart();
    for (int q = 0; q < P && nr == ncclSuccess; ++q) {
        if (plan.send_rows[q] > 0) {
            nr = N.send(xperm + plan.send_offset[q] * H, plan.send_rows[q] * H, ncclFloat16, q, comm->comm, s);
            if (nr == ncclSuccess)
                nr = N.send(wperm + plan.send_offset[q], plan.send_rows[q], ncclFloat32, q, comm->comm, s);
            if (nr == ncclSuccess)
                nr = N.send(sperm + plan.send_offset[q], plan.send_rows[q], ncclFloat32, q, comm->comm, s);
        }
        if (plan.recv_rows[q] > 0 && nr == ncclSuccess) {
            nr = N.recv(xin + plan.recv_offset[q] * H, plan.recv_rows[q] * H, ncclFloat16, q, comm->comm, s);
            if (nr == ncclSuccess)
                nr = N.recv(win + plan.recv_offset[q], plan.recv_rows[q], ncclFloat32, q, comm->comm, s);
            if (nr == ncclSuccess)
                nr = N.recv(scale_in + plan.recv_offset[q], plan.recv_rows[q], ncclFloat32, q, comm->comm, s);
        }
    }
    const ncclResult_t ge = N.groupEnd();
    if (nr != ncclSuccess) return nccl_fail("EP dispatch", nr);
    if (ge != ncclSuccess) return nccl_fail("EP dispatch", ge);

    // 4. this rank's experts over the received (source, expert) segments
    const int Eloc = static_cast<int>(plan.local_experts);
    const int rin = static_cast<int>(plan.recv_total);
    ExpertRun run = local_run(*desc, tokens, ws, w.local);
    run.experts = Eloc + S;
    if (rin > 0) {
        ExpertRun in = run;
        in.xrows = xin;
        in.xscale = scale_in;
        in.weight = win;
        in.tiles = reinterpret_cast<int4*>(ws + w.tiles_in);
        in.tile_count = reinterpret_cast<int32_t*>(ws + w.count_in);
        in.tile_cap = tile_capacity_for(rin, P * Eloc);
        in.rows_cap = rin;
        in.hmid32 = reinterpret_cast<float*>(ws + w.hin);
        in.hmid16 = reinterpret_cast<__nv_bfloat16*>(ws + w.hin);
        in.yrows = yin;
        int max_seg = 0; // rows of the largest (source, expert) segment
        for (int q = 0; q < P; ++q)
            for (int el = 0; el < Eloc; ++el)
                max_seg = std::max(max_seg, comm->host_counts[static_cast<size_t>(q) * E + plan.first_expert + el]);
        in.max_group = max_seg;
        const SegSpec seg{nullptr, counts_all + plan.first_expert, E, P * Eloc, Eloc, 0, 0};
        r = launch_tile_list(seg, const_cast<int4*>(in.tiles), const_cast<int32_t*>(in.tile_count), in.tile_cap, s);
        if (r != HMOE_OK) return r;
        stage(2, s);
        r = run_experts(in, use_gemv(rin, in.H, in.I), true, s);
        if (r != HMOE_OK) return r;
    } else {
        stage(2, s);
        stage(3, s);
        stage(4, s);
    }
    // shared experts: local rows [T*k, T*(k+S)), arena ids Eloc..Eloc+S-1
    if (S > 0 && tokens > 0) {
        ExpertRun sh = run;
        sh.tile_cap = tile_capacity_for(static_cast<long>(tokens) * S, S);
        const SegSpec seg{reinterpret_cast<int32_t*>(ws + w.local.offsets) + E, nullptr, 0, S, S, Eloc, 0};
        r = launch_tile_list(seg, const_cast<int4*>(sh.tiles), const_cast<int32_t*>(sh.tile_count), sh.tile_cap, s);
        if (r == HMOE_OK) r = run_experts(sh, use_gemv(static_cast<long>(tokens) * S, sh.H, sh.I), false, s);
        if (r != HMOE_OK) return r;
    }

    // 5. weighted outputs back to their source rows
    N.groupStart();
    for (int q = 0; q < P && nr == ncclSuccess; ++q) {
        if (plan.recv_rows[q] > 0)
            nr = N.send(yin + plan.recv_offset[q] * H, plan.recv_rows[q] * H, ncclBfloat16, q, comm->comm, s);
        if (plan.send_rows[q] > 0 && nr == ncclSuccess)
            nr = N.recv(yrows + plan.send_offset[q] * H, plan.send_rows[q] * H, ncclBfloat16, q, comm->comm, s);
    }
    const ncclResult_t ge2 = N.groupEnd();
    if (nr != ncclSuccess) return nccl_fail("EP return", nr);
    if (ge2 != ncclSuccess) return nccl_fail("EP return", ge2);

    // 6. combine in ascending expert id
    r = launch_combine(yrows, reinterpret_cast<int32_t*>(ws + w.local.inv),
                       placed ? reinterpret_cast<uint32_t*>(ws + w.local.ids) : nullptr, k, E,
                       static_cast<int>(tokens), slots, static_cast<int>(H), y, s);
    stage(5, s);
    return r;
}

} // extern "C"
