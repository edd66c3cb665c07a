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
#include "rows.cuh"

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
    // Peer-memory path (hmoe_ep_register_workspace): every rank's registered
    // workspace mapped into this process; own entry = reg_ws.
    void* reg_ws = nullptr;
    size_t reg_bytes = 0;
    char* peer_ws[HMOE_EP_MAX_RANKS] = {};
    void* peer_base[HMOE_EP_MAX_RANKS] = {}; // IPC mappings to close
    char** d_peer_ws = nullptr;              // device copy of peer_ws
    uint64_t epoch = 0;                      // forwards since registration
    bool last_peer = false;                  // last forward took the peer path
    int last_parity = 0;
    uint32_t last_E = 0, last_k = 0;        // ... and its layer shape
    size_t last_max_tokens = 0, last_counts_off = 0;
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
// Peer-memory path: the first kEpSyncBytes of the workspace hold the epoch
// flags written by the peers ([3 kinds][HMOE_EP_MAX_RANKS] uint64: counts
// published, rows dispatched, rows returned), a CTA-completion counter, the
// sticky abort word and the device transfer plan.  Zeroed at registration,
// and only there: an abort stays set until the workspace is registered
// again.
// The device transfer plan (see hmoe_ep_peer_plan_t in hmoe.h).
using EpDevPlan = hmoe_ep_peer_plan_t;

// Rows source p sends to owner q: p's routed rows in q's slot range.
// Negative counts count as zero, as the exchange kernel reads them.
__host__ __device__ inline int ep_rows_to_owner(const int32_t* counts, int E, int P, int p, int q) {
    const int base = E / P, extra = E % P;
    const int f = q * base + (q < extra ? q : extra), n = base + (q < extra ? 1 : 0);
    int r = 0;
    for (int sl = f; sl < f + n; ++sl) r += counts[p * E + sl] > 0 ? counts[p * E + sl] : 0;
    return r;
}

// Rank me's plan from R[p * stride + q] = rows of source p for owner q.
// Rows travel source-major into every owner's receive rows (source 0's
// first), and leave a source in owner order (its rows are grouped by slot,
// slots by owner).  `ok` false: a plan that moves nothing.
__host__ __device__ inline void ep_plan_from_rows(const int* R, int stride, int P, int me, bool ok,
                                                   EpDevPlan* plan) {
    int rt = 0, st = 0;
    for (int q = 0; q < P; ++q) {
        int so = 0, db = 0, rb = 0, ro = 0;
        for (int j = 0; j < q; ++j) {
            so += R[me * stride + j];
            rb += R[j * stride + me];
        }
        for (int p = 0; p < me; ++p) db += R[p * stride + q];
        for (int j = 0; j < me; ++j) ro += R[q * stride + j];
        plan->send_off[q] = ok ? so : 0;
        plan->send_rows[q] = ok ? R[me * stride + q] : 0;
        plan->dest_base[q] = ok ? db : 0;
        plan->recv_base[q] = ok ? rb : 0;
        plan->recv_rows[q] = ok ? R[q * stride + me] : 0;
        plan->ret_off[q] = ok ? ro : 0;
        rt += R[q * stride + me];
        st += R[me * stride + q];
    }
    plan->recv_total = ok ? rt : 0;
    plan->sent_total = ok ? st : 0;
}
constexpr size_t kEpFlagsBytes = 3 * HMOE_EP_MAX_RANKS * 8;
constexpr size_t kEpCtrOff = kEpFlagsBytes;           // int32 CTA-completion counter of the dispatch
constexpr size_t kEpAbortOff = kEpFlagsBytes + 64;    // uint32 sticky abort word (any rank may set it)
constexpr size_t kEpPlanOff = kEpFlagsBytes + 256;
constexpr size_t kEpSyncBytes = kEpPlanOff + ((sizeof(EpDevPlan) + 255) / 256) * 256;

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
    // the single-GPU layout (offsets from ws + kEpSyncBytes) follows the sync area
    size_t off = kEpSyncBytes + w.local.total;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align_up(off + bytes, 256);
        return at;
    };
    w.slot_counts = take(static_cast<size_t>(d.experts) * 4);
    w.counts_all = take(2 * P * d.experts * 4); // [epoch parity][P][E]
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

// ------------------------------------------------------------ peer-memory path
//
// With a registered workspace (hmoe_ep_register_workspace) every rank's
// workspace is mapped into every process (CUDA IPC over NVLink), and the
// layer's exchanges are plain stores into the peers' memory, ordered by
// epoch flags: no host synchronisation, no NCCL.
//   ep_exchange_kernel  publish this rank's slot counts into every rank's
//                       counts (epoch-parity buffer), flag them, wait for
//                       every rank's, build the transfer plan on the device
//   ep_permute_kernel   the permutation fused with the dispatch: routed FP16
//                       rows, their scales and routing weights go straight
//                       into the owners' receive rows; the last CTA to
//                       finish flags every rank
//   the down projection the return fused into its epilogue: each output
//                       row is stored straight into its source's own
//                       permuted output rows (PushRows); the owner flags
//                       every rank once its down kernel is done, and each
//                       rank then combines its own rows locally
//   ep_wait_kernel      bounded wait for every rank's flag of this epoch
// A rank can run at most one epoch ahead of another (it needs their counts
// of the same epoch before it writes anything into their buffers), and a
// rank publishes the counts of epoch n only after its kernels of epoch
// n - 1 have run.  So receive rows are never overwritten while their owner
// computes on them, and a source's output rows of epoch n + 1 are written
// by the owners only after the source has combined epoch n (the owners need
// its epoch n + 1 counts first); the counts are double-buffered by epoch
// parity.
//
// Failure: a rank whose flag wait runs out, or whose count exchange fails,
// stores the abort word into every rank's sync area (its own included)
// before anything else it would signal.  Every wait checks the word while it
// spins and once more after its flags arrived (the flag loads acquire, so a
// peer's abort stored before its flag is seen), and fails at once when it is
// set; an aborted rank raises no further flags, moves no rows and reads no
// peer's output rows; every later forward on the workspace fails at its
// count exchange without touching the peers.  All ranks therefore report
// HMOE_TIMEOUT for the failed forward (or, for a rank that was still ahead,
// the next one), nobody computes on rows that were never sent, and epochs
// stop advancing until the ranks register the workspace again, which
// clears the word.
struct PeerCtx {
    char* const* peer; // [P] every rank's workspace base in this address space
    int P, me;
    uint64_t epoch;
    uint64_t limit_ns;
    DeviceStatus* st;
};

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint64_t* ep_flags(char* base, int kind) {
    return reinterpret_cast<uint64_t*>(base) + kind * HMOE_EP_MAX_RANKS;
}

__device__ __forceinline__ uint32_t* ep_abort_word(char* base) {
    return reinterpret_cast<uint32_t*>(base + kEpAbortOff);
}

__device__ __forceinline__ bool ep_aborted(const PeerCtx& c) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ep_abort_word(c.peer[c.me])) : "memory");
    return v != 0;
}

// Marks the failure on every rank (its own workspace included) and in this
// rank's status word.
__device__ void ep_abort_all(const PeerCtx& c) {
    for (int q = 0; q < c.P; ++q)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(ep_abort_word(c.peer[q])), "r"(1u) : "memory");
    __threadfence_system();
    device_fail(c.st, HMOE_TIMEOUT);
}

// Thread-level: every rank's flag `kind` reaches `epoch`, or false after
// limit_ns or as soon as the abort word is set (also when it was set before
// the last flag arrived).
__device__ bool wait_all_flags(const PeerCtx& c, int kind) {
    const uint64_t* f = ep_flags(c.peer[c.me], kind);
    const uint64_t t0 = now_ns();
    for (int p = 0; p < c.P; ++p)
        while (ld_acquire_sys(f + p) < c.epoch) {
            if (ep_aborted(c) || now_ns() - t0 > c.limit_ns) return false;
            __nanosleep(100);
        }
    return !ep_aborted(c);
}

__device__ void signal_all(const PeerCtx& c, int kind) {
    __threadfence_system();
    for (int q = 0; q < c.P; ++q) st_release_sys(ep_flags(c.peer[q], kind) + c.me, c.epoch);
}

// sticky: a wait of a forward (a failure aborts every rank); the flag-wait
// self-test passes false and only records the timeout.
__global__ void ep_wait_kernel(PeerCtx c, int kind, bool sticky) {
    if (threadIdx.x == 0 && !wait_all_flags(c, kind)) {
        if (sticky) ep_abort_all(c);
        else device_fail(c.st, HMOE_TIMEOUT);
    }
}

// One CTA.  counts_off: the [2][P][E] counts in every workspace;
// my_counts: this rank's routed rows per slot; cap_rows: receive rows of
// every workspace.  On a timeout or an inconsistent count the plan moves no
// rows (and the status says why).
__global__ void __launch_bounds__(256) ep_exchange_kernel(PeerCtx c, size_t counts_off, const int32_t* my_counts,
                                                          int E, int parity, int cap_rows) {
    __shared__ int R[HMOE_EP_MAX_RANKS][HMOE_EP_MAX_RANKS + 1]; // rows from p to q
    __shared__ int ok;
    const int P = c.P, me = c.me, tid = threadIdx.x;
    if (tid == 0) ok = ep_aborted(c) ? 0 : 1; // an earlier forward failed on some rank
    __syncthreads();
    for (int q = 0; q < P && ok; ++q) {
        int32_t* dst = reinterpret_cast<int32_t*>(c.peer[q] + counts_off) + (static_cast<size_t>(parity) * P + me) * E;
        for (int e = tid; e < E; e += blockDim.x) dst[e] = my_counts[e];
    }
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
        if (!ok) {
            device_fail(c.st, HMOE_TIMEOUT);
        } else {
            signal_all(c, 0);
            ok = wait_all_flags(c, 0);
            if (!ok) ep_abort_all(c);
        }
    }
    __syncthreads();
    const int32_t* cnt = reinterpret_cast<const int32_t*>(c.peer[me] + counts_off) + static_cast<size_t>(parity) * P * E;
    for (int idx = tid; idx < P * P; idx += blockDim.x) {
        const int p = idx / P, q = idx % P;
        R[p][q] = ok ? ep_rows_to_owner(cnt, E, P, p, q) : 0;
    }
    __syncthreads();
    if (tid == 0) { // every rank's receive rows fit (identical verdict on every rank)
        for (int q = 0; q < P; ++q) {
            long in = 0;
            for (int p = 0; p < P; ++p) in += R[p][q];
            if (in > cap_rows) ok = 0;
        }
        // every rank computes the same verdict, so a rejection needs no abort
        if (!ok && !ep_aborted(c)) device_fail(c.st, HMOE_INVALID_ARGUMENT);
        ep_plan_from_rows(&R[0][0], HMOE_EP_MAX_RANKS + 1, P, me, ok != 0,
                          reinterpret_cast<EpDevPlan*>(c.peer[me] + kEpPlanOff));
    }
}

// Routed rows of this rank live in the expert owners' workspaces: row
// r < routed (a routed slot; shared-expert rows stay local) belongs to the
// rank q whose send range holds it, at q's receive row
// dest_base[q] + r - send_off[q].
struct PeerRowMap {
    char* const* peer;
    int P;
    int routed;
    int send_off[HMOE_EP_MAX_RANKS], send_rows[HMOE_EP_MAX_RANKS], dest_base[HMOE_EP_MAX_RANKS];
    __device__ int owner(int r) const {
        int q = 0;
        while (q + 1 < P && r >= send_off[q] + send_rows[q]) ++q;
        return q;
    }
};

// Dispatch fused into the permutation: routed rows go straight into the
// owners' receive rows (with their scale and routing weight).
struct PeerRows {
    const PeerRowMap* map; // shared memory
    __half* xrows;         // local rows (shared experts)
    float* xscale;
    const float* weight;   // perm_weight
    size_t x_off, s_off, w_off;
    int H;
    __device__ RowDst operator()(int r) const {
        if (r >= map->routed)
            return RowDst{xrows + static_cast<size_t>(r) * H, xscale + r, nullptr, 0.0f};
        const int q = map->owner(r);
        const int d = map->dest_base[q] + r - map->send_off[q];
        char* b = map->peer[q];
        return RowDst{reinterpret_cast<__half*>(b + x_off) + static_cast<size_t>(d) * H,
                      reinterpret_cast<float*>(b + s_off) + d, reinterpret_cast<float*>(b + w_off) + d, weight[r]};
    }
};

__device__ void load_row_map(const PeerCtx& c, int routed, PeerRowMap* m) {
    const EpDevPlan* plan = reinterpret_cast<const EpDevPlan*>(c.peer[c.me] + kEpPlanOff);
    if (threadIdx.x < c.P) {
        m->send_off[threadIdx.x] = plan->send_off[threadIdx.x];
        m->send_rows[threadIdx.x] = plan->send_rows[threadIdx.x];
        m->dest_base[threadIdx.x] = plan->dest_base[threadIdx.x];
    }
    if (threadIdx.x == 0) {
        m->peer = c.peer;
        m->P = c.P;
        // rows past the plan's routed total (a failed exchange moves nothing)
        // stay local
        m->routed = min(routed, plan->sent_total);
    }
    __syncthreads();
}

// One CTA per token; the last CTA out flags the dispatch (kind 1) on every
// rank once every CTA's stores are fenced.
__global__ void __launch_bounds__(256) ep_permute_kernel(PeerCtx c, const float* __restrict__ x,
                                                         const int32_t* __restrict__ inv, int slots, int routed, int H,
                                                         __half* xrows, float* xscale, const float* weight,
                                                         size_t x_off, size_t s_off, size_t w_off) {
    __shared__ PeerRowMap map;
    load_row_map(c, routed, &map);
    permute_token(x, inv, slots, H, blockIdx.x, PeerRows{&map, xrows, xscale, weight, x_off, s_off, w_off, H});
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        int* ctr = reinterpret_cast<int*>(c.peer[c.me] + kEpCtrOff);
        if (atomicAdd(ctr, 1) == static_cast<int>(gridDim.x) - 1) {
            *ctr = 0;
            if (!ep_aborted(c)) signal_all(c, 1);
        }
    }
}

// No rows to dispatch (this rank has no tokens): flag the dispatch anyway;
// also flags the return.  An aborted rank raises no flags.
__global__ void ep_signal_kernel(PeerCtx c, int kind) {
    if (threadIdx.x == 0 && !ep_aborted(c)) signal_all(c, kind);
}

// Peer-memory forward (workspace == comm->reg_ws); the steps of
// hmoe_ep_moe_forward with the count exchange, dispatch and return done by
// the kernels above.
hmoe_status ep_forward_peer(const hmoe_layer_desc* desc, hmoe_ep_comm* comm, const float* x,
                            const float* residual, float* y, __nv_bfloat16* y16, size_t tokens,
                            size_t max_tokens, char* ws, const EpWorkspace& w, cudaStream_t s) {
    const int E = static_cast<int>(desc->experts), S = static_cast<int>(desc->shared_experts);
    const int k = static_cast<int>(desc->top_k), P = comm->size;
    const size_t H = desc->hidden;
    const int slots = k + S;
    char* wsl = ws + kEpSyncBytes; // the single-GPU layout
    const bool placed = comm->placement_experts != 0;
    if (placed && comm->placement_experts != desc->experts) return HMOE_INVALID_ARGUMENT;
    auto* slot_counts = reinterpret_cast<int32_t*>(ws + w.slot_counts);
    const uint64_t epoch = ++comm->epoch;
    const int parity = static_cast<int>(epoch & 1);
    comm->last_peer = true;
    comm->last_parity = parity;
    comm->last_E = desc->experts;
    comm->last_k = desc->top_k;
    comm->last_max_tokens = max_tokens;
    comm->last_counts_off = w.counts_all;
    auto* st = reinterpret_cast<DeviceStatus*>(wsl + w.local.status);
    // every flag wait gives up after the communicator's timeout (at most 10 s)
    const PeerCtx c{comm->d_peer_ws, P, comm->rank, epoch,
                    static_cast<uint64_t>(std::min(comm->timeout_ms, 10000)) * 1000000ull, st};
    const int rin_cap = static_cast<int>(static_cast<size_t>(P) * max_tokens * desc->top_k);

    // 1. route and group this rank's tokens
    stage(0, s);
    hmoe_status r = enqueue_route(*desc, x, tokens, wsl, w.local, false, s,
                                  placed ? comm->d_expert_of_slot : nullptr, placed ? slot_counts : nullptr);
    if (r != HMOE_OK) return r;
    // 2. counts of every (source, slot) and the transfer plan, on the device
    const int32_t* my_counts = placed ? slot_counts : reinterpret_cast<const int32_t*>(wsl + w.local.counts);
    ep_exchange_kernel<<<1, 256, 0, s>>>(c, w.counts_all, my_counts, E, parity, rin_cap);
    r = check_launch("hmoe EP count exchange");
    if (r != HMOE_OK) return r;
    // 3. permutation fused with the dispatch: routed FP16 rows, their scales
    // and routing weights straight into the owners' receive rows
    const int routed = static_cast<int>(tokens) * k;
    if (tokens > 0)
        ep_permute_kernel<<<static_cast<unsigned>(tokens), 256, 0, s>>>(
            c, x, reinterpret_cast<const int32_t*>(wsl + w.local.inv), slots, routed, static_cast<int>(H),
            reinterpret_cast<__half*>(wsl + w.local.xperm), reinterpret_cast<float*>(wsl + w.local.xscale),
            reinterpret_cast<const float*>(wsl + w.local.perm_weight), w.xin, w.scale_in, w.win);
    else
        ep_signal_kernel<<<1, 32, 0, s>>>(c, 1);
    r = check_launch("hmoe EP permute + dispatch");
    if (r != HMOE_OK) return r;
    uint32_t first = 0, Eloc_u = 0;
    hmoe_ep_expert_range(desc->experts, P, comm->rank, &first, &Eloc_u);
    const int Eloc = static_cast<int>(Eloc_u);
    ExpertRun run = local_run(*desc, tokens, wsl, w.local);
    run.experts = Eloc + S;
    ExpertRun in = run;
    in.xrows = reinterpret_cast<const __half*>(ws + w.xin);
    in.xscale = reinterpret_cast<const float*>(ws + w.scale_in);
    in.weight = reinterpret_cast<const float*>(ws + w.win);
    in.tiles = reinterpret_cast<int4*>(ws + w.tiles_in);
    in.tile_count = reinterpret_cast<int32_t*>(ws + w.count_in);
    in.tile_cap = tile_capacity_for(rin_cap, P * Eloc);
    in.rows_cap = rin_cap;
    in.hmid32 = reinterpret_cast<float*>(ws + w.hin);
    in.hmid16 = reinterpret_cast<__nv_bfloat16*>(ws + w.hin);
    in.yrows = reinterpret_cast<__nv_bfloat16*>(ws + w.yin);
    in.max_group = static_cast<int>(std::min<size_t>(static_cast<size_t>(P) * max_tokens, INT_MAX));
    // the return fused into the down projection: each output row goes
    // straight into its source's own permuted output rows
    const EpDevPlan* dplan = reinterpret_cast<const EpDevPlan*>(ws + kEpPlanOff);
    in.push = PushRows{comm->d_peer_ws, kEpSyncBytes + w.local.yrows, dplan->ret_off, dplan->recv_base,
                       reinterpret_cast<const uint32_t*>(ws + kEpAbortOff)};
    const int32_t* counts_all = reinterpret_cast<const int32_t*>(ws + w.counts_all) + static_cast<size_t>(parity) * P * E;
    const SegSpec seg{nullptr, counts_all + first, E, P * Eloc, Eloc, 0, 0};
    r = launch_tile_list(seg, const_cast<int4*>(in.tiles), const_cast<int32_t*>(in.tile_count), in.tile_cap, s);
    if (r != HMOE_OK) return r;
    if (S > 0 && tokens > 0) { // shared experts on the rank's own rows, while the rows arrive
        ExpertRun sh = run;
        sh.tile_cap = tile_capacity_for(static_cast<long>(tokens) * S, S);
        const SegSpec sseg{reinterpret_cast<int32_t*>(wsl + w.local.offsets) + E, nullptr, 0, S, S, Eloc, 0};
        r = launch_tile_list(sseg, const_cast<int4*>(sh.tiles), const_cast<int32_t*>(sh.tile_count), sh.tile_cap, s);
        if (r == HMOE_OK) r = run_experts(sh, use_gemv(static_cast<long>(tokens) * S, sh.H, sh.I), false, s);
        if (r != HMOE_OK) return r;
    }
    ep_wait_kernel<<<1, 32, 0, s>>>(c, 1, true);
    r = check_launch("hmoe EP dispatch wait");
    if (r != HMOE_OK) return r;
    stage(2, s);
    // 4. this rank's experts over the received (source, expert) segments
    r = run_experts(in, use_gemv(rin_cap, in.H, in.I), true, s);
    if (r != HMOE_OK) return r;
    // 5. every output row has been stored into its source: flag it
    ep_signal_kernel<<<1, 32, 0, s>>>(c, 2);
    r = check_launch("hmoe EP return signal");
    if (r != HMOE_OK) return r;
    ep_wait_kernel<<<1, 32, 0, s>>>(c, 2, true);
    r = check_launch("hmoe EP return wait");
    if (r != HMOE_OK) return r;
    // 6. the combine over this rank's own rows (the owners wrote the routed
    // ones), in ascending expert id
    r = launch_combine(reinterpret_cast<const __nv_bfloat16*>(wsl + w.local.yrows),
                       reinterpret_cast<const int32_t*>(wsl + w.local.inv),
                       placed ? reinterpret_cast<const uint32_t*>(wsl + w.local.ids) : nullptr, placed ? k : 0, E,
                       static_cast<int>(tokens), slots, static_cast<int>(H), y, s, residual, y16);

    stage(5, s);
    return r;
}

// Base address and size of the allocation holding p (driver entry point).
bool allocation_range(const void* p, char** base, size_t* size) {
    using Fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static Fn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<Fn>(f);
    });
    if (!fn) return false;
    CUdeviceptr b = 0;
    size_t n = 0;
    if (fn(&b, &n, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) return false;
    *base = reinterpret_cast<char*>(b);
    *size = n;
    return true;
}

void unregister_peers(hmoe_ep_comm* c) {
    for (int q = 0; q < HMOE_EP_MAX_RANKS; ++q) {
        if (c->peer_base[q]) cudaIpcCloseMemHandle(c->peer_base[q]);
        c->peer_base[q] = nullptr;
        c->peer_ws[q] = nullptr;
    }
    if (c->d_peer_ws) cudaFree(c->d_peer_ws);
    c->d_peer_ws = nullptr;
    c->reg_ws = nullptr;
    c->reg_bytes = 0;
    c->epoch = 0;
    c->last_peer = false;
}

struct PeerEntry {
    cudaIpcMemHandle_t handle;
    uint64_t offset, bytes;
};

// All-gather of one fixed-size record per rank through NCCL (blocking).
hmoe_status allgather_host(hmoe_ep_comm* c, const void* mine, void* all, size_t bytes) {
    void* d = nullptr;
    cudaStream_t s = nullptr;
    cudaError_t err = cudaMalloc(&d, bytes * (c->size + 1));
    if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (err == cudaSuccess) err = cudaMemcpy(d, mine, bytes, cudaMemcpyHostToDevice);
    hmoe_status r = HMOE_OK;
    if (err == cudaSuccess) {
        const ncclResult_t nr = nccl().allGather(d, static_cast<char*>(d) + bytes, bytes, ncclChar, c->comm, s);
        if (nr != ncclSuccess) r = nccl_fail("EP registration all-gather", nr);
        err = cudaStreamSynchronize(s);
    }
    if (err == cudaSuccess && r == HMOE_OK)
        err = cudaMemcpy(all, static_cast<char*>(d) + bytes, bytes * c->size, cudaMemcpyDeviceToHost);
    if (s) cudaStreamDestroy(s);
    if (d) cudaFree(d);
    if (err != cudaSuccess && r == HMOE_OK) {
        set_last_error("hmoe EP registration", err);
        r = HMOE_CUDA_ERROR;
    }
    return r;
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
    unregister_peers(c);
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
    if (!comm->last_peer) {
        *plan = comm->last_plan;
        return HMOE_OK;
    }
    // peer path: the plan lives on the device; rebuild it from the
    // exchanged counts (waits for the device)
    const size_t n = static_cast<size_t>(comm->size) * comm->last_E;
    int32_t counts[HMOE_EP_MAX_RANKS * kEpMaxExperts];
    cudaError_t err = cudaDeviceSynchronize();
    if (err == cudaSuccess)
        err = cudaMemcpy(counts, static_cast<const char*>(comm->reg_ws) + comm->last_counts_off +
                                     static_cast<size_t>(comm->last_parity) * n * 4,
                         n * 4, cudaMemcpyDeviceToHost);
    if (err != cudaSuccess) {
        set_last_error("hmoe EP last plan", err);
        return HMOE_CUDA_ERROR;
    }
    return hmoe_ep_plan(counts, comm->last_E, comm->last_k, comm->size, comm->rank, comm->last_max_tokens, plan);
}

hmoe_status hmoe_ep_register_workspace(hmoe_ep_comm* comm, void* workspace, size_t bytes) {
    if (!comm || comm->broken || !comm->comm) return HMOE_INVALID_ARGUMENT;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device) return HMOE_INVALID_ARGUMENT;
    if (workspace && (bytes < kEpSyncBytes || reinterpret_cast<uintptr_t>(workspace) % 256)) return HMOE_INVALID_ARGUMENT;
    // Every rank's earlier work is done before any rank touches the flags.
    cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess) {
        set_last_error("hmoe EP registration", err);
        return HMOE_CUDA_ERROR;
    }
    unregister_peers(comm);
    PeerEntry mine{};
    int ok = 1;
    if (workspace) {
        char* base = nullptr;
        size_t n = 0;
        ok = allocation_range(workspace, &base, &n) &&
             cudaIpcGetMemHandle(&mine.handle, base) == cudaSuccess &&
             cudaMemset(workspace, 0, kEpSyncBytes) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
        mine.offset = static_cast<uint64_t>(static_cast<char*>(workspace) - base);
        mine.bytes = ok ? bytes : 0;
    }
    PeerEntry all[HMOE_EP_MAX_RANKS];
    hmoe_status r = allgather_host(comm, &mine, all, sizeof(PeerEntry));
    if (r != HMOE_OK) return r;
    if (!workspace) return HMOE_OK; // collective unregistration
    // Every rank registers the same size (same layer and max_tokens), or
    // none uses the peer path.
    for (int q = 0; q < comm->size; ++q)
        if (all[q].bytes != bytes) {
            set_last_error_text("hmoe EP registration: the ranks' workspaces differ or one failed to export");
            return HMOE_UNSUPPORTED;
        }
    hmoe_status res = HMOE_OK;
    for (int q = 0; q < comm->size && res == HMOE_OK; ++q) {
        if (q == comm->rank) {
            comm->peer_ws[q] = static_cast<char*>(workspace);
            continue;
        }
        void* p = nullptr;
        err = cudaIpcOpenMemHandle(&p, all[q].handle, cudaIpcMemLazyEnablePeerAccess);
        if (err != cudaSuccess) {
            set_last_error("hmoe EP registration: cudaIpcOpenMemHandle", err);
            res = HMOE_UNSUPPORTED;
            break;
        }
        comm->peer_base[q] = p;
        comm->peer_ws[q] = static_cast<char*>(p) + all[q].offset;
    }
    if (res == HMOE_OK) {
        err = cudaMalloc(&comm->d_peer_ws, sizeof(char*) * comm->size);
        if (err == cudaSuccess)
            err = cudaMemcpy(comm->d_peer_ws, comm->peer_ws, sizeof(char*) * comm->size, cudaMemcpyHostToDevice);
        if (err != cudaSuccess) {
            set_last_error("hmoe EP registration", err);
            res = HMOE_CUDA_ERROR;
        }
    }
    // Every rank learns whether every other rank mapped all peers.
    int32_t flag = res == HMOE_OK ? 1 : 0, flags[HMOE_EP_MAX_RANKS];
    r = allgather_host(comm, &flag, flags, sizeof(flag));
    if (r != HMOE_OK) res = r;
    for (int q = 0; q < comm->size && res == HMOE_OK; ++q)
        if (!flags[q]) {
            set_last_error_text("hmoe EP registration: a peer could not map every workspace");
            res = HMOE_UNSUPPORTED;
        }
    if (res != HMOE_OK) {
        unregister_peers(comm);
        return res;
    }
    comm->reg_ws = workspace;
    comm->reg_bytes = bytes;
    comm->epoch = 0;
    return HMOE_OK;
}

hmoe_status hmoe_ep_peer_plan(const int32_t* slot_counts, uint32_t experts, int32_t ep_size, int32_t ep_rank,
                              int64_t capacity_rows, hmoe_ep_peer_plan_t* plan) {
    if (!slot_counts || !plan || experts == 0 || ep_size < 1 || ep_size > HMOE_EP_MAX_RANKS || ep_rank < 0 ||
        ep_rank >= ep_size || capacity_rows < 0)
        return HMOE_INVALID_ARGUMENT;
    static int R[HMOE_EP_MAX_RANKS * HMOE_EP_MAX_RANKS];
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    const int P = ep_size, E = static_cast<int>(experts);
    for (int p = 0; p < P; ++p)
        for (int q = 0; q < P; ++q) R[p * P + q] = ep_rows_to_owner(slot_counts, E, P, p, q);
    bool ok = true;
    for (int q = 0; q < P; ++q) {
        long long in = 0;
        for (int p = 0; p < P; ++p) in += R[p * P + q];
        if (in > capacity_rows) ok = false;
    }
    std::memset(plan, 0, sizeof(*plan));
    ep_plan_from_rows(R, P, P, ep_rank, ok, plan);
    return ok ? HMOE_OK : HMOE_INVALID_ARGUMENT;
}

hmoe_status hmoe_ep_read_status(void* workspace, int32_t* status, int32_t* near_ties, int32_t* sequential_logits,
                                void* stream) {
    if (!workspace) return HMOE_INVALID_ARGUMENT;
    return hmoe_read_status(static_cast<char*>(workspace) + kEpSyncBytes, status, near_ties, sequential_logits,
                            stream);
}

hmoe_status hmoe_ep_selftest_flag_wait(hmoe_ep_comm* comm, uint64_t limit_ns, int32_t* status) {
    if (!comm || !status || !comm->reg_ws) return HMOE_INVALID_ARGUMENT;
    // waits for an epoch no rank will reach: the bounded wait must give up
    auto* st = reinterpret_cast<DeviceStatus*>(static_cast<char*>(comm->reg_ws) + kEpPlanOff + sizeof(EpDevPlan));
    static_assert(kEpPlanOff + sizeof(EpDevPlan) + sizeof(DeviceStatus) <= kEpSyncBytes, "self-test status slot");
    cudaError_t err = cudaMemset(st, 0, sizeof(DeviceStatus));
    const PeerCtx c{comm->d_peer_ws, comm->size, comm->rank, comm->epoch + (1ull << 40), limit_ns, st};
    if (err == cudaSuccess) {
        ep_wait_kernel<<<1, 32>>>(c, 1, false);
        err = cudaGetLastError();
    }
    DeviceStatus host{};
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    if (err == cudaSuccess) err = cudaMemcpy(&host, st, sizeof(host), cudaMemcpyDeviceToHost);
    if (err != cudaSuccess) {
        set_last_error("hmoe EP flag-wait self-test", err);
        return HMOE_CUDA_ERROR;
    }
    *status = host.status;
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

// Both expert-parallel entry points; residual and y16 as in
// hmoe_moe_forward_residual (both may be null).
static hmoe_status ep_forward(const hmoe_layer_desc* desc, hmoe_ep_comm* comm, const float* x,
                              const float* residual, float* y, __nv_bfloat16* y16, size_t tokens,
                              size_t max_tokens, void* workspace, size_t workspace_bytes, void* stream) {
    const hmoe_status v = validate_ep(desc);
    if (v != HMOE_OK) return v;
    if (!comm || comm->broken || !comm->comm) return HMOE_INVALID_ARGUMENT;
    if (desc->ep_size != comm->size || desc->ep_rank != comm->rank) return HMOE_INVALID_ARGUMENT;
    if (tokens > max_tokens || max_tokens == 0 || max_tokens > static_cast<size_t>(INT_MAX) / 128 ||
        !workspace || (tokens > 0 && (!x || !y)))
        return HMOE_INVALID_ARGUMENT;
    if (!aligned(workspace, 16) ||
        (tokens > 0 && (!aligned(x, 16) || !aligned(y, 16) || !aligned(residual, 16) || !aligned(y16, 16))))
        return HMOE_INVALID_ARGUMENT;
    if (!ep_rows_fit(*desc, max_tokens)) return HMOE_UNSUPPORTED;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device) return HMOE_INVALID_ARGUMENT;
    const EpWorkspace w = plan_ep(*desc, max_tokens);
    if (workspace_bytes < w.total) return HMOE_WORKSPACE_TOO_SMALL;
    if (comm->reg_ws && workspace == comm->reg_ws)
        return ep_forward_peer(desc, comm, x, residual, y, y16, tokens, max_tokens, static_cast<char*>(workspace),
                               w, as_stream(stream));
    comm->last_peer = false;
    const NcclApi& N = nccl();
    char* ws = static_cast<char*>(workspace);
    char* wsl = ws + kEpSyncBytes; // the single-GPU layout
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
    hmoe_status r = enqueue_route(*desc, x, tokens, wsl, w.local, true, s, placed ? comm->d_expert_of_slot : nullptr,
                                  placed ? slot_counts : nullptr);
    if (r != HMOE_OK) return r;

    // 2. counts of every (source, slot), read once on the host
    auto* counts_all = reinterpret_cast<int32_t*>(ws + w.counts_all);
    ncclResult_t nr = N.allGather(placed ? static_cast<void*>(slot_counts) : static_cast<void*>(wsl + w.local.counts),
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
    auto* xperm = reinterpret_cast<__half*>(wsl + w.local.xperm);
    auto* wperm = reinterpret_cast<float*>(wsl + w.local.perm_weight);
    auto* sperm = reinterpret_cast<float*>(wsl + w.local.xscale);
    auto* yrows = reinterpret_cast<__nv_bfloat16*>(wsl + w.local.yrows);
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
    ExpertRun run = local_run(*desc, tokens, wsl, w.local);
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
        const SegSpec seg{reinterpret_cast<int32_t*>(wsl + w.local.offsets) + E, nullptr, 0, S, S, Eloc, 0};
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
    r = launch_combine(yrows, reinterpret_cast<int32_t*>(wsl + w.local.inv),
                       placed ? reinterpret_cast<uint32_t*>(wsl + w.local.ids) : nullptr, k, E,
                       static_cast<int>(tokens), slots, static_cast<int>(H), y, s, residual, y16);
    stage(5, s);
    return r;
}

hmoe_status hmoe_ep_moe_forward(const hmoe_layer_desc* desc, hmoe_ep_comm* comm, const float* x, float* y,
                                size_t tokens, size_t max_tokens, void* workspace, size_t workspace_bytes,
                                void* stream) {
    return ep_forward(desc, comm, x, nullptr, y, nullptr, tokens, max_tokens, workspace, workspace_bytes, stream);
}

hmoe_status hmoe_ep_moe_forward_residual(const hmoe_layer_desc* desc, hmoe_ep_comm* comm, const float* x,
                                         const float* residual, float* y, uint16_t* y_bf16, size_t tokens,
                                         size_t max_tokens, void* workspace, size_t workspace_bytes,
                                         void* stream) {
    return ep_forward(desc, comm, x, residual, y, reinterpret_cast<__nv_bfloat16*>(y_bf16), tokens, max_tokens,
                      workspace, workspace_bytes, stream);
}

} // extern "C"
