// decode_layer.cu -- the whole MoE layer for decode-sized batches in one
// persistent kernel.
//
// At a handful of tokens the multi-kernel layer (router, grouping,
// permutation, tile list, GEMV gate/up, GEMV down, combine) is bound by
// latency: every launch pays its ramp, its cold misses and its drain, while
// the weights it streams are only tens of MB.  Here one cooperative launch
// of one CTA per SM runs the same arithmetic in five phases separated by
// three grid barriers (bounded waits, with a shared abort word):
//
//   A  router partial sums over (128 hidden rows x 32 experts) items, FP64,
//      added into zeroed sums with atomics (the order varies, but every
//      logit is a sum of exact products with a bounded chain of roundings,
//      which the certificate covers); the token scales of the FP16 token
//      rows (as the permutation computes them)
//   B  every CTA, redundantly and identically: the decode router's
//      certification, settling and selection,
//      and the grouping by (expert, token), all in shared memory (no
//      barrier, no global round trip); then L2 prefetches of this CTA's
//      down-projection boxes
//   C  gate/up: (row, projection, K rank) items.  A rank's rows of one
//      projection are contiguous in the packed layout, so an item streams
//      whole-row chunks of up to 32 KB with 1D bulk copies through one ring
//      of ~190 KB per CTA (TMA tensor boxes are row-rate bound on this path:
//      a 256-byte row per box row reaches about half the per-SM rate of a
//      32 KB bulk copy), and stores its rank's partial sums (no atomics).  A
//      row is one (expert, token): an expert with several tokens is streamed
//      once per token, mostly from L2
//   D  down: (row, K rank, column part) items; the item first forms its
//      SwiGLU values from the gate/up rank partials (ranks added in order),
//      then streams its chunks through the same ring, which kept issuing
//      them ahead while C finished; stores rank partials
//   E  combine: per token and column, each routed row's down ranks added
//      in order, weighted and rounded to BF16, the rows added in ascending
//      expert id from zero (plus the residual)
//
// The arithmetic, including every summation order, is the weight-streaming
// GEMV variant's (expert_gemv.cu: row groups rr = g mod 4 within 32-row
// boxes, groups added in order, K ranks added in order from zero, the same
// split of K) and the combine's (rows.cuh), and the router is certified
// exactly as the decode router, so the output equals that variant's bit for
// bit.
#include "common.cuh"
#include "layer.cuh"
#include "route_core.cuh"
#include "sm100.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

namespace hmoe {

namespace {

constexpr int kDlThreads = 256;
constexpr int kDlMaxTokens = 8;  // tokens per call
constexpr int kDlMaxRows = 64;   // T x (k + S)
constexpr int kDlMaxSlots = 16;  // k + S
constexpr int kDlMaxStages = 8;  // ring stages at most
constexpr int kDlStage = 32768;  // bytes per ring stage: whole rows of one projection
constexpr int kDlPartCols = 1024; // columns an item accumulates
constexpr int kDlCw = kDlThreads / 32 - 1; // consumer warps in phases C, D, E; the last warp issues the copies
constexpr int kDlCt = 32 * kDlCw;
constexpr int kDlDynLimit = 232448 - 5120;  // dynamic shared memory (the static arrays take the rest)
constexpr int kDlPrefetchBytes = 768 * 1024; // weight bytes per CTA prefetched into L2 (148 x 768 KB < L2)
constexpr uint64_t kDlWaitNs = 2000000000ull;

// Zeroed control words of one call.
struct DlCtl {
    unsigned bar[4]; // grid barriers
    int abort;       // set by the first CTA that fails; every wait gives up on it
    int pad[11];
};
static_assert(sizeof(DlCtl) == 64, "control header is 64 bytes");

struct DlArgs {
    RouteArgs ra;      // x, router W and bias, T, H, E, k, ...; ids/scores in the workspace
    const float* residual;
    float* y;
    __nv_bfloat16* y16;
    const hmoe_expert_quant* quant;
    int slots, I;
    int KS, kc;        // gate/up: K ranks, rows per rank (multiple of 32)
    int KSd, kcd;      // down: the same
    const int8_t* arena; // expert blobs: gate [H][I] | up [H][I] | down [I][H] at the offsets
    uint64_t stride, gate_off, up_off, down_off;
    int nstage;        // ring stages
    DlCtl* ctl;
    double* racc;      // [T][E] router sums (zeroed)
    double* rwn;       // [E] squared router-column norms (zeroed)
    double* rxn;       // [T] squared token norms (zeroed)
    float* tscale;     // [2][T] s_t, 1/s_t
    float* pgu;        // [KS][R][2I] gate/up rank partials (gate | up)
    float* pdn;        // [KSd][R][H] down rank partials
};

// Shared-memory plan (byte offsets from a 128-byte aligned base).  Phase A
// and phase B work from offset 0 (B may reach into the ring, which is not in
// use yet); C, D and E keep their scratch below `ring`.
struct DlSmem {
    int a_xs, a_red, a_wred, a_end;
    int b_logit, b_evs, b_wn, b_xn, b_bias, b_fb, b_stage, b_grp, b_q, b_end;
    int c_xs, red, d_hs, e_v;
    int ring, bars, total;
};

__host__ __device__ inline int dl_al(int v) { return (v + 127) & ~127; }

__host__ __device__ inline DlSmem dl_smem(int T, int H, int E, int kc, int kcd, int R, int S) {
    DlSmem m{};
    m.a_xs = 0;
    m.a_red = dl_al(m.a_xs + T * kDecRows * 4);
    m.a_wred = dl_al(m.a_red + 8 * T * 32 * 8);
    m.a_end = dl_al(m.a_wred + 8 * 32 * 8);
    m.b_logit = 0;
    m.b_evs = dl_al(m.b_logit + T * E * 4);
    m.b_wn = dl_al(m.b_evs + 8 * kMaxExperts * 4);
    m.b_xn = dl_al(m.b_wn + E * 8);
    m.b_bias = dl_al(m.b_xn + T * 8);
    m.b_fb = dl_al(m.b_bias + E * 4);
    m.b_stage = dl_al(m.b_fb + (1 + kRouteFallbacks) * 4);
    m.b_grp = dl_al(m.b_stage + kDecSlots * staged_logit_doubles(H) * 8);
    m.b_q = dl_al(m.b_grp + 3 * R * 4);
    m.b_end = dl_al(m.b_q + (E + kDlMaxSlots) * 6 * 4);
    // C: token rows of this rank; D: the item's SwiGLU values; C and D: the
    // row classes' partial sums of one item; E: the slot values of one
    // 32-column unit
    m.c_xs = 0;
    m.d_hs = dl_al(m.c_xs + T * kc * 4);
    m.red = dl_al(m.d_hs + kcd * 4);
    m.e_v = dl_al(m.red + kDlPartCols * 4);
    int r = dl_al(m.e_v + kDlMaxSlots * 32 * 4);
    r = r > m.a_end ? r : m.a_end;
    m.ring = dl_al(r);
    m.bars = dl_al(m.ring + S * kDlStage);
    m.total = m.bars + 2 * S * 8 + 128; // full and empty barriers; room to align the base
    return m;
}

__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier `i`: every CTA arrives once; false once the call is aborted.
// The wait is bounded and gives up as soon as another CTA sets the abort
// word.
__device__ bool dl_grid_sync(const DlArgs& d, int i, int& abort_s) {
    __syncthreads();
    if (threadIdx.x == 0 && !abort_s) {
        __threadfence();
        atomicAdd(&d.ctl->bar[i], 1u);
        const uint64_t t0 = sm100::global_timer_ns();
        for (;;) {
            if (ld_acquire(reinterpret_cast<const int*>(&d.ctl->bar[i])) >= static_cast<int>(gridDim.x)) break;
            if (ld_acquire(&d.ctl->abort)) break;
            if (sm100::global_timer_ns() - t0 > kDlWaitNs) {
                device_fail(d.ra.st, HMOE_TIMEOUT);
                atomicExch(&d.ctl->abort, 1);
                break;
            }
            __nanosleep(100);
        }
        if (ld_acquire(&d.ctl->abort)) abort_s = 1; // some CTA failed
        __threadfence();
    }
    __syncthreads();
    return !abort_s;
}

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kDlCt) : "memory"); }

// dl_grid_sync for the consumer warps only (phases C to E, while the
// producer warp may still be issuing copies).
__device__ bool dl_grid_sync_consumers(const DlArgs& d, int i, int& abort_s) {
    consumers_sync();
    if (threadIdx.x == 0 && !abort_s) {
        __threadfence();
        atomicAdd(&d.ctl->bar[i], 1u);
        const uint64_t t0 = sm100::global_timer_ns();
        for (;;) {
            if (ld_acquire(reinterpret_cast<const int*>(&d.ctl->bar[i])) >= static_cast<int>(gridDim.x)) break;
            if (ld_acquire(&d.ctl->abort)) break;
            if (sm100::global_timer_ns() - t0 > kDlWaitNs) {
                device_fail(d.ra.st, HMOE_TIMEOUT);
                atomicExch(&d.ctl->abort, 1);
                break;
            }
            __nanosleep(100);
        }
        if (ld_acquire(&d.ctl->abort)) abort_s = 1;
        __threadfence();
    }
    consumers_sync();
    return !abort_s;
}

// Ring wait: false after a timeout (recorded) or once the abort word is set.
// Threads poll the barrier in shared memory; the abort word and the clock, which live in global memory, are
// read only every 64 polls, so a grid of waiting threads does not flood one
// L2 line.
__device__ __forceinline__ bool dl_wait(const DlArgs& d, uint64_t* bar, uint32_t parity) {
    if (sm100::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = sm100::global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (sm100::mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*reinterpret_cast<const volatile int*>(&d.ctl->abort)) return false;
            if (sm100::global_timer_ns() - t0 > kDlWaitNs) {
                device_fail(d.ra.st, HMOE_TIMEOUT);
                atomicExch(&d.ctl->abort, 1);
                return false;
            }
        }
    }
}

// The k experts a token's router sums rank highest (logit descending, id
// ascending), by one warp, without certification or softmax: the exact
// selection orders by the same key (the softmax is monotone) and differs
// only where the certificate settles a logit across a float boundary.  Used
// only to prefetch weights; NaN sums rank lowest.
template <int C>
__device__ void guess_topk(const double* sums, const float* bias, int E, int k, uint32_t* out) {
    const int lane = threadIdx.x & 31;
    uint32_t key[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int j = lane + 32 * c;
        float v = -FLT_MAX * 2.0f;
        if (j < E) {
            v = static_cast<float>(__ldcg(sums + j) + (bias ? static_cast<double>(bias[j]) : 0.0));
            if (v != v) v = -FLT_MAX * 2.0f;
        }
        uint32_t u = __float_as_uint(v + 0.0f);
        key[c] = j < E ? ((u & 0x80000000u) ? ~u : (u | 0x80000000u)) : 0u;
    }
    unsigned taken = 0;
    for (int r = 0; r < k; ++r) {
        uint32_t bk = 0, bi = 0xffffffffu;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const uint32_t j = lane + 32 * c;
            if (j < static_cast<uint32_t>(E) && !((taken >> c) & 1u) && (key[c] > bk || (key[c] == bk && j < bi))) {
                bk = key[c];
                bi = j;
            }
        }
        const uint32_t kmax = __reduce_max_sync(0xffffffffu, bk);
        const uint32_t imin = __reduce_min_sync(0xffffffffu, bk == kmax ? bi : 0xffffffffu);
        if (imin == 0xffffffffu) break;
        if (static_cast<int>(imin & 31u) == lane) taken |= 1u << (imin >> 5);
        if (lane == 0) out[r] = imin;
    }
}

// L2 prefetch of a contiguous range (no shared memory, no completion to wait for).
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

} // namespace

namespace {

template <int C>
__global__ void __launch_bounds__(kDlThreads, 1) decode_layer_kernel(const __grid_constant__ DlArgs d) {
    extern __shared__ __align__(128) unsigned char dsm[];
    __shared__ int abort_s, nseg_s;
    __shared__ int4 seg_s[kDlMaxRows];     // segment: (expert, first row, rows, 0)
    __shared__ float qs_s[kDlMaxRows][3];  // segment: scales (gate, up, down)
    __shared__ float qz_s[kDlMaxRows][3];  // segment: 2^23 + 128 + zero point (dequantisation offsets)
    __shared__ int rtok_s[kDlMaxRows];     // row: token
    __shared__ float rw_s[kDlMaxRows];     // row: routing weight (1 for shared experts)
    __shared__ float rsc_s[kDlMaxRows];    // row: down scale of its expert
    __shared__ int trow_s[kDlMaxRows];     // [T][slots] the token's rows, ascending
    __shared__ int rseg_s[kDlMaxRows];     // row: its segment
    __shared__ uint32_t ids_s[kDlMaxRows]; // [T][k] selected experts
    __shared__ float scores_s[kDlMaxRows]; // [T][k] their scores
    __shared__ float tsc_s[2 * kDlMaxTokens];
    __shared__ float red_s[8];
    const RouteArgs& a = d.ra;
    const int T = a.T, H = a.H, E = a.E, I = d.I, k = a.k, slots = d.slots;
    const int R = T * slots;
    const int G = static_cast<int>(gridDim.x), b = static_cast<int>(blockIdx.x);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = d.nstage;
    const DlSmem L = dl_smem(T, H, E, d.kc, d.kcd, R, S);
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 127) & ~uintptr_t(127));
    uint8_t* ring = base + L.ring;
    uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bars);
    if (tid == 0) {
        abort_s = 0;
        for (int s = 0; s < S; ++s) {
            sm100::mbar_init(&full[s], 1);          // the producer's expect_tx (or plain) arrival
            sm100::mbar_init(&full[S + s], kDlCw);  // empty: one arrival per consumer warp
        }
        sm100::fence_mbarrier_init();
    }
    __syncthreads();

    // ------------------------------------------------ A: router partial sums
    const int nRC = H / kDecRows, nEC = (E + kDecCols - 1) / kDecCols, nRI = nRC * nEC;
    {
        float* xs0 = reinterpret_cast<float*>(base + L.a_xs);       // [T][128]
        double* red0 = reinterpret_cast<double*>(base + L.a_red);   // [8][T][32]
        double* wred0 = reinterpret_cast<double*>(base + L.a_wred); // [8][32]
        for (int it = b; it < nRI; it += G) {
            const int rc = it / nEC, ec = it % nEC;
            const int r0 = rc * kDecRows, e0 = ec * kDecCols;
            const int e = e0 + lane;
            // this warp's 16 router rows, all loads in flight at once
            double wv[kDecRows / 8];
#pragma unroll
            for (int j = 0; j < kDecRows / 8; ++j)
                wv[j] = e < E ? static_cast<double>(a.w[static_cast<size_t>(r0 + warp * (kDecRows / 8) + j) * E + e])
                              : 0.0;
            __syncthreads(); // the previous item's shared memory is free
            for (int i = tid; i < T * kDecRows; i += kDlThreads)
                xs0[i] = a.x[static_cast<size_t>(i / kDecRows) * H + r0 + i % kDecRows];
            __syncthreads();
            double acc[kDlMaxTokens];
#pragma unroll
            for (int t = 0; t < kDlMaxTokens; ++t) acc[t] = 0.0;
            double wsq = 0.0;
#pragma unroll
            for (int j = 0; j < kDecRows / 8; ++j) {
                const int i = warp * (kDecRows / 8) + j;
                wsq = fma(wv[j], wv[j], wsq);
#pragma unroll
                for (int t = 0; t < kDlMaxTokens; ++t)
                    if (t < T) acc[t] = fma(static_cast<double>(xs0[t * kDecRows + i]), wv[j], acc[t]);
            }
#pragma unroll
            for (int t = 0; t < kDlMaxTokens; ++t)
                if (t < T) red0[(warp * T + t) * 32 + lane] = acc[t];
            wred0[warp * 32 + lane] = wsq;
            __syncthreads();
            for (int idx = tid; idx < T * 32; idx += kDlThreads) {
                const int t = idx / 32, l = idx % 32;
                double s = 0.0;
                for (int w = 0; w < 8; ++w) s += red0[(w * T + t) * 32 + l];
                if (e0 + l < E) atomicAdd(d.racc + static_cast<size_t>(t) * E + e0 + l, s);
            }
            if (tid < 32 && e0 + tid < E) {
                double s = 0.0;
                for (int w = 0; w < 8; ++w) s += wred0[w * 32 + tid];
                atomicAdd(d.rwn + e0 + tid, s);
            }
            if (ec == 0 && tid < T) {
                double s = 0.0;
                for (int i = 0; i < kDecRows; ++i) {
                    const double v = static_cast<double>(xs0[tid * kDecRows + i]);
                    s = fma(v, v, s);
                }
                atomicAdd(d.rxn + tid, s);
            }
        }
        // token scales, exactly as the permutation (rows.cuh permute_token)
        if (b >= G - T) {
            const int t = G - 1 - b;
            __syncthreads();
            const float4* src = reinterpret_cast<const float4*>(a.x + static_cast<size_t>(t) * H);
            float mx = 0.0f;
            for (int c = tid; c < H / 4; c += kDlThreads) {
                const float4 v = src[c];
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane == 0) red_s[warp] = mx;
            __syncthreads();
            if (tid == 0) {
                mx = red_s[0];
                for (int w = 1; w < kDlThreads / 32; ++w) mx = fmaxf(mx, red_s[w]);
                int ex = 0;
                if (mx > 0.0f && isfinite(mx)) frexpf(mx, &ex);
                const int sh = (mx > 0.0f && isfinite(mx)) ? max(-126, min(126, 15 - ex)) : 0;
                d.tscale[t] = ldexpf(1.0f, sh);
                d.tscale[T + t] = ldexpf(1.0f, -sh);
            }
        }
    }
    bool ok = dl_grid_sync(d, 0, abort_s);

    // ------------------------------------------- work of phases C and D
    // C items: (row, projection, column part) for this CTA's K rank
    // r2 = b mod KS, pairs q2, q2 + nq2, ...; D items: (row, K rank, column
    // part), b, b + G, ...  Every item streams the whole rows of its rank's
    // slab in chunks of rc rows (a multiple of 4, so a row's class mod 4 is
    // its index mod 4 within any chunk) and accumulates the columns of its
    // part.  The last warp issues the chunks into the ring (waiting for the
    // consumers to free each stage); the other warps consume them.
    const int KS = d.KS, kc = d.kc, KSd = d.KSd, kcd = d.kcd;
    const int PC = (I + kDlPartCols - 1) / kDlPartCols, WC = ((I + PC - 1) / PC + 15) / 16 * 16;
    const int PD = (H + kDlPartCols - 1) / kDlPartCols, WD = ((H + PD - 1) / PD + 15) / 16 * 16;
    const int rc2 = min(kc, kDlStage / I / 4 * 4), nb2 = (kc + rc2 - 1) / rc2;
    const int rc3 = min(kcd, kDlStage / H / 4 * 4), nb3 = (kcd + rc3 - 1) / rc3;
    const int r2 = b % KS, q2 = b / KS, nq2 = (G - r2 + KS - 1) / KS;
    const int kb2 = r2 * kc; // at or past H for a rank with no rows (its partials stay zero)
    const int pairs2 = R * 2 * PC;
    const int n2 = ok && q2 < pairs2 ? (pairs2 - q2 + nq2 - 1) / nq2 : 0;
    const int tot2 = n2 * nb2;
    const int items3 = R * KSd * PD;
    const int n3 = ok && b < items3 ? (items3 - b + G - 1) / G : 0;
    const int tot = tot2 + n3 * nb3;
    // C item i: row, projection (0 gate, 1 up), part
    auto c_item = [&](int i, int& row, int& pj, int& part) {
        const int j = q2 + i * nq2;
        part = j % PC;
        pj = (j / PC) & 1;
        row = j / (2 * PC);
    };
    // D item i3: row, rank, part
    auto d_item = [&](int i3, int& row, int& r3, int& part) {
        const int idx3 = b + i3 * G;
        part = idx3 % PD;
        r3 = (idx3 / PD) % KSd;
        row = idx3 / (PD * KSd);
    };

    // ------------- speculative L2 prefetch of this CTA's weight slabs
    // The experts the router sums already rank highest are, but for a
    // logit the certificate moves across a float boundary, the ones the
    // exact selection below picks.  Grouping them the same way gives the
    // rows, hence this CTA's items; their slabs start crossing HBM into L2
    // now and the exact selection's 10-20 us overlap that transfer.
    __shared__ int gex_s[kDlMaxRows]; // row -> guessed expert
    if (ok) {
        uint32_t* gid = ids_s; // overwritten by the exact selection below
        for (int t = warp; t < T; t += kDlThreads / 32)
            guess_topk<C>(d.racc + static_cast<size_t>(t) * E, a.bias, E, k, gid + t * k);
        __syncthreads();
        for (int i = tid; i < R; i += kDlThreads) {
            const int t = i / slots, j = i % slots;
            const int e = j < k ? static_cast<int>(gid[t * k + j]) : E + (j - k);
            rtok_s[i] = e * T + t; // sort key, scratch until the exact grouping
        }
        __syncthreads();
        for (int i = tid; i < R; i += kDlThreads) {
            const int ki = rtok_s[i];
            int rnk = 0;
            for (int i2 = 0; i2 < R; ++i2) rnk += rtok_s[i2] < ki;
            gex_s[rnk] = ki / T;
        }
        __syncthreads();
        if (warp == 0) {
            int budget = kDlPrefetchBytes;
            for (int i = lane; i < n2; i += 32) { // gate/up slabs of this CTA's rank
                int row, pj, part;
                c_item(i, row, pj, part);
                const int rows = min(kc, H - kb2);
                if (part == 0 && rows > 0 && (budget -= rows * I * 32) >= 0)
                    bulk_prefetch_l2(d.arena + static_cast<size_t>(gex_s[row]) * d.stride +
                                         (pj ? d.up_off : d.gate_off) + static_cast<size_t>(kb2) * I,
                                     static_cast<uint32_t>(rows * I));
            }
            for (int i3 = lane; i3 < n3; i3 += 32) { // down slabs of this CTA's items
                int row, r3, part;
                d_item(i3, row, r3, part);
                const int rows = min(kcd, I - r3 * kcd);
                if (part == 0 && rows > 0 && (budget -= rows * H * 32) >= 0)
                    bulk_prefetch_l2(d.arena + static_cast<size_t>(gex_s[row]) * d.stride + d.down_off +
                                         static_cast<size_t>(r3) * kcd * H,
                                     static_cast<uint32_t>(rows * H));
            }
        }
    }

    // ------------------------- B: selection and grouping, in every CTA
    if (ok) {
        if (tid < 2 * T) tsc_s[tid] = __ldcg(d.tscale + tid);
        // every expert's dequantisation constants, while the selection runs
        float* qall = reinterpret_cast<float*>(base + L.b_q); // [E + S][scale x3, offset x3]
        for (int e = tid; e < E + slots - k; e += kDlThreads) {
            const hmoe_expert_quant q = d.quant[e];
#pragma unroll
            for (int p = 0; p < 3; ++p) {
                qall[e * 6 + p] = q.scale[p];
                qall[e * 6 + 3 + p] = 8388608.0f + 128.0f + static_cast<float>(q.zero_point[p]);
            }
        }
        __syncthreads();
        // Certify, settle and select.  Every CTA reaches the same result; only
        // CTA 0 counts near-ties and sequential sums and reports failures.
        RouteArgs ra = a;
        ra.ids = ids_s;
        ra.scores = scores_s;
        ra.st = b == 0 ? a.st : nullptr;
        const DecodeTailSmem m{reinterpret_cast<float*>(base + L.b_logit), reinterpret_cast<float*>(base + L.b_evs),
                               reinterpret_cast<double*>(base + L.b_wn), reinterpret_cast<double*>(base + L.b_xn),
                               reinterpret_cast<float*>(base + L.b_bias), reinterpret_cast<int*>(base + L.b_fb),
                               reinterpret_cast<int*>(base + L.b_fb) + 1,
                               reinterpret_cast<double*>(base + L.b_stage)};
        decode_certify(
            ra, [&](int idx) { return __ldcg(d.racc + idx); }, [&](int t) { return __ldcg(d.rxn + t); },
            [&](int e) { return __ldcg(d.rwn + e); }, m);
        decode_select_block(ra, m);
        __syncthreads();
        // Rows in (expert, token) order, shared experts E.. after the routed
        // ones, as the grouping kernel orders them.
        int* key_s = reinterpret_cast<int*>(base + L.b_grp); // [R] assignment -> key
        int* row_of = key_s + R;                              // [R] assignment -> row
        int* ex_s = row_of + R;                               // [R] row -> expert
        for (int i = tid; i < R; i += kDlThreads) {
            const int t = i / slots, j = i % slots;
            const int e = j < k ? static_cast<int>(ids_s[t * k + j]) : E + (j - k);
            key_s[i] = e * T + t;
        }
        __syncthreads();
        for (int i = tid; i < R; i += kDlThreads) {
            const int ki = key_s[i];
            int rnk = 0;
            for (int i2 = 0; i2 < R; ++i2) rnk += key_s[i2] < ki;
            const int t = i / slots, j = i % slots;
            row_of[i] = rnk;
            ex_s[rnk] = ki / T;
            rtok_s[rnk] = t;
            rw_s[rnk] = j < k ? scores_s[t * k + j] : 1.0f;
        }
        __syncthreads();
        for (int i = tid; i < R; i += kDlThreads) {
            const int t = i / slots, r = row_of[i];
            int pos = 0;
            for (int j2 = 0; j2 < slots; ++j2) pos += row_of[t * slots + j2] < r;
            trow_s[t * slots + pos] = r;
        }
        for (int r = tid; r < R; r += kDlThreads) {
            if (r == 0 || ex_s[r] != ex_s[r - 1]) {
                int u = 0;
                for (int r2 = 1; r2 <= r; ++r2) u += ex_s[r2] != ex_s[r2 - 1];
                int len = 1;
                while (r + len < R && ex_s[r + len] == ex_s[r]) ++len;
                const int e = ex_s[r];
                seg_s[u] = make_int4(e, r, len, 0);
#pragma unroll
                for (int p = 0; p < 3; ++p) {
                    qs_s[u][p] = qall[e * 6 + p];
                    qz_s[u][p] = qall[e * 6 + 3 + p];
                }
                for (int rr = r; rr < r + len; ++rr) {
                    rsc_s[rr] = qall[e * 6 + 2];
                    rseg_s[rr] = u;
                }
            }
        }
        if (tid == 0) {
            int n = 1;
            for (int r = 1; r < R; ++r) n += ex_s[r] != ex_s[r - 1];
            nseg_s = n;
        }
        if (b == 0)
            for (int i = tid; i < T * k; i += kDlThreads) {
                a.ids[i] = ids_s[i];
                a.scores[i] = scores_s[i];
            }
    } else if (tid == 0) {
        nseg_s = 0;
    }
    sm100::fence_proxy_async_smem(); // phase B's writes precede the ring's TMA copies
    __syncthreads();

    uint64_t* empty = full + S;

    if (warp == kDlCw) {
        // ------------------------------------------------------ producer
        if (lane == 0 && ok) {
            int issued = 0;
            for (int n = 0; n < tot; ++n) {
                const int s = n % S;
                // the consumers have freed the stage (chunk n - S)
                if (n >= S && !dl_wait(d, &empty[s], ((n / S) - 1) & 1)) break;
                const int8_t* src;
                int rows, N;
                if (n < tot2) {
                    int row, pj, part;
                    c_item(n / nb2, row, pj, part);
                    const int ch = n % nb2, r0 = kb2 + ch * rc2;
                    rows = min(min(rc2, kc - ch * rc2), H - r0);
                    N = I;
                    src = d.arena + static_cast<size_t>(seg_s[rseg_s[row]].x) * d.stride +
                          (pj ? d.up_off : d.gate_off) + static_cast<size_t>(r0) * I;
                } else {
                    int row, r3, part;
                    const int m = n - tot2;
                    d_item(m / nb3, row, r3, part);
                    const int ch = m % nb3, r0 = r3 * kcd + ch * rc3;
                    rows = min(min(rc3, kcd - ch * rc3), I - r0);
                    N = H;
                    src = d.arena + static_cast<size_t>(seg_s[rseg_s[row]].x) * d.stride + d.down_off +
                          static_cast<size_t>(r0) * H;
                }
                // a chunk wholly past K is not copied: its barrier completes
                // with a plain arrival
                if (rows > 0) {
                    sm100::mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(rows * N));
                    sm100::bulk_load(ring + s * kDlStage, src, static_cast<uint32_t>(rows * N), &full[s]);
                } else {
                    sm100::mbar_arrive(&full[s]);
                }
                issued = n + 1;
            }
            // every copy lands before the warp exits (the earlier ones were
            // consumed, which the stage waits above saw)
            for (int n = max(0, issued - S); n < issued; ++n)
                sm100::mbar_wait_for(&full[n % S], (n / S) & 1, kDlWaitNs);
        }
        return; // the producer warp takes no part in the rest
    }

    // ------------------------------------------------------ consumers
    __shared__ int cdead_s; // a consumer's wait failed
    if (tid == 0) cdead_s = !ok;
    consumers_sync();
    float* red = reinterpret_cast<float*>(base + L.red); // [part columns] row classes added in order
    // Accumulates chunk n (rows x N bytes in stage n mod S; columns
    // [c0, c0 + w) of the part) times v[0..rows) into acc, then frees the
    // stage.  Unit u = thread + kDlCt * k (k < 2) is (16-column group
    // u mod JG, row class u / JG): rows g, g + 4, ... of the chunk, in
    // order, as the GEMV's row groups.  Packed FP32 pairs (FADD2 / FFMA2) do
    // the dequantisation and the products, each lane rounding as fmaf.
    auto consume = [&](int n, int N, int nr, int c0, int w, float zoff, const float* v, float2 (&acc)[2][8]) {
        const int s = n % S;
        const bool got = dl_wait(d, &full[s], (n / S) & 1);
        if (got) {
            const uint8_t* chunk = ring + s * kDlStage + c0;
            const int JG = w / 16;
            const float2 noff = make_float2(-zoff, -zoff);
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int u = tid + kDlCt * k;
                if (u < 4 * JG) {
                    const int j = u % JG, g = u / JG;
#pragma unroll 2
                    for (int rr = g; rr < nr; rr += 4) {
                        const float xv = v[rr];
                        const float2 x2 = make_float2(xv, xv);
                        const uint4 q4 = *reinterpret_cast<const uint4*>(chunk + rr * N + 16 * j);
                        const uint32_t qw[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                        for (int h = 0; h < 4; ++h) {
                            const uint32_t q = qw[h] ^ 0x80808080u;
                            float2 lo = make_float2(__uint_as_float(__byte_perm(q, 0x4B000000u, 0x7540)),
                                                    __uint_as_float(__byte_perm(q, 0x4B000000u, 0x7541)));
                            float2 hi = make_float2(__uint_as_float(__byte_perm(q, 0x4B000000u, 0x7542)),
                                                    __uint_as_float(__byte_perm(q, 0x4B000000u, 0x7543)));
                            lo = __fadd2_rn(lo, noff);
                            hi = __fadd2_rn(hi, noff);
                            acc[k][2 * h] = __ffma2_rn(x2, lo, acc[k][2 * h]);
                            acc[k][2 * h + 1] = __ffma2_rn(x2, hi, acc[k][2 * h + 1]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&empty[s]);
        } else {
            cdead_s = 1; // the stage is not freed: the producer stops at the abort word
        }
        return got;
    };
    // The row classes' sums added in order (class 0 stores, 1..3 add in
    // turn) into red[0..w).
    auto fold = [&](const float2 (&acc)[2][8], int w) {
        const int JG = w / 16;
        for (int gg = 0; gg < 4; ++gg) {
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int u = tid + kDlCt * k;
                if (u < 4 * JG && u / JG == gg) {
                    float2* r = reinterpret_cast<float2*>(red + 16 * (u % JG));
#pragma unroll
                    for (int h = 0; h < 8; ++h) {
                        if (gg == 0) {
                            r[h] = acc[k][h];
                        } else {
                            float2 o = r[h];
                            o.x += acc[k][h].x;
                            o.y += acc[k][h].y;
                            r[h] = o;
                        }
                    }
                }
            }
            consumers_sync();
        }
    };
    auto zero = [](float2 (&acc)[2][8]) {
#pragma unroll
        for (int k = 0; k < 2; ++k)
#pragma unroll
            for (int h = 0; h < 8; ++h) acc[k][h] = make_float2(0.0f, 0.0f);
    };

    // ------------------------------------------------------- C: gate/up
    {
        float* xs2 = reinterpret_cast<float*>(base + L.c_xs); // [T][kc] token rows of this rank
        if (n2 > 0) {
            for (int i = tid; i < T * kc; i += kDlCt) {
                const int t = i / kc, kk = i % kc;
                float v = 0.0f;
                if (kb2 + kk < H)
                    v = __half2float(__float2half_rn(a.x[static_cast<size_t>(t) * H + kb2 + kk] * tsc_s[t])) *
                        tsc_s[T + t];
                xs2[i] = v;
            }
        }
        consumers_sync();
        for (int i = 0; i < n2; ++i) {
            int row, pj, part;
            c_item(i, row, pj, part);
            const int u = rseg_s[row];
            const int c0 = part * WC, w = min(WC, I - c0);
            const float zoff = qz_s[u][pj];
            const float* xrow = xs2 + rtok_s[row] * kc;
            float2 acc[2][8];
            zero(acc);
            for (int ch = 0; ch < nb2; ++ch)
                consume(i * nb2 + ch, I, min(min(rc2, kc - ch * rc2), H - (kb2 + ch * rc2)), c0, w, zoff,
                        xrow + ch * rc2, acc);
            fold(acc, w);
            if (cdead_s) break; // uniform: read after a consumer barrier
            for (int c = tid; c < w; c += kDlCt)
                d.pgu[(static_cast<size_t>(r2) * R + row) * (2 * I) + pj * I + c0 + c] = red[c];
            consumers_sync();
        }
    }
    ok = dl_grid_sync_consumers(d, 1, abort_s) && !cdead_s;

    // ---------------------------------------------------------- D: down
    {
        float* hs = reinterpret_cast<float*>(base + L.d_hs); // [kcd] SwiGLU values of the item
        for (int i3 = 0; ok && i3 < n3; ++i3) {
            int row, r3, part;
            d_item(i3, row, r3, part);
            const int u = rseg_s[row];
            const int kb3 = r3 * kcd;
            // SwiGLU values [kb3, kb3 + kcd) of the row: the gate/up ranks
            // added in order, as the GEMV's gate/up epilogue does
            for (int kk = tid; kk < kcd; kk += kDlCt) {
                float v = 0.0f;
                if (kb3 + kk < I) {
                    float v0[8], v1[8];
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        const float* pr = d.pgu + (static_cast<size_t>(r) * R + row) * (2 * I) + kb3 + kk;
                        v0[r] = r < KS ? __ldcg(pr) : 0.0f;
                        v1[r] = r < KS ? __ldcg(pr + I) : 0.0f;
                    }
                    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
                    for (int r = 0; r < 8; ++r)
                        if (r < KS) {
                            s0 += v0[r];
                            s1 += v1[r];
                        }
                    const float gg = qs_s[u][0] * s0;
                    const float uu = qs_s[u][1] * s1;
                    v = silu(gg) * uu;
                }
                hs[kk] = v;
            }
            consumers_sync();
            const int c0 = part * WD, w = min(WD, H - c0);
            const float zoff = qz_s[u][2];
            float2 acc[2][8];
            zero(acc);
            for (int ch = 0; ch < nb3; ++ch)
                consume(tot2 + i3 * nb3 + ch, H, min(min(rc3, kcd - ch * rc3), I - (kb3 + ch * rc3)), c0, w, zoff,
                        hs + ch * rc3, acc);
            fold(acc, w);
            if (cdead_s) break;
            for (int c = tid; c < w; c += kDlCt)
                d.pdn[(static_cast<size_t>(r3) * R + row) * H + c0 + c] = red[c];
            consumers_sync(); // red and hs are rewritten by the next item
        }
    }
    ok = dl_grid_sync_consumers(d, 2, abort_s) && ok && !cdead_s;

    // -------------------------------------------------------- E: combine
    if (ok) {
        float* vb = reinterpret_cast<float*>(base + L.e_v); // [slots][32]
        const int units = T * (H / 32);
        for (int un = b; un < units; un += G) {
            const int t = un / (H / 32), c = (un % (H / 32)) * 32 + lane;
            // warp w: the BF16 output rows of slots w, w + kDlCw, ... (as
            // the down projection rounds them), each the down ranks added in
            // order
            for (int sl = warp; sl < slots; sl += kDlCw) {
                const int r = trow_s[t * slots + sl];
                float v[8];
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    v[q] = q < KSd ? __ldcg(d.pdn + (static_cast<size_t>(q) * R + r) * H + c) : 0.0f;
                float s0 = 0.0f;
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    if (q < KSd) s0 += v[q];
                vb[sl * 32 + lane] = __bfloat162float(__float2bfloat16_rn(rw_s[r] * (rsc_s[r] * s0)));
            }
            consumers_sync();
            if (warp == 0) { // rows in ascending expert id, from zero
                float acc = 0.0f;
                for (int sl = 0; sl < slots; ++sl) acc = __fadd_rn(acc, vb[sl * 32 + lane]);
                const size_t o = static_cast<size_t>(t) * H + c;
                if (d.residual) acc = __fadd_rn(d.residual[o], acc);
                d.y[o] = acc;
                if (d.y16) d.y16[o] = __float2bfloat16_rn(acc);
            }
            consumers_sync();
        }
    }
}

} // namespace

// ------------------------------------------------------------ host side

namespace {

// The GEMV variant's split of K over ranks (expert_gemv.cu gemv_split): the
// same split here gives the same summation order.
int dl_split(int K) {
    int ks = 8;
    while (ks > 1 && (K + ks - 1) / ks < 32) ks /= 2;
    return ks;
}

int dl_rows_per_rank(int K, int ks) {
    const int kc = (K + ks - 1) / ks;
    return (kc + 31) / 32 * 32;
}

struct DlLayout {
    size_t tscale, pgu, pdn, total;
};

DlLayout dl_layout(const hmoe_layer_desc& d, size_t T) {
    const size_t H = d.hidden, I = d.intermediate, slots = d.top_k + d.shared_experts;
    const size_t R = T * slots;
    const size_t KS = dl_split(static_cast<int>(H)), KSd = dl_split(static_cast<int>(I));
    DlLayout l{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align_up(off + bytes, 256);
        return at;
    };
    l.tscale = take(2 * T * 4);
    l.pgu = take(KS * R * 2 * I * 4);
    l.pdn = take(KSd * R * H * 4);
    l.total = off;
    return l;
}

template <int C>
const void* dl_kernel() {
    return reinterpret_cast<const void*>(decode_layer_kernel<C>);
}

const void* dl_pick(int E) {
    const int c = (E + 31) / 32;
    if (c <= 1) return dl_kernel<1>();
    if (c <= 2) return dl_kernel<2>();
    if (c <= 4) return dl_kernel<4>();
    return dl_kernel<8>();
}

// Ring stages for a shape, 0 when the phases' scratch leaves too little.
int dl_stages(int T, int H, int E, int kc, int kcd, int R) {
    const DlSmem L0 = dl_smem(T, H, E, kc, kcd, R, 0);
    int S = std::min(kDlMaxStages, (kDlDynLimit - L0.total) / (kDlStage + 8));
    while (S > 0) {
        const DlSmem L = dl_smem(T, H, E, kc, kcd, R, S);
        if (L.total <= kDlDynLimit && L.b_end <= L.bars) break; // phase B stays clear of the barriers
        --S;
    }
    return S >= 3 ? S : 0;
}

} // namespace

bool decode_layer_shape_ok(const hmoe_layer_desc& d, size_t T) {
    const size_t slots = d.top_k + d.shared_experts;
    if (!(T >= 1 && T <= static_cast<size_t>(kDlMaxTokens) && slots <= static_cast<size_t>(kDlMaxSlots) &&
          T * slots <= static_cast<size_t>(kDlMaxRows) && d.hidden % 256 == 0 && d.intermediate % 128 == 0 &&
          d.intermediate >= 256 && reinterpret_cast<uintptr_t>(d.arena) % 16 == 0 &&
          d.experts <= static_cast<uint32_t>(kMaxExperts) && d.ep_size == 1))
        return false;
    const int H = static_cast<int>(d.hidden), I = static_cast<int>(d.intermediate);
    const int kc = dl_rows_per_rank(H, dl_split(H)), kcd = dl_rows_per_rank(I, dl_split(I));
    return dl_stages(static_cast<int>(T), H, static_cast<int>(d.experts), kc, kcd, static_cast<int>(T * slots)) > 0;
}

// Zeroed per call: the control words, then the router sums [T][E], the
// column norms [E] and the token norms [T] (FP64).
size_t decode_layer_ctl_bytes(const hmoe_layer_desc& d, size_t T) {
    if (!decode_layer_shape_ok(d, T)) return 0;
    return sizeof(DlCtl) + align_up(T * d.experts * 8, 256) + align_up(d.experts * 8, 256) + align_up(T * 8, 256);
}

size_t decode_layer_data_bytes(const hmoe_layer_desc& d, size_t T) {
    return decode_layer_shape_ok(d, T) ? dl_layout(d, T).total : 0;
}

hmoe_status launch_decode_layer(const hmoe_layer_desc& desc, const float* x, const float* residual, float* y,
                                __nv_bfloat16* y16, size_t tokens, char* ws, const Workspace& w,
                                cudaStream_t stream) {
    if (!decode_layer_shape_ok(desc, tokens) || !w.dl_ctl_bytes || !w.dl_data_bytes) return HMOE_UNSUPPORTED;
    if (reinterpret_cast<uintptr_t>(x) % 16) return HMOE_UNSUPPORTED;
    const int T = static_cast<int>(tokens), H = static_cast<int>(desc.hidden), I = static_cast<int>(desc.intermediate);
    const int E = static_cast<int>(desc.experts), S = static_cast<int>(desc.shared_experts);
    const int k = static_cast<int>(desc.top_k), slots = k + S, R = T * slots;
    DlArgs d{};
    d.ra = RouteArgs{x, desc.router_weight, desc.router_bias, T, H, E, k, desc.softmax, desc.renormalize,
                     reinterpret_cast<uint32_t*>(ws + w.ids), reinterpret_cast<float*>(ws + w.scores), nullptr,
                     reinterpret_cast<DeviceStatus*>(ws + w.status), nullptr};
    d.residual = residual;
    d.y = y;
    d.y16 = y16;
    d.quant = desc.quant;
    d.slots = slots;
    d.I = I;
    d.KS = dl_split(H);
    d.kc = dl_rows_per_rank(H, d.KS);
    d.KSd = dl_split(I);
    d.kcd = dl_rows_per_rank(I, d.KSd);
    d.arena = desc.arena;
    d.stride = desc.expert_stride;
    d.gate_off = desc.gate_offset;
    d.up_off = desc.up_offset;
    d.down_off = desc.down_offset;
    d.nstage = dl_stages(T, H, E, d.kc, d.kcd, R);
    const DlSmem L = dl_smem(T, H, E, d.kc, d.kcd, R, d.nstage);
    char* base = ws + w.dl_data;
    const DlLayout l = dl_layout(desc, tokens);
    d.ctl = reinterpret_cast<DlCtl*>(ws + w.dl_ctl);
    char* z = ws + w.dl_ctl + sizeof(DlCtl);
    d.racc = reinterpret_cast<double*>(z);
    d.rwn = reinterpret_cast<double*>(z + align_up(tokens * desc.experts * 8, 256));
    d.rxn = reinterpret_cast<double*>(z + align_up(tokens * desc.experts * 8, 256) + align_up(desc.experts * 8, 256));
    d.tscale = reinterpret_cast<float*>(base + l.tscale);
    d.pgu = reinterpret_cast<float*>(base + l.pgu);
    d.pdn = reinterpret_cast<float*>(base + l.pdn);
    const void* fn = dl_pick(E);
    cudaError_t err = set_smem_limit(fn, L.total);
    if (err != cudaSuccess) {
        set_last_error("hmoe decode layer shared memory", err);
        return HMOE_CUDA_ERROR;
    }
    int per_sm = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kDlThreads, L.total);
    if (err != cudaSuccess || per_sm < 1) return HMOE_UNSUPPORTED;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(current_sm_count()));
    cfg.blockDim = dim3(kDlThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(L.total);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative; // every CTA resident at once: the grid barriers rely on it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {&d};
    err = cudaLaunchKernelExC(&cfg, fn, args);
    if (err != cudaSuccess) {
        set_last_error("hmoe decode layer launch", err);
        return HMOE_CUDA_ERROR;
    }
    return check_launch("hmoe decode layer");
}

} // namespace hmoe
