// router.cu -- router logits, softmax, top-k, renormalisation and the
// device-built expert grouping (histogram, prefix offsets, permutation).
//
// Contract: the selected ids (and therefore the permutation) equal those of
// the reference CPU router, CpuRouterBackend::routeToken
// (src/router/CpuRouterBackend.cpp:35-91), on the same inputs:
//
//  * logits.  The reference computes float(sum_i double(h_i)*double(W_ie))
//    sequentially in i order.  A product of two floats is exact in double,
//    so only the summation order can differ.  Here the sum is formed in P
//    parallel chunks (fixed order), and a rigorous bound on the difference
//    between any two orderings, (H + L + P + 2) * 2^-53 * sum|h_i W_ie|, is
//    checked against the distance to the nearest float rounding boundary.
//    When the bound does not certify that both orders round to the same
//    float, that logit is recomputed in the reference's sequential order.
//    Every logit is therefore bit-identical to the reference's.
//
//  * softmax.  exp(l - max) is evaluated in double and rounded to float
//    (a correctly rounded expf).  The reference calls glibc expf, which is
//    not correctly rounded for ~1e-4 of inputs (always within 1 ulp).  exp
//    is monotone, so the selection can only differ from the reference where
//    two candidate probabilities adjacent in rank are within 2 ulp of each
//    other while their logits differ.  Such near-ties are counted in the
//    workspace status word (hmoe_read_status) so callers and tests can see
//    that the certificate covered every token.
//
//  * the denominator is a double sum in expert order, the probabilities
//    float(double(e)/D), selection (score desc, id asc), renormalisation by
//    a double sum in rank order -- all as in the reference.
#include "common.cuh"
#include "layer.cuh"
#include "route_core.cuh"
#include "sm100.cuh"

#include <cooperative_groups.h>
#include <cub/block/block_scan.cuh>

#include <cfloat>
#include <algorithm>
#include <climits>

namespace cg = cooperative_groups;

namespace hmoe {

// Shared-memory plan of the fused router (byte offsets, 16-byte aligned).
// The router-matrix slab ring and, after the main loop, the per-row-lane
// partial sums share one region.
struct RouteSmem {
    int slab_rows;                  // router rows per bulk copy (power of two)
    int ring, xf, xs, wsq, xn, xw, logit, evs, fb, bars, total;
};

__host__ __device__ inline RouteSmem route_smem(int E, int E_pad, int P) {
    RouteSmem m{};
    int sr = 256;
    while (sr > 8 && sr * E_pad * 4 > 16384) sr >>= 1;
    m.slab_rows = sr;
    auto al = [](int v) { return (v + 15) & ~15; };
    const int ring_bytes = kRouteStages * sr * E * 4;
    const int part_bytes = kRouteTokens * P * E_pad * 8;
    int off = 0;
    m.ring = off;
    off = al(off + (ring_bytes > part_bytes ? ring_bytes : part_bytes));
    m.xf = off;
    off = al(off + kRouteTokens * kRouteChunk * 4);
    m.xs = off;
    off = al(off + kRouteTokens * kRouteChunk * 8);
    m.wsq = off;
    off = al(off + P * E_pad * 4);
    m.xn = off;
    off = al(off + 2 * kRouteTokens * 8);
    m.xw = off;
    off = al(off + 8 * kRouteTokens * 8);
    m.logit = off;
    off = al(off + kRouteTokens * E_pad * 4);
    m.evs = off;
    off = al(off + kRouteTokens * E_pad * 4);
    m.fb = off;
    off = al(off + (1 + kRouteFallbacks) * 4);
    m.bars = off;
    off = al(off + (kRouteStages + 1) * 8);
    m.total = off;
    return m;
}


// Fused router.  Grid (KS, ceil(T/kRouteTokens)), clusters of KS CTAs along
// x: CTA r of a cluster sums hidden rows [r*H/KS, (r+1)*H/KS) for
// kRouteTokens tokens and every expert.  Thread (quad = tid % EQ,
// p = tid / EQ) owns experts 4*quad..4*quad+3 and the rows i = p (mod P)
// of each router slab.  Both operands arrive by bulk copies: the router
// matrix in slabs of contiguous rows through a kRouteStages-deep ring, the
// token rows kRouteChunk floats at a time, converted once to doubles in
// shared memory (so one broadcast load feeds four DFMAs).  Partial sums
// meet in (distributed) shared memory and are added in a fixed order
// (rank, p).  The certificate bounds sum_i |x_i W_ie| by ||x|| ||W_e||
// (Cauchy-Schwarz); ||x_t||^2 is accumulated during the conversion.
template <int C>
__global__ void __launch_bounds__(256, 2) route_kernel(RouteArgs a, int EQ, int P, int KS) {
    extern __shared__ __align__(16) unsigned char smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int H = a.H, E = a.E;
    const int E_pad = 4 * EQ;
    const RouteSmem L = route_smem(E, E_pad, P);
    const int SR = L.slab_rows;
    const int stage_region = L.xf - L.ring; // the slab ring / partials region, free in phase 2b
    float* wsl = reinterpret_cast<float*>(smem + L.ring);                     // [stages][SR][E]
    double* part = reinterpret_cast<double*>(smem + L.ring);                  // [TB][P][E_pad] (after)
    float* xf = reinterpret_cast<float*>(smem + L.xf);                        // [TB][chunk] staging
    double* xs = reinterpret_cast<double*>(smem + L.xs);                      // [TB][chunk]
    float* wsq = reinterpret_cast<float*>(smem + L.wsq);                      // [P][E_pad]
    double* xn_part = reinterpret_cast<double*>(smem + L.xn);                 // [TB] this CTA's rows
    double* xn = xn_part + kRouteTokens;                                      // [TB] all rows
    float* logit = reinterpret_cast<float*>(smem + L.logit);                  // [TB][E_pad]
    float* evs = reinterpret_cast<float*>(smem + L.evs);                      // [TB][E_pad]
    int* fb_count = reinterpret_cast<int*>(smem + L.fb);                      // [1]
    int* fb_list = fb_count + 1;                                              // [kRouteFallbacks]
    uint64_t* wbar = reinterpret_cast<uint64_t*>(smem + L.bars);              // [stages]
    uint64_t* xbar = wbar + kRouteStages;                                     // [1]

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int quad = tid % EQ, p = tid / EQ;
    const bool active = p < P;
    const int t0 = blockIdx.y * kRouteTokens;
    const int nt = min(kRouteTokens, a.T - t0);
    const int h0 = rank * (H / KS), h1 = h0 + H / KS;
    const bool vec4 = (E % 4) == 0;
    const int nslab = (h1 - h0 + SR - 1) / SR;
    const int nchunk = (h1 - h0 + kRouteChunk - 1) / kRouteChunk;

    double acc[kRouteTokens][4];
    double xsq[kRouteTokens];
    float sq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int t = 0; t < kRouteTokens; ++t) {
        xsq[t] = 0.0;
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[t][j] = 0.0;
    }

    auto issue_slab = [&](int sl) {
        const int r0 = h0 + sl * SR;
        const int nr = min(SR, h1 - r0);
        uint64_t* bar = &wbar[sl % kRouteStages];
        sm100::mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nr * E * 4));
        sm100::bulk_load(wsl + (sl % kRouteStages) * SR * E, a.w + static_cast<size_t>(r0) * E,
                         static_cast<uint32_t>(nr * E * 4), bar);
    };
    auto issue_chunk = [&](int c) {
        const int r0 = h0 + c * kRouteChunk;
        const int cn = min(kRouteChunk, h1 - r0);
        sm100::mbar_arrive_expect_tx(xbar, static_cast<uint32_t>(nt * cn * 4));
        for (int t = 0; t < nt; ++t)
            sm100::bulk_load(xf + t * kRouteChunk, a.x + static_cast<size_t>(t0 + t) * H + r0,
                             static_cast<uint32_t>(cn * 4), xbar);
    };
    if (tid == 0) {
        *fb_count = 0;
        for (int s = 0; s < kRouteStages; ++s) sm100::mbar_init(&wbar[s], 1);
        sm100::mbar_init(xbar, 1);
        sm100::fence_mbarrier_init();
        if (nchunk > 0) issue_chunk(0);
        for (int sl = 0; sl < kRouteStages && sl < nslab; ++sl) issue_slab(sl);
    }
    __syncthreads();

    for (int sl = 0; sl < nslab; ++sl) {
        const int r0 = h0 + sl * SR;
        const int nr = min(SR, h1 - r0);
        const int xoff = (r0 - h0) % kRouteChunk;
        if (xoff == 0) { // convert the next token chunk to doubles
            const int c = (r0 - h0) / kRouteChunk;
            const int cn = min(kRouteChunk, h1 - r0);
            if (!sm100::mbar_wait_for(xbar, c & 1, 2000000000ull)) device_fail(a.st, HMOE_TIMEOUT);
            for (int i = tid; i < kRouteChunk; i += blockDim.x) {
#pragma unroll
                for (int t = 0; t < kRouteTokens; ++t) {
                    const double v = (t < nt && i < cn) ? static_cast<double>(xf[t * kRouteChunk + i]) : 0.0;
                    xs[t * kRouteChunk + i] = v;
                    xsq[t] = fma(v, v, xsq[t]);
                }
            }
            __syncthreads(); // xs complete, xf free
            if (tid == 0 && c + 1 < nchunk) issue_chunk(c + 1);
        }
        if (!sm100::mbar_wait_for(&wbar[sl % kRouteStages], (sl / kRouteStages) & 1, 2000000000ull))
            device_fail(a.st, HMOE_TIMEOUT);
        const float* ws = wsl + (sl % kRouteStages) * SR * E;
        if (active) {
            // Two rows per iteration with every shared load issued before the
            // DFMAs, so the load latency of one row overlaps the other's math.
            int i = p;
            for (; i + P < nr; i += 2 * P) {
                float wv[2][4];
                if (vec4) {
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const float4 w4 = *reinterpret_cast<const float4*>(ws + (i + u * P) * E + 4 * quad);
                        wv[u][0] = w4.x; wv[u][1] = w4.y; wv[u][2] = w4.z; wv[u][3] = w4.w;
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < 2; ++u)
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            wv[u][j] = 4 * quad + j < E ? ws[(i + u * P) * E + 4 * quad + j] : 0.0f;
                }
                double xv[2][kRouteTokens];
#pragma unroll
                for (int u = 0; u < 2; ++u)
#pragma unroll
                    for (int t = 0; t < kRouteTokens; ++t) xv[u][t] = xs[t * kRouteChunk + xoff + i + u * P];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    double wd[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        wd[j] = static_cast<double>(wv[u][j]);
                        sq[j] = fmaf(wv[u][j], wv[u][j], sq[j]);
                    }
#pragma unroll
                    for (int t = 0; t < kRouteTokens; ++t)
#pragma unroll
                        for (int j = 0; j < 4; ++j) acc[t][j] = fma(xv[u][t], wd[j], acc[t][j]);
                }
            }
            for (; i < nr; i += P) {
                float wv[4];
                if (vec4) {
                    const float4 w4 = *reinterpret_cast<const float4*>(ws + i * E + 4 * quad);
                    wv[0] = w4.x; wv[1] = w4.y; wv[2] = w4.z; wv[3] = w4.w;
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) wv[j] = 4 * quad + j < E ? ws[i * E + 4 * quad + j] : 0.0f;
                }
                double wd[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    wd[j] = static_cast<double>(wv[j]);
                    sq[j] = fmaf(wv[j], wv[j], sq[j]);
                }
                const double* xr = xs + xoff + i;
#pragma unroll
                for (int t = 0; t < kRouteTokens; ++t) {
                    const double xv = xr[t * kRouteChunk];
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[t][j] = fma(xv, wd[j], acc[t][j]);
                }
            }
        }
        __syncthreads(); // every warp is done with this slot
        if (tid == 0 && sl + kRouteStages < nslab) issue_slab(sl + kRouteStages);
    }
    // ||x_t||^2 over this CTA's rows: warp sums, then a fixed-order sum of
    // the warps (the value only feeds an upper bound).
#pragma unroll
    for (int t = 0; t < kRouteTokens; ++t) {
        double v = xsq[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        xsq[t] = v;
    }
    double* xw = reinterpret_cast<double*>(smem + L.xw); // [8 warps][TB]
    if (lane == 0)
#pragma unroll
        for (int t = 0; t < kRouteTokens; ++t) xw[warp * kRouteTokens + t] = xsq[t];
    if (active) {
#pragma unroll
        for (int t = 0; t < kRouteTokens; ++t)
#pragma unroll
            for (int j = 0; j < 4; ++j) part[(t * P + p) * E_pad + 4 * quad + j] = acc[t][j];
#pragma unroll
        for (int j = 0; j < 4; ++j) wsq[p * E_pad + 4 * quad + j] = sq[j];
    }
    __syncthreads();
    if (tid < kRouteTokens) {
        double v = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += xw[w * kRouteTokens + tid];
        xn_part[tid] = v;
    }
    // Fold this CTA's row lanes in fixed order q = 0..P-1 into row 0 of each
    // token's partial block (and of wsq), so the cluster reduction below
    // reads one value per CTA.
    for (int idx = tid; idx < kRouteTokens * E_pad; idx += blockDim.x) {
        const int t = idx / E_pad, e = idx % E_pad;
        double s = 0.0;
        for (int q = 0; q < P; ++q) s += part[(t * P + q) * E_pad + e];
        part[(t * P) * E_pad + e] = s;
        if (t == 0) {
            float w2 = 0.0f;
            for (int q = 0; q < P; ++q) w2 += wsq[q * E_pad + e];
            wsq[e] = w2;
        }
    }
    cluster.sync();

    if (rank == 0) {
        if (tid < kRouteTokens) {
            double v = 0.0;
            for (int r = 0; r < KS; ++r) v += cluster.map_shared_rank(xn_part, r)[tid];
            xn[tid] = v;
        }
        __syncthreads();
        // Norm factors of the certificate, once per token and per expert:
        // ||x_t|| and ||W_e|| (each rounded up).
        double* wn = reinterpret_cast<double*>(evs); // [E_pad], free until phase 3
        for (int e = tid; e < E; e += blockDim.x) {
            float w2 = 0.0f;
            for (int r = 0; r < KS; ++r) w2 += cluster.map_shared_rank(wsq, r)[e];
            wn[e] = sqrt(static_cast<double>(w2) * (1.0 + (H + 64) * 0x1.0p-22));
        }
        if (tid < kRouteTokens) xn[tid] = sqrt(xn[tid] * (1.0 + 0x1.0p-40));
        __syncthreads();
        // Phase 2: exact float logits; logits the certificate cannot settle
        // are queued and recomputed in the reference's sequential order by
        // whole warps (phase 2b).
        const int L = H / (P * KS) + 1;
        const double gamma = static_cast<double>(H + L + P * KS + 4) * 0x1.0p-53 * 1.01;
        for (int idx = tid; idx < nt * E; idx += blockDim.x) {
            const int t = idx / E, e = idx % E;
            double pr[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) // issue every remote load first
                pr[r] = r < KS ? cluster.map_shared_rank(part, r)[(t * P) * E_pad + e] : 0.0;
            double s = 0.0;
            for (int r = 0; r < KS; ++r) s += pr[r];
            double A = xn[t] * wn[e] * (1.0 + 0x1.0p-40);
            if (a.bias) {
                s += static_cast<double>(a.bias[e]);
                A += fabs(static_cast<double>(a.bias[e]));
            }
            const double beta = gamma * A + 0x1.0p-1060;
            if (!rounding_certified(s, beta)) {
                const int slot = atomicAdd(fb_count, 1);
                if (slot < kRouteFallbacks) fb_list[slot] = t * 256 + e;
                else s = sequential_logit(a, t0 + t, e); // queue full: this thread does it
            }
            if (!isfinite(s)) device_fail(a.st, HMOE_NON_FINITE_ROUTER);
            logit[t * E_pad + e] = static_cast<float>(s);
        }
        __syncthreads();
        // Phase 2b, a warp per queued logit (settle_logit).  This CTA's
        // partials are consumed, so their region stages the products.
        const int nfb = min(*fb_count, kRouteFallbacks);
        const int slots = min(8, stage_region / (8 * staged_logit_doubles(H)));
        for (int f = warp; f < nfb; f += blockDim.x >> 5) {
            const int t = fb_list[f] >> 8, e = fb_list[f] & 255;
            const float lg = settle_logit(a, t0 + t, e, warp < slots ? part + warp * staged_logit_doubles(H) : nullptr);
            if (lane == 0) {
                if (!isfinite(lg)) device_fail(a.st, HMOE_NON_FINITE_ROUTER);
                logit[t * E_pad + e] = lg;
            }
        }
        __syncthreads();
        // Phase 3: softmax, selection, renormalisation; one warp per token.
        for (int t = warp; t < nt; t += blockDim.x >> 5) {
            float lv[C];
#pragma unroll
            for (int c = 0; c < C; ++c) {
                const int j = lane + 32 * c;
                lv[c] = j < E ? logit[t * E_pad + j] : 0.0f;
            }
            const size_t tok = static_cast<size_t>(t0 + t);
            select_token<C>(lv, E, a.k, a.softmax, a.renorm, evs + t * E_pad, a.ids + tok * a.k,
                            a.scores + tok * a.k, a.counts, token_block_counts(a, tok), a.st, false, nullptr);
        }
    }
    cluster.sync(); // keep every CTA's shared memory alive until rank 0 is done
}

// ------------------------------------------------------------ tiled router
//
// Large batches.  The router is a [T, H] x [H, E] product in FP64.  The
// per-8-token CTAs of route_kernel re-stream the whole router matrix for
// every 8 tokens and issue one DFMA per multiply-add with operands from
// shared memory, which holds them near a third of the FP64 rate.  The tiled
// kernel runs the products on the FP64 tensor-core path (mma.sync m8n8k4):
//  * a CTA owns 64 tokens and all (<= 128) experts, split over H across a
//    cluster of KS CTAs; warp (wm, wn) owns tokens 32wm.. and experts
//    32wn.. as 4 x 4 tiles of 8 x 8: 16 MMAs per 8 fragment loads;
//  * 32-row chunks of the FP32 token rows (one [64][32] box) and router
//    rows (four [32][32] boxes) arrive by TMA with the 128-byte swizzle
//    through a four-deep ring; the swizzle keeps an A-fragment load at one
//    shared-memory wavefront and a B-fragment load at two;
//  * fragments are converted float -> double as they are loaded (exact);
//  * a ring stage is refilled by the last warp to finish with it (a shared
//    counter), so the main loop runs no CTA-wide barrier;
//  * the certificate's norms come from the fragments themselves: ||x_t||^2
//    from the A fragments of warps 0 and 3, ||W_e||^2 from the B fragments
//    of warps 1, 2, 5 and 6, each summed in a fixed order.
// Products of two floats are exact in double and the tensor-core path
// rounds each accumulation to nearest (IEEE 754), so every output is a
// summation tree of the exact products with at most H/KS roundings on any
// chain: the rounding certificate of route_kernel covers it, and the
// logits, and all that follows from them, are bit-identical to the
// reference's (uncertified ones are recomputed sequentially).
constexpr int kRtTokens = 64;
constexpr int kRtRows = 32;     // hidden rows per chunk (one 128-byte swizzle row)
constexpr int kRtCols = 128;    // expert columns (E <= 128)
constexpr int kRtStages = 4;
constexpr int kRtFallbacks = 64;
constexpr int kStageW = 4 * kRtRows * 128;       // four [32 rows][32 experts] FP32 boxes
constexpr int kStageX = kRtTokens * 128;         // one [64 tokens][32 rows] FP32 box
constexpr int kStageBytes = kStageW + kStageX;     // 24 KB (multiple of 1024)

struct TiledSmem {
    int ring, xn, wn, xnorm, wnorm, bias, evs, fb, cnt, bars, total;
};

__host__ __device__ constexpr int tiled_al(int v) { return (v + 15) & ~15; }

// Offsets from the 1024-byte aligned base; `total` includes the alignment slack.
__host__ __device__ constexpr TiledSmem tiled_smem() {
    TiledSmem m{};
    int off = 0;
    m.ring = off; // [stages][W boxes | x box]; after the main loop [64][128]
                  // double partials, then [64][128] float logits
    off = tiled_al(off + kRtStages * kStageBytes);
    m.xn = off;   // [KS][64/KS] received ||x_t||^2 partials of this rank's tokens
    off = tiled_al(off + kRtTokens * 8);
    m.wn = off;   // [KS][128] received ||W_e||^2 partials; [8 warps][128] floats in phase 3
    off = tiled_al(off + 8 * kRtCols * 8);
    m.xnorm = off;
    off = tiled_al(off + kRtTokens * 8);
    m.wnorm = off;
    off = tiled_al(off + kRtCols * 8);
    m.bias = off;
    off = tiled_al(off + kRtCols * 4);
    m.evs = m.wn;
    m.fb = off;
    off = tiled_al(off + (1 + kRtFallbacks) * 4);
    m.cnt = off;  // [stages] warps done with the stage's current chunk
    off = tiled_al(off + kRtStages * 4);
    m.bars = off; // full[stages]
    off = tiled_al(off + kRtStages * 8);
    m.total = off + 1024;
    return m;
}

static_assert(kRtTokens * kRtCols * (8 + 4) <= kRtStages * kStageBytes,
              "tiled router: received partials and logits fit the ring");
static_assert(8 * kRtCols * 4 <= 8 * kRtCols * 8, "tiled router: softmax scratch fits the W-norm region");
static_assert(kStageBytes % 1024 == 0, "tiled router: swizzled boxes need 1024-byte alignment");
static_assert(tiled_smem().total <= 112 * 1024, "tiled router: two CTAs per SM");

__device__ __forceinline__ void dmma_8x8x4(double (&d)[2], double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
                 : "+d"(d[0]), "+d"(d[1])
                 : "d"(a), "d"(b));
}

// Grid (KS, ceil(T / kRtTokens)), clusters of KS CTAs along x; CTA r sums
// hidden rows [r*H/KS, (r+1)*H/KS).  mx: token rows [T][H], box [64][32];
// mw: router rows [H][E], box [32][32].  Needs E <= 128, E % 4 == 0 and
// H % (32*KS) == 0.
template <int C>
__global__ void __launch_bounds__(256, 2) route_tiled_kernel(const __grid_constant__ CUtensorMap mx,
                                                             const __grid_constant__ CUtensorMap mw,
                                                             RouteArgs a, int KS) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int H = a.H, E = a.E;
    constexpr TiledSmem L = tiled_smem();
    unsigned char* ring = smem + L.ring;
    double* recv = reinterpret_cast<double*>(ring);                            // [KS][64/KS][128]
    float* logit = reinterpret_cast<float*>(ring + kRtTokens * kRtCols * 8);   // [64/KS][128]
    double* xrecv = reinterpret_cast<double*>(smem + L.xn);                    // [KS][64/KS]
    double* wrecv = reinterpret_cast<double*>(smem + L.wn);                    // [KS][128]
    double* xnorm = reinterpret_cast<double*>(smem + L.xnorm);
    double* wnorm = reinterpret_cast<double*>(smem + L.wnorm);
    float* bias_s = reinterpret_cast<float*>(smem + L.bias);
    float* evs = reinterpret_cast<float*>(smem + L.evs);
    int* fb_count = reinterpret_cast<int*>(smem + L.fb);
    int* fb_list = fb_count + 1;
    int* cnt = reinterpret_cast<int*>(smem + L.cnt);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp & 1, wn4 = warp >> 1;
    const int t0 = blockIdx.y * kRtTokens;
    const int nt = min(kRtTokens, a.T - t0);
    const int rows = H / KS, h0 = rank * rows;
    const int nchunk = rows / kRtRows;

    if (tid == 0) {
        *fb_count = 0;
        for (int s = 0; s < kRtStages; ++s) {
            cnt[s] = 0;
            sm100::mbar_init(&full[s], 1);
        }
        sm100::fence_mbarrier_init();
        sm100::prefetch_tmap(&mx);
        sm100::prefetch_tmap(&mw);
    }
    __syncthreads();

    // Chunk c into stage c % kRtStages (one thread): the token box and the
    // four router boxes; rows past T and columns past E read as zero.
    auto issue = [&](int c) {
        const int s = c % kRtStages;
        const int r0 = h0 + c * kRtRows;
        unsigned char* st = ring + s * kStageBytes;
        sm100::mbar_arrive_expect_tx(&full[s], kStageBytes);
        for (int cb = 0; cb < 4; ++cb) sm100::tma_load_2d(st + cb * kRtRows * 128, &mw, 32 * cb, r0, &full[s]);
        sm100::tma_load_2d(st + kStageW, &mx, r0, t0, &full[s]);
    };
    if (tid == 0)
        for (int c = 0; c < kRtStages && c < nchunk; ++c) issue(c);

    double acc[4][4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;
    // Norm roles (one warp per token block and per expert block, disjoint):
    // role 1 (warps 0, 3): ||x||^2 of tokens 32wm + 8i + lane/4 from the A
    // fragments; role 2 (warps 1, 2, 5, 6): ||W||^2 of experts
    // 32wn + 8j + lane/4 from the B fragments.
    const int role = wn4 == wm ? 1 : (wm == 1 - (wn4 & 1) ? 2 : 0);
    double sq[4] = {0.0, 0.0, 0.0, 0.0};
    bool failed = false;
    const int fr = lane & 3, fc = lane >> 2; // fragment row / column within an 8 x 4 or 4 x 8 tile

    for (int c = 0; c < nchunk; ++c) {
        const int s = c % kRtStages;
        if (!sm100::mbar_wait_for(&full[s], (c / kRtStages) & 1, 2000000000ull)) failed = true;
        // Swizzled box rows are 128 bytes; 16-byte chunk q of row r sits at
        // chunk q ^ (r % 8).  B: row 4kk+fr, column 8j+fc of box wn.  A:
        // token 32wm+8i+fc (so r % 8 = fc), column 4kk+fr.
        const unsigned char* wsb = ring + s * kStageBytes + wn4 * (kRtRows * 128) + fr * 128 + (fc & 3) * 4;
        const unsigned char* xsb = ring + s * kStageBytes + kStageW + (32 * wm + fc) * 128 + fr * 4;
#pragma unroll 2
        for (int kk = 0; kk < kRtRows / 4; ++kk) {
            double av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                av[i] = static_cast<double>(*reinterpret_cast<const float*>(xsb + i * 8 * 128 + ((kk ^ fc) << 4)));
            const int rsw = (4 * kk + fr) & 7;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                bv[j] = static_cast<double>(
                    *reinterpret_cast<const float*>(wsb + kk * 4 * 128 + (((2 * j + (fc >> 2)) ^ rsw) << 4)));
            if (role == 1) {
#pragma unroll
                for (int i = 0; i < 4; ++i) sq[i] = fma(av[i], av[i], sq[i]);
            } else if (role == 2) {
#pragma unroll
                for (int j = 0; j < 4; ++j) sq[j] = fma(bv[j], bv[j], sq[j]);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) dmma_8x8x4(acc[i][j], av[i], bv[j]);
        }
        __syncwarp(); // every lane is done with stage s
        if (lane == 0) {
            __threadfence_block();
            if (atomicAdd(&cnt[s], 1) == 7) { // last warp out refills the stage
                cnt[s] = 0;
                __threadfence_block();
                if (c + kRtStages < nchunk) {
                    sm100::fence_proxy_async_smem();
                    issue(c + kRtStages);
                }
            }
        }
    }
    if (failed) {
        device_fail(a.st, HMOE_TIMEOUT);
        for (int s = 0; s < kRtStages && s < nchunk; ++s) // let issued copies land
            sm100::mbar_wait_for(&full[s], ((nchunk - 1 - s) / kRtStages) & 1, 2000000000ull);
    }
    __syncthreads(); // every warp is done with the ring

    // Partials of this CTA go straight to the rank that finishes them: rank
    // q owns tokens [q*TPR, (q+1)*TPR) of the tile and receives every rank's
    // sums for them (slot = source rank), the x-norm partials of its tokens
    // and every rank's W-norm partials.  The norms are first summed over the
    // four lanes of a fragment column (fixed order).
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        sq[i] += __shfl_xor_sync(0xffffffffu, sq[i], 1);
        sq[i] += __shfl_xor_sync(0xffffffffu, sq[i], 2);
    }
    const int TPR = kRtTokens / KS;
    cluster.sync(); // every CTA of the cluster is done with its ring
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int tok = 32 * wm + 8 * i + fc;
        const int q = tok / TPR, lt = tok % TPR;
        double* dst = cluster.map_shared_rank(recv, q) + (rank * TPR + lt) * kRtCols + 32 * wn4 + 2 * fr;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            *reinterpret_cast<double2*>(dst + 8 * j) = make_double2(acc[i][j][0], acc[i][j][1]);
        if (role == 1 && fr == 0) cluster.map_shared_rank(xrecv, q)[rank * TPR + lt] = sq[i];
    }
    if (role == 2 && fr == 0)
        for (int q = 0; q < KS; ++q) {
            double* dst = cluster.map_shared_rank(wrecv, q) + rank * kRtCols + 32 * wn4 + fc;
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[8 * j] = sq[j];
        }
    cluster.sync(); // everything this rank needs is now in its own shared memory

    // Epilogue: this rank finishes tokens [rank*TPR, (rank+1)*TPR) of the tile.
    const int lt0 = rank * TPR;
    const int ntr = max(0, min(TPR, nt - lt0));
    for (int e = tid; e < E; e += blockDim.x) {
        double w2 = 0.0;
        for (int q = 0; q < KS; ++q) w2 += wrecv[q * kRtCols + e];
        wnorm[e] = sqrt(w2 * (1.0 + (H + 64) * 0x1.0p-52));
        bias_s[e] = a.bias ? a.bias[e] : 0.0f;
    }
    if (tid < ntr) {
        double x2 = 0.0;
        for (int q = 0; q < KS; ++q) x2 += xrecv[q * TPR + tid];
        xnorm[tid] = sqrt(x2 * (1.0 + (H + 64) * 0x1.0p-52));
    }
    __syncthreads();
    // Phase 2: float logits certified against the reference's rounding; the
    // rest are queued for the sequential recomputation (phase 2b).
    const double gamma = static_cast<double>(H + rows + KS + 8) * 0x1.0p-53 * 1.01;
    for (int idx = tid; idx < ntr * E; idx += blockDim.x) {
        const int lt = idx / E, e = idx % E;
        double sum = 0.0;
        for (int q = 0; q < KS; ++q) sum += recv[(q * TPR + lt) * kRtCols + e];
        double A = xnorm[lt] * wnorm[e] * (1.0 + 0x1.0p-40);
        if (a.bias) {
            sum += static_cast<double>(bias_s[e]);
            A += fabs(static_cast<double>(bias_s[e]));
        }
        const double beta = gamma * A + 0x1.0p-1060;
        if (!rounding_certified(sum, beta)) {
            const int slot = atomicAdd(fb_count, 1);
            if (slot < kRtFallbacks) fb_list[slot] = lt * 256 + e;
            else sum = sequential_logit(a, t0 + lt0 + lt, e); // queue full: this thread does it
        }
        if (!isfinite(sum)) device_fail(a.st, HMOE_NON_FINITE_ROUTER);
        logit[lt * kRtCols + e] = static_cast<float>(sum);
    }
    __syncthreads();
    // Phase 2b, a warp per queued logit (settle_logit): the second-level
    // certificate settles almost all of them; the rest are summed in the
    // reference's order.  The received partials are consumed, so their
    // region stages the products.
    const int nfb = min(*fb_count, kRtFallbacks);
    const int slots = min(8, (kRtTokens * kRtCols * 8) / (8 * staged_logit_doubles(H)));
    for (int f = warp; f < nfb; f += blockDim.x >> 5) {
        const int lt = fb_list[f] >> 8, e = fb_list[f] & 255;
        const float lg =
            settle_logit(a, t0 + lt0 + lt, e, warp < slots ? recv + warp * staged_logit_doubles(H) : nullptr);
        if (lane == 0) {
            if (!isfinite(lg)) device_fail(a.st, HMOE_NON_FINITE_ROUTER);
            logit[lt * kRtCols + e] = lg;
        }
    }
    __syncthreads();
    // Phase 3: softmax, selection, renormalisation; one warp per token.
    for (int lt = warp; lt < ntr; lt += blockDim.x >> 5) {
        float lv[C];
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const int j = lane + 32 * c;
            lv[c] = j < E ? logit[lt * kRtCols + j] : 0.0f;
        }
        const size_t tok = static_cast<size_t>(t0 + lt0 + lt);
        select_token<C>(lv, E, a.k, a.softmax, a.renorm, evs + warp * kRtCols, a.ids + tok * a.k,
                        a.scores + tok * a.k, a.counts, token_block_counts(a, tok), a.st, false, nullptr);
    }
}

// ------------------------------------------------------------ decode router
//
// Decode-sized batches (T <= 16).  The per-8-token and tiled kernels split
// H over at most one cluster, so at T = 1 a handful of CTAs stream the whole
// router matrix and the SMs wait on that latency.  Here a grid of
// (H/128) x (E/32) small CTAs each forms FP64 partial dots of all T tokens
// with 32 experts over 128 hidden rows (lane = expert, warp = 16 rows, the
// 8 warps added in a fixed order) and adds them to zeroed [T][E] doubles
// with atomics, together with the norms of the certificate.  Atomic order
// varies from run to run, but every partial is a rounded sum of exact
// products with at most 24 + H/128 roundings on any chain, so the rounding
// certificate holds; certified logits are the reference's exact floats and
// the rest are settled as in the other kernels, so the result does not
// depend on that order.  The last CTA to finish (a ticket) certifies,
// settles and selects.
constexpr int kDecAutoTokens = 8; // chosen automatically up to here (T=1: 26.6 us vs 30.7 us for route_kernel,
                                  // T=4: 26.6 vs 32.7; at T=16 its serial selection tail makes it slower:
                                  // 47.1 vs 36.9)

struct DecodeArgs {
    RouteArgs a;
    double* acc; // [T][E] partial sums (zeroed)
    double* xn2; // [T] squared token norms (zeroed)
    double* wn2; // [E] squared expert-column norms (zeroed)
    int* ticket; // CTAs done (zeroed)
};

// Doubles of zeroed scratch the decode router needs for T tokens.
__host__ __device__ inline size_t decode_scratch_doubles(int T, int E) {
    return static_cast<size_t>(T) * E + T + E + 2;
}

template <int C>
__global__ void __launch_bounds__(256) route_decode_kernel(DecodeArgs d) {
    extern __shared__ __align__(16) double stage_buf[]; // [kDecSlots][H + 32]
    __shared__ float xs[kDecMaxTokens][kDecRows];       // token rows; softmax scratch at the end
    __shared__ double red[8][kDecMaxTokens][kDecCols];  // warp partials; logits at the end
    __shared__ double wred[8][kDecCols];
    __shared__ int last, fb_count, fb_list[kRouteFallbacks];
    __shared__ double wnorm_s[kMaxExperts], xnorm_s[kDecMaxTokens];
    __shared__ float bias_s[kMaxExperts];
    const RouteArgs& a = d.a;
    const int T = a.T, H = a.H, E = a.E;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r0 = blockIdx.x * kDecRows, e0 = blockIdx.y * kDecCols;
    for (int i = tid; i < T * kDecRows; i += blockDim.x)
        xs[i / kDecRows][i % kDecRows] = a.x[static_cast<size_t>(i / kDecRows) * H + r0 + i % kDecRows];
    __syncthreads();
    const int e = e0 + lane;
    double acc[kDecMaxTokens];
#pragma unroll
    for (int t = 0; t < kDecMaxTokens; ++t) acc[t] = 0.0;
    double wsq = 0.0;
#pragma unroll 4
    for (int j = 0; j < kDecRows / 8; ++j) {
        const int i = warp * (kDecRows / 8) + j;
        const double wd = e < E ? static_cast<double>(a.w[static_cast<size_t>(r0 + i) * E + e]) : 0.0;
        wsq = fma(wd, wd, wsq);
#pragma unroll
        for (int t = 0; t < kDecMaxTokens; ++t)
            if (t < T) acc[t] = fma(static_cast<double>(xs[t][i]), wd, acc[t]);
    }
#pragma unroll
    for (int t = 0; t < kDecMaxTokens; ++t)
        if (t < T) red[warp][t][lane] = acc[t];
    wred[warp][lane] = wsq;
    __syncthreads();
    for (int idx = tid; idx < T * kDecCols; idx += blockDim.x) {
        const int t = idx / kDecCols, l = idx % kDecCols;
        double s = 0.0;
        for (int w = 0; w < 8; ++w) s += red[w][t][l];
        if (e0 + l < E) atomicAdd(d.acc + static_cast<size_t>(t) * E + e0 + l, s);
    }
    if (tid < kDecCols && e0 + tid < E) {
        double s = 0.0;
        for (int w = 0; w < 8; ++w) s += wred[w][tid];
        atomicAdd(d.wn2 + e0 + tid, s);
    }
    if (blockIdx.y == 0 && tid < T) {
        double s = 0.0;
        for (int i = 0; i < kDecRows; ++i) {
            const double v = static_cast<double>(xs[tid][i]);
            s = fma(v, v, s);
        }
        atomicAdd(d.xn2 + tid, s);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        last = atomicAdd(d.ticket, 1) == static_cast<int>(gridDim.x * gridDim.y) - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // The last CTA: certify every logit, settle the queued ones, select.
    const DecodeTailSmem m{reinterpret_cast<float*>(&red[0][0][0]), &xs[0][0], wnorm_s, xnorm_s, bias_s, &fb_count,
                           fb_list, stage_buf};
    decode_finish<C>(
        a, [&](int idx) { return __ldcg(d.acc + idx); }, [&](int t) { return __ldcg(d.xn2 + t); },
        [&](int e) { return __ldcg(d.wn2 + e); }, m);
}

static_assert(kDecMaxTokens * kDecRows * 4 >= 8 * kMaxExperts * 4, "decode router: softmax scratch fits");
static_assert(8 * kDecMaxTokens * kDecCols * 8 >= kDecMaxTokens * kMaxExperts * 4, "decode router: logits fit");

// kernels::routerTopK drop-in (CudaKernels.cu:152-204): one warp per token,
// logits given, probabilities written back in place when softmax != 0.
template <int C>
__global__ void router_topk_kernel(float* logits, int T, int E, int k,
                                   int softmax, int renorm, uint32_t* ids,
                                   float* scores) {
    __shared__ float evs[8][kMaxExperts];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + warp;
    if (t >= T) return;
    float* row = logits + static_cast<size_t>(t) * E;
    float lv[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int j = lane + 32 * c;
        lv[c] = j < E ? row[j] : 0.0f;
    }
    select_token<C>(lv, E, k, softmax, renorm, evs[warp], ids + static_cast<size_t>(t) * k,
                    scores + static_cast<size_t>(t) * k, nullptr, nullptr, nullptr, softmax != 0, row);
}

// ------------------------------------------------------------ grouping

struct GroupArgs {
    const uint32_t* ids;   // [T, k]
    const float* scores;   // [T, k]
    const int32_t* counts; // [E] routed counts
    const int32_t* block_counts; // [ceil(T/kGroupBlock)][E] routed counts per token block
    int T, k, E, S;        // S shared experts
    int32_t* offsets;      // [E+S+1]
    uint32_t* perm_token;  // [T*(k+S)] token of each permuted row
    float* perm_weight;    // [T*(k+S)] routing weight of each row
    int32_t* inv;          // [T*(k+S)] row of (token, slot); slots k.. = shared
    const int32_t* expert_of_slot; // [E] placement (group b holds that expert), or null
    int32_t* slot_counts;  // [E] routed rows per placement slot (with a placement)
};

// Expert held by group b (routed groups follow the placement when given).
__device__ __forceinline__ int group_expert(const GroupArgs& g, int b) {
    return (b < g.E && g.expert_of_slot) ? g.expert_of_slot[b] : b;
}

__device__ __forceinline__ int group_count(const GroupArgs& g, int b) {
    return b < g.E ? g.counts[group_expert(g, b)] : g.T;
}

// Stable counting sort of the (token, slot) assignments, one CTA per block
// of kGroupBlock tokens.  Groups are laid out in slot order (ascending
// expert id without a placement), then the shared experts; inside a group
// tokens ascend, exactly as routeBatch appends them
// (CpuRouterBackend.cpp:78-90).  A row's position is the group offset, plus
// the group's rows in earlier token blocks (the router's per-block counts),
// plus the rank of the token among this block's tokens of that expert (a
// bit mask per expert).
__global__ void __launch_bounds__(256) group_kernel(GroupArgs g) {
    using Scan = cub::BlockScan<int, 256>;
    __shared__ typename Scan::TempStorage scan_tmp;
    __shared__ int off_s[2 * 256 + 1];
    __shared__ int slot_of[kMaxExperts];
    __shared__ int pre[kMaxExperts];
    __shared__ uint32_t mask[kMaxExperts][kGroupBlock / 32];
    const int tid = threadIdx.x, blk = blockIdx.x;
    const int tb0 = blk * kGroupBlock;
    const int nt = min(kGroupBlock, g.T - tb0);
    const int nb = g.E + g.S;
    // group offsets: exclusive scan of the group sizes (two per thread)
    int v[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int b = 2 * tid + q;
        v[q] = b < nb ? group_count(g, b) : 0;
    }
    int total = 0;
    Scan(scan_tmp).ExclusiveSum(v, v, total);
#pragma unroll
    for (int q = 0; q < 2; ++q)
        if (2 * tid + q < nb) off_s[2 * tid + q] = v[q];
    if (tid == 0) off_s[nb] = total;
    for (int b = tid; b < g.E; b += blockDim.x) slot_of[group_expert(g, b)] = b;
    for (int e = tid; e < g.E; e += blockDim.x) {
        int p = 0;
        for (int q = 0; q < blk; ++q) p += g.block_counts[q * g.E + e];
        pre[e] = p;
    }
    for (int i = tid; i < g.E * (kGroupBlock / 32); i += blockDim.x) (&mask[0][0])[i] = 0u;
    __syncthreads();
    if (blk == 0) {
        for (int b = tid; b <= nb; b += blockDim.x) g.offsets[b] = off_s[b];
        if (g.slot_counts)
            for (int b = tid; b < g.E; b += blockDim.x) g.slot_counts[b] = group_count(g, b);
    }
    const int t = tb0 + tid;
    const uint32_t* r = g.ids + static_cast<size_t>(t) * g.k;
    if (tid < nt)
        for (int j = 0; j < g.k; ++j) atomicOr(&mask[r[j]][tid >> 5], 1u << (tid & 31));
    __syncthreads();
    if (tid >= nt) return;
    const int slots = g.k + g.S;
    const int w = tid >> 5;
    for (int j = 0; j < g.k; ++j) {
        const int e = static_cast<int>(r[j]);
        int rank = __popc(mask[e][w] & ((1u << (tid & 31)) - 1u));
        for (int q = 0; q < w; ++q) rank += __popc(mask[e][q]);
        const int row = off_s[slot_of[e]] + pre[e] + rank;
        g.perm_token[row] = static_cast<uint32_t>(t);
        g.perm_weight[row] = g.scores[static_cast<size_t>(t) * g.k + j];
        g.inv[static_cast<size_t>(t) * slots + j] = row;
    }
    for (int sx = 0; sx < g.S; ++sx) {
        const int row = off_s[g.E + sx] + t;
        g.perm_token[row] = static_cast<uint32_t>(t);
        g.perm_weight[row] = 1.0f;
        g.inv[static_cast<size_t>(t) * slots + g.k + sx] = row;
    }
}

// ------------------------------------------------------------ launchers


// Router kernel choice: 0 = automatic, 1 = per-8-token cluster kernel,
// 2 = tiled kernel, 3 = decode kernel (hmoe_set_route_variant).
int g_route_variant = 0;
constexpr int kTiledMinTokens = 512;

bool decode_shape_ok(int T, int H, int E) { return T <= kDecMaxTokens && H % kDecRows == 0 && E <= kMaxExperts; }

size_t route_decode_scratch_bytes(size_t T, int H, int E) {
    if (!decode_shape_ok(static_cast<int>(std::min<size_t>(T, INT_MAX)), H, E)) return 0;
    return decode_scratch_doubles(static_cast<int>(T), E) * 8;
}

hmoe_status launch_route_decode(const RouteArgs& a, double* scratch, cudaStream_t stream) {
    DecodeArgs d{a, scratch, scratch + static_cast<size_t>(a.T) * a.E, scratch + static_cast<size_t>(a.T) * a.E + a.T,
                 reinterpret_cast<int*>(scratch + static_cast<size_t>(a.T) * a.E + a.T + a.E)};
    const dim3 grid(static_cast<unsigned>(a.H / kDecRows), static_cast<unsigned>((a.E + kDecCols - 1) / kDecCols));
    const int smem = kDecSlots * staged_logit_doubles(a.H) * 8;
    cudaError_t err = cudaErrorInvalidValue;
#define HMOE_DECODE_CASE(CC)                                                                                 \
    case CC: {                                                                                               \
        err = set_smem_limit(reinterpret_cast<const void*>(route_decode_kernel<CC>), smem);                  \
        if (err != cudaSuccess) break;                                                                       \
        route_decode_kernel<CC><<<grid, 256, smem, stream>>>(d);                                             \
        err = cudaGetLastError();                                                                            \
        break;                                                                                               \
    }
    switch ((a.E + 31) / 32) {
        HMOE_DECODE_CASE(1)
        HMOE_DECODE_CASE(2)
        HMOE_DECODE_CASE(3)
        HMOE_DECODE_CASE(4)
        HMOE_DECODE_CASE(5)
        HMOE_DECODE_CASE(6)
        HMOE_DECODE_CASE(7)
        HMOE_DECODE_CASE(8)
    default: return HMOE_UNSUPPORTED;
    }
#undef HMOE_DECODE_CASE
    if (err != cudaSuccess) {
        set_last_error("hmoe decode route kernel launch", err);
        return HMOE_CUDA_ERROR;
    }
    return check_launch("hmoe decode route kernel");
}

bool tiled_shape_ok(int H, int E) { return E <= kRtCols && E % 4 == 0 && H % kRtRows == 0; }

hmoe_status launch_route_tiled(const RouteArgs& a, cudaStream_t stream) {
    CUtensorMap mx, mw;
    if (!map_f32_rows_sw128(&mx, a.x, static_cast<uint64_t>(a.H), static_cast<uint64_t>(a.T), 32, kRtTokens) ||
        !map_f32_rows_sw128(&mw, a.w, static_cast<uint64_t>(a.E), static_cast<uint64_t>(a.H), 32, kRtRows)) {
        set_last_error_text("hmoe: cuTensorMapEncodeTiled failed (tiled router)");
        return HMOE_CUDA_ERROR;
    }
    const int tiles = (a.T + kRtTokens - 1) / kRtTokens;
    int KS = 1; // split H over a cluster until the tiles fill about two CTAs per SM
    while (KS < 8 && tiles * KS < 250 && a.H % (kRtRows * KS * 2) == 0) KS *= 2;
    constexpr int smem = tiled_smem().total;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(KS), static_cast<unsigned>(tiles));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(KS);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaErrorInvalidValue;
#define HMOE_TILED_CASE(CC)                                                                                 \
    case CC: {                                                                                              \
        err = set_smem_limit(reinterpret_cast<const void*>(route_tiled_kernel<CC>), smem);                  \
        if (err != cudaSuccess) break;                                                                      \
        err = cudaLaunchKernelEx(&cfg, route_tiled_kernel<CC>, mx, mw, a, KS);                              \
        break;                                                                                              \
    }
    switch ((a.E + 31) / 32) {
        HMOE_TILED_CASE(1)
        HMOE_TILED_CASE(2)
        HMOE_TILED_CASE(3)
        HMOE_TILED_CASE(4)
    default: return HMOE_UNSUPPORTED;
    }
#undef HMOE_TILED_CASE
    if (err != cudaSuccess) {
        set_last_error("hmoe tiled route kernel launch", err);
        return HMOE_CUDA_ERROR;
    }
    return check_launch("hmoe tiled route kernel");
}

hmoe_status launch_route(const float* x, const float* w, const float* bias,
                         int T, int H, int E, int k, int softmax, int renorm,
                         uint32_t* ids, float* scores, int32_t* counts,
                         int32_t* block_counts, double* decode_scratch, DeviceStatus* st, cudaStream_t stream) {
    if (T <= 0) return HMOE_OK;
    if (E <= 0 || E > kMaxExperts || k <= 0 || k > E || k > kMaxTopK || H <= 0 || H % 8)
        return HMOE_INVALID_ARGUMENT;
    // hidden rows and router rows arrive by bulk copies (16-byte aligned)
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % 16) return HMOE_INVALID_ARGUMENT;
    const bool tiled_ok = tiled_shape_ok(H, E);
    if (g_route_variant == 2 && !tiled_ok) {
        set_last_error_text("hmoe route: the tiled router needs E <= 128, E % 4 == 0 and H % 32 == 0");
        return HMOE_UNSUPPORTED;
    }
    if (g_route_variant == 2 || (g_route_variant == 0 && tiled_ok && T >= kTiledMinTokens)) {
        RouteArgs a{x, w, bias, T, H, E, k, softmax, renorm, ids, scores, counts, st, block_counts};
        return launch_route_tiled(a, stream);
    }
    const bool decode_ok = decode_shape_ok(T, H, E) && decode_scratch;
    if (g_route_variant == 3 && !decode_ok) {
        set_last_error_text("hmoe route: the decode router needs T <= 16, H % 128 == 0 and its scratch");
        return HMOE_UNSUPPORTED;
    }
    if (g_route_variant == 3 || (g_route_variant == 0 && decode_ok && T <= kDecAutoTokens)) {
        RouteArgs a{x, w, bias, T, H, E, k, softmax, renorm, ids, scores, counts, st, block_counts};
        return launch_route_decode(a, decode_scratch, stream);
    }
    const int EQ = (E + 3) / 4;
    const int P = std::min(32, 256 / EQ); // row lanes; phase 2 maps token t to lane t mod P
    if (EQ * P > 256 || P < 1) return HMOE_UNSUPPORTED;
    const int E_pad = 4 * EQ;
    const int smem = route_smem(E, E_pad, P).total;
    const int rows = (T + kRouteTokens - 1) / kRouteTokens;
    int KS = 1; // split H over a cluster until there are about 2 CTAs per SM
    while (KS < 8 && rows * KS < 2 * 148 && (H / (KS * 2)) % 8 == 0 && H / (KS * 2) >= 64) KS *= 2;
    RouteArgs a{x, w, bias, T, H, E, k, softmax, renorm, ids, scores, counts, st, block_counts};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(KS), static_cast<unsigned>(rows));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(KS);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const int C = (E + 31) / 32;
    cudaError_t err = cudaErrorInvalidValue;
#define HMOE_ROUTE_CASE(CC)                                                                          \
    case CC: {                                                                                       \
        err = set_smem_limit(reinterpret_cast<const void*>(route_kernel<CC>), smem);                \
        if (err != cudaSuccess) break;                                                               \
        err = cudaLaunchKernelEx(&cfg, route_kernel<CC>, a, EQ, P, KS);                              \
        break;                                                                                       \
    }
    switch (C) {
        HMOE_ROUTE_CASE(1)
        HMOE_ROUTE_CASE(2)
        HMOE_ROUTE_CASE(3)
        HMOE_ROUTE_CASE(4)
        HMOE_ROUTE_CASE(5)
        HMOE_ROUTE_CASE(6)
        HMOE_ROUTE_CASE(7)
        HMOE_ROUTE_CASE(8)
    default: return HMOE_UNSUPPORTED;
    }
#undef HMOE_ROUTE_CASE
    if (err != cudaSuccess) {
        set_last_error("hmoe route kernel launch", err);
        return HMOE_CUDA_ERROR;
    }
    return check_launch("hmoe route kernel");
}

hmoe_status launch_group(const uint32_t* ids, const float* scores, const int32_t* counts,
                         const int32_t* block_counts, int T, int k, int E, int S, int32_t* offsets,
                         uint32_t* perm_token, float* perm_weight, int32_t* inv, const int32_t* expert_of_slot,
                         int32_t* slot_counts, cudaStream_t stream) {
    if (T <= 0) return HMOE_OK;
    if (E + S > 2 * 256) return HMOE_UNSUPPORTED;
    GroupArgs g{ids, scores, counts, block_counts, T, k, E, S, offsets, perm_token, perm_weight, inv,
                expert_of_slot, slot_counts};
    group_kernel<<<(T + kGroupBlock - 1) / kGroupBlock, 256, 0, stream>>>(g);
    return check_launch("hmoe group kernel");
}

} // namespace hmoe

extern "C" hmoe_status hmoe_router_topk(float* logits, size_t tokens,
                                        size_t experts, size_t top_k,
                                        int softmax, int renormalize,
                                        uint32_t* selected_ids,
                                        float* selected_scores, void* stream) {
    using namespace hmoe;
    if (tokens == 0) return HMOE_OK;
    if (!logits || !selected_ids || !selected_scores || experts == 0 ||
        top_k == 0 || top_k > experts || experts > kMaxExperts || top_k > kMaxTopK ||
        tokens > static_cast<size_t>(INT_MAX))
        return HMOE_INVALID_ARGUMENT;
    const int C = static_cast<int>((experts + 31) / 32);
    const unsigned grid = static_cast<unsigned>((tokens + 7) / 8);
    const int T = static_cast<int>(tokens), E = static_cast<int>(experts), K = static_cast<int>(top_k);
    cudaStream_t s = as_stream(stream);
#define HMOE_TOPK_CASE(CC)                                                                         \
    case CC:                                                                                       \
        router_topk_kernel<CC><<<grid, 256, 0, s>>>(logits, T, E, K, softmax, renormalize,          \
                                                   selected_ids, selected_scores);                 \
        break;
    switch (C) {
        HMOE_TOPK_CASE(1)
        HMOE_TOPK_CASE(2)
        HMOE_TOPK_CASE(3)
        HMOE_TOPK_CASE(4)
        HMOE_TOPK_CASE(5)
        HMOE_TOPK_CASE(6)
        HMOE_TOPK_CASE(7)
        HMOE_TOPK_CASE(8)
    default: return HMOE_UNSUPPORTED;
    }
#undef HMOE_TOPK_CASE
    return check_launch("CUDA router top-k kernel");
}

extern "C" hmoe_status hmoe_set_route_variant(int32_t variant) {
    if (variant < 0 || variant > 3) return HMOE_INVALID_ARGUMENT;
    hmoe::g_route_variant = variant;
    return HMOE_OK;
}
