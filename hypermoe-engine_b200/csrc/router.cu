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
#include "sm100.cuh"

#include <cooperative_groups.h>

#include <cfloat>
#include <algorithm>
#include <climits>

namespace cg = cooperative_groups;

namespace hmoe {

constexpr int kRouteTokens = 8;     // tokens per CTA in the fused router
constexpr int kRouteChunk = 256;    // hidden rows staged per pass (= threads per CTA)
constexpr int kRouteFallbacks = 64; // queued sequential recomputations per CTA
constexpr int kRouteStages = 4;     // router-matrix slabs in flight
constexpr int kMaxExperts = 256; // E_pad <= 256 (8 candidates per lane)
constexpr int kMaxTopK = 32;

struct RouteArgs {
    const float* x;     // [T, H]
    const float* w;     // [H, E]
    const float* bias;  // [E] or null
    int T, H, E, k, softmax, renorm;
    uint32_t* ids;      // [T, k]
    float* scores;      // [T, k]
    int32_t* counts;    // [E] (zeroed by the caller), may be null
    DeviceStatus* st;
};

__device__ __forceinline__ bool better(float pa, int ia, float pb, int ib) {
    return pa > pb || (pa == pb && ia < ib);
}

// Distance check of a double sum against float rounding boundaries.
__device__ __forceinline__ bool rounding_certified(double s, double beta) {
    const float f = static_cast<float>(s);
    const double fd = static_cast<double>(f);
    const double lo = 0.5 * (fd + static_cast<double>(nextafterf(f, -FLT_MAX * 2.0f)));
    const double hi = 0.5 * (fd + static_cast<double>(nextafterf(f, FLT_MAX * 2.0f)));
    return (s - beta > lo) && (s + beta < hi);
}

// Selection, renormalisation and near-tie accounting for one token held by
// one warp: lanes own candidates j = lane + 32*c.  `lv` are exact logits.
template <int C>
__device__ void select_token(const float (&lv)[C], int E, int k, int softmax,
                             int renorm, float* ev_smem, uint32_t* ids_out,
                             float* scores_out, int32_t* counts,
                             DeviceStatus* st, bool write_probs,
                             float* probs_out) {
    const int lane = threadIdx.x & 31;
    float p[C];
    float m = -FLT_MAX * 2.0f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int j = lane + 32 * c;
        if (j < E) m = fmaxf(m, lv[c]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    bool ok = true;
    if (softmax) {
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const int j = lane + 32 * c;
            const float d = lv[c] - m; // float subtraction, as the reference
            const float e = static_cast<float>(exp(static_cast<double>(d)));
            p[c] = e;
            if (j < E) ev_smem[j] = e;
        }
        __syncwarp();
        // The reference sums the E floats in double in expert order.  When
        // every term is >= 2^-22 all of them are multiples of 2^-45 and the
        // total is below 2^8, so the double sum is exact in any order and a
        // tree sum gives the same bits; otherwise sum sequentially.
        double den = 0.0;
        bool small = false;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const int j = lane + 32 * c;
            if (j < E) {
                den += static_cast<double>(p[c]);
                small |= p[c] < 0x1.0p-22f;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
        if (__any_sync(0xffffffffu, small)) {
            den = 0.0;
            if (lane == 0)
                for (int j = 0; j < E; ++j) den += static_cast<double>(ev_smem[j]);
            den = __shfl_sync(0xffffffffu, den, 0);
        }
        __syncwarp();
        if (!(isfinite(den) && den > 0.0)) ok = false;
#pragma unroll
        for (int c = 0; c < C; ++c) p[c] = static_cast<float>(static_cast<double>(p[c]) / den);
    } else {
#pragma unroll
        for (int c = 0; c < C; ++c) p[c] = lv[c];
    }
    if (write_probs) {
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const int j = lane + 32 * c;
            if (j < E) probs_out[j] = p[c];
        }
    }
    // Selection key: a NaN probability (only possible for a token whose
    // logits or denominator are not finite, which is flagged above and by
    // the logit pass) ranks lowest, so every round still picks a valid id.
#pragma unroll
    for (int c = 0; c < C; ++c)
        if (p[c] != p[c]) {
            p[c] = -FLT_MAX * 2.0f;
            ok = false;
        }
    unsigned selected = 0; // bit c: candidate c of this lane taken
    double rsum = 0.0;
    float prev_p = 0.0f, prev_l = 0.0f;
    float chosen[kMaxTopK];
    bool tie = false;
    const int rounds = k < E ? k + 1 : k; // one extra to see rank k
    for (int r = 0; r < rounds; ++r) {
        float bp = -FLT_MAX * 2.0f, bl = 0.0f;
        int bi = INT_MAX;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const int j = lane + 32 * c;
            if (j < E && !((selected >> c) & 1u) && better(p[c], j, bp, bi)) {
                bp = p[c];
                bi = j;
                bl = lv[c];
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float op = __shfl_xor_sync(0xffffffffu, bp, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const float ol = __shfl_xor_sync(0xffffffffu, bl, o);
            if (better(op, oi, bp, bi)) {
                bp = op;
                bi = oi;
                bl = ol;
            }
        }
        if (r > 0 && softmax && bl != prev_l) {
            const int d = abs(__float_as_int(prev_p) - __float_as_int(bp));
            if (d <= 2) tie = true;
        }
        prev_p = bp;
        prev_l = bl;
        if (r == k) break;
        if (bi >= E) { // unreachable: E - r > 0 candidates remain
            bi = 0;
            ok = false;
        }
        if ((bi & 31) == lane) selected |= 1u << (bi >> 5);
        chosen[r] = bp;
        rsum += static_cast<double>(bp);
        if (lane == 0) {
            ids_out[r] = static_cast<uint32_t>(bi);
            if (counts) atomicAdd(counts + bi, 1);
        }
    }
    if (lane == 0) {
        if (renorm) {
            if (!(isfinite(rsum) && rsum != 0.0)) ok = false;
            if (ok) {
                for (int r = 0; r < k; ++r)
                    scores_out[r] = static_cast<float>(static_cast<double>(chosen[r]) / rsum);
            } else {
                for (int r = 0; r < k; ++r) scores_out[r] = chosen[r];
                scores_out[0] = __int_as_float(0x7fc00000); // NaN, CudaKernels.cu:201-202
            }
        } else {
            for (int r = 0; r < k; ++r) scores_out[r] = chosen[r];
            if (!ok) scores_out[0] = __int_as_float(0x7fc00000);
        }
        if (!ok) device_fail(st, HMOE_NON_FINITE_ROUTER);
        if (tie && st) atomicAdd(&st->near_ties, 1);
    }
}

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

// The reference's sequential double accumulation for one (token, expert),
// by a single thread (used only when the per-CTA queue overflows).
__device__ double sequential_logit(const RouteArgs& a, int tok, int e) {
    const float* xr = a.x + static_cast<size_t>(tok) * a.H;
    double s = 0.0;
    for (int i = 0; i < a.H; ++i)
        s = fma(static_cast<double>(xr[i]), static_cast<double>(a.w[static_cast<size_t>(i) * a.E + e]), s);
    if (a.bias) s = fma(1.0, static_cast<double>(a.bias[e]), s);
    if (a.st) atomicAdd(&a.st->sequential_logits, 1);
    return s;
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
        // Phase 2b: warp-cooperative sequential recomputation.  Each lane
        // forms one exact product per 32-row chunk; the chunks' products are
        // loaded four chunks ahead of the dependent double additions.
        const int nfb = min(*fb_count, kRouteFallbacks);
        for (int f = warp; f < nfb; f += blockDim.x >> 5) {
            const int t = fb_list[f] >> 8, e = fb_list[f] & 255;
            const float* xr = a.x + static_cast<size_t>(t0 + t) * H;
            auto prod_at = [&](int c) {
                const int i = c * 32 + lane;
                // products of two floats are exact in double; rows past H add +0.0
                return i < H ? static_cast<double>(xr[i]) * static_cast<double>(a.w[static_cast<size_t>(i) * E + e])
                             : 0.0;
            };
            const int nch = (H + 31) / 32;
            double q[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) q[u] = prod_at(u);
            double s = 0.0;
            for (int c = 0; c < nch; c += 4) {
                double nq[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) nq[u] = c + 4 + u < nch ? prod_at(c + 4 + u) : 0.0;
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) s += __shfl_sync(0xffffffffu, q[u], jj);
#pragma unroll
                for (int u = 0; u < 4; ++u) q[u] = nq[u];
            }
            if (a.bias) s += static_cast<double>(a.bias[e]);
            if (lane == 0) {
                if (!isfinite(s)) device_fail(a.st, HMOE_NON_FINITE_ROUTER);
                logit[t * E_pad + e] = static_cast<float>(s);
                if (a.st) atomicAdd(&a.st->sequential_logits, 1);
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
                            a.scores + tok * a.k, a.counts, a.st, false, nullptr);
        }
    }
    cluster.sync(); // keep every CTA's shared memory alive until rank 0 is done
}

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
                    scores + static_cast<size_t>(t) * k, nullptr, nullptr, softmax != 0, row);
}

// ------------------------------------------------------------ grouping

struct GroupArgs {
    const uint32_t* ids;   // [T, k]
    const float* scores;   // [T, k]
    const int32_t* counts; // [E] routed counts
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

// One CTA per expert (routed then shared).  Tokens are placed in ascending
// order inside the expert's group, exactly as routeBatch appends them
// (CpuRouterBackend.cpp:78-90); groups are laid out in ascending expert id.
__global__ void __launch_bounds__(256) group_kernel(GroupArgs g) {
    __shared__ int red[8];
    __shared__ int warp_hits[8];
    __shared__ int base_s;
    const int b = blockIdx.x;          // group (placement slot for routed experts)
    const int e = group_expert(g, b);  // expert of the group
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // Offset of group b from the counts of the groups before it.
    int off = 0;
    for (int j = tid; j < b; j += blockDim.x) off += group_count(g, j);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) off += __shfl_xor_sync(0xffffffffu, off, o);
    if (lane == 0) red[warp] = off;
    __syncthreads();
    if (tid == 0) {
        int o = 0;
        for (int w = 0; w < 8; ++w) o += red[w];
        g.offsets[b] = o;
        if (b == g.E + g.S - 1) g.offsets[b + 1] = o + group_count(g, b);
        if (g.slot_counts && b < g.E) g.slot_counts[b] = group_count(g, b);
        base_s = o;
    }
    __syncthreads();
    int base = base_s;
    const int slots = g.k + g.S;
    if (b >= g.E) {
        const int s = b - g.E;
        for (int t = tid; t < g.T; t += blockDim.x) {
            const int row = base + t;
            g.perm_token[row] = static_cast<uint32_t>(t);
            g.perm_weight[row] = 1.0f;
            g.inv[static_cast<size_t>(t) * slots + g.k + s] = row;
        }
        return;
    }
    for (int t0 = 0; t0 < g.T; t0 += blockDim.x) {
        const int t = t0 + tid;
        int slot = -1;
        if (t < g.T) {
            const uint32_t* r = g.ids + static_cast<size_t>(t) * g.k;
            for (int j = 0; j < g.k; ++j)
                if (r[j] == static_cast<uint32_t>(e)) slot = j;
        }
        const unsigned mask = __ballot_sync(0xffffffffu, slot >= 0);
        if (lane == 0) warp_hits[warp] = __popc(mask);
        __syncthreads();
        int before = 0, chunk = 0;
        for (int w = 0; w < 8; ++w) {
            before += w < warp ? warp_hits[w] : 0;
            chunk += warp_hits[w];
        }
        if (slot >= 0) {
            const int row = base + before + __popc(mask & ((1u << lane) - 1u));
            g.perm_token[row] = static_cast<uint32_t>(t);
            g.perm_weight[row] = g.scores[static_cast<size_t>(t) * g.k + slot];
            g.inv[static_cast<size_t>(t) * slots + slot] = row;
        }
        base += chunk;
        __syncthreads();
    }
}

// ------------------------------------------------------------ launchers


hmoe_status launch_route(const float* x, const float* w, const float* bias,
                         int T, int H, int E, int k, int softmax, int renorm,
                         uint32_t* ids, float* scores, int32_t* counts,
                         DeviceStatus* st, cudaStream_t stream) {
    if (T <= 0) return HMOE_OK;
    if (E <= 0 || E > kMaxExperts || k <= 0 || k > E || k > kMaxTopK || H <= 0 || H % 8)
        return HMOE_INVALID_ARGUMENT;
    // hidden rows and router rows arrive by bulk copies (16-byte aligned)
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % 16) return HMOE_INVALID_ARGUMENT;
    const int EQ = (E + 3) / 4;
    const int P = std::min(32, 256 / EQ); // row lanes; phase 2 maps token t to lane t mod P
    if (EQ * P > 256 || P < 1) return HMOE_UNSUPPORTED;
    const int E_pad = 4 * EQ;
    const int smem = route_smem(E, E_pad, P).total;
    const int rows = (T + kRouteTokens - 1) / kRouteTokens;
    int KS = 1; // split H over a cluster until there are about 2 CTAs per SM
    while (KS < 8 && rows * KS < 2 * 148 && (H / (KS * 2)) % 8 == 0 && H / (KS * 2) >= 64) KS *= 2;
    RouteArgs a{x, w, bias, T, H, E, k, softmax, renorm, ids, scores, counts, st};
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
        static int attr_set = 0;                                                                     \
        if (smem > attr_set) {                                                                       \
            cudaFuncSetAttribute(route_kernel<CC>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); \
            attr_set = smem;                                                                         \
        }                                                                                            \
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

hmoe_status launch_group(const uint32_t* ids, const float* scores, const int32_t* counts, int T, int k,
                         int E, int S, int32_t* offsets, uint32_t* perm_token, float* perm_weight,
                         int32_t* inv, const int32_t* expert_of_slot, int32_t* slot_counts,
                         cudaStream_t stream) {
    GroupArgs g{ids, scores, counts, T, k, E, S, offsets, perm_token, perm_weight, inv, expert_of_slot,
                slot_counts};
    group_kernel<<<E + S, 256, 0, stream>>>(g);
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
