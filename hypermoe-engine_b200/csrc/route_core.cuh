// route_core.cuh -- the router's exact-logit and selection building blocks,
// shared by the router kernels (router.cu) and the decode layer kernel
// (decode_layer.cu): the rounding certificate, the settling of queued
// logits (second-level certificate, then the reference's sequential sum),
// the softmax / top-k / renormalisation of one token by one warp, and the
// decode routers' finish over T x E double logits.  The contract these
// implement is stated at the top of router.cu.
#pragma once

#include "common.cuh"
#include "layer.cuh"

#include <cfloat>
#include <climits>

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
    int32_t* block_counts; // [ceil(T/kGroupBlock)][E] per token block (zeroed), may be null
};

// Selected-expert counts of token block tok / kGroupBlock (for the grouping).
__device__ __forceinline__ int32_t* token_block_counts(const RouteArgs& a, size_t tok) {
    return a.block_counts ? a.block_counts + (tok / kGroupBlock) * a.E : nullptr;
}

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
                             float* scores_out, int32_t* counts, int32_t* block_counts,
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
    float mine = 0.0f; // lane r < k: the rank-r probability and expert
    int myid = 0;
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
        // Warp argmax in the order of better(): the largest value of an
        // order-preserving key (-0.0 keyed as +0.0, which compare equal),
        // then the smallest index among the lanes holding it; the owner of
        // that index holds it as its own best candidate.
        {
            uint32_t key = __float_as_uint(bp + 0.0f);
            key = (key & 0x80000000u) ? ~key : (key | 0x80000000u);
            const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
            const uint32_t imin =
                __reduce_min_sync(0xffffffffu, key == kmax ? static_cast<uint32_t>(bi) : 0xffffffffu);
            const int owner = static_cast<int>(imin & 31u);
            bp = __shfl_sync(0xffffffffu, bp, owner);
            bl = __shfl_sync(0xffffffffu, bl, owner);
            bi = static_cast<int>(imin);
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
        if (lane == r) {
            mine = bp;
            myid = bi;
        }
        rsum += static_cast<double>(bp); // rank order, as the reference
    }
    // Lane r writes rank r: the renormalised score (a double division, as
    // the reference) or, for a token flagged non-finite, the raw scores with
    // NaN in slot 0 (CudaKernels.cu:201-202).
    if (renorm && !(isfinite(rsum) && rsum != 0.0)) ok = false;
    ok = __all_sync(0xffffffffu, ok);
    if (lane < k) {
        float sc = mine;
        if (renorm && ok) sc = static_cast<float>(static_cast<double>(mine) / rsum);
        if (!ok && lane == 0) sc = __int_as_float(0x7fc00000);
        ids_out[lane] = static_cast<uint32_t>(myid);
        scores_out[lane] = sc;
        if (counts) atomicAdd(counts + myid, 1);
        if (block_counts) atomicAdd(block_counts + myid, 1);
    }
    if (lane == 0) {
        if (!ok) device_fail(st, HMOE_NON_FINITE_ROUTER);
        if (tie && st) atomicAdd(&st->near_ties, 1);
    }
}

// The reference's sequential double accumulation for one (token, expert),
// by a single thread (used only when the per-CTA queue overflows).
__device__ inline double sequential_logit(const RouteArgs& a, int tok, int e) {
    const float* xr = a.x + static_cast<size_t>(tok) * a.H;
    double s = 0.0;
    for (int i = 0; i < a.H; ++i)
        s = fma(static_cast<double>(xr[i]), static_cast<double>(a.w[static_cast<size_t>(i) * a.E + e]), s);
    if (a.bias) s = fma(1.0, static_cast<double>(a.bias[e]), s);
    if (a.st) atomicAdd(&a.st->sequential_logits, 1);
    return s;
}

// The same sequential sum by a whole warp (result on every lane): each lane
// forms one exact product per 32-row chunk, the products are loaded four
// chunks ahead, and the dependent double additions run in row order through
// shuffles.
__device__ inline double warp_sequential_logit(const RouteArgs& a, int tok, int e) {
    const int lane = threadIdx.x & 31;
    const int H = a.H, E = a.E;
    const float* xr = a.x + static_cast<size_t>(tok) * H;
    auto prod_at = [&](int c) {
        const int i = c * 32 + lane;
        // products of two floats are exact in double; rows past H add +0.0
        return i < H ? static_cast<double>(xr[i]) * static_cast<double>(a.w[static_cast<size_t>(i) * E + e]) : 0.0;
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
    return s;
}

__device__ __forceinline__ void two_sum(double a, double b, double& s, double& err) {
    s = a + b;
    const double bb = s - a;
    err = (a - (s - bb)) + (b - bb);
}

// Shared-memory doubles a warp needs to stage the H products of one logit.
__host__ __device__ constexpr int staged_logit_doubles(int H) { return H + 32; }

// The H exact products x_i * W_ie of one logit, staged by the whole warp in
// 32 segments of H/32 rows: row i at buf[i + i/(H/32)] (one pad per
// segment, so the lanes' segment walks below hit distinct banks).
// Needs H % 32 == 0.
__device__ inline void stage_products(const RouteArgs& a, int tok, int e, double* buf) {
    const int lane = threadIdx.x & 31;
    const int H = a.H, E = a.E, seg = H / 32;
    const float* xr = a.x + static_cast<size_t>(tok) * H;
    // 16 rows per lane in flight at a time: the router column is strided
    // (one 4-byte load per row), so the latency, not the bytes, sets the time
    for (int i0 = lane; i0 < H; i0 += 32 * 16) {
        float xv[16], wv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int i = i0 + 32 * j;
            xv[j] = i < H ? __ldg(xr + i) : 0.0f;
            wv[j] = i < H ? __ldg(a.w + static_cast<size_t>(i) * E + e) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int i = i0 + 32 * j;
            if (i < H) buf[i + i / seg] = static_cast<double>(xv[j]) * static_cast<double>(wv[j]);
        }
    }
    __syncwarp();
}

// Second-level certificate of one logit from its staged products, by a
// whole warp (result on every lane), tried before the sequential
// recomputation.  The reference's sum s_H = fl(...fl(p_1 + p_2)... + p_H)
// differs from the exact sum S_H by at most u/(1-u) * sum_i |s_i| <=
// u/(1-u) * sum_i |S_i| + H^2 u^2 P (S_i the exact partial sums,
// P = sum |p_i|, u = 2^-53).  The partial sums of a random-signed sum grow
// like sqrt(i), so this is far tighter than the (H-1) u P of the first
// certificate.  Lane l walks segment l; S_i comes from compensated (TwoSum)
// sums and a warp scan.  Returns whether the float logit (bias added last,
// as the reference does) is settled, and sets *out to it.
__device__ inline bool refined_logit(const RouteArgs& a, int e, const double* buf, float* out) {
    const int lane = threadIdx.x & 31;
    const int H = a.H, seg = H / 32;
    const double* sb = buf + lane * (seg + 1);
    double hi = 0.0, lo = 0.0, pabs = 0.0;
    for (int i = 0; i < seg; ++i) {
        const double p = sb[i];
        double err;
        two_sum(hi, p, hi, err);
        lo += err;
        pabs += fabs(p);
    }
    // inclusive scan of the segment sums over the lanes (double-double)
    double ih = hi, il = lo;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double oh = __shfl_up_sync(0xffffffffu, ih, o), ol = __shfl_up_sync(0xffffffffu, il, o);
        if (lane >= o) {
            double err;
            two_sum(oh, ih, ih, err);
            il = il + ol + err;
        }
    }
    double sh = __shfl_up_sync(0xffffffffu, ih, 1), sl = __shfl_up_sync(0xffffffffu, il, 1);
    if (lane == 0) sh = sl = 0.0;
    const double th = __shfl_sync(0xffffffffu, ih, 31), tl = __shfl_sync(0xffffffffu, il, 31);
    // walk the segment again from its prefix: sum of |S_i|
    double sabs = 0.0;
    for (int i = 0; i < seg; ++i) {
        double err;
        two_sum(sh, sb[i], sh, err);
        sl += err;
        sabs += fabs(sh + sl);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        sabs += __shfl_xor_sync(0xffffffffu, sabs, o);
        pabs += __shfl_xor_sync(0xffffffffu, pabs, o);
    }
    const double u = 0x1.0p-53;
    const double hh = static_cast<double>(H + 64);
    // |s_H - S_H| (reference) and |t - S_H| (this compensated sum), with
    // generous slack for the roundings of the bound itself.
    const double beta_ref = sabs * u * (1.0 + 0x1.0p-30) + 8.0 * hh * hh * u * u * pabs;
    const double b = a.bias ? static_cast<double>(a.bias[e]) : 0.0;
    const double z = th + (tl + b);
    const double beta = beta_ref * (1.0 + 4.0 * u) + 8.0 * u * (fabs(z) + fabs(b) + fabs(tl) + beta_ref) +
                        8.0 * hh * hh * u * u * pabs + 0x1.0p-1060;
    *out = static_cast<float>(z);
    return isfinite(z) && rounding_certified(z, beta);
}

// The reference's sequential sum over the staged products: lane 0 runs the
// dependent additions in row order (result on lane 0).
__device__ inline double staged_sequential_logit(const RouteArgs& a, int e, const double* buf) {
    const int lane = threadIdx.x & 31;
    const int H = a.H, seg = H / 32;
    double s = 0.0;
    if (lane == 0) {
        for (int l = 0; l < 32; ++l) {
            const double* sb = buf + l * (seg + 1);
#pragma unroll 8
            for (int i = 0; i < seg; ++i) s += sb[i];
        }
        if (a.bias) s += static_cast<double>(a.bias[e]);
    }
    __syncwarp(); // buf is reused by this warp's next logit
    return s;
}

// One queued logit by a whole warp: the second-level certificate over the
// staged products, else the sequential sum (staged when a buffer is given,
// otherwise from global memory).  Result on lane 0; counts the sequential
// recomputations.
__device__ inline float settle_logit(const RouteArgs& a, int tok, int e, double* buf) {
    const int lane = threadIdx.x & 31;
    if (buf && a.H % 32 == 0) {
        stage_products(a, tok, e, buf);
        float lg;
        if (refined_logit(a, e, buf, &lg)) {
            __syncwarp();
            return lg;
        }
        const double s = staged_sequential_logit(a, e, buf);
        if (lane == 0 && a.st) atomicAdd(&a.st->sequential_logits, 1);
        return static_cast<float>(s);
    }
    const double s = warp_sequential_logit(a, tok, e);
    if (lane == 0 && a.st) atomicAdd(&a.st->sequential_logits, 1);
    return static_cast<float>(s);
}

// ------------------------------------------------- decode routers' finish

constexpr int kDecMaxTokens = 16;
constexpr int kDecRows = 128;  // hidden rows per partial sum (row chunk)
constexpr int kDecCols = 32;   // experts per CTA of the decode router
constexpr int kDecSlots = 2;   // staging buffers for settle_logit

// Shared memory the finish works in (caller-provided, any layout).
struct DecodeTailSmem {
    float* logit;  // [T][E]
    float* evs;    // [8][kMaxExperts] softmax scratch, one row per warp
    double* wnorm; // [E]
    double* xnorm; // [T]
    float* bias;   // [E]
    int* fb_count; // [1]
    int* fb_list;  // [kRouteFallbacks]
    double* stage; // [kDecSlots][staged_logit_doubles(H)]
};

// The decode routers' finish, by one CTA of 256 threads: certify the T x E
// double logits acc(t * E + e), each a sum of exact products with at most
// 24 + H / kDecRows roundings on any chain (the order of the row chunks
// does not matter), against the squared norms xn2(t) and wn2(e); settle the
// queued ones; select every token (one warp per token).  Writes a.ids,
// a.scores and the counts RouteArgs names.
template <class Acc, class Xn, class Wn>
__device__ void decode_certify(const RouteArgs& a, const Acc& acc, const Xn& xn2, const Wn& wn2,
                               const DecodeTailSmem& m) {
    const int T = a.T, H = a.H, E = a.E;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) *m.fb_count = 0;
    for (int ee = tid; ee < E; ee += blockDim.x) {
        m.wnorm[ee] = sqrt(wn2(ee) * (1.0 + (H + 64) * 0x1.0p-52));
        m.bias[ee] = a.bias ? a.bias[ee] : 0.0f;
    }
    for (int t = tid; t < T; t += blockDim.x) m.xnorm[t] = sqrt(xn2(t) * (1.0 + (H + 64) * 0x1.0p-52));
    __syncthreads();
    const double gamma = static_cast<double>(H + H / kDecRows + 40) * 0x1.0p-53 * 1.01;
#pragma unroll 4
    for (int idx = tid; idx < T * E; idx += blockDim.x) {
        const int t = idx / E, ee = idx % E;
        double s = acc(idx);
        double A = m.xnorm[t] * m.wnorm[ee] * (1.0 + 0x1.0p-40);
        if (a.bias) {
            s += static_cast<double>(m.bias[ee]);
            A += fabs(static_cast<double>(m.bias[ee]));
        }
        if (!rounding_certified(s, gamma * A + 0x1.0p-1060)) {
            const int slot = atomicAdd(m.fb_count, 1);
            if (slot < kRouteFallbacks) m.fb_list[slot] = t * 256 + ee;
            else s = sequential_logit(a, t, ee); // queue full: this thread does it
        }
        if (!isfinite(s)) device_fail(a.st, HMOE_NON_FINITE_ROUTER);
        m.logit[idx] = static_cast<float>(s);
    }
    __syncthreads();
    const int nfb = min(*m.fb_count, kRouteFallbacks);
    for (int f = warp; f < nfb; f += blockDim.x >> 5) {
        const int t = m.fb_list[f] >> 8, ee = m.fb_list[f] & 255;
        const float lg =
            settle_logit(a, t, ee, warp < kDecSlots ? m.stage + warp * staged_logit_doubles(H) : nullptr);
        if (lane == 0) {
            if (!isfinite(lg)) device_fail(a.st, HMOE_NON_FINITE_ROUTER);
            m.logit[t * E + ee] = lg;
        }
    }
    __syncthreads();
}

// The decode routers' finish: certify (above), then select every token, one
// warp per token (select_token).
template <int C, class Acc, class Xn, class Wn>
__device__ void decode_finish(const RouteArgs& a, const Acc& acc, const Xn& xn2, const Wn& wn2,
                              const DecodeTailSmem& m) {
    decode_certify(a, acc, xn2, wn2, m);
    const int T = a.T, E = a.E;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int t = warp; t < T; t += blockDim.x >> 5) {
        float lv[C];
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const int j = lane + 32 * c;
            lv[c] = j < E ? m.logit[t * E + j] : 0.0f;
        }
        select_token<C>(lv, E, a.k, a.softmax, a.renorm, m.evs + warp * kMaxExperts,
                        a.ids + static_cast<size_t>(t) * a.k, a.scores + static_cast<size_t>(t) * a.k, a.counts,
                        token_block_counts(a, t), a.st, false, nullptr);
    }
}

// select_token's result for every token of m.logit ([T][E], exact logits),
// computed by the whole CTA at once: the exponentials and divisions spread
// over all threads, and each candidate's rank in the order (probability
// descending, id ascending) counted directly instead of k + 1 sequential
// argmax rounds.  The ranks are those rounds' outcome: the order is total
// (ids differ), a NaN probability is keyed lowest as there, and -0.0 and
// +0.0 compare equal as there.  The maximum, the denominator (a tree sum
// exactly when every term is at least 2^-22, else the sequential sum in
// expert order), the probabilities float(e / den), the renormalising sum in
// rank order, the near-tie test between adjacent ranks and the non-finite
// handling are select_token's, operation for operation.  Uses m.evs as
// [T][E] and m.stage as scratch (after decode_certify); T <= 8, k <= 32.
__device__ inline void decode_select_block(const RouteArgs& a, const DecodeTailSmem& m) {
    const int T = a.T, E = a.E, k = a.k;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nth = blockDim.x, nw = nth >> 5;
    const int nk = k < E ? k + 1 : k; // ranks the selection looks at
    constexpr int kRk = 33;           // per-token stride of the rank tables
    const float* lg = m.logit;
    float* pv = m.evs;                // [T][E] exponentials, then probabilities
    double* den_s = m.stage;          // [T]
    float* mx_s = reinterpret_cast<float*>(den_s + T);
    int* ok_s = reinterpret_cast<int*>(mx_s + T);
    int* sel_e = ok_s + T;            // [T][kRk] expert of each rank
    float* sel_p = reinterpret_cast<float*>(sel_e + T * kRk);
    float* sel_l = sel_p + T * kRk;   // its logit
    for (int t = warp; t < T; t += nw) {
        float mm = -FLT_MAX * 2.0f;
        for (int j = lane; j < E; j += 32) mm = fmaxf(mm, lg[t * E + j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
        if (lane == 0) {
            mx_s[t] = mm;
            ok_s[t] = 1;
        }
    }
    __syncthreads();
    for (int i = tid; i < T * E; i += nth) {
        const float x = lg[i];
        pv[i] = a.softmax ? static_cast<float>(exp(static_cast<double>(x - mx_s[i / E]))) : x;
    }
    __syncthreads();
    if (a.softmax) {
        for (int t = warp; t < T; t += nw) {
            double den = 0.0;
            bool small = false;
            for (int j = lane; j < E; j += 32) {
                const float e = pv[t * E + j];
                den += static_cast<double>(e);
                small |= e < 0x1.0p-22f;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
            if (__any_sync(0xffffffffu, small)) {
                den = 0.0;
                if (lane == 0)
                    for (int j = 0; j < E; ++j) den += static_cast<double>(pv[t * E + j]);
                den = __shfl_sync(0xffffffffu, den, 0);
            }
            if (lane == 0) {
                den_s[t] = den;
                if (!(isfinite(den) && den > 0.0)) ok_s[t] = 0;
            }
        }
        __syncthreads();
        for (int i = tid; i < T * E; i += nth)
            pv[i] = static_cast<float>(static_cast<double>(pv[i]) / den_s[i / E]);
        __syncthreads();
    }
    for (int i = tid; i < T * E; i += nth) {
        const float p = pv[i];
        if (p != p) { // ranks lowest; the token is flagged
            pv[i] = -FLT_MAX * 2.0f;
            ok_s[i / E] = 0;
        }
    }
    __syncthreads();
    for (int i = tid; i < T * E; i += nth) {
        const int t = i / E, e = i % E;
        const float p = pv[i];
        const float* row = pv + t * E;
        int r = 0;
        for (int j = 0; j < E; ++j) {
            const float q = row[j];
            r += (q > p) || (q == p && j < e);
        }
        if (r < nk) {
            sel_e[t * kRk + r] = e;
            sel_p[t * kRk + r] = p;
            sel_l[t * kRk + r] = lg[i];
        }
    }
    __syncthreads();
    for (int t = warp; t < T; t += nw) {
        bool ok = ok_s[t] != 0;
        bool tie = false;
        if (a.softmax && lane >= 1 && lane < nk && sel_l[t * kRk + lane] != sel_l[t * kRk + lane - 1]) {
            const int dd = abs(__float_as_int(sel_p[t * kRk + lane - 1]) - __float_as_int(sel_p[t * kRk + lane]));
            tie = dd <= 2;
        }
        tie = __any_sync(0xffffffffu, tie);
        double rsum = 0.0; // rank order
        if (lane == 0)
            for (int r = 0; r < k; ++r) rsum += static_cast<double>(sel_p[t * kRk + r]);
        rsum = __shfl_sync(0xffffffffu, rsum, 0);
        if (a.renorm && !(isfinite(rsum) && rsum != 0.0)) ok = false;
        if (lane < k) {
            const float mine = sel_p[t * kRk + lane];
            const int id = sel_e[t * kRk + lane];
            float sc = mine;
            if (a.renorm && ok) sc = static_cast<float>(static_cast<double>(mine) / rsum);
            if (!ok && lane == 0) sc = __int_as_float(0x7fc00000);
            a.ids[static_cast<size_t>(t) * k + lane] = static_cast<uint32_t>(id);
            a.scores[static_cast<size_t>(t) * k + lane] = sc;
            if (a.counts) atomicAdd(a.counts + id, 1);
            int32_t* bc = token_block_counts(a, t);
            if (bc) atomicAdd(bc + id, 1);
        }
        if (lane == 0) {
            if (!ok) device_fail(a.st, HMOE_NON_FINITE_ROUTER);
            if (tie && a.st) atomicAdd(&a.st->near_ties, 1);
        }
    }
}

} // namespace hmoe
