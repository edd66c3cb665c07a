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
//      stored per row chunk; the token scales of the FP16 token rows (as the
//      permutation computes them)
//   B  every CTA, redundantly and identically: the row chunks added in
//      order, the decode router's certification, settling and selection,
//      and the grouping by (expert, token), all in shared memory (no
//      barrier, no global round trip); then L2 prefetches of this CTA's
//      down-projection boxes
//   C  gate/up: (segment, 128 columns, K rank) items; INT8 boxes stream
//      through one TMA ring of up to ~190 KB per CTA, and each item stores
//      its rank's partial sums (no atomics)
//   D  down: (segment, K rank, group of 256-column blocks) items; the item
//      first forms its SwiGLU rows from the gate/up rank partials (ranks
//      added in order), then streams its down boxes through the same ring,
//      which kept issuing them ahead while C finished; stores rank partials
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
constexpr int kDlStage = 32768;  // bytes per ring stage: a gate box and an up box, or one down box.
                                 // Boxes are 256 bytes wide and 32-128 rows deep: TMA moves
                                 // narrower or shallower boxes at a fraction of the HBM rate
constexpr int kDlDynLimit = 232448 - 5120;  // dynamic shared memory (the static arrays take the rest)
constexpr int kDlPrefetchBytes = 256 * 1024; // down bytes per CTA prefetched into L2
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
    int KS, kc, bk2;   // gate/up: K ranks, rows per rank (multiple of 32), rows per box
    int KSd, kcd, bk3; // down: the same
    int nstage;        // ring stages
    DlCtl* ctl;
    double* rpart;     // [H/128][T][E] router partial sums
    double* wpart;     // [H/128][E] squared router-column norms
    double* xpart;     // [H/128][T] squared token norms
    float* tscale;     // [2][T] s_t, 1/s_t
    float* pgu;        // [KS][R][2I] gate/up rank partials (gate | up)
    float* pdn;        // [KSd][R][H] down rank partials
};

// Shared-memory plan (byte offsets from a 128-byte aligned base).  Phase A
// and phase B work from offset 0 (B may reach into the ring, which is not in
// use yet); C, D and E keep their scratch below `ring`.
struct DlSmem {
    int a_xs, a_red, a_wred, a_end;
    int b_racc, b_wn2, b_xn2, b_logit, b_evs, b_wn, b_xn, b_bias, b_fb, b_stage, b_grp, b_end;
    int c_xs, c_red, d_hs, d_red, e_v;
    int ring, bars, total;
};

__host__ __device__ inline int dl_al(int v) { return (v + 127) & ~127; }

__host__ __device__ inline DlSmem dl_smem(int T, int maxt, int H, int E, int kc, int kcd, int R, int S) {
    DlSmem m{};
    m.a_xs = 0;
    m.a_red = dl_al(m.a_xs + T * kDecRows * 4);
    m.a_wred = dl_al(m.a_red + 8 * T * 32 * 8);
    m.a_end = dl_al(m.a_wred + 8 * 32 * 8);
    m.b_racc = 0;
    m.b_wn2 = dl_al(m.b_racc + T * E * 8);
    m.b_xn2 = dl_al(m.b_wn2 + E * 8);
    m.b_logit = dl_al(m.b_xn2 + T * 8);
    m.b_evs = dl_al(m.b_logit + T * E * 4);
    m.b_wn = dl_al(m.b_evs + 8 * kMaxExperts * 4);
    m.b_xn = dl_al(m.b_wn + E * 8);
    m.b_bias = dl_al(m.b_xn + T * 8);
    m.b_fb = dl_al(m.b_bias + E * 4);
    m.b_stage = dl_al(m.b_fb + (1 + kRouteFallbacks) * 4);
    m.b_grp = dl_al(m.b_stage + kDecSlots * staged_logit_doubles(H) * 8);
    m.b_end = dl_al(m.b_grp + 3 * R * 4);
    // C: token rows of this rank, row-group partials; D: SwiGLU rows of the
    // item, row-group partials; E: the slot values of one 32-column unit
    m.c_xs = 0;
    m.c_red = dl_al(m.c_xs + T * kc * 4);
    const int c_end = dl_al(m.c_red + maxt * 2 * 256 * 4);
    m.d_hs = 0;
    m.d_red = dl_al(m.d_hs + maxt * kcd * 4);
    const int d_end = dl_al(m.d_red + maxt * 256 * 4);
    m.e_v = 0;
    const int e_end = dl_al(m.e_v + kDlMaxSlots * 32 * 4);
    int r = c_end > d_end ? c_end : d_end;
    r = r > e_end ? r : e_end;
    r = r > m.a_end ? r : m.a_end;
    m.ring = dl_al(r);
    m.bars = dl_al(m.ring + S * kDlStage);
    m.total = m.bars + S * 8 + 128; // room to align the base
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

// Ring wait (every thread waits; a timeout or the abort word marks the call
// failed).  The caller combines the threads' results with __syncthreads_or,
// so every thread takes the same branch.  Threads poll the barrier in shared
// memory; the abort word and the clock, which live in global memory, are
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

// L2 prefetch of one tensor box (no shared memory, no completion to wait for).
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap* map, int x, int y, int z) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(map), "r"(x),
                 "r"(y), "r"(z)
                 : "memory");
}

} // namespace

namespace {

template <int C, int MAXT>
__global__ void __launch_bounds__(kDlThreads, 1)
    decode_layer_kernel(const __grid_constant__ CUtensorMap tmg, const __grid_constant__ CUtensorMap tmu,
                        const __grid_constant__ CUtensorMap tmd, DlArgs d) {
    extern __shared__ __align__(128) unsigned char dsm[];
    __shared__ int abort_s, nseg_s;
    __shared__ int4 seg_s[kDlMaxRows];     // segment: (expert, first row, rows, 0)
    __shared__ float qs_s[kDlMaxRows][3];  // segment: scales (gate, up, down)
    __shared__ float qz_s[kDlMaxRows][3];  // segment: 2^23 + 128 + zero point (dequantisation offsets)
    __shared__ int rtok_s[kDlMaxRows];     // row: token
    __shared__ float rw_s[kDlMaxRows];     // row: routing weight (1 for shared experts)
    __shared__ float rsc_s[kDlMaxRows];    // row: down scale of its expert
    __shared__ int trow_s[kDlMaxRows];     // [T][slots] the token's rows, ascending
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
    const DlSmem L = dl_smem(T, MAXT, H, E, d.kc, d.kcd, R, S);
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 127) & ~uintptr_t(127));
    uint8_t* ring = base + L.ring;
    uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bars);
    if (tid == 0) {
        abort_s = 0;
        for (int s = 0; s < S; ++s) sm100::mbar_init(&full[s], 1);
        sm100::fence_mbarrier_init();
        sm100::prefetch_tmap(&tmg);
        sm100::prefetch_tmap(&tmu);
        sm100::prefetch_tmap(&tmd);
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
                if (e0 + l < E) d.rpart[(static_cast<size_t>(rc) * T + t) * E + e0 + l] = s;
            }
            if (tid < 32 && e0 + tid < E) {
                double s = 0.0;
                for (int w = 0; w < 8; ++w) s += wred0[w * 32 + tid];
                d.wpart[static_cast<size_t>(rc) * E + e0 + tid] = s;
            }
            if (ec == 0 && tid < T) {
                double s = 0.0;
                for (int i = 0; i < kDecRows; ++i) {
                    const double v = static_cast<double>(xs0[tid * kDecRows + i]);
                    s = fma(v, v, s);
                }
                d.xpart[static_cast<size_t>(rc) * T + tid] = s;
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

    // ------------------------- B: selection and grouping, in every CTA
    if (ok) {
        double* racc = reinterpret_cast<double*>(base + L.b_racc); // [T][E]
        double* wn2 = reinterpret_cast<double*>(base + L.b_wn2);   // [E]
        double* xn2 = reinterpret_cast<double*>(base + L.b_xn2);   // [T]
        // the row chunks in order (two logits per thread at a time, eight
        // chunk loads each in flight)
        for (int i0 = tid; i0 < T * E; i0 += 2 * kDlThreads) {
            const int i1 = i0 + kDlThreads;
            const int t0 = i0 / E, e0 = i0 % E, t1 = i1 / E, e1 = i1 % E;
            const bool has1 = i1 < T * E;
            double s0 = 0.0, s1 = 0.0;
            for (int c0 = 0; c0 < nRC; c0 += 8) {
                double v0[8], v1[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const bool in = c0 + u < nRC;
                    v0[u] = in ? __ldcg(d.rpart + (static_cast<size_t>(c0 + u) * T + t0) * E + e0) : 0.0;
                    v1[u] = in && has1 ? __ldcg(d.rpart + (static_cast<size_t>(c0 + u) * T + t1) * E + e1) : 0.0;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (c0 + u < nRC) {
                        s0 += v0[u];
                        s1 += v1[u];
                    }
            }
            racc[i0] = s0;
            if (has1) racc[i1] = s1;
        }
        for (int e = tid; e < E; e += kDlThreads) {
            double s = 0.0;
            for (int c = 0; c < nRC; ++c) s += __ldcg(d.wpart + static_cast<size_t>(c) * E + e);
            wn2[e] = s;
        }
        if (tid < T) {
            double s = 0.0;
            for (int c = 0; c < nRC; ++c) s += __ldcg(d.xpart + static_cast<size_t>(c) * T + tid);
            xn2[tid] = s;
        }
        if (tid < 2 * T) tsc_s[tid] = __ldcg(d.tscale + tid);
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
        decode_finish<C>(
            ra, [&](int idx) { return racc[idx]; }, [&](int t) { return xn2[t]; }, [&](int e) { return wn2[e]; }, m);
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
                const hmoe_expert_quant& q = d.quant[e];
#pragma unroll
                for (int p = 0; p < 3; ++p) {
                    qs_s[u][p] = q.scale[p];
                    qz_s[u][p] = 8388608.0f + 128.0f + static_cast<float>(q.zero_point[p]);
                }
                for (int rr = r; rr < r + len; ++rr) rsc_s[rr] = q.scale[2];
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

    // ------------------------------------------- work of phases C and D
    // Phase C items: (segment, 256-column block, K rank), rank r2 = b mod KS
    // fixed per CTA, blocks q2, q2 + nq2, ...; phase D items: (segment, K
    // rank, group of CGW 256-column blocks), b, b + G, ...
    const int nseg = nseg_s;
    const int KS = d.KS, kc = d.kc, bk2 = d.bk2, nb2 = kc / bk2, nCB = (I + 255) / 256;
    const int r2 = b % KS, q2 = b / KS, nq2 = (G - r2 + KS - 1) / KS;
    const int kb2 = r2 * kc; // at or past H for a rank with no rows (its partials stay zero)
    const int pairs2 = nseg * nCB;
    const int n2 = q2 < pairs2 ? (pairs2 - q2 + nq2 - 1) / nq2 : 0;
    const int tot2 = n2 * nb2;
    const int KSd = d.KSd, kcd = d.kcd, bk3 = d.bk3, nb3 = kcd / bk3, nCBd = H / 256;
    const int CGW = nCBd % 4 == 0 ? 4 : (nCBd % 3 == 0 ? 3 : (nCBd % 2 == 0 ? 2 : 1));
    const int nCG = nCBd / CGW, nbi3 = CGW * nb3;
    const int items3 = nseg * KSd * nCG;
    const int n3 = b < items3 ? (items3 - b + G - 1) / G : 0;
    const int tot = tot2 + n3 * nbi3;
    // Down box m of this CTA (m < n3 * nbi3): tensor coordinates.
    auto down_box = [&](int m, int& x, int& y, int& z) {
        const int i3 = m / nbi3, w = m % nbi3;
        const int idx3 = b + i3 * G;
        const int cg = idx3 % nCG, r3 = (idx3 / nCG) % KSd, u = idx3 / (nCG * KSd);
        x = (cg * CGW + w / nb3) * 256;
        y = r3 * kcd + (w % nb3) * bk3;
        z = seg_s[u].x;
    };
    // Box n of the ring sequence (phase C's boxes, then phase D's), issued
    // into stage n mod S.  A box wholly past K is not copied; its barrier
    // completes with a plain arrival.  Columns past N read as zeros.
    auto issue = [&](int n) {
        const int s = n % S;
        uint8_t* dst = ring + s * kDlStage;
        if (n < tot2) {
            const int i = n / nb2, bx = n % nb2;
            const int j = q2 + i * nq2;
            const int e = seg_s[j / nCB].x, c0 = (j % nCB) * 256, kk = kb2 + bx * bk2;
            if (kk < H) {
                sm100::mbar_arrive_expect_tx(&full[s], 2 * 256 * bk2);
                sm100::tma_load_3d(dst, &tmg, c0, kk, e, &full[s]);
                sm100::tma_load_3d(dst + kDlStage / 2, &tmu, c0, kk, e, &full[s]);
            } else {
                sm100::mbar_arrive(&full[s]);
            }
        } else {
            int x, y, z;
            down_box(n - tot2, x, y, z);
            if (y < I) {
                sm100::mbar_arrive_expect_tx(&full[s], 256 * bk3);
                sm100::tma_load_3d(dst, &tmd, x, y, z, &full[s]);
            } else {
                sm100::mbar_arrive(&full[s]);
            }
        }
    };
    int issued = ok ? min(S, tot) : 0; // uniform over the CTA
    int cons = 0;                      // boxes thread 0 has seen complete
    if (warp == 0 && ok) {
        // the ring's first S boxes, then L2 prefetches of the first down
        // boxes, so the down weights cross HBM while gate/up streams
        for (int n = lane; n < issued; n += 32) issue(n);
        const int np = min(n3 * nbi3, kDlPrefetchBytes / (256 * bk3));
        for (int m = lane; m < np; m += 32) {
            int x, y, z;
            down_box(m, x, y, z);
            if (y < I) tma_prefetch_l2_3d(&tmd, x, y, z);
        }
    }
    bool dead = !ok; // uniform over the CTA
    // thread (column quad cq of the 256-column block, row class g): rows
    // g, g + 4, ... of each box, in order, as the GEMV's row groups
    const int cq = tid & 63, g = tid >> 6;

    // ------------------------------------------------------- C: gate/up
    {
        float* xs2 = reinterpret_cast<float*>(base + L.c_xs);  // [T][kc] token rows of this rank
        float* red2 = reinterpret_cast<float*>(base + L.c_red); // [MAXT][2][256] row classes added in order
        if (ok && n2 > 0) {
            for (int i = tid; i < T * kc; i += kDlThreads) {
                const int t = i / kc, kk = i % kc;
                float v = 0.0f;
                if (kb2 + kk < H)
                    v = __half2float(__float2half_rn(a.x[static_cast<size_t>(t) * H + kb2 + kk] * tsc_s[t])) *
                        tsc_s[T + t];
                xs2[i] = v;
            }
        }
        __syncthreads();
        for (int i = 0; i < n2 && !dead; ++i) {
            const int j = q2 + i * nq2, u = j / nCB, cb = j % nCB;
            const int4 sg = seg_s[u];
            const int first = sg.y, tu = min(sg.z, MAXT);
            const float zg = qz_s[u][0], zu = qz_s[u][1];
            int xoff[MAXT];
#pragma unroll
            for (int tt = 0; tt < MAXT; ++tt) xoff[tt] = tt < tu ? rtok_s[first + tt] * kc : 0;
            float acc[MAXT][2][4];
#pragma unroll
            for (int tt = 0; tt < MAXT; ++tt)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[tt][0][c] = acc[tt][1][c] = 0.0f;
            for (int bx = 0; bx < nb2; ++bx) {
                const int n = i * nb2 + bx, s = n % S;
                const bool got = dl_wait(d, &full[s], (n / S) & 1);
                const int nr = got ? min(bk2, H - (kb2 + bx * bk2)) : 0;
                const uint8_t* bg = ring + s * kDlStage;
                const uint8_t* bu = bg + kDlStage / 2;
#pragma unroll 2
                for (int rr = g; rr < bk2; rr += 4) {
                    if (rr < nr) {
                        float wg[4], wu[4];
                        dequant4_fast(*reinterpret_cast<const uint32_t*>(bg + rr * 256 + 4 * cq), zg, wg);
                        dequant4_fast(*reinterpret_cast<const uint32_t*>(bu + rr * 256 + 4 * cq), zu, wu);
                        const float* xr = xs2 + bx * bk2 + rr;
#pragma unroll
                        for (int tt = 0; tt < MAXT; ++tt) {
                            if (tt < tu) {
                                const float xv = xr[xoff[tt]];
#pragma unroll
                                for (int c = 0; c < 4; ++c) {
                                    acc[tt][0][c] = fmaf(xv, wg[c], acc[tt][0][c]);
                                    acc[tt][1][c] = fmaf(xv, wu[c], acc[tt][1][c]);
                                }
                            }
                        }
                    }
                }
                cons += got;
                dead = __syncthreads_or(!got) != 0; // stage s is free
                if (dead) break;
                if (n + S < tot) {
                    if (tid == 0) issue(n + S);
                    issued = n + S + 1;
                }
            }
            if (dead) break;
            // row classes added in order: class 0 stores, 1..3 add in turn
            for (int gg = 0; gg < 4; ++gg) {
                if (g == gg) {
#pragma unroll
                    for (int tt = 0; tt < MAXT; ++tt)
                        if (tt < tu)
#pragma unroll
                            for (int pj = 0; pj < 2; ++pj) {
                                float4* r = reinterpret_cast<float4*>(red2 + (tt * 2 + pj) * 256 + 4 * cq);
                                const float4 v = make_float4(acc[tt][pj][0], acc[tt][pj][1], acc[tt][pj][2],
                                                             acc[tt][pj][3]);
                                if (gg == 0) {
                                    *r = v;
                                } else {
                                    float4 o = *r;
                                    o.x += v.x;
                                    o.y += v.y;
                                    o.z += v.z;
                                    o.w += v.w;
                                    *r = o;
                                }
                            }
                }
                __syncthreads();
            }
            for (int idx = tid; idx < tu * 512; idx += kDlThreads) {
                const int tt = idx / 512, pj = (idx / 256) & 1, c = cb * 256 + idx % 256;
                if (c < I)
                    d.pgu[(static_cast<size_t>(r2) * R + first + tt) * (2 * I) + pj * I + c] = red2[idx];
            }
            __syncthreads();
        }
    }
    ok = dl_grid_sync(d, 1, abort_s) && !dead;

    // ---------------------------------------------------------- D: down
    {
        float* hs = reinterpret_cast<float*>(base + L.d_hs);    // [MAXT][kcd] SwiGLU rows of the item
        float* red3 = reinterpret_cast<float*>(base + L.d_red); // [MAXT][256] row classes added in order
        for (int i3 = 0; ok && !dead && i3 < n3; ++i3) {
            const int idx3 = b + i3 * G;
            const int cg = idx3 % nCG, r3 = (idx3 / nCG) % KSd, u = idx3 / (nCG * KSd);
            const int4 sg = seg_s[u];
            const int first = sg.y, tu = min(sg.z, MAXT);
            const int kb3 = r3 * kcd;
            // SwiGLU rows [kb3, kb3 + kcd) of the segment: the gate/up ranks
            // added in order, as the GEMV's gate/up epilogue does
            for (int x = tid; x < tu * kcd; x += kDlThreads) {
                const int tt = x / kcd, kk = x % kcd;
                float v = 0.0f;
                if (kb3 + kk < I) {
                    const size_t row = static_cast<size_t>(first + tt);
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
                hs[tt * kcd + kk] = v;
            }
            __syncthreads();
            const float zoff = qz_s[u][2];
            for (int cbl = 0; cbl < CGW && !dead; ++cbl) {
                const int cb = cg * CGW + cbl;
                float acc[MAXT][4];
#pragma unroll
                for (int tt = 0; tt < MAXT; ++tt)
#pragma unroll
                    for (int c = 0; c < 4; ++c) acc[tt][c] = 0.0f;
                for (int bx = 0; bx < nb3; ++bx) {
                    const int n = tot2 + i3 * nbi3 + cbl * nb3 + bx, s = n % S;
                    const bool got = dl_wait(d, &full[s], (n / S) & 1);
                    const int nr = got ? min(bk3, I - (kb3 + bx * bk3)) : 0;
                    const uint8_t* box = ring + s * kDlStage;
#pragma unroll 2
                    for (int rr = g; rr < bk3; rr += 4) {
                        if (rr < nr) {
                            float w[4];
                            dequant4_fast(*reinterpret_cast<const uint32_t*>(box + rr * 256 + 4 * cq), zoff, w);
                            const float* hr = hs + bx * bk3 + rr;
#pragma unroll
                            for (int tt = 0; tt < MAXT; ++tt) {
                                if (tt < tu) {
                                    const float xv = hr[tt * kcd];
#pragma unroll
                                    for (int c = 0; c < 4; ++c) acc[tt][c] = fmaf(xv, w[c], acc[tt][c]);
                                }
                            }
                        }
                    }
                    cons += got;
                    dead = __syncthreads_or(!got) != 0;
                    if (dead) break;
                    if (n + S < tot) {
                        if (tid == 0) issue(n + S);
                        issued = n + S + 1;
                    }
                }
                if (dead) break;
                for (int gg = 0; gg < 4; ++gg) {
                    if (g == gg) {
#pragma unroll
                        for (int tt = 0; tt < MAXT; ++tt)
                            if (tt < tu) {
                                float4* r = reinterpret_cast<float4*>(red3 + tt * 256 + 4 * cq);
                                const float4 v = make_float4(acc[tt][0], acc[tt][1], acc[tt][2], acc[tt][3]);
                                if (gg == 0) {
                                    *r = v;
                                } else {
                                    float4 o = *r;
                                    o.x += v.x;
                                    o.y += v.y;
                                    o.z += v.z;
                                    o.w += v.w;
                                    *r = o;
                                }
                            }
                    }
                    __syncthreads();
                }
                for (int idx = tid; idx < tu * 256; idx += kDlThreads)
                    d.pdn[(static_cast<size_t>(r3) * R + first + idx / 256) * H + cb * 256 + idx % 256] = red3[idx];
                __syncthreads();
            }
            __syncthreads(); // hs is rewritten by the next item
        }
    }
    ok = dl_grid_sync(d, 2, abort_s) && !dead;

    // -------------------------------------------------------- E: combine
    if (ok) {
        float* vb = reinterpret_cast<float*>(base + L.e_v); // [slots][32]
        const int units = T * (H / 32);
        for (int un = b; un < units; un += G) {
            const int t = un / (H / 32), c = (un % (H / 32)) * 32 + lane;
            // warp w: the BF16 output rows of slots w, w + 8 (as the down
            // projection rounds them), each the down ranks added in order
            for (int sl = warp; sl < slots; sl += kDlThreads / 32) {
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
            __syncthreads();
            if (warp == 0) { // rows in ascending expert id, from zero
                float acc = 0.0f;
                for (int sl = 0; sl < slots; ++sl) acc = __fadd_rn(acc, vb[sl * 32 + lane]);
                const size_t o = static_cast<size_t>(t) * H + c;
                if (d.residual) acc = __fadd_rn(d.residual[o], acc);
                d.y[o] = acc;
                if (d.y16) d.y16[o] = __float2bfloat16_rn(acc);
            }
            __syncthreads();
        }
    }

    // Every issued box is waited for (bounded) before the CTA exits.
    if (tid == 0)
        for (int n = cons; n < issued; ++n) sm100::mbar_wait_for(&full[n % S], (n / S) & 1, kDlWaitNs);
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

// Rows per TMA box for a rank of kc rows (a multiple of 32): kc split into
// the fewest equal boxes of at most `most` rows (each a multiple of 4, so a
// row's class mod 4 is the same within the box and within the rank).
int dl_box_rows(int kc, int most) {
    int n = (kc + most - 1) / most;
    while (kc % n || (kc / n) % 4) ++n;
    return kc / n;
}

struct DlLayout {
    size_t rpart, wpart, xpart, tscale, pgu, pdn, total;
};

DlLayout dl_layout(const hmoe_layer_desc& d, size_t T) {
    const size_t H = d.hidden, I = d.intermediate, E = d.experts, slots = d.top_k + d.shared_experts;
    const size_t R = T * slots, nRC = H / kDecRows;
    const size_t KS = dl_split(static_cast<int>(H)), KSd = dl_split(static_cast<int>(I));
    DlLayout l{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align_up(off + bytes, 256);
        return at;
    };
    l.rpart = take(nRC * T * E * 8);
    l.wpart = take(nRC * E * 8);
    l.xpart = take(nRC * T * 8);
    l.tscale = take(2 * T * 4);
    l.pgu = take(KS * R * 2 * I * 4);
    l.pdn = take(KSd * R * H * 4);
    l.total = off;
    return l;
}

template <int C, int MAXT>
const void* dl_kernel() {
    return reinterpret_cast<const void*>(decode_layer_kernel<C, MAXT>);
}

const void* dl_pick(int E, int T) {
    const int c = (E + 31) / 32;
    const bool one = T == 1;
    if (c <= 1) return one ? dl_kernel<1, 1>() : dl_kernel<1, 8>();
    if (c <= 2) return one ? dl_kernel<2, 1>() : dl_kernel<2, 8>();
    if (c <= 4) return one ? dl_kernel<4, 1>() : dl_kernel<4, 8>();
    return one ? dl_kernel<8, 1>() : dl_kernel<8, 8>();
}

// Ring stages for a shape, 0 when the phases' scratch leaves too little.
int dl_stages(int T, int H, int E, int kc, int kcd, int R) {
    const int maxt = T == 1 ? 1 : kDlMaxTokens;
    const DlSmem L0 = dl_smem(T, maxt, H, E, kc, kcd, R, 0);
    int S = std::min(kDlMaxStages, (kDlDynLimit - L0.total) / (kDlStage + 8));
    while (S > 0) {
        const DlSmem L = dl_smem(T, maxt, H, E, kc, kcd, R, S);
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
          d.intermediate >= 256 &&
          d.experts <= static_cast<uint32_t>(kMaxExperts) && d.ep_size == 1))
        return false;
    const int H = static_cast<int>(d.hidden), I = static_cast<int>(d.intermediate);
    const int kc = dl_rows_per_rank(H, dl_split(H)), kcd = dl_rows_per_rank(I, dl_split(I));
    return dl_stages(static_cast<int>(T), H, static_cast<int>(d.experts), kc, kcd, static_cast<int>(T * slots)) > 0;
}

size_t decode_layer_ctl_bytes(const hmoe_layer_desc& d, size_t T) {
    return decode_layer_shape_ok(d, T) ? sizeof(DlCtl) : 0;
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
    d.bk2 = dl_box_rows(d.kc, 64);
    d.KSd = dl_split(I);
    d.kcd = dl_rows_per_rank(I, d.KSd);
    d.bk3 = dl_box_rows(d.kcd, 128);
    d.nstage = dl_stages(T, H, E, d.kc, d.kcd, R);
    const int maxt = T == 1 ? 1 : kDlMaxTokens;
    const DlSmem L = dl_smem(T, maxt, H, E, d.kc, d.kcd, R, d.nstage);
    char* base = ws + w.dl_data;
    const DlLayout l = dl_layout(desc, tokens);
    d.ctl = reinterpret_cast<DlCtl*>(ws + w.dl_ctl);
    d.rpart = reinterpret_cast<double*>(base + l.rpart);
    d.wpart = reinterpret_cast<double*>(base + l.wpart);
    d.xpart = reinterpret_cast<double*>(base + l.xpart);
    d.tscale = reinterpret_cast<float*>(base + l.tscale);
    d.pgu = reinterpret_cast<float*>(base + l.pgu);
    d.pdn = reinterpret_cast<float*>(base + l.pdn);
    const int experts = E + S;
    CUtensorMap mg, mu, md;
    if (!map_weights_box(&mg, desc.arena + desc.gate_offset, I, H, experts, desc.expert_stride, 256, d.bk2) ||
        !map_weights_box(&mu, desc.arena + desc.up_offset, I, H, experts, desc.expert_stride, 256, d.bk2) ||
        !map_weights_box(&md, desc.arena + desc.down_offset, H, I, experts, desc.expert_stride, 256, d.bk3)) {
        set_last_error_text("hmoe: cuTensorMapEncodeTiled failed (decode layer)");
        return HMOE_CUDA_ERROR;
    }
    const void* fn = dl_pick(E, T);
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
    void* args[] = {&mg, &mu, &md, &d};
    err = cudaLaunchKernelExC(&cfg, fn, args);
    if (err != cudaSuccess) {
        set_last_error("hmoe decode layer launch", err);
        return HMOE_CUDA_ERROR;
    }
    return check_launch("hmoe decode layer");
}

} // namespace hmoe
