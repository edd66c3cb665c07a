// expert_gemv.cu -- weight-streaming expert MLP for decode-sized groups.
//
// Same math as the tensor-core path and as ExpertMlpExecutor::execute
// (src/experts/ExpertExecutor.cpp:118-131):
//     gate/up:  h[r,c] = SiLU(sg * sum_k x[r,k] Wg[k,c]) * (su * sum_k x[r,k] Wu[k,c])
//     down:     y[r,c] = w_r * (sd * sum_k h[r,k] Wd[k,c])
// with W = q - zp dequantised exactly, FP32 accumulation.
//
// Decode touches each expert for a handful of rows, so the kernel is a
// stream of the expert's INT8 weights at HBM speed.  A thread block cluster
// of KS CTAs owns (tile, 256 output columns); CTA r of the cluster streams
// K rows [r*kc, (r+1)*kc) of the projection(s) through a 4-stage ring of
// TMA boxes [32 k][256 n] (8 KB each, issued by one thread, so each CTA
// keeps up to 64 KB of weights in flight).  Thread (cq, kr) owns columns
// 4cq..4cq+3 and the box rows kr (mod 4): one 32-bit shared load feeds
// four exact dequantisations and four FMAs per token.  The four row groups
// and the KS ranks are added in a fixed order (shared memory, then
// distributed shared memory), so results are deterministic.
#include "common.cuh"
#include "layer.cuh"
#include "sm100.cuh"

#include <cooperative_groups.h>

#include <algorithm>

namespace cg = cooperative_groups;

namespace hmoe {

namespace {

constexpr int kVThreads = 256;
constexpr int kVCols = 256;   // output columns per CTA (box width, bytes)
constexpr int kVRows = 32;    // K rows per box
constexpr int kVStages = 4;   // boxes (per projection) in flight
constexpr int kVGroups = kVThreads / (kVCols / 4); // 4 row groups
constexpr int kVMaxKc = 1024; // K rows per CTA (bounds the token staging)
constexpr uint64_t kVWaitNs = 2000000000ull;

struct GemvSmem {
    int ring, xs, bars, total;
};

__host__ __device__ inline GemvSmem gemv_smem(int NP, int tok, int kc) {
    GemvSmem m{};
    const int ring = kVStages * NP * kVRows * kVCols;
    const int red = kVGroups * tok * NP * kVCols * 4; // partial sums, overlaid on the ring
    m.ring = 0;
    int off = (ring > red ? ring : red);
    off = (off + 15) & ~15;
    m.xs = off;
    off += tok * kc * 4;
    off = (off + 15) & ~15;
    m.bars = off;
    off += kVStages * 8;
    m.total = off + 128; // room to align the base to 128 bytes
    return m;
}

template <bool GATE_UP, int TOK>
__global__ void __launch_bounds__(kVThreads, 2)
    expert_gemv_kernel(const __grid_constant__ CUtensorMap tm0, const __grid_constant__ CUtensorMap tm1, GemvArgs a,
                       int kc) {
    constexpr int NP = GATE_UP ? 2 : 1;
    extern __shared__ __align__(128) unsigned char gsm[];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int KS = a.KS;
    if (static_cast<int>(blockIdx.z) >= *a.tile_count) return; // the whole cluster exits together
    const int4 td = a.tiles[blockIdx.z];
    const int e = td.x, r0 = td.y, n = td.z;
    const int K = a.K, N = a.N;
    const int kb = min(K, rank * kc), ke = min(K, kb + kc);
    const int nbox = (ke - kb + kVRows - 1) / kVRows;
    const int tid = threadIdx.x;
    const int cq = tid % (kVCols / 4), kr = tid / (kVCols / 4);
    const int c0 = blockIdx.y * kVCols;

    const GemvSmem L = gemv_smem(NP, TOK, kc);
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm) + 127) & ~uintptr_t(127));
    uint8_t* ring = base + L.ring;                        // [stage][NP][32 k][256 n] INT8
    float* red = reinterpret_cast<float*>(base + L.ring); // [group][TOK][NP][256] after the stream
    float* xs = reinterpret_cast<float*>(base + L.xs);    // [TOK][kc]
    uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bars);
    __shared__ int abort_s; // set after a timed-out wait: no further copies are issued

    const hmoe_expert_quant qp = a.quant[e];
    const float zoff0 = 8388608.0f + 128.0f + static_cast<float>(qp.zero_point[a.proj0]);
    const float zoff1 = GATE_UP ? 8388608.0f + 128.0f + static_cast<float>(qp.zero_point[a.proj0 + 1]) : 0.0f;
    if (tid == 0) {
        abort_s = 0;
        for (int s = 0; s < kVStages; ++s) sm100::mbar_init(&full[s], 1);
        sm100::fence_mbarrier_init();
        sm100::prefetch_tmap(&tm0);
        if (GATE_UP) sm100::prefetch_tmap(&tm1);
    }
    __syncthreads();

    uint32_t it = 0; // ring slots consumed so far (phase of each slot)
    for (int j0 = 0; j0 < n; j0 += TOK) {
        const int nj = min(TOK, n - j0);
        auto issue = [&](int b) {
            const int s = (it + b) % kVStages;
            sm100::mbar_arrive_expect_tx(&full[s], NP * kVRows * kVCols);
            sm100::tma_load_3d(ring + (s * NP + 0) * kVRows * kVCols, &tm0, c0, kb + b * kVRows, e, &full[s]);
            if (GATE_UP)
                sm100::tma_load_3d(ring + (s * NP + 1) * kVRows * kVCols, &tm1, c0, kb + b * kVRows, e, &full[s]);
        };
        // Every thread tracks how many boxes of this pass were issued (the
        // decision depends only on abort_s, read after a barrier).
        int issued = abort_s ? 0 : min(kVStages, nbox);
        if (tid == 0)
            for (int b = 0; b < issued; ++b) issue(b);
        // token rows of this pass (FP32 in shared memory; zero past the group)
        for (int i = tid; i < TOK * kc; i += kVThreads) {
            const int t = i / kc, kk = i % kc;
            float v = 0.0f;
            if (t < nj && kb + kk < ke) {
                const size_t row = static_cast<size_t>(r0 + j0 + t);
                if constexpr (GATE_UP)
                    v = __half2float(a.act16[row * K + kb + kk]) * a.xscale[row];
                else
                    v = a.act32[row * K + kb + kk];
            }
            xs[t * kc + kk] = v;
        }
        __syncthreads();
        // column pairs in packed FP32 (FADD2 / FFMA2): each lane rounds as
        // the scalar subtraction and fmaf would
        float2 acc[TOK][NP][2];
#pragma unroll
        for (int t = 0; t < TOK; ++t)
#pragma unroll
            for (int p = 0; p < NP; ++p) acc[t][p][0] = acc[t][p][1] = make_float2(0.0f, 0.0f);
        const float2 noff0 = make_float2(-zoff0, -zoff0), noff1 = make_float2(-zoff1, -zoff1);
        for (int b = 0; b < nbox; ++b) {
            const int s = (it + b) % kVStages;
            // Boxes that were issued are always waited for (bounded), so no
            // copy is left in flight when the CTA moves on or exits.
            if (b < issued && !sm100::mbar_wait_for(&full[s], ((it + b) / kVStages) & 1, kVWaitNs)) {
                device_fail(a.st, HMOE_TIMEOUT);
                abort_s = 1;
            }
            const int nr = min(kVRows, ke - (kb + b * kVRows));
            const uint8_t* box = ring + s * NP * kVRows * kVCols;
#pragma unroll 2
            for (int rr = kr; rr < kVRows; rr += kVGroups) {
                if (rr < nr) {
                    float2 w[NP][2];
#pragma unroll
                    for (int p = 0; p < NP; ++p) {
                        const uint32_t q =
                            *reinterpret_cast<const uint32_t*>(box + (p * kVRows + rr) * kVCols + 4 * cq) ^ 0x80808080u;
                        // float(2^23 + (q + 128)) - (2^23 + 128 + zp) = q - zp, exact
                        const float2 lo = make_float2(__uint_as_float(__byte_perm(q, 0x4B000000u, 0x7540)),
                                                      __uint_as_float(__byte_perm(q, 0x4B000000u, 0x7541)));
                        const float2 hi = make_float2(__uint_as_float(__byte_perm(q, 0x4B000000u, 0x7542)),
                                                      __uint_as_float(__byte_perm(q, 0x4B000000u, 0x7543)));
                        w[p][0] = __fadd2_rn(lo, p ? noff1 : noff0);
                        w[p][1] = __fadd2_rn(hi, p ? noff1 : noff0);
                    }
                    const float* xr = xs + b * kVRows + rr;
#pragma unroll
                    for (int t = 0; t < TOK; ++t) {
                        const float xv = xr[t * kc];
                        const float2 x2 = make_float2(xv, xv);
#pragma unroll
                        for (int p = 0; p < NP; ++p) {
                            acc[t][p][0] = __ffma2_rn(x2, w[p][0], acc[t][p][0]);
                            acc[t][p][1] = __ffma2_rn(x2, w[p][1], acc[t][p][1]);
                        }
                    }
                }
            }
            __syncthreads(); // every thread is done with this slot (and sees abort_s)
            if (!abort_s && b + kVStages < nbox && issued == b + kVStages) {
                if (tid == 0) issue(b + kVStages);
                issued = b + kVStages + 1;
            }
        }
        it += nbox;
        // The ring is idle now (every issued box was waited for): reuse it
        // for the row-group partial sums, then fold the groups in order.
#pragma unroll
        for (int t = 0; t < TOK; ++t)
#pragma unroll
            for (int p = 0; p < NP; ++p)
                *reinterpret_cast<float4*>(red + ((kr * TOK + t) * NP + p) * kVCols + 4 * cq) =
                    make_float4(acc[t][p][0].x, acc[t][p][0].y, acc[t][p][1].x, acc[t][p][1].y);
        __syncthreads();
        for (int i = tid; i < TOK * NP * kVCols; i += kVThreads) {
            float v = red[i];
#pragma unroll
            for (int g = 1; g < kVGroups; ++g) v += red[g * TOK * NP * kVCols + i];
            red[i] = v;
        }
        cluster.sync();
        // Rank r finalises a slice of the columns, adding the ranks in order.
        const int slice = kVCols / KS;
        for (int i = tid; i < TOK * slice; i += kVThreads) {
            const int t = i / slice;
            const int cl = rank * slice + i % slice;
            const int c = c0 + cl;
            if (t >= nj || c >= N) continue;
            float s0 = 0.0f, s1 = 0.0f;
            for (int r = 0; r < KS; ++r) {
                const float* rp = cluster.map_shared_rank(red, r);
                s0 += rp[(t * NP + 0) * kVCols + cl];
                if constexpr (GATE_UP) s1 += rp[(t * NP + 1) * kVCols + cl];
            }
            const size_t row = static_cast<size_t>(r0 + j0 + t);
            if constexpr (GATE_UP) {
                const float g = qp.scale[a.proj0] * s0;
                const float u = qp.scale[a.proj0 + 1] * s1;
                a.out32[row * N + c] = silu(g) * u;
            } else if (!a.push.peer || *reinterpret_cast<const volatile uint32_t*>(a.push.abort) == 0) {
                pushed_row(a.push, a.out16, td.w, static_cast<int>(row), N)[c] =
                    __float2bfloat16_rn(a.weight[row] * (qp.scale[a.proj0] * s0));
            }
        }
        cluster.sync(); // peers' partial sums stay alive until read; ring free again
    }
    if (!GATE_UP && a.push.peer) __threadfence_system(); // pushed rows visible before the return flag
}

template <bool GATE_UP, int TOK>
cudaError_t launch_gemv_variant(cudaLaunchConfig_t& cfg, const CUtensorMap& m0, const CUtensorMap& m1,
                                const GemvArgs& args, int kc) {
    const cudaError_t err = set_smem_limit(reinterpret_cast<const void*>(expert_gemv_kernel<GATE_UP, TOK>),
                                           static_cast<int>(cfg.dynamicSmemBytes));
    if (err != cudaSuccess) return err;
    return cudaLaunchKernelEx(&cfg, expert_gemv_kernel<GATE_UP, TOK>, m0, m1, args, kc);
}

// Split of K over the cluster: 8 CTAs (fewer only when a CTA would get
// under one box of rows).  It depends on K alone, so a row's result does not
// depend on how many tiles the launch covers (the expert-parallel path sizes
// its launches by capacity, the single-GPU path by the batch).
int gemv_split(int K) {
    int ks = 8;
    while (ks > 1 && (K + ks - 1) / ks < kVRows) ks /= 2;
    return ks;
}

hmoe_status launch_gemv(bool gate_up, const ExpertRun& r, const CUtensorMap& m0, const CUtensorMap& m1,
                        GemvArgs& g, cudaStream_t stream) {
    if (r.tile_cap <= 0) return HMOE_OK;
    if (r.tile_cap > 65535) return HMOE_UNSUPPORTED;
    const int col_blocks = (g.N + kVCols - 1) / kVCols;
    g.KS = gemv_split(g.K);
    int kc = (g.K + g.KS - 1) / g.KS;
    kc = (kc + kVRows - 1) / kVRows * kVRows;
    if (kc > kVMaxKc) return HMOE_UNSUPPORTED;
    // One token per pass when no expert holds more (a single-token batch
    // without shared experts); otherwise four.
    const int tok = r.max_group <= 1 ? 1 : 4;
    const GemvSmem L = gemv_smem(gate_up ? 2 : 1, tok, kc);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(g.KS), static_cast<unsigned>(col_blocks),
                       static_cast<unsigned>(r.tile_cap));
    cfg.blockDim = dim3(kVThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(L.total);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(g.KS);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err;
    if (gate_up)
        err = tok == 1 ? launch_gemv_variant<true, 1>(cfg, m0, m1, g, kc)
                       : launch_gemv_variant<true, 4>(cfg, m0, m1, g, kc);
    else
        err = tok == 1 ? launch_gemv_variant<false, 1>(cfg, m0, m1, g, kc)
                       : launch_gemv_variant<false, 4>(cfg, m0, m1, g, kc);
    if (err != cudaSuccess) {
        set_last_error("hmoe expert GEMV launch", err);
        return HMOE_CUDA_ERROR;
    }
    return check_launch("hmoe expert GEMV");
}

GemvArgs gemv_common(const ExpertRun& r) {
    GemvArgs g{};
    g.tiles = r.tiles;
    g.tile_count = r.tile_count;
    g.quant = r.quant;
    g.st = r.st;
    return g;
}

} // namespace

// gate/up of every tile, weight-streaming GEMV variant.
hmoe_status gemv_gate_up(const ExpertRun& r, cudaStream_t s) {
    GemvArgs g = gemv_common(r);
    g.act16 = r.xrows;
    g.xscale = r.xscale;
    g.proj0 = 0;
    g.out32 = r.hmid32;
    g.K = r.H;
    g.N = r.I;
    CUtensorMap mg, mu;
    if (!map_weights_box(&mg, r.arena + r.gate_offset, r.I, r.H, r.experts, r.stride, kVCols, kVRows) ||
        !map_weights_box(&mu, r.arena + r.up_offset, r.I, r.H, r.experts, r.stride, kVCols, kVRows)) {
        set_last_error_text("hmoe: cuTensorMapEncodeTiled failed (GEMV gate/up)");
        return HMOE_CUDA_ERROR;
    }
    return launch_gemv(true, r, mg, mu, g, s);
}

// down of every tile with the routing weight, weight-streaming GEMV variant.
hmoe_status gemv_down(const ExpertRun& r, cudaStream_t s) {
    GemvArgs g = gemv_common(r);
    g.act32 = r.hmid32;
    g.weight = r.weight;
    g.proj0 = 2;
    g.out16 = r.yrows;
    g.push = r.push;
    g.K = r.I;
    g.N = r.H;
    CUtensorMap md;
    if (!map_weights_box(&md, r.arena + r.down_offset, r.H, r.I, r.experts, r.stride, kVCols, kVRows)) {
        set_last_error_text("hmoe: cuTensorMapEncodeTiled failed (GEMV down)");
        return HMOE_CUDA_ERROR;
    }
    return launch_gemv(false, r, md, md, g, s);
}

} // namespace hmoe
