// expert_gemv.cu -- split-K weight-streaming INT8 expert projections for
// expert groups with few tokens (decode), where the layer is HBM-bound.
//
// Replaces, for those groups, the per-expert projections of
// ExpertMlpExecutor::execute (src/experts/ExpertExecutor.cpp:118-131) that
// the reference runs as int8WeightMatmulKernel / cooperativeInt8Kernel
// (src/backend/cuda/CudaKernels.cu:30-107) plus activationKernel and a
// cuBLAS multiply.
//
// One launch handles every tile of the device-built tile list.  A thread
// block cluster of KS CTAs owns (tile, 256 output columns); CTA r of the
// cluster streams rows [r*K/KS, (r+1)*K/KS) of the INT8 weight matrix
// ([K,N] row-major, each lane reading 8 consecutive columns with one 64-bit
// load per row) and accumulates x * (q - zp) in FP32 for every token of the
// group.  The KS partial tiles are summed through distributed shared memory
// in rank order -- a fixed order, so results are deterministic and no
// global scratch or atomics are needed.  The epilogue applies the
// projection scale and either SwiGLU (gate/up: h = SiLU(sg*G) * (su*U)) or
// the routing weight (down: y = w * sd * D).
#include "common.cuh"
#include "layer.cuh"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace hmoe {

constexpr int kGemvWarps = 8;
constexpr int kGemvCols = 256; // 32 lanes x 8 columns
constexpr int kGemvRows = 8;   // weight rows in flight per lane



template <bool GATE_UP, int kGemvTokens>
__global__ void __launch_bounds__(kGemvWarps * 32) expert_gemv_kernel(GemvArgs a) {
    constexpr int NP = GATE_UP ? 2 : 1;
    extern __shared__ __align__(16) float gsm[];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int KS = a.KS;
    if (static_cast<int>(blockIdx.z) >= *a.tile_count) return; // whole cluster exits together
    const int4 td = a.tiles[blockIdx.z];
    const int e = td.x;
    const int r0 = td.y;
    const int n = td.z;
    const int K = a.K, N = a.N;
    const int KP = (K + KS - 1) / KS;
    const int kb = min(K, rank * KP), ke = min(K, kb + KP);
    const int kc = ke - kb;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int col = blockIdx.y * kGemvCols + lane * 8;
    const bool col_ok = col < N;

    float* xs = gsm;                                        // [kGemvTokens][KP]
    float* red = xs + kGemvTokens * KP;                     // [warps][tokens][NP][256]
    float* part = red + kGemvWarps * kGemvTokens * NP * kGemvCols; // [tokens][NP][256]

    const int8_t* base = a.arena + static_cast<uint64_t>(e) * a.stride;
    const int8_t* w0 = base + a.off0;
    const int8_t* w1 = base + a.off1;
    const hmoe_expert_quant qp = a.quant[e];
    const float zp0 = static_cast<float>(qp.zero_point[a.proj0]);
    const float zp1 = GATE_UP ? static_cast<float>(qp.zero_point[a.proj0 + 1]) : 0.0f;

    for (int j0 = 0; j0 < n; j0 += kGemvTokens) {
        const int nj = min(kGemvTokens, n - j0);
        for (int i = tid; i < kGemvTokens * kc; i += blockDim.x) {
            const int t = i / kc, kk = i % kc;
            float v = 0.0f;
            if (t < nj) {
                const size_t row = static_cast<size_t>(r0 + j0 + t);
                if constexpr (GATE_UP)
                    v = __bfloat162float(a.act16[row * K + kb + kk]);
                else
                    v = a.act32[row * K + kb + kk];
            }
            xs[t * KP + kk] = v;
        }
        __syncthreads();
        float acc[kGemvTokens][NP][8];
#pragma unroll
        for (int t = 0; t < kGemvTokens; ++t)
#pragma unroll
            for (int p = 0; p < NP; ++p)
#pragma unroll
                for (int c = 0; c < 8; ++c) acc[t][p][c] = 0.0f;
        if (col_ok) {
            // kGemvRows weight rows per lane are loaded before any is used,
            // so every lane keeps kGemvRows x NP 8-byte loads in flight.
            for (int k0 = warp; k0 < kc; k0 += kGemvWarps * kGemvRows) {
                uint2 qv[kGemvRows][NP];
#pragma unroll
                for (int r = 0; r < kGemvRows; ++r) {
                    const int kk = k0 + r * kGemvWarps;
                    if (kk < kc) {
                        const size_t off = static_cast<size_t>(kb + kk) * N + col;
                        qv[r][0] = __ldg(reinterpret_cast<const uint2*>(w0 + off));
                        if constexpr (GATE_UP) qv[r][1] = __ldg(reinterpret_cast<const uint2*>(w1 + off));
                    } else {
                        qv[r][0] = make_uint2(0u, 0u);
                        if constexpr (GATE_UP) qv[r][1] = make_uint2(0u, 0u);
                    }
                }
#pragma unroll
                for (int r = 0; r < kGemvRows; ++r) {
                    const int kk = k0 + r * kGemvWarps;
                    if (kk >= kc) break;
                    float wv[NP][8];
#pragma unroll
                    for (int p = 0; p < NP; ++p) {
                        dequant4(qv[r][p].x, p ? zp1 : zp0, &wv[p][0]);
                        dequant4(qv[r][p].y, p ? zp1 : zp0, &wv[p][4]);
                    }
#pragma unroll
                    for (int t = 0; t < kGemvTokens; ++t) {
                        if (t < nj) {
                            const float xv = xs[t * KP + kk];
#pragma unroll
                            for (int p = 0; p < NP; ++p)
#pragma unroll
                                for (int c = 0; c < 8; ++c) acc[t][p][c] = fmaf(xv, wv[p][c], acc[t][p][c]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kGemvTokens; ++t)
#pragma unroll
            for (int p = 0; p < NP; ++p) {
                float4* dst = reinterpret_cast<float4*>(red + ((warp * kGemvTokens + t) * NP + p) * kGemvCols + lane * 8);
                dst[0] = make_float4(acc[t][p][0], acc[t][p][1], acc[t][p][2], acc[t][p][3]);
                dst[1] = make_float4(acc[t][p][4], acc[t][p][5], acc[t][p][6], acc[t][p][7]);
            }
        __syncthreads();
        for (int i = tid; i < kGemvTokens * NP * kGemvCols; i += blockDim.x) {
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < kGemvWarps; ++w) s += red[w * kGemvTokens * NP * kGemvCols + i];
            part[i] = s;
        }
        cluster.sync();
        // Rank r finalises a slice of the columns, summing ranks in order.
        const int slice = kGemvCols / KS;
        for (int i = tid; i < kGemvTokens * slice; i += blockDim.x) {
            const int t = i / slice;
            const int cl = rank * slice + i % slice;
            const int c = blockIdx.y * kGemvCols + cl;
            if (t >= nj || c >= N) continue;
            float s0 = 0.0f, s1 = 0.0f;
            for (int r = 0; r < KS; ++r) {
                const float* rp = cluster.map_shared_rank(part, r);
                s0 += rp[(t * NP + 0) * kGemvCols + cl];
                if constexpr (GATE_UP) s1 += rp[(t * NP + 1) * kGemvCols + cl];
            }
            const int row = r0 + j0 + t;
            if constexpr (GATE_UP) {
                const float g = qp.scale[a.proj0] * s0;
                const float u = qp.scale[a.proj0 + 1] * s1;
                a.out32[static_cast<size_t>(row) * N + c] = silu(g) * u;
            } else {
                a.out16[static_cast<size_t>(row) * N + c] = __float2bfloat16_rn(a.weight[row] * (qp.scale[a.proj0] * s0));
            }
        }
        cluster.sync();
    }
}

size_t gemv_smem_bytes(int K, int KS, bool gate_up, int tokens) {
    const int NP = gate_up ? 2 : 1;
    const int KP = (K + KS - 1) / KS;
    return static_cast<size_t>(tokens * KP + kGemvWarps * tokens * NP * kGemvCols + tokens * NP * kGemvCols) *
           sizeof(float);
}

template <bool GATE_UP, int TOK>
cudaError_t launch_gemv_variant(cudaLaunchConfig_t& cfg, const GemvArgs& args) {
    static size_t attr_set = 0;
    if (cfg.dynamicSmemBytes > attr_set) {
        cudaFuncSetAttribute(expert_gemv_kernel<GATE_UP, TOK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(cfg.dynamicSmemBytes));
        attr_set = cfg.dynamicSmemBytes;
    }
    return cudaLaunchKernelEx(&cfg, expert_gemv_kernel<GATE_UP, TOK>, args);
}

hmoe_status launch_expert_gemv(bool gate_up, const GemvArgs& args, int list_capacity, int max_tokens,
                               cudaStream_t stream) {
    if (list_capacity <= 0) return HMOE_OK;
    if (list_capacity > 65535) return HMOE_UNSUPPORTED;
    // One token per pass when no expert can hold more (a single-token
    // batch without shared experts); otherwise four.
    const int tok = max_tokens <= 1 ? 1 : 4;
    const size_t smem = gemv_smem_bytes(args.K, args.KS, gate_up, tok);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(args.KS), static_cast<unsigned>((args.N + kGemvCols - 1) / kGemvCols),
                       static_cast<unsigned>(list_capacity));
    cfg.blockDim = dim3(kGemvWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(args.KS);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err;
    if (gate_up)
        err = tok == 1 ? launch_gemv_variant<true, 1>(cfg, args) : launch_gemv_variant<true, 4>(cfg, args);
    else
        err = tok == 1 ? launch_gemv_variant<false, 1>(cfg, args) : launch_gemv_variant<false, 4>(cfg, args);
    if (err != cudaSuccess) {
        set_last_error("hmoe expert GEMV launch", err);
        return HMOE_CUDA_ERROR;
    }
    return check_launch("hmoe expert GEMV");
}

namespace {

int gemv_split(int capacity, int col_blocks) {
    int ks = 1;
    while (ks < 8 && static_cast<long>(capacity) * col_blocks * ks < 2L * 148) ks *= 2;
    return ks;
}

GemvArgs gemv_common(const ExpertRun& r) {
    GemvArgs g{};
    g.tiles = r.tiles;
    g.tile_count = r.tile_count;
    g.arena = r.arena;
    g.stride = r.stride;
    g.quant = r.quant;
    return g;
}

} // namespace

// gate/up of every tile, weight-streaming GEMV variant.
hmoe_status gemv_gate_up(const ExpertRun& r, cudaStream_t s) {
    GemvArgs g = gemv_common(r);
    g.act16 = r.xrows;
    g.off0 = r.gate_offset;
    g.off1 = r.up_offset;
    g.proj0 = 0;
    g.out32 = r.hmid32;
    g.K = r.H;
    g.N = r.I;
    g.KS = gemv_split(r.tile_cap, (r.I + 255) / 256);
    return launch_expert_gemv(true, g, r.tile_cap, r.max_group, s);
}

// down of every tile with the routing weight, weight-streaming GEMV variant.
hmoe_status gemv_down(const ExpertRun& r, cudaStream_t s) {
    GemvArgs g = gemv_common(r);
    g.act32 = r.hmid32;
    g.weight = r.weight;
    g.off0 = r.down_offset;
    g.proj0 = 2;
    g.out16 = r.yrows;
    g.K = r.I;
    g.N = r.H;
    g.KS = gemv_split(r.tile_cap, (r.H + 255) / 256);
    return launch_expert_gemv(false, g, r.tile_cap, r.max_group, s);
}

} // namespace hmoe
