// expert_gemm_sm100.cu -- grouped INT8-weight expert GEMM on the 5th-
// generation tensor cores (tcgen05 + TMEM), for expert groups with many
// tokens (prefill).
//
// Replaces, for those groups, the three per-expert INT8 projections of
// ExpertMlpExecutor::execute (src/experts/ExpertExecutor.cpp:118-131),
// out[r,c] = sum_k x[r,k] * (float(q[k,c] - zp) * scale)
// (CpuTensorBackend.cpp:173-186 / CudaKernels.cu:30-107), together with
// the SiLU, the multiply and the routing weight.
//
// Formulation ("weights as M"): for expert e, output features n and tokens
// t, D[n, t] = sum_k W[k, n] * X[t, k].  The INT8 weight tile W[k0:k0+64,
// n0:n0+128] ([in,out] row-major, i.e. the packed layout as stored) is the
// MN-major A operand; the token tile (BF16 rows, K contiguous) is the
// K-major B operand; M = 128 features, N = up to 128 tokens, so one tile
// serves 1..128 tokens of an expert and decode-sized and prefill-sized
// groups use the same code.
//
// Per CTA (192 threads, one output tile):
//   warp 0     TMA producer: INT8 weight tile(s) (3-D map over the expert
//              arena) and the BF16 token tile (128-byte swizzle) per
//              64-deep K block, into a 3/4-stage ring.
//   warp 1     MMA issuer: one thread issues tcgen05.mma (BF16 x BF16 ->
//              FP32 in TMEM) and tcgen05.commit to release each stage.
//   warps 2-5  dequantise: INT8 -> exact BF16 (q - zp, |q - zp| <= 255) into
//              the swizzled MN-major A layout, fence to the async proxy,
//              signal the MMA thread; then the epilogue: tcgen05.ld the
//              accumulators, apply the projection scale, SwiGLU (gate/up,
//              BF16 out) or the routing weight (down, FP32 out).
// Every mbarrier wait is bounded in time; on expiry the CTA records
// HMOE_TIMEOUT in the workspace status word, drains its own TMA loads and
// MMAs (again bounded), frees its TMEM and exits.
#include "common.cuh"
#include "layer.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>

#include <mutex>

namespace hmoe {

namespace {

constexpr int kTileM = 128;   // output features per CTA (MMA M)
constexpr int kTileT = 128;   // tokens per tile (MMA N <= 128)
constexpr int kBK = 64;       // K per stage (128 bytes of BF16)
constexpr int kThreadsGemm = 192;
constexpr uint64_t kWaitNs = 2000000000ull; // 2 s per wait

constexpr int kABytes = kTileM * kBK * 2;   // 16 KB BF16 A tile
constexpr int kBBytes = kTileT * kBK * 2;   // 16 KB BF16 B tile
constexpr int kSBytes = kTileM * kBK;       // 8 KB INT8 staging tile

template <bool GATE_UP>
struct Cfg {
    static constexpr int NP = GATE_UP ? 2 : 1;                  // projections
    static constexpr int kStages = GATE_UP ? 3 : 4;
    static constexpr int kStageBytes = NP * (kABytes + kSBytes) + kBBytes;
    static constexpr int kTmemCols = GATE_UP ? 256 : 128;
    static constexpr int kSmem = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

struct GemmArgs {
    const int4* tiles;          // (expert, first row, rows, 0)
    const int32_t* tile_count;
    const hmoe_expert_quant* quant;
    int proj0;                  // quant index of the first projection
    const float* perm_weight;   // down: routing weight per row
    void* out;                  // gate/up: BF16 hmid [R,N]; down: FP32 rows [R,N]
    int K, N;
    DeviceStatus* st;
};

__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// 16 INT8 weights (one 16-byte chunk of a staging row) -> 16 BF16 values
// q - zp, exact.  (u + 2^23) - (2^23 + 128 + zp) with u = q + 128.
__device__ __forceinline__ void dequant16(const uint4 q, float off, uint32_t (&o)[8]) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t u = w[i] ^ 0x80808080u;
        const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - off;
        const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - off;
        const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - off;
        const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - off;
        o[2 * i] = bf16x2(f0, f1);
        o[2 * i + 1] = bf16x2(f2, f3);
    }
}

// Staging [64 k][128 n] INT8 -> A [2 atoms of 64 n][64 k][128 B], 128-byte
// swizzle (16-byte chunk index XOR (k mod 8)).  128 threads, 4 chunks each.
__device__ __forceinline__ void dequant_tile(const uint8_t* stage, uint8_t* a, float off, int dt) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int c = dt + 128 * i;  // 16-byte chunk of the staging tile
        const int k = c >> 3, j = c & 7;
        const uint4 q = *reinterpret_cast<const uint4*>(stage + k * 128 + j * 16);
        uint32_t o[8];
        dequant16(q, off, o);
        const int atom = j >> 2, cc = (j & 3) * 2;
        uint8_t* row = a + atom * 8192 + k * 128;
        *reinterpret_cast<uint4*>(row + ((cc ^ (k & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(row + (((cc + 1) ^ (k & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

template <bool GATE_UP>
__global__ void __launch_bounds__(kThreadsGemm, 1)
    expert_gemm_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                       const __grid_constant__ CUtensorMap tm_b, GemmArgs a) {
    using C = Cfg<GATE_UP>;
    constexpr int S = C::kStages;
    const int tile = blockIdx.y;
    if (tile >= *a.tile_count) return; // whole CTA, before any barrier or TMEM use

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // stage s: [A0 | A1 | B | S0 | S1]
    auto A = [&](int s, int p) { return smem + s * C::kStageBytes + p * kABytes; };
    auto B = [&](int s) { return smem + s * C::kStageBytes + C::NP * kABytes; };
    auto Sg = [&](int s, int p) { return smem + s * C::kStageBytes + C::NP * kABytes + kBBytes + p * kSBytes; };
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * C::kStageBytes);
    uint64_t* full = bars;
    uint64_t* aready = bars + S;
    uint64_t* empty = bars + 2 * S;
    uint64_t* accfull = bars + 3 * S;
    uint32_t* tmem_s = reinterpret_cast<uint32_t*>(bars + 3 * S + 1);
    volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_s + 1);

    const int4 td = a.tiles[tile];
    const int e = td.x, row0 = td.y, rows = td.z;
    const int n0 = blockIdx.x * kTileM;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkb = a.K / kBK;

    if (warp == 0) {
        sm100::tmem_alloc(tmem_s, C::kTmemCols);
        sm100::tmem_relinquish();
    }
    if (threadIdx.x == 32) {
        for (int s = 0; s < S; ++s) {
            sm100::mbar_init(&full[s], 1);
            sm100::mbar_init(&aready[s], 4);
            sm100::mbar_init(&empty[s], 1);
        }
        sm100::mbar_init(accfull, 1);
        *abort_s = 0;
        sm100::fence_mbarrier_init();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = *tmem_s;
    const uint32_t nmma = static_cast<uint32_t>((rows + 15) & ~15);

    auto fail = [&]() {
        *abort_s = 1;
        device_fail(a.st, HMOE_TIMEOUT);
    };

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------ TMA producer
        sm100::prefetch_tmap(&tm_w0);
        if (GATE_UP) sm100::prefetch_tmap(&tm_w1);
        sm100::prefetch_tmap(&tm_b);
        constexpr uint32_t bytes = C::NP * kSBytes + kBBytes;
        int issued = 0;
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % S;
            if (kb >= S && !sm100::mbar_wait(&empty[s], ((kb / S) - 1) & 1, abort_s, kWaitNs)) {
                fail();
                break;
            }
            sm100::mbar_arrive_expect_tx(&full[s], bytes);
            sm100::tma_load_3d(Sg(s, 0), &tm_w0, n0, kb * kBK, e, &full[s]);
            if (GATE_UP) sm100::tma_load_3d(Sg(s, 1), &tm_w1, n0, kb * kBK, e, &full[s]);
            sm100::tma_load_2d(B(s), &tm_b, kb * kBK, row0, &full[s]);
            issued = kb + 1;
        }
        if (*abort_s) {
            // drain this CTA's own loads still in flight before exit
            for (int kb = (issued > S ? issued - S : 0); kb < issued; ++kb)
                sm100::mbar_wait_for(&full[kb % S], (kb / S) & 1, kWaitNs);
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------ MMA issuer
        const uint32_t idesc = sm100::make_idesc_bf16(kTileM, nmma, true, false);
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % S;
            if (!sm100::mbar_wait(&full[s], (kb / S) & 1, abort_s, kWaitNs) ||
                !sm100::mbar_wait(&aready[s], (kb / S) & 1, abort_s, kWaitNs)) {
                fail();
                break;
            }
            sm100::tc_fence_after();
            const uint32_t b0 = sm100::smem_u32(B(s));
#pragma unroll
            for (int ks = 0; ks < kBK / 16; ++ks) {
                const uint64_t bd = sm100::make_smem_desc(b0 + ks * 32, 16, 1024, 2);
#pragma unroll
                for (int p = 0; p < C::NP; ++p) {
                    const uint64_t ad = sm100::make_smem_desc(sm100::smem_u32(A(s, p)) + ks * 2048, 8192, 1024, 2);
                    sm100::mma_bf16(tmem + p * 128, ad, bd, idesc, (kb | ks) != 0);
                }
            }
            sm100::mma_commit(&empty[s]);
        }
        sm100::mma_commit(accfull); // also on abort: completes once issued MMAs finish
    } else if (warp >= 2) {
        // ------------------------------------------------ dequant + epilogue
        const int dt = threadIdx.x - 64;
        const hmoe_expert_quant qp = a.quant[e];
        const float off0 = 8388608.0f + 128.0f + static_cast<float>(qp.zero_point[a.proj0]);
        const float off1 = GATE_UP ? 8388608.0f + 128.0f + static_cast<float>(qp.zero_point[a.proj0 + 1]) : 0.0f;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % S;
            if (!sm100::mbar_wait(&full[s], (kb / S) & 1, abort_s, kWaitNs)) {
                fail();
                ok = false;
                break;
            }
            dequant_tile(Sg(s, 0), A(s, 0), off0, dt);
            if (GATE_UP) dequant_tile(Sg(s, 1), A(s, 1), off1, dt);
            sm100::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&aready[s]);
        }
        if (ok && sm100::mbar_wait(accfull, 0, abort_s, kWaitNs)) {
            sm100::tc_fence_after();
            const int q = warp & 3;            // TMEM lane quarter of this warp
            const int m = q * 32 + lane;       // output feature within the tile
            const int n = n0 + m;
            const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
            if (GATE_UP) {
                const float sg = qp.scale[a.proj0], su = qp.scale[a.proj0 + 1];
                __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
                for (uint32_t c0 = 0; c0 < nmma; c0 += 32) {
                    uint32_t g[32], u[32];
                    sm100::tmem_ld32(lane_addr + c0, g);
                    sm100::tmem_ld32(lane_addr + 128 + c0, u);
                    sm100::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int t = static_cast<int>(c0) + j;
                        if (t < rows && n < a.N) {
                            const float gv = sg * __uint_as_float(g[j]);
                            const float uv = su * __uint_as_float(u[j]);
                            out[static_cast<size_t>(row0 + t) * a.N + n] = __float2bfloat16_rn(silu(gv) * uv);
                        }
                    }
                }
            } else {
                const float sd = qp.scale[a.proj0];
                float* out = static_cast<float*>(a.out);
                for (uint32_t c0 = 0; c0 < nmma; c0 += 32) {
                    uint32_t d[32];
                    sm100::tmem_ld32(lane_addr + c0, d);
                    sm100::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int t = static_cast<int>(c0) + j;
                        if (t < rows && n < a.N)
                            out[static_cast<size_t>(row0 + t) * a.N + n] =
                                a.perm_weight[row0 + t] * (sd * __uint_as_float(d[j]));
                    }
                }
            }
        } else if (ok) {
            fail();
        }
    }
    // teardown: every thread arrives here, including after an abort
    sm100::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        // after an abort, let the MMAs already issued finish before freeing TMEM
        if (*abort_s) sm100::mbar_wait_for(accfull, 0, kWaitNs);
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem, C::kTmemCols);
    }
}

// Builds the GEMM tile list: every expert on the large list is cut into
// tiles of at most kTileT consecutive permuted rows.
__global__ void tile_list_kernel(const int32_t* large_list, const int32_t* list_sizes, const int32_t* offsets,
                                 int4* tiles, int32_t* tile_count, int capacity) {
    if (threadIdx.x != 0) return;
    int n = 0;
    const int nl = list_sizes[1];
    for (int i = 0; i < nl; ++i) {
        const int e = large_list[i];
        const int r0 = offsets[e], cnt = offsets[e + 1] - r0;
        for (int j = 0; j < cnt && n < capacity; j += kTileT) tiles[n++] = make_int4(e, r0 + j, min(kTileT, cnt - j), 0);
    }
    *tile_count = n;
}

// X_perm[row] = BF16(x[perm_token[row]]) for the rows of every GEMM tile.
__global__ void __launch_bounds__(256) permute_kernel(const float* __restrict__ x, const uint32_t* __restrict__ perm_token,
                                                      const int4* tiles, const int32_t* tile_count, int H,
                                                      __nv_bfloat16* __restrict__ xperm) {
    if (static_cast<int>(blockIdx.x) >= *tile_count) return;
    const int4 td = tiles[blockIdx.x];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = warp; r < td.z; r += 8) {
        const int row = td.y + r;
        const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(perm_token[row]) * H);
        uint4* dst = reinterpret_cast<uint4*>(xperm + static_cast<size_t>(row) * H);
        for (int c = lane; c < H / 8; c += 32) {
            const float4 v0 = src[2 * c], v1 = src[2 * c + 1];
            dst[c] = make_uint4(bf16x2(v0.x, v0.y), bf16x2(v0.z, v0.w), bf16x2(v1.x, v1.y), bf16x2(v1.z, v1.w));
        }
    }
}

// ---------------------------------------------------------------- host

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// INT8 weights of one projection across all experts: dims {N, K, experts}.
bool map_weights(CUtensorMap* m, const int8_t* base, int N, int K, int experts, uint64_t stride) {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(K),
                                static_cast<cuuint64_t>(experts)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(N), stride};
    const cuuint32_t box[3] = {kTileM, kBK, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(base), dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// BF16 rows [rows, K] (K contiguous), 128-byte swizzle, box 64 x kTileT.
bool map_rows(CUtensorMap* m, const void* base, int K, int rows) {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {kBK, kTileT};
    const cuuint32_t es[2] = {1, 1};
    return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool GATE_UP>
hmoe_status launch_gemm(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& b, const GemmArgs& args,
                        int tile_capacity, cudaStream_t s) {
    using C = Cfg<GATE_UP>;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(expert_gemm_kernel<GATE_UP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
        attr = true;
    }
    const dim3 grid(static_cast<unsigned>((args.N + kTileM - 1) / kTileM), static_cast<unsigned>(tile_capacity));
    expert_gemm_kernel<GATE_UP><<<grid, kThreadsGemm, C::kSmem, s>>>(w0, w1, b, args);
    return check_launch(GATE_UP ? "hmoe expert GEMM gate/up" : "hmoe expert GEMM down");
}

int tile_capacity(const hmoe_layer_desc& d, size_t T, int list_capacity) {
    const long rows = static_cast<long>(T) * (d.top_k + d.shared_experts);
    return static_cast<int>(rows / kTileT + list_capacity + 1);
}

} // namespace

bool gemm_available() {
    static int avail = -1;
    if (avail < 0) {
        int dev = 0, major = 0, minor = 0;
        avail = cudaGetDevice(&dev) == cudaSuccess &&
                cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess &&
                cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) == cudaSuccess &&
                major == 10 && minor == 0 && encode_fn() != nullptr;
        cudaGetLastError();
    }
    return avail == 1;
}

hmoe_status launch_expert_gemm_gate_up(const hmoe_layer_desc& d, const float* x, size_t T, char* ws,
                                       const Workspace& w, int list_capacity, cudaStream_t s) {
    const int H = static_cast<int>(d.hidden), I = static_cast<int>(d.intermediate);
    const int E = static_cast<int>(d.experts + d.shared_experts);
    const int cap = tile_capacity(d, T, list_capacity);
    const int R = static_cast<int>(T * (d.top_k + d.shared_experts));
    auto* tiles = reinterpret_cast<int4*>(ws + w.tiles);
    auto* tcount = reinterpret_cast<int32_t*>(ws + w.tile_count);
    tile_list_kernel<<<1, 32, 0, s>>>(reinterpret_cast<int32_t*>(ws + w.large_list),
                                      reinterpret_cast<int32_t*>(ws + w.list_sizes),
                                      reinterpret_cast<int32_t*>(ws + w.offsets), tiles, tcount, cap);
    hmoe_status r = check_launch("hmoe tile list");
    if (r != HMOE_OK) return r;
    auto* xperm = reinterpret_cast<__nv_bfloat16*>(ws + w.xperm);
    permute_kernel<<<cap, 256, 0, s>>>(x, reinterpret_cast<uint32_t*>(ws + w.perm_token), tiles, tcount, H, xperm);
    r = check_launch("hmoe permute");
    if (r != HMOE_OK) return r;
    CUtensorMap mg, mu, mb;
    if (!map_weights(&mg, d.arena + d.gate_offset, I, H, E, d.expert_stride) ||
        !map_weights(&mu, d.arena + d.up_offset, I, H, E, d.expert_stride) || !map_rows(&mb, xperm, H, R)) {
        set_last_error_text("hmoe: cuTensorMapEncodeTiled failed (gate/up)");
        return HMOE_CUDA_ERROR;
    }
    GemmArgs a{tiles, tcount, d.quant, 0, nullptr, ws + w.hmid16, H, I,
               reinterpret_cast<DeviceStatus*>(ws + w.status)};
    return launch_gemm<true>(mg, mu, mb, a, cap, s);
}

hmoe_status launch_expert_gemm_down(const hmoe_layer_desc& d, size_t T, char* ws, const Workspace& w,
                                    int list_capacity, cudaStream_t s) {
    const int H = static_cast<int>(d.hidden), I = static_cast<int>(d.intermediate);
    const int E = static_cast<int>(d.experts + d.shared_experts);
    const int cap = tile_capacity(d, T, list_capacity);
    const int R = static_cast<int>(T * (d.top_k + d.shared_experts));
    CUtensorMap md, mb;
    if (!map_weights(&md, d.arena + d.down_offset, H, I, E, d.expert_stride) ||
        !map_rows(&mb, ws + w.hmid16, I, R)) {
        set_last_error_text("hmoe: cuTensorMapEncodeTiled failed (down)");
        return HMOE_CUDA_ERROR;
    }
    GemmArgs a{reinterpret_cast<int4*>(ws + w.tiles), reinterpret_cast<int32_t*>(ws + w.tile_count), d.quant, 2,
               reinterpret_cast<float*>(ws + w.perm_weight), ws + w.yrows, I, H,
               reinterpret_cast<DeviceStatus*>(ws + w.status)};
    return launch_gemm<false>(md, md, mb, a, cap, s);
}

} // namespace hmoe
