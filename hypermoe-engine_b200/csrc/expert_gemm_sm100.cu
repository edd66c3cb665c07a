// expert_gemm_sm100.cu -- grouped INT8-weight expert GEMM on the 5th-
// generation tensor cores (tcgen05 + TMEM).
//
// Replaces the three per-expert INT8 projections of ExpertMlpExecutor::
// execute (src/experts/ExpertExecutor.cpp:118-131),
//     out[r,c] = sum_k x[r,k] * (float(q[k,c] - zp) * scale)
// (CpuTensorBackend.cpp:173-186; the reference's CUDA kernels
// CudaKernels.cu:30-107), together with the SiLU, the elementwise multiply
// and the routing weight, for every expert of the layer in one launch per
// projection pair.
//
// Formulation ("weights as M"): for expert e, output features n and tokens
// t, D[n, t] = sum_k W[k, n] * X[t, k].  The INT8 weight tile W[k0:k0+128,
// n0:n0+128] -- the packed [in,out] layout exactly as stored -- becomes the
// MN-major 16-bit A operand after an exact in-shared-memory dequantisation
// (q - zp is an integer in [-255, 255], exact in FP16 and BF16); the
// expert's token rows (K contiguous, TMA with 128-byte swizzle) are the
// K-major B operand: FP16 rows scaled per token by a power of two for
// gate/up, BF16 SwiGLU rows for down.  M = 256 features per CTA pair,
// N = 16..256 tokens, FP32 accumulation in TMEM.
//
// Persistent kernel over CTA pairs (thread-block clusters of 2), one CTA per
// SM.  The pair runs the 2-SM MMA (tcgen05 .cta_group::2, M = 256): each CTA
// holds half of the A rows and half of the token tile, which halves the
// shared-memory traffic per MMA FLOP compared with one CTA.  For gate/up a
// CTA's 128 A rows are 64 gate features and the same 64 up features, so
// both projections come out of one MMA and SwiGLU stays inside the CTA.
// K advances 128 per stage: the issuing thread checks one barrier, issues 8
// MMAs and one commit per stage (its per-instruction issue cost, not the
// tensor core, bounds narrow tiles).
// Warp roles (19 warps per CTA):
//   warp 0      TMA producer of INT8 weight tiles (two [128 k][64 n] boxes per
//               stage, 3-deep staging ring)
//   warp 1      TMA producer of this CTA's half of the 16-bit token tile
//               (two 64-k boxes per stage; bytes counted on the leader's barrier)
//   warp 2      TMEM owner; in the leader CTA one thread issues the pair MMA
//               and multicasts tcgen05.commit to both CTAs' barriers
//   warps 3-10  dequantise INT8 -> FP16 (gate/up) or BF16 (down) into the
//               swizzled A layout; in the leader they also wait for the token
//               tile, so one barrier tells the MMA issuer the stage is ready
//   warps 11-18 epilogue: tcgen05.ld from double-buffered accumulators,
//               projection scale, SwiGLU (gate/up) or routing weight (down),
//               BF16 rows staged in shared memory and stored coalesced,
//               overlapping the next main loop.
// Work items are (token tile of <= 256 rows of one expert, feature block),
// longest tiles first, dealt round-robin to the pairs.
//
#include "common.cuh"
#include "layer.cuh"
#include "rows.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>
#include <cub/block/block_scan.cuh>

#include <algorithm>
#include <atomic>
#include <mutex>

namespace hmoe {

bool map_weights_box(CUtensorMap* m, const int8_t* base, int N, int K, int experts, uint64_t stride, int box_n,
                     int box_k);

namespace {

constexpr int kTileT = 256;   // tokens per work item (pair MMA N <= 256)
static_assert(kTileT == kTileRows, "GEMM work items are whole tiles");
constexpr int kBK = 128;      // K per stage: 8 MMAs (K = 16 each) per barrier round trip
constexpr int kDequantWarps = 8;
constexpr int kEpiWarps = 8;                // two groups of 4 (one per column half)
constexpr int kThreadsGemm = 32 * (3 + kDequantWarps + kEpiWarps);
constexpr uint64_t kWaitNs = 2000000000ull; // 2 s per wait
constexpr uint32_t kTmemCols = 512;         // 2 accumulator buffers x 256 columns

constexpr int kAAtom = 128 * kBK;           // one 64-row MN atom: 128 B x kBK k rows (16 KB)
constexpr int kABytes = 2 * kAAtom;         // 32 KB: 128 A rows (two 64-row atoms)
constexpr int kSBytes = 64 * kBK;           // 8 KB: one [128 k][64 n] INT8 box
// Epilogue scratch per column-half group, 8 KB: the gate/up exchange (2 x 64
// x 16 FP32), whose outputs are stored straight from registers (a warp's 32
// lanes hold 32 consecutive features of a token: one 64-byte run per token
// row); for down, the staging tile of 32 tokens x 128 BF16 features.
constexpr int kXchBytes = 2 * 64 * 16 * 4;  // 8 KB
constexpr int kXBytes = 2 * kXchBytes;

// Shared-memory plan of a kernel whose CTAs hold HT token rows (the token
// box height).  HT = 128 takes tiles of up to 256 rows.  HT = 32 takes tiles
// of up to 64 rows (decode-sized batches): its token stages are a quarter of
// the size, and the room they free deepens all three rings.  A narrow
// tile's MMAs take little time, so each ring's round trip (an INT8 stage:
// HBM latency; a token stage: L2 latency; an A stage: dequantise, arrive,
// MMA, commit) over its depth sets the pace.
template <int HT>
struct GemmCfg {
    static constexpr int kWStages = HT == 128 ? 3 : 4;   // INT8 staging ring
    static constexpr int kAStages = HT == 128 ? 2 : 3;   // A ring (dequantised weights)
    static constexpr int kBStages = HT == 128 ? 3 : 6;   // B ring (token rows): one more stage hides the L2 latency
    static constexpr int kBBox = HT * 64 * 2;            // one TMA box: HT token rows x 64 k
    static constexpr int kBBytes = 2 * kBBox;            // HT token rows x 128 k
    static constexpr int kSOff = 0;
    static constexpr int kAOff = kSOff + kWStages * 2 * kSBytes;
    static constexpr int kBOff = kAOff + kAStages * kABytes;
    static constexpr int kXOff = kBOff + kBStages * kBBytes;
    static constexpr int kBarOff = kXOff + kXBytes;
    static constexpr int kSmem = kBarOff + 512 + 1024 /*alignment slack*/;
    static_assert(HT == 128 || HT == 32, "token box heights");
    static_assert(kSmem <= 232448, "shared memory budget");
};
constexpr int kNarrowRows = 64; // largest tile of the HT = 32 kernel (two CTAs x 32 rows)

struct GemmArgs {
    const int4* tiles;          // (expert, first row, rows, 0), longest first
    const int32_t* tile_count;
    int nblocks;                // feature blocks per pair
    const hmoe_expert_quant* quant;
    const float* perm_weight;   // down: routing weight per row
    const float* xscale;        // gate/up: 1 / (power-of-two scale of each token row)
    void* out;                  // BF16 rows [R,N]: gate/up SwiGLU output; down weighted output
    int K, N;
    DeviceStatus* st;
    PushRows push;              // down: rows pushed to their sources (peer != null)
};

__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
}

// 16 INT8 weights -> 16 16-bit values q - zp, exact.
//  BF16: float(2^23 + u) - (2^23 + 128 + zp) with u = q + 128, packed
//        (BF16 keeps the integer exactly: |q - zp| <= 255 needs 8 bits).
//  FP16: two bytes at a time: the half pair (1024 + u0, 1024 + u1) built by
//        one byte permute, minus (1152 + zp) in both halves -- exact in FP16.
template <bool F16>
__device__ __forceinline__ void dequant16(const uint4 q, float off, uint32_t offh2, uint32_t (&o)[8]) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t u = w[i] ^ 0x80808080u;
        if constexpr (F16) {
            o[2 * i] = hsub2_u32(__byte_perm(u, 0x64646464u, 0x4140), offh2);
            o[2 * i + 1] = hsub2_u32(__byte_perm(u, 0x64646464u, 0x4342), offh2);
        } else {
            const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - off;
            const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - off;
            const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - off;
            const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - off;
            o[2 * i] = bf16x2(f0, f1);
            o[2 * i + 1] = bf16x2(f2, f3);
        }
    }
}

// (1152 + zp) in both halves of a half pair (exact: an integer below 2048).
__device__ __forceinline__ uint32_t f16_offset_pair(int zp) {
    const __half h = __int2half_rn(1152 + zp);
    const __half2 p = __halves2half2(h, h);
    return *reinterpret_cast<const uint32_t*>(&p);
}

// Two staging boxes [kBK k][64 n] INT8 (atom 0 and atom 1) -> A [2 atoms of
// 64 MN][kBK k][128 B] with the 128-byte swizzle (16-byte chunk index XOR
// (k mod 8)).  256 threads, four 16-byte input chunks each.  Eight
// consecutive threads cover rows k, k+1 (k even) of one box: their loads
// read two 64-byte rows that fall in different bank halves, and their
// 16-byte stores land in 8 distinct chunk positions (row k gets even
// chunks, row k+1 odd ones), so neither side has bank conflicts.
template <bool F16>
__device__ __forceinline__ void dequant_stage(const uint8_t* s0, const uint8_t* s1, uint8_t* a, float off0,
                                              float off1, uint32_t offh0, uint32_t offh1, int dt) {
#pragma unroll
    for (int i = 0; i < kBK / 32; ++i) {
        const int u = dt + 256 * i;
        const int q = u & 3, r = (u >> 2) & 1, atom = (u >> 3) & 1, kp = u >> 4;
        const int k = 2 * kp + r;
        const uint4 v = *reinterpret_cast<const uint4*>((atom ? s1 : s0) + k * 64 + q * 16);
        uint32_t o[8];
        dequant16<F16>(v, atom ? off1 : off0, atom ? offh1 : offh0, o);
        uint8_t* row = a + atom * kAAtom + k * 128;
        const int cc = 2 * q;
        *reinterpret_cast<uint4*>(row + ((cc ^ (k & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(row + (((cc + 1) ^ (k & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

// Named barrier of one epilogue group (4 warps; ids 1, 2; 0 = __syncthreads).
__device__ __forceinline__ void epi_barrier(int group) {
    asm volatile("bar.sync %0, 128;" ::"r"(group + 1) : "memory");
}

__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

template <bool GATE_UP, int HT>
__global__ void __launch_bounds__(kThreadsGemm, 1)
    expert_gemm_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                       const __grid_constant__ CUtensorMap tm_b, GemmArgs a) {
    using G = GemmCfg<HT>;
    constexpr int kWStages = G::kWStages, kAStages = G::kAStages, kBStages = G::kBStages;
    constexpr int kBBox = G::kBBox, kBBytes = G::kBBytes;
    constexpr int kSOff = G::kSOff, kAOff = G::kAOff, kBOff = G::kBOff, kXOff = G::kXOff, kBarOff = G::kBarOff;
    const int n_items = *a.tile_count * a.nblocks;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    if (pair >= n_items) return; // both CTAs of the pair, before any barrier/TMEM use
    const uint32_t rank = sm100::cluster_rank();
    const bool leader = rank == 0;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    auto S = [&](int s, int p) { return smem + kSOff + (s * 2 + p) * kSBytes; };
    auto A = [&](int s) { return smem + kAOff + s * kABytes; };
    auto B = [&](int s) { return smem + kBOff + s * kBBytes; };
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
    uint64_t* full_w = bars;                  // [kWStages] local: weights landed
    uint64_t* empty_w = full_w + kWStages;    // [kWStages] local: staging consumed
    uint64_t* full_b = empty_w + kWStages;    // [kBStages] leader: both token halves landed
    uint64_t* empty_b = full_b + kBStages;    // [kBStages] both: MMA done with the token stage
    uint64_t* aready = empty_b + kBStages;    // [kAStages] leader: A written in both CTAs, B landed
    uint64_t* empty_a = aready + kAStages;    // [kAStages] both: MMA done with the A stage
    uint64_t* accfull = empty_a + kAStages;   // [2] both: accumulator ready
    uint64_t* accempty = accfull + 2;         // [2] leader: both epilogues drained it
    uint64_t* drain = accempty + 2;           // [1] both: every MMA done
    uint32_t* tmem_s = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_s + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkb = a.K / kBK;

    if (warp == 2) {
        sm100::tmem_alloc_pair(tmem_s, kTmemCols);
        sm100::tmem_relinquish_pair();
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < kWStages; ++s) {
            sm100::mbar_init(&full_w[s], 1);
            sm100::mbar_init(&empty_w[s], kDequantWarps);
        }
        for (int s = 0; s < kBStages; ++s) {
            sm100::mbar_init(&full_b[s], 1);
            sm100::mbar_init(&empty_b[s], 1);
        }
        for (int s = 0; s < kAStages; ++s) {
            sm100::mbar_init(&aready[s], 2 * kDequantWarps);
            sm100::mbar_init(&empty_a[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            sm100::mbar_init(&accfull[b], 1);
            sm100::mbar_init(&accempty[b], 2 * kEpiWarps);
        }
        sm100::mbar_init(drain, 1);
        *abort_s = 0;
        sm100::fence_mbarrier_init();
    }
    sm100::tc_fence_before();
    sm100::cluster_sync_all(); // barriers of both CTAs initialised, TMEM allocated
    sm100::tc_fence_after();
    const uint32_t tmem = *tmem_s;

    auto fail = [&]() {
        *abort_s = 1;
        device_fail(a.st, HMOE_TIMEOUT);
    };

    // Role loops keep every warp converged: all 32 lanes run the loop and the
    // waits, lane 0 alone issues TMA / MMA instructions, then __syncwarp.
    if (warp == 0) {
        // ------------------------------------------------ INT8 weight producer
        if (lane == 0) {
            sm100::prefetch_tmap(&tm_w0);
            sm100::prefetch_tmap(&tm_w1);
        }
        uint32_t it = 0;
        for (int item = pair; item < n_items && !*abort_s; item += npairs) {
            const int4 td = a.tiles[item / a.nblocks];
            const int nb = item % a.nblocks;
            // gate/up: both boxes at the CTA's 64 features; down: two
            // adjacent 64-feature boxes of the CTA's 128 features
            const int x0 = GATE_UP ? nb * 128 + 64 * static_cast<int>(rank) : nb * 256 + 128 * static_cast<int>(rank);
            const int x1 = GATE_UP ? x0 : x0 + 64;
            bool ok = true;
            for (int kb = 0; kb < nkb; ++kb, ++it) {
                const int s = it % kWStages;
                if (it >= kWStages &&
                    !sm100::mbar_wait(&empty_w[s], ((it / kWStages) - 1) & 1, abort_s, kWaitNs)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    sm100::mbar_arrive_expect_tx(&full_w[s], 2 * kSBytes);
                    sm100::tma_load_3d(S(s, 0), &tm_w0, x0, kb * kBK, td.x, &full_w[s]);
                    sm100::tma_load_3d(S(s, 1), &tm_w1, x1, kb * kBK, td.x, &full_w[s]);
                }
                __syncwarp();
            }
            if (!ok) {
                if (lane == 0) fail();
                break;
            }
        }
        if (*abort_s) // drain this CTA's own loads before it exits
            for (uint32_t i = (it > kWStages ? it - kWStages : 0); i < it; ++i)
                sm100::mbar_wait_for(&full_w[i % kWStages], (i / kWStages) & 1, kWaitNs);
    } else if (warp == 1) {
        // ------------------------------------------------ 16-bit token-tile producer
        if (lane == 0) sm100::prefetch_tmap(&tm_b);
        uint32_t it = 0;
        for (int item = pair; item < n_items && !*abort_s; item += npairs) {
            const int4 td = a.tiles[item / a.nblocks];
            const int half = ((td.z + 15) & ~15) >> 1;
            const int y = td.y + static_cast<int>(rank) * half;
            bool ok = true;
            for (int kb = 0; kb < nkb; ++kb, ++it) {
                const int s = it % kBStages;
                if (it >= kBStages &&
                    !sm100::mbar_wait(&empty_b[s], ((it / kBStages) - 1) & 1, abort_s, kWaitNs)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint32_t bar = sm100::map_shared(sm100::smem_u32(&full_b[s]), 0);
                    if (leader) sm100::mbar_arrive_expect_tx(&full_b[s], 2 * kBBytes);
                    sm100::tma_load_2d_pair(B(s), &tm_b, kb * kBK, y, bar);
                    sm100::tma_load_2d_pair(B(s) + kBBox, &tm_b, kb * kBK + 64, y, bar);
                }
                __syncwarp();
            }
            if (!ok) {
                if (lane == 0) fail();
                break;
            }
        }
        // Both CTAs' token loads complete on the leader's barriers: after an
        // abort the leader waits for the last stages it saw issued, and the
        // teardown cluster barrier keeps the follower alive until then.
        if (*abort_s && leader)
            for (uint32_t i = (it > kBStages ? it - kBStages : 0); i < it; ++i)
                sm100::mbar_wait_for(&full_b[i % kBStages], (i / kBStages) & 1, kWaitNs);
    } else if (warp == 2) {
        // ------------------------------------------------ MMA issuer (leader)
        if (leader) {
            uint32_t it = 0;
            int j = 0;
            for (int item = pair; item < n_items && !*abort_s; item += npairs, ++j) {
                const int4 td = a.tiles[item / a.nblocks];
                const uint32_t nmma = static_cast<uint32_t>((td.z + 15) & ~15);
                // gate/up: FP16 operands (scaled token rows); down: BF16
                const uint32_t idesc = sm100::make_idesc_f16kind(256, nmma, true, false, !GATE_UP);
                const int buf = j & 1;
                if (j >= 2 && !sm100::mbar_wait_cluster(&accempty[buf], ((j >> 1) - 1) & 1, abort_s, kWaitNs)) {
                    if (lane == 0) fail();
                    break;
                }
                sm100::tc_fence_after();
                const uint32_t d0 = tmem + static_cast<uint32_t>(buf * kTileT);
                bool ok = true;
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % kAStages, bs = it % kBStages;
                    // aready implies the token tile landed: the leader's
                    // dequantisation warps wait for it before arriving.
                    if (!sm100::mbar_wait_cluster(&aready[s], (it / kAStages) & 1, abort_s, kWaitNs)) {
                        ok = false;
                        break;
                    }
                    sm100::tc_fence_after();
                    if (lane == 0) {
                        const uint32_t a0 = sm100::smem_u32(A(s)), b0 = sm100::smem_u32(B(bs));
#pragma unroll
                        for (int ks = 0; ks < kBK / 16; ++ks) {
                            const uint64_t ad = sm100::make_smem_desc(a0 + ks * 2048, kAAtom, 1024, 2);
                            const uint64_t bd =
                                sm100::make_smem_desc(b0 + (ks >> 2) * kBBox + (ks & 3) * 32, 16, 1024, 2);
                            sm100::mma_bf16_pair(d0, ad, bd, idesc, (kb | ks) != 0);
                        }
                        sm100::mma_commit_pair(&empty_a[s], 0x3);
                        sm100::mma_commit_pair(&empty_b[bs], 0x3);
                    }
                    __syncwarp();
                }
                if (!ok) {
                    if (lane == 0) fail();
                    break;
                }
                if (lane == 0) sm100::mma_commit_pair(&accfull[buf], 0x3);
                __syncwarp();
            }
            if (lane == 0) sm100::mma_commit_pair(drain, 0x3); // completes once every MMA has finished
            __syncwarp();
        }
    } else if (warp < 3 + kDequantWarps) {
        // ------------------------------------------------ dequantise
        const int dt = threadIdx.x - 96;
        uint32_t wi = 0, ai = 0;
        for (int item = pair; item < n_items && !*abort_s; item += npairs) {
            const int4 td = a.tiles[item / a.nblocks];
            const hmoe_expert_quant qp = a.quant[td.x];
            const float off0 = 8388608.0f + 128.0f + static_cast<float>(qp.zero_point[GATE_UP ? 0 : 2]);
            const float off1 = 8388608.0f + 128.0f + static_cast<float>(qp.zero_point[GATE_UP ? 1 : 2]);
            const uint32_t offh0 = f16_offset_pair(qp.zero_point[GATE_UP ? 0 : 2]);
            const uint32_t offh1 = f16_offset_pair(qp.zero_point[GATE_UP ? 1 : 2]);
            bool ok = true;
            for (int kb = 0; kb < nkb; ++kb, ++wi, ++ai) {
                const int ws = wi % kWStages, as = ai % kAStages, bs = ai % kBStages;
                if (!sm100::mbar_wait(&full_w[ws], (wi / kWStages) & 1, abort_s, kWaitNs) ||
                    (ai >= kAStages &&
                     !sm100::mbar_wait_cluster(&empty_a[as], ((ai / kAStages) - 1) & 1, abort_s, kWaitNs))) {
                    fail();
                    ok = false;
                    break;
                }
                dequant_stage<GATE_UP>(S(ws, 0), S(ws, 1), A(as), off0, off1, offh0, offh1, dt);
                sm100::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) sm100::mbar_arrive(&empty_w[ws]);
                if (leader && !sm100::mbar_wait(&full_b[bs], (ai / kBStages) & 1, abort_s, kWaitNs)) {
                    fail();
                    ok = false;
                    break;
                }
                if (lane == 0) sm100::mbar_arrive_remote(sm100::map_shared(sm100::smem_u32(&aready[as]), 0));
            }
            if (!ok) break;
        }
    } else {
        // ------------------------------------------------ epilogue
        // Two groups of 4 warps; group h handles the 32-column chunks with
        // index = h (mod 2).  Each warp reads its TMEM lane quarter q.
        const int e = warp - (3 + kDequantWarps);
        const int grp = e >> 2;
        const int q = warp & 3;                 // TMEM lane quarter of this warp
        const int m = q * 32 + lane;            // accumulator row (TMEM lane)
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
        uint8_t* xbase = smem + kXOff + grp * kXchBytes;
        float* xg = reinterpret_cast<float*>(xbase);            // [16 t][64 f] gate, tokens 16..31
        float* xu = xg + 64 * 16;                               // [16 t][64 f] up, tokens 0..15
        int j = 0;
        for (int item = pair; item < n_items && !*abort_s; item += npairs, ++j) {
            const int4 td = a.tiles[item / a.nblocks];
            const int row0 = td.y, rows = td.z;
            const int nb = item % a.nblocks;
            const uint32_t nmma = static_cast<uint32_t>((rows + 15) & ~15);
            const int buf = j & 1;
            if (!sm100::mbar_wait_cluster(&accfull[buf], (j >> 1) & 1, abort_s, kWaitNs)) {
                fail();
                break;
            }
            sm100::tc_fence_after();
            const hmoe_expert_quant qp = a.quant[td.x];
            const uint32_t col = static_cast<uint32_t>(buf * kTileT);
            for (uint32_t c0 = 32u * grp; c0 < nmma; c0 += 64) {
                uint32_t v[32];
                sm100::tmem_ld32(lane_addr + col + c0, v);
                sm100::tmem_wait_ld();
                const int nt = min(32, rows - static_cast<int>(c0)); // valid tokens in the chunk
                if (GATE_UP) {
                    // rows 0-63: gate of features f, rows 64-127: up of the same
                    // f.  Warps q<2 finish tokens 0..15, warps q>=2 tokens 16..31.
                    // The token rows were scaled by powers of two; xs undoes it.
                    const float sg = qp.scale[0], su = qp.scale[1];
                    const float isl = lane < nt ? a.xscale[row0 + c0 + lane] : 0.0f;
                    if (q < 2) {
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            xg[i * 64 + m] = sg * (__uint_as_float(v[16 + i]) * __shfl_sync(0xffffffffu, isl, 16 + i));
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            xu[i * 64 + (m - 64)] = su * (__uint_as_float(v[i]) * __shfl_sync(0xffffffffu, isl, i));
                    }
                    epi_barrier(grp);
                    // SwiGLU of feature f0 + f for 16 tokens per thread,
                    // stored straight to the row (lanes: consecutive f)
                    const int f = m & 63;
                    const int f0 = nb * 128 + 64 * static_cast<int>(rank);
                    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out) + f0 + f;
                    const bool fin = f0 + f < a.N;
                    if (q < 2) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const float gv = sg * (__uint_as_float(v[i]) * __shfl_sync(0xffffffffu, isl, i));
                            const float uv = xu[i * 64 + f];
                            if (i < nt && fin)
                                out[static_cast<size_t>(row0 + c0 + i) * a.N] = __float2bfloat16_rn(silu_fast(gv) * uv);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const float gv = xg[i * 64 + f];
                            const float uv = su * (__uint_as_float(v[16 + i]) * __shfl_sync(0xffffffffu, isl, 16 + i));
                            if (16 + i < nt && fin)
                                out[static_cast<size_t>(row0 + c0 + 16 + i) * a.N] =
                                    __float2bfloat16_rn(silu_fast(gv) * uv);
                        }
                    }
                    epi_barrier(grp); // exchange buffers free for the next chunk
                } else {
                    // weighted rows: [32 t][128 f] BF16 staged in the group's
                    // (otherwise unused) exchange buffer, then stored as
                    // 16-byte pieces, coalesced per row
                    const float sd = qp.scale[2];
                    const float wl = lane < nt ? a.perm_weight[row0 + c0 + lane] : 0.0f;
                    __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(xbase);
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float wt = __shfl_sync(0xffffffffu, wl, i);
                        st[i * 128 + m] = __float2bfloat16_rn(wt * (sd * __uint_as_float(v[i])));
                    }
                    epi_barrier(grp);
                    const int f0 = nb * 256 + 128 * static_cast<int>(rank);
                    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
                    const int gt = q * 32 + lane; // thread index inside the group
                    // pushed rows: none after an abort (no store into a peer)
                    const bool store = !a.push.peer || *reinterpret_cast<const volatile uint32_t*>(a.push.abort) == 0;
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const int idx = gt + 128 * p; // 512 pieces of 8 BF16
                        const int t = idx >> 4, c = idx & 15;
                        if (store && t < nt && f0 + c * 8 < a.N)
                            *reinterpret_cast<uint4*>(pushed_row(a.push, out, td.w, row0 + c0 + t, a.N) + f0 + c * 8) =
                                *reinterpret_cast<const uint4*>(st + t * 128 + c * 8);
                    }
                    epi_barrier(grp);
                }
            }
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive_remote(sm100::map_shared(sm100::smem_u32(&accempty[buf]), 0));
        }
        if (a.push.peer) __threadfence_system(); // pushed rows visible to their sources before the return flag
    }
    // teardown: every thread of both CTAs arrives here, also after an abort
    if (warp == 2) {
        sm100::mbar_wait_for(drain, 0, kWaitNs); // every pair MMA has completed
    }
    sm100::tc_fence_before();
    sm100::cluster_sync_all();
    if (warp == 2) {
        sm100::tc_fence_after();
        sm100::tmem_dealloc_pair(tmem, kTmemCols);
    }
}

// Cuts every segment (a run of consecutive permuted rows of one expert)
// into ceil(rows / kTileRows) tiles of near-equal size (the first rows %
// tiles of them one row longer), so no expert leaves a sliver tile that
// runs at the MMA issue floor.  Segments are ordered by their longest tile,
// largest first (ties by segment order), all tiles of a segment together,
// so the persistent CTAs start with the longest work items.  One CTA, one
// thread per segment.
// The tile list by one CTA of NT threads (kMaxSegments / NT segments per
// thread, blocked): each segment of r rows is cut into ceil(r / kTileRows)
// near-equal tiles (expert, first row, rows, segment group), and the tiles
// are ordered longest first (ties by segment index).
template <int NT>
__device__ void build_tile_list(const SegSpec& sp, int4* tiles, int32_t* tile_count, int capacity) {
    constexpr int IPT = kMaxSegments / NT;
    using Scan = cub::BlockScan<int, NT>;
    __shared__ typename Scan::TempStorage scan_s;
    __shared__ int2 kn_s[kMaxSegments]; // (longest tile, tiles) of each segment
    __shared__ int total_s;
    const int tid = threadIdx.x;
    int r0[IPT], cnt[IPT];
#pragma unroll
    for (int q = 0; q < IPT; ++q) {
        const int i = tid * IPT + q;
        r0[q] = 0;
        cnt[q] = 0;
        if (i < sp.nseg) {
            if (sp.offsets) {
                r0[q] = sp.offsets[i];
                cnt[q] = sp.offsets[i + 1] - r0[q];
            } else {
                cnt[q] = sp.counts[(i / sp.eps) * sp.count_stride + i % sp.eps];
            }
        }
    }
    if (!sp.offsets) {
        Scan(scan_s).ExclusiveSum(cnt, r0);
#pragma unroll
        for (int q = 0; q < IPT; ++q) r0[q] += sp.row_base;
        __syncthreads();
    }
    int ntile[IPT], base[IPT], extra[IPT], key[IPT];
#pragma unroll
    for (int q = 0; q < IPT; ++q) {
        ntile[q] = cnt[q] > 0 ? (cnt[q] + kTileRows - 1) / kTileRows : 0;
        base[q] = ntile[q] > 0 ? cnt[q] / ntile[q] : 0;
        extra[q] = ntile[q] > 0 ? cnt[q] % ntile[q] : 0;
        key[q] = ntile[q] > 0 ? base[q] + (extra[q] > 0) : 0; // longest tile of the segment
        kn_s[tid * IPT + q] = make_int2(key[q], ntile[q]);
    }
    int excl[IPT], total = 0;
    Scan(scan_s).ExclusiveSum(ntile, excl, total);
    if (tid == 0) total_s = total;
    __syncthreads();
    if (tid == 0) *tile_count = min(capacity, total_s);
    const int nseg = sp.nseg;
#pragma unroll
    for (int q = 0; q < IPT; ++q) {
        const int i = tid * IPT + q;
        if (i >= nseg || ntile[q] == 0) continue;
        const int group = i / sp.eps;
        // tiles of segments ordered before this one: longer tiles, or equal
        // tiles and a lower segment index (independent partial sums so that
        // the shared-memory loads pipeline)
        int pos4[4] = {0, 0, 0, 0};
#pragma unroll 4
        for (int j = 0; j < nseg; ++j) {
            const int2 kj = kn_s[j];
            pos4[j & 3] += (kj.x > key[q] || (kj.x == key[q] && j < i)) ? kj.y : 0;
        }
        const int pos = pos4[0] + pos4[1] + pos4[2] + pos4[3];
        const int e = sp.expert_base + i % sp.eps;
        int row = r0[q];
        for (int f = 0; f < ntile[q]; ++f) {
            const int rows = base[q] + (f < extra[q]);
            if (pos + f < capacity) tiles[pos + f] = make_int4(e, row, rows, group);
            row += rows;
        }
    }
}

__global__ void __launch_bounds__(kMaxSegments) tile_list_kernel(SegSpec sp, int4* tiles, int32_t* tile_count,
                                                                 int capacity) {
    build_tile_list<kMaxSegments>(sp, tiles, tile_count, capacity);
}

// Token-major permutation (permute_token) into this GPU's rows.
struct LocalRows {
    __half* xrows;
    float* xscale;
    int H;
    __device__ RowDst operator()(int r) const {
        return RowDst{xrows + static_cast<size_t>(r) * H, xscale + r, nullptr, 0.0f};
    }
};

// One CTA per token; with a segment spec, CTA 0 (scheduled first, so it
// overlaps the permutation) builds the tile list, which needs only the
// group offsets, saving its own launch.
__global__ void __launch_bounds__(256) permute_kernel(const float* __restrict__ x, const int32_t* __restrict__ inv,
                                                      int first_token_block, int slots, int H,
                                                      __half* __restrict__ xrows, float* __restrict__ xscale,
                                                      SegSpec seg, int4* tiles, int32_t* tile_count, int capacity) {
    if (static_cast<int>(blockIdx.x) < first_token_block) {
        build_tile_list<256>(seg, tiles, tile_count, capacity);
        return;
    }
    permute_token(x, inv, slots, H, blockIdx.x - first_token_block, LocalRows{xrows, xscale, H});
}

// The grouping of a batch of at most kGroupBlock tokens, the permutation and
// the tile list in one launch.  Every CTA scans the group sizes into the
// group offsets (routed experts in id order, then the shared experts).
// CTA 0 stores the offsets and builds the tile list from them.  CTA 1 + t
// places token t's rows where group_kernel's stable counting sort puts them
// -- the group offset plus the number of earlier tokens routed to that
// expert (CpuRouterBackend.cpp:78-90 appends tokens in order) -- writes the
// permutation and the inverse map, and permutes the token.
__global__ void __launch_bounds__(256) group_permute_kernel(const float* __restrict__ x, int H,
                                                            __half* __restrict__ xrows, float* __restrict__ xscale,
                                                            SmallGroup g, SegSpec seg, int4* tiles,
                                                            int32_t* tile_count, int capacity) {
    using Scan = cub::BlockScan<int, 256>;
    __shared__ typename Scan::TempStorage scan_s;
    __shared__ int off_s[2 * 256 + 1];
    __shared__ int e_s[kMaxSlots], cnt_s[kMaxSlots];
    const int tid = threadIdx.x, nb = g.E + g.S, k = g.k;
    int v[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int b = 2 * tid + q;
        v[q] = b < nb ? (b < g.E ? g.counts[b] : g.T) : 0;
    }
    int total = 0;
    Scan(scan_s).ExclusiveSum(v, v, total);
#pragma unroll
    for (int q = 0; q < 2; ++q)
        if (2 * tid + q < nb) off_s[2 * tid + q] = v[q];
    if (tid == 0) off_s[nb] = total;
    __syncthreads();
    if (blockIdx.x == 0) {
        for (int b = tid; b <= nb; b += blockDim.x) g.offsets[b] = off_s[b];
        __syncthreads(); // the tile list reads the offsets back
        build_tile_list<256>(seg, tiles, tile_count, capacity);
        return;
    }
    const int t = static_cast<int>(blockIdx.x) - 1, slots = k + g.S;
    if (tid < k) {
        e_s[tid] = static_cast<int>(g.ids[static_cast<size_t>(t) * k + tid]);
        cnt_s[tid] = 0;
    }
    __syncthreads();
    // earlier tokens routed to each of this token's experts (a token's k
    // experts are distinct, so each earlier token counts once per expert)
    for (int tp = tid; tp < t; tp += blockDim.x) {
        const uint32_t* r = g.ids + static_cast<size_t>(tp) * k;
        for (int jj = 0; jj < k; ++jj) {
            const int ep = static_cast<int>(r[jj]);
            for (int j = 0; j < k; ++j)
                if (ep == e_s[j]) atomicAdd(&cnt_s[j], 1);
        }
    }
    __syncthreads();
    if (tid < slots) {
        const int row = tid < k ? off_s[e_s[tid]] + cnt_s[tid] : off_s[g.E + (tid - k)] + t;
        g.perm_token[row] = static_cast<uint32_t>(t);
        g.perm_weight[row] = tid < k ? g.scores[static_cast<size_t>(t) * k + tid] : 1.0f;
        g.inv[static_cast<size_t>(t) * slots + tid] = row;
    }
    __syncthreads(); // permute_token reads the inverse map back
    permute_token(x, g.inv, slots, H, t, LocalRows{xrows, xscale, H});
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

// INT8 weights of one projection across all experts: dims {N, K, experts},
// box [64 k][64 n].
bool map_weights(CUtensorMap* m, const int8_t* base, int N, int K, int experts, uint64_t stride) {
    return map_weights_box(m, base, N, K, experts, stride, 64, kBK);
}

// 16-bit rows [rows, K] (K contiguous), 128-byte swizzle, box 64 x box_rows.
bool map_rows(CUtensorMap* m, const void* base, int K, int rows, bool f16, int box_rows) {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)}; // 128 bytes: the swizzle span
    const cuuint32_t es[2] = {1, 1};
    return encode_fn()(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                       const_cast<void*>(base), dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() { return current_sm_count(); }

template <bool GATE_UP, int HT>
hmoe_status launch_gemm(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& b, const GemmArgs& args,
                        int item_capacity, cudaStream_t s) {
    constexpr int kSmem = GemmCfg<HT>::kSmem;
    const cudaError_t aerr = set_smem_limit(reinterpret_cast<const void*>(expert_gemm_kernel<GATE_UP, HT>), kSmem);
    if (aerr != cudaSuccess) {
        set_last_error("hmoe expert GEMM shared-memory limit", aerr);
        return HMOE_CUDA_ERROR;
    }
    const int pairs = std::max(1, std::min(sm_count() / 2, item_capacity));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    cfg.blockDim = dim3(kThreadsGemm);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = 2;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, expert_gemm_kernel<GATE_UP, HT>, w0, w1, b, args);
    if (err != cudaSuccess) {
        set_last_error(GATE_UP ? "hmoe expert GEMM gate/up launch" : "hmoe expert GEMM down launch", err);
        return HMOE_CUDA_ERROR;
    }
    return check_launch(GATE_UP ? "hmoe expert GEMM gate/up" : "hmoe expert GEMM down");
}

} // namespace

// FP32 row-major matrix [rows][cols] (cols contiguous, cols % 4 == 0), box
// [box_rows][box_cols] with box_cols * 4 == 128 bytes, 128-byte swizzle;
// elements outside the matrix read as zero.
bool map_f32_rows_sw128(CUtensorMap* m, const float* base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                        uint32_t box_rows) {
    if (!encode_fn()) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// INT8 weights of one projection across all experts, dims {N, K, experts}
// (the packed [in,out] layout, N contiguous), box [box_k][box_n], no swizzle.
bool map_weights_box(CUtensorMap* m, const int8_t* base, int N, int K, int experts, uint64_t stride, int box_n,
                     int box_k) {
    if (!encode_fn()) return false;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(K),
                                static_cast<cuuint64_t>(experts)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(N), stride};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(box_n), static_cast<cuuint32_t>(box_k), 1};
    const cuuint32_t es[3] = {1, 1, 1};
    return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(base), dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int device_sm_count() { return sm_count(); }

// Per device ordinal (a process may drive devices of different kinds):
// 0 unknown, 1 no, 2 yes.  Racing first calls compute the same answer.
bool gemm_available() {
    static std::atomic<int> avail[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return false;
    }
    int v = avail[dev].load();
    if (v == 0) {
        int major = 0, minor = 0;
        const bool ok = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess &&
                        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) == cudaSuccess &&
                        major == 10 && minor == 0 && encode_fn() != nullptr;
        cudaGetLastError();
        v = ok ? 2 : 1;
        avail[dev].store(v);
    }
    return v == 2;
}

hmoe_status launch_tile_list(const SegSpec& spec, int4* tiles, int32_t* tile_count, int capacity,
                             cudaStream_t s) {
    if (spec.nseg <= 0 || spec.nseg > kMaxSegments || spec.eps <= 0 || capacity <= 0)
        return HMOE_INVALID_ARGUMENT;
    tile_list_kernel<<<1, kMaxSegments, 0, s>>>(spec, tiles, tile_count, capacity);
    return check_launch("hmoe tile list");
}

hmoe_status launch_permute(const float* x, const int32_t* inv, int tokens, int slots, int H, __half* xrows,
                           float* xscale, cudaStream_t s, const SegSpec* seg, int4* tiles, int32_t* tile_count,
                           int capacity) {
    if (tokens <= 0) return HMOE_OK;
    const bool with_tiles = seg != nullptr;
    if (with_tiles && (seg->nseg <= 0 || seg->nseg > kMaxSegments || seg->eps <= 0 || capacity <= 0))
        return HMOE_INVALID_ARGUMENT;
    const int first = with_tiles ? 1 : 0;
    permute_kernel<<<static_cast<unsigned>(tokens + first), 256, 0, s>>>(
        x, inv, first, slots, H, xrows, xscale, with_tiles ? *seg : SegSpec{}, tiles, tile_count, capacity);
    return check_launch("hmoe permute");
}

hmoe_status launch_group_permute(const SmallGroup& g, const float* x, int H, __half* xrows, float* xscale,
                                 const SegSpec& seg, int4* tiles, int32_t* tile_count, int capacity,
                                 cudaStream_t s) {
    if (g.T <= 0) return HMOE_OK;
    if (g.T > kGroupBlock || g.E + g.S > 2 * 256 || g.k + g.S > kMaxSlots || seg.nseg <= 0 ||
        seg.nseg > kMaxSegments || seg.eps <= 0 || capacity <= 0)
        return HMOE_INVALID_ARGUMENT;
    group_permute_kernel<<<static_cast<unsigned>(g.T + 1), 256, 0, s>>>(x, H, xrows, xscale, g, seg, tiles,
                                                                         tile_count, capacity);
    return check_launch("hmoe group and permute");
}

// Full tiles are at most rows / kTileRows; each segment with rows adds at
// most one partial tile, and at most `rows` segments have rows.
int tile_capacity_for(long rows, int segments) {
    return static_cast<int>(rows / kTileRows + std::min<long>(segments, rows) + 1);
}

extern int g_variant; // layer.cu: 4 forces the wide-tile kernel

// Every tile of the run fits the narrow kernel: no expert holds more than
// kNarrowRows rows.
bool narrow_run(const ExpertRun& r) { return g_variant != 4 && r.max_group >= 0 && r.max_group <= kNarrowRows; }

hmoe_status gemm_gate_up(const ExpertRun& r, cudaStream_t s) {
    const bool narrow = narrow_run(r);
    CUtensorMap mg, mu, mb;
    if (!map_weights(&mg, r.arena + r.gate_offset, r.I, r.H, r.experts, r.stride) ||
        !map_weights(&mu, r.arena + r.up_offset, r.I, r.H, r.experts, r.stride) ||
        !map_rows(&mb, r.xrows, r.H, r.rows_cap, true, narrow ? 32 : 128)) {
        set_last_error_text("hmoe: cuTensorMapEncodeTiled failed (gate/up)");
        return HMOE_CUDA_ERROR;
    }
    const int nb = (r.I + 127) / 128; // 128 features (64 per CTA) per pair
    GemmArgs a{r.tiles, r.tile_count, nb, r.quant, nullptr, r.xscale, r.hmid16, r.H, r.I, r.st, PushRows{}};
    return narrow ? launch_gemm<true, 32>(mg, mu, mb, a, r.tile_cap * nb, s)
                  : launch_gemm<true, 128>(mg, mu, mb, a, r.tile_cap * nb, s);
}

hmoe_status gemm_down(const ExpertRun& r, cudaStream_t s) {
    const bool narrow = narrow_run(r);
    CUtensorMap md, mb;
    if (!map_weights(&md, r.arena + r.down_offset, r.H, r.I, r.experts, r.stride) ||
        !map_rows(&mb, r.hmid16, r.I, r.rows_cap, false, narrow ? 32 : 128)) {
        set_last_error_text("hmoe: cuTensorMapEncodeTiled failed (down)");
        return HMOE_CUDA_ERROR;
    }
    const int nb = (r.H + 255) / 256; // 256 features (128 per CTA) per pair
    GemmArgs a{r.tiles, r.tile_count, nb, r.quant, r.weight, nullptr, r.yrows, r.I, r.H, r.st, r.push};
    return narrow ? launch_gemm<false, 32>(md, md, mb, a, r.tile_cap * nb, s)
                  : launch_gemm<false, 128>(md, md, mb, a, r.tile_cap * nb, s);
}

} // namespace hmoe
