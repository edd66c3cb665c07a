// rows.cuh -- the per-token bodies of the permutation and of the combine,
// shared by the single-GPU kernels (rows in this GPU's workspace) and the
// expert-parallel ones (routed rows in the expert owners' workspaces,
// reached by peer-memory stores and loads).  A row locator maps a permuted
// row index to where that row lives.
#pragma once

#include "layer.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <climits>

namespace hmoe {

// Destination of one permuted row: its FP16 elements, its 1/scale and (for
// rows that carry it along) its routing weight.
struct RowDst {
    __half* row;
    float* scale;
    float* weight; // null: the weight stays in perm_weight
    float wval;
};

// Token t of the permutation: its FP32 row is read once, scaled by the power
// of two s_t that puts its largest magnitude in [2^14, 2^15), converted to
// FP16 (11-bit significand, no overflow) and written to each of its rows
// inv[t, 0..slots) at loc(row); 1/s_t goes with every row.  One CTA.
template <class Loc>
__device__ __forceinline__ void permute_token(const float* __restrict__ x, const int32_t* __restrict__ inv, int slots,
                                              int H, int t, const Loc& loc) {
    __shared__ RowDst dst_s[kMaxSlots];
    __shared__ float red_s[8];
    for (int s = threadIdx.x; s < slots; s += blockDim.x) dst_s[s] = loc(inv[static_cast<size_t>(t) * slots + s]);
    const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * H);
    float mx = 0.0f;
    for (int c = threadIdx.x; c < H / 4; c += blockDim.x) {
        const float4 v = src[c];
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red_s[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red_s[0];
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) mx = fmaxf(mx, red_s[w]);
    int ex = 0;
    if (mx > 0.0f && isfinite(mx)) frexpf(mx, &ex); // mx = m * 2^ex, m in [0.5, 1)
    const int sh = (mx > 0.0f && isfinite(mx)) ? max(-126, min(126, 15 - ex)) : 0;
    const float sc = ldexpf(1.0f, sh), isc = ldexpf(1.0f, -sh);
    for (int s = threadIdx.x; s < slots; s += blockDim.x) {
        *dst_s[s].scale = isc;
        if (dst_s[s].weight) *dst_s[s].weight = dst_s[s].wval;
    }
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
        const float4 v0 = src[2 * c], v1 = src[2 * c + 1];
        const __half2 h0 = __floats2half2_rn(v0.x * sc, v0.y * sc), h1 = __floats2half2_rn(v0.z * sc, v0.w * sc);
        const __half2 h2 = __floats2half2_rn(v1.x * sc, v1.y * sc), h3 = __floats2half2_rn(v1.z * sc, v1.w * sc);
        const uint4 o = make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                                   *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
        for (int s = 0; s < slots; ++s) reinterpret_cast<uint4*>(dst_s[s].row)[c] = o;
    }
}

// Token t of the combine: its rows (routed slots, then shared) ordered
// ascending by expert id (routing ids when given, else row order, which is
// expert order without a placement) and accumulated in that order from zero,
// as the reference's combine loop does (MoERuntime.cpp:311-325).  src(row)
// gives the BF16 row.  With `residual`, the finished sum is added to
// residual[t] with one FP32 rounding, as the reference's layer adds the MoE
// output to its residual (MoELayer.cpp:37-39); residual may be `out`
// itself.  With `out16`, the result is also written as BF16 (round to
// nearest even).  One CTA.
template <class Src>
__device__ __forceinline__ void combine_token(const int32_t* __restrict__ inv, const uint32_t* __restrict__ ids,
                                              int k, int E, int slots, int H, int t, float* out,
                                              const Src& src, const float* residual = nullptr,
                                              __nv_bfloat16* __restrict__ out16 = nullptr) {
    __shared__ const __nv_bfloat16* rows_s[kMaxSlots];
    __shared__ int keys_s[kMaxSlots];
    if (threadIdx.x < 32) { // warp 0: every slot's key at once, then its rank among the keys
        const int lane = threadIdx.x;
        int key[3], row[3];
#pragma unroll
        for (int q = 0; q < 3; ++q) {
            const int s = lane + 32 * q;
            key[q] = INT_MAX;
            row[q] = 0;
            if (s < slots) {
                row[q] = inv[static_cast<size_t>(t) * slots + s];
                key[q] = ids ? (s < k ? static_cast<int>(ids[static_cast<size_t>(t) * k + s]) : E + (s - k)) : row[q];
                keys_s[s] = key[q];
            }
        }
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 3; ++q) {
            const int s = lane + 32 * q;
            if (s < slots) {
                int rank = 0; // keys are distinct: a token's rows, or its experts
                for (int j = 0; j < slots; ++j) rank += keys_s[j] < key[q];
                rows_s[rank] = src(row[q]);
            }
        }
    }
    __syncthreads();
    const int H8 = H / 8;
    constexpr int kBatch = 8; // rows whose loads are in flight together
    for (int c = threadIdx.x; c < H8; c += blockDim.x) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int s0 = 0; s0 < slots; s0 += kBatch) {
            uint4 v[kBatch];
#pragma unroll
            for (int b = 0; b < kBatch; ++b)
                if (s0 + b < slots) v[b] = reinterpret_cast<const uint4*>(rows_s[s0 + b])[c];
#pragma unroll
            for (int b = 0; b < kBatch; ++b) { // still added in row order
                if (s0 + b >= slots) break;
                const uint32_t w[4] = {v[b].x, v[b].y, v[b].z, v[b].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    acc[2 * i] = __fadd_rn(acc[2 * i], __uint_as_float(w[i] << 16));
                    acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __uint_as_float(w[i] & 0xffff0000u));
                }
            }
        }
        if (residual) {
            const float4* rs = reinterpret_cast<const float4*>(residual + static_cast<size_t>(t) * H) + 2 * c;
            const float4 r0 = rs[0], r1 = rs[1];
            const float r[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(r[i], acc[i]);
        }
        float4* o = reinterpret_cast<float4*>(out + static_cast<size_t>(t) * H) + 2 * c;
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
        if (out16) {
            uint32_t b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const __nv_bfloat162 v = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
                b[i] = *reinterpret_cast<const uint32_t*>(&v);
            }
            reinterpret_cast<uint4*>(out16 + static_cast<size_t>(t) * H)[c] = make_uint4(b[0], b[1], b[2], b[3]);
        }
    }
}

} // namespace hmoe
