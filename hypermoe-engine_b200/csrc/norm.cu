// norm.cu -- hmoe_rms_norm: RMSNorm of token rows, the normalisation a
// transformer block applies to the residual stream before its MoE layer
// (TransformerBlock::execute, src/transformer/runtime/TransformerBlock.cpp:90-92).
// Stacks of MoE blocks need it: without it the SwiGLU output grows with the
// square of its input and the residual stream overflows after a few layers.
//
// Arithmetic of the reference's CPU RMSNorm (src/transformer/norm/RMSNorm.cpp:64-77):
// each square of a float is exact in double and summed in double (here as a
// tree over the CTA, where the reference adds sequentially: the two sums
// differ by a few double roundings), inverse RMS = 1/sqrt(sum/H + eps) in
// double, and out = float(double(x) * inv * double(w)) with one rounding.
//
// One CTA of 256 threads per token.  HBM-bound: 4H bytes read and 4H
// written per token (the second read of the row hits L1/L2).
#include "common.cuh"

#include <climits>
#include <cmath>

namespace hmoe {
namespace {

constexpr int kNormThreads = 256;

// x and out may alias (in place): each thread reads the elements it writes
// before writing them, and every read of the first pass precedes the CTA
// barrier of the reduction.
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const float* x, const float* __restrict__ w,
                                                                float* out, int H, float eps, int vec) {
    __shared__ double red_s[kNormThreads / 32];
    __shared__ double inv_s;
    const size_t base = static_cast<size_t>(blockIdx.x) * static_cast<size_t>(H);
    const float* row = x + base;
    float* orow = out + base;
    double ss = 0.0;
    if (vec) {
        const float4* r4 = reinterpret_cast<const float4*>(row);
        for (int c = threadIdx.x; c < H / 4; c += kNormThreads) {
            const float4 v = r4[c];
            ss += static_cast<double>(v.x) * v.x;
            ss += static_cast<double>(v.y) * v.y;
            ss += static_cast<double>(v.z) * v.z;
            ss += static_cast<double>(v.w) * v.w;
        }
    } else {
        for (int i = threadIdx.x; i < H; i += kNormThreads) {
            const double v = row[i];
            ss += v * v;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red_s[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double total = 0.0;
        for (int i = 0; i < kNormThreads / 32; ++i) total += red_s[i];
        inv_s = 1.0 / sqrt(total / static_cast<double>(H) + static_cast<double>(eps));
    }
    __syncthreads();
    const double inv = inv_s;
    if (vec) {
        const float4* r4 = reinterpret_cast<const float4*>(row);
        const float4* w4 = reinterpret_cast<const float4*>(w);
        float4* o4 = reinterpret_cast<float4*>(orow);
        for (int c = threadIdx.x; c < H / 4; c += kNormThreads) {
            const float4 v = r4[c], g = w4[c];
            o4[c] = make_float4(static_cast<float>(static_cast<double>(v.x) * inv * static_cast<double>(g.x)),
                                static_cast<float>(static_cast<double>(v.y) * inv * static_cast<double>(g.y)),
                                static_cast<float>(static_cast<double>(v.z) * inv * static_cast<double>(g.z)),
                                static_cast<float>(static_cast<double>(v.w) * inv * static_cast<double>(g.w)));
        }
    } else {
        for (int i = threadIdx.x; i < H; i += kNormThreads)
            orow[i] = static_cast<float>(static_cast<double>(row[i]) * inv * static_cast<double>(w[i]));
    }
}

} // namespace
} // namespace hmoe

extern "C" {

hmoe_status hmoe_rms_norm(const float* input, const float* weight, float* output, size_t tokens, size_t hidden,
                          float epsilon, void* stream) {
    using namespace hmoe;
    // RMSNorm's constructor and execute checks (RMSNorm.cpp:17-22,41-52)
    if (hidden == 0 || !(epsilon > 0.0f) || !std::isfinite(epsilon)) return HMOE_INVALID_ARGUMENT;
    if (tokens == 0) return HMOE_OK;
    if (!input || !weight || !output) return HMOE_INVALID_ARGUMENT;
    if (hidden > static_cast<size_t>(INT_MAX) || tokens > static_cast<size_t>(INT_MAX)) return HMOE_UNSUPPORTED;
    const bool vec = hidden % 4 == 0 && reinterpret_cast<uintptr_t>(input) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(weight) % 16 == 0 && reinterpret_cast<uintptr_t>(output) % 16 == 0;
    rms_norm_kernel<<<static_cast<unsigned>(tokens), kNormThreads, 0, as_stream(stream)>>>(
        input, weight, output, static_cast<int>(hidden), epsilon, vec ? 1 : 0);
    return check_launch("hmoe rms norm kernel");
}

} // extern "C"
