// synth.cpp -- seeded synthetic inputs and the INT8 expert packer.
//
// The benchmark configurations have no public dataset; inputs are seeded
// synthetic tensors with the shapes and distributions the configurations
// name (activations ~N(0,1), router and expert weights ~N(0, 0.02^2),
// Zipf(1.1)-skewed routing).  Everything is generated on the host by a
// counter-based generator so that any element can be produced
// independently (threads split the work without changing the values).
//
// hmoe_quantize_int8 restates quantizeInt8
// (src/tensor/quantization/Quantization.cpp:45-79) and hmoe_synth_arena
// lays experts out as ExpertPacker does (tools/model_convert/
// ExpertPacker.cpp:150-247: per expert gate|up|down, [in,out] row-major).

#include "hmoe.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

constexpr std::uint64_t kGolden = 0x9E3779B97F4A7C15ULL;

inline std::uint64_t mix64(std::uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

// SplitMix64 keyed by (seed, stream); value n of the sequence.
inline std::uint64_t draw(std::uint64_t key, std::uint64_t n) {
    return mix64(key + (n + 1) * kGolden);
}

inline std::uint64_t streamKey(std::uint64_t seed, std::uint64_t stream) {
    return seed ^ mix64(stream ^ 0xD1B54A32D192ED03ULL);
}

// Pair j of normals (Box-Muller on two 53-bit uniforms, all in double).
inline void normalPair(std::uint64_t key, std::uint64_t j, double& a, double& b) {
    const double u1 = static_cast<double>((draw(key, 2 * j) >> 11) + 1) * 0x1.0p-53;
    const double u2 = static_cast<double>(draw(key, 2 * j + 1) >> 11) * 0x1.0p-53;
    const double r = std::sqrt(-2.0 * std::log(u1));
    const double t = 6.283185307179586476925286766559 * u2;
    a = r * std::cos(t);
    b = r * std::sin(t);
}

void fillNormal(std::uint64_t key, float sigma, float* out, std::size_t begin,
                std::size_t end) {
    for (std::size_t i = begin; i < end;) {
        double a, b;
        normalPair(key, i / 2, a, b);
        if ((i & 1) == 0) {
            out[i] = static_cast<float>(a * sigma);
            if (i + 1 < end) out[i + 1] = static_cast<float>(b * sigma);
            i += 2;
        } else {
            out[i] = static_cast<float>(b * sigma);
            i += 1;
        }
    }
}

template <class F>
void parallelFor(std::size_t n, int threads, F&& body) {
    const int t = std::max(1, std::min<int>(threads, static_cast<int>(std::max<std::size_t>(n, 1))));
    if (t == 1) {
        for (std::size_t i = 0; i < n; ++i) body(i);
        return;
    }
    std::vector<std::thread> pool;
    for (int w = 0; w < t; ++w) {
        pool.emplace_back([&, w]() {
            for (std::size_t i = static_cast<std::size_t>(w); i < n; i += static_cast<std::size_t>(t)) body(i);
        });
    }
    for (auto& th : pool) th.join();
}

} // namespace

extern "C" {

void hmoe_synth_normal(std::uint64_t seed, std::uint64_t stream, float sigma,
                       float* out, std::size_t n, int threads) {
    const auto key = streamKey(seed, stream);
    constexpr std::size_t kChunk = 1 << 16; // even, so pairs never straddle
    const std::size_t chunks = (n + kChunk - 1) / kChunk;
    parallelFor(chunks, threads, [&](std::size_t c) {
        fillNormal(key, sigma, out, c * kChunk, std::min(n, (c + 1) * kChunk));
    });
}

void hmoe_synth_zipf_bias(std::uint64_t seed, float alpha, float* bias,
                          std::size_t E) {
    std::vector<std::uint32_t> perm(E);
    for (std::size_t e = 0; e < E; ++e) perm[e] = static_cast<std::uint32_t>(e);
    const auto key = streamKey(seed, 3);
    for (std::size_t i = E; i > 1; --i) { // Fisher-Yates
        const auto j = draw(key, i) % i;
        std::swap(perm[i - 1], perm[j]);
    }
    for (std::size_t e = 0; e < E; ++e)
        bias[e] = static_cast<float>(-static_cast<double>(alpha) * std::log(static_cast<double>(perm[e]) + 1.0));
}

hmoe_status hmoe_quantize_int8(const float* w, std::size_t n, std::int8_t* q,
                               float* scale, std::int32_t* zero_point,
                               float* max_abs_error) {
    if (n == 0 || !w || !q || !scale || !zero_point) return HMOE_INVALID_ARGUMENT;
    float m = 0.0F;
    for (std::size_t i = 0; i < n; ++i) {
        if (!std::isfinite(w[i])) return HMOE_INVALID_ARGUMENT;
        m = std::max(m, std::fabs(w[i]));
    }
    const float s = m == 0.0F ? 1.0F : m / 127.0F;
    float err = 0.0F;
    for (std::size_t i = 0; i < n; ++i) {
        const float r = std::clamp(std::round(w[i] / s), -127.0F, 127.0F);
        const auto v = static_cast<std::int8_t>(r);
        q[i] = v;
        err = std::max(err, std::fabs(w[i] - static_cast<float>(static_cast<std::int32_t>(v)) * s));
    }
    *scale = s;
    *zero_point = 0;
    if (max_abs_error) *max_abs_error = err;
    return HMOE_OK;
}

void hmoe_synth_arena(std::uint64_t seed, std::uint32_t layer, std::uint32_t first,
                      std::uint32_t count, std::uint32_t H, std::uint32_t I,
                      float sigma, std::int8_t* arena, std::uint64_t expert_stride,
                      std::uint64_t gate_offset, std::uint64_t up_offset,
                      std::uint64_t down_offset, hmoe_expert_quant* quant,
                      int threads) {
    const std::size_t n = static_cast<std::size_t>(H) * I;
    const std::uint64_t offs[3] = {gate_offset, up_offset, down_offset};
    parallelFor(static_cast<std::size_t>(count) * 3, threads, [&](std::size_t job) {
        const auto local = static_cast<std::uint32_t>(job / 3);
        const auto p = static_cast<std::uint32_t>(job % 3);
        const std::uint64_t e = first + local;
        const std::uint64_t stream = 0x1000ULL + (static_cast<std::uint64_t>(layer) << 24) + e * 4 + p;
        std::vector<float> w(n);
        fillNormal(streamKey(seed, stream), sigma, w.data(), 0, n);
        float s = 1.0F;
        std::int32_t z = 0;
        hmoe_quantize_int8(w.data(), n, arena + local * expert_stride + offs[p], &s, &z, nullptr);
        quant[local].scale[p] = s;
        quant[local].zero_point[p] = z;
    });
}

} // extern "C"
