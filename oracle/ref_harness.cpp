// ref_harness.cpp -- C entry points over the UNMODIFIED HyperMoE CPU path.
//
// TEST INFRASTRUCTURE ONLY (the checker, never the product).  oracle/Makefile
// compiles this file together with the reference's own sources, read in place
// from the reference tree, into oracle/_ref/libhmoe_ref.so.  Nothing here
// re-implements arithmetic: every number comes from the reference classes
//   router::CpuRouterBackend::routeBatch   src/router/CpuRouterBackend.cpp:125-160
//   tensor::CpuTensorBackend::matmulInt8Weights
//                                          src/tensor/backend/CpuTensorBackend.cpp:133-190
//   ExpertMlpExecutor::execute             src/experts/ExpertExecutor.cpp:43-138
//   tensor::quantization::quantizeInt8     src/tensor/quantization/Quantization.cpp:45-79
// and the layer loop restates the CPU branch of MoERuntime::executeBatch
// (src/core/runtime/MoERuntime.cpp:182-325: gather by memcpy, expert MLP,
// combine `out[tok] += w * y` in ascending expert order).  The scheduler,
// residency and storage layers that MoERuntime also drives are out of scope
// (all experts resident), so they are not linked.
//
// Used by tests/golden/make_golden.py (fixtures), by tests that cross-check
// oracle/hmoe_oracle.c, and by bench.py's reference arm (timed on the host).

#include "experts/ExpertExecutor.hpp"
#include "router/CpuRouterBackend.hpp"
#include "router/RouterConfig.hpp"
#include "tensor/backend/CpuTensorBackend.hpp"
#include "tensor/quantization/Quantization.hpp"
#include "transformer/norm/RMSNorm.hpp"

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <thread>
#include <vector>

using namespace hypermoe;
using tensor::DType;
using tensor::Shape;

namespace {

constexpr int kOk = 0;
constexpr int kInvalid = 1;
constexpr int kFailed = 2;

tensor::Tensor hostTensor(tensor::CpuTensorBackend& cpu, Shape shape,
                          DType dtype, const void* src, std::size_t bytes) {
    auto t = cpu.allocateTensor(shape, dtype);
    if (src && bytes) std::memcpy(t.data(), src, bytes);
    return t;
}

// Routes through CpuRouterBackend.  A non-null bias is folded in by
// extending each hidden row with a constant 1 and the router matrix with the
// bias row, so the reference's own double accumulation adds it last.
router::BatchRouterDecision route(tensor::CpuTensorBackend& cpu,
                                  const float* hidden, const float* weights,
                                  const float* bias, std::size_t T,
                                  std::size_t H, std::size_t E, std::size_t k,
                                  int softmax, int renorm) {
    const std::size_t Hx = bias ? H + 1 : H;
    auto h = cpu.allocateTensor({T, Hx}, DType::FP32);
    auto w = cpu.allocateTensor({Hx, E}, DType::FP32);
    auto* hp = static_cast<float*>(h.data());
    auto* wp = static_cast<float*>(w.data());
    for (std::size_t t = 0; t < T; ++t) {
        std::memcpy(hp + t * Hx, hidden + t * H, H * sizeof(float));
        if (bias) hp[t * Hx + H] = 1.0F;
    }
    std::memcpy(wp, weights, H * E * sizeof(float));
    if (bias) std::memcpy(wp + H * E, bias, E * sizeof(float));
    const router::RouterConfig config{
        E, k,
        softmax ? router::RoutingNormalization::Softmax
                : router::RoutingNormalization::None,
        renorm != 0};
    router::CpuRouterBackend backend;
    return backend.routeBatch(0, h, w, config);
}

struct Layer {
    std::size_t H, I, E, k, shared;
    int softmax, renorm;
    std::vector<float> routerW, bias;
    bool hasBias;
    tensor::CpuTensorBackend cpu;
    tensor::Tensor arena;
    std::size_t stride, gateOff, upOff, downOff;
    std::vector<float> scale;
    std::vector<std::int32_t> zp;

    ExpertMlpWeights weights(std::size_t e) const {
        tensor::TensorView all(arena);
        const auto base = e * stride;
        using QP = tensor::quantization::QuantizationParameters;
        return {all.sliceBytes(base + gateOff, {H, I}, DType::INT8),
                all.sliceBytes(base + upOff, {H, I}, DType::INT8),
                all.sliceBytes(base + downOff, {I, H}, DType::INT8),
                QP{scale[3 * e + 0], zp[3 * e + 0]},
                QP{scale[3 * e + 1], zp[3 * e + 1]},
                QP{scale[3 * e + 2], zp[3 * e + 2]}};
    }
};

} // namespace

extern "C" {

int hmr_route_batch(const float* hidden, const float* weights,
                    const float* bias, std::size_t T, std::size_t H,
                    std::size_t E, std::size_t k, int softmax, int renorm,
                    std::uint32_t* ids, float* scores, std::int32_t* offsets,
                    std::uint32_t* group_tokens, float* group_scores) {
    try {
        tensor::CpuTensorBackend cpu;
        const auto d = route(cpu, hidden, weights, bias, T, H, E, k, softmax, renorm);
        for (std::size_t t = 0; t < T; ++t) {
            for (std::size_t r = 0; r < k; ++r) {
                ids[t * k + r] = d.tokens[t].selectedExpertIds[r];
                scores[t * k + r] = d.tokens[t].routingScores[r];
            }
        }
        if (offsets) {
            std::fill(offsets, offsets + E + 1, 0);
            std::size_t pos = 0;
            for (const auto& g : d.expertGroups) {
                offsets[g.expertId + 1] = static_cast<std::int32_t>(g.tokenIndices.size());
                for (std::size_t j = 0; j < g.tokenIndices.size(); ++j, ++pos) {
                    if (group_tokens) group_tokens[pos] = static_cast<std::uint32_t>(g.tokenIndices[j]);
                    if (group_scores) group_scores[pos] = g.routingScores[j];
                }
            }
            for (std::size_t e = 0; e < E; ++e) offsets[e + 1] += offsets[e];
        }
        return kOk;
    } catch (const std::invalid_argument&) {
        return kInvalid;
    } catch (const std::exception&) {
        return kFailed;
    }
}

int hmr_int8_matmul(const float* left, const std::int8_t* q, float* out,
                    std::size_t rows, std::size_t K, std::size_t N,
                    float scale, std::int32_t zp) {
    try {
        tensor::CpuTensorBackend cpu;
        auto a = hostTensor(cpu, {rows, K}, DType::FP32, left, rows * K * 4);
        auto b = hostTensor(cpu, {K, N}, DType::INT8, q, K * N);
        auto c = cpu.allocateTensor({rows, N}, DType::FP32);
        cpu.matmulInt8Weights(a, b, {scale, zp}, c);
        std::memcpy(out, c.data(), rows * N * 4);
        return kOk;
    } catch (const std::invalid_argument&) {
        return kInvalid;
    } catch (const std::exception&) {
        return kFailed;
    }
}

int hmr_expert_mlp(const float* x, std::size_t rows, std::size_t H,
                   std::size_t I, const std::int8_t* gate,
                   const std::int8_t* up, const std::int8_t* down,
                   const float* scale, const std::int32_t* zp, float* y) {
    try {
        auto cpu = std::make_shared<tensor::CpuTensorBackend>();
        auto in = hostTensor(*cpu, {rows, H}, DType::FP32, x, rows * H * 4);
        auto g = hostTensor(*cpu, {H, I}, DType::INT8, gate, H * I);
        auto u = hostTensor(*cpu, {H, I}, DType::INT8, up, H * I);
        auto d = hostTensor(*cpu, {I, H}, DType::INT8, down, I * H);
        auto out = cpu->allocateTensor({rows, H}, DType::FP32);
        using QP = tensor::quantization::QuantizationParameters;
        ExpertMlpExecutor(cpu).execute(
            in, {g, u, d, QP{scale[0], zp[0]}, QP{scale[1], zp[1]}, QP{scale[2], zp[2]}},
            out);
        std::memcpy(y, out.data(), rows * H * 4);
        return kOk;
    } catch (const std::invalid_argument&) {
        return kInvalid;
    } catch (const std::exception&) {
        return kFailed;
    }
}

// RMSNorm::execute on the CPU backend (src/transformer/norm/RMSNorm.cpp:35-77).
int hmr_rms_norm(const float* x, const float* w, float* out, std::size_t T, std::size_t H, float eps) {
    try {
        auto cpu = std::make_shared<tensor::CpuTensorBackend>();
        auto in = hostTensor(*cpu, {T, H}, DType::FP32, x, T * H * 4);
        auto g = hostTensor(*cpu, {H}, DType::FP32, w, H * 4);
        transformer::norm::RMSNorm norm(cpu, H, eps);
        auto o = norm.execute(in.view(), g.view());
        std::memcpy(out, o.data(), T * H * 4);
        return kOk;
    } catch (const std::invalid_argument&) {
        return kInvalid;
    } catch (const std::exception&) {
        return kFailed;
    }
}

int hmr_quantize_int8(const float* w, std::size_t n, std::int8_t* q,
                      float* scale, std::int32_t* zp, float* max_err) {
    try {
        const auto r = tensor::quantization::quantizeInt8(std::span<const float>(w, n));
        std::memcpy(q, r.bytes.data(), n);
        *scale = r.parameters.scale;
        *zp = r.parameters.zeroPoint;
        if (max_err) *max_err = r.maximumAbsoluteError;
        return kOk;
    } catch (const std::invalid_argument&) {
        return kInvalid;
    } catch (const std::exception&) {
        return kFailed;
    }
}

// A resident layer: the arena (ExpertPacker layout, uniform expert stride) is
// copied once into a reference Tensor so that hmr_layer_forward times only
// the forward pass, as the reference runs it with every expert resident.
void* hmr_layer_create(std::size_t H, std::size_t I, std::size_t E,
                       std::size_t k, int softmax, int renorm,
                       const float* router_w, const float* router_bias,
                       std::size_t n_shared, const std::int8_t* arena,
                       std::size_t stride, std::size_t gate_off,
                       std::size_t up_off, std::size_t down_off,
                       const float* qscale, const std::int32_t* qzp) {
    try {
        auto* L = new Layer();
        L->H = H; L->I = I; L->E = E; L->k = k; L->shared = n_shared;
        L->softmax = softmax; L->renorm = renorm;
        L->routerW.assign(router_w, router_w + H * E);
        L->hasBias = router_bias != nullptr;
        if (router_bias) L->bias.assign(router_bias, router_bias + E);
        const auto total = E + n_shared;
        L->arena = hostTensor(L->cpu, {total * stride}, DType::INT8, arena, total * stride);
        L->stride = stride; L->gateOff = gate_off; L->upOff = up_off; L->downOff = down_off;
        L->scale.assign(qscale, qscale + 3 * total);
        L->zp.assign(qzp, qzp + 3 * total);
        return L;
    } catch (const std::exception&) {
        return nullptr;
    }
}

void hmr_layer_destroy(void* layer) { delete static_cast<Layer*>(layer); }

// One layer forward.  `threads` > 1 runs different expert groups on
// different host threads (each with its own CpuTensorBackend, which is
// single-threaded by construction); the combine then runs in ascending
// expert order exactly as the single-threaded loop does, so the output is
// bit-identical for every thread count.
int hmr_layer_forward(void* layer, const float* x, std::size_t T, float* out,
                      std::uint32_t* ids, float* scores, std::int32_t* offsets,
                      int threads) {
    auto* L = static_cast<Layer*>(layer);
    if (!L || T == 0) return kInvalid;
    try {
        tensor::CpuTensorBackend cpu;
        const auto d = route(cpu, x, L->routerW.data(), L->hasBias ? L->bias.data() : nullptr,
                             T, L->H, L->E, L->k, L->softmax, L->renorm);
        if (ids && scores) {
            for (std::size_t t = 0; t < T; ++t) {
                for (std::size_t r = 0; r < L->k; ++r) {
                    ids[t * L->k + r] = d.tokens[t].selectedExpertIds[r];
                    scores[t * L->k + r] = d.tokens[t].routingScores[r];
                }
            }
        }
        if (offsets) {
            std::fill(offsets, offsets + L->E + 1, 0);
            for (const auto& g : d.expertGroups)
                offsets[g.expertId + 1] = static_cast<std::int32_t>(g.tokenIndices.size());
            for (std::size_t e = 0; e < L->E; ++e) offsets[e + 1] += offsets[e];
        }
        struct Job { std::size_t expert; std::vector<std::size_t> tokens; std::vector<float> w; };
        std::vector<Job> jobs;
        for (const auto& g : d.expertGroups) jobs.push_back({g.expertId, g.tokenIndices, g.routingScores});
        for (std::size_t s = 0; s < L->shared; ++s) {
            Job j{L->E + s, {}, {}};
            for (std::size_t t = 0; t < T; ++t) { j.tokens.push_back(t); j.w.push_back(1.0F); }
            jobs.push_back(std::move(j));
        }
        std::vector<std::vector<float>> results(jobs.size());
        std::atomic<std::size_t> next{0};
        std::atomic<bool> failed{false};
        const auto worker = [&]() {
            try {
                auto backend = std::make_shared<tensor::CpuTensorBackend>();
                ExpertMlpExecutor executor(backend);
                for (;;) {
                    const auto j = next.fetch_add(1);
                    if (j >= jobs.size() || failed) break;
                    const auto n = jobs[j].tokens.size();
                    auto in = backend->allocateTensor({n, L->H}, DType::FP32);
                    auto* ip = static_cast<float*>(in.data());
                    for (std::size_t r = 0; r < n; ++r)
                        std::memcpy(ip + r * L->H, x + jobs[j].tokens[r] * L->H, L->H * 4);
                    auto y = backend->allocateTensor({n, L->H}, DType::FP32);
                    executor.execute(in, L->weights(jobs[j].expert), y);
                    const auto* yp = static_cast<const float*>(y.data());
                    results[j].assign(yp, yp + n * L->H);
                }
            } catch (const std::exception&) {
                failed = true;
            }
        };
        const int nthreads = std::max(1, threads);
        std::vector<std::thread> pool;
        for (int i = 1; i < nthreads; ++i) pool.emplace_back(worker);
        worker();
        for (auto& t : pool) t.join();
        if (failed) return kFailed;
        std::fill(out, out + T * L->H, 0.0F);
        for (std::size_t j = 0; j < jobs.size(); ++j) {
            for (std::size_t r = 0; r < jobs[j].tokens.size(); ++r) {
                const auto tok = jobs[j].tokens[r];
                const auto wt = jobs[j].w[r];
                for (std::size_t h = 0; h < L->H; ++h)
                    out[tok * L->H + h] += wt * results[j][r * L->H + h];
            }
        }
        return kOk;
    } catch (const std::invalid_argument&) {
        return kInvalid;
    } catch (const std::exception&) {
        return kFailed;
    }
}

} // extern "C"
