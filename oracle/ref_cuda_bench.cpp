// ref_cuda_bench.cpp -- times the reference's own CUDA path for one MoE layer.
//
// TEST / MEASUREMENT INFRASTRUCTURE ONLY: this is the bar the B200 path is
// measured against, never the product.  oracle/Makefile compiles it together
// with the reference's sources, read in place from the reference tree and
// built with its CUDA backend enabled (HYPERMOE_HAS_CUDA, HYPERMOE_HAS_CUBLAS,
// HYPERMOE_HAS_CUDA_KERNELS; CudaKernels.cu by nvcc for sm_100a), into the
// standalone executable oracle/_ref/ref_cuda_bench.  It runs in a process of
// its own, so neither libhmoe.so nor torch shares its CUDA context.
//
// One step is the layer as MoERuntime::executeBatch runs it on a CUDA
// backend with every expert resident (src/core/runtime/MoERuntime.cpp:
// 182-349, `nativeCuda` branch):
//   CudaRouterBackend::routeBatch            cuBLAS FP32 logits, routerTopKKernel,
//                                            device->host readback, host grouping
//                                            (src/router/CudaRouterBackend.cpp:104-116,
//                                             CudaTensorBackend.cpp:601-652)
//   CudaTensorBackend::zero(output)          MoERuntime.cpp:188
//   per expert group, ascending expert id:
//     CudaTensorBackend::gatherRows          MoERuntime.cpp:285-286
//     ExpertMlpExecutor::execute             MoERuntime.cpp:302-303 (three INT8
//                                            GEMMs through planInt8Gemm's Auto mode,
//                                            SiLU, multiply)
//     CudaTensorBackend::scatterAddRows      MoERuntime.cpp:309-310
// The scheduler, residency leases and storage that MoERuntime also drives
// are not part of this all-resident path and are not linked.
//
// Inputs are the same seeded synthetic layer and tokens the B200 benchmark
// uses (hypermoe-engine_b200/host/synth.cpp compiled into this executable).
// The optional router bias (Zipf skew) is folded in the way the CPU harness
// folds it: the hidden rows get a constant 1 column and the router matrix a
// bias row, so the reference's own router computes logit + bias.
//
// Usage:
//   ref_cuda_bench --hidden H --inter I --experts E --topk k --softmax 0|1
//                  --renorm 0|1 --shared S --zipf A --tokens T --seed s
//                  --steps K --warmup W [--dump out.f32]
// Prints one JSON object: per-step wall-clock milliseconds (the path
// synchronises with the device inside every step, so host time is device
// time), tokens/s, experts touched.  --dump writes the last step's output
// [T, H] FP32.

#include "hmoe.h"

#include "backend/cuda/Int8GemmPlan.hpp"
#include "experts/ExpertExecutor.hpp"
#include "router/CudaRouterBackend.hpp"
#include "router/RouterConfig.hpp"
#include "tensor/backend/CpuTensorBackend.hpp"
#include "tensor/backend/CudaTensorBackend.hpp"

#include <cuda_runtime_api.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <map>
#include <memory>
#include <string>
#include <thread>
#include <vector>

using namespace hypermoe;
using tensor::DType;

namespace {

struct Args {
    std::size_t H = 0, I = 0, E = 0, k = 0, S = 0, T = 0;
    int softmax = 1, renorm = 1, steps = 5, warmup = 2;
    float zipf = 0.0F;
    std::uint64_t seed = 0;
    std::string dump;
};

Args parse(int argc, char** argv) {
    Args a;
    std::map<std::string, std::string> kv;
    for (int i = 1; i + 1 < argc; i += 2) kv[argv[i]] = argv[i + 1];
    auto num = [&](const char* key, double dflt) {
        const auto it = kv.find(key);
        return it == kv.end() ? dflt : std::strtod(it->second.c_str(), nullptr);
    };
    a.H = static_cast<std::size_t>(num("--hidden", 0));
    a.I = static_cast<std::size_t>(num("--inter", 0));
    a.E = static_cast<std::size_t>(num("--experts", 0));
    a.k = static_cast<std::size_t>(num("--topk", 0));
    a.S = static_cast<std::size_t>(num("--shared", 0));
    a.T = static_cast<std::size_t>(num("--tokens", 0));
    a.softmax = static_cast<int>(num("--softmax", 1));
    a.renorm = static_cast<int>(num("--renorm", 1));
    a.zipf = static_cast<float>(num("--zipf", 0));
    a.seed = static_cast<std::uint64_t>(num("--seed", 0));
    a.steps = static_cast<int>(num("--steps", 5));
    a.warmup = static_cast<int>(num("--warmup", 2));
    if (kv.count("--dump")) a.dump = kv["--dump"];
    return a;
}

tensor::Tensor upload(tensor::CudaTensorBackend& cuda, tensor::CpuTensorBackend& cpu, tensor::Shape shape,
                      DType dtype, const void* src, std::size_t bytes) {
    auto host = cpu.allocateTensor(shape, dtype);
    std::memcpy(host.data(), src, bytes);
    auto dev = cuda.allocateTensor(shape, dtype);
    cuda.copyTensor(host.view(), dev.view());
    return dev;
}

} // namespace

int main(int argc, char** argv) {
    const Args a = parse(argc, argv);
    if (!a.H || !a.I || !a.E || !a.k || !a.T || a.k > a.E) {
        std::fprintf(stderr, "ref_cuda_bench: missing or invalid shape arguments\n");
        return 2;
    }
    try {
        const int threads = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
        const std::size_t total = a.E + a.S;
        const std::size_t proj = a.H * a.I;
        const std::size_t stride = (3 * proj + 4095) / 4096 * 4096; // ExpertPacker blob alignment
        // The benchmark's seeded layer (hmoe_api.make_host_layer, layer 0).
        std::vector<float> routerW(a.H * a.E), bias(a.E), x(a.T * a.H);
        hmoe_synth_normal(a.seed, 2, 0.02F, routerW.data(), routerW.size(), threads);
        const bool hasBias = a.zipf > 0.0F;
        if (hasBias) hmoe_synth_zipf_bias(a.seed, a.zipf, bias.data(), a.E);
        std::vector<std::int8_t> arena(total * stride, 0);
        std::vector<hmoe_expert_quant> quant(total);
        hmoe_synth_arena(a.seed, 0, 0, static_cast<std::uint32_t>(total), static_cast<std::uint32_t>(a.H),
                         static_cast<std::uint32_t>(a.I), 0.02F, arena.data(), stride, 0, proj, 2 * proj,
                         quant.data(), threads);
        hmoe_synth_normal(a.seed, 1, 1.0F, x.data(), x.size(), threads);

        auto cuda = std::make_shared<tensor::CudaTensorBackend>(0, nullptr, backend::cuda::Int8GemmMode::Auto);
        if (!cuda->available() || !cuda->nativeKernelsAvailable()) {
            std::fprintf(stderr, "ref_cuda_bench: the reference CUDA backend is unavailable\n");
            return 3;
        }
        tensor::CpuTensorBackend cpu;
        const std::size_t Hx = hasBias ? a.H + 1 : a.H;
        std::vector<float> wExt(Hx * a.E), xExt(a.T * Hx);
        std::memcpy(wExt.data(), routerW.data(), routerW.size() * 4);
        if (hasBias) std::memcpy(wExt.data() + a.H * a.E, bias.data(), a.E * 4);
        for (std::size_t t = 0; t < a.T; ++t) {
            std::memcpy(xExt.data() + t * Hx, x.data() + t * a.H, a.H * 4);
            if (hasBias) xExt[t * Hx + a.H] = 1.0F;
        }
        auto dW = upload(*cuda, cpu, {Hx, a.E}, DType::FP32, wExt.data(), wExt.size() * 4);
        auto dXr = upload(*cuda, cpu, {a.T, Hx}, DType::FP32, xExt.data(), xExt.size() * 4);
        auto dX = upload(*cuda, cpu, {a.T, a.H}, DType::FP32, x.data(), x.size() * 4);
        auto dArena = upload(*cuda, cpu, {total * stride}, DType::INT8, arena.data(), arena.size());
        auto out = cuda->allocateTensor({a.T, a.H}, DType::FP32);

        using QP = tensor::quantization::QuantizationParameters;
        auto weights = [&](std::size_t e) {
            tensor::TensorView all(dArena);
            const std::size_t base = e * stride;
            return ExpertMlpWeights{all.sliceBytes(base, {a.H, a.I}, DType::INT8),
                                    all.sliceBytes(base + proj, {a.H, a.I}, DType::INT8),
                                    all.sliceBytes(base + 2 * proj, {a.I, a.H}, DType::INT8),
                                    QP{quant[e].scale[0], quant[e].zero_point[0]},
                                    QP{quant[e].scale[1], quant[e].zero_point[1]},
                                    QP{quant[e].scale[2], quant[e].zero_point[2]}};
        };
        const router::RouterConfig config{
            a.E, a.k, a.softmax ? router::RoutingNormalization::Softmax : router::RoutingNormalization::None,
            a.renorm != 0};
        router::CudaRouterBackend router(cuda);
        ExpertMlpExecutor executor(cuda);
        std::vector<std::size_t> allTokens(a.T);
        std::vector<float> ones(a.T, 1.0F);
        for (std::size_t t = 0; t < a.T; ++t) allTokens[t] = t;

        std::size_t touched = 0;
        auto step = [&]() {
            const auto decision = router.routeBatch(0, dXr.view(), dW.view(), config);
            cuda->zero(out.view());
            touched = decision.expertGroups.size();
            for (const auto& g : decision.expertGroups) { // ascending expert id
                const std::size_t n = g.tokenIndices.size();
                auto in = cuda->allocateTensor({n, a.H}, DType::FP32);
                cuda->gatherRows(dX.view(), g.tokenIndices, in.view());
                auto y = cuda->allocateTensor({n, a.H}, DType::FP32);
                executor.execute(in.view(), weights(g.expertId), y.view());
                cuda->scatterAddRows(y.view(), g.tokenIndices, g.routingScores, out.view());
            }
            for (std::size_t s = 0; s < a.S; ++s) { // always-on experts after the routed ones
                auto in = cuda->allocateTensor({a.T, a.H}, DType::FP32);
                cuda->gatherRows(dX.view(), allTokens, in.view());
                auto y = cuda->allocateTensor({a.T, a.H}, DType::FP32);
                executor.execute(in.view(), weights(a.E + s), y.view());
                cuda->scatterAddRows(y.view(), allTokens, ones, out.view());
            }
            cuda->synchronizeExecution();
        };

        // L2 flush between steps (larger than the 126 MB L2).
        void* flush = nullptr;
        const std::size_t flushBytes = std::size_t(256) << 20;
        if (cudaMalloc(&flush, flushBytes) != cudaSuccess) flush = nullptr;
        for (int i = 0; i < a.warmup; ++i) step();
        std::vector<double> ms;
        for (int i = 0; i < a.steps; ++i) {
            if (flush) {
                cudaMemset(flush, i & 0xff, flushBytes);
                cudaDeviceSynchronize();
            }
            const auto t0 = std::chrono::steady_clock::now();
            step();
            const auto t1 = std::chrono::steady_clock::now();
            ms.push_back(std::chrono::duration<double, std::milli>(t1 - t0).count());
        }
        if (flush) cudaFree(flush);
        if (!a.dump.empty()) {
            auto host = cpu.allocateTensor({a.T, a.H}, DType::FP32);
            cuda->copyTensor(out.view(), host.view());
            std::FILE* f = std::fopen(a.dump.c_str(), "wb");
            if (f) {
                std::fwrite(host.data(), 4, a.T * a.H, f);
                std::fclose(f);
            }
        }
        std::vector<double> sorted = ms;
        std::sort(sorted.begin(), sorted.end());
        double mean = 0.0;
        for (double v : ms) mean += v;
        mean /= static_cast<double>(ms.size());
        const double median = sorted[sorted.size() / 2];
        std::printf("{\"impl\": \"reference-cuda\", \"tokens\": %zu, \"steps\": %d, \"warmup\": %d, "
                    "\"ms_mean\": %.6f, \"ms_median\": %.6f, \"ms_min\": %.6f, \"value\": %.3f, "
                    "\"unique_experts\": %zu, \"int8_gemm_mode\": \"auto\", \"ms\": [",
                    a.T, a.steps, a.warmup, mean, median, sorted.front(),
                    static_cast<double>(a.T) / (median * 1e-3), touched + a.S);
        for (std::size_t i = 0; i < ms.size(); ++i) std::printf(i ? ", %.6f" : "%.6f", ms[i]);
        std::printf("]}\n");
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "ref_cuda_bench: %s\n", e.what());
        return 1;
    }
}
