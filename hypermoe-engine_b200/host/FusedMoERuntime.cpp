// FusedMoERuntime.cpp -- see FusedMoERuntime.hpp.
#include "FusedMoERuntime.hpp"

#include "hmoe.h"

#include "tensor/TensorView.hpp"
#include "tensor/backend/CpuTensorBackend.hpp"

#include <cuda_runtime_api.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <stdexcept>
#include <string>
#include <utility>

namespace hypermoe::runtime {

namespace {

void check(hmoe_status status, const char* what) {
    if (status == HMOE_OK) return;
    if (status == HMOE_INVALID_ARGUMENT) throw std::invalid_argument(std::string(what) + ": invalid argument");
    if (status == HMOE_CUDA_ERROR) throw std::runtime_error(std::string(what) + ": " + hmoe_last_error());
    throw std::runtime_error(std::string(what) + ": hmoe status " + std::to_string(static_cast<int>(status)));
}

void checkCuda(cudaError_t err, const char* what) {
    if (err != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(err));
}

} // namespace

struct FusedMoERuntime::Impl {
    std::shared_ptr<tensor::TensorBackend> backend;
    router::RouterConfig config;
    std::size_t H, I, S, stride, gateOffset, upOffset, downOffset;
    tensor::TensorView arena, bias;
    tensor::Tensor ownedArena; // fromPackedStore: the device arena the runtime owns
    tensor::Tensor quant;     // device hmoe_expert_quant[E + S]
    tensor::Tensor workspace; // device scratch, grown to the largest batch seen
    cudaStream_t stream{};
    std::mutex mutex;         // one layer call at a time, as MoERuntime::executionMutex_

    hmoe_layer_desc desc(const void* routerWeights) const {
        hmoe_layer_desc d{};
        d.hidden = static_cast<std::uint32_t>(H);
        d.intermediate = static_cast<std::uint32_t>(I);
        d.experts = static_cast<std::uint32_t>(config.expertCount);
        d.top_k = static_cast<std::uint32_t>(config.topK);
        d.softmax = config.normalization == router::RoutingNormalization::Softmax ? 1 : 0;
        d.renormalize = config.renormalizeSelected ? 1 : 0;
        d.shared_experts = static_cast<std::uint32_t>(S);
        d.router_weight = static_cast<const float*>(routerWeights);
        d.router_bias = bias ? static_cast<const float*>(bias.data()) : nullptr;
        d.arena = static_cast<const std::int8_t*>(arena.data());
        d.expert_stride = stride;
        d.gate_offset = gateOffset;
        d.up_offset = upOffset;
        d.down_offset = downOffset;
        d.quant = static_cast<const hmoe_expert_quant*>(quant.data());
        d.ep_rank = 0;
        d.ep_size = 1;
        return d;
    }

    void* scratch(std::size_t bytes) {
        if (!workspace || workspace.bytes() < bytes)
            workspace = backend->allocateTensor({bytes}, tensor::DType::INT8);
        return workspace.data();
    }

    void validate(tensor::TensorView hidden, tensor::TensorView router) const {
        const auto cuda = backend->device();
        if (!hidden || hidden.shape().rank() != 2 || hidden.dtype() != tensor::DType::FP32 ||
            hidden.device() != cuda || !hidden.isContiguous() || hidden.shape().dimensions()[1] != H)
            throw std::invalid_argument("fused MoE runtime requires contiguous FP32 hidden states [T, H] on the device");
        if (!router || router.shape().rank() != 2 || router.dtype() != tensor::DType::FP32 ||
            router.device() != cuda || !router.isContiguous() || router.shape().dimensions()[0] != H ||
            router.shape().dimensions()[1] != config.expertCount)
            throw std::invalid_argument("fused MoE runtime requires contiguous FP32 router weights [H, E] on the device");
    }
};

FusedMoERuntime::FusedMoERuntime(std::shared_ptr<tensor::TensorBackend> backend, router::RouterConfig config,
                                 std::size_t hidden, std::size_t intermediate, tensor::TensorView arena,
                                 std::size_t expertStride, std::size_t gateOffset, std::size_t upOffset,
                                 std::size_t downOffset, std::vector<ExpertQuantization> quantization,
                                 std::size_t sharedExperts, tensor::TensorView routerBias)
    : impl_(std::make_unique<Impl>()) {
    config.validate(); // RouterConfig::validate, RouterConfig.cpp:9-22
    if (!backend || !backend->available() || backend->device().type != tensor::DeviceType::CUDA)
        throw std::invalid_argument("fused MoE runtime requires an available CUDA tensor backend");
    const std::size_t experts = config.expertCount + sharedExperts;
    if (!arena || arena.device() != backend->device() || arena.bytes() < experts * expertStride)
        throw std::invalid_argument("fused MoE runtime: the expert arena must hold every expert on the device");
    if (quantization.size() != experts)
        throw std::invalid_argument("fused MoE runtime: one quantisation entry per expert is required");
    if (routerBias && (routerBias.device() != backend->device() || routerBias.dtype() != tensor::DType::FP32 ||
                       routerBias.bytes() != config.expertCount * sizeof(float)))
        throw std::invalid_argument("fused MoE runtime: router bias must be [E] FP32 on the device");
    auto& m = *impl_;
    m.backend = std::move(backend);
    m.config = config;
    m.H = hidden;
    m.I = intermediate;
    m.S = sharedExperts;
    m.stride = expertStride;
    m.gateOffset = gateOffset;
    m.upOffset = upOffset;
    m.downOffset = downOffset;
    m.arena = arena;
    m.bias = routerBias;
    // Parameters are checked as the reference's runtime checks them
    // (validateParameters, Quantization.cpp:24-40), then uploaded once.
    tensor::CpuTensorBackend cpu;
    auto host = cpu.allocateTensor({experts * sizeof(hmoe_expert_quant)}, tensor::DType::INT8);
    auto* q = static_cast<hmoe_expert_quant*>(host.data());
    for (std::size_t e = 0; e < experts; ++e) {
        for (int p = 0; p < 3; ++p) {
            tensor::quantization::validateParameters(tensor::quantization::QuantizedDType::INT8, quantization[e][p]);
            q[e].scale[p] = quantization[e][p].scale;
            q[e].zero_point[p] = quantization[e][p].zeroPoint;
        }
    }
    m.quant = m.backend->allocateTensor(host.shape(), tensor::DType::INT8);
    m.backend->copyTensor(host.view(), m.quant.view());
    // The descriptor's shape limits are checked once here.
    hmoe_layer_desc d = m.desc(nullptr);
    d.router_weight = reinterpret_cast<const float*>(m.quant.data()); // any non-null device pointer
    std::size_t bytes = 0;
    check(hmoe_workspace_size(&d, 1, &bytes), "fused MoE runtime layer descriptor");
    checkCuda(cudaSetDevice(m.backend->device().ordinal), "cudaSetDevice");
    checkCuda(cudaStreamCreateWithFlags(&m.stream, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
}

FusedMoERuntime::~FusedMoERuntime() {
    if (impl_ && impl_->stream) {
        cudaStreamSynchronize(impl_->stream);
        cudaStreamDestroy(impl_->stream);
    }
}

BatchLayerExecutionResult FusedMoERuntime::executeBatch(LayerId layerId, tensor::TensorView hiddenStates,
                                                        tensor::TensorView routerWeights,
                                                        bool materializeRouting) {
    auto& m = *impl_;
    std::lock_guard<std::mutex> lock(m.mutex);
    m.validate(hiddenStates, routerWeights);
    const std::size_t T = hiddenStates.shape().dimensions()[0];
    const std::size_t k = m.config.topK, E = m.config.expertCount, H = m.H;
    if (T == 0) throw std::invalid_argument("fused MoE runtime requires at least one token");
    checkCuda(cudaSetDevice(m.backend->device().ordinal), "cudaSetDevice");
    // Inputs were produced on the backend's streams: complete them first, as
    // the reference's runtime does at its own synchronisation points.
    m.backend->synchronizeExecution();

    BatchLayerExecutionResult result;
    result.output = m.backend->allocateTensor({T, H}, tensor::DType::FP32);
    const hmoe_layer_desc d = m.desc(routerWeights.data());
    std::size_t bytes = 0;
    check(hmoe_workspace_size(&d, T, &bytes), "fused MoE runtime workspace size");
    void* ws = m.scratch(bytes);
    const auto start = std::chrono::steady_clock::now();
    check(hmoe_moe_forward(&d, static_cast<const float*>(hiddenStates.data()),
                           static_cast<float*>(result.output.data()), T, ws, bytes, m.stream),
          "fused MoE layer");
    std::int32_t status = 0, ties = 0, sequential = 0;
    check(hmoe_read_status(ws, &status, &ties, &sequential, m.stream), "fused MoE layer status");
    if (status == HMOE_NON_FINITE_ROUTER)
        throw std::runtime_error("router produced a non-finite score"); // CudaTensorBackend.cpp:642-645
    check(static_cast<hmoe_status>(status), "fused MoE layer (device)");
    const auto end = std::chrono::steady_clock::now();

    result.execution.expertAssignments = T * k;
    result.execution.tensorBackend = "hmoe fused sm_100a layer";
    result.execution.expertExecutionTime = end - start;
    result.routing.layerId = layerId;
    if (!materializeRouting) return result;

    // Routing decision and expert batches (the grouping of
    // CpuRouterBackend::routeBatch, CpuRouterBackend.cpp:140-158): selected
    // ids and scores per token in rank order, groups by ascending expert id
    // with tokens ascending.
    tensor::Tensor ids = m.backend->allocateTensor({T, k}, tensor::DType::FP32); // 4-byte slots
    tensor::Tensor scores = m.backend->allocateTensor({T, k}, tensor::DType::FP32);
    tensor::Tensor offsets = m.backend->allocateTensor({E + 1}, tensor::DType::FP32);
    tensor::Tensor gtok = m.backend->allocateTensor({T * k}, tensor::DType::FP32);
    tensor::Tensor gsc = m.backend->allocateTensor({T * k}, tensor::DType::FP32);
    check(hmoe_route(&d, static_cast<const float*>(hiddenStates.data()), T, static_cast<std::uint32_t*>(ids.data()),
                     static_cast<float*>(scores.data()), static_cast<std::int32_t*>(offsets.data()),
                     static_cast<std::uint32_t*>(gtok.data()), static_cast<float*>(gsc.data()), ws, bytes,
                     m.stream),
          "fused MoE routing");
    std::vector<std::uint32_t> hid(T * k), htok(T * k);
    std::vector<float> hsc(T * k), hgsc(T * k);
    std::vector<std::int32_t> hoff(E + 1);
    checkCuda(cudaMemcpyAsync(hid.data(), ids.data(), T * k * 4, cudaMemcpyDeviceToHost, m.stream), "routing ids");
    checkCuda(cudaMemcpyAsync(hsc.data(), scores.data(), T * k * 4, cudaMemcpyDeviceToHost, m.stream), "routing scores");
    checkCuda(cudaMemcpyAsync(hoff.data(), offsets.data(), (E + 1) * 4, cudaMemcpyDeviceToHost, m.stream), "offsets");
    checkCuda(cudaMemcpyAsync(htok.data(), gtok.data(), T * k * 4, cudaMemcpyDeviceToHost, m.stream), "groups");
    checkCuda(cudaMemcpyAsync(hgsc.data(), gsc.data(), T * k * 4, cudaMemcpyDeviceToHost, m.stream), "group scores");
    checkCuda(cudaStreamSynchronize(m.stream), "routing readback");
    result.routing.tokens.resize(T);
    for (std::size_t t = 0; t < T; ++t) {
        auto& r = result.routing.tokens[t];
        r.layerId = layerId;
        r.selectedExpertIds.assign(hid.begin() + t * k, hid.begin() + (t + 1) * k);
        r.routingScores.assign(hsc.begin() + t * k, hsc.begin() + (t + 1) * k);
    }
    for (std::size_t e = 0; e < E; ++e) {
        const auto b = static_cast<std::size_t>(hoff[e]), n = static_cast<std::size_t>(hoff[e + 1]) - b;
        if (n == 0) continue;
        router::ExpertTokenGroup g;
        g.expertId = static_cast<ExpertId>(e);
        g.tokenIndices.assign(htok.begin() + b, htok.begin() + b + n);
        g.routingScores.assign(hgsc.begin() + b, hgsc.begin() + b + n);
        result.expertBatches.push_back({layerId, g.expertId, g.tokenIndices, g.routingScores});
        result.routing.expertGroups.push_back(std::move(g));
    }
    result.execution.uniqueExperts = result.routing.expertGroups.size();
    return result;
}

std::unique_ptr<FusedMoERuntime> FusedMoERuntime::fromPackedStore(std::shared_ptr<tensor::TensorBackend> backend,
                                                                   const storage::ExpertStore& store,
                                                                   const models::ExpertWeightMap& weights,
                                                                   LayerId layer, router::RouterConfig config,
                                                                   tensor::TensorView routerBias) {
    config.validate();
    if (!backend || !backend->available())
        throw std::invalid_argument("fused MoE runtime requires an available CUDA tensor backend");
    const std::size_t E = config.expertCount;
    std::size_t H = 0, I = 0;
    tensor::CpuTensorBackend cpu;
    std::vector<ExpertQuantization> quant(E);
    tensor::Tensor host;
    std::size_t stride = 0;
    for (std::size_t e = 0; e < E; ++e) {
        const auto id = static_cast<std::uint32_t>(e);
        const auto record = store.index().find(layer, id);
        if (!record) throw std::invalid_argument("packed store lacks an expert of the layer");
        const auto payload = store.mappedExpert(layer, id); // CRC-checked
        // a TensorView does not own its storage: keep the buffer alive here
        const auto buffer = std::make_shared<const std::vector<std::byte>>(payload.begin(), payload.end());
        const auto view = tensor::TensorView::fromHostBuffer({payload.size()}, tensor::DType::INT8, buffer, false);
        const auto w = weights.createViews(layer, id, view, record->offset);
        const auto& g = w.gateProjection.shape().dimensions();
        const auto& d = w.downProjection.shape().dimensions();
        if (w.gateProjection.dtype() != tensor::DType::INT8 || w.upProjection.dtype() != tensor::DType::INT8 ||
            w.downProjection.dtype() != tensor::DType::INT8 || g.size() != 2 || d.size() != 2 ||
            w.upProjection.shape() != w.gateProjection.shape() || d[0] != g[1] || d[1] != g[0] ||
            !w.gateQuantization || !w.upQuantization || !w.downQuantization)
            throw std::invalid_argument("fused MoE runtime needs INT8 [H,I] gate/up and [I,H] down projections");
        if (e == 0) {
            H = g[0];
            I = g[1];
            stride = (3 * H * I + 4095) / 4096 * 4096; // ExpertPacker's blob alignment
            host = cpu.allocateTensor({E * stride}, tensor::DType::INT8);
            std::memset(host.data(), 0, E * stride);
        } else if (g[0] != H || g[1] != I) {
            throw std::invalid_argument("experts of one layer differ in shape");
        }
        auto* dst = static_cast<std::byte*>(host.data()) + e * stride;
        std::memcpy(dst, w.gateProjection.data(), H * I);
        std::memcpy(dst + H * I, w.upProjection.data(), H * I);
        std::memcpy(dst + 2 * H * I, w.downProjection.data(), H * I);
        quant[e] = {*w.gateQuantization, *w.upQuantization, *w.downQuantization};
    }
    auto arena = backend->allocateTensor(host.shape(), tensor::DType::INT8);
    backend->copyTensor(host.view(), arena.view());
    auto runtime = std::make_unique<FusedMoERuntime>(backend, config, H, I, arena.view(), stride, 0, H * I,
                                                     2 * H * I, std::move(quant), 0, routerBias);
    runtime->impl_->ownedArena = std::move(arena);
    return runtime;
}

bool FusedMoERuntime::coversAllExperts(std::size_t deviceBudgetBytes, const storage::ExpertStore& store) {
    std::size_t total = 0;
    for (const auto& record : store.index().records()) {
        if (record.size > deviceBudgetBytes - std::min(total, deviceBudgetBytes)) return false;
        total += static_cast<std::size_t>(record.size);
    }
    return true;
}

tensor::Tensor FusedMoERuntime::executeWithResidual(LayerId, tensor::TensorView hiddenStates,
                                                    tensor::TensorView routerWeights, tensor::TensorView residual,
                                                    tensor::Tensor* bf16Output) {
    auto& m = *impl_;
    std::lock_guard<std::mutex> lock(m.mutex);
    m.validate(hiddenStates, routerWeights);
    const std::size_t T = hiddenStates.shape().dimensions()[0], H = m.H;
    if (T == 0) throw std::invalid_argument("fused MoE runtime requires at least one token");
    if (!residual || residual.shape() != hiddenStates.shape() || residual.dtype() != tensor::DType::FP32 ||
        residual.device() != m.backend->device() || !residual.isContiguous())
        throw std::invalid_argument("MoE output is incompatible with residual input");
    checkCuda(cudaSetDevice(m.backend->device().ordinal), "cudaSetDevice");
    m.backend->synchronizeExecution();
    auto output = m.backend->allocateTensor({T, H}, tensor::DType::FP32);
    std::uint16_t* y16 = nullptr;
    if (bf16Output) {
        *bf16Output = m.backend->allocateTensor({T, H}, tensor::DType::BF16);
        y16 = static_cast<std::uint16_t*>(bf16Output->data());
    }
    const hmoe_layer_desc d = m.desc(routerWeights.data());
    std::size_t bytes = 0;
    check(hmoe_workspace_size(&d, T, &bytes), "fused MoE runtime workspace size");
    void* ws = m.scratch(bytes);
    check(hmoe_moe_forward_residual(&d, static_cast<const float*>(hiddenStates.data()),
                                    static_cast<const float*>(residual.data()), static_cast<float*>(output.data()),
                                    y16, T, ws, bytes, m.stream),
          "fused MoE layer with residual");
    std::int32_t status = 0, ties = 0, sequential = 0;
    check(hmoe_read_status(ws, &status, &ties, &sequential, m.stream), "fused MoE layer status"); // synchronises
    if (status == HMOE_NON_FINITE_ROUTER) throw std::runtime_error("router produced a non-finite score");
    check(static_cast<hmoe_status>(status), "fused MoE layer (device)");
    return output;
}

LayerExecutionResult FusedMoERuntime::executeLayer(LayerId layerId, tensor::TensorView hiddenState,
                                                   tensor::TensorView routerWeights) {
    if (hiddenState && hiddenState.shape().rank() == 1)
        hiddenState = hiddenState.reshape({1, hiddenState.shape().dimensions()[0]});
    auto batch = executeBatch(layerId, hiddenState, routerWeights, true);
    if (batch.routing.tokens.size() != 1)
        throw std::invalid_argument("single-token MoE layer received multiple tokens");
    return {std::move(batch.routing.tokens.front()), std::move(batch.output)};
}

} // namespace hypermoe::runtime
