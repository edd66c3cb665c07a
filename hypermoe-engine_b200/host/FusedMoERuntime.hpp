// FusedMoERuntime.hpp -- the reference's layer-runtime contract over the
// fused sm_100a layer (libhmoe.so, include/hmoe.h).
//
// A drop-in for MoERuntime::executeBatch / executeLayer
// (src/core/runtime/MoERuntime.hpp:57-60, MoERuntime.cpp:58-349) for a layer
// whose experts are all resident on the CUDA device: the same inputs
// (layer id, hidden states [T, H] FP32 on the device, router weights [H, E]
// FP32 on the device), the same result types (BatchLayerExecutionResult,
// LayerExecutionResult, MoERuntime.hpp:28-39) and the same errors
// (std::invalid_argument for bad arguments, std::runtime_error for a
// non-finite router score or a CUDA failure).  It plugs in under
// MoELayer::executeExpertsBatch (src/transformer/MoELayer.cpp:50-55) in
// place of MoERuntime when the expert budget covers the whole layer.
//
// What differs, by design:
//   * one fused call (route, group, permute, grouped INT8 expert MLP, combine
//     in ascending expert id) instead of a host loop over experts with a
//     synchronisation after every gather and scatter;
//   * routing decisions and expert batches are materialised on the host only
//     when asked for (`materializeRouting`), because building them needs a
//     device-to-host copy the fused path otherwise never makes;
//   * expertOutputs stays empty: per-expert FP32 outputs are never formed
//     (each expert's rows are weighted and combined inside the device).
//
// This file compiles against the reference's headers (its src/ and include/
// on the include path) and links with libhmoe.so; oracle/Makefile builds it
// into the GPU check program oracle/_ref/fused_runtime_check.
#pragma once

#include "core/runtime/MoERuntime.hpp"
#include "models/ExpertWeightMap.hpp"
#include "router/RouterConfig.hpp"
#include "storage/ExpertStore.hpp"
#include "tensor/Tensor.hpp"
#include "tensor/backend/TensorBackend.hpp"
#include "tensor/quantization/Quantization.hpp"

#include <array>
#include <cstddef>
#include <memory>
#include <mutex>
#include <vector>

namespace hypermoe::runtime {

class FusedMoERuntime {
public:
    // gate, up, down (ExpertMlpWeights, src/experts/ExpertExecutor.hpp:18-43)
    using ExpertQuantization = std::array<tensor::quantization::QuantizationParameters, 3>;

    // `arena`: every expert of the layer, resident on the backend's device, in
    // the ExpertPacker layout (tools/model_convert/ExpertPacker.cpp:150-247):
    // expert e's blob at e * expertStride holds gate [H, I], up [H, I] and
    // down [I, H] INT8 [in, out] views at the given offsets.  `quantization`
    // has one entry per expert (routed experts, then `sharedExperts`
    // always-on experts).  `routerBias` (optional, [E] FP32 on the device) is
    // added to each logit as the last term of the reference's double sum.
    FusedMoERuntime(std::shared_ptr<tensor::TensorBackend> backend,
                    router::RouterConfig config,
                    std::size_t hidden,
                    std::size_t intermediate,
                    tensor::TensorView arena,
                    std::size_t expertStride,
                    std::size_t gateOffset,
                    std::size_t upOffset,
                    std::size_t downOffset,
                    std::vector<ExpertQuantization> quantization,
                    std::size_t sharedExperts = 0,
                    tensor::TensorView routerBias = {});
    ~FusedMoERuntime();

    FusedMoERuntime(const FusedMoERuntime&) = delete;
    FusedMoERuntime& operator=(const FusedMoERuntime&) = delete;

    // All-resident expert mode (the packed model runtime's expert path,
    // src/models/runtime/PackedModelRuntime.cpp:345-400, with nothing left for
    // its scheduler, residency manager or transfer workers to do): every
    // expert of `layer` is read once from the reference's own packed store,
    // sliced with its ExpertWeightMap (ExpertWeightMap::createViews: the
    // same views and quantisation checks), repacked gate|up|down into one
    // device arena owned by the returned runtime, and uploaded through
    // `backend`.  The routed experts are ids 0..config.expertCount-1.
    [[nodiscard]] static std::unique_ptr<FusedMoERuntime> fromPackedStore(
        std::shared_ptr<tensor::TensorBackend> backend, const storage::ExpertStore& store,
        const models::ExpertWeightMap& weights, LayerId layer, router::RouterConfig config,
        tensor::TensorView routerBias = {});

    // Whether a device expert budget holds every expert the store indexes
    // (the condition under which a packed runtime can run its MoE layers on
    // fusedRuntime instances instead of the tiered MoERuntime).
    [[nodiscard]] static bool coversAllExperts(std::size_t deviceBudgetBytes, const storage::ExpertStore& store);

    // The transformer block's MoE stage with its residual add fused into the
    // combine (TransformerBlock.cpp:93-104, MoELayer.cpp:37-39): returns
    // residual + moe(hiddenStates) with one FP32 rounding, as the backend's
    // add gives, and writes its BF16 copy into *bf16Output ([T, H], DType
    // BF16, on the device) when given.  No [T, H] MoE output is materialised
    // and no separate add runs; the call returns once the result is complete
    // (the reference's CUDA tensor backend exposes no stream to order later
    // work against).
    [[nodiscard]] tensor::Tensor executeWithResidual(LayerId layerId, tensor::TensorView hiddenStates,
                                                     tensor::TensorView routerWeights,
                                                     tensor::TensorView residual,
                                                     tensor::Tensor* bf16Output = nullptr);

    [[nodiscard]] BatchLayerExecutionResult executeBatch(LayerId layerId,
                                                         tensor::TensorView hiddenStates,
                                                         tensor::TensorView routerWeights,
                                                         bool materializeRouting = false);
    // One token: routing is always materialised, as LayerExecutionResult
    // carries it.
    [[nodiscard]] LayerExecutionResult executeLayer(LayerId layerId,
                                                    tensor::TensorView hiddenState,
                                                    tensor::TensorView routerWeights);

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

} // namespace hypermoe::runtime
