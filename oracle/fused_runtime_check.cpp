// fused_runtime_check.cpp -- GPU check of hypermoe-engine_b200/host/
// FusedMoERuntime.cpp against the reference's own CPU path.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile links this program with the
// reference's library sources (CUDA backend enabled), ref_harness.cpp (the
// reference's CPU classes behind C entry points) and libhmoe.so.  It
//   1. builds the benchmark's seeded layer (host/synth.cpp),
//   2. places the expert arena, router matrix and bias on the device through
//      the reference's own CudaTensorBackend,
//   3. runs FusedMoERuntime::executeBatch with the routing materialised, and
//      executeLayer on one token,
//   4. runs the same layer through the reference's CPU classes
//      (hmr_layer_forward: CpuRouterBackend, ExpertMlpExecutor on
//      CpuTensorBackend, combine in ascending expert id),
// and compares: selected ids and expert groups bit for bit, scores to
// within the CPU expf's last-place rounding (2e-7 relative), expert
// batches equal to the groups, outputs within the INT8 layer tolerance
// (abs 2e-2 + rel 2e-2 element-wise, normwise <= 2e-2, cosine >= 0.9995;
// CorrectnessOracle::toleranceFor(INT8), CorrectnessOracle.cpp:34-42).
// Prints one JSON line; exit status 0 when every check holds.
//
// Usage: fused_runtime_check --hidden H --inter I --experts E --topk k
//          --softmax 0|1 --renorm 0|1 --shared S --zipf A --tokens T --seed s
#include "FusedMoERuntime.hpp"
#include "hmoe.h"

#include "models/ExpertWeightMap.hpp"
#include "storage/ExpertStore.hpp"
#include "tensor/backend/CpuTensorBackend.hpp"
#include "tensor/backend/CudaTensorBackend.hpp"

#include <filesystem>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <map>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include <unistd.h>

extern "C" {
void* hmr_layer_create(std::size_t H, std::size_t I, std::size_t E, std::size_t k, int softmax, int renorm,
                       const float* router_w, const float* router_bias, std::size_t n_shared,
                       const std::int8_t* arena, std::size_t stride, std::size_t gate_off, std::size_t up_off,
                       std::size_t down_off, const float* qscale, const std::int32_t* qzp);
void hmr_layer_destroy(void* layer);
int hmr_layer_forward(void* layer, const float* x, std::size_t T, float* out, std::uint32_t* ids, float* scores,
                      std::int32_t* offsets, int threads);
}

using namespace hypermoe;
using tensor::DType;

namespace {

tensor::Tensor upload(tensor::TensorBackend& dev, tensor::Shape shape, DType dtype, const void* src,
                      std::size_t bytes) {
    tensor::CpuTensorBackend cpu;
    auto host = cpu.allocateTensor(shape, dtype);
    std::memcpy(host.data(), src, bytes);
    auto d = dev.allocateTensor(shape, dtype);
    dev.copyTensor(host.view(), d.view());
    return d;
}

std::vector<float> download(tensor::TensorBackend& dev, const tensor::Tensor& t) {
    tensor::CpuTensorBackend cpu;
    auto host = cpu.allocateTensor(t.shape(), DType::FP32);
    dev.copyTensor(t.view(), host.view());
    const auto* p = static_cast<const float*>(host.data());
    return std::vector<float>(p, p + t.shape().elementCount());
}

struct Closeness {
    bool elementwise = true;
    double normwise = 0, cosine = 0, maxAbs = 0;
    bool ok() const { return elementwise && normwise <= 2e-2 && cosine >= 0.9995; }
};

Closeness compare(const std::vector<float>& a, const std::vector<float>& e) {
    Closeness c;
    double dd = 0, ee = 0, aa = 0, ae = 0;
    for (std::size_t i = 0; i < a.size(); ++i) {
        const double d = std::fabs(double(a[i]) - double(e[i]));
        if (!std::isfinite(a[i]) || d > 2e-2 + 2e-2 * std::fabs(double(e[i]))) c.elementwise = false;
        c.maxAbs = std::max(c.maxAbs, d);
        dd += d * d;
        ee += double(e[i]) * e[i];
        aa += double(a[i]) * a[i];
        ae += double(a[i]) * e[i];
    }
    c.normwise = std::sqrt(dd) / std::max(std::sqrt(ee), 1e-30);
    c.cosine = ae / std::max(std::sqrt(aa) * std::sqrt(ee), 1e-30);
    return c;
}

} // namespace

int main(int argc, char** argv) {
    std::map<std::string, double> a;
    for (int i = 1; i + 1 < argc; i += 2) a[argv[i]] = std::strtod(argv[i + 1], nullptr);
    const std::size_t H = a["--hidden"], I = a["--inter"], E = a["--experts"], k = a["--topk"], S = a["--shared"],
                      T = a["--tokens"];
    const int softmax = a.count("--softmax") ? int(a["--softmax"]) : 1;
    const int renorm = a.count("--renorm") ? int(a["--renorm"]) : 1;
    const float zipf = static_cast<float>(a["--zipf"]);
    const std::uint64_t seed = static_cast<std::uint64_t>(a["--seed"]);
    if (!H || !I || !E || !k || !T) {
        std::fprintf(stderr, "fused_runtime_check: missing shape arguments\n");
        return 2;
    }
    try {
        const int threads = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
        const std::size_t total = E + S, proj = H * I, stride = (3 * proj + 4095) / 4096 * 4096;
        std::vector<float> w(H * E), bias(E), x(T * H);
        hmoe_synth_normal(seed, 2, 0.02F, w.data(), w.size(), threads);
        if (zipf > 0) hmoe_synth_zipf_bias(seed, zipf, bias.data(), E);
        std::vector<std::int8_t> arena(total * stride, 0);
        std::vector<hmoe_expert_quant> q(total);
        hmoe_synth_arena(seed, 0, 0, static_cast<std::uint32_t>(total), static_cast<std::uint32_t>(H),
                         static_cast<std::uint32_t>(I), 0.02F, arena.data(), stride, 0, proj, 2 * proj, q.data(),
                         threads);
        hmoe_synth_normal(seed, 1, 1.0F, x.data(), x.size(), threads);

        // The reference's CPU path on the same layer.
        std::vector<float> qs(3 * total);
        std::vector<std::int32_t> qz(3 * total);
        for (std::size_t e = 0; e < total; ++e)
            for (int p = 0; p < 3; ++p) {
                qs[3 * e + p] = q[e].scale[p];
                qz[3 * e + p] = q[e].zero_point[p];
            }
        void* ref = hmr_layer_create(H, I, E, k, softmax, renorm, w.data(), zipf > 0 ? bias.data() : nullptr, S,
                                     arena.data(), stride, 0, proj, 2 * proj, qs.data(), qz.data());
        if (!ref) throw std::runtime_error("hmr_layer_create failed");
        std::vector<float> outRef(T * H), scRef(T * k);
        std::vector<std::uint32_t> idsRef(T * k);
        std::vector<std::int32_t> offRef(E + 1);
        if (hmr_layer_forward(ref, x.data(), T, outRef.data(), idsRef.data(), scRef.data(), offRef.data(),
                              threads) != 0)
            throw std::runtime_error("hmr_layer_forward failed");

        // The fused runtime on the reference's own CUDA tensor backend.
        auto cuda = std::make_shared<tensor::CudaTensorBackend>(0);
        if (!cuda->available()) {
            std::fprintf(stderr, "fused_runtime_check: no CUDA device\n");
            return 3;
        }
        auto dArena = upload(*cuda, {total * stride}, DType::INT8, arena.data(), arena.size());
        auto dW = upload(*cuda, {H, E}, DType::FP32, w.data(), w.size() * 4);
        auto dBias = upload(*cuda, {E}, DType::FP32, bias.data(), bias.size() * 4);
        auto dX = upload(*cuda, {T, H}, DType::FP32, x.data(), x.size() * 4);
        std::vector<runtime::FusedMoERuntime::ExpertQuantization> quant(total);
        for (std::size_t e = 0; e < total; ++e)
            for (int p = 0; p < 3; ++p) quant[e][p] = {q[e].scale[p], q[e].zero_point[p]};
        const router::RouterConfig config{
            E, k, softmax ? router::RoutingNormalization::Softmax : router::RoutingNormalization::None, renorm != 0};
        runtime::FusedMoERuntime fused(cuda, config, H, I, dArena.view(), stride, 0, proj, 2 * proj, quant, S,
                                       zipf > 0 ? tensor::TensorView(dBias) : tensor::TensorView());
        auto res = fused.executeBatch(7, dX.view(), dW.view(), true);
        const auto out = download(*cuda, res.output);

        bool idsOk = res.routing.tokens.size() == T && res.routing.layerId == 7;
        bool scoresOk = idsOk;
        for (std::size_t t = 0; idsOk && t < T; ++t)
            for (std::size_t r = 0; r < k; ++r) {
                idsOk = idsOk && res.routing.tokens[t].selectedExpertIds[r] == idsRef[t * k + r];
                // the device's exp is correctly rounded, the CPU's expf may be
                // one ulp off: scores agree to within that
                const double sa = res.routing.tokens[t].routingScores[r], sb = scRef[t * k + r];
                scoresOk = scoresOk && std::fabs(sa - sb) <= 2e-7 * std::fabs(sb) + 1e-7;
            }
        bool groupsOk = res.routing.valid();
        std::size_t touched = 0;
        for (std::size_t e = 0; e < E; ++e) touched += offRef[e + 1] > offRef[e];
        groupsOk = groupsOk && res.routing.expertGroups.size() == touched &&
                   res.expertBatches.size() == touched && res.execution.uniqueExperts == touched;
        for (std::size_t g = 0; groupsOk && g < res.routing.expertGroups.size(); ++g) {
            const auto& grp = res.routing.expertGroups[g];
            const auto n = static_cast<std::size_t>(offRef[grp.expertId + 1] - offRef[grp.expertId]);
            groupsOk = grp.tokenIndices.size() == n && res.expertBatches[g].expertId == grp.expertId &&
                       res.expertBatches[g].tokenIndices == grp.tokenIndices &&
                       res.expertBatches[g].routingWeights == grp.routingScores;
            for (std::size_t j = 0; groupsOk && j + 1 < n; ++j)
                groupsOk = grp.tokenIndices[j] < grp.tokenIndices[j + 1];
            if (g > 0) groupsOk = groupsOk && res.routing.expertGroups[g - 1].expertId < grp.expertId;
        }
        const Closeness close = compare(out, outRef);

        // One token through executeLayer.
        auto one = dX.view().sliceBytes(0, {1, H}, DType::FP32);
        auto layer = fused.executeLayer(7, one, dW.view());
        const auto out1 = download(*cuda, layer.output);
        bool layerOk = layer.routing.selectedExpertIds.size() == k;
        for (std::size_t r = 0; layerOk && r < k; ++r) layerOk = layer.routing.selectedExpertIds[r] == idsRef[r];
        const Closeness close1 = compare(out1, std::vector<float>(outRef.begin(), outRef.begin() + H));
        hmr_layer_destroy(ref);

        // All-resident mode from the reference's own packed store: the
        // experts written with ExpertStore::create (blob = gate|up|down) and
        // mapped as the packer's manifest maps them; the runtime built from
        // it must give the arena-built runtime's output bit for bit, and the
        // fused residual stage out + residual (one FP32 rounding) with its
        // BF16 copy.
        bool packedOk = true, residualOk = true, coversOk = true;
        if (S == 0) {
            const auto dir = std::filesystem::temp_directory_path() /
                             ("hmoe_packed_" + std::to_string(static_cast<long>(::getpid())));
            std::filesystem::remove_all(dir);
            std::filesystem::create_directories(dir);
            std::vector<storage::ExpertBlob> blobs(E);
            for (std::size_t e = 0; e < E; ++e) {
                blobs[e].layerId = 3;
                blobs[e].expertId = static_cast<std::uint32_t>(e);
                blobs[e].quantizationType = 1;
                const auto* src = reinterpret_cast<const std::byte*>(arena.data() + e * stride);
                blobs[e].data.assign(src, src + 3 * proj);
            }
            storage::ExpertStore::create(dir, blobs, "{}");
            storage::ExpertStore store(dir);
            models::ExpertWeightMap mappings;
            const models::ExpertWeightType types[3] = {models::ExpertWeightType::GATE, models::ExpertWeightType::UP,
                                                       models::ExpertWeightType::DOWN};
            for (std::size_t e = 0; e < E; ++e) {
                const auto rec = store.index().find(3, static_cast<std::uint32_t>(e)).value();
                for (int p = 0; p < 3; ++p)
                    mappings.add(3, static_cast<std::uint32_t>(e), types[p],
                                 {"expert", p < 2 ? tensor::Shape{H, I} : tensor::Shape{I, H}, DType::INT8,
                                  tensor::quantization::QuantizedDType::INT8, rec.offset + p * proj, proj, 3,
                                  static_cast<std::uint32_t>(e),
                                  tensor::quantization::QuantizationParameters{q[e].scale[p], q[e].zero_point[p]}});
            }
            std::size_t totalBytes = 0;
            for (const auto& rec : store.index().records()) totalBytes += static_cast<std::size_t>(rec.size);
            coversOk = runtime::FusedMoERuntime::coversAllExperts(totalBytes, store) &&
                       !runtime::FusedMoERuntime::coversAllExperts(totalBytes - 1, store);
            auto packed = runtime::FusedMoERuntime::fromPackedStore(
                cuda, store, mappings, 3, config, zipf > 0 ? tensor::TensorView(dBias) : tensor::TensorView());
            auto pres = packed->executeBatch(3, dX.view(), dW.view());
            packedOk = download(*cuda, pres.output) == out;
            tensor::Tensor out16;
            auto withRes = packed->executeWithResidual(3, dX.view(), dW.view(), dX.view(), &out16);
            const auto yr = download(*cuda, withRes);
            tensor::CpuTensorBackend cpu;
            auto h16 = cpu.allocateTensor({T, H}, DType::BF16);
            cuda->copyTensor(out16.view(), h16.view());
            const auto* b16 = static_cast<const std::uint16_t*>(h16.data());
            for (std::size_t i = 0; i < T * H && residualOk; ++i) {
                const float sum = x[i] + out[i];
                residualOk = yr[i] == sum;
                // round to nearest even of the FP32 result
                std::uint32_t u;
                std::memcpy(&u, &sum, 4);
                const std::uint32_t r = (u + 0x7fffu + ((u >> 16) & 1u)) >> 16;
                residualOk = residualOk && b16[i] == static_cast<std::uint16_t>(r);
            }
            std::filesystem::remove_all(dir);
        }

        const bool ok = idsOk && scoresOk && groupsOk && close.ok() && layerOk && close1.ok() && packedOk &&
                        residualOk && coversOk;
        std::printf("{\"ok\": %s, \"tokens\": %zu, \"ids_equal\": %s, \"scores_equal\": %s, \"groups_equal\": %s, "
                    "\"elementwise\": %s, \"normwise\": %.3e, \"cosine\": %.7f, \"max_abs\": %.3e, "
                    "\"execute_layer_ok\": %s, \"packed_store_ok\": %s, \"residual_ok\": %s, \"covers_ok\": %s, "
                    "\"unique_experts\": %zu, \"backend\": \"%s\"}\n",
                    ok ? "true" : "false", T, idsOk ? "true" : "false", scoresOk ? "true" : "false",
                    groupsOk ? "true" : "false", close.elementwise ? "true" : "false", close.normwise, close.cosine,
                    close.maxAbs, (layerOk && close1.ok()) ? "true" : "false", packedOk ? "true" : "false",
                    residualOk ? "true" : "false", coversOk ? "true" : "false", touched,
                    res.execution.tensorBackend.c_str());
        return ok ? 0 : 1;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "fused_runtime_check: %s\n", e.what());
        return 1;
    }
}
