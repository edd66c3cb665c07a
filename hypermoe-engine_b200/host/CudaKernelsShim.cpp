// CudaKernelsShim.cpp -- the reference's CUDA kernel launchers
// (namespace hypermoe::backend::cuda::kernels, src/backend/cuda/
// CudaKernels.hpp:10-46) defined over the libhmoe.so C ABI.
//
// Linked into the reference's build in place of the hot-path definitions of
// src/backend/cuda/CudaKernels.cu, this file makes CudaTensorBackend (and so
// ExpertMlpExecutor, activation::apply, MoERuntime and CudaRouterBackend)
// run the sm_100a kernels with no change to any caller.  Same arguments,
// same stream semantics (enqueue and return), same exceptions:
//   * a launch failure throws std::runtime_error("<op>: <CUDA error>")
//     (CudaKernels.cu:293-299);
//   * int8WeightMatmulCooperative throws std::invalid_argument on a plan or
//     scratch mismatch (CudaKernels.cu:330-333).
// rmsNorm, rope and causalAttention are not on the MoE hot path and stay
// the reference's own.
//
// With HMOE_SHIM_TRACE set in the environment, the process prints at exit
// how often each launcher here was called (stderr, one line), so a caller
// can see that its kernel launches went through this file.
//
// Build modes:
//   * inside the reference tree: -DHMOE_SHIM_WITH_REFERENCE_HEADERS and the
//     reference's src/ on the include path; the header's declarations are
//     then the ones defined here, and the static_asserts at the end fail to
//     compile if any signature drifted;
//   * standalone (libhmoe_shim.so, used by the tests): the declarations
//     below, which spell the same signatures.
#include "hmoe.h"

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <type_traits>

#ifdef HMOE_SHIM_WITH_REFERENCE_HEADERS
#include "backend/cuda/CudaKernels.hpp"
#else
namespace hypermoe::backend {
using StreamHandle = void*; // src/backend/Backend.hpp:12
}
namespace hypermoe::backend::cuda::kernels {
void activation(int type, const float* input, float* output, std::size_t elements, StreamHandle stream);
void int8WeightMatmul(const float* left, const std::int8_t* right, float* output, std::size_t rows,
                      std::size_t inner, std::size_t columns, float scale, std::int32_t zeroPoint,
                      StreamHandle stream);
void int8WeightMatmulCooperative(const float* left, const std::int8_t* right, float* output, float* partials,
                                 std::size_t rows, std::size_t inner, std::size_t columns,
                                 std::size_t partitions, float scale, std::int32_t zeroPoint,
                                 StreamHandle stream);
void routerTopK(float* logits, std::size_t tokens, std::size_t experts, std::size_t topK, bool softmax,
                bool renormalize, std::uint32_t* selectedIds, float* selectedScores, StreamHandle stream);
void gatherRows(const float* input, float* output, const std::uint32_t* rows, std::size_t rowCount,
                std::size_t width, StreamHandle stream);
void scatterAddRows(const float* input, float* output, const std::uint32_t* rows, const float* weights,
                    std::size_t rowCount, std::size_t width, StreamHandle stream);
void zero(float* output, std::size_t elements, StreamHandle stream);
} // namespace hypermoe::backend::cuda::kernels
#endif

namespace hypermoe::backend::cuda::kernels {
namespace {

enum Op { kActivation, kMatmul, kCooperative, kRouterTopK, kGather, kScatter, kZero, kOps };
const char* const kOpNames[kOps] = {"activation", "int8WeightMatmul", "int8WeightMatmulCooperative",
                                    "routerTopK", "gatherRows", "scatterAddRows", "zero"};
std::atomic<long long> g_calls[kOps];

struct CallReport {
    ~CallReport() {
        if (!std::getenv("HMOE_SHIM_TRACE")) return;
        std::fprintf(stderr, "hmoe shim calls:");
        for (int i = 0; i < kOps; ++i) std::fprintf(stderr, " %s=%lld", kOpNames[i], g_calls[i].load());
        std::fprintf(stderr, "\n");
    }
} g_report;

void note(Op op) { g_calls[op].fetch_add(1, std::memory_order_relaxed); }

// Converts a status into the reference's exception for that failure.
void raise(hmoe_status status, const char* operation) {
    if (status == HMOE_OK) return;
    if (status == HMOE_CUDA_ERROR) throw std::runtime_error(hmoe_last_error());
    if (status == HMOE_INVALID_ARGUMENT) throw std::invalid_argument(std::string(operation) + ": invalid argument");
    throw std::runtime_error(std::string(operation) + ": hmoe status " + std::to_string(static_cast<int>(status)));
}

} // namespace

void activation(int type, const float* input, float* output, std::size_t elements, StreamHandle stream) {
    note(kActivation);
    raise(hmoe_activation(type, input, output, elements, stream), "CUDA activation kernel");
}

void int8WeightMatmul(const float* left, const std::int8_t* right, float* output, std::size_t rows,
                      std::size_t inner, std::size_t columns, float scale, std::int32_t zeroPoint,
                      StreamHandle stream) {
    note(kMatmul);
    raise(hmoe_int8_weight_matmul(left, right, output, rows, inner, columns, scale, zeroPoint, stream),
          "CUDA INT8 weight matmul kernel");
}

void int8WeightMatmulCooperative(const float* left, const std::int8_t* right, float* output, float* partials,
                                 std::size_t rows, std::size_t inner, std::size_t columns,
                                 std::size_t partitions, float scale, std::int32_t zeroPoint,
                                 StreamHandle stream) {
    note(kCooperative);
    const hmoe_status st = hmoe_int8_weight_matmul_cooperative(left, right, output, partials, rows, inner, columns,
                                                               partitions, scale, zeroPoint, stream);
    if (st == HMOE_INVALID_ARGUMENT)
        throw std::invalid_argument("cooperative INT8 GEMM scratch/partition mismatch");
    raise(st, "CUDA cooperative INT8 weight matmul kernel");
}

void routerTopK(float* logits, std::size_t tokens, std::size_t experts, std::size_t topK, bool softmax,
                bool renormalize, std::uint32_t* selectedIds, float* selectedScores, StreamHandle stream) {
    note(kRouterTopK);
    raise(hmoe_router_topk(logits, tokens, experts, topK, softmax ? 1 : 0, renormalize ? 1 : 0, selectedIds,
                           selectedScores, stream),
          "CUDA router top-k kernel");
}

void gatherRows(const float* input, float* output, const std::uint32_t* rows, std::size_t rowCount,
                std::size_t width, StreamHandle stream) {
    note(kGather);
    raise(hmoe_gather_rows(input, output, rows, rowCount, width, stream), "CUDA gather kernel");
}

void scatterAddRows(const float* input, float* output, const std::uint32_t* rows, const float* weights,
                    std::size_t rowCount, std::size_t width, StreamHandle stream) {
    note(kScatter);
    raise(hmoe_scatter_add_rows(input, output, rows, weights, rowCount, width, stream), "CUDA scatter kernel");
}

void zero(float* output, std::size_t elements, StreamHandle stream) {
    note(kZero);
    raise(hmoe_zero(output, elements, stream), "CUDA zero kernel");
}

// One definition per name: with the reference header included, a signature
// that differs from its declaration would add an overload and make these
// expressions ambiguous.
static_assert(std::is_same_v<decltype(&activation), void (*)(int, const float*, float*, std::size_t, StreamHandle)>);
static_assert(std::is_same_v<decltype(&int8WeightMatmul),
                             void (*)(const float*, const std::int8_t*, float*, std::size_t, std::size_t,
                                      std::size_t, float, std::int32_t, StreamHandle)>);
static_assert(std::is_same_v<decltype(&int8WeightMatmulCooperative),
                             void (*)(const float*, const std::int8_t*, float*, float*, std::size_t, std::size_t,
                                      std::size_t, std::size_t, float, std::int32_t, StreamHandle)>);
static_assert(std::is_same_v<decltype(&routerTopK), void (*)(float*, std::size_t, std::size_t, std::size_t, bool,
                                                             bool, std::uint32_t*, float*, StreamHandle)>);
static_assert(std::is_same_v<decltype(&gatherRows), void (*)(const float*, float*, const std::uint32_t*,
                                                             std::size_t, std::size_t, StreamHandle)>);
static_assert(std::is_same_v<decltype(&scatterAddRows),
                             void (*)(const float*, float*, const std::uint32_t*, const float*, std::size_t,
                                      std::size_t, StreamHandle)>);
static_assert(std::is_same_v<decltype(&zero), void (*)(float*, std::size_t, StreamHandle)>);

} // namespace hypermoe::backend::cuda::kernels
