// Calls the reference-signature launchers of libhmoe_shim.so on the host and
// reports which exception each failure path throws.  Only argument checks
// that fail before any CUDA call are exercised, so no GPU is needed.
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <stdexcept>

namespace hypermoe::backend::cuda::kernels {
void int8WeightMatmulCooperative(const float* left, const std::int8_t* right, float* output, float* partials,
                                 std::size_t rows, std::size_t inner, std::size_t columns,
                                 std::size_t partitions, float scale, std::int32_t zeroPoint, void* stream);
}

int main() {
    using namespace hypermoe::backend::cuda::kernels;
    float dummy = 0.0f;
    std::int8_t q = 0;
    // rows=1, inner=4096, columns=256 plans several partitions; 1 is a mismatch
    try {
        int8WeightMatmulCooperative(&dummy, &q, &dummy, &dummy, 1, 4096, 256, 1, 1.0f, 0, nullptr);
        std::puts("no exception");
    } catch (const std::invalid_argument& e) {
        std::printf("invalid_argument: %s\n", e.what());
    } catch (const std::exception& e) {
        std::printf("other: %s\n", e.what());
    }
    return 0;
}
