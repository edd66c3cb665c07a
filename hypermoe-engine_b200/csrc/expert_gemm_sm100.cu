// expert_gemm_sm100.cu -- tcgen05 grouped expert GEMM (placeholder until
// the tensor-core path lands; every expert then takes the GEMV path).
#include "layer.cuh"

namespace hmoe {

bool gemm_available() { return false; }

hmoe_status launch_expert_gemm_gate_up(const hmoe_layer_desc&, const float*, size_t, char*,
                                       const Workspace&, int, cudaStream_t) {
    return HMOE_UNSUPPORTED;
}

hmoe_status launch_expert_gemm_down(const hmoe_layer_desc&, size_t, char*, const Workspace&, int,
                                    cudaStream_t) {
    return HMOE_UNSUPPORTED;
}

} // namespace hmoe
