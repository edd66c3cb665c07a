// noalloc.cu -- hmoe_moe_forward_noalloc: the fused layer forward with its
// scratch in a file-scope device array instead of a caller workspace.
//
// For callers that cannot allocate device memory at the call site (e.g. a
// host runtime whose allocator is not reachable from the layer call, or a
// decode loop that must not touch the allocator between steps).  The array
// holds up to kNoAllocScratchBytes (16 MiB): enough for decode-sized batches
// (C3 layer up to 185 tokens, C2 up to 150).  Larger batches are rejected
// with HMOE_WORKSPACE_TOO_SMALL and a message naming the limit.
//
// One array per device (the module is loaded per context), shared by every
// call on that device: calls that overlap in time -- on different streams,
// or from different host threads -- race on it.  The first call on a device
// looks the array up with cudaGetSymbolAddress; make that first call before
// any stream capture on that device.  The address is remembered for the life
// of the process, so it is not valid across cudaDeviceReset.
//
// The layer's device status word (router non-finite input, bounded-wait
// timeouts, near-tie counts) sits at the start of the array, as it sits at
// the start of a caller workspace; hmoe_noalloc_read_status reads it.
#include "common.cuh"

#include <mutex>
#include <string>

namespace hmoe {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of this device's scratch array (looked up once per device,
// with that device current).
hmoe_status noalloc_scratch(void** out) {
    int dev = -1;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) {
        set_last_error("hmoe_moe_forward_noalloc: cudaGetDevice", err);
        return HMOE_CUDA_ERROR;
    }
    if (dev < 0 || dev >= kNoAllocMaxDevices) {
        set_last_error_text("hmoe_moe_forward_noalloc: device ordinal out of range");
        return HMOE_UNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess || !p) {
            set_last_error("hmoe_moe_forward_noalloc: cudaGetSymbolAddress", err);
            return HMOE_CUDA_ERROR;
        }
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return HMOE_OK;
}

} // namespace
} // namespace hmoe

extern "C" hmoe_status hmoe_moe_forward_noalloc(const hmoe_layer_desc* desc, const float* x, float* y,
                                                size_t tokens, void* stream) {
    using namespace hmoe;
    if (tokens == 0) return HMOE_OK;
    size_t need = 0;
    hmoe_status st = hmoe_workspace_size(desc, tokens, &need);
    if (st != HMOE_OK) return st;
    if (need > kNoAllocScratchBytes) {
        const std::string msg = "hmoe_moe_forward_noalloc: " + std::to_string(tokens) + " tokens need " +
                                std::to_string(need) + " scratch bytes; the static scratch holds " +
                                std::to_string(kNoAllocScratchBytes) + " (16 MiB)";
        set_last_error_text(msg.c_str());
        return HMOE_WORKSPACE_TOO_SMALL;
    }
    void* scratch = nullptr;
    st = noalloc_scratch(&scratch);
    if (st != HMOE_OK) return st;
    // hmoe_moe_forward clears the status word and the expert counters (the
    // parts that must start at zero) with one cudaMemsetAsync on `stream`.
    return hmoe_moe_forward(desc, x, y, tokens, scratch, kNoAllocScratchBytes, stream);
}

// The status word the last hmoe_moe_forward_noalloc on this device left in
// the static scratch (hmoe_read_status on the array).
extern "C" hmoe_status hmoe_noalloc_read_status(int32_t* status, int32_t* near_ties, int32_t* sequential_logits,
                                                void* stream) {
    using namespace hmoe;
    void* scratch = nullptr;
    const hmoe_status st = noalloc_scratch(&scratch);
    if (st != HMOE_OK) return st;
    return hmoe_read_status(scratch, status, near_ties, sequential_logits, stream);
}
