// common.cuh -- shared helpers for the sm_100a HyperMoE kernels.
#pragma once

#include "hmoe.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace hmoe {

// Device status word at the start of every layer workspace.
struct DeviceStatus {
    int32_t status;            // hmoe_status of the last failing device check
    int32_t near_ties;         // router selections within 2 ulp (see router.cu)
    int32_t sequential_logits; // logits recomputed in the CPU's sequential order
    int32_t reserved[13];
};

// Records `what: cudaGetErrorString(err)` for hmoe_last_error().
void set_last_error(const char* what, cudaError_t err);
void set_last_error_text(const char* text);

// Counts this library's kernel launches (hmoe_launch_count).
void count_launch();

// Raises `func`'s dynamic shared-memory limit to at least `bytes` on the
// current device.  Function attributes belong to a device context, so the
// setting is remembered per (kernel, device ordinal); several host threads
// may call this at once.
cudaError_t set_smem_limit(const void* func, int bytes);

// Multiprocessor count of the current device (remembered per ordinal).
int current_sm_count();

// checkLaunch (reference CudaKernels.cu:293-299) as a status.
inline hmoe_status check_launch(const char* what) {
    count_launch();
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) {
        set_last_error(what, err);
        return HMOE_CUDA_ERROR;
    }
    return HMOE_OK;
}

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Whether p (null allowed) is a multiple of `a` bytes.  Token rows, the
// workspace, the router matrix and the expert arena are read and written
// with 16-byte vector accesses and bulk/tensor copies, which fault on
// misaligned addresses, so the entry points check them on the host.
inline bool aligned(const void* p, size_t a) { return reinterpret_cast<uintptr_t>(p) % a == 0; }

constexpr unsigned kThreads = 256;

inline unsigned blocks_for(size_t n, unsigned per = kThreads) {
    return static_cast<unsigned>((n + per - 1) / per);
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Sets err->status once (first error wins).
__device__ __forceinline__ void device_fail(DeviceStatus* st, int32_t code) {
    if (st) atomicCAS(&st->status, 0, code);
}

// int8x4 (packed in a 32-bit word) minus zero point -> 4 exact floats.
// q - zp lies in [-255, 255]: exact in FP32 and in BF16.
__device__ __forceinline__ void dequant4(uint32_t w, float zp, float out[4]) {
    out[0] = static_cast<float>(static_cast<int8_t>(w & 0xff)) - zp;
    out[1] = static_cast<float>(static_cast<int8_t>((w >> 8) & 0xff)) - zp;
    out[2] = static_cast<float>(static_cast<int8_t>((w >> 16) & 0xff)) - zp;
    out[3] = static_cast<float>(static_cast<int8_t>(w >> 24)) - zp;
}

// Four INT8 weights -> q - zp, exact, without integer-to-float conversions:
// float(2^23 + (q + 128)) - off with off = 2^23 + 128 + zp.
__device__ __forceinline__ void dequant4_fast(uint32_t w, float off, float out[4]) {
    const uint32_t u = w ^ 0x80808080u;
    out[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - off;
    out[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - off;
    out[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - off;
    out[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - off;
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

} // namespace hmoe
