// ops.cu -- per-operator drop-ins for hypermoe::backend::cuda::kernels::*
// (reference src/backend/cuda/CudaKernels.hpp:10-46) and planInt8Gemm
// (src/backend/cuda/Int8GemmPlan.cpp:29-53).  FP32 arithmetic, results
// within the reference's own CUDA-vs-CPU tolerance (1e-5 + 1e-5*|ref|).
#include "common.cuh"

#include <cooperative_groups.h>

#include <atomic>
#include <climits>
#include <cstring>
#include <limits>
#include <map>
#include <mutex>
#include <string>
#include <utility>

namespace cg = cooperative_groups;

namespace hmoe {

namespace {
thread_local std::string g_last_error;
std::atomic<long long> g_launches{0};
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

namespace {
std::mutex g_attr_mutex;
std::map<std::pair<const void*, int>, int> g_smem_limit; // (kernel, device) -> bytes set
std::map<int, int> g_sm_count;                           // device -> multiprocessors
}

cudaError_t set_smem_limit(const void* func, int bytes) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    int& have = g_smem_limit[{func, dev}];
    if (bytes <= have) return cudaSuccess;
    err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (err == cudaSuccess) have = bytes;
    return err;
}

int current_sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    int& n = g_sm_count[dev];
    if (n <= 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            return 148;
        }
    }
    return n;
}

void set_last_error(const char* what, cudaError_t err) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(err);
}

void set_last_error_text(const char* text) { g_last_error = text; }

// ------------------------------------------------------------ activation

__global__ void activation_kernel(int type, const float* __restrict__ in,
                                  float* __restrict__ out, size_t n) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = in[i];
    if (type == 0) {
        out[i] = v / (1.0f + expf(-v));
    } else {
        out[i] = 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
    }
}

// -------------------------------------------- INT8-weight matmul (general)
//
// Any shape (the reference's tests use N = 7, 31, 33, 65, 67, ...), so the
// weight loads are bytes: a warp reads 32 consecutive columns of a row.  A
// cluster of KS CTAs splits K; partial tiles meet in distributed shared
// memory and are summed in rank order (deterministic, no scratch).
constexpr int kMmCols = 128;
constexpr int kMmRows = 4;

// ldl: row stride of `left` (K, or the full K when this launch is one pass
// of a longer K); accumulate: add to `out` instead of overwriting it.
__global__ void __launch_bounds__(kMmCols) int8_matmul_kernel(
    const float* __restrict__ left, const int8_t* __restrict__ right,
    float* __restrict__ out, int rows, int K, int N, float scale, int zp, int KS, int ldl, int accumulate) {
    extern __shared__ __align__(16) float msm[];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int KP = (K + KS - 1) / KS;
    const int kb = min(K, rank * KP), ke = min(K, kb + KP), kc = ke - kb;
    const int r0 = blockIdx.z * kMmRows;
    const int nr = min(kMmRows, rows - r0);
    const int col = blockIdx.y * kMmCols + threadIdx.x;
    float* xs = msm;                     // [kMmRows][KP]
    float* part = msm + kMmRows * KP;    // [kMmRows][kMmCols]
    for (int i = threadIdx.x; i < kMmRows * kc; i += blockDim.x) {
        const int r = i / kc, kk = i % kc;
        xs[r * KP + kk] = r < nr ? left[static_cast<size_t>(r0 + r) * ldl + kb + kk] : 0.0f;
    }
    __syncthreads();
    float acc[kMmRows] = {0.0f, 0.0f, 0.0f, 0.0f};
    const float fzp = static_cast<float>(zp);
    if (col < N) {
        const int8_t* wp = right + static_cast<size_t>(kb) * N + col;
#pragma unroll 4
        for (int kk = 0; kk < kc; ++kk) {
            const float w = static_cast<float>(wp[static_cast<size_t>(kk) * N]) - fzp;
#pragma unroll
            for (int r = 0; r < kMmRows; ++r) acc[r] = fmaf(xs[r * KP + kk], w, acc[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < kMmRows; ++r) part[r * kMmCols + threadIdx.x] = acc[r];
    cluster.sync();
    const int slice = kMmCols / KS;
    for (int i = threadIdx.x; i < kMmRows * slice; i += blockDim.x) {
        const int r = i / slice, cl = rank * slice + i % slice;
        const int c = blockIdx.y * kMmCols + cl;
        if (r >= nr || c >= N) continue;
        float s = 0.0f;
        for (int q = 0; q < KS; ++q) s += cluster.map_shared_rank(part, q)[r * kMmCols + cl];
        const size_t o = static_cast<size_t>(r0 + r) * N + c;
        out[o] = accumulate ? out[o] + scale * s : scale * s;
    }
    cluster.sync();
}

hmoe_status launch_int8_matmul(const float* left, const int8_t* right, float* out,
                               size_t rows, size_t K, size_t N, float scale, int32_t zp,
                               cudaStream_t stream) {
    if (rows == 0 || K == 0 || N == 0) return HMOE_INVALID_ARGUMENT;
    if (!left || !right || !out) return HMOE_INVALID_ARGUMENT;
    if (!(scale > 0.0f) || !(scale < std::numeric_limits<float>::infinity()) || zp < -128 || zp > 127)
        return HMOE_INVALID_ARGUMENT; // validateParameters, Quantization.cpp:24-40
    if (rows > INT_MAX || K > INT_MAX || N > INT_MAX) return HMOE_UNSUPPORTED;
    const size_t col_blocks = (N + kMmCols - 1) / kMmCols;
    if (col_blocks > 65535) return HMOE_UNSUPPORTED;
    // Rows beyond one grid's z extent go in further launches.
    constexpr size_t kRowsPerLaunch = static_cast<size_t>(65535) * kMmRows;
    const size_t row_blocks_all = (rows + kMmRows - 1) / kMmRows;
    const size_t row_blocks = std::min<size_t>(row_blocks_all, 65535);
    int KS = 1;
    while (KS < 8 && col_blocks * row_blocks * KS < 296 && K / (KS * 2) >= 64) KS *= 2;
    // The CTA's x rows ([kMmRows][K / KS] FP32) live in shared memory: a long
    // K is split over more cluster ranks, and beyond 8 ranks into passes
    // whose partial products are added into `out` (each pass's sum is
    // deterministic; the passes add in K order).
    constexpr size_t kSmemCap = 200 * 1024;
    constexpr size_t kMaxKP = kSmemCap / sizeof(float) / kMmRows - kMmCols; // K per rank
    while (KS < 8 && (K + KS - 1) / KS > kMaxKP) KS *= 2;
    const size_t k_pass = static_cast<size_t>(KS) * kMaxKP;
    for (size_t r0 = 0; r0 < rows; r0 += kRowsPerLaunch) {
        const size_t nrows = std::min(kRowsPerLaunch, rows - r0);
        for (size_t k0 = 0; k0 < K; k0 += k_pass) {
            const size_t kc = std::min(k_pass, K - k0);
            const int KP = static_cast<int>((kc + KS - 1) / KS);
            const size_t smem = static_cast<size_t>(kMmRows * KP + kMmRows * kMmCols) * sizeof(float);
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(static_cast<unsigned>(KS), static_cast<unsigned>(col_blocks),
                               static_cast<unsigned>((nrows + kMmRows - 1) / kMmRows));
            cfg.blockDim = dim3(kMmCols);
            cfg.dynamicSmemBytes = smem;
            cfg.stream = stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = static_cast<unsigned>(KS);
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            cudaError_t err = set_smem_limit(reinterpret_cast<const void*>(int8_matmul_kernel), static_cast<int>(smem));
            if (err == cudaSuccess)
                err = cudaLaunchKernelEx(&cfg, int8_matmul_kernel, left + r0 * K + k0, right + k0 * N, out + r0 * N,
                                         static_cast<int>(nrows), static_cast<int>(kc), static_cast<int>(N), scale,
                                         static_cast<int>(zp), KS, static_cast<int>(K), k0 > 0 ? 1 : 0);
            if (err != cudaSuccess) {
                set_last_error("CUDA INT8 weight matmul kernel", err);
                return HMOE_CUDA_ERROR;
            }
            const hmoe_status st = check_launch("CUDA INT8 weight matmul kernel");
            if (st != HMOE_OK) return st;
        }
    }
    return HMOE_OK;
}

// ------------------------------------------------------- gather / scatter

__global__ void gather_rows_kernel(const float* __restrict__ in, float* __restrict__ out,
                                   const uint32_t* __restrict__ rows, size_t count, size_t width) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count * width) return;
    const size_t r = i / width, c = i % width;
    out[i] = in[static_cast<size_t>(rows[r]) * width + c];
}

__global__ void gather_rows_vec4_kernel(const float4* __restrict__ in, float4* __restrict__ out,
                                        const uint32_t* __restrict__ rows, size_t count, size_t w4) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count * w4) return;
    const size_t r = i / w4, c = i % w4;
    out[i] = in[static_cast<size_t>(rows[r]) * w4 + c];
}

__global__ void scatter_add_rows_kernel(const float* __restrict__ in, float* out,
                                        const uint32_t* __restrict__ rows,
                                        const float* __restrict__ weights, size_t count,
                                        size_t width) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count * width) return;
    const size_t r = i / width, c = i % width;
    atomicAdd(out + static_cast<size_t>(rows[r]) * width + c, in[i] * weights[r]);
}

__global__ void scatter_add_rows_vec4_kernel(const float4* __restrict__ in, float4* out,
                                             const uint32_t* __restrict__ rows,
                                             const float* __restrict__ weights, size_t count,
                                             size_t w4) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count * w4) return;
    const size_t r = i / w4, c = i % w4;
    const float wt = weights[r];
    const float4 v = in[i];
    atomicAdd(out + static_cast<size_t>(rows[r]) * w4 + c,
              make_float4(v.x * wt, v.y * wt, v.z * wt, v.w * wt));
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

} // namespace hmoe

using namespace hmoe;

extern "C" {

const char* hmoe_last_error(void) { return g_last_error.c_str(); }

int64_t hmoe_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

hmoe_status hmoe_activation(int type, const float* input, float* output, size_t elements,
                            void* stream) {
    if (elements == 0) return HMOE_OK;
    if (!input || !output || (type != 0 && type != 1)) return HMOE_INVALID_ARGUMENT;
    activation_kernel<<<blocks_for(elements), kThreads, 0, as_stream(stream)>>>(type, input, output, elements);
    return check_launch("CUDA activation kernel");
}

hmoe_status hmoe_int8_weight_matmul(const float* left, const int8_t* right, float* output,
                                    size_t rows, size_t inner, size_t columns, float scale,
                                    int32_t zero_point, void* stream) {
    return launch_int8_matmul(left, right, output, rows, inner, columns, scale, zero_point,
                              as_stream(stream));
}

hmoe_status hmoe_int8_gemm_plan(size_t rows, size_t inner, size_t columns, int32_t mode,
                                hmoe_int8_gemm_plan_t* plan) {
    if (!plan || rows == 0 || inner == 0 || columns == 0 || mode < 0 || mode > 2)
        return HMOE_INVALID_ARGUMENT;
    const auto mul_ok = [](size_t a, size_t b) { return b == 0 || a <= SIZE_MAX / b; };
    if (!mul_ok(rows, columns) || !mul_ok(rows, inner) || !mul_ok(inner, columns))
        return HMOE_INVALID_ARGUMENT; // std::overflow_error in the reference
    const auto div_up = [](size_t v, size_t d) { return v / d + static_cast<size_t>(v % d != 0); };
    const size_t elements = rows * columns;
    hmoe_int8_gemm_plan_t r{};
    r.partitions = 1;
    r.implementation = mode == HMOE_INT8_GEMM_AUTO
                           ? (inner >= 256 && columns >= 64 ? HMOE_INT8_GEMM_COOPERATIVE : HMOE_INT8_GEMM_REFERENCE)
                           : mode;
    if (r.implementation == HMOE_INT8_GEMM_REFERENCE) {
        r.blocks = div_up(elements, 256);
    } else {
        r.partitions = div_up(inner, 512) < 8 ? div_up(inner, 512) : 8;
        if (!mul_ok(rows, r.partitions) || !mul_ok(rows * r.partitions, div_up(columns, 32)))
            return HMOE_INVALID_ARGUMENT;
        r.blocks = rows * r.partitions * div_up(columns, 32);
        if (r.partitions > 1) {
            if (!mul_ok(elements, r.partitions)) return HMOE_INVALID_ARGUMENT;
            r.scratch_elements = elements * r.partitions;
        }
    }
    if (r.blocks > static_cast<size_t>(INT_MAX) || r.scratch_elements > SIZE_MAX / sizeof(float))
        return HMOE_INVALID_ARGUMENT;
    *plan = r;
    return HMOE_OK;
}

hmoe_status hmoe_int8_weight_matmul_cooperative(const float* left, const int8_t* right,
                                                float* output, float* partials, size_t rows,
                                                size_t inner, size_t columns, size_t partitions,
                                                float scale, int32_t zero_point, void* stream) {
    hmoe_int8_gemm_plan_t plan;
    const hmoe_status st = hmoe_int8_gemm_plan(rows, inner, columns, HMOE_INT8_GEMM_COOPERATIVE, &plan);
    if (st != HMOE_OK) return st;
    if (partitions != plan.partitions || (partitions > 1 && partials == nullptr))
        return HMOE_INVALID_ARGUMENT; // CudaKernels.cu:330-333
    // The split-K partials meet in distributed shared memory, so the caller's
    // scratch buffer is accepted for interface compatibility but not needed.
    return launch_int8_matmul(left, right, output, rows, inner, columns, scale, zero_point,
                              as_stream(stream));
}

hmoe_status hmoe_gather_rows(const float* input, float* output, const uint32_t* rows,
                             size_t row_count, size_t width, void* stream) {
    if (row_count == 0 || width == 0) return HMOE_OK;
    if (!input || !output || !rows) return HMOE_INVALID_ARGUMENT;
    cudaStream_t s = as_stream(stream);
    if (width % 4 == 0 && aligned16(input) && aligned16(output)) {
        const size_t n = row_count * (width / 4);
        gather_rows_vec4_kernel<<<blocks_for(n), kThreads, 0, s>>>(
            reinterpret_cast<const float4*>(input), reinterpret_cast<float4*>(output), rows, row_count, width / 4);
    } else {
        gather_rows_kernel<<<blocks_for(row_count * width), kThreads, 0, s>>>(input, output, rows, row_count, width);
    }
    return check_launch("CUDA gather kernel");
}

hmoe_status hmoe_scatter_add_rows(const float* input, float* output, const uint32_t* rows,
                                  const float* weights, size_t row_count, size_t width,
                                  void* stream) {
    if (row_count == 0 || width == 0) return HMOE_OK;
    if (!input || !output || !rows || !weights) return HMOE_INVALID_ARGUMENT;
    cudaStream_t s = as_stream(stream);
    if (width % 4 == 0 && aligned16(input) && aligned16(output)) {
        const size_t n = row_count * (width / 4);
        scatter_add_rows_vec4_kernel<<<blocks_for(n), kThreads, 0, s>>>(
            reinterpret_cast<const float4*>(input), reinterpret_cast<float4*>(output), rows, weights,
            row_count, width / 4);
    } else {
        scatter_add_rows_kernel<<<blocks_for(row_count * width), kThreads, 0, s>>>(input, output, rows, weights,
                                                                                 row_count, width);
    }
    return check_launch("CUDA scatter kernel");
}

hmoe_status hmoe_zero(float* output, size_t elements, void* stream) {
    if (elements == 0) return HMOE_OK;
    if (!output) return HMOE_INVALID_ARGUMENT;
    const cudaError_t err = cudaMemsetAsync(output, 0, elements * sizeof(float), as_stream(stream));
    if (err != cudaSuccess) {
        set_last_error("CUDA zero", err);
        return HMOE_CUDA_ERROR;
    }
    return HMOE_OK;
}

} // extern "C"
