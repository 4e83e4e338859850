// Shared helpers of the scope_b200 kernels: status codes, launch checks,
// bf16 conversion and the bounded waits every pipelined kernel uses.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "scope_b200.h"

void scope_note_launch();

// after every kernel launch: count it, and map a launch failure to a status
#define SCOPE_CHECK_LAUNCH()                                  \
    do {                                                      \
        scope_note_launch();                                  \
        cudaError_t e__ = cudaGetLastError();                 \
        if (e__ != cudaSuccess) return SCOPE_ERR_CUDA;        \
    } while (0)

namespace scope {

__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
    return __uint_as_float(uint32_t(b) << 16);
}

__device__ __forceinline__ void set_err(int32_t *flag, int bits) {
    if (flag) atomicOr(flag, bits);
}

template <typename T> struct Elem;
template <> struct Elem<float> {
    __device__ __forceinline__ static float load(const float *p) { return *p; }
    __device__ __forceinline__ static void store(float *p, float v) { *p = v; }
};
template <> struct Elem<__nv_bfloat16> {
    __device__ __forceinline__ static float load(const __nv_bfloat16 *p) { return __bfloat162float(*p); }
    __device__ __forceinline__ static void store(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }
};

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Upper bound on the wall time of any wait on an mbarrier or flag.  A wait
// that reaches it records SCOPE_DEVERR_TIMEOUT and the kernel winds down
// instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // 2 s

}  // namespace scope
