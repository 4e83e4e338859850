// Self-test of the failure path every pipelined kernel uses: a bounded
// mbarrier wait that gives up.  The kernel allocates TMEM as the attention
// kernels do, waits (with the same mbar_wait) on a barrier that nothing ever
// arrives on, sets SCOPE_DEVERR_TIMEOUT in the error word when the wait
// returns unsuccessful, frees TMEM and exits -- the context stays usable.
#include "common.cuh"
#include "tc_ptx.cuh"

namespace scope {
namespace selftest {

using namespace tc;

__global__ void wait_timeout_kernel(int32_t *err, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    __shared__ uint32_t tslot;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    if (threadIdx.x < 32) {
        tmem_alloc(&tslot, 32);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0 && !mbar_wait(&bar, 0, limit_ns)) set_err(err, SCOPE_DEVERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x < 32) {
        tc_fence_after();
        tmem_dealloc(tslot, 32);
    }
}

// ex2_fma2 over a vector (the FMA-pipe exponential of the attention forward),
// so a test can hold it against exp2's error bound
__global__ void exp2_fma_kernel(const float *__restrict__ x, float *__restrict__ y, int n) {
    const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (i >= n) return;
    const float x1 = (i + 1 < n) ? x[i + 1] : 0.f;
    const float2 r = f2_unpack(ex2_fma2(x[i], x1));
    y[i] = r.x;
    if (i + 1 < n) y[i + 1] = r.y;
}

}  // namespace selftest
}  // namespace scope

extern "C" int scope_selftest_wait_timeout(int32_t *err_flag, uint32_t limit_us, scope_stream_t stream) {
    if (!err_flag || limit_us == 0 || limit_us > 1000000) return SCOPE_ERR_INVALID;
    scope::selftest::wait_timeout_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        err_flag, (uint64_t)limit_us * 1000ull);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

extern "C" int scope_selftest_exp2_fma(const float *x, float *y, int32_t n, scope_stream_t stream) {
    if (!x || !y || n < 0) return SCOPE_ERR_INVALID;
    if (n == 0) return SCOPE_OK;
    const int pairs = (n + 1) / 2;
    scope::selftest::exp2_fma_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0,
                                       reinterpret_cast<cudaStream_t>(stream)>>>(x, y, n);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}
