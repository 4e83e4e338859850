// Backward entry point that allocates nothing and needs no caller workspace.
//
// Some callers cannot hand the backward a workspace: plugin hosts that own
// every device allocation themselves and give a library no allocator, or FFI
// bindings that have no device allocator at all.  For them the backward's
// scratch (per-row softmax statistics, the work plan of the dK/dV pass)
// lives in one fixed-size, file-scope device array instead.  Every GPU that
// loads this library holds that array (kStaticScratchBytes) until the process
// exits.  The array's device address is looked up once per device and kept:
// a cudaDeviceReset() between calls is not supported (the library's module
// is reloaded and the kept address would be stale).
#include <mutex>

#include "common.cuh"

namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;   // 32 MiB
__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
void *g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of the array on the current device; looked up once per device.
int scratch_address(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SCOPE_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) return SCOPE_ERR_CUDA;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return SCOPE_OK;
}

}  // namespace

extern "C" size_t scope_static_scratch_bytes(void) { return kStaticScratchBytes; }

extern "C" int scope_attn_bwd_static_scratch(const ScopeAttnArgs *args, scope_stream_t stream) {
    if (!args) return SCOPE_ERR_INVALID;
    if (scope_workspace_bytes(args) > kStaticScratchBytes) return SCOPE_ERR_WORKSPACE;
    void *scratch = nullptr;
    int st = scratch_address(&scratch);
    if (st != SCOPE_OK) return st;
    ScopeAttnArgs a = *args;
    a.workspace = scratch;
    a.workspace_bytes = kStaticScratchBytes;
    return scope_attn_bwd(&a, stream);
}
