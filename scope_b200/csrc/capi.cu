// extern "C" attention entry points: argument validation and dispatch.
//
// bf16 inputs with 128-token blocks run on the tcgen05 tensor-core kernels: no
// bias, the qk_aug bias, and the score_mod closure when its Fourier sum comes
// with augmented dims (q_aug / k_aug); float32 inputs, and score_mod without
// them, run on the CUDA-core kernels.  Nothing here falls back silently: a
// combination neither path supports returns an error status.
#include <atomic>
#include <cmath>
#include <cstddef>
#include <cstring>

#include "common.cuh"

int scope_simt_fwd(const ScopeAttnArgs &a, cudaStream_t s);
int scope_simt_bwd(const ScopeAttnArgs &a, cudaStream_t s);
int scope_tc_fwd(const ScopeAttnArgs &a, cudaStream_t s);
int scope_tc_bwd(const ScopeAttnArgs &a, cudaStream_t s);
bool scope_tc_eligible(const ScopeAttnArgs &a, bool bwd);
size_t scope_bwd_workspace_bytes(int H, int T, int block_size, int d_aug, bool smod);

namespace {

int validate(const ScopeAttnArgs &a, bool bwd) {
    if (a.H <= 0 || a.T <= 0 || a.D != 64) return SCOPE_ERR_INVALID;
    if (a.block_size != 64 && a.block_size != 128 && a.block_size != 256) return SCOPE_ERR_INVALID;
    if (a.T % a.block_size != 0) return SCOPE_ERR_INVALID;
    if (a.dtype != SCOPE_F32 && a.dtype != SCOPE_BF16) return SCOPE_ERR_DTYPE;
    if (!a.q || !a.k || !a.v || !a.out || !a.kv_num || !a.kv_indices || a.kv_stride < 1) return SCOPE_ERR_INVALID;
    if (!(a.scale > 0.f) || !std::isfinite(a.scale)) return SCOPE_ERR_INVALID;
    switch (a.bias_mode) {
        case SCOPE_BIAS_NONE:
            if (a.d_aug != 0) return SCOPE_ERR_INVALID;
            break;
        case SCOPE_BIAS_SCORE_MOD:
            if (a.K < 1 || a.K > 16 || !a.coeff_cos || !a.coeff_sin || !a.cos_tab || !a.sin_tab) return SCOPE_ERR_INVALID;
            if (a.tab_len < a.T) return SCOPE_ERR_INVALID;
            // d_aug 0: CUDA cores; else the Fourier dims from scope_qk_aug_prepare (no slope column)
            if (a.d_aug != 0 && (!a.q_aug || !a.k_aug || a.d_aug != (2 * a.K + 15) / 16 * 16)) return SCOPE_ERR_INVALID;
            if (a.gate != SCOPE_GATE_NONE && (!a.delta_main || !a.width || !(a.gate_tau != 0.f))) return SCOPE_ERR_INVALID;
            if (a.gate < 0 || a.gate > 2) return SCOPE_ERR_INVALID;
            break;
        case SCOPE_BIAS_QK_AUG:
            if (!a.q_aug || !a.k_aug || a.d_aug < 16 || a.d_aug > 64 || a.d_aug % 16) return SCOPE_ERR_INVALID;
            if (bwd && (a.dcoeff_cos || a.dcoeff_sin) && (a.K < 1 || !a.cos_tab || !a.sin_tab || a.tab_len < a.T ||
                                                          2 * a.K + (a.slope ? 1 : 0) > a.d_aug))
                return SCOPE_ERR_INVALID;
            break;
        default:
            return SCOPE_ERR_INVALID;
    }
    if (bwd) {
        if (!a.dout || !a.dq || !a.dk || !a.dv || !a.lse || !a.q_bitmap) return SCOPE_ERR_INVALID;
        if (!a.workspace || a.workspace_bytes < scope_workspace_bytes(&a)) return SCOPE_ERR_WORKSPACE;
        if (reinterpret_cast<uintptr_t>(a.workspace) & 255) return SCOPE_ERR_ALIGN;
    }
    return SCOPE_OK;
}

}  // namespace

extern "C" size_t scope_workspace_bytes(const ScopeAttnArgs *a) {
    if (!a || a->H <= 0 || a->T <= 0 || a->block_size <= 0 || a->T % a->block_size) return 0;
    // delta_i = rowsum(dO * O), lse_i * log2(e) (float32 [H, T] each), the dK/dV work plan and
    // the fp32 dQ accumulator of the tensor-core backward
    const bool aug = a->bias_mode == SCOPE_BIAS_QK_AUG || (a->bias_mode == SCOPE_BIAS_SCORE_MOD && a->d_aug > 0);
    return scope_bwd_workspace_bytes(a->H, a->T, a->block_size, aug ? a->d_aug : 0,
                                     a->bias_mode == SCOPE_BIAS_SCORE_MOD && a->d_aug > 0);
}

extern "C" int scope_attn_fwd(const ScopeAttnArgs *args, scope_stream_t stream) {
    if (!args) return SCOPE_ERR_INVALID;
    int st = validate(*args, false);
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (!(args->flags & SCOPE_FLAG_CUDA_CORES) && scope_tc_eligible(*args, false)) return scope_tc_fwd(*args, s);
    if (args->block_size > 128) return SCOPE_ERR_UNSUPPORTED;
    return scope_simt_fwd(*args, s);
}

extern "C" int scope_attn_bwd(const ScopeAttnArgs *args, scope_stream_t stream) {
    if (!args) return SCOPE_ERR_INVALID;
    int st = validate(*args, true);
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (!(args->flags & SCOPE_FLAG_CUDA_CORES) && scope_tc_eligible(*args, true)) return scope_tc_bwd(*args, s);
    if (args->block_size > 128) return SCOPE_ERR_UNSUPPORTED;
    return scope_simt_bwd(*args, s);
}

extern "C" const char *scope_error_string(int status) {
    switch (status) {
        case SCOPE_OK: return "ok";
        case SCOPE_ERR_INVALID: return "invalid argument";
        case SCOPE_ERR_DTYPE: return "unsupported dtype";
        case SCOPE_ERR_ALIGN: return "misaligned pointer or stride";
        case SCOPE_ERR_CUDA: return "CUDA error";
        case SCOPE_ERR_UNSUPPORTED: return "unsupported device or configuration";
        case SCOPE_ERR_WORKSPACE: return "workspace missing or too small";
        default: return "unknown status";
    }
}

extern "C" size_t scope_abi_layout(int which, int what) {
    // which: 0 ScopeMaskArgs, 1 ScopeAttnArgs, 2 ScopeCoeffArgs, 3 ScopeCoeffBwdArgs, 4 ScopeCoeffMlpBwdArgs;
    // what: 0 sizeof, 1 offset of the last field
    if (which == 0) return what == 0 ? sizeof(ScopeMaskArgs) : offsetof(ScopeMaskArgs, err_flag);
    if (which == 1) return what == 0 ? sizeof(ScopeAttnArgs) : offsetof(ScopeAttnArgs, err_flag);
    if (which == 2) return what == 0 ? sizeof(ScopeCoeffArgs) : offsetof(ScopeCoeffArgs, err_flag);
    if (which == 3) return what == 0 ? sizeof(ScopeCoeffBwdArgs) : offsetof(ScopeCoeffBwdArgs, err_flag);
    if (which == 4) return what == 0 ? sizeof(ScopeCoeffMlpBwdArgs) : offsetof(ScopeCoeffMlpBwdArgs, err_flag);
    return 0;
}

static std::atomic<uint64_t> g_launches{0};
void scope_note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
extern "C" uint64_t scope_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int scope_device_supported(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    return (major == 10 && minor == 0) ? 1 : 0;
}
