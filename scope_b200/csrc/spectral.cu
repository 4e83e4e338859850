// Spectral-bias helpers: the bf16 trig tables and the qk_aug augmented dims.
//
// Trig tables follow SpectralBias._get_trig_tables (model/attn_bias.py:326-340):
// cos/sin of the float32 product w_k * d, rounded to bf16.  The augmented
// dims follow the qk_aug branch of CausalSelfAttention.forward
// (scoped_medium.py:380-421): the bias sum_k A_k cos(w_k (i-j)) + B_k sin(w_k (i-j))
// is rewritten with cos(a-b) = cos a cos b + sin a sin b so it rides inside
// the QK^T contraction, which on B200 is a tensor-core MMA.
#include <cmath>

#include "common.cuh"

namespace scope {
namespace spectral {

__global__ void trig_kernel(const float *__restrict__ w, int K, int L, uint16_t *__restrict__ cos_out,
                            uint16_t *__restrict__ sin_out) {
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)K * L) return;
    int k = (int)(idx / L);
    int d = (int)(idx - (int64_t)k * L);
    float ph = __fmul_rn(w[k], (float)d);
    __nv_bfloat16 c = __float2bfloat16_rn(cosf(ph));
    __nv_bfloat16 s = __float2bfloat16_rn(sinf(ph));
    cos_out[idx] = *reinterpret_cast<uint16_t *>(&c);
    sin_out[idx] = *reinterpret_cast<uint16_t *>(&s);
}

template <typename T>
__device__ __forceinline__ void store_elem(T *p, float v);
template <>
__device__ __forceinline__ void store_elem<float>(float *p, float v) { *p = v; }
template <>
__device__ __forceinline__ void store_elem<__nv_bfloat16>(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

// one thread per (h, t) row of q_aug; head 0 also writes the k_aug row.
// Operation order mirrors the eager reference: (A*c) + (B*s), then * s_scale.
template <typename E>
__global__ void qk_aug_kernel(const float *__restrict__ cc, const float *__restrict__ cs,
                              const float *__restrict__ slope, const uint16_t *__restrict__ ct,
                              const uint16_t *__restrict__ st, int tab_len, int H, int T, int K, int da,
                              float s, E *__restrict__ q_aug, E *__restrict__ k_aug) {
    int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= (int64_t)H * T) return;
    int t = (int)(row % T);
    E *qo = q_aug + row * da;
    for (int k = 0; k < K; ++k) {
        float c = bf16_to_f32(ct[(int64_t)k * tab_len + t]);
        float sn = bf16_to_f32(st[(int64_t)k * tab_len + t]);
        float A = cc[row * K + k], B = cs[row * K + k];
        float qc = __fadd_rn(__fmul_rn(A, c), __fmul_rn(B, sn));
        float qs = __fsub_rn(__fmul_rn(A, sn), __fmul_rn(B, c));
        store_elem(qo + k, __fmul_rn(qc, s));
        store_elem(qo + K + k, __fmul_rn(qs, s));
    }
    int used = 2 * K;
    if (slope) {
        store_elem(qo + used, __fmul_rn(-slope[row], s));
        ++used;
    }
    for (int j = used; j < da; ++j) store_elem(qo + j, 0.0f);
    if (row < T) {   // head 0 row t: the head-independent k_aug row
        E *ko = k_aug + (int64_t)t * da;
        for (int k = 0; k < K; ++k) {
            store_elem(ko + k, __fmul_rn(bf16_to_f32(ct[(int64_t)k * tab_len + t]), s));
            store_elem(ko + K + k, __fmul_rn(bf16_to_f32(st[(int64_t)k * tab_len + t]), s));
        }
        int u = 2 * K;
        if (slope) {
            store_elem(ko + u, __fmul_rn((float)t, s));
            ++u;
        }
        for (int j = u; j < da; ++j) store_elem(ko + j, 0.0f);
    }
}

}  // namespace spectral
}  // namespace scope

using namespace scope;

extern "C" int scope_trig_tables(const float *omegas, int32_t K, int32_t L, uint16_t *cos_out, uint16_t *sin_out,
                                 scope_stream_t stream) {
    if (!omegas || !cos_out || !sin_out || K <= 0 || L <= 0) return SCOPE_ERR_INVALID;
    int64_t n = (int64_t)K * L;
    spectral::trig_kernel<<<(unsigned)((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        omegas, K, L, cos_out, sin_out);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

extern "C" int scope_qk_aug_prepare(const float *coeff_cos, const float *coeff_sin, const float *slope,
                                    const uint16_t *cos_tab, const uint16_t *sin_tab, int32_t tab_len, int32_t H,
                                    int32_t T, int32_t K, int32_t d_aug, float beta, float scale, int32_t dtype,
                                    void *q_aug, void *k_aug, scope_stream_t stream) {
    if (!coeff_cos || !coeff_sin || !cos_tab || !sin_tab || !q_aug || !k_aug) return SCOPE_ERR_INVALID;
    if (H <= 0 || T <= 0 || K <= 0 || tab_len < T) return SCOPE_ERR_INVALID;
    int need = 2 * K + (slope ? 1 : 0);
    if (d_aug < need || d_aug % 16 != 0) return SCOPE_ERR_INVALID;
    if (!(scale > 0.f) || beta < 0.f) return SCOPE_ERR_INVALID;
    // the reference forms s = sqrt(beta/scale) in double precision and rounds it once
    float s = (float)sqrt((double)beta / (double)scale);
    int64_t rows = (int64_t)H * T;
    unsigned grid = (unsigned)((rows + 127) / 128);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == SCOPE_BF16)
        spectral::qk_aug_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(
            coeff_cos, coeff_sin, slope, cos_tab, sin_tab, tab_len, H, T, K, d_aug, s,
            reinterpret_cast<__nv_bfloat16 *>(q_aug), reinterpret_cast<__nv_bfloat16 *>(k_aug));
    else if (dtype == SCOPE_F32)
        spectral::qk_aug_kernel<float><<<grid, 128, 0, st>>>(coeff_cos, coeff_sin, slope, cos_tab, sin_tab, tab_len,
                                                              H, T, K, d_aug, s, reinterpret_cast<float *>(q_aug),
                                                              reinterpret_cast<float *>(k_aug));
    else
        return SCOPE_ERR_DTYPE;
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}
