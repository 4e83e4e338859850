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

// one thread per (h, t) row of q_aug (head 0's threads also write the k_aug
// row t); each row is assembled in registers and stored as 16-byte vectors.
// Operation order mirrors the eager reference: (A*c) + (B*s), then * s_scale.
template <typename E>
__device__ __forceinline__ void store_row(E *dst, const float *v, int n);
template <>
__device__ __forceinline__ void store_row<__nv_bfloat16>(__nv_bfloat16 *dst, const float *v, int n) {
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    for (int j = 0; j < n; j += 8) {
        __nv_bfloat162 w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = __floats2bfloat162_rn(v[j + 2 * e], v[j + 2 * e + 1]);
        d[j / 8] = *reinterpret_cast<uint4 *>(w);
    }
}
template <>
__device__ __forceinline__ void store_row<float>(float *dst, const float *v, int n) {
    float4 *d = reinterpret_cast<float4 *>(dst);
    for (int j = 0; j < n; j += 4) d[j / 4] = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
}

template <typename E, int DA>
__global__ void qk_aug_kernel(const float *__restrict__ cc, const float *__restrict__ cs,
                              const float *__restrict__ slope, const uint16_t *__restrict__ ct,
                              const uint16_t *__restrict__ st, int tab_len, int H, int T, int K, float s,
                              E *__restrict__ q_aug, E *__restrict__ k_aug) {
    const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= (int64_t)H * T) return;
    const int t = (int)(row % T);
    float v[DA], w[DA];
#pragma unroll
    for (int j = 0; j < DA; ++j) {
        float qv = 0.f, kv = 0.f;
        if (j < 2 * K) {
            const int k = j < K ? j : j - K;
            const float c = bf16_to_f32(__ldg(ct + (int64_t)k * tab_len + t));
            const float sn = bf16_to_f32(__ldg(st + (int64_t)k * tab_len + t));
            const float A = __ldg(cc + row * K + k), B = __ldg(cs + row * K + k);
            const float x = j < K ? __fadd_rn(__fmul_rn(A, c), __fmul_rn(B, sn))
                                  : __fsub_rn(__fmul_rn(A, sn), __fmul_rn(B, c));
            qv = __fmul_rn(x, s);
            kv = __fmul_rn(j < K ? c : sn, s);
        } else if (j == 2 * K && slope) {
            qv = __fmul_rn(-__ldg(slope + row), s);
            kv = __fmul_rn((float)t, s);
        }
        v[j] = qv;
        w[j] = kv;
    }
    store_row<E>(q_aug + row * DA, v, DA);
    if (row < T) store_row<E>(k_aug + (int64_t)t * DA, w, DA);   // head 0 row t: the head-independent k_aug row
}

template <typename E>
int launch_aug(const float *cc, const float *cs, const float *slope, const uint16_t *ct, const uint16_t *st,
               int tab_len, int H, int T, int K, int da, float s, void *q_aug, void *k_aug, cudaStream_t stream) {
    const int64_t rows = (int64_t)H * T;
    const unsigned grid = (unsigned)((rows + 127) / 128);
    E *qa = reinterpret_cast<E *>(q_aug), *ka = reinterpret_cast<E *>(k_aug);
    switch (da) {
        case 16: qk_aug_kernel<E, 16><<<grid, 128, 0, stream>>>(cc, cs, slope, ct, st, tab_len, H, T, K, s, qa, ka); break;
        case 32: qk_aug_kernel<E, 32><<<grid, 128, 0, stream>>>(cc, cs, slope, ct, st, tab_len, H, T, K, s, qa, ka); break;
        case 48: qk_aug_kernel<E, 48><<<grid, 128, 0, stream>>>(cc, cs, slope, ct, st, tab_len, H, T, K, s, qa, ka); break;
        case 64: qk_aug_kernel<E, 64><<<grid, 128, 0, stream>>>(cc, cs, slope, ct, st, tab_len, H, T, K, s, qa, ka); break;
        default: return SCOPE_ERR_INVALID;
    }
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
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
    if (d_aug > 64) return SCOPE_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(q_aug) | reinterpret_cast<uintptr_t>(k_aug)) & 15) return SCOPE_ERR_ALIGN;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == SCOPE_BF16)
        return spectral::launch_aug<__nv_bfloat16>(coeff_cos, coeff_sin, slope, cos_tab, sin_tab, tab_len, H, T, K,
                                                   d_aug, s, q_aug, k_aug, st);
    if (dtype == SCOPE_F32)
        return spectral::launch_aug<float>(coeff_cos, coeff_sin, slope, cos_tab, sin_tab, tab_len, H, T, K, d_aug, s,
                                           q_aug, k_aug, st);
    return SCOPE_ERR_DTYPE;
}
