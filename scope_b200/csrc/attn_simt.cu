// Block-sparse attention on CUDA cores: the float32 path and the exact
// score_mod path.
//
// This is the kernel for what the tensor-core kernel does not cover: float32
// inputs (the reference's fp32 flex_attention, tolerance 1e-4) and the full
// score_mod closure of scoped_medium.py:425-457 with its exact bf16 table
// lookups, b0, slope and softplus/relu gate, including the gradients flex
// computes for those captured tensors.  The qk_aug mode runs here too in
// float32.  One thread owns one query row (forward, dQ) or one key row
// (dK/dV); K/V (or Q/dO) tiles named by the block lists are staged in shared
// memory.  Every listed block is a partial block: the document-causal
// mask_mod of model/attn_bias.py:674-679 is applied to every element.
#include <cmath>

#include "common.cuh"

namespace scope {
namespace simt {

constexpr int kD = 64;
constexpr int kMaxK = 16;

__device__ __forceinline__ float softplus_t(float x) {   // torch softplus, beta=1, threshold=20
    return x > 20.f ? x : log1pf(expf(x));
}
__device__ __forceinline__ float softplus_grad(float x) {
    return x > 20.f ? 1.f : 1.f / (1.f + expf(-x));
}

template <typename T>
__device__ __forceinline__ float ld(const T *p) { return Elem<T>::load(p); }

// per-row parameters of the score_mod closure
struct RowBias {
    float A[kMaxK], B[kMaxK];
    float b0, slope, dm, w;
};

__device__ __forceinline__ void load_rowbias(const ScopeAttnArgs &a, int64_t hrow, RowBias &rb) {
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) {
        rb.A[k] = (k < a.K) ? a.coeff_cos[hrow * a.K + k] : 0.f;
        rb.B[k] = (k < a.K) ? a.coeff_sin[hrow * a.K + k] : 0.f;
    }
    rb.b0 = a.b0 ? a.b0[hrow] : 0.f;
    rb.slope = a.slope ? a.slope[hrow] : 0.f;
    rb.dm = (a.gate && a.delta_main) ? a.delta_main[hrow] : 0.f;
    rb.w = (a.gate && a.width) ? a.width[hrow] : 0.f;
}

// bias(i,j) of scoped_medium.py:425-457 for delta = max(i-j, 0)
__device__ __forceinline__ float eval_bias(const ScopeAttnArgs &a, const RowBias &rb, int delta) {
    float bias = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) {
        if (k < a.K) {
            float c = bf16_to_f32(__ldg(a.cos_tab + (int64_t)k * a.tab_len + delta));
            float s = bf16_to_f32(__ldg(a.sin_tab + (int64_t)k * a.tab_len + delta));
            bias = __fadd_rn(__fadd_rn(bias, __fmul_rn(rb.A[k], c)), __fmul_rn(rb.B[k], s));
        }
    }
    float df = (float)delta;
    if (a.b0) bias = bias - rb.b0;
    if (a.slope) bias = bias + rb.slope * df;
    if (a.gate != SCOPE_GATE_NONE && a.gate_lambda > 0.f) {
        float x = (fabsf(df - rb.dm) - rb.w) / a.gate_tau;
        float g = (a.gate == SCOPE_GATE_RELU) ? fmaxf(x, 0.f) : softplus_t(x);
        bias = bias - a.gate_lambda * g;
    }
    return bias;
}

template <typename T, int DA>
struct Tiles {
    static constexpr int KS = kD + DA;        // row stride of a K (or Q) tile
    static constexpr int OS = kD + DA + 1;    // padded stride of a thread-owned row
};

// --------------------------------------------------------------------------
// forward
// --------------------------------------------------------------------------
template <typename T, int DA, int MODE>
__global__ void __launch_bounds__(128) fwd_kernel(const ScopeAttnArgs a) {
    using TL = Tiles<T, DA>;
    extern __shared__ float sm[];
    const int bs = a.block_size, QB = a.T / bs;
    const int qb = blockIdx.x, h = blockIdx.y, r = threadIdx.x;
    const int i = qb * bs + r;
    float *Ks = sm;                        // [bs][KS]
    float *Vs = Ks + bs * TL::KS;          // [bs][64]
    float *Qo = Vs + bs * kD;              // [bs][OS] own rows
    int *dks = reinterpret_cast<int *>(Qo + bs * TL::OS);   // [bs]
    const T *Q = reinterpret_cast<const T *>(a.q), *Kp = reinterpret_cast<const T *>(a.k),
            *Vp = reinterpret_cast<const T *>(a.v);
    const T *QA = reinterpret_cast<const T *>(a.q_aug), *KA = reinterpret_cast<const T *>(a.k_aug);
    float *qrow = Qo + r * TL::OS;
    for (int d = 0; d < kD; ++d) qrow[d] = ld(Q + h * a.q_sh + (int64_t)i * a.q_st + d);
    if (DA) for (int e = 0; e < DA; ++e) qrow[kD + e] = ld(QA + ((int64_t)h * a.T + i) * DA + e);
    RowBias rb;
    if (MODE == SCOPE_BIAS_SCORE_MOD) load_rowbias(a, (int64_t)h * a.T + i, rb);
    const int dq = a.docs ? a.docs[i] : 0;
    float m = -INFINITY, l = 0.f, acc[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) acc[d] = 0.f;
    const int64_t mrow = (int64_t)h * QB + qb;
    const int n = a.kv_num[mrow];
    for (int jj = 0; jj < n; ++jj) {
        const int kb = a.kv_indices[mrow * a.kv_stride + jj];
        if (kb < 0 || kb >= QB) {
            if (r == 0) set_err(a.err_flag, SCOPE_DEVERR_INDEX);
            continue;
        }
        __syncthreads();
        for (int e = r; e < bs * kD; e += blockDim.x) {
            int c = e / kD, d = e - c * kD;
            int64_t t = (int64_t)kb * bs + c;
            Ks[c * TL::KS + d] = ld(Kp + h * a.k_sh + t * a.k_st + d);
            Vs[c * kD + d] = ld(Vp + h * a.v_sh + t * a.v_st + d);
        }
        if (DA)
            for (int e = r; e < bs * DA; e += blockDim.x) {
                int c = e / DA, d = e - c * DA;
                Ks[c * TL::KS + kD + d] = ld(KA + ((int64_t)kb * bs + c) * DA + d);
            }
        for (int c = r; c < bs; c += blockDim.x) dks[c] = a.docs ? a.docs[kb * bs + c] : 0;
        __syncthreads();
        for (int c0 = 0; c0 < bs; c0 += 16) {
            float s[16];
            float mx = -INFINITY;
#pragma unroll
            for (int cc = 0; cc < 16; ++cc) {
                const int c = c0 + cc, j = kb * bs + c;
                const float *kr = Ks + c * TL::KS;
                float dot = 0.f;
#pragma unroll 16
                for (int d = 0; d < TL::KS; ++d) dot = fmaf(qrow[d], kr[d], dot);
                float sc = dot * a.scale;
                if (MODE == SCOPE_BIAS_SCORE_MOD) sc = sc + a.beta * eval_bias(a, rb, max(i - j, 0));
                bool valid = (j <= i) && (dks[c] == dq);
                s[cc] = valid ? sc : -INFINITY;
                mx = fmaxf(mx, s[cc]);
            }
            float mn = fmaxf(m, mx);
            if (mn == -INFINITY) continue;
            float corr = expf(m - mn);
            l *= corr;
#pragma unroll
            for (int d = 0; d < kD; ++d) acc[d] *= corr;
#pragma unroll
            for (int cc = 0; cc < 16; ++cc) {
                float p = expf(s[cc] - mn);
                l += p;
                const float *vr = Vs + (c0 + cc) * kD;
#pragma unroll
                for (int d = 0; d < kD; ++d) acc[d] = fmaf(p, vr[d], acc[d]);
            }
            m = mn;
        }
    }
    T *O = reinterpret_cast<T *>(a.out);
    float inv = (l > 0.f) ? 1.f / l : 0.f;
#pragma unroll
    for (int d = 0; d < kD; ++d) Elem<T>::store(O + h * a.o_sh + (int64_t)i * a.o_st + d, acc[d] * inv);
    if (a.lse) a.lse[(int64_t)h * a.T + i] = (l > 0.f) ? m + logf(l) : -INFINITY;
}

// --------------------------------------------------------------------------
// backward: delta_i = sum_d dO_i . O_i
// --------------------------------------------------------------------------
template <typename T>
__global__ void bwd_delta_kernel(const ScopeAttnArgs a, float *__restrict__ delta) {
    int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= (int64_t)a.H * a.T) return;
    int h = (int)(row / a.T), t = (int)(row % a.T);
    const T *O = reinterpret_cast<const T *>(a.out), *dO = reinterpret_cast<const T *>(a.dout);
    float s = 0.f;
    for (int d = 0; d < kD; ++d)
        s = fmaf(ld(O + h * a.o_sh + (int64_t)t * a.o_st + d), ld(dO + h * a.do_sh + (int64_t)t * a.do_st + d), s);
    delta[row] = s;
}

// dQ (and the gradients of the per-query bias tensors), walking kv lists
template <typename T, int DA, int MODE>
__global__ void __launch_bounds__(128) bwd_dq_kernel(const ScopeAttnArgs a, const float *__restrict__ delta) {
    using TL = Tiles<T, DA>;
    extern __shared__ float sm[];
    const int bs = a.block_size, QB = a.T / bs;
    const int qb = blockIdx.x, h = blockIdx.y, r = threadIdx.x;
    const int i = qb * bs + r;
    const int64_t hrow = (int64_t)h * a.T + i;
    float *Ks = sm;                        // [bs][KS]
    float *Vs = Ks + bs * TL::KS;          // [bs][64]
    float *Qo = Vs + bs * kD;              // [bs][OS] own q rows
    float *Do = Qo + bs * TL::OS;          // [bs][65] own dO rows
    float *Ga = Do + bs * (kD + 1);        // [bs][DA+1] own dq_aug accumulators
    int *dks = reinterpret_cast<int *>(Ga + bs * (DA + 1));
    const T *Q = reinterpret_cast<const T *>(a.q), *Kp = reinterpret_cast<const T *>(a.k),
            *Vp = reinterpret_cast<const T *>(a.v), *DO = reinterpret_cast<const T *>(a.dout);
    const T *QA = reinterpret_cast<const T *>(a.q_aug), *KA = reinterpret_cast<const T *>(a.k_aug);
    float *qrow = Qo + r * TL::OS, *drow = Do + r * (kD + 1), *garow = Ga + r * (DA + 1);
    for (int d = 0; d < kD; ++d) {
        qrow[d] = ld(Q + h * a.q_sh + (int64_t)i * a.q_st + d);
        drow[d] = ld(DO + h * a.do_sh + (int64_t)i * a.do_st + d);
    }
    if (DA) for (int e = 0; e < DA; ++e) {
        qrow[kD + e] = ld(QA + hrow * DA + e);
        garow[e] = 0.f;
    }
    RowBias rb;
    if (MODE == SCOPE_BIAS_SCORE_MOD) load_rowbias(a, hrow, rb);
    float gA[kMaxK], gB[kMaxK], gb0 = 0.f, gsl = 0.f, gdm = 0.f, gw = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) gA[k] = gB[k] = 0.f;
    const int dq = a.docs ? a.docs[i] : 0;
    const float lse = a.lse[hrow], dlt = delta[hrow];
    float acc[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) acc[d] = 0.f;
    const int64_t mrow = (int64_t)h * QB + qb;
    const int n = a.kv_num[mrow];
    for (int jj = 0; jj < n; ++jj) {
        const int kb = a.kv_indices[mrow * a.kv_stride + jj];
        if (kb < 0 || kb >= QB) continue;
        __syncthreads();
        for (int e = r; e < bs * kD; e += blockDim.x) {
            int c = e / kD, d = e - c * kD;
            int64_t t = (int64_t)kb * bs + c;
            Ks[c * TL::KS + d] = ld(Kp + h * a.k_sh + t * a.k_st + d);
            Vs[c * kD + d] = ld(Vp + h * a.v_sh + t * a.v_st + d);
        }
        if (DA)
            for (int e = r; e < bs * DA; e += blockDim.x) {
                int c = e / DA, d = e - c * DA;
                Ks[c * TL::KS + kD + d] = ld(KA + ((int64_t)kb * bs + c) * DA + d);
            }
        for (int c = r; c < bs; c += blockDim.x) dks[c] = a.docs ? a.docs[kb * bs + c] : 0;
        __syncthreads();
        for (int c = 0; c < bs; ++c) {
            const int j = kb * bs + c;
            const bool valid = (j <= i) && (dks[c] == dq) && (lse != -INFINITY);
            if (!valid) continue;
            const float *kr = Ks + c * TL::KS;
            float dot = 0.f;
#pragma unroll 16
            for (int d = 0; d < TL::KS; ++d) dot = fmaf(qrow[d], kr[d], dot);
            float sc = dot * a.scale;
            const int dl = max(i - j, 0);
            if (MODE == SCOPE_BIAS_SCORE_MOD) sc = sc + a.beta * eval_bias(a, rb, dl);
            const float p = expf(sc - lse);
            const float *vr = Vs + c * kD;
            float dp = 0.f;
#pragma unroll 16
            for (int d = 0; d < kD; ++d) dp = fmaf(drow[d], vr[d], dp);
            const float ds = p * (dp - dlt);
#pragma unroll
            for (int d = 0; d < kD; ++d) acc[d] = fmaf(ds, kr[d], acc[d]);
            if (DA) for (int e = 0; e < DA; ++e) garow[e] = fmaf(ds, kr[kD + e], garow[e]);
            if (MODE == SCOPE_BIAS_SCORE_MOD) {
#pragma unroll
                for (int k = 0; k < kMaxK; ++k) {
                    if (k < a.K) {
                        gA[k] = fmaf(ds, bf16_to_f32(__ldg(a.cos_tab + (int64_t)k * a.tab_len + dl)), gA[k]);
                        gB[k] = fmaf(ds, bf16_to_f32(__ldg(a.sin_tab + (int64_t)k * a.tab_len + dl)), gB[k]);
                    }
                }
                const float df = (float)dl;
                gb0 -= ds;
                gsl = fmaf(ds, df, gsl);
                if (a.gate != SCOPE_GATE_NONE && a.gate_lambda > 0.f) {
                    float x = (fabsf(df - rb.dm) - rb.w) / a.gate_tau;
                    float gp = (a.gate == SCOPE_GATE_RELU) ? (x > 0.f ? 1.f : 0.f) : softplus_grad(x);
                    float sg = (df > rb.dm) ? 1.f : ((df < rb.dm) ? -1.f : 0.f);
                    gdm = fmaf(ds, a.gate_lambda * gp * sg / a.gate_tau, gdm);
                    gw = fmaf(ds, a.gate_lambda * gp / a.gate_tau, gw);
                }
            }
        }
    }
    T *DQ = reinterpret_cast<T *>(a.dq);
#pragma unroll
    for (int d = 0; d < kD; ++d) Elem<T>::store(DQ + h * a.dq_sh + (int64_t)i * a.dq_st + d, acc[d] * a.scale);
    if (MODE == SCOPE_BIAS_SCORE_MOD) {
        const float bt = a.beta;
        for (int k = 0; k < a.K; ++k) {
            if (a.dcoeff_cos) a.dcoeff_cos[hrow * a.K + k] = bt * gA[k];
            if (a.dcoeff_sin) a.dcoeff_sin[hrow * a.K + k] = bt * gB[k];
        }
        if (a.db0) a.db0[hrow] = bt * gb0;
        if (a.dslope) a.dslope[hrow] = bt * gsl;
        if (a.ddelta_main) a.ddelta_main[hrow] = bt * gdm;
        if (a.dwidth) a.dwidth[hrow] = bt * gw;
    }
    if (MODE == SCOPE_BIAS_QK_AUG && DA) {
        // q_aug = s*[A c + B s', A s' - B c, -slope]  ->  chain rule to the coefficients
        const float sa = (float)sqrt((double)a.beta / (double)a.scale);
        for (int k = 0; k < a.K; ++k) {
            float c = bf16_to_f32(a.cos_tab[(int64_t)k * a.tab_len + i]);
            float sn = bf16_to_f32(a.sin_tab[(int64_t)k * a.tab_len + i]);
            float g0 = garow[k] * a.scale, g1 = garow[a.K + k] * a.scale;
            if (a.dcoeff_cos) a.dcoeff_cos[hrow * a.K + k] = sa * (g0 * c + g1 * sn);
            if (a.dcoeff_sin) a.dcoeff_sin[hrow * a.K + k] = sa * (g0 * sn - g1 * c);
        }
        if (a.slope && a.dslope) a.dslope[hrow] = -sa * garow[2 * a.K] * a.scale;
    }
}

// dK, dV walking the q-side bitmap (q blocks ascending)
template <typename T, int DA, int MODE>
__global__ void __launch_bounds__(128) bwd_dkv_kernel(const ScopeAttnArgs a, const float *__restrict__ delta) {
    using TL = Tiles<T, DA>;
    extern __shared__ float sm[];
    const int bs = a.block_size, QB = a.T / bs, words = (QB + 31) / 32;
    const int kb = blockIdx.x, h = blockIdx.y, c = threadIdx.x;
    const int j = kb * bs + c;
    float *Qs = sm;                            // [bs][KS] q tile
    float *Ds = Qs + bs * TL::KS;              // [bs][64] dO tile
    float *Ko = Ds + bs * kD;                  // [bs][OS] own k rows
    float *Vo = Ko + bs * TL::OS;              // [bs][65] own v rows
    float *Rb = Vo + bs * (kD + 1);            // [bs][2K+4] tile row bias params (score_mod)
    const int RBS = (MODE == SCOPE_BIAS_SCORE_MOD) ? 2 * a.K + 4 : 0;
    float *Ls = Rb + bs * RBS;                 // [bs] lse
    float *Dl = Ls + bs;                       // [bs] delta
    int *dqs = reinterpret_cast<int *>(Dl + bs);   // [bs] docs of the q tile
    const T *Q = reinterpret_cast<const T *>(a.q), *Kp = reinterpret_cast<const T *>(a.k),
            *Vp = reinterpret_cast<const T *>(a.v), *DO = reinterpret_cast<const T *>(a.dout);
    const T *QA = reinterpret_cast<const T *>(a.q_aug), *KA = reinterpret_cast<const T *>(a.k_aug);
    float *krow = Ko + c * TL::OS, *vrow = Vo + c * (kD + 1);
    for (int d = 0; d < kD; ++d) {
        krow[d] = ld(Kp + h * a.k_sh + (int64_t)j * a.k_st + d);
        vrow[d] = ld(Vp + h * a.v_sh + (int64_t)j * a.v_st + d);
    }
    if (DA) for (int e = 0; e < DA; ++e) krow[kD + e] = ld(KA + (int64_t)j * DA + e);
    const int dk_doc = a.docs ? a.docs[j] : 0;
    float gk[kD], gv[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) gk[d] = gv[d] = 0.f;
    const uint32_t *brow = a.q_bitmap + ((int64_t)h * QB + kb) * words;
    for (int w = 0; w < words; ++w) {
        uint32_t bits = brow[w];
        while (bits) {
            const int b = __ffs(bits) - 1;
            bits &= bits - 1;
            const int qb = w * 32 + b;
            __syncthreads();
            for (int e = c; e < bs * kD; e += blockDim.x) {
                int rr = e / kD, d = e - rr * kD;
                int64_t t = (int64_t)qb * bs + rr;
                Qs[rr * TL::KS + d] = ld(Q + h * a.q_sh + t * a.q_st + d);
                Ds[rr * kD + d] = ld(DO + h * a.do_sh + t * a.do_st + d);
            }
            if (DA)
                for (int e = c; e < bs * DA; e += blockDim.x) {
                    int rr = e / DA, d = e - rr * DA;
                    Qs[rr * TL::KS + kD + d] = ld(QA + ((int64_t)h * a.T + (int64_t)qb * bs + rr) * DA + d);
                }
            for (int rr = c; rr < bs; rr += blockDim.x) {
                int64_t hr = (int64_t)h * a.T + (int64_t)qb * bs + rr;
                Ls[rr] = a.lse[hr];
                Dl[rr] = delta[hr];
                dqs[rr] = a.docs ? a.docs[qb * bs + rr] : 0;
                if (MODE == SCOPE_BIAS_SCORE_MOD) {
                    float *p = Rb + rr * RBS;
                    for (int k = 0; k < a.K; ++k) {
                        p[k] = a.coeff_cos[hr * a.K + k];
                        p[a.K + k] = a.coeff_sin[hr * a.K + k];
                    }
                    p[2 * a.K] = a.b0 ? a.b0[hr] : 0.f;
                    p[2 * a.K + 1] = a.slope ? a.slope[hr] : 0.f;
                    p[2 * a.K + 2] = (a.gate && a.delta_main) ? a.delta_main[hr] : 0.f;
                    p[2 * a.K + 3] = (a.gate && a.width) ? a.width[hr] : 0.f;
                }
            }
            __syncthreads();
            for (int rr = 0; rr < bs; ++rr) {
                const int i = qb * bs + rr;
                if (!(j <= i && dqs[rr] == dk_doc && Ls[rr] != -INFINITY)) continue;
                const float *qr = Qs + rr * TL::KS;
                float dot = 0.f;
#pragma unroll 16
                for (int d = 0; d < TL::KS; ++d) dot = fmaf(qr[d], krow[d], dot);
                float sc = dot * a.scale;
                if (MODE == SCOPE_BIAS_SCORE_MOD) {
                    RowBias rb;
                    const float *p = Rb + rr * RBS;
#pragma unroll
                    for (int k = 0; k < kMaxK; ++k) {
                        rb.A[k] = (k < a.K) ? p[k] : 0.f;
                        rb.B[k] = (k < a.K) ? p[a.K + k] : 0.f;
                    }
                    rb.b0 = p[2 * a.K];
                    rb.slope = p[2 * a.K + 1];
                    rb.dm = p[2 * a.K + 2];
                    rb.w = p[2 * a.K + 3];
                    sc = sc + a.beta * eval_bias(a, rb, max(i - j, 0));
                }
                const float pr = expf(sc - Ls[rr]);
                const float *dr = Ds + rr * kD;
                float dp = 0.f;
#pragma unroll 16
                for (int d = 0; d < kD; ++d) dp = fmaf(dr[d], vrow[d], dp);
                const float ds = pr * (dp - Dl[rr]);
#pragma unroll
                for (int d = 0; d < kD; ++d) {
                    gv[d] = fmaf(pr, dr[d], gv[d]);
                    gk[d] = fmaf(ds, qr[d], gk[d]);
                }
            }
        }
    }
    T *DK = reinterpret_cast<T *>(a.dk), *DV = reinterpret_cast<T *>(a.dv);
#pragma unroll
    for (int d = 0; d < kD; ++d) {
        Elem<T>::store(DK + h * a.dk_sh + (int64_t)j * a.dk_st + d, gk[d] * a.scale);
        Elem<T>::store(DV + h * a.dv_sh + (int64_t)j * a.dv_st + d, gv[d]);
    }
}

template <typename T, int DA, int MODE>
size_t fwd_smem(int bs) { return sizeof(float) * ((size_t)bs * (Tiles<T, DA>::KS + kD + Tiles<T, DA>::OS) + bs); }
template <typename T, int DA, int MODE>
size_t dq_smem(int bs) {
    return sizeof(float) * ((size_t)bs * (Tiles<T, DA>::KS + kD + Tiles<T, DA>::OS + (kD + 1) + (DA + 1)) + bs);
}
template <typename T, int DA, int MODE>
size_t dkv_smem(int bs, int K) {
    int rbs = (MODE == SCOPE_BIAS_SCORE_MOD) ? 2 * K + 4 : 0;
    return sizeof(float) * ((size_t)bs * (Tiles<T, DA>::KS + kD + Tiles<T, DA>::OS + (kD + 1) + rbs + 3));
}

template <typename K>
static int set_smem(K kern, size_t bytes) {
    if (bytes > 227 * 1024) return SCOPE_ERR_INVALID;
    if (bytes > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
        return SCOPE_ERR_CUDA;
    return SCOPE_OK;
}

template <typename T, int DA, int MODE>
int run_fwd(const ScopeAttnArgs &a, cudaStream_t s) {
    size_t sm = fwd_smem<T, DA, MODE>(a.block_size);
    int st = set_smem(fwd_kernel<T, DA, MODE>, sm);
    if (st) return st;
    dim3 grid(a.T / a.block_size, a.H);
    fwd_kernel<T, DA, MODE><<<grid, a.block_size, sm, s>>>(a);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

template <typename T, int DA, int MODE>
int run_bwd(const ScopeAttnArgs &a, cudaStream_t s) {
    float *delta = reinterpret_cast<float *>(a.workspace);
    int64_t rows = (int64_t)a.H * a.T;
    bwd_delta_kernel<T><<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(a, delta);
    SCOPE_CHECK_LAUNCH();
    dim3 grid(a.T / a.block_size, a.H);
    size_t sm = dq_smem<T, DA, MODE>(a.block_size);
    int st = set_smem(bwd_dq_kernel<T, DA, MODE>, sm);
    if (st) return st;
    bwd_dq_kernel<T, DA, MODE><<<grid, a.block_size, sm, s>>>(a, delta);
    SCOPE_CHECK_LAUNCH();
    sm = dkv_smem<T, DA, MODE>(a.block_size, a.K);
    st = set_smem(bwd_dkv_kernel<T, DA, MODE>, sm);
    if (st) return st;
    bwd_dkv_kernel<T, DA, MODE><<<grid, a.block_size, sm, s>>>(a, delta);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

template <typename T, int MODE>
int dispatch_da(const ScopeAttnArgs &a, cudaStream_t s, bool bwd) {
    switch (a.d_aug) {
        case 0: return bwd ? run_bwd<T, 0, MODE>(a, s) : run_fwd<T, 0, MODE>(a, s);
        case 16: return bwd ? run_bwd<T, 16, MODE>(a, s) : run_fwd<T, 16, MODE>(a, s);
        case 32: return bwd ? run_bwd<T, 32, MODE>(a, s) : run_fwd<T, 32, MODE>(a, s);
        case 48: return bwd ? run_bwd<T, 48, MODE>(a, s) : run_fwd<T, 48, MODE>(a, s);
        case 64: return bwd ? run_bwd<T, 64, MODE>(a, s) : run_fwd<T, 64, MODE>(a, s);
        default: return SCOPE_ERR_INVALID;
    }
}

template <typename T>
int dispatch_mode(const ScopeAttnArgs &a, cudaStream_t s, bool bwd) {
    switch (a.bias_mode) {
        case SCOPE_BIAS_NONE:
            if (a.d_aug) return SCOPE_ERR_INVALID;
            return bwd ? run_bwd<T, 0, SCOPE_BIAS_NONE>(a, s) : run_fwd<T, 0, SCOPE_BIAS_NONE>(a, s);
        case SCOPE_BIAS_SCORE_MOD:
            if (a.d_aug) return SCOPE_ERR_INVALID;
            return bwd ? run_bwd<T, 0, SCOPE_BIAS_SCORE_MOD>(a, s) : run_fwd<T, 0, SCOPE_BIAS_SCORE_MOD>(a, s);
        case SCOPE_BIAS_QK_AUG: return dispatch_da<T, SCOPE_BIAS_QK_AUG>(a, s, bwd);
        default: return SCOPE_ERR_INVALID;
    }
}

}  // namespace simt
}  // namespace scope

// entry points used by capi.cu
int scope_simt_fwd(const ScopeAttnArgs &a, cudaStream_t s) {
    using namespace scope::simt;
    return a.dtype == SCOPE_F32 ? dispatch_mode<float>(a, s, false) : dispatch_mode<__nv_bfloat16>(a, s, false);
}
int scope_simt_bwd(const ScopeAttnArgs &a, cudaStream_t s) {
    using namespace scope::simt;
    return a.dtype == SCOPE_F32 ? dispatch_mode<float>(a, s, true) : dispatch_mode<__nv_bfloat16>(a, s, true);
}
