// SpectralBias coefficient block, forward (model/attn_bias.py:306-324, 419-478):
// the per-query MLP q -> y and the mixture that turns y into the Fourier
// coefficients the attention bias consumes, fused so that none of the
// reference's [B,H,L,M,K] intermediates is materialised.
//
// One CTA of 256 threads per 128-token tile of one head (two CTAs per SM):
//   TMA      q tile [128 x 64] bf16, W1 [128 x 64], W2 [n_out x 128] (zero rows
//            up to NP = n_out rounded up to 16), 128-byte swizzled, K-major
//   tcgen05  D1 = q W1^T into TMEM columns [0, 128)
//   threads  x = bf16(D1 + b1), h = bf16(silu(x)), written back to shared memory
//            in the same swizzled K-major layout as the A operand of
//   tcgen05  D2 = h W2^T into TMEM columns [128, 128 + NP)
//   threads  y = bf16(D2 + b2) (the reference runs both linears in the dtype of
//            q, bf16; with one weight set per head its einsum rounds D to bf16
//            before the bias add, and so does this kernel), then per token: delta* = sigmoid * cap, mu, sigma, pi =
//            softmax, budget logits, slope = c tanh, the Gaussian weights a_mk
//            over log omega, and coeff_cos/sin[k] = sum_m pi_m a_mk cos/sin(w_k delta*_m),
//            b0 = sum_k coeff_cos, delta_main, width.
// Threads r and r + 128 share token row r (TMEM lane r): each forms half of
// the hidden units and the mixture over half of the pointers, and the two
// halves of the coefficient sums meet in shared memory.  The arithmetic
// follows the reference's operation order with explicit roundings (no
// contraction into FMAs where the reference rounds twice); divisions by a
// per-row or per-pointer value are multiplications by its correctly rounded
// reciprocal, cos/sin take the phase reduced to [-pi, pi] by a two-term 2*pi
// (Cody and Waite), and the SiLU (rounded to bf16 right after) and the
// Gaussian weights use the hardware exponent -- each within a few ulp of the
// reference; delta*, mu, sigma and pi keep the accurate exponent.
#include <cmath>
#include <cstring>

#include "common.cuh"
#include "tc_host.cuh"
#include "tc_ptx.cuh"

namespace scope {
namespace coeff {

using namespace tc;

constexpr int BM = 128;       // tokens per tile
constexpr int HD = 64;        // head dim (q)
constexpr int HID = 128;      // MLP hidden width: max(128, 2 * head_dim)
constexpr uint32_t kTmemCols = 256;

struct Maps {
    CUtensorMap q, w1, w2;
};

struct Params {
    int H, T, K, M, n_out, use_slope, subtract_b0, w_heads;
    const uint16_t *b1, *b2;
    const float *omegas, *log_omegas;
    float delta_cap, logw_min, logw_max, c_scale, width_min, width_max, eps;
    float *coeff_cos, *coeff_sin, *slope, *b0, *delta_star, *pi, *budget, *delta_main, *width;
    uint16_t *mlp_out;
    float *omega_reg;
    int32_t *err;
};

__host__ __device__ constexpr uint32_t align1k(uint32_t x) { return (x + 1023u) & ~1023u; }

template <int NP>
struct Layout {
    static constexpr uint32_t Q = 0, W1 = 16384, W2 = 32768;
    static constexpr uint32_t W2SUB = align1k(NP * 128);       // one 64-column half of W2
    static constexpr uint32_t HB = W2 + 2 * W2SUB;              // silu(x): two 64-column halves
    static constexpr uint32_t BAR = HB + 2 * 16384;
    static constexpr uint32_t TOTAL = BAR + 64;
    static constexpr uint32_t TX = 2 * 16384 + 2 * NP * 128;    // bytes the TMA loads deliver
};

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float sigmoid_ref(float x) { return __frcp_rn(__fadd_rn(1.f, expf(-x))); }
// cos / sin of a float32 phase: reduce by the nearest multiple of 2*pi, split
// in two float32 terms, then the hardware approximation on [-pi, pi]
__device__ __forceinline__ void sincos_phase(float ph, float *s, float *c) {
    constexpr float kTwoPiHi = 6.28318548202514648f, kTwoPiLo = -1.7484555314695172e-07f, kInvTwoPi = 0.159154943091895336f;
    const float k = rintf(__fmul_rn(ph, kInvTwoPi));
    float r = fmaf(-k, kTwoPiHi, ph);
    r = fmaf(-k, kTwoPiLo, r);
    __sincosf(r, s, c);
}

template <int K, int M, int NP>
__global__ void __launch_bounds__(256, 2) coeff_kernel(const __grid_constant__ Maps maps, const Params p) {
    using L = Layout<NP>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR);   // [0] loads, [1] MMA 1, [2] MMA 2
    uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + L::BAR + 32);

    const int warp = threadIdx.x >> 5, r = threadIdx.x & 127, half = threadIdx.x >> 7;
    const int tiles_per_head = p.T / BM;
    const int h = blockIdx.x / tiles_per_head, t0 = (blockIdx.x - h * tiles_per_head) * BM;
    const bool per_head = p.w_heads > 1;
    const int hw = per_head ? h : 0;

    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_init(&bars[2], 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tslot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t lb = (uint32_t)((warp & 3) * 32) << 16;

    if (threadIdx.x == 0) {
        mbar_expect_tx(&bars[0], L::TX);
        tma_load_3d(&maps.q, smem + L::Q, &bars[0], 0, t0, h);
        tma_load_3d(&maps.w1, smem + L::W1, &bars[0], 0, 0, hw);
        tma_load_3d(&maps.w2, smem + L::W2, &bars[0], 0, 0, hw);
        tma_load_3d(&maps.w2, smem + L::W2 + L::W2SUB, &bars[0], 64, 0, hw);
    }
    bool ok = mbar_wait(&bars[0], 0);
    const uint32_t sQ = smem_u32(smem + L::Q), sW1 = smem_u32(smem + L::W1), sW2 = smem_u32(smem + L::W2),
                   sH = smem_u32(smem + L::HB);
    if (threadIdx.x == 0 && ok) {
        tc_fence_after();
        constexpr uint32_t id1 = idesc_bf16(128, HID, false, false);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
            mma_ss(tmem, kmajor_desc(sQ + kk * 32, 128), kmajor_desc(sW1 + kk * 32, 128), id1, kk > 0);
        tc_commit(&bars[1]);
    }
    ok = __syncthreads_and(ok);
    ok = ok && mbar_wait(&bars[1], 0);
    tc_fence_after();

    // ---- x = bf16(q W1^T + b1), h = bf16(silu(x)) -> shared memory (swizzled K-major rows)
    if (ok) {
        const uint16_t *b1 = p.b1 + (size_t)hw * HID;
#pragma unroll 1
        for (int c4 = 2 * half; c4 < 2 * half + 2; ++c4) {
            uint32_t v[32];
            tmem_ld32(tmem + lb + 32 * c4, v);
            tmem_wait_ld();
            pin(v);
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
                float s2[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int j = 32 * c4 + e + u;
                    // per-head weights: the reference's einsum rounds to bf16 before its bias add
                    const float acc = per_head ? bf16r(__uint_as_float(v[e + u])) : __uint_as_float(v[e + u]);
                    const float x = bf16r(__fadd_rn(acc, bf16_to_f32(__ldg(b1 + j))));
                    // rounded to bf16 at once: the hardware exponent and divide change it
                    // only where x / (1 + e^-x) lies within ~1e-7 of a bf16 rounding boundary
                    s2[u] = bf16r(__fdividef(x, __fadd_rn(1.f, __expf(-x))));
                }
                pk[e / 2] = pack_bf16(s2[0], s2[1]);
            }
            // hidden columns [32 c4, 32 c4 + 32): half a = c4 / 2, 16-byte chunks (c4 % 2) * 4 .. + 3
            uint8_t *half = smem + L::HB + (c4 >> 1) * 16384 + r * 128;
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                const int chunk = (c4 & 1) * 4 + q4;
                *reinterpret_cast<uint4 *>(half + ((chunk ^ (r & 7)) << 4)) =
                    make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
            }
        }
    }
    // generic-proxy writes of h must be visible to the tensor core's reads
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    ok = __syncthreads_and(ok);
    if (threadIdx.x == 0 && ok) {
        tc_fence_after();
        constexpr uint32_t id2 = idesc_bf16(128, NP, false, false);
#pragma unroll
        for (int kk = 0; kk < HID / 16; ++kk) {
            const uint32_t a = (uint32_t)(kk >> 2) * 16384u + (kk & 3) * 32, b = (uint32_t)(kk >> 2) * L::W2SUB + (kk & 3) * 32;
            mma_ss(tmem + HID, kmajor_desc(sH + a, 128), kmajor_desc(sW2 + b, 128), id2, kk > 0);
        }
        tc_commit(&bars[2]);
    }
    ok = ok && mbar_wait(&bars[2], 0);
    ok = __syncthreads_and(ok);   // uniform: the exchange below synchronises all 256 threads
    tc_fence_after();

    if (ok) {
        // ---- y = bf16(h W2^T + b2)
        float y[NP];
        const uint16_t *b2 = p.b2 + (size_t)hw * p.n_out;
#pragma unroll
        for (int c = 0; c < NP; c += 16) {
            uint32_t v[16];
            tmem_ld16(tmem + lb + HID + c, v);
            tmem_wait_ld();
            pin(v);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const float acc = per_head ? bf16r(__uint_as_float(v[e])) : __uint_as_float(v[e]);
                y[c + e] = c + e < p.n_out ? bf16r(__fadd_rn(acc, bf16_to_f32(__ldg(b2 + c + e)))) : 0.f;
            }
        }
        const int64_t row = (int64_t)h * p.T + t0 + r;
        if (p.mlp_out) {
            // the tile's 128 rows of y are contiguous in global memory: staged in shared
            // memory (the q tile is idle now) and written out 16 bytes at a time
            uint16_t *sy = reinterpret_cast<uint16_t *>(smem + L::Q);
            if (!half) {
#pragma unroll
                for (int o = 0; o < NP; ++o) {
                    if (o < p.n_out) {
                        __nv_bfloat16 b = __float2bfloat16_rn(y[o]);
                        sy[r * p.n_out + o] = *reinterpret_cast<uint16_t *>(&b);
                    }
                }
            }
            asm volatile("bar.sync 1, 256;" ::: "memory");
            uint16_t *g = p.mlp_out + ((int64_t)h * p.T + t0) * p.n_out;
            const int bytes = BM * p.n_out * 2;           // a multiple of 256
            if ((reinterpret_cast<uintptr_t>(g) & 15) == 0) {
                for (int o = threadIdx.x; o < bytes / 16; o += 256)
                    reinterpret_cast<uint4 *>(g)[o] = reinterpret_cast<const uint4 *>(sy)[o];
            } else {
                for (int o = threadIdx.x; o < bytes / 2; o += 256) g[o] = sy[o];
            }
            asm volatile("bar.sync 1, 256;" ::: "memory");   // the region is reused for the exchange below
        }
        // ---- heads (model/attn_bias.py:437-478), y columns: delta | mu | sigma | pi | budget | (slope)
        float ds[M], mu[M], sg[M], pi[M];
        float musum = 0.f, pmax = -INFINITY, dmain = 0.f;   // delta* of the first largest pi logit
#pragma unroll
        for (int m = 0; m < M; ++m) {
            ds[m] = __fmul_rn(sigmoid_ref(y[m]), p.delta_cap);
            mu[m] = __fadd_rn(p.logw_min, __fmul_rn(__fsub_rn(p.logw_max, p.logw_min), sigmoid_ref(y[M + m])));
            sg[m] = __fadd_rn(0.25f, __fmul_rn(1.75f, sigmoid_ref(y[2 * M + m])));
            musum = __fadd_rn(musum, mu[m]);
            if (y[3 * M + m] > pmax) {
                pmax = y[3 * M + m];
                dmain = ds[m];
            }
        }
        float psum = 0.f;
#pragma unroll
        for (int m = 0; m < M; ++m) {
            pi[m] = expf(__fsub_rn(y[3 * M + m], pmax));
            psum = __fadd_rn(psum, pi[m]);
        }
        const float rps = __frcp_rn(psum);
#pragma unroll
        for (int m = 0; m < M; ++m) pi[m] = __fmul_rn(pi[m], rps);
        // the mixture over this thread's half of the pointers
        float cc[K], cs[K], om = 0.f;   // om: sum over this half's pointers of sum_k w_k^2 a_hat^2
#pragma unroll
        for (int k = 0; k < K; ++k) cc[k] = cs[k] = 0.f;
#pragma unroll
        for (int mm = 0; mm < M / 2; ++mm) {
            const int m = half * (M / 2) + mm;
            float dsm = ds[0], sgm = sg[0], mum = mu[0], pim = pi[0];
#pragma unroll
            for (int i = 1; i < M; ++i)
                if (i == m) dsm = ds[i], sgm = sg[i], mum = mu[i], pim = pi[i];
            const float rden = __frcp_rn(__fmul_rn(2.f, __fmul_rn(sgm, sgm)));
            float a[K], asum = 0.f;
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const float d = __fsub_rn(__ldg(p.log_omegas + k), mum);
                a[k] = __expf(__fmul_rn(-__fmul_rn(d, d), rden));   // relative error ~1e-7
                asum = __fadd_rn(asum, a[k]);
            }
            const float ran = __frcp_rn(__fadd_rn(asum, p.eps));
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const float ah = __fmul_rn(a[k], ran), wk = __ldg(p.omegas + k);
                om = __fadd_rn(om, __fmul_rn(__fmul_rn(wk, wk), __fmul_rn(ah, ah)));
                const float w = __fmul_rn(pim, ah);
                float sn, c;
                sincos_phase(__fmul_rn(__ldg(p.omegas + k), dsm), &sn, &c);
                cc[k] = __fadd_rn(cc[k], __fmul_rn(w, c));
                cs[k] = __fadd_rn(cs[k], __fmul_rn(w, sn));
            }
        }
        // exchange: half 0 finishes coeff_cos (needs half 1's cos sums), half 1 coeff_sin
        float *xch = reinterpret_cast<float *>(smem + L::Q);   // [2][K][128] (16 KB at most): the q tile is idle now
#pragma unroll
        for (int k = 0; k < K; ++k) xch[(half * K + k) * 128 + r] = half ? cc[k] : cs[k];
        float *xom = reinterpret_cast<float *>(smem + L::W1);   // [128]: W1 is idle now too
        if (half) xom[r] = om;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        float fin[K];
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const float other = xch[((1 - half) * K + k) * 128 + r];
            fin[k] = half ? __fadd_rn(other, cs[k]) : __fadd_rn(cc[k], other);
        }
        float b0 = 0.f;
        if (p.subtract_b0 && !half) {
#pragma unroll
            for (int k = 0; k < K; ++k) b0 = __fadd_rn(b0, fin[k]);
        }
        // ---- stores: [H,T,K] coefficients (cos by half 0, sin by half 1), [H,T,M], [H,T]
        float *oc = (half ? p.coeff_sin : p.coeff_cos) + row * K;
        if constexpr (K % 4 == 0) {
#pragma unroll
            for (int k = 0; k < K; k += 4) *reinterpret_cast<float4 *>(oc + k) = make_float4(fin[k], fin[k + 1], fin[k + 2], fin[k + 3]);
        } else {
#pragma unroll
            for (int k = 0; k < K; ++k) oc[k] = fin[k];
        }
        if (!half) {
#pragma unroll
            for (int m = 0; m < M; ++m) {
                p.delta_star[row * M + m] = ds[m];
                p.pi[row * M + m] = pi[m];
                p.budget[row * M + m] = y[4 * M + m];
            }
            p.b0[row] = b0;
            if (p.omega_reg) p.omega_reg[row] = __fadd_rn(om, xom[r]);
        } else {
            p.slope[row] = p.use_slope ? __fmul_rn(p.c_scale, tanhf(y[5 * M])) : 0.f;
            p.delta_main[row] = dmain;
            p.width[row] = __fadd_rn(
                p.width_min, __fmul_rn(__fsub_rn(p.width_max, p.width_min), sigmoid_ref(__fmul_rn(musum, 1.f / M))));
        }
    } else if (threadIdx.x == 0) {
        set_err(p.err, SCOPE_DEVERR_TIMEOUT);
    }

    // the MMAs are complete (or their wait gave up: wait once more, bounded) before TMEM is freed
    if (!ok && threadIdx.x == 0) {
        mbar_wait(&bars[1], 0, 500000000ull);
        mbar_wait(&bars[2], 0, 500000000ull);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ============================================================================ backward
// dL/dy for the MLP output y from the upstream gradients of the block's outputs
// (model/attn_bias.py:437-478 differentiated): one thread per token recomputes
// the heads from y and applies the chain rule through the mixture, the
// Gaussian normalisation, the softmax and the squashing functions.  The MLP's
// own backward (two bf16 linears and a SiLU) is left to the caller.
struct BwdParams {
    int rows, K, M, n_out, use_slope, subtract_b0;
    const uint16_t *y;
    const float *dcc, *dcs, *db0, *dslope, *ddelta_main, *dwidth, *dds, *dpi, *dbudget, *dom;
    const float *omegas, *log_omegas;
    float delta_cap, logw_min, logw_max, c_scale, width_min, width_max, eps;
    float *dy;
    uint16_t *dyb;    // or bf16 rows of dyb_ld (zero padded), written 16 bytes at a time
    int dyb_ld;
};

// Two threads per token (lanes 2t, 2t+1): each takes half of the M mixture
// components -- the K-frequency inner loops, the expensive part -- and the
// few sums over all components (softmax max / sum, the mean of mu, the
// argmax for delta_main, sum_m pi dpi) are completed with one shuffle each.
template <int K, int M>
__global__ void __launch_bounds__(256) coeff_bwd_kernel(const BwdParams p) {
    constexpr int MH = M / 2;
    const int half = threadIdx.x & 1;
    const int64_t row0 = (int64_t)blockIdx.x * 128 + (threadIdx.x >> 1);
    const bool valid = row0 < p.rows;
    const int64_t row = valid ? row0 : p.rows - 1;   // both lanes take part in the shuffles
    const uint16_t *yr = p.y + row * p.n_out;
    const int mb = half * MH;                        // this lane's first component
    float sd[MH], sm[MH], ss[MH], ds[MH], mu[MH], sg[MH], pi[MH], pl[MH];
    float pmax = -INFINITY, musum = 0.f;
    int imax = 0;
#pragma unroll
    for (int mm = 0; mm < MH; ++mm) {
        const int m = mb + mm;
        sd[mm] = sigmoid_ref(bf16_to_f32(yr[m]));
        sm[mm] = sigmoid_ref(bf16_to_f32(yr[M + m]));
        ss[mm] = sigmoid_ref(bf16_to_f32(yr[2 * M + m]));
        ds[mm] = sd[mm] * p.delta_cap;
        mu[mm] = p.logw_min + (p.logw_max - p.logw_min) * sm[mm];
        sg[mm] = 0.25f + 1.75f * ss[mm];
        musum += mu[mm];
        pl[mm] = bf16_to_f32(yr[3 * M + m]);
        if (pl[mm] > pmax) {
            pmax = pl[mm];
            imax = m;
        }
    }
    // the first largest pi logit over both halves (lane 0's components come first)
    {
        const float op = __shfl_xor_sync(0xffffffffu, pmax, 1);
        const int oi = __shfl_xor_sync(0xffffffffu, imax, 1);
        if (op > pmax || (op == pmax && oi < imax)) {
            pmax = op;
            imax = oi;
        }
    }
    musum += __shfl_xor_sync(0xffffffffu, musum, 1);
    float psum = 0.f;
#pragma unroll
    for (int mm = 0; mm < MH; ++mm) {
        pi[mm] = expf(pl[mm] - pmax);
        psum += pi[mm];
    }
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    {
        const float rps = __frcp_rn(psum);
#pragma unroll
        for (int mm = 0; mm < MH; ++mm) pi[mm] *= rps;
    }
    // upstream gradients of the per-frequency outputs; b0 = sum_k coeff_cos adds db0 to each
    float e[K], f[K];
    const float g_b0 = (p.subtract_b0 && p.db0) ? p.db0[row] : 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        e[k] = (p.dcc ? p.dcc[row * K + k] : 0.f) + g_b0;
        f[k] = p.dcs ? p.dcs[row * K + k] : 0.f;
    }
    float dpi[MH], dds[MH], dmu[MH], dsg[MH];
    const float g_om = p.dom ? p.dom[row] : 0.f;   // gradient of sum_m sum_k w_k^2 a_hat_mk^2
#pragma unroll
    for (int mm = 0; mm < MH; ++mm) {
        const int m = mb + mm;
        const float rden = __frcp_rn(2.f * sg[mm] * sg[mm]);
        float a[K], S = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const float d = __ldg(p.log_omegas + k) - mu[mm];
            a[k] = __expf(-(d * d) * rden);
            S += a[k];
        }
        const float Se = S + p.eps, rSe = __frcp_rn(Se);
        float gpi = 0.f, gdl = 0.f, dah[K], dot = 0.f;
#pragma unroll
        for (int k = 0; k < K; ++k) {
            float sn, c;
            sincos_phase(__ldg(p.omegas + k) * ds[mm], &sn, &c);
            const float ah = a[k] * rSe;
            const float g = e[k] * c + f[k] * sn;
            gpi += ah * g;
            gdl += ah * __ldg(p.omegas + k) * (f[k] * c - e[k] * sn);
            dah[k] = pi[mm] * g + g_om * 2.f * __ldg(p.omegas + k) * __ldg(p.omegas + k) * ah;
            dot += dah[k] * a[k];
        }
        dpi[mm] = gpi + (p.dpi ? p.dpi[row * M + m] : 0.f);
        dds[mm] = pi[mm] * gdl + (p.dds ? p.dds[row * M + m] : 0.f);
        // a_hat = a / (S + eps): da_k = dah_k / Se - sum_j dah_j a_j / Se^2
        float gm = 0.f, gs = 0.f;
        const float inv_s2 = 1.f / (sg[mm] * sg[mm]);
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const float da = (dah[k] - dot * rSe) * rSe;
            const float d = __ldg(p.log_omegas + k) - mu[mm];
            gm += da * a[k] * d * inv_s2;                    // d a / d mu    = a (l - mu) / sigma^2
            gs += da * a[k] * d * d * inv_s2 / sg[mm];       // d a / d sigma = a (l - mu)^2 / sigma^3
        }
        dmu[mm] = gm;
        dsg[mm] = gs;
    }
    if (p.ddelta_main) {
        const float g = p.ddelta_main[row];
#pragma unroll
        for (int mm = 0; mm < MH; ++mm)
            if (mb + mm == imax) dds[mm] += g;
    }
    if (p.dwidth) {
        const float sw = sigmoid_ref(musum / (float)M);
        const float g = p.dwidth[row] * (p.width_max - p.width_min) * sw * (1.f - sw) / (float)M;
#pragma unroll
        for (int mm = 0; mm < MH; ++mm) dmu[mm] += g;
    }
    float pd = 0.f;
#pragma unroll
    for (int mm = 0; mm < MH; ++mm) pd += pi[mm] * dpi[mm];
    pd += __shfl_xor_sync(0xffffffffu, pd, 1);
    // this lane's outputs: column g M + mb + mm of each group g (delta | mu | sigma | pi | budget)
    float o[5][MH];
#pragma unroll
    for (int mm = 0; mm < MH; ++mm) {
        const int m = mb + mm;
        o[0][mm] = dds[mm] * p.delta_cap * sd[mm] * (1.f - sd[mm]);
        o[1][mm] = dmu[mm] * (p.logw_max - p.logw_min) * sm[mm] * (1.f - sm[mm]);
        o[2][mm] = dsg[mm] * 1.75f * ss[mm] * (1.f - ss[mm]);
        o[3][mm] = pi[mm] * (dpi[mm] - pd);
        o[4][mm] = p.dbudget ? p.dbudget[row * M + m] : 0.f;
    }
    float oslope = 0.f;
    if (p.use_slope) {
        const float t = tanhf(bf16_to_f32(yr[5 * M]));
        oslope = (p.dslope ? p.dslope[row] : 0.f) * p.c_scale * (1.f - t * t);
    }
    if (p.dyb) {
        // the whole row in both lanes (the partner's components by shuffle), then each
        // lane writes half of its 16-byte chunks (bf16 pairs, zero past n_out)
        constexpr int NO = 5 * M + 1;
        constexpr int NPD = (NO + 15) / 16 * 16;
        float full[NO];
#pragma unroll
        for (int g = 0; g < 5; ++g) {
#pragma unroll
            for (int mm = 0; mm < MH; ++mm) {
                const float other = __shfl_xor_sync(0xffffffffu, o[g][mm], 1);
                full[g * M + mm] = half ? other : o[g][mm];
                full[g * M + MH + mm] = half ? o[g][mm] : other;
            }
        }
        full[5 * M] = oslope;
        uint4 *d = reinterpret_cast<uint4 *>(p.dyb + row * p.dyb_ld);
#pragma unroll
        for (int c8 = 0; c8 < NPD / 8; ++c8) {
            if (valid && (c8 & 1) == half && 8 * c8 < p.dyb_ld) {
                uint32_t w[4];
#pragma unroll
                for (int e4 = 0; e4 < 4; ++e4) {
                    const int c0 = 8 * c8 + 2 * e4, c1 = c0 + 1;
                    const float v0 = (c0 < NO && c0 < p.n_out) ? full[c0 < NO ? c0 : 0] : 0.f;
                    const float v1 = (c1 < NO && c1 < p.n_out) ? full[c1 < NO ? c1 : 0] : 0.f;
                    __nv_bfloat162 b = __floats2bfloat162_rn(v0, v1);
                    w[e4] = *reinterpret_cast<uint32_t *>(&b);
                }
                d[c8] = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
    } else if (valid) {
        float *dy = p.dy + row * p.n_out;
#pragma unroll
        for (int g = 0; g < 5; ++g) {
#pragma unroll
            for (int mm = 0; mm < MH; ++mm) dy[g * M + mb + mm] = o[g][mm];
        }
        if (p.use_slope && half == 0) dy[5 * M] = oslope;
    }
}

// bf16 [rows][inner] weights per head: [w_heads][rows][inner], box (64, box_rows, 1)
static bool map_weights(CUtensorMap *m, const void *base, int inner, int rows, int heads, int box_rows) {
    cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)heads};
    cuuint64_t strides[2] = {(cuuint64_t)inner * 2, (cuuint64_t)inner * rows * 2};
    cuuint32_t box[3] = {64u, (cuuint32_t)box_rows, 1u};
    cuuint32_t es[3] = {1, 1, 1};
    auto fn = tchost::encode_fn();
    return fn && fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int K, int M>
static int launch(const ScopeCoeffArgs &a, cudaStream_t s) {
    constexpr int NP = ((5 * M + 1) + 15) / 16 * 16;
    using L = Layout<NP>;
    Maps maps;
    std::memset(&maps, 0, sizeof(maps));
    if (!tchost::map3d(&maps.q, a.q, HD, a.T, a.H, a.q_st, a.q_sh, HD) ||
        !map_weights(&maps.w1, a.w1, HD, HID, a.w_heads, HID) ||
        !map_weights(&maps.w2, a.w2, HID, 5 * M + (a.use_slope ? 1 : 0), a.w_heads, NP))
        return SCOPE_ERR_ALIGN;
    Params p;
    std::memset(&p, 0, sizeof(p));
    p.H = a.H;
    p.T = a.T;
    p.K = K;
    p.M = M;
    p.n_out = 5 * M + (a.use_slope ? 1 : 0);
    p.use_slope = a.use_slope;
    p.subtract_b0 = a.subtract_b0;
    p.w_heads = a.w_heads;
    p.b1 = reinterpret_cast<const uint16_t *>(a.b1);
    p.b2 = reinterpret_cast<const uint16_t *>(a.b2);
    p.omegas = a.omegas;
    p.log_omegas = a.log_omegas;
    p.delta_cap = a.delta_cap;
    p.logw_min = a.logw_min;
    p.logw_max = a.logw_max;
    p.c_scale = a.c_scale;
    p.width_min = a.width_min;
    p.width_max = a.width_max;
    p.eps = a.eps;
    p.coeff_cos = a.coeff_cos;
    p.coeff_sin = a.coeff_sin;
    p.slope = a.slope;
    p.b0 = a.b0;
    p.delta_star = a.delta_star;
    p.pi = a.pi;
    p.budget = a.budget_logits;
    p.delta_main = a.delta_main;
    p.width = a.width;
    p.mlp_out = a.mlp_out;
    p.omega_reg = a.omega_reg;
    p.err = a.err_flag;
    const size_t smem = L::TOTAL + 1024;
    if (cudaFuncSetAttribute(coeff_kernel<K, M, NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return SCOPE_ERR_CUDA;
    coeff_kernel<K, M, NP><<<(unsigned)(a.H * (a.T / BM)), 256, smem, s>>>(maps, p);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

template <int K>
static int launch_m(const ScopeCoeffArgs &a, cudaStream_t s) {
    switch (a.M) {
        case 2: return launch<K, 2>(a, s);
        case 4: return launch<K, 4>(a, s);
        case 8: return launch<K, 8>(a, s);
        default: return SCOPE_ERR_UNSUPPORTED;
    }
}

template <int K, int M>
static int launch_bwd(const ScopeCoeffBwdArgs &a, cudaStream_t s) {
    BwdParams p;
    std::memset(&p, 0, sizeof(p));
    p.rows = a.H * a.T;
    p.K = K;
    p.M = M;
    p.n_out = 5 * M + (a.use_slope ? 1 : 0);
    p.use_slope = a.use_slope;
    p.subtract_b0 = a.subtract_b0;
    p.y = a.mlp_out;
    p.dcc = a.dcoeff_cos;
    p.dcs = a.dcoeff_sin;
    p.db0 = a.db0;
    p.dslope = a.dslope;
    p.ddelta_main = a.ddelta_main;
    p.dwidth = a.dwidth;
    p.dds = a.ddelta_star;
    p.dpi = a.dpi;
    p.dbudget = a.dbudget_logits;
    p.dom = a.domega_reg;
    p.omegas = a.omegas;
    p.log_omegas = a.log_omegas;
    p.delta_cap = a.delta_cap;
    p.logw_min = a.logw_min;
    p.logw_max = a.logw_max;
    p.c_scale = a.c_scale;
    p.width_min = a.width_min;
    p.width_max = a.width_max;
    p.eps = a.eps;
    p.dy = a.dy;
    p.dyb = reinterpret_cast<uint16_t *>(a.dy_bf16);
    p.dyb_ld = a.dy_ld;
    if (p.dyb) {
        constexpr int NPD = (5 * M + 1 + 15) / 16 * 16;
        if (p.dy || a.dy_ld % 8 || a.dy_ld < p.n_out || a.dy_ld > NPD) return SCOPE_ERR_INVALID;
        if (reinterpret_cast<uintptr_t>(a.dy_bf16) & 15) return SCOPE_ERR_ALIGN;
    }
    coeff_bwd_kernel<K, M><<<(unsigned)((p.rows + 127) / 128), 256, 0, s>>>(p);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

template <int K>
static int launch_bwd_m(const ScopeCoeffBwdArgs &a, cudaStream_t s) {
    switch (a.M) {
        case 2: return launch_bwd<K, 2>(a, s);
        case 4: return launch_bwd<K, 4>(a, s);
        case 8: return launch_bwd<K, 8>(a, s);
        default: return SCOPE_ERR_UNSUPPORTED;
    }
}

}  // namespace coeff
}  // namespace scope

extern "C" int scope_spectral_coeffs_bwd(const ScopeCoeffBwdArgs *args, scope_stream_t stream) {
    using namespace scope::coeff;
    if (!args) return SCOPE_ERR_INVALID;
    const ScopeCoeffBwdArgs &a = *args;
    if (a.H <= 0 || a.T <= 0 || !a.mlp_out || !a.omegas || !a.log_omegas || (!a.dy && !a.dy_bf16))
        return SCOPE_ERR_INVALID;
    if ((int64_t)a.H * a.T > INT32_MAX) return SCOPE_ERR_INVALID;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (a.K) {
        case 6: return launch_bwd_m<6>(a, s);
        case 8: return launch_bwd_m<8>(a, s);
        case 16: return launch_bwd_m<16>(a, s);
        default: return SCOPE_ERR_UNSUPPORTED;
    }
}

extern "C" int scope_spectral_coeffs(const ScopeCoeffArgs *args, scope_stream_t stream) {
    using namespace scope::coeff;
    if (!args) return SCOPE_ERR_INVALID;
    const ScopeCoeffArgs &a = *args;
    if (a.H <= 0 || a.T <= 0 || a.T % BM != 0 || a.D != HD || a.hidden != HID) return SCOPE_ERR_INVALID;
    if (a.w_heads != 1 && a.w_heads != a.H) return SCOPE_ERR_INVALID;
    if (!a.q || !a.w1 || !a.b1 || !a.w2 || !a.b2 || !a.omegas || !a.log_omegas || !a.coeff_cos || !a.coeff_sin ||
        !a.slope || !a.b0 || !a.delta_star || !a.pi || !a.budget_logits || !a.delta_main || !a.width)
        return SCOPE_ERR_INVALID;
    if ((a.q_st * 2) % 16 != 0 || (a.q_sh * 2) % 16 != 0) return SCOPE_ERR_ALIGN;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (a.K) {
        case 6: return launch_m<6>(a, s);
        case 8: return launch_m<8>(a, s);
        case 16: return launch_m<16>(a, s);
        default: return SCOPE_ERR_UNSUPPORTED;
    }
}
