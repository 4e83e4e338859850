// Backward of the SpectralBias coefficient MLP (model/attn_bias.py:306-324,
// shared weights) on the sm_100a tensor cores: from dL/dy to dL/dq, dL/dW1,
// dL/db1 and dL/dW2 in one pass over the tokens, with the roundings of the
// reference's bf16 autograd (each linear's output, the SiLU and its backward
// rounded to bf16).
//
// Persistent: one CTA per SM walks the 128-token tiles (all heads share the
// weights).  Per tile:
//   TMA      q [128 x 64] and dy [128 x NP] (bf16, NP = n_out padded to 16),
//            double buffered: tile t+1's loads are issued right after tile t's
//            first MMAs, so their latency overlaps tile t's work
//   tcgen05  X = q W1^T (128 hidden columns) and DH = dy W2 (128)
//   threads  x = bf16(X + b1), s = sigmoid(x), h = bf16(x s), dh = bf16(DH),
//            dx = bf16(dh s (1 + x (1 - s))); h and dx into shared memory
//   tcgen05  DQ = dx W1 (into X's first 64 columns), W2A += dy^T h,
//            W1A += dx^T [q | 1] (the extra column of ones gives db1)
//   threads  dq = bf16(DQ) -> global memory
// The accumulators W2A [NP x 128] and W1A [128 x (64 + 1)] stay in TMEM
// across the CTA's tiles and are added into fp32 global sums at the end.
// TMEM columns: X [0,128) (DQ reuses [0,64)), DH [128,256), W2A [256,384),
// W1A [384,464).  Every wait is bounded (SCOPE_DEVERR_TIMEOUT).
#include <cmath>
#include <cstring>

#include "common.cuh"
#include "tc_host.cuh"
#include "tc_ptx.cuh"

namespace scope {
namespace coeffbwd {

using namespace tc;

constexpr int BM = 128, HD = 64, HID = 128;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t TX = 0, TDH = 128, TW2 = 256, TW1 = 384;

__host__ __device__ constexpr uint32_t align1k(uint32_t x) { return (x + 1023u) & ~1023u; }

template <int NP>
struct Lay {
    static constexpr uint32_t W1 = 0;                               // [128 hid][64 d], 128-byte swizzle
    static constexpr uint32_t W2SUB = align1k(NP * 128);             // W2 [NP][64 hid] per half
    static constexpr uint32_t W2 = 16384;
    static constexpr uint32_t Q = align1k(W2 + 2 * W2SUB);           // 2 x [128 tok][64 d]
    // [128 tok][64]: column 0 = 1, the second N atom of [q | 1] for either q buffer (LBO = ONES - q)
    static constexpr uint32_t ONES = Q + 2 * 16384;
    static constexpr uint32_t DY = ONES + 16384;                     // 2 x 8 sub-tiles [128 tok][16], 32-byte swizzle
    static constexpr uint32_t DYB = 8 * 4096;                        // one dy buffer
    static constexpr uint32_t H = DY + 2 * DYB;                      // [128 tok][128 hid]: two halves
    static constexpr uint32_t DX = H + 32768;
    static constexpr uint32_t BAR = DX + 32768;
    static constexpr uint32_t TOTAL = BAR + 128;
    static constexpr uint32_t W_BYTES = 16384 + 2 * NP * 128;
    static constexpr uint32_t T_BYTES = 16384 + (NP / 16) * 4096;
};

struct Maps {
    CUtensorMap q, w1, w2, dy;
};

struct Params {
    int H, T, tiles, n_out;
    const uint16_t *b1;
    __nv_bfloat16 *dq;            // [H, T, 64] contiguous
    float *dw1, *db1, *dw2;       // fp32 sums, zeroed by the caller
    int32_t *err;
};

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <int NP>
__global__ void __launch_bounds__(256, 1) mlp_bwd_kernel(const __grid_constant__ Maps maps, const Params p) {
    using L = Lay<NP>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    // 0 weights, 1 / 5 tile in buffer 0 / 1, 2 X/DH, 3 DQ, 4 accumulators
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(smem + L::BAR + 64);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int quad = warp & 3, half = warp >> 2;
    const int r = quad * 32 + lane;                  // token row of the tile (TMEM lane)
    const uint32_t lb = (uint32_t)(quad * 32) << 16;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 6; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tslot, kTmemCols);
        tmem_relinquish();
    }
    // the ones column and the zero sub-tiles of dy beyond NP (rows of W2A that must stay 0)
    {
        uint4 *ones = reinterpret_cast<uint4 *>(smem + L::ONES);
        for (int i = threadIdx.x; i < 16384 / 16; i += blockDim.x) {
            const int row = i >> 3, chunk = i & 7;
            // element (row, 0) sits in chunk 0 ^ (row & 7) of the row (128-byte swizzle)
            ones[i] = (chunk == (row & 7)) ? make_uint4(0x3F80u, 0u, 0u, 0u) : make_uint4(0u, 0u, 0u, 0u);
        }
        for (int b = 0; b < 2; ++b) {
            uint4 *pad = reinterpret_cast<uint4 *>(smem + L::DY + b * L::DYB + (NP / 16) * 4096);
            for (int i = threadIdx.x; i < (8 - NP / 16) * 4096 / 16; i += blockDim.x) pad[i] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t sW1 = smem_u32(smem + L::W1), sW2 = smem_u32(smem + L::W2), sQ = smem_u32(smem + L::Q),
                   sDY = smem_u32(smem + L::DY), sH = smem_u32(smem + L::H), sDX = smem_u32(smem + L::DX);
    if (threadIdx.x == 0) {
        mbar_expect_tx(&bars[0], L::W_BYTES);
        tma_load_3d(&maps.w1, smem + L::W1, &bars[0], 0, 0, 0);
        tma_load_3d(&maps.w2, smem + L::W2, &bars[0], 0, 0, 0);
        tma_load_3d(&maps.w2, smem + L::W2 + L::W2SUB, &bars[0], 64, 0, 0);
    }
    const int tiles_per_head = p.T / BM;
    const uint16_t *b1 = p.b1;
    // tile loads into buffer b (its barrier: bars[1] for buffer 0, bars[5] for buffer 1)
    auto load_tile = [&](int tile, int b) {
        const int h = tile / tiles_per_head, t0 = (tile - h * tiles_per_head) * BM;
        uint64_t *bar = &bars[b ? 5 : 1];
        mbar_expect_tx(bar, L::T_BYTES);
        tma_load_3d(&maps.q, smem + L::Q + b * 16384, bar, 0, t0, h);
#pragma unroll
        for (int a = 0; a < NP / 16; ++a)
            tma_load_2d(&maps.dy, smem + L::DY + b * L::DYB + a * 4096, bar, 16 * a, h * p.T + t0);
    };
    int pend_b = -1, pend_par = 0;   // a prefetch not yet consumed (thread 0): drained before exit
    if (threadIdx.x == 0 && (int)blockIdx.x < p.tiles) {
        load_tile(blockIdx.x, 0);
        pend_b = 0;
    }
    bool ok = true;
    int it = 0;
    for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, ++it) {
        const int h = tile / tiles_per_head, t0 = (tile - h * tiles_per_head) * BM;
        const int b = it & 1;
        const uint32_t sQb = sQ + b * 16384, sDYb = sDY + b * L::DYB;
        // ---- the first two MMAs (one thread), then the next tile's loads into the other
        // buffer once the previous tile's MMAs, which read it (and h, dx), completed
        if (threadIdx.x == 0) {
            ok = (it > 0 || mbar_wait(&bars[0], 0)) && mbar_wait(&bars[b ? 5 : 1], (it >> 1) & 1);
            if (ok) pend_b = -1;
            if (ok) {
                tc_fence_after();
                constexpr uint32_t idX = idesc_bf16(128, HID, false, false);
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    mma_ss(tmem + TX, kmajor_desc(sQb + kk * 32, 128), kmajor_desc(sW1 + kk * 32, 128), idX, kk > 0);
                constexpr uint32_t idDH = idesc_bf16(128, HID, false, true);
#pragma unroll
                for (int kk = 0; kk < NP / 16; ++kk)
                    mma_ss(tmem + TDH, kmajor_desc(sDYb + kk * 4096, 32), smem_desc(sW2 + kk * 2048, L::W2SUB, 1024, SW128),
                           idDH, kk > 0);
                tc_commit(&bars[2]);
            }
            if (ok && it > 0) ok = mbar_wait(&bars[4], (it - 1) & 1);
            if (ok && tile + (int)gridDim.x < p.tiles) {
                load_tile(tile + gridDim.x, b ^ 1);
                pend_b = b ^ 1;
                pend_par = ((it + 1) >> 1) & 1;
            }
        }
        ok = __syncthreads_and(ok);
        if (!ok) break;
        // ---- h and dx for this thread's row, hidden columns [64 half, 64 half + 64)
        ok = mbar_wait(&bars[2], it & 1);
        ok = __syncthreads_and(ok);
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
            const int j0 = 64 * half + 32 * c;
            uint32_t vx[32], vd[32];
            tmem_ld32_nw(tmem + lb + TX + j0, vx);
            tmem_ld32_nw(tmem + lb + TDH + j0, vd);
            tmem_wait_ld();
            pin(vx);
            pin(vd);
            uint32_t ph[16], pdx[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
                float hv[2], dv[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const float x = bf16r(__fadd_rn(__uint_as_float(vx[e + u]), bf16_to_f32(__ldg(b1 + j0 + e + u))));
                    const float sg = 1.f / (1.f + __expf(-x));
                    hv[u] = bf16r(x * sg);
                    const float dh = bf16r(__uint_as_float(vd[e + u]));
                    dv[u] = bf16r(dh * sg * (1.f + x * (1.f - sg)));
                }
                ph[e / 2] = pack_bf16(hv[0], hv[1]);
                pdx[e / 2] = pack_bf16(dv[0], dv[1]);
            }
            // hidden columns j0..j0+31: half (j0 / 64), 16-byte chunks (j0 % 64) / 8 .. + 3
            uint8_t *hrow = smem + L::H + (j0 >> 6) * 16384 + r * 128;
            uint8_t *xrow = smem + L::DX + (j0 >> 6) * 16384 + r * 128;
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                const int chunk = ((j0 & 63) >> 3) + q4;
                *reinterpret_cast<uint4 *>(hrow + ((chunk ^ (r & 7)) << 4)) =
                    make_uint4(ph[4 * q4], ph[4 * q4 + 1], ph[4 * q4 + 2], ph[4 * q4 + 3]);
                *reinterpret_cast<uint4 *>(xrow + ((chunk ^ (r & 7)) << 4)) =
                    make_uint4(pdx[4 * q4], pdx[4 * q4 + 1], pdx[4 * q4 + 2], pdx[4 * q4 + 3]);
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncthreads();
        // ---- DQ = dx W1; the weight-gradient sums
        if (threadIdx.x == 0) {
            tc_fence_after();
            constexpr uint32_t idQ = idesc_bf16(128, HD, false, true);
#pragma unroll
            for (int kk = 0; kk < HID / 16; ++kk)
                mma_ss(tmem + TX, kmajor_desc(sDX + (kk >> 2) * 16384 + (kk & 3) * 32, 128), mnmajor128_desc(sW1 + kk * 2048),
                       idQ, kk > 0);
            tc_commit(&bars[3]);
            constexpr uint32_t idW2 = idesc_bf16(128, HID, true, true);
            constexpr uint32_t idW1 = idesc_bf16(128, HD + 16, true, true);
#pragma unroll
            for (int kk = 0; kk < BM / 16; ++kk) {
                const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
                mma_ss(tmem + TW2, mnmajor32_desc(sDYb + kk * 512), mnmajor128_desc(sH + kk * 2048), idW2, acc);
                // [q | 1]: the B operand's second 64-column atom is the ones tile, LBO bytes after q
                mma_ss(tmem + TW1, mnmajor128_desc(sDX + kk * 2048),
                       smem_desc(sQb + kk * 2048, (uint32_t)(L::ONES - L::Q) - b * 16384u, 1024, SW128), idW1, acc);
            }
            tc_commit(&bars[4]);
        }
        // ---- dq of this thread's row, d columns [32 half, 32 half + 32)
        ok = mbar_wait(&bars[3], it & 1);
        ok = __syncthreads_and(ok);
        if (!ok) break;
        tc_fence_after();
        {
            uint32_t v[32];
            tmem_ld32(tmem + lb + TX + 32 * half, v);
            tmem_wait_ld();
            pin(v);
            uint32_t w[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) w[e] = pack_bf16(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
            uint4 *dst = reinterpret_cast<uint4 *>(p.dq + ((int64_t)h * p.T + t0 + r) * HD + 32 * half);
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
        }
        // X is rewritten by the next tile's first MMA: every thread has read DQ first
        tc_fence_before();
        __syncthreads();
    }
    if (!ok) set_err(p.err, SCOPE_DEVERR_TIMEOUT);
    // never leave the CTA with a TMA write still in flight
    if (threadIdx.x == 0 && pend_b >= 0) mbar_wait(&bars[pend_b ? 5 : 1], pend_par, 500000000ull);
    // ---- the CTA's weight-gradient sums -> global
    bool fin = ok && it > 0;
    if (threadIdx.x == 0 && fin) fin = mbar_wait(&bars[4], (it - 1) & 1);
    fin = __syncthreads_and(fin);
    if (fin) {
        tc_fence_after();
        if (half == 0) {
            // W2A: lane = output o, 128 hidden columns
#pragma unroll 1
            for (int c = 0; c < HID; c += 32) {
                uint32_t v[32];
                tmem_ld32(tmem + lb + TW2 + c, v);
                tmem_wait_ld();
                pin(v);
                if (r < p.n_out)
                    for (int e = 0; e < 32; ++e) atomicAdd(p.dw2 + r * HID + c + e, __uint_as_float(v[e]));
            }
        } else {
            // W1A: lane = hidden unit, 64 d columns then the db1 column
#pragma unroll 1
            for (int c = 0; c < HD; c += 32) {
                uint32_t v[32];
                tmem_ld32(tmem + lb + TW1 + c, v);
                tmem_wait_ld();
                pin(v);
                for (int e = 0; e < 32; ++e) atomicAdd(p.dw1 + r * HD + c + e, __uint_as_float(v[e]));
            }
            uint32_t v1;
            tmem_ld1(tmem + lb + TW1 + HD, v1);
            tmem_wait_ld();
            atomicAdd(p.db1 + r, __uint_as_float(v1));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// [heads][rows][inner] bf16 weights, box (64, box_rows, 1), 128-byte swizzle
static bool map_w(CUtensorMap *m, const void *base, int inner, int rows, int box_rows) {
    cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, 1};
    cuuint64_t strides[2] = {(cuuint64_t)inner * 2, (cuuint64_t)inner * rows * 2};
    cuuint32_t box[3] = {64u, (cuuint32_t)box_rows, 1u};
    cuuint32_t es[3] = {1, 1, 1};
    auto fn = tchost::encode_fn();
    return fn && fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NP>
static int launch(const ScopeCoeffMlpBwdArgs &a, cudaStream_t s) {
    using L = Lay<NP>;
    Maps maps;
    std::memset(&maps, 0, sizeof(maps));
    if (!tchost::map3d(&maps.q, a.q, HD, a.T, a.H, a.q_st, a.q_sh, HD) || !map_w(&maps.w1, a.w1, HD, HID, HID) ||
        !map_w(&maps.w2, a.w2, HID, a.n_out, NP) ||
        !tchost::map2d(&maps.dy, a.dy, NP, (int)((int64_t)a.H * a.T), 16))
        return SCOPE_ERR_ALIGN;
    Params p;
    std::memset(&p, 0, sizeof(p));
    p.H = a.H;
    p.T = a.T;
    p.tiles = a.H * (a.T / BM);
    p.n_out = a.n_out;
    p.b1 = reinterpret_cast<const uint16_t *>(a.b1);
    p.dq = reinterpret_cast<__nv_bfloat16 *>(a.dq);
    p.dw1 = a.dw1;
    p.db1 = a.db1;
    p.dw2 = a.dw2;
    p.err = a.err_flag;
    const size_t smem = L::TOTAL + 1024;
    if (cudaFuncSetAttribute(mlp_bwd_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return SCOPE_ERR_CUDA;
    int dev = 0, n_sm = 148;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return SCOPE_ERR_CUDA;
    mlp_bwd_kernel<NP><<<(unsigned)std::min(p.tiles, n_sm), 256, smem, s>>>(maps, p);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

}  // namespace coeffbwd
}  // namespace scope

extern "C" int scope_spectral_mlp_bwd(const ScopeCoeffMlpBwdArgs *args, scope_stream_t stream) {
    using namespace scope::coeffbwd;
    if (!args) return SCOPE_ERR_INVALID;
    const ScopeCoeffMlpBwdArgs &a = *args;
    if (a.H <= 0 || a.T <= 0 || a.T % BM != 0 || a.n_out < 1 || a.n_out > 96) return SCOPE_ERR_INVALID;
    if (!a.q || !a.w1 || !a.b1 || !a.w2 || !a.dy || !a.dq || !a.dw1 || !a.db1 || !a.dw2) return SCOPE_ERR_INVALID;
    if ((int64_t)a.H * a.T > INT32_MAX) return SCOPE_ERR_INVALID;
    if ((a.q_st * 2) % 16 != 0 || (a.q_sh * 2) % 16 != 0 || !scope::tchost::aligned16(a.q) ||
        !scope::tchost::aligned16(a.dq) || !scope::tchost::aligned16(a.dy))
        return SCOPE_ERR_ALIGN;
    if (!scope_device_supported() || !scope::tchost::encode_fn()) return SCOPE_ERR_UNSUPPORTED;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int np = (a.n_out + 15) / 16 * 16;
    switch (np) {
        case 16: return launch<16>(a, s);
        case 32: return launch<32>(a, s);
        case 48: return launch<48>(a, s);
        case 64: return launch<64>(a, s);
        case 80: return launch<80>(a, s);
        case 96: return launch<96>(a, s);
        default: return SCOPE_ERR_UNSUPPORTED;
    }
}
