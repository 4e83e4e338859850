// Block-sparse SCOPE attention backward on the sm_100a tensor cores.
//
// Launches, all on the caller's stream:
//   prep    delta_i = sum_d dO_i . O_i  and  lse2_i = lse_i * log2(e)   (workspace)
//   plan    per (head, kv block) the number of q blocks that see it (from the
//           builder's q-side bitmap) and the work items: a kv block and a run
//           of the q blocks that see it, ascending
//   dkvq    persistent, one CTA per SM walking the work items.  Per (kv block,
//           q block) tile it recomputes S^T and dP^T once and produces all
//           three gradients: dV += P^T dO and dK += dS^T Q accumulate in TMEM
//           over the item; dQ (and, for the qk_aug spectral bias, the gradient
//           of the augmented q dims) = dS [K | K_aug] is formed in TMEM per
//           tile and added into an fp32 accumulator in global memory by
//           dedicated drain warps (red.global.add, L2-resident adds).
//   finish  dQ accumulator -> bf16 dq (x scale); the augmented-dim gradient ->
//           dcoeff_cos / dcoeff_sin / dslope by the chain rule of
//           scoped_medium.py:380-421.
// A kv block that many q blocks see (a global / sink block is seen by every q
// block of its document) would make one CTA walk a list of up to QB tiles;
// `plan` cuts such lists into chunks of at most kChunk q tiles handled by
// separate items, whose fp32 dK / dV partial sums meet in a small slot buffer
// that the last chunk of the row converts to bf16.
//
// dkvq, per CTA (one per SM, 768 threads, all 512 TMEM columns):
//   warp 0       producer (TMA): per item K (+ K_aug) and V; per tile Q
//                (+ Q_aug), dO, lse2, delta into an NST-stage ring
//   warp 1       S / dP issuer: S^T = K Q^T (+ K_aug Q_aug^T) into SB once the
//                previous tile's dV MMAs read their P^T from it; dP^T = V dO^T
//                into DPB once the previous tile's dK MMAs read their dS^T
//   warp 2       gradient issuer: dV += P^T dO (P^T from TMEM), dK += dS^T Q
//                (dS^T from TMEM); it releases the tile's stage
//   warp 3       dQ issuer: dQ = dS [K | K_aug] (dS from shared memory) into DQ
//                once the drain warps copied out the previous tile's.  Each
//                tcgen05.mma holds its issuing warp about as long as the tensor
//                pipe takes to run it, and that cost lands on the warp's
//                sub-partition: three issuing warps spread it
//   warps 4-19   elementwise (four per TMEM lane quadrant): thread = kv row,
//                32 q columns each: P = exp2(S scale log2e - lse2) (masked),
//                P^T as bf16 pairs over the warp's own S^T columns; then dP^T 16
//                columns at a time, dS = P (dP - delta) as bf16 pairs over the
//                chunk's own dP^T columns and into the shared-memory dS tile
//   warps 20-23  dQ drain: per tile, the dQ accumulator rows of their lane
//                quadrant out of TMEM and added into global memory
// TMEM columns: SB [0,128) S^T, then P^T as bf16 pairs over the read columns;
// DPB [128,256) dP^T, then dS^T as bf16 pairs; DV [256,320); DK [320,384);
// DQ [384, 448 + DA) dQ | aug-dim gradient.  The kernel is bound by shared-memory
// bandwidth: per tile the SS MMAs read ~170 KB of operands, TMA writes ~41 KB,
// dS and the dQ staging boxes add ~80 KB.  Every wait is bounded
// (SCOPE_DEVERR_TIMEOUT).
#include <algorithm>
#include <cmath>
#include <cstring>

#include "tc_host.cuh"
#include "tc_ptx.cuh"

namespace scope {
namespace tcbwd {

using namespace tc;

constexpr int BM = 128;
constexpr int HD = 64;
constexpr int kElemWarps = 16;          // four per TMEM lane quadrant, 32 tile columns each
constexpr int kElemWarp0 = 4;           // warpgroups 1-4
constexpr int kDrainWarp0 = kElemWarp0 + kElemWarps;   // warpgroup 5
constexpr int kThreads = 32 * (kDrainWarp0 + 4);       // 768: six warpgroups
constexpr int kElem = 32 * kElemWarps;  // elementwise threads
constexpr int kDrain = 128;             // drain threads
constexpr int kDrainBoxes = 3;          // staging boxes per drain warp (reduces in flight)
constexpr int kIdxWarps = 3 + kElemWarps + 4;   // the issuers, elementwise and drain warps read each item index
constexpr int kChunk = 64;              // max q tiles per dK/dV work item
constexpr int kSlotCap = 128;           // max kv rows whose q list is split
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t SB = 0, DPB = 128, DV = 256, DK = 320, DQ = 384;
// TMEM column of the bf16 P^T pairs of K step kk (q rows 16kk..16kk+15) of the dV MMA:
// warp kk/2's chunk kk%2, written over the first 16 of that warp's 32 S^T columns
__device__ __forceinline__ uint32_t pcol(int kk) { return (uint32_t)(32 * (kk >> 1) + 8 * (kk & 1)); }
constexpr uint32_t kSmemBudget = 227 * 1024;   // dynamic shared memory per CTA
constexpr float kLog2e = 1.4426950408889634f;

__host__ __device__ constexpr uint32_t align1k(uint32_t x) { return (x + 1023u) & ~1023u; }

// ------------------------------------------------------------------ prep
// score_mod mode: the forward's lse includes the row constant -beta b0, which
// the recomputed scores leave out, so it is added back here; the per-row slope,
// Δ_main and width are copied next to each other (zeros for absent terms) for
// the producer's per-tile bulk loads.
struct PrepSmod {
    const float *b0, *slope, *dmain, *width;
    float beta;
    float *par;   // [3][H*T]: slope, Δ_main, width
};

__global__ void prep_kernel(const __nv_bfloat16 *__restrict__ out, int64_t o_sh, int64_t o_st,
                            const __nv_bfloat16 *__restrict__ dout, int64_t do_sh, int64_t do_st,
                            const float *__restrict__ lse, int H, int T, float *__restrict__ delta,
                            float *__restrict__ lse2, const PrepSmod sm) {
    int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= (int64_t)H * T) return;
    const int h = (int)(row / T), t = (int)(row % T);
    const uint4 *o = reinterpret_cast<const uint4 *>(out + h * o_sh + (int64_t)t * o_st);
    const uint4 *d = reinterpret_cast<const uint4 *>(dout + h * do_sh + (int64_t)t * do_st);
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        uint4 a = o[k], b = d[k];
        const __nv_bfloat162 *pa = reinterpret_cast<const __nv_bfloat162 *>(&a);
        const __nv_bfloat162 *pb = reinterpret_cast<const __nv_bfloat162 *>(&b);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float2 fa = __bfloat1622float2(pa[e]), fb = __bfloat1622float2(pb[e]);
            s = fmaf(fa.x, fb.x, s);
            s = fmaf(fa.y, fb.y, s);
        }
    }
    delta[row] = s;
    float l = lse[row];
    if (sm.par) {
        if (sm.b0 && l != -INFINITY) l += sm.beta * sm.b0[row];
        const int64_t n = (int64_t)H * T;
        sm.par[row] = sm.slope ? sm.slope[row] : 0.f;
        sm.par[n + row] = sm.dmain ? sm.dmain[row] : 0.f;
        sm.par[2 * n + row] = sm.width ? sm.width[row] : 0.f;
    }
    lse2[row] = (l == -INFINITY) ? INFINITY : l * kLog2e;   // rows that saw nothing get P = 0
}

struct Plan {
    const int32_t *n_items;   // [1]
    const int4 *items;        // (h, kb, first q rank, count)
    const int32_t *item_slot; // split slot or -1
    const int32_t *slot_chunks;
    int32_t *slot_done;
    float *partial;           // [kSlotCap][128 rows][128]: dV (64) | dK (64)
    int32_t *next_item;       // items handed out beyond the first G (zeroed by the plan kernel)
};

struct Params {
    int H, T, QB, words;
    const uint32_t *q_bitmap;
    const int32_t *block_info, *docs;
    const float *lse2, *delta;
    float scale, scale_log2;
    __nv_bfloat16 *dk, *dv;
    int64_t dk_sh, dk_st, dv_sh, dv_st;
    float *dq_acc;            // [H, T, 64 + DA] fp32, zeroed before the launch
    float *slope_acc;         // [H, T] fp32 (qk_aug with slope; score_mod: sum_j dS_ij (i - j)), zeroed
    float s_aug;
    // score_mod: per-row slope, Δ_main, width [3][H*T] (staged per tile), the gate
    // sums [H, T] (zeroed), beta*log2(e), the gate's lambda and 1/tau
    const float *par;
    float *dm_acc, *w_acc;
    float bias2, gate_lambda, gate_itau;
    Plan plan;
    int32_t *err;
};

struct Maps {
    CUtensorMap q, k16, v, dout, qa, ka;   // k16: K in 16-column boxes (32-byte swizzle)
    CUtensorMap dqa;                       // the fp32 dQ accumulator [H*T, 64 + DA], 32 x 16 boxes
};

struct Ctx {
    volatile int *abort_flag;
    int32_t *err;
    __device__ void give_up() {
        *abort_flag = 1;
        set_err(err, SCOPE_DEVERR_TIMEOUT);
    }
    __device__ bool wait1(uint64_t *bar, uint32_t parity) {      // single thread
        if (*abort_flag) return false;
        if (mbar_wait(bar, parity)) return true;
        give_up();
        return false;
    }
    __device__ bool waitw(uint64_t *bar, uint32_t parity) {      // a whole warp, uniform result
        bool ok = !*abort_flag && mbar_wait(bar, parity);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) give_up();
        return ok;
    }
};

__device__ __forceinline__ void elem_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kElem) : "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }


// mbarriers and small shared state of a backward CTA
struct Bars {
    uint64_t res_full;                 // an item's K (+aug), V are in shared memory (tx bytes)
    uint64_t acc_done;                 // every gradient MMA of an item completed
    uint64_t acc_free;                 // the item's epilogue read dV / dK (elementwise arrivals)
    uint64_t idx_taken;                // every consuming warp read the item index (one arrival per warp)
    uint64_t full[4], empty[4];        // streamed stage ring
    uint64_t s_full;                   // S^T of a tile is in SB
    uint64_t p_full;                   // all of P^T is back in the S buffer
    uint64_t pv_done;                  // the dV MMAs that read P^T completed
    uint64_t dp_full;                  // dP^T of a tile is in DPB
    uint64_t ds_ready;                 // dS^T back in DPB and dS in shared memory
    uint64_t dp_free;                  // the dK MMAs that read dS^T completed
    uint64_t dq_full;                  // dQ of a tile is in DQ (and the dS tile in shared memory is free)
    uint64_t dq_free;                  // the drain warps copied DQ out
    uint64_t drain[3];                 // each issuing warp's MMAs completed (before TMEM is freed)
    volatile int stage_blk[4];         // q block of the tile in each stage
    volatile int stage_mk[4];          // its mask kind
    uint32_t tmem_slot;
    volatile int abort_flag, last_flag, item_of;
    __device__ void init(int nst) {
        mbar_init(&res_full, 1);
        mbar_init(&acc_done, 2);   // the gradient issuer and the dQ issuer
        mbar_init(&acc_free, kElem);
        mbar_init(&idx_taken, kIdxWarps);
        for (int i = 0; i < nst; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(&s_full, 1);
        mbar_init(&dq_full, 1);
        mbar_init(&dq_free, kDrain);
        mbar_init(&p_full, kElem);
        mbar_init(&pv_done, 1);
        mbar_init(&dp_full, 1);
        mbar_init(&ds_ready, kElem);
        mbar_init(&dp_free, 1);
        mbar_init(&drain[0], 1);
        mbar_init(&drain[1], 1);
        mbar_init(&drain[2], 1);
        abort_flag = 0;
        last_flag = 0;
        item_of = 0;
        fence_mbar_init();
    }
};

// N (16 or 32) fp32 accumulator columns -> 2N bytes of a bf16 row in global memory
template <int N>
__device__ __forceinline__ void store_row(uint32_t taddr, float mul, __nv_bfloat16 *dst, bool have) {
    uint32_t o[N];
    if (have) {
        if constexpr (N == 32) {
            tmem_ld32_nw(taddr, o);
        } else {
            tmem_ld16(taddr, o);
        }
        tmem_wait_ld();
        pin(o);
    } else {
#pragma unroll
        for (int e = 0; e < N; ++e) o[e] = 0u;
    }
    uint32_t w[N / 2];
#pragma unroll
    for (int e = 0; e < N / 2; ++e) w[e] = pack_bf16(__uint_as_float(o[2 * e]) * mul, __uint_as_float(o[2 * e + 1]) * mul);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
    for (int e = 0; e < N / 8; ++e) d[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
}

// Tile masking: every element of a full tile is visible; a tile whose q and kv
// blocks lie in one document needs only the causal test (one compare); only
// tiles that straddle a document boundary read document ids per element.
// The producer thread classifies each tile (it runs ahead of the elementwise
// warps) and hands the class over in shared memory with the tile's block index.
enum MaskKind { MASK_FULL = 0, MASK_CAUSAL = 1, MASK_DOCS = 2 };
__device__ __forceinline__ int tile_mask_kind(int qb, int kb, bool have_docs, const int32_t *block_info, int QB) {
    bool same_doc = !have_docs;
    if (have_docs && block_info) {
        const int a = block_info[2 * QB + qb], b = block_info[3 * QB + qb];
        const int c = block_info[2 * QB + kb], d = block_info[3 * QB + kb];
        same_doc = (a == b) & (c == d) & (a == c);
    }
    if (kb < qb && same_doc) return MASK_FULL;
    return same_doc ? MASK_CAUSAL : MASK_DOCS;
}

// Bias of the score_mod mode beyond the Fourier sum, for Δ = i - j
// (scoped_medium.py:425-457): slope Δ - lambda gate((|Δ - Δ_main| - width) / tau).
// SM: 0 off, 1 no gate, 2 softplus gate (torch's, threshold 20), 3 relu gate.
template <int SM>
__device__ __forceinline__ float smod_bias(float dl, float slope, float dm, float w, float lam, float itau) {
    float b = slope * dl;
    if constexpr (SM >= 2) {
        const float u = (fabsf(dl - dm) - w) * itau;
        float g;
        if constexpr (SM == 3) {
            g = fmaxf(u, 0.f);
        } else {
            g = u > 20.f ? u : 0.69314718055994531f * lg2(1.f + ex2(u * kLog2e));
        }
        b = fmaf(-lam, g, b);
    }
    return b;
}

// score_mod parameters of the 32 q rows of a thread's columns (staged per tile)
struct SmodCols {
    const float *slope, *dm, *w;
};

// P for 16 columns, thread = kv row j: P = exp2(S * scale*log2e - lse2), zero
// where the element is masked (column e visible iff e >= lim, and in j's
// document on boundary tiles).
template <bool MASKED, int SM = 0>
__device__ __forceinline__ void p_piece(float *s, const float4 *LS, uint64_t c2, int mk, int lim,
                                        const int32_t *docs, int i0, int doc_j, const SmodCols &sc = SmodCols{},
                                        float bias2 = 0.f, float lam = 0.f, float itau = 0.f) {
#pragma unroll
    for (int e4 = 0; e4 < 4; ++e4) {
        const float4 l4 = LS[e4];
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
            const int e = e4 * 4 + 2 * q2;
            uint64_t nl = q2 ? f2_pack(-l4.z, -l4.w) : f2_pack(-l4.x, -l4.y);
            if constexpr (SM != 0) {
                // + beta log2(e) (slope Δ - lambda gate), Δ = i - j = e - lim
                const float2 n2 = f2_unpack(nl);
                const float b0v = smod_bias<SM>((float)(e - lim), sc.slope[e], sc.dm[e], sc.w[e], lam, itau);
                const float b1v = smod_bias<SM>((float)(e + 1 - lim), sc.slope[e + 1], sc.dm[e + 1], sc.w[e + 1], lam, itau);
                nl = f2_pack(fmaf(bias2, b0v, n2.x), fmaf(bias2, b1v, n2.y));
            }
            const float2 x = f2_unpack(ffma2(f2_pack(s[e], s[e + 1]), c2, nl));
            float p0 = ex2(x.x), p1 = ex2(x.y);
            if (MASKED) {
                bool v0 = e >= lim, v1 = e + 1 >= lim;
                if (mk == MASK_DOCS) {
                    v0 = v0 && (__ldg(docs + i0 + e) == doc_j);
                    v1 = v1 && (__ldg(docs + i0 + e + 1) == doc_j);
                }
                p0 = v0 ? p0 : 0.f;
                p1 = v1 ? p1 : 0.f;
            }
            s[e] = p0;
            s[e + 1] = p1;
        }
    }
}

// dS = P (dP - delta) for 16 columns, into dp
__device__ __forceinline__ void ds_piece(const float *p, float *dp, const float4 *DL) {
#pragma unroll
    for (int e4 = 0; e4 < 4; ++e4) {
        const float4 d4 = DL[e4];
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
            const int e = e4 * 4 + 2 * q2;
            const uint64_t nd = q2 ? f2_pack(-d4.z, -d4.w) : f2_pack(-d4.x, -d4.y);
            const float2 ds = f2_unpack(fmul2(f2_pack(p[e], p[e + 1]), fadd2(f2_pack(dp[e], dp[e + 1]), nd)));
            dp[e] = ds.x;
            dp[e + 1] = ds.y;
        }
    }
}

// Column sums of a warp's 32-row x 16-column block: lane l returns the sum over
// the 32 lanes of v[l & 15] (a butterfly that halves the values each lane carries
// every round, then the two 16-lane halves added).
__device__ __forceinline__ float warp_column_sums16(float (&v)[16]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int w = 8; w >= 1; w >>= 1) {
        const bool hi = (lane & w) != 0;
#pragma unroll
        for (int e = 0; e < w; ++e) {
            const float send = hi ? v[e] : v[e + w];
            const float keep = hi ? v[e + w] : v[e];
            v[e] = keep + __shfl_xor_sync(0xffffffffu, send, w);
        }
    }
    return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 16);
}

// rank-th set bit onward of a bitmap row: the word index and remaining bits
__device__ __forceinline__ void seek_rank(const uint32_t *row, int words, int rank, int &w, uint32_t &bits) {
    w = 0;
    bits = 0;
    for (; w < words; ++w) {
        bits = row[w];
        const int c = __popc(bits);
        if (rank < c) break;
        rank -= c;
    }
    for (; rank > 0 && bits; --rank) bits &= bits - 1;
}
// next set bit of the walk (-1 past the end)
__device__ __forceinline__ int next_bit(const uint32_t *row, int words, int &w, uint32_t &bits) {
    while (!bits) {
        if (++w >= words) return -1;
        bits = row[w];
    }
    const int qb = w * 32 + __ffs(bits) - 1;
    bits &= bits - 1;
    return qb;
}

// Shared memory of a dkvq CTA.  K and the aug dims of a kv block are 16-column
// sub-tiles (32-byte swizzle) 4 KiB apart, so [K | K_aug] is one MN-major B
// operand of N = 64 + DA for dQ and K-major A operands (one per K step) for S^T.
// dS is stored MN-major (128-byte swizzle, two 64-column halves 16 KiB apart),
// the A operand of dQ = dS [K | K_aug].
template <int DA, int SM = 0>
struct FL {
    static constexpr int NA = DA / 16;
    static constexpr int NKA = 4 + NA;                        // K + K_aug sub-tiles
    static constexpr uint32_t TILE = BM * HD * 2, ATILE = BM * 16 * 2;
    static constexpr uint32_t RK = 0, RV = align1k(NKA * ATILE);
    static constexpr uint32_t RESB = align1k(RV + TILE);
    static constexpr uint32_t DS = RESB;                      // dS tile, 32 KiB
    static constexpr uint32_t STAGE0 = DS + 2 * TILE;
    static constexpr uint32_t SQ = 0, SQA = TILE, SDO = align1k(TILE + NA * ATILE), SLSE = SDO + TILE,
                              SDEL = SLSE + 512, SPAR = SDEL + 512;   // SPAR: score_mod slope, Δ_main, width
    static constexpr uint32_t PAR_BYTES = SM ? 3 * 512 : 0;
    static constexpr uint32_t STAGE = align1k(SPAR + PAR_BYTES);
    static constexpr uint32_t EXTRA = 1024 + 1024;            // barriers, base alignment
    static constexpr uint32_t DRN_BYTES = 4 * kDrainBoxes * 2048;   // drain staging: 32 x 16 fp32 boxes
    static constexpr int NST = STAGE0 + 4 * STAGE + DRN_BYTES + EXTRA <= kSmemBudget
                                   ? 4
                                   : (STAGE0 + 3 * STAGE + DRN_BYTES + EXTRA <= kSmemBudget ? 3 : 2);
    static constexpr uint32_t DRN = STAGE0 + NST * STAGE;       // 1024-aligned (STAGE0, STAGE are)
    static constexpr uint32_t BAR = DRN + DRN_BYTES;
    static constexpr uint32_t RES_BYTES = NKA * ATILE + TILE;
    static constexpr uint32_t Q_BYTES = 2 * TILE + NA * ATILE + 1024 + PAR_BYTES;
    static constexpr uint32_t TOTAL = BAR + sizeof(Bars);
    static constexpr int DQN = 64 + DA;                       // dQ accumulator columns
    static_assert(TOTAL + 1024 <= kSmemBudget, "shared memory");
    static_assert(DQ + DQN <= kTmemCols, "tensor memory");
};

template <int DA, bool SLOPE, int SM>
__global__ void __launch_bounds__(kThreads, 1) dkvq_kernel(const __grid_constant__ Maps maps, const Params p) {
    using L = FL<DA, SM>;
    constexpr int NA = L::NA, NST = L::NST;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    Bars &B = *reinterpret_cast<Bars *>(smem + L::BAR);
    Ctx cx{&B.abort_flag, p.err};

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = *p.plan.n_items, G = gridDim.x;

    if (threadIdx.x == 0) B.init(NST);
    if (warp == 1) {
        tmem_alloc(&B.tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = B.tmem_slot;
    const uint32_t sK = smem_u32(smem + L::RK), sV = smem_u32(smem + L::RV), sDS = smem_u32(smem + L::DS);

    if (warp == 0) {
        // ---------------- producer: per item K (+aug) / V, then the q tiles that see the kv block
        if (lane == 0) {
            int gt = 0, last_res = -1;
            bool ok = true;
            for (int ci = 0; ok; ++ci) {
                // the first item of each CTA is its block index, the rest are handed out in order
                const int it = ci == 0 ? (int)blockIdx.x : G + atomicAdd(p.plan.next_item, 1);
                // the item index may be replaced once every warp read the previous one, the
                // residents once every MMA of the previous item completed
                if (ci >= 1 && (!cx.wait1(&B.idx_taken, (ci - 1) & 1) || !cx.wait1(&B.acc_done, (ci - 1) & 1))) break;
                last_res = -1;
                B.item_of = it < n_items ? it : -1;
                if (it >= n_items) {
                    mbar_arrive(&B.res_full);      // publishes "no item left"
                    break;
                }
                const int4 item = p.plan.items[it];
                const int h = item.x, kb = item.y, first = item.z, nq = item.w;
                if (nq > 0) {
                    mbar_expect_tx(&B.res_full, L::RES_BYTES);
#pragma unroll
                    for (int a = 0; a < 4; ++a)
                        tma_load_3d(&maps.k16, smem + L::RK + a * L::ATILE, &B.res_full, 16 * a, kb * BM, h);
#pragma unroll
                    for (int a = 0; a < NA; ++a)
                        tma_load_2d(&maps.ka, smem + L::RK + (4 + a) * L::ATILE, &B.res_full, 16 * a, kb * BM);
                    tma_load_3d(&maps.v, smem + L::RV, &B.res_full, 0, kb * BM, h);
                    last_res = ci;
                } else {
                    mbar_arrive(&B.res_full);      // keeps the phases in step
                }
                const uint32_t *brow = p.q_bitmap + ((int64_t)h * p.QB + kb) * p.words;
                int w;
                uint32_t bits;
                seek_rank(brow, p.words, first, w, bits);
                int t = 0;
                for (; t < nq; ++t) {
                    const int qb = next_bit(brow, p.words, w, bits);
                    if (qb < 0) break;
                    const int st = gt % NST;
                    if (gt >= NST && !cx.wait1(&B.empty[st], ((gt / NST) - 1) & 1)) { ok = false; break; }
                    uint8_t *sb = smem + L::STAGE0 + st * L::STAGE;
                    B.stage_blk[st] = qb;
                    B.stage_mk[st] = tile_mask_kind(qb, kb, p.docs != nullptr, p.block_info, p.QB);
                    mbar_expect_tx(&B.full[st], L::Q_BYTES);
                    tma_load_3d(&maps.q, sb + L::SQ, &B.full[st], 0, qb * BM, h);
#pragma unroll
                    for (int a = 0; a < NA; ++a)
                        tma_load_3d(&maps.qa, sb + L::SQA + a * L::ATILE, &B.full[st], 16 * a, qb * BM, h);
                    tma_load_3d(&maps.dout, sb + L::SDO, &B.full[st], 0, qb * BM, h);
                    const int64_t off = (int64_t)h * p.T + (int64_t)qb * BM;
                    bulk_load(sb + L::SLSE, p.lse2 + off, 512, &B.full[st]);
                    bulk_load(sb + L::SDEL, p.delta + off, 512, &B.full[st]);
                    if constexpr (SM != 0) {
                        const int64_t n = (int64_t)p.H * p.T;
#pragma unroll
                        for (int a = 0; a < 3; ++a)
                            bulk_load(sb + L::SPAR + a * 512, p.par + a * n + off, 512, &B.full[st]);
                    }
                    ++gt;
                }
                if (ok && t < nq) {   // the plan promised more q blocks than the bitmap row holds
                    set_err(p.err, SCOPE_DEVERR_INDEX);
                    cx.give_up();
                    ok = false;
                }
            }
            // never leave the CTA with a TMA write still in flight
            if (last_res >= 0) mbar_wait(&B.res_full, last_res & 1, 500000000ull);
            for (int j = (gt > NST ? gt - NST : 0); j < gt; ++j) mbar_wait(&B.full[j % NST], (j / NST) & 1, 500000000ull);
        }
    } else if (warp == 1) {
        // ---------------- S / dP issuer (the whole warp waits, lane 0 issues)
        constexpr uint32_t idS = idesc_bf16(128, 128, false, false);
        int gt = 0;
        bool ok = true;
        for (int ci = 0; ok; ++ci) {
            if (!cx.waitw(&B.res_full, ci & 1)) { ok = false; break; }
            const int it = B.item_of;
            __syncwarp();
            if (lane == 0) mbar_arrive(&B.idx_taken);
            if (it < 0) break;
            const int nq = p.plan.items[it].w;
            for (int t = 0; t < nq; ++t, ++gt) {
                const int st = gt % NST;
                if (!cx.waitw(&B.full[st], (gt / NST) & 1)) { ok = false; break; }
                const uint32_t sb = smem_u32(smem + L::STAGE0 + st * L::STAGE);
                // S^T = K Q^T (+ K_aug Q_aug^T) into SB once the dV MMAs of the previous tile
                // read their P^T from it
                if (gt >= 1 && !cx.waitw(&B.pv_done, (gt - 1) & 1)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_ss(tmem + SB, kmajor_desc(sK + kk * L::ATILE, 32),
                               kmajor_desc(sb + L::SQ + kk * 32, 128), idS, kk > 0);
#pragma unroll
                    for (int a = 0; a < NA; ++a)
                        mma_ss(tmem + SB, kmajor_desc(sK + (4 + a) * L::ATILE, 32),
                               kmajor_desc(sb + L::SQA + a * L::ATILE, 32), idS, 1);
                    tc_commit(&B.s_full);
                }
                __syncwarp();
                // dP^T = V dO^T once the dK MMAs of the previous tile read its dS^T
                if (gt >= 1 && !cx.waitw(&B.dp_free, (gt - 1) & 1)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_ss(tmem + DPB, kmajor_desc(sV + kk * 32, 128), kmajor_desc(sb + L::SDO + kk * 32, 128), idS,
                               kk > 0);
                    tc_commit(&B.dp_full);
                }
                __syncwarp();
            }
        }
        if (!ok) cx.give_up();
        if (lane == 0) tc_commit(&B.drain[0]);   // TMEM is freed only after this warp's MMAs completed
        mbar_wait(&B.drain[0], 0, 500000000ull);
    } else if (warp == 2) {
        // ---------------- gradient issuer (whole warp): dV and dK
        constexpr uint32_t idG = idesc_bf16(128, 64, false, true);
        int gt = 0;
        bool ok = true;
        for (int ci = 0; ok; ++ci) {
            if (!cx.waitw(&B.res_full, ci & 1)) { ok = false; break; }
            const int it = B.item_of;
            __syncwarp();
            if (lane == 0) mbar_arrive(&B.idx_taken);
            if (it < 0) break;
            const int nq = p.plan.items[it].w;
            for (int t = 0; t < nq; ++t, ++gt) {
                const int st = gt % NST;
                const uint32_t sb = smem_u32(smem + L::STAGE0 + st * L::STAGE);
                // dV += P^T dO
                if (!cx.waitw(&B.p_full, gt & 1)) { ok = false; break; }
                // the first MMA of an item overwrites dV / dK: the previous item's epilogue must have read them
                if (t == 0 && ci >= 1 && !cx.waitw(&B.acc_free, (ci - 1) & 1)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        mma_ts(tmem + DV, tmem + SB + pcol(kk), mnmajor128_desc(sb + L::SDO + kk * 2048), idG,
                               (t > 0 || kk > 0) ? 1u : 0u);
                    tc_commit(&B.pv_done);
                }
                __syncwarp();
                // dK += dS^T Q
                if (!cx.waitw(&B.ds_ready, gt & 1)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        mma_ts(tmem + DK, tmem + DPB + pcol(kk), mnmajor128_desc(sb + L::SQ + kk * 2048), idG,
                               (t > 0 || kk > 0) ? 1u : 0u);
                    tc_commit(&B.dp_free);
                    tc_commit(&B.empty[st]);   // the stage's last readers were dV and dK
                }
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) tc_commit(&B.acc_done);   // every item, so the phases stay in step
            __syncwarp();
        }
        if (!ok) cx.give_up();
        if (lane == 0) tc_commit(&B.drain[1]);
        mbar_wait(&B.drain[1], 0, 500000000ull);
    } else if (warp < kElemWarp0) {
        // ---------------- dQ issuer (whole warp): dQ (| aug-dim gradient) = dS [K | K_aug]
        // once dS is in shared memory and the drain warps took the previous tile's
        constexpr uint32_t idQ = idesc_bf16(128, L::DQN, true, true);
        int gt = 0;
        bool ok = true;
        for (int ci = 0; ok; ++ci) {
            if (!cx.waitw(&B.res_full, ci & 1)) { ok = false; break; }
            const int it = B.item_of;
            __syncwarp();
            if (lane == 0) mbar_arrive(&B.idx_taken);
            if (it < 0) break;
            const int nq = p.plan.items[it].w;
            for (int t = 0; t < nq; ++t, ++gt) {
                if (!cx.waitw(&B.ds_ready, gt & 1)) { ok = false; break; }
                if (gt >= 1 && !cx.waitw(&B.dq_free, (gt - 1) & 1)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        mma_ss(tmem + DQ, mnmajor128_desc(sDS + kk * 2048), mnmajor32_desc(sK + kk * 512), idQ,
                               kk > 0 ? 1u : 0u);
                    tc_commit(&B.dq_full);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) tc_commit(&B.acc_done);   // the item's dQ MMAs read K: the residents wait for them too
            __syncwarp();
        }
        if (!ok) cx.give_up();
        if (lane == 0) tc_commit(&B.drain[2]);
        mbar_wait(&B.drain[2], 0, 500000000ull);
    } else if (warp < kDrainWarp0) {
        // ---------------- elementwise: thread = kv row c, tile columns [32qc, 32qc+32)
        const int quad = warp & 3;
        const int qc = (warp - kElemWarp0) >> 2;
        const int c = quad * 32 + lane;
        const uint32_t lb = (uint32_t)(quad * 32) << 16;
        const bool have_docs = p.docs != nullptr;
        const uint64_t c2 = f2_pack(p.scale_log2, p.scale_log2);
        // this thread's row of the dS tile (MN-major, 128-byte swizzle): two 16-byte chunks per 16 columns
        uint8_t *ds_row = smem + L::DS + (qc >> 1) * 16384 + c * 128;
        const int ch0 = (qc & 1) * 4;                   // 16-byte chunk of column 32qc within its half
        int gt = 0;
        bool alive = true;
        for (int ci = 0; alive; ++ci) {
            if (!cx.waitw(&B.res_full, ci & 1)) { alive = false; break; }
            const int it = B.item_of;
            __syncwarp();
            if (lane == 0) mbar_arrive(&B.idx_taken);
            if (it < 0) break;
            const int4 item = p.plan.items[it];
            const int slot = p.plan.item_slot[it];
            const int h = item.x, kb = item.y, nq = item.w;
            const int j = kb * BM + c;
            const int doc_j = have_docs ? p.docs[j] : 0;
            const float kpos_j = SLOPE ? __bfloat162float(__float2bfloat16_rn(__fmul_rn((float)j, p.s_aug))) : 0.f;
            for (int t = 0; t < nq; ++t, ++gt) {
                const int st = gt % NST;
                if (!cx.waitw(&B.full[st], (gt / NST) & 1)) { alive = false; break; }
                const int qb = B.stage_blk[st];
                const int mk = B.stage_mk[st];
                const uint8_t *sbp = smem + L::STAGE0 + st * L::STAGE;
                const int i0 = qb * BM + qc * 32;
                const int lim = j - i0;                  // column e visible iff e >= lim (causal: j <= i)
                const float4 *LS = reinterpret_cast<const float4 *>(sbp + L::SLSE) + qc * 8;
                const float4 *DL = reinterpret_cast<const float4 *>(sbp + L::SDEL) + qc * 8;
                // S^T -> registers; P; P^T back over the warp's own (already read) columns:
                // 16-column chunk cc at columns [32qc + 8cc, +8) as bf16 pairs
                if (!cx.waitw(&B.s_full, gt & 1)) { alive = false; break; }
                tc_fence_after();
                float s[32];
                {
                    uint32_t r[32];
                    tmem_ld32(tmem + lb + SB + qc * 32, r);
                    tmem_wait_ld();
                    pin(r);
#pragma unroll
                    for (int e = 0; e < 32; ++e) s[e] = __uint_as_float(r[e]);
                }
                // score_mod: slope, Δ_main, width of this thread's 32 q rows
                const float *spar = reinterpret_cast<const float *>(sbp + L::SPAR) + qc * 32;
                const SmodCols sc0{spar, spar + 128, spar + 256}, sc1{spar + 16, spar + 144, spar + 272};
                if (mk == MASK_FULL) {
                    p_piece<false, SM>(s, LS, c2, mk, lim, p.docs, i0, doc_j, sc0, p.bias2, p.gate_lambda, p.gate_itau);
                    p_piece<false, SM>(s + 16, LS + 4, c2, mk, lim - 16, p.docs, i0 + 16, doc_j, sc1, p.bias2,
                                       p.gate_lambda, p.gate_itau);
                } else {
                    p_piece<true, SM>(s, LS, c2, mk, lim, p.docs, i0, doc_j, sc0, p.bias2, p.gate_lambda, p.gate_itau);
                    p_piece<true, SM>(s + 16, LS + 4, c2, mk, lim - 16, p.docs, i0 + 16, doc_j, sc1, p.bias2,
                                      p.gate_lambda, p.gate_itau);
                }
                {
                    uint32_t w[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) w[e] = pack_bf16(s[2 * e], s[2 * e + 1]);
                    tmem_st16(tmem + lb + SB + qc * 32, w);
                }
                tmem_wait_st();
                tc_fence_before();
                // the gradient issuer consumed the previous tile's P^T (its dV MMAs completed)
                // before this arrival starts the next phase
                if (gt >= 1 && !cx.waitw(&B.pv_done, (gt - 1) & 1)) { alive = false; break; }
                mbar_arrive_warp(&B.p_full);
                // dP^T -> registers; dS = P (dP - delta); dS^T as bf16 pairs over the warp's
                // first 16 dP^T columns and dS into the shared-memory tile
                if (!cx.waitw(&B.dp_full, gt & 1)) { alive = false; break; }
                tc_fence_after();
                float d[32];
                {
                    uint32_t r[32];
                    tmem_ld32(tmem + lb + DPB + qc * 32, r);
                    tmem_wait_ld();
                    pin(r);
#pragma unroll
                    for (int e = 0; e < 32; ++e) d[e] = __uint_as_float(r[e]);
                }
                ds_piece(s, d, DL);
                ds_piece(s + 16, d + 16, DL + 4);
                if constexpr (SLOPE) {
                    // slope column of the aug-dim gradient in fp32 from the unrounded dS,
                    // against positions relative to each query row: sum_j dS_ij = 0 in exact
                    // arithmetic, so subtracting k_aug[i] changes nothing but the rounding,
                    // which would otherwise amplify the small residual of that sum by ~i*s
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        float v[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            const float kpos_i =
                                __bfloat162float(__float2bfloat16_rn(__fmul_rn((float)(i0 + 16 * cc + e), p.s_aug)));
                            v[e] = d[16 * cc + e] * (kpos_j - kpos_i);
                        }
                        const float col = warp_column_sums16(v);
                        if (lane < 16) atomicAdd(p.slope_acc + (int64_t)h * p.T + i0 + 16 * cc + lane, col);
                    }
                }
                if constexpr (SM != 0) {
                    // gradients of the per-row score_mod terms, summed over this tile's kv rows
                    // (the warp's 32 lanes) per q row: dS Δ for the slope; for the gate
                    // dS gate'(u) sign(Δ - Δ_main) and dS gate'(u), scaled in the finish kernel
                    const int64_t rowq = (int64_t)h * p.T + i0;
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        float v[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) v[e] = d[16 * cc + e] * (float)(16 * cc + e - lim);
                        const float col = warp_column_sums16(v);
                        if (lane < 16) atomicAdd(p.slope_acc + rowq + 16 * cc + lane, col);
                        if constexpr (SM >= 2) {
                            float vg[16], vd[16];
#pragma unroll
                            for (int e = 0; e < 16; ++e) {
                                const int ee = 16 * cc + e;
                                const float dl = (float)(ee - lim), dm = spar[128 + ee];
                                const float u = (fabsf(dl - dm) - spar[256 + ee]) * p.gate_itau;
                                float gp;
                                if constexpr (SM == 3) {
                                    gp = u > 0.f ? 1.f : 0.f;
                                } else {
                                    gp = u > 20.f ? 1.f : __frcp_rn(1.f + ex2(-u * kLog2e));
                                }
                                vg[e] = d[ee] * gp;
                                vd[e] = dl > dm ? vg[e] : (dl < dm ? -vg[e] : 0.f);
                            }
                            const float cg = warp_column_sums16(vg);
                            const float cd = warp_column_sums16(vd);
                            if (lane < 16) {
                                atomicAdd(p.w_acc + rowq + 16 * cc + lane, cg);
                                atomicAdd(p.dm_acc + rowq + 16 * cc + lane, cd);
                            }
                        }
                    }
                }
                {
                    uint32_t w[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) w[e] = pack_bf16(d[2 * e], d[2 * e + 1]);
                    tmem_st16(tmem + lb + DPB + qc * 32, w);
                    // the dS tile in shared memory is free once the previous tile's dQ MMAs completed
                    if (gt >= 1 && !cx.waitw(&B.dq_full, (gt - 1) & 1)) { alive = false; break; }
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4)
                        *reinterpret_cast<uint4 *>(ds_row + (((ch0 + q4) ^ (c & 7)) << 4)) =
                            make_uint4(w[4 * q4], w[4 * q4 + 1], w[4 * q4 + 2], w[4 * q4 + 3]);
                }
                tmem_wait_st();
                fence_async_smem();
                tc_fence_before();
                mbar_arrive_warp(&B.ds_ready);
            }
            if (!alive) break;
            // ---------------- epilogue of the item: dV, dK * scale
            if (!cx.waitw(&B.acc_done, ci & 1)) { alive = false; break; }
            tc_fence_after();
            const bool have = nq > 0;
            const int half = qc >> 1, c32 = (qc & 1) * 32;
            const uint32_t acc = tmem + lb + (half == 0 ? DV : DK) + c32;
            const float mul = half == 0 ? 1.f : p.scale;
            __nv_bfloat16 *dst = (half == 0 ? p.dv + (int64_t)h * p.dv_sh + (int64_t)j * p.dv_st
                                            : p.dk + (int64_t)h * p.dk_sh + (int64_t)j * p.dk_st) + c32;
            if (slot < 0) {
                store_row<32>(acc, mul, dst, have);
            } else {
                // a chunk of a split row: add into the row's fp32 slot; the last chunk writes bf16
                float *part = p.plan.partial + ((size_t)slot * BM + c) * 128 + qc * 32;
                if (have) {
                    uint32_t o[32];
                    tmem_ld32_nw(acc, o);
                    tmem_wait_ld();
                    pin(o);
#pragma unroll
                    for (int e = 0; e < 32; ++e) atomicAdd(part + e, __uint_as_float(o[e]) * mul);
                }
                __threadfence();
                elem_bar();
                if (threadIdx.x == 32 * kElemWarp0) {
                    const int done = atomicAdd(p.plan.slot_done + slot, 1);
                    B.last_flag = (done == p.plan.slot_chunks[slot] - 1) ? 1 : 0;
                }
                elem_bar();
                const bool last = B.last_flag != 0;
                elem_bar();   // every thread read the flag before a later item writes it again
                if (last) {
                    __threadfence();
                    uint32_t w[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) w[e] = pack_bf16(__ldcg(part + 2 * e), __ldcg(part + 2 * e + 1));
                    uint4 *dd = reinterpret_cast<uint4 *>(dst);
#pragma unroll
                    for (int e = 0; e < 4; ++e) dd[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
                }
            }
            tc_fence_before();
            mbar_arrive_warp(&B.acc_free);   // dV / dK read
        }
    } else {
        // ---------------- dQ drain: the 32 q rows of this warp's lane quadrant, DQN fp32 columns
        // each, added into the accumulator 16 columns at a time: TMEM -> registers (a row per
        // thread) -> a 32 x 16 box in shared memory (64-byte swizzle, so the row-per-lane
        // stores are conflict free) -> one TMA tensor reduce-add of the box.  The warp's
        // boxes rotate; a box is rewritten once the reduce that read it is done reading.
        // The q blocks come from the same bitmap walk the producer makes.
        const int quad = warp & 3;
        const uint32_t lb = (uint32_t)(quad * 32) << 16;
        constexpr int DQN = L::DQN;
        uint8_t *stg = smem + L::DRN + (warp - kDrainWarp0) * (kDrainBoxes * 2048);
        int issued = 0;                                  // reduces issued by lane 0 (bulk groups)
        int gt = 0;
        bool alive = true;
        for (int ci = 0; alive; ++ci) {
            if (!cx.waitw(&B.res_full, ci & 1)) { alive = false; break; }
            const int it = B.item_of;
            __syncwarp();
            if (lane == 0) mbar_arrive(&B.idx_taken);
            if (it < 0) break;
            const int4 item = p.plan.items[it];
            const int h = item.x, kb = item.y, first = item.z, nq = item.w;
            const uint32_t *brow = p.q_bitmap + ((int64_t)h * p.QB + kb) * p.words;
            int w;
            uint32_t bits;
            seek_rank(brow, p.words, first, w, bits);
            for (int t = 0; t < nq; ++t, ++gt) {
                const int qb = next_bit(brow, p.words, w, bits);
                if (!cx.waitw(&B.dq_full, gt & 1)) { alive = false; break; }
                tc_fence_after();
                const int row0 = (int)((int64_t)h * p.T + (int64_t)qb * BM + quad * 32);
#pragma unroll
                for (int c0 = 0; c0 < DQN; c0 += 16) {
                    uint8_t *box = stg + (issued % kDrainBoxes) * 2048;
                    if (lane == 0 && issued >= kDrainBoxes) bulk_wait_group_read<kDrainBoxes - 1>();   // this box's previous reduce
                    __syncwarp();
                    uint32_t o[16];
                    tmem_ld16(tmem + lb + DQ + c0, o);
                    tmem_wait_ld();
                    pin(o);
                    if (c0 + 16 >= DQN) {
                        tc_fence_before();
                        mbar_arrive_warp(&B.dq_free);   // the accumulator is in registers
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        *reinterpret_cast<uint4 *>(box + lane * 64 + ((e ^ ((lane >> 1) & 3)) << 4)) =
                            make_uint4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3]);
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0 && qb >= 0) {
                        tma_reduce_add_2d(&maps.dqa, box, c0, row0);
                        bulk_commit_group();
                    }
                    ++issued;
                }
            }
        }
        if (lane == 0) bulk_wait_group_all();            // every reduce completed before the CTA exits
    }
    __syncwarp();   // every warp reaches the CTA barrier converged (the producer ran on lane 0 alone)
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ============================================================================ dK/dV work plan
// per (h, kb) row: number of q blocks that see it
__global__ void plan_count_kernel(const uint32_t *__restrict__ bm, int rows, int words, int32_t *__restrict__ nq) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= rows) return;
    int c = 0;
    for (int w = lane; w < words; w += 32) c += __popc(bm[(int64_t)row * words + w]);
#pragma unroll
    for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) nq[row] = c;
}

__device__ int block_exclusive_scan(int v, int *sh, int &total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh[w] = x;
    __syncthreads();
    if (w == 0) {
        int y = lane < nw ? sh[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int z = __shfl_up_sync(0xffffffffu, y, o);
            if (lane >= o) y += z;
        }
        sh[lane] = y;
    }
    __syncthreads();
    const int excl = x - v + (w > 0 ? sh[w - 1] : 0);
    total = sh[nw - 1];
    __syncthreads();
    return excl;
}

// one CTA: split items (long rows) first, then one item per remaining row
__global__ void __launch_bounds__(1024) plan_items_kernel(const int32_t *__restrict__ nq, int rows, int KB,
                                                          Plan plan, int4 *items, int32_t *item_slot,
                                                          int32_t *slot_chunks, int32_t *n_items) {
    __shared__ int sh[32];
    const int per = (rows + blockDim.x - 1) / blockDim.x;
    const int r0 = threadIdx.x * per, r1 = min(rows, r0 + per);
    for (int i = threadIdx.x; i < kSlotCap; i += blockDim.x) plan.slot_done[i] = 0;
    if (threadIdx.x == 0) plan.next_item[0] = plan.next_item[1] = 0;   // dK/dV and dQ item counters
    int nsplit = 0;
    for (int r = r0; r < r1; ++r) nsplit += nq[r] > kChunk;
    int tot;
    const int slot0 = block_exclusive_scan(nsplit, sh, tot);
    int ns_items = 0, nu_items = 0, slot = slot0;
    for (int r = r0; r < r1; ++r) {
        const int n = nq[r];
        if (n > kChunk && slot < kSlotCap) {
            ns_items += (n + kChunk - 1) / kChunk;
            ++slot;
        } else {
            nu_items += 1;
            if (n > kChunk) ++slot;
        }
    }
    int tot_s, tot_u;
    const int s_base = block_exclusive_scan(ns_items, sh, tot_s);
    const int u_base = block_exclusive_scan(nu_items, sh, tot_u);
    int so = s_base, uo = tot_s + u_base;
    slot = slot0;
    for (int r = r0; r < r1; ++r) {
        const int n = nq[r];
        const int h = r / KB, kb = r - h * KB;
        if (n > kChunk && slot < kSlotCap) {
            const int nc = (n + kChunk - 1) / kChunk;
            slot_chunks[slot] = nc;
            for (int c = 0; c < nc; ++c) {
                items[so] = make_int4(h, kb, c * kChunk, min(kChunk, n - c * kChunk));
                item_slot[so] = slot;
                ++so;
            }
            ++slot;
        } else {
            items[uo] = make_int4(h, kb, 0, n);
            item_slot[uo] = -1;
            ++uo;
            if (n > kChunk) ++slot;
        }
    }
    if (threadIdx.x == 0) *n_items = tot_s + tot_u;
}

// ============================================================================ finish
// One warp per (head, row): dq = bf16(scale * acc[0:64]); the aug-dim gradient
// g = scale * acc[64:] -> dcoeff_cos[k] = s (g_k cos_ik + g_{K+k} sin_ik),
// dcoeff_sin[k] = s (g_k sin_ik - g_{K+k} cos_ik) (q_aug = s [A c + B s', A s' - B c, -slope]),
// dslope = -s * scale * (the fp32 slope sums).
struct FinishParams {
    const float *acc;
    int ld, H, T, K, tab_len;
    float scale, s_aug;
    __nv_bfloat16 *dq;
    int64_t dq_sh, dq_st;
    const uint16_t *cos_tab, *sin_tab;
    float *dcoeff_cos, *dcoeff_sin;
    const float *slope_acc;
    float *dslope;
    // score_mod: dslope = beta * sum dS (i - j); dΔ_main / dwidth = beta lambda / tau * the
    // gate sums; db0 = 0 (a per-row constant of the scores: softmax is invariant to it)
    int smod;
    float beta, gate_k;
    const float *dm_acc, *w_acc;
    float *ddelta_main, *dwidth, *db0;
};

__global__ void finish_kernel(const FinishParams f) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= (int64_t)f.H * f.T) return;
    const int h = (int)(row / f.T), i = (int)(row % f.T);
    const float *a = f.acc + row * f.ld;
    if (lane < 16) {
        const float4 v = *reinterpret_cast<const float4 *>(a + 4 * lane);
        uint2 o = make_uint2(pack_bf16(v.x * f.scale, v.y * f.scale), pack_bf16(v.z * f.scale, v.w * f.scale));
        *reinterpret_cast<uint2 *>(f.dq + h * f.dq_sh + (int64_t)i * f.dq_st + 4 * lane) = o;
    } else if (f.dcoeff_cos) {
        for (int k = lane - 16; k < f.K; k += 16) {
            const float g0 = a[64 + k] * f.scale, g1 = a[64 + f.K + k] * f.scale;
            const float cv = bf16_to_f32(f.cos_tab[(int64_t)k * f.tab_len + i]);
            const float sv = bf16_to_f32(f.sin_tab[(int64_t)k * f.tab_len + i]);
            f.dcoeff_cos[row * f.K + k] = f.s_aug * (g0 * cv + g1 * sv);
            f.dcoeff_sin[row * f.K + k] = f.s_aug * (g0 * sv - g1 * cv);
        }
    }
    if (lane == 0) {
        if (f.smod) {
            if (f.dslope) f.dslope[row] = f.beta * f.slope_acc[row];
            if (f.ddelta_main) f.ddelta_main[row] = f.gate_k * f.dm_acc[row];
            if (f.dwidth) f.dwidth[row] = f.gate_k * f.w_acc[row];
            if (f.db0) f.db0[row] = 0.f;
        } else if (f.dslope) {
            f.dslope[row] = -f.s_aug * (f.slope_acc[row] * f.scale);
        }
    }
}

}  // namespace tcbwd

namespace tchost {

// Workspace of the backward: delta, lse*log2(e), the work plan, the dK/dV
// slot partials, the fp32 dQ accumulator [H, T, 64 + DA] and the fp32 slope
// sums [H, T].
struct BwdWorkspace {
    size_t delta, lse2, nq, items, item_slot, n_items, slot_chunks, slot_done, partial, par, dq_acc, slope_acc,
        dm_acc, w_acc, total;
    int max_items, dq_ld;
};

// smod: the score_mod mode's per-row parameters [3][H*T] and gate sums [2][H*T]
BwdWorkspace bwd_workspace(int H, int T, int block_size, int d_aug, bool smod) {
    auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
    BwdWorkspace w;
    const int QB = T / block_size;
    w.max_items = H * QB + tcbwd::kSlotCap * ((QB + tcbwd::kChunk - 1) / tcbwd::kChunk);
    w.dq_ld = 64 + d_aug;
    size_t o = 0;
    w.delta = o;       o += up((size_t)H * T * 4);
    w.lse2 = o;        o += up((size_t)H * T * 4);
    w.nq = o;          o += up((size_t)H * QB * 4);
    w.items = o;       o += up((size_t)w.max_items * 16);
    w.item_slot = o;   o += up((size_t)w.max_items * 4);
    w.n_items = o;     o += up(16);
    w.slot_chunks = o; o += up((size_t)tcbwd::kSlotCap * 4);
    w.slot_done = o;   o += up((size_t)tcbwd::kSlotCap * 4);
    w.partial = o;     o += up((size_t)tcbwd::kSlotCap * 128 * 128 * 4);
    w.par = o;         o += smod ? up((size_t)3 * H * T * 4) : 0;
    w.dq_acc = o;      o += up((size_t)H * T * w.dq_ld * 4);
    w.slope_acc = o;   o += up((size_t)H * T * 4);
    w.dm_acc = o;      o += smod ? up((size_t)H * T * 4) : 0;
    w.w_acc = o;       o += smod ? up((size_t)H * T * 4) : 0;
    w.total = o;
    return w;
}

template <int DA, bool SLOPE, int SM>
int launch_bwd(const ScopeAttnArgs &a, cudaStream_t s) {
    const int QB = a.T / 128;
    const BwdWorkspace ws = bwd_workspace(a.H, a.T, 128, DA, SM != 0);
    uint8_t *base = reinterpret_cast<uint8_t *>(a.workspace);
    float *delta = reinterpret_cast<float *>(base + ws.delta);
    float *lse2 = reinterpret_cast<float *>(base + ws.lse2);
    float *dq_acc = reinterpret_cast<float *>(base + ws.dq_acc);
    float *slope_acc = reinterpret_cast<float *>(base + ws.slope_acc);
    const int64_t rows = (int64_t)a.H * a.T;
    tcbwd::PrepSmod psm;
    std::memset(&psm, 0, sizeof(psm));
    if (SM) {
        psm.b0 = a.b0;
        psm.slope = a.slope;
        psm.dmain = SM >= 2 ? a.delta_main : nullptr;
        psm.width = SM >= 2 ? a.width : nullptr;
        psm.beta = a.beta;
        psm.par = reinterpret_cast<float *>(base + ws.par);
    }
    tcbwd::prep_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16 *>(a.out), a.o_sh, a.o_st, reinterpret_cast<const __nv_bfloat16 *>(a.dout),
        a.do_sh, a.do_st, a.lse, a.H, a.T, delta, lse2, psm);
    SCOPE_CHECK_LAUNCH();

    // work plan: long q lists are cut into chunks
    tcbwd::Plan plan;
    int32_t *nq = reinterpret_cast<int32_t *>(base + ws.nq);
    int4 *items = reinterpret_cast<int4 *>(base + ws.items);
    int32_t *item_slot = reinterpret_cast<int32_t *>(base + ws.item_slot);
    int32_t *n_items = reinterpret_cast<int32_t *>(base + ws.n_items);
    int32_t *slot_chunks = reinterpret_cast<int32_t *>(base + ws.slot_chunks);
    plan.n_items = n_items;
    plan.items = items;
    plan.item_slot = item_slot;
    plan.slot_chunks = slot_chunks;
    plan.slot_done = reinterpret_cast<int32_t *>(base + ws.slot_done);
    plan.partial = reinterpret_cast<float *>(base + ws.partial);
    plan.next_item = n_items + 1;   // the second word of the n_items allocation (256 bytes)
    const int prow = a.H * QB, words = (QB + 31) / 32;
    tcbwd::plan_count_kernel<<<(unsigned)((prow * 32 + 255) / 256), 256, 0, s>>>(a.q_bitmap, prow, words, nq);
    SCOPE_CHECK_LAUNCH();
    tcbwd::plan_items_kernel<<<1, 1024, 0, s>>>(nq, prow, QB, plan, items, item_slot, slot_chunks, n_items);
    SCOPE_CHECK_LAUNCH();
    if (cudaMemsetAsync(plan.partial, 0, (size_t)tcbwd::kSlotCap * 128 * 128 * 4, s) != cudaSuccess)
        return SCOPE_ERR_CUDA;
    // the dQ accumulator, the slope and gate sums start at zero (adjacent in the workspace)
    if (cudaMemsetAsync(dq_acc, 0, ws.total - ws.dq_acc, s) != cudaSuccess) return SCOPE_ERR_CUDA;

    tcbwd::Maps maps;
    std::memset(&maps, 0, sizeof(maps));
    bool ok = map3d(&maps.q, a.q, 64, a.T, a.H, a.q_st, a.q_sh, 64) &&
              map3d(&maps.k16, a.k, 64, a.T, a.H, a.k_st, a.k_sh, 16) &&
              map3d(&maps.v, a.v, 64, a.T, a.H, a.v_st, a.v_sh, 64) &&
              map3d(&maps.dout, a.dout, 64, a.T, a.H, a.do_st, a.do_sh, 64);
    if (DA) ok = ok && map3d(&maps.qa, a.q_aug, DA, a.T, a.H, DA, (int64_t)a.T * DA, 16) &&
                 map2d(&maps.ka, a.k_aug, DA, a.T, 16);
    ok = ok && map2d_f32_sw64(&maps.dqa, dq_acc, ws.dq_ld, (int64_t)a.H * a.T, 32);
    if (!ok) return SCOPE_ERR_ALIGN;

    tcbwd::Params p;
    std::memset(&p, 0, sizeof(p));
    p.H = a.H;
    p.T = a.T;
    p.QB = QB;
    p.words = words;
    p.q_bitmap = a.q_bitmap;
    p.block_info = a.block_info;
    p.docs = a.docs;
    p.lse2 = lse2;
    p.delta = delta;
    p.scale = a.scale;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.dk = reinterpret_cast<__nv_bfloat16 *>(a.dk);
    p.dk_sh = a.dk_sh;
    p.dk_st = a.dk_st;
    p.dv = reinterpret_cast<__nv_bfloat16 *>(a.dv);
    p.dv_sh = a.dv_sh;
    p.dv_st = a.dv_st;
    p.dq_acc = dq_acc;
    p.slope_acc = slope_acc;
    p.s_aug = (float)sqrt((double)a.beta / (double)a.scale);
    if (SM) {
        p.par = psm.par;
        p.dm_acc = reinterpret_cast<float *>(base + ws.dm_acc);
        p.w_acc = reinterpret_cast<float *>(base + ws.w_acc);
        p.bias2 = a.beta * 1.4426950408889634f;
        p.gate_lambda = a.gate_lambda;
        p.gate_itau = (a.gate_tau != 0.f) ? 1.f / a.gate_tau : 0.f;
    }
    p.plan = plan;
    p.err = a.err_flag;

    // each CTA takes all 512 TMEM columns, so ask for enough shared memory that a
    // second CTA never lands on the SM just to wait inside tcgen05.alloc
    const size_t kOneCtaPerSm = 120 * 1024;
    const size_t smem = std::max<size_t>(tcbwd::FL<DA, SM>::TOTAL + 1024, kOneCtaPerSm);
    if (cudaFuncSetAttribute(tcbwd::dkvq_kernel<DA, SLOPE, SM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return SCOPE_ERR_CUDA;
    int dev = 0, n_sm = 148;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return SCOPE_ERR_CUDA;
    // persistent: one CTA per SM walks the plan's items
    tcbwd::dkvq_kernel<DA, SLOPE, SM><<<std::min(ws.max_items, n_sm), tcbwd::kThreads, smem, s>>>(maps, p);
    SCOPE_CHECK_LAUNCH();

    tcbwd::FinishParams f;
    std::memset(&f, 0, sizeof(f));
    f.acc = dq_acc;
    f.ld = ws.dq_ld;
    f.H = a.H;
    f.T = a.T;
    f.scale = a.scale;
    f.s_aug = p.s_aug;
    f.dq = reinterpret_cast<__nv_bfloat16 *>(a.dq);
    f.dq_sh = a.dq_sh;
    f.dq_st = a.dq_st;
    if (DA && a.dcoeff_cos) {
        f.K = a.K;
        f.tab_len = a.tab_len;
        f.cos_tab = a.cos_tab;
        f.sin_tab = a.sin_tab;
        f.dcoeff_cos = a.dcoeff_cos;
        f.dcoeff_sin = a.dcoeff_sin;
        if (SLOPE) {
            f.slope_acc = slope_acc;
            f.dslope = a.dslope;
        }
    }
    if (SM) {
        f.smod = 1;
        f.beta = a.beta;
        f.gate_k = a.beta * p.gate_lambda * p.gate_itau;
        f.slope_acc = slope_acc;
        f.dm_acc = p.dm_acc;
        f.w_acc = p.w_acc;
        f.dslope = a.slope ? a.dslope : nullptr;
        f.ddelta_main = SM >= 2 ? a.ddelta_main : nullptr;
        f.dwidth = SM >= 2 ? a.dwidth : nullptr;
        f.db0 = a.b0 ? a.db0 : nullptr;
    }
    tcbwd::finish_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(f);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

}  // namespace tchost
}  // namespace scope

size_t scope_bwd_workspace_bytes(int H, int T, int block_size, int d_aug, bool smod) {
    return scope::tchost::bwd_workspace(H, T, block_size, d_aug, smod).total;
}

int scope_tc_smod(const ScopeAttnArgs &a);

int scope_tc_bwd(const ScopeAttnArgs &a, cudaStream_t s) {
    using namespace scope::tchost;
    const int sm = scope_tc_smod(a);
    if (sm) {
        const bool d16 = a.d_aug == 16;
        switch (sm) {
            case 1: return d16 ? launch_bwd<16, false, 1>(a, s) : launch_bwd<32, false, 1>(a, s);
            case 2: return d16 ? launch_bwd<16, false, 2>(a, s) : launch_bwd<32, false, 2>(a, s);
            default: return d16 ? launch_bwd<16, false, 3>(a, s) : launch_bwd<32, false, 3>(a, s);
        }
    }
    const bool slope = a.bias_mode == SCOPE_BIAS_QK_AUG && a.slope && a.dslope && a.dcoeff_cos;
    switch (a.bias_mode == SCOPE_BIAS_QK_AUG ? a.d_aug : 0) {
        case 0: return launch_bwd<0, false, 0>(a, s);
        case 16: return slope ? launch_bwd<16, true, 0>(a, s) : launch_bwd<16, false, 0>(a, s);
        case 32: return slope ? launch_bwd<32, true, 0>(a, s) : launch_bwd<32, false, 0>(a, s);
        case 48: return slope ? launch_bwd<48, true, 0>(a, s) : launch_bwd<48, false, 0>(a, s);
        case 64: return slope ? launch_bwd<64, true, 0>(a, s) : launch_bwd<64, false, 0>(a, s);
        default: return SCOPE_ERR_INVALID;
    }
}
