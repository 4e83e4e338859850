// Block-sparse SCOPE attention backward on the sm_100a tensor cores.
//
// Launches, all on the caller's stream:
//   prep   delta_i = sum_d dO_i . O_i  and  lse2_i = lse_i * log2(e)   (workspace)
//   plan   per (head, kv block) the number of q blocks that see it (from the
//          builder's q-side bitmap) and the dK/dV work items
//   dkv    persistent, one CTA per SM walking the work items (a kv block and a
//          run of the q blocks that see it, ascending): dV += P^T dO and
//          dK += dS^T Q in TMEM.
//   dq     persistent, one CTA per SM walking the (head, q block) items: the kv
//          list like the forward, dQ += dS K (and, for the qk_aug spectral bias,
//          the gradient of the augmented dims, turned into dcoeff_cos /
//          dcoeff_sin / dslope in the epilogue by the chain rule of
//          scoped_medium.py:380-421).
// dQ is computed by its own kernel rather than with atomics so every output
// is written once, deterministically.  A kv block that many q blocks see (a
// global / sink block is seen by every q block of its document) would make one
// dK/dV CTA walk a list of up to QB tiles; `plan` cuts such lists into chunks of
// at most kChunk q tiles handled by separate CTAs, whose fp32 partial sums meet
// in a small slot buffer that the last chunk of the row converts to bf16.
//
// Both kernels share one pipeline on whole 128x128 tiles (608 threads, one CTA
// per SM, all 512 TMEM columns): a producer warp (TMA), an S / dP issuing warp,
// a gradient issuing warp and sixteen elementwise warps (four per TMEM lane
// quadrant, 32 columns each in two chunks of 16).  S is double buffered in
// TMEM; dP is single buffered, read by every elementwise warp at the start of
// a tile and released at once, and the next dP is issued before the next S.
// P / dS go back into the S buffer as bf16 pairs within each chunk's own
// columns, where the gradient MMAs read them as their A operand (the even
// chunks' K steps as soon as they are written).  Every wait is bounded
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
constexpr int kElemWarps = 16;         // four per TMEM lane quadrant, 32 tile columns each
constexpr int kThreads = 32 * (kElemWarps + 3);   // producer, S/dP issuer, elementwise warps, gradient issuer
constexpr int kGradWarp = kElemWarps + 2;
constexpr int kElem = 32 * kElemWarps; // elementwise threads
constexpr int kChunk = 64;             // max q tiles per dK/dV work item
constexpr int kSlotCap = 128;          // max kv rows whose q list is split
constexpr uint32_t kTmemCols = 512;
// TMEM columns (one CTA per SM owns all 512):
//   [0, 256)    two S buffers: S (dq) or S^T (dkv) of a 128 x 128 tile, fp32;
//               P / dS of the 16 columns [16g, 16g+16) go back into those same
//               columns as bf16 pairs (dkv: P^T at 16g, dS^T at 16g + 8; dq: dS
//               at 16g), so every warp writes only over columns it has read
//   [256, 384)  DP: dP (dq) or dP^T (dkv) of the tile, fp32, one buffer
//   [384, 448)  ACC0: dV (dkv) | dQ (dq)
//   [448, 512)  ACC1: dK (dkv) | gradient of the qk_aug dims (dq)
// S is double buffered so S of tile j+1 is computed while the elementwise
// warps work on tile j; dP of tile j+1 starts once they have read dP of j.
constexpr uint32_t DPC = 256, ACC0 = 384, ACC1 = 448;
constexpr uint32_t kSmemBudget = 227 * 1024;   // dynamic shared memory per CTA
constexpr float kLog2e = 1.4426950408889634f;

__host__ __device__ constexpr uint32_t align1k(uint32_t x) { return (x + 1023u) & ~1023u; }
__device__ __forceinline__ uint32_t sbuf(int b) { return (uint32_t)b * 128u; }
// K step kk of the gradient contraction (16 tile columns, 8 packed TMEM
// columns) of the TMEM A operand starts at a_col(kk); in dkv the dS^T pairs
// follow at +8.
__device__ __forceinline__ uint32_t a_col(int kk) { return (uint32_t)(16 * kk); }

// ------------------------------------------------------------------ prep
__global__ void prep_kernel(const __nv_bfloat16 *__restrict__ out, int64_t o_sh, int64_t o_st,
                            const __nv_bfloat16 *__restrict__ dout, int64_t do_sh, int64_t do_st,
                            const float *__restrict__ lse, int H, int T, float *__restrict__ delta,
                            float *__restrict__ lse2) {
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
    const float l = lse[row];
    lse2[row] = (l == -INFINITY) ? INFINITY : l * kLog2e;   // rows that saw nothing get P = 0
}

struct Plan {
    const int32_t *n_items;   // [1]
    const int4 *items;        // (h, kb, first q rank, count)
    const int32_t *item_slot; // split slot or -1
    const int32_t *slot_chunks;
    int32_t *slot_done;
    float *partial;           // [kSlotCap][128 rows][128]: dV (64) | dK (64)
    int32_t *next_item;       // [2]: dK/dV, dQ items handed out beyond the first G (zeroed by the plan kernel)
};

struct Params {
    int H, T, QB, words, kv_stride;
    const uint32_t *q_bitmap;
    const int32_t *kv_num, *kv_idx;
    const int32_t *block_info, *docs;
    const float *lse2, *delta;
    float scale, scale_log2;
    __nv_bfloat16 *g0, *g1;           // dkv: dK, dV      dq: dQ, (unused)
    int64_t g0_sh, g0_st, g1_sh, g1_st;
    // dq epilogue for the qk_aug bias
    int K, has_slope, tab_len, tab_smem;   // tab_smem: table rows 16-byte aligned, staged by the producer
    const uint16_t *cos_tab, *sin_tab;
    float s_aug;
    float *dcoeff_cos, *dcoeff_sin, *dslope;
    Plan plan;
    int32_t *err;
};

struct Maps {
    CUtensorMap q, k, v, dout, qa, ka;
};

// helpers shared by both kernels ------------------------------------------------
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

// mbarriers and small shared state of a backward CTA
struct Bars {
    uint64_t res_full[2];              // a work item's resident tiles are in shared memory (buffer ci & 1)
    uint64_t acc_done;                 // every gradient MMA of a work item completed
    uint64_t acc_free[2];              // the epilogue of work item ci read the accumulators and is done
                                       // with resident buffer ci & 1 (elementwise arrivals)
    uint64_t full[4], empty[4];        // streamed stage ring
    uint64_t s_full[2];                // S of a tile is in its buffer
    uint64_t p_half[2];                // P / dS of the even 16-column chunks are back (elementwise arrivals)
    uint64_t p_full[2];                // P / dS of every chunk are back in the buffer (elementwise arrivals)
    uint64_t s_free[2];                // the gradient MMAs that read the buffer completed
    uint64_t dp_full;                  // dP of a tile is in DP
    uint64_t dp_free;                  // the elementwise warps have read DP (elementwise arrivals)
    uint64_t drain[2];                 // each issuing warp's MMAs completed (before TMEM is freed)
    volatile int stage_blk[4];         // block index of the tile in each stage
    volatile int stage_mk[4];          // its mask kind
    uint32_t tmem_slot;
    volatile int abort_flag, last_flag, pad;
    volatile int item_of[2];           // dkv: the work item in resident buffer b, -1 when none is left
    __device__ void init(int nst, int acc_free_count) {
        mbar_init(&res_full[0], 1);
        mbar_init(&res_full[1], 1);
        mbar_init(&acc_done, 1);
        mbar_init(&acc_free[0], acc_free_count);
        mbar_init(&acc_free[1], acc_free_count);
        for (int i = 0; i < nst; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_half[i], kElem);
            mbar_init(&p_full[i], kElem);
            mbar_init(&s_free[i], 1);
        }
        mbar_init(&dp_full, 1);
        mbar_init(&dp_free, kElem);
        mbar_init(&drain[0], 1);
        mbar_init(&drain[1], 1);
        abort_flag = 0;
        last_flag = 0;
        fence_mbar_init();
    }
};

// A warp's start of a tile: its 32 dP columns and the first 16 S columns of
// this thread's TMEM lane in one wait, so dP can be released right away
__device__ __forceinline__ void ld_tile_start(uint32_t ts, uint32_t tdp, uint32_t (&s0)[16], uint32_t (&dp0)[16],
                                              uint32_t (&dp1)[16]) {
    tmem_ld16(ts, s0);
    tmem_ld16(tdp, dp0);
    tmem_ld16(tdp + 16, dp1);
    tmem_wait_ld();
    pin(s0);
    pin(dp0);
    pin(dp1);
}
__device__ __forceinline__ void ld_cols16(uint32_t taddr, uint32_t (&r)[16]) {
    tmem_ld16(taddr, r);
    tmem_wait_ld();
    pin(r);
}
// 16 values as 8 bf16 pairs at taddr
__device__ __forceinline__ void st_bf16x16(uint32_t taddr, const float (&x)[16]) {
    uint32_t pk[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) pk[e] = pack_bf16(x[2 * e], x[2 * e + 1]);
    tmem_st8(taddr, pk);
}
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

// One 16-column piece of the dK/dV elementwise stage, thread = kv row j:
// P = exp2(S * scale*log2e - lse2), dS = P (dP - delta), masked when MASKED.
template <bool MASKED>
__device__ __forceinline__ void dkv_piece(float (&s)[16], float (&dp)[16], const float4 *LS, const float4 *DL,
                                          uint64_t c2, int mk, int lim, const int32_t *docs, int i0, int doc_j) {
#pragma unroll
    for (int e4 = 0; e4 < 4; ++e4) {
        const float4 l4 = LS[e4], d4 = DL[e4];
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
            const int e = e4 * 4 + 2 * q2;
            const uint64_t nl = q2 ? f2_pack(-l4.z, -l4.w) : f2_pack(-l4.x, -l4.y);
            const uint64_t nd = q2 ? f2_pack(-d4.z, -d4.w) : f2_pack(-d4.x, -d4.y);
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
            const float2 ds = f2_unpack(fmul2(f2_pack(p0, p1), fadd2(f2_pack(dp[e], dp[e + 1]), nd)));
            s[e] = p0;
            s[e + 1] = p1;
            dp[e] = ds.x;
            dp[e + 1] = ds.y;
        }
    }
}

// One 16-column piece of the dQ elementwise stage, thread = q row i; dS -> s.
template <bool MASKED>
__device__ __forceinline__ void dq_piece(float (&s)[16], const float (&dp)[16], uint64_t c2, uint64_t nl2,
                                         uint64_t nd2, int mk, int lim, bool bad, const int32_t *docs, int j0,
                                         int doc_i) {
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
        const float2 x = f2_unpack(ffma2(f2_pack(s[e], s[e + 1]), c2, nl2));
        float p0 = ex2(x.x), p1 = ex2(x.y);
        if (MASKED) {
            bool v0 = e <= lim && !bad, v1 = e + 1 <= lim && !bad;
            if (mk == MASK_DOCS && docs && !bad) {
                v0 = v0 && (__ldg(docs + j0 + e) == doc_i);
                v1 = v1 && (__ldg(docs + j0 + e + 1) == doc_i);
            }
            p0 = v0 ? p0 : 0.f;
            p1 = v1 ? p1 : 0.f;
        }
        const float2 ds = f2_unpack(fmul2(f2_pack(p0, p1), fadd2(f2_pack(dp[e], dp[e + 1]), nd2)));
        s[e] = ds.x;
        s[e + 1] = ds.y;
    }
}

// ============================================================================ dK / dV
// Persistent: one CTA per SM walks work items of the plan (its block index
// first, then the next unclaimed one from an atomic counter: the items range
// from 1 to kChunk q tiles), so that the next item's resident tiles load and
// its first tiles run while the previous item's epilogue drains.  The
// producer publishes each item's index with the resident buffer's barrier.  Resident per item (two
// buffers, item ci in buffer ci & 1): K, the k_aug dims, V.  Streamed per q tile
// (ring of NST stages, one tile counter across items): Q, the q_aug dims, dO,
// lse2, delta.
template <int DA>
struct KVL {
    static constexpr int NA = DA / 16;
    static constexpr uint32_t TILE = BM * HD * 2, ATILE = BM * 16 * 2;
    static constexpr uint32_t K = 0, KA = TILE, V = align1k(TILE + NA * ATILE);   // within a resident buffer
    static constexpr uint32_t RESB = align1k(V + TILE);
    static constexpr uint32_t STAGE0 = 2 * RESB;
    static constexpr uint32_t SQ = 0, SQA = TILE, SDO = align1k(TILE + NA * ATILE), SLSE = SDO + TILE,
                              SDEL = SLSE + 512;
    static constexpr uint32_t STAGE = align1k(SDEL + 512);
    static constexpr uint32_t EXTRA = 1024 + 1024;                  // barriers, base alignment
    static constexpr int NST = STAGE0 + 4 * STAGE + EXTRA <= kSmemBudget
                                   ? 4
                                   : (STAGE0 + 3 * STAGE + EXTRA <= kSmemBudget ? 3 : 2);
    static constexpr uint32_t BAR = STAGE0 + NST * STAGE;
    static constexpr uint32_t RES_BYTES = 2 * TILE + NA * ATILE;
    static constexpr uint32_t TOTAL = BAR + sizeof(Bars);
    static constexpr uint32_t Q_BYTES = 2 * TILE + NA * ATILE + 1024;
    static_assert(TOTAL + 1024 <= kSmemBudget, "shared memory");
};

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

template <int DA>
__global__ void __launch_bounds__(kThreads, 1) dkv_kernel(const __grid_constant__ Maps maps, const Params p) {
    using L = KVL<DA>;
    constexpr int NA = L::NA, NST = L::NST;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    Bars &B = *reinterpret_cast<Bars *>(smem + L::BAR);
    Ctx cx{&B.abort_flag, p.err};

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = *p.plan.n_items, G = gridDim.x;

    // acc_free of a resident buffer: the elementwise threads after the item's epilogue,
    // and each issuing warp once it has read the item's index
    if (threadIdx.x == 0) B.init(NST, kElem + 2);
    if (warp == 1) {
        tmem_alloc(&B.tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    __syncwarp();   // every warp reaches the CTA barrier converged (the producer ran on lane 0 alone)
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = B.tmem_slot;

    if (warp == 0) {
        // ---------------- producer: per item K / V into its resident buffer, then the q tiles
        // that see the kv block, ascending
        if (lane == 0) {
            int gt = 0, last_res = -1;
            bool ok = true;
            for (int ci = 0; ok; ++ci) {
                // the first item of each CTA is its block index, the rest are handed out in order
                const int it = ci == 0 ? (int)blockIdx.x : G + atomicAdd(p.plan.next_item, 1);
                const int rb = ci & 1;
                uint8_t *res = smem + rb * L::RESB;
                // buffer rb is free once every role is done with item ci - 2
                if (ci >= 2 && !cx.wait1(&B.acc_free[rb], ((ci >> 1) - 1) & 1)) break;
                if (last_res == ci - 2) last_res = -1;   // its tiles were consumed, so they landed
                B.item_of[rb] = it < n_items ? it : -1;
                if (it >= n_items) {
                    mbar_arrive(&B.res_full[rb]);      // publishes "no item left"
                    break;
                }
                const int4 item = p.plan.items[it];
                const int h = item.x, kb = item.y, first = item.z, nq = item.w;
                if (nq > 0) {
                    mbar_expect_tx(&B.res_full[rb], L::RES_BYTES);
                    tma_load_3d(&maps.k, res + L::K, &B.res_full[rb], 0, kb * BM, h);
#pragma unroll
                    for (int a = 0; a < NA; ++a)
                        tma_load_2d(&maps.ka, res + L::KA + a * L::ATILE, &B.res_full[rb], 16 * a, kb * BM);
                    tma_load_3d(&maps.v, res + L::V, &B.res_full[rb], 0, kb * BM, h);
                    last_res = ci;
                } else {
                    mbar_arrive(&B.res_full[rb]);      // keeps the buffer's phases in step
                }
                const uint32_t *brow = p.q_bitmap + ((int64_t)h * p.QB + kb) * p.words;
                int w;
                uint32_t bits;
                seek_rank(brow, p.words, first, w, bits);
                int t = 0;
                while (t < nq && w < p.words) {
                    if (!bits) {
                        if (++w < p.words) bits = brow[w];
                        continue;
                    }
                    const int qb = w * 32 + __ffs(bits) - 1;
                    bits &= bits - 1;
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
                    ++t;
                    ++gt;
                }
                if (ok && t < nq) {   // the plan promised more q blocks than the bitmap row holds
                    set_err(p.err, SCOPE_DEVERR_INDEX);
                    cx.give_up();
                    ok = false;
                }
            }
            // never leave the CTA with a TMA write still in flight
            if (last_res >= 0) mbar_wait(&B.res_full[last_res & 1], (last_res >> 1) & 1, 500000000ull);
            for (int j = (gt > NST ? gt - NST : 0); j < gt; ++j) mbar_wait(&B.full[j % NST], (j / NST) & 1, 500000000ull);
        }
    } else if (warp == 1) {
        // ---------------- S / dP issuer (the whole warp waits, lane 0 issues)
        constexpr uint32_t idS = idesc_bf16(128, 128, false, false);
        int gt = 0;
        bool ok = true;
        for (int ci = 0; ok; ++ci) {
            const int rb = ci & 1;
            if (!cx.waitw(&B.res_full[rb], (ci >> 1) & 1)) { ok = false; break; }
            const int it = B.item_of[rb];
            if (lane == 0) mbar_arrive(&B.acc_free[rb]);   // the index is read
            if (it < 0) break;
            const int nq = p.plan.items[it].w;
            const uint32_t res = smem_u32(smem + rb * L::RESB);
            const uint32_t sK = res + L::K, sKA = res + L::KA, sV = res + L::V;
            for (int t = 0; t < nq; ++t, ++gt) {
                const int st = gt % NST, b = gt & 1;
                if (!cx.waitw(&B.full[st], (gt / NST) & 1)) { ok = false; break; }
                const uint32_t sb = smem_u32(smem + L::STAGE0 + st * L::STAGE);
                // dP^T = V dO^T first: the elementwise warps release dP^T of the previous tile
                // as they start it, while S^T waits for the gradient MMAs of tile gt-2
                if (gt >= 1 && !cx.waitw(&B.dp_free, (gt - 1) & 1)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_ss(tmem + DPC, kmajor_desc(sV + kk * 32, 128), kmajor_desc(sb + L::SDO + kk * 32, 128), idS,
                               kk > 0);
                    tc_commit(&B.dp_full);
                }
                __syncwarp();
                // S^T = K Q^T (+ Kaug Qaug^T): 128 kv rows x 128 q columns
                if (gt >= 2 && !cx.waitw(&B.s_free[b], ((gt >> 1) - 1) & 1)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_ss(tmem + sbuf(b), kmajor_desc(sK + kk * 32, 128), kmajor_desc(sb + L::SQ + kk * 32, 128),
                               idS, kk > 0);
#pragma unroll
                    for (int a = 0; a < NA; ++a)
                        mma_ss(tmem + sbuf(b), kmajor_desc(sKA + a * L::ATILE, 32),
                               kmajor_desc(sb + L::SQA + a * L::ATILE, 32), idS, 1);
                    tc_commit(&B.s_full[b]);
                }
                __syncwarp();
            }
        }
        if (!ok) cx.give_up();
        if (lane == 0) tc_commit(&B.drain[0]);   // TMEM is freed only after this warp's MMAs completed
        mbar_wait(&B.drain[0], 0, 500000000ull);
    } else if (warp == kGradWarp) {
        // ---------------- gradient issuer (whole warp): a second issuing warp, so
        // the S / dP MMAs and these queue on the tensor pipe side by side
        constexpr uint32_t idG = idesc_bf16(128, 64, false, true);
        int gt = 0;
        bool ok = true;
        for (int ci = 0; ok; ++ci) {
            const int rb = ci & 1;
            if (!cx.waitw(&B.res_full[rb], (ci >> 1) & 1)) { ok = false; break; }
            const int it = B.item_of[rb];
            if (lane == 0) mbar_arrive(&B.acc_free[rb]);   // the index is read
            if (it < 0) break;
            const int nq = p.plan.items[it].w;
            for (int t = 0; t < nq; ++t, ++gt) {
                const int st = gt % NST, b = gt & 1;
                const uint32_t sb = smem_u32(smem + L::STAGE0 + st * L::STAGE);
                // dV += P^T dO, dK += dS^T Q over the tile's 128 q rows: the even K steps
                // (16-column chunks) as soon as every warp has written them, then the odd
                for (int half = 0; half < 2; ++half) {
                    if (!cx.waitw(half ? &B.p_full[b] : &B.p_half[b], (gt >> 1) & 1)) { ok = false; break; }
                    // the first MMA of an item overwrites the accumulators: the previous
                    // item's epilogue must have read them
                    if (!half && t == 0 && ci >= 1 && !cx.waitw(&B.acc_free[(ci - 1) & 1], ((ci - 1) >> 1) & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (lane == 0) {
#pragma unroll
                        for (int k2 = 0; k2 < 4; ++k2) {
                            const int kk = 2 * k2 + half;
                            const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
                            mma_ts(tmem + ACC0, tmem + sbuf(b) + a_col(kk), mnmajor128_desc(sb + L::SDO + kk * 2048),
                                   idG, acc);
                            mma_ts(tmem + ACC1, tmem + sbuf(b) + a_col(kk) + 8, mnmajor128_desc(sb + L::SQ + kk * 2048),
                                   idG, acc);
                        }
                        if (half) {
                            tc_commit(&B.s_free[b]);
                            tc_commit(&B.empty[st]);
                        }
                    }
                    __syncwarp();
                }
                if (!ok) break;
            }
            if (!ok) break;
            if (lane == 0) tc_commit(&B.acc_done);   // every item, so the epilogue's phases stay in step
            __syncwarp();
        }
        if (!ok) cx.give_up();
        if (lane == 0) tc_commit(&B.drain[1]);
        mbar_wait(&B.drain[1], 0, 500000000ull);
    } else {
        // ---------------- elementwise: thread = kv row c, tile columns [32qc, 32qc+32) in two chunks of 16
        const int quad = warp & 3;
        const int qc = (warp - 2) >> 2;
        const int c = quad * 32 + lane;
        const uint32_t lb = (uint32_t)(quad * 32) << 16;
        const bool have_docs = p.docs != nullptr;
        const uint64_t c2 = f2_pack(p.scale_log2, p.scale_log2);
        int gt = 0;
        bool alive = true;
        for (int ci = 0; alive; ++ci) {
            const int rb = ci & 1;
            if (!cx.waitw(&B.res_full[rb], (ci >> 1) & 1)) { alive = false; break; }
            const int it = B.item_of[rb];
            if (it < 0) break;
            const int4 item = p.plan.items[it];
            const int slot = p.plan.item_slot[it];
            const int h = item.x, kb = item.y, nq = item.w;
            const int j = kb * BM + c;
            const int doc_j = have_docs ? p.docs[j] : 0;
            for (int t = 0; t < nq; ++t, ++gt) {
                const int st = gt % NST, b = gt & 1;
                if (!cx.waitw(&B.full[st], (gt / NST) & 1)) { alive = false; break; }
                const int qb = B.stage_blk[st];
                const int mk = B.stage_mk[st];
                if (!cx.waitw(&B.s_full[b], (gt >> 1) & 1) || !cx.waitw(&B.dp_full, gt & 1)) { alive = false; break; }
                tc_fence_after();
                const uint8_t *sbp = smem + L::STAGE0 + st * L::STAGE;
                uint32_t rs[16], rp0[16], rp1[16];
                ld_tile_start(tmem + lb + sbuf(b) + qc * 32, tmem + lb + DPC + qc * 32, rs, rp0, rp1);
                tc_fence_before();
                mbar_arrive_warp(&B.dp_free);           // this warp's dP^T columns are in registers
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int col0 = qc * 32 + cc * 16;  // q row within the tile of the chunk's first column
                    const uint32_t tc = tmem + lb + sbuf(b) + col0;
                    if (cc == 1) ld_cols16(tc, rs);
                    float s[16], dp[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        s[e] = __uint_as_float(rs[e]);
                        dp[e] = __uint_as_float(cc ? rp1[e] : rp0[e]);
                    }
                    const float4 *LS = reinterpret_cast<const float4 *>(sbp + L::SLSE) + col0 / 4;
                    const float4 *DL = reinterpret_cast<const float4 *>(sbp + L::SDEL) + col0 / 4;
                    const int i0 = qb * BM + col0;
                    const int lim = j - i0;              // column e visible iff e >= lim (causal: j <= i)
                    if (mk == MASK_FULL) dkv_piece<false>(s, dp, LS, DL, c2, mk, lim, p.docs, i0, doc_j);
                    else dkv_piece<true>(s, dp, LS, DL, c2, mk, lim, p.docs, i0, doc_j);
                    st_bf16x16(tc, s);                   // P^T pairs, then dS^T pairs, over the chunk's own columns
                    st_bf16x16(tc + 8, dp);
                    if (cc == 0) {
                        tmem_wait_st();
                        tc_fence_before();
                        mbar_arrive_warp(&B.p_half[b]);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive_warp(&B.p_full[b]);
            }
            if (!alive) break;
            // ---------------- epilogue of the item
            if (!cx.waitw(&B.acc_done, ci & 1)) { alive = false; break; }
            tc_fence_after();
            const bool have = nq > 0;
            // dV from ACC0 (quarters 0, 1), dK * scale from ACC1 (quarters 2, 3): 32 columns per warp
            const int half = qc >> 1, c32 = (qc & 1) * 32;
            const uint32_t acc = tmem + lb + (half == 0 ? ACC0 : ACC1) + c32;
            const float mul = half == 0 ? 1.f : p.scale;
            __nv_bfloat16 *dst = (half == 0 ? p.g1 + (int64_t)h * p.g1_sh + (int64_t)j * p.g1_st
                                            : p.g0 + (int64_t)h * p.g0_sh + (int64_t)j * p.g0_st) + c32;
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
                if (threadIdx.x == 64) {
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
                    uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
                    for (int e = 0; e < 4; ++e) d[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
                }
            }
            tc_fence_before();
            mbar_arrive_warp(&B.acc_free[rb]);   // accumulators read, resident buffer rb released
        }
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

// ============================================================================ dQ
// Persistent: one CTA per SM walks the work items (head, q block): its block
// index first, then the next unclaimed one from an atomic counter (kv lists
// run from 1 to ~80 tiles), so that the next item's resident tiles load and
// its first tiles run while the previous item's epilogue drains.  Resident per item
// (two buffers, item ci in buffer ci & 1): Q, the q_aug dims, dO and the item's
// rows of the cos / sin tables.  Streamed per kv tile (ring of NST stages, one
// tile counter across items): K, the k_aug dims, V.
template <int DA>
struct QL {
    static constexpr int NA = DA / 16;
    static constexpr int KM = DA > 0 ? DA / 2 : 1;                 // coefficients per row, K <= DA / 2
    static constexpr int KM4 = (KM + 3) / 4;                        // per elementwise warp of a quadrant
    static constexpr uint32_t TILE = BM * HD * 2, ATILE = BM * 16 * 2;
    static constexpr uint32_t Q = 0, QA = TILE, DO = align1k(TILE + NA * ATILE);
    static constexpr uint32_t TAB = DO + TILE;                       // bf16 [2][KM][128]: cos rows, sin rows
    static constexpr uint32_t RESB = align1k(TAB + (NA > 0 ? KM * 512 : 0));
    static constexpr uint32_t STAGE0 = 2 * RESB;
    static constexpr uint32_t SK = 0, SKA = TILE, SV = align1k(TILE + NA * ATILE);
    static constexpr uint32_t STAGE = SV + TILE;
    static constexpr uint32_t EXTRA = 1024 + 1024;                  // barriers, base alignment
    static constexpr int NST = STAGE0 + 4 * STAGE + EXTRA <= kSmemBudget
                                   ? 4
                                   : (STAGE0 + 3 * STAGE + EXTRA <= kSmemBudget ? 3 : 2);
    static constexpr uint32_t BAR = STAGE0 + NST * STAGE;
    static constexpr uint32_t TOTAL = BAR + sizeof(Bars);
    static constexpr uint32_t RES_BYTES = 2 * TILE + NA * ATILE;
    static constexpr uint32_t KV_BYTES = 2 * TILE + NA * ATILE;
    static_assert(TOTAL + 1024 <= kSmemBudget, "shared memory");
};

template <int DA>
__global__ void __launch_bounds__(kThreads, 1) dq_kernel(const __grid_constant__ Maps maps, const Params p) {
    using L = QL<DA>;
    constexpr int NA = L::NA, NST = L::NST, KM = L::KM, KM4 = L::KM4;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    Bars &B = *reinterpret_cast<Bars *>(smem + L::BAR);
    Ctx cx{&B.abort_flag, p.err};

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = p.H * p.QB, G = gridDim.x;
    const bool tab = NA > 0 && p.dcoeff_cos && p.tab_smem;

    // acc_free of a resident buffer: the elementwise threads after the item's epilogue,
    // and each issuing warp once it has read the item's index
    if (threadIdx.x == 0) B.init(NST, kElem + 2);
    if (warp == 1) {
        tmem_alloc(&B.tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    __syncwarp();   // every warp reaches the CTA barrier converged (the producer ran on lane 0 alone)
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = B.tmem_slot;

    if (warp == 0) {
        // ---------------- producer: per item the resident tiles, then its kv tiles in list order
        if (lane == 0) {
            int gt = 0, last_res = -1;
            bool ok = true;
            for (int ci = 0; ok; ++ci) {
                // the first item of each CTA is its block index, the rest are handed out in order
                const int it = ci == 0 ? (int)blockIdx.x : G + atomicAdd(p.plan.next_item + 1, 1);
                const int rb = ci & 1;
                uint8_t *res = smem + rb * L::RESB;
                // buffer rb is free once every role is done with item ci - 2
                if (ci >= 2 && !cx.wait1(&B.acc_free[rb], ((ci >> 1) - 1) & 1)) break;
                if (last_res == ci - 2) last_res = -1;   // its tiles were consumed, so they landed
                B.item_of[rb] = it < n_items ? it : -1;
                if (it >= n_items) {
                    mbar_arrive(&B.res_full[rb]);      // publishes "no item left"
                    break;
                }
                const int h = it / p.QB, qb = it - h * p.QB;
                const int64_t mrow = (int64_t)h * p.QB + qb;
                const int n = p.kv_num[mrow];
                const int32_t *list = p.kv_idx + mrow * p.kv_stride;
                if (n > 0) {
                    mbar_expect_tx(&B.res_full[rb], L::RES_BYTES + (tab ? 2u * p.K * 256u : 0u));
                    if (tab) {
                        for (int k = 0; k < p.K; ++k) {
                            bulk_load(res + L::TAB + k * 256, p.cos_tab + (int64_t)k * p.tab_len + qb * BM, 256,
                                      &B.res_full[rb]);
                            bulk_load(res + L::TAB + (KM + k) * 256, p.sin_tab + (int64_t)k * p.tab_len + qb * BM, 256,
                                      &B.res_full[rb]);
                        }
                    }
                    tma_load_3d(&maps.q, res + L::Q, &B.res_full[rb], 0, qb * BM, h);
#pragma unroll
                    for (int a = 0; a < NA; ++a)
                        tma_load_3d(&maps.qa, res + L::QA + a * L::ATILE, &B.res_full[rb], 16 * a, qb * BM, h);
                    tma_load_3d(&maps.dout, res + L::DO, &B.res_full[rb], 0, qb * BM, h);
                    last_res = ci;
                } else {
                    mbar_arrive(&B.res_full[rb]);      // keeps the buffer's phases in step
                }
                for (int jj = 0; jj < n; ++jj, ++gt) {
                    const int st = gt % NST;
                    if (gt >= NST && !cx.wait1(&B.empty[st], ((gt / NST) - 1) & 1)) { ok = false; break; }
                    int kb = list[jj];
                    B.stage_blk[st] = kb;
                    const bool bad = kb < 0 || kb >= p.QB;
                    B.stage_mk[st] = bad ? MASK_DOCS : tile_mask_kind(qb, kb, p.docs != nullptr, p.block_info, p.QB);
                    if (bad) kb = 0;   // masked by the elementwise warps
                    uint8_t *sb = smem + L::STAGE0 + st * L::STAGE;
                    mbar_expect_tx(&B.full[st], L::KV_BYTES);
                    tma_load_3d(&maps.k, sb + L::SK, &B.full[st], 0, kb * BM, h);
#pragma unroll
                    for (int a = 0; a < NA; ++a)
                        tma_load_2d(&maps.ka, sb + L::SKA + a * L::ATILE, &B.full[st], 16 * a, kb * BM);
                    tma_load_3d(&maps.v, sb + L::SV, &B.full[st], 0, kb * BM, h);
                }
            }
            // never leave the CTA with a TMA write still in flight
            if (last_res >= 0) mbar_wait(&B.res_full[last_res & 1], (last_res >> 1) & 1, 500000000ull);
            for (int j = (gt > NST ? gt - NST : 0); j < gt; ++j) mbar_wait(&B.full[j % NST], (j / NST) & 1, 500000000ull);
        }
    } else if (warp == 1) {
        // ---------------- S / dP issuer (the whole warp waits, lane 0 issues)
        constexpr uint32_t idS = idesc_bf16(128, 128, false, false);
        int gt = 0;
        bool ok = true;
        for (int ci = 0; ok; ++ci) {
            const int rb = ci & 1;
            if (!cx.waitw(&B.res_full[rb], (ci >> 1) & 1)) { ok = false; break; }
            const int it = B.item_of[rb];
            if (lane == 0) mbar_arrive(&B.acc_free[rb]);   // the index is read
            if (it < 0) break;
            const int h = it / p.QB, qb = it - h * p.QB;
            const int n = p.kv_num[(int64_t)h * p.QB + qb];
            if (n == 0) continue;
            const uint32_t res = smem_u32(smem + rb * L::RESB);
            const uint32_t sQ = res + L::Q, sQA = res + L::QA, sDO = res + L::DO;
            for (int jj = 0; jj < n; ++jj, ++gt) {
                const int st = gt % NST, b = gt & 1;
                if (!cx.waitw(&B.full[st], (gt / NST) & 1)) { ok = false; break; }
                const uint32_t sb = smem_u32(smem + L::STAGE0 + st * L::STAGE);
                // dP = dO V^T first: the elementwise warps release dP of the previous tile as
                // they start it, while S waits for the gradient MMAs of tile gt-2
                if (gt >= 1 && !cx.waitw(&B.dp_free, (gt - 1) & 1)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_ss(tmem + DPC, kmajor_desc(sDO + kk * 32, 128), kmajor_desc(sb + L::SV + kk * 32, 128), idS,
                               kk > 0);
                    tc_commit(&B.dp_full);
                }
                __syncwarp();
                // S = Q K^T (+ Qaug Kaug^T): 128 q rows x 128 kv columns
                if (gt >= 2 && !cx.waitw(&B.s_free[b], ((gt >> 1) - 1) & 1)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_ss(tmem + sbuf(b), kmajor_desc(sQ + kk * 32, 128), kmajor_desc(sb + L::SK + kk * 32, 128),
                               idS, kk > 0);
#pragma unroll
                    for (int a = 0; a < NA; ++a)
                        mma_ss(tmem + sbuf(b), kmajor_desc(sQA + a * L::ATILE, 32),
                               kmajor_desc(sb + L::SKA + a * L::ATILE, 32), idS, 1);
                    tc_commit(&B.s_full[b]);
                }
                __syncwarp();
            }
        }
        if (!ok) cx.give_up();
        if (lane == 0) tc_commit(&B.drain[0]);   // TMEM is freed only after this warp's MMAs completed
        mbar_wait(&B.drain[0], 0, 500000000ull);
    } else if (warp == kGradWarp) {
        // ---------------- gradient issuer (whole warp): a second issuing warp, so
        // the S / dP MMAs and these queue on the tensor pipe side by side
        constexpr uint32_t idG = idesc_bf16(128, 64, false, true);
        // the DA/16 aug sub-tiles (16 columns, 32-byte swizzle) lie 4 KiB apart:
        // one MN-major operand of N = DA whose atoms the descriptor's
        // leading byte offset (4 KiB) steps through
        constexpr uint32_t idA = idesc_bf16(128, DA > 0 ? DA : 16, false, true);
        int gt = 0;
        bool ok = true;
        for (int ci = 0; ok; ++ci) {
            const int rb = ci & 1;
            if (!cx.waitw(&B.res_full[rb], (ci >> 1) & 1)) { ok = false; break; }
            const int it = B.item_of[rb];
            if (lane == 0) mbar_arrive(&B.acc_free[rb]);   // the index is read
            if (it < 0) break;
            const int h = it / p.QB, qb = it - h * p.QB;
            const int n = p.kv_num[(int64_t)h * p.QB + qb];
            for (int jj = 0; jj < n; ++jj, ++gt) {
                const int st = gt % NST, b = gt & 1;
                const uint32_t sb = smem_u32(smem + L::STAGE0 + st * L::STAGE);
                // dQ += dS K (+ dQaug += dS Kaug) over the tile's 128 kv rows: the even K
                // steps as soon as every warp has written them, then the odd
                for (int half = 0; half < 2; ++half) {
                    if (!cx.waitw(half ? &B.p_full[b] : &B.p_half[b], (gt >> 1) & 1)) { ok = false; break; }
                    // the first MMA of an item overwrites the accumulators: the previous
                    // item's epilogue must have read them
                    if (!half && jj == 0 && ci >= 1 && !cx.waitw(&B.acc_free[(ci - 1) & 1], ((ci - 1) >> 1) & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (lane == 0) {
#pragma unroll
                        for (int k2 = 0; k2 < 4; ++k2) {
                            const int kk = 2 * k2 + half;
                            const uint32_t acc = (jj > 0 || kk > 0) ? 1u : 0u;
                            mma_ts(tmem + ACC0, tmem + sbuf(b) + a_col(kk), mnmajor128_desc(sb + L::SK + kk * 2048),
                                   idG, acc);
                            if (NA > 0)
                                mma_ts(tmem + ACC1, tmem + sbuf(b) + a_col(kk), mnmajor32_desc(sb + L::SKA + kk * 512),
                                       idA, acc);
                        }
                        if (half) {
                            tc_commit(&B.s_free[b]);
                            tc_commit(&B.empty[st]);
                        }
                    }
                    __syncwarp();
                }
                if (!ok) break;
            }
            if (!ok) break;
            if (lane == 0) tc_commit(&B.acc_done);   // every item, so the epilogue's phases stay in step
            __syncwarp();
        }
        if (!ok) cx.give_up();
        if (lane == 0) tc_commit(&B.drain[1]);
        mbar_wait(&B.drain[1], 0, 500000000ull);
    } else {
        // ---------------- elementwise: thread = q row i, tile columns [32qc, 32qc+32) in two chunks of 16
        const int quad = warp & 3;
        const int qc = (warp - 2) >> 2;
        const int r = quad * 32 + lane;
        const uint32_t lb = (uint32_t)(quad * 32) << 16;
        const bool have_docs = p.docs != nullptr;
        const bool slope_acc = NA > 0 && p.has_slope && p.dslope;
        const uint64_t c2 = f2_pack(p.scale_log2, p.scale_log2);
        int gt = 0;
        bool alive = true;
        for (int ci = 0; alive; ++ci) {
            const int rb = ci & 1;
            if (!cx.waitw(&B.res_full[rb], (ci >> 1) & 1)) { alive = false; break; }
            const int it = B.item_of[rb];
            if (it < 0) break;
            const int h = it / p.QB, qb = it - h * p.QB;
            const int n = p.kv_num[(int64_t)h * p.QB + qb];
            uint8_t *res = smem + rb * L::RESB;
            const int i = qb * BM + r;
            const int doc_i = have_docs ? p.docs[i] : 0;
            const int64_t hrow = (int64_t)h * p.T + i;
            const float l2 = p.lse2[hrow], dl = p.delta[hrow];
            const uint64_t nl2 = f2_pack(-l2, -l2), nd2 = f2_pack(-dl, -dl);
            // The slope column of k_aug holds positions * s (up to ~T*s).  Its dS sum
            // is accumulated here in fp32 from the unrounded dS, against positions
            // relative to this query row: sum_j dS_ij = 0 in exact arithmetic, so
            // subtracting k_aug[i] changes nothing but the rounding, which would
            // otherwise amplify the small residual of that sum by ~i*s.
            const float kpos_i = __bfloat162float(__float2bfloat16_rn(__fmul_rn((float)i, p.s_aug)));
            float gsl = 0.f;
            for (int jj = 0; jj < n; ++jj, ++gt) {
                const int st = gt % NST, b = gt & 1;
                if (!cx.waitw(&B.full[st], (gt / NST) & 1)) { alive = false; break; }
                const int kb = B.stage_blk[st];
                const bool bad = kb < 0 || kb >= p.QB;
                const int mk = B.stage_mk[st];
                if (!cx.waitw(&B.s_full[b], (gt >> 1) & 1) || !cx.waitw(&B.dp_full, gt & 1)) { alive = false; break; }
                tc_fence_after();
                uint32_t rs[16], rp0[16], rp1[16];
                ld_tile_start(tmem + lb + sbuf(b) + qc * 32, tmem + lb + DPC + qc * 32, rs, rp0, rp1);
                tc_fence_before();
                mbar_arrive_warp(&B.dp_free);       // this warp's dP columns are in registers
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int col0 = qc * 32 + cc * 16;
                    const uint32_t tc = tmem + lb + sbuf(b) + col0;
                    if (cc == 1) ld_cols16(tc, rs);
                    float s[16], dp[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        s[e] = __uint_as_float(rs[e]);
                        dp[e] = __uint_as_float(cc ? rp1[e] : rp0[e]);
                    }
                    const int j0 = kb * BM + col0;
                    const int lim = i - j0;              // column e visible iff e <= lim (causal: j <= i)
                    if (mk == MASK_FULL) dq_piece<false>(s, dp, c2, nl2, nd2, mk, lim, bad, p.docs, j0, doc_i);
                    else dq_piece<true>(s, dp, c2, nl2, nd2, mk, lim, bad, p.docs, j0, doc_i);
                    if (slope_acc && !bad) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            // the value scope_qk_aug_prepare stored: bf16(fp32(j) * s)
                            const float kpos =
                                __bfloat162float(__float2bfloat16_rn(__fmul_rn((float)(j0 + e), p.s_aug)));
                            gsl = fmaf(s[e], kpos - kpos_i, gsl);
                        }
                    }
                    st_bf16x16(tc, s);                   // dS pairs over the chunk's own columns
                    if (cc == 0) {
                        tmem_wait_st();
                        tc_fence_before();
                        mbar_arrive_warp(&B.p_half[b]);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive_warp(&B.p_full[b]);
            }
            if (!alive) break;
            // ---------------- epilogue of the item
            if (!cx.waitw(&B.acc_done, ci & 1)) { alive = false; break; }
            tc_fence_after();
            const bool have = n > 0;
            // dQ: each of the quadrant's four warps stores 16 of the 64 columns
            store_row<16>(tmem + lb + ACC0 + qc * 16, p.scale,
                          p.g0 + (int64_t)h * p.g0_sh + (int64_t)i * p.g0_st + qc * 16, have);
            if (NA > 0 && p.dcoeff_cos) {
                // gradient of the augmented dims -> coefficients (q_aug = s [A c + B s', A s' - B c, -slope]);
                // the four warps of a quadrant split the K coefficients, reading the two
                // accumulator columns (k, K + k) of each coefficient k directly
                const int K = p.K;
                const int kq = (K + 3) >> 2;
                const int k0 = qc * kq, nk = max(0, min(kq, K - k0));
                float cv[KM4], sv[KM4], g0[KM4], g1[KM4];
                {
                    uint32_t o0[KM4], o1[KM4];
#pragma unroll
                    for (int e = 0; e < KM4; ++e) {
                        o0[e] = o1[e] = 0u;
                        if (have && e < nk) {
                            tmem_ld1(tmem + lb + ACC1 + k0 + e, o0[e]);
                            tmem_ld1(tmem + lb + ACC1 + K + k0 + e, o1[e]);
                        }
                    }
                    tmem_wait_ld();
                    pin(o0);
                    pin(o1);
#pragma unroll
                    for (int e = 0; e < KM4; ++e) {
                        g0[e] = __uint_as_float(o0[e]) * p.scale;
                        g1[e] = __uint_as_float(o1[e]) * p.scale;
                    }
                }
                if (tab && have) {
                    // the producer staged this item's table rows with its resident tiles
                    const bool ok = cx.waitw(&B.res_full[rb], (ci >> 1) & 1);
                    const uint16_t *tc = reinterpret_cast<const uint16_t *>(res + L::TAB);
#pragma unroll
                    for (int e = 0; e < KM4; ++e) {
                        if (e < nk) {
                            cv[e] = ok ? bf16_to_f32(tc[(k0 + e) * BM + r]) : 0.f;
                            sv[e] = ok ? bf16_to_f32(tc[(KM + k0 + e) * BM + r]) : 0.f;
                        }
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < KM4; ++e) {          // independent table loads, issued together
                        if (e < nk) {
                            cv[e] = bf16_to_f32(p.cos_tab[(int64_t)(k0 + e) * p.tab_len + i]);
                            sv[e] = bf16_to_f32(p.sin_tab[(int64_t)(k0 + e) * p.tab_len + i]);
                        }
                    }
                }
                float *oc = p.dcoeff_cos + hrow * K + k0, *os = p.dcoeff_sin + hrow * K + k0;
#pragma unroll
                for (int e = 0; e < KM4; ++e) {
                    if (e < nk) {
                        oc[e] = p.s_aug * (g0[e] * cv[e] + g1[e] * sv[e]);
                        os[e] = p.s_aug * (g0[e] * sv[e] - g1[e] * cv[e]);
                    }
                }
                if (slope_acc) {
                    // the quadrant's four partial sums meet in shared memory, in the item's Q
                    // tile (idle once its MMAs completed, ours until acc_free); the second
                    // barrier keeps every read before the buffer is released
                    float *slope_part = reinterpret_cast<float *>(res + L::Q);
                    if (qc > 0) slope_part[(qc - 1) * BM + r] = gsl;
                    elem_bar();
                    if (qc == 0)
                        p.dslope[hrow] =
                            -p.s_aug * ((gsl + slope_part[r] + slope_part[BM + r] + slope_part[2 * BM + r]) * p.scale);
                    elem_bar();
                }
            }
            tc_fence_before();
            mbar_arrive_warp(&B.acc_free[rb]);   // accumulators read, resident buffer rb released
        }
    }
    __syncwarp();   // every warp reaches the CTA barrier converged (the producer ran on lane 0 alone)
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace tcbwd

namespace tchost {

// Workspace of the backward: delta, lse*log2(e), and the dK/dV work plan.
struct BwdWorkspace {
    size_t delta, lse2, nq, items, item_slot, n_items, slot_chunks, slot_done, partial, total;
    int max_items;
};

BwdWorkspace bwd_workspace(int H, int T, int block_size) {
    auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
    BwdWorkspace w;
    const int QB = T / block_size;
    w.max_items = H * QB + tcbwd::kSlotCap * ((QB + tcbwd::kChunk - 1) / tcbwd::kChunk);
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
    w.total = o;
    return w;
}

template <int DA>
int launch_bwd(const ScopeAttnArgs &a, cudaStream_t s) {
    const int QB = a.T / 128;
    const BwdWorkspace ws = bwd_workspace(a.H, a.T, 128);
    uint8_t *base = reinterpret_cast<uint8_t *>(a.workspace);
    float *delta = reinterpret_cast<float *>(base + ws.delta);
    float *lse2 = reinterpret_cast<float *>(base + ws.lse2);
    const int64_t rows = (int64_t)a.H * a.T;
    tcbwd::prep_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16 *>(a.out), a.o_sh, a.o_st, reinterpret_cast<const __nv_bfloat16 *>(a.dout),
        a.do_sh, a.do_st, a.lse, a.H, a.T, delta, lse2);
    SCOPE_CHECK_LAUNCH();

    // dK/dV work plan: long q lists are cut into chunks
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

    tcbwd::Maps maps;
    std::memset(&maps, 0, sizeof(maps));
    bool ok = map3d(&maps.q, a.q, 64, a.T, a.H, a.q_st, a.q_sh, 64) &&
              map3d(&maps.k, a.k, 64, a.T, a.H, a.k_st, a.k_sh, 64) &&
              map3d(&maps.v, a.v, 64, a.T, a.H, a.v_st, a.v_sh, 64) &&
              map3d(&maps.dout, a.dout, 64, a.T, a.H, a.do_st, a.do_sh, 64);
    if (DA) ok = ok && map3d(&maps.qa, a.q_aug, DA, a.T, a.H, DA, (int64_t)a.T * DA, 16) &&
                 map2d(&maps.ka, a.k_aug, DA, a.T, 16);
    if (!ok) return SCOPE_ERR_ALIGN;

    tcbwd::Params p;
    std::memset(&p, 0, sizeof(p));
    p.H = a.H;
    p.T = a.T;
    p.QB = QB;
    p.words = words;
    p.kv_stride = a.kv_stride;
    p.q_bitmap = a.q_bitmap;
    p.kv_num = a.kv_num;
    p.kv_idx = a.kv_indices;
    p.block_info = a.block_info;
    p.docs = a.docs;
    p.lse2 = lse2;
    p.delta = delta;
    p.scale = a.scale;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.plan = plan;
    p.err = a.err_flag;

    // dK, dV
    p.g0 = reinterpret_cast<__nv_bfloat16 *>(a.dk);
    p.g0_sh = a.dk_sh;
    p.g0_st = a.dk_st;
    p.g1 = reinterpret_cast<__nv_bfloat16 *>(a.dv);
    p.g1_sh = a.dv_sh;
    p.g1_st = a.dv_st;
    // each CTA takes all 512 TMEM columns, so ask for enough shared memory that a
    // second CTA never lands on the SM just to wait inside tcgen05.alloc
    const size_t kOneCtaPerSm = 120 * 1024;
    size_t smem = std::max<size_t>(tcbwd::KVL<DA>::TOTAL + 1024, kOneCtaPerSm);
    if (cudaFuncSetAttribute(tcbwd::dkv_kernel<DA>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return SCOPE_ERR_CUDA;
    // persistent: one CTA per SM walks the plan's items
    int dev = 0, n_sm = 148;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return SCOPE_ERR_CUDA;
    tcbwd::dkv_kernel<DA><<<std::min(ws.max_items, n_sm), tcbwd::kThreads, smem, s>>>(maps, p);
    SCOPE_CHECK_LAUNCH();

    // dQ (+ coefficient gradients)
    p.g0 = reinterpret_cast<__nv_bfloat16 *>(a.dq);
    p.g0_sh = a.dq_sh;
    p.g0_st = a.dq_st;
    p.g1 = nullptr;
    if (a.bias_mode == SCOPE_BIAS_QK_AUG) {
        p.K = a.K;
        p.has_slope = a.slope != nullptr;
        p.tab_len = a.tab_len;
        p.tab_smem = (a.tab_len % 8 == 0) && aligned16(a.cos_tab) && aligned16(a.sin_tab) && a.K <= DA / 2;
        p.cos_tab = a.cos_tab;
        p.sin_tab = a.sin_tab;
        p.s_aug = (float)sqrt((double)a.beta / (double)a.scale);
        p.dcoeff_cos = a.dcoeff_cos;
        p.dcoeff_sin = a.dcoeff_sin;
        p.dslope = a.dslope;
    }
    smem = std::max<size_t>(tcbwd::QL<DA>::TOTAL + 1024, kOneCtaPerSm);
    if (cudaFuncSetAttribute(tcbwd::dq_kernel<DA>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return SCOPE_ERR_CUDA;
    // persistent: one CTA per SM (at most one per work item)
    const int grid_q = std::min(a.H * QB, n_sm);
    tcbwd::dq_kernel<DA><<<grid_q, tcbwd::kThreads, smem, s>>>(maps, p);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

}  // namespace tchost
}  // namespace scope

size_t scope_bwd_workspace_bytes(int H, int T, int block_size) {
    return scope::tchost::bwd_workspace(H, T, block_size).total;
}

int scope_tc_bwd(const ScopeAttnArgs &a, cudaStream_t s) {
    using namespace scope::tchost;
    switch (a.bias_mode == SCOPE_BIAS_QK_AUG ? a.d_aug : 0) {
        case 0: return launch_bwd<0>(a, s);
        case 16: return launch_bwd<16>(a, s);
        case 32: return launch_bwd<32>(a, s);
        case 48: return launch_bwd<48>(a, s);
        case 64: return launch_bwd<64>(a, s);
        default: return SCOPE_ERR_INVALID;
    }
}
