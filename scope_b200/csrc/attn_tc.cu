// Block-sparse SCOPE attention forward on the sm_100a tensor cores.
//
// One CTA computes one 128-row query block of one head against the kv
// blocks its list names (kv_indices, in order), flash-attention style:
//
//   warp 0      TMA producer: Q (+ the qk_aug dims) once, then K (+aug) and V
//               of each listed kv block into 2-stage rings with their own
//               barriers (K is released once the S MMA that read it is done,
//               V once P V is).  Tiles are addressed by block index, so the
//               sparse gather is just the TMA coordinate.  No multicast.
//               The same thread issues O += P V_j (P read from TMEM as the A
//               operand) once P_j is ready, just before it reloads V_j's stage.
//   warp 1      S issuer (the warp waits, lane 0 issues): S = Q K^T (+ Qaug
//               Kaug^T, the spectral bias) into TMEM as soon as the softmax
//               holds the previous S in registers, with sleeping waits.  It
//               also owns the TMEM allocation.
//   warps 2..9  softmax: two threads per query row (one per 64-column half,
//               the halves trading row max and row sum through shared memory
//               behind a bounded mbarrier).  S comes out of TMEM with
//               tcgen05.ld, the document-causal mask is applied only on tiles
//               the producer classified as needing it (diagonal, document
//               boundary; branch-free selects, document ids read 16 bytes at a
//               time), exponentials are taken in the log2 domain (one pair in
//               eight on the FMA pipe, ex2_fma2, the rest on the MUFU), P goes
//               back to TMEM as bf16, and the running max is only moved when
//               it grows by more than 2^8 (otherwise O would need a rescale
//               through TMEM every tile).
//
// TMEM (256 columns per CTA, two CTAs per SM): S [0,128), O [128,192),
// P (bf16 pairs) [192,256).  S is single buffered: the issuer starts
// S_{j+1} as soon as the softmax threads have copied S_j to registers, so the
// QK^T of the next tile overlaps the softmax of the current one and P V_j
// overlaps the next softmax.
//
// Every mbarrier wait is bounded; a wait that gives up sets
// SCOPE_DEVERR_TIMEOUT in the error word and the CTA winds down (draining
// its own TMA loads, freeing TMEM) instead of hanging.
//
// The same kernel with MASS set computes the spectral teacher's dense block
// mass (scoped_medium.py:1793-1819, entry point scope_block_mass): no V, the
// kv blocks from the document start of the q block to the diagonal, walked
// twice (row statistics, then the probabilities summed per kv block).
#include <cmath>
#include <cstring>

#include "tc_host.cuh"
#include "tc_ptx.cuh"

namespace scope {
namespace tcfwd {

using namespace tc;

constexpr int BM = 128;
constexpr int HD = 64;
constexpr int kThreads = 320;   // producer, issuer, 8 softmax warps (two per TMEM lane quadrant)
constexpr int kSoftmax = 256;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t S_COL = 0, O_COL = 128, P_COL = 192;
// of every 8 exponential pairs, this many are evaluated on the FMA pipe
// (ex2_fma2) and the rest on the MUFU: the two pipes then share the softmax's
// exponentials instead of the MUFU alone bounding it
#ifndef SCOPE_FWD_POLY_PAIRS
#define SCOPE_FWD_POLY_PAIRS 1
#endif
constexpr int kPolyPairs = SCOPE_FWD_POLY_PAIRS;

__host__ __device__ constexpr uint32_t align1k(uint32_t x) { return (x + 1023u) & ~1023u; }

// qk_aug dims are staged as DA/16 sub-tiles of 16 bf16 columns (32-byte rows,
// 32-byte swizzle), one MMA K-step each, so every aug width 16..64 uses the
// same layout.
template <int DA>
struct Layout {
    static constexpr int NA = DA / 16;                           // aug sub-tiles
    static constexpr uint32_t TILE = BM * HD * 2;                // 16 KiB
    static constexpr uint32_t ATILE = BM * 16 * 2;               // 4 KiB
    static constexpr uint32_t Q = 0;
    static constexpr uint32_t QA = TILE;                         // + a * ATILE
    static constexpr uint32_t STAGE0 = align1k(QA + NA * ATILE);
    static constexpr uint32_t K = 0, KA = TILE;                  // + a * ATILE
    static constexpr uint32_t V = align1k(TILE + NA * ATILE);
    static constexpr uint32_t STAGE = V + TILE;
    static constexpr uint32_t BAR = STAGE0 + 2 * STAGE;
    static constexpr uint32_t XCH = BAR + 256;                   // float[2 parity][2 halves][128 rows] + l[2][128]
    static constexpr uint32_t TOTAL = XCH + 3 * 1024;
    static constexpr uint32_t K_BYTES = TILE + NA * ATILE;       // expected TMA bytes: K (+aug) of a stage
    static constexpr uint32_t V_BYTES = TILE;                    // V of a stage
    static constexpr uint32_t Q_BYTES = TILE + NA * ATILE;
};

// Tile classes: 0 every element visible (kv block before the q block, one
// document), 1 one document (causal test only), 2 straddles a document boundary
// (element document ids needed).  block_info rows 2, 3: per-block doc min / max.
__device__ __forceinline__ int tile_kind(int qb, int kb, bool have_docs, const int32_t *block_info, int QB) {
    bool same_doc = !have_docs;
    if (have_docs && block_info) {
        const int a = block_info[2 * QB + qb], b = block_info[3 * QB + qb];
        const int c = block_info[2 * QB + kb], d = block_info[3 * QB + kb];
        same_doc = (a == b) & (c == d) & (a == c);
    }
    return (kb < qb && same_doc) ? 0 : (same_doc ? 1 : 2);
}

struct FwdParams {
    int H, T, QB, kv_stride;
    const int32_t *kv_num, *kv_idx, *block_info, *docs;
    float scale_log2;
    __nv_bfloat16 *out;
    int64_t o_sh, o_st;
    float *lse;
    int32_t *err;
};

// score_mod mode (the Fourier sum is in the aug dims): per-row slope, Δ_main,
// width and b0 [H,T] (or null), the gate's lambda and 1/tau, beta / scale
// (bias units -> unscaled score units), and beta for the lse's b0 term
struct SmodParams {
    const float *slope, *dmain, *width, *b0;
    float gate_lambda, gate_itau, bias_k, beta;
    float *mass;   // block-mass variant: [H, QB, QB] output, zeroed before the launch
};

struct Maps {
    CUtensorMap q, k, v, qa, ka;   // qa / ka: 16-column boxes of the qk_aug dims
};

// Bias of the score_mod mode beyond the Fourier sum, for Δ = i - j
// (scoped_medium.py:425-457): slope Δ - lambda gate((|Δ - Δ_main| - width) / tau),
// gate = softplus (torch's, threshold 20) or relu.  SM: 0 off, 1 no gate,
// 2 softplus gate, 3 relu gate.
template <int SM>
__device__ __forceinline__ float smod_bias(float dl, float slope, float dm, float w, float lam, float itau) {
    float b = slope * dl;
    if constexpr (SM >= 2) {
        const float u = (fabsf(dl - dm) - w) * itau;
        float g;
        if constexpr (SM == 3) {
            g = fmaxf(u, 0.f);
        } else {
            g = u > 20.f ? u : 0.69314718055994531f * lg2(1.f + ex2(u * 1.4426950408889634f));
        }
        b = fmaf(-lam, g, b);
    }
    return b;
}

// MASS: the teacher's dense block mass (scoped_medium.py:1793-1819) instead of
// attention: the kv list is implicit (every block from the document start of
// the q block's first row up to the diagonal), the tiles run twice -- once for
// the row max and sum, once for the probabilities, whose sum over each tile is
// added into mass[h, qb, kb] -- and no V is loaded or multiplied.
template <int DA, int SM, bool MASS = false>
__global__ void __launch_bounds__(kThreads, 2) fwd_kernel(const __grid_constant__ Maps maps, const FwdParams p,
                                                          const __grid_constant__ SmodParams sp) {
    using L = Layout<DA>;
    constexpr int NA = L::NA;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR);
    // K (+aug) and V of a stage have their own barriers: K is released when
    // the S MMA that read it completes, long before P V frees V, so the next
    // K load gets a whole softmax period of lead time.
    uint64_t *q_full = bars + 0, *kv_full = bars + 1, *kv_empty = bars + 3;   // K halves of the stages
    uint64_t *v_full = bars + 20, *v_empty = bars + 22;
    uint64_t *s_full = bars + 5, *s_free = bars + 6, *p_full = bars + 7, *o_done = bars + 8;
    uint64_t *xchg = bars + 9;                                   // [4]: one per TMEM lane quadrant
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 13);
    // kv block and mask kind of tile j at [j & 3]: the producer may refill a
    // stage's K (tile j+2) while the softmax has yet to read tile j's entry
    volatile int *stage_kb = reinterpret_cast<volatile int *>(bars + 14);   // [4]
    volatile int *stage_mk = stage_kb + 4;                                  // [4]
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    float *xmax = reinterpret_cast<float *>(smem + L::XCH);      // [2][2][128]
    float *xsum = xmax + 512;                                    // [2][128]

    const int qb = blockIdx.x, h = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t mrow = (int64_t)h * p.QB + qb;
    // the mass variant's blocks: kb0 .. qb, kb0 the document start block of the q block's first row
    const int kb0 = MASS ? ((p.docs && p.block_info) ? min(max(p.block_info[p.QB + qb], 0), qb) : 0) : 0;
    const int n = MASS ? qb - kb0 + 1 : p.kv_num[mrow];
    const int ntile = MASS ? 2 * n : n;   // tiles the producer, the issuer and the softmax walk
    const int32_t *list = p.kv_idx + mrow * p.kv_stride;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(kv_full + 0, 1);
        mbar_init(kv_full + 1, 1);
        mbar_init(kv_empty + 0, 1);
        mbar_init(kv_empty + 1, 1);
        for (int q = 0; q < 2; ++q) {
            mbar_init(v_full + q, 1);
            mbar_init(v_empty + q, 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, kSoftmax);
        mbar_init(p_full, kSoftmax);
        mbar_init(o_done, 1);
        for (int q = 0; q < 4; ++q) mbar_init(xchg + q, 64);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    __syncwarp();   // every warp reaches the CTA barrier converged (the producer ran on lane 0 alone)
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto give_up = [&]() {
        *abort_flag = 1;
        set_err(p.err, SCOPE_DEVERR_TIMEOUT);
    };
    // softmax warps run warp-collective tcgen05.ld/st, so they agree on every wait's outcome
    auto warp_wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        bool ok = !*abort_flag && mbar_wait(bar, parity);
        return __all_sync(0xffffffffu, ok);
    };
    // the issuer warp only waits: it sleeps between polls
    auto idle_wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        bool ok = !*abort_flag && mbar_wait_idle(bar, parity);
        return __all_sync(0xffffffffu, ok);
    };

    // P V_j, issued by the producer thread: once P_j is in TMEM and V_j has landed
    auto issue_pv = [&](int j) -> bool {
        if (*abort_flag || !mbar_wait_idle(p_full, j & 1) || !mbar_wait_idle(v_full + (j & 1), (j >> 1) & 1))
            return false;
        tc_fence_after();
        constexpr uint32_t idO = idesc_bf16(128, 64, false, true);
        const uint32_t sv = smem_u32(smem + L::STAGE0 + (j & 1) * L::STAGE + L::V);
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk)
            mma_ts(tmem + O_COL, tmem + P_COL + kk * 8, mnmajor128_desc(sv + kk * 2048), idO, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(o_done);
        if (j + 2 < n) tc_commit(v_empty + (j & 1));
        return true;
    };
    if (warp == 0 && MASS) {
        // ------------------------------------------------------------ producer (mass): K only, both passes
        if (lane == 0 && n > 0) {
            mbar_expect_tx(q_full, L::Q_BYTES);
            tma_load_3d(&maps.q, smem + L::Q, q_full, 0, qb * BM, h);
#pragma unroll
            for (int a = 0; a < NA; ++a) tma_load_3d(&maps.qa, smem + L::QA + a * L::ATILE, q_full, 16 * a, qb * BM, h);
            int kissued = 0;
            for (int j = 0; j < ntile; ++j) {
                const int s = j & 1;
                if (j >= 2 && (*abort_flag || !mbar_wait_idle(kv_empty + s, ((j >> 1) - 1) & 1))) {
                    give_up();
                    break;
                }
                const int kb = kb0 + (j < n ? j : j - n);
                uint8_t *st = smem + L::STAGE0 + s * L::STAGE;
                mbar_expect_tx(kv_full + s, L::K_BYTES);
                tma_load_3d(&maps.k, st + L::K, kv_full + s, 0, kb * BM, h);
#pragma unroll
                for (int a = 0; a < NA; ++a) tma_load_2d(&maps.ka, st + L::KA + a * L::ATILE, kv_full + s, 16 * a, kb * BM);
                kissued = j + 1;
            }
            // never leave the CTA with a TMA write still in flight
            mbar_wait(q_full, 0, 500000000ull);
            for (int j = (kissued > 2 ? kissued - 2 : 0); j < kissued; ++j)
                mbar_wait(kv_full + (j & 1), (j >> 1) & 1, 500000000ull);
        }
    } else if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0 && n > 0) {
            mbar_expect_tx(q_full, L::Q_BYTES);
            tma_load_3d(&maps.q, smem + L::Q, q_full, 0, qb * BM, h);
#pragma unroll
            for (int a = 0; a < NA; ++a) tma_load_3d(&maps.qa, smem + L::QA + a * L::ATILE, q_full, 16 * a, qb * BM, h);
            int issued = 0, kissued = 0;   // stages whose V / K loads were issued
            for (int j = 0; j < n; ++j) {
                const int s = j & 1;
                if (j >= 2 && (*abort_flag || !mbar_wait_idle(kv_empty + s, ((j >> 1) - 1) & 1))) {
                    give_up();
                    break;
                }
                int kb = list[j];
                const bool bad = kb < 0 || kb >= p.QB;
                stage_kb[j & 3] = kb;
                stage_mk[j & 3] = bad ? 3 : tile_kind(qb, kb, p.docs != nullptr, p.block_info, p.QB);
                if (bad) kb = 0;   // the softmax masks this tile and flags it
                uint8_t *st = smem + L::STAGE0 + s * L::STAGE;
                mbar_expect_tx(kv_full + s, L::K_BYTES);
                tma_load_3d(&maps.k, st + L::K, kv_full + s, 0, kb * BM, h);
#pragma unroll
                for (int a = 0; a < NA; ++a) tma_load_2d(&maps.ka, st + L::KA + a * L::ATILE, kv_full + s, 16 * a, kb * BM);
                // P V of two tiles back, once its P is ready (its V stage is reloaded next)
                if (j >= 2 && !issue_pv(j - 2)) {
                    give_up();
                    issued = j;
                    kissued = j + 1;
                    break;
                }
                if (j >= 2 && (*abort_flag || !mbar_wait_idle(v_empty + s, ((j >> 1) - 1) & 1))) {
                    give_up();
                    issued = j;
                    kissued = j + 1;
                    break;
                }
                mbar_expect_tx(v_full + s, L::V_BYTES);
                tma_load_3d(&maps.v, st + L::V, v_full + s, 0, kb * BM, h);
                issued = kissued = j + 1;
            }
            for (int j = (n > 2 ? n - 2 : 0); j < n && issued == n; ++j)
                if (!issue_pv(j)) {
                    give_up();
                    break;
                }
            // never leave the CTA with a TMA write still in flight
            mbar_wait(q_full, 0, 500000000ull);
            for (int j = (kissued > 2 ? kissued - 2 : 0); j < kissued; ++j)
                mbar_wait(kv_full + (j & 1), (j >> 1) & 1, 500000000ull);
            for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j)
                mbar_wait(v_full + (j & 1), (j >> 1) & 1, 500000000ull);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ tcgen05 issuer
        if (n > 0) {   // the whole warp waits; lane 0 issues
            constexpr uint32_t idS = idesc_bf16(128, 128, false, false);
            const uint32_t tS = tmem + S_COL;
            const uint32_t sq = smem_u32(smem + L::Q);
            bool ok = idle_wait(q_full, 0);
            auto issue_S = [&](int j) -> bool {
                const int s = j & 1;
                if (!idle_wait(kv_full + s, (j >> 1) & 1)) return false;
                tc_fence_after();
                const uint32_t sk = smem_u32(smem + L::STAGE0 + s * L::STAGE);
                if (lane == 0) {
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk)
                        mma_ss(tS, kmajor_desc(sq + L::Q + kk * 32, 128), kmajor_desc(sk + L::K + kk * 32, 128), idS,
                               kk > 0);
#pragma unroll
                    for (int a = 0; a < NA; ++a)
                        mma_ss(tS, kmajor_desc(sq + L::QA + a * L::ATILE, 32), kmajor_desc(sk + L::KA + a * L::ATILE, 32),
                               idS, 1);
                    tc_commit(s_full);
                    // mass variant: K of this stage may be reloaded once S is done (only when a
                    // later tile will be)
                    if (MASS && j + 2 < ntile) tc_commit(kv_empty + s);
                }
                __syncwarp();
                return true;
            };
            ok = ok && issue_S(0);
            // S_{j+1} as soon as the softmax holds S_j in registers and K_{j+1} has
            // landed; the waits block in the barrier (the warp sleeps instead of
            // polling issue slots away from the softmax warps on its sub-partition).
            // P V is issued by the producer thread: each tcgen05.mma holds its
            // issuing warp for about its execution time, so splitting the two kinds
            // of MMA over two warps (on two sub-partitions, other ones for the SM's
            // second CTA) spreads that cost instead of piling it on one.
            for (int j = 0; ok && j + 1 < ntile; ++j) {
                ok = idle_wait(s_free, j & 1);
                // attention variant: K_j's stage is released once the softmax holds S_j (so
                // S_j is done), not when S_j completes: the softmax warps wait on kv_full of
                // tile j before they read S_j, and K_{j+2} must not land there first
                if (!MASS && ok && lane == 0 && j + 2 < ntile) mbar_arrive(kv_empty + (j & 1));
                ok = ok && issue_S(j + 1);
            }
            if (!ok) give_up();
        }
    } else {
        // ------------------------------------------------------------ softmax + epilogue
        // thread = (query row r, column half ch): S columns [64ch, 64ch+64), O and P columns [32ch, 32ch+32)
        const int quad = warp & 3;
        const int ch = (warp - 2) >> 2;
        const int r = quad * 32 + lane;
        const int i = qb * BM + r;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const uint32_t tS = tmem + lane_base + S_COL + ch * 64, tO = tmem + lane_base + O_COL + ch * 32,
                       tP = tmem + lane_base + P_COL + ch * 32;
        const bool have_docs = p.docs != nullptr;
        const bool docs_vec = (reinterpret_cast<uintptr_t>(p.docs) & 15) == 0;
        float sm_slope = 0.f, sm_dm = 0.f, sm_w = 0.f;
        if constexpr (SM != 0) {
            const int64_t hrow = (int64_t)h * p.T + i;
            sm_slope = sp.slope ? sp.slope[hrow] : 0.f;
            if constexpr (SM >= 2) {
                sm_dm = sp.dmain[hrow];
                sm_w = sp.width[hrow];
            }
        }
        const int doc_i = have_docs ? p.docs[i] : 0;
        // scores are kept unscaled until the exponent: max(x) * c = max(x * c) for c > 0,
        // and a negative scale is folded into the sign of the loaded scores
        const bool neg = p.scale_log2 < 0.f;
        const float cabs = fabsf(p.scale_log2);
        const uint64_t c2 = f2_pack(cabs, cabs);
        float m = -INFINITY, l = 0.f;
        bool alive = true;
        int xphase = 0;                         // completed phases of this quadrant's exchange barrier
        float mlse = 0.f;                       // mass variant, second pass: m + log2(row sum)
        for (int j = 0; j < ntile && alive; ++j) {
            if (MASS && j == n) {
                // between the passes: the row sum across the two column halves
                xsum[ch * 128 + r] = l;
                mbar_arrive(xchg + quad);
                if (!warp_wait(xchg + quad, xphase & 1)) { give_up(); alive = false; break; }
                ++xphase;
                const float ltot = l + xsum[(1 - ch) * 128 + r];
                mlse = (ltot > 0.f && m != -INFINITY) ? m + lg2(ltot) : INFINITY;
            }
            // this tile's kv block and mask kind: 0 full, 1 causal only, 2 document ids,
            // 3 bad index.  The producer classified it; the mass variant, whose producer
            // refills a K stage as soon as the S MMA that read it is done (which can move
            // kv_full two phases on before these warps wait on it), computes both itself.
            int kb, mk;
            if constexpr (MASS) {
                kb = kb0 + (j < n ? j : j - n);
                mk = tile_kind(qb, kb, have_docs, p.block_info, p.QB);
            } else {
                if (!warp_wait(kv_full + (j & 1), (j >> 1) & 1)) { give_up(); alive = false; break; }
                kb = stage_kb[j & 3];
                mk = stage_mk[j & 3];
            }
            if (mk == 3 && r == 0 && ch == 0) set_err(p.err, SCOPE_DEVERR_INDEX);
            if (!warp_wait(s_full, j & 1)) { give_up(); alive = false; break; }
            tc_fence_after();
            float x[64];
            {
                uint32_t u0[32], u1[32];
                tmem_ld32_nw(tS, u0);
                tmem_ld32_nw(tS + 32, u1);
                tmem_wait_ld();
                pin(u0);
                pin(u1);
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    x[e] = __uint_as_float(u0[e]);
                    x[32 + e] = __uint_as_float(u1[e]);
                }
                if (neg) {
#pragma unroll
                    for (int e = 0; e < 64; ++e) x[e] = -x[e];
                }
            }
            tc_fence_before();
            mbar_arrive(s_free);
            if constexpr (SM != 0) {
                // the elementwise terms of the score_mod bias, in unscaled score units
                const float dbase = (float)(i - (kb * BM + ch * 64));
#pragma unroll
                for (int c = 0; c < 64; ++c)
                    x[c] = fmaf(sp.bias_k,
                                smod_bias<SM>(dbase - (float)c, sm_slope, sm_dm, sm_w, sp.gate_lambda, sp.gate_itau), x[c]);
            }
            if (mk != 0) {
                const int j0 = kb * BM + ch * 64;
                const int lim = mk == 3 ? -1 : i - j0;  // column c visible iff c <= lim
                // document ids of the 64 columns (tiles of kind 2 only), 16 bytes at a time
                // where the pointer allows it (j0 is a multiple of 64)
                const int32_t *dp = have_docs ? p.docs + j0 : p.docs;
#pragma unroll
                for (int c4 = 0; c4 < 16; ++c4) {
                    int4 d = make_int4(doc_i, doc_i, doc_i, doc_i);
                    if (mk == 2)
                        d = docs_vec ? __ldg(reinterpret_cast<const int4 *>(dp) + c4)
                                     : make_int4(__ldg(dp + 4 * c4), __ldg(dp + 4 * c4 + 1), __ldg(dp + 4 * c4 + 2),
                                                 __ldg(dp + 4 * c4 + 3));
                    const int c = 4 * c4;
                    x[c] = (c <= lim && d.x == doc_i) ? x[c] : -INFINITY;
                    x[c + 1] = (c + 1 <= lim && d.y == doc_i) ? x[c + 1] : -INFINITY;
                    x[c + 2] = (c + 2 <= lim && d.z == doc_i) ? x[c + 2] : -INFINITY;
                    x[c + 3] = (c + 3 <= lim && d.w == doc_i) ? x[c + 3] : -INFINITY;
                }
            }
            if (MASS && j >= n) {
                // second pass: this tile's probabilities 2^(x c - mlse), summed over the
                // thread's 64 columns, the warp's 32 rows, and added into the block mass
                const uint64_t nl2 = f2_pack(-mlse, -mlse);
                uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
                for (int c = 0; c < 64; c += 2) {
                    const float2 d = f2_unpack(ffma2(f2_pack(x[c], x[c + 1]), c2, nl2));
                    const uint64_t pp = (((c >> 1) & 7) < kPolyPairs) ? ex2_fma2(d.x, d.y) : f2_pack(ex2(d.x), ex2(d.y));
                    acc[(c >> 1) & 3] = fadd2(acc[(c >> 1) & 3], pp);
                }
                const float2 a01 = f2_unpack(fadd2(acc[0], acc[1])), a23 = f2_unpack(fadd2(acc[2], acc[3]));
                float rs = (a01.x + a01.y) + (a23.x + a23.y);
#pragma unroll
                for (int o = 16; o; o >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o);
                if (lane == 0) atomicAdd(sp.mass + mrow * p.QB + kb, rs);
                continue;
            }
            // row max over this thread's 64 columns: 8 independent chains of
            // three-input maxima (column c in chain c & 7), then a tree
            float pm[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                pm[k] = fmax3(x[k], x[8 + k], x[16 + k]);
                pm[k] = fmax3(pm[k], x[24 + k], x[32 + k]);
                pm[k] = fmax3(pm[k], x[40 + k], x[48 + k]);
                pm[k] = fmaxf(pm[k], x[56 + k]);
            }
            const float pmx = fmax3(fmax3(pm[0], pm[1], pm[2]), fmax3(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7])) * cabs;
            // row max across the two column halves
            xmax[(j & 1) * 256 + ch * 128 + r] = pmx;
            mbar_arrive(xchg + quad);
            if (!warp_wait(xchg + quad, xphase & 1)) { give_up(); alive = false; break; }
            ++xphase;
            const float mx = fmaxf(pmx, xmax[(j & 1) * 256 + (1 - ch) * 128 + r]);
            float alpha = 1.f;
            bool rescale = false;
            if (mx > m + 8.f) {     // move the reference max only when it grows by > 2^8
                alpha = (m == -INFINITY) ? 0.f : ex2(m - mx);
                m = mx;
                rescale = true;
            }
            const float mref = (m == -INFINITY) ? 0.f : m;
            const uint64_t nm2 = f2_pack(-mref, -mref);
            // p = 2^(x c - m) in one packed FMA per pair; the row sum in four packed partials
            uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
            uint32_t pk[32];                  // P as bf16 pairs, packed as it is formed
#pragma unroll
            for (int c = 0; c < 64; c += 2) {
                const float2 d = f2_unpack(ffma2(f2_pack(x[c], x[c + 1]), c2, nm2));
                uint64_t pp;
                if (((c >> 1) & 7) < kPolyPairs) {
                    pp = ex2_fma2(d.x, d.y);   // this share of the pairs on the FMA pipe
                } else {
                    pp = f2_pack(ex2(d.x), ex2(d.y));
                }
                const float2 pf = f2_unpack(pp);
                pk[c >> 1] = pack_bf16(pf.x, pf.y);
                acc[(c >> 1) & 3] = fadd2(acc[(c >> 1) & 3], pp);
            }
            const float2 a01 = f2_unpack(fadd2(acc[0], acc[1])), a23 = f2_unpack(fadd2(acc[2], acc[3]));
            const float rs = (a01.x + a01.y) + (a23.x + a23.y);
            l = l * alpha + rs;
            if (MASS) continue;   // first pass of the mass variant: statistics only
            // P V of the previous tile has read P and written O: P can be replaced, O rescaled
            if (j > 0) {
                if (!warp_wait(o_done, (j - 1) & 1)) { give_up(); alive = false; break; }
                tc_fence_after();
            }
            tmem_st32(tP, pk);
            // tcgen05.ld/st are warp-collective: rescale O whenever any row of the warp needs it
            if (j > 0 && __any_sync(0xffffffffu, rescale)) {
                uint32_t o[32];
                tmem_ld32_nw(tO, o);
                tmem_wait_ld();
                pin(o);
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                tmem_st32(tO, o);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(p_full);
        }
        // epilogue: row sum across the halves, O / l -> bf16, lse (the mass
        // variant wrote its output in the second pass)
        if constexpr (!MASS) {
            bool have_o = false;
            if (alive) {
                xsum[ch * 128 + r] = l;
                mbar_arrive(xchg + quad);
                alive = warp_wait(xchg + quad, xphase & 1);
                if (!alive) give_up();
            }
            const float ltot = alive ? l + xsum[(1 - ch) * 128 + r] : 0.f;
            if (alive && n > 0) {
                have_o = warp_wait(o_done, (n - 1) & 1);
                if (!have_o) give_up();
                tc_fence_after();
            }
            __nv_bfloat16 *orow = p.out + (int64_t)h * p.o_sh + (int64_t)i * p.o_st + ch * 32;
            const float inv = (ltot > 0.f) ? 1.f / ltot : 0.f;
            {
                uint32_t o[32];
                if (have_o) {
                    tmem_ld32_nw(tO, o);
                    tmem_wait_ld();
                    pin(o);
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] = 0u;
                }
                uint32_t w[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) w[e] = pack_bf16(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
                uint4 *dst = reinterpret_cast<uint4 *>(orow);
#pragma unroll
                for (int e = 0; e < 4; ++e) dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
            }
            if (p.lse && ch == 0) {
                float lse = (ltot > 0.f) ? (m + log2f(ltot)) * 0.69314718055994531f : -INFINITY;
                if constexpr (SM != 0) {
                    if (sp.b0) lse -= sp.beta * sp.b0[(int64_t)h * p.T + i];   // the score_mod bias's row constant -beta b0
                }
                p.lse[(int64_t)h * p.T + i] = lse;
            }
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

}  // namespace tcfwd

// ---------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------
namespace tchost {

template <int DA, int SM>
int launch_fwd(const ScopeAttnArgs &a, cudaStream_t s) {
    using L = tcfwd::Layout<DA>;
    tcfwd::Maps maps;
    std::memset(&maps, 0, sizeof(maps));
    bool ok = map3d(&maps.q, a.q, 64, a.T, a.H, a.q_st, a.q_sh, 64) &&
              map3d(&maps.k, a.k, 64, a.T, a.H, a.k_st, a.k_sh, 64) &&
              map3d(&maps.v, a.v, 64, a.T, a.H, a.v_st, a.v_sh, 64);
    if (DA) ok = ok && map3d(&maps.qa, a.q_aug, DA, a.T, a.H, DA, (int64_t)a.T * DA, 16) &&
                 map2d(&maps.ka, a.k_aug, DA, a.T, 16);
    if (!ok) return SCOPE_ERR_ALIGN;
    tcfwd::FwdParams p;
    p.H = a.H;
    p.T = a.T;
    p.QB = a.T / 128;
    p.kv_stride = a.kv_stride;
    p.kv_num = a.kv_num;
    p.kv_idx = a.kv_indices;
    p.block_info = a.block_info;
    p.docs = a.docs;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.out = reinterpret_cast<__nv_bfloat16 *>(a.out);
    p.o_sh = a.o_sh;
    p.o_st = a.o_st;
    p.lse = a.lse;
    p.err = a.err_flag;
    tcfwd::SmodParams sp;
    sp.slope = a.slope;
    sp.dmain = a.delta_main;
    sp.width = a.width;
    sp.b0 = a.b0;
    sp.gate_lambda = a.gate_lambda;
    sp.gate_itau = (a.gate_tau != 0.f) ? 1.f / a.gate_tau : 0.f;
    sp.bias_k = a.beta / a.scale;
    sp.beta = a.beta;
    const size_t smem = L::TOTAL + 1024;
    if (cudaFuncSetAttribute(tcfwd::fwd_kernel<DA, SM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return SCOPE_ERR_CUDA;
    dim3 grid(p.QB, a.H);
    tcfwd::fwd_kernel<DA, SM><<<grid, tcfwd::kThreads, smem, s>>>(maps, p, sp);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

// the teacher's block mass: fwd_kernel's mass variant over the implicit
// document-causal lists, into a zeroed [H, QB, QB] float32 buffer
template <int DA>
int launch_mass(const ScopeAttnArgs &a, float *mass, cudaStream_t s) {
    using L = tcfwd::Layout<DA>;
    tcfwd::Maps maps;
    std::memset(&maps, 0, sizeof(maps));
    bool ok = map3d(&maps.q, a.q, 64, a.T, a.H, a.q_st, a.q_sh, 64) &&
              map3d(&maps.k, a.k, 64, a.T, a.H, a.k_st, a.k_sh, 64);
    if (DA) ok = ok && map3d(&maps.qa, a.q_aug, DA, a.T, a.H, DA, (int64_t)a.T * DA, 16) &&
                 map2d(&maps.ka, a.k_aug, DA, a.T, 16);
    if (!ok) return SCOPE_ERR_ALIGN;
    tcfwd::FwdParams p;
    std::memset(&p, 0, sizeof(p));
    p.H = a.H;
    p.T = a.T;
    p.QB = a.T / 128;
    p.block_info = a.block_info;
    p.docs = a.docs;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.err = a.err_flag;
    tcfwd::SmodParams sp;
    std::memset(&sp, 0, sizeof(sp));
    sp.mass = mass;
    if (cudaMemsetAsync(mass, 0, sizeof(float) * (size_t)a.H * p.QB * p.QB, s) != cudaSuccess) return SCOPE_ERR_CUDA;
    const size_t smem = L::TOTAL + 1024;
    if (cudaFuncSetAttribute(tcfwd::fwd_kernel<DA, 0, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return SCOPE_ERR_CUDA;
    dim3 grid(p.QB, a.H);
    tcfwd::fwd_kernel<DA, 0, true><<<grid, tcfwd::kThreads, smem, s>>>(maps, p, sp);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

}  // namespace tchost
}  // namespace scope

using namespace scope;

extern "C" int scope_block_mass(const ScopeAttnArgs *args, float *mass, scope_stream_t stream) {
    if (!args || !mass) return SCOPE_ERR_INVALID;
    const ScopeAttnArgs &a = *args;
    if (a.H <= 0 || a.T <= 0 || a.block_size != 128 || a.T % 128 != 0 || a.D != 64 || !a.q || !a.k)
        return SCOPE_ERR_INVALID;
    if (a.dtype != SCOPE_BF16) return SCOPE_ERR_DTYPE;
    if (a.bias_mode != SCOPE_BIAS_NONE && a.bias_mode != SCOPE_BIAS_QK_AUG) return SCOPE_ERR_INVALID;
    const int da = a.bias_mode == SCOPE_BIAS_QK_AUG ? a.d_aug : 0;
    if (da && (!a.q_aug || !a.k_aug || (da != 16 && da != 32 && da != 48 && da != 64))) return SCOPE_ERR_INVALID;
    if (!tchost::aligned16(a.q) || !tchost::aligned16(a.k) || a.q_sh % 8 || a.q_st % 8 || a.k_sh % 8 || a.k_st % 8 ||
        (da && (!tchost::aligned16(a.q_aug) || !tchost::aligned16(a.k_aug))))
        return SCOPE_ERR_ALIGN;
    if (!scope_device_supported() || !tchost::encode_fn()) return SCOPE_ERR_UNSUPPORTED;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    switch (da) {
        case 0: return tchost::launch_mass<0>(a, mass, s);
        case 16: return tchost::launch_mass<16>(a, mass, s);
        case 32: return tchost::launch_mass<32>(a, mass, s);
        case 48: return tchost::launch_mass<48>(a, mass, s);
        default: return tchost::launch_mass<64>(a, mass, s);
    }
}

// score_mod variant of the kernels: 0 (no score_mod), 1 (no gate), 2 (softplus), 3 (relu)
int scope_tc_smod(const ScopeAttnArgs &a) {
    if (a.bias_mode != SCOPE_BIAS_SCORE_MOD) return 0;
    if (a.gate == SCOPE_GATE_NONE || !(a.gate_lambda > 0.f)) return 1;
    return a.gate == SCOPE_GATE_SOFTPLUS ? 2 : 3;
}

bool scope_tc_eligible(const ScopeAttnArgs &a, bool bwd) {
    if (a.dtype != SCOPE_BF16 || a.block_size != 128 || a.D != 64) return false;
    // score_mod runs here with its Fourier sum in the aug dims (q_aug / k_aug from
    // scope_qk_aug_prepare without the slope column); without them, on the CUDA cores
    if (a.bias_mode == SCOPE_BIAS_SCORE_MOD &&
        (!a.q_aug || !a.k_aug || a.d_aug != (2 * a.K + 15) / 16 * 16 || a.d_aug > 32))
        return false;
    if (a.bias_mode == SCOPE_BIAS_QK_AUG && a.d_aug != 16 && a.d_aug != 32 && a.d_aug != 48 && a.d_aug != 64)
        return false;
    if (!scope_device_supported() || !tchost::encode_fn()) return false;
    // TMA: 16-byte aligned bases and strides; epilogues write 16-byte vectors
    const void *ptrs[8] = {a.q, a.k, a.v, a.out, a.dout, a.dq, a.dk, a.dv};
    const int64_t strides[16] = {a.q_sh, a.q_st, a.k_sh, a.k_st, a.v_sh, a.v_st, a.o_sh, a.o_st,
                                 a.do_sh, a.do_st, a.dq_sh, a.dq_st, a.dk_sh, a.dk_st, a.dv_sh, a.dv_st};
    const int n = bwd ? 8 : 4;
    for (int i = 0; i < n; ++i)
        if (!tchost::aligned16(ptrs[i]) || strides[2 * i] % 8 || strides[2 * i + 1] % 8) return false;
    if (a.bias_mode != SCOPE_BIAS_NONE && (!tchost::aligned16(a.q_aug) || !tchost::aligned16(a.k_aug))) return false;
    if (bwd && (!a.q_bitmap || !a.lse)) return false;
    return true;
}

int scope_tc_fwd(const ScopeAttnArgs &a, cudaStream_t s) {
    const int sm = scope_tc_smod(a);
    if (sm) {
        const bool d16 = a.d_aug == 16;
        switch (sm) {
            case 1: return d16 ? tchost::launch_fwd<16, 1>(a, s) : tchost::launch_fwd<32, 1>(a, s);
            case 2: return d16 ? tchost::launch_fwd<16, 2>(a, s) : tchost::launch_fwd<32, 2>(a, s);
            default: return d16 ? tchost::launch_fwd<16, 3>(a, s) : tchost::launch_fwd<32, 3>(a, s);
        }
    }
    switch (a.bias_mode == SCOPE_BIAS_QK_AUG ? a.d_aug : 0) {
        case 0: return tchost::launch_fwd<0, 0>(a, s);
        case 16: return tchost::launch_fwd<16, 0>(a, s);
        case 32: return tchost::launch_fwd<32, 0>(a, s);
        case 48: return tchost::launch_fwd<48, 0>(a, s);
        case 64: return tchost::launch_fwd<64, 0>(a, s);
        default: return SCOPE_ERR_INVALID;
    }
}

