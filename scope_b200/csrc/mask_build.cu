// Pointer block-mask builder for B200.
//
// Replaces SpectralBias.build_pointer_blockmask (model/attn_bias.py:623-874).
// Design: one warp owns one (head, query block) row for the whole build --
// pointer selection (a warp-wide Gumbel top-M over the causal candidates),
// radius allocation, the union of local / pointer / global windows and the
// de-duplicating pack all happen in registers and a per-warp shared-memory
// list, so a row costs one pass over its candidate logits and nothing else
// touches HBM.  The torch BlockMask's q-side transpose, which the reference
// gets from a dense [H,QB,QB] matrix and an argsort
// (torch/nn/attention/flex_attention.py:412-415), becomes one bit per
// (kb, qb) pair set with atomicOr into a bitmap the backward walks directly.
//
// Float32 steps use explicitly rounded intrinsics in the reference's
// operation order (no FMA contraction), so integer outputs are bit-identical
// to the reference given the same inputs and noise.
#include <algorithm>
#include <climits>
#include <cmath>

#include "common.cuh"

namespace scope {
namespace mask {

constexpr int kMaxM = 16;
constexpr int kWarps = 8;

// --------------------------------------------------------------------------
// document / reset starts per block (model/attn_bias.py:681-709)
// --------------------------------------------------------------------------
// Pass 1, one warp per block: the last change point inside the block, whether
// the block's first token is a change point, and the block's doc id range.
__global__ void block_info_pass1(const int32_t *__restrict__ docs, int T, int bs, int QB,
                                 int32_t *__restrict__ out) {
    int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (b >= QB) return;
    int base = b * bs;
    int last = -1, mn = INT_MAX, mx = INT_MIN;
    for (int i = lane; i < bs; i += 32) {
        int t = base + i;
        int d = docs ? docs[t] : 0;
        bool chg = (t == 0) || (docs && docs[t] != docs[t - 1]);
        if (chg) last = t;
        mn = min(mn, d);
        mx = max(mx, d);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
        mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 0) {
        bool first_chg = (base == 0) || (docs && docs[base] != docs[base - 1]);
        out[b] = last;
        out[QB + b] = first_chg ? base : -1;
        out[2 * QB + b] = mn;
        out[3 * QB + b] = mx;
    }
}

// Pass 2, one CTA: running max of change points -> doc_start_token at the
// representative (last) and first token of each block, then the clamps.
__global__ void __launch_bounds__(1024) block_info_pass2(int QB, int bs, int doc_clamp, int reset_active,
                                                        int reset_len, int32_t *__restrict__ out) {
    __shared__ int warp_max[32];
    const int tid = threadIdx.x, nt = blockDim.x;
    const int per = (QB + nt - 1) / nt;
    const int b0 = tid * per, b1 = min(QB, b0 + per);
    int local = -1;
    for (int b = b0; b < b1; ++b) local = max(local, out[b]);
    // exclusive block-wide max-scan of the per-thread maxima
    int lane = tid & 31, w = tid >> 5;
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = max(incl, y);
    }
    if (lane == 31) warp_max[w] = incl;
    __syncthreads();
    if (w == 0) {
        int v = (lane < (nt >> 5)) ? warp_max[lane] : -1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v = max(v, y);
        }
        warp_max[lane] = v;
    }
    __syncthreads();
    int excl = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) excl = -1;
    if (w > 0) excl = max(excl, warp_max[w - 1]);
    int run = excl;
    for (int b = b0; b < b1; ++b) {
        int last = out[b], first = out[QB + b];
        int dsl_tok = max(run, first);
        run = max(run, last);
        int dsp_tok = run;
        int dsp = dsp_tok / bs, dsl = dsl_tok / bs;
        if (!doc_clamp) dsp = dsl = 0;
        if (reset_active && reset_len > 0) {
            long long t_rep = (long long)(b + 1) * bs - 1;
            long long st = (long long)b * bs;
            dsp = max(dsp, (int)(((t_rep / reset_len) * reset_len) / bs));
            dsl = max(dsl, (int)(((st / reset_len) * reset_len) / bs));
        }
        out[b] = dsp;
        out[QB + b] = dsl;
    }
}

// --------------------------------------------------------------------------
// the per-row builder
// --------------------------------------------------------------------------
struct BuildParams {
    ScopeMaskArgs a;
    int max_kv;      // entries before de-duplication
    uint32_t span_mul;   // ceil(2^32 / span), span = 2 half_blocks + 1 (0 when span is 1): q / span = umulhi(q, span_mul)
    int per_warp;    // ints of shared memory per warp
    int np2;         // max_kv rounded up to a power of two (the sort buffer)
    int n_stats;     // ints of the statistics block
    int words;       // bitmap words per row
};

// x / d, with the division replaced by an exact multiply when d is a power of
// two (the configurations' temperatures): identical results, and the selection
// scan over ~QB/2 candidates per row stops being bound by IEEE division.
struct Divider {
    float d, inv;
    bool pow2;
    __device__ explicit Divider(float d_) : d(d_) {
        int e;
        const float m = frexpf(d_, &e);
        pow2 = (m == 0.5f) && e > -125 && e < 126;    // d = 2^(e-1): 1/d is exact and normal
        inv = pow2 ? ldexpf(1.0f, 1 - e) : 0.f;
    }
    __device__ __forceinline__ float operator()(float x) const { return pow2 ? __fmul_rn(x, inv) : __fdiv_rn(x, d); }
};

__device__ __forceinline__ bool better(float av, int ai, float bv, int bi) {
    return av > bv || (av == bv && ai < bi);
}

// insert (s, kb) into a descending top-M list held in registers
__device__ __forceinline__ void topm_insert(float (&v)[kMaxM], int (&id)[kMaxM], int M, float s, int kb) {
    if (!better(s, kb, v[M - 1], id[M - 1])) return;
    bool done = false;
#pragma unroll
    for (int j = kMaxM - 1; j >= 0; --j) {
        if (j < M && !done) {
            if (j > 0 && better(s, kb, v[j - 1], id[j - 1])) {
                v[j] = v[j - 1];
                id[j] = id[j - 1];
            } else {
                v[j] = s;
                id[j] = kb;
                done = true;
            }
        }
    }
}

__device__ __forceinline__ void topm_pop(float (&v)[kMaxM], int (&id)[kMaxM], int M) {
#pragma unroll
    for (int j = 0; j < kMaxM - 1; ++j) {
        if (j + 1 < M) {
            v[j] = v[j + 1];
            id[j] = id[j + 1];
        }
    }
    v[M - 1] = -INFINITY;
    id[M - 1] = INT_MAX;
}

// Gumbel top-M over candidates kb in [0, qb]; winners in descending score
// order (ties to the lower block) go to cen[0..M); missing ones become qb.
__device__ void select_row(const ScopeMaskArgs &a, int h, int qb, int lane, int *cen) {
    const int M = a.M;
    float v[kMaxM];
    int id[kMaxM];
#pragma unroll
    for (int j = 0; j < kMaxM; ++j) {
        v[j] = -INFINITY;
        id[j] = INT_MAX;
    }
    const float *lrow = a.sel_logits + (int64_t)h * a.sel_head_stride + (int64_t)qb * a.sel_row_stride;
    const float *grow = a.sel_gumbel + (int64_t)h * a.sel_head_stride + (int64_t)qb * a.sel_row_stride;
    const Divider tau(a.sel_tau);
    const int n = qb + 1;
    const bool vec = (a.QB % 4 == 0) && (a.sel_row_stride % 4 == 0) && (a.sel_head_stride % 4 == 0) &&
                     ((reinterpret_cast<uintptr_t>(a.sel_logits) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(a.sel_gumbel) & 15) == 0);
    if (vec) {
        // two float4 pairs in flight per lane per step
        for (int base = lane * 4; base < n; base += 256) {
            int b2 = base + 128;
            float4 l0 = __ldg(reinterpret_cast<const float4 *>(lrow + base));
            float4 g0 = __ldg(reinterpret_cast<const float4 *>(grow + base));
            float4 l1 = make_float4(0.f, 0.f, 0.f, 0.f), g1 = l1;
            if (b2 < n) {
                l1 = __ldg(reinterpret_cast<const float4 *>(lrow + b2));
                g1 = __ldg(reinterpret_cast<const float4 *>(grow + b2));
            }
            float lv[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
            float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                int kb = (e < 4) ? base + e : b2 + e - 4;
                if (kb < n) topm_insert(v, id, M, __fadd_rn(tau(lv[e]), gv[e]), kb);
            }
        }
    } else {
        for (int kb = lane; kb < n; kb += 32) {
            float s = __fadd_rn(tau(__ldg(lrow + kb)), __ldg(grow + kb));
            topm_insert(v, id, M, s, kb);
        }
    }
    for (int r = 0; r < M; ++r) {
        float bv = v[0];
        int bi = id[0];
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (bi != INT_MAX && id[0] == bi) topm_pop(v, id, M);
        if (lane == 0) cen[r] = (bi == INT_MAX) ? qb : bi;
    }
    __syncwarp();
}

// The same selection for rows of at most 32 * 32 candidates with every score in
// registers (compile-time indices, nothing in local memory): lane l holds the
// candidates kb = l + 32 e and a bitmask of those already taken; each lane
// keeps its best (score, block) among the untaken cached; per round a warp
// argmax picks the winner and only the winning lane rescans.  Order and ties
// as select_row; once every candidate is taken the rest of the centres are qb.
__device__ void select_row_regs(const ScopeMaskArgs &a, int h, int qb, int lane, int *cen) {
    constexpr int NE = 32;
    const float *lrow = a.sel_logits + (int64_t)h * a.sel_head_stride + (int64_t)qb * a.sel_row_stride;
    const float *grow = a.sel_gumbel + (int64_t)h * a.sel_head_stride + (int64_t)qb * a.sel_row_stride;
    const Divider tau(a.sel_tau);
    const int n = qb + 1;
    float sc[NE];
#pragma unroll
    for (int e = 0; e < NE; ++e) {
        const int kb = lane + 32 * e;
        sc[e] = (kb < n) ? __fadd_rn(tau(__ldg(lrow + kb)), __ldg(grow + kb)) : -INFINITY;
    }
    uint32_t taken = 0u;
    auto lane_best = [&](float &bv, int &bi) {
        bv = -INFINITY;
        bi = INT_MAX;
#pragma unroll
        for (int e = 0; e < NE; ++e) {
            const int kb = lane + 32 * e;
            if (kb < n && !((taken >> e) & 1u) && better(sc[e], kb, bv, bi)) {
                bv = sc[e];
                bi = kb;
            }
        }
    };
    float lv;
    int li;
    lane_best(lv, li);
    for (int r = 0; r < a.M; ++r) {
        float bv = lv;
        int bi = li;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) cen[r] = (bi == INT_MAX) ? qb : bi;
        if (bi != INT_MAX && li == bi) {
            // the winner is this lane's cached best: mark it taken and rescan
            taken |= 1u << ((bi - lane) >> 5);
            lane_best(lv, li);
        }
    }
    __syncwarp();
}

// The same selection by a threshold filter, 1,024 candidates (a chunk) at a
// time: lane l holds kb = c0 + 128 g + 4 l + c (g < 8, c < 4) of chunk c0.
// The M-th largest of the 32 lane maxima bounds the chunk's own M-th best
// score (those lane maxima are M distinct candidates), and the running M-th
// best of the earlier chunks bounds what can still enter, so only candidates
// scoring at least both are compacted into shared memory, next to the running
// top-M, and ranked by one warp bitonic sort under the order better() uses.
// Returns false, leaving cen untouched, when a chunk passes more candidates
// than fit beside the running list or a score is NaN: the caller then runs an
// exact path, so the result is the same either way.
__device__ bool select_row_thr(const ScopeMaskArgs &a, int h, int qb, int lane, int *cen, float *sv, int *si) {
    const float *lrow = a.sel_logits + (int64_t)h * a.sel_head_stride + (int64_t)qb * a.sel_row_stride;
    const float *grow = a.sel_gumbel + (int64_t)h * a.sel_head_stride + (int64_t)qb * a.sel_row_stride;
    const Divider tau(a.sel_tau);
    const int n = qb + 1, M = a.M;
    const bool vec = (a.QB % 4 == 0) && (a.sel_row_stride % 4 == 0) && (a.sel_head_stride % 4 == 0) &&
                     ((reinterpret_cast<uintptr_t>(a.sel_logits) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(a.sel_gumbel) & 15) == 0);
    // the running top-M: lane r < kept holds entry r, best first
    float v = -INFINITY;
    int id = INT_MAX;
    int kept = 0;
    float thr_run = -INFINITY;   // its M-th score once M are kept
    for (int c0 = 0; c0 < n; c0 += 1024) {
        float sc[32];
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const int b = c0 + 128 * g + 4 * lane;
            float lv[4] = {0.f, 0.f, 0.f, 0.f}, gv[4] = {0.f, 0.f, 0.f, 0.f};
            if (b < n) {
                if (vec) {
                    const float4 l4 = __ldg(reinterpret_cast<const float4 *>(lrow + b));
                    const float4 g4 = __ldg(reinterpret_cast<const float4 *>(grow + b));
                    lv[0] = l4.x; lv[1] = l4.y; lv[2] = l4.z; lv[3] = l4.w;
                    gv[0] = g4.x; gv[1] = g4.y; gv[2] = g4.z; gv[3] = g4.w;
                } else {
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        if (b + c < n) {
                            lv[c] = __ldg(lrow + b + c);
                            gv[c] = __ldg(grow + b + c);
                        }
                }
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) sc[4 * g + c] = (b + c < n) ? __fadd_rn(tau(lv[c]), gv[c]) : -INFINITY;
        }
        // lane maximum with NaN propagation (max.NaN), so a NaN anywhere shows in it
        float lm = sc[0];
#pragma unroll
        for (int e = 1; e < 32; e += 2) {
            if (e + 1 < 32) {
                asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(lm) : "f"(lm), "f"(sc[e]), "f"(sc[e + 1]));
            } else {
                asm("max.NaN.f32 %0, %1, %2;" : "=f"(lm) : "f"(lm), "f"(sc[e]));
            }
        }
        if (__any_sync(0xffffffffu, isnan(lm))) return false;
        // the M-th largest lane maximum: a descending bitonic sort of the 32 values
        float t = lm;
#pragma unroll
        for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
            for (int j = k >> 1; j > 0; j >>= 1) {
                const float o = __shfl_xor_sync(0xffffffffu, t, j);
                const bool desc = (lane & k) == 0, lower = (lane & j) == 0;
                t = (lower == desc) ? fmaxf(t, o) : fminf(t, o);
            }
        }
        const float thr = fmaxf(__shfl_sync(0xffffffffu, t, M - 1), thr_run);
        // the candidates that can still win, compacted in lane order after the running list
        uint32_t hit = 0u;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            const int kb = c0 + 128 * (e >> 2) + 4 * lane + (e & 3);
            if (kb < n && sc[e] >= thr) hit |= 1u << e;
        }
        const int cnt = __popc(hit);
        int pre = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, pre, o);
            if (lane >= o) pre += y;
        }
        const int total = __shfl_sync(0xffffffffu, pre, 31);
        if (kept + total > 32) return false;
        if (lane < kept) {
            sv[lane] = v;
            si[lane] = id;
        }
        int pos = kept + pre - cnt;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            if ((hit >> e) & 1u) {
                sv[pos] = sc[e];
                si[pos] = c0 + 128 * (e >> 2) + 4 * lane + (e & 3);
                ++pos;
            }
        }
        __syncwarp();
        const int m = kept + total;
        v = lane < m ? sv[lane] : -INFINITY;
        id = lane < m ? si[lane] : INT_MAX;
        __syncwarp();
        // warp bitonic sort, best first under better()
#pragma unroll
        for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
            for (int j = k >> 1; j > 0; j >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, v, j);
                const int oi = __shfl_xor_sync(0xffffffffu, id, j);
                const bool desc = (lane & k) == 0, lower = (lane & j) == 0;
                if ((lower == desc) ? better(ov, oi, v, id) : better(v, id, ov, oi)) {
                    v = ov;
                    id = oi;
                }
            }
        }
        kept = min(m, M);
        if (lane >= kept) {
            v = -INFINITY;
            id = INT_MAX;
        }
        if (kept == M) thr_run = __shfl_sync(0xffffffffu, v, M - 1);
    }
    if (lane < M) cen[lane] = (id == INT_MAX) ? qb : id;
    __syncwarp();
    return true;
}

// Ascending bitonic sort of 32 E ints held E per lane (element i = E lane + k):
// partners closer than E are in the same lane, the others one shuffle away.
template <int E>
__device__ __forceinline__ void warp_sort_regs(int (&v)[E], int lane) {
#pragma unroll
    for (int k = 2; k <= 32 * E; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j < E) {
#pragma unroll
                for (int q = 0; q < E; ++q) {
                    const int pq = q ^ j;
                    if (pq > q) {
                        const bool asc = ((E * lane + q) & k) == 0;
                        const int lo = min(v[q], v[pq]), hi = max(v[q], v[pq]);
                        v[q] = asc ? lo : hi;
                        v[pq] = asc ? hi : lo;
                    }
                }
            } else {
                const int lj = j / E;
                const bool lower = (lane & lj) == 0;
#pragma unroll
                for (int q = 0; q < E; ++q) {
                    const int o = __shfl_xor_sync(0xffffffffu, v[q], lj);
                    const bool asc = ((E * lane + q) & k) == 0;
                    v[q] = (lower == asc) ? min(v[q], o) : max(v[q], o);
                }
            }
        }
    }
}

// The window entries of a row (model/attn_bias.py:786-825): entry pos of the
// local blocks, the M pointer windows and the global blocks.
__device__ __forceinline__ int window_entry(const ScopeMaskArgs &a, uint32_t span_mul, int pos, int qb, int dsp,
                                            int dsl, const int *cen, const int *rad) {
    const int L = a.local_blocks, M = a.M, p = a.half_blocks, span = 2 * p + 1;
    if (pos < L) return max(max(qb - pos, 0), dsl);
    if (pos < L + M * span) {
        const int q = pos - L, m = span_mul ? (int)__umulhi((uint32_t)q, span_mul) : q, c = cen[m];
        if (p > 0) {
            const int o = q - m * span - p;
            int w = min(max(c + o, 0), a.QB - 1);
            w = max(min(w, qb), dsp);
            return (abs(o) <= rad[m]) ? w : c;
        }
        return c;
    }
    const int i = pos - L - M * span;
    const int g = min(dsp + i, qb);
    return (i < a.global_active) ? g : qb;
}

// Window entries sorted and packed in registers (rows of at most 32 E
// entries): unique blocks ascending, then the repeats ascending, into outl;
// returns the number of unique blocks.
template <int E>
__device__ int pack_row_regs(const ScopeMaskArgs &a, uint32_t span_mul, int n, int qb, int dsp, int dsl, const int *cen,
                             const int *rad, int lane, int *outl) {
    int v[E];
#pragma unroll
    for (int q = 0; q < E; ++q) {
        const int pos = E * lane + q;
        v[q] = pos < n ? window_entry(a, span_mul, pos, qb, dsp, dsl, cen, rad) : INT_MAX;   // INT_MAX sorts past every block
    }
    warp_sort_regs<E>(v, lane);
    const int prev_lane_last = __shfl_up_sync(0xffffffffu, v[E - 1], 1);
    bool first[E];
    int cnt = 0;
#pragma unroll
    for (int q = 0; q < E; ++q) {
        const int pos = E * lane + q;
        const int prev = q > 0 ? v[q - 1] : prev_lane_last;
        first[q] = pos < n && (pos == 0 || prev != v[q]);
        cnt += first[q] ? 1 : 0;
    }
    int pre = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, pre, o);
        if (lane >= o) pre += y;
    }
    const int num = __shfl_sync(0xffffffffu, pre, 31);
    int fb = pre - cnt;   // firsts before this lane's first element
#pragma unroll
    for (int q = 0; q < E; ++q) {
        const int pos = E * lane + q;
        if (pos < n) outl[first[q] ? fb : num + (pos - fb)] = v[q];
        fb += first[q] ? 1 : 0;
    }
    __syncwarp();
    return num;
}

// four CTAs (32 warps) per SM: the row's selection and sort are latency chains
// that more warps in flight hide better than more registers per thread would
__global__ void __launch_bounds__(kWarps * 32, 4) build_kernel(const BuildParams P) {
    extern __shared__ int smem[];
    const ScopeMaskArgs &a = P.a;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int *vals = smem + wid * P.per_warp;  // [np2]: the row's window entries, sorted in place
    int *outl = vals + P.np2;             // [max_kv]: packed list
    int *cen = outl + P.max_kv;           // [kMaxM]
    int *rad = cen + kMaxM;               // [kMaxM]
    float *alloc = reinterpret_cast<float *>(rad + kMaxM);  // [kMaxM]
    float *frac = alloc + kMaxM;          // [kMaxM]
    float *selv = frac + kMaxM;           // [32]: select_row_thr's candidates
    int *seli = reinterpret_cast<int *>(selv + 32);   // [32]
    int *hist = smem + nw * P.per_warp;   // [n_stats] per CTA
    const bool want_stats = a.stats != nullptr;
    if (want_stats)
        for (int i = threadIdx.x; i < P.n_stats; i += blockDim.x) hist[i] = 0;
    __syncthreads();

    const int H = a.H, QB = a.QB, M = a.M, L = a.local_blocks, p = a.half_blocks, G = a.global_max;
    const int span = 2 * p + 1;
    const int n = P.max_kv;
    const int *dspA = a.block_info;
    const int *dslA = a.block_info + QB;
    const int rows = H * QB;
    const int hist_r = n + 1;                       // radius histogram offset
    const int hist_e = hist_r + p + 1;              // extra-sum histogram offset
    const int max_extra = max(1, p * M);
    const int hist_z = hist_e + max_extra + 1;      // zero-radius count

    for (int row = blockIdx.x * nw + wid; row < rows; row += gridDim.x * nw) {
        const int h = row / QB, qb = row - h * QB;
        const int dsp = dspA[qb], dsl = dslA[qb];

        // ---- pointer centres (model/attn_bias.py:779-784) ----
        if (a.sel_logits) {
            if (!select_row_thr(a, h, qb, lane, cen, selv, seli)) {
                if (qb < 32 * 32) select_row_regs(a, h, qb, lane, cen);
                else select_row(a, h, qb, lane, cen);
            }
        } else if (lane < M) {
            float d = a.delta_rep[(int64_t)h * a.delta_head_stride + (int64_t)qb * a.delta_row_stride +
                                  (int64_t)lane * a.delta_m_stride];
            float key = __fsub_rn((float)((qb + 1) * a.block_size - 1), d);
            key = fmaxf(key, 0.0f);
            long long kt = (long long)key;
            long long cb = kt / a.block_size;
            cen[lane] = (int)(cb < (long long)INT_MAX ? cb : (long long)INT_MAX);
        }
        __syncwarp();
        if (lane < M) {
            int c = min(cen[lane], qb);
            if (!a.ptr_enabled) c = qb;
            cen[lane] = max(c, dsp);
        }

        // ---- radius allocation (model/attn_bias.py:721-761) ----
        const float *brow = a.budget_rep + (int64_t)h * a.budget_head_stride + (int64_t)qb * a.budget_row_stride;
        int r = 0;
        if (a.radius_mode == 0) {
            r = a.half_active;
        } else if (a.budget_rem > 0) {
            // the M - 1 stick fractions are independent: one lane each; only the
            // breaking itself (two dependent roundings per stick) runs in lane 0
            if (lane < M - 1) {
                float u = __fdiv_rn(brow[(int64_t)lane * a.budget_m_stride], a.budget_temp);
                alloc[lane] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-u)));
            }
            __syncwarp();
            if (lane == 0) {
                float rem = (float)a.budget_rem;
                for (int m = 0; m < M - 1; ++m) {
                    float bb = __fmul_rn(alloc[m], rem);
                    alloc[m] = bb;
                    rem = __fsub_rn(rem, bb);
                }
                alloc[M - 1] = rem;
            }
            __syncwarp();
            float fl = 0.f, fr = 0.f;
            if (lane < M) {
                fl = floorf(alloc[lane]);
                fr = __fsub_rn(alloc[lane], fl);
                frac[lane] = fr;
            }
            int fsum = (lane < M) ? (int)fl : 0;
#pragma unroll
            for (int o = 16; o; o >>= 1) fsum += __shfl_xor_sync(0xffffffffu, fsum, o);
            __syncwarp();
            if (lane < M) {
                int rem_int = min(max(a.budget_rem - fsum, 0), M);
                int rank = 0;
                for (int j = 0; j < M; ++j) {
                    float fj = frac[j];
                    rank += (fj > fr) || (fj == fr && j < lane);
                }
                float extra = fl + ((rank < rem_int) ? 1.0f : 0.0f);
                r = min(max((int)extra, 0), p);
            }
        }
        r = min(r, a.half_active);
        if (!a.ptr_enabled) r = 0;
        // Gumbel peak masking (model/attn_bias.py:763-777)
        if (a.peak_gumbel && a.gumbel_k > 0 && a.gumbel_k < M && p > 0) {
            float s = -INFINITY;
            if (lane < M)
                s = __fadd_rn(__fdiv_rn(brow[(int64_t)lane * a.budget_m_stride], a.gumbel_tau),
                              a.peak_gumbel[(int64_t)row * M + lane]);
            int rank = 0;
            for (int j = 0; j < M; ++j) {
                float sj = __shfl_sync(0xffffffffu, s, j);
                rank += (sj > s) || (sj == s && j < lane);
            }
            if (rank >= a.gumbel_k) r = 0;
        }
        if (lane < M) rad[lane] = r;
        __syncwarp();

        // ---- window pieces (model/attn_bias.py:786-825), de-duplicated and packed
        // (model/attn_bias.py:828-837): in registers for rows of up to 128 entries ----
        int num = 0;
        if (P.np2 <= 128) {
            if (P.np2 == 32) num = pack_row_regs<1>(a, P.span_mul, n, qb, dsp, dsl, cen, rad, lane, outl);
            else if (P.np2 == 64) num = pack_row_regs<2>(a, P.span_mul, n, qb, dsp, dsl, cen, rad, lane, outl);
            else num = pack_row_regs<4>(a, P.span_mul, n, qb, dsp, dsl, cen, rad, lane, outl);
        } else {
        for (int pos = lane; pos < n; pos += 32) {
            int val;
            if (pos < L) {
                val = max(max(qb - pos, 0), dsl);
            } else if (pos < L + M * span) {
                int q = pos - L;
                int m = q / span;
                int c = cen[m];
                if (p > 0) {
                    int o = q - m * span - p;
                    int w = min(max(c + o, 0), QB - 1);
                    w = max(min(w, qb), dsp);
                    val = (abs(o) <= rad[m]) ? w : c;
                } else {
                    val = c;
                }
            } else {
                int i = pos - L - M * span;
                int g = min(dsp + i, qb);
                val = (i < a.global_active) ? g : qb;
            }
            vals[pos] = val;
        }
        for (int pos = n + lane; pos < P.np2; pos += 32) vals[pos] = INT_MAX;   // sorts past every block
        __syncwarp();

        // ---- de-duplicate and pack (model/attn_bias.py:828-837) ----
        // The reference sorts, keeps the first of each run, and stably re-sorts on
        // (!keep, value): the unique blocks ascending, then the repeats ascending.
        // Here: a warp bitonic sort of the entries in shared memory, then runs
        // are found by comparing neighbours and packed with ballot prefix counts.
        const int N2 = P.np2;
        for (int kk = 2; kk <= N2; kk <<= 1) {
            for (int jj = kk >> 1; jj > 0; jj >>= 1) {
                for (int t = lane; t < (N2 >> 1); t += 32) {
                    const int i = ((t & ~(jj - 1)) << 1) | (t & (jj - 1));   // lower element of pair t
                    const int l = i + jj;
                    const int x = vals[i], y = vals[l];
                    if ((x > y) == ((i & kk) == 0)) {
                        vals[i] = y;
                        vals[l] = x;
                    }
                }
                __syncwarp();
            }
        }
        for (int c0 = 0; c0 < n; c0 += 32) {
            const int pos = c0 + lane;
            const bool first = pos < n && (pos == 0 || vals[pos - 1] != vals[pos]);
            num += __popc(__ballot_sync(0xffffffffu, first));
        }
        int firsts_before = 0;
        for (int c0 = 0; c0 < n; c0 += 32) {
            const int pos = c0 + lane;
            const int v = pos < n ? vals[pos] : 0;
            const bool first = pos < n && (pos == 0 || vals[pos - 1] != v);
            const unsigned fb = __ballot_sync(0xffffffffu, first);
            const int pre = firsts_before + __popc(fb & ((1u << lane) - 1u));
            if (pos < n) outl[first ? pre : num + (pos - pre)] = v;
            firsts_before += __popc(fb);
        }
        __syncwarp();
        }

        // ---- outputs ----
        if (lane == 0) a.kv_num[row] = num;
        int32_t *krow = a.kv_indices + (int64_t)row * a.kv_stride;
        if (a.flex_padded) {
            for (int j = lane; j < QB; j += 32) krow[j] = (j < n) ? outl[j] : outl[0];
        } else {
            int wlen = min(n, a.kv_stride);
            for (int j = lane; j < wlen; j += 32) krow[j] = outl[j];
            if (n > a.kv_stride && lane == 0) set_err(a.err_flag, SCOPE_DEVERR_SHAPE);
        }
        if (a.q_bitmap) {
            for (int j = lane; j < num; j += 32) {
                int kb = outl[j];
                if (kb >= 0 && kb < QB)
                    atomicOr(a.q_bitmap + ((int64_t)h * QB + kb) * P.words + (qb >> 5), 1u << (qb & 31));
                else
                    set_err(a.err_flag, SCOPE_DEVERR_INDEX);
            }
        }
        if (lane < M) {
            if (a.r_m_out) a.r_m_out[(int64_t)row * M + lane] = rad[lane];
            if (a.centres_out) a.centres_out[(int64_t)row * M + lane] = cen[lane];
        }
        if (want_stats) {
            int rr = (lane < M) ? rad[lane] : 0;
            int esum = rr;
#pragma unroll
            for (int o = 16; o; o >>= 1) esum += __shfl_xor_sync(0xffffffffu, esum, o);
            if (lane == 0) {
                atomicAdd(&hist[min(num, n)], 1);
                atomicAdd(&hist[hist_e + min(esum, max_extra)], 1);
            }
            if (lane < M) {
                atomicAdd(&hist[hist_r + min(max(rr, 0), p)], 1);
                if (rr == 0) atomicAdd(&hist[hist_z], 1);
            }
        }
        __syncwarp();
    }
    if (want_stats) {
        __syncthreads();
        for (int i = threadIdx.x; i < P.n_stats; i += blockDim.x)
            if (hist[i]) atomicAdd(a.stats + i, hist[i]);
    }
}

// --------------------------------------------------------------------------
// q-side lists in torch's layout, from the bitmap
// --------------------------------------------------------------------------
__global__ void transpose_kernel(const uint32_t *__restrict__ bm, int H, int QB, int words,
                                 int32_t *__restrict__ q_num, int32_t *__restrict__ q_idx) {
    int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;   // (h, kb)
    int lane = threadIdx.x & 31;
    if (row >= H * QB) return;
    const uint32_t *r = bm + (int64_t)row * words;
    int cnt = 0;
    for (int w = lane; w < words; w += 32) cnt += __popc(r[w]);
#pragma unroll
    for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if (lane == 0) q_num[row] = cnt;
    if (!q_idx) return;
    int32_t *out = q_idx + (int64_t)row * QB;
    int seen_set = 0, seen_unset = 0;   // running counts over earlier chunks
    for (int w0 = 0; w0 < words; w0 += 32) {
        int w = w0 + lane;
        uint32_t bits = (w < words) ? r[w] : 0u;
        int nvalid = min(32, QB - w * 32);
        if (w >= words) nvalid = 0;
        uint32_t vmask = (nvalid >= 32) ? 0xffffffffu : ((nvalid > 0) ? ((1u << nvalid) - 1u) : 0u);
        bits &= vmask;
        int ns = __popc(bits), nu = __popc(vmask & ~bits);
        int ps = ns, pu = nu;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int ys = __shfl_up_sync(0xffffffffu, ps, o), yu = __shfl_up_sync(0xffffffffu, pu, o);
            if (lane >= o) {
                ps += ys;
                pu += yu;
            }
        }
        int es = seen_set + ps - ns, eu = seen_unset + pu - nu;
        for (int b = 0; b < nvalid; ++b) {
            int qb = w * 32 + b;
            if ((bits >> b) & 1u) out[es++] = qb;
            else out[cnt + eu++] = qb;
        }
        seen_set += __shfl_sync(0xffffffffu, ps, 31);
        seen_unset += __shfl_sync(0xffffffffu, pu, 31);
    }
}

}  // namespace mask
}  // namespace scope

using namespace scope;

extern "C" int32_t scope_mask_max_kv(int32_t local_blocks, int32_t M, int32_t half_blocks, int32_t global_max) {
    return local_blocks + (half_blocks > 0 ? M * (2 * half_blocks + 1) : M) + global_max;
}

extern "C" int scope_block_info(const int32_t *docs, int32_t T, int32_t block_size, int32_t doc_clamp,
                                int32_t reset_active, int32_t reset_len, int32_t *out, scope_stream_t stream) {
    if (T <= 0 || block_size <= 0 || T % block_size != 0 || !out) return SCOPE_ERR_INVALID;
    int QB = T / block_size;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    mask::block_info_pass1<<<ceil_div(QB * 32, 256), 256, 0, s>>>(docs, T, block_size, QB, out);
    SCOPE_CHECK_LAUNCH();
    mask::block_info_pass2<<<1, 1024, 0, s>>>(QB, block_size, doc_clamp, reset_active, reset_len, out);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

extern "C" int scope_mask_build(const ScopeMaskArgs *args, scope_stream_t stream) {
    if (!args) return SCOPE_ERR_INVALID;
    const ScopeMaskArgs &a = *args;
    if (a.H <= 0 || a.QB <= 0 || a.M <= 0 || a.M > mask::kMaxM || a.block_size <= 0) return SCOPE_ERR_INVALID;
    if ((a.sel_logits == nullptr) == (a.delta_rep == nullptr)) return SCOPE_ERR_INVALID;
    if (a.sel_logits && (!a.sel_gumbel || a.sel_row_stride < a.QB)) return SCOPE_ERR_INVALID;
    if (!a.budget_rep && a.radius_mode == 1 && a.budget_rem > 0) return SCOPE_ERR_INVALID;
    if (!a.block_info || !a.kv_num || !a.kv_indices) return SCOPE_ERR_INVALID;
    if (a.local_blocks < 1 || a.local_blocks > a.QB || a.half_blocks < 0 || a.global_max < 0 ||
        a.global_max > a.QB || a.global_active < 0 || a.global_active > a.global_max)
        return SCOPE_ERR_INVALID;
    if (a.radius_mode == 1 && a.budget_rem > 0 && !(a.budget_temp > 0.f)) return SCOPE_ERR_INVALID;
    if (a.sel_logits && !(a.sel_tau > 0.f)) return SCOPE_ERR_INVALID;
    if (a.peak_gumbel && !(a.gumbel_tau > 0.f)) return SCOPE_ERR_INVALID;
    int max_kv = scope_mask_max_kv(a.local_blocks, a.M, a.half_blocks, a.global_max);
    if (a.flex_padded ? (a.kv_stride != a.QB) : (a.kv_stride < max_kv)) return SCOPE_ERR_INVALID;
    mask::BuildParams P;
    P.a = a;
    P.max_kv = max_kv;
    P.np2 = 32;
    while (P.np2 < max_kv) P.np2 <<= 1;
    P.per_warp = P.np2 + max_kv + 4 * mask::kMaxM + 64;
    P.n_stats = (max_kv + 1) + (a.half_blocks + 1) + (std::max(1, a.half_blocks * a.M) + 1) + 1;
    P.words = (a.QB + 31) / 32;
    {
        // 0 stands for span 1 (q / 1 = q); otherwise exact for every q the rows hold (q < 2^20)
        const uint64_t span = 2ull * (uint64_t)a.half_blocks + 1ull;
        P.span_mul = span == 1 ? 0u : (uint32_t)(((1ull << 32) + span - 1) / span);
    }
    int nwarps = mask::kWarps;
    size_t smem = (size_t)(nwarps * P.per_warp + P.n_stats) * sizeof(int);
    while (smem > 160 * 1024 && nwarps > 1) {
        nwarps >>= 1;
        smem = (size_t)(nwarps * P.per_warp + P.n_stats) * sizeof(int);
    }
    if (smem > 200 * 1024) return SCOPE_ERR_INVALID;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(mask::build_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return SCOPE_ERR_CUDA;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int rows = a.H * a.QB;
    // one wave of resident CTAs, rows taken in a grid-stride loop
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mask::build_kernel, nwarps * 32, smem) != cudaSuccess ||
        per_sm < 1)
        per_sm = 1;
    int grid = std::min(ceil_div(rows, nwarps), sms * per_sm);
    mask::build_kernel<<<grid, nwarps * 32, smem, s>>>(P);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

extern "C" int scope_mask_transpose(const uint32_t *q_bitmap, int32_t H, int32_t QB, int32_t *q_num,
                                    int32_t *q_indices, scope_stream_t stream) {
    if (!q_bitmap || !q_num || H <= 0 || QB <= 0) return SCOPE_ERR_INVALID;
    int words = (QB + 31) / 32;
    int rows = H * QB;
    mask::transpose_kernel<<<ceil_div(rows * 32, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        q_bitmap, H, QB, words, q_num, q_indices);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

// ---------------------------------------------------------------------------
// Kernel tiles of a coarse mask: block_size 2*bs -> bs.  Fine q block
// q' = 2*qb + s sees fine kv blocks 2*kb and 2*kb + 1 of every coarse kb in
// its coarse row, minus those wholly in its causal future (fine kv block >
// q', where every key follows every query); order stays ascending.  The
// element mask (document-causal) is applied inside the tiles as before.
namespace scope {
namespace mask {
__global__ void refine_kernel(const int32_t *__restrict__ kv_num, const int32_t *__restrict__ kv_idx, int H, int QB,
                              int kv_stride, int32_t *__restrict__ kv_num_out, int32_t *__restrict__ kv_idx_out,
                              int kv_stride_out, uint32_t *__restrict__ q_bitmap_out, int32_t *err) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;   // (h, fine q block)
    const int QF = 2 * QB;
    if (row >= H * QF) return;
    const int h = row / QF, qf = row - h * QF, qb = qf >> 1;
    const int words = (QF + 31) / 32;
    const int32_t *src = kv_idx + ((int64_t)h * QB + qb) * kv_stride;
    int32_t *dst = kv_idx_out + (int64_t)row * kv_stride_out;
    const int n = kv_num[(int64_t)h * QB + qb];
    int m = 0;
    for (int e = 0; e < n; ++e) {
        const int kb = src[e];
        if (kb < 0 || kb >= QB) {          // skipped, as the attention kernels would
            set_err(err, SCOPE_DEVERR_INDEX);
            continue;
        }
        for (int t = 0; t < 2; ++t) {
            const int kf = 2 * kb + t;
            if (kf > qf) break;
            dst[m++] = kf;
            atomicOr(q_bitmap_out + ((int64_t)h * QF + kf) * words + (qf >> 5), 1u << (qf & 31));
        }
    }
    kv_num_out[row] = m;
}
}  // namespace mask
}  // namespace scope

extern "C" int scope_mask_refine(const int32_t *kv_num, const int32_t *kv_indices, int32_t H, int32_t QB,
                                 int32_t kv_stride, int32_t *kv_num_out, int32_t *kv_indices_out,
                                 int32_t kv_stride_out, uint32_t *q_bitmap_out, int32_t *err_flag,
                                 scope_stream_t stream) {
    if (!kv_num || !kv_indices || !kv_num_out || !kv_indices_out || !q_bitmap_out || H <= 0 || QB <= 0 ||
        kv_stride <= 0 || kv_stride_out < 2 * kv_stride)
        return SCOPE_ERR_INVALID;
    const int rows = H * 2 * QB;
    scope::mask::refine_kernel<<<ceil_div(rows, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        kv_num, kv_indices, H, QB, kv_stride, kv_num_out, kv_indices_out, kv_stride_out, q_bitmap_out, err_flag);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}

// ---------------------------------------------------------------------------
// q-side bitmap of a mask given only its kv lists (a torch BlockMask handed to
// the attention drop-in): bit qb of row (h, kb) set for every kb among the
// first kv_num[h, qb] entries of row (h, qb).  The caller zeroes the bitmap.
namespace scope {
namespace mask {
__global__ void lists_bitmap_kernel(const int32_t *__restrict__ kv_num, const int32_t *__restrict__ kv_idx, int H,
                                    int QB, int kv_stride, uint32_t *__restrict__ q_bitmap, int32_t *err) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;   // (h, q block)
    if (row >= H * QB) return;
    const int h = row / QB, qb = row - h * QB;
    const int words = (QB + 31) / 32;
    const int32_t *src = kv_idx + (int64_t)row * kv_stride;
    int n = kv_num[row];
    if (n < 0 || n > kv_stride) {
        set_err(err, SCOPE_DEVERR_SHAPE);
        n = n < 0 ? 0 : kv_stride;
    }
    for (int e = 0; e < n; ++e) {
        const int kb = src[e];
        if (kb < 0 || kb >= QB) {            // skipped, as the attention kernels skip it
            set_err(err, SCOPE_DEVERR_INDEX);
            continue;
        }
        atomicOr(q_bitmap + ((int64_t)h * QB + kb) * words + (qb >> 5), 1u << (qb & 31));
    }
}
}  // namespace mask
}  // namespace scope

extern "C" int scope_mask_bitmap_from_lists(const int32_t *kv_num, const int32_t *kv_indices, int32_t H, int32_t QB,
                                            int32_t kv_stride, uint32_t *q_bitmap, int32_t *err_flag,
                                            scope_stream_t stream) {
    if (!kv_num || !kv_indices || !q_bitmap || H <= 0 || QB <= 0 || kv_stride <= 0) return SCOPE_ERR_INVALID;
    const int rows = H * QB;
    scope::mask::lists_bitmap_kernel<<<ceil_div(rows, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        kv_num, kv_indices, H, QB, kv_stride, q_bitmap, err_flag);
    SCOPE_CHECK_LAUNCH();
    return SCOPE_OK;
}
