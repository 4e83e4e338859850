// sm_100a building blocks written directly in PTX: mbarriers with bounded
// waits, TMA tile loads, and the tcgen05 tensor-core / tensor-memory ops.
//
// Encodings of the shared-memory matrix descriptor and the kind::f16
// instruction descriptor follow the PTX ISA's tcgen05 chapter (the same bit
// layout CUTLASS's UMMA::SmemDescriptor / UMMA::InstrDescriptor spell out).
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace scope {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// One arrival per thread of the calling warp, made by lane 0 after the warp
// synchronised (bar.warp.sync orders the lanes' prior memory operations, and
// tcgen05 operations fenced with tcgen05.fence::before_thread_sync, before it).
__device__ __forceinline__ void mbar_arrive_warp(uint64_t *bar) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0)
        asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], 32;" ::"r"(smem_u32(bar)) : "memory");
    __syncwarp();
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
// try_wait without a suspend-time hint: the thread blocks for a
// system-dependent time and wakes when the phase completes.  (A hint made the
// measured arrive -> wake round trip between two warps ~35% longer on B200.)
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Wait for the phase with the given parity to complete, for at most
// `limit_ns` nanoseconds of wall time.  Returns false when the wait gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait(a, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// The same bounded wait for warps that only wait (the TMA producer and the
// tcgen05 issuer): each poll carries a suspend-time hint, so the warp sleeps in
// the barrier until the phase completes instead of re-polling.
__device__ __forceinline__ bool mbar_wait_idle(uint64_t *bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok)
            : "r"(a), "r"(parity), "r"(1000000u)
            : "memory");
        if (ok) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// Non-blocking test of a phase, decided by lane 0 of a converged warp and
// broadcast, so the whole warp takes the same branch.
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok = 0;
    if ((threadIdx.x & 31) == 0) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(const CUtensorMap *m, void *dst, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(const CUtensorMap *m, void *dst, uint64_t *bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// element-wise add of a shared-memory box into the tensor map's box at (x, y) (fp32
// maps: x must be a multiple of 4); tracked by the issuing thread's bulk groups
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *m, const void *src, int x, int y) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N of this thread's bulk groups are still reading shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// wait until every bulk group of this thread completed
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// contiguous global -> shared copy of `bytes` (multiple of 16, both ends 16-byte aligned)
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// arrive on `bar` once every tcgen05 op this thread issued so far has completed
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
// Issuing: the whole issuing warp waits on its mbarriers (warp-uniform
// control flow), then one lane issues a batch of MMAs and the commits that
// track them, followed by __syncwarp().  (An elect.sync per instruction cost
// the warps sharing the SM sub-partition ~5x more issue slots per MMA in a
// measurement on B200.)
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// After tcgen05.wait::ld: make the loaded registers opaque so no use of them
// is scheduled above the wait (tcgen05.ld writes them asynchronously).
template <int N>
__device__ __forceinline__ void pin(uint32_t (&r)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

#define SCOPE_R8(b) "=r"(r[b + 0]), "=r"(r[b + 1]), "=r"(r[b + 2]), "=r"(r[b + 3]), "=r"(r[b + 4]), "=r"(r[b + 5]), "=r"(r[b + 6]), "=r"(r[b + 7])
#define SCOPE_W8(b) "r"(r[b + 0]), "r"(r[b + 1]), "r"(r[b + 2]), "r"(r[b + 3]), "r"(r[b + 4]), "r"(r[b + 5]), "r"(r[b + 6]), "r"(r[b + 7])

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets lane
// (lane base of taddr + t), columns [col, col+32) of taddr.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : SCOPE_R8(0), SCOPE_R8(8), SCOPE_R8(16), SCOPE_R8(24)
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        SCOPE_W8(0), SCOPE_W8(8), SCOPE_W8(16), SCOPE_W8(24)
        : "memory");
}
// loads without the wait (issue several, then one tmem_wait_ld)
__device__ __forceinline__ void tmem_ld32_nw(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : SCOPE_R8(0), SCOPE_R8(8), SCOPE_R8(16), SCOPE_R8(24)
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : SCOPE_R8(0), SCOPE_R8(8)
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld1(uint32_t taddr, uint32_t &r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        SCOPE_W8(0), SCOPE_W8(8)
        : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), SCOPE_W8(0)
                 : "memory");
}
#undef SCOPE_R8
#undef SCOPE_W8

// Shared-memory matrix descriptor: start address, leading / stride byte
// offsets (16-byte units), descriptor version 1 (sm_100), swizzle mode.
enum Swizzle : uint32_t { SW_NONE = 0, SW128 = 2, SW64 = 4, SW32 = 6 };
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t swz) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46) | ((uint64_t)swz << 61);
}
// K-major tile whose rows are `row_bytes` long (32, 64 or 128 = one swizzle
// span): 8-row core groups are 8*row_bytes apart.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t addr, uint32_t row_bytes) {
    uint32_t swz = row_bytes == 128 ? SW128 : (row_bytes == 64 ? SW64 : SW32);
    return smem_desc(addr, 16, 8 * row_bytes, swz);
}
// MN-major tile of 64 bf16 columns (128-byte rows along N), K rows: 8-row
// groups 1024 bytes apart.
__device__ __forceinline__ uint64_t mnmajor128_desc(uint32_t addr) { return smem_desc(addr, 16384, 1024, SW128); }
// MN-major tile of 16 bf16 columns (32-byte rows along N): 8-row groups 256 bytes apart.
__device__ __forceinline__ uint64_t mnmajor32_desc(uint32_t addr) { return smem_desc(addr, 4096, 256, SW32); }

// kind::f16 instruction descriptor: bf16 A and B, f32 accumulate, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float lg2(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// packed fp32x2 arithmetic (one instruction for two lanes of work on sm_100)
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// max of three (one instruction on sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// 2^x of a pair on the FMA pipe, to take load off the MUFU ex2.  Cody-Waite
// style reduction for base 2: x = n + f with n = round(x) (x + 1.5*2^23 puts n
// in the low mantissa bits; the subtractions are exact), 2^f by a degree-3
// polynomial whose coefficients minimise the relative error on [-1/2, 1/2]
// (Remez exchange, gen_exp2_poly.py: 7.5e-5 max relative error in float32),
// then n added to the exponent field.  x is clamped below at -125 so the
// exponent stays normal (-inf gives about 2^-125, not 0); x must be <= 127.
__device__ __forceinline__ uint64_t ex2_fma2(float x0, float x1) {
    constexpr float kMagic = 12582912.f, C0 = 0.9999280571937561f, C1 = 0.6932609677314758f,
                    C2 = 0.2426111251115799f, C3 = 0.0551716685295105f;
    const uint64_t d = f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
    const uint64_t t = fadd2(d, f2_pack(kMagic, kMagic));
    const uint64_t r = fadd2(t, f2_pack(-kMagic, -kMagic));
    const uint64_t f = ffma2(r, f2_pack(-1.f, -1.f), d);
    uint64_t q = ffma2(f2_pack(C3, C3), f, f2_pack(C2, C2));
    q = ffma2(q, f, f2_pack(C1, C1));
    q = ffma2(q, f, f2_pack(C0, C0));
    uint32_t t0, t1, q0, q1;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(t0), "=r"(t1) : "l"(t));
    asm("mov.b64 {%0, %1}, %2;" : "=r"(q0), "=r"(q1) : "l"(q));
    uint64_t out;
    asm("mov.b64 %0, {%1, %2};" : "=l"(out) : "r"(q0 + (t0 << 23)), "r"(q1 + (t1 << 23)));
    return out;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

}  // namespace tc
}  // namespace scope
