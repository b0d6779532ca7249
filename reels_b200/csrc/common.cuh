// Shared device helpers for the reels low-VRAM kernels (sm_100a only).
//
// Thin inline-PTX wrappers for mbarriers, TMA tile loads and the 5th-gen
// tensor core (tcgen05 / TMEM), plus the element-type helpers.  Every
// spin-wait in this library goes through `wait_bar`, which gives up after a
// bounded time, records an error code in a device word and lets the kernel
// unwind; nothing here traps.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace reels {

enum DType : int { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };

// Device-side status bits, OR-ed into the error word by a failing CTA.
enum DevErr : unsigned {
    DEVERR_TIMEOUT_AB_FULL = 1u,
    DEVERR_TIMEOUT_AB_EMPTY = 2u,
    DEVERR_TIMEOUT_W_FULL = 4u,
    DEVERR_TIMEOUT_W_EMPTY = 8u,
    DEVERR_TIMEOUT_ACC = 16u,
    DEVERR_NONFINITE_WEIGHT = 256u,
    DEVERR_OPT_TABLE = 512u,  // an optimizer workspace that was not prepared
    // a row whose max|w| / 127 underflows to 0 holds a zero: 0 / 0 is NaN
    DEVERR_QUANT_NAN = 1024u,
};

// ---------------------------------------------------------------- elements
template <int DT> struct Elem;
template <> struct Elem<DT_BF16> {
    using T = __nv_bfloat16;
    static __device__ __forceinline__ float to_f(T v) { return __bfloat162float(v); }
    static __device__ __forceinline__ T from_f(float v) { return __float2bfloat16_rn(v); }
    static __device__ __forceinline__ uint32_t pack2(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&h);
    }
};
template <> struct Elem<DT_F16> {
    using T = __half;
    static __device__ __forceinline__ float to_f(T v) { return __half2float(v); }
    static __device__ __forceinline__ T from_f(float v) { return __float2half_rn(v); }
    static __device__ __forceinline__ uint32_t pack2(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&h);
    }
};
template <> struct Elem<DT_F32> {
    using T = float;
    static __device__ __forceinline__ float to_f(T v) { return v; }
    static __device__ __forceinline__ T from_f(float v) { return v; }
};

__device__ __forceinline__ float load_act(const void *p, int64_t i, int dt) {
    if (dt == DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
    if (dt == DT_F16) return __half2float(reinterpret_cast<const __half *>(p)[i]);
    return reinterpret_cast<const float *>(p)[i];
}
// v rounded to the element type dt (kept in fp32 form).
__device__ __forceinline__ float round_dt(float v, int dt) {
    if (dt == DT_BF16) return __bfloat162float(__float2bfloat16_rn(v));
    if (dt == DT_F16) return __half2float(__float2half_rn(v));
    return v;
}
__device__ __forceinline__ void store_act(void *p, int64_t i, int dt, float v) {
    if (dt == DT_BF16) reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
    else if (dt == DT_F16) reinterpret_cast<__half *>(p)[i] = __float2half_rn(v);
    else reinterpret_cast<float *>(p)[i] = v;
}

// ------------------------------------------------------------------ PTX
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// try_wait with a suspend-time hint: a waiting thread is parked (it issues
// nothing) until the phase completes or the hint (ns) elapses, so pipeline
// waits do not steal issue slots from the warps doing the work.
#ifndef REELS_SUSPEND_HINT_NS
#define REELS_SUSPEND_HINT_NS 1000000u
#endif
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(REELS_SUSPEND_HINT_NS)
        : "memory");
    return ok != 0;
}

// Non-blocking check of a phase (no suspend): the cheap first probe of a wait.
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Upper bound on a single wait: about two seconds at the B200 boost clock.
// A pipeline stage normally completes in well under a microsecond.
#ifndef REELS_WAIT_LIMIT_CYCLES
#define REELS_WAIT_LIMIT_CYCLES 4000000000ll
#endif

// Bounded wait on an mbarrier phase.  `abort` is a CTA-shared flag: once any
// wait in the CTA has given up, every later wait returns at once so the
// CTA unwinds instead of serialising one timeout per stage.
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, volatile int *abort,
                                         unsigned *err, unsigned code) {
    if (mbar_test_wait(bar, parity)) return true;
    if (mbar_try_wait(bar, parity)) return true;
    long long t0 = clock64();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > REELS_WAIT_LIMIT_CYCLES) {
            *abort = 1;
            if (err) atomicOr(err, code);
            return false;
        }
    }
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Prefetch one 2-D tensor-map box into L2 (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_l2_2d(const void *tmap, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                     reinterpret_cast<uint64_t>(tmap)),
                 "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory (no multicast).
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const void *tmap, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// ------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16 or fp16 in, fp32 accum).
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on `bar` when every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit columns; thread t gets lane (base + t).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

// Shared-memory matrix descriptor for a 128-byte-swizzled canonical layout.
//  K-major : rows of 128 B (64 16-bit elements of K), 8-row groups SBO apart.
//  MN-major: 64 MN-elements contiguous (128 B) per K-row, 8-K-row groups SBO
//            apart, 64-element MN blocks LBO apart.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
    d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16 with fp32 accumulation.
// ab_type: 0 = fp16, 1 = bf16.  a_mn/b_mn: operand is MN-major.
__host__ __device__ constexpr uint32_t idesc_f16(int ab_type, int a_mn, int b_mn, int M, int N) {
    return (1u << 4) | (static_cast<uint32_t>(ab_type) << 7) | (static_cast<uint32_t>(ab_type) << 10) |
           (static_cast<uint32_t>(a_mn) << 15) | (static_cast<uint32_t>(b_mn) << 16) |
           (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Byte offset of 16-byte chunk `c` (0..7) of row `row` inside a 1024-byte
// aligned 128B-swizzled region whose rows are 128 B apart.
__device__ __forceinline__ uint32_t sw128_off(uint32_t row, uint32_t c) {
    return row * 128u + ((c ^ (row & 7u)) << 4);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ uint2 ld_shared_v2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization is queued early; griddep_wait() blocks until the previous
// kernel in the stream has completed and its memory is visible, so every such
// kernel calls it before its first global-memory access (read or write), on
// every path: a kernel whose CTAs could all exit without waiting would finish
// ahead of its predecessor and release the next kernel early, so the
// stream's order is transitive only if every kernel waits.  The kernels do
// not signal griddepcontrol.launch_dependents: with every kernel waiting an
// early trigger is correct, but it measured no faster.  Data written by an
// earlier kernel is read through L2 (__ldcg), not through the SM's L1 or the
// read-only path.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// 32-byte global stores (sm_100): one instruction per 16 bf16/fp16 or 8 fp32.
__device__ __forceinline__ void st_global_v8(void *p, uint4 a, uint4 b) {
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w),
                 "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
                 : "memory");
}

}  // namespace reels
