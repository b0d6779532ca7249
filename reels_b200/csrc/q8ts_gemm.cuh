// Persistent tcgen05 GEMM over an Int8 frozen weight with the dequantised
// weight held in tensor memory (sm_100a).
//
// Same product as q8_gemm.cuh,
//   D[M x Nout] = [act | ext_act] . [dequant(W) ; ext_w],
// computed transposed: the tensor core's A operand is a 128-row slice of the
// weight (128 output columns of D), written by the dequant warps straight
// into TMEM with tcgen05.st, and its B operand is the activation tile (BT
// tokens) that TMA leaves in shared memory.  The dequantised weight therefore
// never touches shared memory: per 64-wide reduction block the SM's shared
// memory sees the activation tile twice (TMA write, MMA read) and the int8
// tile twice (TMA write, ldmatrix read), about 60% of the traffic of the
// SMEM x SMEM kernel, whose 16-bit weight tile is written once and read by
// both 128-row MMAs.  The accumulator holds D^T (lanes = output columns,
// columns = tokens); the epilogue transposes through warp shuffles into
// row-major D.
//
// Dequant fragment (both weight orientations): thread t of a warp working on
// TMEM lane quarter q holds, for 16 reduction indices k0..k0+15, the four
// bytes k0 + 4(t%4) .. +3 of lanes 32q + 8i + t/4 (i = 0..3).  Weight tiles
// whose rows are output columns (64 reduction bytes per row, TMA 64B swizzle)
// are read with ldmatrix.m8n8.x4.b16; tiles whose rows are reduction indices
// (128 output-column bytes per row, TMA 128B swizzle) with
// ldmatrix.m16n16.x2.trans.b8, which transposes the bytes on the way.  Each
// byte quad becomes two bf16x2/f16x2 words, stored with tcgen05.st.16x256b
// (thread t -> lane t/4 and t/4 + 8, columns 2(t%4), 2(t%4)+1), the operand
// layout of a K-major TMEM A operand (lane = row, column c = elements 2c, 2c+1).
//
// Warp roles: 0 activation TMA, 1 MMA issue, 2 int8 (+ scale) TMA,
// 3..10 dequant (two groups of four, one warp per TMEM lane quarter; the
//          groups take alternate reduction blocks so two are in flight),
// 11..18 epilogue (two per lane quarter, half of the tile's tokens each),
// 19 (128-token tiles only) a second MMA issuer, used when each CTA runs one
//          work unit: the two issuers take alternate stages into the two
//          accumulators, which the epilogue adds.
//
// Rings: the activation ring is a ring of 64-wide atoms (released per atom on
// the double-buffered rings of single-CTA 128-wide stages), the int8 ring is
// shared by the two dequant groups (a group waits for the slot's previous use
// to be released before waiting for its load), and NA TMEM stages hold the
// dequantised weight.  PAIR = 1 runs each tile on a cluster of two CTAs
// (tcgen05.mma.cta_group::2): 256 weight rows per MMA, each CTA's 128 in its
// own TMEM, each CTA holding half of the token tile; see the pair helpers.
#pragma once
#include "act.cuh"
#include "q8_gemm.cuh"

namespace reels {

constexpr int TS_NDW = 8;  // dequant warps
constexpr int TS_NG = 2;   // dequant groups (one warp per TMEM lane quarter each), alternate reduction blocks
constexpr int TS_GW = TS_NDW / TS_NG;  // warps per group
constexpr int TS_NEW = 8;  // epilogue warps
constexpr int TS_THREADS = 32 * (3 + TS_NDW + TS_NEW);

// Debug builds only (-DREELS_TS_TRACE, never the shipped library): per CTA and
// warp, clock64 cycles spent in each wait and in the work between them,
// summed into g_ts_trace[cta][warp][4] (CTAs < 256).
#ifdef REELS_TS_TRACE
__device__ unsigned long long g_ts_trace[256 * (TS_THREADS / 32) * 4];
#define TSW(k, expr)                                   \
    ([&]() {                                           \
        const long long t0_ = clock64();               \
        const bool r_ = (expr);                        \
        tr_[k] += (unsigned long long)(clock64() - t0_); \
        return r_;                                     \
    }())
#define TS_MARK(v) const long long v = clock64()
#define TS_ADD(k, v) tr_[k] += (unsigned long long)(clock64() - (v))
#else
#define TSW(k, expr) (expr)
#define TS_MARK(v)
#define TS_ADD(k, v)
#endif

// A pipeline stage covers SK = 64*KB2 reduction elements, KB2 = 1 or 2 as the
// planner picks per shape: a 128-wide stage spreads the MMA warp's per-stage
// synchronisation over twice the tensor work and weight bytes.
// TMEM (512 columns): NACC accumulators of BT columns and NA A-operand stages
// of SK/2 columns.  BT = 256 leaves room for one accumulator only; BT <= 192
// double-buffers it so the epilogue overlaps the next tile's MMAs.
// PAIR = 1: the tile is shared by a CTA pair (see the pair helpers above);
// this CTA holds XT = BT/2 tokens of each activation atom.
template <int BT, int KB2, int PAIR = 0>
struct TsGeom {
    static constexpr int SK = 64 * KB2;
    static constexpr int NACC = BT == 256 ? 1 : 2;
    static constexpr int ACOLS = SK / 2;
    static constexpr int NA = (BT == 192 ? 4 : 8) / KB2;
    static constexpr int W_BYTES = 128 * SK;        // int8 tile: 128 output columns x SK
    static constexpr int SC_BYTES = 4 * SK;         // SK fp32 reduction scales
    static constexpr int EPI_BYTES = 4096;          // per epilogue warp: two 32 x 32 16-bit staging tiles
#ifndef REELS_TS_SX
#define REELS_TS_SX 0
#endif
#ifndef REELS_TS_S8
#define REELS_TS_S8 0
#endif
    static constexpr int XT = PAIR ? BT / 2 : BT;  // tokens of the activation tile in this CTA
    // A pair's half-height atoms leave room for a ring as deep as the TMEM stages.
    static constexpr int SX = PAIR ? NA
                                   : (REELS_TS_SX ? REELS_TS_SX
                                                  : (KB2 == 2 ? (BT == 128 ? 4 : 2) : (BT == 128 ? 6 : 4)));
    static constexpr int S8 = REELS_TS_S8 ? REELS_TS_S8 : (KB2 == 2 ? 3 : (BT == 256 ? 6 : 8));
    // The activation ring holds SXA slots of one 64-wide atom (BT x 64
    // elements) each; stage ga reads atoms ga*KB2 .. ga*KB2 + KB2 - 1, atom ax
    // in slot ax % SXA.
    static constexpr int XA_BYTES = XT * 128;
    static constexpr int SXA = SX * KB2;
    // Atom release: with 128-wide stages on a double-buffered ring, a slot is
    // handed back as soon as the MMAs that read its atom are done (x_empty),
    // not when the whole stage is, so the refill of one atom overlaps the
    // multiplication of the next.  With an even ring a stage's last atom
    // always sits in an odd slot and is released by the stage's kb_empty
    // commit, so only the first atom costs an extra commit.  Deep rings (the
    // 128-token tiles) and 64-wide stages release whole stages through kb_empty.
    static constexpr bool ATOM_REL = !PAIR && KB2 == 2 && BT != 128;
    static constexpr bool LAST_VIA_KB = ATOM_REL && (SXA % KB2 == 0);
    static constexpr int SXS = SXA / KB2;  // whole stages in the ring (when released by kb_empty)
    static_assert(ATOM_REL || SXA == SX * KB2, "stage-level release needs stage-aligned atom slots");
    static constexpr int NXE = ATOM_REL ? SXA : 0;  // x_empty barriers
    static constexpr int X_OFF = 0;
    static constexpr int W_OFF = X_OFF + SXA * XA_BYTES;
    static constexpr int SC_OFF = W_OFF + S8 * W_BYTES;
    static constexpr int EPI_OFF = (SC_OFF + S8 * SC_BYTES + 1023) / 1024 * 1024;
    static constexpr int BAR_OFF = EPI_OFF + TS_NEW * EPI_BYTES;
    // w_full, w_empty, kb_full, kb_empty, acc_full, acc_empty, mma_done, one
    // pre-activation load per epilogue warp, x_empty
    static constexpr int NBAR = 2 * S8 + 2 * NA + 2 * NACC + 1 + TS_NEW + NXE;
    static constexpr int MISC_OFF = BAR_OFF + NBAR * 8;
    static constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;
    static_assert(SMEM_BYTES <= 232448, "shared memory plan exceeds 227 KB");
    static_assert(NACC * BT + NA * ACOLS <= 512, "TMEM plan exceeds 512 columns");
    // Second MMA issuer (128-token tiles, TsArgs::iss2).  One thread issues an
    // N = 128 MMA every ~85 cycles against 64 of tensor work, and two threads
    // in different warps keep the pipe at its nominal rate.  The issuers take
    // alternate stages of a tile, each into its own accumulator (the two that
    // otherwise double-buffer tiles), and the epilogue adds the two.
    static constexpr bool ISS2 = BT == 128;
    static constexpr int ISS_WARP = TS_THREADS / 32;  // the extra warp
    static constexpr int THREADS = TS_THREADS + (ISS2 ? 32 : 0);
    static_assert(!ISS2 || NA % 2 == 0, "two issuers split the stage barrier ring by parity");
    // Stage ga uses barrier slot ga % NA: kb_full is completed by the
    // activation TMA and the dequant group, kb_empty (which frees the TMEM A
    // stage) by the MMA commit once the stage's MMAs are done.  The producer
    // arrives on kb_full[ga % NA] only after the slot of the stage's first
    // atom was released by its previous occupant, an atom of stage
    // ga - ceil(SXA / KB2) or later; with ceil(SXA / KB2) <= NA, stage
    // ga - NA's kb_full phase has then completed, so the arrival cannot land
    // in an older phase.
    static_assert((SXA + KB2 - 1) / KB2 <= NA, "activation ring deeper than the stage barrier ring");

    // Accumulator a starts at column 256 * a; A stages fill the columns left over.
    static __device__ __forceinline__ uint32_t acc_col(int a) { return 256u * a; }
    static __device__ __forceinline__ uint32_t a_col(int s) {
        if constexpr (NACC == 1) return 256u + (uint32_t)ACOLS * s;
        else return (s < NA / 2) ? (uint32_t)BT + ACOLS * s : 256u + BT + (uint32_t)ACOLS * (s - NA / 2);
    }
};

struct TsArgs {
    int M;             // rows of D (tokens)
    int Nout;          // columns of D
    int kb_total;      // main reduction blocks of 64
    int kb_per_split;
    int splits;
    int ntiles, mtiles;
    int w_rows_red;    // 1: int8 tile rows are reduction indices (transposed read)
    int scale_mode;    // 0 none, 1 per output column (dequant), 2 per reduction index (dequant)
    int wscale_len;
    const float *wscale;
    int r;             // LoRA rank (0: none)
    int ext_ld;        // row pitch (elements) of ext_w, which is [Nout][rp], rp = r rounded up to 32
    const void *ext_w;
    int epi_partial;
    const float *col_scale;  // per output column, applied in the epilogue
    const void *bias;
    void *out;
    long long ldo;
    int epi_act;       // EpiAct: gelu_tanh after the output, or its derivative (act.cuh)
    void *pre;         // the rounded pre-activation [M][Nout]: written (gelu), read (gradient); nullable for gelu
    float *partial;    // [splits][M][Nout]
    unsigned *err;
    int iss2;          // 128-token tiles: two MMA issuers (every unit has >= 2 stages)
};

__device__ __forceinline__ void ldsm_x4_b16(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// Four 8x8 16-bit matrices read transposed into mma-fragment registers (the
// inverse of stsm_x4_trans with the same addresses).
__device__ __forceinline__ void ldsm_x4_trans_b16(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_trans_b8(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m16n16.x2.trans.shared.b8 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// 16 lanes x 16 columns: thread t -> lanes t/4 (v[0..1], v[4..5]) and t/4 + 8
// (v[2..3], v[6..7]), columns 2(t%4), 2(t%4)+1 and 8 + the same.
__device__ __forceinline__ void tmem_st_16x256b_x2(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.16x256b.x2.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// TMA tile store from this CTA's shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const void *tmap, uint32_t smem_src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(tmap)),
                 "r"(x), "r"(y), "r"(smem_src)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 16 lanes x 32 columns: thread t gets lanes t/4 and t/4 + 8, columns
// 8g + 2(t%4) and 8g + 2(t%4) + 1 for g = 0..3 (r[4g .. 4g+3]).
__device__ __forceinline__ void tmem_ld_16x256b_x4(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
// Four 8x8 16-bit matrices from mma-fragment registers, each written
// transposed (fragment row -> shared-memory column); threads 8i..8i+7 give
// the row addresses of matrix i.
__device__ __forceinline__ void stsm_x4_trans(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b),
                 "r"(c), "r"(d)
                 : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns; thread t gets lane (base + t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// ------------------------------------------------------------ CTA pairs
// The pair variant (PAIR = 1) runs each tile on a cluster of two CTAs on
// neighbouring SMs with tcgen05.mma.cta_group::2: one MMA covers both CTAs'
// 128 weight rows (M = 256; each CTA's rows in its own TMEM) against the
// token tile, whose first half lives in the leader's shared memory and the
// second in the peer's.  Loads stay plain TMA loads into the issuing CTA's
// own shared memory (no multicast); the .cta_group::2 form only lets their
// completion count on the leader's barrier.  Commits go to both CTAs.
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
    return d;
}
// Arrive on a barrier of another CTA of the cluster.  The arrivals that use it
// follow tcgen05.wait::st + tcgen05.fence::before_thread_sync (the TMEM
// stores are complete) or tcgen05.ld completion, so the default CTA-scope
// release suffices; a cluster-scope release would also order every earlier
// global and shared write of the warp, and costs far more.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// try_wait that acquires at cluster scope (phases completed by the peer CTA).
__device__ __forceinline__ bool mbar_try_wait_cl(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(REELS_SUSPEND_HINT_NS)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool wait_bar_cl(uint64_t *bar, uint32_t parity, volatile int *abort, unsigned *err,
                                            unsigned code) {
    if (mbar_try_wait_cl(bar, parity)) return true;
    long long t0 = clock64();
    while (true) {
        if (mbar_try_wait_cl(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > REELS_WAIT_LIMIT_CYCLES) {
            *abort = 1;
            if (err) atomicOr(err, code);
            return false;
        }
    }
}
// Every thread of both CTAs.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc] over both CTAs of the pair, issued by the leader.
__device__ __forceinline__ void mma_f16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on `bar` in both CTAs of the pair when the pair MMAs issued so far are done.
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)0x3)
        : "memory");
}
// TMA load into this CTA's shared memory whose completion counts on the
// leader's mbarrier (`bar_leader`, a shared::cluster address from mapa).
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const void *tmap, int x, int y,
                                                 uint32_t bar_leader) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar_leader)
        : "memory");
}

// Bounded wait executed by every lane of a warp (the warp stays converged);
// the result is the same in all lanes.
__device__ __forceinline__ bool wait_bar_all(uint64_t *bar, uint32_t parity, volatile int *abort, unsigned *err,
                                             unsigned code) {
    const bool ok = wait_bar(bar, parity, abort, err, code);
    return __all_sync(0xffffffffu, ok);
}

// Four int8 (one 32-bit word, element 0 in the low byte) -> two 16-bit pairs.
template <int DT, int SMODE>
__device__ __forceinline__ void i8x4_convert(uint32_t v, const float *s, uint32_t &w0, uint32_t &w1) {
    if constexpr (SMODE == 0) {
        if constexpr (DT == DT_BF16) {
            w0 = bytes01_to_bf16x2(v, 0x4140u);
            w1 = bytes01_to_bf16x2(v, 0x4342u);
        } else {
            const uint32_t a = v ^ 0x80808080u;
            w0 = bytes01_to_f16x2(a, 0x4140u);
            w1 = bytes01_to_f16x2(a, 0x4342u);
        }
    } else {
        const uint32_t a = v ^ 0x80808080u;
        w0 = scaled_pair<DT>(a, 0, s[0], s[1]);
        w1 = scaled_pair<DT>(a, 2, s[2], s[3]);
    }
}

// fp16 with a scale: Float16(q) * Float16(s) rounded to fp16, the
// reference's own fp16 dequantisation (src/layers/quantization.jl:61-62):
// the exact int8 -> fp16 conversion, then one packed fp16 multiply by the
// scale pair (s01 = scales of elements 0, 1; s23 of elements 2, 3).
__device__ __forceinline__ void i8x4_f16_scaled(uint32_t v, uint32_t s01, uint32_t s23, uint32_t &w0,
                                                uint32_t &w1) {
    const uint32_t a = v ^ 0x80808080u;
    uint32_t q0 = bytes01_to_f16x2(a, 0x4140u), q1 = bytes01_to_f16x2(a, 0x4342u);
    __half2 p0 = __hmul2(*reinterpret_cast<__half2 *>(&q0), *reinterpret_cast<const __half2 *>(&s01));
    __half2 p1 = __hmul2(*reinterpret_cast<__half2 *>(&q1), *reinterpret_cast<const __half2 *>(&s23));
    w0 = *reinterpret_cast<uint32_t *>(&p0);
    w1 = *reinterpret_cast<uint32_t *>(&p1);
}
__device__ __forceinline__ uint32_t half2_bits(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

// 64 reduction indices (sub-block h2 of the stage) into TMEM columns 32*h2 .. 32*h2 + 31.
template <int DT, int ROWS_RED, int SMODE, int SK>
__device__ __forceinline__ void ts_dequant_sub(uint32_t w_base, uint32_t sc_base, uint32_t a_tm, int q, int lane,
                                               const float (&lane_s)[4], int h2) {
    uint32_t raw[4][4];
#pragma unroll
    for (int jl = 0; jl < 4; ++jl) {  // 16-wide reduction chunk j = 4*h2 + jl of the stage
        const uint32_t j = 4u * h2 + jl;
        if constexpr (ROWS_RED == 0) {
            // rows = output columns: thread t addresses row 32q + t, 16-byte chunk j
            const uint32_t row = 32u * q + lane;
            if constexpr (SK == 64) ldsm_x4_b16(w_base + row * 64u + ((j ^ ((row >> 1) & 3u)) << 4), raw[jl]);
            else ldsm_x4_b16(w_base + row * 128u + ((j ^ (row & 7u)) << 4), raw[jl]);
        } else {
            // rows = reduction indices (128 B): threads 0-15 chunk 2q, 16-31 chunk 2q+1
            const uint32_t row = 16u * j + (lane & 15);
            const uint32_t c = 2u * q + (lane >> 4);
            ldsm_x2_trans_b8(w_base + row * 128u + ((c ^ (row & 7u)) << 4), raw[jl]);
        }
    }
    // raw[j][i]: lanes 32q + 8i + t/4, reduction 16j + 4(t%4) .. +3
    // fp16 with a scale: the scales as fp16 pairs (per lane for SMODE 1)
    uint32_t ls2[4];
    if constexpr (DT == DT_F16 && SMODE == 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) ls2[i] = half2_bits(lane_s[i], lane_s[i]);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // reduction indices 32h .. 32h+31 = TMEM columns 16h .. 16h+15
        float rs[2][4];
        uint32_t rh[2][2];
        if constexpr (SMODE == 2) {
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                const float4 s4 = *reinterpret_cast<const float4 *>(
                    __cvta_shared_to_generic(sc_base + 4u * (64u * h2 + 16u * (2 * h + jj) + 4u * (lane & 3))));
                rs[jj][0] = s4.x;
                rs[jj][1] = s4.y;
                rs[jj][2] = s4.z;
                rs[jj][3] = s4.w;
                if constexpr (DT == DT_F16) {
                    rh[jj][0] = half2_bits(s4.x, s4.y);
                    rh[jj][1] = half2_bits(s4.z, s4.w);
                }
            }
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            uint32_t v[8];
#pragma unroll
            for (int jj = 0; jj < 2; ++jj)
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int i = 2 * half + u;
                    if constexpr (DT == DT_F16 && SMODE == 1) {
                        i8x4_f16_scaled(raw[2 * h + jj][i], ls2[i], ls2[i], v[4 * jj + 2 * u], v[4 * jj + 2 * u + 1]);
                    } else if constexpr (DT == DT_F16 && SMODE == 2) {
                        i8x4_f16_scaled(raw[2 * h + jj][i], rh[jj][0], rh[jj][1], v[4 * jj + 2 * u],
                                        v[4 * jj + 2 * u + 1]);
                    } else {
                        float sc[4];
                        if constexpr (SMODE == 1) sc[0] = sc[1] = sc[2] = sc[3] = lane_s[i];
                        if constexpr (SMODE == 2) {
                            sc[0] = rs[jj][0];
                            sc[1] = rs[jj][1];
                            sc[2] = rs[jj][2];
                            sc[3] = rs[jj][3];
                        }
                        i8x4_convert<DT, SMODE>(raw[2 * h + jj][i], sc, v[4 * jj + 2 * u], v[4 * jj + 2 * u + 1]);
                    }
                }
            tmem_st_16x256b_x2(a_tm + ((uint32_t)(32 * q + 16 * half) << 16) + 32u * h2 + 16u * h, v);
        }
    }
}


// One pipeline stage (SK reduction indices) of the weight into TMEM A stage
// `a_tm` (lane 0 address of the stage), 64 indices (sub-block h2) at a time.
// Warp q: lanes 32q..32q+31.  `lane_s` are the per-lane scales of SMODE 1
// (lanes 32q + 8i + t/4); SMODE 2 reads the stage's reduction scales from
// `sc_base`.  Tiles whose rows are output columns have SK-byte rows (64B
// swizzle for 64, 128B swizzle for 128); tiles whose rows are reduction
// indices have 128-byte rows (128B swizzle).
template <int DT, int ROWS_RED, int SMODE, int SK>
__device__ __forceinline__ void ts_dequant_block(uint32_t w_base, uint32_t sc_base, uint32_t a_tm, int q, int lane,
                                                 const float (&lane_s)[4]) {
#pragma unroll
    for (int h2 = 0; h2 < SK / 64; ++h2)
        ts_dequant_sub<DT, ROWS_RED, SMODE, SK>(w_base, sc_base, a_tm, q, lane, lane_s, h2);
}


struct TsTile {
    int n0, m0, sp, kb0, n_main, n_ext;
};

// Tiles run output-column tile fastest, so the CTAs in flight share one
// activation tile through L2 while the (small) weight stays resident there.
// With a CTA pair, a tile covers 256 output columns and `rank` picks this
// CTA's 128 (ntiles then counts 256-column tiles).
template <int BT, int SK, int PAIR = 0>
__device__ __forceinline__ TsTile ts_tile(const TsArgs &a, int t, uint32_t rank = 0) {
    TsTile c;
    const int nt = t % a.ntiles;
    const int rest = t / a.ntiles;
    const int mt = rest % a.mtiles;
    c.sp = rest / a.mtiles;
    c.n0 = PAIR ? nt * 256 + 128 * (int)rank : nt * 128;
    c.m0 = mt * BT;
    c.kb0 = c.sp * a.kb_per_split;
    c.n_main = max(0, min(a.kb_total, c.kb0 + a.kb_per_split) - c.kb0);
    c.n_ext = (c.sp == a.splits - 1 && a.r > 0) ? (a.r + SK - 1) / SK : 0;
    return c;
}

template <int DT, int BT, int KB2, int ACT, int PAIR = 0>
__global__ void __launch_bounds__(TsGeom<BT, KB2, PAIR>::THREADS, 1)
    q8ts_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmE, const __grid_constant__ CUtensorMap tmS,
                     const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmP,
                     const TsArgs args) {
    using G = TsGeom<BT, KB2, PAIR>;
    using E = Elem<DT>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    const uint32_t sbase = smem_u32(smem);

    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + G::BAR_OFF);
    uint64_t *w_full = bars;
    uint64_t *w_empty = w_full + G::S8;
    uint64_t *kb_full = w_empty + G::S8;
    uint64_t *kb_empty = kb_full + G::NA;
    uint64_t *acc_full = kb_empty + G::NA;
    uint64_t *acc_empty = acc_full + G::NACC;
    uint64_t *mma_done = acc_empty + G::NACC;
    uint64_t *pre_bar = mma_done + 1;
    uint64_t *x_empty = pre_bar + TS_NEW;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + G::MISC_OFF);
    volatile int *abort = reinterpret_cast<volatile int *>(smem + G::MISC_OFF + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int total_tiles = args.ntiles * args.mtiles * args.splits;
    // A pair walks the tiles together; the leader (rank 0) issues the MMAs and
    // owns the barriers both CTAs' producers complete.
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    const int t_first = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int t_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const bool two = G::ISS2 && args.iss2 != 0;  // two MMA issuers, one accumulator each

    if (threadIdx.x == 0) {
        for (int i = 0; i < G::S8; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], TS_GW);
        }
        for (int i = 0; i < G::NA; ++i) {
            // activation TMA (expect_tx) + one dequant group (of each CTA of a pair)
            mbar_init(&kb_full[i], 1 + (PAIR ? 2 : 1) * TS_GW);
            mbar_init(&kb_empty[i], 1);
        }
        for (int i = 0; i < G::NACC; ++i) {
            mbar_init(&acc_full[i], two ? 2 : 1);  // one commit per issuer
            mbar_init(&acc_empty[i], (PAIR ? 2 : 1) * TS_NEW);
        }
        mbar_init(mma_done, two ? 2 : 1);
        for (int i = 0; i < TS_NEW; ++i) mbar_init(&pre_bar[i], 1);
        for (int i = 0; i < G::NXE; ++i) mbar_init(&x_empty[i], 1);  // one MMA commit per use
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmW);
        if (args.r > 0) tma_prefetch_desc(&tmE);
        if (args.scale_mode == 2) tma_prefetch_desc(&tmS);
        if (!args.epi_partial) tma_prefetch_desc(&tmO);
        if (!args.epi_partial && args.epi_act != ACT_NONE && args.pre) tma_prefetch_desc(&tmP);
    }
    if (warp == 1) {
        if (PAIR) {
            tmem_alloc_pair(tmem_slot, 512);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, 512);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrival
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddep_wait();  // the previous kernel's outputs are complete from here on
    bool aborted_here = false;
    // arrive on the leader's copy of a barrier (local for the leader)
    auto arrive_leader = [&](uint64_t *bar) {
        if (!PAIR || leader) mbar_arrive(bar);
        else mbar_arrive_cluster(mapa_shared(smem_u32(bar), 0));
    };
    // MMA-side waits see the peer's arrivals at cluster scope
    auto wait_mma = [&](uint64_t *bar, uint32_t parity, unsigned code) {
        return PAIR ? wait_bar_cl(bar, parity, abort, args.err, code) : wait_bar(bar, parity, abort, args.err, code);
    };
    auto commit = [&](uint64_t *bar) {
        if (PAIR) mma_commit_pair(bar);
        else mma_commit(bar);
    };
#ifdef REELS_TS_TRACE
    unsigned long long tr_[4] = {0, 0, 0, 0};
    const long long tr_start = clock64();
#endif

    // Producer and MMA warps run converged; one lane issues the TMA copies,
    // MMAs and commits.
    if (warp == 0) {
        // ------------------------------------------------ activation producer
        // One lane runs the loop: no warp-wide votes or syncs per stage.
        if (lane == 0) {
            uint32_t gx = 0;
            for (int t = t_first; t < total_tiles && !aborted_here; t += t_step) {
                const TsTile c = ts_tile<BT, G::SK, PAIR>(args, t, rank);
                for (int it = 0; it < c.n_main + c.n_ext && !aborted_here; ++it, ++gx) {
                    uint64_t *full = &kb_full[gx % G::NA];
                    // main: KB2 K-major atoms of [BT tokens][64 K]; ext: rank atoms of
                    // [64 ranks][BT tokens], tokens contiguous (BT/64 boxes of 64 x 64),
                    // atoms wholly past r not loaded (the MMA does not read them)
                    const int e = it - c.n_main;
                    const int na = it < c.n_main ? KB2 : min(KB2, (args.r - G::SK * e + 63) / 64);
#pragma unroll
                    for (int a = 0; a < KB2; ++a) {
                        const uint32_t ax = gx * KB2 + a;
                        const int slot = ax % G::SXA;
                        // Wait for the slot's previous atom to be released; every slot is
                        // waited for and released once per use, loaded or not.
                        bool ok = true;
                        if (G::ATOM_REL && (a < KB2 - 1 || !G::LAST_VIA_KB)) {
                            if (ax >= (uint32_t)G::SXA)
                                ok = TSW(0, wait_bar(&x_empty[slot], ((ax / G::SXA) & 1) ^ 1, abort, args.err,
                                                     DEVERR_TIMEOUT_AB_EMPTY));
                        } else if (a == (G::ATOM_REL ? KB2 - 1 : 0) && gx >= (uint32_t)G::SXS) {
                            const uint32_t j = gx - G::SXS;  // the stage that last used these slots
                            ok = TSW(0, wait_bar(&kb_empty[j % G::NA], (j / G::NA) & 1, abort, args.err,
                                                 DEVERR_TIMEOUT_AB_EMPTY));
                        }
                        if (!ok) {
                            aborted_here = true;
                            break;
                        }
                        // the stage's bytes (both CTAs' halves for a pair) on the leader's barrier
                        if (a == 0 && (!PAIR || leader)) mbar_arrive_expect_tx(full, na * BT * 128);
                        if (a >= na) continue;
                        uint8_t *dst = smem + G::X_OFF + slot * G::XA_BYTES;
                        const int xm0 = c.m0 + (int)rank * G::XT;  // this CTA's tokens
                        auto load = [&](void *d, const CUtensorMap *m, int x, int y) {
                            if (PAIR) tma_load_2d_pair(d, m, x, y, mapa_shared(smem_u32(full), 0));
                            else tma_load_2d(d, m, x, y, full);
                        };
                        if (it < c.n_main) {
                            load(dst, &tmX, (c.kb0 + it) * G::SK + 64 * a, xm0);
                        } else {
#pragma unroll
                            for (int b = 0; b < G::XT / 64; ++b)
                                load(dst + b * 8192, &tmE, xm0 + 64 * b, G::SK * e + 64 * a);
                        }
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == 2) {
        // ------------------------------------------------ int8 weight (+ scale) producer
        if (lane == 0) {
            uint32_t gw = 0;
            const uint32_t bytes = G::W_BYTES + (args.scale_mode == 2 ? G::SC_BYTES : 0);
            for (int t = t_first; t < total_tiles && !aborted_here; t += t_step) {
                const TsTile c = ts_tile<BT, G::SK, PAIR>(args, t, rank);
                for (int it = 0; it < c.n_main; ++it, ++gw) {
                    const int s = gw % G::S8;
                    if (!TSW(0, wait_bar(&w_empty[s], ((gw / G::S8) & 1) ^ 1, abort, args.err,
                                         DEVERR_TIMEOUT_W_EMPTY))) {
                        aborted_here = true;
                        break;
                    }
                    uint8_t *dst = smem + G::W_OFF + s * G::W_BYTES;
                    mbar_arrive_expect_tx(&w_full[s], bytes);
                    const int kb = c.kb0 + it;
                    if (args.w_rows_red == 0) tma_load_2d(dst, &tmW, kb * G::SK, c.n0, &w_full[s]);
                    else tma_load_2d(dst, &tmW, c.n0, kb * G::SK, &w_full[s]);
                    if (args.scale_mode == 2)
                        tma_load_2d(smem + G::SC_OFF + s * G::SC_BYTES, &tmS, kb * G::SK, 0, &w_full[s]);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1 || (G::ISS2 && warp == G::ISS_WARP)) {
        // ------------------------------------------------ MMA issuer(s)
        // One lane runs the loop.  Each stage's MMAs are queued, then its
        // commit (releasing the stage once they complete), then the wait for
        // the next stage: the tensor pipe keeps the queued work while the
        // thread waits, and no warp-wide vote or sync sits between stages.
        // With two issuers, issuer `iss` takes the stages ga % 2 == iss into
        // accumulator iss; both wait for the tile's accumulators to be free and
        // both commit acc_full (count 2).  Splitting by the running stage count
        // (not by the stage's index in its tile) keeps each barrier slot
        // ga % NA (NA even) with one issuer, which waits its phases in order.
        const int iss = warp == 1 ? 0 : 1;
        if (lane == 0 && (!PAIR || leader) && (iss == 0 || two)) {
            const int ab = (DT == DT_BF16) ? 1 : 0;
            const uint32_t id_main = idesc_f16(ab, 0, 0, PAIR ? 256 : 128, BT);
            const uint32_t id_ext = idesc_f16(ab, 0, 1, PAIR ? 256 : 128, BT);
            auto mma = [&](uint32_t d, uint32_t a_t, uint64_t b, uint32_t id, uint32_t acc) {
                if (PAIR) mma_f16_ts_pair(d, a_t, b, id, acc);
                else mma_f16_ts(d, a_t, b, id, acc);
            };
            // Descriptors of X stage 0; a stage or K offset adds (bytes >> 4) to the address field.
            const uint64_t dmain0 = sdesc_sw128(sbase + G::X_OFF, 16, 1024);
            const uint64_t dext0 = sdesc_sw128(sbase + G::X_OFF, 8192, 1024);
            uint32_t ga = 0, local = 0;
            for (int t = t_first; t < total_tiles && !aborted_here; t += t_step, ++local) {
                const TsTile c = ts_tile<BT, G::SK, PAIR>(args, t, rank);
                const int acc = two ? 0 : (int)(local % G::NACC);  // barrier slot
                const uint32_t acc_par = two ? (local & 1) : ((local / G::NACC) & 1);
                if (!TSW(0, wait_mma(&acc_empty[acc], acc_par ^ 1, DEVERR_TIMEOUT_ACC))) {
                    aborted_here = true;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tm = tmem + G::acc_col(two ? iss : acc);
                const int n_iter = c.n_main + c.n_ext;
                bool fresh = true;  // this issuer's first stage of the tile overwrites its accumulator
                for (int it = 0; it < n_iter; ++it, ++ga) {
                    if (two && (int)(ga & 1) != iss) continue;
                    const int sa = ga % G::NA;
                    if (!TSW(1, wait_mma(&kb_full[sa], (ga / G::NA) & 1, DEVERR_TIMEOUT_AB_FULL))) {
                        aborted_here = true;
                        break;
                    }
                    tc_fence_after();
                    TS_MARK(tr_issue);
                    const uint32_t a_tm = tmem + G::a_col(sa);
                    // atom slot of K step kk: (ga * KB2 + kk / 4) % SXA; 32 bytes per step
                    // inside a K-major atom, 2048 inside a rank atom
                    auto xslot = [&](int a) { return (int)((ga * KB2 + a) % G::SXA); };
                    auto xoff = [&](int a) { return (uint64_t)((xslot(a) * G::XA_BYTES) >> 4); };
                    auto release = [&](int a) {
                        if (G::ATOM_REL && (a < KB2 - 1 || !G::LAST_VIA_KB)) mma_commit(&x_empty[xslot(a)]);
                    };
                    if (it < c.n_main) {
#pragma unroll
                        for (int kk = 0; kk < 4 * KB2; ++kk) {
                            mma(d_tm, a_tm + 8 * kk, dmain0 + xoff(kk >> 2) + (uint64_t)(((kk & 3) * 32) >> 4), id_main,
                                (!fresh || kk > 0) ? 1u : 0u);
                            if ((kk & 3) == 3) release(kk >> 2);  // this atom has been read
                        }
                    } else {
                        const int e = it - c.n_main;
                        const int nk = (min(G::SK, args.r - G::SK * e) + 15) / 16;
                        for (int kk = 0; kk < nk; ++kk)
                            mma(d_tm, a_tm + 8 * kk, dext0 + xoff(kk >> 2) + (uint64_t)(((kk & 3) * 2048) >> 4),
                                id_ext, (!fresh || kk > 0) ? 1u : 0u);
#pragma unroll
                        for (int a = 0; a < KB2; ++a) release(a);
                    }
                    commit(&kb_empty[sa]);
                    fresh = false;
                    TS_ADD(2, tr_issue);
                }
                if (aborted_here) break;
                commit(&acc_full[acc]);
            }
            commit(mma_done);
        }
        __syncwarp();
    } else if (warp < 3 + TS_NDW) {
        // ------------------------------------------------ dequant warps
        const int q = warp & 3;               // TMEM lane quarter
        const int g = (warp - 3) / TS_GW;     // group: reduction blocks with ga % TS_NG == g
        uint32_t ga = 0, gw = 0;
        for (int t = t_first; t < total_tiles && !aborted_here; t += t_step) {
            const TsTile c = ts_tile<BT, G::SK, PAIR>(args, t, rank);
            // Per-lane scales (lanes 32q + 8i + t/4) for SMODE 1.
            float lane_s[4] = {0.f, 0.f, 0.f, 0.f};
            if (args.scale_mode == 1) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int n = c.n0 + 32 * q + 8 * i + (lane >> 2);
                    lane_s[i] = n < args.wscale_len ? args.wscale[n] : 0.0f;
                }
            }
            const int n_iter = c.n_main + c.n_ext;
            for (int it = 0; it < n_iter; ++it, ++ga) {
                const bool main_blk = it < c.n_main;
                const uint32_t gw_this = gw;
                if (main_blk) ++gw;
                if ((int)(ga % TS_NG) != g) continue;
                const int sw = gw_this % G::S8;
                // The groups share the int8 ring, so the slot's previous use may
                // belong to the other group.  Waiting for that use to be released
                // first (w_empty) means w_full can only be in this use's phase:
                // otherwise, with the previous use's load still in flight, a
                // parity wait for this use would see that older phase's parity
                // and pass at once.
                if (main_blk && gw_this >= (uint32_t)G::S8 &&
                    !TSW(0, wait_bar_all(&w_empty[sw], ((gw_this / G::S8) & 1) ^ 1, abort, args.err,
                                         DEVERR_TIMEOUT_W_EMPTY))) {
                    aborted_here = true;
                    break;
                }
                if (main_blk &&
                    !TSW(0, wait_bar_all(&w_full[sw], (gw_this / G::S8) & 1, abort, args.err, DEVERR_TIMEOUT_W_FULL))) {
                    aborted_here = true;
                    break;
                }
                const int sa = ga % G::NA;
                if (!TSW(1, wait_bar_all(&kb_empty[sa], ((ga / G::NA) & 1) ^ 1, abort, args.err, DEVERR_TIMEOUT_AB_EMPTY))) {
                    aborted_here = true;
                    break;
                }
                tc_fence_after();
                TS_MARK(tr_work);
                const uint32_t a_tm = tmem + G::a_col(sa);
                if (main_blk) {
                    const uint32_t w_base = sbase + G::W_OFF + sw * G::W_BYTES;
                    const uint32_t sc_base = sbase + G::SC_OFF + sw * G::SC_BYTES;
                    switch (args.w_rows_red * 3 + args.scale_mode) {
                        case 0: ts_dequant_block<DT, 0, 0, G::SK>(w_base, sc_base, a_tm, q, lane, lane_s); break;
                        case 1: ts_dequant_block<DT, 0, 1, G::SK>(w_base, sc_base, a_tm, q, lane, lane_s); break;
                        case 2: ts_dequant_block<DT, 0, 2, G::SK>(w_base, sc_base, a_tm, q, lane, lane_s); break;
                        case 3: ts_dequant_block<DT, 1, 0, G::SK>(w_base, sc_base, a_tm, q, lane, lane_s); break;
                        case 4: ts_dequant_block<DT, 1, 1, G::SK>(w_base, sc_base, a_tm, q, lane, lane_s); break;
                        default: ts_dequant_block<DT, 1, 2, G::SK>(w_base, sc_base, a_tm, q, lane, lane_s); break;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&w_empty[sw]);
                } else {
                    // LoRA block: rows n0 + lane of the prepared [Nout][rp] operand,
                    // 16-bit pairs already in TMEM column order.
                    const int e = it - c.n_main;
                    const uint16_t *src = reinterpret_cast<const uint16_t *>(args.ext_w);
                    // 32 ranks per h; the MMAs read ceil(ranks / 16) K-steps of 8 columns
                    const int nh = min(2 * KB2, (min(G::SK, args.r - G::SK * e) + 31) / 32);
#pragma unroll
                    for (int h = 0; h < 2 * KB2; ++h)
                        if (h < nh)
#pragma unroll
                        for (int half = 0; half < 2; ++half) {
                            uint32_t v[8];
#pragma unroll
                            for (int jj = 0; jj < 2; ++jj)
#pragma unroll
                                for (int u = 0; u < 2; ++u) {
                                    const int n = c.n0 + 32 * q + 16 * half + 8 * u + (lane >> 2);
                                    const int k = G::SK * e + 16 * (2 * h + jj) + 4 * (lane & 3);
                                    uint2 w = make_uint2(0, 0);
                                    if (n < args.Nout)
                                        w = __ldcg(reinterpret_cast<const uint2 *>(src + (long long)n * args.ext_ld + k));
                                    v[4 * jj + 2 * u] = w.x;
                                    v[4 * jj + 2 * u + 1] = w.y;
                                }
                            tmem_st_16x256b_x2(a_tm + ((uint32_t)(32 * q + 16 * half) << 16) + 16u * h, v);
                        }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) arrive_leader(&kb_full[sa]);
                TS_ADD(2, tr_work);
            }
        }
    } else {
        // ------------------------------------------------ epilogue warps
        // 32 x 32 chunks of D^T (32 output columns of this warp's TMEM lane
        // quarter x 32 tokens).  Split partials: fp32 straight from a
        // thread-per-column load (a warp writes 128 contiguous bytes per
        // token).  Otherwise the 16x256b load gives mma fragments (rows =
        // columns of D, column pairs = tokens); after scale, bias and rounding
        // stmatrix.trans writes them token-major into a 64B-swizzled staging
        // tile that one TMA store copies to D.
        const int ew = warp - (3 + TS_NDW);
        const int q = warp & 3;
        const int set = ew >> 2;
        const uint32_t stage0 = sbase + G::EPI_OFF + ew * G::EPI_BYTES;
        int buf = 0;
        uint32_t pre_phase = 0;
        bool pre_pending = false;  // a pre-activation load is in flight
        uint32_t local = 0;
        // The activation is a compile-time variant: no branches in the
        // per-element code, and ACT_NONE carries none of its registers.
        constexpr int act = ACT;
        const bool store_pre = act == ACT_GELU_TANH && args.pre != nullptr;
        // Gradient: the pre-activation tile of a chunk is loaded (TMA, 32 x 32,
        // 64B swizzle) into the second staging tile while the chunk before it
        // is computed, once that chunk has read its own; chunk 0's load and an
        // L2 prefetch of the tile's other chunks are issued before the
        // accumulator wait, under the MMAs.
        auto load_pre = [&](const TsTile &c, int j0) {
            fence_proxy_async_smem();  // earlier ldmatrix reads of the tile come first
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_expect_tx(&pre_bar[ew], 2048);
                tma_load_2d(reinterpret_cast<void *>(smem + (stage0 + 2048 - sbase)), &tmP, c.n0 + 32 * q,
                            c.m0 + j0, &pre_bar[ew]);
            }
            pre_pending = true;
        };
        for (int t = t_first; t < total_tiles && !aborted_here; t += t_step, ++local) {
            const TsTile c = ts_tile<BT, G::SK, PAIR>(args, t, rank);
            const int acc = two ? 0 : (int)(local % G::NACC);
            if (act == ACT_GELU_TANH_GRAD && c.m0 + set * (BT / 2) < args.M) {
                if (lane == 0)
                    for (int ch = 1; ch < BT / 64; ++ch)
                        if (c.m0 + set * (BT / 2) + 32 * ch < args.M)
                            tma_prefetch_l2_2d(&tmP, c.n0 + 32 * q, c.m0 + set * (BT / 2) + 32 * ch);
                load_pre(c, set * (BT / 2));
            }
            if (!TSW(0, wait_bar_all(&acc_full[acc], two ? (local & 1) : ((local / G::NACC) & 1), abort, args.err,
                                     DEVERR_TIMEOUT_ACC))) {
                aborted_here = true;
                break;
            }
            tc_fence_after();
            const uint32_t t_base = tmem + ((uint32_t)(32 * q) << 16) + G::acc_col(acc);
            // two issuers: the second accumulator, added to the first in a fixed order
            const uint32_t t_base1 = tmem + ((uint32_t)(32 * q) << 16) + G::acc_col(1);
            constexpr int NCH = BT / 64;  // 32-column chunks per epilogue set
            if (args.epi_partial) {
                const int n = c.n0 + 32 * q + lane;
                const bool n_ok = n < args.Nout;
                for (int ch = 0; ch < NCH; ++ch) {
                    const int j0 = set * (BT / 2) + 32 * ch;
                    uint32_t v[32];
                    tmem_ld32(t_base + j0, v);
                    tmem_wait_ld();
                    if (G::ISS2 && two) {
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            uint32_t w[16];
                            tmem_ld16(t_base1 + j0 + 16 * h, w);
                            tmem_wait_ld();
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                v[16 * h + j] = __float_as_uint(__uint_as_float(v[16 * h + j]) + __uint_as_float(w[j]));
                        }
                    }
                    if (ch == NCH - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) arrive_leader(&acc_empty[acc]);
                    }
                    const int m_base = c.m0 + j0;
                    float *dst = args.partial + ((long long)c.sp * args.M + m_base) * args.Nout + n;
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (n_ok && m_base + j < args.M) dst[(long long)j * args.Nout] = __uint_as_float(v[j]);
                }
                continue;
            }
            // Column scale and bias of the four output columns this thread holds:
            // 32q + 16hh + 8k + t/4.
            float cs[2][2], bs[2][2];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                for (int k = 0; k < 2; ++k) {
                    const int n = c.n0 + 32 * q + 16 * hh + 8 * k + (lane >> 2);
                    cs[hh][k] = 1.0f;
                    bs[hh][k] = 0.0f;
                    if (n < args.Nout) {
                        if (args.col_scale) cs[hh][k] = args.col_scale[n];
                        if (args.bias) bs[hh][k] = E::to_f(reinterpret_cast<const typename E::T *>(args.bias)[n]);
                    }
                }
            for (int ch = 0; ch < NCH; ++ch) {
                const int j0 = set * (BT / 2) + 32 * ch;  // first token column of the chunk
                uint32_t r[2][16];
                tmem_ld_16x256b_x4(t_base + j0, r[0]);
                tmem_ld_16x256b_x4(t_base + (16u << 16) + j0, r[1]);
                tmem_wait_ld();
                if (G::ISS2 && two) {
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        uint32_t w[16];
                        tmem_ld_16x256b_x4(t_base1 + ((uint32_t)(16 * hh) << 16) + j0, w);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            r[hh][j] = __float_as_uint(__uint_as_float(r[hh][j]) + __uint_as_float(w[j]));
                    }
                }
                if (ch == NCH - 1) {
                    // all of this warp's accumulator columns are in registers
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) arrive_leader(&acc_empty[acc]);
                }
                const int m_base = c.m0 + j0;
                const bool rows_ok = m_base < args.M;  // rows past M are clipped by the TMA unit
                uint32_t st_tile, pre_tile;
                if (act == ACT_NONE) {
                    // The staging tile this chunk reuses was last read by the TMA
                    // store issued two chunks ago.
                    if (lane == 0) bulk_wait_group_read<1>();
                    __syncwarp();
                    st_tile = stage0 + buf * 2048;
                    pre_tile = st_tile;
                    buf ^= 1;
                } else {
                    // Both staging tiles serve this chunk: the output and the
                    // pre-activation (stored for gelu, loaded for its gradient).
                    if (lane == 0) bulk_wait_group_read<0>();
                    __syncwarp();
                    st_tile = stage0;
                    pre_tile = stage0 + 2048;
                }
                if (act == ACT_GELU_TANH_GRAD && rows_ok) {
                    if (!wait_bar_all(&pre_bar[ew], pre_phase & 1, abort, args.err, DEVERR_TIMEOUT_ACC)) {
                        aborted_here = true;
                        break;
                    }
                    ++pre_phase;
                    pre_pending = false;
                }
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    // matrix (column block nb = 2hh + k, token block g)
                    uint32_t pm[4], pp[4];
                    // thread 8i + j: row (token) 8g + j of matrix i, 16-byte chunk i (64B swizzle)
                    const uint32_t row = 8 * g + (lane & 7);
                    const uint32_t nb = lane >> 3;
                    const uint32_t off = row * 64 + ((nb ^ ((row >> 1) & 3)) << 4);
                    uint32_t hp[4];  // gradient: the rounded pre-activation, in the accumulator's fragment layout
                    if (act == ACT_GELU_TANH_GRAD) {
                        ldsm_x4_trans_b16(pre_tile + off, hp);
                        // the last read of this chunk's pre-activation tile: the next chunk's may load
                        if (g == 3 && rows_ok && ch + 1 < NCH && m_base + 32 < args.M) load_pre(c, j0 + 32);
                    }
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                        for (int k = 0; k < 2; ++k) {
                            const float v0 = fmaf(__uint_as_float(r[hh][4 * g + 2 * k]), cs[hh][k], bs[hh][k]);
                            const float v1 = fmaf(__uint_as_float(r[hh][4 * g + 2 * k + 1]), cs[hh][k], bs[hh][k]);
                            const int i = 2 * hh + k;
                            if (act == ACT_NONE) {
                                pm[i] = E::pack2(v0, v1);
                            } else if (act == ACT_GELU_TANH) {
                                const float h0 = round_act<DT>(v0), h1 = round_act<DT>(v1);
                                pp[i] = pack_rounded<DT>(h0, h1);
                                pm[i] = E::pack2(gelu_tanh_f32(h0), gelu_tanh_f32(h1));
                            } else {
                                float h0, h1;
                                unpack2<DT>(hp[i], h0, h1);
                                pm[i] = E::pack2(round_act<DT>(v0) * gelu_tanh_grad_f32(h0),
                                                 round_act<DT>(v1) * gelu_tanh_grad_f32(h1));
                            }
                        }
                    stsm_x4_trans(st_tile + off, pm[0], pm[1], pm[2], pm[3]);
                    if (store_pre) stsm_x4_trans(pre_tile + off, pp[0], pp[1], pp[2], pp[3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && rows_ok) {
                    tma_store_2d(&tmO, st_tile, c.n0 + 32 * q, m_base);
                    if (store_pre) tma_store_2d(&tmP, pre_tile, c.n0 + 32 * q, m_base);
                    bulk_commit_group();
                }
            }
            if (aborted_here) break;
        }
        // Stores must finish reading shared memory before the CTA exits, and an
        // abandoned pre-activation load must land (bounded wait).
        if (lane == 0) bulk_wait_group<0>();
        if (pre_pending) {
            const long long t0 = clock64();
            while (!mbar_try_wait(&pre_bar[ew], pre_phase & 1) && clock64() - t0 < REELS_WAIT_LIMIT_CYCLES) {
            }
        }
        __syncwarp();
    }

#ifdef REELS_TS_TRACE
    tr_[3] = (unsigned long long)(clock64() - tr_start);
    if (lane == 0 && blockIdx.x < 256 && warp < TS_THREADS / 32)
        for (int k = 0; k < 4; ++k) atomicAdd(&g_ts_trace[((size_t)blockIdx.x * (TS_THREADS / 32) + warp) * 4 + k], tr_[k]);
#endif
    if (aborted_here && (warp == 0 || warp == 2)) {
        for (int i = 0; i < 64; ++i) __nanosleep(2000);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        if (lane == 0) {
            long long t0 = clock64();
            while (!mbar_try_wait(mma_done, 0)) {
                if (clock64() - t0 > REELS_WAIT_LIMIT_CYCLES) {
                    atomicOr(args.err, DEVERR_TIMEOUT_ACC);
                    break;
                }
            }
        }
        __syncwarp();
    }
    // A pair's CTAs read each other's shared memory (the MMA) and barriers
    // (remote arrivals): neither leaves before both are done.
    if (PAIR) cluster_sync_all();
    if (warp == 1) {
        if (PAIR) tmem_dealloc_pair(tmem, 512);
        else tmem_dealloc(tmem, 512);
    }
}

}  // namespace reels
