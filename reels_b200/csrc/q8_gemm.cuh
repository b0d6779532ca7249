// Persistent tcgen05 GEMM over an Int8 frozen weight (sm_100a).
//
//   D[M x Nout] = [act | ext_act] . [dequant(W) ; ext_w]
//
// act is the 16-bit activation (x for the forward Y, dy for dX), W the int8
// weight with one fp32 scale per output row of the reference matrix, and the
// "ext" blocks append the rank-r LoRA term to the same accumulation:
//   forward (src/layers/quantization.jl:73-74 + lora.jl:86-94):
//       ext_act = A.x, ext_w = (alpha/r) B (divided by the column scale when
//       that scale is applied in the epilogue)
//   dX (quantization.jl:75-76 + lora.jl:115-116):
//       ext_act = (alpha/r) B'.dy, ext_w = A
//
// Pipeline per CTA (one CTA per SM, tiles handed out round-robin):
//   warp 0      TMA loads of activation tiles into the A ring
//   warp 2      TMA loads of int8 weight tiles into the W ring
//   warps 3-10  dequant: int8 tile -> bf16/fp16 in the 128B-swizzled K- or
//               MN-major layout tcgen05 reads, into the B ring (the LoRA
//               ext tile is copied from a prepared buffer instead)
//   warp 1      one thread issues tcgen05.mma into fp32 accumulators in TMEM
//   warps 11-18 epilogue: TMEM -> registers, column scale / bias, store
// The rings are decoupled, so the next tile's loads and dequant proceed while
// the epilogue drains the accumulator; with MT = 1 the accumulator is double
// buffered in TMEM and the MMA does not wait for the epilogue either.
#pragma once
#include "common.cuh"
#include "convert.cuh"
#include "sk_gemm.cuh"

namespace reels {

#ifndef REELS_Q8_DEQUANT_WARPS
#define REELS_Q8_DEQUANT_WARPS 8
#endif
constexpr int Q8_NCW = REELS_Q8_DEQUANT_WARPS;  // dequant warps (3 .. 2 + Q8_NCW)
constexpr int Q8_NDT = 32 * Q8_NCW;             // dequant threads
constexpr int Q8_NEW = 8;         // epilogue warps (11..18)
constexpr int Q8_THREADS = 32 * (3 + Q8_NCW + Q8_NEW);

struct Q8Args {
    int M;             // rows of D (tokens)
    int Nout;          // columns of D
    int kb_total;      // main reduction blocks of 64
    int kb_per_split;  // main blocks per split
    int splits;
    int ntiles, mtiles;
    int w_orient;      // 0: int8 staging rows are D columns  -> K-major B operand
                       // 1: int8 staging rows are reduction  -> MN-major B operand
    int scale_mode;    // 0 none, 1 per staging row, 2 per staging column
    int wscale_len;
    const float *wscale;
    // LoRA extension blocks
    int r;             // rank (0: none)
    int ext_kind;      // 0: ext_w is [rp][Nout] (MN-major);  1: ext_w is [Nout][rp] (K-major)
    int ext_ld;        // row pitch of ext_w in elements
    const void *ext_w; // prepared, rows/columns beyond r are zero
    // epilogue
    int epi_partial;
    const float *col_scale;
    const void *bias;
    void *out;
    long long ldo;
    int out_v8;        // out rows are 32-byte aligned: single 32-byte stores
    float *partial;    // [splits][M][Nout] (256-byte aligned)
    unsigned *err;
};

// Shared-memory plan per (MT, BN): A ring (activation tiles), B ring (16-bit
// weight tiles written by the dequant warps), W ring (int8 TMA staging),
// at most 224 KB.  For 2x256 a sweep on B200 put the third B stage ahead of
// a third A or fourth W stage (+10% forward): the MMA and the dequant warps
// run at similar rates, and two B stages made them wait on each other.  TMEM holds 512 fp32 columns: two accumulators of
// MT*BN columns when that is 256 (double buffered), one when it is 512.
template <int MT, int BN>
struct Q8Geom {
    static constexpr int ACC_COLS = MT * BN;
    static constexpr int NACC = 512 / ACC_COLS;
    static constexpr int A_BYTES = MT * 128 * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int W_BYTES = BN * BK;
    // Ring depths of the 2x256 plan; tuning builds may override them.
#ifndef REELS_Q8_SA
#define REELS_Q8_SA 2
#endif
#ifndef REELS_Q8_SB
#define REELS_Q8_SB 3
#endif
#ifndef REELS_Q8_S8
#define REELS_Q8_S8 3
#endif
    // 128-row tiles serve few tokens (M < 256): the int8 weight then streams
    // from HBM, so most of the budget goes to the W ring to keep ~128 KB of
    // weight in flight per SM (Little's law at ~2 us DRAM latency).
    static constexpr int SA = (MT == 2) ? (BN == 256 ? REELS_Q8_SA : 4) : 2;
    static constexpr int SB = (MT == 2) ? (BN == 256 ? REELS_Q8_SB : 3) : (BN == 256 ? 2 : 3);
    static constexpr int S8 = (MT == 2) ? (BN == 256 ? REELS_Q8_S8 : 6) : (BN == 256 ? 8 : 16);
    static constexpr int CPT = W_BYTES / 8 / Q8_NDT;  // 8-byte chunks per dequant thread
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = A_OFF + SA * A_BYTES;
    static constexpr int W_OFF = B_OFF + SB * B_BYTES;
    static constexpr int BAR_OFF = W_OFF + S8 * W_BYTES;
    // a_full, a_empty, b_full, b_empty, w_full, w_empty, acc_full, acc_empty, mma_done
    static constexpr int NBAR = 2 * SA + 2 * SB + 2 * S8 + 2 * NACC + 1;
    static constexpr int MISC_OFF = BAR_OFF + NBAR * 8;
    static constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;
    static constexpr int TMEM_COLS = 512;
    static_assert(SMEM_BYTES <= 232448, "shared memory plan exceeds 227 KB");
};

struct TileCoord {
    int n0, m0, sp, kb0, n_main, n_ext;
};

template <int MT, int BN>
__device__ __forceinline__ TileCoord q8_tile(const Q8Args &a, int t) {
    TileCoord c;
    const int nt = t % a.ntiles;
    const int rest = t / a.ntiles;
    const int mt = rest % a.mtiles;
    c.sp = rest / a.mtiles;
    c.n0 = nt * BN;
    c.m0 = mt * (MT * 128);
    c.kb0 = c.sp * a.kb_per_split;
    c.n_main = max(0, min(a.kb_total, c.kb0 + a.kb_per_split) - c.kb0);
    c.n_ext = (c.sp == a.splits - 1 && a.r > 0) ? (a.r + 63) / 64 : 0;
    return c;
}

// Epilogue for 16 consecutive accumulator columns of one row: fp32 partial
// sums (split reduction), or column scale + bias, rounding and a 32-byte store.
template <int DT>
__device__ __forceinline__ void epilogue_store16(const Q8Args &args, const uint32_t (&v)[16], int row, int col,
                                                 int sp) {
    using E = Elem<DT>;
    if (args.epi_partial) {
        float *dst = args.partial + ((long long)sp * args.M + row) * args.Nout + col;
        st_global_v8(dst, make_uint4(v[0], v[1], v[2], v[3]), make_uint4(v[4], v[5], v[6], v[7]));
        st_global_v8(dst + 8, make_uint4(v[8], v[9], v[10], v[11]), make_uint4(v[12], v[13], v[14], v[15]));
        return;
    }
    float f[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) f[u] = __uint_as_float(v[u]);
    if (args.col_scale) {
        const float4 *cs = reinterpret_cast<const float4 *>(args.col_scale + col);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float4 s4 = cs[u];
            f[4 * u] *= s4.x;
            f[4 * u + 1] *= s4.y;
            f[4 * u + 2] *= s4.z;
            f[4 * u + 3] *= s4.w;
        }
    }
    if (args.bias) {
        const typename E::T *bp = reinterpret_cast<const typename E::T *>(args.bias) + col;
#pragma unroll
        for (int u = 0; u < 16; ++u) f[u] += E::to_f(bp[u]);
    }
    uint4 o0, o1;
    o0.x = E::pack2(f[0], f[1]);
    o0.y = E::pack2(f[2], f[3]);
    o0.z = E::pack2(f[4], f[5]);
    o0.w = E::pack2(f[6], f[7]);
    o1.x = E::pack2(f[8], f[9]);
    o1.y = E::pack2(f[10], f[11]);
    o1.z = E::pack2(f[12], f[13]);
    o1.w = E::pack2(f[14], f[15]);
    typename E::T *dst = reinterpret_cast<typename E::T *>(args.out) + (long long)row * args.ldo + col;
    if (args.out_v8) {
        st_global_v8(dst, o0, o1);
    } else {
        reinterpret_cast<uint4 *>(dst)[0] = o0;
        reinterpret_cast<uint4 *>(dst)[1] = o1;
    }
}

// One int8 staging tile (BN x 64 bytes, row-major as TMA left it) to the
// 16-bit B-operand tile.  Each of the Q8_NDT dequant threads handles
// BN*8/Q8_NDT 8-byte chunks; their shared loads are issued back to back before any
// conversion so the latencies overlap.
//   ORIENT 0: staging rows are D columns, 64 B each   -> K-major B (SW128)
//   ORIENT 1: staging rows are reduction, BN B each   -> MN-major B (SW128,
//             64-column blocks 8 KB apart)
//   SMODE 0: exact int8 (scale applied elsewhere); 1: one fp32 scale per
//   staging row; 2: one fp32 scale per staging column.  The scale index is
//   the staging coordinate in the weight (row y0 + row, column x0 + col).
template <int DT, int BN, int ORIENT, int SMODE>
__device__ __forceinline__ void dequant_stage(uint32_t w_base, uint32_t b_base, int ct, int x0, int y0,
                                              const float *wscale, int wlen) {
    constexpr int CPT = BN * 8 / Q8_NDT;
    constexpr int BATCH = CPT < 4 ? CPT : 4;
    static_assert(CPT % BATCH == 0, "dequant chunks per thread must split into equal batches");
    constexpr int RC = (ORIENT == 0) ? 8 : BN / 8;  // chunks per staging row
    const int c8 = ct % RC;
    float cs[8];
    if constexpr (SMODE == 2) {
        const int gi = x0 + c8 * 8;
#pragma unroll
        for (int q = 0; q < 8; ++q) cs[q] = (gi + q) < wlen ? wscale[gi + q] : 0.0f;
    }
    // Batches of four chunks: four loads in flight, then convert and store.
#pragma unroll
    for (int jb = 0; jb < CPT; jb += BATCH) {
        uint2 v[BATCH];
        float rs[BATCH];
#pragma unroll
        for (int j = 0; j < BATCH; ++j) v[j] = ld_shared_v2(w_base + (ct + Q8_NDT * (jb + j)) * 8);
        if constexpr (SMODE == 1) {
#pragma unroll
            for (int j = 0; j < BATCH; ++j) {
                const int row = (ct + Q8_NDT * (jb + j)) / RC;
                rs[j] = (y0 + row) < wlen ? wscale[y0 + row] : 0.0f;
            }
        }
#pragma unroll
        for (int j = 0; j < BATCH; ++j) {
            const int row = (ct + Q8_NDT * (jb + j)) / RC;
            uint32_t dst;
            if constexpr (ORIENT == 0) dst = b_base + sw128_off(row, c8);
            else dst = b_base + (c8 >> 3) * 8192 + sw128_off(row, c8 & 7);
            uint4 o;
            if constexpr (SMODE == 0) o = i8x8_exact<DT>(v[j]);
            else if constexpr (SMODE == 1) o = i8x8_scaled1<DT>(v[j], rs[j]);
            else o = i8x8_scaled<DT>(v[j], cs);
            st_shared_v4(dst, o);
        }
    }
}

template <int DT, int MT, int BN>
__global__ void __launch_bounds__(Q8_THREADS, 1)
    q8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmE, const Q8Args args) {
    using G = Q8Geom<MT, BN>;
    using E = Elem<DT>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    const uint32_t sbase = smem_u32(smem);

    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + G::BAR_OFF);
    uint64_t *a_full = bars;
    uint64_t *a_empty = a_full + G::SA;
    uint64_t *b_full = a_empty + G::SA;
    uint64_t *b_empty = b_full + G::SB;
    uint64_t *w_full = b_empty + G::SB;
    uint64_t *w_empty = w_full + G::S8;
    uint64_t *acc_full = w_empty + G::S8;
    uint64_t *acc_empty = acc_full + G::NACC;
    uint64_t *mma_done = acc_empty + G::NACC;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + G::MISC_OFF);
    volatile int *abort = reinterpret_cast<volatile int *>(smem + G::MISC_OFF + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int total_tiles = args.ntiles * args.mtiles * args.splits;

    if (threadIdx.x == 0) {
        for (int i = 0; i < G::SA; ++i) {
            mbar_init(&a_full[i], 1);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < G::SB; ++i) {
            mbar_init(&b_full[i], Q8_NCW);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < G::S8; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], Q8_NCW);
        }
        for (int i = 0; i < G::NACC; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], Q8_NEW);
        }
        mbar_init(mma_done, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmW);
        if (args.r > 0) tma_prefetch_desc(&tmE);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, G::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddep_wait();  // the previous kernel's outputs are complete from here on
    bool aborted_here = false;

    if (warp == 0) {
        // ------------------------------------------------ activation producer
        if (lane == 0) {
            uint32_t ga = 0;
            for (int t = blockIdx.x; t < total_tiles && !aborted_here; t += gridDim.x) {
                const TileCoord c = q8_tile<MT, BN>(args, t);
                for (int it = 0; it < c.n_main + c.n_ext; ++it, ++ga) {
                    const int s = ga % G::SA;
                    if (!wait_bar(&a_empty[s], ((ga / G::SA) & 1) ^ 1, abort, args.err, DEVERR_TIMEOUT_AB_EMPTY)) {
                        aborted_here = true;
                        break;
                    }
                    uint8_t *dst = smem + G::A_OFF + s * G::A_BYTES;
                    mbar_arrive_expect_tx(&a_full[s], G::A_BYTES);
                    if (it < c.n_main) {
                        tma_load_2d(dst, &tmA, (c.kb0 + it) * BK, c.m0, &a_full[s]);
                    } else {
                        const int e = it - c.n_main;
#pragma unroll
                        for (int b = 0; b < 2 * MT; ++b)
                            tma_load_2d(dst + b * 8192, &tmE, c.m0 + 64 * b, 64 * e, &a_full[s]);
                    }
                }
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------ int8 weight producer
        if (lane == 0) {
            uint32_t gw = 0;
            for (int t = blockIdx.x; t < total_tiles && !aborted_here; t += gridDim.x) {
                const TileCoord c = q8_tile<MT, BN>(args, t);
                for (int it = 0; it < c.n_main; ++it, ++gw) {
                    const int s = gw % G::S8;
                    if (!wait_bar(&w_empty[s], ((gw / G::S8) & 1) ^ 1, abort, args.err, DEVERR_TIMEOUT_W_EMPTY)) {
                        aborted_here = true;
                        break;
                    }
                    uint8_t *dst = smem + G::W_OFF + s * G::W_BYTES;
                    mbar_arrive_expect_tx(&w_full[s], G::W_BYTES);
                    const int kb = c.kb0 + it;
                    if (args.w_orient == 0) tma_load_2d(dst, &tmW, kb * BK, c.n0, &w_full[s]);
                    else tma_load_2d(dst, &tmW, c.n0, kb * BK, &w_full[s]);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            const int ab = (DT == DT_BF16) ? 1 : 0;
            const uint32_t id_main = idesc_f16(ab, 0, args.w_orient == 1 ? 1 : 0, 128, BN);
            const uint32_t id_ext = idesc_f16(ab, 1, args.ext_kind == 0 ? 1 : 0, 128, BN);
            uint32_t ga = 0, gb = 0, local = 0;
            for (int t = blockIdx.x; t < total_tiles && !aborted_here; t += gridDim.x, ++local) {
                const TileCoord c = q8_tile<MT, BN>(args, t);
                const int acc = local % G::NACC;
                if (!wait_bar(&acc_empty[acc], ((local / G::NACC) & 1) ^ 1, abort, args.err, DEVERR_TIMEOUT_ACC)) {
                    aborted_here = true;
                    break;
                }
                tc_fence_after();
                const uint32_t d_base = tmem + acc * G::ACC_COLS;
                const int n_iter = c.n_main + c.n_ext;
                for (int it = 0; it < n_iter; ++it, ++ga, ++gb) {
                    const int sa = ga % G::SA, sb = gb % G::SB;
                    if (!wait_bar(&a_full[sa], (ga / G::SA) & 1, abort, args.err, DEVERR_TIMEOUT_AB_FULL) ||
                        !wait_bar(&b_full[sb], (gb / G::SB) & 1, abort, args.err, DEVERR_TIMEOUT_AB_FULL)) {
                        aborted_here = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_base = sbase + G::A_OFF + sa * G::A_BYTES;
                    const uint32_t b_base = sbase + G::B_OFF + sb * G::B_BYTES;
                    if (it < c.n_main) {
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                            for (int kk = 0; kk < BK / 16; ++kk) {
                                const uint64_t ad = sdesc_sw128(a_base + mt * 16384 + kk * 32, 16, 1024);
                                const uint64_t bd = (args.w_orient == 0)
                                                        ? sdesc_sw128(b_base + kk * 32, 16, 1024)
                                                        : sdesc_sw128(b_base + kk * 2048, 8192, 1024);
                                mma_f16_ss(d_base + mt * BN, ad, bd, id_main, (it > 0 || kk > 0) ? 1u : 0u);
                            }
                    } else {
                        const int e = it - c.n_main;
                        const int nk = (min(64, args.r - 64 * e) + 15) / 16;
                        for (int mt = 0; mt < MT; ++mt)
                            for (int kk = 0; kk < nk; ++kk) {
                                const uint64_t ad = sdesc_sw128(a_base + mt * 16384 + kk * 2048, 8192, 1024);
                                const uint64_t bd = (args.ext_kind == 0)
                                                        ? sdesc_sw128(b_base + kk * 2048, 8192, 1024)
                                                        : sdesc_sw128(b_base + kk * 32, 16, 1024);
                                mma_f16_ss(d_base + mt * BN, ad, bd, id_ext, (it > 0 || kk > 0) ? 1u : 0u);
                            }
                    }
                    mma_commit(&a_empty[sa]);
                    mma_commit(&b_empty[sb]);
                }
                if (aborted_here) break;
                mma_commit(&acc_full[acc]);
            }
            // Completes once every MMA issued above has finished, also after an
            // abort; the teardown waits on it before freeing tensor memory.
            mma_commit(mma_done);
        }
    } else if (warp < 3 + Q8_NCW) {
        // ------------------------------------------------ dequant warps
        const int ct = threadIdx.x - 3 * 32;  // 0 .. Q8_NDT-1
        uint32_t gb = 0, gw = 0;
        for (int t = blockIdx.x; t < total_tiles && !aborted_here; t += gridDim.x) {
            const TileCoord c = q8_tile<MT, BN>(args, t);
            const int n_iter = c.n_main + c.n_ext;
            for (int it = 0; it < n_iter; ++it, ++gb) {
                const bool main_blk = it < c.n_main;
                const int sw = gw % G::S8;
                if (main_blk &&
                    !warp_wait(&w_full[sw], (gw / G::S8) & 1, abort, args.err, DEVERR_TIMEOUT_W_FULL)) {
                    aborted_here = true;
                    break;
                }
                const int sb = gb % G::SB;
                if (!warp_wait(&b_empty[sb], ((gb / G::SB) & 1) ^ 1, abort, args.err, DEVERR_TIMEOUT_AB_EMPTY)) {
                    aborted_here = true;
                    break;
                }
                const uint32_t b_base = sbase + G::B_OFF + sb * G::B_BYTES;
                if (main_blk) {
                    const uint32_t w_base = sbase + G::W_OFF + sw * G::W_BYTES;
                    const int kb = c.kb0 + it;
                    // TMA coordinates of the staging tile: x = column origin, y = row origin.
                    const int x0 = (args.w_orient == 0) ? kb * BK : c.n0;
                    const int y0 = (args.w_orient == 0) ? c.n0 : kb * BK;
                    switch (args.w_orient * 3 + args.scale_mode) {
                        case 0: dequant_stage<DT, BN, 0, 0>(w_base, b_base, ct, x0, y0, args.wscale, args.wscale_len); break;
                        case 1: dequant_stage<DT, BN, 0, 1>(w_base, b_base, ct, x0, y0, args.wscale, args.wscale_len); break;
                        case 2: dequant_stage<DT, BN, 0, 2>(w_base, b_base, ct, x0, y0, args.wscale, args.wscale_len); break;
                        case 3: dequant_stage<DT, BN, 1, 0>(w_base, b_base, ct, x0, y0, args.wscale, args.wscale_len); break;
                        case 4: dequant_stage<DT, BN, 1, 1>(w_base, b_base, ct, x0, y0, args.wscale, args.wscale_len); break;
                        default: dequant_stage<DT, BN, 1, 2>(w_base, b_base, ct, x0, y0, args.wscale, args.wscale_len); break;
                    }
                } else {
                    // LoRA ext tile: a straight copy of the prepared operand.
                    const int e = it - c.n_main;
                    const typename E::T *src = reinterpret_cast<const typename E::T *>(args.ext_w);
#pragma unroll
                    for (int j = 0; j < G::CPT; ++j) {
                        const int i = ct + Q8_NDT * j;
                        uint4 o = make_uint4(0, 0, 0, 0);
                        uint32_t dst;
                        if (args.ext_kind == 0) {
                            const int jr = i / (BN / 8), cc = i % (BN / 8);
                            const int n = c.n0 + cc * 8;
                            dst = b_base + (cc >> 3) * 8192 + sw128_off(jr, cc & 7);
                            if (n < args.Nout)
                                o = __ldcg(reinterpret_cast<const uint4 *>(src + (long long)(64 * e + jr) * args.ext_ld + n));
                        } else {
                            const int row = i >> 3, cc = i & 7;
                            const int k = c.n0 + row;
                            dst = b_base + sw128_off(row, cc);
                            if (k < args.Nout)
                                o = __ldcg(reinterpret_cast<const uint4 *>(src + (long long)k * args.ext_ld + 64 * e + cc * 8));
                        }
                        st_shared_v4(dst, o);
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if (main_blk) mbar_arrive(&w_empty[sw]);
                    mbar_arrive(&b_full[sb]);
                }
                if (main_blk) ++gw;
            }
        }
    } else {
        // ------------------------------------------------ epilogue warps
        const int ew = warp - (3 + Q8_NCW);  // 0..7 (epilogue warp index)
        const int q = warp & 3;              // TMEM lane quarter this warp may read
        const int set = ew >> 2;             // 0 or 1
        uint32_t local = 0;
        for (int t = blockIdx.x; t < total_tiles && !aborted_here; t += gridDim.x, ++local) {
            const TileCoord c = q8_tile<MT, BN>(args, t);
            const int acc = local % G::NACC;
            if (!warp_wait(&acc_full[acc], (local / G::NACC) & 1, abort, args.err, DEVERR_TIMEOUT_ACC)) {
                aborted_here = true;
                break;
            }
            tc_fence_after();
            int mt, c_begin, c_end;
            if (MT == 2) {
                mt = set;
                c_begin = 0;
                c_end = BN;
            } else {
                mt = 0;
                c_begin = set * (BN / 2);
                c_end = c_begin + BN / 2;
            }
            const int row = c.m0 + mt * 128 + 32 * q + lane;
            const uint32_t t_base = tmem + ((uint32_t)(32 * q) << 16) + acc * G::ACC_COLS + mt * BN;
            for (int cb = c_begin; cb < c_end; cb += 32) {
                // Two TMEM loads in flight per wait.
                uint32_t v[2][16];
                tmem_ld16(t_base + cb, v[0]);
                tmem_ld16(t_base + cb + 16, v[1]);
                tmem_wait_ld();
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int col = c.n0 + cb + 16 * h;
                    if (row < args.M && col < args.Nout)
                        epilogue_store16<DT>(args, v[h], row, col, c.sp);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
    }

    if (aborted_here && (warp == 0 || warp == 2)) {
        // Give TMA copies already issued time to land before the CTA exits.
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
        tmem_dealloc(tmem, G::TMEM_COLS);
    }
}

}  // namespace reels
