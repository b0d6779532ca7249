// Pair-CTA (cta_group::2) variant of the Int8-weight LoRA GEMM (sm_100a).
//
// Same product as q8_gemm_kernel (see q8_gemm.cuh) on 256 x 256 tiles, but
// each tile is shared by a cluster of two CTAs on neighbouring SMs:
//   - CTA r of the pair holds tokens m0 + 128 r .. +127 of the activation
//     tile and output columns n0 + 128 r .. +127 of the weight tile, so each
//     SM dequantises only half of the weight tile;
//   - the leader (rank 0) issues tcgen05.mma.cta_group::2 (M = 256, N = 256)
//     which reads both CTAs' shared memory and writes 128 accumulator rows
//     into each CTA's tensor memory;
//   - each CTA's accumulator is 256 columns, so two fit in TMEM and the
//     epilogue of one tile overlaps the MMAs of the next.
// Compared with one CTA on a 256 x 256 tile this halves the shared-memory
// reads of the weight operand and the dequant work per SM, and hides the
// epilogue.  Measured on B200 it nevertheless reaches only about 770 TFLOP/s
// (forward, bf16) against 920-1130 for the single-CTA kernel, independent of
// ring depths: the library therefore runs it only when REELS_Q8_TILE=pair
// asks for it.
//
// Synchronisation: the "full" side of every pipeline lives in the leader.
// Both CTAs' TMA loads complete on the leader's a_full barrier (the
// cta_group::2 form of the TMA load), both CTAs' dequant warps arrive on the
// leader's b_full and both epilogues on the leader's acc_empty (remote
// arrivals at cluster scope), so the MMA thread waits on local barriers only.
// Its commits arrive on both CTAs' "empty" / acc_full barriers at once
// (tcgen05.commit with a CTA mask), releasing each CTA's own stages.  No TMA
// load uses multicast: every CTA loads only its own data into its own shared
// memory.
#pragma once
#include "q8_gemm.cuh"

namespace reels {

#ifndef REELS_PAIR_S
#define REELS_PAIR_S 5
#endif
#ifndef REELS_PAIR_S8
#define REELS_PAIR_S8 8
#endif
struct Q8PairGeom {
    static constexpr int S = REELS_PAIR_S;    // A and B stages (one index for both)
    static constexpr int S8 = REELS_PAIR_S8;  // int8 staging stages
    static constexpr int NACC = 2;    // double-buffered accumulators
    static constexpr int HALF = 128;  // tokens / weight columns per CTA
    static constexpr int A_BYTES = HALF * 128;
    static constexpr int B_BYTES = HALF * 128;
    static constexpr int W_BYTES = HALF * BK;
    static constexpr int CPT = W_BYTES / 8 / Q8_NDT;
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = A_OFF + S * A_BYTES;
    static constexpr int W_OFF = B_OFF + S * B_BYTES;
    static constexpr int BAR_OFF = W_OFF + S8 * W_BYTES;
    // a_full, a_empty, b_full, b_empty (S each), w_full, w_empty, acc_full,
    // acc_empty, mma_done
    static constexpr int NBAR = 4 * S + 2 * S8 + 2 * NACC + 1;
    static constexpr int MISC_OFF = BAR_OFF + NBAR * 8;
    static constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;
    static constexpr int ACC_COLS = 256;
    static constexpr int TMEM_COLS = 512;
    static_assert(SMEM_BYTES <= 232448, "shared memory plan exceeds 227 KB");
};

template <int DT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Q8_THREADS, 1)
    q8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                        const __grid_constant__ CUtensorMap tmE, const Q8Args args) {
    using G = Q8PairGeom;
    using E = Elem<DT>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    const uint32_t sbase = smem_u32(smem);

    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + G::BAR_OFF);
    uint64_t *a_full = bars;
    uint64_t *a_empty = a_full + G::S;
    uint64_t *b_full = a_empty + G::S;
    uint64_t *b_empty = b_full + G::S;
    uint64_t *w_full = b_empty + G::S;
    uint64_t *w_empty = w_full + G::S8;
    uint64_t *acc_full = w_empty + G::S8;
    uint64_t *acc_empty = acc_full + G::NACC;
    uint64_t *mma_done = acc_empty + G::NACC;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + G::MISC_OFF);
    volatile int *abort = reinterpret_cast<volatile int *>(smem + G::MISC_OFF + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();  // 0 = leader
    const int pair_id = blockIdx.x >> 1;
    const int npairs = gridDim.x >> 1;
    const int total_tiles = args.ntiles * args.mtiles * args.splits;

    if (threadIdx.x == 0) {
        // Leader-side counts cover both CTAs (the peer's copies are unused).
        for (int i = 0; i < G::S; ++i) {
            mbar_init(&a_full[i], 1);
            mbar_init(&a_empty[i], 1);
            mbar_init(&b_full[i], 2 * Q8_NCW);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < G::S8; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], Q8_NCW);
        }
        for (int i = 0; i < G::NACC; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 2 * Q8_NEW);
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
        tmem_alloc_pair(tmem_slot, G::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    // Both CTAs' barriers must be initialised before any remote arrival.
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool aborted_here = false;

    if (warp == 0) {
        // ------------------------------------------------ activation producer (own 128 tokens)
        if (lane == 0) {
            uint32_t ga = 0;
            for (int t = pair_id; t < total_tiles && !aborted_here; t += npairs) {
                const TileCoord c = q8_tile<2, 256>(args, t);
                const int mrow = c.m0 + G::HALF * rank;
                for (int it = 0; it < c.n_main + c.n_ext; ++it, ++ga) {
                    const int s = ga % G::S;
                    if (!wait_bar(&a_empty[s], ((ga / G::S) & 1) ^ 1, abort, args.err, DEVERR_TIMEOUT_AB_EMPTY)) {
                        aborted_here = true;
                        break;
                    }
                    uint8_t *dst = smem + G::A_OFF + s * G::A_BYTES;
                    const uint32_t fb = mapa_shared(smem_u32(&a_full[s]), 0);
                    if (rank == 0) mbar_arrive_expect_tx(&a_full[s], 2 * G::A_BYTES);
                    if (it < c.n_main) {
                        tma_load_2d_pair(dst, &tmA, (c.kb0 + it) * BK, mrow, fb);
                    } else {
                        const int e = it - c.n_main;
                        tma_load_2d_pair(dst, &tmE, mrow, 64 * e, fb);
                        tma_load_2d_pair(dst + 8192, &tmE, mrow + 64, 64 * e, fb);
                    }
                }
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------ int8 weight producer (own 128 columns)
        if (lane == 0) {
            uint32_t gw = 0;
            for (int t = pair_id; t < total_tiles && !aborted_here; t += npairs) {
                const TileCoord c = q8_tile<2, 256>(args, t);
                const int ncol = c.n0 + G::HALF * rank;
                for (int it = 0; it < c.n_main; ++it, ++gw) {
                    const int s = gw % G::S8;
                    if (!wait_bar(&w_empty[s], ((gw / G::S8) & 1) ^ 1, abort, args.err, DEVERR_TIMEOUT_W_EMPTY)) {
                        aborted_here = true;
                        break;
                    }
                    uint8_t *dst = smem + G::W_OFF + s * G::W_BYTES;
                    mbar_arrive_expect_tx(&w_full[s], G::W_BYTES);
                    const int kb = c.kb0 + it;
                    if (args.w_orient == 0) tma_load_2d(dst, &tmW, kb * BK, ncol, &w_full[s]);
                    else tma_load_2d(dst, &tmW, ncol, kb * BK, &w_full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // -------------------------------------------- MMA issuer (leader)
            const int ab = (DT == DT_BF16) ? 1 : 0;
            const uint32_t id_main = idesc_f16(ab, 0, args.w_orient == 1 ? 1 : 0, 256, 256);
            const uint32_t id_ext = idesc_f16(ab, 1, args.ext_kind == 0 ? 1 : 0, 256, 256);
            uint32_t g = 0, local = 0;
            for (int t = pair_id; t < total_tiles && !aborted_here; t += npairs, ++local) {
                const TileCoord c = q8_tile<2, 256>(args, t);
                const int acc = local % G::NACC;
                const uint32_t pe = ((local / G::NACC) & 1) ^ 1;
                if (!wait_bar(&acc_empty[acc], pe, abort, args.err, DEVERR_TIMEOUT_ACC)) {
                    aborted_here = true;
                    break;
                }
                tc_fence_after();
                const uint32_t d_base = tmem + acc * G::ACC_COLS;
                const int n_iter = c.n_main + c.n_ext;
                for (int it = 0; it < n_iter; ++it, ++g) {
                    const int s = g % G::S;
                    const uint32_t ph = (g / G::S) & 1;
                    if (!wait_bar(&a_full[s], ph, abort, args.err, DEVERR_TIMEOUT_AB_FULL) ||
                        !wait_bar(&b_full[s], ph, abort, args.err, DEVERR_TIMEOUT_AB_FULL)) {
                        aborted_here = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_base = sbase + G::A_OFF + s * G::A_BYTES;
                    const uint32_t b_base = sbase + G::B_OFF + s * G::B_BYTES;
                    if (it < c.n_main) {
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            const uint64_t ad = sdesc_sw128(a_base + kk * 32, 16, 1024);
                            const uint64_t bd = (args.w_orient == 0) ? sdesc_sw128(b_base + kk * 32, 16, 1024)
                                                                     : sdesc_sw128(b_base + kk * 2048, 8192, 1024);
                            mma_f16_ss_pair(d_base, ad, bd, id_main, (it > 0 || kk > 0) ? 1u : 0u);
                        }
                    } else {
                        const int e = it - c.n_main;
                        const int nk = (min(64, args.r - 64 * e) + 15) / 16;
                        for (int kk = 0; kk < nk; ++kk) {
                            const uint64_t ad = sdesc_sw128(a_base + kk * 2048, 8192, 1024);
                            const uint64_t bd = (args.ext_kind == 0) ? sdesc_sw128(b_base + kk * 2048, 8192, 1024)
                                                                     : sdesc_sw128(b_base + kk * 32, 16, 1024);
                            mma_f16_ss_pair(d_base, ad, bd, id_ext, (it > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                    mma_commit_pair(&a_empty[s], 0x3);
                    mma_commit_pair(&b_empty[s], 0x3);
                }
                if (aborted_here) break;
                mma_commit_pair(&acc_full[acc], 0x3);
            }
            mma_commit_pair(mma_done, 0x1);
        }
    } else if (warp < 3 + Q8_NCW) {
        // ------------------------------------------------ dequant warps (own 128 weight columns)
        const int ct = threadIdx.x - 3 * 32;
        uint32_t g = 0, gw = 0;
        for (int t = pair_id; t < total_tiles && !aborted_here; t += npairs) {
            const TileCoord c = q8_tile<2, 256>(args, t);
            const int ncol = c.n0 + G::HALF * rank;
            const int n_iter = c.n_main + c.n_ext;
            for (int it = 0; it < n_iter; ++it, ++g) {
                const bool main_blk = it < c.n_main;
                const int sw = gw % G::S8;
                if (main_blk &&
                    !warp_wait(&w_full[sw], (gw / G::S8) & 1, abort, args.err, DEVERR_TIMEOUT_W_FULL)) {
                    aborted_here = true;
                    break;
                }
                const int s = g % G::S;
                if (!warp_wait(&b_empty[s], ((g / G::S) & 1) ^ 1, abort, args.err, DEVERR_TIMEOUT_AB_EMPTY)) {
                    aborted_here = true;
                    break;
                }
                const uint32_t b_base = sbase + G::B_OFF + s * G::B_BYTES;
                if (main_blk) {
                    const uint32_t w_base = sbase + G::W_OFF + sw * G::W_BYTES;
                    const int kb = c.kb0 + it;
                    const int x0 = (args.w_orient == 0) ? kb * BK : ncol;
                    const int y0 = (args.w_orient == 0) ? ncol : kb * BK;
                    switch (args.w_orient * 3 + args.scale_mode) {
                        case 0: dequant_stage<DT, 128, 0, 0>(w_base, b_base, ct, x0, y0, args.wscale, args.wscale_len); break;
                        case 1: dequant_stage<DT, 128, 0, 1>(w_base, b_base, ct, x0, y0, args.wscale, args.wscale_len); break;
                        case 2: dequant_stage<DT, 128, 0, 2>(w_base, b_base, ct, x0, y0, args.wscale, args.wscale_len); break;
                        case 3: dequant_stage<DT, 128, 1, 0>(w_base, b_base, ct, x0, y0, args.wscale, args.wscale_len); break;
                        case 4: dequant_stage<DT, 128, 1, 1>(w_base, b_base, ct, x0, y0, args.wscale, args.wscale_len); break;
                        default: dequant_stage<DT, 128, 1, 2>(w_base, b_base, ct, x0, y0, args.wscale, args.wscale_len); break;
                    }
                } else {
                    // LoRA ext tile: copy of the prepared operand, own half.
                    const int e = it - c.n_main;
                    const typename E::T *src = reinterpret_cast<const typename E::T *>(args.ext_w);
#pragma unroll
                    for (int j = 0; j < G::CPT; ++j) {
                        const int i = ct + Q8_NDT * j;
                        uint4 o = make_uint4(0, 0, 0, 0);
                        uint32_t dst;
                        if (args.ext_kind == 0) {
                            const int jr = i / 16, cc = i % 16;
                            const int n = ncol + cc * 8;
                            dst = b_base + (cc >> 3) * 8192 + sw128_off(jr, cc & 7);
                            if (n < args.Nout)
                                o = __ldcg(reinterpret_cast<const uint4 *>(src + (long long)(64 * e + jr) * args.ext_ld + n));
                        } else {
                            const int row = i >> 3, cc = i & 7;
                            const int k = ncol + row;
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
                    if (rank == 0) mbar_arrive(&b_full[s]);
                    else mbar_arrive_remote(mapa_shared(smem_u32(&b_full[s]), 0));
                }
                if (main_blk) ++gw;
            }
        }
    } else {
        // ------------------------------------------------ epilogue warps (own 128 rows)
        const int ew = warp - (3 + Q8_NCW);
        const int q = warp & 3;
        const int set = ew >> 2;  // column half of the 256-wide accumulator
        uint32_t local = 0;
        for (int t = pair_id; t < total_tiles && !aborted_here; t += npairs, ++local) {
            const TileCoord c = q8_tile<2, 256>(args, t);
            const int acc = local % G::NACC;
            if (!warp_wait(&acc_full[acc], (local / G::NACC) & 1, abort, args.err, DEVERR_TIMEOUT_ACC)) {
                aborted_here = true;
                break;
            }
            tc_fence_after();
            const int row = c.m0 + G::HALF * rank + 32 * q + lane;
            const uint32_t t_base = tmem + ((uint32_t)(32 * q) << 16) + acc * G::ACC_COLS;
            for (int cb = set * 128; cb < set * 128 + 128; cb += 32) {
                uint32_t v[2][16];
                tmem_ld16(t_base + cb, v[0]);
                tmem_ld16(t_base + cb + 16, v[1]);
                tmem_wait_ld();
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int col = c.n0 + cb + 16 * h;
                    if (row < args.M && col < args.Nout) epilogue_store16<DT>(args, v[h], row, col, c.sp);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (rank == 0) mbar_arrive(&acc_empty[acc]);
                else mbar_arrive_remote(mapa_shared(smem_u32(&acc_empty[acc]), 0));
            }
        }
    }

    if (aborted_here && (warp == 0 || warp == 2)) {
        for (int i = 0; i < 64; ++i) __nanosleep(2000);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1 && lane == 0 && rank == 0) {
        // Every MMA of the pair has finished writing both CTAs' TMEM.
        long long t0 = clock64();
        while (!mbar_try_wait(mma_done, 0)) {
            if (clock64() - t0 > REELS_WAIT_LIMIT_CYCLES) {
                atomicOr(args.err, DEVERR_TIMEOUT_ACC);
                break;
            }
        }
    }
    __syncwarp();
    // Neither CTA leaves while its peer may still read its shared memory or
    // arrive on its barriers, or while MMAs may still write its TMEM.
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, G::TMEM_COLS);
    }
}

}  // namespace reels
