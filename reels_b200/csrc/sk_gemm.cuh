// Skinny rank-r GEMMs on tcgen05 (sm_100a): both operands 16-bit and fed by
// TMA, N = r <= 256.  They compute T = A.x and G = s.(B'.dy) (lora.jl:86 and
// lora.jl:112-116) with the token dimension as rows, and the adapter
// gradients dA, dB (lora.jl:113-114) with the token dimension as the
// reduction, split across CTAs when the output alone does not fill the GPU.
#pragma once
#include "common.cuh"

namespace reels {

constexpr int BK = 64;  // reduction elements per pipeline stage (128 B of 16-bit)

__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort, unsigned *err,
                                          unsigned code) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = wait_bar(bar, parity, abort, err, code) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    return ok != 0;
}

// ------------------------------------------------------------ skinny gemm
// Persistent: each CTA walks work units u = blockIdx.x, blockIdx.x + gridDim.x,
// ... (a unit is one 128-row tile of D over one reduction split).  The TMA
// ring runs on across units, so a CTA's next tile streams in while the
// current one is multiplied, and the TMEM accumulator is double-buffered so
// the epilogue of one unit overlaps the MMAs of the next: the pipeline fill
// and the epilogue are paid once per CTA, not once per tile.
constexpr int SK_THREADS = 192;  // warp0 TMA, warp1 MMA, warps 2..5 epilogue
// The activation (or dy) tile SK_PF stages ahead of each TMA load is
// prefetched into L2: more DRAM requests in flight per SM than the shared-
// memory ring holds.  8 measured ~1.5% faster on the block step than none
// (4: no change).
constexpr int SK_PF = 8;
constexpr int SK_A_BYTES = 128 * 128;
constexpr int SK_MAX_STAGES = 8;
// Ring buffer for the stages; the stage count is chosen per launch from the
// B tile size (rank): these kernels stream x or dy from HBM, so they keep as
// many bytes in flight as the budget allows (8 stages up to rank 64).
constexpr int SK_RING_BYTES = 200 * 1024;
constexpr int SK_BAR_OFF = SK_RING_BYTES;
constexpr int SK_NBAR = 2 * SK_MAX_STAGES + 5;  // full, empty, acc_full[2], acc_empty[2], mma_done
constexpr int SK_SMEM_BYTES = SK_BAR_OFF + SK_NBAR * 8 + 16 + 1024;

__host__ __device__ constexpr int sk_stage_bytes(int npad) { return SK_A_BYTES + npad * 128; }
__host__ __device__ constexpr int sk_stages(int npad) {
    return SK_RING_BYTES / sk_stage_bytes(npad) < SK_MAX_STAGES ? SK_RING_BYTES / sk_stage_bytes(npad)
                                                                 : SK_MAX_STAGES;
}

struct SkArgs {
    int rows;          // rows of D
    int kb_total;      // reduction blocks of 64
    int kb_per_split;
    int splits;
    int npad;          // MMA N = B-operand rows (multiple of 16, <= 256)
    int a_mn;          // A operand MN-major (rows of D contiguous in memory)
    int epi;           // 0 transposed store act dtype, 1 fp32 accumulate, 2 fp32 partial
    int ncols;         // valid D columns (rank)
    float alpha;
    int accumulate;
    void *out;
    long long ldo;     // epi 0: row pitch of out[j][row]
    long long rs, cs;  // epi 1: out[row*rs + j*cs]
    float *partial;    // epi 2: [splits][rows][npad], or [splits][npad][rows] with pcol
    unsigned *err;
    int pcol;          // partial layout with rows contiguous (see sk_reduce_kernel)
};

struct SkUnit {
    int row0, sp, kb0, n_iter;
};
__device__ __forceinline__ SkUnit sk_unit(const SkArgs &a, int tiles, int u) {
    SkUnit w;
    w.sp = u / tiles;
    w.row0 = (u - w.sp * tiles) * 128;
    w.kb0 = w.sp * a.kb_per_split;
    w.n_iter = max(0, min(a.kb_total, w.kb0 + a.kb_per_split) - w.kb0);
    return w;
}

template <int DT>
__global__ void __launch_bounds__(SK_THREADS, 1)
    sk_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const SkArgs args) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    const uint32_t sbase = smem_u32(smem);
    const int NS = sk_stages(args.npad);
    const int STAGE = sk_stage_bytes(args.npad);  // multiple of 1024: A tile 16 KB + npad*128 B
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + SK_BAR_OFF);
    uint64_t *empty = full + SK_MAX_STAGES;
    uint64_t *acc_full = full + 2 * SK_MAX_STAGES;
    uint64_t *acc_empty = acc_full + 2;
    uint64_t *mma_done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + SK_BAR_OFF + SK_NBAR * 8);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = (args.rows + 127) / 128;
    const int units = tiles * args.splits;
    const uint32_t b_bytes = (uint32_t)args.npad * 128u;
    const uint32_t acc_cols = args.npad <= 32 ? 32u : (args.npad <= 64 ? 64u : (args.npad <= 128 ? 128u : 256u));

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 4);  // one arrival per epilogue warp
        }
        mbar_init(mma_done, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * acc_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddep_wait();  // the previous kernel's outputs are complete from here on
    bool aborted_here = false;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0;
            for (int u = blockIdx.x; u < units && !aborted_here; u += gridDim.x) {
                const SkUnit w = sk_unit(args, tiles, u);
                for (int it = 0; it < w.n_iter; ++it, ++g) {
                    const int s = g % NS;
                    const uint32_t ph = (g / NS) & 1;
                    if (!wait_bar(&empty[s], ph ^ 1, abort, args.err, DEVERR_TIMEOUT_AB_EMPTY)) {
                        aborted_here = true;
                        break;
                    }
                    uint8_t *a_dst = smem + s * STAGE;
                    uint8_t *b_dst = a_dst + SK_A_BYTES;
                    const int kb = w.kb0 + it;
                    mbar_arrive_expect_tx(&full[s], SK_A_BYTES + b_bytes);
                    if (args.a_mn) {
                        tma_load_2d(a_dst, &tmA, w.row0, kb * BK, &full[s]);
                        tma_load_2d(a_dst + 8192, &tmA, w.row0 + 64, kb * BK, &full[s]);
                    } else {
                        tma_load_2d(a_dst, &tmA, kb * BK, w.row0, &full[s]);
                    }
                    tma_load_2d(b_dst, &tmB, kb * BK, 0, &full[s]);
                    if (SK_PF > 0 && it + SK_PF < w.n_iter) {
                        // the activation block SK_PF stages ahead, into L2 only
                        const int kp = kb + SK_PF;
                        if (args.a_mn) {
                            tma_prefetch_l2_2d(&tmA, w.row0, kp * BK);
                            tma_prefetch_l2_2d(&tmA, w.row0 + 64, kp * BK);
                        } else {
                            tma_prefetch_l2_2d(&tmA, kp * BK, w.row0);
                        }
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const int ab = (DT == DT_BF16) ? 1 : 0;
            const uint32_t id = idesc_f16(ab, args.a_mn, 0, 128, args.npad);
            uint32_t g = 0, lu = 0;
            for (int u = blockIdx.x; u < units && !aborted_here; u += gridDim.x, ++lu) {
                const SkUnit w = sk_unit(args, tiles, u);
                const int acc = lu & 1;
                if (!wait_bar(&acc_empty[acc], ((lu >> 1) & 1) ^ 1, abort, args.err, DEVERR_TIMEOUT_ACC)) {
                    aborted_here = true;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tm = tmem + acc * acc_cols;
                for (int it = 0; it < w.n_iter; ++it, ++g) {
                    const int s = g % NS;
                    const uint32_t ph = (g / NS) & 1;
                    if (!wait_bar(&full[s], ph, abort, args.err, DEVERR_TIMEOUT_AB_FULL)) {
                        aborted_here = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_base = sbase + s * STAGE;
                    const uint32_t b_base = a_base + SK_A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t ad = args.a_mn ? sdesc_sw128(a_base + kk * 2048, 8192, 1024)
                                                      : sdesc_sw128(a_base + kk * 32, 16, 1024);
                        const uint64_t bd = sdesc_sw128(b_base + kk * 32, 16, 1024);
                        mma_f16_ss(d_tm, ad, bd, id, (it > 0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit(&empty[s]);
                }
                if (aborted_here) break;
                mma_commit(&acc_full[acc]);
            }
            mma_commit(mma_done);
        }
    } else {
        const int q = warp & 3;
        uint32_t lu = 0;
        for (int u = blockIdx.x; u < units && !aborted_here; u += gridDim.x, ++lu) {
            const SkUnit w = sk_unit(args, tiles, u);
            const int acc = lu & 1;
            if (!warp_wait(&acc_full[acc], (lu >> 1) & 1, abort, args.err, DEVERR_TIMEOUT_ACC)) {
                aborted_here = true;
                break;
            }
            tc_fence_after();
            const int row = w.row0 + 32 * q + lane;
            for (int c = 0; c < args.npad; c += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + acc * acc_cols + c, v);
                tmem_wait_ld();
                if (c + 16 >= args.npad) {
                    // the whole accumulator is in registers: the next unit may use it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[acc]);
                }
                if (row >= args.rows) continue;
                if (w.n_iter == 0) {
#pragma unroll
                    for (int t = 0; t < 16; ++t) v[t] = 0u;
                }
                if (args.epi == 2 && args.pcol) {
                    // rows contiguous: lanes (consecutive rows) write 128 bytes per column
                    float *dst = args.partial + ((long long)w.sp * args.npad + c) * args.rows + row;
#pragma unroll
                    for (int t = 0; t < 16; ++t) dst[(long long)t * args.rows] = __uint_as_float(v[t]);
                } else if (args.epi == 2) {
                    float *dst = args.partial + ((long long)w.sp * args.rows + row) * args.npad + c;
#pragma unroll
                    for (int t = 0; t < 16; t += 4)
                        *reinterpret_cast<float4 *>(dst + t) =
                            make_float4(__uint_as_float(v[t]), __uint_as_float(v[t + 1]), __uint_as_float(v[t + 2]),
                                        __uint_as_float(v[t + 3]));
                } else if (args.epi == 0) {
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        const int j = c + t;
                        if (j < args.ncols)
                            store_act(args.out, (long long)j * args.ldo + row, DT, args.alpha * __uint_as_float(v[t]));
                    }
                } else {
                    float *o = reinterpret_cast<float *>(args.out);
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        const int j = c + t;
                        if (j < args.ncols) {
                            const long long idx = (long long)row * args.rs + (long long)j * args.cs;
                            const float prev = args.accumulate ? o[idx] : 0.0f;
                            o[idx] = prev + args.alpha * __uint_as_float(v[t]);
                        }
                    }
                }
            }
        }
    }

    if (aborted_here && warp == 0) {
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
        tmem_dealloc(tmem, 2 * acc_cols);
    }
}

// ------------------------------------------------------------ one pass over dy
// Both rank-r products of the backward that read dy (lora.jl:112-114):
//     G[m][j]  = sum_n dy[m][n] B[j][n]          (tokens are the rows)
//     dB[j][n] = sum_m T[j][m] dy[m][n]          (tokens are the reduction)
// from ONE read of dy.  The work is a grid of token ranges x output-feature
// ranges, one CTA each.  A CTA walks its token tiles (128 tokens) and, inside
// each, its feature tiles (128 features); every stage is one 128 x 128 tile
// of dy plus the matching 128 columns of B and 128 tokens of T, and feeds two
// MMA chains:
//   G  (K-major dy, M = tokens):    one accumulator per token tile, complete
//                                   over the CTA's feature range when the
//                                   tile ends (double-buffered);
//   dB (MN-major dy, M = features): one accumulator per feature tile of the
//                                   range, complete over the CTA's token
//                                   range when the CTA ends.
// Each output is a final value when its range covers the whole reduction,
// else an fp32 partial that sk_reduce_kernel sums in a fixed order.
constexpr int DU_DY_BYTES = 2 * 128 * 128;  // 128 tokens x 128 features, two 64-feature boxes
constexpr int DU_NBAR = 2 * SK_MAX_STAGES + 6;  // full, empty, g_full[2], g_empty[2], db_full, mma_done
constexpr int DU_SMEM_BYTES = SK_BAR_OFF + DU_NBAR * 8 + 16 + 1024;

__host__ __device__ constexpr int du_stage_bytes(int npad) { return DU_DY_BYTES + 4 * npad * 128; }
__host__ __device__ constexpr int du_stages(int npad) {
    return SK_RING_BYTES / du_stage_bytes(npad) < SK_MAX_STAGES ? SK_RING_BYTES / du_stage_bytes(npad)
                                                                 : SK_MAX_STAGES;
}
__host__ __device__ constexpr int du_acc_cols(int npad) {
    return npad <= 32 ? 32 : (npad <= 64 ? 64 : (npad <= 128 ? 128 : 256));
}
// Feature tiles one CTA can hold dB accumulators for (TMEM has 512 columns,
// two of them go to the G double buffer).
__host__ __device__ constexpr int du_max_ftiles(int npad) { return 512 / du_acc_cols(npad) - 2; }

struct SkDualArgs {
    int M, N;              // tokens, output features
    int tm_tiles, tn_tiles;
    int splits_m, splits_n;
    int npad, ncols;
    int tmem_cols;         // power of two >= (2 + max feature tiles per CTA) * acc columns
    void *g_out;           // splits_n == 1: 16-bit G [ncols][ldm], scaled by g_alpha
    long long ldm;
    float g_alpha;
    float *g_part;         // splits_n > 1: [splits_n][npad][M]
    float *db_out;         // splits_m == 1: fp32 dB [ncols][N], db_alpha * sum (+ previous)
    float db_alpha;
    int accumulate;
    float *db_part;        // splits_m > 1: [splits_m][npad][N]
    unsigned *err;
};

template <int DT>
__global__ void __launch_bounds__(SK_THREADS, 1)
    sk_dual_kernel(const __grid_constant__ CUtensorMap tmDy, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmT, const SkDualArgs args) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    const uint32_t sbase = smem_u32(smem);
    const int NS = du_stages(args.npad);
    const int STAGE = du_stage_bytes(args.npad);  // multiple of 8 KB
    const uint32_t bbox = (uint32_t)args.npad * 128u;  // one [npad][64] box of B or T
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + SK_BAR_OFF);
    uint64_t *empty = full + SK_MAX_STAGES;
    uint64_t *g_full = full + 2 * SK_MAX_STAGES;
    uint64_t *g_empty = g_full + 2;
    uint64_t *db_full = g_empty + 2;
    uint64_t *mma_done = db_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + SK_BAR_OFF + DU_NBAR * 8);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sm = blockIdx.x / args.splits_n, sn = blockIdx.x - sm * args.splits_n;
    const int tm0 = (int)((long long)sm * args.tm_tiles / args.splits_m);
    const int tm1 = (int)((long long)(sm + 1) * args.tm_tiles / args.splits_m);
    const int tn0 = (int)((long long)sn * args.tn_tiles / args.splits_n);
    const int tn1 = (int)((long long)(sn + 1) * args.tn_tiles / args.splits_n);
    const uint32_t acc_cols = (uint32_t)du_acc_cols(args.npad);

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&g_full[i], 1);
            mbar_init(&g_empty[i], 4);  // one arrival per epilogue warp
        }
        mbar_init(db_full, 1);
        mbar_init(mma_done, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmDy);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmT);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, (uint32_t)args.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddep_wait();  // the previous kernel's outputs (T) are complete from here on
    bool aborted_here = false;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0;
            for (int t = tm0; t < tm1 && !aborted_here; ++t) {
                for (int nt = tn0; nt < tn1; ++nt, ++g) {
                    const int s = g % NS;
                    const uint32_t ph = (g / NS) & 1;
                    if (!wait_bar(&empty[s], ph ^ 1, abort, args.err, DEVERR_TIMEOUT_AB_EMPTY)) {
                        aborted_here = true;
                        break;
                    }
                    uint8_t *st = smem + s * STAGE;
                    mbar_arrive_expect_tx(&full[s], DU_DY_BYTES + 4 * bbox);
                    tma_load_2d(st, &tmDy, nt * 128, t * 128, &full[s]);
                    tma_load_2d(st + 16384, &tmDy, nt * 128 + 64, t * 128, &full[s]);
                    tma_load_2d(st + DU_DY_BYTES, &tmB, nt * 128, 0, &full[s]);
                    tma_load_2d(st + DU_DY_BYTES + bbox, &tmB, nt * 128 + 64, 0, &full[s]);
                    tma_load_2d(st + DU_DY_BYTES + 2 * bbox, &tmT, t * 128, 0, &full[s]);
                    tma_load_2d(st + DU_DY_BYTES + 3 * bbox, &tmT, t * 128 + 64, 0, &full[s]);
                    if (SK_PF > 0) {
                        // the dy tile SK_PF stages ahead, into L2 only
                        const int kn = tn1 - tn0;
                        const int f = (t - tm0) * kn + (nt - tn0) + SK_PF;
                        const int tp = tm0 + f / kn, np = tn0 + f % kn;
                        if (tp < tm1) {
                            tma_prefetch_l2_2d(&tmDy, np * 128, tp * 128);
                            tma_prefetch_l2_2d(&tmDy, np * 128 + 64, tp * 128);
                        }
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const int ab = (DT == DT_BF16) ? 1 : 0;
            const uint32_t id_g = idesc_f16(ab, 0, 0, 128, args.npad);
            const uint32_t id_b = idesc_f16(ab, 1, 0, 128, args.npad);
            uint32_t g = 0, lt = 0;
            for (int t = tm0; t < tm1 && !aborted_here; ++t, ++lt) {
                const int gb = lt & 1;
                if (!wait_bar(&g_empty[gb], ((lt >> 1) & 1) ^ 1, abort, args.err, DEVERR_TIMEOUT_ACC)) {
                    aborted_here = true;
                    break;
                }
                tc_fence_after();
                const uint32_t g_tm = tmem + gb * acc_cols;
                for (int nt = tn0; nt < tn1; ++nt, ++g) {
                    const int s = g % NS;
                    const uint32_t ph = (g / NS) & 1;
                    if (!wait_bar(&full[s], ph, abort, args.err, DEVERR_TIMEOUT_AB_FULL)) {
                        aborted_here = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t dy_base = sbase + s * STAGE;
                    const uint32_t b_base = dy_base + DU_DY_BYTES;
                    const uint32_t t_base = b_base + 2 * bbox;
                    const uint32_t db_tm = tmem + (2 + nt - tn0) * acc_cols;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {  // G: reduction over this tile's 128 features
                        const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                        const uint32_t boff = (kk >> 2) * bbox + (kk & 3) * 32;
                        mma_f16_ss(g_tm, sdesc_sw128(dy_base + off, 16, 1024), sdesc_sw128(b_base + boff, 16, 1024),
                                   id_g, (nt > tn0 || kk > 0) ? 1u : 0u);
                    }
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {  // dB: reduction over this tile's 128 tokens
                        const uint32_t boff = (kk >> 2) * bbox + (kk & 3) * 32;
                        mma_f16_ss(db_tm, sdesc_sw128(dy_base + kk * 2048, 16384, 1024),
                                   sdesc_sw128(t_base + boff, 16, 1024), id_b, (t > tm0 || kk > 0) ? 1u : 0u);
                    }
                    mma_commit(&empty[s]);
                }
                if (aborted_here) break;
                mma_commit(&g_full[gb]);
            }
            if (!aborted_here) mma_commit(db_full);
            mma_commit(mma_done);
        }
    } else {
        const int q = warp & 3;
        const uint32_t lane_off = (uint32_t)(32 * q) << 16;
        uint32_t lt = 0;
        for (int t = tm0; t < tm1 && !aborted_here; ++t, ++lt) {
            const int gb = lt & 1;
            if (!warp_wait(&g_full[gb], (lt >> 1) & 1, abort, args.err, DEVERR_TIMEOUT_ACC)) {
                aborted_here = true;
                break;
            }
            tc_fence_after();
            const int row = t * 128 + 32 * q + lane;  // token
            for (int c = 0; c < args.npad; c += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + lane_off + gb * acc_cols + c, v);
                tmem_wait_ld();
                if (c + 16 >= args.npad) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&g_empty[gb]);
                }
                if (row >= args.M) continue;
                if (args.splits_n > 1) {
                    float *dst = args.g_part + ((long long)sn * args.npad + c) * args.M + row;
#pragma unroll
                    for (int u = 0; u < 16; ++u) dst[(long long)u * args.M] = __uint_as_float(v[u]);
                } else {
#pragma unroll
                    for (int u = 0; u < 16; ++u)
                        if (c + u < args.ncols)
                            store_act(args.g_out, (long long)(c + u) * args.ldm + row, DT,
                                      args.g_alpha * __uint_as_float(v[u]));
                }
            }
        }
        if (!aborted_here && warp_wait(db_full, 0, abort, args.err, DEVERR_TIMEOUT_ACC)) {
            tc_fence_after();
            for (int nt = tn0; nt < tn1; ++nt) {
                const int col = nt * 128 + 32 * q + lane;  // output feature
                for (int c = 0; c < args.npad; c += 16) {
                    uint32_t v[16];
                    tmem_ld16(tmem + lane_off + (2 + nt - tn0) * acc_cols + c, v);
                    tmem_wait_ld();
                    if (col >= args.N) continue;
                    if (args.splits_m > 1) {
                        float *dst = args.db_part + ((long long)sm * args.npad + c) * args.N + col;
#pragma unroll
                        for (int u = 0; u < 16; ++u) dst[(long long)u * args.N] = __uint_as_float(v[u]);
                    } else {
#pragma unroll
                        for (int u = 0; u < 16; ++u) {
                            if (c + u < args.ncols) {
                                float *o = args.db_out + (long long)(c + u) * args.N + col;
                                *o = (args.accumulate ? *o : 0.0f) + args.db_alpha * __uint_as_float(v[u]);
                            }
                        }
                    }
                }
            }
        }
    }

    if (aborted_here && warp == 0) {
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
        tmem_dealloc(tmem, (uint32_t)args.tmem_cols);
    }
}

}  // namespace reels
