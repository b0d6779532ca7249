// tcgen05 / TMA kernels for the Int8-weight LoRA linear (sm_100a).
//
// q8_gemm_kernel: D[M x Nout] = [act | lora_act] . [dequant(W) ; lora_w]
//   The frozen weight arrives as int8 tiles through TMA, eight "dequant" warps
//   widen them to bf16/fp16 straight into the 128B-swizzled shared-memory
//   layout the tensor core reads, and one thread issues tcgen05.mma into an
//   fp32 accumulator in tensor memory.  The rank-r LoRA term rides along as
//   extra reduction blocks at the end of the same accumulation, so the
//   adapter costs one more pipeline stage, not another GEMM over Y.
//   Used for the forward Y (src/layers/quantization.jl:73-74 + lora.jl:86-94)
//   and for dX (quantization.jl:75-76 + the A'(B'dy) term of lora.jl:115-116).
//
// sk_gemm_kernel: the skinny rank-r GEMMs (N = r <= 256) with both operands
//   16-bit and fed by TMA: T = A.x, G = B'.dy (lora.jl:86, 112-113) and the
//   adapter gradients dA, dB (lora.jl:113-114), the latter reducing over the
//   token dimension and split across CTAs.
#pragma once
#include "common.cuh"
#include "convert.cuh"

namespace reels {

constexpr int BK = 64;       // reduction elements per pipeline stage (128 B of 16-bit)
constexpr int Q8_BN = 256;   // output columns per CTA
constexpr int Q8_THREADS = 352;  // 11 warps
constexpr int Q8_NCW = 8;        // dequant / epilogue warps (warps 3..10)

// ------------------------------------------------------------ q8 gemm
struct Q8Args {
    int M;             // rows of D (tokens)
    int Nout;          // columns of D
    int kb_total;      // main reduction blocks of 64
    int kb_per_split;  // main blocks per split (gridDim.z splits)
    int w_orient;      // 0: int8 staging rows are D columns  -> K-major B operand
                       // 1: int8 staging rows are reduction  -> MN-major B operand
    int scale_mode;    // 0 none, 1 per staging row, 2 per staging column
    int wscale_len;    // length of wscale (valid scale indices)
    const float *wscale;
    // LoRA extension blocks
    int r;             // rank (0: no extension)
    int ext_kind;      // 0: B-op = lora[r][Nout] (MN-major); 1: B-op = lora[Nout][r] (K-major)
    const void *lora;
    float ext_scale;
    const float *ext_div;  // per-column divisor for ext_kind 0 (nullable)
    // epilogue
    int epi_partial;         // 1: write fp32 partial sums
    const float *col_scale;  // per output column multiplier (nullable)
    const void *bias;        // act dtype [Nout] (nullable)
    void *out;
    long long ldo;
    float *partial;          // [splits][M][Nout]
    unsigned *err;
};

template <int MT>
struct Q8Geom {
    static constexpr int SAB = (MT == 2) ? 3 : 4;  // activation+weight (bf16) stages
    static constexpr int S8 = 2;                    // int8 staging stages
    static constexpr int A_BYTES = MT * 128 * 128;
    static constexpr int B_BYTES = Q8_BN * 128;
    static constexpr int W_BYTES = Q8_BN * BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int W_OFF = SAB * STAGE_BYTES;
    static constexpr int BAR_OFF = W_OFF + S8 * W_BYTES;
    // barriers: ab_full[SAB], ab_empty[SAB], w_full[S8], w_empty[S8], acc_full
    static constexpr int NBAR = 2 * SAB + 2 * S8 + 1;
    static constexpr int MISC_OFF = BAR_OFF + NBAR * 8;
    static constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;  // + alignment slack
    static constexpr int TMEM_COLS = MT * 256;
};

__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort, unsigned *err,
                                          unsigned code) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = wait_bar(bar, parity, abort, err, code) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    return ok != 0;
}

template <int DT>
__device__ __forceinline__ uint4 load8_act_scaled(const void *base, long long idx, int valid, float mul) {
    using E = Elem<DT>;
    const typename E::T *p = reinterpret_cast<const typename E::T *>(base) + idx;
    float f[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) f[t] = (t < valid) ? E::to_f(p[t]) * mul : 0.0f;
    uint4 o;
    o.x = E::pack2(f[0], f[1]);
    o.y = E::pack2(f[2], f[3]);
    o.z = E::pack2(f[4], f[5]);
    o.w = E::pack2(f[6], f[7]);
    return o;
}

template <int DT, int MT>
__global__ void __launch_bounds__(Q8_THREADS, 1)
    q8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmE, const Q8Args args) {
    using G = Q8Geom<MT>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    const uint32_t sbase = smem_u32(smem);

    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + G::BAR_OFF);
    uint64_t *ab_full = bars;
    uint64_t *ab_empty = bars + G::SAB;
    uint64_t *w_full = bars + 2 * G::SAB;
    uint64_t *w_empty = bars + 2 * G::SAB + G::S8;
    uint64_t *acc_full = bars + 2 * G::SAB + 2 * G::S8;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + G::MISC_OFF);
    volatile int *abort = reinterpret_cast<volatile int *>(smem + G::MISC_OFF + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * Q8_BN;
    const int m0 = blockIdx.y * (MT * 128);
    const int sp = blockIdx.z;
    const int splits = gridDim.z;
    const int kb0 = sp * args.kb_per_split;
    const int kb1 = min(args.kb_total, kb0 + args.kb_per_split);
    const int n_main = max(0, kb1 - kb0);
    const int n_ext = (sp == splits - 1 && args.r > 0) ? (args.r + 63) / 64 : 0;
    const int n_iter = n_main + n_ext;

    if (threadIdx.x == 0) {
        for (int i = 0; i < G::SAB; ++i) {
            mbar_init(&ab_full[i], 1 + Q8_NCW);
            mbar_init(&ab_empty[i], 1);
        }
        for (int i = 0; i < G::S8; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], Q8_NCW);
        }
        mbar_init(acc_full, 1);
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
    bool aborted_here = false;

    if (warp == 0) {
        // ---------------- activation producer (TMA) ----------------
        if (lane == 0) {
            for (int it = 0; it < n_iter; ++it) {
                const int s = it % G::SAB;
                const uint32_t ph = (it / G::SAB) & 1;
                if (!wait_bar(&ab_empty[s], ph ^ 1, abort, args.err, DEVERR_TIMEOUT_AB_EMPTY)) {
                    aborted_here = true;
                    break;
                }
                uint8_t *a_dst = smem + s * G::STAGE_BYTES;
                mbar_arrive_expect_tx(&ab_full[s], G::A_BYTES);
                if (it < n_main) {
                    tma_load_2d(a_dst, &tmA, (kb0 + it) * BK, m0, &ab_full[s]);
                } else {
                    const int e = it - n_main;
#pragma unroll
                    for (int b = 0; b < 2 * MT; ++b)
                        tma_load_2d(a_dst + b * 8192, &tmE, m0 + 64 * b, 64 * e, &ab_full[s]);
                }
            }
        }
    } else if (warp == 2) {
        // ---------------- int8 weight producer (TMA) ----------------
        if (lane == 0) {
            for (int it = 0; it < n_main; ++it) {
                const int s8 = it % G::S8;
                const uint32_t ph8 = (it / G::S8) & 1;
                if (!wait_bar(&w_empty[s8], ph8 ^ 1, abort, args.err, DEVERR_TIMEOUT_W_EMPTY)) {
                    aborted_here = true;
                    break;
                }
                uint8_t *w_dst = smem + G::W_OFF + s8 * G::W_BYTES;
                mbar_arrive_expect_tx(&w_full[s8], G::W_BYTES);
                const int kb = kb0 + it;
                if (args.w_orient == 0) tma_load_2d(w_dst, &tmW, kb * BK, n0, &w_full[s8]);
                else tma_load_2d(w_dst, &tmW, n0, kb * BK, &w_full[s8]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const int ab = (DT == DT_BF16) ? 1 : 0;
            const uint32_t id_main = idesc_f16(ab, 0, args.w_orient == 1 ? 1 : 0, 128, Q8_BN);
            const uint32_t id_ext = idesc_f16(ab, 1, args.ext_kind == 0 ? 1 : 0, 128, Q8_BN);
            for (int it = 0; it < n_iter; ++it) {
                const int s = it % G::SAB;
                const uint32_t ph = (it / G::SAB) & 1;
                if (!wait_bar(&ab_full[s], ph, abort, args.err, DEVERR_TIMEOUT_AB_FULL)) {
                    aborted_here = true;
                    break;
                }
                tc_fence_after();
                const uint32_t a_base = sbase + s * G::STAGE_BYTES;
                const uint32_t b_base = a_base + G::A_BYTES;
                if (it < n_main) {
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            const uint64_t ad = sdesc_sw128(a_base + mt * 16384 + kk * 32, 16, 1024);
                            const uint64_t bd = (args.w_orient == 0)
                                                    ? sdesc_sw128(b_base + kk * 32, 16, 1024)
                                                    : sdesc_sw128(b_base + kk * 2048, 8192, 1024);
                            mma_f16_ss(tmem + mt * 256, ad, bd, id_main, (it > 0 || kk > 0) ? 1u : 0u);
                        }
                } else {
                    const int e = it - n_main;
                    const int kext = min(64, args.r - 64 * e);
                    const int nk = (kext + 15) / 16;
                    for (int mt = 0; mt < MT; ++mt)
                        for (int kk = 0; kk < nk; ++kk) {
                            const uint64_t ad = sdesc_sw128(a_base + mt * 16384 + kk * 2048, 8192, 1024);
                            const uint64_t bd = (args.ext_kind == 0)
                                                    ? sdesc_sw128(b_base + kk * 2048, 8192, 1024)
                                                    : sdesc_sw128(b_base + kk * 32, 16, 1024);
                            mma_f16_ss(tmem + mt * 256, ad, bd, id_ext, (it > 0 || kk > 0) ? 1u : 0u);
                        }
                }
                mma_commit(&ab_empty[s]);
            }
            // Always committed, also after an abort: the teardown waits on it so
            // that no MMA is still writing tensor memory when it is freed.
            mma_commit(acc_full);
        }
    } else {
        // ---------------- dequant warps, then epilogue ----------------
        const int ct = threadIdx.x - 3 * 32;  // 0..255
        using E = Elem<DT>;
        for (int it = 0; it < n_iter; ++it) {
            const int s = it % G::SAB;
            const uint32_t ph = (it / G::SAB) & 1;
            const bool main_blk = it < n_main;
            const int s8 = it % G::S8;
            if (main_blk) {
                if (!warp_wait(&w_full[s8], (it / G::S8) & 1, abort, args.err, DEVERR_TIMEOUT_W_FULL)) {
                    aborted_here = true;
                    break;
                }
            }
            if (!warp_wait(&ab_empty[s], ph ^ 1, abort, args.err, DEVERR_TIMEOUT_AB_EMPTY)) {
                aborted_here = true;
                break;
            }
            const uint32_t b_base = sbase + s * G::STAGE_BYTES + G::A_BYTES;
            if (main_blk) {
                const uint32_t w_base = sbase + G::W_OFF + s8 * G::W_BYTES;
                const int kb = kb0 + it;
                // TMA coordinates of this staging tile: x = column origin, y = row origin.
                const int x0 = (args.w_orient == 0) ? kb * BK : n0;
                const int y0 = (args.w_orient == 0) ? n0 : kb * BK;
#pragma unroll 2
                for (int j = 0; j < 8; ++j) {
                    const int i = ct + 256 * j;
                    const uint2 v = ld_shared_v2(w_base + i * 8);
                    int row, c8;  // staging row and 8-byte column chunk
                    uint32_t dst;
                    if (args.w_orient == 0) {
                        row = i >> 3;
                        c8 = i & 7;
                        dst = b_base + sw128_off(row, c8);
                    } else {
                        row = i >> 5;
                        c8 = i & 31;
                        dst = b_base + (c8 >> 3) * 8192 + sw128_off(row, c8 & 7);
                    }
                    uint4 o;
                    if (args.scale_mode == 0) {
                        o = i8x8_exact<DT>(v);
                    } else if (args.scale_mode == 1) {
                        const int gi = y0 + row;
                        const float sc = gi < args.wscale_len ? __ldg(args.wscale + gi) : 0.0f;
                        o = i8x8_scaled1<DT>(v, sc);
                    } else {
                        float sc[8];
                        const int gi = x0 + c8 * 8;
#pragma unroll
                        for (int t = 0; t < 8; ++t)
                            sc[t] = (gi + t) < args.wscale_len ? __ldg(args.wscale + gi + t) : 0.0f;
                        o = i8x8_scaled<DT>(v, sc);
                    }
                    st_shared_v4(dst, o);
                }
            } else {
                const int e = it - n_main;
#pragma unroll 2
                for (int j = 0; j < 8; ++j) {
                    const int i = ct + 256 * j;
                    uint4 o;
                    uint32_t dst;
                    if (args.ext_kind == 0) {
                        // B-op rows = rank j, columns = output n (MN-major)
                        const int jr = i >> 5, c8 = i & 31;
                        const int jj = 64 * e + jr;
                        const int n = n0 + c8 * 8;
                        dst = b_base + (c8 >> 3) * 8192 + sw128_off(jr, c8 & 7);
                        if (jj < args.r && n < args.Nout) {
                            const typename E::T *p =
                                reinterpret_cast<const typename E::T *>(args.lora) + (long long)jj * args.Nout + n;
                            float f[8];
#pragma unroll
                            for (int t = 0; t < 8; ++t) {
                                f[t] = 0.0f;
                                if (n + t < args.Nout) {
                                    float m = args.ext_scale;
                                    if (args.ext_div) m = m / __ldg(args.ext_div + n + t);
                                    f[t] = E::to_f(p[t]) * m;
                                }
                            }
                            o.x = E::pack2(f[0], f[1]);
                            o.y = E::pack2(f[2], f[3]);
                            o.z = E::pack2(f[4], f[5]);
                            o.w = E::pack2(f[6], f[7]);
                        } else {
                            o = make_uint4(0, 0, 0, 0);
                        }
                    } else {
                        // B-op rows = output k, columns = rank j (K-major)
                        const int row = i >> 3, c8 = i & 7;
                        const int k = n0 + row;
                        const int jj = 64 * e + c8 * 8;
                        dst = b_base + sw128_off(row, c8);
                        if (k < args.Nout && jj < args.r) {
                            o = load8_act_scaled<DT>(args.lora, (long long)k * args.r + jj, min(8, args.r - jj),
                                                     args.ext_scale);
                        } else {
                            o = make_uint4(0, 0, 0, 0);
                        }
                    }
                    st_shared_v4(dst, o);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                if (main_blk) mbar_arrive(&w_empty[s8]);
                mbar_arrive(&ab_full[s]);
            }
        }

        // ---------------- epilogue ----------------
        if (!aborted_here && warp_wait(acc_full, 0, abort, args.err, DEVERR_TIMEOUT_ACC)) {
            tc_fence_after();
            const int ew = warp - 3;     // 0..7
            const int q = warp & 3;      // TMEM lane quarter this warp may read
            int mt, c_begin, c_end;
            if (MT == 2) {
                mt = ew >> 2;
                c_begin = 0;
                c_end = Q8_BN;
            } else {
                mt = 0;
                c_begin = (ew >> 2) * (Q8_BN / 2);
                c_end = c_begin + Q8_BN / 2;
            }
            const int row = m0 + mt * 128 + 32 * q + lane;
            for (int c = c_begin; c < c_end; c += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + mt * 256 + c, v);
                tmem_wait_ld();
                const int col = n0 + c;
                if (row < args.M && col < args.Nout) {
                    if (args.epi_partial) {
                        float *dst = args.partial + ((long long)sp * args.M + row) * args.Nout + col;
#pragma unroll
                        for (int t = 0; t < 16; t += 4)
                            *reinterpret_cast<float4 *>(dst + t) =
                                make_float4(__uint_as_float(v[t]), __uint_as_float(v[t + 1]),
                                            __uint_as_float(v[t + 2]), __uint_as_float(v[t + 3]));
                    } else {
                        float f[16];
#pragma unroll
                        for (int t = 0; t < 16; ++t) {
                            float x = __uint_as_float(v[t]);
                            if (args.col_scale) x *= __ldg(args.col_scale + col + t);
                            if (args.bias)
                                x += E::to_f(reinterpret_cast<const typename E::T *>(args.bias)[col + t]);
                            f[t] = x;
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
                        uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<typename E::T *>(args.out) +
                                                               (long long)row * args.ldo + col);
                        dst[0] = o0;
                        dst[1] = o1;
                    }
                }
            }
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
            // Bounded: the final commit arrives once every issued MMA is done.
            long long t0 = clock64();
            while (!mbar_try_wait(acc_full, 0)) {
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

// ------------------------------------------------------------ skinny gemm
constexpr int SK_THREADS = 192;  // warp0 TMA, warp1 MMA, warps 2..5 epilogue
constexpr int SK_STAGES = 4;
constexpr int SK_A_BYTES = 128 * 128;
constexpr int SK_B_MAX = 256 * 128;
constexpr int SK_STAGE_BYTES = SK_A_BYTES + SK_B_MAX;
constexpr int SK_BAR_OFF = SK_STAGES * SK_STAGE_BYTES;
constexpr int SK_SMEM_BYTES = SK_BAR_OFF + (2 * SK_STAGES + 1) * 8 + 16 + 1024;

struct SkArgs {
    int rows;          // rows of D
    int kb_total;      // reduction blocks of 64
    int kb_per_split;
    int npad;          // MMA N = B-operand rows (multiple of 16, <= 256)
    int a_mn;          // A operand MN-major (rows of D contiguous in memory)
    int epi;           // 0 transposed store act dtype, 1 fp32 accumulate, 2 fp32 partial
    int ncols;         // valid D columns (rank)
    float alpha;
    int accumulate;
    void *out;
    long long ldo;     // epi 0: row pitch of out[j][row]
    long long rs, cs;  // epi 1: out[row*rs + j*cs]
    float *partial;    // epi 2: [splits][rows][npad]
    unsigned *err;
};

template <int DT>
__global__ void __launch_bounds__(SK_THREADS, 1)
    sk_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const SkArgs args) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    const uint32_t sbase = smem_u32(smem);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + SK_BAR_OFF);
    uint64_t *empty = full + SK_STAGES;
    uint64_t *acc_full = full + 2 * SK_STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + SK_BAR_OFF + (2 * SK_STAGES + 1) * 8);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * 128;
    const int sp = blockIdx.y;
    const int kb0 = sp * args.kb_per_split;
    const int kb1 = min(args.kb_total, kb0 + args.kb_per_split);
    const int n_iter = max(0, kb1 - kb0);
    const uint32_t b_bytes = (uint32_t)args.npad * 128u;
    const uint32_t tmem_cols = args.npad <= 32 ? 32u : (args.npad <= 64 ? 64u : (args.npad <= 128 ? 128u : 256u));

    if (threadIdx.x == 0) {
        for (int i = 0; i < SK_STAGES; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(acc_full, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool aborted_here = false;

    if (warp == 0) {
        if (lane == 0) {
            for (int it = 0; it < n_iter; ++it) {
                const int s = it % SK_STAGES;
                const uint32_t ph = (it / SK_STAGES) & 1;
                if (!wait_bar(&empty[s], ph ^ 1, abort, args.err, DEVERR_TIMEOUT_AB_EMPTY)) {
                    aborted_here = true;
                    break;
                }
                uint8_t *a_dst = smem + s * SK_STAGE_BYTES;
                uint8_t *b_dst = a_dst + SK_A_BYTES;
                const int kb = kb0 + it;
                mbar_arrive_expect_tx(&full[s], SK_A_BYTES + b_bytes);
                if (args.a_mn) {
                    tma_load_2d(a_dst, &tmA, row0, kb * BK, &full[s]);
                    tma_load_2d(a_dst + 8192, &tmA, row0 + 64, kb * BK, &full[s]);
                } else {
                    tma_load_2d(a_dst, &tmA, kb * BK, row0, &full[s]);
                }
                tma_load_2d(b_dst, &tmB, kb * BK, 0, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const int ab = (DT == DT_BF16) ? 1 : 0;
            const uint32_t id = idesc_f16(ab, args.a_mn, 0, 128, args.npad);
            for (int it = 0; it < n_iter; ++it) {
                const int s = it % SK_STAGES;
                const uint32_t ph = (it / SK_STAGES) & 1;
                if (!wait_bar(&full[s], ph, abort, args.err, DEVERR_TIMEOUT_AB_FULL)) {
                    aborted_here = true;
                    break;
                }
                tc_fence_after();
                const uint32_t a_base = sbase + s * SK_STAGE_BYTES;
                const uint32_t b_base = a_base + SK_A_BYTES;
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t ad = args.a_mn ? sdesc_sw128(a_base + kk * 2048, 8192, 1024)
                                                  : sdesc_sw128(a_base + kk * 32, 16, 1024);
                    const uint64_t bd = sdesc_sw128(b_base + kk * 32, 16, 1024);
                    mma_f16_ss(tmem, ad, bd, id, (it > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&empty[s]);
            }
            mma_commit(acc_full);
        }
    } else {
        const int q = warp & 3;
        if (warp_wait(acc_full, 0, abort, args.err, DEVERR_TIMEOUT_ACC)) {
            tc_fence_after();
            const int row = row0 + 32 * q + lane;
            for (int c = 0; c < args.npad; c += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + c, v);
                tmem_wait_ld();
                if (row >= args.rows) continue;
                if (n_iter == 0) {
#pragma unroll
                    for (int t = 0; t < 16; ++t) v[t] = 0u;
                }
                if (args.epi == 2) {
                    float *dst = args.partial + ((long long)sp * args.rows + row) * args.npad + c;
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
            while (!mbar_try_wait(acc_full, 0)) {
                if (clock64() - t0 > REELS_WAIT_LIMIT_CYCLES) {
                    atomicOr(args.err, DEVERR_TIMEOUT_ACC);
                    break;
                }
            }
        }
        __syncwarp();
        tmem_dealloc(tmem, tmem_cols);
    }
}

}  // namespace reels
