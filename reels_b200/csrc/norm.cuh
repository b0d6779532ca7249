// The producer of the linears' input in the Wan block: LayerNorm followed by
// the AdaLN modulation,
//   out = mixed_affine(layernorm(x; epsilon, weight, bias), scale, shift)
// (src/layers/linear.jl:26-36,49-59; the block calls it at
// src/models/wan21/transformer.jl:287-289), in one pass over each row, and
// its backward.  The reference evaluates it as about eight full-array
// broadcasts and reductions with fp32 temporaries.
//
// Forward, per row of K features (token m, sample b = m / tokens_per_sample):
//   mean = sum(x) / K ; var = sum((x - mean)^2) / K ; d = sqrt(var + eps)
//   y = (x - mean) / d  (* weight) (+ bias) ; ln = round(y)
//   out = round(ln * (1 + scale[b]) + shift[b])
// every operation in fp32 and rounded once (no fused multiply-adds), the two
// sums in a fixed tree order.
// Backward: g = round(dout * (1 + scale[b])) (the modulation's pullback,
// modulation.jl:13-22), gw = g * weight, and with yhat = (x - mean) / d
//   dx = (gw - mean(gw) - yhat * mean(gw * yhat)) / d
// plus the per-sample parameter gradients dscale[b] = sum_m dout * ln and
// dshift[b] = sum_m dout over the sample's tokens, reduced in a fixed order.
#pragma once
#include "act.cuh"
#include "common.cuh"

namespace reels {

constexpr int LN_THREADS = 256;
constexpr int64_t LN_MAX_K = 16384;  // the row (x, and g in the backward) is staged in shared memory
constexpr int LN_COL_ROWS = 128;  // rows per block of the parameter-gradient reduction

// Block-wide fp32 sum in a fixed order (warp shuffles, then warp totals).
__device__ __forceinline__ float ln_block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5;
    __syncthreads();  // red may still be read by the previous sum
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float s = 0.0f;
    for (int i = 0; i < LN_THREADS / 32; ++i) s += red[i];
    return s;
}

// Loads row m of x into shared memory as fp32 and returns (mean, d).
template <int DT>
__device__ __forceinline__ float2 ln_row_stats(const void *x, int64_t m, int64_t K, float eps, float *row, float *red) {
    const typename Elem<DT>::T *xr = reinterpret_cast<const typename Elem<DT>::T *>(x) + m * K;
    float s = 0.0f;
    for (int64_t k = threadIdx.x; k < K; k += LN_THREADS) {
        const float v = Elem<DT>::to_f(xr[k]);
        row[k] = v;
        s = __fadd_rn(s, v);
    }
    const float mean = __fdiv_rn(ln_block_sum(s, red), (float)K);
    float q = 0.0f;
    for (int64_t k = threadIdx.x; k < K; k += LN_THREADS) {
        const float c = __fsub_rn(row[k], mean);
        q = __fadd_rn(q, __fmul_rn(c, c));
    }
    const float var = __fdiv_rn(ln_block_sum(q, red), (float)K);
    return make_float2(mean, __fsqrt_rn(__fadd_rn(var, eps)));
}

// ln (the rounded LayerNorm output) of one element.
template <int DT>
__device__ __forceinline__ float ln_value(float xv, float mean, float d, const void *lnw, const void *lnb, int64_t k) {
    float y = __fdiv_rn(__fsub_rn(xv, mean), d);
    if (lnw) y = __fmul_rn(y, Elem<DT>::to_f(reinterpret_cast<const typename Elem<DT>::T *>(lnw)[k]));
    if (lnb) y = __fadd_rn(y, Elem<DT>::to_f(reinterpret_cast<const typename Elem<DT>::T *>(lnb)[k]));
    return round_act<DT>(y);
}

// Row statistics with 16-byte loads (8 elements of a 16-bit type; K % 8 == 0,
// x 16-byte aligned).  Each thread owns runs of 8 consecutive elements
// instead of every LN_THREADS-th one, so its partial sums run in a different
// (still fixed) order from ln_row_stats'.
template <int DT>
__device__ __forceinline__ float2 ln_row_stats_v8(const void *x, int64_t m, int64_t K, float eps, float *row,
                                                  float *red) {
    const uint4 *xr = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(x) + m * K);
    float s = 0.0f;
    for (int64_t v = threadIdx.x; v < K / 8; v += LN_THREADS) {
        const uint4 w = xr[v];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        float f[8];
#pragma unroll
        for (int h = 0; h < 4; ++h) unpack2<DT>(ws[h], f[2 * h], f[2 * h + 1]);
        reinterpret_cast<float4 *>(row)[2 * v] = make_float4(f[0], f[1], f[2], f[3]);
        reinterpret_cast<float4 *>(row)[2 * v + 1] = make_float4(f[4], f[5], f[6], f[7]);
#pragma unroll
        for (int e = 0; e < 8; ++e) s = __fadd_rn(s, f[e]);
    }
    const float mean = __fdiv_rn(ln_block_sum(s, red), (float)K);
    float q = 0.0f;
    for (int64_t v = threadIdx.x; v < K / 8; v += LN_THREADS) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float c = __fsub_rn(row[8 * v + e], mean);
            q = __fadd_rn(q, __fmul_rn(c, c));
        }
    }
    const float var = __fdiv_rn(ln_block_sum(q, red), (float)K);
    return make_float2(mean, __fsqrt_rn(__fadd_rn(var, eps)));
}

template <int DT>
__global__ void __launch_bounds__(LN_THREADS) ln_modulate_kernel(const void *x, int64_t M, int64_t K, int64_t tps,
                                                                 const void *scale, const void *shift,
                                                                 const void *lnw, const void *lnb, float eps,
                                                                 void *out) {
    griddep_wait();
    extern __shared__ float row[];
    __shared__ float red[LN_THREADS / 32];
    using T = typename Elem<DT>::T;
    if constexpr (DT != DT_F32) {
        // 16-byte path: x, out, scale, shift 16-byte aligned, K % 8 == 0, no LayerNorm affine
        const bool vec = (K & 7) == 0 && !lnw && !lnb &&
                         ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
                           reinterpret_cast<uintptr_t>(scale) | reinterpret_cast<uintptr_t>(shift)) & 15) == 0;
        if (vec) {
            for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
                const float2 st = ln_row_stats_v8<DT>(x, m, K, eps, row, red);
                const int64_t b = m / tps;
                const uint4 *sc = scale ? reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(scale) + b * K) : nullptr;
                const uint4 *sh = shift ? reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(shift) + b * K) : nullptr;
                uint4 *o = reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(out) + m * K);
                for (int64_t v = threadIdx.x; v < K / 8; v += LN_THREADS) {
                    float f[8], fs[8], fh[8];
                    uint4 sw = sc ? sc[v] : make_uint4(0, 0, 0, 0), hw = sh ? sh[v] : make_uint4(0, 0, 0, 0);
                    const uint32_t sws[4] = {sw.x, sw.y, sw.z, sw.w}, hws[4] = {hw.x, hw.y, hw.z, hw.w};
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        unpack2<DT>(sws[h], fs[2 * h], fs[2 * h + 1]);
                        unpack2<DT>(hws[h], fh[2 * h], fh[2 * h + 1]);
                    }
                    uint32_t ow[4];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        float vv = round_act<DT>(__fdiv_rn(__fsub_rn(row[8 * v + e], st.x), st.y));
                        if (sc) vv = __fmul_rn(vv, __fadd_rn(1.0f, fs[e]));
                        if (sh) vv = __fadd_rn(vv, fh[e]);
                        f[e] = vv;
                    }
#pragma unroll
                    for (int h = 0; h < 4; ++h) ow[h] = Elem<DT>::pack2(f[2 * h], f[2 * h + 1]);
                    o[v] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
                }
            }
            return;
        }
    }
    for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
        const float2 st = ln_row_stats<DT>(x, m, K, eps, row, red);
        const int64_t b = m / tps;
        const T *sc = scale ? reinterpret_cast<const T *>(scale) + b * K : nullptr;
        const T *sh = shift ? reinterpret_cast<const T *>(shift) + b * K : nullptr;
        T *o = reinterpret_cast<T *>(out) + m * K;
        for (int64_t k = threadIdx.x; k < K; k += LN_THREADS) {
            float v = ln_value<DT>(row[k], st.x, st.y, lnw, lnb, k);
            if (sc) v = __fmul_rn(v, __fadd_rn(1.0f, Elem<DT>::to_f(sc[k])));
            if (sh) v = __fadd_rn(v, Elem<DT>::to_f(sh[k]));
            o[k] = Elem<DT>::from_f(v);
        }
    }
}

// ------------------------------------------------------------ one row per warp
// The 16-byte path (16-bit types, K % 8 == 0, 16-byte aligned rows, no
// LayerNorm affine) runs one row per warp: sums are warp shuffles in a fixed
// order, nothing waits on a block barrier, and a CTA keeps eight rows in
// flight.  The row is read from DRAM once; its second and third passes hit
// L2 (or L1).  Each element takes the same single-rounded operation
// sequence as the block kernels; the sums run in another fixed order.
__device__ __forceinline__ float warp_sum_fixed(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// (mean, d) of row xr (K / 8 16-byte chunks), lane-strided chunks.
template <int DT>
__device__ __forceinline__ float2 ln_warp_stats(const uint4 *xr, int64_t nv, int64_t K, float eps, int lane) {
    float s = 0.0f;
    for (int64_t v = lane; v < nv; v += 32) {
        const uint4 w = xr[v];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            float a, b;
            unpack2<DT>(ws[h], a, b);
            s = __fadd_rn(__fadd_rn(s, a), b);
        }
    }
    const float mean = __fdiv_rn(warp_sum_fixed(s), (float)K);
    float q = 0.0f;
    for (int64_t v = lane; v < nv; v += 32) {
        const uint4 w = xr[v];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            float a, b;
            unpack2<DT>(ws[h], a, b);
            const float ca = __fsub_rn(a, mean), cb = __fsub_rn(b, mean);
            q = __fadd_rn(__fadd_rn(q, __fmul_rn(ca, ca)), __fmul_rn(cb, cb));
        }
    }
    const float var = __fdiv_rn(warp_sum_fixed(q), (float)K);
    return make_float2(mean, __fsqrt_rn(__fadd_rn(var, eps)));
}

template <int DT>
__global__ void __launch_bounds__(LN_THREADS) ln_modulate_warp_kernel(const void *x, int64_t M, int64_t K,
                                                                      int64_t tps, const void *scale,
                                                                      const void *shift, float eps, void *out) {
    griddep_wait();
    const int lane = threadIdx.x & 31;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t nv = K / 8;
    for (int64_t m = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; m < M; m += nw) {
        const uint4 *xr = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(x) + m * K);
        const float2 st = ln_warp_stats<DT>(xr, nv, K, eps, lane);
        const int64_t b = m / tps;
        const uint4 *sc = scale ? reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(scale) + b * K) : nullptr;
        const uint4 *sh = shift ? reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(shift) + b * K) : nullptr;
        uint4 *o = reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(out) + m * K);
        for (int64_t v = lane; v < nv; v += 32) {
            const uint4 w = xr[v];
            const uint4 sw = sc ? sc[v] : make_uint4(0, 0, 0, 0), hw = sh ? sh[v] : make_uint4(0, 0, 0, 0);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w}, sws[4] = {sw.x, sw.y, sw.z, sw.w},
                           hws[4] = {hw.x, hw.y, hw.z, hw.w};
            uint32_t ow[4];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                float xv[2], fs[2], fh[2], f[2];
                unpack2<DT>(ws[h], xv[0], xv[1]);
                unpack2<DT>(sws[h], fs[0], fs[1]);
                unpack2<DT>(hws[h], fh[0], fh[1]);
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float vv = round_act<DT>(__fdiv_rn(__fsub_rn(xv[e], st.x), st.y));
                    if (sc) vv = __fmul_rn(vv, __fadd_rn(1.0f, fs[e]));
                    if (sh) vv = __fadd_rn(vv, fh[e]);
                    f[e] = vv;
                }
                ow[h] = Elem<DT>::pack2(f[0], f[1]);
            }
            o[v] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        }
    }
}

// dx per row, one row per warp (the 16-byte path, no LayerNorm weight);
// also the row's (mean, d) for the parameter reduction.  g is recomputed from
// dout in the last pass instead of being kept.
template <int DT>
__global__ void __launch_bounds__(LN_THREADS) ln_modulate_bwd_warp_kernel(const void *x, const void *dout, int64_t M,
                                                                          int64_t K, int64_t tps, const void *scale,
                                                                          float eps, void *dx, float2 *stats) {
    griddep_wait();
    const int lane = threadIdx.x & 31;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t nv = K / 8;
    for (int64_t m = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; m < M; m += nw) {
        const uint4 *xr = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(x) + m * K);
        const uint4 *dr = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(dout) + m * K);
        const float2 st = ln_warp_stats<DT>(xr, nv, K, eps, lane);
        if (lane == 0 && stats) stats[m] = st;
        const int64_t b = m / tps;
        const uint4 *sc = scale ? reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(scale) + b * K) : nullptr;
        // g (the modulation's pullback, rounded) and yhat of 8 elements
        auto load8 = [&](int64_t v, float (&g)[8], float (&yh)[8]) {
            const uint4 w = xr[v], dw = dr[v];
            const uint4 sw = sc ? sc[v] : make_uint4(0, 0, 0, 0);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w}, dws[4] = {dw.x, dw.y, dw.z, dw.w},
                           sws[4] = {sw.x, sw.y, sw.z, sw.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                float xv[2], dv[2], sv[2];
                unpack2<DT>(ws[h], xv[0], xv[1]);
                unpack2<DT>(dws[h], dv[0], dv[1]);
                unpack2<DT>(sws[h], sv[0], sv[1]);
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float gg = dv[e];
                    if (sc) gg = round_act<DT>(__fmul_rn(gg, __fadd_rn(1.0f, sv[e])));
                    g[2 * h + e] = gg;
                    yh[2 * h + e] = __fdiv_rn(__fsub_rn(xv[e], st.x), st.y);
                }
            }
        };
        float s1 = 0.0f, s2 = 0.0f;
        for (int64_t v = lane; v < nv; v += 32) {
            float g[8], yh[8];
            load8(v, g, yh);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                s1 = __fadd_rn(s1, g[e]);
                s2 = __fadd_rn(s2, __fmul_rn(g[e], yh[e]));
            }
        }
        const float mg = __fdiv_rn(warp_sum_fixed(s1), (float)K);
        const float mgy = __fdiv_rn(warp_sum_fixed(s2), (float)K);
        uint4 *o = reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(dx) + m * K);
        for (int64_t v = lane; v < nv; v += 32) {
            float g[8], yh[8];
            load8(v, g, yh);
            uint32_t ow[4];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                float f[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const float t = __fsub_rn(__fsub_rn(g[2 * h + e], mg), __fmul_rn(yh[2 * h + e], mgy));
                    f[e] = __fdiv_rn(t, st.y);
                }
                ow[h] = Elem<DT>::pack2(f[0], f[1]);
            }
            o[v] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        }
    }
}

// dx per row; also the row's (mean, d) for the parameter reduction.
template <int DT>
__global__ void __launch_bounds__(LN_THREADS) ln_modulate_bwd_kernel(const void *x, const void *dout, int64_t M,
                                                                     int64_t K, int64_t tps, const void *scale,
                                                                     const void *lnw, float eps, void *dx,
                                                                     float2 *stats) {
    griddep_wait();
    extern __shared__ float row[];  // [K] x, then [K] g
    __shared__ float red[LN_THREADS / 32];
    using T = typename Elem<DT>::T;
    float *gr = row + K;
    for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
        const float2 st = ln_row_stats<DT>(x, m, K, eps, row, red);
        if (threadIdx.x == 0 && stats) stats[m] = st;
        const int64_t b = m / tps;
        const T *sc = scale ? reinterpret_cast<const T *>(scale) + b * K : nullptr;
        const T *dr = reinterpret_cast<const T *>(dout) + m * K;
        float s1 = 0.0f, s2 = 0.0f;
        for (int64_t k = threadIdx.x; k < K; k += LN_THREADS) {
            float g = Elem<DT>::to_f(dr[k]);
            if (sc) g = round_act<DT>(__fmul_rn(g, __fadd_rn(1.0f, Elem<DT>::to_f(sc[k]))));
            if (lnw) g = __fmul_rn(g, Elem<DT>::to_f(reinterpret_cast<const T *>(lnw)[k]));
            gr[k] = g;
            const float yh = __fdiv_rn(__fsub_rn(row[k], st.x), st.y);
            s1 = __fadd_rn(s1, g);
            s2 = __fadd_rn(s2, __fmul_rn(g, yh));
        }
        const float mg = __fdiv_rn(ln_block_sum(s1, red), (float)K);
        const float mgy = __fdiv_rn(ln_block_sum(s2, red), (float)K);
        T *o = reinterpret_cast<T *>(dx) + m * K;
        for (int64_t k = threadIdx.x; k < K; k += LN_THREADS) {
            const float yh = __fdiv_rn(__fsub_rn(row[k], st.x), st.y);
            const float t = __fsub_rn(__fsub_rn(gr[k], mg), __fmul_rn(yh, mgy));
            o[k] = Elem<DT>::from_f(__fdiv_rn(t, st.y));
        }
        __syncthreads();  // row/gr are rewritten by the next row
    }
}

// Partial sums over LN_COL_ROWS tokens of one sample: dscale = sum dout * ln,
// dshift = sum dout, into part[chunk][2][K] (chunk = sample-local row block).
template <int DT>
__global__ void __launch_bounds__(LN_THREADS) ln_param_partial_kernel(const void *x, const void *dout,
                                                                      const float2 *stats, int64_t M, int64_t K,
                                                                      int64_t tps, const void *lnw, const void *lnb,
                                                                      int64_t chunks_per_sample, float *part) {
    griddep_wait();
    using T = typename Elem<DT>::T;
    const int64_t k = (int64_t)blockIdx.x * LN_THREADS + threadIdx.x;
    const int64_t b = blockIdx.y / chunks_per_sample, c = blockIdx.y % chunks_per_sample;
    const int64_t m0 = b * tps + c * LN_COL_ROWS, m1 = min(min(m0 + LN_COL_ROWS, (b + 1) * tps), M);
    if (k >= K) return;
    float ds = 0.0f, dh = 0.0f;
#pragma unroll 4
    for (int64_t m = m0; m < m1; ++m) {
        const float2 st = __ldcg(&stats[m]);
        const float g = Elem<DT>::to_f(reinterpret_cast<const T *>(dout)[m * K + k]);
        const float ln = ln_value<DT>(Elem<DT>::to_f(reinterpret_cast<const T *>(x)[m * K + k]), st.x, st.y, lnw, lnb, k);
        ds = __fadd_rn(ds, __fmul_rn(g, ln));
        dh = __fadd_rn(dh, g);
    }
    float *p = part + (int64_t)blockIdx.y * 2 * K;
    p[k] = ds;
    p[K + k] = dh;
}

// dscale[b][k] (+)= sum over the sample's chunks, in chunk order; same for dshift.
__global__ void ln_param_final_kernel(const float *part, int64_t K, int64_t batch, int64_t chunks_per_sample,
                                      int accumulate, float *dscale, float *dshift) {
    griddep_wait();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < batch * K; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / K, k = i % K;
        float ds = 0.0f, dh = 0.0f;
        for (int64_t c = 0; c < chunks_per_sample; ++c) {
            const float *p = part + (b * chunks_per_sample + c) * 2 * K;
            ds = __fadd_rn(ds, __ldcg(p + k));
            dh = __fadd_rn(dh, __ldcg(p + K + k));
        }
        if (dscale) dscale[i] = accumulate ? __fadd_rn(dscale[i], ds) : ds;
        if (dshift) dshift[i] = accumulate ? __fadd_rn(dshift[i], dh) : dh;
    }
}

}  // namespace reels

namespace reels {

// The gated residual after a block's output projection,
//   out = mixed_add(x, mixed_mul(y, gate[b]))       (transformer.jl:272,293)
// = round(x + round(y * gate[b])) per element, b = token / tokens_per_sample,
// in one pass (the reference's two broadcasts write an intermediate).  out may
// be x itself.  Its pullback: dx = dout; dy = round(dout * gate[b]) (the
// product's pullback); dgate[b] = sum over the sample's tokens of dout * y.
// 16-bit types with N % 8 == 0 and 16-byte aligned pointers: eight elements
// of one row per 16-byte access.
template <int DT>
__device__ __forceinline__ bool gr_vec(int64_t N, const void *a, const void *b, const void *c, const void *d) {
    return DT != DT_F32 && (N & 7) == 0 &&
           ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c) |
             reinterpret_cast<uintptr_t>(d)) & 15) == 0;
}

template <int DT>
__global__ void gated_residual_kernel(const void *x, const void *y, const void *gate, int64_t M, int64_t N,
                                      int64_t tps, void *out) {
    griddep_wait();
    using T = typename Elem<DT>::T;
    const T *xp = reinterpret_cast<const T *>(x);
    const T *yp = reinterpret_cast<const T *>(y);
    const T *gp = reinterpret_cast<const T *>(gate);
    T *op = reinterpret_cast<T *>(out);
    if constexpr (DT != DT_F32) {
        if (gr_vec<DT>(N, x, y, gate, out)) {
            const int64_t nv = M * N / 8, rowv = N / 8;
            for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
                const int64_t m = v / rowv, nb = v - m * rowv;
                const uint4 xw = reinterpret_cast<const uint4 *>(xp)[v], yw = reinterpret_cast<const uint4 *>(yp)[v];
                const uint4 gw = reinterpret_cast<const uint4 *>(gp + (m / tps) * N)[nb];
                const uint32_t xs[4] = {xw.x, xw.y, xw.z, xw.w}, ys[4] = {yw.x, yw.y, yw.z, yw.w},
                               gs[4] = {gw.x, gw.y, gw.z, gw.w};
                uint32_t os[4];
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    float x0, x1, y0, y1, g0, g1;
                    unpack2<DT>(xs[h], x0, x1);
                    unpack2<DT>(ys[h], y0, y1);
                    unpack2<DT>(gs[h], g0, g1);
                    os[h] = Elem<DT>::pack2(__fadd_rn(x0, round_act<DT>(__fmul_rn(y0, g0))),
                                            __fadd_rn(x1, round_act<DT>(__fmul_rn(y1, g1))));
                }
                reinterpret_cast<uint4 *>(op)[v] = make_uint4(os[0], os[1], os[2], os[3]);
            }
            return;
        }
    }
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M * N; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / N, n = i - m * N;
        const float prod = round_act<DT>(__fmul_rn(Elem<DT>::to_f(yp[i]), Elem<DT>::to_f(gp[(m / tps) * N + n])));
        op[i] = Elem<DT>::from_f(__fadd_rn(Elem<DT>::to_f(xp[i]), prod));
    }
}

template <int DT>
__global__ void gated_residual_dy_kernel(const void *dout, const void *gate, int64_t M, int64_t N, int64_t tps,
                                         void *dy) {
    griddep_wait();
    using T = typename Elem<DT>::T;
    const T *dp = reinterpret_cast<const T *>(dout);
    const T *gp = reinterpret_cast<const T *>(gate);
    T *o = reinterpret_cast<T *>(dy);
    if constexpr (DT != DT_F32) {
        if (gr_vec<DT>(N, dout, gate, dy, dy)) {
            const int64_t nv = M * N / 8, rowv = N / 8;
            for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
                const int64_t m = v / rowv, nb = v - m * rowv;
                const uint4 dw = reinterpret_cast<const uint4 *>(dp)[v];
                const uint4 gw = reinterpret_cast<const uint4 *>(gp + (m / tps) * N)[nb];
                const uint32_t ds[4] = {dw.x, dw.y, dw.z, dw.w}, gs[4] = {gw.x, gw.y, gw.z, gw.w};
                uint32_t os[4];
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    float d0, d1, g0, g1;
                    unpack2<DT>(ds[h], d0, d1);
                    unpack2<DT>(gs[h], g0, g1);
                    os[h] = Elem<DT>::pack2(__fmul_rn(d0, g0), __fmul_rn(d1, g1));
                }
                reinterpret_cast<uint4 *>(o)[v] = make_uint4(os[0], os[1], os[2], os[3]);
            }
            return;
        }
    }
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M * N; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / N, n = i - m * N;
        o[i] = Elem<DT>::from_f(__fmul_rn(Elem<DT>::to_f(dp[i]), Elem<DT>::to_f(gp[(m / tps) * N + n])));
    }
}

// Partial sums over LN_COL_ROWS tokens of one sample of dout * y, into
// part[chunk][N]; then the same final reduction as the modulation's.
template <int DT>
__global__ void __launch_bounds__(LN_THREADS) gate_grad_partial_kernel(const void *dout, const void *y, int64_t M,
                                                                       int64_t N, int64_t tps,
                                                                       int64_t chunks_per_sample, float *part) {
    griddep_wait();
    using T = typename Elem<DT>::T;
    const int64_t n = (int64_t)blockIdx.x * LN_THREADS + threadIdx.x;
    const int64_t b = blockIdx.y / chunks_per_sample, c = blockIdx.y % chunks_per_sample;
    const int64_t m0 = b * tps + c * LN_COL_ROWS, m1 = min(min(m0 + LN_COL_ROWS, (b + 1) * tps), M);
    if (n >= N) return;
    float acc = 0.0f;
    for (int64_t m = m0; m < m1; ++m)
        acc = __fadd_rn(acc, __fmul_rn(Elem<DT>::to_f(reinterpret_cast<const T *>(dout)[m * N + n]),
                                       Elem<DT>::to_f(reinterpret_cast<const T *>(y)[m * N + n])));
    part[(int64_t)blockIdx.y * N + n] = acc;
}

__global__ void gate_grad_final_kernel(const float *part, int64_t N, int64_t batch, int64_t chunks_per_sample,
                                       int accumulate, float *dgate) {
    griddep_wait();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < batch * N; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / N, n = i % N;
        float acc = 0.0f;
        for (int64_t c = 0; c < chunks_per_sample; ++c) acc = __fadd_rn(acc, __ldcg(part + (b * chunks_per_sample + c) * N + n));
        dgate[i] = accumulate ? __fadd_rn(dgate[i], acc) : acc;
    }
}

}  // namespace reels
