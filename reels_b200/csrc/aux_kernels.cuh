// Memory-bound helper kernels: the bit-exact quantiser, weight
// materialisation, the rank-r transpose, split-K reductions, and the
// CUDA-core "generic" path that serves shapes and dtypes the tensor-core
// path does not take (ragged feature sizes, fp32 activations).
#pragma once
#include "act.cuh"
#include "common.cuh"

namespace reels {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// ----------------------------------------------------------- quantiser
// src/layers/quantization.jl:35-44, per output row n:
//   m = max_k |w[n,k]| (fp32),  s = m / 127 (IEEE),  s = 1 if m == 0,
//   q = Int8(round(clamp(w / s, -127, 127)))   with round = ties-to-even.
// Only m == 0 is replaced, so a row whose m is at most 63 * 2^-149 gets s = 0
// (m / 127 underflows).  Its nonzero elements divide to +-Inf and clamp to
// +-127; a zero element gives 0 / 0 = NaN, which Julia's clamp passes through
// and Int8(NaN) rejects with InexactError.  The kernels flag that NaN
// (DEVERR_QUANT_NAN) instead of clamping it: fminf/fmaxf would turn it into
// a number.
// Layout 0 (Julia (out, in) column-major): w[k*N + n].  One block handles
// 32 consecutive rows n (one per lane, coalesced along n); its 8 warps split
// the k range and combine maxima in shared memory.
template <typename T>
__global__ void __launch_bounds__(256) quantize_outcontig_kernel(const T *__restrict__ w, int64_t N, int64_t K,
                                                                 int8_t *__restrict__ q, float *__restrict__ scales,
                                                                 unsigned *err) {
    __shared__ float smax[8][32];
    __shared__ float sscale[32];
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
    const int64_t n = (int64_t)blockIdx.x * 32 + lane;
    float m = 0.0f;
    bool bad = false;
    if (n < N) {
        for (int64_t k = wp; k < K; k += 8) {
            float v = to_f32(w[k * N + n]);
            bad |= !isfinite(v);
            m = fmaxf(m, fabsf(v));
        }
    }
    smax[wp][lane] = m;
    __syncthreads();
    if (wp == 0) {
        float mm = smax[0][lane];
        for (int i = 1; i < 8; ++i) mm = fmaxf(mm, smax[i][lane]);
        const float s = (mm == 0.0f) ? 1.0f : __fdiv_rn(mm, 127.0f);
        sscale[lane] = s;
        if (n < N) scales[n] = s;
    }
    if (bad) atomicOr(err, DEVERR_NONFINITE_WEIGHT);
    __syncthreads();
    if (n < N) {
        const float s = sscale[lane];
        bool nan = false;
        for (int64_t k = wp; k < K; k += 8) {
            float t = __fdiv_rn(to_f32(w[k * N + n]), s);
            nan |= isnan(t);
            t = fminf(fmaxf(t, -127.0f), 127.0f);
            q[k * N + n] = (int8_t)__float2int_rn(t);
        }
        if (nan) atomicOr(err, DEVERR_QUANT_NAN);
    }
}

// Layout 1 (PyTorch nn.Linear): w[n*K + k]; one warp per row.
template <typename T>
__global__ void __launch_bounds__(256) quantize_incontig_kernel(const T *__restrict__ w, int64_t N, int64_t K,
                                                                int8_t *__restrict__ q, float *__restrict__ scales,
                                                                unsigned *err) {
    const int lane = threadIdx.x & 31;
    const int64_t n = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (n >= N) return;
    const T *row = w + n * K;
    float m = 0.0f;
    bool bad = false;
    for (int64_t k = lane; k < K; k += 32) {
        float v = to_f32(row[k]);
        bad |= !isfinite(v);
        m = fmaxf(m, fabsf(v));
    }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(err, DEVERR_NONFINITE_WEIGHT);
    const float s = (m == 0.0f) ? 1.0f : __fdiv_rn(m, 127.0f);
    if (lane == 0) scales[n] = s;
    int8_t *qr = q + n * K;
    bool nan = false;
    for (int64_t k = lane; k < K; k += 32) {
        float t = __fdiv_rn(to_f32(row[k]), s);
        nan |= isnan(t);
        t = fminf(fmaxf(t, -127.0f), 127.0f);
        qr[k] = (int8_t)__float2int_rn(t);
    }
    if (__any_sync(0xffffffffu, nan) && lane == 0) atomicOr(err, DEVERR_QUANT_NAN);
}

// ------------------------------------------------------- materialise
// quantization.jl:54-64: fp16 -> Float16(q) * Float16(s) rounded to fp16;
// fp32 -> Float32(q) * s; bf16 (not offered by the reference) -> the fp32
// product rounded once to bf16, the rule of interface.jl:19-25.
__global__ void materialize_kernel(const int8_t *__restrict__ q, const float *__restrict__ scales, int layout,
                                   int64_t N, int64_t K, int out_dt, void *out) {
    const int64_t total = N * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = (layout == 0) ? (i % N) : (i / K);
        const float s = scales[n];
        const float qv = (float)q[i];
        if (out_dt == DT_F16) {
            reinterpret_cast<__half *>(out)[i] = __hmul(__float2half_rn(qv), __float2half_rn(s));
        } else if (out_dt == DT_BF16) {
            reinterpret_cast<__nv_bfloat16 *>(out)[i] = __float2bfloat16_rn(qv * s);
        } else {
            reinterpret_cast<float *>(out)[i] = qv * s;
        }
    }
}

// A [K][r] -> At [r][K] (same element type, 2 bytes).  K * r < 2^31.
__global__ void transpose_rank_kernel(const uint16_t *a, int K, int r, uint16_t *__restrict__ at) {
    griddep_wait();
    const int total = K * r;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int j = i / K, k = i - j * K;
        at[i] = a[k * r + j];
    }
}

// -------------------------------------------------- split-K reductions
// The output epilogue of one element: value v (column scale and bias applied),
// optionally through gelu_tanh (writing the rounded pre-activation) or its
// derivative (reading it); see act.cuh.
__device__ __forceinline__ void epilogue_value(float v, int act, int dt, void *out, void *pre, int64_t idx) {
    if (act == ACT_GELU_TANH) {
        store_act(out, idx, dt, v);
        const float h = load_act(out, idx, dt);  // the rounded pre-activation
        if (pre) store_act(pre, idx, dt, h);
        store_act(out, idx, dt, gelu_tanh_f32(h));
    } else if (act == ACT_GELU_TANH_GRAD) {
        store_act(out, idx, dt, v);
        store_act(out, idx, dt, load_act(out, idx, dt) * gelu_tanh_grad_f32(load_act(pre, idx, dt)));
    } else {
        store_act(out, idx, dt, v);
    }
}

// Sum q8 partials [splits][M][Nout] and apply the output epilogue.  Four
// consecutive columns per thread (Nout is a multiple of 16 on the tensor-core
// path), 16-byte loads, the split loop unrolled so its loads are in flight
// together; the sum runs over s = 0 .. splits-1 in order.
__global__ void q8_reduce_kernel(const float *partial, int splits, int64_t M, int64_t Nout,
                                 const float *col_scale, const void *bias, int dt, void *out,
                                 int64_t ldo, int act, void *pre) {
    griddep_wait();
    const int64_t total4 = M * Nout / 4;
    const float4 *p4 = reinterpret_cast<const float4 *>(partial);
    for (int64_t i4 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i4 < total4;
         i4 += (int64_t)gridDim.x * blockDim.x) {
        float4 acc = __ldcg(p4 + i4);
#pragma unroll 4
        for (int s = 1; s < splits; ++s) {
            const float4 v = __ldcg(p4 + (int64_t)s * total4 + i4);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        const int64_t i = i4 * 4, row = i / Nout, col = i % Nout;
        float a[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (col_scale) a[u] *= col_scale[col + u];
            if (bias) a[u] += load_act(bias, col + u, dt);
            epilogue_value(a[u], act, dt, out, pre, row * ldo + col + u);
        }
    }
}

// Sum skinny partials [splits][rows][npad] and apply epi 0 (transposed
// store, act dtype) or epi 1 (fp32 accumulate into out[row*rs + j*cs]).
// The outputs are few and the splits many, so the sum is latency-bound: four
// threads share an output, thread t of the four adds the splits s = t mod 4
// in order with eight loads in flight, and the four partial sums are
// combined in a fixed order (deterministic from run to run).
// pcol selects the partials' layout and the order of the outputs, so that
// both follow the output's contiguous dimension: pcol = 0, partials
// [splits][rows][npad] and consecutive outputs are consecutive columns j of a
// row (out[row*rs + j] with cs = 1); pcol = 1, partials [splits][npad][rows]
// and consecutive outputs are consecutive rows (the transposed store
// out[j*ldo + row], or out[row + j*cs] with rs = 1).
// With few splits (vec = 1: pcol layout, rows % 4 == 0, 16-byte aligned
// output) a lane instead owns four consecutive outputs, adds the splits in
// order with float4 loads and writes the four results at once: a warp covers
// 128 outputs per step instead of eight.
// One launch sums one or two such jobs (G and dB of the one-pass dy kernel):
// the warps take the first job's groups of outputs, then the second's.
struct RedJob {
    const float *partial;
    int splits;
    int64_t rows;
    int npad, ncols, epi;
    float alpha;
    int accumulate;
    void *out;
    int64_t ldo, rs, cs;
    int pcol;
    int vec;
};

constexpr int RED_VEC_MAX = 8;  // most splits of the vector path

__device__ __forceinline__ int64_t red_groups(const RedJob &J) {
    const int64_t total = J.rows * (int64_t)J.ncols;
    return J.vec ? (total + 127) / 128 : (total + 7) / 8;
}

__device__ __forceinline__ void reduce_group_vec(const RedJob &J, int64_t w, int lane, int dt) {
    const int64_t o = w * 128 + 4 * lane;  // four consecutive rows of one column j
    if (o >= J.rows * (int64_t)J.ncols) return;
    const int64_t j = o / J.rows, row = o % J.rows;
    const int64_t stride = J.rows * (int64_t)J.npad;
    const float *p = J.partial + j * J.rows + row;
    float4 v[RED_VEC_MAX];
#pragma unroll
    for (int s = 0; s < RED_VEC_MAX; ++s)  // every load in flight, then the sum in split order
        if (s < J.splits) v[s] = __ldcg(reinterpret_cast<const float4 *>(p + (int64_t)s * stride));
    float4 acc = v[0];
#pragma unroll
    for (int s = 1; s < RED_VEC_MAX; ++s) {
        if (s < J.splits) {
            acc.x += v[s].x;
            acc.y += v[s].y;
            acc.z += v[s].z;
            acc.w += v[s].w;
        }
    }
    if (J.epi == 0) {
        const int64_t idx = j * J.ldo + row;
        if (dt == DT_BF16) {
            *reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(J.out) + idx) =
                make_uint2(Elem<DT_BF16>::pack2(J.alpha * acc.x, J.alpha * acc.y),
                           Elem<DT_BF16>::pack2(J.alpha * acc.z, J.alpha * acc.w));
        } else {
            *reinterpret_cast<uint2 *>(reinterpret_cast<__half *>(J.out) + idx) =
                make_uint2(Elem<DT_F16>::pack2(J.alpha * acc.x, J.alpha * acc.y),
                           Elem<DT_F16>::pack2(J.alpha * acc.z, J.alpha * acc.w));
        }
    } else {
        float4 *o4 = reinterpret_cast<float4 *>(reinterpret_cast<float *>(J.out) + row + j * J.cs);
        float4 prev = J.accumulate ? *o4 : make_float4(0.f, 0.f, 0.f, 0.f);
        prev.x += J.alpha * acc.x;
        prev.y += J.alpha * acc.y;
        prev.z += J.alpha * acc.z;
        prev.w += J.alpha * acc.w;
        *o4 = prev;
    }
}

__device__ __forceinline__ void reduce_group(const RedJob &J, int64_t w, int lane, int dt) {
    const int sl = lane & 3;
    const int64_t total = J.rows * (int64_t)J.ncols;
    const int64_t stride = J.rows * (int64_t)J.npad;
    const int64_t o = w * 8 + (lane >> 2);  // eight consecutive outputs per warp
    float acc = 0.0f;
    int64_t row = 0, j = 0;
    if (o < total) {
        if (J.pcol) {
            j = o / J.rows;
            row = o % J.rows;
        } else {
            row = o / J.ncols;
            j = o % J.ncols;
        }
        const float *p = J.pcol ? J.partial + j * J.rows + row : J.partial + row * J.npad + j;
        int s = sl;
        for (; s + 28 < J.splits; s += 32) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = __ldcg(p + (int64_t)(s + 4 * u) * stride);
#pragma unroll
            for (int u = 0; u < 8; ++u) acc += v[u];
        }
        for (; s < J.splits; s += 4) acc += __ldcg(p + (int64_t)s * stride);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (sl == 0 && o < total) {
        if (J.epi == 0) {
            store_act(J.out, j * J.ldo + row, dt, J.alpha * acc);
        } else {
            float *o32 = reinterpret_cast<float *>(J.out);
            const int64_t idx = row * J.rs + j * J.cs;
            o32[idx] = (J.accumulate ? o32[idx] : 0.0f) + J.alpha * acc;
        }
    }
}

__global__ void sk_reduce_kernel(const RedJob j0, const RedJob j1, int njobs, int dt) {
    griddep_wait();
    const int lane = threadIdx.x & 31;
    const int64_t g0 = red_groups(j0);
    const int64_t g1 = njobs > 1 ? red_groups(j1) : 0;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < g0 + g1; w += nw) {
        const RedJob &J = w < g0 ? j0 : j1;
        const int64_t wl = w < g0 ? w : w - g0;
        if (J.vec) reduce_group_vec(J, wl, lane, dt);
        else reduce_group(J, wl, lane, dt);
    }
}

// The fused activation as a separate pass, for the kernels without it in
// their epilogue: gelu reads the GEMM output from `pre` and writes `out`;
// the gradient rescales `out` in place by gelu'(pre).
__global__ void act_apply_kernel(int act, int dt, int64_t total, void *out, const void *pre) {
    griddep_wait();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float h = load_act(pre, i, dt);
        if (act == ACT_GELU_TANH) store_act(out, i, dt, gelu_tanh_f32(h));
        else store_act(out, i, dt, load_act(out, i, dt) * gelu_tanh_grad_f32(h));
    }
}

// ------------------------------------------------- generic (CUDA cores)
// One thread per output element, fp32 accumulation, any shape.  Weight
// element (n, k) is dequantised as fp32(q) * s[n] (quantization.jl:63-64).
__device__ __forceinline__ float wdq(const int8_t *q, const float *s, int layout, int64_t N, int64_t K, int64_t n,
                                     int64_t k) {
    const int64_t idx = (layout == 0) ? (k * N + n) : (n * K + k);
    return (float)q[idx] * s[n];
}

// T[j][m] (act dtype, pitch ldt) = sum_k X[m][k] * A[k][j]
__global__ void gen_rank_down_kernel(const void *x, const void *a, int64_t M, int64_t K, int r, int dt, void *t,
                                     int64_t ldt) {
    const int64_t total = M * (int64_t)r;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i / M, m = i % M;
        float acc = 0.0f;
        for (int64_t k = 0; k < K; ++k) acc += load_act(x, m * K + k, dt) * load_act(a, k * r + j, dt);
        store_act(t, j * ldt + m, dt, acc);
    }
}

// G[j][m] (act dtype) = alpha * sum_n dY[m][n] * B[j][n]
__global__ void gen_rank_grad_kernel(const void *dy, const void *b, int64_t M, int64_t N, int r, float alpha, int dt,
                                     void *g, int64_t ldg) {
    const int64_t total = M * (int64_t)r;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i / M, m = i % M;
        float acc = 0.0f;
        for (int64_t n = 0; n < N; ++n) acc += load_act(dy, m * N + n, dt) * load_act(b, j * N + n, dt);
        store_act(g, j * ldg + m, dt, alpha * acc);
    }
}

// Y[m][n] = sum_k X[m][k] Wdq(n,k) + bias[n] + s * sum_j T[j][m] B[j][n]
__global__ void gen_forward_kernel(const void *x, const int8_t *q, const float *sc, int layout, const void *bias,
                                   const void *t, int64_t ldt, const void *b, int64_t M, int64_t K, int64_t N, int r,
                                   float s, int dt, void *y) {
    const int64_t total = M * N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / N, n = i % N;
        float acc = 0.0f;
        for (int64_t k = 0; k < K; ++k) acc += load_act(x, m * K + k, dt) * wdq(q, sc, layout, N, K, n, k);
        if (bias) acc += load_act(bias, n, dt);
        float lora = 0.0f;
        for (int j = 0; j < r; ++j) lora += load_act(t, j * ldt + m, dt) * load_act(b, (int64_t)j * N + n, dt);
        store_act(y, i, dt, acc + s * lora);
    }
}

// dX[m][k] = sum_n dY[m][n] Wdq(n,k) + sum_j G[j][m] A[k][j]   (G already * s)
__global__ void gen_dx_kernel(const void *dy, const int8_t *q, const float *sc, int layout, const void *g,
                              int64_t ldg, const void *a, int64_t M, int64_t K, int64_t N, int r, int dt, void *dx) {
    const int64_t total = M * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / K, k = i % K;
        float acc = 0.0f;
        for (int64_t n = 0; n < N; ++n) acc += load_act(dy, m * N + n, dt) * wdq(q, sc, layout, N, K, n, k);
        float lora = 0.0f;
        for (int j = 0; j < r; ++j) lora += load_act(g, j * ldg + m, dt) * load_act(a, k * r + j, dt);
        store_act(dx, i, dt, acc + lora);
    }
}

// dA[k][j] = beta*dA + alpha * sum_m G[j][m] X[m][k]
__global__ void gen_da_kernel(const void *g, int64_t ldg, const void *x, int64_t M, int64_t K, int r, float alpha,
                              int accumulate, int dt, float *da) {
    const int64_t total = K * (int64_t)r;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t k = i / r, j = i % r;
        float acc = 0.0f;
        for (int64_t m = 0; m < M; ++m) acc += load_act(g, j * ldg + m, dt) * load_act(x, m * K + k, dt);
        da[i] = (accumulate ? da[i] : 0.0f) + alpha * acc;
    }
}

// dB[j][n] = beta*dB + alpha * sum_m dY[m][n] T[j][m]
__global__ void gen_db_kernel(const void *dy, const void *t, int64_t ldt, int64_t M, int64_t N, int r, float alpha,
                              int accumulate, int dt, float *db) {
    const int64_t total = N * (int64_t)r;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i / N, n = i % N;
        float acc = 0.0f;
        for (int64_t m = 0; m < M; ++m) acc += load_act(dy, m * N + n, dt) * load_act(t, j * ldt + m, dt);
        db[i] = (accumulate ? db[i] : 0.0f) + alpha * acc;
    }
}

}  // namespace reels
