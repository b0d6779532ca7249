/*
 * CPU oracle for the Int8-weight LoRA linear (TEST INFRASTRUCTURE ONLY).
 *
 * This file restates, in plain C, the arithmetic of Reels.jl's quantised LoRA
 * linear so that the CUDA path can be checked against it.  It is linked only by
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, never by the
 * product library.
 *
 * Layout convention (matches the reference's column-major, feature-first
 * arrays, written here as row-major C arrays):
 *   X  [M][K]   activations  (Julia `x`  is (in, tokens))
 *   Y  [M][N]   outputs      (Julia `y`  is (out, tokens))
 *   W  [K][N]   "out-contiguous" (Julia weight (out, in))      layout 0
 *      [N][K]   "in-contiguous"  (PyTorch nn.Linear weight)     layout 1
 *   A  [K][r]   (Julia A is (rank, in))
 *   B  [r][N]   (Julia B is (out, rank))
 *   scales[N]   one fp32 scale per output row of the weight
 *
 * Parity status: the reference is Julia, which is not installed here, so no
 * reference output could be generated.  The quantiser is pinned by hand-derived
 * known answers (exact scales, ties-to-even), the linear algebra by the
 * reference test properties (B = 0 identity, merged weight, finite
 * differences).  Against reference-produced vectors parity is UNPINNED.
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <stdlib.h>

#define OIDX_W(layout, n, k, N, K) ((layout) == 0 ? ((int64_t)(k) * (N) + (n)) : ((int64_t)(n) * (K) + (k)))

/* quantization.jl:35-44 `quantize_frozen_matrix`:
 *   maxima = maximum(abs, host; dims=2)       (fp32, per output row)
 *   scales = maxima ./ 127f0                  (IEEE fp32 division)
 *   scales[maxima .== 0f0] .= 1f0
 *   values = Int8.(round.(clamp.(host ./ scales, -127f0, 127f0)))
 * Julia's `round` is RoundNearest (ties to even); `rintf` under the default
 * FE_TONEAREST mode is the same rule.  Julia's clamp is
 * ifelse(x > hi, hi, ifelse(x < lo, lo, x)), so a NaN quotient passes through
 * and Int8(NaN) raises InexactError.  Two inputs reach that:
 *   - a non-finite weight (max or quotient NaN): returns -1;
 *   - a row whose maximum m is nonzero but m/127 rounds to 0 (m <= 63*2^-149;
 *     only m == 0 is replaced by 1) and which holds a zero element: 0/0 = NaN.
 *     Returns -2.  The row's nonzero elements divide to +-Inf and clamp to
 *     +-127, so a row without zeros quantises with scale 0.
 * NaN is never cast to an integer (that is undefined behaviour in C). */
int oracle_quantize(const float *w, int layout, int64_t N, int64_t K, int8_t *q, float *scales)
{
    int bad = 0, nan_quotient = 0;
    for (int64_t n = 0; n < N; ++n) {
        float m = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            float v = w[OIDX_W(layout, n, k, N, K)];
            if (!isfinite(v)) bad = 1;
            float a = fabsf(v);
            if (a > m) m = a;
        }
        volatile float s = m / 127.0f;          /* keep the IEEE division */
        float sc = (m == 0.0f) ? 1.0f : s;
        scales[n] = sc;
        for (int64_t k = 0; k < K; ++k) {
            int64_t i = OIDX_W(layout, n, k, N, K);
            volatile float t = w[i] / sc;
            float c = t;
            if (c > 127.0f) c = 127.0f;
            if (c < -127.0f) c = -127.0f;
            if (isnan(c)) {
                if (isfinite(w[i])) nan_quotient = 1;
                q[i] = 0;
                continue;
            }
            q[i] = (int8_t)(int)rintf(c);
        }
    }
    return bad ? -1 : (nan_quotient ? -2 : 0);
}

/* quantization.jl:63-64 `_dequantize_for_compute(values, scales, Float32)`:
 * Float32.(values) .* Float32.(scales), written in the weight's own layout. */
void oracle_dequantize_f32(const int8_t *q, const float *scales, int layout, int64_t N, int64_t K, float *out)
{
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k) {
            int64_t i = OIDX_W(layout, n, k, N, K);
            out[i] = (float)q[i] * scales[n];
        }
}

/* quantization.jl:61-62 `_dequantize_for_compute(values, scales, Float16)`:
 * Float16.(values) .* Float16.(scales); the product is rounded to fp16.
 * Output is the fp16 bit pattern. */
void oracle_dequantize_f16(const int8_t *q, const float *scales, int layout, int64_t N, int64_t K, uint16_t *out)
{
    for (int64_t n = 0; n < N; ++n) {
        _Float16 s = (_Float16)scales[n];
        for (int64_t k = 0; k < K; ++k) {
            int64_t i = OIDX_W(layout, n, k, N, K);
            _Float16 v = (_Float16)(float)q[i];
            _Float16 p = v * s;
            memcpy(&out[i], &p, 2);
        }
    }
}

/* interface.jl:19-25 `bfloat16_values`: round fp32 to bf16 with
 * (bits + 0x7fff + ((bits >> 16) & 1)) >> 16. */
uint16_t oracle_bf16_from_f32(float x)
{
    uint32_t b;
    memcpy(&b, &x, 4);
    b = b + 0x7fffu + ((b >> 16) & 1u);
    return (uint16_t)(b >> 16);
}

/* interface.jl:13-17 `float32_values`: bf16 bits << 16. */
float oracle_f32_from_bf16(uint16_t h)
{
    uint32_t b = (uint32_t)h << 16;
    float x;
    memcpy(&x, &b, 4);
    return x;
}

void oracle_bf16_round_array(const float *x, int64_t n, uint16_t *out)
{
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_bf16_from_f32(x[i]);
}

void oracle_bf16_materialise_array(const int8_t *q, const float *scales, int layout, int64_t N, int64_t K, uint16_t *out)
{
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k) {
            int64_t i = OIDX_W(layout, n, k, N, K);
            out[i] = oracle_bf16_from_f32((float)q[i] * scales[n]);
        }
}

/* Forward, lora.jl:56-95 with training=false / dropout 0, on the fp32
 * dequantised weight Wdq = Float32(q) * scale (quantization.jl:63-64):
 *   y  = Wdq * x            (quantization.jl:73-74)
 *   y += bias               (lora.jl:64-67, mixed_add)
 *   T  = A * x              (lora.jl:86, inner product)
 *   y += (alpha/r) * B * T  (lora.jl:86-94)
 * Inputs are fp32 (bf16/fp16 inputs are widened exactly by the caller);
 * accumulation is fp64, the result is rounded once to fp32.
 * T_out (nullable) receives T as [M][r]. */
/* Z (nullable): the adapter's input when it differs from X (LoRA dropout,
 * lora.jl:71-85): T = A * Z, the frozen weight still multiplies X. */
void oracle_lora_forward_z(const float *X, const float *Z, const int8_t *q, const float *scales, int layout,
                           const float *A, const float *B, const float *bias,
                           int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                           float *Y, float *T_out)
{
    double s = r > 0 ? (double)(alpha / (float)r) : 0.0;  /* r = 0: no adapter */
    double *T = (double *)malloc(sizeof(double) * (size_t)(M * (r > 0 ? r : 1)));
    float *Wd = (float *)malloc(sizeof(float) * (size_t)(N * K));
    oracle_dequantize_f32(q, scales, layout, N, K, Wd);
    #pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        const float *x = X + m * K;
        const float *z = (Z ? Z : X) + m * K;
        for (int64_t j = 0; j < r; ++j) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; ++k) acc += (double)z[k] * (double)A[k * r + j];
            T[m * r + j] = acc;
            if (T_out) T_out[m * r + j] = (float)acc;
        }
        for (int64_t n = 0; n < N; ++n) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; ++k)
                acc += (double)x[k] * (double)Wd[OIDX_W(layout, n, k, N, K)];
            if (bias) acc += (double)bias[n];
            double lora = 0.0;
            for (int64_t j = 0; j < r; ++j) lora += T[m * r + j] * (double)B[j * N + n];
            Y[m * N + n] = (float)(acc + s * lora);
        }
    }
    free(Wd);
    free(T);
}

void oracle_lora_forward(const float *X, const int8_t *q, const float *scales, int layout,
                         const float *A, const float *B, const float *bias,
                         int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                         float *Y, float *T_out)
{
    oracle_lora_forward_z(X, NULL, q, scales, layout, A, B, bias, M, K, N, r, alpha, Y, T_out);
}

/* Backward, lora.jl:106-118 (identical to Zygote's pullback of lora_forward
 * through the rrule at ad_rules.jl:70-80):
 *   ax = A * x
 *   dA = s * (B' * dy) * x'           -> [K][r] here (Julia (r, in))
 *   dB = s * dy * ax'                 -> [r][N] here (Julia (out, r))
 *   dx = Wdq' * dy + s * A' * (B' * dy)
 * fp64 accumulation, fp32 results.  Any of dX, dA, dB may be NULL. */
/* With LoRA dropout the adapter saw Z = X * keep / (1 - p): T = A * Z,
 * dA = s * G * Z', and the adapter's part of dX is scaled per element by
 * dscale = keep / (1 - p) ([M][K]).  Z and dscale NULL: no dropout. */
void oracle_lora_backward_z(const float *X, const float *Z, const float *dscale, const float *dY, const int8_t *q,
                            const float *scales, int layout, const float *A, const float *B,
                            int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                            float *dX, float *dA, float *dB)
{
    if (!Z) Z = X;
    double s = r > 0 ? (double)(alpha / (float)r) : 0.0;  /* r = 0: no adapter */
    double *G = (double *)malloc(sizeof(double) * (size_t)(M * (r > 0 ? r : 1)));
    double *T = (double *)malloc(sizeof(double) * (size_t)(M * (r > 0 ? r : 1)));
    float *Wd = (float *)malloc(sizeof(float) * (size_t)(N * K));
    oracle_dequantize_f32(q, scales, layout, N, K, Wd);
    #pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t j = 0; j < r; ++j) {
            double g = 0.0, t = 0.0;
            for (int64_t n = 0; n < N; ++n) g += (double)dY[m * N + n] * (double)B[j * N + n];
            for (int64_t k = 0; k < K; ++k) t += (double)Z[m * K + k] * (double)A[k * r + j];
            G[m * r + j] = g;
            T[m * r + j] = t;
        }
    }
    if (dX) {
        #pragma omp parallel for schedule(static)
        for (int64_t m = 0; m < M; ++m) {
            for (int64_t k = 0; k < K; ++k) {
                double acc = 0.0;
                for (int64_t n = 0; n < N; ++n)
                    acc += (double)dY[m * N + n] * (double)Wd[OIDX_W(layout, n, k, N, K)];
                double lora = 0.0;
                for (int64_t j = 0; j < r; ++j) lora += (double)A[k * r + j] * G[m * r + j];
                if (dscale) lora *= (double)dscale[m * K + k];
                dX[m * K + k] = (float)(acc + s * lora);
            }
        }
    }
    if (dA) {
        #pragma omp parallel for schedule(static)
        for (int64_t k = 0; k < K; ++k)
            for (int64_t j = 0; j < r; ++j) {
                double acc = 0.0;
                for (int64_t m = 0; m < M; ++m) acc += G[m * r + j] * (double)Z[m * K + k];
                dA[k * r + j] = (float)(s * acc);
            }
    }
    if (dB) {
        #pragma omp parallel for schedule(static)
        for (int64_t n = 0; n < N; ++n)
            for (int64_t j = 0; j < r; ++j) {
                double acc = 0.0;
                for (int64_t m = 0; m < M; ++m) acc += (double)dY[m * N + n] * T[m * r + j];
                dB[j * N + n] = (float)(s * acc);
            }
    }
    free(Wd);
    free(T);
    free(G);
}

void oracle_lora_backward(const float *X, const float *dY, const int8_t *q, const float *scales, int layout,
                          const float *A, const float *B,
                          int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                          float *dX, float *dA, float *dB)
{
    oracle_lora_backward_z(X, NULL, NULL, dY, q, scales, layout, A, B, M, K, N, r, alpha, dX, dA, dB);
}

/* The LoRA dropout mask of the library (its counter-based generator,
 * restated): key = seed xor (stream * 0x9e3779b97f4a7c15) (lora.jl:41-43);
 * for element i, z = key + (i + 1) * 0x9e3779b97f4a7c15 through the SplitMix64
 * output function (Steele, Lea, Flood 2014); u = (z >> 40) * 2^-24 in fp32;
 * keep = u >= p. */
void oracle_dropout_keep(int64_t n, float p, uint64_t seed, uint64_t stream, uint8_t *keep)
{
    const uint64_t golden = 0x9e3779b97f4a7c15ull;
    const uint64_t key = seed ^ (stream * golden);
    for (int64_t i = 0; i < n; ++i) {
        uint64_t z = key + ((uint64_t)i + 1) * golden;
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        z ^= z >> 31;
        const float u = (float)(uint32_t)(z >> 40) * 0x1p-24f;
        keep[i] = u >= p ? 1 : 0;
    }
}

/* gelu_tanh of src/layers/linear.jl:61-68, elementwise in fp32 as written
 * there: cubic = x^3 (Julia's literal power, (x*x)*x), inner = x +
 * 0.044715f*cubic, y = 0.5f*x*(1 + tanh(sqrt(Float32(2/pi))*inner)).  The
 * caller rounds the input from and the output to the element type. */
#define GELU_K0 0.7978845238685608f /* sqrt(Float32(2/pi)) rounded to fp32 */
#define GELU_K1 0.044715f
void oracle_gelu_tanh(const float *x, int64_t n, float *out)
{
    for (int64_t i = 0; i < n; ++i) {
        const float v = x[i];
        const float cubic = (v * v) * v;
        const float inner = v + GELU_K1 * cubic;
        const float t = tanhf(GELU_K0 * inner);
        out[i] = (0.5f * v) * (1.0f + t);
    }
}

/* The derivative of gelu_tanh, the factor the pullback multiplies the
 * incoming gradient by (chain rule through linear.jl:63-66, fp32):
 *   0.5*(1 + t) + 0.5*x*(1 - t^2)*K0*(1 + 3*K1*x^2),  t = tanh(K0*inner). */
void oracle_gelu_tanh_grad(const float *x, int64_t n, float *out)
{
    for (int64_t i = 0; i < n; ++i) {
        const float v = x[i];
        const float x2 = v * v;
        const float inner = v + GELU_K1 * (x2 * v);
        const float t = tanhf(GELU_K0 * inner);
        const float dinner = GELU_K0 * (1.0f + 3.0f * GELU_K1 * x2);
        out[i] = 0.5f * (1.0f + t) + (0.5f * v) * (1.0f - t * t) * dinner;
    }
}

/* update! of src/training/optimizer.jl:63-71 over one tensor, with the clip
 * of src/training/wan_runner.jl:218-221 applied to the gradient first when
 * `clip` is set.  fp32 throughout, each operation rounded once (this file is
 * built with -ffp-contract=off, and Julia's broadcasts do not fuse):
 *   g = gs*g; g = g*clip_scale; m = b1*m + (1-b1)*g; v = b2*v + (1-b2)*g*g
 *   w = w - lr*((m/c1)/(sqrt(v/c2) + eps) + decay*w)
 * The model's copy of the parameter is w rounded to its element type, which
 * the caller does. */
void oracle_adamw_update(const float *g, float *m, float *v, float *w, int64_t n, float lr, float b1, float b2,
                         float eps, float decay, float c1, float c2, float gs, int clip, float clip_scale)
{
    const float omb1 = 1.0f - b1, omb2 = 1.0f - b2;
    for (int64_t i = 0; i < n; ++i) {
        float gi = g[i];
        if (gs != 1.0f) gi = gi * gs;
        if (clip) gi = gi * clip_scale;
        const float mi = b1 * m[i] + omb1 * gi;
        const float g2 = gi * gi;
        const float vi = b2 * v[i] + omb2 * g2;
        const float t1 = mi / c1;
        const float t2 = vi / c2;
        const float t3 = sqrtf(t2);
        const float t4 = t3 + eps;
        const float t5 = t1 / t4;
        const float t6 = decay * w[i];
        const float t7 = t5 + t6;
        const float t8 = lr * t7;
        m[i] = mi;
        v[i] = vi;
        w[i] = w[i] - t8;
    }
}

/* sum of (gs*g)^2 in fp64: the reference's norm_squared (wan_runner.jl:215)
 * without its fp32 summation-order dependence. */
double oracle_sumsq(const float *g, int64_t n, float gs)
{
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        const float a = g[i] * gs;
        s += (double)a * (double)a;
    }
    return s;
}

/* mixed_affine(layernorm(x; eps, w, b), scale, shift) (src/layers/linear.jl:
 * 26-36,49-59) per row of X [M][K]; sample = row / tps.  The mean and the
 * variance are summed in fp64 and rounded to fp32 (the reference sums in fp32
 * in its reduction's order); the rest is the reference's fp32 sequence:
 *   y = (x - mean) / sqrt(var + eps) (* w) (+ b)   -> LN (the caller rounds)
 * Out receives y; the caller rounds it to the element type, then forms
 * round(ln * (1 + scale) + shift) with oracle_modulate. */
void oracle_layernorm(const float *X, int64_t M, int64_t K, float eps, const float *w, const float *b, float *Y)
{
    for (int64_t m = 0; m < M; ++m) {
        const float *x = X + m * K;
        double s = 0.0;
        for (int64_t k = 0; k < K; ++k) s += x[k];
        const float mean = (float)s / (float)K;
        double q = 0.0;
        for (int64_t k = 0; k < K; ++k) {
            const float c = x[k] - mean;
            q += (double)c * (double)c;
        }
        const float var = (float)q / (float)K;
        const float d = sqrtf(var + eps);
        for (int64_t k = 0; k < K; ++k) {
            float y = (x[k] - mean) / d;
            if (w) y = y * w[k];
            if (b) y = y + b[k];
            Y[m * K + k] = y;
        }
    }
}

/* mixed_affine's fp32 part: ln * (1 + scale[b]) + shift[b]. */
void oracle_modulate(const float *LN, int64_t M, int64_t K, int64_t tps, const float *scale, const float *shift,
                     float *Out)
{
    for (int64_t m = 0; m < M; ++m) {
        const int64_t b = m / tps;
        for (int64_t k = 0; k < K; ++k) {
            float v = LN[m * K + k];
            if (scale) v = v * (1.0f + scale[b * K + k]);
            if (shift) v = v + shift[b * K + k];
            Out[m * K + k] = v;
        }
    }
}

/* The LayerNorm's pullback in fp64 from G = the gradient reaching its
 * (rounded) output, per row: with yhat = (x - mean)/d and gw = G * w,
 *   dx = (gw - mean(gw) - yhat * mean(gw * yhat)) / d. */
void oracle_layernorm_backward(const float *X, const float *G, int64_t M, int64_t K, float eps, const float *w,
                               float *DX)
{
    for (int64_t m = 0; m < M; ++m) {
        const float *x = X + m * K;
        double s = 0.0;
        for (int64_t k = 0; k < K; ++k) s += x[k];
        const double mean = s / (double)K;
        double q = 0.0;
        for (int64_t k = 0; k < K; ++k) q += (x[k] - mean) * (x[k] - mean);
        const double d = sqrt(q / (double)K + (double)eps);
        double s1 = 0.0, s2 = 0.0;
        for (int64_t k = 0; k < K; ++k) {
            const double gw = (double)G[m * K + k] * (w ? (double)w[k] : 1.0);
            s1 += gw;
            s2 += gw * (x[k] - mean) / d;
        }
        s1 /= (double)K;
        s2 /= (double)K;
        for (int64_t k = 0; k < K; ++k) {
            const double gw = (double)G[m * K + k] * (w ? (double)w[k] : 1.0);
            DX[m * K + k] = (float)((gw - s1 - (x[k] - mean) / d * s2) / d);
        }
    }
}

/* Relative L2 error ||a - b|| / ||b|| in fp64 (the north-star metric). */
double oracle_rel_l2(const float *a, const float *b, int64_t n)
{
    double num = 0.0, den = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        double d = (double)a[i] - (double)b[i];
        num += d * d;
        den += (double)b[i] * (double)b[i];
    }
    if (den == 0.0) return num == 0.0 ? 0.0 : INFINITY;
    return sqrt(num / den);
}
