// The optimizer step over the adapter tensors after the gradient all-reduce:
// the clip norm (wan_runner.jl:213-221) and AdamW with fp32 masters
// (optimizer.jl:48-73), each one launch over every tensor.
//
// Work is split into chunks of OPT_CHUNK elements of one tensor; a block
// walks chunks c = blockIdx.x, blockIdx.x + gridDim.x, ... and finds the
// tensor of a chunk by binary search over the prepared table's first-chunk
// indices.  Both kernels stream each element once (the norm reads g, the
// update reads g, m, v, master and writes m, v, master, param): HBM-bound, so
// the loads are 16-byte vectors wherever the tensor's pointers allow.
#pragma once
#include "common.cuh"

namespace reels {

constexpr int OPT_CHUNK = 8192;       // elements per work unit (a multiple of 4)
constexpr int OPT_THREADS = 256;
constexpr int OPT_MAX_BLOCKS = 1024;  // partial sums of the norm
constexpr uint32_t OPT_MAGIC = 0x5245'4f50u;

struct OptEntry {
    reels_opt_tensor t;
    int64_t chunk0;  // global index of the tensor's first chunk
    int vec;         // 1: every pointer allows 4-element vectors
    int pad;
};

struct OptHeader {
    uint32_t magic;
    int count;
    int64_t total_chunks;
};

// Workspace: header | fp64 partial sums of the norm | descriptor table.
constexpr size_t OPT_PARTIALS_OFF = 256;
constexpr size_t OPT_TABLE_OFF = OPT_PARTIALS_OFF + sizeof(double) * OPT_MAX_BLOCKS;
inline size_t opt_table_end(int count) { return OPT_TABLE_OFF + (size_t)count * sizeof(OptEntry); }

// Largest i with tab[i].chunk0 <= chunk (entries with no chunks share the
// next entry's chunk0; the search lands on the last of them that is <= chunk,
// which owns the chunk because later ones start later).
__device__ __forceinline__ int opt_find(const OptEntry *tab, int count, int64_t chunk) {
    int lo = 0, hi = count - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (tab[mid].chunk0 <= chunk) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ bool opt_header_ok(const OptHeader *h, unsigned *err) {
    if (h->magic != OPT_MAGIC || h->count < 0) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(err, DEVERR_OPT_TABLE);
        return false;
    }
    return true;
}

// Per-block fp64 partial sums of (gs * g)^2.
__global__ void __launch_bounds__(OPT_THREADS) grad_sumsq_kernel(const char *ws, float gs, double *partials,
                                                                   unsigned *err) {
    griddep_wait();
    const OptHeader *h = reinterpret_cast<const OptHeader *>(ws);
    __shared__ double red[OPT_THREADS / 32];
    double acc = 0.0;
    if (opt_header_ok(h, err)) {
        const OptEntry *tab = reinterpret_cast<const OptEntry *>(ws + OPT_TABLE_OFF);
        for (int64_t c = blockIdx.x; c < h->total_chunks; c += gridDim.x) {
            const OptEntry &e = tab[opt_find(tab, h->count, c)];
            const int64_t i0 = (c - e.chunk0) * OPT_CHUNK;
            const int64_t len = min((int64_t)OPT_CHUNK, e.t.n - i0);
            const float *g = e.t.grad + i0;
            if (e.vec) {
                // four 16-byte loads in flight per thread before they are summed
                const int64_t nv = len >> 2;
                for (int64_t j = threadIdx.x; j < nv; j += 4 * OPT_THREADS) {
                    float4 x[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        x[u] = j + u * OPT_THREADS < nv
                                   ? __ldcs(reinterpret_cast<const float4 *>(g) + j + u * OPT_THREADS)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float a = __fmul_rn(x[u].x, gs), b = __fmul_rn(x[u].y, gs);
                        const float cc = __fmul_rn(x[u].z, gs), d = __fmul_rn(x[u].w, gs);
                        acc += (double)a * a + (double)b * b + (double)cc * cc + (double)d * d;
                    }
                }
                for (int64_t j = (nv << 2) + threadIdx.x; j < len; j += OPT_THREADS) {
                    const float a = __fmul_rn(g[j], gs);
                    acc += (double)a * a;
                }
            } else {
                for (int64_t j = threadIdx.x; j < len; j += OPT_THREADS) {
                    const float a = __fmul_rn(g[j], gs);
                    acc += (double)a * a;
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int w = 0; w < OPT_THREADS / 32; ++w) s += red[w];
        partials[blockIdx.x] = s;
    }
}

// One block: the partials in a fixed order, rounded to fp32.
__global__ void __launch_bounds__(OPT_MAX_BLOCKS) grad_sumsq_final_kernel(const double *partials, int n,
                                                                           float *sumsq) {
    griddep_wait();
    __shared__ double red[OPT_MAX_BLOCKS];
    red[threadIdx.x] = threadIdx.x < n ? partials[threadIdx.x] : 0.0;
    __syncthreads();
    for (int s = OPT_MAX_BLOCKS / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) *sumsq = (float)red[0];
}

struct AdamArgs {
    float lr, beta1, beta2, omb1, omb2, eps, wd, c1, c2, gs, max_norm;
    const float *sumsq;
};

// One element of update! (optimizer.jl:63-71), every operation rounded once
// (the __f*_rn forms are never contracted into fused multiply-adds).
__device__ __forceinline__ void adam_elem(float g, float &m, float &v, float &w, const AdamArgs &a, float decay,
                                          bool clip, float clip_scale) {
    if (a.gs != 1.0f) g = __fmul_rn(g, a.gs);
    if (clip) g = __fmul_rn(g, clip_scale);
    m = __fadd_rn(__fmul_rn(a.beta1, m), __fmul_rn(a.omb1, g));
    v = __fadd_rn(__fmul_rn(a.beta2, v), __fmul_rn(a.omb2, __fmul_rn(g, g)));
    const float step = __fdiv_rn(__fdiv_rn(m, a.c1), __fadd_rn(__fsqrt_rn(__fdiv_rn(v, a.c2)), a.eps));
    w = __fsub_rn(w, __fmul_rn(a.lr, __fadd_rn(step, __fmul_rn(decay, w))));
}

__device__ __forceinline__ void store_param(void *p, int64_t i, int dt, float w) {
    if (dt == DT_BF16) reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(w);
    else if (dt == DT_F16) reinterpret_cast<__half *>(p)[i] = __float2half_rn(w);
    else reinterpret_cast<float *>(p)[i] = w;
}

__global__ void __launch_bounds__(OPT_THREADS) adamw_kernel(const char *ws, AdamArgs a, unsigned *err) {
    griddep_wait();
    const OptHeader *h = reinterpret_cast<const OptHeader *>(ws);
    if (!opt_header_ok(h, err)) return;
    // Clip (wan_runner.jl:215-221): gradient_norm = Float32(sqrt(norm_squared)).
    bool clip = false;
    float clip_scale = 1.0f;
    if (a.sumsq) {
        const float norm = __fsqrt_rn(*a.sumsq);
        clip = norm > a.max_norm;
        clip_scale = __fdiv_rn(a.max_norm, norm);
    }
    const OptEntry *tab = reinterpret_cast<const OptEntry *>(ws + OPT_TABLE_OFF);
    for (int64_t c = blockIdx.x; c < h->total_chunks; c += gridDim.x) {
        const OptEntry &e = tab[opt_find(tab, h->count, c)];
        const int64_t i0 = (c - e.chunk0) * OPT_CHUNK;
        const int64_t len = min((int64_t)OPT_CHUNK, e.t.n - i0);
        const float decay = e.t.decay ? a.wd : 0.0f;
        const int dt = e.t.param_dtype;
        const float *g = e.t.grad + i0;
        float *m = e.t.m + i0, *v = e.t.v + i0, *w = e.t.master + i0;
        char *p = reinterpret_cast<char *>(e.t.param) + i0 * (dt == DT_F32 ? 4 : 2);
        int64_t done = 0;
        if (e.vec) {
            const int64_t nv = len >> 2;
            for (int64_t j = threadIdx.x; j < nv; j += OPT_THREADS) {
                const float4 gg = __ldcs(reinterpret_cast<const float4 *>(g) + j);
                float4 mm = reinterpret_cast<float4 *>(m)[j];
                float4 vv = reinterpret_cast<float4 *>(v)[j];
                float4 ww = reinterpret_cast<float4 *>(w)[j];
                adam_elem(gg.x, mm.x, vv.x, ww.x, a, decay, clip, clip_scale);
                adam_elem(gg.y, mm.y, vv.y, ww.y, a, decay, clip, clip_scale);
                adam_elem(gg.z, mm.z, vv.z, ww.z, a, decay, clip, clip_scale);
                adam_elem(gg.w, mm.w, vv.w, ww.w, a, decay, clip, clip_scale);
                reinterpret_cast<float4 *>(m)[j] = mm;
                reinterpret_cast<float4 *>(v)[j] = vv;
                reinterpret_cast<float4 *>(w)[j] = ww;
                if (dt == DT_F32) {
                    reinterpret_cast<float4 *>(p)[j] = ww;
                } else if (dt == DT_BF16) {
                    __nv_bfloat162 lo = __floats2bfloat162_rn(ww.x, ww.y), hi = __floats2bfloat162_rn(ww.z, ww.w);
                    uint2 u;
                    u.x = *reinterpret_cast<uint32_t *>(&lo);
                    u.y = *reinterpret_cast<uint32_t *>(&hi);
                    reinterpret_cast<uint2 *>(p)[j] = u;
                } else {
                    __half2 lo = __floats2half2_rn(ww.x, ww.y), hi = __floats2half2_rn(ww.z, ww.w);
                    uint2 u;
                    u.x = *reinterpret_cast<uint32_t *>(&lo);
                    u.y = *reinterpret_cast<uint32_t *>(&hi);
                    reinterpret_cast<uint2 *>(p)[j] = u;
                }
            }
            done = nv << 2;
        }
        for (int64_t j = done + threadIdx.x; j < len; j += OPT_THREADS) {
            float mj = m[j], vj = v[j], wj = w[j];
            adam_elem(g[j], mj, vj, wj, a, decay, clip, clip_scale);
            m[j] = mj;
            v[j] = vj;
            w[j] = wj;
            store_param(e.t.param, i0 + j, dt, wj);
        }
    }
}

}  // namespace reels
