// LoRA dropout (lora.jl:71-85): the adapter's input is z = x * keep / (1 - p)
// with keep = (u >= p) for a uniform u per element; the frozen weight's
// product still uses x.
//
// The reference draws u from Julia's Xoshiro256++ seeded with
// seed xor (stream * 0x9e3779b97f4a7c15) (lora.jl:41-52) and copies the mask
// from the host.  Here u comes from a counter-based generator evaluated where
// it is used: the key is the reference's combined seed, the counter is the
// element's linear index in x (token-major, the reference's column-major
// order), and the value is the SplitMix64 output function (Steele, Lea and
// Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014)
// applied to key + (index + 1) * 0x9e3779b97f4a7c15.  Its top 24 bits make
// u = k * 2^-24, the resolution of rand(Float32).  The stream differs from
// Xoshiro's, so agreement with the reference is statistical (the kept
// fraction, uniformity, independence); the mask is the same wherever it is
// recomputed (forward, backward, oracle).
#pragma once
#include "act.cuh"
#include "common.cuh"

namespace reels {

constexpr uint64_t kDropoutGolden = 0x9e3779b97f4a7c15ull;

// _dropout_seed (lora.jl:41-43)
__host__ __device__ __forceinline__ uint64_t dropout_key(uint64_t seed, uint64_t stream) {
    return seed ^ (stream * kDropoutGolden);
}

__host__ __device__ __forceinline__ uint64_t dropout_bits(uint64_t key, uint64_t index) {
    uint64_t z = key + (index + 1) * kDropoutGolden;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// keep = rand >= p, rand = (top 24 bits) * 2^-24 compared in fp32
__device__ __forceinline__ bool dropout_keep(uint64_t key, uint64_t index, float p) {
    return (float)(uint32_t)(dropout_bits(key, index) >> 40) * 0x1p-24f >= p;
}

// The mask as bytes (1 kept, 0 dropped).
__global__ void dropout_mask_kernel(int64_t n, float p, uint64_t key, uint8_t *keep) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        keep[i] = dropout_keep(key, (uint64_t)i, p) ? 1 : 0;
}

// z = cast(float32(x .* mask) ./ (1f0 - p)) (lora.jl:80-83): the product with
// 0 or 1 is exact (a dropped negative x gives -0), the division is fp32.
// 16-bit types with n % 8 == 0 and 16-byte aligned pointers move eight
// elements per 16-byte access.
__global__ void dropout_input_kernel(const void *x, int64_t n, int dt, float p, uint64_t key, void *z) {
    griddep_wait();
    const float keep_scale = 1.0f - p;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool vec = dt != DT_F32 && (n & 7) == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(z)) & 15) == 0;
    if (vec) {
        for (int64_t v = t0; v < n / 8; v += stride) {
            uint4 in = reinterpret_cast<const uint4 *>(x)[v], out;
            const uint32_t *iw = &in.x;
            uint32_t *ow = &out.x;
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                float a, b;
                if (dt == DT_BF16) unpack2<DT_BF16>(iw[h], a, b);
                else unpack2<DT_F16>(iw[h], a, b);
                const uint64_t i = (uint64_t)(8 * v + 2 * h);
                a = __fdiv_rn(__fmul_rn(a, dropout_keep(key, i, p) ? 1.0f : 0.0f), keep_scale);
                b = __fdiv_rn(__fmul_rn(b, dropout_keep(key, i + 1, p) ? 1.0f : 0.0f), keep_scale);
                ow[h] = dt == DT_BF16 ? Elem<DT_BF16>::pack2(a, b) : Elem<DT_F16>::pack2(a, b);
            }
            reinterpret_cast<uint4 *>(z)[v] = out;
        }
        return;
    }
    for (int64_t i = t0; i < n; i += stride) {
        const float kept = __fmul_rn(load_act(x, i, dt), dropout_keep(key, (uint64_t)i, p) ? 1.0f : 0.0f);
        store_act(z, i, dt, __fdiv_rn(kept, keep_scale));
    }
}

// The adapter's part of dx through the dropout, added to the frozen weight's
// part already in dx:
//   dz = round(A' g')  (g' = s B' dy, [r][ldg]),  d = round(round(dz / (1 - p)) * keep)
//   dx = round(dx + d)
// Tile: 32 tokens x 256 input features per block, g' of the tokens in shared
// memory (read as 16-byte broadcasts), one feature per thread with 32
// accumulators.  The feature's row of A streams through registers eight
// ranks (16 bytes) at a time, the next eight loaded while the current ones
// are used: the loop is otherwise bound by that load's latency.
constexpr int DROP_TOK = 32;
template <int DT>
__global__ void __launch_bounds__(256) dropout_dx_kernel(const void *a, const void *g, int64_t ldg, int64_t M,
                                                         int64_t K, int r, float p, uint64_t key, void *dx) {
    griddep_wait();
    extern __shared__ float gs[];  // [r][DROP_TOK]
    const int64_t m0 = (int64_t)blockIdx.y * DROP_TOK;
    for (int i = threadIdx.x; i < r * DROP_TOK; i += blockDim.x) {
        const int j = i / DROP_TOK, t = i % DROP_TOK;
        gs[i] = m0 + t < M ? load_act(g, (int64_t)j * ldg + m0 + t, DT) : 0.0f;
    }
    __syncthreads();
    const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= K) return;
    float acc[DROP_TOK];
#pragma unroll
    for (int t = 0; t < DROP_TOK; ++t) acc[t] = 0.0f;
    auto rank_step = [&](float av, int j) {
        const float4 *g4 = reinterpret_cast<const float4 *>(gs + j * DROP_TOK);  // same address in every lane
#pragma unroll
        for (int t4 = 0; t4 < DROP_TOK / 4; ++t4) {
            const float4 gv = g4[t4];
            acc[4 * t4] = fmaf(av, gv.x, acc[4 * t4]);
            acc[4 * t4 + 1] = fmaf(av, gv.y, acc[4 * t4 + 1]);
            acc[4 * t4 + 2] = fmaf(av, gv.z, acc[4 * t4 + 2]);
            acc[4 * t4 + 3] = fmaf(av, gv.w, acc[4 * t4 + 3]);
        }
    };
    if constexpr (DT != DT_F32) {
        if ((r & 7) == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0) {
            const uint4 *row = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(a) + k * r);
            const int nc = r / 8;
            uint4 cur = row[0];
            for (int c = 0; c < nc; ++c) {
                const uint4 nxt = c + 1 < nc ? row[c + 1] : cur;
                const uint32_t w[4] = {cur.x, cur.y, cur.z, cur.w};
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    float a0, a1;
                    unpack2<DT>(w[h], a0, a1);
                    rank_step(a0, 8 * c + 2 * h);
                    rank_step(a1, 8 * c + 2 * h + 1);
                }
                cur = nxt;
            }
        } else {
            for (int j = 0; j < r; ++j) rank_step(load_act(a, k * r + j, DT), j);
        }
    } else {
        for (int j = 0; j < r; ++j) rank_step(load_act(a, k * r + j, DT), j);
    }
    const float keep_scale = 1.0f - p;
    // fully unrolled (a loop that could stop early would index acc[] at run
    // time and move it to local memory)
#pragma unroll
    for (int t = 0; t < DROP_TOK; ++t) {
        if (m0 + t < M) {
            const int64_t idx = (m0 + t) * K + k;
            float d = 0.0f;
            if (dropout_keep(key, (uint64_t)idx, p)) d = round_dt(__fdiv_rn(round_dt(acc[t], DT), keep_scale), DT);
            store_act(dx, idx, DT, load_act(dx, idx, DT) + d);
        }
    }
}

}  // namespace reels
