// Host side of libreels_lowvram.so: argument checks, tile planning, TMA
// tensor maps and kernel launches behind the C ABI of include/reels_lowvram.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

#include "../../include/reels_lowvram.h"
#include "aux_kernels.cuh"
#include "q8_gemm.cuh"
#include "dropout.cuh"
#include "norm.cuh"
#include "optim.cuh"
#include "q8ts_gemm.cuh"

using namespace reels;

// Status words the kernels OR error bits into (one per device context).
__device__ unsigned g_dev_status;
__device__ unsigned g_quant_status;

namespace {

thread_local std::string t_last_error;
thread_local int t_last_path = REELS_PATH_NONE;

// Opt-in profiling: events around each q8 GEMM launch on its own stream.
struct Profile {
    bool on = false;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pool;
    size_t used = 0;
    double flops = 0.0;
};
thread_local Profile t_prof;
thread_local long long t_launches = 0;

inline void count_launch(int n = 1) { t_launches += n; }

int fail(const std::string &msg) {
    t_last_error = msg;
    return REELS_EINVAL;
}
int fail_dev(const std::string &msg) {
    t_last_error = msg;
    return REELS_EDEVICE;
}
int ok(int path) {
    t_last_error.clear();
    t_last_path = path;
    return REELS_OK;
}

#define REELS_LAUNCHED()                                                                                \
    do {                                                                                                \
        cudaError_t e_ = cudaGetLastError();                                                            \
        if (e_ != cudaSuccess) return fail_dev(std::string("kernel launch: ") + cudaGetErrorString(e_)); \
        count_launch();                                                                                 \
    } while (0)

#define REELS_CUDA(call)                                                                                \
    do {                                                                                                \
        cudaError_t e_ = (call);                                                                        \
        if (e_ != cudaSuccess) return fail_dev(std::string(#call) + ": " + cudaGetErrorString(e_));    \
    } while (0)

// Launch with programmatic stream serialization (see griddep_wait in
// common.cuh): the launch is queued ahead of the previous kernel's completion
// and every kernel launched this way waits for that kernel before touching
// global memory.  REELS_NO_PDL=1 launches everything in plain stream order.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    static const bool pdl = [] {
        const char *e = getenv("REELS_NO_PDL");
        return !(e && atoi(e) != 0);
    }();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// The same with a cluster of `cx` CTAs along x (the CTA pairs of the
// weight-in-TMEM kernel); the grid is a multiple of cx.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cx,
                               Args... args) {
    static const bool pdl = [] {
        const char *e = getenv("REELS_NO_PDL");
        return !(e && atoi(e) != 0);
    }();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)cx;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// ------------------------------------------------------------ device state
constexpr int kMaxDevices = 64;
struct DeviceState {
    bool ready = false;
    int index = -1;
    int sms = 148;
    unsigned *status = nullptr;
    unsigned *quant_status = nullptr;
};
DeviceState g_dev[kMaxDevices];
std::mutex g_dev_mu;

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

template <int DT, int MT, int BN>
cudaError_t set_q8_attr() {
    return cudaFuncSetAttribute(q8_gemm_kernel<DT, MT, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                Q8Geom<MT, BN>::SMEM_BYTES);
}
template <int DT>
cudaError_t set_q8_attrs() {
    cudaError_t e;
    if ((e = set_q8_attr<DT, 1, 128>()) != cudaSuccess) return e;
    if ((e = set_q8_attr<DT, 1, 256>()) != cudaSuccess) return e;
    if ((e = set_q8_attr<DT, 2, 128>()) != cudaSuccess) return e;
    return set_q8_attr<DT, 2, 256>();
}

template <int DT, int BT, int KB2>
cudaError_t set_ts_attr() {
    cudaError_t e = cudaFuncSetAttribute(q8ts_gemm_kernel<DT, BT, KB2, ACT_NONE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, TsGeom<BT, KB2>::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(q8ts_gemm_kernel<DT, BT, KB2, ACT_GELU_TANH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             TsGeom<BT, KB2>::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(q8ts_gemm_kernel<DT, BT, KB2, ACT_GELU_TANH_GRAD>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, TsGeom<BT, KB2>::SMEM_BYTES);
}
template <int DT, int BT, int KB2>
cudaError_t set_ts_pair_attr() {
    using G = TsGeom<BT, KB2, 1>;
    cudaError_t e = cudaFuncSetAttribute(q8ts_gemm_kernel<DT, BT, KB2, ACT_NONE, 1>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(q8ts_gemm_kernel<DT, BT, KB2, ACT_GELU_TANH, 1>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(q8ts_gemm_kernel<DT, BT, KB2, ACT_GELU_TANH_GRAD, 1>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM_BYTES);
}

template <int DT>
cudaError_t set_ts_attrs() {
    cudaError_t e;
    if ((e = set_ts_attr<DT, 256, 1>()) != cudaSuccess) return e;
    if ((e = set_ts_attr<DT, 192, 1>()) != cudaSuccess) return e;
    if ((e = set_ts_attr<DT, 128, 1>()) != cudaSuccess) return e;
    if ((e = set_ts_attr<DT, 256, 2>()) != cudaSuccess) return e;
    if ((e = set_ts_attr<DT, 192, 2>()) != cudaSuccess) return e;
    if ((e = set_ts_attr<DT, 128, 2>()) != cudaSuccess) return e;
    if ((e = set_ts_pair_attr<DT, 256, 2>()) != cudaSuccess) return e;
    return set_ts_pair_attr<DT, 128, 2>();
}

// The calling thread's current context is restored when an entry point
// returns: a caller that passes device-1 buffers while device 0 is current
// gets device 0 back.  Contexts (not device indices) are compared and
// restored, so a thread that had no current context is left with none and
// no primary context is created on a device the caller never used.
using CtxGetFn = CUresult (*)(CUcontext *);
using CtxSetFn = CUresult (*)(CUcontext);
CtxGetFn g_ctx_get = nullptr;
CtxSetFn g_ctx_set = nullptr;
std::once_flag g_ctx_once;

struct DeviceScope {
    CUcontext prev = nullptr;
    bool restore = false;
    DeviceScope() = default;
    DeviceScope(const DeviceScope &) = delete;
    DeviceScope &operator=(const DeviceScope &) = delete;
    ~DeviceScope() {
        if (restore && g_ctx_set) g_ctx_set(prev);
    }
};

void resolve_ctx_calls() {
    std::call_once(g_ctx_once, [] {
        void *fg = nullptr, *fs = nullptr;
        cudaDriverEntryPointQueryResult q1, q2;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fg, cudaEnableDefault, &q1) == cudaSuccess &&
            cudaGetDriverEntryPoint("cuCtxSetCurrent", &fs, cudaEnableDefault, &q2) == cudaSuccess &&
            q1 == cudaDriverEntryPointSuccess && q2 == cudaDriverEntryPointSuccess && fg && fs) {
            g_ctx_get = reinterpret_cast<CtxGetFn>(fg);
            g_ctx_set = reinterpret_cast<CtxSetFn>(fs);
        } else {
            cudaGetLastError();
        }
    });
}

int bind_device(const void *ptr, DeviceState **out, DeviceScope &scope) {
    int dev = -1;
    cudaPointerAttributes attr;
    if (ptr && cudaPointerGetAttributes(&attr, ptr) == cudaSuccess && attr.type == cudaMemoryTypeDevice) {
        dev = attr.device;
    } else {
        cudaGetLastError();
        REELS_CUDA(cudaGetDevice(&dev));
    }
    if (dev < 0 || dev >= kMaxDevices) return fail("device index out of range");
    // Always bind: on a thread that has not used this device yet (e.g. an
    // autograd worker) this also makes the primary context current, which
    // the driver-API tensor-map encoder needs.  `scope` puts the caller's
    // context back when the entry point returns.
    resolve_ctx_calls();
    CUcontext before = nullptr, after = nullptr;
    if (g_ctx_get && g_ctx_get(&before) != CUDA_SUCCESS) before = nullptr;
    REELS_CUDA(cudaSetDevice(dev));
    if (g_ctx_get && g_ctx_get(&after) == CUDA_SUCCESS && after != before && !scope.restore) {
        scope.prev = before;
        scope.restore = true;
    }
    std::lock_guard<std::mutex> lock(g_dev_mu);
    DeviceState &st = g_dev[dev];
    if (!st.ready) {
        st.index = dev;
        int major = 0, minor = 0;
        REELS_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
        REELS_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
        if (major != 10 || minor != 0)
            return fail("libreels_lowvram is built for sm_100a (B200); device " + std::to_string(dev) +
                        " is sm_" + std::to_string(major) + std::to_string(minor));
        REELS_CUDA(cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, dev));
        REELS_CUDA(cudaGetSymbolAddress(reinterpret_cast<void **>(&st.status), g_dev_status));
        REELS_CUDA(cudaGetSymbolAddress(reinterpret_cast<void **>(&st.quant_status), g_quant_status));
        REELS_CUDA(set_q8_attrs<DT_BF16>());
        REELS_CUDA(set_q8_attrs<DT_F16>());
        REELS_CUDA(set_ts_attrs<DT_BF16>());
        REELS_CUDA(set_ts_attrs<DT_F16>());
        for (auto fn : {(const void *)ln_modulate_kernel<DT_BF16>, (const void *)ln_modulate_kernel<DT_F16>,
                        (const void *)ln_modulate_kernel<DT_F32>, (const void *)ln_modulate_bwd_kernel<DT_BF16>,
                        (const void *)ln_modulate_bwd_kernel<DT_F16>, (const void *)ln_modulate_bwd_kernel<DT_F32>})
            REELS_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * LN_MAX_K * 4));
        REELS_CUDA(cudaFuncSetAttribute(sk_gemm_kernel<DT_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SK_SMEM_BYTES));
        REELS_CUDA(cudaFuncSetAttribute(sk_gemm_kernel<DT_F16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SK_SMEM_BYTES));
        REELS_CUDA(cudaFuncSetAttribute(sk_dual_kernel<DT_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        DU_SMEM_BYTES));
        REELS_CUDA(cudaFuncSetAttribute(sk_dual_kernel<DT_F16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        DU_SMEM_BYTES));
        if (!g_encode) {
            void *fn = nullptr;
            cudaDriverEntryPointQueryResult qr;
            REELS_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr));
            if (qr != cudaDriverEntryPointSuccess || !fn) return fail_dev("cuTensorMapEncodeTiled unavailable");
            g_encode = reinterpret_cast<EncodeTiledFn>(fn);
        }
        st.ready = true;
    }
    *out = &st;
    return REELS_OK;
}

// ------------------------------------------------------------- tensor maps
int tmap_2d(CUtensorMap *tm, const void *base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
            uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {pitch_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(tm, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[200];
        snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu pitch %llu box %u x %u", (int)r,
                 (unsigned long long)inner, (unsigned long long)outer, (unsigned long long)pitch_bytes, box_inner,
                 box_outer);
        return fail(buf);
    }
    return REELS_OK;
}

CUtensorMapDataType tma_act_type(int dt) {
    return dt == REELS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// ---------------------------------------------------------------- planning
int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
int64_t round_up(int64_t a, int64_t b) { return cdiv(a, b) * b; }
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
int esize(int dt) { return dt == REELS_F32 ? 4 : 2; }
int64_t ld_tokens(int64_t M) { return round_up(std::max<int64_t>(M, 1), 8); }

struct Split {
    int splits = 1;
    int kb_per = 1;
};

// Split of the reduction for the skinny kernels: the split count that
// minimises (waves of CTAs) x (reduction blocks per CTA) plus the fp32
// partial traffic, in units of one reduction block of one tile (16 KB of
// 16-bit activations; a partial tile of 128 x npad fp32 is written once and
// read once).  Each CTA runs one (tile, split) unit and the SK kernel is one
// CTA per SM, so a count that spills a few CTAs into a second wave roughly
// doubles the time.
Split plan_split(int64_t tiles, int64_t kb, int sms, int64_t min_kb, int64_t npad) {
    Split best;
    kb = std::max<int64_t>(kb, 1);
    double best_cost = 1e300;
    const int64_t max_want = std::max<int64_t>(1, kb / min_kb);
    const double part_cost = 2.0 * 128.0 * (double)npad * 4.0 / 16384.0;  // per partial tile, in block units
    for (int64_t want = 1; want <= max_want; ++want) {
        Split s;
        s.kb_per = (int)cdiv(kb, want);
        s.splits = (int)cdiv(kb, s.kb_per);
        if (want > 1 && s.splits != want) continue;
        const double waves = (double)cdiv(tiles * s.splits, sms);
        double cost = waves * s.kb_per;
        if (s.splits > 1) cost += part_cost * (double)(tiles * s.splits) / sms + 2.0;
        if (cost < best_cost * 0.999) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

int npad_of(int64_t r) { return (int)std::max<int64_t>(16, round_up(r, 16)); }

struct Q8Plan {
    int mt = 1, bn = 256;
    int ts = 0;         // > 0: weight-in-TMEM kernel, 128 output columns x ts tokens
    int ts_kb2 = 1;     // its pipeline stages cover 64 * ts_kb2 reduction elements
    int pair = 0;       // 1: CTA pairs (cta_group::2), 256 output columns per tile
    int64_t ntiles = 1, mtiles = 1;
    Split split;
};

// Kernel, tile shape and reduction split from a time model fitted to B200
// measurements (microseconds per pipeline stage of one tile, plus a per-tile
// epilogue cost the kernel cannot overlap; least squares over whole-tile
// rounds of the Wan 1.3B/14B linears at 512..32760 tokens):
//   weight-in-TMEM kernel (q8ts_gemm.cuh), 128 output columns x bt tokens,
//   stages of 64 reduction elements: bt 256: 0.51 + 0.54 per tile (single
//       accumulator), bt 192: 0.47 + 0.23, bt 128: 0.46 + 0.37;
//   stages of 128: bt 256: 0.84 + 1.14, bt 192: 0.79 + 0.28, bt 128: 0.64 + 0.20.
//   The MMA warp's per-stage waits and commit cost about the same whatever
//   the stage width, so 128-wide stages move more weight per round trip; the
//   256-token tiles' 128-wide stages also hand their activation atoms back
//   one at a time (q8ts_gemm.cuh), which hides most of their refill.
//   CTA pairs (256 output columns per tile on two SMs, 74 tiles in flight):
//   bt 256: 0.80 + 1.05, bt 128: 0.62 + 0.30 (128-wide stages; the ratios
//   to the single-CTA plans measured on one box, 3-7% and 2-5% faster).
//   128-token tiles with 128-wide stages whose launch gives each CTA one
//   unit run two MMA issuers: per stage x0.89 single, x0.98 on pairs.
//   SMEM x SMEM kernel (q8_gemm.cuh), 128*mt tokens x bn output columns:
//       2x256: 1.18 + 4.0, 2x128: 0.85, 1x256: 1.0, 1x128: 0.75 (+ 1.5).
// The kernels are persistent, so a CTA runs ceil(work units / SMs) units; a
// split reduction adds the write and re-read of fp32 partials (~5 TB/s).
// REELS_Q8_TILE ("MTxBN") and REELS_Q8_TS (256, 192, 128; 2562,
// 1922, 1282 for 128-wide stages; 0 for off) force a plan for measurements.
// Two MMA issuers on 128-token tiles (q8ts_gemm.cuh) when each CTA (or CTA
// pair) runs a single work unit.  REELS_Q8_ISS2=0 turns them off.
bool q8_iss2_env_on() {
    static const int env = [] {
        const char *e = getenv("REELS_Q8_ISS2");
        return e ? atoi(e) : 1;
    }();
    return env != 0;
}
bool q8_iss2_ok(const Q8Plan &p, int sms) {
    const int64_t units = p.ntiles * p.mtiles * p.split.splits;
    return q8_iss2_env_on() && p.ts == 128 && units <= (p.pair ? sms / 2 : sms);
}

Q8Plan plan_q8(int64_t M, int64_t Nout, int64_t Kred, int sms, bool allow_ts, int act) {
    static const int forced = [] {
        const char *e = getenv("REELS_Q8_TILE");  // "MTxBN" (e.g. "2x128")
        if (!e) return 0;
        int a = 0, b = 0;
        if (sscanf(e, "%dx%d", &a, &b) == 2 && (a == 1 || a == 2) && (b == 128 || b == 256)) return a * 1000 + b;
        return 0;
    }();
    static const int forced_ts = [] {
        const char *e = getenv("REELS_Q8_TS");  // 256, 192, 128 (64-wide stages), 2562, 1922, 1282 (128-wide), 0 = off
        if (!e) return -1;                      // automatic
        const int v = atoi(e);
        return (v == 256 || v == 192 || v == 128 || v == 2562 || v == 1922 || v == 1282) ? v : 0;
    }();
    // REELS_Q8_PAIR: 1 runs the plans that have a CTA-pair variant on pairs,
    // 0 never; unset, the model decides.
    static const int pair_env = [] {
        const char *e = getenv("REELS_Q8_PAIR");
        return e ? (atoi(e) == 1 ? 1 : 0) : -1;
    }();
    struct Cand {
        int mt, bn, ts, kb2;
        double per_kb, epi;  // per_kb: per pipeline stage (64 * kb2 reduction elements)
        int pair;            // CTA pair: 256 output columns per tile on two SMs
    };
    const Cand cands[] = {
        {0, 0, 256, 1, 0.51, 0.54, 0}, {0, 0, 192, 1, 0.47, 0.23, 0}, {0, 0, 128, 1, 0.46, 0.37, 0},
        {0, 0, 128, 2, 0.64, 0.20, 0}, {0, 0, 256, 2, 0.84, 1.14, 0}, {0, 0, 192, 2, 0.79, 0.28, 0},
        {0, 0, 256, 2, 0.80, 1.05, 1}, {0, 0, 128, 2, 0.62, 0.30, 1},
        {2, 256, 0, 1, 1.18, 4.0, 0}, {2, 128, 0, 1, 0.85, 1.5, 0}, {1, 256, 0, 1, 1.0, 1.5, 0},
        {1, 128, 0, 1, 0.75, 1.5, 0},
    };
    double best = 1e300;
    Q8Plan bestp;
    for (const Cand &cd : cands) {
        const int64_t kb = cdiv(Kred, BK * cd.kb2);
        if (cd.pair && pair_env == 0) continue;
        if (!cd.pair && cd.ts && pair_env == 1 && cd.kb2 == 2 && (cd.ts == 256 || cd.ts == 128)) continue;
        if (cd.ts) {
            if (!allow_ts || forced || forced_ts == 0) continue;
            if (forced_ts > 0 && forced_ts != cd.ts * 10 + cd.kb2 && forced_ts != cd.ts) continue;
            if (forced_ts > 0 && forced_ts == cd.ts && cd.kb2 != 1) continue;
        } else {
            if (forced_ts > 0) continue;
            if (forced && forced != cd.mt * 1000 + cd.bn) continue;
            if (!forced && cd.mt == 2 && M < 256) continue;
        }
        const int64_t ntiles = cd.ts ? cdiv(Nout, cd.pair ? 256 : 128) : cdiv(Nout, cd.bn);
        const int slots = cd.pair ? sms / 2 : sms;  // tiles in flight
        const int64_t mtiles = cd.ts ? cdiv(M, cd.ts) : cdiv(M, 128 * cd.mt);
        const int64_t tiles = ntiles * mtiles;
        for (int64_t want = 1; want <= std::max<int64_t>(1, kb / 4); want = want < 4 ? want + 1 : want * 2) {
            Split sp;
            sp.kb_per = (int)cdiv(kb, want);
            sp.splits = (int)cdiv(kb, sp.kb_per);
            if (want > 1 && sp.splits == 1) continue;
            const double units = (double)cdiv(tiles * sp.splits, slots);
            // A fused activation lengthens the epilogue; with one accumulator
            // (256-token tiles) the MMAs wait for it.
            const double act_epi = act == ACT_NONE || sp.splits > 1 ? 0.0 : (cd.ts == 256 ? 1.5 : 0.1);
            // 128-token tiles with 128-wide stages, one unit per CTA: two MMA
            // issuers (fwd / dX at 128 x 5120 x 13824: 11% faster single, 2% on pairs)
            double per_kb = cd.per_kb;
            if (cd.ts == 128 && cd.kb2 == 2 && units == 1.0 && q8_iss2_env_on()) per_kb *= cd.pair ? 0.98 : 0.89;
            double cost = units * (sp.kb_per * per_kb + cd.epi + act_epi);
            if (sp.splits > 1) cost += 2.0 * sp.splits * (double)M * (double)Nout * 4.0 / 5.0e6 + 3.0;
            if (cost < best * 0.999) {
                best = cost;
                bestp = Q8Plan();
                bestp.mt = cd.ts ? 1 : cd.mt;
                bestp.bn = cd.ts ? 128 : cd.bn;
                bestp.ts = cd.ts;
                bestp.ts_kb2 = cd.kb2;
                bestp.pair = cd.pair;
                bestp.ntiles = ntiles;
                bestp.mtiles = mtiles;
                bestp.split = sp;
            }
            if (tiles >= slots) break;  // enough tiles: never split
        }
    }
    return bestp;
}

Split plan_sk(int64_t rows, int64_t red, int sms, int64_t r) {
    return plan_split(cdiv(rows, 128), cdiv(red, BK), sms, 4, npad_of(r));
}

// Grid of the one-pass dy kernel (sk_dual_kernel): splits_m token ranges x
// splits_n feature ranges, one CTA each.  Cost, in units of 16 KB streamed
// into one SM: the largest CTA's stages (each a 128 x 128 tile of dy, 32 KB,
// plus 128 columns of B and 128 tokens of T, npad x 256 B each), plus the
// fp32 partials written and read back (G's when the features are split, dB's
// when the tokens are), spread over the SMs, plus a fixed charge for the
// reduce launch.  The separate G and dB passes are costed the same way
// (plan_split; each 16 KB block of dy brings npad x 128 B of B or T); the
// cheaper plan wins.  Ranks above 128 leave no TMEM for the dB accumulators:
// separate passes.
struct DualPlan {
    bool use = false;
    int splits_m = 1, splits_n = 1, tmem_cols = 0;
    int64_t part_g = 0, part_db = 0;  // partial bytes
};

DualPlan plan_dual(int64_t M, int64_t N, int64_t r, int sms) {
    DualPlan best;
    const int np = npad_of(r);
    const int kmax = np <= 128 ? du_max_ftiles(np) : 0;
    if (kmax < 1 || M <= 0 || N <= 0 || r <= 0) return best;
    if (const char *e = getenv("REELS_SK_DUAL"))
        if (atoi(e) == 0) return best;
    const int64_t TM = cdiv(M, 128), TN = cdiv(N, 128);
    const double blk = 16384.0 * sms;  // bytes the GPU streams per block round
    double best_cost = 1e300;
    for (int64_t sn = cdiv(TN, kmax); sn <= std::min<int64_t>(TN, sms); ++sn) {
        const int64_t kn = cdiv(TN, sn);
        if (kn > kmax) continue;
        const int64_t sm_max = std::min<int64_t>(TM, sms / sn);
        for (int64_t smm = 1; smm <= sm_max; ++smm) {
            const double part_g = sn > 1 ? (double)sn * M * np * 4 : 0.0;
            const double part_db = smm > 1 ? (double)smm * N * np * 4 : 0.0;
            double cost = (2.0 + np / 32.0) * (double)(cdiv(TM, smm) * kn) + 2.0 * (part_g + part_db) / blk;
            if (sn > 1 || smm > 1) cost += 2.0;
            if (cost < best_cost * 0.999) {
                best_cost = cost;
                best.splits_m = (int)smm;
                best.splits_n = (int)sn;
                best.part_g = (int64_t)part_g;
                best.part_db = (int64_t)part_db;
            }
        }
    }
    // the separate passes: G (rows = tokens, reduction = features) and dB
    // (rows = features, reduction = tokens), each with its own split
    auto sep = [&](int64_t rows, int64_t red) {
        const Split s = plan_split(cdiv(rows, 128), cdiv(red, BK), sms, 4, np);
        double c = (double)cdiv(cdiv(rows, 128) * s.splits, sms) * s.kb_per * (1.0 + np / 128.0);
        if (s.splits > 1) c += 2.0 * 128.0 * np * 4.0 * (double)(cdiv(rows, 128) * s.splits) / blk + 2.0;
        return c + 2.0;  // launch
    };
    const double sep_cost = sep(M, N) + sep(N, M);
    if (best_cost + 2.0 < sep_cost) {
        best.use = true;
        const int64_t kn = cdiv(TN, best.splits_n);
        const int need = (int)(2 + kn) * du_acc_cols(np);
        int cols = 32;
        while (cols < need) cols <<= 1;
        best.tmem_cols = cols;
    }
    return best;
}


// Workspace layout shared by the forward and backward passes.
struct Ws {
    size_t at = 0, tbuf = 0, gbuf = 0, ext = 0, zbuf = 0, part = 0, total = 0;
};

// Rank padding of the prepared LoRA operands: a multiple of the widest
// pipeline stage (128 reduction elements).
int64_t rank_pad(int64_t r) { return round_up(std::max<int64_t>(r, 1), 128); }
// The weight-in-TMEM kernel reads its LoRA operand 32 ranks at a time.
int64_t ts_rank_pad(int64_t r) { return round_up(std::max<int64_t>(r, 1), 32); }

Ws ws_layout(int64_t M, int64_t K, int64_t N, int64_t r, int dt, int pass_flags, int sms) {
    Ws w;
    const int pass = pass_flags & 1;
    const bool dropout = (pass_flags & REELS_PASS_DROPOUT) && r > 0;
    const int64_t ldm = ld_tokens(M);
    size_t off = 0;
    const size_t at_bytes = r > 0 ? align256((size_t)r * K * 2) : 0;
    const size_t tg_bytes = r > 0 ? align256((size_t)r * ldm * esize(dt)) : 0;
    w.at = off;
    off += at_bytes;
    w.tbuf = off;
    off += tg_bytes;
    w.gbuf = off;
    if (pass == REELS_PASS_BACKWARD) off += tg_bytes;
    w.ext = off;
    if (r > 0) off += align256((size_t)rank_pad(r) * std::max(N, K) * 2);
    w.zbuf = off;  // the dropped-out adapter input z [M][K]
    if (dropout) off += align256((size_t)M * K * esize(dt));
    size_t part = 0;
    const int64_t np = npad_of(r);
    auto sk_part = [&](int64_t rows, int64_t red) {
        Split s = plan_sk(rows, red, sms, r);
        if (s.splits > 1) part = std::max(part, (size_t)s.splits * rows * np * 4);
    };
    auto q8_part = [&](int64_t rows, int64_t cols, int64_t red) {
        // the TMEM-weight plan may fall back to the other; a fused activation
        // weighs the plans differently
        for (int ts = 0; ts < 2; ++ts)
            for (int act : {(int)ACT_NONE, (int)ACT_GELU_TANH}) {
                Q8Plan p = plan_q8(rows, cols, red, sms, ts == 1, act);
                if (p.split.splits > 1) part = std::max(part, (size_t)p.split.splits * rows * cols * 4);
            }
    };
    if (M > 0) {
        if (r > 0) sk_part(M, K);  // A*x (forward, or recompute in the backward)
        if (pass == REELS_PASS_FORWARD) {
            q8_part(M, N, K);
        } else {
            if (r > 0) {
                sk_part(M, N);  // B'*dy
                sk_part(K, M);  // dA
                sk_part(N, M);  // dB
                const DualPlan d = plan_dual(M, N, r, sms);  // G and dB in one pass over dy
                if (d.use) part = std::max(part, align256((size_t)d.part_g) + (size_t)d.part_db);
            }
            q8_part(M, K, N);
        }
    }
    w.part = off;
    off += align256(part);
    w.total = off;
    return w;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_common(int64_t M, int64_t K, int64_t N, int64_t r, int dt, int layout) {
    if (M < 0 || K <= 0 || N <= 0) return fail("dimensions must be positive (M may be 0)");
    if (r < 0 || r > 256) return fail("LoRA rank must be in [0, 256]");
    if (dt != REELS_F32 && dt != REELS_F16 && dt != REELS_BF16) return fail("unknown activation dtype");
    if (layout != REELS_W_OUT_CONTIGUOUS && layout != REELS_W_IN_CONTIGUOUS) return fail("unknown weight layout");
    if (K > INT32_MAX / 2 || N > INT32_MAX / 2 || M > INT32_MAX / 2) return fail("dimension too large");
    return REELS_OK;
}

int launch_grid(int64_t total) { return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(total, 256), 148 * 16)); }

// -------------------------------------------------------- tensor-core ops
// D[rows][r] = act[rows][red] . Bop[r][red]^T  (A-op K-major), or
// D[rows][r] = act[red][rows]^T . Bop[r][red]^T (A-op MN-major), epilogue epi.
struct SkCall {
    const void *act;     // 16-bit activation tensor
    int64_t act_inner;   // contiguous extent of act
    int64_t act_outer;
    bool a_mn;
    const void *bop;     // 16-bit [r][red], row pitch bop_pitch elements
    int64_t bop_pitch;
    int64_t rows, red, r;
    int epi_final;       // 0 transposed store, 1 fp32 accumulate
    float alpha;
    int accumulate;
    void *out;
    int64_t ldo, rs, cs;
};

// The reduction's vector path (four consecutive outputs per lane, float4
// partial loads): few splits, rows-contiguous partials and outputs whose
// four-row groups are aligned (8 B for 16-bit stores, 16 B for fp32).
int red_vec_ok(const RedJob &j) {
    if (!j.pcol || j.splits > RED_VEC_MAX || j.rows % 4 != 0) return 0;
    const uintptr_t o = reinterpret_cast<uintptr_t>(j.out);
    if (j.epi == 0) return (o % 8 == 0 && j.ldo % 4 == 0) ? 1 : 0;
    return (j.rs == 1 && o % 16 == 0 && j.cs % 4 == 0) ? 1 : 0;
}

int run_sk(const SkCall &c, int dt, const DeviceState &ds, char *ws_base, const Ws &wl, cudaStream_t st) {
    CUtensorMap ta, tb;
    int rc;
    const uint64_t pitch = (uint64_t)c.act_inner * 2;
    if (c.a_mn) rc = tmap_2d(&ta, c.act, tma_act_type(dt), c.act_inner, c.act_outer, pitch, 64, 64,
                             CU_TENSOR_MAP_SWIZZLE_128B);
    else rc = tmap_2d(&ta, c.act, tma_act_type(dt), c.act_inner, c.act_outer, pitch, 64, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const int np = npad_of(c.r);
    rc = tmap_2d(&tb, c.bop, tma_act_type(dt), c.red, c.r, (uint64_t)c.bop_pitch * 2, 64, np,
                 CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    Split s = plan_sk(c.rows, c.red, ds.sms, c.r);
    SkArgs a;
    a.rows = (int)c.rows;
    a.kb_total = (int)cdiv(c.red, BK);
    a.kb_per_split = s.kb_per;
    a.npad = np;
    a.a_mn = c.a_mn ? 1 : 0;
    a.ncols = (int)c.r;
    a.alpha = c.alpha;
    a.accumulate = c.accumulate;
    a.out = c.out;
    a.ldo = c.ldo;
    a.rs = c.rs;
    a.cs = c.cs;
    a.partial = reinterpret_cast<float *>(ws_base + wl.part);
    a.err = ds.status;
    a.epi = s.splits > 1 ? 2 : c.epi_final;
    a.splits = s.splits;
    // split partials follow the output's contiguous dimension
    a.pcol = (c.epi_final == 0 || c.rs == 1) ? 1 : 0;
    // persistent CTAs, one per SM at most (200 KB of ring each)
    const dim3 grid((unsigned)std::min<int64_t>(cdiv(c.rows, 128) * s.splits, ds.sms));
    if (dt == REELS_BF16) launch_pdl(sk_gemm_kernel<DT_BF16>, dim3(grid), dim3(SK_THREADS), SK_SMEM_BYTES, st, ta, tb, a);
    else launch_pdl(sk_gemm_kernel<DT_F16>, dim3(grid), dim3(SK_THREADS), SK_SMEM_BYTES, st, ta, tb, a);
    REELS_LAUNCHED();
    if (s.splits > 1) {
        RedJob j{a.partial, s.splits, c.rows, np, (int)c.r, c.epi_final, c.alpha, c.accumulate, c.out,
                 c.ldo, c.rs, c.cs, a.pcol, 0};
        j.vec = red_vec_ok(j);
        launch_pdl(sk_reduce_kernel, dim3(launch_grid(c.rows * c.r * 4)), dim3(256), 0, st, j, j, 1, dt);
        REELS_LAUNCHED();
    }
    return REELS_OK;
}

// G = s*(B'*dy) into gbuf ([r][ldm], 16-bit) and dB = alpha_db * T*dy (fp32
// [r][N], accumulated when asked) from one pass over dy (sk_dual_kernel), then
// one reduce launch for whichever of the two was split.
int run_dual(const DualPlan &d, const void *dy, const void *B, const void *tbuf, int64_t M, int64_t N, int64_t r,
             float s, float alpha_db, int accumulate, void *gbuf, float *dB, int dt, const DeviceState &ds,
             char *ws_base, const Ws &wl, cudaStream_t st) {
    CUtensorMap tdy, tb, tt;
    const int np = npad_of(r);
    const int64_t ldm = ld_tokens(M);
    int rc = tmap_2d(&tdy, dy, tma_act_type(dt), N, M, (uint64_t)N * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = tmap_2d(&tb, B, tma_act_type(dt), N, r, (uint64_t)N * 2, 64, np, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = tmap_2d(&tt, tbuf, tma_act_type(dt), M, r, (uint64_t)ldm * 2, 64, np, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (align256((size_t)d.part_g) + (size_t)d.part_db > wl.total - wl.part)
        return fail("workspace partial region too small for the one-pass dy plan");
    SkDualArgs a;
    a.M = (int)M;
    a.N = (int)N;
    a.tm_tiles = (int)cdiv(M, 128);
    a.tn_tiles = (int)cdiv(N, 128);
    a.splits_m = d.splits_m;
    a.splits_n = d.splits_n;
    a.npad = np;
    a.ncols = (int)r;
    a.tmem_cols = d.tmem_cols;
    a.g_out = gbuf;
    a.ldm = ldm;
    a.g_alpha = s;
    float *part = reinterpret_cast<float *>(ws_base + wl.part);
    a.g_part = part;
    a.db_out = dB;
    a.db_alpha = alpha_db;
    a.accumulate = accumulate;
    a.db_part = reinterpret_cast<float *>(reinterpret_cast<char *>(part) + align256((size_t)d.part_g));
    a.err = ds.status;
    const dim3 grid((unsigned)(d.splits_m * d.splits_n));
    if (dt == REELS_BF16) launch_pdl(sk_dual_kernel<DT_BF16>, grid, dim3(SK_THREADS), DU_SMEM_BYTES, st, tdy, tb, tt, a);
    else launch_pdl(sk_dual_kernel<DT_F16>, grid, dim3(SK_THREADS), DU_SMEM_BYTES, st, tdy, tb, tt, a);
    REELS_LAUNCHED();
    RedJob jobs[2];
    int n = 0;
    if (d.splits_n > 1) jobs[n++] = RedJob{a.g_part, d.splits_n, M, np, (int)r, 0, s, 0, gbuf, ldm, 0, 0, 1, 0};
    if (d.splits_m > 1) jobs[n++] = RedJob{a.db_part, d.splits_m, N, np, (int)r, 1, alpha_db, accumulate, dB, 0, 1, N, 1, 0};
    for (int i = 0; i < n; ++i) jobs[i].vec = red_vec_ok(jobs[i]);
    if (n > 0) {
        const int64_t outs = (n > 1 ? M + N : (d.splits_n > 1 ? M : N)) * r;
        launch_pdl(sk_reduce_kernel, dim3(launch_grid(outs * 4)), dim3(256), 0, st, jobs[0], jobs[n - 1], n, dt);
        REELS_LAUNCHED();
    }
    return REELS_OK;
}

// Q8 GEMM: D[M][Nout] over reduction Kred of act[M][Kred] and the int8 weight,
// plus the LoRA extension.  `fwd` selects the weight orientation.
// Prepared LoRA operand of the q8 GEMM's extension blocks (rows or columns
// past r are zero):  forward  E[j][n] = B[j][n] * s (/ scale[n] when the
//                     column scale is applied in the epilogue), [rp][N]
//                     dX       E[k][j] = A[k][j],                  [K][rp]
template <typename T>
__global__ void prep_ext_fwd_kernel(const T *B, const float *scales, float s, int divide,
                                    int64_t r, int64_t rp, int64_t N, T *__restrict__ out) {
    griddep_wait();
    const int64_t total = rp * N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i / N, n = i % N;
        float v = 0.0f;
        if (j < r) {
            v = to_f32(B[j * N + n]) * s;
            if (divide) v = v / scales[n];
        }
        out[i] = Elem<std::is_same<T, __half>::value ? DT_F16 : DT_BF16>::from_f(v);
    }
}

// The LoRA operands of one pass in a single launch.  Blocks [0, nb_ext)
// write the weight-in-TMEM kernel's extension operand:
//   ext_kind 0 (forward): E[n][j] = B[j][n] * s (/ scale[n]), [nrows = N][rp];
//     a block transposes 32 output columns through shared memory (B read
//     along n, E written along j);
//   ext_kind 1 (dX):      E[k][j] = A[k][j], [nrows = K][rp], eight ranks per
//     thread and one 16-byte store;
// columns j >= r are zero.  The other blocks write At = A^T [r][K], the
// rank-down GEMM's operand (none when gridDim.x == nb_ext).
template <typename T>
__global__ void prep_lora_kernel(int ext_kind, const T *B, const float *scales, float s, int divide, int r, int rp,
                                 int nrows, T *__restrict__ ext, int nb_ext, const uint16_t *A, int K,
                                 uint16_t *__restrict__ At) {
    griddep_wait();
    __shared__ float tile[128][33];
    if ((int)blockIdx.x < nb_ext) {
        if (ext_kind == 0) {
            const int n0 = blockIdx.x * 32;
            for (int jb = 0; jb < rp; jb += 128) {
                for (int e = threadIdx.x; e < 128 * 32; e += blockDim.x) {
                    const int jj = e >> 5, nn = e & 31;
                    const int j = jb + jj, n = n0 + nn;
                    float v = 0.0f;
                    if (j < r && n < nrows) {
                        v = to_f32(B[(int64_t)j * nrows + n]) * s;
                        if (divide) v = v / scales[n];
                    }
                    tile[jj][nn] = v;
                }
                __syncthreads();
                const int jw = min(128, rp - jb);
                for (int e = threadIdx.x; e < 32 * jw; e += blockDim.x) {
                    const int nn = e / jw, jj = e - nn * jw;
                    const int n = n0 + nn;
                    if (n < nrows)
                        ext[(int64_t)n * rp + jb + jj] =
                            Elem<std::is_same<T, __half>::value ? DT_F16 : DT_BF16>::from_f(tile[jj][nn]);
                }
                __syncthreads();
            }
        } else {
            const uint16_t *a16 = A;
            uint16_t *e16 = reinterpret_cast<uint16_t *>(ext);
            const int per_row = rp / 8;
            const int total = nrows * per_row;
            for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += nb_ext * blockDim.x) {
                const int k = i / per_row, j0 = (i - k * per_row) * 8;
                uint16_t v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = (j0 + u < r) ? a16[(int64_t)k * r + j0 + u] : (uint16_t)0;
                uint4 w;
                w.x = v[0] | ((uint32_t)v[1] << 16);
                w.y = v[2] | ((uint32_t)v[3] << 16);
                w.z = v[4] | ((uint32_t)v[5] << 16);
                w.w = v[6] | ((uint32_t)v[7] << 16);
                *reinterpret_cast<uint4 *>(e16 + (int64_t)k * rp + j0) = w;
            }
        }
        return;
    }
    const int total = K * r;
    const int nb = gridDim.x - nb_ext;
    for (int i = (blockIdx.x - nb_ext) * blockDim.x + threadIdx.x; i < total; i += nb * blockDim.x) {
        const int j = i / K, k = i - j * K;
        At[i] = A[k * r + j];
    }
}

struct Q8Call {
    bool fwd;
    const void *act;   // [M][Kred]
    int64_t M, Nout, Kred;
    const int8_t *q;
    const float *scales;
    int layout;
    int64_t N_w, K_w;  // weight dims (out, in)
    int64_t r;
    const void *ext_act;  // [r][ldm] 16-bit
    const void *lora;     // fwd: B [r][N]; dX: A [K][r]
    float ext_scale;
    void *ext_buf;        // workspace for the prepared ext operand
    const void *bias;
    void *out;
    int epi_act = ACT_NONE;  // fused output activation (act.cuh)
    void *pre = nullptr;     // its rounded pre-activation [M][Nout]
    bool ext_ready = false;  // the weight-in-TMEM kernel's LoRA operand is already in ext_buf
};

template <int DT, int MT, int BN>
void launch_q8_t(dim3 grid, cudaStream_t st, const CUtensorMap &ta, const CUtensorMap &tw, const CUtensorMap &te,
                 const Q8Args &a) {
    launch_pdl(q8_gemm_kernel<DT, MT, BN>, dim3(grid), dim3(Q8_THREADS), Q8Geom<MT, BN>::SMEM_BYTES, st, ta, tw, te, a);
}

void launch_q8(int dt, int mt, int bn, dim3 grid, cudaStream_t st, const CUtensorMap &ta, const CUtensorMap &tw,
               const CUtensorMap &te, const Q8Args &a) {
    const int key = (dt == REELS_BF16 ? 100 : 0) + mt * 10 + (bn == 256 ? 1 : 0);
    switch (key) {
        case 110: launch_q8_t<DT_BF16, 1, 128>(grid, st, ta, tw, te, a); break;
        case 111: launch_q8_t<DT_BF16, 1, 256>(grid, st, ta, tw, te, a); break;
        case 120: launch_q8_t<DT_BF16, 2, 128>(grid, st, ta, tw, te, a); break;
        case 121: launch_q8_t<DT_BF16, 2, 256>(grid, st, ta, tw, te, a); break;
        case 10: launch_q8_t<DT_F16, 1, 128>(grid, st, ta, tw, te, a); break;
        case 11: launch_q8_t<DT_F16, 1, 256>(grid, st, ta, tw, te, a); break;
        case 20: launch_q8_t<DT_F16, 2, 128>(grid, st, ta, tw, te, a); break;
        default: launch_q8_t<DT_F16, 2, 256>(grid, st, ta, tw, te, a); break;
    }
}

template <int DT, int BT, int KB2>
void launch_ts_t(dim3 grid, cudaStream_t st, const CUtensorMap &tx, const CUtensorMap &tw, const CUtensorMap &te,
                 const CUtensorMap &tsc, const CUtensorMap &to, const CUtensorMap &tp, const TsArgs &a) {
    // The activation variant only when the kernel writes the output itself
    // (split partials leave the activation to the reduce).
    using G = TsGeom<BT, KB2>;
    const int act = a.epi_partial ? ACT_NONE : a.epi_act;
    if (act == ACT_GELU_TANH)
        launch_pdl(q8ts_gemm_kernel<DT, BT, KB2, ACT_GELU_TANH>, dim3(grid), dim3(G::THREADS), G::SMEM_BYTES, st, tx,
                   tw, te, tsc, to, tp, a);
    else if (act == ACT_GELU_TANH_GRAD)
        launch_pdl(q8ts_gemm_kernel<DT, BT, KB2, ACT_GELU_TANH_GRAD>, dim3(grid), dim3(G::THREADS), G::SMEM_BYTES,
                   st, tx, tw, te, tsc, to, tp, a);
    else
        launch_pdl(q8ts_gemm_kernel<DT, BT, KB2, ACT_NONE>, dim3(grid), dim3(G::THREADS), G::SMEM_BYTES, st, tx, tw,
                   te, tsc, to, tp, a);
}
template <int DT, int BT, int KB2>
void launch_ts_pair_t(dim3 grid, cudaStream_t st, const CUtensorMap &tx, const CUtensorMap &tw,
                      const CUtensorMap &te, const CUtensorMap &tsc, const CUtensorMap &to, const CUtensorMap &tp,
                      const TsArgs &a) {
    using G = TsGeom<BT, KB2, 1>;
    const int act = a.epi_partial ? ACT_NONE : a.epi_act;
    if (act == ACT_GELU_TANH)
        launch_pdl_cluster(q8ts_gemm_kernel<DT, BT, KB2, ACT_GELU_TANH, 1>, grid, dim3(G::THREADS), G::SMEM_BYTES,
                           st, 2, tx, tw, te, tsc, to, tp, a);
    else if (act == ACT_GELU_TANH_GRAD)
        launch_pdl_cluster(q8ts_gemm_kernel<DT, BT, KB2, ACT_GELU_TANH_GRAD, 1>, grid, dim3(G::THREADS),
                           G::SMEM_BYTES, st, 2, tx, tw, te, tsc, to, tp, a);
    else
        launch_pdl_cluster(q8ts_gemm_kernel<DT, BT, KB2, ACT_NONE, 1>, grid, dim3(G::THREADS), G::SMEM_BYTES, st, 2,
                           tx, tw, te, tsc, to, tp, a);
}

// Profiling hook shared by both q8 launch paths: events around the GEMM.
cudaEvent_t prof_begin(cudaStream_t st, const Q8Call &c) {
    if (!t_prof.on) return nullptr;
    if (t_prof.used == t_prof.pool.size()) {
        cudaEvent_t a, b;
        if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess) return nullptr;
        t_prof.pool.emplace_back(a, b);
    }
    auto &pr = t_prof.pool[t_prof.used++];
    cudaEventRecord(pr.first, st);
    t_prof.flops += 2.0 * (double)c.M * (double)c.Nout * (double)(c.Kred + c.r);
    return pr.second;
}

int prep_lora(int dt, int ext_kind, const void *B, const float *scales, float s, bool divide, int64_t r, int64_t rp,
              int64_t nrows, void *ext, const void *A, int64_t K, void *at, cudaStream_t st);

// The weight-in-TMEM kernel (q8ts_gemm.cuh).
int run_q8_ts(const Q8Call &c, int dt, const DeviceState &ds, char *ws_base, const Ws &wl, cudaStream_t st,
              const Q8Plan &p) {
    const int bt = p.ts;
    const int sk = 64 * p.ts_kb2;  // reduction elements per pipeline stage
    CUtensorMap tx, tw, te, tsc, to, tp;
    // a CTA of a pair loads half of the token tile
    int rc = tmap_2d(&tx, c.act, tma_act_type(dt), c.Kred, c.M, (uint64_t)c.Kred * 2, 64, p.pair ? bt / 2 : bt,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const uint64_t w_inner = c.layout == REELS_W_OUT_CONTIGUOUS ? c.N_w : c.K_w;
    const uint64_t w_outer = c.layout == REELS_W_OUT_CONTIGUOUS ? c.K_w : c.N_w;
    const bool inner_is_red = c.fwd ? (c.layout == REELS_W_IN_CONTIGUOUS) : (c.layout == REELS_W_OUT_CONTIGUOUS);
    // Rows of output columns carry sk reduction bytes (64B swizzle for 64,
    // 128B for 128); rows of reduction indices carry 128 output-column bytes
    // (128B swizzle), sk of them.
    if (inner_is_red)
        rc = tmap_2d(&tw, c.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_inner, w_outer, w_inner, sk, 128,
                     sk == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
    else
        rc = tmap_2d(&tw, c.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_inner, w_outer, w_inner, 128, sk,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const int64_t ldm = ld_tokens(c.M);
    if (c.r > 0) {
        rc = tmap_2d(&te, c.ext_act, tma_act_type(dt), c.M, c.r, (uint64_t)ldm * 2, 64, 64,
                     CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    } else {
        te = tx;
    }
    TsArgs a;
    memset(&a, 0, sizeof a);
    a.M = (int)c.M;
    a.Nout = (int)c.Nout;
    a.kb_total = (int)cdiv(c.Kred, sk);
    a.kb_per_split = p.split.kb_per;
    a.splits = p.split.splits;
    a.ntiles = (int)p.ntiles;
    a.mtiles = (int)p.mtiles;
    a.w_rows_red = inner_is_red ? 0 : 1;
    a.wscale = c.scales;
    a.wscale_len = (int)c.N_w;
    bool ext_divide = false;
    if (c.fwd) {
        // bf16: exact int8 in the MMA, scale per output column in the epilogue;
        // fp16: scale in the dequant (keeps B*s in fp16 range).
        if (dt == REELS_BF16) {
            a.scale_mode = 0;
            a.col_scale = c.scales;
            ext_divide = true;
        } else {
            a.scale_mode = 1;
        }
    } else {
        a.scale_mode = 2;  // dX: the scale sits on the reduction index
    }
    if (a.scale_mode == 2) {
        rc = tmap_2d(&tsc, c.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, c.N_w, 1, (uint64_t)round_up(c.N_w * 4, 16),
                     sk, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    } else {
        tsc = tx;
    }
    a.r = (int)c.r;
    if (c.r > 0 && c.ext_ready) {
        a.ext_w = c.ext_buf;
        a.ext_ld = (int)ts_rank_pad(c.r);
    } else if (c.r > 0) {
        a.ext_w = c.ext_buf;
        a.ext_ld = (int)ts_rank_pad(c.r);
        const int64_t rp = ts_rank_pad(c.r);
        rc = c.fwd ? prep_lora(dt, 0, c.lora, c.scales, c.ext_scale, ext_divide, c.r, rp, c.Nout, c.ext_buf, nullptr,
                               0, nullptr, st)
                   : prep_lora(dt, 1, nullptr, c.scales, 1.0f, false, c.r, rp, c.Nout, c.ext_buf, c.lora, 0, nullptr,
                               st);
        if (rc) return rc;
    }
    a.bias = c.bias;
    a.out = c.out;
    a.ldo = c.Nout;
    a.partial = reinterpret_cast<float *>(ws_base + wl.part);
    a.epi_partial = p.split.splits > 1 ? 1 : 0;
    a.err = ds.status;
    a.epi_act = c.epi_act;
    a.pre = c.pre;
    {
        // 128-token tiles: a second MMA issuer (q8ts_gemm.cuh), when every CTA
        // runs one work unit (with more, the two accumulators serve to overlap
        // a tile's epilogue with the next tile's MMAs) and every unit has two
        // stages or more (each issuer's accumulator gets at least one).
        // REELS_Q8_ISS2=0 keeps one issuer (for measurements).
        const int n_ext = c.r > 0 ? (int)cdiv(c.r, sk) : 0;
        const int last_main = a.kb_total - a.kb_per_split * (a.splits - 1);
        a.iss2 = (bt == 128 && q8_iss2_ok(p, ds.sms) && a.kb_per_split >= 2 && last_main + n_ext >= 2) ? 1 : 0;
    }
    tp = tx;
    if (!a.epi_partial) {
        // D tiles of 32 columns x 32 tokens, stored from the epilogue's staging.
        rc = tmap_2d(&to, c.out, tma_act_type(dt), c.Nout, c.M, (uint64_t)c.Nout * 2, 32, 32,
                     CU_TENSOR_MAP_SWIZZLE_64B);
        if (rc) return rc;
        if (c.epi_act != ACT_NONE && c.pre) {
            rc = tmap_2d(&tp, c.pre, tma_act_type(dt), c.Nout, c.M, (uint64_t)c.Nout * 2, 32, 32,
                         CU_TENSOR_MAP_SWIZZLE_64B);
            if (rc) return rc;
        }
    } else {
        to = tx;
    }
    const int64_t total_tiles = p.ntiles * p.mtiles * p.split.splits;
    const dim3 grid(p.pair ? 2u * (unsigned)std::min<int64_t>(total_tiles, ds.sms / 2)
                           : (unsigned)std::min<int64_t>(total_tiles, ds.sms));
    cudaEvent_t ev_stop = prof_begin(st, c);
    const int key = (dt == REELS_BF16 ? 10000 : 0) + bt * 10 + p.ts_kb2;
    if (p.pair) {
        switch (key) {
            case 12562: launch_ts_pair_t<DT_BF16, 256, 2>(grid, st, tx, tw, te, tsc, to, tp, a); break;
            case 11282: launch_ts_pair_t<DT_BF16, 128, 2>(grid, st, tx, tw, te, tsc, to, tp, a); break;
            case 2562: launch_ts_pair_t<DT_F16, 256, 2>(grid, st, tx, tw, te, tsc, to, tp, a); break;
            case 1282: launch_ts_pair_t<DT_F16, 128, 2>(grid, st, tx, tw, te, tsc, to, tp, a); break;
            default: return fail("no CTA-pair variant of this tile plan");
        }
    } else switch (key) {
        case 12561: launch_ts_t<DT_BF16, 256, 1>(grid, st, tx, tw, te, tsc, to, tp, a); break;
        case 11921: launch_ts_t<DT_BF16, 192, 1>(grid, st, tx, tw, te, tsc, to, tp, a); break;
        case 11281: launch_ts_t<DT_BF16, 128, 1>(grid, st, tx, tw, te, tsc, to, tp, a); break;
        case 11282: launch_ts_t<DT_BF16, 128, 2>(grid, st, tx, tw, te, tsc, to, tp, a); break;
        case 12562: launch_ts_t<DT_BF16, 256, 2>(grid, st, tx, tw, te, tsc, to, tp, a); break;
        case 11922: launch_ts_t<DT_BF16, 192, 2>(grid, st, tx, tw, te, tsc, to, tp, a); break;
        case 2562: launch_ts_t<DT_F16, 256, 2>(grid, st, tx, tw, te, tsc, to, tp, a); break;
        case 1922: launch_ts_t<DT_F16, 192, 2>(grid, st, tx, tw, te, tsc, to, tp, a); break;
        case 2561: launch_ts_t<DT_F16, 256, 1>(grid, st, tx, tw, te, tsc, to, tp, a); break;
        case 1921: launch_ts_t<DT_F16, 192, 1>(grid, st, tx, tw, te, tsc, to, tp, a); break;
        case 1281: launch_ts_t<DT_F16, 128, 1>(grid, st, tx, tw, te, tsc, to, tp, a); break;
        default: launch_ts_t<DT_F16, 128, 2>(grid, st, tx, tw, te, tsc, to, tp, a); break;
    }
    REELS_LAUNCHED();
    if (ev_stop) REELS_CUDA(cudaEventRecord(ev_stop, st));
    if (p.split.splits > 1) {
        launch_pdl(q8_reduce_kernel, dim3(launch_grid(c.M * c.Nout / 4)), dim3(256), 0, st, a.partial, p.split.splits, c.M, c.Nout,
                                                                    a.col_scale, c.bias, dt, c.out, c.Nout, c.epi_act, c.pre);
        REELS_LAUNCHED();
    }
    return REELS_OK;
}

int run_q8(const Q8Call &c, int dt, const DeviceState &ds, char *ws_base, const Ws &wl, cudaStream_t st) {
    // The TMEM-weight kernel loads the reduction scales by TMA (16-byte aligned base).
    const bool ts_ok = aligned16(c.scales);
    Q8Plan p = plan_q8(c.M, c.Nout, c.Kred, ds.sms, ts_ok, c.epi_act);
    if (p.ts) return run_q8_ts(c, dt, ds, ws_base, wl, st, p);
    if (c.epi_act != ACT_NONE) {
        // The SMEM-operand kernels have no activation epilogue: the GEMM
        // writes the linear's output (gelu: into `pre` when given), then one
        // elementwise pass applies the activation or its derivative.
        Q8Call plain = c;
        plain.epi_act = ACT_NONE;
        plain.pre = nullptr;
        if (c.epi_act == ACT_GELU_TANH && c.pre) plain.out = c.pre;
        int rc = run_q8(plain, dt, ds, ws_base, wl, st);
        if (rc) return rc;
        const void *h = c.epi_act == ACT_GELU_TANH ? plain.out : c.pre;
        launch_pdl(act_apply_kernel, dim3(launch_grid(c.M * c.Nout)), dim3(256), 0, st, c.epi_act, dt,
                   c.M * c.Nout, c.out, h);
        REELS_LAUNCHED();
        return REELS_OK;
    }
    CUtensorMap ta, tw, te;
    const int a_rows = 128 * p.mt;
    const int w_box = p.bn;
    int rc = tmap_2d(&ta, c.act, tma_act_type(dt), c.Kred, c.M, (uint64_t)c.Kred * 2, 64, a_rows,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    // Weight tensor as stored: layout 0 is [K][N] (inner N), layout 1 is [N][K] (inner K).
    const uint64_t w_inner = c.layout == REELS_W_OUT_CONTIGUOUS ? c.N_w : c.K_w;
    const uint64_t w_outer = c.layout == REELS_W_OUT_CONTIGUOUS ? c.K_w : c.N_w;
    // Orientation 0 (staging rows = D columns) when the weight's contiguous
    // dimension is the reduction: forward on [N][K], dX on [K][N].
    const bool inner_is_red = c.fwd ? (c.layout == REELS_W_IN_CONTIGUOUS) : (c.layout == REELS_W_OUT_CONTIGUOUS);
    const int orient = inner_is_red ? 0 : 1;
    if (orient == 0) rc = tmap_2d(&tw, c.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_inner, w_outer, w_inner, 64, w_box,
                                  CU_TENSOR_MAP_SWIZZLE_NONE);
    else rc = tmap_2d(&tw, c.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_inner, w_outer, w_inner, w_box, 64,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    const int64_t ldm = ld_tokens(c.M);
    if (c.r > 0) {
        rc = tmap_2d(&te, c.ext_act, tma_act_type(dt), c.M, c.r, (uint64_t)ldm * 2, 64, 64,
                     CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
    } else {
        te = ta;
    }
    Q8Args a;
    memset(&a, 0, sizeof a);
    a.M = (int)c.M;
    a.Nout = (int)c.Nout;
    a.kb_total = (int)cdiv(c.Kred, BK);
    a.kb_per_split = p.split.kb_per;
    a.splits = p.split.splits;
    a.ntiles = (int)p.ntiles;
    a.mtiles = (int)p.mtiles;
    a.w_orient = orient;
    a.wscale = c.scales;
    a.wscale_len = (int)c.N_w;
    bool ext_divide = false;
    if (c.fwd) {
        // bf16: exact int8 in the MMA, per-column scale in the epilogue.
        // fp16: scale folded into the dequant (keeps B*s in fp16 range).
        if (dt == REELS_BF16) {
            a.scale_mode = 0;
            a.col_scale = c.scales;
            ext_divide = true;
        } else {
            a.scale_mode = orient == 0 ? 1 : 2;
            a.col_scale = nullptr;
        }
        a.ext_kind = 0;
    } else {
        // dX: the scale sits on the reduction index n.
        a.scale_mode = orient == 1 ? 1 : 2;
        a.col_scale = nullptr;
        a.ext_kind = 1;
    }
    a.r = (int)c.r;
    if (c.r > 0) {
        const int64_t rp = rank_pad(c.r);
        a.ext_w = c.ext_buf;
        if (c.fwd) {
            a.ext_ld = (int)c.Nout;
            if (dt == REELS_BF16)
                launch_pdl(prep_ext_fwd_kernel<__nv_bfloat16>, dim3(launch_grid(rp * c.Nout)), dim3(256), 0, st, 
                    (const __nv_bfloat16 *)c.lora, c.scales, c.ext_scale, ext_divide ? 1 : 0, c.r, rp, c.Nout,
                    (__nv_bfloat16 *)c.ext_buf);
            else
                launch_pdl(prep_ext_fwd_kernel<__half>, dim3(launch_grid(rp * c.Nout)), dim3(256), 0, st, 
                    (const __half *)c.lora, c.scales, c.ext_scale, 0, c.r, rp, c.Nout, (__half *)c.ext_buf);
        } else {
            a.ext_ld = (int)rp;
            int rc2 = prep_lora(dt, 1, nullptr, c.scales, 1.0f, false, c.r, rp, c.Nout, c.ext_buf, c.lora, 0, nullptr,
                                st);
            if (rc2) return rc2;
        }
        if (c.fwd) REELS_LAUNCHED();
    }
    a.bias = c.bias;
    a.out = c.out;
    a.ldo = c.Nout;
    a.out_v8 = (reinterpret_cast<uintptr_t>(c.out) & 31u) == 0 ? 1 : 0;
    a.partial = reinterpret_cast<float *>(ws_base + wl.part);
    a.epi_partial = p.split.splits > 1 ? 1 : 0;
    a.err = ds.status;
    const int64_t total_tiles = p.ntiles * p.mtiles * p.split.splits;
    dim3 grid((unsigned)std::min<int64_t>(total_tiles, ds.sms));
    cudaEvent_t ev_stop = prof_begin(st, c);
    launch_q8(dt, p.mt, p.bn, grid, st, ta, tw, te, a);
    REELS_LAUNCHED();
    if (ev_stop) REELS_CUDA(cudaEventRecord(ev_stop, st));
    if (p.split.splits > 1) {
        launch_pdl(q8_reduce_kernel, dim3(launch_grid(c.M * c.Nout / 4)), dim3(256), 0, st, a.partial, p.split.splits, c.M, c.Nout,
                                                                    a.col_scale, c.bias, dt, c.out, c.Nout, c.epi_act, c.pre);
        REELS_LAUNCHED();
    }
    return REELS_OK;
}

bool tc_eligible(int64_t K, int64_t N, int dt, std::initializer_list<const void *> ptrs) {
    if (dt == REELS_F32) return false;
    if (K % 16 != 0 || N % 16 != 0) return false;
    for (const void *p : ptrs)
        if (p && !aligned16(p)) return false;
    return true;
}

int check_ws(void *ws, size_t ws_bytes, const Ws &wl) {
    if (wl.total == 0) return REELS_OK;
    if (!ws) return fail("workspace is NULL; size it with reels_q8lora_workspace_bytes");
    if (ws_bytes < wl.total)
        return fail("workspace too small: need " + std::to_string(wl.total) + " bytes, got " +
                    std::to_string(ws_bytes));
    if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return fail("workspace must be 256-byte aligned");
    return REELS_OK;
}

// A [K][r] -> At [r][K]
int transpose_rank(const void *A, int64_t K, int64_t r, void *At, cudaStream_t st) {
    launch_pdl(transpose_rank_kernel, dim3(launch_grid(K * r)), dim3(256), 0, st, reinterpret_cast<const uint16_t *>(A), (int)K, (int)r,
                                                              reinterpret_cast<uint16_t *>(At));
    REELS_LAUNCHED();
    return REELS_OK;
}

int rank_down_tc(const void *x, const void *A, int64_t M, int64_t K, int64_t r, int dt, void *tbuf, void *at,
                 const DeviceState &ds, char *ws, const Ws &wl, cudaStream_t st, bool at_ready = false) {
    if (!at_ready) {
        int rc = transpose_rank(A, K, r, at, st);
        if (rc) return rc;
    }
    SkCall c{};
    c.act = x;
    c.act_inner = K;
    c.act_outer = M;
    c.a_mn = false;
    c.bop = at;
    c.bop_pitch = K;
    c.rows = M;
    c.red = K;
    c.r = r;
    c.epi_final = 0;
    c.alpha = 1.0f;
    c.out = tbuf;
    c.ldo = ld_tokens(M);
    return run_sk(c, dt, ds, ws, wl, st);
}

// One launch of prep_lora_kernel: the extension operand of a weight-in-TMEM
// q8 GEMM (ext != nullptr) and/or A^T (at != nullptr).
int prep_lora(int dt, int ext_kind, const void *B, const float *scales, float s, bool divide, int64_t r, int64_t rp,
              int64_t nrows, void *ext, const void *A, int64_t K, void *at, cudaStream_t st) {
    const int nb_ext = ext ? (ext_kind == 0 ? (int)cdiv(nrows, 32) : launch_grid(nrows * rp / 8)) : 0;
    const int nb_at = at ? launch_grid(K * r) : 0;
    if (nb_ext + nb_at == 0) return REELS_OK;
    const dim3 grid((unsigned)(nb_ext + nb_at));
    if (dt == REELS_BF16)
        launch_pdl(prep_lora_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, ext_kind, (const __nv_bfloat16 *)B,
                   scales, s, divide ? 1 : 0, (int)r, (int)rp, (int)nrows, (__nv_bfloat16 *)ext, nb_ext,
                   (const uint16_t *)A, (int)K, (uint16_t *)at);
    else
        launch_pdl(prep_lora_kernel<__half>, grid, dim3(256), 0, st, ext_kind, (const __half *)B, scales, s,
                   divide ? 1 : 0, (int)r, (int)rp, (int)nrows, (__half *)ext, nb_ext, (const uint16_t *)A, (int)K,
                   (uint16_t *)at);
    REELS_LAUNCHED();
    return REELS_OK;
}

}  // namespace

// Calls f with the element type as a compile-time constant.
template <typename F>
void dispatch_dt(int dt, F &&f) {
    if (dt == REELS_BF16) f(std::integral_constant<int, DT_BF16>{});
    else if (dt == REELS_F16) f(std::integral_constant<int, DT_F16>{});
    else f(std::integral_constant<int, DT_F32>{});
}

// =====================================================================
extern "C" {

const char *reels_lowvram_last_error(void) { return t_last_error.c_str(); }
int reels_lowvram_abi_version(void) { return REELS_LOWVRAM_ABI_VERSION; }
int reels_lowvram_last_path(void) { return t_last_path; }

static int current_sms() {
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) sms = v;
    } else {
        cudaGetLastError();
    }
    return sms;
}

int reels_q8_plan(int64_t M, int64_t Nout, int64_t Kred, int act, int sms, int64_t *info) {
    if (!info) return fail("null info");
    if (M <= 0 || Nout <= 0 || Kred <= 0) return fail("plan needs positive M, Nout and Kred");
    if (act != REELS_ACT_NONE && act != REELS_ACT_GELU_TANH) return fail("unknown activation");
    const Q8Plan p = plan_q8(M, Nout, Kred, sms > 0 ? sms : current_sms(), true,
                             act == REELS_ACT_NONE ? ACT_NONE : ACT_GELU_TANH);
    info[0] = p.ts ? (p.pair ? 2 : 1) : 0;
    info[1] = p.ts ? p.ts : 128 * p.mt;
    info[2] = p.ts ? 64 * p.ts_kb2 : BK;
    info[3] = p.split.splits;
    info[4] = p.split.kb_per;
    info[5] = p.ntiles;
    info[6] = p.mtiles;
    return REELS_OK;
}

int reels_sk_plan(int64_t rows, int64_t red, int64_t r, int sms, int64_t *info) {
    if (!info) return fail("null info");
    if (rows <= 0 || red <= 0 || r <= 0 || r > 256) return fail("plan needs positive rows, red and 0 < r <= 256");
    const Split sp = plan_sk(rows, red, sms > 0 ? sms : current_sms(), r);
    info[0] = sp.splits;
    info[1] = sp.kb_per;
    return REELS_OK;
}

int reels_sk_dual_plan(int64_t M, int64_t N, int64_t r, int sms, int64_t *info) {
    if (!info) return fail("null info");
    if (M <= 0 || N <= 0 || r <= 0 || r > 256) return fail("plan needs positive M, N and 0 < r <= 256");
    const DualPlan d = plan_dual(M, N, r, sms > 0 ? sms : current_sms());
    info[0] = d.use ? 1 : 0;
    info[1] = d.splits_m;
    info[2] = d.splits_n;
    info[3] = d.tmem_cols;
    info[4] = d.part_g;
    info[5] = d.part_db;
    return REELS_OK;
}

int reels_lowvram_profile_enable(int enable) {
    t_prof.on = enable != 0;
    t_prof.used = 0;
    t_prof.flops = 0.0;
    t_launches = 0;
    return REELS_OK;
}

int reels_lowvram_profile_read(double *q8_ms, int64_t *q8_launches, double *q8_flops, int64_t *kernel_launches) {
    double total = 0.0;
    for (size_t i = 0; i < t_prof.used; ++i) {
        REELS_CUDA(cudaEventSynchronize(t_prof.pool[i].second));
        float ms = 0.0f;
        REELS_CUDA(cudaEventElapsedTime(&ms, t_prof.pool[i].first, t_prof.pool[i].second));
        total += ms;
    }
    if (q8_ms) *q8_ms = total;
    if (q8_launches) *q8_launches = (int64_t)t_prof.used;
    if (q8_flops) *q8_flops = t_prof.flops;
    if (kernel_launches) *kernel_launches = t_launches;
    t_prof.used = 0;
    t_prof.flops = 0.0;
    t_launches = 0;
    return REELS_OK;
}

int reels_lowvram_check_device_status(void *stream) {
    DeviceState *ds;
    DeviceScope scope;

    int rc = bind_device(nullptr, &ds, scope);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned h = 0, zero = 0;
    REELS_CUDA(cudaStreamSynchronize(st));
    REELS_CUDA(cudaMemcpy(&h, ds->status, 4, cudaMemcpyDeviceToHost));
    if (h) {
        REELS_CUDA(cudaMemcpy(ds->status, &zero, 4, cudaMemcpyHostToDevice));
        char buf[128];
        snprintf(buf, sizeof buf, "device status 0x%x: %s", h,
                 (h & DEVERR_OPT_TABLE) ? "an optimizer call on a workspace that reels_opt_prepare did not set up"
                                        : "a pipeline wait timed out");
        return fail_dev(buf);
    }
    t_last_error.clear();
    return REELS_OK;
}

int reels_q8_quantize(const void *w, int w_dtype, int layout, int64_t N, int64_t K, int8_t *q, float *scales,
                      void *stream) {
    if (!w || !q || !scales) return fail("null pointer passed to reels_q8_quantize");
    if (N <= 0 || K <= 0) return fail("weight dimensions must be positive");
    if (layout != REELS_W_OUT_CONTIGUOUS && layout != REELS_W_IN_CONTIGUOUS) return fail("unknown weight layout");
    if (w_dtype != REELS_F32 && w_dtype != REELS_F16 && w_dtype != REELS_BF16) return fail("unknown weight dtype");
    DeviceState *ds;
    DeviceScope scope;

    int rc = bind_device(w, &ds, scope);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    REELS_CUDA(cudaMemsetAsync(ds->quant_status, 0, 4, st));
    if (layout == REELS_W_OUT_CONTIGUOUS) {
        dim3 grid((unsigned)cdiv(N, 32));
        if (w_dtype == REELS_F32)
            quantize_outcontig_kernel<float><<<grid, 256, 0, st>>>((const float *)w, N, K, q, scales,
                                                                   ds->quant_status);
        else if (w_dtype == REELS_F16)
            quantize_outcontig_kernel<__half><<<grid, 256, 0, st>>>((const __half *)w, N, K, q, scales,
                                                                    ds->quant_status);
        else
            quantize_outcontig_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16 *)w, N, K, q,
                                                                           scales, ds->quant_status);
    } else {
        dim3 grid((unsigned)cdiv(N, 8));
        if (w_dtype == REELS_F32)
            quantize_incontig_kernel<float><<<grid, 256, 0, st>>>((const float *)w, N, K, q, scales,
                                                                  ds->quant_status);
        else if (w_dtype == REELS_F16)
            quantize_incontig_kernel<__half><<<grid, 256, 0, st>>>((const __half *)w, N, K, q, scales,
                                                                   ds->quant_status);
        else
            quantize_incontig_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16 *)w, N, K, q,
                                                                          scales, ds->quant_status);
    }
    REELS_LAUNCHED();
    unsigned h = 0;
    REELS_CUDA(cudaMemcpyAsync(&h, ds->quant_status, 4, cudaMemcpyDeviceToHost, st));
    REELS_CUDA(cudaStreamSynchronize(st));
    if (h & DEVERR_NONFINITE_WEIGHT) return fail("frozen weight contains non-finite values (NaN or Inf)");
    if (h & DEVERR_QUANT_NAN)
        return fail("a row's max|w| / 127 underflows to 0 while the row holds a zero: 0/0 is NaN, which Int8 "
                    "rejects (InexactError in quantize_frozen_matrix)");
    return ok(REELS_PATH_CUDACORE);
}

int reels_q8_materialize(const int8_t *q, const float *scales, int layout, int64_t N, int64_t K, int out_dtype,
                         void *out, void *stream) {
    if (!q || !scales || !out) return fail("null pointer passed to reels_q8_materialize");
    if (N <= 0 || K <= 0) return fail("weight dimensions must be positive");
    if (layout != REELS_W_OUT_CONTIGUOUS && layout != REELS_W_IN_CONTIGUOUS) return fail("unknown weight layout");
    if (out_dtype != REELS_F32 && out_dtype != REELS_F16 && out_dtype != REELS_BF16) return fail("unknown dtype");
    DeviceState *ds;
    DeviceScope scope;

    int rc = bind_device(q, &ds, scope);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    materialize_kernel<<<launch_grid(N * K), 256, 0, st>>>(q, scales, layout, N, K, out_dtype, out);
    REELS_LAUNCHED();
    return ok(REELS_PATH_CUDACORE);
}

size_t reels_q8lora_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r, int act_dtype, int pass) {
    if (M < 0 || K <= 0 || N <= 0 || r < 0) return 0;
    return ws_layout(M, K, N, r, act_dtype, pass, current_sms()).total;
}

size_t reels_q8lora_saved_bytes(int64_t M, int64_t r, int act_dtype) {
    if (M < 0 || r <= 0) return 0;
    return (size_t)r * ld_tokens(M) * esize(act_dtype);
}

static int check_dropout(float dropout, int64_t M) {
    if (!(dropout >= 0.0f && dropout < 1.0f)) return fail("dropout must be in [0, 1)");
    if (dropout > 0.0f && cdiv(M, DROP_TOK) > 65535) return fail("too many tokens for the dropout kernels");
    return REELS_OK;
}

// z = dropout(x) into the workspace (lora.jl:71-83)
static int launch_dropout_input(const void *x, int64_t n, int dt, float p, uint64_t key, void *z, cudaStream_t st) {
    launch_pdl(dropout_input_kernel, dim3(launch_grid(n)), dim3(256), 0, st, x, n, dt, p, key, z);
    REELS_LAUNCHED();
    return REELS_OK;
}

static int q8lora_forward_impl(const void *x, const int8_t *q, const float *scales, int layout, const void *A,
                               const void *B, const void *bias, int64_t M, int64_t K, int64_t N, int64_t r,
                               float alpha, int dt, int act, float dropout, uint64_t key, void *y, void *pre,
                               void *saved, void *workspace, size_t ws_bytes, void *stream) {
    int rc = check_common(M, K, N, r, dt, layout);
    if (rc) return rc;
    // With M == 0 the token-sized buffers (x, y, pre, saved) may be NULL.
    if (!q || !scales) return fail("null q or scales");
    if (M > 0 && (!x || !y)) return fail("null x or y");
    if (act != REELS_ACT_NONE && act != REELS_ACT_GELU_TANH) return fail("unknown activation");
    if (pre && pre == y) return fail("pre and y must be different buffers");
    if (r > 0 && (!A || !B)) return fail("null LoRA A or B");
    if (r > 0 && !std::isfinite(alpha)) return fail("alpha must be finite");
    rc = check_dropout(dropout, M);
    if (rc) return rc;
    if (M == 0) return ok(REELS_PATH_NONE);
    DeviceState *ds;
    DeviceScope scope;

    rc = bind_device(x, &ds, scope);
    if (rc) return rc;
    const bool drop = dropout > 0.0f && r > 0;
    const Ws wl = ws_layout(M, K, N, r, dt, REELS_PASS_FORWARD | (drop ? REELS_PASS_DROPOUT : 0), ds->sms);
    rc = check_ws(workspace, ws_bytes, wl);
    if (rc) return rc;
    if (saved && !aligned16(saved)) return fail("saved buffer must be 16-byte aligned");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    char *ws = reinterpret_cast<char *>(workspace);
    const float s = r > 0 ? alpha / (float)r : 0.0f;
    const int64_t ldm = ld_tokens(M);
    void *tbuf = r > 0 ? (saved ? saved : ws + wl.tbuf) : nullptr;
    // The adapter's input: x, or with dropout z = x * keep / (1 - p).
    const void *ax = x;
    if (drop) {
        rc = launch_dropout_input(x, M * K, dt, dropout, key, ws + wl.zbuf, st);
        if (rc) return rc;
        ax = ws + wl.zbuf;
    }

    if (tc_eligible(K, N, dt, {x, q, y, B, saved})) {
        // With the weight-in-TMEM plan, one launch prepares both LoRA
        // operands (A^T for the rank-down GEMM, the scaled B for the q8 GEMM).
        const int epi = act == REELS_ACT_GELU_TANH ? ACT_GELU_TANH : ACT_NONE;
        const bool ts_prep = r > 0 && plan_q8(M, N, K, ds->sms, aligned16(scales), epi).ts > 0;
        if (ts_prep) {
            rc = prep_lora(dt, 0, B, scales, s, dt == REELS_BF16, r, ts_rank_pad(r), N, ws + wl.ext, A, K, ws + wl.at,
                           st);
            if (rc) return rc;
        }
        if (r > 0) {
            rc = rank_down_tc(ax, A, M, K, r, dt, tbuf, ws + wl.at, *ds, ws, wl, st, ts_prep);
            if (rc) return rc;
        }
        Q8Call c{};
        c.fwd = true;
        c.act = x;
        c.M = M;
        c.Nout = N;
        c.Kred = K;
        c.q = q;
        c.scales = scales;
        c.layout = layout;
        c.N_w = N;
        c.K_w = K;
        c.r = r;
        c.ext_act = tbuf;
        c.lora = B;
        c.ext_scale = s;
        c.ext_buf = ws + wl.ext;
        c.bias = bias;
        c.out = y;
        c.epi_act = epi;
        c.pre = act == REELS_ACT_NONE ? nullptr : pre;
        c.ext_ready = ts_prep;
        rc = run_q8(c, dt, *ds, ws, wl, st);
        if (rc) return rc;
        return ok(REELS_PATH_TENSORCORE);
    }
    if (r > 0) {
        gen_rank_down_kernel<<<launch_grid(M * r), 256, 0, st>>>(ax, A, M, K, (int)r, dt, tbuf, ldm);
        REELS_LAUNCHED();
    }
    void *lin = act != REELS_ACT_NONE && pre ? pre : y;  // the linear's output
    gen_forward_kernel<<<launch_grid(M * N), 256, 0, st>>>(x, q, scales, layout, bias, tbuf, ldm, B, M, K, N,
                                                           (int)r, s, dt, lin);
    REELS_LAUNCHED();
    if (act != REELS_ACT_NONE) {
        act_apply_kernel<<<launch_grid(M * N), 256, 0, st>>>(ACT_GELU_TANH, dt, M * N, y, lin);
        REELS_LAUNCHED();
    }
    return ok(REELS_PATH_CUDACORE);
}

int reels_q8lora_forward(const void *x, const int8_t *q, const float *scales, int layout, const void *A,
                         const void *B, const void *bias, int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                         int dt, void *y, void *saved, void *workspace, size_t ws_bytes, void *stream) {
    return q8lora_forward_impl(x, q, scales, layout, A, B, bias, M, K, N, r, alpha, dt, REELS_ACT_NONE, 0.0f, 0, y,
                               nullptr, saved, workspace, ws_bytes, stream);
}

int reels_q8lora_forward_act(const void *x, const int8_t *q, const float *scales, int layout, const void *A,
                             const void *B, const void *bias, int64_t M, int64_t K, int64_t N, int64_t r,
                             float alpha, int act_dtype, int act, void *y, void *pre, void *saved, void *workspace,
                             size_t ws_bytes, void *stream) {
    return q8lora_forward_impl(x, q, scales, layout, A, B, bias, M, K, N, r, alpha, act_dtype, act, 0.0f, 0, y, pre,
                               saved, workspace, ws_bytes, stream);
}

int reels_q8lora_forward_dropout(const void *x, const int8_t *q, const float *scales, int layout, const void *A,
                                 const void *B, const void *bias, int64_t M, int64_t K, int64_t N, int64_t r,
                                 float alpha, int act_dtype, float dropout, uint64_t seed, uint64_t stream_id, void *y,
                                 void *saved, void *workspace, size_t ws_bytes, void *stream) {
    return q8lora_forward_impl(x, q, scales, layout, A, B, bias, M, K, N, r, alpha, act_dtype, REELS_ACT_NONE,
                               dropout, dropout_key(seed, stream_id), y, nullptr, saved, workspace, ws_bytes, stream);
}

int reels_q8_weight_mul(const void *x, const int8_t *q, const float *scales, int layout, const void *bias, int64_t M,
                        int64_t K, int64_t N, int act_dtype, void *y, void *workspace, size_t ws_bytes,
                        void *stream) {
    return reels_q8lora_forward(x, q, scales, layout, nullptr, nullptr, bias, M, K, N, 0, 1.0f, act_dtype, y,
                                nullptr, workspace, ws_bytes, stream);
}

static int q8lora_backward_impl(const void *x, const void *dy, const int8_t *q, const float *scales, int layout,
                                const void *A, const void *B, const void *saved, int64_t M, int64_t K, int64_t N,
                                int64_t r, float alpha, float grad_scale, int dt, int act, const void *pre_x,
                                float dropout, uint64_t key, void *dx, float *dA, float *dB, int accumulate,
                                void *workspace, size_t ws_bytes, void *stream) {
    int rc = check_common(M, K, N, r, dt, layout);
    if (rc) return rc;
    // With M == 0 the token-sized buffers (x, dy, pre_x, dx, saved) may be NULL.
    if (!q || !scales) return fail("null q or scales");
    if (M > 0 && !dy) return fail("null dy");
    if (act != REELS_ACT_NONE && act != REELS_ACT_GELU_TANH) return fail("unknown activation");
    if (act != REELS_ACT_NONE && dx && !pre_x) return fail("null pre-activation of x");
    if (act != REELS_ACT_NONE && dx && pre_x == dx) return fail("pre_x and dx must be different buffers");
    rc = check_dropout(dropout, M);
    if (rc) return rc;
    if (dropout > 0.0f && act != REELS_ACT_NONE) return fail("dropout is not combined with a fused activation");
    if (r > 0 && (!A || !B || !dA || !dB)) return fail("null A, B, dA or dB with r > 0");
    if (r > 0 && M > 0 && !x) return fail("null x with r > 0");
    if (r > 0 && !std::isfinite(alpha)) return fail("alpha must be finite");
    if (!std::isfinite(grad_scale)) return fail("grad_scale must be finite");
    if (!dx && r == 0) return ok(REELS_PATH_NONE);
    DeviceState *ds;
    DeviceScope scope;

    rc = bind_device(M > 0 ? dy : static_cast<const void *>(q), &ds, scope);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (M == 0) {
        // No tokens: gradients are zero (or unchanged when accumulating).
        if (r > 0 && !accumulate) {
            REELS_CUDA(cudaMemsetAsync(dA, 0, sizeof(float) * K * r, st));
            REELS_CUDA(cudaMemsetAsync(dB, 0, sizeof(float) * N * r, st));
        }
        return ok(REELS_PATH_NONE);
    }
    const bool drop = dropout > 0.0f && r > 0;
    const Ws wl = ws_layout(M, K, N, r, dt, REELS_PASS_BACKWARD | (drop ? REELS_PASS_DROPOUT : 0), ds->sms);
    rc = check_ws(workspace, ws_bytes, wl);
    if (rc) return rc;
    if (saved && !aligned16(saved)) return fail("saved buffer must be 16-byte aligned");
    char *ws = reinterpret_cast<char *>(workspace);
    const float s = r > 0 ? alpha / (float)r : 0.0f;
    const int64_t ldm = ld_tokens(M);
    const void *tbuf = r > 0 ? (saved ? saved : (const void *)(ws + wl.tbuf)) : nullptr;
    void *gbuf = r > 0 ? (void *)(ws + wl.gbuf) : nullptr;
    // The adapter's input of the forward: x, or with dropout z, recomputed
    // from the same key (the mask is a function of the key and the index).
    const void *ax = x;
    if (drop) {
        rc = launch_dropout_input(x, M * K, dt, dropout, key, ws + wl.zbuf, st);
        if (rc) return rc;
        ax = ws + wl.zbuf;
    }
    // With dropout the adapter's part of dx is masked, so the dx GEMM takes
    // the frozen weight alone and dropout_dx_kernel adds that part.
    auto add_dropout_dx = [&]() -> int {
        const size_t smem = sizeof(float) * (size_t)r * DROP_TOK;
        const dim3 grid((unsigned)cdiv(K, 256), (unsigned)cdiv(M, DROP_TOK));
        if (dt == REELS_BF16)
            launch_pdl(dropout_dx_kernel<DT_BF16>, grid, dim3(256), smem, st, A, (const void *)gbuf, ldm, M, K, (int)r,
                       dropout, key, dx);
        else if (dt == REELS_F16)
            launch_pdl(dropout_dx_kernel<DT_F16>, grid, dim3(256), smem, st, A, (const void *)gbuf, ldm, M, K, (int)r,
                       dropout, key, dx);
        else
            launch_pdl(dropout_dx_kernel<DT_F32>, grid, dim3(256), smem, st, A, (const void *)gbuf, ldm, M, K, (int)r,
                       dropout, key, dx);
        REELS_LAUNCHED();
        return REELS_OK;
    };

    if (tc_eligible(K, N, dt, {x, dy, q, dx, B, saved})) {
        // With the weight-in-TMEM plan for dX, one launch prepares its LoRA
        // operand (A, zero-padded) and, when A*x is recomputed, A^T.
        const int epi = act == REELS_ACT_GELU_TANH ? ACT_GELU_TANH_GRAD : ACT_NONE;
        const bool ts_prep = r > 0 && dx && !drop && plan_q8(M, K, N, ds->sms, aligned16(scales), epi).ts > 0;
        const DualPlan dual = plan_dual(M, N, r, ds->sms);
        if (ts_prep) {
            rc = prep_lora(dt, 1, nullptr, scales, 1.0f, false, r, ts_rank_pad(r), K, ws + wl.ext, A, K,
                           saved ? nullptr : ws + wl.at, st);
            if (rc) return rc;
        }
        if (r > 0) {
            if (!saved) {
                rc = rank_down_tc(ax, A, M, K, r, dt, ws + wl.tbuf, ws + wl.at, *ds, ws, wl, st, ts_prep);
                if (rc) return rc;
            }
            if (dual.use) {
                // g' and dB from one pass over dy
                rc = run_dual(dual, dy, B, tbuf, M, N, r, s, grad_scale * s, accumulate, gbuf, dB, dt, *ds, ws, wl, st);
                if (rc) return rc;
            } else {
                // g' = s * (B' * dy), stored [r][ldm]
                SkCall g{};
                g.act = dy;
                g.act_inner = N;
                g.act_outer = M;
                g.a_mn = false;
                g.bop = B;
                g.bop_pitch = N;
                g.rows = M;
                g.red = N;
                g.r = r;
                g.epi_final = 0;
                g.alpha = s;
                g.out = gbuf;
                g.ldo = ldm;
                rc = run_sk(g, dt, *ds, ws, wl, st);
                if (rc) return rc;
            }
        }
        if (dx) {
            Q8Call c{};
            c.fwd = false;
            c.act = dy;
            c.M = M;
            c.Nout = K;
            c.Kred = N;
            c.q = q;
            c.scales = scales;
            c.layout = layout;
            c.N_w = N;
            c.K_w = K;
            c.r = drop ? 0 : r;
            c.ext_act = gbuf;
            c.lora = A;
            c.ext_scale = 1.0f;
            c.ext_buf = ws + wl.ext;
            c.bias = nullptr;
            c.out = dx;
            c.epi_act = epi;
            c.pre = act == REELS_ACT_NONE ? nullptr : const_cast<void *>(pre_x);
            c.ext_ready = ts_prep;
            rc = run_q8(c, dt, *ds, ws, wl, st);
            if (rc) return rc;
            if (drop) {
                rc = add_dropout_dx();
                if (rc) return rc;
            }
        }
        if (r > 0) {
            // dA[k][j] = grad_scale * sum_m g'[j][m] z[m][k]  (z = x without dropout)
            SkCall da{};
            da.act = ax;
            da.act_inner = K;
            da.act_outer = M;
            da.a_mn = true;
            da.bop = gbuf;
            da.bop_pitch = ldm;
            da.rows = K;
            da.red = M;
            da.r = r;
            da.epi_final = 1;
            da.alpha = grad_scale;
            da.accumulate = accumulate;
            da.out = dA;
            da.rs = r;
            da.cs = 1;
            rc = run_sk(da, dt, *ds, ws, wl, st);
            if (rc) return rc;
        }
        if (r > 0 && !dual.use) {
            // dB[j][n] = grad_scale * s * sum_m dy[m][n] t[j][m]
            SkCall db{};
            db.act = dy;
            db.act_inner = N;
            db.act_outer = M;
            db.a_mn = true;
            db.bop = tbuf;
            db.bop_pitch = ldm;
            db.rows = N;
            db.red = M;
            db.r = r;
            db.epi_final = 1;
            db.alpha = grad_scale * s;
            db.accumulate = accumulate;
            db.out = dB;
            db.rs = 1;
            db.cs = N;
            rc = run_sk(db, dt, *ds, ws, wl, st);
            if (rc) return rc;
        }
        return ok(REELS_PATH_TENSORCORE);
    }

    if (r > 0) {
        if (!saved) {
            gen_rank_down_kernel<<<launch_grid(M * r), 256, 0, st>>>(ax, A, M, K, (int)r, dt, ws + wl.tbuf, ldm);
            REELS_LAUNCHED();
        }
        gen_rank_grad_kernel<<<launch_grid(M * r), 256, 0, st>>>(dy, B, M, N, (int)r, s, dt, gbuf, ldm);
        REELS_LAUNCHED();
    }
    if (dx) {
        gen_dx_kernel<<<launch_grid(M * K), 256, 0, st>>>(dy, q, scales, layout, gbuf, ldm, A, M, K, N,
                                                          drop ? 0 : (int)r, dt, dx);
        REELS_LAUNCHED();
        if (drop) {
            rc = add_dropout_dx();
            if (rc) return rc;
        }
        if (act != REELS_ACT_NONE) {
            act_apply_kernel<<<launch_grid(M * K), 256, 0, st>>>(ACT_GELU_TANH_GRAD, dt, M * K, dx, pre_x);
            REELS_LAUNCHED();
        }
    }
    if (r > 0) {
        gen_da_kernel<<<launch_grid(K * r), 256, 0, st>>>(gbuf, ldm, ax, M, K, (int)r, grad_scale, accumulate, dt, dA);
        REELS_LAUNCHED();
        gen_db_kernel<<<launch_grid(N * r), 256, 0, st>>>(dy, tbuf, ldm, M, N, (int)r, grad_scale * s, accumulate, dt,
                                                          dB);
        REELS_LAUNCHED();
    }
    return ok(REELS_PATH_CUDACORE);
}

int reels_q8lora_backward(const void *x, const void *dy, const int8_t *q, const float *scales, int layout,
                          const void *A, const void *B, const void *saved, int64_t M, int64_t K, int64_t N, int64_t r,
                          float alpha, float grad_scale, int dt, void *dx, float *dA, float *dB, int accumulate,
                          void *workspace, size_t ws_bytes, void *stream) {
    return q8lora_backward_impl(x, dy, q, scales, layout, A, B, saved, M, K, N, r, alpha, grad_scale, dt,
                                REELS_ACT_NONE, nullptr, 0.0f, 0, dx, dA, dB, accumulate, workspace, ws_bytes, stream);
}

int reels_q8lora_backward_dropout(const void *x, const void *dy, const int8_t *q, const float *scales, int layout,
                                  const void *A, const void *B, const void *saved, int64_t M, int64_t K, int64_t N,
                                  int64_t r, float alpha, float grad_scale, int act_dtype, float dropout, uint64_t seed,
                                  uint64_t stream_id, void *dx, float *dA, float *dB, int accumulate, void *workspace,
                                  size_t ws_bytes, void *stream) {
    return q8lora_backward_impl(x, dy, q, scales, layout, A, B, saved, M, K, N, r, alpha, grad_scale, act_dtype,
                                REELS_ACT_NONE, nullptr, dropout, dropout_key(seed, stream_id), dx, dA, dB, accumulate,
                                workspace, ws_bytes, stream);
}

int reels_dropout_mask(int64_t n, float dropout, uint64_t seed, uint64_t stream_id, uint8_t *keep, void *stream) {
    if (n < 0) return fail("negative length");
    if (!(dropout >= 0.0f && dropout < 1.0f)) return fail("dropout must be in [0, 1)");
    if (n == 0) return ok(REELS_PATH_NONE);
    if (!keep) return fail("null mask");
    DeviceState *ds;
    DeviceScope scope;

    int rc = bind_device(keep, &ds, scope);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    dropout_mask_kernel<<<launch_grid(n), 256, 0, st>>>(n, dropout, dropout_key(seed, stream_id), keep);
    REELS_LAUNCHED();
    return ok(REELS_PATH_CUDACORE);
}

int reels_q8lora_backward_act(const void *x, const void *dy, const int8_t *q, const float *scales, int layout,
                              const void *A, const void *B, const void *saved, int64_t M, int64_t K, int64_t N,
                              int64_t r, float alpha, float grad_scale, int act_dtype, int act, const void *pre_x,
                              void *dx, float *dA, float *dB, int accumulate, void *workspace, size_t ws_bytes,
                              void *stream) {
    return q8lora_backward_impl(x, dy, q, scales, layout, A, B, saved, M, K, N, r, alpha, grad_scale, act_dtype, act,
                                pre_x, 0.0f, 0, dx, dA, dB, accumulate, workspace, ws_bytes, stream);
}

static int check_ln(const void *x, int64_t M, int64_t K, int64_t tps, float eps, int dt) {
    if (!x && M > 0) return fail("null x");
    if (M < 0 || K <= 0 || K > LN_MAX_K) return fail("LayerNorm needs 0 <= M and 0 < K <= " + std::to_string(LN_MAX_K));
    if (tps <= 0) return fail("tokens_per_sample must be positive");
    if (!(eps >= 0.0f) || !std::isfinite(eps)) return fail("epsilon must be finite and non-negative");
    if (dt != REELS_F32 && dt != REELS_F16 && dt != REELS_BF16) return fail("unknown act_dtype");
    return REELS_OK;
}

static int64_t ln_chunks(int64_t tps) { return cdiv(tps, LN_COL_ROWS); }

size_t reels_layernorm_modulate_workspace_bytes(int64_t M, int64_t K, int64_t tokens_per_sample) {
    if (M < 0 || K <= 0 || tokens_per_sample <= 0) return 0;
    const int64_t batch = cdiv(M, tokens_per_sample);
    return align256((size_t)M * 8) + align256((size_t)batch * ln_chunks(tokens_per_sample) * 2 * K * 4);
}

int reels_layernorm_modulate(const void *x, int64_t M, int64_t K, int64_t tokens_per_sample, const void *scale,
                             const void *shift, const void *ln_weight, const void *ln_bias, float epsilon, int dt,
                             void *out, void *stream) {
    int rc = check_ln(x, M, K, tokens_per_sample, epsilon, dt);
    if (rc) return rc;
    if (!out && M > 0) return fail("null out");
    if (M == 0) return ok(REELS_PATH_NONE);
    DeviceState *ds;
    DeviceScope scope;

    rc = bind_device(x, &ds, scope);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // one row per warp on the 16-byte path (no LayerNorm affine)
    const bool warp_rows = dt != REELS_F32 && (K & 7) == 0 && !ln_weight && !ln_bias &&
                           ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
                             reinterpret_cast<uintptr_t>(scale) | reinterpret_cast<uintptr_t>(shift)) & 15) == 0;
    if (warp_rows) {
        const dim3 wg((unsigned)std::min<int64_t>(cdiv(M, LN_THREADS / 32), 16LL * ds->sms));
        if (dt == REELS_BF16)
            launch_pdl(ln_modulate_warp_kernel<DT_BF16>, wg, dim3(LN_THREADS), 0, st, x, M, K, tokens_per_sample,
                       scale, shift, epsilon, out);
        else
            launch_pdl(ln_modulate_warp_kernel<DT_F16>, wg, dim3(LN_THREADS), 0, st, x, M, K, tokens_per_sample,
                       scale, shift, epsilon, out);
        REELS_LAUNCHED();
        return ok(REELS_PATH_CUDACORE);
    }
    const dim3 grid((unsigned)std::min<int64_t>(M, 16LL * ds->sms));
    const size_t smem = (size_t)K * 4;
    if (dt == REELS_BF16)
        launch_pdl(ln_modulate_kernel<DT_BF16>, grid, dim3(LN_THREADS), smem, st, x, M, K, tokens_per_sample, scale,
                   shift, ln_weight, ln_bias, epsilon, out);
    else if (dt == REELS_F16)
        launch_pdl(ln_modulate_kernel<DT_F16>, grid, dim3(LN_THREADS), smem, st, x, M, K, tokens_per_sample, scale,
                   shift, ln_weight, ln_bias, epsilon, out);
    else
        launch_pdl(ln_modulate_kernel<DT_F32>, grid, dim3(LN_THREADS), smem, st, x, M, K, tokens_per_sample, scale,
                   shift, ln_weight, ln_bias, epsilon, out);
    REELS_LAUNCHED();
    return ok(REELS_PATH_CUDACORE);
}

int reels_layernorm_modulate_backward(const void *x, const void *dout, int64_t M, int64_t K,
                                      int64_t tokens_per_sample, const void *scale, const void *ln_weight,
                                      const void *ln_bias, float epsilon, int dt, void *dx, float *dscale,
                                      float *dshift, int accumulate, void *workspace, size_t ws_bytes,
                                      void *stream) {
    int rc = check_ln(x, M, K, tokens_per_sample, epsilon, dt);
    if (rc) return rc;
    if (!dout && M > 0) return fail("null dout");
    if (!dx && M > 0) return fail("null dx (the parameter gradients reuse its row statistics)");
    const bool params = dscale || dshift;
    const int64_t batch = cdiv(M, tokens_per_sample);
    if (params && M > 0) {
        if (!workspace) return fail("null workspace; size it with reels_layernorm_modulate_workspace_bytes");
        if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return fail("workspace must be 256-byte aligned");
        if (ws_bytes < reels_layernorm_modulate_workspace_bytes(M, K, tokens_per_sample))
            return fail("workspace too small");
    }
    DeviceState *ds;
    DeviceScope scope;

    rc = bind_device(x, &ds, scope);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (M == 0) {
        if (params && !accumulate) {
            if (dscale) REELS_CUDA(cudaMemsetAsync(dscale, 0, sizeof(float) * batch * K, st));
            if (dshift) REELS_CUDA(cudaMemsetAsync(dshift, 0, sizeof(float) * batch * K, st));
        }
        return ok(REELS_PATH_NONE);
    }
    float2 *stats = params ? reinterpret_cast<float2 *>(workspace) : nullptr;
    float *part = params ? reinterpret_cast<float *>(reinterpret_cast<char *>(workspace) + align256((size_t)M * 8))
                         : nullptr;
    const dim3 grid((unsigned)std::min<int64_t>(M, 16LL * ds->sms));
    const size_t smem = (size_t)K * 8;
    // dx, and the row statistics the parameter reduction reads
    void *dxo = dx;
    const bool warp_rows = dt != REELS_F32 && (K & 7) == 0 && !ln_weight &&
                           ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dout) |
                             reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(scale)) & 15) == 0;
    const dim3 wg((unsigned)std::min<int64_t>(cdiv(M, LN_THREADS / 32), 16LL * ds->sms));
    if (warp_rows && dt == REELS_BF16)
        launch_pdl(ln_modulate_bwd_warp_kernel<DT_BF16>, wg, dim3(LN_THREADS), 0, st, x, dout, M, K,
                   tokens_per_sample, scale, epsilon, dxo, stats);
    else if (warp_rows)
        launch_pdl(ln_modulate_bwd_warp_kernel<DT_F16>, wg, dim3(LN_THREADS), 0, st, x, dout, M, K,
                   tokens_per_sample, scale, epsilon, dxo, stats);
    else if (dt == REELS_BF16)
        launch_pdl(ln_modulate_bwd_kernel<DT_BF16>, grid, dim3(LN_THREADS), smem, st, x, dout, M, K,
                   tokens_per_sample, scale, ln_weight, epsilon, dxo, stats);
    else if (dt == REELS_F16)
        launch_pdl(ln_modulate_bwd_kernel<DT_F16>, grid, dim3(LN_THREADS), smem, st, x, dout, M, K,
                   tokens_per_sample, scale, ln_weight, epsilon, dxo, stats);
    else
        launch_pdl(ln_modulate_bwd_kernel<DT_F32>, grid, dim3(LN_THREADS), smem, st, x, dout, M, K,
                   tokens_per_sample, scale, ln_weight, epsilon, dxo, stats);
    REELS_LAUNCHED();
    if (params) {
        const int64_t cps = ln_chunks(tokens_per_sample);
        if (batch * cps > 65535) return fail("too many token blocks for the parameter reduction");
        const dim3 pg((unsigned)cdiv(K, LN_THREADS), (unsigned)(batch * cps));
        if (dt == REELS_BF16)
            launch_pdl(ln_param_partial_kernel<DT_BF16>, pg, dim3(LN_THREADS), 0, st, x, dout, (const float2 *)stats,
                       M, K, tokens_per_sample, ln_weight, ln_bias, cps, part);
        else if (dt == REELS_F16)
            launch_pdl(ln_param_partial_kernel<DT_F16>, pg, dim3(LN_THREADS), 0, st, x, dout, (const float2 *)stats, M,
                       K, tokens_per_sample, ln_weight, ln_bias, cps, part);
        else
            launch_pdl(ln_param_partial_kernel<DT_F32>, pg, dim3(LN_THREADS), 0, st, x, dout, (const float2 *)stats, M,
                       K, tokens_per_sample, ln_weight, ln_bias, cps, part);
        REELS_LAUNCHED();
        launch_pdl(ln_param_final_kernel, dim3(launch_grid(batch * K)), dim3(256), 0, st, (const float *)part, K, batch,
                   cps, accumulate, dscale, dshift);
        REELS_LAUNCHED();
    }
    return ok(REELS_PATH_CUDACORE);
}

static int check_gate(int64_t M, int64_t N, int64_t tps, int dt) {
    if (M < 0 || N <= 0) return fail("gated residual needs 0 <= M and 0 < N");
    if (tps <= 0) return fail("tokens_per_sample must be positive");
    if (dt != REELS_F32 && dt != REELS_F16 && dt != REELS_BF16) return fail("unknown act_dtype");
    return REELS_OK;
}

int reels_gated_residual(const void *x, const void *y, const void *gate, int64_t M, int64_t N,
                         int64_t tokens_per_sample, int dt, void *out, void *stream) {
    int rc = check_gate(M, N, tokens_per_sample, dt);
    if (rc) return rc;
    if (M == 0) return ok(REELS_PATH_NONE);
    if (!x || !y || !gate || !out) return fail("null x, y, gate or out");
    DeviceState *ds;
    DeviceScope scope;

    rc = bind_device(x, &ds, scope);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    dispatch_dt(dt, [&](auto d) {
        launch_pdl(gated_residual_kernel<decltype(d)::value>, dim3(launch_grid(M * N)), dim3(256), 0, st, x, y, gate,
                   M, N, tokens_per_sample, out);
    });
    REELS_LAUNCHED();
    return ok(REELS_PATH_CUDACORE);
}

size_t reels_gated_residual_workspace_bytes(int64_t M, int64_t N, int64_t tokens_per_sample) {
    if (M < 0 || N <= 0 || tokens_per_sample <= 0) return 0;
    return align256((size_t)cdiv(M, tokens_per_sample) * ln_chunks(tokens_per_sample) * N * 4);
}

int reels_gated_residual_backward(const void *dout, const void *y, const void *gate, int64_t M, int64_t N,
                                  int64_t tokens_per_sample, int dt, void *dy, float *dgate, int accumulate,
                                  void *workspace, size_t ws_bytes, void *stream) {
    int rc = check_gate(M, N, tokens_per_sample, dt);
    if (rc) return rc;
    if (M > 0 && (!dout || !gate)) return fail("null dout or gate");
    if (M > 0 && dgate && !y) return fail("dgate needs y");
    if (dgate && M > 0) {
        if (!workspace) return fail("null workspace; size it with reels_gated_residual_workspace_bytes");
        if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return fail("workspace must be 256-byte aligned");
        if (ws_bytes < reels_gated_residual_workspace_bytes(M, N, tokens_per_sample)) return fail("workspace too small");
    }
    if (!dy && !dgate) return ok(REELS_PATH_NONE);
    DeviceState *ds;
    DeviceScope scope;

    rc = bind_device(dout, &ds, scope);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int64_t batch = cdiv(M, tokens_per_sample);
    if (M == 0) {
        if (dgate && !accumulate) REELS_CUDA(cudaMemsetAsync(dgate, 0, sizeof(float) * batch * N, st));
        return ok(REELS_PATH_NONE);
    }
    if (dy) {
        dispatch_dt(dt, [&](auto d) {
            launch_pdl(gated_residual_dy_kernel<decltype(d)::value>, dim3(launch_grid(M * N)), dim3(256), 0, st, dout,
                       gate, M, N, tokens_per_sample, dy);
        });
        REELS_LAUNCHED();
    }
    if (dgate) {
        const int64_t cps = ln_chunks(tokens_per_sample);
        if (batch * cps > 65535) return fail("too many token blocks for the gate reduction");
        float *part = reinterpret_cast<float *>(workspace);
        const dim3 pg((unsigned)cdiv(N, LN_THREADS), (unsigned)(batch * cps));
        dispatch_dt(dt, [&](auto d) {
            launch_pdl(gate_grad_partial_kernel<decltype(d)::value>, pg, dim3(LN_THREADS), 0, st, dout, y, M, N,
                       tokens_per_sample, cps, part);
        });
        REELS_LAUNCHED();
        launch_pdl(gate_grad_final_kernel, dim3(launch_grid(batch * N)), dim3(256), 0, st, (const float *)part, N,
                   batch, cps, accumulate, dgate);
        REELS_LAUNCHED();
    }
    return ok(REELS_PATH_CUDACORE);
}

size_t reels_opt_workspace_bytes(int count) {
    if (count < 0) return 0;
    return opt_table_end(count);
}

int reels_opt_prepare(const reels_opt_tensor *tensors, int count, void *workspace, size_t ws_bytes, void *stream) {
    if (count < 0) return fail("negative tensor count");
    if (count > 0 && !tensors) return fail("null tensor table");
    if (!workspace) return fail("null optimizer workspace");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return fail("optimizer workspace must be 256-byte aligned");
    if (ws_bytes < reels_opt_workspace_bytes(count))
        return fail("optimizer workspace too small: need " + std::to_string(reels_opt_workspace_bytes(count)) +
                    " bytes, got " + std::to_string(ws_bytes));
    // header and table (the partials in between are scratch: not copied)
    std::vector<char> host(opt_table_end(count), 0);
    OptHeader *h = reinterpret_cast<OptHeader *>(host.data());
    OptEntry *tab = reinterpret_cast<OptEntry *>(host.data() + OPT_TABLE_OFF);
    int64_t chunks = 0;
    for (int i = 0; i < count; ++i) {
        const reels_opt_tensor &t = tensors[i];
        if (t.n < 0) return fail("tensor " + std::to_string(i) + ": negative length");
        if (t.param_dtype != REELS_F32 && t.param_dtype != REELS_F16 && t.param_dtype != REELS_BF16)
            return fail("tensor " + std::to_string(i) + ": unknown param_dtype");
        if (t.n > 0 && (!t.param || !t.grad || !t.m || !t.v || !t.master))
            return fail("tensor " + std::to_string(i) + ": null pointer");
        tab[i].t = t;
        tab[i].chunk0 = chunks;
        const size_t pal = t.param_dtype == REELS_F32 ? 16 : 8;
        tab[i].vec = aligned16(t.grad) && aligned16(t.m) && aligned16(t.v) && aligned16(t.master) &&
                     (reinterpret_cast<uintptr_t>(t.param) % pal) == 0;
        chunks += (t.n + OPT_CHUNK - 1) / OPT_CHUNK;
    }
    h->magic = OPT_MAGIC;
    h->count = count;
    h->total_chunks = chunks;
    DeviceState *ds;
    DeviceScope scope;

    int rc = bind_device(workspace, &ds, scope);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    char *dws = reinterpret_cast<char *>(workspace);
    REELS_CUDA(cudaMemcpyAsync(dws, host.data(), sizeof(OptHeader), cudaMemcpyHostToDevice, st));
    if (count > 0)
        REELS_CUDA(cudaMemcpyAsync(dws + OPT_TABLE_OFF, host.data() + OPT_TABLE_OFF, host.size() - OPT_TABLE_OFF,
                                   cudaMemcpyHostToDevice, st));
    REELS_CUDA(cudaStreamSynchronize(st));
    return ok(REELS_PATH_CUDACORE);
}

static int opt_blocks(const DeviceState &ds) { return std::min(OPT_MAX_BLOCKS, 4 * ds.sms); }

int reels_grad_norm_sq(void *workspace, float grad_scale, float *sumsq, void *stream) {
    if (!workspace || !sumsq) return fail("null workspace or sumsq");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return fail("optimizer workspace must be 256-byte aligned");
    if (!std::isfinite(grad_scale)) return fail("grad_scale must be finite");
    DeviceState *ds;
    DeviceScope scope;

    int rc = bind_device(workspace, &ds, scope);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const char *ws = reinterpret_cast<const char *>(workspace);
    double *partials = reinterpret_cast<double *>(reinterpret_cast<char *>(workspace) + OPT_PARTIALS_OFF);
    const int nb = opt_blocks(*ds);
    launch_pdl(grad_sumsq_kernel, dim3(nb), dim3(OPT_THREADS), 0, st, ws, grad_scale, partials, ds->status);
    REELS_LAUNCHED();
    launch_pdl(grad_sumsq_final_kernel, dim3(1), dim3(OPT_MAX_BLOCKS), 0, st, (const double *)partials, nb, sumsq);
    REELS_LAUNCHED();
    return ok(REELS_PATH_CUDACORE);
}

int reels_adamw_update(void *workspace, float lr, float beta1, float beta2, float eps, float weight_decay,
                       float correction1, float correction2, float grad_scale, const float *sumsq, float max_norm,
                       void *stream) {
    if (!workspace) return fail("null optimizer workspace");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return fail("optimizer workspace must be 256-byte aligned");
    for (float f : {lr, beta1, beta2, eps, weight_decay, correction1, correction2, grad_scale})
        if (!std::isfinite(f)) return fail("optimizer hyperparameters must be finite");
    if (!(correction1 > 0.0f) || !(correction2 > 0.0f)) return fail("bias corrections must be positive");
    if (sumsq && !(max_norm > 0.0f)) return fail("max_norm must be positive when clipping");
    DeviceState *ds;
    DeviceScope scope;

    int rc = bind_device(workspace, &ds, scope);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    AdamArgs a;
    a.lr = lr;
    a.beta1 = beta1;
    a.beta2 = beta2;
    a.omb1 = 1.0f - beta1;  // (1f0 - opt.beta1), rounded in fp32 as the reference forms it
    a.omb2 = 1.0f - beta2;
    a.eps = eps;
    a.wd = weight_decay;
    a.c1 = correction1;
    a.c2 = correction2;
    a.gs = grad_scale;
    a.max_norm = max_norm;
    a.sumsq = sumsq;
    launch_pdl(adamw_kernel, dim3(opt_blocks(*ds)), dim3(OPT_THREADS), 0, st, (const char *)workspace, a,
               ds->status);
    REELS_LAUNCHED();
    return ok(REELS_PATH_CUDACORE);
}

int reels_q8_weight_transpose_mul(const void *dy, const int8_t *q, const float *scales, int layout, int64_t M,
                                  int64_t K, int64_t N, int act_dtype, void *dx, void *workspace, size_t ws_bytes,
                                  void *stream) {
    if (!dx && M > 0) return fail("null dx");
    return reels_q8lora_backward(nullptr, dy, q, scales, layout, nullptr, nullptr, nullptr, M, K, N, 0, 1.0f, 1.0f,
                                 act_dtype, dx, nullptr, nullptr, 0, workspace, ws_bytes, stream);
}

}  // extern "C"

#ifdef REELS_TS_TRACE
// Debug builds only: copy out and clear the weight-in-TMEM kernel's per-role
// cycle counters (q8ts_gemm.cuh, g_ts_trace).
extern "C" int reels_ts_trace_read(unsigned long long *dst, size_t n) {
    static unsigned long long zero[256 * (TS_THREADS / 32) * 4];
    n = std::min(n, sizeof(zero) / 8);
    REELS_CUDA(cudaDeviceSynchronize());
    if (dst) REELS_CUDA(cudaMemcpyFromSymbol(dst, g_ts_trace, n * 8));
    REELS_CUDA(cudaMemcpyToSymbol(g_ts_trace, zero, sizeof(zero)));
    return REELS_OK;
}
#endif

// =====================================================================
// Forward with library-owned scratch, for callers that cannot allocate
// device memory (see include/reels_lowvram.h).  The scratch is this
// file-scope array; in host code its name is only a stand-in, so the device
// address is looked up with cudaGetSymbolAddress, once per device, with that
// device current, and handed to the kernels as an ordinary pointer.
static __device__ __align__(256) unsigned char g_static_ws[REELS_STATIC_WS_BYTES];

namespace {
void *g_static_ws_addr[kMaxDevices];
std::mutex g_static_ws_mu;
}  // namespace

extern "C" int reels_q8lora_forward_static_ws(const void *x, const int8_t *q, const float *scales, int layout,
                                              const void *A, const void *B, const void *bias, int64_t M, int64_t K,
                                              int64_t N, int64_t r, float alpha, int act_dtype, void *y, void *saved,
                                              void *stream) {
    int rc = check_common(M, K, N, r, act_dtype, layout);
    if (rc) return rc;
    if (M == 0) return ok(REELS_PATH_NONE);
    if (!x) return fail("null x");
    // Binds x's device (refusing a GPU the library was not built for) before
    // the array's address is looked up with that device current.
    DeviceScope scope;
    DeviceState *ds;
    rc = bind_device(x, &ds, scope);
    if (rc) return rc;
    const int dev = ds->index;
    void *ws = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_static_ws_mu);
        if (!g_static_ws_addr[dev]) {
            void *p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_static_ws);
            if (e != cudaSuccess || !p)
                return fail_dev(std::string("cudaGetSymbolAddress(static scratch): ") + cudaGetErrorString(e));
            g_static_ws_addr[dev] = p;
        }
        ws = g_static_ws_addr[dev];
    }
    const size_t need = ws_layout(M, K, N, r, act_dtype, REELS_PASS_FORWARD, ds->sms).total;
    if (need > REELS_STATIC_WS_BYTES) {
        char buf[200];
        snprintf(buf, sizeof buf,
                 "shape needs %zu bytes of scratch, more than the %u-byte static array; use reels_q8lora_forward "
                 "with a caller workspace",
                 need, (unsigned)REELS_STATIC_WS_BYTES);
        return fail(buf);
    }
    return reels_q8lora_forward(x, q, scales, layout, A, B, bias, M, K, N, r, alpha, act_dtype, y, saved, ws,
                                REELS_STATIC_WS_BYTES, stream);
}
