// chronos_moe.cu — the C ABI (include/chronos_moe.h): argument checks,
// workspace layout, TMA descriptors and the launch sequence of one MoE layer.
//
//   route -> plan -> scatter -> gate/up GEMM [-> act] -> down GEMM -> finalize
//
// All launches go to the caller's stream; nothing synchronises the host.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cmath>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>
#include <string>
#include <unordered_map>
#include <vector>

#include "chronos_attention.h"
#include "chronos_ep.h"
#include "chronos_lookahead.h"
#include "chronos_moe.h"
#include "common.cuh"
#include "attention.cuh"
#include "ep.cuh"
#include "lookahead.cuh"
#include "gemm_simt.cuh"
#include "gemm_tc.cuh"
#include "plan.cuh"
#include "router.cuh"
#include "route_fused.cuh"

namespace chronos {
namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

#define CHRONOS_CUDA_CHECK(expr)                                                              \
    do {                                                                                      \
        cudaError_t err_ = (expr);                                                            \
        if (err_ != cudaSuccess)                                                              \
            return fail(CHRONOS_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,                     \
                        cudaGetErrorString(err_), __FILE__, __LINE__);                        \
    } while (0)

constexpr int kDownWideMinTokens = 1024;  // batches from this size use token-major down tiles
constexpr int kDmPass = 64;  // token-major down: output columns per epilogue pass

std::atomic<uint64_t> g_kernel_launches{0};

// Decode routing as one cluster launch (route_fused.cuh); off: the two-kernel
// path.  Set by chronos_moe_set_option("fused_route", 0/1).
std::atomic<bool> g_fused_route_enabled{false};

// Prefill-sized calls (token-major down GEMM, shared experts last): combine the
// routed rows in two phases (stores + an ordered per-token sum, bitwise
// reproducible) instead of fp32 reduce-adds.  Off by default: measured slower
// (8192-token prefill 1.30 ms with it, 1.14 ms without).  Set by
// chronos_moe_set_option("two_phase_combine", 0/1).
std::atomic<bool> g_two_phase_enabled{false};

// Weight-major calls with shared experts: the down GEMM writes the output as
// each column tile completes (no finalize kernel).  Off by default: waiting
// for each unit's reduce-adds before counting it in stalls the epilogue, and
// measured slower than the finalize kernel it replaces (decode batches of 32
// and 64 tokens: 225 and 265 us per call with it, 198 and 203 us without).
// Set by chronos_moe_set_option("fold_finalize", 0/1).
std::atomic<bool> g_fold_enabled{false};

// Weight-major down GEMM: K is split until the call has about this many units
// per SM (0: no split); -1 (default): the split that best fills the last round
// of units (see forward_impl).  Set by chronos_moe_set_option("down_split_target", n).
std::atomic<int> g_down_split_target{-1};

// Decode batches of 9..32 tokens: selection + plan in one block of a warp per
// token (no ticket) instead of blocks of 8 tokens and a last-block plan.  Off by
// default: measured slower (32 tokens: 200.6-201.5 us per decode call with it,
// 196.3-196.9 without; 8-layer model 795 vs 785 us per step).  Set by
// chronos_moe_set_option("select_plan_one_block", 0/1).
std::atomic<bool> g_select_one_block{false};

inline void count_launch() { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }

// Launch with programmatic stream serialisation (`pdl`): the kernel may start
// while its predecessor in the stream runs and waits for it with pdl_wait().
// The first kernel of a call is launched without it, so a call never overlaps
// the previous call's kernels.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t st, bool pdl, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl ? attr : nullptr;
    cfg.numAttrs = pdl ? 1 : 0;
    count_launch();
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// stage profiling: CUDA events at the stage boundaries of profiled calls
// ---------------------------------------------------------------------------
constexpr int kBoundaries = CHRONOS_NUM_STAGES + 1;

struct ProfileState {
    int max_calls = 0;
    int calls = 0;
    std::vector<cudaEvent_t> events;           // [max_calls * kBoundaries]
    std::vector<uint8_t> ran;                  // [max_calls * CHRONOS_NUM_STAGES]
};
thread_local ProfileState g_prof;

// Slot of the current call in the profile, or -1.
int prof_begin_call() {
    if (g_prof.calls >= g_prof.max_calls) return -1;
    return g_prof.calls++;
}

void prof_mark(int slot, int boundary, cudaStream_t st) {
    if (slot >= 0) cudaEventRecord(g_prof.events[static_cast<size_t>(slot) * kBoundaries + boundary], st);
}

void prof_ran(int slot, int stage) {
    if (slot >= 0) g_prof.ran[static_cast<size_t>(slot) * CHRONOS_NUM_STAGES + stage] = 1;
}

size_t elem_size(int dtype) { return dtype == CHRONOS_DTYPE_FP32 ? 4 : 2; }

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Workspace regions, a function of the shape only.
struct Layout {
    size_t grp_count, grp_off, act_rows, act_xrow, act_hrow, act_wslot, act_eid, ustart_gu, partials,
        ustart_dn, hdr, pos, sel_coef, shared_coef, topk_idx, topk_w, slot_tok, slot_coef, slot_map, pair_slot,
        tile_cnt, gu_cnt, gu_part, xp, hid, y_acc, total;
};

// Decode gate/up K splits (weight-major, dense mode, N <= 64): when the call's
// routed and shared units would not cover the SMs (a batch of one token: 6
// routed experts x 11 weight-row tiles + 22 shared units for 148 SMs), the
// routed units are split along K (2 or 4 ways, >= 4 k tiles each) and the last
// split of a tile to finish sums the fp32 partials in split order and applies
// SiLU-mul.  The shared experts' units run before the plan exists and stay
// whole.  A function of the shape and the SM count, so the workspace layout
// and the call agree.  Off by default: measured slower (batch 1: 53.6-54.3 us
// per call split, 51.4 unsplit; the split gate/up kernel alone 36.7 vs 24.6 us
// in a serialised replay): the extra routed units all start after the routing
// wait, and the CTAs that get two of them finish last.  Set by
// chronos_moe_set_option("gateup_split", 0/1) before sizing a workspace.
std::atomic<bool> g_gateup_split_enabled{false};
// MB of routed gate/up weights the decode GEMM's idle CTAs prefetch into L2
// while the routing kernels run (batches that select nearly every expert); 0: off
std::atomic<int> g_gateup_prefetch_mb{128};
// Programmatic (early) launch of the norm, attention, lookahead and arg-max
// kernels; each waits for its predecessor before touching memory.  Off by
// default: the 8-layer decode step measured 761.0 us with it, 758.7 without.
std::atomic<bool> g_model_pdl{false};

int sm_count();

int gateup_splits(const ChronosMoeShape& s) {
    if (!g_gateup_split_enabled || s.num_tokens < 1 || s.num_tokens > kSelectPlanMaxTokens ||
        s.dtype == CHRONOS_DTYPE_FP32 || s.hidden % kTcBK || s.ffn % kTcBK)
        return 1;
    const int kt = s.hidden / kTcBK;
    const int mt = (s.ffn + kTcBM - 1) / kTcBM;
    const double draws = static_cast<double>(s.num_tokens) * s.top_k;
    const double routed = s.num_experts * (1.0 - std::pow(1.0 - 1.0 / s.num_experts, draws));
    const double pre = static_cast<double>(s.num_shared) * mt;
    int sp = 1;
    while (routed * mt * sp + pre < sm_count() && sp < 4 && kt / (2 * sp) >= 4) sp *= 2;
    return sp;
}

Layout make_layout(const ChronosMoeShape& s) {
    Layout L{};
    const size_t N = static_cast<size_t>(s.num_tokens);
    const size_t E = s.num_experts, K = s.top_k, S = s.num_shared, H = s.hidden, F = s.ffn;
    const size_t G = E + S;
    const size_t es = elem_size(s.dtype);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    L.grp_count = take(4 * (E + 1));  // + the ticket of the decode select + plan kernel
    L.grp_off = take(4 * E);
    L.act_rows = take(4 * G);
    L.act_xrow = take(4 * G);
    L.act_hrow = take(4 * G);
    L.act_wslot = take(4 * G);
    L.act_eid = take(4 * G);
    L.ustart_gu = take(4 * (G + 1));
    L.ustart_dn = take(4 * (G + 1));
    L.hdr = take(sizeof(PlanHeader));
    L.pos = take(4 * N * K);
    L.sel_coef = take(4 * N * K);
    L.shared_coef = take(4 * N);
    L.topk_idx = take(4 * N * K);
    L.topk_w = take(4 * N * K);
    L.partials = take(4 * N * E * route_chunks(s.hidden));
    L.slot_tok = take(4 * (N * K + S * N));
    L.slot_coef = take(4 * (N * K + S * N));
    L.slot_map = N <= static_cast<size_t>(kSelectPlanMaxTokens) ? take(4 * E * N) : off;
    L.pair_slot = take(4 * N * K);
    L.tile_cnt = take(4 * ((H + 127) / 128));
    {
        // decode gate/up K-split partials: [routed tile][split][G, U][token][128 rows] fp32
        const size_t sp = static_cast<size_t>(gateup_splits(s));
        const size_t routed = std::min(E, N * K);
        const size_t mt = (F + 127) / 128;
        L.gu_cnt = sp > 1 ? take(4 * routed * mt) : off;
        L.gu_part = sp > 1 ? take(4 * routed * mt * sp * 2 * N * 128) : off;
    }
    // x rows in expert order for the gate/up GEMM; once that GEMM is done, the
    // two-phase down GEMM's scaled slot rows (same size) go here
    L.xp = take(es * N * K * H);
    L.hid = take(es * (N * K + S * N) * F);
    L.y_acc = take(4 * N * H);
    L.total = off;
    return L;
}

int validate_shape(const ChronosMoeShape* s) {
    if (s == nullptr) return fail(CHRONOS_ERR_INVALID_ARG, "shape is NULL");
    if (s->num_tokens < 0 || s->num_tokens > (int64_t(1) << 24))
        return fail(CHRONOS_ERR_INVALID_ARG, "num_tokens %lld out of range [0, 2^24]",
                    static_cast<long long>(s->num_tokens));
    if (s->num_experts < 1 || s->num_experts > kMaxExperts)
        return fail(CHRONOS_ERR_INVALID_ARG, "num_experts %d out of range [1, %d]", s->num_experts,
                    kMaxExperts);
    if (s->top_k < 1 || s->top_k > kMaxTopK || s->top_k > s->num_experts)
        return fail(CHRONOS_ERR_INVALID_ARG, "top_k %d out of range [1, min(E, %d)]", s->top_k,
                    kMaxTopK);
    if (s->num_shared < 0 || s->num_shared > 8)
        return fail(CHRONOS_ERR_INVALID_ARG, "num_shared %d out of range [0, 8]", s->num_shared);
    if (s->hidden < 4 || s->hidden % 4 != 0 || s->hidden > 65536)
        return fail(CHRONOS_ERR_INVALID_ARG, "hidden %d must be a multiple of 4 in [4, 65536]",
                    s->hidden);
    if (s->ffn < 1 || s->ffn > 65536)
        return fail(CHRONOS_ERR_INVALID_ARG, "ffn %d out of range [1, 65536]", s->ffn);
    if (s->dtype != CHRONOS_DTYPE_BF16 && s->dtype != CHRONOS_DTYPE_FP16 &&
        s->dtype != CHRONOS_DTYPE_FP32)
        return fail(CHRONOS_ERR_INVALID_ARG, "unknown dtype %d", s->dtype);
    const int64_t slots = s->num_tokens * (s->top_k + s->num_shared);
    if (slots > (int64_t(1) << 30))
        return fail(CHRONOS_ERR_INVALID_ARG, "num_tokens * (top_k + num_shared) too large");
    return CHRONOS_OK;
}

// ---------------------------------------------------------------------------
// TMA descriptors (cuTensorMapEncodeTiled through the runtime's driver entry
// point), cached by (address, extents, box).
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

struct MapKey {
    uint64_t ptr, rows, cols, box_rows, dtype;
    bool operator==(const MapKey& o) const {
        return ptr == o.ptr && rows == o.rows && cols == o.cols && box_rows == o.box_rows &&
               dtype == o.dtype;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey& k) const {
        uint64_t h = k.ptr * 0x9E3779B97F4A7C15ull;
        h ^= k.rows + 0x632BE59BD9B4E019ull + (h << 6) + (h >> 2);
        h ^= k.cols + (h << 6) + (h >> 2);
        h ^= k.box_rows * 131 + k.dtype + (h << 6) + (h >> 2);
        return static_cast<size_t>(h);
    }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// 2-D row-major [rows, cols] tensor, tile box [box_rows, 64 columns], 128-B swizzle.
int make_map(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
             int dtype) {
    const MapKey key{reinterpret_cast<uint64_t>(base), rows, cols, box_rows,
                     static_cast<uint64_t>(dtype)};
    {
        std::lock_guard<std::mutex> lk(g_map_mu);
        auto it = g_maps.find(key);
        if (it != g_maps.end()) {
            *out = it->second;
            return CHRONOS_OK;
        }
    }
    EncodeTiledFn enc = get_encode_fn();
    if (enc == nullptr) return fail(CHRONOS_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
        return fail(CHRONOS_ERR_INVALID_ARG, "TMA operand %p is not 16-byte aligned", base);
    const cuuint64_t dims[2] = {cols, rows == 0 ? 1 : rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTcBK), box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = dtype == CHRONOS_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap m;
    const CUresult r = enc(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(CHRONOS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu",
                    static_cast<int>(r), static_cast<unsigned long long>(rows),
                    static_cast<unsigned long long>(cols));
    {
        std::lock_guard<std::mutex> lk(g_map_mu);
        if (g_maps.size() > 4096) g_maps.clear();
        g_maps.emplace(key, m);
    }
    *out = m;
    return CHRONOS_OK;
}

int sm_count() {
    int dev = 0;
    cudaGetDevice(&dev);
    static int cached[64] = {0};
    if (dev < 64 && cached[dev] > 0) return cached[dev];
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    if (dev < 64) cached[dev] = n;
    return n;
}

template <typename K>
int set_smem(K kernel, int bytes) {
    // The attribute is a limit that sticks to the function on its device, and
    // setting it costs host time on every layer call: raise it only when a launch
    // needs more than the largest value set so far on this device (a smaller
    // launch fits under a larger limit; lowering it would break a later larger
    // launch that found its size "already set").
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> limit;
    int dev = 0;
    cudaGetDevice(&dev);
    const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
    std::lock_guard<std::mutex> lk(mu);
    auto it = limit.find(key);
    if (it != limit.end() && it->second >= bytes) return CHRONOS_OK;
    CHRONOS_CUDA_CHECK(
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    limit[key] = bytes;
    return CHRONOS_OK;
}

struct Ptrs {
    uint8_t* ws;
    const Layout* L;
    float* acc_out = nullptr;  // the caller's fp32 output as the accumulator (CHRONOS_FLAG_ACC_OUT)
    template <typename P>
    P* at(size_t off) const { return reinterpret_cast<P*>(ws + off); }
    float* y_acc() const { return acc_out != nullptr ? acc_out : at<float>(L->y_acc); }
};

// ---------------------------------------------------------------------------
// launch helpers
// ---------------------------------------------------------------------------
int experts_per_lane(int num_experts) {
    return num_experts <= 32 ? 1 : num_experts <= 64 ? 2 : num_experts <= 128 ? 4 : 8;
}

RouteParams route_params(const ChronosMoeArgs* a, const Ptrs& w, bool prerouted, int32_t* topk_idx,
                         float* topk_w, bool zero_acc, void* y_direct) {
    const ChronosMoeShape& s = a->shape;
    RouteParams rp{};
    rp.x = a->x;
    rp.w = a->router_w;
    rp.bias = a->router_bias;
    rp.avail = a->avail;
    rp.avail_mask = (a->flags & CHRONOS_FLAG_AVAIL_MASK) ? 1 : 0;
    rp.slot_of_expert = a->slot_of_expert;
    rp.n = s.num_tokens;
    rp.h = s.hidden;
    rp.e = s.num_experts;
    rp.k = s.top_k;
    rp.num_shared = s.num_shared;
    rp.norm_topk = a->norm_topk ? 1 : 0;
    rp.prerouted = prerouted ? 1 : 0;
    rp.probs = prerouted ? nullptr : a->router_probs;
    rp.topk_idx = topk_idx;
    rp.topk_w = topk_w;
    rp.counts_all = prerouted ? nullptr : a->expert_counts;
    rp.mass_all = prerouted ? nullptr : a->expert_mass;
    rp.grp_count = w.at<int32_t>(w.L->grp_count);
    rp.pos = w.at<int32_t>(w.L->pos);
    rp.sel_coef = w.at<float>(w.L->sel_coef);
    rp.shared_coef = w.at<float>(w.L->shared_coef);
    rp.y_acc = (zero_acc && y_direct == nullptr) ? w.y_acc() : nullptr;
    rp.y_direct = y_direct;
    rp.partials = w.at<float>(w.L->partials);
    rp.nchunks = route_chunks(s.hidden);
    return rp;
}

// The cluster shape of the fused decode routing kernel for this call, or
// false when the call takes the two-kernel path (a batch above 64 tokens,
// d_model above 4096, shared memory above the limit, or a cluster this GPU
// cannot place).  The placement check runs once per (kernel, shape).
template <typename T, int EPL>
bool fused_route_fits_epl(int ncta, size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<int, size_t>, bool> seen;
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_pair(ncta, smem);
    auto it = seen.find(key);
    if (it != seen.end()) return it->second;
    bool ok = set_smem(route_decode_fused_kernel<T, EPL>, static_cast<int>(smem)) == CHRONOS_OK;
    if (ok) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(ncta);
        cfg.blockDim = dim3(kFusedRouteThreads);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = ncta;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        ok = cudaOccupancyMaxActiveClusters(&clusters, route_decode_fused_kernel<T, EPL>, &cfg) == cudaSuccess &&
             clusters >= 1;
        cudaGetLastError();   // a refused query leaves no error behind
    }
    seen[key] = ok;
    return ok;
}

template <typename T>
bool fused_route_shape(const ChronosMoeShape& s, int* ncta, int* cpc, size_t* smem) {
    if (s.num_tokens < 1 || s.num_tokens > kFusedRouteMaxTokens) return false;
    const int C = route_chunks(s.hidden);
    *ncta = std::min(kFusedRouteMaxCtas, C);
    *cpc = (C + *ncta - 1) / *ncta;
    if (*ncta * *cpc > kFusedRouteMaxChunks) return false;
    *smem = fused_route_smem<T>(s.num_tokens, s.num_experts, *cpc);
    if (*smem > static_cast<size_t>(180 << 10)) return false;
    switch (experts_per_lane(s.num_experts)) {
        case 1: return fused_route_fits_epl<T, 1>(*ncta, *smem);
        case 2: return fused_route_fits_epl<T, 2>(*ncta, *smem);
        case 4: return fused_route_fits_epl<T, 4>(*ncta, *smem);
        default: return fused_route_fits_epl<T, 8>(*ncta, *smem);
    }
}

template <typename T, int EPL>
cudaError_t launch_fused_route_epl(const RouteParams& rp, const PlanParams& pp, const ScatterParams& sp,
                                   int ncta, int cpc, size_t smem, cudaStream_t st) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(ncta);
    cfg.blockDim = dim3(kFusedRouteThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = ncta;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    count_launch();
    return cudaLaunchKernelEx(&cfg, route_decode_fused_kernel<T, EPL>, rp, pp, sp, cpc);
}

template <typename T>
int launch_fused_route(const RouteParams& rp, const PlanParams& pp, const ScatterParams& sp, int ncta, int cpc,
                       size_t smem, cudaStream_t st) {
    cudaError_t err;
    switch (experts_per_lane(rp.e)) {
        case 1: err = launch_fused_route_epl<T, 1>(rp, pp, sp, ncta, cpc, smem, st); break;
        case 2: err = launch_fused_route_epl<T, 2>(rp, pp, sp, ncta, cpc, smem, st); break;
        case 4: err = launch_fused_route_epl<T, 4>(rp, pp, sp, ncta, cpc, smem, st); break;
        default: err = launch_fused_route_epl<T, 8>(rp, pp, sp, ncta, cpc, smem, st); break;
    }
    CHRONOS_CUDA_CHECK(err);
    return CHRONOS_OK;
}

// Launches the logit kernel and (unless `out_params` is given, in which case
// the parameters are returned for the fused select + plan kernel) the select kernel.
template <typename T>
int launch_route(const ChronosMoeArgs* a, const Ptrs& w, cudaStream_t st, bool prerouted,
                 int32_t* topk_idx, float* topk_w, bool zero_acc, RouteParams* out_params = nullptr,
                 void* y_direct = nullptr) {
    const ChronosMoeShape& s = a->shape;
    RouteParams rp = route_params(a, w, prerouted, topk_idx, topk_w, zero_acc, y_direct);
    const int64_t N = s.num_tokens;
    const bool small = N <= kRouteSmallMax;
    // the logit kernel is the call's first launch (no PDL) and zeroes the counters;
    // with pre-routed inputs the caller zeroed them and the select kernel comes first
    if (!prerouted) {
        if (small) {
            const dim3 grid(static_cast<unsigned>((N + kRouteGroup - 1) / kRouteGroup),
                            static_cast<unsigned>(rp.nchunks),
                            static_cast<unsigned>((s.num_experts + kPartialThreads - 1) / kPartialThreads));
            CHRONOS_CUDA_CHECK(launch_kernel(route_partials_kernel<T>, grid, dim3(kPartialThreads), 0, st,
                                             false, rp));
        } else {
            const dim3 grid(static_cast<unsigned>((N + kTiledTokens - 1) / kTiledTokens),
                            static_cast<unsigned>((s.num_experts + kRouteTile - 1) / kRouteTile),
                            static_cast<unsigned>((rp.nchunks + kTiledChunks - 1) / kTiledChunks));
            constexpr int smem = tiled_smem_bytes<T>();
            if (int rc = set_smem(route_tiled_kernel<T>, smem)) return rc;
            CHRONOS_CUDA_CHECK(launch_kernel(route_tiled_kernel<T>, grid, dim3(kTiledThreads), smem, st,
                                             false, rp));
        }
    }
    if (out_params != nullptr) {  // the caller launches the fused select + plan kernel
        *out_params = rp;
        return CHRONOS_OK;
    }
    const unsigned sgrid = static_cast<unsigned>((N + kSelectThreads / 32 - 1) / (kSelectThreads / 32));
    const dim3 g(sgrid), b(kSelectThreads);
    const int epl = experts_per_lane(s.num_experts);
    cudaError_t err;
    switch (epl) {
        case 1: err = launch_kernel(route_select_kernel<T, 1>, g, b, 0, st, !prerouted, rp); break;
        case 2: err = launch_kernel(route_select_kernel<T, 2>, g, b, 0, st, !prerouted, rp); break;
        case 4: err = launch_kernel(route_select_kernel<T, 4>, g, b, 0, st, !prerouted, rp); break;
        default: err = launch_kernel(route_select_kernel<T, 8>, g, b, 0, st, !prerouted, rp); break;
    }
    CHRONOS_CUDA_CHECK(err);
    return CHRONOS_OK;
}

template <typename T>
int launch_select_plan(const RouteParams& rp, const PlanParams& pp, const ScatterParams& sp, int num_experts,
                       bool pdl, cudaStream_t st) {
    int32_t* ticket = rp.grp_count + num_experts;
    cudaError_t err;
    if (g_select_one_block && rp.n > kSelectPlanWarps && rp.n <= kSelectPlanWideThreads / 32) {
        // 9..32 tokens: one block of a warp per token, no ticket, fence or re-reads
        constexpr int NT = kSelectPlanWideThreads;
        const dim3 g(1), b(NT);
        switch (experts_per_lane(num_experts)) {
            case 1: err = launch_kernel(route_select_plan_kernel<T, 1, NT>, g, b, 0, st, pdl, rp, pp, sp, ticket); break;
            case 2: err = launch_kernel(route_select_plan_kernel<T, 2, NT>, g, b, 0, st, pdl, rp, pp, sp, ticket); break;
            case 4: err = launch_kernel(route_select_plan_kernel<T, 4, NT>, g, b, 0, st, pdl, rp, pp, sp, ticket); break;
            default: err = launch_kernel(route_select_plan_kernel<T, 8, NT>, g, b, 0, st, pdl, rp, pp, sp, ticket); break;
        }
        CHRONOS_CUDA_CHECK(err);
        return CHRONOS_OK;
    }
    const dim3 g(static_cast<unsigned>((rp.n + kSelectPlanWarps - 1) / kSelectPlanWarps)), b(kSelectPlanThreads);
    switch (experts_per_lane(num_experts)) {
        case 1: err = launch_kernel(route_select_plan_kernel<T, 1>, g, b, 0, st, pdl, rp, pp, sp, ticket); break;
        case 2: err = launch_kernel(route_select_plan_kernel<T, 2>, g, b, 0, st, pdl, rp, pp, sp, ticket); break;
        case 4: err = launch_kernel(route_select_plan_kernel<T, 4>, g, b, 0, st, pdl, rp, pp, sp, ticket); break;
        default: err = launch_kernel(route_select_plan_kernel<T, 8>, g, b, 0, st, pdl, rp, pp, sp, ticket); break;
    }
    CHRONOS_CUDA_CHECK(err);
    return CHRONOS_OK;
}

template <typename T, int BN, bool GATEUP, bool DENSE = false>
int launch_tc(const CUtensorMap& a0r, const CUtensorMap& a1r, const CUtensorMap& a0s,
              const CUtensorMap& a1s, const CUtensorMap& br, const CUtensorMap& bs,
              const TcGemmParams& p, int grid, cudaStream_t st) {
    constexpr int smem = tc_smem_bytes(BN, GATEUP);
    auto kern = tc_grouped_gemm<T, BN, GATEUP, DENSE>;
    if (int rc = set_smem(kern, smem)) return rc;
    CHRONOS_CUDA_CHECK(launch_kernel(kern, dim3(grid), dim3(kTcThreads), smem, st, true, a0r, a1r, a0s,
                                     a1s, br, bs, p));
    return CHRONOS_OK;
}

template <typename T, int BN, int BN_DN, bool TM_DN = false>
int launch_tc_pair(const ChronosMoeArgs* a, const Ptrs& w, cudaStream_t st, int kt_per_split_dn, int slot,
                   bool direct, bool shared_last, bool two_phase = false, bool fold = false, int gu_splits = 1) {
    const ChronosMoeShape& s = a->shape;
    const int dt = s.dtype;
    const uint64_t N = static_cast<uint64_t>(s.num_tokens), H = s.hidden, F = s.ffn;
    const uint64_t K = s.top_k, S = s.num_shared, P = a->pool_slots;
    const uint64_t slots = N * K + S * N;
    CUtensorMap g_r, u_r, g_s, u_s, xp_m, x_m, d_r, d_s, h_m;
    int rc;
    if ((rc = make_map(&g_r, a->w_gate, P * F, H, kTcBM, dt))) return rc;
    if ((rc = make_map(&u_r, a->w_up, P * F, H, kTcBM, dt))) return rc;
    if ((rc = make_map(&d_r, a->w_down, P * H, F, kTcBM, dt))) return rc;
    if (S > 0) {
        if ((rc = make_map(&g_s, a->w_shared_gate, S * F, H, kTcBM, dt))) return rc;
        if ((rc = make_map(&u_s, a->w_shared_up, S * F, H, kTcBM, dt))) return rc;
        if ((rc = make_map(&d_s, a->w_shared_down, S * H, F, kTcBM, dt))) return rc;
    } else {
        g_s = g_r;
        u_s = u_r;
        d_s = d_r;
    }
    // decode tiles (BN >= N): every group's B operand is x itself (DENSE), no
    // expert-ordered copy of x exists
    constexpr bool kDense = BN <= kSelectPlanMaxTokens;
    if ((rc = make_map(&x_m, a->x, N, H, BN, dt))) return rc;
    if (kDense) {
        xp_m = x_m;
    } else if ((rc = make_map(&xp_m, w.ws + w.L->xp, N * K, H, BN, dt))) {
        return rc;
    }
    if ((rc = make_map(&h_m, w.ws + w.L->hid, slots, F, BN_DN, dt))) return rc;

    TcGemmParams p{};
    p.hdr = w.at<PlanHeader>(w.L->hdr);
    p.act_rows = w.at<int32_t>(w.L->act_rows);
    p.act_xrow = w.at<int32_t>(w.L->act_xrow);
    p.act_hrow = w.at<int32_t>(w.L->act_hrow);
    p.act_wslot = w.at<int32_t>(w.L->act_wslot);
    p.act_eid = w.at<int32_t>(w.L->act_eid);
    p.f = static_cast<int>(F);
    p.h = static_cast<int>(H);
    p.hid = w.ws + w.L->hid;
    p.y_acc = w.y_acc();
    p.slot_tok = w.at<int32_t>(w.L->slot_tok);
    p.slot_coef = w.at<float>(w.L->slot_coef);
    p.ready_flags = a->ready_flags;
    p.ready_epoch = a->ready_epoch;
    p.ready_limit_ns = a->spin_limit_ns > 0 ? static_cast<uint64_t>(a->spin_limit_ns)
                                            : 2000000000ull;
    p.status = a->status;
    p.slot_map = w.at<int32_t>(w.L->slot_map);
    p.n_tokens = s.num_tokens;
    const int grid = (a->max_ctas > 0 && a->max_ctas < sm_count()) ? a->max_ctas : sm_count();

    // gate/up
    TcGemmParams pg = p;
    pg.ustart = w.at<int32_t>(w.L->ustart_gu);
    pg.k_tiles = static_cast<int>(H / kTcBK);
    pg.kt_per_split = static_cast<int>(H / kTcBK);
    pg.m_tiles = static_cast<int>((F + kTcBM - 1) / kTcBM);
    pg.w_rows = static_cast<int>(F);
    pg.out_cols = static_cast<int>(F);
    if (kDense && S > 0) {
        // decode: the shared experts' units run before the plan of the call exists
        pg.pre_units = static_cast<int>(S) * pg.m_tiles;
        pg.sh_hrow = static_cast<int64_t>(N * K);
    }
    if (kDense && gu_splits > 1) {
        // routed units split along K; the shared (pre-plan) units stay whole
        pg.kt_per_split = (pg.k_tiles + gu_splits - 1) / gu_splits;
        pg.gu_splits = gu_splits;
        pg.gu_cnt = w.at<int32_t>(w.L->gu_cnt);
        pg.gu_part = w.at<float>(w.L->gu_part);
        pg.num_shared = static_cast<int>(S);
    }
    if (kDense && gu_splits <= 1 && a->slot_of_expert == nullptr) {
        // speculative L2 prefetch of each idle CTA's first routed unit, when an
        // expert is left unselected with probability (1 - k/E)^N <= 10 %
        const int mb = g_gateup_prefetch_mb.load();
        const double p_idle = std::pow(1.0 - static_cast<double>(K) / static_cast<double>(s.num_experts),
                                       static_cast<double>(N));
        const int ctas = grid - pg.pre_units;
        if (mb > 0 && p_idle <= 0.1 && ctas > 0) {
            const uint64_t per_kt = 2ull * kTcBM * kTcBK * 2;   // gate + up boxes, 16-bit types
            const uint64_t kt = (static_cast<uint64_t>(mb) << 20) / (static_cast<uint64_t>(ctas) * per_kt);
            pg.spec_kt = static_cast<int>(std::min<uint64_t>(kt, static_cast<uint64_t>(pg.k_tiles)));
            pg.spec_experts = s.num_experts;
            pg.spec_avail = a->avail;
        }
    }
    prof_mark(slot, CHRONOS_STAGE_GATEUP, st);
    if constexpr (BN == kTmTokens) {
        // large batches: token-major tiles (one N = 256 MMA for gate and up)
        if ((rc = set_smem(tc_gateup_tm<T>, kTmSmemBytes))) return rc;
        CHRONOS_CUDA_CHECK(launch_kernel(tc_gateup_tm<T>, dim3(grid), dim3(kTcThreads), kTmSmemBytes, st, true,
                                         g_r, u_r, g_s, u_s, xp_m, x_m, pg));
    } else if ((rc = launch_tc<T, BN, true, kDense>(g_r, u_r, g_s, u_s, xp_m, x_m, pg, grid, st))) {
        return rc;
    }
    prof_ran(slot, CHRONOS_STAGE_GATEUP);
    prof_mark(slot, CHRONOS_STAGE_ACT, st);  // SiLU-mul is fused into the gate/up epilogue
    prof_mark(slot, CHRONOS_STAGE_DOWN, st);
    // down
    TcGemmParams pd = p;
    pd.ustart = w.at<int32_t>(w.L->ustart_dn);
    pd.k_tiles = static_cast<int>(F / kTcBK);
    pd.kt_per_split = kt_per_split_dn;
    pd.m_tiles = static_cast<int>(TM_DN ? (H + kDmCols - 1) / kDmCols : (H + kTcBM - 1) / kTcBM);
    pd.w_rows = static_cast<int>(H);
    pd.out_cols = static_cast<int>(H);
    pd.y_direct = direct ? a->y : nullptr;
    if (fold) {
        pd.tile_cnt = w.at<int32_t>(w.L->tile_cnt);
        pd.y_fold = a->y;
    }
    if (shared_last) {
        pd.sf_shared = static_cast<int>(S);
        pd.sh_hrow = static_cast<int64_t>(N * K);
        pd.dn_done = &w.at<PlanHeader>(w.L->hdr)->dn_done;
        pd.y_out = a->y;
        if (two_phase) {
            pd.ys = w.ws + w.L->xp;
            pd.pair_slot = w.at<int32_t>(w.L->pair_slot);
            pd.k_pairs = static_cast<int>(K);
        }
    }
    if constexpr (TM_DN) {
        // large batches: token-major tiles (128 tokens x 256 output columns)
        constexpr int smem = tc_dm_smem_bytes(kDmPass);
        if ((rc = set_smem(tc_down_tm<T, kDmPass>, smem))) return rc;
        CHRONOS_CUDA_CHECK(launch_kernel(tc_down_tm<T, kDmPass>, dim3(grid), dim3(kTcThreads), smem, st, true,
                                         d_r, d_s, h_m, pd));
    } else if ((rc = launch_tc<T, BN_DN, false>(d_r, d_r, d_s, d_s, h_m, h_m, pd, grid, st))) {
        return rc;
    }
    prof_ran(slot, CHRONOS_STAGE_DOWN);
    return CHRONOS_OK;
}

template <typename T>
int launch_simt(const ChronosMoeArgs* a, const Ptrs& w, cudaStream_t st, int slot) {
    const ChronosMoeShape& s = a->shape;
    SimtGemmParams p{};
    p.hdr = w.at<PlanHeader>(w.L->hdr);
    p.act_rows = w.at<int32_t>(w.L->act_rows);
    p.act_hrow = w.at<int32_t>(w.L->act_hrow);
    p.act_wslot = w.at<int32_t>(w.L->act_wslot);
    p.act_eid = w.at<int32_t>(w.L->act_eid);
    p.f = s.ffn;
    p.h = s.hidden;
    p.x = a->x;
    p.hid_in = w.ws + w.L->hid;
    p.hid_out = w.ws + w.L->hid;
    p.y_acc = w.y_acc();
    p.slot_tok = w.at<int32_t>(w.L->slot_tok);
    p.slot_coef = w.at<float>(w.L->slot_coef);
    p.ready_flags = a->ready_flags;
    p.ready_epoch = a->ready_epoch;
    p.ready_limit_ns = a->spin_limit_ns > 0 ? static_cast<uint64_t>(a->spin_limit_ns) : 2000000000ull;
    p.status = a->status;
    const int grid = 4 * sm_count();

    SimtGemmParams pg = p;
    pg.ustart = w.at<int32_t>(w.L->ustart_gu);
    pg.m_tiles = (s.ffn + kSimtTile - 1) / kSimtTile;
    pg.kdim = s.hidden;
    pg.out_cols = s.ffn;
    pg.w0r = a->w_gate;
    pg.w1r = a->w_up;
    pg.w0s = a->w_shared_gate;
    pg.w1s = a->w_shared_up;
    prof_mark(slot, CHRONOS_STAGE_GATEUP, st);
    CHRONOS_CUDA_CHECK(launch_kernel(simt_grouped_gemm<T, true>, dim3(grid), dim3(kSimtThreads), 0, st,
                                     true, pg));
    prof_ran(slot, CHRONOS_STAGE_GATEUP);
    prof_mark(slot, CHRONOS_STAGE_ACT, st);
    prof_mark(slot, CHRONOS_STAGE_DOWN, st);

    SimtGemmParams pd = p;
    pd.ustart = w.at<int32_t>(w.L->ustart_dn);
    pd.m_tiles = (s.hidden + kSimtTile - 1) / kSimtTile;
    pd.kdim = s.ffn;
    pd.out_cols = s.hidden;
    pd.w0r = a->w_down;
    pd.w0s = a->w_shared_down;
    CHRONOS_CUDA_CHECK(launch_kernel(simt_grouped_gemm<T, false>, dim3(grid), dim3(kSimtThreads), 0, st,
                                     true, pd));
    prof_ran(slot, CHRONOS_STAGE_DOWN);
    return CHRONOS_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int validate_args(const ChronosMoeArgs* a, bool need_experts) {
    if (a == nullptr) return fail(CHRONOS_ERR_INVALID_ARG, "args is NULL");
    if (int rc = validate_shape(&a->shape)) return rc;
    const ChronosMoeShape& s = a->shape;
    if (s.num_tokens == 0) return CHRONOS_OK;
    if (a->x == nullptr || a->router_w == nullptr)
        return fail(CHRONOS_ERR_INVALID_ARG, "x and router_w are required");
    if (a->workspace == nullptr && make_layout(s).total > 0)
        return fail(CHRONOS_ERR_INVALID_ARG, "workspace is NULL");
    if ((reinterpret_cast<uintptr_t>(a->workspace) & 255) != 0)
        return fail(CHRONOS_ERR_INVALID_ARG, "workspace must be 256-byte aligned");
    if (a->workspace_bytes < make_layout(s).total)
        return fail(CHRONOS_ERR_WORKSPACE_TOO_SMALL, "workspace %zu bytes < %zu required",
                    a->workspace_bytes, make_layout(s).total);
    if (!need_experts) return CHRONOS_OK;
    if (a->y == nullptr) return fail(CHRONOS_ERR_INVALID_ARG, "y is required");
    if (a->w_gate == nullptr || a->w_up == nullptr || a->w_down == nullptr)
        return fail(CHRONOS_ERR_INVALID_ARG, "routed expert weights are required");
    if (a->pool_slots < 1) return fail(CHRONOS_ERR_INVALID_ARG, "pool_slots must be >= 1");
    if (a->slot_of_expert == nullptr && a->pool_slots < s.num_experts)
        return fail(CHRONOS_ERR_INVALID_ARG, "pool_slots %d < num_experts %d without slot_of_expert",
                    a->pool_slots, s.num_experts);
    if (s.num_shared > 0 &&
        (a->w_shared_gate == nullptr || a->w_shared_up == nullptr || a->w_shared_down == nullptr))
        return fail(CHRONOS_ERR_INVALID_ARG, "shared expert weights are required (num_shared=%d)",
                    s.num_shared);
    if ((a->flags & CHRONOS_FLAG_PREROUTED) && (a->topk_idx == nullptr || a->topk_weight == nullptr))
        return fail(CHRONOS_ERR_INVALID_ARG, "CHRONOS_FLAG_PREROUTED needs topk_idx and topk_weight");
    return CHRONOS_OK;
}

template <typename T>
int forward_impl(const ChronosMoeArgs* a, cudaStream_t st) {
    const ChronosMoeShape& s = a->shape;
    const Layout L = make_layout(s);
    Ptrs w{static_cast<uint8_t*>(a->workspace), &L};
    const bool prerouted = (a->flags & CHRONOS_FLAG_PREROUTED) != 0;
    int32_t* topk_idx = a->topk_idx ? a->topk_idx : w.at<int32_t>(L.topk_idx);
    float* topk_w = a->topk_weight ? a->topk_weight : w.at<float>(L.topk_w);
    const int64_t N = s.num_tokens;

    const bool tc = (s.dtype != CHRONOS_DTYPE_FP32) && s.hidden % kTcBK == 0 &&
                    s.ffn % kTcBK == 0 && aligned16(a->x) && aligned16(a->w_gate) &&
                    aligned16(a->w_up) && aligned16(a->w_down) &&
                    (s.num_shared == 0 || (aligned16(a->w_shared_gate) &&
                                           aligned16(a->w_shared_up) &&
                                           aligned16(a->w_shared_down)));
    int bn = 128;
    if (tc) bn = N <= 16 ? 16 : N <= 32 ? 32 : N <= 64 ? 64 : 128;
    // large batches: token-major down tiles, 128 tokens x 256 output columns (the
    // MMA's N = 256 halves the weight-operand traffic per FLOP of 128-column
    // tiles; 128-token tiles keep small expert groups' padding low)
    const bool tm_dn = tc && N >= kDownWideMinTokens;
    const int bn_dn = tm_dn ? kTmTokens : bn;
    const int tok_tile = tc ? bn : kSimtTile;
    const int tok_tile_dn = tc ? bn_dn : kSimtTile;
    const int mt_gu = tc ? (s.ffn + kTcBM - 1) / kTcBM : (s.ffn + kSimtTile - 1) / kSimtTile;
    const int mt_dn = tm_dn ? (s.hidden + kDmCols - 1) / kDmCols
                      : tc  ? (s.hidden + kTcBM - 1) / kTcBM
                            : (s.hidden + kSimtTile - 1) / kSimtTile;

    // decode gate/up K split (dense mode only; the layout reserved its partials)
    const int gu_splits = (tc && N <= kSelectPlanMaxTokens) ? gateup_splits(s) : 1;
    int splits_dn = 1, kt_dn = s.ffn / kTcBK;
    if (tc && !tm_dn) {
        const int kt_total = s.ffn / kTcBK;
        // expected distinct routed experts of N*k draws over E, plus the shared ones
        const double draws = static_cast<double>(N) * s.top_k;
        const double groups_est =
            s.num_experts * (1.0 - std::pow(1.0 - 1.0 / s.num_experts, draws)) + s.num_shared;
        const double tiles_est = groups_est * static_cast<double>((N + bn_dn - 1) / bn_dn) * mt_dn;
        const int target_units = g_down_split_target.load();
        if (target_units >= 0) {
            const double target = static_cast<double>(target_units) * sm_count();
            while (tiles_est * splits_dn < target && splits_dn * 2 * 4 <= kt_total) splits_dn *= 2;
        } else {
            // halve K once the unsplit units fill at least two rounds of the SMs: the
            // half-size units shorten the last round's tail.  With fewer units the
            // split only adds reduce traffic and per-unit work (measured: batch 1 of
            // the 64-expert shape and the 16-expert model shape are faster unsplit,
            // batches 8 and 32 faster split, 64 even)
            if (tiles_est >= 2.0 * sm_count() && kt_total >= 8) splits_dn = 2;
        }
        kt_dn = (kt_total + splits_dn - 1) / splits_dn;
        splits_dn = (kt_total + kt_dn - 1) / kt_dn;
    }

    // one contribution per token (k = 1, no shared experts, e.g. the rows an
    // expert-parallel rank received): the down GEMM stores the output rows
    // itself; no fp32 accumulator, no finalize pass
    // the caller takes the fp32 accumulator as the output: every path that writes
    // the layer dtype itself (direct, shared-last, folded finalize) is off
    const bool acc_out = (a->flags & CHRONOS_FLAG_ACC_OUT) != 0;
    if (acc_out) {
        if (!aligned16(a->y)) return fail(CHRONOS_ERR_INVALID_ARG, "CHRONOS_FLAG_ACC_OUT: y must be 16-byte aligned");
        w.acc_out = static_cast<float*>(a->y);
    }
    const bool direct = tc && !acc_out && s.top_k == 1 && s.num_shared == 0 && aligned16(a->y);
    if (direct) {
        splits_dn = 1;
        kt_dn = s.ffn / kTcBK;
    }
    // shared experts present: they run last in the down GEMM as one K = S_h * F
    // product per output tile, whose epilogue adds the routed accumulator and
    // writes the output (no finalize pass, no shared reduce-adds)
    // (when its tiles, one per 128 or BN tokens and output-column tile, cover the SMs)
    const bool shared_last = tc && !direct && !acc_out && s.num_shared > 0 && aligned16(a->y) &&
                             (N + bn_dn - 1) / bn_dn * mt_dn >= sm_count();
    // token-major shared-last calls combine in two phases: the routed units store
    // their scaled rows (layer dtype) into the expert-ordered x buffer, dead once
    // gate/up is done, and the shared units sum each token's rows in choice order
    // (no fp32 accumulator: no zeroing, no reduce-adds)
    const bool two_phase = tm_dn && shared_last && g_two_phase_enabled;
    // weight-major calls with shared experts (every output tile has units): the
    // down GEMM writes the output tile by tile as the last contribution lands
    const bool fold = tc && !tm_dn && !direct && !shared_last && !acc_out && s.num_shared > 0 && g_fold_enabled;

    int rc;
    // counters: zeroed by the logit kernel, or here when routing is skipped
    if (prerouted)
        CHRONOS_CUDA_CHECK(cudaMemsetAsync(w.ws + L.grp_count, 0, 4 * (s.num_experts + 1), st));
    const int slot = prof_begin_call();
    // decode batches: the routing selection, plan and slot tables run in one block;
    // with a cluster the logits run in that same launch (route_fused.cuh)
    const bool fused_plan = N <= kSelectPlanMaxTokens;
    int f_ncta = 0, f_cpc = 0;
    size_t f_smem = 0;
    const bool cluster_route = fused_plan && !prerouted && g_fused_route_enabled &&
                               fused_route_shape<T>(s, &f_ncta, &f_cpc, &f_smem);
    RouteParams rp{};
    prof_mark(slot, CHRONOS_STAGE_ROUTE, st);
    if (cluster_route)
        rp = route_params(a, w, false, topk_idx, topk_w, true, direct ? a->y : nullptr);
    else if ((rc = launch_route<T>(a, w, st, prerouted, topk_idx, topk_w, !two_phase,
                                   fused_plan ? &rp : nullptr, direct ? a->y : nullptr)))
        return rc;
    prof_ran(slot, CHRONOS_STAGE_ROUTE);
    prof_mark(slot, CHRONOS_STAGE_PLAN, st);

    PlanParams pp{};
    pp.n = N;
    pp.e = s.num_experts;
    pp.k = s.top_k;
    pp.num_shared = s.num_shared;
    pp.tok_tile = tok_tile;
    pp.tok_tile_dn = tok_tile_dn;
    pp.mt_gu = mt_gu;
    pp.mt_dn = mt_dn;
    pp.splits_dn = splits_dn;
    pp.shared_fin = shared_last ? 1 : 0;
    pp.grp_count = w.at<int32_t>(L.grp_count);
    pp.slot_of_expert = a->slot_of_expert;
    pp.hdr = w.at<PlanHeader>(L.hdr);
    pp.grp_off = w.at<int32_t>(L.grp_off);
    pp.act_rows = w.at<int32_t>(L.act_rows);
    pp.act_xrow = w.at<int32_t>(L.act_xrow);
    pp.act_hrow = w.at<int32_t>(L.act_hrow);
    pp.act_wslot = w.at<int32_t>(L.act_wslot);
    pp.act_eid = w.at<int32_t>(L.act_eid);
    pp.ustart_gu = w.at<int32_t>(L.ustart_gu);
    pp.ustart_dn = w.at<int32_t>(L.ustart_dn);
    pp.tile_cnt = fold ? w.at<int32_t>(L.tile_cnt) : nullptr;
    pp.n_tile_cnt = fold ? mt_dn : 0;
    pp.splits_gu = (tc && bn <= kSelectPlanMaxTokens) ? gu_splits : 1;
    pp.gu_cnt = pp.splits_gu > 1 ? w.at<int32_t>(L.gu_cnt) : nullptr;
    pp.n_gu_cnt = pp.splits_gu > 1 ? static_cast<int>(std::min<int64_t>(s.num_experts, N * s.top_k)) * mt_gu : 0;
    // the plan is computed inside the scatter launch (stage "plan" stays empty)
    prof_mark(slot, CHRONOS_STAGE_SCATTER, st);

    ScatterParams sp{};
    sp.x = a->x;
    sp.n = N;
    sp.h = s.hidden;
    sp.k = s.top_k;
    sp.num_shared = s.num_shared;
    sp.topk_idx = topk_idx;
    sp.pos = w.at<int32_t>(L.pos);
    sp.sel_coef = w.at<float>(L.sel_coef);
    sp.shared_coef = w.at<float>(L.shared_coef);
    sp.grp_off = w.at<int32_t>(L.grp_off);
    sp.xp = w.ws + L.xp;
    sp.slot_tok = w.at<int32_t>(L.slot_tok);
    sp.slot_coef = w.at<float>(L.slot_coef);
    sp.copy_rows = tc ? 1 : 0;
    sp.pair_slot = two_phase ? w.at<int32_t>(L.pair_slot) : nullptr;
    if (fused_plan) {
        sp.copy_rows = 0;
        sp.slot_map = tc ? w.at<int32_t>(L.slot_map) : nullptr;
        sp.e = s.num_experts;
        if (cluster_route) {
            if ((rc = launch_fused_route<T>(rp, pp, sp, f_ncta, f_cpc, f_smem, st))) return rc;
        } else if ((rc = launch_select_plan<T>(rp, pp, sp, s.num_experts, !prerouted, st))) {
            // (the first launch of the call when routing was skipped: pre-routed inputs)
            return rc;
        }
    } else {
        const int64_t warps = N * s.top_k;
        const unsigned blocks =
            static_cast<unsigned>(std::max<int64_t>(1, (warps + kScatterWarps - 1) / kScatterWarps));
        CHRONOS_CUDA_CHECK(launch_kernel(plan_scatter_kernel<T>, dim3(blocks), dim3(kScatterThreads), 0,
                                         st, true, pp, sp));
    }
    prof_ran(slot, CHRONOS_STAGE_SCATTER);

    if (tc) {
        if constexpr (std::is_same<T, float>::value) {
            return fail(CHRONOS_ERR_INVALID_ARG, "internal: fp32 on the tensor-core path");
        } else {
            switch (bn) {
                case 16: rc = launch_tc_pair<T, 16, 16>(a, w, st, kt_dn, slot, direct, shared_last, false, fold, gu_splits); break;
                case 32: rc = launch_tc_pair<T, 32, 32>(a, w, st, kt_dn, slot, direct, shared_last, false, fold, gu_splits); break;
                case 64: rc = launch_tc_pair<T, 64, 64>(a, w, st, kt_dn, slot, direct, shared_last, false, fold, gu_splits); break;
                default:
                    rc = tm_dn ? launch_tc_pair<T, 128, 128, true>(a, w, st, kt_dn, slot, direct, shared_last,
                                                                    two_phase)
                               : launch_tc_pair<T, 128, 128>(a, w, st, kt_dn, slot, direct, shared_last, false,
                                                             fold);
                    break;
            }
        }
    } else {
        rc = launch_simt<T>(a, w, st, slot);
    }
    if (rc) return rc;

    prof_mark(slot, CHRONOS_STAGE_FINALIZE, st);
    if (direct || shared_last || fold || acc_out) {
        prof_mark(slot, kBoundaries - 1, st);
        return CHRONOS_OK;
    }
    const int64_t count4 = N * s.hidden / 4;
    const int blocks = static_cast<int>(std::min<int64_t>((count4 + 255) / 256, 8 * sm_count()));
    CHRONOS_CUDA_CHECK(launch_kernel(finalize_kernel<T>, dim3(blocks), dim3(256), 0, st, true,
                                     static_cast<const float*>(w.y_acc()),
                                     static_cast<T*>(a->y), count4));
    prof_ran(slot, CHRONOS_STAGE_FINALIZE);
    prof_mark(slot, kBoundaries - 1, st);
    return CHRONOS_OK;
}

template <typename T>
int route_impl(const ChronosMoeArgs* a, cudaStream_t st) {
    const ChronosMoeShape& s = a->shape;
    const Layout L = make_layout(s);
    Ptrs w{static_cast<uint8_t*>(a->workspace), &L};
    // the logit kernel zeroes the group counters and the per-expert statistics
    return launch_route<T>(a, w, st, false, a->topk_idx, a->topk_weight, false);
}

}  // namespace
}  // namespace chronos

using namespace chronos;

extern "C" size_t chronos_moe_workspace_size(const ChronosMoeShape* shape) {
    if (validate_shape(shape) != CHRONOS_OK) return 0;
    return make_layout(*shape).total;
}

extern "C" int chronos_moe_forward(const ChronosMoeArgs* args, void* cuda_stream) {
    g_last_error.clear();
    if (int rc = validate_args(args, true)) return rc;
    if (args->shape.num_tokens == 0) return CHRONOS_OK;
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    switch (args->shape.dtype) {
        case CHRONOS_DTYPE_BF16: return forward_impl<__nv_bfloat16>(args, st);
        case CHRONOS_DTYPE_FP16: return forward_impl<__half>(args, st);
        default: return forward_impl<float>(args, st);
    }
}

extern "C" int chronos_moe_route(const ChronosMoeArgs* args, void* cuda_stream) {
    g_last_error.clear();
    if (int rc = validate_args(args, false)) return rc;
    if (args->shape.num_tokens == 0) return CHRONOS_OK;
    if (args->topk_idx == nullptr || args->topk_weight == nullptr)
        return fail(CHRONOS_ERR_INVALID_ARG, "chronos_moe_route needs topk_idx and topk_weight");
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    switch (args->shape.dtype) {
        case CHRONOS_DTYPE_BF16: return route_impl<__nv_bfloat16>(args, st);
        case CHRONOS_DTYPE_FP16: return route_impl<__half>(args, st);
        default: return route_impl<float>(args, st);
    }
}

// ---------------------------------------------------------------------------
// No-allocation variant: the workspace is a scratch array compiled into the
// library instead of caller memory.  Host code must not use the array's name
// as a device address (on the host it names a shadow object), so its device
// address is looked up per device with cudaGetSymbolAddress and cached.
// ---------------------------------------------------------------------------
static __device__ __align__(256) uint8_t g_noalloc_scratch[CHRONOS_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {nullptr};

int noalloc_scratch(void** out) {
    int dev = -1;
    CHRONOS_CUDA_CHECK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices)
        return fail(CHRONOS_ERR_INVALID_ARG, "device %d out of range for the scratch table", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        CHRONOS_CUDA_CHECK(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        if (p == nullptr || (reinterpret_cast<uintptr_t>(p) & 255) != 0)
            return fail(CHRONOS_ERR_CUDA, "scratch array address %p is unusable", p);
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return CHRONOS_OK;
}
}  // namespace

extern "C" int chronos_moe_forward_noalloc(const ChronosMoeArgs* args, void* cuda_stream) {
    g_last_error.clear();
    if (args == nullptr) return fail(CHRONOS_ERR_INVALID_ARG, "args is NULL");
    if (int rc = validate_shape(&args->shape)) return rc;
    const size_t need = make_layout(args->shape).total;
    if (need > CHRONOS_NOALLOC_SCRATCH_BYTES)
        return fail(CHRONOS_ERR_INVALID_ARG,
                    "this shape needs %zu bytes of scratch; chronos_moe_forward_noalloc serves at "
                    "most %u (use chronos_moe_forward with a caller workspace)",
                    need, CHRONOS_NOALLOC_SCRATCH_BYTES);
    if (args->shape.num_tokens == 0) return CHRONOS_OK;
    ChronosMoeArgs a = *args;
    if (int rc = noalloc_scratch(&a.workspace)) return rc;
    a.workspace_bytes = CHRONOS_NOALLOC_SCRATCH_BYTES;
    if (int rc = validate_args(&a, true)) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    switch (a.shape.dtype) {
        case CHRONOS_DTYPE_BF16: return forward_impl<__nv_bfloat16>(&a, st);
        case CHRONOS_DTYPE_FP16: return forward_impl<__half>(&a, st);
        default: return forward_impl<float>(&a, st);
    }
}

extern "C" const char* chronos_moe_last_error(void) { return g_last_error.c_str(); }

extern "C" int chronos_moe_abi_version(void) { return CHRONOS_MOE_ABI_VERSION; }

extern "C" size_t chronos_moe_args_size(void) { return sizeof(ChronosMoeArgs); }

extern "C" int chronos_moe_profile_begin(int max_calls) {
    g_last_error.clear();
    if (max_calls < 1 || max_calls > 100000)
        return fail(CHRONOS_ERR_INVALID_ARG, "max_calls %d out of range [1, 100000]", max_calls);
    const size_t need = static_cast<size_t>(max_calls) * kBoundaries;
    while (g_prof.events.size() < need) {
        cudaEvent_t ev;
        CHRONOS_CUDA_CHECK(cudaEventCreate(&ev));
        g_prof.events.push_back(ev);
    }
    g_prof.ran.assign(static_cast<size_t>(max_calls) * CHRONOS_NUM_STAGES, 0);
    g_prof.max_calls = max_calls;
    g_prof.calls = 0;
    return CHRONOS_OK;
}

extern "C" int chronos_moe_profile_end(float* stage_ms, int32_t* stage_launches, int max_stages) {
    g_last_error.clear();
    const int calls = g_prof.calls;
    g_prof.max_calls = 0;
    g_prof.calls = 0;
    const int ns = std::min(max_stages, CHRONOS_NUM_STAGES);
    for (int i = 0; i < ns; ++i) {
        if (stage_ms) stage_ms[i] = 0.0f;
        if (stage_launches) stage_launches[i] = 0;
    }
    for (int c = 0; c < calls; ++c) {
        cudaEvent_t* ev = g_prof.events.data() + static_cast<size_t>(c) * kBoundaries;
        cudaError_t e = cudaEventSynchronize(ev[kBoundaries - 1]);
        if (e != cudaSuccess)
            return -fail(CHRONOS_ERR_CUDA, "cudaEventSynchronize: %s", cudaGetErrorString(e));
        for (int i = 0; i < ns; ++i) {
            float ms = 0.0f;
            e = cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
            if (e != cudaSuccess)
                return -fail(CHRONOS_ERR_CUDA, "cudaEventElapsedTime: %s", cudaGetErrorString(e));
            if (stage_ms) stage_ms[i] += ms;
            if (stage_launches)
                stage_launches[i] += g_prof.ran[static_cast<size_t>(c) * CHRONOS_NUM_STAGES + i];
        }
    }
    return calls;
}

extern "C" uint64_t chronos_moe_kernel_launches(void) {
    return g_kernel_launches.load(std::memory_order_relaxed);
}

extern "C" int chronos_moe_set_option(const char* name, int64_t value) {
    g_last_error.clear();
    if (name != nullptr && std::strcmp(name, "fused_route") == 0) {
        g_fused_route_enabled.store(value != 0);
        return CHRONOS_OK;
    }
    if (name != nullptr && std::strcmp(name, "fold_finalize") == 0) {
        g_fold_enabled.store(value != 0);
        return CHRONOS_OK;
    }
    if (name != nullptr && std::strcmp(name, "two_phase_combine") == 0) {
        g_two_phase_enabled.store(value != 0);
        return CHRONOS_OK;
    }
    if (name != nullptr && std::strcmp(name, "gateup_split") == 0) {
        g_gateup_split_enabled.store(value != 0);
        return CHRONOS_OK;
    }
    if (name != nullptr && std::strcmp(name, "gateup_prefetch_mb") == 0) {
        if (value < 0 || value > 1024) return fail(CHRONOS_ERR_INVALID_ARG, "gateup_prefetch_mb %lld (0..1024)",
                                                   static_cast<long long>(value));
        g_gateup_prefetch_mb.store(static_cast<int>(value));
        return CHRONOS_OK;
    }
    if (name != nullptr && std::strcmp(name, "model_pdl") == 0) {
        g_model_pdl.store(value != 0);
        return CHRONOS_OK;
    }
    if (name != nullptr && std::strcmp(name, "select_plan_one_block") == 0) {
        g_select_one_block.store(value != 0);
        return CHRONOS_OK;
    }
    if (name != nullptr && std::strcmp(name, "down_split_target") == 0) {
        if (value < -1 || value > 64) return fail(CHRONOS_ERR_INVALID_ARG, "down_split_target %lld (-1..64)",
                                                  static_cast<long long>(value));
        g_down_split_target.store(static_cast<int>(value));
        return CHRONOS_OK;
    }
    return fail(CHRONOS_ERR_INVALID_ARG, "unknown option %s", name ? name : "(null)");
}

// ---------------------------------------------------------------------------
// expert-parallel dispatch / combine (include/chronos_ep.h)
// ---------------------------------------------------------------------------
namespace chronos {
namespace {

int validate_ep_rows(int64_t n, int32_t h, int32_t k, int32_t dtype) {
    if (n < 0 || n > (int64_t(1) << 24)) return fail(CHRONOS_ERR_INVALID_ARG, "num_tokens %lld out of range",
                                                     static_cast<long long>(n));
    if (dtype != CHRONOS_DTYPE_BF16 && dtype != CHRONOS_DTYPE_FP16 && dtype != CHRONOS_DTYPE_FP32)
        return fail(CHRONOS_ERR_INVALID_ARG, "dtype %d unknown", dtype);
    if (h <= 0 || (static_cast<size_t>(h) * elem_size(dtype)) % 16 != 0)
        return fail(CHRONOS_ERR_INVALID_ARG, "hidden %d: rows must be a multiple of 16 bytes", h);
    if (k < 1 || k > kMaxTopKEp) return fail(CHRONOS_ERR_INVALID_ARG, "top_k %d out of range [1, %d]", k,
                                             kMaxTopKEp);
    return CHRONOS_OK;
}

template <typename T>
int ep_dispatch_impl(const ChronosEpDispatchArgs* a, cudaStream_t st) {
    EpParams p{};
    p.x = a->x;
    p.n = a->num_tokens;
    p.h = a->hidden;
    p.e = a->num_experts;
    p.k = a->top_k;
    p.g = a->world_size;
    p.epr = a->num_experts / a->world_size;
    const int chunks = a->num_chunks < 1 ? 1 : a->num_chunks;
    p.chunks = chunks;
    p.chunk_experts = p.epr / chunks;
    p.pairs = a->meta_pairs > 1 ? a->meta_pairs : 1;
    p.topk_idx = a->topk_idx;
    p.topk_w = a->topk_weight;
    p.avail = a->avail;
    p.counts = a->send_counts;
    p.pos = a->scratch;
    p.send_x = a->send_x;
    p.send_meta = a->send_meta;
    p.pair_slot = a->pair_slot;
    p.shared_w = a->shared_weight;
    p.seg_rows = a->seg_rows > 0 ? a->seg_rows : 0;
    CHRONOS_CUDA_CHECK(cudaMemsetAsync(a->send_counts, 0, sizeof(int32_t) * a->world_size * chunks, st));
    const int64_t pairs = p.n * p.k;
    // no selections: nothing to send, unless fixed segments need their padding metadata
    if (pairs == 0 && p.seg_rows == 0) return CHRONOS_OK;
    const int64_t work = std::max<int64_t>(pairs, 1);
    const unsigned cb = static_cast<unsigned>((work + kEpPackThreads - 1) / kEpPackThreads);
    CHRONOS_CUDA_CHECK(launch_kernel(ep_count_kernel, dim3(cb), dim3(kEpPackThreads), 0, st, false, p));
    const int64_t wpb = kEpPackThreads / 32;
    const unsigned pb = static_cast<unsigned>((work + wpb - 1) / wpb);
    CHRONOS_CUDA_CHECK(launch_kernel(ep_pack_kernel<T>, dim3(pb), dim3(kEpPackThreads), 0, st, true, p));
    return CHRONOS_OK;
}

template <typename T>
int ep_combine_impl(const ChronosEpCombineArgs* a, cudaStream_t st) {
    EpCombineParams p{};
    p.y_shared = a->y_shared;
    p.recv_y = a->recv_y;
    p.pair_slot = a->pair_slot;
    p.y = a->y;
    p.n = a->num_tokens;
    p.h = a->hidden;
    p.k = a->top_k;
    if (p.n == 0) return CHRONOS_OK;
    CHRONOS_CUDA_CHECK(launch_kernel(ep_combine_kernel<T>, dim3(static_cast<unsigned>(p.n)),
                                     dim3(kEpCombineThreads), 0, st, false, p));
    return CHRONOS_OK;
}

}  // namespace
}  // namespace chronos

extern "C" int chronos_ep_dispatch(const ChronosEpDispatchArgs* a, void* stream) {
    using namespace chronos;
    if (a == nullptr) return fail(CHRONOS_ERR_INVALID_ARG, "args is NULL");
    if (int rc = validate_ep_rows(a->num_tokens, a->hidden, a->top_k, a->dtype)) return rc;
    if (a->world_size < 1 || a->world_size > CHRONOS_EP_MAX_RANKS)
        return fail(CHRONOS_ERR_INVALID_ARG, "world_size %d out of range [1, %d]", a->world_size,
                    CHRONOS_EP_MAX_RANKS);
    if (static_cast<int64_t>(a->num_chunks < 1 ? 1 : a->num_chunks) * a->world_size > CHRONOS_EP_MAX_RANKS)
        return fail(CHRONOS_ERR_INVALID_ARG, "num_chunks %d x world_size %d exceeds %d", a->num_chunks,
                    a->world_size, CHRONOS_EP_MAX_RANKS);
    if (a->num_experts < 1 || a->num_experts % a->world_size != 0 || a->num_experts < a->top_k)
        return fail(CHRONOS_ERR_INVALID_ARG, "num_experts %d must be >= top_k and a multiple of world_size %d",
                    a->num_experts, a->world_size);
    if ((a->num_experts / a->world_size) % (a->num_chunks < 1 ? 1 : a->num_chunks) != 0)
        return fail(CHRONOS_ERR_INVALID_ARG, "num_chunks %d does not divide the %d experts of a rank",
                    a->num_chunks, a->num_experts / a->world_size);
    if (a->meta_pairs > 1 &&
        (a->num_chunks > 1 || a->meta_pairs > kMaxTopKEp ||
         a->meta_pairs < std::min(a->top_k, a->num_experts / a->world_size)))
        return fail(CHRONOS_ERR_INVALID_ARG, "meta_pairs %d: deduplicated rows need one expert chunk and "
                    "min(top_k %d, experts per rank %d) <= meta_pairs <= %d", a->meta_pairs, a->top_k,
                    a->num_experts / a->world_size, kMaxTopKEp);
    if (a->send_counts == nullptr) return fail(CHRONOS_ERR_INVALID_ARG, "send_counts is required");
    if (a->seg_rows < 0 ||
        (a->seg_rows > 0 &&
         (a->num_chunks > 1 ||
          a->seg_rows < a->num_tokens * (a->meta_pairs > 1 ? 1 : std::min(a->top_k, a->num_experts / a->world_size)) ||
          a->seg_rows * a->world_size > (int64_t(1) << 31) - 1)))
        return fail(CHRONOS_ERR_INVALID_ARG, "seg_rows %lld: fixed segments need one expert chunk and room for "
                    "every row a rank can receive (num_tokens, or num_tokens * min(top_k, experts per rank) "
                    "without deduplication)", static_cast<long long>(a->seg_rows));
    if (a->seg_rows > 0 && a->send_meta == nullptr)
        return fail(CHRONOS_ERR_INVALID_ARG, "send_meta is required with fixed segments");
    if (a->num_tokens > 0 &&
        (a->x == nullptr || a->topk_idx == nullptr || a->topk_weight == nullptr || a->send_x == nullptr ||
         a->send_meta == nullptr || a->pair_slot == nullptr ||
         a->shared_weight == nullptr || a->scratch == nullptr))
        return fail(CHRONOS_ERR_INVALID_ARG, "a required pointer is NULL");
    if ((reinterpret_cast<uintptr_t>(a->x) | reinterpret_cast<uintptr_t>(a->send_x)) & 15)
        return fail(CHRONOS_ERR_INVALID_ARG, "x and send_x must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (a->dtype) {
        case CHRONOS_DTYPE_BF16: return ep_dispatch_impl<__nv_bfloat16>(a, st);
        case CHRONOS_DTYPE_FP16: return ep_dispatch_impl<__half>(a, st);
        default: return ep_dispatch_impl<float>(a, st);
    }
}

extern "C" int chronos_ep_combine(const ChronosEpCombineArgs* a, void* stream) {
    using namespace chronos;
    if (a == nullptr) return fail(CHRONOS_ERR_INVALID_ARG, "args is NULL");
    if (int rc = validate_ep_rows(a->num_tokens, a->hidden, a->top_k, a->dtype)) return rc;
    if (a->num_tokens > 0 && (a->recv_y == nullptr || a->pair_slot == nullptr || a->y == nullptr))
        return fail(CHRONOS_ERR_INVALID_ARG, "recv_y, pair_slot and y are required");
    if ((reinterpret_cast<uintptr_t>(a->recv_y) | reinterpret_cast<uintptr_t>(a->y) |
         reinterpret_cast<uintptr_t>(a->y_shared)) & 15)
        return fail(CHRONOS_ERR_INVALID_ARG, "row buffers must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (a->dtype) {
        case CHRONOS_DTYPE_BF16: return ep_combine_impl<__nv_bfloat16>(a, st);
        case CHRONOS_DTYPE_FP16: return ep_combine_impl<__half>(a, st);
        default: return ep_combine_impl<float>(a, st);
    }
}

extern "C" size_t chronos_ep_dispatch_args_size(void) { return sizeof(ChronosEpDispatchArgs); }
extern "C" size_t chronos_ep_combine_args_size(void) { return sizeof(ChronosEpCombineArgs); }

// ---------------------------------------------------------------------------
// lookahead router (include/chronos_lookahead.h)
// ---------------------------------------------------------------------------
namespace chronos {
namespace {

// Whether a cluster of `cs` lookahead CTAs with `smem` bytes each can be
// placed on this GPU (checked once per shape and device).
template <typename T>
bool lookahead_cluster_fits(int cs, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, size_t>, bool> seen;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_tuple(dev, cs, smem);
    auto it = seen.find(key);
    if (it != seen.end()) return it->second;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(cs);
    cfg.blockDim = dim3(kLookaheadThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    const bool ok = cudaOccupancyMaxActiveClusters(&clusters, lookahead_kernel<T>, &cfg) == cudaSuccess &&
                    clusters >= 1;
    cudaGetLastError();   // a refused query leaves no error behind
    seen[key] = ok;
    return ok;
}

template <typename T>
int lookahead_impl(const ChronosLookaheadArgs* a, cudaStream_t st) {
    LookaheadParams p{};
    p.x = a->x;
    p.w1 = a->w1;
    p.w2 = a->w2;
    p.probs = a->probs;
    p.n = a->num_tokens;
    p.h = a->hidden;
    p.inner = a->inner;
    p.e = a->num_experts;
    p.k = a->steps;
    if (p.n == 0) return CHRONOS_OK;
    auto aligned16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    p.vec1 = (p.h % 8 == 0 && aligned16(p.x) && aligned16(p.w1)) ? 1 : 0;
    p.vec2 = (p.inner % 8 == 0 && aligned16(p.w2)) ? 1 : 0;
    // one CTA per 32 W1 rows (a pass of 8 warps x 4 rows), at most 8
    int cs = std::min(kLookaheadMaxCluster, std::max(1, (p.inner + 31) / 32));
    // tokens per cluster: up to 8 (every W1 row read once per 8 tokens), fewer
    // when that leaves SMs idle (a 32-token decode batch: 2 per cluster, 128 CTAs)
    const int64_t fill = (p.n * cs + sm_count() - 1) / sm_count();
    p.tb = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({static_cast<int64_t>(kLookaheadMaxTB), fill,
                                                                    kLookaheadXBytes / (p.h * 4)})));
    size_t smem = 0;
    for (;; cs /= 2) {
        p.rpc = (p.inner + cs - 1) / cs;
        smem = lookahead_smem(p.tb, p.h, p.rpc, p.inner, p.e * p.k);
        if (int rc = set_smem(lookahead_kernel<T>, static_cast<int>(smem))) return rc;
        if (cs == 1 || lookahead_cluster_fits<T>(cs, smem)) break;
    }
    const int64_t groups = (p.n + p.tb - 1) / p.tb;
    if (groups * cs > (int64_t(1) << 31) - 1)
        return fail(CHRONOS_ERR_INVALID_ARG, "lookahead: %lld tokens need too many blocks",
                    static_cast<long long>(p.n));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(groups * cs));
    cfg.blockDim = dim3(kLookaheadThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_model_pdl.load() ? 2 : 1;
    count_launch();
    CHRONOS_CUDA_CHECK(cudaLaunchKernelEx(&cfg, lookahead_kernel<T>, p));
    return CHRONOS_OK;
}

}  // namespace
}  // namespace chronos

extern "C" int chronos_lookahead_forward(const ChronosLookaheadArgs* a, void* stream) {
    using namespace chronos;
    if (a == nullptr) return fail(CHRONOS_ERR_INVALID_ARG, "args is NULL");
    if (a->num_tokens < 0 || a->num_tokens > (int64_t(1) << 24))
        return fail(CHRONOS_ERR_INVALID_ARG, "num_tokens %lld out of range", static_cast<long long>(a->num_tokens));
    if (a->hidden < 1 || a->hidden > 8192 || a->inner < 1 || a->inner > 2048 || a->num_experts < 1 ||
        a->steps < 1 || static_cast<int64_t>(a->num_experts) * a->steps > 4096)
        return fail(CHRONOS_ERR_INVALID_ARG, "lookahead shape out of range (H %d, inner %d, E %d, K %d)",
                    a->hidden, a->inner, a->num_experts, a->steps);
    if (a->dtype != CHRONOS_DTYPE_BF16 && a->dtype != CHRONOS_DTYPE_FP16 && a->dtype != CHRONOS_DTYPE_FP32)
        return fail(CHRONOS_ERR_INVALID_ARG, "dtype %d unknown", a->dtype);
    if (a->num_tokens > 0 && (a->x == nullptr || a->w1 == nullptr || a->w2 == nullptr || a->probs == nullptr))
        return fail(CHRONOS_ERR_INVALID_ARG, "x, w1, w2 and probs are required");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (a->dtype) {
        case CHRONOS_DTYPE_BF16: return lookahead_impl<__nv_bfloat16>(a, st);
        case CHRONOS_DTYPE_FP16: return lookahead_impl<__half>(a, st);
        default: return lookahead_impl<float>(a, st);
    }
}

extern "C" size_t chronos_lookahead_args_size(void) { return sizeof(ChronosLookaheadArgs); }

// ---------------------------------------------------------------------------
// hybrid-attention decode and residual add + RMSNorm (include/chronos_attention.h)
// ---------------------------------------------------------------------------
namespace chronos {
namespace {

constexpr int kAttnMaxSmem = 200 << 10;
constexpr int kAttnMaxSplits = 8;   // CTAs per (kv head, batch row): a portable cluster

bool known_dtype(int32_t d) {
    return d == CHRONOS_DTYPE_BF16 || d == CHRONOS_DTYPE_FP16 || d == CHRONOS_DTYPE_FP32;
}

int attn_common_checks(const ChronosAttnArgs* a, const char* what) {
    if (a == nullptr) return fail(CHRONOS_ERR_INVALID_ARG, "%s: args is NULL", what);
    if (a->batch < 0 || a->heads < 1 || a->kv_heads < 1 || a->heads % a->kv_heads != 0 ||
        a->heads / a->kv_heads > kAttnMaxRep)
        return fail(CHRONOS_ERR_INVALID_ARG, "%s: batch %d, heads %d, kv_heads %d (heads must be a "
                    "multiple of kv_heads, at most %d per kv head)", what, a->batch, a->heads, a->kv_heads,
                    kAttnMaxRep);
    if (a->head_dim < 8 || a->head_dim > 256 || (a->head_dim % 8))
        return fail(CHRONOS_ERR_INVALID_ARG, "%s: head_dim %d (a multiple of 8, <= 256)", what, a->head_dim);
    if (!known_dtype(a->dtype)) return fail(CHRONOS_ERR_INVALID_ARG, "%s: dtype %d unknown", what, a->dtype);
    if (a->table_len < 1) return fail(CHRONOS_ERR_INVALID_ARG, "%s: table_len %d", what, a->table_len);
    if (a->batch > 0 && (a->pos == nullptr || a->proj == nullptr || a->norm_q == nullptr ||
                         a->norm_q2 == nullptr || a->cos == nullptr || a->sin == nullptr ||
                         a->cache_a == nullptr || a->cache_b == nullptr || a->out == nullptr))
        return fail(CHRONOS_ERR_INVALID_ARG, "%s: a required pointer is NULL", what);
    return CHRONOS_OK;
}

AttnParams attn_params(const ChronosAttnArgs* a) {
    AttnParams p{};
    p.heads = a->heads;
    p.kv_heads = a->kv_heads;
    p.rep = a->heads / a->kv_heads;
    p.head_dim = a->head_dim;
    p.rope_dim = a->rope_dim;
    p.nope = a->head_dim - a->rope_dim;
    p.latent = a->latent;
    p.window = a->window;
    p.max_len = a->max_len;
    p.table_len = a->table_len;
    p.eps = a->eps;
    p.scale = 1.0f / sqrtf(static_cast<float>(a->head_dim));
    p.pos = a->pos;
    p.proj = a->proj;
    p.norm_q = a->norm_q;
    p.norm_q2 = a->norm_q2;
    p.norm_kv = a->norm_kv;
    p.w_krope = a->w_krope;
    p.w_knope = a->w_knope;
    p.w_v = a->w_v;
    p.cos = a->cos;
    p.sin = a->sin;
    p.cache_a = a->cache_a;
    p.cache_b = a->cache_b;
    p.out = a->out;
    return p;
}

// Shared memory of one decode CTA, in the order the kernels lay it out.
// The weight slices of an MLA CTA (k_nope_proj and k_rope_proj slices of its
// kv head, its share of the v_proj rows), when staged in shared memory.
size_t mla_wstage_bytes(const AttnParams& p, size_t elem) {
    const int dper = (p.head_dim + p.splits - 1) / p.splits;
    return elem * static_cast<size_t>(p.latent) * (p.nope + p.rope_dim + dper);
}

size_t mla_smem_base(const AttnParams& p) {
    const size_t rep = static_cast<size_t>(p.rep);
    return sizeof(float) * (rep * p.nope               // qn
                            + rep * p.rope_dim         // qr
                            + 3 * rep * p.latent       // qabs, ctx, part
                            + p.latent + p.rope_dim    // cnew, krn
                            + (rep + 1) * p.rope_dim   // tmp
                            + p.nope + p.rope_dim + p.latent   // norm weights
                            + 2 * p.rope_dim           // cos, sin
                            + 2 * kAttnMaxRep          // red
                            + attn_red_floats(p.rep, p.latent)   // weighted-sum reduction
                            + rep * p.cap);            // scores
}

size_t sw_smem(const AttnParams& p) {
    const size_t rep = static_cast<size_t>(p.rep);
    return sizeof(float) * (rep * p.head_dim           // q
                            + 2 * p.head_dim           // kn, vn
                            + (rep + 1) * p.head_dim   // tmp
                            + 4 * p.head_dim           // norm weights, cos, sin
                            + rep * p.head_dim         // part
                            + 2 * kAttnMaxRep          // red
                            + attn_red_floats(p.rep, p.head_dim)   // weighted-sum reduction
                            + rep * p.cap);            // scores
}

// How many clusters of `splits` CTAs of `kernel` with `smem` bytes each this
// GPU runs at once (0: none can be placed); queried once per kernel, device
// and shape.
int attn_active_clusters(void (*kernel)(AttnParams), int splits, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int, size_t>, int> seen;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_tuple(reinterpret_cast<const void*>(kernel), dev, splits, smem);
    auto it = seen.find(key);
    if (it != seen.end()) return it->second;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(splits);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) clusters = 0;
    cudaGetLastError();   // a refused query leaves no error behind
    seen[key] = clusters;
    return clusters;
}

// Split the positions over `splits` CTAs: the score capacity per CTA and, for
// MLA, whether the weight slices fit in shared memory beside everything else.
size_t attn_layout(AttnParams& p, bool mla, int splits, size_t elem) {
    p.splits = splits;
    p.cap = ((mla ? p.max_len : p.window) + splits - 1) / splits;
    if (!mla) return sw_smem(p);
    const size_t base = mla_smem_base(p), w = mla_wstage_bytes(p, elem);
    p.stage_w = base + w <= static_cast<size_t>(kAttnMaxSmem) ? 1 : 0;
    return base + (p.stage_w ? w : 0);
}

// Choose the split of this call: the most CTAs per (kv head, row) pair (at
// most a portable cluster of 8) whose clusters all run in one wave; the fewest
// whose shared memory fits when no split runs in one wave.  0 or an error.
int attn_plan(AttnParams& p, bool mla, int batch, size_t elem, void (*kernel)(AttnParams), size_t* smem,
              const char* what) {
    int s_min = 1;
    *smem = attn_layout(p, mla, s_min, elem);
    while (*smem > static_cast<size_t>(kAttnMaxSmem) && s_min < kAttnMaxSplits)
        *smem = attn_layout(p, mla, ++s_min, elem);
    if (*smem > static_cast<size_t>(kAttnMaxSmem))
        return fail(CHRONOS_ERR_INVALID_ARG, "%s: %d cached positions x %d heads per kv head need %zu bytes of "
                    "shared memory per CTA at %d CTAs per head group (limit %d)", what,
                    mla ? p.max_len : p.window, p.rep, *smem, s_min, kAttnMaxSmem);
    if (batch == 0) return CHRONOS_OK;
    const int64_t items = static_cast<int64_t>(p.kv_heads) * batch;
    int best = 0;
    for (int sp = kAttnMaxSplits; sp >= s_min && best == 0; --sp) {
        const size_t sm = attn_layout(p, mla, sp, elem);
        if (int rc = set_smem(kernel, static_cast<int>(sm))) return rc;
        if (attn_active_clusters(kernel, sp, sm) >= items) best = sp;
    }
    if (best == 0) {
        best = s_min;
        while (best <= kAttnMaxSplits && attn_active_clusters(kernel, best, attn_layout(p, mla, best, elem)) < 1)
            ++best;
        if (best > kAttnMaxSplits)
            return fail(CHRONOS_ERR_CUDA, "%s: no cluster of %d..%d CTAs can be placed", what, s_min,
                        kAttnMaxSplits);
    }
    *smem = attn_layout(p, mla, best, elem);
    return set_smem(kernel, static_cast<int>(*smem));
}

int attn_launch(void (*kernel)(AttnParams), const AttnParams& p, int batch, size_t smem, cudaStream_t st) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(p.kv_heads * p.splits), static_cast<unsigned>(batch));
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = p.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_model_pdl.load() ? 2 : 1;
    count_launch();
    CHRONOS_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, p));
    return CHRONOS_OK;
}

// The decode kernel for `rep` query heads per kv head (1..8).
template <typename T, int REP>
void (*attn_kernel_rep(bool mla))(AttnParams) {
    return mla ? mla_decode_kernel<T, REP> : sw_decode_kernel<T, REP>;
}
template <typename T>
void (*attn_kernel(bool mla, int rep))(AttnParams) {
    switch (rep) {
        case 1: return attn_kernel_rep<T, 1>(mla);
        case 2: return attn_kernel_rep<T, 2>(mla);
        case 3: return attn_kernel_rep<T, 3>(mla);
        case 4: return attn_kernel_rep<T, 4>(mla);
        case 5: return attn_kernel_rep<T, 5>(mla);
        case 6: return attn_kernel_rep<T, 6>(mla);
        case 7: return attn_kernel_rep<T, 7>(mla);
        default: return attn_kernel_rep<T, 8>(mla);
    }
}

template <typename T>
int attn_impl(AttnParams p, bool mla, int batch, cudaStream_t st, const char* what) {
    void (*kernel)(AttnParams) = attn_kernel<T>(mla, p.rep);
    size_t smem = 0;
    if (int rc = attn_plan(p, mla, batch, sizeof(T), kernel, &smem, what)) return rc;
    if (batch == 0) return CHRONOS_OK;
    return attn_launch(kernel, p, batch, smem, st);
}

template <typename T>
int norm_impl(const ChronosNormArgs* a, cudaStream_t st) {
    NormParams p{};
    p.rows = a->rows;
    p.width = a->width;
    p.eps = a->eps;
    p.x_fp32 = a->x_fp32 ? 1 : 0;
    p.x = a->x;
    p.residual = a->residual;
    p.sum_out = a->sum_out;
    p.weight = a->weight;
    p.out = a->out;
    auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    if (a->width % 8 == 0 && a->width <= 8 * 256 && a16(a->x) && a16(a->weight) && a16(a->out) &&
        (a->residual == nullptr || a16(a->residual)) && (a->sum_out == nullptr || a16(a->sum_out))) {
        // one warp per row, the row in registers
        const unsigned grid = static_cast<unsigned>((a->rows + kAttnWarps - 1) / kAttnWarps);
        const int vpl = (a->width + 255) / 256;
        void (*kernel)(NormParams) = vpl <= 1 ? add_rmsnorm_warp_kernel<T, 1>
                                     : vpl <= 2 ? add_rmsnorm_warp_kernel<T, 2>
                                     : vpl <= 4 ? add_rmsnorm_warp_kernel<T, 4>
                                                : add_rmsnorm_warp_kernel<T, 8>;
        CHRONOS_CUDA_CHECK(launch_kernel(kernel, dim3(grid), dim3(kAttnThreads), 0, st, g_model_pdl.load(), p));
        return CHRONOS_OK;
    }
    const int smem = static_cast<int>(sizeof(float) * (a->width + kAttnWarps));
    if (int rc = set_smem(add_rmsnorm_kernel<T>, smem)) return rc;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(a->rows, 1 << 20));
    CHRONOS_CUDA_CHECK(launch_kernel(add_rmsnorm_kernel<T>, dim3(grid), dim3(kAttnThreads), smem, st,
                                     g_model_pdl.load(), p));
    return CHRONOS_OK;
}

}  // namespace
}  // namespace chronos

extern "C" int chronos_mla_decode(const ChronosAttnArgs* a, void* stream) {
    using namespace chronos;
    g_last_error.clear();
    if (int rc = attn_common_checks(a, "chronos_mla_decode")) return rc;
    if (a->rope_dim < 8 || (a->rope_dim % 8) || a->rope_dim >= a->head_dim || a->latent < 8 ||
        a->latent > 256 || (a->latent % 8) || a->max_len < 1 || a->max_len > 8192)
        return fail(CHRONOS_ERR_INVALID_ARG, "chronos_mla_decode: rope_dim %d (a multiple of 8, < head_dim %d), "
                    "latent %d (a multiple of 8, <= 256), max_len %d (1..8192)", a->rope_dim, a->head_dim,
                    a->latent, a->max_len);
    if (a->batch > 0 && (a->norm_kv == nullptr || a->w_krope == nullptr || a->w_knope == nullptr ||
                         a->w_v == nullptr))
        return fail(CHRONOS_ERR_INVALID_ARG, "chronos_mla_decode: norm_kv, w_krope, w_knope and w_v are required");
    const AttnParams p = attn_params(a);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (a->dtype) {
        case CHRONOS_DTYPE_BF16: return attn_impl<__nv_bfloat16>(p, true, a->batch, st, "chronos_mla_decode");
        case CHRONOS_DTYPE_FP16: return attn_impl<__half>(p, true, a->batch, st, "chronos_mla_decode");
        default: return attn_impl<float>(p, true, a->batch, st, "chronos_mla_decode");
    }
}

extern "C" int chronos_sw_decode(const ChronosAttnArgs* a, void* stream) {
    using namespace chronos;
    g_last_error.clear();
    if (int rc = attn_common_checks(a, "chronos_sw_decode")) return rc;
    if (a->rope_dim != a->head_dim || a->window < 1 || a->max_len != a->window)
        return fail(CHRONOS_ERR_INVALID_ARG, "chronos_sw_decode: rope_dim %d must equal head_dim %d, window %d "
                    ">= 1 and max_len %d == window", a->rope_dim, a->head_dim, a->window, a->max_len);
    const AttnParams p = attn_params(a);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (a->dtype) {
        case CHRONOS_DTYPE_BF16: return attn_impl<__nv_bfloat16>(p, false, a->batch, st, "chronos_sw_decode");
        case CHRONOS_DTYPE_FP16: return attn_impl<__half>(p, false, a->batch, st, "chronos_sw_decode");
        default: return attn_impl<float>(p, false, a->batch, st, "chronos_sw_decode");
    }
}

extern "C" int chronos_add_rmsnorm(const ChronosNormArgs* a, void* stream) {
    using namespace chronos;
    g_last_error.clear();
    if (a == nullptr) return fail(CHRONOS_ERR_INVALID_ARG, "chronos_add_rmsnorm: args is NULL");
    if (a->rows < 0 || a->width < 1 || a->width > 16384 || !known_dtype(a->dtype))
        return fail(CHRONOS_ERR_INVALID_ARG, "chronos_add_rmsnorm: rows %lld, width %d (1..16384), dtype %d",
                    static_cast<long long>(a->rows), a->width, a->dtype);
    if (a->rows > 0 && (a->x == nullptr || a->weight == nullptr || a->out == nullptr))
        return fail(CHRONOS_ERR_INVALID_ARG, "chronos_add_rmsnorm: x, weight and out are required");
    if (a->rows == 0) return CHRONOS_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (a->dtype) {
        case CHRONOS_DTYPE_BF16: return norm_impl<__nv_bfloat16>(a, st);
        case CHRONOS_DTYPE_FP16: return norm_impl<__half>(a, st);
        default: return norm_impl<float>(a, st);
    }
}

extern "C" int chronos_argmax_rows(const void* x, int64_t rows, int32_t cols, int32_t dtype, int64_t* out,
                                   void* stream) {
    using namespace chronos;
    g_last_error.clear();
    if (rows < 0 || cols < 1 || !known_dtype(dtype))
        return fail(CHRONOS_ERR_INVALID_ARG, "chronos_argmax_rows: rows %lld, cols %d, dtype %d",
                    static_cast<long long>(rows), cols, dtype);
    if (rows > 0 && (x == nullptr || out == nullptr))
        return fail(CHRONOS_ERR_INVALID_ARG, "chronos_argmax_rows: x and out are required");
    if (rows == 0) return CHRONOS_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const dim3 grid(static_cast<unsigned>(std::min<int64_t>(rows, 1 << 20)));
    switch (dtype) {
        case CHRONOS_DTYPE_BF16:
            CHRONOS_CUDA_CHECK(launch_kernel(argmax_rows_kernel<__nv_bfloat16>, grid, dim3(kAttnThreads), 0, st,
                                             g_model_pdl.load(), static_cast<const __nv_bfloat16*>(x), rows, static_cast<int>(cols), out));
            break;
        case CHRONOS_DTYPE_FP16:
            CHRONOS_CUDA_CHECK(launch_kernel(argmax_rows_kernel<__half>, grid, dim3(kAttnThreads), 0, st,
                                             g_model_pdl.load(),
                                             static_cast<const __half*>(x), rows, static_cast<int>(cols), out));
            break;
        default:
            CHRONOS_CUDA_CHECK(launch_kernel(argmax_rows_kernel<float>, grid, dim3(kAttnThreads), 0, st,
                                             g_model_pdl.load(),
                                             static_cast<const float*>(x), rows, static_cast<int>(cols), out));
    }
    return CHRONOS_OK;
}

extern "C" size_t chronos_attn_args_size(void) { return sizeof(ChronosAttnArgs); }
extern "C" size_t chronos_norm_args_size(void) { return sizeof(ChronosNormArgs); }
