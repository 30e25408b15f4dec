// C ABI of libmoelab_b200 (declared in include/moelab_b200.h). Plain pointers and sizes, int status,
// no allocation, no host synchronisation except moeb_read_error.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <tuple>
#include <unordered_map>

#include "../../include/moelab_b200.h"
#include "common.cuh"
#include "kernels.h"

using namespace moeb;

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char *fmt, const char *detail = "") {
    snprintf(g_err, sizeof g_err, fmt, detail);
    return code;
}

int check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        snprintf(g_err, sizeof g_err, "%s: %s", what, cudaGetErrorString(e));
        return MOEB_ELAUNCH;
    }
    return MOEB_OK;
}

int sm_count() {
    static std::mutex mu;
    static std::unordered_map<int, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(dev);
    if (it != cache.end()) return it->second;
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n;
    return n;
}

int occupancy(const void *fn, int threads, size_t smem) {
    static std::mutex mu;
    static std::unordered_map<const void *, int> cache;
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(fn);
    if (it != cache.end()) return it->second;
    int n = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem);
    if (n < 1) n = 1;
    cache[fn] = n;
    return n;
}

// Launch with programmatic dependent launch so the kernel's prologue overlaps the previous kernel's tail;
// every kernel calls griddepcontrol.wait before touching data produced upstream.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// The same with thread-block clusters of cluster_x CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster_x,
                           Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Workspace layout for up to Tc tokens. The first region holds counters that must be zero before the first
// call (moeb_workspace_init); every kernel leaves them zero again.
struct Layout {
    size_t err, cnt_all, rcnt, ycnt, zero_end;
    size_t logits, idx, wts, xsum, ntiles, tiles, sorted, h, hsum, yp, xg, drec, total;
};

// with_yp = false: no per-slot output region (expert-parallel calls write the slot outputs to the caller's buffer).
Layout layout(long Tc, int d, int f, int E, int k, bool with_yp = true) {
    Layout L;
    const long TK = Tc * k;
    size_t o = 0;
    L.err = o; o += 256;
    L.cnt_all = o; o += 256;
    L.rcnt = o; o = align256(o + 4 * (size_t)Tc);  // one counter per router token block (>= 1 token each)
    L.ycnt = o; o = align256(o + 4 * (size_t)Tc * (d / 16));
    L.zero_end = o;
    L.logits = o; o = align256(o + 4 * (size_t)Tc * E);
    L.idx = o; o = align256(o + 4 * (size_t)TK);
    L.wts = o; o = align256(o + 4 * (size_t)TK);
    L.xsum = o; o = align256(o + 4 * (size_t)Tc * xsum_stride(d));
    L.ntiles = o; o += 256;
    L.tiles = o; o = align256(o + 16 * (size_t)(TK + E + 1));
    L.sorted = o; o = align256(o + 4 * (size_t)TK);
    L.h = o; o = align256(o + 2 * (size_t)TK * f);
    L.hsum = o; o = align256(o + 4 * (size_t)TK * (f / 16));
    L.yp = o; o = align256(o + (with_yp ? 4 * (size_t)TK * d : 0));
    // expert-parallel rows gathered in expert order for the tensor-core kernels (a layer call uses the slot-row
    // region for that)
    L.xg = o; o = align256(o + (with_yp ? 0 : 2 * (size_t)TK * d));
    // single-kernel decode (<= 16 slots): tagged 64-bit records of h [slot][f] and of the slot outputs [slot][d]
    L.drec = o; o = align256(o + (with_yp ? 8 * (size_t)std::min<long>(TK, 16) * (f + d) : 0));
    L.total = o;
    return L;
}

// Largest token capacity whose layout fits in `bytes` (layout size is monotone in T).
long capacity(size_t bytes, int d, int f, int E, int k, bool with_yp = true) {
    long lo = 0, hi = 1;
    while (layout(hi, d, f, E, k, with_yp).total <= bytes && hi < (1L << 24)) hi *= 2;
    while (lo < hi) {
        long mid = (lo + hi + 1) / 2;
        if (layout(mid, d, f, E, k, with_yp).total <= bytes) lo = mid; else hi = mid - 1;
    }
    return lo;
}

template <typename T>
T *at(void *ws, size_t off) { return reinterpret_cast<T *>(static_cast<char *>(ws) + off); }

int check_shape(int T, int d, int f, int E, int k) {
    if (T < 0 || d <= 0 || f <= 0 || E <= 0 || k <= 0) return fail(MOEB_EINVAL, "non-positive dimension%s");
    if (d % 64 || f % 64) return fail(MOEB_EINVAL, "d and f must be multiples of 64%s");
    if (k > 32 || k > E) return fail(MOEB_EINVAL, "k must be <= min(E, 32)%s");
    if (E > 1024) return fail(MOEB_EINVAL, "E must be <= 1024%s");
    return MOEB_OK;
}

// ------------------------------------------------------------------ dispatcher
// Load = T*k/E (average slots per expert; the reference's policy variable, metal_q4_moe.py:42-46).
// Measured on B200 (Qwen3-30B shape, 16 layers cycled, CUDA graph): the split-K decode kernels win up to 16
// slots (T <= 2 at k = 8); above that the warp-specialized tensor-map pipeline beats the register tiles at
// every load (T = 4: 50.8 vs 55.6 us, T = 32: 126 vs 145 us), with tiles of 8 slots up to load ~4 and tiles of
// 16 at high load (T = 256, load 16: 291 vs 329 us).
// From 24 slots per expert the tcgen05 kernels (weights dequantized once per tile, A operand in TMEM) win:
// Qwen3-30B T = 384 / 512 / 1024 (load 24 / 32 / 64): 235 / 263 / 429 us vs ring16 275 / 346 / 603 us; below
// that the tile kernels do (T = 256, load 16: 228 vs 208 us). Each M = 128, K = 16 tensor-core step costs about
// the same up to N = 128 slots, so small tiles leave the tensor pipe mostly idle.
int choose_policy(int T, int E, int k, int d, int f) {
    const long TK = (long)T * k;
    if (TK <= 16) return MOEB_POLICY_SLOTS;
    // tcgen05 from 14 slots per expert (Qwen3-30B T = 192 / 224 / 256: 179.7 / 181.4 / 183.5 us against 172.9 /
    // 206.5 / 216.6 with tiles of 16 and 207.5 / 211.1 / 215.9 with tiles of 24)
    if (TK >= 14L * E && d % 128 == 0 && f % 128 == 0) return MOEB_POLICY_TC;
    if (TK >= 16L * E) return MOEB_POLICY_TILES24_RING;  // shapes the tcgen05 kernels do not take
    return TK >= 8L * E ? MOEB_POLICY_TILES16_RING : MOEB_POLICY_TILES8_RING;
}

// tcgen05 tile size: the smallest of 32, 64, 128, 192, 256 at or above 1.5 x the average expert's slots, so that
// most experts fit one tile (weights are dequantized once per tile; a second, partial tile reads them again).
int tc_nt(long TK, int E) {
    const long load = TK / std::max(E, 1), need = load + load / 2;
    return need > 192 ? 256 : need > 128 ? 192 : need > 64 ? 128 : need > 32 ? 64 : 32;
}

int nt_of(int policy, long TK, int E) {
    if (policy == MOEB_POLICY_TC) return tc_nt(TK, E);
    if (policy == MOEB_POLICY_TILES24_RING) return 24;
    return (policy == MOEB_POLICY_TILES16 || policy == MOEB_POLICY_TILES16_RING) ? 16 : 8;
}
bool is_tiles(int policy) {
    return (policy >= MOEB_POLICY_TILES8 && policy <= MOEB_POLICY_TC) || policy == MOEB_POLICY_TILES24_RING;
}

// One expert kernel launch: per_warp kernels run one (tile, 16-row block) unit per warp; the others one unit
// per CTA, where a warp-specialized kernel's unit is `rows` consecutive row blocks (rows > 1 also means it
// reads the weights through tensor maps whose box is rows x sg).
struct KLaunch {
    void (*fn)(ExpArgs);
    int threads;
    size_t smem;
    bool per_warp;
    int rows, sg;
    bool tc = false;  // tensor-core kernel: reads the activations through the expert-sorted row map
    bool tmem_a = false;  // tensor-core kernel with A in TMEM: activations in the permuted 64-group k order
};
struct ExpLaunch {
    KLaunch gu, dn;
};

constexpr int WS_RBC = 8, WS_SG = 4, WS_NS_GU = 2, WS_NS_DN = 4, WS_NS_DN24 = 3;  // (3: two CTAs per SM at 24 slots)

template <int FMT>
KLaunch ws_kernel_fmt(int nt8, bool down) {
    void (*fn)(ExpArgs) = nullptr;
    if (nt8 == 1) fn = down ? k_experts_ws<FMT, 1, WS_RBC, WS_SG, WS_NS_DN, true, 2>
                            : k_experts_ws<FMT, 1, WS_RBC, WS_SG, WS_NS_GU, false, 2>;
    else if (nt8 == 2) fn = down ? k_experts_ws<FMT, 2, WS_RBC, WS_SG, WS_NS_DN, true, 2>
                                 : k_experts_ws<FMT, 2, WS_RBC, WS_SG, WS_NS_GU, false, 2>;
    else fn = down ? k_experts_ws<FMT, 3, WS_RBC, WS_SG, WS_NS_DN24, true, 2>
                   : k_experts_ws<FMT, 3, WS_RBC, WS_SG, WS_NS_GU, false, 2>;
    const int ns = down ? (nt8 == 3 ? WS_NS_DN24 : WS_NS_DN) : WS_NS_GU;
    return {fn, 32 * (WS_RBC + 1), experts_ws_smem(nt8, WS_RBC, WS_SG, ns, down, FMT), false, WS_RBC, WS_SG};
}
KLaunch ws_kernel(int fmt, int nt8, bool down) {
    return fmt == FMT_FP4 ? ws_kernel_fmt<FMT_FP4>(nt8, down) : ws_kernel_fmt<FMT_Q4>(nt8, down);
}

KLaunch tc_kernel(int fmt, int nt, bool down) {
    const TcInfo t = experts_tc_info(fmt, nt, down);
    return {t.fn, t.threads, t.smem, false, 8, t.sg, true, t.tmem_a};
}

// Kernels per policy: TILES8 / TILES16 run the register-pipelined tile kernels, the *_RING policies the
// warp-specialized tensor-map pipeline (faster on B200 for both projections, so the dispatcher picks it).
ExpLaunch pick_kernels(int fmt, int policy, int d, int f, int nt) {
    const KLaunch none = {nullptr, 0, 0, false, 1, 0};
    if (fmt != FMT_Q4 && fmt != FMT_FP4) return {none, none};
    if (policy == MOEB_POLICY_SLOTS) {
        if (fmt == FMT_FP4)
            return {{k_gate_up_slots<FMT_FP4, 8, 4>, 256, (size_t)d * 2, false, 1, 0},
                    {k_down_slots<FMT_FP4, 4, 4>, 128, (size_t)f * 2 + (size_t)f / 16 * 4, false, 1, 0}};
        // int4: 4 warps split K, 8 groups each loaded at once (Qwen3-30B T=1: 20.64 us against 20.99 with 8 warps x
        // 4 groups and 22.48 with 16 x 2)
        return {{k_gate_up_slots<FMT_Q4, 4, 8>, 128, (size_t)d * 2, false, 1, 0},
                {k_down_slots<FMT_Q4, 4, 4>, 128, (size_t)f * 2 + (size_t)f / 16 * 4, false, 1, 0}};
    }
    if (policy == MOEB_POLICY_TC) {
        if (d % 128 || f % 128) return {none, none};
        return {tc_kernel(fmt, nt, false), tc_kernel(fmt, nt, true)};
    }
    if (policy == MOEB_POLICY_TILES24_RING) return {ws_kernel(fmt, 3, false), ws_kernel(fmt, 3, true)};
    if (policy == MOEB_POLICY_TILES16_RING) return {ws_kernel(fmt, 2, false), ws_kernel(fmt, 2, true)};
    if (policy == MOEB_POLICY_TILES8_RING) return {ws_kernel(fmt, 1, false), ws_kernel(fmt, 1, true)};
    if (fmt == FMT_FP4) {
        if (policy == MOEB_POLICY_TILES16)
            return {{k_gate_up_tiles_reg<FMT_FP4, 2, 1>, 128, 0, true, 1, 0},
                    {k_down_tiles_reg<FMT_FP4, 2, 1>, 128, 0, true, 1, 0}};
        return {{k_gate_up_tiles_reg<FMT_FP4, 1, 2>, 128, 0, true, 1, 0},
                {k_down_tiles_reg<FMT_FP4, 1, 2>, 128, 0, true, 1, 0}};
    }
    if (policy == MOEB_POLICY_TILES16)
        return {{k_gate_up_tiles_reg<FMT_Q4, 2, 1>, 128, 0, true, 1, 0},
                {k_down_tiles_reg<FMT_Q4, 2, 1>, 128, 0, true, 1, 0}};
    return {{k_gate_up_tiles_reg<FMT_Q4, 1, 2>, 128, 0, true, 1, 0}, {k_down_tiles_reg<FMT_Q4, 1, 2>, 128, 0, true, 1, 0}};
}

// ---- tensor maps for the warp-specialized kernels (driver entry point, cached per weight array and shape)
PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D view of a fragment-major projection: rows = row blocks of all experts, each row the K/64 groups' bytes
// (codes: 512 B per group as uint64 elements; scale|bias: 64 B per group as uint32); box = brows rows x
// bgroups groups. words = 32-bit words per group (128 or 16).
bool encode_weights_map(CUtensorMap *out, const void *base, int words, long groups, long rows, int bgroups,
                        int brows) {
    using Key = std::tuple<const void *, int, long, long, int, int>;
    static std::mutex mu;
    static std::map<Key, CUtensorMap> cache;
    const Key key{base, words, groups, rows, bgroups, brows};
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    auto fn = tmap_encoder();
    if (!fn) return false;
    const bool wide = words == 128;  // codes: 8-byte elements keep the box row (SG * 512 B) within 256 elements
    const int esz = wide ? 8 : 4, per_group = words * 4 / esz;
    const cuuint64_t dims[2] = {(cuuint64_t)groups * per_group, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)groups * words * 4};
    const cuuint32_t box[2] = {(cuuint32_t)(bgroups * per_group), (cuuint32_t)brows};
    const cuuint32_t es[2] = {1, 1};
    if (box[0] > 256 || box[1] > 256) return false;
    CUtensorMap m;
    if (fn(&m, wide ? CU_TENSOR_MAP_DATA_TYPE_UINT64 : CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(base),
           dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    if (cache.size() > 4096) cache.clear();  // bounded: a long-lived process cycling through many weight sets
    cache[key] = m;
    *out = m;
    return true;
}

// Opt a kernel in to more than 48 KB of dynamic shared memory (once per kernel).
bool allow_smem(const void *fn, size_t bytes) {
    if (bytes <= 48 * 1024) return true;
    static std::mutex mu;
    static std::unordered_map<const void *, size_t> done;
    std::lock_guard<std::mutex> lk(mu);
    auto it = done.find(fn);
    if (it != done.end() && it->second >= bytes) return true;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess) return false;
    done[fn] = bytes;
    return true;
}

// The warp-specialized down kernel can combine in its epilogue (the last of a token's k slots to finish a 16-row
// block sums them, as the decode kernels do) or leave the weighted slot rows to a separate combine pass; the
// tensor-core down kernel always leaves them. MOEB_WS_COMBINE=fused|separate overrides the default (measurements).
bool separate_combine(const KLaunch &dn) {
    static const int mode = [] {
        const char *s = getenv("MOEB_WS_COMBINE");
        return s ? (strcmp(s, "fused") == 0 ? 1 : strcmp(s, "separate") == 0 ? 2 : 0) : 0;
    }();
    if (dn.tc) return true;
    if (dn.sg == 0) return false;
    return mode != 1;
}

// 2-D map over rows x d bf16 activations (row stride d * 2 bytes), box 64 x brows, 128-byte swizzle.
bool encode_rows_map(CUtensorMap *out, const void *base, long rows, int d, int brows) {
    auto fn = tmap_encoder();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)std::max<long>(rows, 1)};
    const cuuint64_t strides[1] = {(cuuint64_t)d * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)brows};
    const cuuint32_t es[2] = {1, 1};
    return fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int grid_for(const KLaunch &k, long units) {
    const long ctas = k.per_warp ? (units + k.threads / 32 - 1) / (k.threads / 32) : units;
    const long cap = (long)occupancy((const void *)k.fn, k.threads, k.smem) * sm_count();
    return (int)std::max<long>(1, std::min(ctas, cap));
}

// Warps per slot of the token-major decode down kernel: 2 (Qwen3-30B T=1 / 2: 20.02 / 32.93 us against 20.57 /
// 33.83 with 4, whose 1024-thread CTAs are capped at 64 registers and spill, and 20.68 / 33.30 with 1).
// MOEB_DOWN_TOK_KS=4 selects the 4-warp kernel (measurements).
int down_tok_ks() {
    static const int v = [] {
        const char *s = getenv("MOEB_DOWN_TOK_KS");
        return s && atoi(s) == 4 ? 4 : 2;
    }();
    return v;
}

// The decode down kernel reads its ids, weights and first weight batch before waiting for gate/up, and the
// warp-specialized down issues the weight copies of its first NS stages before it (MOEB_DOWN_EARLY=0: after, for
// measurements).
bool down_early() {
    static const int v = [] {
        const char *s = getenv("MOEB_DOWN_EARLY");
        return s ? atoi(s) : 1;
    }();
    return v != 0;
}

int run_experts(int fmt, ExpArgs a, int policy, const Layout &L, void *ws, cudaStream_t st,
                void *const *ev) {
    const long TK = (long)a.T * a.k;
    // tile size from the rows that carry work: a peer-exchange call's P blocks of Cs rows hold about Cs valid rows
    const int nt = nt_of(policy, a.ypeers ? (long)a.C : TK, a.E);
    const long max_tiles = a.tile_mode ? std::min<long>(TK, (long)a.E + TK / nt) : TK;
    ExpLaunch K = pick_kernels(fmt, policy, a.d, a.f, nt);
    if (!K.gu.fn) return fail(MOEB_EUNSUP, "format not supported%s");
    if (policy == MOEB_POLICY_SLOTS && (K.gu.smem > 48 * 1024 || K.dn.smem > 48 * 1024))
        return fail(MOEB_EINVAL, "d or f too large for the decode kernels%s");
    if (!allow_smem((const void *)K.gu.fn, K.gu.smem) || !allow_smem((const void *)K.dn.fn, K.dn.smem))
        return check_launch("cudaFuncSetAttribute");
    const int RBf = a.f / 16, RBd = a.d / 16;
    const int sw = fmt == FMT_FP4 ? 8 : 16;  // scale words per (row block, group)
    if (K.gu.sg) {
        if (!encode_weights_map(&a.tmq[0], a.g.q, 128, a.d / 64, (long)a.E * RBf, K.gu.sg, K.gu.rows) ||
            !encode_weights_map(&a.tmsb[0], a.g.sb, sw, a.d / 64, (long)a.E * RBf, K.gu.sg, K.gu.rows) ||
            !encode_weights_map(&a.tmq[1], a.u.q, 128, a.d / 64, (long)a.E * RBf, K.gu.sg, K.gu.rows) ||
            !encode_weights_map(&a.tmsb[1], a.u.sb, sw, a.d / 64, (long)a.E * RBf, K.gu.sg, K.gu.rows))
            return fail(MOEB_ELAUNCH, "tensor map encoding failed (gate/up)%s");
    }
    if (K.dn.sg) {
        if (!encode_weights_map(&a.tmq[2], a.dn.q, 128, a.f / 64, (long)a.E * RBd, K.dn.sg, K.dn.rows) ||
            !encode_weights_map(&a.tmsb[2], a.dn.sb, sw, a.f / 64, (long)a.E * RBd, K.dn.sg, K.dn.rows))
            return fail(MOEB_ELAUNCH, "tensor map encoding failed (down)%s");
    }
    a.h_kperm = K.dn.tc && K.dn.tmem_a ? 1 : 0;
    if (K.gu.tc) {  // activations in expert-sorted order: in the slot-row region (free until down writes it) of a
                    // layer call, in their own region for expert-parallel rows (whose slot outputs go elsewhere)
        uint16_t *xs = a.slot_out ? at<uint16_t>(ws, L.xg) : reinterpret_cast<uint16_t *>(a.yp);
        if (launch(k_gather_rows, dim3((unsigned)((TK + 7) / 8)), dim3(256), 0, st, a.x, (const int *)a.sorted, (int)TK,
                   a.k, a.d, a.xs, K.gu.tmem_a ? 1 : 0, xs) != cudaSuccess)
            return check_launch("gather");
        if (!encode_rows_map(&a.tmx, xs, TK, a.d, nt)) return fail(MOEB_ELAUNCH, "tensor map encoding failed (x)%s");
    }
    // Warp-specialized pair at up to 2 slots per expert: down issues its first ring of weight copies before waiting
    // for gate/up, which then releases it only after its own wait (both kernels read the flag). Qwen3-30B, us per
    // layer, with / without: T = 4 45.7 / 47.5, 16 82.9 / 83.0, 32 111.5 / 111.7, 64 123.4 / 122.5, 128 160.8 / 159.1.
    a.early_ids = K.dn.sg && !K.dn.tc && K.gu.sg && !K.gu.tc && TK <= 2L * a.E && down_early() ? 1 : 0;
    {
        const long units = max_tiles * ((RBf + K.gu.rows - 1) / K.gu.rows);
        if (launch(K.gu.fn, dim3(grid_for(K.gu, units)), dim3(K.gu.threads), K.gu.smem, st, a) != cudaSuccess)
            return check_launch("gate_up");
    }
    if (K.dn.tc && !encode_rows_map(&a.tmx, a.h, TK, a.f, nt))
        return fail(MOEB_ELAUNCH, "tensor map encoding failed (h)%s");
    if (ev) cudaEventRecord(static_cast<cudaEvent_t>(ev[2]), st);
    // combine: fused into down (last arrival per (token, row block) sums the k slot rows), or a separate pass
    // over the weighted slot rows when down is the warp-specialized kernel (no fences / counters in its epilogue)
    const bool sep = !a.slot_out && separate_combine(K.dn);
    if (sep) a.slot_out = 1;
    // decode: one CTA per (token, 16-row block) with the token's k slots combined in shared memory. Only for
    // short K: each warp then runs f / 256 groups, and the CTA count is T * d / 16 rather than T * k * d / 16
    // (Mixtral, f = 14336, k = 2: 134 vs 95 us; Qwen3-30B, f = 768: 21.1 vs 23.1 us)
    if (policy == MOEB_POLICY_SLOTS && !a.slot_out && a.k <= 8 && a.f <= 2048) {
        const int ks = down_tok_ks();
        a.early_ids = down_early() ? 1 : 0;
        // both carry the 4-warp K split of k_down_slots (2 warps x 2 shares, or 4 x 1): the same bits per slot
        const KLaunch tk = ks == 2 ? KLaunch{fmt == FMT_FP4 ? k_down_tok<FMT_FP4, 2, 2, 6> : k_down_tok<FMT_Q4, 2, 2, 6>,
                                             64 * a.k, down_tok_smem(a.k, a.f, 4), false, 1, 0}
                                   : KLaunch{fmt == FMT_FP4 ? k_down_tok<FMT_FP4, 4, 1, 4> : k_down_tok<FMT_Q4, 4, 1, 4>,
                                             128 * a.k, down_tok_smem(a.k, a.f, 4), false, 1, 0};
        if (tk.smem <= 200 * 1024) {
            if (!allow_smem((const void *)tk.fn, tk.smem)) return check_launch("cudaFuncSetAttribute");
            if (launch(tk.fn, dim3(grid_for(tk, (long)a.T * RBd)), dim3(tk.threads), tk.smem, st, a) != cudaSuccess)
                return check_launch("down");
            if (ev) cudaEventRecord(static_cast<cudaEvent_t>(ev[3]), st);
            return MOEB_OK;
        }
    }
    {
        const long units = max_tiles * ((RBd + K.dn.rows - 1) / K.dn.rows);
        if (launch(K.dn.fn, dim3(grid_for(K.dn, units)), dim3(K.dn.threads), K.dn.smem, st, a) != cudaSuccess)
            return check_launch("down");
    }
    if (sep && launch(k_combine, dim3((unsigned)(((long)a.T * (a.d / 4) + 127) / 128)), dim3(128), 0, st,
                      (const float *)a.yp, a.T, a.d, a.k, a.residual, a.y) != cudaSuccess)
        return check_launch("combine");
    if (ev) cudaEventRecord(static_cast<cudaEvent_t>(ev[3]), st);
    (void)L;
    (void)ws;
    return MOEB_OK;
}

template <int TPB, int U, bool PRE = false>
void (*router_kernel(int E))(RouterArgs) {
    const int J = (E + 31) / 32;
    if (J <= 1) return k_router<TPB, 1, U, PRE>;
    if (J <= 2) return k_router<TPB, 2, U, PRE>;
    if (J <= 4) return k_router<TPB, 4, U, PRE>;
    if (J <= 8) return k_router<TPB, 8, U, PRE>;
    if (J <= 16) return k_router<TPB, 16, U, PRE>;
    return k_router<TPB, 32, U, PRE>;
}

// Slot-mode router calls with E <= 128 and T <= 16 (at most 16 clusters of up to 8 one-per-SM CTAs: one wave) use
// k_router_cl, a cluster per token with the top-k in shared memory (Qwen3-30B T=1 / 2: 18.1 / 30.2 us per layer
// against 18.9 / 31.3). MOEB_ROUTER_CL=0: the last-arriver k_router (measurements).
bool router_cluster() {
    static const int v = [] {
        const char *s = getenv("MOEB_ROUTER_CL");
        return s ? atoi(s) : 1;
    }();
    return v != 0;
}

// One-token router CTAs load their gate rows before the PDL wait when the grid (T * E/4 CTAs) stays within 768 CTAs:
// the held registers cut residency from 6 to 4 CTAs per SM. Qwen3-30B (E = 128), us per layer, with / without:
// T = 1 18.6 / 19.1, 16 82.9 / 84.4, 24 95.3 / 98.3, 32 111.1 / 111.1, 48 119.4 / 118.7, 64 123.0 / 121.9.
// MOEB_ROUTER_PRE_T=n replaces the rule with T <= n (measurements).
bool router_pre(int T, int E) {
    static const int v = [] {
        const char *s = getenv("MOEB_ROUTER_PRE_T");
        return s ? atoi(s) : -1;
    }();
    return v >= 0 ? T <= v : (long)T * ((E + 3) / 4) <= 768;
}

// The register-tiled router needs enough (token block, expert block) CTAs to fill the GPU. Measured (CUDA graph,
// router alone): E = 128, d = 2048, T = 256 / 1024 / 4096: 11.4 / 34.5 / 127 us vs 21.9 / 68.7 / 277 us for the
// one-expert-per-warp kernel, which stays ahead below T * E = 16384 (E = 128, T = 32: 8.5 vs 9.1 us; E = 32,
// T = 256: 9.6 vs 11.5 us) and for few experts up to T = 4096 (E = 8, T = 1024: 11.2 vs 15.2 us).
// MOEB_ROUTER_TILED_T, if set, replaces the rule with "T >= value" (for measurements).
bool router_tiled(int T, int E) {
    static const int v = [] {
        const char *s = getenv("MOEB_ROUTER_TILED_T");
        return s ? atoi(s) : -1;
    }();
    if (v >= 0) return T >= v;
    return E >= 32 ? (long)T * E >= 16384 : T >= 4096;
}

template <int TW, int EW>
void (*router_t_kernel(int E))(RouterArgs) {
    const int J = (E + 31) / 32;
    if (J <= 1) return k_router_t<TW, EW, 1>;
    if (J <= 2) return k_router_t<TW, EW, 2>;
    if (J <= 4) return k_router_t<TW, EW, 4>;
    if (J <= 8) return k_router_t<TW, EW, 8>;
    if (J <= 16) return k_router_t<TW, EW, 16>;
    return k_router_t<TW, EW, 32>;
}

// Tokens per warp of the register-tiled router with 4 experts per warp: 8 from T = MOEB_ROUTER_TW8_T (default
// 512), else 4.
int router_tw(int T) {
    static const int v = [] {
        const char *s = getenv("MOEB_ROUTER_TW8_T");
        return s ? atoi(s) : 512;
    }();
    return T >= v ? 8 : 4;
}

// E, k: routed experts / slots; ns shared experts follow as ids E .. E + ns - 1 (slots per token k + ns).
int launch_router(const void *x, const void *wg, const void *bias, int T, int d, int E, int k, int norm,
                  float scale, int *idx, float *wts, float *logits, bool want_xsum, int policy, const Layout &L,
                  void *ws, cudaStream_t st, int ns = 0) {
    RouterArgs r = {};
    r.ns = ns;
    r.x = static_cast<const uint16_t *>(x);
    r.wg = static_cast<const uint16_t *>(wg);
    r.bias = static_cast<const uint16_t *>(bias);
    r.T = T; r.d = d; r.E = E; r.k = k; r.norm = norm; r.scale = scale;
    r.logits = logits ? logits : at<float>(ws, L.logits);
    r.idx = idx;
    r.wts = wts;
    r.xsum = want_xsum ? at<float>(ws, L.xsum) : nullptr;
    r.cnt = at<unsigned>(ws, L.rcnt);
    r.cnt_all = at<unsigned>(ws, L.cnt_all);
    r.err = at<unsigned>(ws, L.err);
    const bool tiles = is_tiles(policy);
    r.NT = nt_of(policy, (long)T * (k + ns), E + ns);
    r.tiles = tiles ? at<int4>(ws, L.tiles) : nullptr;
    r.ntiles = at<int>(ws, L.ntiles);
    r.sorted = at<int>(ws, L.sorted);
    // the tile builder keeps the slot ids in shared memory for its second pass when that stays small (every
    // router CTA carries this allocation, so it is capped to keep the logits phase at full occupancy)
    const bool tiled = router_tiled(T, E);
    const int tpb = T <= 64 ? 1 : 4;
    const size_t smem = tiles ? tiles_smem(tiled ? 256 : 128, E + ns, (long)T * (k + ns), 16 * 1024) : 0;
    // one expert per warp and 1 (T <= 64) or 4 tokens, or the register-tiled kernel (4 tokens x EW experts per
    // warp, EW = 4 from 32 experts on)
    cudaError_t e;
    if (!tiles && E <= 128 && T <= 16 && router_cluster()) {
        // slot mode: one cluster per token selects its experts in shared memory
        const int rc = (E + 15) / 16, J = (E + 31) / 32;
        void (*kern)(RouterArgs) = J <= 1 ? k_router_cl<1> : J <= 2 ? k_router_cl<2> : k_router_cl<4>;
        e = launch_cluster(kern, dim3(rc, T), dim3(512), 0, st, rc, r);
    } else if (tiled) {
        const int ew = E >= 32 ? 4 : E >= 16 ? 2 : 1, tw = ew == 4 ? router_tw(T) : 4;
        void (*kern)(RouterArgs) = ew == 4 ? (tw == 8 ? router_t_kernel<8, 4>(E) : router_t_kernel<4, 4>(E))
                                 : ew == 2 ? router_t_kernel<4, 2>(E) : router_t_kernel<4, 1>(E);
        e = launch(kern, dim3((E + 8 * ew - 1) / (8 * ew), (T + tw - 1) / tw), dim3(256), smem, st, r);
    } else {
        void (*kern)(RouterArgs) = tpb == 4             ? router_kernel<4, 4>(E)
                                   : router_pre(T, E)    ? router_kernel<1, 8, true>(E)
                                                         : router_kernel<1, 8>(E);
        e = launch(kern, dim3((E + 3) / 4, (T + tpb - 1) / tpb), dim3(128), smem, st, r);
    }
    if (e != cudaSuccess)
        return check_launch("router");
    return MOEB_OK;
}

// ------------------------------------------------------------------ single-kernel decode (decode.cu)
size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Work split and shared-memory layout of one decode launch over G CTAs; false when it does not fit an SM (the
// caller then uses the three-launch decode path).
bool decode_plan(int fmt, int T, int d, int f, int ks, int Er, bool routing, int G, size_t static_smem, DecodePlan *P) {
    const int S = T * ks, RBf = f / 16, RBd = d / 16, Gd = d / 64, Gf = f / 64;
    if (S < 1 || S > 16 || G < 1) return false;
    P->NW = DEC_NW;
    // groups per item: the largest chunk size up to DEC_CG that divides the projection's group count (every item
    // full, one unrolled item body per projection)
    auto chunk = [](int G) {
        for (int c : {8, 6, 5, 4, 3, 2})
            if (c <= DEC_CG && G % c == 0) return c;
        return 1;
    };
    P->CGd = chunk(Gd);
    P->CGf = chunk(Gf);
    P->NCd = Gd / P->CGd;
    P->NCf = Gf / P->CGf;
    const long Ugu = (long)S * RBf, Udn = (long)S * RBd;
    P->max_gu_units = (int)((Ugu + G - 1) / G);
    P->max_dn_units = (int)((Udn + G - 1) / G);
    const long max_items = (long)P->max_gu_units * 2 * P->NCd + (long)P->max_dn_units * P->NCf;
    P->NSL = std::min(S, (std::max(P->max_dn_units, 1) + RBd - 2) / RBd + 1);
    const int sbw = fmt == FMT_FP4 ? 8 : 16;
    const int cg = std::max(P->CGd, P->CGf);
    P->slot_bytes = (int)align_up((size_t)cg * 512 + (size_t)cg * sbw * 4, 128);
    // the partials array also holds the logits [T][Er] while the CTA selects its experts
    const size_t part_bytes = std::max((size_t)max_items * 64, routing ? (size_t)T * ((Er + 15) & ~15) * 4 : 0);
    const size_t fixed = align_up((size_t)T * d * 2, 16) + align_up((size_t)T * Gd * 4, 16) + 2 * align_up((size_t)S * 4, 16) +
                         align_up(part_bytes, 16) +
                         align_up((size_t)(P->max_gu_units + P->max_dn_units) * 4, 16) +
                         align_up((size_t)P->NSL * (f * 2 + f / 16 * 4), 16) + align_up((size_t)P->NSL * 4, 16);
    const size_t cap = 227 * 1024 - static_smem;
    if (fixed + 256 >= cap) return false;
    long nslot = std::min<long>(max_items, (long)((cap - fixed - 256) / (P->slot_bytes + 16)));
    if (nslot < max_items && nslot < 32) return false;
    P->NSLOT = (int)std::max<long>(nslot, 1);
    size_t o = 0;
    P->o_ring = 0;
    o = (size_t)P->NSLOT * P->slot_bytes;
    P->o_bar = (int)o; o = align_up(o + 16 * (size_t)P->NSLOT, 16);
    P->o_x = (int)o; o = align_up(o + (size_t)T * d * 2, 16);
    P->o_xsum = (int)o; o = align_up(o + (size_t)T * Gd * 4, 16);
    P->o_idx = (int)o; o = align_up(o + (size_t)S * 4, 16);
    P->o_wts = (int)o; o = align_up(o + (size_t)S * 4, 16);
    P->o_part = (int)o; o = align_up(o + part_bytes, 16);
    P->o_ucnt = (int)o; o = align_up(o + (size_t)(P->max_gu_units + P->max_dn_units) * 4, 16);
    P->o_h = (int)o; o = align_up(o + (size_t)P->NSL * (f * 2 + f / 16 * 4), 16);
    P->o_hstate = (int)o; o = align_up(o + (size_t)P->NSL * 4, 16);
    P->total = (int)o;
    if ((size_t)P->total > cap) return false;
    P->nR = routing ? std::min(G, (Er + DEC_NW - 1) / DEC_NW) : 0;
    return true;
}

void (*decode_fn(int fmt, int E))(DecodeArgs) {
    (void)E;
    return fmt == FMT_FP4 ? k_decode<FMT_FP4> : k_decode<FMT_Q4>;
}

size_t static_smem_of(const void *fn) {
    static std::mutex mu;
    static std::unordered_map<const void *, size_t> cache;
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(fn);
    if (it != cache.end()) return it->second;
    cudaFuncAttributes fa;
    const size_t v = cudaFuncGetAttributes(&fa, fn) == cudaSuccess ? fa.sharedSizeBytes : 1024;
    cache[fn] = v;
    return v;
}

// Whether the single-kernel decode serves this call (routed experts Er for the router's top-k kernel variant).
bool decode_fits(int fmt, int T, int d, int f, int ks, int Er, bool routing) {
    DecodePlan P;
    auto fn = decode_fn(fmt, routing ? Er : 1);
    return decode_plan(fmt, T, d, f, ks, Er, routing, sm_count(), static_smem_of((const void *)fn), &P);
}

// Decode words in the workspace: the arrival counter sits in the zeroed counter region, the generation word in
// the error region (byte 8; never cleared by moeb_read_error), the records in their own region.
constexpr size_t DEC_ARR_OFF = 16, DEC_GEN_OFF = 8;

int launch_decode(int fmt, const ExpArgs &a, const RouterArgs &r, const Layout &L, void *ws, cudaStream_t st) {
    const bool routing = r.wg != nullptr;
    void (*kern)(DecodeArgs) = decode_fn(fmt, routing ? r.E : 1);
    DecodeArgs A;
    A.a = a;
    A.r = r;
    A.arr = at<unsigned>(ws, L.cnt_all + DEC_ARR_OFF);
    A.gen = at<unsigned>(ws, L.err + DEC_GEN_OFF);
    A.hrec = at<unsigned long long>(ws, L.drec);
    A.yrec = A.hrec + (size_t)a.T * a.k * a.f;
    const int G = sm_count();
    if (!decode_plan(fmt, a.T, a.d, a.f, a.k, routing ? r.E : 0, routing, G, static_smem_of((const void *)kern), &A.p))
        return fail(MOEB_EUNSUP, "decode kernel: this shape does not fit one SM's shared memory%s");
    if (!allow_smem((const void *)kern, (size_t)A.p.total)) return check_launch("decode smem");
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, DEC_THREADS, A.p.total) != cudaSuccess || occ < 1)
        return fail(MOEB_ELAUNCH, "decode kernel does not fit an SM%s");
    // every CTA must be resident at once (they wait on each other's counters): cooperative launch, one per SM
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(DEC_THREADS);
    cfg.dynamicSmemBytes = A.p.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    static std::atomic<int> with_pdl{1};  // cleared if the runtime refuses the pair of attributes
    cfg.numAttrs = with_pdl.load() ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, A);
    if (e != cudaSuccess && cfg.numAttrs == 2) {
        cudaGetLastError();
        with_pdl.store(0);
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, kern, A);
    }
    if (e != cudaSuccess) return check_launch("decode");
    return MOEB_OK;
}

}  // namespace

namespace moeb {
void set_error(const char *msg) { snprintf(g_err, sizeof g_err, "%s", msg); }

// Bytes at the start of a workspace of `ws_bytes` that hold counters and the error word (must read zero before
// a call); 0 if the workspace cannot hold a single token.
size_t zero_region_bytes(size_t ws_bytes, int d, int f, int E, int k) {
    const long cap = capacity(ws_bytes, d, f, E, k);
    return cap < 1 ? 0 : layout(cap, d, f, E, k).zero_end;
}

// The decode records' byte range in a workspace of `ws_bytes` (their tags must not match a later call's tag:
// a caller that resets the counter region before every call clears these too).
void decode_record_span(size_t ws_bytes, int d, int f, int E, int k, size_t *off, size_t *len) {
    const long cap = capacity(ws_bytes, d, f, E, k);
    if (cap < 1) {
        *off = *len = 0;
        return;
    }
    const Layout L = layout(cap, d, f, E, k);
    *off = L.drec;
    *len = L.total - L.drec;
}
}  // namespace moeb

extern "C" {

int moeb_version(void) { return MOEB_VERSION; }

const char *moeb_last_error(void) { return g_err; }

size_t moeb_workspace_bytes(int T, int d, int f, int E, int k) {
    if (T < 1) T = 1;
    return layout(T, d, f, E, k).total;
}

int moeb_workspace_init(void *ws, size_t ws_bytes, cudaStream_t st) {
    if (!ws) return fail(MOEB_EINVAL, "null workspace%s");
    if (cudaMemsetAsync(ws, 0, ws_bytes, st) != cudaSuccess) return check_launch("workspace_init");
    return MOEB_OK;
}

int moeb_read_error(void *ws, unsigned *out, cudaStream_t st) {
    unsigned v = 0;
    if (cudaMemcpyAsync(&v, ws, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return check_launch("read_error");
    if (cudaStreamSynchronize(st) != cudaSuccess) return check_launch("read_error sync");
    if (cudaMemsetAsync(ws, 0, 4, st) != cudaSuccess) return check_launch("read_error clear");
    *out = v;
    return MOEB_OK;
}

int moeb_policy(int T, int E, int k) { return choose_policy(T, E, k, 128, 128); }

// ------------------------------------------------------------------ quantizers
static int check_rows(long rows, long K) {
    if (K <= 0 || K % 64) return fail(MOEB_EINVAL, "K must be a positive multiple of 64%s");
    if (rows < 0 || rows % 16) return fail(MOEB_EINVAL, "rows must be a multiple of 16 (16-row weight blocks)%s");
    return MOEB_OK;
}

int moeb_quantize_q4(const void *w, long rows, long K, void *qw, void *sb, cudaStream_t st) {
    if (int rc = check_rows(rows, K)) return rc;
    const long n = rows * (K / 64);
    if (n == 0) return MOEB_OK;
    k_q4_quantize<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(static_cast<const uint16_t *>(w), rows, K,
                                                             static_cast<uint32_t *>(qw), static_cast<uint32_t *>(sb));
    return check_launch("quantize_q4");
}

int moeb_dequant_q4(const void *qw, const void *sb, long rows, long K, float *out, cudaStream_t st) {
    if (int rc = check_rows(rows, K)) return rc;
    const long n = rows * (K / 8);
    if (n == 0) return MOEB_OK;
    k_q4_dequant<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(static_cast<const uint32_t *>(qw),
                                                            static_cast<const uint32_t *>(sb), rows, K, out);
    return check_launch("dequant_q4");
}

int moeb_q4_from_mlx(const void *wq, const void *scales, const void *biases, long rows, long K, void *qw, void *sb,
                     cudaStream_t st) {
    if (int rc = check_rows(rows, K)) return rc;
    const long n = rows * (K / 8);
    if (n == 0) return MOEB_OK;
    k_q4_from_mlx<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
        static_cast<const uint32_t *>(wq), static_cast<const uint16_t *>(scales), static_cast<const uint16_t *>(biases),
        rows, K, static_cast<uint32_t *>(qw), static_cast<uint32_t *>(sb));
    return check_launch("q4_from_mlx");
}

int moeb_quantize_mxfp4(const void *w, long rows, long K, void *qw, void *sc, cudaStream_t st) {
    if (int rc = check_rows(rows, K)) return rc;
    const long n = rows * (K / 32);
    if (n == 0) return MOEB_OK;
    k_fp4_quantize<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(static_cast<const uint16_t *>(w), rows, K,
                                                              static_cast<uint32_t *>(qw), static_cast<uint8_t *>(sc));
    return check_launch("quantize_mxfp4");
}

int moeb_dequant_mxfp4(const void *qw, const void *sc, long rows, long K, float *out, cudaStream_t st) {
    if (int rc = check_rows(rows, K)) return rc;
    const long n = rows * (K / 8);
    if (n == 0) return MOEB_OK;
    k_fp4_dequant<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(static_cast<const uint32_t *>(qw),
                                                             static_cast<const uint8_t *>(sc), rows, K, out);
    return check_launch("dequant_mxfp4");
}

int moeb_mxfp4_from_mlx(const void *wq, const void *scales, long rows, long K, void *qw, void *sc, cudaStream_t st) {
    if (int rc = check_rows(rows, K)) return rc;
    const long n = rows * (K / 8);
    if (n == 0) return MOEB_OK;
    k_fp4_from_mlx<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(static_cast<const uint32_t *>(wq),
                                                              static_cast<const uint8_t *>(scales), rows, K,
                                                              static_cast<uint32_t *>(qw), static_cast<uint8_t *>(sc));
    return check_launch("mxfp4_from_mlx");
}

// ------------------------------------------------------------------ router
int moeb_router(const void *x, const void *wg, const void *bias, int T, int d, int E, int k, int norm, float scale,
                int *idx, float *wts, float *logits, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (d <= 0 || d % 8) return fail(MOEB_EINVAL, "d must be a positive multiple of 8%s");
    if (E <= 0 || E > 1024 || k <= 0 || k > 32 || k > E) return fail(MOEB_EINVAL, "need 0 < k <= min(E, 32), E <= 1024%s");
    if (T == 0) return MOEB_OK;
    const long cap = capacity(ws_bytes, d, 64, E, k);
    if (cap < T) return fail(MOEB_EINVAL, "workspace too small%s");
    const Layout L = layout(cap, d, 64, E, k);
    return launch_router(x, wg, bias, T, d, E, k, norm, scale, idx, wts, logits, false, MOEB_POLICY_SLOTS, L, ws, st);
}

// ------------------------------------------------------------------ routing tables (the routing step alone)
int moeb_route_tables(const int *idx, int T, int k, int E, int nt, int *counts, int *offsets, int *sorted, int *tiles,
                      int *ntiles, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (T < 0 || k <= 0 || k > 32 || E <= 0 || E > 1024 || nt < 1) return fail(MOEB_EINVAL, "bad T, k, E or nt%s");
    if (!idx || !sorted || !tiles || !ntiles) return fail(MOEB_EINVAL, "idx, sorted, tiles and ntiles are required%s");
    const long cap = capacity(ws_bytes, 64, 64, E, k);
    if (cap < std::max(T, 1)) return fail(MOEB_EINVAL, "workspace too small%s");
    const Layout L = layout(cap, 64, 64, E, k);
    PrepArgs p = {};
    p.idx = idx;
    p.T = T; p.d = 64; p.E = E; p.k = k; p.xs = 64;
    p.cnt_all = at<unsigned>(ws, L.cnt_all);
    p.NT = nt;
    p.tiles = reinterpret_cast<int4 *>(tiles);
    p.ntiles = ntiles;
    p.sorted = sorted;
    p.err = at<unsigned>(ws, L.err);
    p.counts = counts;
    p.offsets = offsets;
    const size_t smem = tiles_smem(256, E, (long)T * k, 48 * 1024);
    if (launch(k_prep, dim3((unsigned)std::max(1, (T + 7) / 8)), dim3(256), smem, st, p) != cudaSuccess)
        return check_launch("route_tables");
    return MOEB_OK;
}

// ------------------------------------------------------------------ experts (ids given) and full layer
struct P2PParams {
    const unsigned *rflag;
    const int *rcnt;
    const unsigned *epoch;
    const unsigned long long *wait_ns;
    int C, me;  // C: this call's rows per source block
    unsigned char *const *peers;
    size_t yoff;
};

static int experts_common(int fmt, const void *x, const void *qg, const void *sbg, const void *qu, const void *sbu,
                          const void *qd, const void *sbd, const float *bg, const float *bu, const float *bd,
                          const int *idx, const float *wts, int T, int d, int f, int E, int k, int act, int policy,
                          const void *residual, void *y, void *ws, size_t ws_bytes, cudaStream_t st,
                          const void *gate_w, const void *gate_b, int norm, float rscale, int *idx_out,
                          float *wts_out, void *const *ev, float *yp_out = nullptr, int ns = 0,
                          const P2PParams *pp = nullptr) {
    // yp_out != null or pp != null: expert-parallel rows (k = 1, each x row of d + 8 values ends in its
    // {expert, weight} tail); down writes the weighted fp32 slot outputs to yp_out (or straight into the owners'
    // return blocks, pp) and nothing is combined here.
    const bool ep = yp_out != nullptr || pp != nullptr;
    int rc = check_shape(T, d, f, E, k);
    if (rc) return rc;
    if (act < 0 || act > 2) return fail(MOEB_EINVAL, "act must be 0, 1 or 2%s");
    if (T == 0) return MOEB_OK;
    const long cap = capacity(ws_bytes, d, f, E, k, !ep);
    if (cap < T) return fail(MOEB_EINVAL, "workspace too small for T tokens%s");
    const Layout L = layout(cap, d, f, E, k, !ep);
    const int xs = ep ? d + 8 : d;
    if (policy == MOEB_POLICY_AUTO) policy = choose_policy(T, E, k, d, f);
    // the single-kernel decode: layer and expert calls of <= 16 slots whose plan fits an SM
    if (policy == MOEB_POLICY_DECODE &&
        (ep || (long)T * k > 16 || !decode_fits(fmt, T, d, f, k, gate_w ? E - ns : 0, gate_w != nullptr)))
        policy = MOEB_POLICY_SLOTS;
    if (policy != MOEB_POLICY_SLOTS && policy != MOEB_POLICY_DECODE && !is_tiles(policy))
        return fail(MOEB_EINVAL, "unknown policy%s");
    if (policy == MOEB_POLICY_TC && (d % 128 || f % 128))
        return fail(MOEB_EINVAL, "the tensor-core policy needs d, f multiples of 128%s");
    const bool fused = policy == MOEB_POLICY_DECODE;
    const bool tiles = policy != MOEB_POLICY_SLOTS && !fused;
    if (ev) cudaEventRecord(static_cast<cudaEvent_t>(ev[0]), st);
    if (fused) {  // the single decode kernel routes (or checks the given ids) itself
        if (gate_w) {
            idx = idx_out ? idx_out : at<int>(ws, L.idx);
            wts = wts_out ? wts_out : at<float>(ws, L.wts);
        }
    } else if (gate_w) {  // layer call: router produces ids, weights, x group sums and (tile mode) the tiles
        int *ri = idx_out ? idx_out : at<int>(ws, L.idx);
        float *rw = wts_out ? wts_out : at<float>(ws, L.wts);
        // E, k count the ns shared experts / slots; the router picks among the E - ns routed experts
        rc = launch_router(x, gate_w, gate_b, T, d, E - ns, k - ns, norm, rscale, ri, rw, nullptr, true, policy, L,
                           ws, st, ns);
        if (rc) return rc;
        idx = ri;
        wts = rw;
    } else {
        PrepArgs p = {};
        p.x = static_cast<const uint16_t *>(x);
        p.idx = idx;
        p.T = T; p.d = d; p.E = E; p.k = k;
        p.xs = xs;
        if (ep) {
            idx = p.idx = p.idx_w = at<int>(ws, L.idx);
            wts = p.wts_w = at<float>(ws, L.wts);
        }
        if (pp) {
            p.rflag = pp->rflag;
            p.rcnt = pp->rcnt;
            p.epoch = pp->epoch;
            p.wait_ns = pp->wait_ns;
            p.C = pp->C;
        }
        p.xsum = at<float>(ws, L.xsum);
        p.cnt_all = at<unsigned>(ws, L.cnt_all);
        p.NT = nt_of(policy, pp ? (long)pp->C : (long)T * k, E);  // as run_experts picks it
        p.tiles = tiles ? at<int4>(ws, L.tiles) : nullptr;
        p.ntiles = at<int>(ws, L.ntiles);
        p.sorted = at<int>(ws, L.sorted);
        p.err = at<unsigned>(ws, L.err);
        const size_t smem = tiles ? tiles_smem(256, E, (long)T * k, 48 * 1024) : 0;  // ids cached when they fit
        if (launch(k_prep, dim3((T + 7) / 8), dim3(256), smem, st, p) != cudaSuccess) return check_launch("prep");
    }
    if (ev) cudaEventRecord(static_cast<cudaEvent_t>(ev[1]), st);
    ExpArgs a = {};
    a.x = static_cast<const uint16_t *>(x);
    a.xs = xs;
    a.xsum = at<float>(ws, L.xsum);
    a.g = {static_cast<const uint32_t *>(qg), static_cast<const uint32_t *>(sbg)};
    a.u = {static_cast<const uint32_t *>(qu), static_cast<const uint32_t *>(sbu)};
    a.dn = {static_cast<const uint32_t *>(qd), static_cast<const uint32_t *>(sbd)};
    a.bg = bg; a.bu = bu; a.bd = bd;
    if ((bg == nullptr) != (bu == nullptr)) return fail(MOEB_EINVAL, "gate and up biases go together%s");
    a.idx = idx;
    a.wts = wts;
    a.tiles = at<int4>(ws, L.tiles);
    a.ntiles = at<int>(ws, L.ntiles);
    a.sorted = at<int>(ws, L.sorted);
    a.h = at<uint16_t>(ws, L.h);
    a.hsum = at<float>(ws, L.hsum);
    a.yp = yp_out ? yp_out : at<float>(ws, L.yp);
    a.slot_out = ep ? 1 : 0;
    if (pp) {
        a.ypeers = pp->peers;
        a.yoff = pp->yoff;
        a.C = pp->C;
        a.me = pp->me;
    }
    a.ycnt = at<unsigned>(ws, L.ycnt);
    a.residual = static_cast<const uint16_t *>(residual);
    a.y = static_cast<uint16_t *>(y);
    a.err = at<unsigned>(ws, L.err);
    a.T = T; a.d = d; a.f = f; a.E = E; a.k = k; a.act = act; a.tile_mode = tiles ? 1 : 0;
    a.fmt = fmt;
    // the down weights of the routed experts are prefetched into L2 while gate/up runs only when gate/up,
    // down and the prefetch all fit comfortably in L2 (otherwise the gate/up stream evicts them again)
    {
        const double U = std::min<double>(E, (double)T * k);
        const double layer_bytes = U * 3.0 * d * f * (fmt == FMT_FP4 ? 4.25 : 4.5) / 8.0;
        a.dn_prefetch = layer_bytes < 48.0 * (1 << 20) ? 1 : 0;
    }
    if (fused) {
        RouterArgs r = {};
        if (gate_w) {
            r.x = static_cast<const uint16_t *>(x);
            r.wg = static_cast<const uint16_t *>(gate_w);
            r.bias = static_cast<const uint16_t *>(gate_b);
            r.T = T; r.d = d; r.E = E - ns; r.k = k - ns; r.norm = norm; r.ns = ns; r.scale = rscale;
            r.logits = at<float>(ws, L.logits);
            r.idx = const_cast<int *>(idx);
            r.wts = const_cast<float *>(wts);
            r.xsum = at<float>(ws, L.xsum);
            r.err = at<unsigned>(ws, L.err);
        }
        rc = launch_decode(fmt, a, r, L, ws, st);
        if (ev)
            for (int i = 1; i < 4; ++i) cudaEventRecord(static_cast<cudaEvent_t>(ev[i]), st);
        return rc;
    }
    return run_experts(fmt, a, policy, L, ws, st, ev);
}

int moeb_experts_q4(const void *x, const void *qg, const void *sbg, const void *qu, const void *sbu, const void *qd,
                    const void *sbd, const float *bg, const float *bu, const float *bd, const int *idx,
                    const float *wts, int T, int d, int f, int E, int k, int act, int policy, const void *residual,
                    void *y, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (!idx || !wts) return fail(MOEB_EINVAL, "idx and wts are required%s");
    return experts_common(FMT_Q4, x, qg, sbg, qu, sbu, qd, sbd, bg, bu, bd, idx, wts, T, d, f, E, k, act, policy,
                          residual, y, ws, ws_bytes, st, nullptr, nullptr, 0, 1.f, nullptr, nullptr, nullptr);
}

int moeb_experts_mxfp4(const void *x, const void *qg, const void *scg, const void *qu, const void *scu,
                       const void *qd, const void *scd, const float *bg, const float *bu, const float *bd,
                       const int *idx, const float *wts, int T, int d, int f, int E, int k, int act, int policy,
                       const void *residual, void *y, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (!idx || !wts) return fail(MOEB_EINVAL, "idx and wts are required%s");
    return experts_common(FMT_FP4, x, qg, scg, qu, scu, qd, scd, bg, bu, bd, idx, wts, T, d, f, E, k, act, policy,
                          residual, y, ws, ws_bytes, st, nullptr, nullptr, 0, 1.f, nullptr, nullptr, nullptr);
}

int moeb_layer_mxfp4(const void *x, const void *gate_w, const void *gate_b, int norm, float rscale, const void *qg,
                     const void *scg, const void *qu, const void *scu, const void *qd, const void *scd,
                     const float *bg, const float *bu, const float *bd, int T, int d, int f, int E, int k, int act,
                     int policy, const void *residual, void *y, int *idx_out, float *wts_out,
                     void *const *stage_events, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (!gate_w) return fail(MOEB_EINVAL, "gate weights are required%s");
    return experts_common(FMT_FP4, x, qg, scg, qu, scu, qd, scd, bg, bu, bd, nullptr, nullptr, T, d, f, E, k, act,
                          policy, residual, y, ws, ws_bytes, st, gate_w, gate_b, norm, rscale, idx_out, wts_out,
                          stage_events);
}

int moeb_layer_q4_shared(const void *x, const void *gate_w, const void *gate_b, int norm, float rscale, int n_shared,
                         const void *qg, const void *sbg, const void *qu, const void *sbu, const void *qd,
                         const void *sbd, const float *bg, const float *bu, const float *bd, int T, int d, int f, int E,
                         int k, int act, int policy, const void *residual, void *y, int *idx_out, float *wts_out,
                         void *const *stage_events, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (!gate_w) return fail(MOEB_EINVAL, "gate weights are required%s");
    if (n_shared < 0 || k <= 0 || k + n_shared > 32 || k > E)
        return fail(MOEB_EINVAL, "need n_shared >= 0, 0 < k <= E and k + n_shared <= 32%s");
    return experts_common(FMT_Q4, x, qg, sbg, qu, sbu, qd, sbd, bg, bu, bd, nullptr, nullptr, T, d, f, E + n_shared,
                          k + n_shared, act, policy, residual, y, ws, ws_bytes, st, gate_w, gate_b, norm, rscale,
                          idx_out, wts_out, stage_events, nullptr, n_shared);
}

int moeb_layer_q4(const void *x, const void *gate_w, const void *gate_b, int norm, float rscale, const void *qg,
                  const void *sbg, const void *qu, const void *sbu, const void *qd, const void *sbd, const float *bg,
                  const float *bu, const float *bd, int T, int d, int f, int E, int k, int act, int policy,
                  const void *residual, void *y, int *idx_out, float *wts_out, void *const *stage_events, void *ws,
                  size_t ws_bytes, cudaStream_t st) {
    if (!gate_w) return fail(MOEB_EINVAL, "gate weights are required%s");
    return experts_common(FMT_Q4, x, qg, sbg, qu, sbu, qd, sbd, bg, bu, bd, nullptr, nullptr, T, d, f, E, k, act,
                          policy, residual, y, ws, ws_bytes, st, gate_w, gate_b, norm, rscale, idx_out, wts_out,
                          stage_events);
}

// ------------------------------------------------------------------ expert parallelism
static int check_ep(int T, int d, int k, int E, int P) {
    if (T < 0 || d <= 0 || d % 64 || k <= 0 || k > 32 || k > E) return fail(MOEB_EINVAL, "bad T, d or k%s");
    if (P < 1 || P > 32 || E % P) return fail(MOEB_EINVAL, "need 1 <= P <= 32 ranks and E a multiple of P%s");
    return MOEB_OK;
}

int moeb_ep_dispatch(const void *x, const int *idx, const float *wts, int T, int d, int k, int E, int P,
                     void *send_rows, int *send_counts, int *slot_pos, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (int rc = check_ep(T, d, k, E, P)) return rc;
    if (!ws || ws_bytes < 256) return fail(MOEB_EINVAL, "workspace required (its error word is used)%s");
    if (T == 0) {
        if (cudaMemsetAsync(send_counts, 0, sizeof(int) * P, st) != cudaSuccess) return check_launch("ep_dispatch");
        return MOEB_OK;
    }
    EPArgs a = {};
    a.x = static_cast<const uint16_t *>(x);
    a.idx = idx;
    a.wts = wts;
    a.T = T; a.d = d; a.k = k; a.E = E; a.P = P;
    a.send_counts = send_counts;
    a.slot_pos = slot_pos;
    a.rows = static_cast<uint16_t *>(send_rows);
    a.err = static_cast<unsigned *>(ws);
    if (launch(k_ep_plan, dim3(1), dim3(1024), 0, st, a) != cudaSuccess) return check_launch("ep_plan");
    if (launch(k_ep_pack, dim3((unsigned)(((long)T * k + 7) / 8)), dim3(256), 0, st, a) != cudaSuccess)
        return check_launch("ep_pack");
    return MOEB_OK;
}

size_t moeb_ep_workspace_bytes(int R, int d, int f, int E_local) {
    if (R < 1) R = 1;
    return layout(R, d, f, E_local, 1, false).total;
}

int moeb_ep_experts_q4(const void *rows, int R, int d, int f, int E_local, const void *qg, const void *sbg,
                       const void *qu, const void *sbu, const void *qd, const void *sbd, const float *bg,
                       const float *bu, const float *bd, int act, int policy, float *yp, void *ws, size_t ws_bytes,
                       cudaStream_t st) {
    if (!yp) return fail(MOEB_EINVAL, "yp is required%s");
    return experts_common(FMT_Q4, rows, qg, sbg, qu, sbu, qd, sbd, bg, bu, bd, nullptr, nullptr, R, d, f, E_local,
                          1, act, policy, nullptr, nullptr, ws, ws_bytes, st, nullptr, nullptr, 0, 1.f, nullptr,
                          nullptr, nullptr, yp);
}

int moeb_ep_experts_mxfp4(const void *rows, int R, int d, int f, int E_local, const void *qg, const void *scg,
                          const void *qu, const void *scu, const void *qd, const void *scd, const float *bg,
                          const float *bu, const float *bd, int act, int policy, float *yp, void *ws,
                          size_t ws_bytes, cudaStream_t st) {
    if (!yp) return fail(MOEB_EINVAL, "yp is required%s");
    return experts_common(FMT_FP4, rows, qg, scg, qu, scu, qd, scd, bg, bu, bd, nullptr, nullptr, R, d, f, E_local,
                          1, act, policy, nullptr, nullptr, ws, ws_bytes, st, nullptr, nullptr, 0, 1.f, nullptr,
                          nullptr, nullptr, yp);
}

// ---- peer-memory exchange (CUDA IPC mappings of plain device allocations; no multicast objects)
size_t moeb_ep_p2p_bytes(int P, int C, int d) { return p2p_layout(P, C, d).total; }

int moeb_ep_ipc_alloc(size_t bytes, void **ptr) {
    if (!ptr || bytes == 0) return fail(MOEB_EINVAL, "bad allocation request%s");
    if (cudaMalloc(ptr, bytes) != cudaSuccess) return check_launch("ipc_alloc");
    if (cudaMemset(*ptr, 0, bytes) != cudaSuccess) return check_launch("ipc_alloc memset");
    if (cudaDeviceSynchronize() != cudaSuccess) return check_launch("ipc_alloc sync");
    return MOEB_OK;
}
int moeb_ep_ipc_free(void *ptr) {
    if (ptr && cudaFree(ptr) != cudaSuccess) return check_launch("ipc_free");
    return MOEB_OK;
}
int moeb_ep_ipc_handle(void *ptr, void *handle) {
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return check_launch("ipc_handle");
    memcpy(handle, &h, sizeof h);
    return MOEB_OK;
}
int moeb_ep_ipc_open(const void *handle, void **ptr) {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return check_launch("ipc_open");
    return MOEB_OK;
}
int moeb_ep_ipc_close(void *ptr) {
    if (ptr && cudaIpcCloseMemHandle(ptr) != cudaSuccess) return check_launch("ipc_close");
    return MOEB_OK;
}

int moeb_ep_p2p_dispatch(const void *x, const int *idx, const float *wts, int T, int d, int k, int E, int P, int me,
                         int C, int Cs, void *const *peers, void *self, int *send_counts, int *slot_pos,
                         cudaStream_t st) {
    if (int rc = check_ep(T, d, k, E, P)) return rc;
    if (me < 0 || me >= P || !peers || !self) return fail(MOEB_EINVAL, "bad rank or exchange buffers%s");
    if (Cs <= 0) Cs = C;
    if (Cs > C) return fail(MOEB_EINVAL, "Cs exceeds the exchange capacity C%s");
    if ((long)T * k > Cs) return fail(MOEB_EINVAL, "T*k exceeds the call's rows per source Cs%s");
    EPArgs a = {};
    a.x = static_cast<const uint16_t *>(x);
    a.idx = idx;
    a.wts = wts;
    a.T = T; a.d = d; a.k = k; a.E = E; a.P = P;
    a.send_counts = send_counts;
    a.slot_pos = slot_pos;
    a.err = reinterpret_cast<unsigned *>(static_cast<unsigned char *>(self) + p2p_layout(P, C, d).err);
    a.C = C;
    a.Cs = Cs;
    a.me = me;
    a.peers = reinterpret_cast<unsigned char *const *>(peers);
    a.self = static_cast<unsigned char *>(self);
    if (launch(k_ep_plan, dim3(1), dim3(1024), 0, st, a) != cudaSuccess) return check_launch("ep_plan");
    // the sending kernel runs even for T = 0: it still publishes the (zero) counts and the epoch flags
    if (launch(k_ep_send, dim3((unsigned)std::max<long>(1, ((long)T * k + 7) / 8)), dim3(256), 0, st, a) != cudaSuccess)
        return check_launch("ep_send");
    return MOEB_OK;
}

static int p2p_experts(int fmt, void *const *peers, void *self, int P, int me, int C, int Cs, int d, int f,
                       int E_local, const void *qg, const void *sg, const void *qu, const void *su, const void *qd,
                       const void *sd, const float *bg, const float *bu, const float *bd, int act, int policy,
                       void *ws, size_t ws_bytes, cudaStream_t st) {
    if (Cs <= 0) Cs = C;
    if (P < 1 || P > 32 || me < 0 || me >= P || C < 1 || Cs > C || !peers || !self)
        return fail(MOEB_EINVAL, "bad exchange parameters%s");
    const P2PLayout L = p2p_layout(P, C, d);
    unsigned char *b = static_cast<unsigned char *>(self);
    P2PParams pp;
    pp.rflag = reinterpret_cast<const unsigned *>(b + L.rflag);
    pp.rcnt = reinterpret_cast<const int *>(b + L.rcnt);
    pp.epoch = reinterpret_cast<const unsigned *>(b + L.epoch);
    pp.wait_ns = reinterpret_cast<const unsigned long long *>(b + L.wait);
    pp.C = Cs;
    pp.me = me;
    pp.peers = reinterpret_cast<unsigned char *const *>(peers);
    pp.yoff = L.back;
    // kernels that skip padding rows and fence their peer stores: the decode kernels for small calls (each
    // padding unit exits at once), the warp-specialized tiles otherwise. With every rank sending about Cs slots
    // spread over the P owners, an owner receives about Cs rows: the load is Cs / E_local rows per expert.
    if (policy == MOEB_POLICY_AUTO)
        policy = (Cs <= 16 && (long)P * Cs <= 128) ? MOEB_POLICY_SLOTS
                 : ((long)Cs >= 14L * E_local && d % 128 == 0 && f % 128 == 0)
                     ? MOEB_POLICY_TC  // weights dequantized once per tile (the single-GPU dispatcher's rule)
                     : (long)Cs >= 16L * E_local ? MOEB_POLICY_TILES24_RING
                     : ((long)Cs >= 8L * E_local ? MOEB_POLICY_TILES16_RING : MOEB_POLICY_TILES8_RING);
    else if (policy != MOEB_POLICY_SLOTS && policy != MOEB_POLICY_TILES8_RING && policy != MOEB_POLICY_TILES16_RING &&
             policy != MOEB_POLICY_TILES24_RING &&
             policy != MOEB_POLICY_TC)
        policy = MOEB_POLICY_TILES8_RING;  // (TC on request: its down epilogue stores into the owners' blocks)
    int rc = experts_common(fmt, b + L.rows, qg, sg, qu, su, qd, sd, bg, bu, bd, nullptr, nullptr, P * Cs, d, f,
                            E_local, 1, act, policy, nullptr, nullptr, ws, ws_bytes, st, nullptr, nullptr, 0, 1.f,
                            nullptr, nullptr, nullptr, nullptr, 0, &pp);
    if (rc) return rc;
    if (launch(k_ep_signal, dim3(1), dim3(32), 0, st, reinterpret_cast<unsigned char *const *>(peers), b, P, C, d, me) !=
        cudaSuccess)
        return check_launch("ep_signal");
    return MOEB_OK;
}

int moeb_ep_p2p_experts_q4(void *const *peers, void *self, int P, int me, int C, int Cs, int d, int f, int E_local,
                           const void *qg, const void *sbg, const void *qu, const void *sbu, const void *qd,
                           const void *sbd, const float *bg, const float *bu, const float *bd, int act, int policy,
                           void *ws, size_t ws_bytes, cudaStream_t st) {
    return p2p_experts(FMT_Q4, peers, self, P, me, C, Cs, d, f, E_local, qg, sbg, qu, sbu, qd, sbd, bg, bu, bd, act,
                       policy, ws, ws_bytes, st);
}

int moeb_ep_p2p_combine(void *self, const int *slot_pos, int P, int C, int T, int d, int k, const void *residual,
                        void *y, cudaStream_t st) {
    if (T < 0 || d <= 0 || d % 64 || k <= 0 || k > 32 || P < 1 || P > 32) return fail(MOEB_EINVAL, "bad shape%s");
    if (T == 0) return MOEB_OK;
    unsigned char *b = static_cast<unsigned char *>(self);
    if (launch(k_ep_combine_p2p, dim3((unsigned)(((long)T * (d / 4) + 127) / 128)), dim3(128), 0, st,
               (const unsigned char *)b, slot_pos, P, C, T, d, k, static_cast<const uint16_t *>(residual),
               static_cast<uint16_t *>(y), reinterpret_cast<unsigned *>(b + p2p_layout(P, C, d).err)) != cudaSuccess)
        return check_launch("ep_combine_p2p");
    return MOEB_OK;
}

int moeb_ep_p2p_set_wait_limit(void *self, int P, int C, int d, double seconds, cudaStream_t st) {
    if (!self || !(seconds >= 0.0) || seconds > 3600.0) return fail(MOEB_EINVAL, "need 0 <= seconds <= 3600%s");
    const unsigned long long v = (unsigned long long)(seconds * 1e9);
    unsigned char *b = static_cast<unsigned char *>(self) + p2p_layout(P, C, d).wait;
    if (cudaMemcpyAsync(b, &v, sizeof v, cudaMemcpyHostToDevice, st) != cudaSuccess) return check_launch("set_wait");
    if (cudaStreamSynchronize(st) != cudaSuccess) return check_launch("set_wait sync");
    return MOEB_OK;
}

int moeb_ep_p2p_read_error(void *self, int P, int C, int d, unsigned *out, cudaStream_t st) {
    unsigned char *b = static_cast<unsigned char *>(self) + p2p_layout(P, C, d).err;
    return moeb_read_error(b, out, st);
}

int moeb_ep_combine(const float *back, const int *slot_pos, int T, int d, int k, const void *residual, void *y,
                    cudaStream_t st) {
    if (T < 0 || d <= 0 || d % 64 || k <= 0 || k > 32) return fail(MOEB_EINVAL, "bad T, d or k%s");
    if (T == 0) return MOEB_OK;
    if (launch(k_ep_combine, dim3(T), dim3(256), 0, st, back, slot_pos, T, d, k,
               static_cast<const uint16_t *>(residual), static_cast<uint16_t *>(y)) != cudaSuccess)
        return check_launch("ep_combine");
    return MOEB_OK;
}

}  // extern "C"
