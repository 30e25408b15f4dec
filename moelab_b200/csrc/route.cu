// Router and routing kernels.
//
// k_router: the fused router of the layer call (moelab/e2e.py:51-65 composes gate -> top-k -> experts; the
// reference's fused tail is moelab/router.py:15-80). One launch does
//   1. logits[t][e] = x[t] . Wg[e] (+ bias[e]) in fp32, summation order fixed (lane l of a warp takes the
//      8-element chunks l, l+32, ... with fmaf, then a xor butterfly) so the CPU oracle reproduces the
//      logits - and hence the expert ids - bit for bit;
//   2. in the last CTA of each token block (last-arriver counter, no spin): top-k with router.py's rules
//      (NaN = -inf, ties to the lowest id, fewer than k finite -> lowest unused ids with weight 0), softmax
//      over the top-k (norm) or full-softmax probabilities (!norm), times the routed scaling factor; plus the
//      per-64-group sums of x used by the expert kernels' scale/bias promotion;
//   3. in the last of those (tile mode only): the routing step - per-expert histogram, prefix sum and the
//      slot permutation grouped by expert, cut into tiles of <= NT slots (replaces the O(TK^2) map kernels
//      metal_q4_tiles_v2.py:362-373 / metal_mxfp4_moe.py:143-153).
// k_prep: the same steps 2b-3 for the harness contract run(state, x, idx, wts), where ids come from outside.
#include <cooperative_groups.h>

#include "route_common.cuh"

namespace moeb {

// ------------------------------------------------------------------ tile builder (one CTA)
// Exclusive scan over the CTA (blockDim.x <= 1024): warp shuffles, then one warp over the warp totals.
__device__ __forceinline__ int block_exclusive_scan(int v, int *total) {
    __shared__ int wsum[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += n;
    }
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nw ? wsum[lane] : 0;
        int winc = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, winc, o);
            if (lane >= o) winc += n;
        }
        if (lane < nw) wsum[lane] = winc - w;
        if (lane == 31) wsum[31] = winc;  // nw <= 32; lane 31 holds the grand total
    }
    __syncthreads();
    const int r = wsum[warp] + inc - v;
    *total = wsum[31];
    __syncthreads();
    return r;
}

// Stable counting sort of the TK slots by expert (the routing step), one CTA. The slots are cut into one
// contiguous segment per warp; each warp walks its segment in slot order, 32 at a time, grouping equal ids with a
// warp match. A slot's place inside its expert is (slots of that expert in earlier segments) + (earlier slots of
// that expert in this segment), so the slots of one expert keep increasing slot order and every array written here
// is a deterministic function of the ids. Tiles are cut from each expert's run, NT slots at a time: the grouping
// contract of the reference's map kernel (metal_q4_tiles_v2.py:362-373, a tile holds up to VT consecutive
// same-expert slots in slot order), listed here in expert order.
// Dynamic shared memory: hist [warps][E] and tot [E] ints, then (when it fits) the TK ids.
// Ids equal to SLOT_SKIP (capacity padding) are skipped; other ids outside [0, E) set ERR_EXPERT_ID and are
// grouped under expert 0 (the expert kernels compute them there with weight 0).
// counts / offsets (may be null): per-expert slot counts and their exclusive prefix sums (offsets into sorted).
__device__ void build_tiles(const int *__restrict__ idx, int TK, int E, int NT, int4 *__restrict__ tiles,
                            int *__restrict__ ntiles, int *__restrict__ sorted, unsigned *__restrict__ err,
                            int *__restrict__ counts, int *__restrict__ offsets) {
    constexpr int BT = 8;  // ids loaded per lane per batch (independent loads in flight)
    extern __shared__ int smem[];
    const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nth >> 5;
    int *hist = smem;                  // [nw][E]: counts, then each warp's first position per expert
    int *tot = smem + nw * E;          // [E]
    int *ids = smem + (nw + 1) * E;    // [TK] when it fits
    unsigned dsm;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dsm));
    const bool cache = (size_t)((nw + 1) * E + TK) * 4 <= dsm;
    const int seg = (TK + nw - 1) / nw;
    const int s_beg = min(TK, warp * seg), s_end = min(TK, s_beg + seg);
    const unsigned lt = (1u << lane) - 1u;
    for (int i = tid; i < nw * E; i += nth) hist[i] = 0;
    __syncthreads();
    // pass 1: per-warp histograms of the warp's segment (only warp w writes row w: no atomics)
    bool bad = false;
    for (int b0 = s_beg; b0 < s_end; b0 += 32 * BT) {
        int ev[BT];
#pragma unroll
        for (int i = 0; i < BT; ++i) {
            const int s = b0 + 32 * i + lane;
            ev[i] = s < s_end ? __ldcg(idx + s) : SLOT_SKIP;
        }
#pragma unroll
        for (int i = 0; i < BT; ++i) {
            const int s = b0 + 32 * i + lane;
            int e = ev[i];
            if (cache && s < s_end) ids[s] = e;
            if (e != SLOT_SKIP && (e < 0 || e >= E)) { bad = true; e = 0; }
            const unsigned peers = __match_any_sync(0xffffffffu, e);
            if (e != SLOT_SKIP && (peers & lt) == 0u) hist[warp * E + e] += __popc(peers);
            __syncwarp();
        }
    }
    if (bad) atomicOr(err, ERR_EXPERT_ID);
    __syncthreads();
    // per expert: total and per-warp exclusive prefix; each thread owns a contiguous chunk of experts, two CTA-wide
    // scans give the slot and tile offsets
    const int per = (E + nth - 1) / nth;
    const int e0 = min(E, tid * per), e1 = min(E, e0 + per);
    int sc = 0, st = 0;
    for (int e = e0; e < e1; ++e) {
        int c = 0;
        for (int w = 0; w < nw; ++w) {
            const int h = hist[w * E + e];
            hist[w * E + e] = c;
            c += h;
        }
        tot[e] = c;
        sc += c;
        st += (c + NT - 1) / NT;
    }
    int tot_s, tot_t;
    int base_s = block_exclusive_scan(sc, &tot_s);
    int base_t = block_exclusive_scan(st, &tot_t);
    if (tid == 0) *ntiles = tot_t;
    for (int e = e0; e < e1; ++e) {
        const int c = tot[e];
        for (int w = 0; w < nw; ++w) hist[w * E + e] += base_s;
        if (counts) counts[e] = c;
        if (offsets) offsets[e] = base_s;
        const int nt = (c + NT - 1) / NT;
        for (int i = 0; i < nt; ++i) tiles[base_t + i] = make_int4(e, base_s + i * NT, min(NT, c - i * NT), 0);
        base_s += c;
        base_t += nt;
    }
    __syncthreads();
    // pass 2: scatter, the same walk (a slot's position = its warp's running position + its rank among the
    // earlier lanes with the same id)
    for (int b0 = s_beg; b0 < s_end; b0 += 32 * BT) {
        int ev[BT];
#pragma unroll
        for (int i = 0; i < BT; ++i) {
            const int s = b0 + 32 * i + lane;
            ev[i] = s >= s_end ? SLOT_SKIP : cache ? ids[s] : __ldcg(idx + s);
        }
#pragma unroll
        for (int i = 0; i < BT; ++i) {
            const int s = b0 + 32 * i + lane;
            int e = ev[i];
            if (e != SLOT_SKIP && (e < 0 || e >= E)) e = 0;
            const unsigned peers = __match_any_sync(0xffffffffu, e);
            if (e != SLOT_SKIP) {
                const int pos = hist[warp * E + e] + __popc(peers & lt);
                sorted[pos] = s;
            }
            __syncwarp();
            if (e != SLOT_SKIP && (peers & lt) == 0u) hist[warp * E + e] += __popc(peers);
            __syncwarp();
        }
    }
}

// Dynamic shared memory the tile builder uses in a CTA of `threads` threads: per-warp histograms and totals,
// plus the ids when that stays under `cap` bytes.
size_t tiles_smem(int threads, int E, long TK, size_t cap) {
    const size_t base = 4 * (size_t)(threads / 32 + 1) * E;
    return base + 4 * (size_t)TK <= cap ? base + 4 * (size_t)TK : base;
}

// After a router CTA has written its logits: the last CTA of each token block (last-arriver counter, no spin)
// runs top-k for the block's tokens; in tile mode the last token block to finish builds the tiles.
template <int JMAX>
__device__ __forceinline__ void router_tail(const RouterArgs &a, int t0, int nt, int warp, int lane) {
    // the barrier orders the CTA's logits before thread 0's fence (cumulative), the counter picks the last CTA
    // of the token block, whose thread 0 fences again before the reads
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) s_last = atom_add_acq_rel_gpu(a.cnt + blockIdx.y, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    const int nw = blockDim.x >> 5;
    for (int i = warp; i < nt; i += nw) topk_token<JMAX>(a, t0 + i, lane);
    if (threadIdx.x == 0) a.cnt[blockIdx.y] = 0;
    if (a.tiles == nullptr) return;
    // routing step in the last token block to finish
    __syncthreads();
    if (threadIdx.x == 0) s_last = atom_add_acq_rel_gpu(a.cnt_all, 1u) == gridDim.y - 1;
    __syncthreads();
    if (!s_last) return;
    build_tiles(a.idx, a.T * (a.k + a.ns), a.E + a.ns, a.NT, a.tiles, a.ntiles, a.sorted, a.err, nullptr, nullptr);
    if (threadIdx.x == 0) *a.cnt_all = 0;
}

// grid (ceil(E / 4), ceil(T / TPB)), block 128: warp w computes expert blockIdx.x * 4 + w for TPB tokens.
// Each lane loads U chunks of the gate row and of every token row at once, then runs the fmaf chains; warp 0 of
// the first expert block also turns its x registers into the per-64-group sums.
template <int TPB, int JMAX, int U, bool PRE>
__global__ void __launch_bounds__(128) k_router(RouterArgs a) {
    pdl_launch();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e = blockIdx.x * 4 + warp;
    const int nch = a.d / 8;
    const uint16_t *wr = a.wg + (size_t)min(e, a.E - 1) * a.d;
    // PRE: the gate is a weight (written before any call), so the first chunks of its row are loaded before waiting
    // for the kernel that produced x (decode-sized calls, whose router latency is on the critical path; the held
    // registers cost occupancy, so larger calls do not)
    uint4 w0[U];
    if (PRE)
#pragma unroll
        for (int u = 0; u < U; ++u) w0[u] = *reinterpret_cast<const uint4 *>(wr + 8 * min(lane + 32 * u, nch - 1));
    pdl_wait();
    const int t0 = blockIdx.y * TPB;
    const int nt = min(TPB, a.T - t0);
    const bool do_xsum = a.xsum != nullptr && blockIdx.x == 0 && warp == 0;
    if (e < a.E) {
        float acc[TPB];
#pragma unroll
        for (int i = 0; i < TPB; ++i) acc[i] = 0.f;
        for (int c0 = lane; c0 - lane < nch; c0 += 32 * U) {  // same trip count on every lane (shuffles below)
            uint4 w[U], xv[TPB][U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = min(c0 + 32 * u, nch - 1);  // clamped: a repeated load, never used
                w[u] = PRE && c0 == lane ? w0[u] : *reinterpret_cast<const uint4 *>(wr + 8 * c);
#pragma unroll
                for (int i = 0; i < TPB; ++i)
                    xv[i][u] = *reinterpret_cast<const uint4 *>(a.x + (size_t)(t0 + min(i, nt - 1)) * a.d + 8 * c);
            }
#pragma unroll
            for (int i = 0; i < TPB; ++i) {
                float s = acc[i];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if (c0 + 32 * u < nch) {
                        const uint32_t xx[4] = {xv[i][u].x, xv[i][u].y, xv[i][u].z, xv[i][u].w};
                        const uint32_t ww[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            s = __fmaf_rn(bf16lo(xx[j]), bf16lo(ww[j]), s);
                            s = __fmaf_rn(bf16hi(xx[j]), bf16hi(ww[j]), s);
                        }
                    }
                }
                acc[i] = s;
            }
            if (do_xsum) {  // chunk c of lane l covers group c / 8: 8 consecutive lanes share a group
#pragma unroll
                for (int i = 0; i < TPB; ++i) {
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        const int c = c0 + 32 * u;
                        const uint4 v = xv[i][u];
                        float p = bf16lo(v.x) + bf16hi(v.x) + bf16lo(v.y) + bf16hi(v.y) + bf16lo(v.z) +
                                  bf16hi(v.z) + bf16lo(v.w) + bf16hi(v.w);
                        p += __shfl_xor_sync(0xffffffffu, p, 1);
                        p += __shfl_xor_sync(0xffffffffu, p, 2);
                        p += __shfl_xor_sync(0xffffffffu, p, 4);
                        if (i < nt && c < nch && (lane & 7) == 0) a.xsum[(size_t)(t0 + i) * xsum_stride(a.d) + c / 8] = p;
                    }
                }
            }
        }
        const float bias = a.bias ? bf2f(a.bias[e]) : 0.f;
#pragma unroll
        for (int i = 0; i < TPB; ++i) {
            float v = acc[i];
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
            if (a.bias) v = __fadd_rn(v, bias);
            if (lane == 0 && i < nt) a.logits[(size_t)(t0 + i) * a.E + e] = v;
        }
    }
    router_tail<JMAX>(a, t0, nt, warp, lane);
}

// Decode router (slot mode, E <= 128): one cluster of ceil(E / 16) <= 8 CTAs per token (grid (ceil(E / 16), T)),
// 16 warps per CTA, one expert per warp. Each logit is computed exactly as in k_router (lane l sums chunks l, l + 32,
// ... with fmaf in order, then the xor butterfly; the gate row is loaded before the PDL wait) and stored into cluster
// rank 0's shared memory; after one cluster barrier rank 0's warp 0 selects the token's experts there with
// topk_token_to's rules and arithmetic. No global counter and no reload of the logits through L2.
template <int JMAX>
__global__ void __launch_bounds__(512, 1) k_router_cl(RouterArgs a) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    __shared__ float s_lg[128];
    constexpr int U = 8;
    pdl_launch();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e = blockIdx.x * 16 + warp, t = blockIdx.y;
    const int nch = a.d / 8;
    const uint16_t *wr = a.wg + (size_t)min(e, a.E - 1) * a.d;
    uint4 w0[U];
#pragma unroll
    for (int u = 0; u < U; ++u) w0[u] = *reinterpret_cast<const uint4 *>(wr + 8 * min(lane + 32 * u, nch - 1));
    pdl_wait();
    const bool do_xsum = a.xsum != nullptr && blockIdx.x == 0 && warp == 0;
    const uint16_t *xr = a.x + (size_t)t * a.d;
    float acc = 0.f;
    for (int c0 = lane; c0 - lane < nch; c0 += 32 * U) {  // same trip count on every lane (shuffles below)
        uint4 w[U], xv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = min(c0 + 32 * u, nch - 1);  // clamped: a repeated load, never used
            w[u] = c0 == lane ? w0[u] : *reinterpret_cast<const uint4 *>(wr + 8 * c);
            xv[u] = *reinterpret_cast<const uint4 *>(xr + 8 * c);
        }
        float s = acc;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (c0 + 32 * u < nch) {
                const uint32_t xx[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
                const uint32_t ww[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    s = __fmaf_rn(bf16lo(xx[j]), bf16lo(ww[j]), s);
                    s = __fmaf_rn(bf16hi(xx[j]), bf16hi(ww[j]), s);
                }
            }
        }
        acc = s;
        if (do_xsum) {  // chunk c of lane l covers group c / 8: 8 consecutive lanes share a group
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = c0 + 32 * u;
                const uint4 v = xv[u];
                float p = bf16lo(v.x) + bf16hi(v.x) + bf16lo(v.y) + bf16hi(v.y) + bf16lo(v.z) + bf16hi(v.z) +
                          bf16lo(v.w) + bf16hi(v.w);
                p += __shfl_xor_sync(0xffffffffu, p, 1);
                p += __shfl_xor_sync(0xffffffffu, p, 2);
                p += __shfl_xor_sync(0xffffffffu, p, 4);
                if (c < nch && (lane & 7) == 0) a.xsum[(size_t)t * xsum_stride(a.d) + c / 8] = p;
            }
        }
    }
    float v = acc;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (a.bias) v = __fadd_rn(v, bf2f(a.bias[min(e, a.E - 1)]));
    if (lane == 0 && e < a.E) {
        *cl.map_shared_rank(s_lg + e, 0) = v;
        a.logits[(size_t)t * a.E + e] = v;
    }
    cl.sync();  // release / acquire across the cluster: rank 0 sees every logit
    if (cl.block_rank() == 0 && warp == 0) topk_token_to<JMAX>(a, t, lane, a.idx, a.wts, s_lg);
}

// Register-tiled logits for larger T. grid (ceil(E / (8 EW)), ceil(T / TW)), block 256: warp w computes
// experts (blockIdx.x * 8 + w) * EW .. + EW - 1 for the block's TW tokens. Every (token, expert) dot product is
// summed exactly as in k_router (lane l: chunks l, l + 32, ... in order, fmaf over each chunk's 8 elements, then
// the xor butterfly), so the logits and ids are bit-identical; the tile only reuses each loaded x / gate chunk
// and its bf16 -> fp32 conversion across EW experts / TW tokens.
template <int TW, int EW, int JMAX>
__global__ void __launch_bounds__(256) k_router_t(RouterArgs a) {
    pdl_launch();
    pdl_wait();
    constexpr int U = TW * EW >= 32 ? 1 : 2;  // chunks loaded per lane per step (registers: 8 x 4 tiles keep one)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e0 = (blockIdx.x * 8 + warp) * EW;
    const int t0 = blockIdx.y * TW;
    const int nt = min(TW, a.T - t0);
    const int nch = a.d / 8;
    const bool do_xsum = a.xsum != nullptr && blockIdx.x == 0 && warp == 0;
    if (e0 < a.E) {
        float acc[TW][EW];
#pragma unroll
        for (int i = 0; i < TW; ++i)
#pragma unroll
            for (int j = 0; j < EW; ++j) acc[i][j] = 0.f;
        const uint16_t *wr[EW];
        const uint16_t *xr[TW];
#pragma unroll
        for (int j = 0; j < EW; ++j) wr[j] = a.wg + (size_t)min(e0 + j, a.E - 1) * a.d;  // clamped rows: never stored
#pragma unroll
        for (int i = 0; i < TW; ++i) xr[i] = a.x + (size_t)(t0 + min(i, nt - 1)) * a.d;
        for (int c0 = lane; c0 - lane < nch; c0 += 32 * U) {  // same trip count on every lane (shuffles below)
            uint4 w[U][EW], xv[U][TW];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = min(c0 + 32 * u, nch - 1);  // clamped: a repeated load, never used
#pragma unroll
                for (int j = 0; j < EW; ++j) w[u][j] = *reinterpret_cast<const uint4 *>(wr[j] + 8 * c);
#pragma unroll
                for (int i = 0; i < TW; ++i) xv[u][i] = *reinterpret_cast<const uint4 *>(xr[i] + 8 * c);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (c0 + 32 * u < nch) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        float wl[EW], wh[EW];
#pragma unroll
                        for (int j = 0; j < EW; ++j) {
                            const uint32_t ww = q == 0 ? w[u][j].x : q == 1 ? w[u][j].y : q == 2 ? w[u][j].z : w[u][j].w;
                            wl[j] = bf16lo(ww);
                            wh[j] = bf16hi(ww);
                        }
#pragma unroll
                        for (int i = 0; i < TW; ++i) {
                            const uint32_t xx = q == 0 ? xv[u][i].x : q == 1 ? xv[u][i].y : q == 2 ? xv[u][i].z : xv[u][i].w;
                            const float xl = bf16lo(xx), xh = bf16hi(xx);
#pragma unroll
                            for (int j = 0; j < EW; ++j) {
                                acc[i][j] = __fmaf_rn(xl, wl[j], acc[i][j]);
                                acc[i][j] = __fmaf_rn(xh, wh[j], acc[i][j]);
                            }
                        }
                    }
                }
            }
            if (do_xsum) {  // chunk c of lane l covers group c / 8: 8 consecutive lanes share a group
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int c = c0 + 32 * u;
#pragma unroll
                    for (int i = 0; i < TW; ++i) {
                        const uint4 v = xv[u][i];
                        float p = bf16lo(v.x) + bf16hi(v.x) + bf16lo(v.y) + bf16hi(v.y) + bf16lo(v.z) +
                                  bf16hi(v.z) + bf16lo(v.w) + bf16hi(v.w);
                        p += __shfl_xor_sync(0xffffffffu, p, 1);
                        p += __shfl_xor_sync(0xffffffffu, p, 2);
                        p += __shfl_xor_sync(0xffffffffu, p, 4);
                        if (i < nt && c < nch && (lane & 7) == 0) a.xsum[(size_t)(t0 + i) * xsum_stride(a.d) + c / 8] = p;
                    }
                }
            }
        }
#pragma unroll
        for (int j = 0; j < EW; ++j) {
            const int e = e0 + j;
            const float bias = (a.bias && e < a.E) ? bf2f(a.bias[e]) : 0.f;
#pragma unroll
            for (int i = 0; i < TW; ++i) {
                float v = acc[i][j];
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
                if (a.bias) v = __fadd_rn(v, bias);
                if (lane == 0 && i < nt && e < a.E) a.logits[(size_t)(t0 + i) * a.E + e] = v;
            }
        }
    }
    router_tail<JMAX>(a, t0, nt, warp, lane);
}

// Harness path (ids given): grid ceil(T / 8), block 256. Per-token x group sums; tile mode: the last CTA
// builds the tiles.
__global__ void __launch_bounds__(256) k_prep(PrepArgs a) {
    pdl_launch();
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t = blockIdx.x * 8 + warp;
    if (t < a.T && a.x) {  // (no rows: the routing tables alone, moeb_route_tables)
        const uint16_t *xr = a.x + (size_t)t * a.xs;
        bool valid = true;
        if (a.rflag) {  // peer-memory exchange: row t is slot t % C of source t / C; wait for that source
            const int src = t / a.C;
            if (lane == 0) wait_flag_sys(a.rflag + src, *a.epoch, a.err, a.wait_ns ? *a.wait_ns : 0ull);
            __syncwarp();
            valid = (t % a.C) < *reinterpret_cast<const volatile int *>(a.rcnt + src);
        }
        if (valid) row_group_sums(xr, a.d, a.xsum + (size_t)t * xsum_stride(a.d), lane);
        if (a.idx_w && lane == 0) {  // expert-parallel row (k = 1): unpack and validate its tail
            if (valid) {
                const int2 m = *reinterpret_cast<const int2 *>(xr + a.d);
                if (m.x < 0 || m.x >= a.E) atomicOr(a.err, ERR_EXPERT_ID);
                a.idx_w[t] = m.x;
                a.wts_w[t] = __int_as_float(m.y);
            } else {
                a.idx_w[t] = SLOT_SKIP;
                a.wts_w[t] = 0.f;
            }
            __threadfence();  // the tile builder (last CTA) reads the ids
        }
    }
    if (a.tiles == nullptr) {
        if (a.idx_w) return;  // ids validated with their rows
        // slot mode: only validate ids
        for (int s = blockIdx.x * 256 + threadIdx.x; s < a.T * a.k; s += gridDim.x * 256) {
            const int e = a.idx[s];
            if (e < 0 || e >= a.E) atomicOr(a.err, ERR_EXPERT_ID);
        }
        return;
    }
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(a.cnt_all, 1u);
        s_last = prev == gridDim.x - 1;
        if (s_last) __threadfence();
    }
    __syncthreads();
    if (!s_last) return;
    build_tiles(a.idx, a.T * a.k, a.E, a.NT, a.tiles, a.ntiles, a.sorted, a.err, a.counts, a.offsets);
    if (threadIdx.x == 0) *a.cnt_all = 0;
}

#define MOEB_ROUTER_INST(TPB, U, PRE)                          \
    template __global__ void k_router<TPB, 1, U, PRE>(RouterArgs);  \
    template __global__ void k_router<TPB, 2, U, PRE>(RouterArgs);  \
    template __global__ void k_router<TPB, 4, U, PRE>(RouterArgs);  \
    template __global__ void k_router<TPB, 8, U, PRE>(RouterArgs);  \
    template __global__ void k_router<TPB, 16, U, PRE>(RouterArgs); \
    template __global__ void k_router<TPB, 32, U, PRE>(RouterArgs);
MOEB_ROUTER_INST(1, 8, false)
MOEB_ROUTER_INST(1, 8, true)
MOEB_ROUTER_INST(4, 4, false)
#undef MOEB_ROUTER_INST
#define MOEB_ROUTER_T_INST(EW)                               \
    template __global__ void k_router_t<4, EW, 1>(RouterArgs);  \
    template __global__ void k_router_t<4, EW, 2>(RouterArgs);  \
    template __global__ void k_router_t<4, EW, 4>(RouterArgs);  \
    template __global__ void k_router_t<4, EW, 8>(RouterArgs);  \
    template __global__ void k_router_t<4, EW, 16>(RouterArgs); \
    template __global__ void k_router_t<4, EW, 32>(RouterArgs);
MOEB_ROUTER_T_INST(1)
MOEB_ROUTER_T_INST(2)
MOEB_ROUTER_T_INST(4)
#undef MOEB_ROUTER_T_INST
template __global__ void k_router_cl<1>(RouterArgs);
template __global__ void k_router_cl<2>(RouterArgs);
template __global__ void k_router_cl<4>(RouterArgs);
// 8 tokens x 4 experts per warp (large T: each gate chunk loaded from L2 serves twice the tokens)
template __global__ void k_router_t<8, 4, 1>(RouterArgs);
template __global__ void k_router_t<8, 4, 2>(RouterArgs);
template __global__ void k_router_t<8, 4, 4>(RouterArgs);
template __global__ void k_router_t<8, 4, 8>(RouterArgs);
template __global__ void k_router_t<8, 4, 16>(RouterArgs);
template __global__ void k_router_t<8, 4, 32>(RouterArgs);

}  // namespace moeb
