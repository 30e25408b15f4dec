// Decode layer in ONE kernel (T * k <= 16 slots): router, gate/up, down and the weighted combine.
//
// At decode sizes the layer is a few tens of MB of expert weights read once, and what limits it is how soon and
// how many of those bytes are in flight, not arithmetic. So every CTA (one per SM, cooperative launch: all
// co-resident) does:
//   1. router (CTAs [0, nR)): one warp per expert computes its logits for every token in the router's fixed fp32
//      order (lane l sums the 8-element chunks l, l + 32, ... with fmaf, then a xor butterfly - bit-identical to
//      k_router), stores them and arrives on a counter (release);
//   2. every CTA waits for the counter (bounded), and runs top-k itself for every token (router.py rules, the
//      same code as k_router's tail), so no CTA waits for another one's selection;
//   3. the CTA's share of the work is a contiguous range of gate/up units (slot, 16 rows of f) and one of down
//      units (slot, 16 rows of d). Its producer warp turns them into items (unit, projection, <= CG 64-groups of
//      K) and issues every item's packed codes and scales at once with 1-D bulk copies into a ring of shared
//      memory slots - the down weights included, before any h exists - so the SM has its whole share of the layer
//      in flight right after routing;
//   4. consumer warps take items in order: warp MMAs on the raw int4 codes with the per-group fp32 promotion
//      (or exact E2M1 x E8M0 operands), a 16-row partial per item in shared memory; the warp that completes a
//      unit sums its partials in item order (deterministic) and runs the epilogue:
//        gate/up: bias, activation, bf16 h and its 16-row sum to global memory, then +1 on the slot's counter;
//        down:    waits (bounded) until the slot's counter shows all f/16 row blocks of h, stages h once per CTA
//                 and slot, and at the end writes weight * (W_down h + b_down) and arrives on the (token, row
//                 block) counter; the last of the token's k slots sums them in slot order + residual -> y;
//   5. the last CTA to leave resets the counters for the next call.
// Every wait is bounded (mbarrier polls, or ~2 s of %globaltimer); a timeout records MOEB_DEVERR_TIMEOUT, the CTA
// stops consuming, waits (bounded) for its copies in flight and leaves.
// Reference kernels: GATE_UP_SRC / DOWN_SRC of moelab/variants/mlx/metal_q4_decode_v4.py:67-144 (int4) and the
// MXFP4 GEMV kernels of moelab/variants/mlx/metal_mxfp4_moe.py:74-141.
#include <algorithm>

#include "experts_common.cuh"
#include "route_common.cuh"

namespace moeb {

namespace {

MOEB_DEV unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
MOEB_DEV void st_release_gpu(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// logits of expert e for every token: k_router's per-lane chunk order and butterfly (bit-identical)
MOEB_DEV void logits_expert(const RouterArgs &r, int e, int lane) {
    constexpr int U = 8;
    const int nch = r.d / 8;
    const uint16_t *wr = r.wg + (size_t)e * r.d;
    const float bias = r.bias ? bf2f(r.bias[e]) : 0.f;
    for (int t = 0; t < r.T; ++t) {
        float s = 0.f;
        for (int c0 = lane; c0 - lane < nch; c0 += 32 * U) {
            uint4 w[U], xv[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = min(c0 + 32 * u, nch - 1);  // clamped: a repeated load, never used
                w[u] = *reinterpret_cast<const uint4 *>(wr + 8 * c);
                xv[u] = *reinterpret_cast<const uint4 *>(r.x + (size_t)t * r.d + 8 * c);
            }
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
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        if (r.bias) s = __fadd_rn(s, bias);
        if (lane == 0) r.logits[(size_t)t * r.E + e] = s;
    }
}

// What one item of the CTA's list is: unit (global index), projection (0 gate, 1 up, 2 down), first group,
// group count, and its place in the CTA's partial / unit-counter arrays.
struct Item {
    int unit, proj, g0, ng, ulocal, slot, rb;
};

MOEB_DEV Item item_of(const DecodePlan &P, int i, int gu0, int n_gu_items, int dn0, int RBf, int RBd, int Gd, int Gf) {
    Item it;
    if (i < n_gu_items) {
        const int per = 2 * P.NCd;
        const int ul = i / per, rem = i - ul * per;
        it.proj = rem / P.NCd;
        const int ch = rem - it.proj * P.NCd;
        it.unit = gu0 + ul;
        it.ulocal = ul;
        it.slot = it.unit / RBf;
        it.rb = it.unit - it.slot * RBf;
        it.g0 = ch * P.CGd;
        it.ng = P.CGd;
    } else {
        const int j = i - n_gu_items;
        const int vl = j / P.NCf, ch = j - vl * P.NCf;
        it.proj = 2;
        it.unit = dn0 + vl;
        it.ulocal = P.max_gu_units + vl;
        it.slot = it.unit / RBd;
        it.rb = it.unit - it.slot * RBd;
        it.g0 = ch * P.CGf;
        it.ng = P.CGf;
    }
    return it;
}

// One item's dot products: 16 weight rows x the slot's activation row over NG groups of K starting at g0. Branch
// free, so the NG groups' loads, unpacks and MMAs interleave. act: this lane's B source (lanes with gq == 0: the
// activation row (x or h, bf16, in shared memory) + 16 c; the others: a zero block read at the same offsets as
// group 0 - astr 0); sums: int4 only - per-group sums of the row (SUMS4: four 16-row sums per group). Partial rows
// gq, gq + 8 land in lanes with c == 0.
template <int FMT, int NG, bool SUMS4>
MOEB_DEV void item_dot_n(const unsigned char *slot_mem, int cg_bytes, int g0, const uint16_t *act, int astr,
                         const float *sums, int lane, float &p0, float &p1) {
    const int gq = lane >> 2, c = lane & 3;
    const uint4 *wq = reinterpret_cast<const uint4 *>(slot_mem);
    const uint32_t *wsb = reinterpret_cast<const uint32_t *>(slot_mem + cg_bytes);
    float C[2][1][4] = {{{0.f, 0.f, 0.f, 0.f}}, {{0.f, 0.f, 0.f, 0.f}}};  // two chains (alternate groups)
    uint4 w[NG];
    uint2 sb[NG];
#pragma unroll
    for (int gl = 0; gl < NG; ++gl) {
        w[gl] = wq[gl * 32 + lane];
        if (FMT == FMT_FP4) sb[gl] = make_uint2(wsb[gl * 8 + gq], 0u);
        else sb[gl] = *reinterpret_cast<const uint2 *>(wsb + (gl * 8 + gq) * 2);
    }
#pragma unroll
    for (int gl = 0; gl < NG; ++gl) {
        const int g = g0 + gl;
        const uint4 u0 = *reinterpret_cast<const uint4 *>(act + g * astr);
        const uint4 u1 = *reinterpret_cast<const uint4 *>(act + g * astr + 8);
        const uint32_t xb[1][8] = {{u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w}};
        float s0 = 0.f;
        if (FMT == FMT_Q4) {
            if (SUMS4) {
                const float4 v = *reinterpret_cast<const float4 *>(sums + 4 * g);
                s0 = (v.x + v.y) + (v.z + v.w);
            } else {
                s0 = sums[g];
            }
            s0 = c == 0 ? s0 : 0.f;  // column 0 (the slot's row) of the D fragment sits in lanes with c == 0
        }
        const float sx[1][2] = {{s0, 0.f}};
        wgroup<FMT, 1>(w[gl], sb[gl], c, xb, sx, C[gl & 1]);
    }
    p0 = C[0][0][0] + C[1][0][0];
    p1 = C[0][0][2] + C[1][0][2];
}

template <int FMT, bool SUMS4>
MOEB_DEV void item_dot(const unsigned char *slot_mem, int cg_bytes, int ng, int g0, const uint16_t *act, int astr,
                       const float *sums, int lane, float &p0, float &p1) {
    // ng is one of the chunk sizes decode_plan picks (a divisor of the projection's group count)
    switch (ng) {
        case 8: item_dot_n<FMT, 8, SUMS4>(slot_mem, cg_bytes, g0, act, astr, sums, lane, p0, p1); break;
        case 6: item_dot_n<FMT, 6, SUMS4>(slot_mem, cg_bytes, g0, act, astr, sums, lane, p0, p1); break;
        case 5: item_dot_n<FMT, 5, SUMS4>(slot_mem, cg_bytes, g0, act, astr, sums, lane, p0, p1); break;
        case 4: item_dot_n<FMT, 4, SUMS4>(slot_mem, cg_bytes, g0, act, astr, sums, lane, p0, p1); break;
        case 3: item_dot_n<FMT, 3, SUMS4>(slot_mem, cg_bytes, g0, act, astr, sums, lane, p0, p1); break;
        case 2: item_dot_n<FMT, 2, SUMS4>(slot_mem, cg_bytes, g0, act, astr, sums, lane, p0, p1); break;
        default: item_dot_n<FMT, 1, SUMS4>(slot_mem, cg_bytes, g0, act, astr, sums, lane, p0, p1); break;
    }
}

}  // namespace

MOEB_DEV unsigned long long ld_volatile_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Shared-memory layout and work split of one launch: DecodePlan (decode_plan in api.cu).
template <int FMT>
__global__ void __launch_bounds__(DEC_THREADS, 1) k_decode(const __grid_constant__ DecodeArgs A) {
    const ExpArgs &a = A.a;
    const RouterArgs &r = A.r;
    const DecodePlan &P = A.p;
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char *ring = smem + P.o_ring;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + P.o_bar);
    uint64_t *empty = full + P.NSLOT;
    uint16_t *xs = reinterpret_cast<uint16_t *>(smem + P.o_x);
    float *xsum = reinterpret_cast<float *>(smem + P.o_xsum);
    int *sidx = reinterpret_cast<int *>(smem + P.o_idx);
    float *swts = reinterpret_cast<float *>(smem + P.o_wts);
    float *part = reinterpret_cast<float *>(smem + P.o_part);  // also the logits [T][E4] before the items start
    int *ucnt = reinterpret_cast<int *>(smem + P.o_ucnt);
    unsigned char *hbuf = smem + P.o_h;
    int *hstate = reinterpret_cast<int *>(smem + P.o_hstate);
    __shared__ int s_abort;
    __shared__ unsigned s_epoch;
    __shared__ __align__(16) uint16_t zeros[16];  // B operand of the lanes that carry no activation column
    __shared__ int s_sel[16 * 32];                  // top-k scratch [T][k]

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int T = a.T, d = a.d, f = a.f, ks = a.k, S = T * ks;
    const int RBf = f >> 4, RBd = d >> 4, Gd = d >> 6, Gf = f >> 6;
    const int hrow_bytes = f * 2 + (f / 16) * 4;
    const int cg_bytes = max(P.CGd, P.CGf) * 512;  // codes of a ring slot; its scales follow
    // ---- prologue (overlaps the previous kernel's tail): barriers, counters
    if (warp == P.NW && lane == 0) {
        for (int i = 0; i < P.NSLOT; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, 1);
        }
        mbar_fence_init();
    }
    for (int i = threadIdx.x; i < P.max_gu_units + P.max_dn_units; i += blockDim.x) ucnt[i] = 0;
    for (int i = threadIdx.x; i < P.NSL; i += blockDim.x) hstate[i] = 0;
    if (threadIdx.x < 16) zeros[threadIdx.x] = 0;
    if (threadIdx.x == 0) s_abort = 0;
    pdl_launch();
    pdl_wait();
    // the call's generation: read before this CTA arrives; the last CTA to arrive advances it (after every CTA's
    // read and every logit), so it is this call's tag for the h and output records
    unsigned g0 = 0;
    if (threadIdx.x == 0) g0 = *(volatile unsigned *)A.gen;
    // ---- router: logits of this CTA's experts (one expert per warp, every token; x and gate rows straight from
    // global memory, one round trip), spread one expert per CTA first
    const bool routing = r.wg != nullptr;
    if (routing && warp < P.NW)
        for (int e = blockIdx.x + gridDim.x * warp; e < r.E; e += gridDim.x * P.NW) logits_expert(r, e, lane);
    __syncthreads();
    if (threadIdx.x == 0) {
        if (atom_add_acq_rel_gpu(A.arr, 1u) == gridDim.x - 1) {
            *(volatile unsigned *)A.arr = 0u;
            __threadfence();
            st_release_gpu(A.gen, g0 + 1u);
        }
    }
    // ---- x rows into shared memory, per-64-group sums (int4 promotion)
    {
        const int n4 = T * d / 8;
        for (int i = threadIdx.x; i < n4; i += blockDim.x) {
            const int t = i / (d / 8), c = i - t * (d / 8);
            reinterpret_cast<uint4 *>(xs)[i] = *reinterpret_cast<const uint4 *>(a.x + (size_t)t * a.xs + 8 * c);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < T * Gd; i += blockDim.x) {
        const int t = i / Gd, g = i - t * Gd;
        const uint4 *p = reinterpret_cast<const uint4 *>(xs + (size_t)t * d + g * 64);
        float sm = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const uint4 u = p[q];
            sm += bf16lo(u.x) + bf16hi(u.x) + bf16lo(u.y) + bf16hi(u.y) + bf16lo(u.z) + bf16hi(u.z) + bf16lo(u.w) +
                  bf16hi(u.w);
        }
        xsum[i] = sm;
    }
    if (threadIdx.x == 0) {
        // bounded wait for the generation to advance (every CTA arrived: all logits are stored)
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_gpu(A.gen) == g0) {
            if (globaltimer_ns() - t0 > 2000000000ull) {
                atomicOr(a.err, ERR_TIMEOUT);
                s_abort = 1;
                break;
            }
            __nanosleep(20);
        }
        s_epoch = g0 + 1u;
    }
    __syncthreads();
    const unsigned epoch = s_epoch;
    // ---- top-k in every CTA (from the stored logits) or the given ids
    if (routing) {
        float *lg = part;
        const int E4 = (r.E + 15) & ~15;
        for (int i = threadIdx.x; i < T * E4; i += blockDim.x) {
            const int t = i / E4, e = i - t * E4;
            const float l = e < r.E ? __ldcg(r.logits + (size_t)t * r.E + e) : -INFINITY;
            lg[i] = isnan(l) ? -INFINITY : l + 0.f;  // NaN = -inf; -0 -> +0
        }
        __syncthreads();
        topk_rank(r, T, lg, s_sel, sidx, swts);
        __syncthreads();
        if (blockIdx.x == 0)
            for (int s = threadIdx.x; s < S; s += blockDim.x) {
                r.idx[s] = sidx[s];
                r.wts[s] = swts[s];
            }
    } else {
        for (int s = threadIdx.x; s < S; s += blockDim.x) {
            sidx[s] = a.idx[s];
            swts[s] = a.wts[s];
            if (blockIdx.x == 0 && (a.idx[s] < 0 || a.idx[s] >= a.E)) atomicOr(a.err, ERR_EXPERT_ID);
        }
    }
    __syncthreads();
    // ---- this CTA's units and items
    const int Ugu = S * RBf, Udn = S * RBd;
    const int gu0 = (int)((long)blockIdx.x * Ugu / gridDim.x), gu1 = (int)((long)(blockIdx.x + 1) * Ugu / gridDim.x);
    const int dn0 = (int)((long)blockIdx.x * Udn / gridDim.x), dn1 = (int)((long)(blockIdx.x + 1) * Udn / gridDim.x);
    const int n_gu_items = (gu1 - gu0) * 2 * P.NCd;
    const int n_items = n_gu_items + (dn1 - dn0) * P.NCf;
    const int s_first = dn0 / RBd;  // first slot of the down range (h staging index base)
    const uint32_t sbw = FMT == FMT_FP4 ? 8 : 16;  // scale words per (row block, group)

    if (warp == P.NW) {
        // ---------------- producer: every item's codes and scales, 32 items per step (one per lane)
        const uint64_t pol = l2_evict_first_policy();
        for (int base = 0; base < n_items; base += 32) {
            const int i = base + lane;
            bool ok = true;
            if (i < n_items) {
                const int sl = i % P.NSLOT;
                if (i >= P.NSLOT) ok = mbar_wait_bounded(empty + sl, ((i / P.NSLOT) - 1) & 1);
                if (ok && !*(volatile int *)&s_abort) {
                    const Item it = item_of(P, i, gu0, n_gu_items, dn0, RBf, RBd, Gd, Gf);
                    int e = sidx[it.slot];
                    if (e < 0 || e >= a.E) e = 0;
                    const QProj &Q = it.proj == 0 ? a.g : it.proj == 1 ? a.u : a.dn;
                    const int G = it.proj == 2 ? Gf : Gd;
                    const size_t blk = (size_t)e * (it.proj == 2 ? RBd : RBf) + it.rb;
                    const size_t gi = blk * G + it.g0;
                    unsigned char *dst = ring + (size_t)sl * P.slot_bytes;
                    mbar_expect_tx(full + sl, (unsigned)it.ng * (512u + sbw * 4u));
                    tma_load_1d(dst, Q.q + gi * 128, (unsigned)it.ng * 512u, full + sl, pol);
                    tma_load_1d(dst + cg_bytes, Q.sb + gi * sbw, (unsigned)it.ng * sbw * 4u, full + sl, pol);
                } else if (!ok) {
                    atomicOr(a.err, ERR_TIMEOUT);
                    s_abort = 1;
                }
            }
            if (__any_sync(0xffffffffu, !ok) || *(volatile int *)&s_abort) break;
        }
    } else {
        // ---------------- consumers: items w, w + NW, ...
        const int gq = lane >> 2, c = lane & 3;
        for (int i = warp; i < n_items; i += P.NW) {
            if (*(volatile int *)&s_abort) break;
            const int sl = i % P.NSLOT;
            if (!mbar_wait_bounded(full + sl, (i / P.NSLOT) & 1)) {
                if (lane == 0) {
                    atomicOr(a.err, ERR_TIMEOUT);
                    s_abort = 1;
                }
                break;
            }
            const Item it = item_of(P, i, gu0, n_gu_items, dn0, RBf, RBd, Gd, Gf);
            const int slot = it.slot;
            const unsigned char *sm = ring + (size_t)sl * P.slot_bytes;
            float p0, p1;
            if (it.proj < 2) {
                const int t = slot / ks;
                const uint16_t *act = gq == 0 ? xs + (size_t)t * d + 16 * c : zeros;
                item_dot<FMT, false>(sm, cg_bytes, it.ng, it.g0, act, gq == 0 ? 64 : 0, xsum + (size_t)t * Gd, lane,
                                     p0, p1);
            } else {
                // the slot's h (all f rows), staged once per CTA and slot: its records carry this call's tag
                const int hs = slot - s_first;
                uint16_t *hsm = reinterpret_cast<uint16_t *>(hbuf + (size_t)hs * hrow_bytes);
                float *hsum_sm = reinterpret_cast<float *>(hbuf + (size_t)hs * hrow_bytes + f * 2);
                int own = 0;
                if (lane == 0) own = atomicCAS(hstate + hs, 0, 1) == 0;
                own = __shfl_sync(0xffffffffu, own, 0);
                bool ready = true;
                if (own) {
                    const unsigned long long *rec = A.hrec + (size_t)slot * f;
                    const uint64_t t0 = globaltimer_ns();
                    for (;;) {
                        bool mine = true;
                        for (int q = lane; q < f; q += 32) {
                            const unsigned long long v = ld_volatile_u64(rec + q);
                            if ((unsigned)(v >> 32) == epoch) hsm[q] = (uint16_t)v;
                            else mine = false;
                        }
                        if (__all_sync(0xffffffffu, mine)) break;
                        if (globaltimer_ns() - t0 > 2000000000ull) {
                            if (lane == 0) atomicOr(a.err, ERR_TIMEOUT);
                            ready = false;
                            break;
                        }
                        __nanosleep(20);
                    }
                    __syncwarp();
                    for (int q = lane; q < f / 16; q += 32) {  // 16-row sums of the bf16 h (int4 promotion)
                        float hf = 0.f;
#pragma unroll
                        for (int j = 0; j < 16; ++j) hf += bf2f(hsm[q * 16 + j]);
                        hsum_sm[q] = hf;
                    }
                    __syncwarp();
                    if (lane == 0) {
                        __threadfence_block();
                        atomicExch(hstate + hs, 2);
                    }
                } else if (lane == 0) {
                    const uint64_t t0 = globaltimer_ns();
                    while (*(volatile int *)(hstate + hs) != 2) {
                        if (globaltimer_ns() - t0 > 2000000000ull) {
                            atomicOr(a.err, ERR_TIMEOUT);
                            ready = false;
                            break;
                        }
                        __nanosleep(20);
                    }
                    __threadfence_block();
                }
                ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
                if (!ready) {
                    if (lane == 0) s_abort = 1;
                    break;
                }
                __syncwarp();
                const uint16_t *act = gq == 0 ? hsm + 16 * c : zeros;
                item_dot<FMT, true>(sm, cg_bytes, it.ng, it.g0, act, gq == 0 ? 64 : 0, hsum_sm, lane, p0, p1);
            }
            if (c == 0) {
                part[i * 16 + gq] = p0;
                part[i * 16 + gq + 8] = p1;
            }
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                mbar_arrive(empty + sl);  // the slot's bytes are consumed
                __threadfence_block();
                last = atomicAdd(ucnt + it.ulocal, 1) == (it.proj < 2 ? 2 * P.NCd : P.NCf) - 1;
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) continue;
            __threadfence_block();
            const int e_raw = sidx[slot];
            const bool valid = e_raw >= 0 && e_raw < a.E;
            const int e = valid ? e_raw : 0;
            if (it.proj < 2) {
                // gate/up epilogue: rows rb*16 + lane (lane < 16), partials summed in item order; h goes out as
                // tagged 64-bit records {tag, bf16 h}, each one store
                const int ib = it.ulocal * 2 * P.NCd;
                if (lane < 16) {
                    float gv = 0.f, uv = 0.f;
                    for (int ch = 0; ch < P.NCd; ++ch) gv += part[(ib + ch) * 16 + lane];
                    for (int ch = 0; ch < P.NCd; ++ch) uv += part[(ib + P.NCd + ch) * 16 + lane];
                    const int row = it.rb * 16 + lane;
                    if (a.bg) {
                        gv += a.bg[(size_t)e * f + row];
                        uv += a.bu[(size_t)e * f + row];
                    }
                    const uint16_t hb = f2bf(act_glu(a.act, gv, uv));
                    __stcg(A.hrec + (size_t)slot * f + row, ((unsigned long long)epoch << 32) | hb);
                }
            } else {
                // down epilogue: weight * (acc + bias) as tagged records {tag, fp32}
                const int ib = n_gu_items + (it.ulocal - P.max_gu_units) * P.NCf;
                if (lane < 16) {
                    const int row = it.rb * 16 + lane;
                    float acc = 0.f;
                    for (int ch = 0; ch < P.NCf; ++ch) acc += part[(ib + ch) * 16 + lane];
                    if (a.bd) acc += a.bd[(size_t)e * d + row];
                    const float v = (valid ? swts[slot] : 0.f) * acc;
                    __stcg(A.yrec + (size_t)slot * d + row, ((unsigned long long)epoch << 32) | __float_as_uint(v));
                }
            }
        }
        // ---------------- combine: this CTA's (token, 16-row block) pairs, one per warp: the token's k slot
        // records (polled until they carry this call's tag) summed in slot order, + residual
        const int NP = T * RBd;
        const int p0_ = (int)((long)blockIdx.x * NP / gridDim.x), p1_ = (int)((long)(blockIdx.x + 1) * NP / gridDim.x);
        for (int pr = p0_ + warp; pr < p1_ && !*(volatile int *)&s_abort; pr += P.NW) {
            const int t = pr / RBd, rb = pr - t * RBd;
            const int row = rb * 16 + (lane & 15);
            float acc = 0.f;
            bool ok = true;
            if (lane < 16) {
                const uint64_t t0 = globaltimer_ns();
                for (int j = 0; j < ks; ++j) {
                    const unsigned long long *rp = A.yrec + ((size_t)t * ks + j) * d + row;
                    unsigned long long v = ld_volatile_u64(rp);
                    while ((unsigned)(v >> 32) != epoch) {
                        if (globaltimer_ns() - t0 > 2000000000ull) {
                            atomicOr(a.err, ERR_TIMEOUT);
                            ok = false;
                            break;
                        }
                        __nanosleep(20);
                        v = ld_volatile_u64(rp);
                    }
                    if (!ok) break;
                    acc += __uint_as_float((unsigned)v);
                }
                if (a.residual) acc += bf2f(a.residual[(size_t)t * d + row]);
                a.y[(size_t)t * d + row] = f2bf(acc);
            }
            if (!__all_sync(0xffffffffu, ok)) {
                if (lane == 0) s_abort = 1;
            }
        }
    }
    __syncthreads();
    // ---- copies still in flight after an abort: wait for them (bounded) before the CTA's shared memory goes
    if (s_abort && warp == P.NW) {
        for (int sl = lane; sl < P.NSLOT && sl < n_items; sl += 32) {
            const int last_i = sl + ((n_items - 1 - sl) / P.NSLOT) * P.NSLOT;  // the slot's last item
            mbar_wait_bounded(full + sl, (last_i / P.NSLOT) & 1, 1u << 16);
        }
    }
}

template __global__ void k_decode<FMT_Q4>(const __grid_constant__ DecodeArgs);
template __global__ void k_decode<FMT_FP4>(const __grid_constant__ DecodeArgs);

}  // namespace moeb
