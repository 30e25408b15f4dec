// Fused decode layer: router, gate/up and down (+ combine) of a decode call (T*k <= 16 slots) in ONE
// cooperative kernel, so the three phases hand over through device-memory counters instead of kernel
// boundaries (each boundary costs a launch and a drain on the critical path of a ~20 us layer).
//
//   phase A  CTAs [0, nR): warp w of CTA c computes the logits of experts c*8 + w (+ 8 * grid stride) for every
//            token, in the router's fixed fp32 order (bit-identical logits). Each CTA then arrives on a counter;
//            the last one runs top-k per token (router.py rules), the x group sums, and releases the "routed"
//            flag. With ids given (harness run()), CTA 0 computes the group sums and releases the flag.
//   phase B  every CTA waits for the flag, then takes (slot, 16-row block) gate/up units (slots_common.cuh)
//            grid-stride; after each unit it adds one to the slot's "rows of h ready" counter.
//   phase C  every WARP takes (slot, 16-row block) down units grid-stride (whole K per warp, h from L2); each
//            first waits until its slot's h is complete (all f/16 row blocks), then runs the unit with the fused
//            weighted combine.
//   exit     the last CTA to leave resets the flag and the counters for the next call.
// All CTAs are co-resident (cooperative launch sized from the occupancy), and every CTA finishes all its phase-B
// units before any of its warps waits in phase C, so every wait is satisfied by work already assigned to running
// CTAs. Each
// wait is bounded (~2 s of wall time): a timeout records MOEB_DEVERR_TIMEOUT and the CTA carries on.
#include <algorithm>

#include "route_common.cuh"
#include "slots_common.cuh"

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
// Bounded wait (thread 0 of the CTA) until *p >= want; the CTA barrier afterwards publishes the acquire.
MOEB_DEV void wait_at_least(const unsigned *p, unsigned want, unsigned *err) {
    if (threadIdx.x == 0 && ld_acquire_gpu(p) < want) {
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_gpu(p) < want) {
            if (globaltimer_ns() - t0 > 2000000000ull) {
                atomicOr(err, ERR_TIMEOUT);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
}

// logits of expert e for every token, the same per-lane chunk order and butterfly as k_router
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
                const int c = min(c0 + 32 * u, nch - 1);
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

// One down unit (slot, 16-row block) by one warp over the whole K: the h row and its sums come straight from L2
// (written by other CTAs of this kernel, published by the slot counter the caller waited on).
template <int FMT, int GPW>
MOEB_DEV void down_warp_unit(const ExpArgs &a, int unit, int lane) {
    const int gq = lane >> 2, c = lane & 3;
    const int d = a.d, f = a.f, RB = d >> 4, G = f >> 6;
    const int slot = unit / RB, rb = unit - slot * RB;
    const TileInfo ti = tile_info(a, slot);
    const size_t blk = (size_t)ti.e * RB + rb;
    const uint16_t *hrow = a.h + (size_t)slot * f;
    const float *hsr = a.hsum + (size_t)slot * (f / 16);
    float C[1][4] = {{0.f, 0.f, 0.f, 0.f}};
    for (int g0 = 0; g0 < G; g0 += GPW) {
        uint4 w[GPW];
        uint2 b[GPW];
#pragma unroll
        for (int i = 0; i < GPW; ++i) {
            const int g = min(g0 + i, G - 1);  // clamped: a repeated load, never used
            w[i] = ld_w(a.dn, blk, G, g, lane);
            b[i] = ld_scales<FMT>(a.dn, blk, G, g, gq);
        }
#pragma unroll
        for (int i = 0; i < GPW; ++i) {
            if (g0 + i < G) {
                const int g = g0 + i;
                uint32_t hb[1][8];
                if (gq == 0) {
                    const uint4 u0 = __ldcg(reinterpret_cast<const uint4 *>(hrow + g * 64 + 16 * c));
                    const uint4 u1 = __ldcg(reinterpret_cast<const uint4 *>(hrow + g * 64 + 16 * c + 8));
                    hb[0][0] = u0.x; hb[0][1] = u0.y; hb[0][2] = u0.z; hb[0][3] = u0.w;
                    hb[0][4] = u1.x; hb[0][5] = u1.y; hb[0][6] = u1.z; hb[0][7] = u1.w;
                } else {
#pragma unroll
                    for (int q = 0; q < 8; ++q) hb[0][q] = 0u;
                }
                float s0 = 0.f;
                if (FMT == FMT_Q4 && c == 0 && gq == 0) {
                    const float4 v = __ldcg(reinterpret_cast<const float4 *>(hsr + 4 * g));
                    s0 = (v.x + v.y) + (v.z + v.w);
                }
                const float sx[1][2] = {{__shfl_sync(0xffffffffu, s0, 0), 0.f}};
                wgroup<FMT, 1>(w[i], b[i], c, hb, sx, C);
            }
        }
    }
    down_store_combine<1>(a, ti, rb, C, lane);
}

}  // namespace

// Workspace counters (in the zeroed counter region, left zero on exit): ctr[0] router arrivals, ctr[1] routed
// flag, ctr[2] CTAs done, ctr[16 + s] rows of h ready for slot s (s < 16).
template <int FMT, int JMAX>
__global__ void __launch_bounds__(256, 2) k_decode(ExpArgs a, RouterArgs r, unsigned *ctr) {
    extern __shared__ uint4 dsm[];  // max(x row, h row + h sums)
    __shared__ float red[8 * 2 * 4 * 32];
    __shared__ int s_last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int TK = a.T * a.k, RBf = a.f >> 4, RBd = a.d >> 4;
    // ------------------------------------------------------------ phase A: routing
    if (r.wg) {
        const int nR = min((int)gridDim.x, (r.E + 7) / 8);
        if ((int)blockIdx.x < nR) {
            for (int e = blockIdx.x * 8 + warp; e < r.E; e += nR * 8) logits_expert(r, e, lane);
            __syncthreads();
            if (threadIdx.x == 0) {
                __threadfence();
                s_last = atomicAdd(ctr + 0, 1u) == (unsigned)(nR - 1);
                if (s_last) __threadfence();
            }
            __syncthreads();
            if (s_last) {
                for (int t = warp; t < r.T; t += 8) topk_token<JMAX>(r, t, lane);
                if (r.xsum)
                    for (int t = warp; t < r.T; t += 8)
                        row_group_sums(r.x + (size_t)t * r.d, r.d, r.xsum + (size_t)t * xsum_stride(r.d), lane);
                __syncthreads();
                if (threadIdx.x == 0) {
                    ctr[0] = 0u;
                    __threadfence();
                    st_release_gpu(ctr + 1, 1u);
                }
            }
        }
    } else if (blockIdx.x == 0) {  // ids given: group sums (int4 promotion) and id checks, then release
        for (int t = warp; t < a.T; t += 8)
            row_group_sums(a.x + (size_t)t * a.xs, a.d, const_cast<float *>(a.xsum) + (size_t)t * xsum_stride(a.d), lane);
        for (int s = threadIdx.x; s < TK; s += blockDim.x) {
            const int e = a.idx[s];
            if (e < 0 || e >= a.E) atomicOr(a.err, ERR_EXPERT_ID);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            st_release_gpu(ctr + 1, 1u);
        }
    }
    wait_at_least(ctr + 1, 1u, a.err);
    // ------------------------------------------------------------ phase B: gate/up units
    for (int unit = blockIdx.x; unit < TK * RBf; unit += gridDim.x) {
        gate_up_slot_unit<FMT, 8, 4>(a, unit, dsm, red);
        if (threadIdx.x == 0) {  // h rows of this unit (written by warp 0, ordered by the barrier) before the count
            __threadfence();
            atomicAdd(ctr + 16 + unit / RBf, 1u);
        }
    }
    // ------------------------------------------------------------ phase C: down units, one per warp
    for (int unit = blockIdx.x * 8 + warp; unit < TK * RBd; unit += gridDim.x * 8) {
        if (lane == 0) {  // bounded wait for the slot's h (all f/16 row blocks)
            const unsigned *p = ctr + 16 + unit / RBd;
            if (ld_acquire_gpu(p) < (unsigned)RBf) {
                const uint64_t t0 = globaltimer_ns();
                while (ld_acquire_gpu(p) < (unsigned)RBf) {
                    if (globaltimer_ns() - t0 > 2000000000ull) {
                        atomicOr(a.err, ERR_TIMEOUT);
                        break;
                    }
                    __nanosleep(64);
                }
            }
        }
        __syncwarp();
        down_warp_unit<FMT, 4>(a, unit, lane);
    }
    // ------------------------------------------------------------ exit: the last CTA resets the counters
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(ctr + 2, 1u) == gridDim.x - 1) {
            __threadfence();
            for (int s = 0; s < TK; ++s) ctr[16 + s] = 0u;
            ctr[1] = 0u;
            ctr[2] = 0u;
            __threadfence();
        }
    }
}

size_t decode_smem(int d, int f) { return std::max((size_t)d * 2, (size_t)f * 2 + (size_t)f / 16 * 4); }

#define MOEB_DECODE(FMT)                                                        \
    template __global__ void k_decode<FMT, 1>(ExpArgs, RouterArgs, unsigned *);  \
    template __global__ void k_decode<FMT, 2>(ExpArgs, RouterArgs, unsigned *);  \
    template __global__ void k_decode<FMT, 4>(ExpArgs, RouterArgs, unsigned *);  \
    template __global__ void k_decode<FMT, 8>(ExpArgs, RouterArgs, unsigned *);  \
    template __global__ void k_decode<FMT, 16>(ExpArgs, RouterArgs, unsigned *); \
    template __global__ void k_decode<FMT, 32>(ExpArgs, RouterArgs, unsigned *);
MOEB_DECODE(FMT_Q4)
MOEB_DECODE(FMT_FP4)

}  // namespace moeb
