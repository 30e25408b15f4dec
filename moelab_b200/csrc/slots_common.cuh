// Decode (slot mode) unit bodies: one (slot, 16-row block) of gate/up or down with KS warps splitting the K
// groups and GPW groups per warp loaded at once. Used by k_gate_up_slots / k_down_slots / k_down_tok (experts.cu).
// Every thread of the CTA calls them (they use __syncthreads).
#pragma once
#include "experts_common.cuh"

namespace moeb {

// xs4: d bf16 of shared memory; red: KS * 2 * 4 * 32 floats of shared memory.
template <int FMT, int KS, int GPW>
__device__ __forceinline__ void gate_up_slot_unit(const ExpArgs &a, int unit, uint4 *xs4, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gq = lane >> 2, c = lane & 3;
    const int d = a.d, f = a.f;
    const int RB = f >> 4, G = d >> 6;
    const int g_beg = warp * G / KS, g_end = (warp + 1) * G / KS;
    const uint16_t *xs = reinterpret_cast<const uint16_t *>(xs4);
    const int slot = unit / RB, rb = unit - slot * RB;
    if (a.idx[slot] == SLOT_SKIP) return;  // padding row of a peer-exchange block (uniform across the CTA)
    const TileInfo ti = tile_info(a, slot);
    const size_t blk = (size_t)ti.e * RB + rb;
    if (warp == KS - 1 && a.dn_prefetch) prefetch_down(a, ti.e, rb, RB, lane);
    const uint4 *xsrc = reinterpret_cast<const uint4 *>(a.x + (size_t)(slot / a.k) * a.xs);
    const float *sxr = a.xsum + (size_t)(slot / a.k) * xsum_stride(d);
    float Cg[1][4] = {{0.f, 0.f, 0.f, 0.f}}, Cu[1][4] = {{0.f, 0.f, 0.f, 0.f}};
    bool synced = false;
    for (int g0 = g_beg; g0 < g_end; g0 += GPW) {
        uint4 wg[GPW], wu[GPW];
        uint2 bg[GPW], bu[GPW];
#pragma unroll
        for (int i = 0; i < GPW; ++i) {
            const int g = min(g0 + i, g_end - 1);  // clamped: a repeated load, never used
            wg[i] = ld_w(a.g, blk, G, g, lane);
            wu[i] = ld_w(a.u, blk, G, g, lane);
            bg[i] = ld_scales<FMT>(a.g, blk, G, g, gq);
            bu[i] = ld_scales<FMT>(a.u, blk, G, g, gq);
        }
        if (!synced) {  // stage the x row while the first weight batch is in flight
            for (int i = threadIdx.x; i < d / 8; i += 32 * KS) xs4[i] = xsrc[i];
            __syncthreads();
            synced = true;
        }
#pragma unroll
        for (int i = 0; i < GPW; ++i) {
            if (g0 + i < g_end) {
                const int g = g0 + i;
                uint32_t xb[1][8];
                load_b16(gq == 0 ? xs + g * 64 + 16 * c : nullptr, xb[0]);
                const float sx[1][2] = {{c == 0 ? sxr[g] : 0.f, 0.f}};
                wgroup<FMT, 1>(wg[i], bg[i], c, xb, sx, Cg);
                wgroup<FMT, 1>(wu[i], bu[i], c, xb, sx, Cu);
            }
        }
    }
    if (!synced) {  // a warp without groups (G < KS) still stages its share
        for (int i = threadIdx.x; i < d / 8; i += 32 * KS) xs4[i] = xsrc[i];
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        red[((warp * 2 + 0) * 4 + i) * 32 + lane] = Cg[0][i];
        red[((warp * 2 + 1) * 4 + i) * 32 + lane] = Cu[0][i];
    }
    __syncthreads();
    if (warp == 0) {
        float gs[4], us[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            gs[i] = red[(0 * 4 + i) * 32 + lane];
            us[i] = red[(1 * 4 + i) * 32 + lane];
#pragma unroll
            for (int w = 1; w < KS; ++w) {
                gs[i] += red[((w * 2 + 0) * 4 + i) * 32 + lane];
                us[i] += red[((w * 2 + 1) * 4 + i) * 32 + lane];
            }
        }
        gate_up_store<1>(a, ti, rb, 0, gs, us, lane);
    }
    __syncthreads();
}

// One slot's down dot products for this warp's share of K (warp lw of the KS splitting the f/64 groups), with
// the slot's h row and block sums staged into hs4 by the KS * 32 threads ltid = 0 .. (the first weight batch is
// issued before the staging). Contains exactly one __syncthreads; every thread of the CTA must call it.
template <int FMT, int KS, int GPW>
__device__ __forceinline__ void down_slot_partial(const ExpArgs &a, int slot, size_t blk, int lw, int ltid,
                                                  uint4 *hs4, float (&C)[1][4]) {
    const int lane = threadIdx.x & 31, gq = lane >> 2, c = lane & 3;
    const int f = a.f, G = f >> 6;
    const int g_beg = lw * G / KS, g_end = (lw + 1) * G / KS;
    const uint16_t *hs = reinterpret_cast<const uint16_t *>(hs4);
    const float *hsum_s = reinterpret_cast<const float *>(hs4 + f / 8);
    const uint4 *hsrc = reinterpret_cast<const uint4 *>(a.h + (size_t)slot * f);
    const uint4 *ssrc = reinterpret_cast<const uint4 *>(a.hsum + (size_t)slot * (f / 16));
#pragma unroll
    for (int i = 0; i < 4; ++i) C[0][i] = 0.f;
    bool synced = false;
    for (int g0 = g_beg; g0 < g_end; g0 += GPW) {
        uint4 w[GPW];
        uint2 b[GPW];
#pragma unroll
        for (int i = 0; i < GPW; ++i) {
            const int g = min(g0 + i, g_end - 1);
            w[i] = ld_w(a.dn, blk, G, g, lane);
            b[i] = ld_scales<FMT>(a.dn, blk, G, g, gq);
        }
        if (!synced) {  // stage the h row and its block sums while the first weight batch is in flight
            for (int i = ltid; i < f / 8; i += 32 * KS) hs4[i] = __ldcg(hsrc + i);
            for (int i = ltid; i < f / 64; i += 32 * KS) hs4[f / 8 + i] = __ldcg(ssrc + i);
            __syncthreads();
            synced = true;
        }
#pragma unroll
        for (int i = 0; i < GPW; ++i) {
            if (g0 + i < g_end) {
                const int g = g0 + i;
                uint32_t hb[1][8];
                load_b16(gq == 0 ? hs + g * 64 + 16 * c : nullptr, hb[0]);
                const float4 v = *reinterpret_cast<const float4 *>(hsum_s + 4 * g);
                const float sx[1][2] = {{c == 0 ? (v.x + v.y) + (v.z + v.w) : 0.f, 0.f}};
                wgroup<FMT, 1>(w[i], b[i], c, hb, sx, C);
            }
        }
    }
    if (!synced) {
        for (int i = ltid; i < f / 8; i += 32 * KS) hs4[i] = __ldcg(hsrc + i);
        for (int i = ltid; i < f / 64; i += 32 * KS) hs4[f / 8 + i] = __ldcg(ssrc + i);
        __syncthreads();
    }
}

// down_slot_partial with the K split of KS * VW warps carried by KS warps: warp lw computes the VW consecutive
// shares lw * VW .. lw * VW + VW - 1 of that split into separate accumulators (each in the same group order as the
// warp that would own it), so the partials summed in share order equal k_down_slots with KS * VW warps bit for bit.
// All loads of the warp's groups (GPW per batch) are issued together. wait_h: the kernel has not yet waited for
// its upstream grid (the gate/up kernel writing h); the wait is taken after the first weight batch is issued and
// before h is read.
template <int FMT, int KS, int VW, int GPW>
__device__ __forceinline__ void down_slot_partial_v(const ExpArgs &a, int slot, size_t blk, int lw, int ltid,
                                                    uint4 *hs4, float (&C)[VW][1][4], bool wait_h) {
    constexpr int KV = KS * VW;
    const int lane = threadIdx.x & 31, gq = lane >> 2, c = lane & 3;
    const int f = a.f, G = f >> 6;
    int vb[VW + 1];  // share boundaries (groups), as g_beg / g_end of warps lw * VW + v of the KV split
#pragma unroll
    for (int v = 0; v <= VW; ++v) vb[v] = (lw * VW + v) * G / KV;
    const int g_beg = vb[0], g_end = vb[VW];
    const uint16_t *hs = reinterpret_cast<const uint16_t *>(hs4);
    const float *hsum_s = reinterpret_cast<const float *>(hs4 + f / 8);
    const uint4 *hsrc = reinterpret_cast<const uint4 *>(a.h + (size_t)slot * f);
    const uint4 *ssrc = reinterpret_cast<const uint4 *>(a.hsum + (size_t)slot * (f / 16));
#pragma unroll
    for (int v = 0; v < VW; ++v)
#pragma unroll
        for (int i = 0; i < 4; ++i) C[v][0][i] = 0.f;
    bool synced = false;
    for (int g0 = g_beg; g0 < g_end; g0 += GPW) {
        uint4 w[GPW];
        uint2 b[GPW];
#pragma unroll
        for (int i = 0; i < GPW; ++i) {
            const int g = min(g0 + i, g_end - 1);
            w[i] = ld_w(a.dn, blk, G, g, lane);
            b[i] = ld_scales<FMT>(a.dn, blk, G, g, gq);
        }
        if (!synced) {  // stage the h row and its block sums while the first weight batch is in flight
            if (wait_h) pdl_wait();
            for (int i = ltid; i < f / 8; i += 32 * KS) hs4[i] = __ldcg(hsrc + i);
            for (int i = ltid; i < f / 64; i += 32 * KS) hs4[f / 8 + i] = __ldcg(ssrc + i);
            __syncthreads();
            synced = true;
        }
#pragma unroll
        for (int i = 0; i < GPW; ++i) {
            if (g0 + i < g_end) {
                const int g = g0 + i;
                uint32_t hb[1][8];
                load_b16(gq == 0 ? hs + g * 64 + 16 * c : nullptr, hb[0]);
                const float4 v4 = *reinterpret_cast<const float4 *>(hsum_s + 4 * g);
                const float sx[1][2] = {{c == 0 ? (v4.x + v4.y) + (v4.z + v4.w) : 0.f, 0.f}};
#pragma unroll
                for (int v = 0; v < VW; ++v)
                    if (g >= vb[v] && g < vb[v + 1]) wgroup<FMT, 1>(w[i], b[i], c, hb, sx, C[v]);
            }
        }
    }
    if (!synced) {
        if (wait_h) pdl_wait();
        for (int i = ltid; i < f / 8; i += 32 * KS) hs4[i] = __ldcg(hsrc + i);
        for (int i = ltid; i < f / 64; i += 32 * KS) hs4[f / 8 + i] = __ldcg(ssrc + i);
        __syncthreads();
    }
}

// The KS partial accumulators of one slot (red[w][4][32], warp w's lanes) summed in warp order.
template <int KS>
__device__ __forceinline__ void down_slot_reduce(const float *red, int lane, float (&cs)[1][4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        cs[0][i] = red[i * 32 + lane];
#pragma unroll
        for (int w = 1; w < KS; ++w) cs[0][i] += red[(w * 4 + i) * 32 + lane];
    }
}

// hs4: f bf16 + f/16 floats of shared memory; red: KS * 4 * 32 floats of shared memory.
template <int FMT, int KS, int GPW>
__device__ __forceinline__ void down_slot_unit(const ExpArgs &a, int unit, uint4 *hs4, float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int RB = a.d >> 4;
    const int slot = unit / RB, rb = unit - slot * RB;
    if (a.idx[slot] == SLOT_SKIP) return;
    const TileInfo ti = tile_info(a, slot);
    const size_t blk = (size_t)ti.e * RB + rb;
    float C[1][4];
    down_slot_partial<FMT, KS, GPW>(a, slot, blk, warp, threadIdx.x, hs4, C);
#pragma unroll
    for (int i = 0; i < 4; ++i) red[(warp * 4 + i) * 32 + lane] = C[0][i];
    __syncthreads();
    if (warp == 0) {
        float cs[1][4];
        down_slot_reduce<KS>(red, lane, cs);
        down_store_combine<1>(a, ti, rb, cs, lane);
    }
    __syncthreads();
}

}  // namespace moeb
