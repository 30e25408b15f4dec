// Device helpers shared by the expert kernels (experts.cu, experts_ws.cu).
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace moeb {

struct TileInfo {
    int e, start, n;
};

__device__ __forceinline__ TileInfo tile_info(const ExpArgs &a, int tile) {
    TileInfo ti;
    if (a.tile_mode) {
        const int4 t = a.tiles[tile];
        ti.e = t.x;
        ti.start = t.y;
        ti.n = t.z;
    } else {
        ti.e = a.idx[tile];
        ti.start = tile;
        ti.n = 1;
    }
    if (ti.e < 0 || ti.e >= a.E) ti.e = 0;  // invalid id: computed on expert 0, weighted 0 in the down epilogue
    return ti;
}

__device__ __forceinline__ int tile_slot(const ExpArgs &a, const TileInfo &ti, int col) {
    if (col >= ti.n) return -1;
    return a.tile_mode ? a.sorted[ti.start + col] : ti.start;
}

// A work tile's record {expert, first sorted position, slots}: from the tile list, or slot `tile` alone
__device__ __forceinline__ int4 tile_rec(const ExpArgs &a, int tile) {
    return a.tile_mode ? a.tiles[tile] : make_int4(a.idx[tile], tile, 1, 0);
}
__device__ __forceinline__ TileInfo tile_info_of(const ExpArgs &a, const int4 t) {
    TileInfo ti;
    ti.e = (t.x < 0 || t.x >= a.E) ? 0 : t.x;  // invalid id: computed on expert 0, weighted 0 in the down epilogue
    ti.start = t.y;
    ti.n = t.z;
    return ti;
}

// The epilogue's per-lane metadata (lane 4gq + c owns columns 8j + 2c + hf): slot ids, and the down combine
// weights (0 for an invalid expert id). Loaded early by kernels that can hide the global-load latency.
template <int NT8>
__device__ __forceinline__ void epi_slots(const ExpArgs &a, const TileInfo &ti, int lane, int (&sl)[NT8][2]) {
#pragma unroll
    for (int j = 0; j < NT8; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) sl[j][hf] = tile_slot(a, ti, j * 8 + 2 * (lane & 3) + hf);
}
template <int NT8>
__device__ __forceinline__ void epi_weights(const ExpArgs &a, const int (&sl)[NT8][2], float (&wv)[NT8][2]) {
#pragma unroll
    for (int j = 0; j < NT8; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int s = sl[j][hf];
            if (s >= 0) {
                const int e_raw = a.idx[s];
                const float w = a.wts[s];
                wv[j][hf] = (e_raw >= 0 && e_raw < a.E) ? w : 0.f;
            } else {
                wv[j][hf] = 0.f;
            }
        }
}

// One 64-group of one projection: 4 k-steps x NT8 column tiles into P, then promotion into C.
// w: {row gq: word 2c, 2c+1; row gq+8: word 2c, 2c+1}; sb: {row gq, row gq+8} scale|bias.
template <int NT8>
__device__ __forceinline__ void q4_group(const uint4 w, const uint2 sb, const uint32_t (&xb)[NT8][8],
                                         const float (&sx)[NT8][2], float (&C)[NT8][4]) {
    float P[NT8][4];
#pragma unroll
    for (int j = 0; j < NT8; ++j) P[j][0] = P[j][1] = P[j][2] = P[j][3] = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const uint32_t wa0 = (s < 2) ? w.x : w.y, wa1 = (s < 2) ? w.z : w.w;
        const int p0 = (2 * s) & 3, p1 = (2 * s + 1) & 3;
        const uint32_t A[4] = {q4pair(wa0, p0), q4pair(wa1, p0), q4pair(wa0, p1), q4pair(wa1, p1)};
#pragma unroll
        for (int j = 0; j < NT8; ++j) mma_bf16(P[j], A, xb[j][2 * s], xb[j][2 * s + 1]);
    }
    const float s0 = bf16lo(sb.x), s1 = bf16lo(sb.y);
    const float b0 = __fmaf_rn(-128.f, s0, bf16hi(sb.x)), b1 = __fmaf_rn(-128.f, s1, bf16hi(sb.y));
#pragma unroll
    for (int j = 0; j < NT8; ++j) {
        C[j][0] = __fmaf_rn(s0, P[j][0], __fmaf_rn(b0, sx[j][0], C[j][0]));
        C[j][1] = __fmaf_rn(s0, P[j][1], __fmaf_rn(b0, sx[j][1], C[j][1]));
        C[j][2] = __fmaf_rn(s1, P[j][2], __fmaf_rn(b1, sx[j][0], C[j][2]));
        C[j][3] = __fmaf_rn(s1, P[j][3], __fmaf_rn(b1, sx[j][1], C[j][3]));
    }
}

// ---- MXFP4 (E2M1 codes, E8M0 scale per 32 inputs)
// Each lane's 16 elements of a 64-group (16c .. 16c+15) lie in one 32-element scale block (c / 2), so the scale
// is folded into the A fragment exactly: e2m1 * 2^(S-127) is representable in bf16 for S in 1..254. The MMA
// then accumulates straight into C (no per-group promotion).
// bf16 bytes of the 8 E2M1 magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}: high bytes and low bytes, 4 per register.
constexpr uint32_t FP4_HI0 = 0x3F3F3F00u, FP4_HI1 = 0x40404040u, FP4_LO0 = 0xC0800000u, FP4_LO1 = 0xC0804000u;

// bf16x2 (2^(S-127), 2^(S-127)); S = 0 gives the bf16 subnormal 2^-127.
__device__ __forceinline__ uint32_t fp4_scale2(uint32_t S) {
    const uint32_t b = S ? (S << 7) : 0x40u;
    return b | (b << 16);
}

// The 4 bf16x2 pairs (elements 2p, 2p+1) of one interleaved code word, scaled by scale2.
__device__ __forceinline__ void fp4_word(uint32_t w, uint32_t scale2, uint32_t (&pr)[4]) {
    const uint32_t mag = w & 0x77777777u;
    const uint32_t LA = __byte_perm(FP4_LO0, FP4_LO1, mag), HA = __byte_perm(FP4_HI0, FP4_HI1, mag);
    const uint32_t LB = __byte_perm(FP4_LO0, FP4_LO1, mag >> 16), HB = __byte_perm(FP4_HI0, FP4_HI1, mag >> 16);
    const uint32_t L01 = __byte_perm(LA, LB, 0x5140), H01 = __byte_perm(HA, HB, 0x5140);
    const uint32_t L23 = __byte_perm(LA, LB, 0x7362), H23 = __byte_perm(HA, HB, 0x7362);
    pr[0] = __byte_perm(L01, H01, 0x5140) | ((w << 12) & 0x80008000u);
    pr[1] = __byte_perm(L01, H01, 0x7362) | ((w << 8) & 0x80008000u);
    pr[2] = __byte_perm(L23, H23, 0x5140) | ((w << 4) & 0x80008000u);
    pr[3] = __byte_perm(L23, H23, 0x7362) | (w & 0x80008000u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162 *>(&pr[i]);
        const __nv_bfloat162 s2 = *reinterpret_cast<const __nv_bfloat162 *>(&scale2);
        v = __hmul2(v, s2);
        pr[i] = *reinterpret_cast<uint32_t *>(&v);
    }
}

// One 64-group of an MXFP4 projection: sc4 = E8M0 bytes {row gq half 0, half 1, row gq+8 half 0, half 1}.
template <int NT8>
__device__ __forceinline__ void fp4_group(const uint4 w, const uint32_t sc4, int c, const uint32_t (&xb)[NT8][8],
                                          float (&C)[NT8][4]) {
    const uint32_t s0 = fp4_scale2((sc4 >> (8 * (c >> 1))) & 0xFFu);
    const uint32_t s1 = fp4_scale2((sc4 >> (8 * (2 + (c >> 1)))) & 0xFFu);
    uint32_t r0a[4], r0b[4], r1a[4], r1b[4];
    fp4_word(w.x, s0, r0a);
    fp4_word(w.y, s0, r0b);
    fp4_word(w.z, s1, r1a);
    fp4_word(w.w, s1, r1b);
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const int p0 = (2 * s) & 3, p1 = (2 * s + 1) & 3;
        const uint32_t A[4] = {s < 2 ? r0a[p0] : r0b[p0], s < 2 ? r1a[p0] : r1b[p0], s < 2 ? r0a[p1] : r0b[p1],
                               s < 2 ? r1a[p1] : r1b[p1]};
#pragma unroll
        for (int j = 0; j < NT8; ++j) mma_bf16(C[j], A, xb[j][2 * s], xb[j][2 * s + 1]);
    }
}

__device__ __forceinline__ void load_b16(const uint16_t *p, uint32_t (&o)[8]) {
    if (p) {
        const uint4 u0 = *reinterpret_cast<const uint4 *>(p), u1 = *reinterpret_cast<const uint4 *>(p + 8);
        o[0] = u0.x; o[1] = u0.y; o[2] = u0.z; o[3] = u0.w;
        o[4] = u1.x; o[5] = u1.y; o[6] = u1.z; o[7] = u1.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = 0u;
    }
}

// L2 prefetch of the 16-byte-aligned part of [p, p + bytes), in 4 KB pieces spread over a warp's lanes. The
// range is shrunk inward to 16-byte boundaries, so nothing outside it is touched.
__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes, int lane, int nlanes = 32) {
    const uintptr_t b = ((uintptr_t)p + 15) & ~(uintptr_t)15, e = ((uintptr_t)p + bytes) & ~(uintptr_t)15;
    for (uintptr_t q = b + (uintptr_t)lane * 4096; q < e; q += (uintptr_t)nlanes * 4096) {
        const uint32_t n = (uint32_t)(e - q < 4096 ? e - q : 4096);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(q), "r"(n) : "memory");
    }
}

// Pull the share [rb/RB, (rb+1)/RB) of expert e's down projection into L2 (it streams right after gate/up).
// Called by `nlanes` lanes of a warp (lane in [0, nlanes)).
__device__ __forceinline__ void prefetch_down(const ExpArgs &a, int e, int rb, int RB, int lane, int nlanes = 32) {
    const int rb0 = (int)((long)rb * (a.d / 16) / RB), rb1 = (int)((long)(rb + 1) * (a.d / 16) / RB);
    if (rb1 <= rb0) return;
    const size_t blk = (size_t)e * (a.d / 16) + rb0;
    prefetch_l2(a.dn.q + blk * (size_t)(a.f / 64) * 128, (size_t)(rb1 - rb0) * (a.f / 64) * 512, lane, nlanes);
    // scale words: int4 16 uint32 per (row block, group), MXFP4 8 (32 bytes of E8M0)
    const int spg = a.fmt == FMT_FP4 ? 8 : 16;
    prefetch_l2(a.dn.sb + blk * (size_t)(a.f / 64) * spg, (size_t)(rb1 - rb0) * (a.f / 64) * spg * 4, lane, nlanes);
}

// Weights of one (16-row block, 64-group) for this lane.
__device__ __forceinline__ uint4 ld_w(const QProj &P, size_t blk, int G, int g, int lane) {
    return ld_stream_u4(P.q + ((blk * G + g) * 32 + lane) * 4);
}
__device__ __forceinline__ uint2 ld_sb(const QProj &P, size_t blk, int G, int g, int gq) {
    return ld_stream_u2(P.sb + ((blk * G + g) * 8 + gq) * 2);
}
// Per-lane scale words of one (row block, group): int4 -> {scale|bias row gq, row gq+8}; MXFP4 -> the 4 E8M0
// bytes of rows gq, gq+8 in .x (.y unused).
template <int FMT>
__device__ __forceinline__ uint2 ld_scales(const QProj &P, size_t blk, int G, int g, int gq) {
    if (FMT == FMT_FP4) return make_uint2(ld_stream_u32(P.sb + (blk * G + g) * 8 + gq), 0u);
    return ld_sb(P, blk, G, g, gq);
}
// One group of either format into C (int4 uses the group sums sx; MXFP4 ignores them).
template <int FMT, int NT8>
__device__ __forceinline__ void wgroup(const uint4 w, const uint2 sc, int c, const uint32_t (&xb)[NT8][8],
                                       const float (&sx)[NT8][2], float (&C)[NT8][4]) {
    if (FMT == FMT_FP4) fp4_group<NT8>(w, sc.x, c, xb, C);
    else q4_group<NT8>(w, sc, xb, sx, C);
}

// gate/up epilogue for one column tile j of a unit: bias, activation, bf16 h, block sums.
// slot_of(hf): the slot of this lane's column hf, or -1.
template <class SlotOf>
__device__ __forceinline__ void gate_up_store_impl(const ExpArgs &a, const TileInfo &ti, int rb, const float (&gs)[4],
                                                   const float (&us)[4], int lane, SlotOf slot_of) {
    const int gq = lane >> 2, f = a.f;
    const int r0 = rb * 16 + gq, r1 = r0 + 8;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        const int slot = slot_of(hf);
        float g0v = gs[hf], g1v = gs[2 + hf], u0v = us[hf], u1v = us[2 + hf];
        if (a.bg) {
            g0v += a.bg[(size_t)ti.e * f + r0];
            g1v += a.bg[(size_t)ti.e * f + r1];
            u0v += a.bu[(size_t)ti.e * f + r0];
            u1v += a.bu[(size_t)ti.e * f + r1];
        }
        const uint16_t h0 = f2bf(act_glu(a.act, g0v, u0v)), h1 = f2bf(act_glu(a.act, g1v, u1v));
        float part = slot >= 0 ? bf2f(h0) + bf2f(h1) : 0.f;
        part += __shfl_xor_sync(0xffffffffu, part, 4);
        part += __shfl_xor_sync(0xffffffffu, part, 8);
        part += __shfl_xor_sync(0xffffffffu, part, 16);
        if (slot >= 0) {
            a.h[(size_t)slot * f + r0] = h0;
            a.h[(size_t)slot * f + r1] = h1;
            if (gq == 0) a.hsum[(size_t)slot * (f / 16) + rb] = part;
        }
    }
}
template <int NT8>
__device__ __forceinline__ void gate_up_store(const ExpArgs &a, const TileInfo &ti, int rb, int j,
                                              const float (&gs)[4], const float (&us)[4], int lane) {
    gate_up_store_impl(a, ti, rb, gs, us, lane, [&](int hf) { return tile_slot(a, ti, j * 8 + 2 * (lane & 3) + hf); });
}
// the same with the slot ids loaded ahead (epi_slots)
__device__ __forceinline__ void gate_up_store_sl(const ExpArgs &a, const TileInfo &ti, int rb, const int (&sl)[2],
                                                 const float (&gs)[4], const float (&us)[4], int lane) {
    gate_up_store_impl(a, ti, rb, gs, us, lane, [&](int hf) { return sl[hf]; });
}

// down epilogue of one warp: write the weighted per-slot rows, arrive on the (token, row block) counters and
// combine every token this arrival completed. Warp-synchronous; no CTA barrier.
// slot_of(j, hf): the slot of this lane's column 8j + 2c + hf, or -1; weight_of(j, hf, slot): its combine weight.
template <int NT8, class SlotOf, class WeightOf>
__device__ __forceinline__ void down_store_combine_impl(const ExpArgs &a, const TileInfo &ti, int rb,
                                                        const float (&C)[NT8][4], int lane, SlotOf slot_of,
                                                        WeightOf weight_of) {
    const int gq = lane >> 2, d = a.d, k = a.k, RB = d >> 4;
    const int r0 = rb * 16 + gq, r1 = r0 + 8;
#pragma unroll
    for (int j = 0; j < NT8; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int slot = slot_of(j, hf);
            if (slot >= 0) {
                const float wsl = weight_of(j, hf, slot);
                float v0 = C[j][hf], v1 = C[j][2 + hf];
                if (a.bd) {
                    v0 += a.bd[(size_t)ti.e * d + r0];
                    v1 += a.bd[(size_t)ti.e * d + r1];
                }
                float *yrow = a.ypeers ? reinterpret_cast<float *>(a.ypeers[slot / a.C] + a.yoff) +
                                             ((size_t)a.me * a.C + slot % a.C) * d
                                       : a.yp + (size_t)slot * d;
                yrow[r0] = wsl * v0;
                yrow[r1] = wsl * v1;
            }
        }
    if (a.slot_out) {  // expert-parallel or separate combine pass: the rows are combined later
        if (a.ypeers && NT8 == 1 && !a.tile_mode) {  // decode kernels: peers' rows visible before the kernel ends
            __syncwarp();
            if (lane == 0) __threadfence_system();
        }
        return;
    }
    __syncwarp();
    if (lane == 0) __threadfence();  // cumulative over the warp's writes ordered by the __syncwarp
    __syncwarp();
    int tok = -1;
    bool done = false;
    if (lane < 8 * NT8) {
        const int slot = tile_slot(a, ti, lane);
        if (slot >= 0) {
            tok = slot / k;
            done = atomicAdd(a.ycnt + (size_t)tok * RB + rb, 1u) == (unsigned)(k - 1);
        }
    }
    unsigned m = __ballot_sync(0xffffffffu, done);
    if (m) {
        if (lane == 0) __threadfence();
        __syncwarp();
    }
    while (m) {
        const int src = __ffs(m) - 1;
        m &= m - 1;
        const int t = __shfl_sync(0xffffffffu, tok, src);
        if (lane < 16) {
            const int r = rb * 16 + lane;
            float acc = 0.f;
            for (int jj = 0; jj < k; ++jj) acc += __ldcg(a.yp + ((size_t)t * k + jj) * d + r);
            if (a.residual) acc += bf2f(a.residual[(size_t)t * d + r]);
            a.y[(size_t)t * d + r] = f2bf(acc);
        }
        if (lane == 0) a.ycnt[(size_t)t * RB + rb] = 0u;
    }
}

template <int NT8>
__device__ __forceinline__ void down_store_combine(const ExpArgs &a, const TileInfo &ti, int rb,
                                                   const float (&C)[NT8][4], int lane) {
    down_store_combine_impl<NT8>(
        a, ti, rb, C, lane, [&](int j, int hf) { return tile_slot(a, ti, j * 8 + 2 * (lane & 3) + hf); },
        [&](int, int, int slot) {
            const int e_raw = a.idx[slot];
            return (e_raw >= 0 && e_raw < a.E) ? a.wts[slot] : 0.f;
        });
}
// the same with the slot ids and weights loaded ahead (epi_slots, epi_weights)
template <int NT8>
__device__ __forceinline__ void down_store_combine_sl(const ExpArgs &a, const TileInfo &ti, int rb,
                                                      const float (&C)[NT8][4], int lane, const int (&sl)[NT8][2],
                                                      const float (&wv)[NT8][2]) {
    down_store_combine_impl<NT8>(
        a, ti, rb, C, lane, [&](int j, int hf) { return sl[j][hf]; }, [&](int j, int hf, int) { return wv[j][hf]; });
}

}  // namespace moeb
