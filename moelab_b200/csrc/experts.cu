// Grouped expert kernels, warp-MMA path (all loads; the HBM-bound regime).
//
// Work unit = (tile, 16-row block). A tile is up to 8 * NT8 slots routed to one expert (tile mode, built by
// the routing step) or exactly one slot (slot mode, T*k small). The CTA's KS warps split K; each warp runs
// m16n8k16 bf16 MMAs with
//   A = 16 weight rows x 16 k, the raw int4 codes as exact bf16 (128 + q, one lop3 per two codes), loaded
//       straight from HBM into the MMA fragment (8 bytes per row per 64-group per thread);
//   B = the tile's activations (x rows for gate/up, h rows for down), 16 contiguous elements per thread;
// and promotes every 64-wide scale group in fp32: C += s * P + (b - 128 s) * sum(x_group)
// (the same algebra as the reference's raw-code MMA, metal_q4_tiles_v2.py:255-262), so the result equals the
// dot product with the fp32-dequantised weights w = s*q + b up to fp32 rounding.
//
// K permutation: inside each 64-group, MMA k-step s / fragment half hf / lane-in-quad c address the physical
// elements 16c + 4s + 2hf + {0,1}, for A and B alike (a bijection of the group), so every thread reads 16
// contiguous activations and two contiguous 32-bit code words per row.
//
// gate/up (reference GATE_UP_SRC metal_q4_decode_v4.py:67-93, GATE_UP_E_SRC metal_q4_tiles_v2.py:179-275):
//   h[slot][r] = bf16(act(g + bg, u + bu)), plus hsum[slot][r/16] = sum of the 16 bf16 h values of the block
// down + combine (DOWN_SRC metal_q4_decode_v4.py:95-144, DOWN_E_SRC + COMBINE_SRC metal_q4_tiles_v2.py):
//   yp[slot][r] = w_slot * (Wd h + bd), then the last CTA to finish a (token, 16-row block) sums the k slots
//   in fixed slot order j = 0..k-1 (deterministic, no float atomics), adds the optional residual, writes y.
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

// One 64-group of one projection: 4 k-steps x NT8 column tiles into P (zeroed here), then promotion into C.
template <int NT8>
__device__ __forceinline__ void q4_group(const uint2 w0, const uint2 w1, const uint32_t sb0, const uint32_t sb1,
                                         const uint32_t (&xb)[NT8][8], const float (&sx)[NT8][2],
                                         float (&C)[NT8][4]) {
    float P[NT8][4];
#pragma unroll
    for (int j = 0; j < NT8; ++j) P[j][0] = P[j][1] = P[j][2] = P[j][3] = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        // pair index i = 2s + hf -> word (i / 4) of the row's two words, nibble pair i % 4
        const uint32_t wa0 = (s < 2) ? w0.x : w0.y, wa1 = (s < 2) ? w1.x : w1.y;
        const int p0 = (2 * s) & 3, p1 = (2 * s + 1) & 3;
        const uint32_t A[4] = {q4pair(wa0, p0), q4pair(wa1, p0), q4pair(wa0, p1), q4pair(wa1, p1)};
#pragma unroll
        for (int j = 0; j < NT8; ++j) mma_bf16(P[j], A, xb[j][2 * s], xb[j][2 * s + 1]);
    }
    const float s0 = bf16lo(sb0), s1 = bf16lo(sb1);
    const float b0 = __fmaf_rn(-128.f, s0, bf16hi(sb0)), b1 = __fmaf_rn(-128.f, s1, bf16hi(sb1));
#pragma unroll
    for (int j = 0; j < NT8; ++j) {
        C[j][0] = __fmaf_rn(s0, P[j][0], __fmaf_rn(b0, sx[j][0], C[j][0]));
        C[j][1] = __fmaf_rn(s0, P[j][1], __fmaf_rn(b0, sx[j][1], C[j][1]));
        C[j][2] = __fmaf_rn(s1, P[j][2], __fmaf_rn(b1, sx[j][0], C[j][2]));
        C[j][3] = __fmaf_rn(s1, P[j][3], __fmaf_rn(b1, sx[j][1], C[j][3]));
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
__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes, int lane) {
    const uintptr_t b = ((uintptr_t)p + 15) & ~(uintptr_t)15, e = ((uintptr_t)p + bytes) & ~(uintptr_t)15;
    for (uintptr_t q = b + (uintptr_t)lane * 4096; q < e; q += 32 * 4096) {
        const uint32_t n = (uint32_t)(e - q < 4096 ? e - q : 4096);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(q), "r"(n) : "memory");
    }
}

// ------------------------------------------------------------------ gate/up
// GPW = 64-groups per warp per batch: all loads of a batch (codes, scale|bias, activations, group sums) are
// issued before the first MMA, so one warp keeps GPW * 56 bytes per lane in flight.
template <int FMT, int NT8, int KS, int GPW>
__global__ void __launch_bounds__(32 * KS, 2) k_gate_up(ExpArgs a) {
    pdl_launch();
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gq = lane >> 2, c = lane & 3;
    const int d = a.d, f = a.f;
    const int RB = f >> 4, G = d >> 6;
    const int n_tiles = a.tile_mode ? *a.ntiles : a.T * a.k;
    const int g_beg = warp * G / KS, g_end = (warp + 1) * G / KS;
    __shared__ float red[KS][2][NT8][4][32];
    for (int unit = blockIdx.x; unit < n_tiles * RB; unit += gridDim.x) {
        const int tile = unit / RB, rb = unit - tile * RB;
        const TileInfo ti = tile_info(a, tile);
        // the down projection of this expert streams next: pull this unit's share of it into L2 now
        if (warp == KS - 1 && a.dn_prefetch) {
            const int r0 = (int)((long)rb * d / RB), r1 = (int)((long)(rb + 1) * d / RB);
            const size_t row = (size_t)ti.e * d + r0;
            prefetch_l2(a.dn.q + row * (f / 8), (size_t)(r1 - r0) * (f / 2), lane);
            prefetch_l2(a.dn.sb + row * (f / 64), (size_t)(r1 - r0) * (f / 16), lane);
        }
        const uint16_t *xrow[NT8];
        const float *sxrow[NT8][2];
#pragma unroll
        for (int j = 0; j < NT8; ++j) {
            const int sb_ = tile_slot(a, ti, j * 8 + gq);
            xrow[j] = sb_ >= 0 ? a.x + (size_t)(sb_ / a.k) * d + 16 * c : nullptr;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int sc_ = tile_slot(a, ti, j * 8 + 2 * c + hf);
                sxrow[j][hf] = sc_ >= 0 ? a.xsum + (size_t)(sc_ / a.k) * G : nullptr;
            }
        }
        const size_t row0 = (size_t)ti.e * f + rb * 16 + gq;
        const uint32_t *qg0 = a.g.q + row0 * (d / 8) + 2 * c, *qg1 = qg0 + 8 * (size_t)(d / 8);
        const uint32_t *qu0 = a.u.q + row0 * (d / 8) + 2 * c, *qu1 = qu0 + 8 * (size_t)(d / 8);
        const uint32_t *sg0 = a.g.sb + row0 * G, *sg1 = sg0 + 8 * (size_t)G;
        const uint32_t *su0 = a.u.sb + row0 * G, *su1 = su0 + 8 * (size_t)G;
        float Cg[NT8][4], Cu[NT8][4];
#pragma unroll
        for (int j = 0; j < NT8; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) Cg[j][i] = Cu[j][i] = 0.f;
        for (int g0 = g_beg; g0 < g_end; g0 += GPW) {
            uint2 wg0[GPW], wg1[GPW], wu0[GPW], wu1[GPW];
            uint32_t bg0[GPW], bg1[GPW], bu0[GPW], bu1[GPW];
            uint32_t xb[GPW][NT8][8];
            float sx[GPW][NT8][2];
#pragma unroll
            for (int i = 0; i < GPW; ++i) {
                const int g = min(g0 + i, g_end - 1);  // clamped: a repeated load, never used
                wg0[i] = ld_stream_u2(qg0 + g * 8);
                wg1[i] = ld_stream_u2(qg1 + g * 8);
                wu0[i] = ld_stream_u2(qu0 + g * 8);
                wu1[i] = ld_stream_u2(qu1 + g * 8);
                bg0[i] = ld_stream_u32(sg0 + g);
                bg1[i] = ld_stream_u32(sg1 + g);
                bu0[i] = ld_stream_u32(su0 + g);
                bu1[i] = ld_stream_u32(su1 + g);
#pragma unroll
                for (int j = 0; j < NT8; ++j) {
                    load_b16(xrow[j] ? xrow[j] + g * 64 : nullptr, xb[i][j]);
                    sx[i][j][0] = sxrow[j][0] ? sxrow[j][0][g] : 0.f;
                    sx[i][j][1] = sxrow[j][1] ? sxrow[j][1][g] : 0.f;
                }
            }
#pragma unroll
            for (int i = 0; i < GPW; ++i) {
                if (g0 + i < g_end) {
                    q4_group<NT8>(wg0[i], wg1[i], bg0[i], bg1[i], xb[i], sx[i], Cg);
                    q4_group<NT8>(wu0[i], wu1[i], bu0[i], bu1[i], xb[i], sx[i], Cu);
                }
            }
        }
        // split-K reduction in fixed warp order
#pragma unroll
        for (int j = 0; j < NT8; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                red[warp][0][j][i][lane] = Cg[j][i];
                red[warp][1][j][i][lane] = Cu[j][i];
            }
        __syncthreads();
        if (warp == 0) {
#pragma unroll
            for (int j = 0; j < NT8; ++j) {
                float gs[4], us[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    gs[i] = red[0][0][j][i][lane];
                    us[i] = red[0][1][j][i][lane];
#pragma unroll
                    for (int w = 1; w < KS; ++w) {
                        gs[i] += red[w][0][j][i][lane];
                        us[i] += red[w][1][j][i][lane];
                    }
                }
                const int r0 = rb * 16 + gq, r1 = r0 + 8;
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int slot = tile_slot(a, ti, j * 8 + 2 * c + hf);
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
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------ down + combine
template <int FMT, int NT8, int KS, int GPW>
__global__ void __launch_bounds__(32 * KS, 4) k_down(ExpArgs a) {
    pdl_launch();
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gq = lane >> 2, c = lane & 3;
    const int d = a.d, f = a.f, k = a.k;
    const int RB = d >> 4, G = f >> 6;
    const int n_tiles = a.tile_mode ? *a.ntiles : a.T * a.k;
    const int g_beg = warp * G / KS, g_end = (warp + 1) * G / KS;
    __shared__ float red[KS][NT8][4][32];
    __shared__ int s_done[8 * NT8];
    __shared__ int s_ndone;
    for (int unit = blockIdx.x; unit < n_tiles * RB; unit += gridDim.x) {
        const int tile = unit / RB, rb = unit - tile * RB;
        const TileInfo ti = tile_info(a, tile);
        const uint16_t *hrow[NT8];
        const float *hsrow[NT8][2];
#pragma unroll
        for (int j = 0; j < NT8; ++j) {
            const int sb_ = tile_slot(a, ti, j * 8 + gq);
            hrow[j] = sb_ >= 0 ? a.h + (size_t)sb_ * f + 16 * c : nullptr;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int sc_ = tile_slot(a, ti, j * 8 + 2 * c + hf);
                hsrow[j][hf] = sc_ >= 0 ? a.hsum + (size_t)sc_ * (f / 16) : nullptr;
            }
        }
        const size_t row0 = (size_t)ti.e * d + rb * 16 + gq;
        const uint32_t *qd0 = a.dn.q + row0 * (f / 8) + 2 * c, *qd1 = qd0 + 8 * (size_t)(f / 8);
        const uint32_t *sd0 = a.dn.sb + row0 * G, *sd1 = sd0 + 8 * (size_t)G;
        float C[NT8][4];
#pragma unroll
        for (int j = 0; j < NT8; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) C[j][i] = 0.f;
        for (int g0 = g_beg; g0 < g_end; g0 += GPW) {
            uint2 w0[GPW], w1[GPW];
            uint32_t b0[GPW], b1[GPW];
            uint32_t hb[GPW][NT8][8];
            float4 hs[GPW][NT8][2];
#pragma unroll
            for (int i = 0; i < GPW; ++i) {
                const int g = min(g0 + i, g_end - 1);
                w0[i] = ld_stream_u2(qd0 + g * 8);
                w1[i] = ld_stream_u2(qd1 + g * 8);
                b0[i] = ld_stream_u32(sd0 + g);
                b1[i] = ld_stream_u32(sd1 + g);
#pragma unroll
                for (int j = 0; j < NT8; ++j) {
                    load_b16(hrow[j] ? hrow[j] + g * 64 : nullptr, hb[i][j]);
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf)
                        hs[i][j][hf] = hsrow[j][hf] ? *reinterpret_cast<const float4 *>(hsrow[j][hf] + 4 * g)
                                                    : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int i = 0; i < GPW; ++i) {
                if (g0 + i < g_end) {
                    float sx[NT8][2];
#pragma unroll
                    for (int j = 0; j < NT8; ++j)
#pragma unroll
                        for (int hf = 0; hf < 2; ++hf) {
                            const float4 v = hs[i][j][hf];
                            sx[j][hf] = (v.x + v.y) + (v.z + v.w);
                        }
                    q4_group<NT8>(w0[i], w1[i], b0[i], b1[i], hb[i], sx, C);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < NT8; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) red[warp][j][i][lane] = C[j][i];
        if (threadIdx.x == 0) s_ndone = 0;
        __syncthreads();
        if (warp == 0) {
            const int r0 = rb * 16 + gq, r1 = r0 + 8;
#pragma unroll
            for (int j = 0; j < NT8; ++j) {
                float cs[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    cs[i] = red[0][j][i][lane];
#pragma unroll
                    for (int w = 1; w < KS; ++w) cs[i] += red[w][j][i][lane];
                }
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int slot = tile_slot(a, ti, j * 8 + 2 * c + hf);
                    if (slot >= 0) {
                        const int e_raw = a.idx[slot];
                        const float wsl = (e_raw >= 0 && e_raw < a.E) ? a.wts[slot] : 0.f;
                        float v0 = cs[hf], v1 = cs[2 + hf];
                        if (a.bd) {
                            v0 += a.bd[(size_t)ti.e * d + r0];
                            v1 += a.bd[(size_t)ti.e * d + r1];
                        }
                        a.yp[(size_t)slot * d + r0] = wsl * v0;
                        a.yp[(size_t)slot * d + r1] = wsl * v1;
                    }
                }
            }
            __threadfence();
        }
        __syncthreads();
        // one arrival per slot column on its (token, row block) counter; the last arrival combines
        if (threadIdx.x < 8 * NT8) {
            const int slot = tile_slot(a, ti, threadIdx.x);
            if (slot >= 0) {
                const int t = slot / k;
                const unsigned prev = atomicAdd(a.ycnt + (size_t)t * RB + rb, 1u);
                if (prev == (unsigned)(k - 1)) s_done[atomicAdd(&s_ndone, 1)] = t;
            }
        }
        __syncthreads();
        const int nd = s_ndone;
        if (nd > 0) {
            __threadfence();
            for (int m = warp; m < nd; m += KS) {
                const int t = s_done[m];
                if (lane < 16) {
                    const int r = rb * 16 + lane;
                    float acc = 0.f;
                    for (int j = 0; j < k; ++j) acc += __ldcg(a.yp + ((size_t)t * k + j) * d + r);
                    if (a.residual) acc += bf2f(a.residual[(size_t)t * d + r]);
                    a.y[(size_t)t * d + r] = f2bf(acc);
                }
                if (lane == 0) a.ycnt[(size_t)t * RB + rb] = 0u;
            }
        }
        __syncthreads();
    }
}

template __global__ void k_gate_up<FMT_Q4, 1, 8, 4>(ExpArgs);
template __global__ void k_gate_up<FMT_Q4, 2, 8, 2>(ExpArgs);
template __global__ void k_down<FMT_Q4, 1, 4, 4>(ExpArgs);
template __global__ void k_down<FMT_Q4, 2, 4, 2>(ExpArgs);

}  // namespace moeb
