// Grouped expert kernels, warp-MMA path (the HBM-bound regime).
//
// Math. m16n8k16 bf16 MMAs with
//   A = 16 weight rows x 16 k: the raw int4 codes as exact bf16 (128 + q, one lop3 per two codes), read from the
//       fragment-major weight layout (quant.cu) with one coalesced 16-byte load per lane per 64-group;
//   B = the activations (x rows for gate/up, h rows for down), 16 contiguous elements per lane per group;
// and every 64-wide scale group is promoted in fp32: C += s * P + (b - 128 s) * sum(x_group), the algebra of the
// reference's raw-code MMA (metal_q4_tiles_v2.py:255-262), so the result is the dot product with the
// fp32-dequantised weights w = s*q + b up to fp32 rounding.
// K permutation: inside a 64-group, MMA k-step s / fragment half hf / lane-in-quad c address the physical
// elements 16c + 4s + 2hf + {0,1}, for A and B alike (a bijection of the group).
//
// Two launch shapes over work units (tile, 16-row block):
//   *_slots (decode, one slot per tile): one CTA per unit, the KS warps split K with every load issued up
//     front, the token's activation row staged in shared memory, fixed-order split-K reduction.
//   *_tiles (slots grouped by expert into tiles of 8*NT8): one warp per unit over the whole K, a register
//     double-buffered load pipeline, and a per-warp epilogue (no CTA barriers).
// gate/up (reference GATE_UP_SRC metal_q4_decode_v4.py:67-93, GATE_UP_E_SRC metal_q4_tiles_v2.py:179-275):
//   h[slot][r] = bf16(act(g + bg, u + bu)); hsum[slot][r/16] = sum of the block's 16 bf16 h values.
// down + combine (DOWN_SRC metal_q4_decode_v4.py:95-144, DOWN_E_SRC + COMBINE_SRC metal_q4_tiles_v2.py):
//   yp[slot][r] = w_slot * (Wd h + bd); the last unit to finish a (token, 16-row block) sums its k slots in
//   fixed order j = 0..k-1 (deterministic, no float atomics), adds the optional residual and writes y.
#include "experts_common.cuh"

namespace moeb {

// ================================================================== slot mode (decode)
// One CTA per (slot, 16-row block); KS warps split the K groups; GPW groups per warp are loaded at once.
template <int FMT, int KS, int GPW>
__global__ void __launch_bounds__(32 * KS, 3) k_gate_up_slots(ExpArgs a) {
    pdl_launch();
    pdl_wait();
    extern __shared__ uint4 xs4[];  // the slot's x row, d bf16
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gq = lane >> 2, c = lane & 3;
    const int d = a.d, f = a.f;
    const int RB = f >> 4, G = d >> 6;
    const int g_beg = warp * G / KS, g_end = (warp + 1) * G / KS;
    __shared__ float red[KS][2][4][32];
    const uint16_t *xs = reinterpret_cast<const uint16_t *>(xs4);
    for (int unit = blockIdx.x; unit < a.T * a.k * RB; unit += gridDim.x) {
        const int slot = unit / RB, rb = unit - slot * RB;
        const TileInfo ti = tile_info(a, slot);
        const size_t blk = (size_t)ti.e * RB + rb;
        if (warp == KS - 1 && a.dn_prefetch) prefetch_down(a, ti.e, rb, RB, lane);
        const uint4 *xsrc = reinterpret_cast<const uint4 *>(a.x + (size_t)(slot / a.k) * d);
        for (int i = threadIdx.x; i < d / 8; i += 32 * KS) xs4[i] = xsrc[i];
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
                bg[i] = ld_sb(a.g, blk, G, g, gq);
                bu[i] = ld_sb(a.u, blk, G, g, gq);
            }
            if (!synced) {
                __syncthreads();  // x row staged (weights already in flight)
                synced = true;
            }
#pragma unroll
            for (int i = 0; i < GPW; ++i) {
                if (g0 + i < g_end) {
                    const int g = g0 + i;
                    uint32_t xb[1][8];
                    load_b16(gq == 0 ? xs + g * 64 + 16 * c : nullptr, xb[0]);
                    const float sx[1][2] = {{c == 0 ? sxr[g] : 0.f, 0.f}};
                    q4_group<1>(wg[i], bg[i], xb, sx, Cg);
                    q4_group<1>(wu[i], bu[i], xb, sx, Cu);
                }
            }
        }
        if (!synced) __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            red[warp][0][i][lane] = Cg[0][i];
            red[warp][1][i][lane] = Cu[0][i];
        }
        __syncthreads();
        if (warp == 0) {
            float gs[4], us[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                gs[i] = red[0][0][i][lane];
                us[i] = red[0][1][i][lane];
#pragma unroll
                for (int w = 1; w < KS; ++w) {
                    gs[i] += red[w][0][i][lane];
                    us[i] += red[w][1][i][lane];
                }
            }
            gate_up_store<1>(a, ti, rb, 0, gs, us, lane);
        }
        __syncthreads();
    }
}

template <int FMT, int KS, int GPW>
__global__ void __launch_bounds__(32 * KS, 8) k_down_slots(ExpArgs a) {
    pdl_launch();
    pdl_wait();
    extern __shared__ uint4 hs4[];  // the slot's h row (f bf16) followed by its f/16 block sums
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gq = lane >> 2, c = lane & 3;
    const int d = a.d, f = a.f;
    const int RB = d >> 4, G = f >> 6;
    const int g_beg = warp * G / KS, g_end = (warp + 1) * G / KS;
    __shared__ float red[KS][4][32];
    const uint16_t *hs = reinterpret_cast<const uint16_t *>(hs4);
    const float *hsum_s = reinterpret_cast<const float *>(hs4 + f / 8);
    for (int unit = blockIdx.x; unit < a.T * a.k * RB; unit += gridDim.x) {
        const int slot = unit / RB, rb = unit - slot * RB;
        const TileInfo ti = tile_info(a, slot);
        const size_t blk = (size_t)ti.e * RB + rb;
        const uint4 *hsrc = reinterpret_cast<const uint4 *>(a.h + (size_t)slot * f);
        for (int i = threadIdx.x; i < f / 8; i += 32 * KS) hs4[i] = hsrc[i];
        const uint4 *ssrc = reinterpret_cast<const uint4 *>(a.hsum + (size_t)slot * (f / 16));
        for (int i = threadIdx.x; i < f / 64; i += 32 * KS) hs4[f / 8 + i] = ssrc[i];
        float C[1][4] = {{0.f, 0.f, 0.f, 0.f}};
        bool synced = false;
        for (int g0 = g_beg; g0 < g_end; g0 += GPW) {
            uint4 w[GPW];
            uint2 b[GPW];
#pragma unroll
            for (int i = 0; i < GPW; ++i) {
                const int g = min(g0 + i, g_end - 1);
                w[i] = ld_w(a.dn, blk, G, g, lane);
                b[i] = ld_sb(a.dn, blk, G, g, gq);
            }
            if (!synced) {
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
                    q4_group<1>(w[i], b[i], hb, sx, C);
                }
            }
        }
        if (!synced) __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; ++i) red[warp][i][lane] = C[0][i];
        __syncthreads();
        if (warp == 0) {
            float cs[1][4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                cs[0][i] = red[0][i][lane];
#pragma unroll
                for (int w = 1; w < KS; ++w) cs[0][i] += red[w][i][lane];
            }
            down_store_combine<1>(a, ti, rb, cs, lane);
        }
        __syncthreads();
    }
}

// ================================================================== tile mode, register pipeline
// One warp per (tile, 16-row block) over the whole K; loads run one GPW-group batch ahead of the MMAs in
// registers (no shared memory), so more warps fit per SM than with the cp.async ring below.
template <int NT8, int GPW>
struct GUBatch {
    uint4 wg[GPW], wu[GPW];
    uint2 bg[GPW], bu[GPW];
    uint32_t xb[GPW][NT8][8];
    float sx[GPW][NT8][2];
};

template <int NT8, int GPW>
__device__ __forceinline__ void gu_load(GUBatch<NT8, GPW> &B, const ExpArgs &a, size_t blk, int G, int g0,
                                        const uint16_t *const (&xrow)[NT8], const float *const (&sxrow)[NT8][2],
                                        int lane) {
    const int gq = lane >> 2;
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
        const int g = min(g0 + i, G - 1);
        B.wg[i] = ld_w(a.g, blk, G, g, lane);
        B.wu[i] = ld_w(a.u, blk, G, g, lane);
        B.bg[i] = ld_sb(a.g, blk, G, g, gq);
        B.bu[i] = ld_sb(a.u, blk, G, g, gq);
#pragma unroll
        for (int j = 0; j < NT8; ++j) {
            load_b16(xrow[j] ? xrow[j] + g * 64 : nullptr, B.xb[i][j]);
            B.sx[i][j][0] = sxrow[j][0] ? sxrow[j][0][g] : 0.f;
            B.sx[i][j][1] = sxrow[j][1] ? sxrow[j][1][g] : 0.f;
        }
    }
}

template <int NT8, int GPW>
__device__ __forceinline__ void gu_compute(const GUBatch<NT8, GPW> &B, int g0, int G, float (&Cg)[NT8][4],
                                           float (&Cu)[NT8][4]) {
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
        if (g0 + i < G) {
            q4_group<NT8>(B.wg[i], B.bg[i], B.xb[i], B.sx[i], Cg);
            q4_group<NT8>(B.wu[i], B.bu[i], B.xb[i], B.sx[i], Cu);
        }
    }
}

template <int FMT, int NT8, int GPW>
__global__ void __launch_bounds__(128) k_gate_up_tiles_reg(ExpArgs a) {
    pdl_launch();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int gq = lane >> 2, c = lane & 3;
    const int d = a.d, f = a.f;
    const int RB = f >> 4, G = d >> 6;
    const int n_units = *a.ntiles * RB;
    const int nwarps = gridDim.x * 4;
    for (int unit = blockIdx.x * 4 + (threadIdx.x >> 5); unit < n_units; unit += nwarps) {
        const int tile = unit / RB, rb = unit - tile * RB;
        const TileInfo ti = tile_info(a, tile);
        const size_t blk = (size_t)ti.e * RB + rb;
        if (a.dn_prefetch) prefetch_down(a, ti.e, rb, RB, lane);
        const uint16_t *xrow[NT8];
        const float *sxrow[NT8][2];
#pragma unroll
        for (int j = 0; j < NT8; ++j) {
            const int sb_ = tile_slot(a, ti, j * 8 + gq);
            xrow[j] = sb_ >= 0 ? a.x + (size_t)(sb_ / a.k) * d + 16 * c : nullptr;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int sc_ = tile_slot(a, ti, j * 8 + 2 * c + hf);
                sxrow[j][hf] = sc_ >= 0 ? a.xsum + (size_t)(sc_ / a.k) * xsum_stride(d) : nullptr;
            }
        }
        float Cg[NT8][4], Cu[NT8][4];
#pragma unroll
        for (int j = 0; j < NT8; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) Cg[j][i] = Cu[j][i] = 0.f;
        GUBatch<NT8, GPW> A, B;
        gu_load(A, a, blk, G, 0, xrow, sxrow, lane);
        for (int g0 = 0; g0 < G; g0 += 2 * GPW) {
            if (g0 + GPW < G) gu_load(B, a, blk, G, g0 + GPW, xrow, sxrow, lane);
            gu_compute(A, g0, G, Cg, Cu);
            if (g0 + GPW < G) {
                if (g0 + 2 * GPW < G) gu_load(A, a, blk, G, g0 + 2 * GPW, xrow, sxrow, lane);
                gu_compute(B, g0 + GPW, G, Cg, Cu);
            }
        }
#pragma unroll
        for (int j = 0; j < NT8; ++j) gate_up_store<NT8>(a, ti, rb, j, Cg[j], Cu[j], lane);
    }
}

template <int NT8, int GPW>
struct DNBatch {
    uint4 w[GPW];
    uint2 b[GPW];
    uint32_t hb[GPW][NT8][8];
    float4 hs[GPW][NT8][2];
};

template <int NT8, int GPW>
__device__ __forceinline__ void dn_load(DNBatch<NT8, GPW> &B, const ExpArgs &a, size_t blk, int G, int g0,
                                        const uint16_t *const (&hrow)[NT8], const float *const (&hsrow)[NT8][2],
                                        int lane) {
    const int gq = lane >> 2;
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
        const int g = min(g0 + i, G - 1);
        B.w[i] = ld_w(a.dn, blk, G, g, lane);
        B.b[i] = ld_sb(a.dn, blk, G, g, gq);
#pragma unroll
        for (int j = 0; j < NT8; ++j) {
            load_b16(hrow[j] ? hrow[j] + g * 64 : nullptr, B.hb[i][j]);
#pragma unroll
            for (int hf = 0; hf < 2; ++hf)
                B.hs[i][j][hf] = hsrow[j][hf] ? *reinterpret_cast<const float4 *>(hsrow[j][hf] + 4 * g)
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

template <int NT8, int GPW>
__device__ __forceinline__ void dn_compute(const DNBatch<NT8, GPW> &B, int g0, int G, float (&C)[NT8][4]) {
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
        if (g0 + i < G) {
            float sx[NT8][2];
#pragma unroll
            for (int j = 0; j < NT8; ++j)
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const float4 v = B.hs[i][j][hf];
                    sx[j][hf] = (v.x + v.y) + (v.z + v.w);
                }
            q4_group<NT8>(B.w[i], B.b[i], B.hb[i], sx, C);
        }
    }
}

template <int FMT, int NT8, int GPW>
__global__ void __launch_bounds__(128) k_down_tiles_reg(ExpArgs a) {
    pdl_launch();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int gq = lane >> 2, c = lane & 3;
    const int d = a.d, f = a.f;
    const int RB = d >> 4, G = f >> 6;
    const int n_units = *a.ntiles * RB;
    const int nwarps = gridDim.x * 4;
    for (int unit = blockIdx.x * 4 + (threadIdx.x >> 5); unit < n_units; unit += nwarps) {
        const int tile = unit / RB, rb = unit - tile * RB;
        const TileInfo ti = tile_info(a, tile);
        const size_t blk = (size_t)ti.e * RB + rb;
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
        float C[NT8][4];
#pragma unroll
        for (int j = 0; j < NT8; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) C[j][i] = 0.f;
        DNBatch<NT8, GPW> A, B;
        dn_load(A, a, blk, G, 0, hrow, hsrow, lane);
        for (int g0 = 0; g0 < G; g0 += 2 * GPW) {
            if (g0 + GPW < G) dn_load(B, a, blk, G, g0 + GPW, hrow, hsrow, lane);
            dn_compute(A, g0, G, C);
            if (g0 + GPW < G) {
                if (g0 + 2 * GPW < G) dn_load(A, a, blk, G, g0 + 2 * GPW, hrow, hsrow, lane);
                dn_compute(B, g0 + GPW, G, C);
            }
        }
        down_store_combine<NT8>(a, ti, rb, C, lane);
    }
}

// ================================================================== tile mode, TMA ring
// One warp per (tile, 16-row block) over the whole K. In the fragment-major layout a unit's codes for groups
// [g0, g0 + SG) are one contiguous block per projection (and likewise the scale|bias words), so lane 0 of each
// warp streams whole stages with 1-D TMA bulk copies (evict-first in L2) into a ring of NS shared-memory stages
// completing on per-stage mbarriers; the warp's MMAs read the ring. Activations and group sums (L2-resident,
// reused by every row block of a tile) come through plain loads one group ahead. Every wait is bounded: on a
// timeout the warp records MOEB_DEVERR_TIMEOUT and stops issuing.
template <int NT8>
struct UnitSrc {
    int unit = -1;
    TileInfo ti;
    size_t blk;
    const uint16_t *row[NT8];   // activation row of B column gq of each n8 tile (x or h), or null
    const float *srow[NT8][2];  // group-sum rows of C columns 2c, 2c+1 (xsum or hsum), or null
};

template <int NT8, bool DOWN>
__device__ __forceinline__ void unit_src(UnitSrc<NT8> &u, const ExpArgs &a, int unit, int RB, int lane) {
    const int gq = lane >> 2, c = lane & 3;
    u.unit = unit;
    const int tile = unit / RB, rb = unit - tile * RB;
    u.ti = tile_info(a, tile);
    u.blk = (size_t)u.ti.e * RB + rb;
#pragma unroll
    for (int j = 0; j < NT8; ++j) {
        const int sb_ = tile_slot(a, u.ti, j * 8 + gq);
        if (DOWN) u.row[j] = sb_ >= 0 ? a.h + (size_t)sb_ * a.f + 16 * c : nullptr;
        else u.row[j] = sb_ >= 0 ? a.x + (size_t)(sb_ / a.k) * a.d + 16 * c : nullptr;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int sc_ = tile_slot(a, u.ti, j * 8 + 2 * c + hf);
            if (DOWN) u.srow[j][hf] = sc_ >= 0 ? a.hsum + (size_t)sc_ * (a.f / 16) : nullptr;
            else u.srow[j][hf] = sc_ >= 0 ? a.xsum + (size_t)(sc_ / a.k) * xsum_stride(a.d) : nullptr;
        }
    }
}

// B operand (16 activations per lane) and the two group sums of one group.
template <int NT8, bool DOWN>
__device__ __forceinline__ void load_act(const UnitSrc<NT8> &u, int g, uint32_t (&xb)[NT8][8], float (&sx)[NT8][2]) {
#pragma unroll
    for (int j = 0; j < NT8; ++j) {
        load_b16(u.row[j] ? u.row[j] + g * 64 : nullptr, xb[j]);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const float *p = u.srow[j][hf];
            if (DOWN) {
                if (p) {
                    const float4 v = *reinterpret_cast<const float4 *>(p + 4 * g);
                    sx[j][hf] = (v.x + v.y) + (v.z + v.w);
                } else {
                    sx[j][hf] = 0.f;
                }
            } else {
                sx[j][hf] = p ? p[g] : 0.f;
            }
        }
    }
}

// NP projections (2 for gate/up, 1 for down) of SG groups per stage
template <int NP, int SG>
struct RingStage {
    static constexpr int Q_BYTES = SG * 512, SB_BYTES = SG * 64;
    static constexpr int BYTES = NP * (Q_BYTES + SB_BYTES);
};

template <int FMT, int NT8, int NS, int SG, bool DOWN>
__device__ __forceinline__ void tiles_tma_body(const ExpArgs &a) {
    constexpr int NP = DOWN ? 1 : 2;
    using RS = RingStage<NP, SG>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int RB = DOWN ? (a.d >> 4) : (a.f >> 4);
    const int G = DOWN ? (a.f >> 6) : (a.d >> 6);
    const int SPU = (G + SG - 1) / SG;  // stages per unit
    const int n_units = *a.ntiles * RB;
    const int w0 = blockIdx.x * 4 + warp, nw = gridDim.x * 4;
    const int my_units = w0 < n_units ? (n_units - w0 + nw - 1) / nw : 0;
    const int total = my_units * SPU;
    unsigned char *ring = smem_raw + (size_t)warp * NS * RS::BYTES;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem_raw + 4 * NS * RS::BYTES) + warp * NS;
    const QProj P0 = DOWN ? a.dn : a.g, P1 = a.u;
    const uint64_t pol = l2_evict_first_policy();
    if (lane == 0) {
        for (int i = 0; i < NS; ++i) mbar_init(bar + i, 1);
        mbar_fence_init();
    }
    __syncwarp();
    int p_unit = -1;
    size_t p_blk = 0;
    auto issue = [&](int k) {  // lane 0 only
        if (k >= total) return;
        const int unit = w0 + (k / SPU) * nw, g0 = (k % SPU) * SG;
        if (unit != p_unit) {
            p_unit = unit;
            const int tile = unit / RB;
            int e = a.tile_mode ? a.tiles[tile].x : a.idx[tile];
            if (e < 0 || e >= a.E) e = 0;
            p_blk = (size_t)e * RB + (unit - tile * RB);
            if (!DOWN && g0 == 0 && a.dn_prefetch) prefetch_down(a, e, unit - tile * RB, RB, 0, 1);
        }
        const int ng = min(SG, G - g0);
        uint64_t *b = bar + (k % NS);
        unsigned char *st = ring + (size_t)(k % NS) * RS::BYTES;
        mbar_expect_tx(b, (unsigned)(NP * ng * (512 + 64)));
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            const QProj &PP = p == 0 ? P0 : P1;
            tma_load_1d(st + p * RS::Q_BYTES, PP.q + (p_blk * G + g0) * 128, ng * 512, b, pol);
            tma_load_1d(st + NP * RS::Q_BYTES + p * RS::SB_BYTES, PP.sb + (p_blk * G + g0) * 16, ng * 64, b, pol);
        }
    };
    if (lane == 0)
        for (int k = 0; k < NS - 1; ++k) issue(k);
    UnitSrc<NT8> U;
    float C0[NT8][4], C1[NT8][4];
#pragma unroll
    for (int j = 0; j < NT8; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) C0[j][i] = C1[j][i] = 0.f;
    uint32_t xb[NT8][8];
    float sx[NT8][2];
    bool ok = true;
    for (int k = 0; k < total && ok; ++k) {
        if (lane == 0) issue(k + NS - 1);
        const int unit = w0 + (k / SPU) * nw, g0 = (k % SPU) * SG;
        if (g0 == 0) {
            unit_src<NT8, DOWN>(U, a, unit, RB, lane);
            load_act<NT8, DOWN>(U, 0, xb, sx);
        }
        ok = mbar_wait_bounded(bar + (k % NS), (unsigned)((k / NS) & 1));
        if (!ok) {
            if (lane == 0) atomicOr(a.err, ERR_TIMEOUT);
            break;
        }
        const unsigned char *st = ring + (size_t)(k % NS) * RS::BYTES;
        const int ng = min(SG, G - g0);
#pragma unroll 1
        for (int i = 0; i < ng; ++i) {
            uint32_t xn[NT8][8];
            float sn[NT8][2];
            if (g0 + i + 1 < G) load_act<NT8, DOWN>(U, g0 + i + 1, xn, sn);  // next group's activations
            const uint4 w0v = reinterpret_cast<const uint4 *>(st)[i * 32 + lane];
            const uint2 s0v = reinterpret_cast<const uint2 *>(st + NP * RS::Q_BYTES)[i * 8 + (lane >> 2)];
            q4_group<NT8>(w0v, s0v, xb, sx, C0);
            if (!DOWN) {
                const uint4 w1v = reinterpret_cast<const uint4 *>(st + RS::Q_BYTES)[i * 32 + lane];
                const uint2 s1v = reinterpret_cast<const uint2 *>(st + NP * RS::Q_BYTES + RS::SB_BYTES)[i * 8 + (lane >> 2)];
                q4_group<NT8>(w1v, s1v, xb, sx, C1);
            }
#pragma unroll
            for (int j = 0; j < NT8; ++j) {
#pragma unroll
                for (int q = 0; q < 8; ++q) xb[j][q] = xn[j][q];
                sx[j][0] = sn[j][0];
                sx[j][1] = sn[j][1];
            }
        }
        __syncwarp();  // every lane is done with this stage before lane 0 refills it
        if (k % SPU == SPU - 1) {
            const int rb = unit - (unit / RB) * RB;
            if (DOWN) {
                down_store_combine<NT8>(a, U.ti, rb, C0, lane);
            } else {
#pragma unroll
                for (int j = 0; j < NT8; ++j) gate_up_store<NT8>(a, U.ti, rb, j, C0[j], C1[j], lane);
            }
#pragma unroll
            for (int j = 0; j < NT8; ++j)
#pragma unroll
                for (int i = 0; i < 4; ++i) C0[j][i] = C1[j][i] = 0.f;
        }
    }
    if (!ok) {  // drain: give every issued stage a bounded chance to land before the CTA exits
        for (int k = 0; k < NS; ++k) mbar_wait_bounded(bar + k, 0u, 1u << 12), mbar_wait_bounded(bar + k, 1u, 1u << 12);
    }
}

template <int FMT, int NT8, int NS, int SG>
__global__ void __launch_bounds__(128) k_gate_up_tiles(ExpArgs a) {
    pdl_launch();
    pdl_wait();
    tiles_tma_body<FMT, NT8, NS, SG, false>(a);
}

template <int FMT, int NT8, int NS, int SG>
__global__ void __launch_bounds__(128) k_down_tiles(ExpArgs a) {
    pdl_launch();
    pdl_wait();
    tiles_tma_body<FMT, NT8, NS, SG, true>(a);
}

// shared-memory bytes of the TMA-ring tile kernels (4 warps per CTA, plus one mbarrier per stage and warp)
size_t gate_up_tiles_smem(int nt8, int ns, int sg) {
    (void)nt8;
    return (size_t)4 * ns * 2 * sg * (512 + 64) + 4 * ns * 8;
}
size_t down_tiles_smem(int nt8, int ns, int sg) {
    (void)nt8;
    return (size_t)4 * ns * sg * (512 + 64) + 4 * ns * 8;
}

template __global__ void k_gate_up_slots<FMT_Q4, 8, 4>(ExpArgs);
template __global__ void k_down_slots<FMT_Q4, 4, 4>(ExpArgs);
template __global__ void k_gate_up_tiles_reg<FMT_Q4, 1, 2>(ExpArgs);
template __global__ void k_gate_up_tiles_reg<FMT_Q4, 2, 1>(ExpArgs);
template __global__ void k_down_tiles_reg<FMT_Q4, 1, 2>(ExpArgs);
template __global__ void k_down_tiles_reg<FMT_Q4, 2, 1>(ExpArgs);
template __global__ void k_gate_up_tiles<FMT_Q4, 1, 3, 8>(ExpArgs);
template __global__ void k_gate_up_tiles<FMT_Q4, 2, 3, 8>(ExpArgs);
template __global__ void k_down_tiles<FMT_Q4, 1, 3, 8>(ExpArgs);
template __global__ void k_down_tiles<FMT_Q4, 2, 3, 8>(ExpArgs);

}  // namespace moeb
