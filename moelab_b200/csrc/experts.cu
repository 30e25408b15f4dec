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
//   *_tiles_reg (slots grouped by expert into tiles of 8*NT8): one warp per unit over the whole K, a register
//     double-buffered load pipeline, and a per-warp epilogue (no CTA barriers). The warp-specialized TMA
//     variant of the tile kernels is in experts_ws.cu.
// Both weight formats share these kernels (FMT): int4 promotes per 64-group in fp32; MXFP4 folds its E8M0 scale
// into exact bf16 A fragments (experts_common.cuh).
// gate/up (reference GATE_UP_SRC metal_q4_decode_v4.py:67-93, GATE_UP_E_SRC metal_q4_tiles_v2.py:179-275):
//   h[slot][r] = bf16(act(g + bg, u + bu)); hsum[slot][r/16] = sum of the block's 16 bf16 h values.
// down + combine (DOWN_SRC metal_q4_decode_v4.py:95-144, DOWN_E_SRC + COMBINE_SRC metal_q4_tiles_v2.py):
//   yp[slot][r] = w_slot * (Wd h + bd); the last unit to finish a (token, 16-row block) sums its k slots in
//   fixed order j = 0..k-1 (deterministic, no float atomics), adds the optional residual and writes y.
#include "slots_common.cuh"

namespace moeb {

// ================================================================== slot mode (decode)
// One CTA per (slot, 16-row block); KS warps split the K groups; GPW groups per warp are loaded at once. The unit
// bodies live in slots_common.cuh (shared with the fused decode kernel).
// The dependents are released only after this grid's own wait: the decode down kernel then reads the ids and
// weights (written upstream of this kernel) before it waits for h.
template <int FMT, int KS, int GPW>
__global__ void __launch_bounds__(32 * KS, FMT == FMT_FP4 ? 2 : 3) k_gate_up_slots(ExpArgs a) {
    pdl_wait();
    pdl_launch();
    extern __shared__ uint4 xs4[];  // the slot's x row, d bf16
    __shared__ float red[KS * 2 * 4 * 32];
    for (int unit = blockIdx.x; unit < a.T * a.k * (a.f >> 4); unit += gridDim.x)
        gate_up_slot_unit<FMT, KS, GPW>(a, unit, xs4, red);
}

template <int FMT, int KS, int GPW>
__global__ void __launch_bounds__(32 * KS, FMT == FMT_FP4 ? 4 : 8) k_down_slots(ExpArgs a) {
    pdl_launch();
    pdl_wait();
    extern __shared__ uint4 hs4[];  // the slot's h row (f bf16) followed by its f/16 block sums
    __shared__ float red[KS * 4 * 32];
    for (int unit = blockIdx.x; unit < a.T * a.k * (a.d >> 4); unit += gridDim.x)
        down_slot_unit<FMT, KS, GPW>(a, unit, hs4, red);
}

// Decode down with the combine in shared memory: one CTA per (token, 16-row block of d), the token's k slots as k
// groups of KS warps, each warp carrying VW shares of a KS * VW split of K. Each slot's value is computed exactly as
// in k_down_slots with 4 warps when KS * VW = 4 (same shares, partials summed in share order, weight * (acc + bias));
// the k values are then summed in slot order plus the residual, as down_store_combine's last arrival does - without
// the global slot rows, fences and counters. k <= 32 / KS; the CTA has 32 * KS * k threads (at most 256 * KS, the
// launch bound).
// The expert ids and combine weights come from upstream of the gate/up kernel, which releases this grid only
// after its own wait, so they are read through L2 (never a stale L1 line) before this grid waits for gate/up; the
// first weight batch of every slot is issued before the wait too, and h after it (a.early_ids = 0: wait first).
template <int FMT, int KS, int VW, int GPW>
__global__ void __launch_bounds__(256 * KS, 1) k_down_tok(ExpArgs a) {
    constexpr int KV = KS * VW;
    pdl_launch();
    if (!a.early_ids) pdl_wait();
    extern __shared__ uint4 tsm4[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int grp = warp / KS, lw = warp - grp * KS;  // slot j = grp of the token; local warp
    const int k = a.k, d = a.d, f = a.f, RB = d >> 4;
    const int hs_u4 = (f * 2 + f / 16 * 4) / 16;     // h row + block sums, in uint4
    uint4 *hs4 = tsm4 + (size_t)grp * hs_u4;
    float *red = reinterpret_cast<float *>(tsm4 + (size_t)k * hs_u4);  // [k][KV][4][32]
    float *vals = red + k * KV * 4 * 32;                                // [k][16]
    for (int unit = blockIdx.x; unit < a.T * RB; unit += gridDim.x) {
        const int t = unit / RB, rb = unit - t * RB;
        const int slot = t * k + grp;
        const int e_raw = __ldcg(a.idx + slot);
        const float w_raw = __ldcg(a.wts + slot);
        const TileInfo ti = {(e_raw >= 0 && e_raw < a.E) ? e_raw : 0, slot, 1};
        float C[VW][1][4];
        down_slot_partial_v<FMT, KS, VW, GPW>(a, slot, (size_t)ti.e * RB + rb, lw, threadIdx.x - grp * KS * 32, hs4,
                                              C, a.early_ids != 0);
#pragma unroll
        for (int v = 0; v < VW; ++v)
#pragma unroll
            for (int i = 0; i < 4; ++i) red[((grp * KV + lw * VW + v) * 4 + i) * 32 + lane] = C[v][0][i];
        __syncthreads();
        if (lw == 0 && (lane & 3) == 0) {  // column 0 (the slot) of rows gq, gq + 8
            float cs[1][4];
            down_slot_reduce<KV>(red + grp * KV * 4 * 32, lane, cs);
            const int gq = lane >> 2, r0 = rb * 16 + gq, r1 = r0 + 8;
            const float wsl = (e_raw >= 0 && e_raw < a.E) ? w_raw : 0.f;
            float v0 = cs[0][0], v1 = cs[0][2];
            if (a.bd) {
                v0 += a.bd[(size_t)ti.e * d + r0];
                v1 += a.bd[(size_t)ti.e * d + r1];
            }
            vals[grp * 16 + gq] = wsl * v0;
            vals[grp * 16 + gq + 8] = wsl * v1;
        }
        __syncthreads();
        if (threadIdx.x < 16) {
            const int r = rb * 16 + threadIdx.x;
            float acc = 0.f;
            for (int j = 0; j < k; ++j) acc += vals[j * 16 + threadIdx.x];
            if (a.residual) acc += bf2f(a.residual[(size_t)t * d + r]);
            a.y[(size_t)t * d + r] = f2bf(acc);
        }
        __syncthreads();  // the shared buffers are reused by the next unit
    }
}

size_t down_tok_smem(int k, int f, int ks) { return (size_t)k * ((f * 2 + f / 16 * 4) + ks * 4 * 32 * 4 + 16 * 4); }

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

template <int FMT, int NT8, int GPW>
__device__ __forceinline__ void gu_load(GUBatch<NT8, GPW> &B, const ExpArgs &a, size_t blk, int G, int g0,
                                        const uint16_t *const (&xrow)[NT8], const float *const (&sxrow)[NT8][2],
                                        int lane) {
    const int gq = lane >> 2;
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
        const int g = min(g0 + i, G - 1);
        B.wg[i] = ld_w(a.g, blk, G, g, lane);
        B.wu[i] = ld_w(a.u, blk, G, g, lane);
        B.bg[i] = ld_scales<FMT>(a.g, blk, G, g, gq);
        B.bu[i] = ld_scales<FMT>(a.u, blk, G, g, gq);
#pragma unroll
        for (int j = 0; j < NT8; ++j) {
            load_b16(xrow[j] ? xrow[j] + g * 64 : nullptr, B.xb[i][j]);
            B.sx[i][j][0] = sxrow[j][0] ? sxrow[j][0][g] : 0.f;
            B.sx[i][j][1] = sxrow[j][1] ? sxrow[j][1][g] : 0.f;
        }
    }
}

template <int FMT, int NT8, int GPW>
__device__ __forceinline__ void gu_compute(const GUBatch<NT8, GPW> &B, int g0, int G, int c, float (&Cg)[NT8][4],
                                           float (&Cu)[NT8][4]) {
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
        if (g0 + i < G) {
            wgroup<FMT, NT8>(B.wg[i], B.bg[i], c, B.xb[i], B.sx[i], Cg);
            wgroup<FMT, NT8>(B.wu[i], B.bu[i], c, B.xb[i], B.sx[i], Cu);
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
            xrow[j] = sb_ >= 0 ? a.x + (size_t)(sb_ / a.k) * a.xs + 16 * c : nullptr;
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
        gu_load<FMT>(A, a, blk, G, 0, xrow, sxrow, lane);
        for (int g0 = 0; g0 < G; g0 += 2 * GPW) {
            if (g0 + GPW < G) gu_load<FMT>(B, a, blk, G, g0 + GPW, xrow, sxrow, lane);
            gu_compute<FMT>(A, g0, G, c, Cg, Cu);
            if (g0 + GPW < G) {
                if (g0 + 2 * GPW < G) gu_load<FMT>(A, a, blk, G, g0 + 2 * GPW, xrow, sxrow, lane);
                gu_compute<FMT>(B, g0 + GPW, G, c, Cg, Cu);
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

template <int FMT, int NT8, int GPW>
__device__ __forceinline__ void dn_load(DNBatch<NT8, GPW> &B, const ExpArgs &a, size_t blk, int G, int g0,
                                        const uint16_t *const (&hrow)[NT8], const float *const (&hsrow)[NT8][2],
                                        int lane) {
    const int gq = lane >> 2;
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
        const int g = min(g0 + i, G - 1);
        B.w[i] = ld_w(a.dn, blk, G, g, lane);
        B.b[i] = ld_scales<FMT>(a.dn, blk, G, g, gq);
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

template <int FMT, int NT8, int GPW>
__device__ __forceinline__ void dn_compute(const DNBatch<NT8, GPW> &B, int g0, int G, int c, float (&C)[NT8][4]) {
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
            wgroup<FMT, NT8>(B.w[i], B.b[i], c, B.hb[i], sx, C);
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
        dn_load<FMT>(A, a, blk, G, 0, hrow, hsrow, lane);
        for (int g0 = 0; g0 < G; g0 += 2 * GPW) {
            if (g0 + GPW < G) dn_load<FMT>(B, a, blk, G, g0 + GPW, hrow, hsrow, lane);
            dn_compute<FMT>(A, g0, G, c, C);
            if (g0 + GPW < G) {
                if (g0 + 2 * GPW < G) dn_load<FMT>(A, a, blk, G, g0 + 2 * GPW, hrow, hsrow, lane);
                dn_compute<FMT>(B, g0 + GPW, G, c, C);
            }
        }
        down_store_combine<NT8>(a, ti, rb, C, lane);
    }
}

template __global__ void k_gate_up_slots<FMT_Q4, 4, 8>(ExpArgs);
template __global__ void k_down_slots<FMT_Q4, 4, 4>(ExpArgs);
template __global__ void k_gate_up_slots<FMT_FP4, 8, 4>(ExpArgs);
template __global__ void k_down_slots<FMT_FP4, 4, 4>(ExpArgs);
template __global__ void k_down_tok<FMT_Q4, 4, 1, 4>(ExpArgs);
template __global__ void k_down_tok<FMT_FP4, 4, 1, 4>(ExpArgs);
template __global__ void k_down_tok<FMT_Q4, 2, 2, 6>(ExpArgs);
template __global__ void k_down_tok<FMT_FP4, 2, 2, 6>(ExpArgs);
template __global__ void k_gate_up_tiles_reg<FMT_FP4, 1, 2>(ExpArgs);
template __global__ void k_down_tiles_reg<FMT_FP4, 1, 2>(ExpArgs);
template __global__ void k_gate_up_tiles_reg<FMT_FP4, 2, 1>(ExpArgs);
template __global__ void k_down_tiles_reg<FMT_FP4, 2, 1>(ExpArgs);
template __global__ void k_gate_up_tiles_reg<FMT_Q4, 1, 2>(ExpArgs);
template __global__ void k_gate_up_tiles_reg<FMT_Q4, 2, 1>(ExpArgs);
template __global__ void k_down_tiles_reg<FMT_Q4, 1, 2>(ExpArgs);
template __global__ void k_down_tiles_reg<FMT_Q4, 2, 1>(ExpArgs);

}  // namespace moeb
