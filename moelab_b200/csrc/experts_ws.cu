// Grouped expert kernels, warp-specialized TMA pipeline (tile mode: slots grouped by expert).
//
// CTA = 1 producer warp + RBC consumer warps. A CTA work item ("super-unit") is one tile (<= 8*NT8 slots of one
// expert) and RBC consecutive 16-row blocks of the projection. K is streamed in stages of SG 64-groups through
// an NS-deep shared-memory ring:
//   producer: per stage, lane 0 issues one 2-D tensor copy per projection for the codes (RBC row blocks x SG
//     groups x 512 B) and one for the scale|bias words (x 64 B), evict-first in L2, no multicast; the lanes
//     of the tile's columns each issue a 1-D bulk copy of their activation row chunk (x for gate/up, h for
//     down; rows padded by 16 bytes in shared memory to spread banks) and of its group sums. Everything
//     completes on the stage's "full" mbarrier. (A bulk copy has a fixed issue cost, so few large copies per
//     stage matter: the tensor copies replace 2*NP*RBC row-block copies.)
//   consumers: each warp owns one row block, waits on "full", runs the m16n8k16 raw-code MMAs and fp32 scale
//     promotion of experts_common.cuh on the stage, and arrives on the stage's "empty" mbarrier.
// The activation tile is fetched once per CTA and shared by all row blocks; consumers never touch global
// memory until their epilogue (gate/up: bias, activation, h, hsum; down: weighted rows + deterministic combine).
// Every mbarrier wait is bounded; a timeout records MOEB_DEVERR_TIMEOUT and the CTA stops.
#include "experts_common.cuh"

namespace moeb {

template <int FMT, int NT8, int RBC, int SG, bool DOWN>
struct WSL {
    static constexpr int NP = DOWN ? 1 : 2;
    static constexpr int COLS = 8 * NT8;
    static constexpr int SBG = FMT == FMT_FP4 ? 32 : 64;  // scale bytes per (row block, group)
    static constexpr int W_BYTES = NP * RBC * SG * 512;
    static constexpr int SB_BYTES = NP * RBC * SG * SBG;
    static constexpr int X_ROW = SG * 128 + 16;
    static constexpr int X_BYTES = COLS * X_ROW;
    // group sums: down 16 bytes per group; gate/up 4 bytes per group, copied from the 16-byte boundary at or
    // below the stage's first group (a bulk copy must start 16-byte aligned), so up to 3 extra leading floats
    // (down rows get 16 bytes of padding: lanes 2c + hf then read float4s from distinct bank groups)
    static constexpr int S_ROW = DOWN ? SG * 16 + 16 : (SG % 4 == 0 ? SG * 4 : ((SG + 3) * 4 + 15) / 16 * 16);
    static constexpr int S_BYTES = COLS * S_ROW;
    static constexpr int STAGE = W_BYTES + SB_BYTES + X_BYTES + S_BYTES;
    static_assert(STAGE % 128 == 0 && W_BYTES % 128 == 0 && SB_BYTES % 128 == 0 && (RBC * SG * SBG) % 128 == 0,
                  "tensor-copy destinations must stay 128-byte aligned");
};

// This lane's scale words of one (row block, group) in a stage: int4 {scale|bias row gq, row gq+8}; MXFP4 the
// 4 E8M0 bytes of rows gq, gq+8 in .x
template <int FMT>
MOEB_DEV uint2 stage_scales(const unsigned char *p, int gq) {
    if (FMT == FMT_FP4) return make_uint2(reinterpret_cast<const uint32_t *>(p)[gq], 0u);
    return reinterpret_cast<const uint2 *>(p)[gq];
}

template <int FMT, int NT8, int RBC, int SG, int NS, bool DOWN, int MB>
__global__ void __launch_bounds__(32 * (RBC + 1), MB) k_experts_ws(const __grid_constant__ ExpArgs a) {
    using L = WSL<FMT, NT8, RBC, SG, DOWN>;
    if (DOWN || !a.early_ids) pdl_launch();
    extern __shared__ __align__(128) unsigned char smem_raw[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem_raw + NS * L::STAGE);
    uint64_t *empty = full + NS;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // barrier setup overlaps the upstream kernel's tail (it touches no upstream data)
    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, RBC);
        }
        mbar_fence_init();
    }
    __syncthreads();
    // Early down (a.early_ids, set for both kernels of the pair): the gate/up kernel releases this grid only after
    // its own wait (releasing it at the start measured faster when down does not start early), so the routing tables
    // (written upstream of gate/up) are complete; the producer reads them through L2 and issues the weight copies of
    // its first NS stages before waiting for h, then the activation copies of those stages.
    const bool early = DOWN && a.early_ids && warp == RBC;
    if (!early) pdl_wait();
    if (!DOWN && a.early_ids) pdl_launch();  // after this grid's own wait: the early down producer relies on it
    const int RB = DOWN ? (a.d >> 4) : (a.f >> 4);
    const int G = DOWN ? (a.f >> 6) : (a.d >> 6);
    const int RBS = (RB + RBC - 1) / RBC;  // super-units per tile
    const int SPU = (G + SG - 1) / SG;     // stages per super-unit
    const int n_tiles = a.tile_mode ? __ldcg(a.ntiles) : a.T * a.k;
    const int n_su = n_tiles * RBS;
    const int my_su = (int)blockIdx.x < n_su ? (n_su - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    const int total = my_su * SPU;

    if (warp == RBC) {
        // ------------------------------------------------------------ producer warp
        // Lane 0 issues the weight tensor copies; lanes [CL0, CL0 + COLS) copy one activation column each (CL0 = 16,
        // or 32 - COLS for tiles of more than 16 slots). Per work item every lane computes its source bases once;
        // the item's tile record and slot ids are fetched one item ahead so no global load sits on the issue path.
        constexpr int CL0 = L::COLS <= 16 ? 16 : 32 - L::COLS;
        static_assert(L::COLS <= 31, "producer lane roles: lane 0 issues the tensor copies");
        const uint64_t pol = l2_evict_first_policy();
        const int col = lane - CL0;  // column lane: column index
        const bool clane = col >= 0 && col < L::COLS;
        const int m0 = DOWN ? 2 : 0;  // tensor maps of this kernel's projections
        if (lane == 0)
            for (int p = 0; p < L::NP; ++p) {
                tmap_prefetch(&a.tmq[m0 + p]);
                tmap_prefetch(&a.tmsb[m0 + p]);
            }
        auto fetch_tile = [&](int su) {  // tile record (expert, start, n), through L2
            const int tile = su / RBS;
            return a.tile_mode ? __ldcg(a.tiles + tile) : make_int4(__ldcg(a.idx + tile), tile, 1, 0);
        };
        auto fetch_slot = [&](const int4 &tr) {  // this lane's slot id, or -1
            return (clane && col < tr.z) ? (a.tile_mode ? __ldcg(a.sorted + tr.y + col) : tr.y) : -1;
        };
        // activation copies of the first `nearly` stages, deferred until the upstream grid is complete
        const int nearly = early ? min(NS, total) : 0;
        const unsigned char *ps0[NS], *ps1[NS];
        auto issue_x = [&](int k, const unsigned char *s0, const unsigned char *s1) {
            const int g0 = (k % SPU) * SG, ng = min(SG, G - g0);
            const int ga = DOWN ? g0 : (g0 & ~3);
            const int sum_bytes = DOWN ? ng * 16 : ((g0 + ng - ga + 3) / 4) * 16;
            unsigned char *st = smem_raw + (size_t)(k % NS) * L::STAGE;
            tma_load_1d(st + L::W_BYTES + L::SB_BYTES + col * L::X_ROW, s0 + (size_t)g0 * 128, ng * 128,
                        full + k % NS);
            tma_load_1d(st + L::W_BYTES + L::SB_BYTES + L::X_BYTES + col * L::S_ROW, s1 + (size_t)ga * (DOWN ? 16 : 4),
                        sum_bytes, full + k % NS);
        };
        auto flush_early = [&]() {
            pdl_wait();
#pragma unroll
            for (int q = 0; q < NS; ++q)
                if (q < nearly && lane != 0 && ps0[q] != nullptr) issue_x(q, ps0[q], ps1[q]);
        };
        int4 tr_n = make_int4(0, 0, 0, 0);
        int sl_n = -1;
        if (my_su > 0) {
            tr_n = fetch_tile(blockIdx.x);
            sl_n = fetch_slot(tr_n);
        }
        const unsigned char *src0 = nullptr, *src1 = nullptr;
        int ncol = 0, row0 = 0;
        for (int k = 0; k < total; ++k) {
            const int slot = k % NS;
            const int g0 = (k % SPU) * SG, ng = min(SG, G - g0);
            if (g0 == 0) {  // new work item: take the prefetched metadata, prefetch the next item's
                const int su = (int)blockIdx.x + (k / SPU) * (int)gridDim.x;
                const int rb0 = (su - (su / RBS) * RBS) * RBC;
                const int e = (tr_n.x < 0 || tr_n.x >= a.E) ? 0 : tr_n.x;
                ncol = min(L::COLS, tr_n.z);
                row0 = e * RB + rb0;
                const int s_ = sl_n;
                if (clane && s_ >= 0) {
                    src0 = reinterpret_cast<const unsigned char *>(DOWN ? a.h + (size_t)s_ * a.f
                                                                        : a.x + (size_t)(s_ / a.k) * a.xs);
                    src1 = reinterpret_cast<const unsigned char *>(DOWN ? a.hsum + (size_t)s_ * (a.f / 16)
                                                                        : a.xsum + (size_t)(s_ / a.k) * xsum_stride(a.d));
                } else {
                    src0 = src1 = nullptr;
                }
                if (!DOWN && lane == 0 && a.dn_prefetch)
                    for (int r = 0; r < min(RBC, RB - rb0); ++r) prefetch_down(a, e, rb0 + r, RB, 0, 1);
                const int nsu = su + (int)gridDim.x;
                if (nsu < n_su) {
                    tr_n = fetch_tile(nsu);                 // in flight during this item's stages
                    if (SPU == 1) sl_n = fetch_slot(tr_n);  // no later stage to hide it behind
                }
            } else if (g0 == SG) {
                const int nsu = (int)blockIdx.x + (k / SPU + 1) * (int)gridDim.x;
                if (nsu < n_su) sl_n = fetch_slot(tr_n);
            }
            if (k == nearly && nearly > 0) flush_early();  // before any wait on a consumed stage
            if (k >= NS && !mbar_wait_bounded(empty + slot, (unsigned)(((k / NS) - 1) & 1))) {
                if (lane == 0) atomicOr(a.err, ERR_TIMEOUT);
                return;
            }
            const int ga = DOWN ? g0 : (g0 & ~3);  // first group of the sums copy (16-byte aligned source)
            const int sum_bytes = DOWN ? ng * 16 : ((g0 + ng - ga + 3) / 4) * 16;
            // a tensor copy always delivers its whole box (rows or groups past the end arrive as zeros)
            if (lane == 0)
                mbar_expect_tx(full + slot, (unsigned)(L::NP * RBC * SG * (512 + L::SBG) + ncol * (ng * 128 + sum_bytes)));
            __syncwarp();
            unsigned char *st = smem_raw + (size_t)slot * L::STAGE;
            if (lane == 0) {
                for (int p = 0; p < L::NP; ++p) {
                    tma_load_2d(st + p * RBC * SG * 512, &a.tmq[m0 + p], g0 * 64, row0, full + slot, pol);
                    tma_load_2d(st + L::W_BYTES + p * RBC * SG * L::SBG, &a.tmsb[m0 + p], g0 * (L::SBG / 4), row0,
                                full + slot, pol);
                }
            } else if (k < nearly) {
#pragma unroll
                for (int q = 0; q < NS; ++q)
                    if (q == k) {
                        ps0[q] = src0;
                        ps1[q] = src1;
                    }
            } else if (src0 != nullptr) {
                issue_x(k, src0, src1);
            }
        }
        if (nearly > 0 && total == nearly) flush_early();  // every stage fit the first ring
        return;
    }

    // ---------------------------------------------------------------- consumer warps (one row block each)
    // Global metadata is loaded ahead of its use, so no dependent global load sits between two stages: the next
    // item's tile record during this item and, for tiles of up to 16 slots (EARLY; 24 would spill), the epilogue's
    // slot ids at the item's first stage and (down) the combine weights at its second.
    constexpr bool EARLY = NT8 <= 2;
    const int gq = lane >> 2, c = lane & 3;
    float C0[NT8][4], C1[NT8][4];
    int sl[NT8][2];
    float wv[NT8][2];
    TileInfo ti;
    int rb = 0;
    int4 tr_next = my_su > 0 ? tile_rec(a, (int)blockIdx.x / RBS) : make_int4(0, 0, 0, 0);
    for (int k = 0; k < total; ++k) {
        const int slot = k % NS;
        const int su = (int)blockIdx.x + (k / SPU) * (int)gridDim.x;
        const int tile = su / RBS;
        const int g0 = (k % SPU) * SG, ng = min(SG, G - g0);
        if (g0 == 0) {
            ti = tile_info_of(a, tr_next);
            if (su + (int)gridDim.x < n_su) tr_next = tile_rec(a, (su + (int)gridDim.x) / RBS);
            rb = (su - tile * RBS) * RBC + warp;
            if (EARLY) epi_slots<NT8>(a, ti, lane, sl);
#pragma unroll
            for (int j = 0; j < NT8; ++j)
#pragma unroll
                for (int i = 0; i < 4; ++i) C0[j][i] = C1[j][i] = 0.f;
        }
        if (EARLY && DOWN && k % SPU == (SPU > 1 ? 1 : 0)) epi_weights<NT8>(a, sl, wv);
        if (!mbar_wait_bounded(full + slot, (unsigned)((k / NS) & 1))) {
            if (lane == 0) atomicOr(a.err, ERR_TIMEOUT);
            // give the copies that may still be in flight into this CTA's ring a bounded chance to land
            for (int q = 1; q < NS && k + q < total; ++q)
                mbar_wait_bounded(full + (k + q) % NS, (unsigned)(((k + q) / NS) & 1), 1u << 12);
            return;
        }
        const unsigned char *st = smem_raw + (size_t)slot * L::STAGE;
        if (rb < RB) {
            const unsigned char *xs = st + L::W_BYTES + L::SB_BYTES;
            const unsigned char *ss = xs + L::X_BYTES;
#pragma unroll
            for (int i = 0; i < SG; ++i) {
                if (i < ng) {
                    uint32_t xb[NT8][8];
                    float sx[NT8][2];
#pragma unroll
                    for (int j = 0; j < NT8; ++j) {
                        const int col = j * 8 + gq;
                        if (col < ti.n) {
                            const uint4 *xp = reinterpret_cast<const uint4 *>(xs + col * L::X_ROW + i * 128 + 32 * c);
                            const uint4 u0 = xp[0], u1 = xp[1];
                            xb[j][0] = u0.x; xb[j][1] = u0.y; xb[j][2] = u0.z; xb[j][3] = u0.w;
                            xb[j][4] = u1.x; xb[j][5] = u1.y; xb[j][6] = u1.z; xb[j][7] = u1.w;
                        } else {
#pragma unroll
                            for (int q = 0; q < 8; ++q) xb[j][q] = 0u;
                        }
#pragma unroll
                        for (int hf = 0; hf < 2; ++hf) {
                            const int cc = j * 8 + 2 * c + hf;
                            if (FMT == FMT_Q4 && cc < ti.n) {  // group sums: int4 promotion only
                                if (DOWN) {
                                    const float4 v = *reinterpret_cast<const float4 *>(ss + cc * L::S_ROW + i * 16);
                                    sx[j][hf] = (v.x + v.y) + (v.z + v.w);
                                } else {
                                    sx[j][hf] = reinterpret_cast<const float *>(ss + cc * L::S_ROW)[(g0 & 3) + i];
                                }
                            } else {
                                sx[j][hf] = 0.f;
                            }
                        }
                    }
                    const uint4 w0 = reinterpret_cast<const uint4 *>(st + (warp * SG + i) * 512)[lane];
                    wgroup<FMT, NT8>(w0, stage_scales<FMT>(st + L::W_BYTES + (warp * SG + i) * L::SBG, gq), c, xb, sx, C0);
                    if (!DOWN) {
                        const uint4 w1 = reinterpret_cast<const uint4 *>(st + ((RBC + warp) * SG + i) * 512)[lane];
                        wgroup<FMT, NT8>(w1, stage_scales<FMT>(st + L::W_BYTES + ((RBC + warp) * SG + i) * L::SBG, gq),
                                         c, xb, sx, C1);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot);
        if (k % SPU == SPU - 1 && rb < RB) {
            if (!EARLY) {
                epi_slots<NT8>(a, ti, lane, sl);
                if (DOWN) epi_weights<NT8>(a, sl, wv);
            }
            if (DOWN) {
                down_store_combine_sl<NT8>(a, ti, rb, C0, lane, sl, wv);
            } else {
#pragma unroll
                for (int j = 0; j < NT8; ++j) gate_up_store_sl(a, ti, rb, sl[j], C0[j], C1[j], lane);
            }
        }
    }
    if (DOWN && a.ypeers) {  // rows stored into peers' memory: make them visible system-wide before exiting
        __syncwarp();
        if (lane == 0) __threadfence_system();
    }
}

size_t experts_ws_smem(int nt8, int rbc, int sg, int ns, bool down, int fmt) {
    const int np = down ? 1 : 2, cols = 8 * nt8, sbg = fmt == FMT_FP4 ? 32 : 64;
    const int s_row = down ? sg * 16 + 16 : (sg % 4 == 0 ? sg * 4 : ((sg + 3) * 4 + 15) / 16 * 16);
    const size_t stage = (size_t)np * rbc * sg * (512 + sbg) + (size_t)cols * (sg * 128 + 16) + (size_t)cols * s_row;
    return ns * stage + 2 * ns * 8;
}

// gate/up: 4 groups per stage, 2 stages, 2 CTAs per SM; down: 4 groups per stage, 4 stages, 2 CTAs per SM
// (measured best of the (SG, NS, CTAs/SM) sweep on the Qwen3-30B shape at T = 4, 32, 256)
#define MOEB_WS(FMT)                                                                         \
    template __global__ void k_experts_ws<FMT, 1, 8, 4, 2, false, 2>(const __grid_constant__ ExpArgs); \
    template __global__ void k_experts_ws<FMT, 2, 8, 4, 2, false, 2>(const __grid_constant__ ExpArgs); \
    template __global__ void k_experts_ws<FMT, 1, 8, 4, 4, true, 2>(const __grid_constant__ ExpArgs);  \
    template __global__ void k_experts_ws<FMT, 2, 8, 4, 4, true, 2>(const __grid_constant__ ExpArgs);  \
    template __global__ void k_experts_ws<FMT, 3, 8, 4, 2, false, 2>(const __grid_constant__ ExpArgs); \
    template __global__ void k_experts_ws<FMT, 3, 8, 4, 3, true, 2>(const __grid_constant__ ExpArgs);
MOEB_WS(FMT_Q4)
MOEB_WS(FMT_FP4)

}  // namespace moeb
