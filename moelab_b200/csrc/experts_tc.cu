// Grouped expert kernels on the 5th-generation tensor cores (tcgen05, accumulators in TMEM), for medium and high
// loads (tiles of up to NT = 32 .. 256 slots of one expert: the weights are dequantized once per tile). Two
// kernels: k_experts_tc below keeps the dequantized A operand in shared memory (gate/up tiles of 256, whose two
// accumulators fill TMEM); k_experts_tca further down writes A into TMEM (every other tile size).
//
// k_experts_tc. A work item is (tile, 128 output rows). D[128 rows][NT slots] = W[128][K] . X[NT][K]^T accumulates in TMEM
// (fp32, lane = row, column = slot). K advances one 64-group per step through three shared-memory rings, so
// that each resource is only as deep as its own latency needs:
//   raw ring (NR stages, 4.5 KB per projection): the packed int4 codes and scale|bias words (or MXFP4 codes and
//     E8M0 scales) of the item's 8 row blocks for one group. They come from HBM, so this ring is the deep one;
//   X ring (NX stages, NT x 128 B): the tile's activation rows for the group (64 k, 128-byte swizzle: the UMMA
//     K-major layout), from L2;
//   A ring (NA stages, 16 KB per projection): the dequantized bf16 weight tile in the same swizzled layout.
// Roles (one CTA per SM):
//   warp 0, one lane: tensor copies of the raw stages ("rfull" mbarrier with transaction bytes; "rempty" frees);
//   warp 2, one lane: tensor copies of the X stages ("xfull" / "xempty"). No multicast anywhere;
//   warps 3 .. 3 + DQW - 1 (one per (projection, row block)): wait for a raw stage, read their block into
//     registers, wait for a free A stage, dequantize (int4: q|0x4300 = 128+q exactly, one HSUB2 and one HFMA2,
//     a single bf16 rounding of s*q + b; MXFP4: E2M1 * 2^(S-127), exact), write it swizzled, fence the proxy
//     (generic writes -> tensor-core reads), then arrive on "afull" and release the raw stage;
//   warp 1, one lane: per step waits "afull" and "xfull", issues 4 k-steps of tcgen05.mma per projection
//     (M = 128, N = the tile's slots rounded up to 16, K = 16, bf16 x bf16 -> fp32) and commits "aempty" and
//     "xempty"; after the item's last group it commits the accumulator set ("accf");
//   EPW epilogue warps: tcgen05.ld 16 columns at a time (warp w reads TMEM lanes 32 * (w % 4) .. + 31, its
//     rows; with 8 warps two share a lane quarter and split the columns); gate/up: bias + activation -> h in
//     slot-sorted order; down: weight * (acc + bias) -> the slot's fp32 row for the separate combine pass; then
//     "acce" frees the set. With ACC = 2 sets the next item's MMAs run while the epilogue drains.
// The activations arrive in expert-sorted order (x gathered by k_gather_rows; gate/up writes h sorted), so each
// tile's rows are contiguous for the tensor copy (rows past the tile belong to other tiles or are zero-filled
// past the end; their columns are never read).
// Every wait is bounded (timeout -> MOEB_DEVERR_TIMEOUT, the roles stop, in-flight copies and MMAs are drained
// with bounded waits, TMEM is released).
#include "experts_common.cuh"

namespace moeb {

namespace {

constexpr int TC_M = 128;
// K-major operand descriptor, 128-byte swizzle: 8-row groups 1024 B apart (SBO), rows of 128 B.
MOEB_DEV uint64_t sdesc_sw128(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
    d |= (uint64_t)1 << 46;             // descriptor version (tcgen05)
    d |= (uint64_t)2 << 61;             // SWIZZLE_128B
    return d;
}
// kind::f16 instruction descriptor: fp32 accumulate, A = B = bf16, both K-major, M x N.
MOEB_DEV uint32_t idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
MOEB_DEV void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
MOEB_DEV void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
MOEB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MOEB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
MOEB_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
MOEB_DEV void mbar_arrive1(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
MOEB_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// A from tensor memory: D[tmem] (+)= A[tmem] . B[smem desc]^T (no output lanes disabled)
MOEB_DEV void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
// 16 TMEM lanes x 32 columns from the warp: thread 4i + j supplies lanes i, i + 8, columns 8m + 2j, 8m + 2j + 1
// (register 4m + 2h + c = lane i + 8h, column 8m + 2j + c)
MOEB_DEV void tmem_st_16x256_x4(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
MOEB_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Dequantize this lane's share of one (16-row block, 64-group): rows gq (out[0]) and gq + 8 (out[1]), k-pairs
// 8c .. 8c + 7 of the group (k = 16c .. 16c + 15) as bf16x2 words. int4: q|0x4300 = 128+q exactly, one HSUB2 and
// one HFMA2 (a single bf16 rounding of s*q + b); MXFP4: E2M1 * 2^(S-127), exact in bf16.
template <int FMT>
MOEB_DEV void dequant_block(uint4 w, uint32_t sb0, uint32_t sb1, int c, uint32_t (&out)[2][8]) {
    const uint32_t k128 = 0x43004300u;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        const uint32_t wa = hf ? w.z : w.x, wb = hf ? w.w : w.y;
        if (FMT == FMT_FP4) {
            const uint32_t S = (sb0 >> (8 * (hf * 2 + (c >> 1)))) & 0xFFu;
            uint32_t lo[4], hi[4];
            fp4_word(wa, fp4_scale2(S), lo);
            fp4_word(wb, fp4_scale2(S), hi);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                out[hf][i] = lo[i];
                out[hf][4 + i] = hi[i];
            }
        } else {
            const uint32_t sv = hf ? sb1 : sb0;
            const uint32_t s2 = (sv & 0xFFFFu) | (sv << 16), b2 = (sv >> 16) | (sv & 0xFFFF0000u);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t v = q4pair(i < 4 ? wa : wb, i & 3);  // (128 + q_2p, 128 + q_2p+1)
                __nv_bfloat162 qv = *reinterpret_cast<const __nv_bfloat162 *>(&v);
                qv = __hsub2(qv, *reinterpret_cast<const __nv_bfloat162 *>(&k128));
                const __nv_bfloat162 r2 = __hfma2(qv, *reinterpret_cast<const __nv_bfloat162 *>(&s2),
                                                  *reinterpret_cast<const __nv_bfloat162 *>(&b2));
                out[hf][i] = *reinterpret_cast<const uint32_t *>(&r2);
            }
        }
    }
}

// The fp32 output row of a slot: the workspace's slot rows, or - expert-parallel over peer memory - the slot's row
// in its owner's return block (as the decode and tile epilogues store it)
MOEB_DEV float *slot_row(const ExpArgs &a, int slot) {
    return a.ypeers ? reinterpret_cast<float *>(a.ypeers[slot / a.C] + a.yoff) + ((size_t)a.me * a.C + slot % a.C) * a.d
                    : a.yp + (size_t)slot * a.d;
}

// Tile record of this CTA's work item `it` (items blockIdx.x + it * gridDim.x; MT items per tile). The roles keep the
// next item's record in flight while they work on the current one.
MOEB_DEV int4 item_tile(const ExpArgs &a, int it, int MT) {
    return a.tiles[((int)blockIdx.x + it * (int)gridDim.x) / MT];
}

// The down epilogue's per-column metadata for one warp, loaded before its accumulator is ready: lane l holds, for
// chunk q (columns c0 = c_first + q * c_step .. c0 + 15), the slot and combine weight of column c0 + (l & 15)
// (slot -1 past the tile). Loading them per column next to the row stores serialises two dependent global-load
// round trips per column: a load after a store that may alias it stays behind that store.
template <int NCH>
MOEB_DEV void down_epi_meta(const ExpArgs &a, const int4 tr, int c_first, int c_step, int lane, int (&msl)[NCH],
                            float (&mw)[NCH]) {
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
        const int n = c_first + q * c_step + (lane & 15);
        msl[q] = n < tr.z ? a.sorted[tr.y + n] : -1;
    }
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
        const int s = msl[q];
        float w = 0.f;
        if (s >= 0) {
            const int e_raw = a.idx[s];
            const float wt = a.wts[s];
            w = (e_raw >= 0 && e_raw < a.E) ? wt : 0.f;
        }
        mw[q] = w;
    }
}

// k order of the tensor-core operands inside a 64-group when A lives in TMEM (see k_experts_tca)
MOEB_DEV int kperm64(int k) { return (k & ~63) | (((k >> 2) & 3) << 4) | (((k >> 4) & 3) << 2) | (k & 3); }

template <int FMT, int NT, int NR, int NA, int NX, int ACC, bool DOWN>
struct TCL {
    static constexpr int NP = DOWN ? 1 : 2;
    static constexpr int DQW = 8 * NP;                   // dequant warps: one (projection, row block) each
    static constexpr int EPW = DOWN ? 4 : 8;             // epilogue warps
    static constexpr int THREADS = 32 * (3 + DQW + EPW);
    static constexpr int SBG = FMT == FMT_FP4 ? 32 : 64;  // scale bytes per (row block, group)
    static constexpr int A_BYTES = TC_M * 128;           // one projection's 128 rows x 64 k, bf16, swizzled
    static constexpr int A_STAGE = NP * A_BYTES;
    static constexpr int X_STAGE = NT * 128;             // NT rows x 64 k
    static constexpr int Q_BYTES = 8 * 512;              // packed codes, 8 row blocks x one group
    static constexpr int S_BYTES = 8 * SBG;              // int4 scale|bias words / MXFP4 E8M0 bytes
    static constexpr int R_STAGE = NP * (Q_BYTES + S_BYTES);
    static constexpr int OFF_X = NA * A_STAGE;
    static constexpr int OFF_R = OFF_X + NX * X_STAGE;
    static constexpr int OFF_BAR = OFF_R + NR * R_STAGE;
    static constexpr int NBAR = 2 * (NR + NA + NX + ACC);
    static constexpr int SMEM = 1024 + OFF_BAR + NBAR * 8;  // + alignment slack
    static constexpr int TMEM_RAW = ACC * NP * NT;
    static constexpr int TMEM_COLS = TMEM_RAW < 32 ? 32 : TMEM_RAW;
    static_assert((TMEM_COLS & (TMEM_COLS - 1)) == 0 && TMEM_COLS <= 512, "TMEM allocation");
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static_assert(X_STAGE % 1024 == 0 && R_STAGE % 128 == 0, "stage alignment");
};

}  // namespace

template <int FMT, int NT, int NR, int NA, int NX, int ACC, bool DOWN>
__global__ void __launch_bounds__(TCL<FMT, NT, NR, NA, NX, ACC, DOWN>::THREADS, 1)
    k_experts_tc(const __grid_constant__ ExpArgs a) {
    using L = TCL<FMT, NT, NR, NA, NX, ACC, DOWN>;
    pdl_launch();
    extern __shared__ __align__(1024) unsigned char tsm_raw[];
    // 1024-byte aligned base for the swizzled tiles
    unsigned char *tsm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(tsm_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char *Ab = tsm, *Xb = tsm + L::OFF_X, *Rb = tsm + L::OFF_R;
    uint64_t *rfull = reinterpret_cast<uint64_t *>(tsm + L::OFF_BAR);
    uint64_t *rempty = rfull + NR, *afull = rempty + NR, *aempty = afull + NA, *xfull = aempty + NA,
             *xempty = xfull + NX, *accf = xempty + NX, *acce = accf + ACC;
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int RB = DOWN ? (a.d >> 4) : (a.f >> 4);     // 16-row blocks of the output rows
    const int G = DOWN ? (a.f >> 6) : (a.d >> 6);      // 64-groups of K
    const int MT = RB / 8;                             // 128-row work items per tile
    if (threadIdx.x == 0) {
        for (int i = 0; i < NR; ++i) {
            mbar_init(rfull + i, 1);
            mbar_init(rempty + i, L::DQW);
        }
        for (int i = 0; i < NA; ++i) {
            mbar_init(afull + i, L::DQW);
            mbar_init(aempty + i, 1);
        }
        for (int i = 0; i < NX; ++i) {
            mbar_init(xfull + i, 1);
            mbar_init(xempty + i, 1);
        }
        for (int b = 0; b < ACC; ++b) {
            mbar_init(accf + b, 1);
            mbar_init(acce + b, L::EPW);
        }
        mbar_fence_init();
        s_fail = 0;
    }
    if (warp == 1) {  // TMEM: ACC accumulator sets of NP x NT fp32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"((uint32_t)L::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pdl_wait();  // barrier setup and the TMEM allocation above overlap the upstream kernel's tail
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const int n_tiles = *a.ntiles;
    const int n_items = n_tiles * MT;
    const int my_items = (int)blockIdx.x < n_items ? (n_items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    const int m0 = DOWN ? 2 : 0;  // tensor maps of this kernel's projections
    const unsigned timeout_err = ERR_TIMEOUT;

    if (warp == 0) {
        // ------------------------------------------------------------ raw producer (codes + scales, from HBM)
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            for (int p = 0; p < L::NP; ++p) {
                tmap_prefetch(&a.tmq[m0 + p]);
                tmap_prefetch(&a.tmsb[m0 + p]);
            }
            int k = 0;
            bool ok = true;
            int4 tr_n = my_items > 0 ? item_tile(a, 0, MT) : make_int4(0, 0, 0, 0);
            for (int it = 0; it < my_items && ok; ++it) {
                const int item = (int)blockIdx.x + it * (int)gridDim.x;
                const int tile = item / MT, mt = item - tile * MT;
                const int4 tr = tr_n;
                if (it + 1 < my_items) tr_n = item_tile(a, it + 1, MT);
                const int e = (tr.x < 0 || tr.x >= a.E) ? 0 : tr.x;
                const int row0 = e * RB + mt * 8;
                for (int g = 0; g < G; ++g, ++k) {
                    const int r = k % NR;
                    if (k >= NR && !mbar_wait_bounded(rempty + r, (unsigned)(((k / NR) - 1) & 1))) {
                        atomicOr(a.err, timeout_err);
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    unsigned char *q = Rb + (size_t)r * L::R_STAGE;
                    mbar_expect_tx(rfull + r, (unsigned)L::R_STAGE);
                    for (int p = 0; p < L::NP; ++p) {
                        tma_load_2d(q + p * L::Q_BYTES, &a.tmq[m0 + p], g * 64, row0, rfull + r, pol);
                        tma_load_2d(q + L::NP * L::Q_BYTES + p * L::S_BYTES, &a.tmsb[m0 + p], g * (L::SBG / 4), row0,
                                    rfull + r, pol);
                    }
                }
            }
            // let the copies this CTA issued land before it can exit (bounded)
            for (int q = k - NR; q < k; ++q)
                if (q >= 0) mbar_wait_bounded(rfull + q % NR, (unsigned)((q / NR) & 1), 1u << 16);
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ X producer (the tile's activation rows, L2)
        if (lane == 0) {
            const uint64_t pol_x = l2_evict_last_policy();  // re-read for every 128-row item of the tile
            tmap_prefetch(&a.tmx);
            int k = 0;
            bool ok = true;
            int4 tr_n = my_items > 0 ? item_tile(a, 0, MT) : make_int4(0, 0, 0, 0);
            for (int it = 0; it < my_items && ok; ++it) {
                const int4 tr = tr_n;
                if (it + 1 < my_items) tr_n = item_tile(a, it + 1, MT);
                for (int g = 0; g < G; ++g, ++k) {
                    const int x = k % NX;
                    if (k >= NX && !mbar_wait_bounded(xempty + x, (unsigned)(((k / NX) - 1) & 1))) {
                        atomicOr(a.err, timeout_err);
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(xfull + x, (unsigned)L::X_STAGE);
                    tma_load_2d(Xb + (size_t)x * L::X_STAGE, &a.tmx, g * 64, tr.y, xfull + x, pol_x);
                }
            }
            for (int q = k - NX; q < k; ++q)
                if (q >= 0) mbar_wait_bounded(xfull + q % NX, (unsigned)((q / NX) & 1), 1u << 16);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int k = 0;
            bool ok = true;
            int4 tr_n = my_items > 0 ? item_tile(a, 0, MT) : make_int4(0, 0, 0, 0);
            for (int it = 0; it < my_items && ok; ++it) {
                const int b = it % ACC, use = it / ACC;  // accumulator set and how often it was used before
                const int nslot = tr_n.z;
                if (it + 1 < my_items) tr_n = item_tile(a, it + 1, MT);
                // MMA width: the tile's slots rounded up to 16 (columns past them are never read)
                const uint32_t idesc = idesc_bf16(TC_M, min(NT, max(16, (nslot + 15) & ~15)));
                if (use >= 1 && !mbar_wait_bounded(acce + b, (unsigned)((use - 1) & 1))) {
                    atomicOr(a.err, timeout_err);
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                for (int g = 0; g < G; ++g, ++k) {
                    const int sa = k % NA, sx = k % NX;
                    if (!mbar_wait_bounded(afull + sa, (unsigned)((k / NA) & 1)) ||
                        !mbar_wait_bounded(xfull + sx, (unsigned)((k / NX) & 1))) {
                        atomicOr(a.err, timeout_err);
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bdesc = sdesc_sw128(smem_u32(Xb + (size_t)sx * L::X_STAGE));
#pragma unroll
                    for (int p = 0; p < L::NP; ++p) {
                        const uint64_t adesc = sdesc_sw128(smem_u32(Ab + (size_t)sa * L::A_STAGE + p * L::A_BYTES));
                        const uint32_t d_tmem = tmem + (uint32_t)((b * L::NP + p) * NT);
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks)  // 16 k = 32 bytes along the swizzled row: +2 in 16-byte units
                            umma_bf16(d_tmem, adesc + 2 * ks, bdesc + 2 * ks, idesc, (g > 0 || ks > 0) ? 1u : 0u);
                    }
                    umma_commit(aempty + sa);  // both stages are free once these MMAs have read them
                    umma_commit(xempty + sx);
                }
                if (ok) umma_commit(accf + b);
            }
            // MMAs still in flight finish before TMEM is released (bounded)
            if (k > 0) mbar_wait_bounded(aempty + (k - 1) % NA, (unsigned)(((k - 1) / NA) & 1), 1u << 16);
        }
    } else if (warp < 3 + L::DQW) {
        // ------------------------------------------------------------ dequant (one (projection, row block) each)
        const int dw = warp - 3;
        const int p = dw >> 3, rb = dw & 7;
        const int gq = lane >> 2, c = lane & 3;
        int k = 0;
        for (int it = 0; it < my_items && !*reinterpret_cast<volatile int *>(&s_fail); ++it) {
            bool ok = true;
            for (int g = 0; g < G; ++g, ++k) {
                const int r = k % NR, sa = k % NA;
                if (!mbar_wait_bounded(rfull + r, (unsigned)((k / NR) & 1))) {
                    if (lane == 0) atomicOr(a.err, timeout_err);
                    ok = false;
                    break;
                }
                const unsigned char *q = Rb + (size_t)r * L::R_STAGE;
                const uint4 w = reinterpret_cast<const uint4 *>(q + p * L::Q_BYTES + rb * 512)[lane];
                const uint32_t *sbw = reinterpret_cast<const uint32_t *>(q + L::NP * L::Q_BYTES + p * L::S_BYTES + rb * L::SBG);
                uint32_t sbv[2];
                if (FMT == FMT_FP4) {
                    sbv[0] = sbw[gq];
                    sbv[1] = 0;
                } else {
                    sbv[0] = sbw[gq * 2];
                    sbv[1] = sbw[gq * 2 + 1];
                }
                if (k >= NA && !mbar_wait_bounded(aempty + sa, (unsigned)(((k / NA) - 1) & 1))) {
                    if (lane == 0) atomicOr(a.err, timeout_err);
                    ok = false;
                    break;
                }
                unsigned char *A = Ab + (size_t)sa * L::A_STAGE + p * L::A_BYTES;
                uint32_t out[2][8];
                dequant_block<FMT>(w, sbv[0], sbv[1], c, out);
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {  // rows gq and gq + 8
                    const int rr = rb * 16 + gq + 8 * hf;
                    // elements 16c .. 16c+15 of row rr = chunks 2c, 2c+1 (16 B each), swizzled by rr % 8
                    uint4 *row = reinterpret_cast<uint4 *>(A + rr * 128);
                    row[(2 * c) ^ (rr & 7)] = make_uint4(out[hf][0], out[hf][1], out[hf][2], out[hf][3]);
                    row[(2 * c + 1) ^ (rr & 7)] = make_uint4(out[hf][4], out[hf][5], out[hf][6], out[hf][7]);
                }
                fence_async_smem();  // generic-proxy writes of A -> the tensor core's reads
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive1(afull + sa);
                    mbar_arrive1(rempty + r);  // the raw stage was consumed (its values are in A)
                }
            }
            if (!ok) {
                s_fail = 1;
                break;
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (TMEM lane quarter warp % 4)
        const int ew = warp - 3 - L::DQW;
        const int quarter = warp & 3;
        constexpr int HALVES = L::EPW / 4;  // warps sharing a quarter split the columns
        const int half = ew >> 2;
        for (int it = 0; it < my_items && !*reinterpret_cast<volatile int *>(&s_fail); ++it) {
            const int item = (int)blockIdx.x + it * (int)gridDim.x;
            const int tile = item / MT, mt = item - tile * MT;
            const int4 tr = a.tiles[tile];
            const int e = (tr.x < 0 || tr.x >= a.E) ? 0 : tr.x;
            const int b = it % ACC;
            constexpr int NCH = DOWN ? NT / (16 * HALVES) : 1;
            int msl[NCH];
            float mw[NCH];
            if (DOWN) down_epi_meta<NCH>(a, tr, 16 * half, 16 * HALVES, lane, msl, mw);
            if (!mbar_wait_bounded(accf + b, (unsigned)((it / ACC) & 1))) {
                if (lane == 0) atomicOr(a.err, timeout_err);
                break;
            }
            tc_fence_after();
            const int row = mt * TC_M + quarter * 32 + lane;  // output row (f for gate/up, d for down)
            const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16);
            // this warp's columns: 16-column chunks half, half + HALVES, ... below the tile's slot count
            if (!DOWN) {
                const float bgr = a.bg ? a.bg[(size_t)e * a.f + row] : 0.f, bur = a.bu ? a.bu[(size_t)e * a.f + row] : 0.f;
                const int hrow = a.h_kperm ? kperm64(row) : row;  // the down kernel's k order
                for (int c0 = 16 * half; c0 < tr.z; c0 += 16 * HALVES) {
                    float gv[16], uv[16];
                    tmem_ld16(tl + (uint32_t)((b * 2 + 0) * NT + c0), gv);
                    tmem_ld16(tl + (uint32_t)((b * 2 + 1) * NT + c0), uv);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = c0 + j;
                        if (n < tr.z) a.h[(size_t)(tr.y + n) * a.f + hrow] = f2bf(act_glu(a.act, gv[j] + bgr, uv[j] + bur));
                    }
                }
            } else {
                const float bdr = a.bd ? a.bd[(size_t)e * a.d + row] : 0.f;
#pragma unroll
                for (int q = 0; q < NCH; ++q) {
                    const int c0 = 16 * half + q * 16 * HALVES;
                    if (c0 >= tr.z) break;
                    float dv[16];
                    tmem_ld16(tl + (uint32_t)(b * NT + c0), dv);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int slot = __shfl_sync(0xffffffffu, msl[q], j);
                        const float wsl = __shfl_sync(0xffffffffu, mw[q], j);
                        if (c0 + j < tr.z) slot_row(a, slot)[row] = wsl * (dv[j] + bdr);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive1(acce + b);
        }
        if (DOWN && a.ypeers) __threadfence_system();  // peer stores visible before the signal kernel runs
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)L::TMEM_COLS)
                     : "memory");
    }
}


// ==================================================================== A operand in tensor memory
// The same work decomposition with the dequantized weights written straight into TMEM (tcgen05.st) instead of
// shared memory: no shared-memory stores or reads of A, no proxy fence. Rings:
//   raw ring (NR stages): packed codes + scales from HBM (as above);
//   operand ring (NS stages): the A tile in TMEM columns and the X tile in shared memory share one "ofull"
//     barrier (DQW dequant arrivals + the X copy's transaction bytes) and one "oempty" (MMA commit).
// The 16x256b TMEM store gives lane 4i + j of a warp columns 8m + 2j, 8m + 2j + 1 of rows i, i + 8, while the
// int4 fragment gives it k = 16j .. 16j + 15. So inside every 64-group the operands use the k order
// "position 16a + 4b + r holds k = 16b + 4a + r" (a digit swap, its own inverse): A by where the lanes store,
// X by the gather that builds the expert-sorted rows, h by the gate/up epilogue that writes it (h_kperm). The
// MMA sums over k, so the order does not change the products, only which bf16 pairs meet in the tensor core.

namespace {
template <int FMT, int NT, int NR, int NS, int ACC, bool DOWN, int SGK>
struct TAL {
    static constexpr int NP = DOWN ? 1 : 2;
    static constexpr int DQW = 8 * NP;                   // dequant warps: one (projection, row block) each
    static constexpr int EPW = 8;                        // epilogue warps (two per TMEM lane quarter)
    static constexpr int THREADS = 32 * (3 + DQW + EPW);
    static constexpr int SBG = FMT == FMT_FP4 ? 32 : 64;
    static constexpr int X_SUB = NT * 128;               // one 64-group of the tile's activation rows
    static constexpr int X_STAGE = SGK * X_SUB;
    static constexpr int Q_BYTES = 8 * 512;              // per group: 8 row blocks of packed codes
    static constexpr int S_BYTES = 8 * SBG;
    static constexpr int R_STAGE = NP * SGK * (Q_BYTES + S_BYTES);
    static constexpr int OFF_R = NS * X_STAGE;
    static constexpr int OFF_BAR = OFF_R + NR * R_STAGE;
    static constexpr int NBAR = 2 * (NR + NS + ACC);
    static constexpr int SMEM = 1024 + OFF_BAR + NBAR * 8;
    static constexpr int A_COL0 = ACC * NP * NT;         // accumulators first, then the A stages (32 columns each)
    static constexpr int TMEM_RAW = A_COL0 + NS * NP * SGK * 32;
    static constexpr int TMEM_COLS = TMEM_RAW <= 32 ? 32 : TMEM_RAW <= 64 ? 64 : TMEM_RAW <= 128 ? 128
                                   : TMEM_RAW <= 256 ? 256 : 512;
    static_assert(TMEM_RAW <= 512, "TMEM allocation");
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static_assert(X_STAGE % 1024 == 0 && R_STAGE % 128 == 0, "stage alignment");
};
}  // namespace

template <int FMT, int NT, int NR, int NS, int ACC, bool DOWN, int SGK>
__global__ void __launch_bounds__(TAL<FMT, NT, NR, NS, ACC, DOWN, SGK>::THREADS, 1)
    k_experts_tca(const __grid_constant__ ExpArgs a) {
    using L = TAL<FMT, NT, NR, NS, ACC, DOWN, SGK>;
    pdl_launch();
    extern __shared__ __align__(1024) unsigned char tsm_raw[];
    unsigned char *tsm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(tsm_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char *Xb = tsm, *Rb = tsm + L::OFF_R;
    uint64_t *rfull = reinterpret_cast<uint64_t *>(tsm + L::OFF_BAR);
    uint64_t *rempty = rfull + NR, *ofull = rempty + NR, *oempty = ofull + NS, *accf = oempty + NS, *acce = accf + ACC;
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int RB = DOWN ? (a.d >> 4) : (a.f >> 4);
    const int GS = (DOWN ? (a.f >> 6) : (a.d >> 6)) / SGK;  // stages per item (SGK groups each; G % SGK == 0)
    const int MT = RB / 8;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NR; ++i) {
            mbar_init(rfull + i, 1);
            mbar_init(rempty + i, L::DQW);
        }
        for (int i = 0; i < NS; ++i) {
            mbar_init(ofull + i, L::DQW + 1);
            mbar_init(oempty + i, 1);
        }
        for (int b = 0; b < ACC; ++b) {
            mbar_init(accf + b, 1);
            mbar_init(acce + b, L::EPW);
        }
        mbar_fence_init();
        s_fail = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"((uint32_t)L::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pdl_wait();  // barrier setup and the TMEM allocation above overlap the upstream kernel's tail
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const int n_tiles = *a.ntiles;
    const int n_items = n_tiles * MT;
    const int my_items = (int)blockIdx.x < n_items ? (n_items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    const int m0 = DOWN ? 2 : 0;
    const unsigned timeout_err = ERR_TIMEOUT;

    if (warp == 0) {
        // ------------------------------------------------------------ raw producer (codes + scales, from HBM)
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            for (int p = 0; p < L::NP; ++p) {
                tmap_prefetch(&a.tmq[m0 + p]);
                tmap_prefetch(&a.tmsb[m0 + p]);
            }
            int k = 0;
            bool ok = true;
            int4 tr_n = my_items > 0 ? item_tile(a, 0, MT) : make_int4(0, 0, 0, 0);
            for (int it = 0; it < my_items && ok; ++it) {
                const int item = (int)blockIdx.x + it * (int)gridDim.x;
                const int tile = item / MT, mt = item - tile * MT;
                const int4 tr = tr_n;
                if (it + 1 < my_items) tr_n = item_tile(a, it + 1, MT);
                const int e = (tr.x < 0 || tr.x >= a.E) ? 0 : tr.x;
                const int row0 = e * RB + mt * 8;
                for (int gs = 0; gs < GS; ++gs, ++k) {
                    const int r = k % NR, g = gs * SGK;
                    if (k >= NR && !mbar_wait_bounded(rempty + r, (unsigned)(((k / NR) - 1) & 1))) {
                        atomicOr(a.err, timeout_err);
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    unsigned char *q = Rb + (size_t)r * L::R_STAGE;
                    mbar_expect_tx(rfull + r, (unsigned)L::R_STAGE);
                    for (int p = 0; p < L::NP; ++p) {  // boxes of 8 row blocks x SGK groups
                        tma_load_2d(q + p * SGK * L::Q_BYTES, &a.tmq[m0 + p], g * 64, row0, rfull + r, pol);
                        tma_load_2d(q + L::NP * SGK * L::Q_BYTES + p * SGK * L::S_BYTES, &a.tmsb[m0 + p],
                                    g * (L::SBG / 4), row0, rfull + r, pol);
                    }
                }
            }
            for (int q = k - NR; q < k; ++q)
                if (q >= 0) mbar_wait_bounded(rfull + q % NR, (unsigned)((q / NR) & 1), 1u << 16);
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ X producer (operand stage's B half, from L2)
        if (lane == 0) {
            const uint64_t pol_x = l2_evict_last_policy();
            tmap_prefetch(&a.tmx);
            int k = 0;
            bool ok = true;
            int4 tr_n = my_items > 0 ? item_tile(a, 0, MT) : make_int4(0, 0, 0, 0);
            for (int it = 0; it < my_items && ok; ++it) {
                const int4 tr = tr_n;
                if (it + 1 < my_items) tr_n = item_tile(a, it + 1, MT);
                for (int gs = 0; gs < GS; ++gs, ++k) {
                    const int s = k % NS;
                    if (k >= NS && !mbar_wait_bounded(oempty + s, (unsigned)(((k / NS) - 1) & 1))) {
                        atomicOr(a.err, timeout_err);
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(ofull + s, (unsigned)L::X_STAGE);
                    for (int gi = 0; gi < SGK; ++gi)
                        tma_load_2d(Xb + (size_t)s * L::X_STAGE + gi * L::X_SUB, &a.tmx, (gs * SGK + gi) * 64, tr.y,
                                    ofull + s, pol_x);
                }
            }
            for (int q = k - NS; q < k; ++q)
                if (q >= 0) mbar_wait_bounded(ofull + q % NS, (unsigned)((q / NS) & 1), 1u << 16);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int k = 0;
            bool ok = true;
            int4 tr_n = my_items > 0 ? item_tile(a, 0, MT) : make_int4(0, 0, 0, 0);
            for (int it = 0; it < my_items && ok; ++it) {
                const int b = it % ACC, use = it / ACC;
                const int nslot = tr_n.z;
                if (it + 1 < my_items) tr_n = item_tile(a, it + 1, MT);
                const uint32_t idesc = idesc_bf16(TC_M, min(NT, max(16, (nslot + 15) & ~15)));
                if (use >= 1 && !mbar_wait_bounded(acce + b, (unsigned)((use - 1) & 1))) {
                    atomicOr(a.err, timeout_err);
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                for (int gs = 0; gs < GS; ++gs, ++k) {
                    const int s = k % NS;
                    if (!mbar_wait_bounded(ofull + s, (unsigned)((k / NS) & 1))) {
                        atomicOr(a.err, timeout_err);
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int gi = 0; gi < SGK; ++gi) {
                        const uint64_t bdesc = sdesc_sw128(smem_u32(Xb + (size_t)s * L::X_STAGE + gi * L::X_SUB));
#pragma unroll
                        for (int p = 0; p < L::NP; ++p) {
                            const uint32_t d_tmem = tmem + (uint32_t)((b * L::NP + p) * NT);
                            const uint32_t a_tmem = tmem + (uint32_t)(L::A_COL0 + ((s * L::NP + p) * SGK + gi) * 32);
#pragma unroll
                            for (int ks = 0; ks < 4; ++ks)  // 16 k = 8 TMEM columns of A, 32 bytes of the X row
                                umma_bf16_ts(d_tmem, a_tmem + 8 * ks, bdesc + 2 * ks, idesc,
                                             (gs > 0 || gi > 0 || ks > 0) ? 1u : 0u);
                        }
                    }
                    umma_commit(oempty + s);
                }
                if (ok) umma_commit(accf + b);
            }
            if (k > 0) mbar_wait_bounded(oempty + (k - 1) % NS, (unsigned)(((k - 1) / NS) & 1), 1u << 16);
        }
    } else if (warp < 3 + L::DQW) {
        // ------------------------------------------------------------ dequant: warp -> (projection, row block)
        // whose 16 rows lie in its TMEM lane quarter (warp % 4)
        const int i = warp - 3, quarter = warp & 3, j = i >> 2;
        const int p = L::NP == 2 ? (j >> 1) : 0, rb = 2 * quarter + (j & 1);
        const int gq = lane >> 2, c = lane & 3;
        const uint32_t lane_addr = (uint32_t)(rb * 16) << 16;
        int k = 0;
        for (int it = 0; it < my_items && !*reinterpret_cast<volatile int *>(&s_fail); ++it) {
            bool ok = true;
            for (int gs = 0; gs < GS; ++gs, ++k) {
                const int r = k % NR, s = k % NS;
                if (!mbar_wait_bounded(rfull + r, (unsigned)((k / NR) & 1))) {
                    if (lane == 0) atomicOr(a.err, timeout_err);
                    ok = false;
                    break;
                }
                const unsigned char *q = Rb + (size_t)r * L::R_STAGE;
                uint32_t out[SGK][2][8];
#pragma unroll
                for (int gi = 0; gi < SGK; ++gi) {  // this warp's block of each of the stage's groups
                    const uint4 w = reinterpret_cast<const uint4 *>(q + p * SGK * L::Q_BYTES + rb * (SGK * 512) + gi * 512)[lane];
                    const uint32_t *sbw = reinterpret_cast<const uint32_t *>(q + L::NP * SGK * L::Q_BYTES + p * SGK * L::S_BYTES +
                                                                             rb * (SGK * L::SBG) + gi * L::SBG);
                    const uint32_t sb0 = FMT == FMT_FP4 ? sbw[gq] : sbw[gq * 2], sb1 = FMT == FMT_FP4 ? 0u : sbw[gq * 2 + 1];
                    dequant_block<FMT>(w, sb0, sb1, c, out[gi]);
                }
                __syncwarp();  // every lane's reads of the raw stage are complete (their values are in out)
                if (lane == 0) mbar_arrive1(rempty + r);
                if (k >= NS && !mbar_wait_bounded(oempty + s, (unsigned)(((k / NS) - 1) & 1))) {
                    if (lane == 0) atomicOr(a.err, timeout_err);
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int gi = 0; gi < SGK; ++gi) {
                    uint32_t v[16];
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        v[4 * m + 0] = out[gi][0][2 * m];
                        v[4 * m + 1] = out[gi][0][2 * m + 1];
                        v[4 * m + 2] = out[gi][1][2 * m];
                        v[4 * m + 3] = out[gi][1][2 * m + 1];
                    }
                    tmem_st_16x256_x4(tmem + lane_addr + (uint32_t)(L::A_COL0 + ((s * L::NP + p) * SGK + gi) * 32), v);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive1(ofull + s);
            }
            if (!ok) {
                s_fail = 1;
                break;
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (TMEM lane quarter warp % 4)
        const int ew = warp - 3 - L::DQW;
        const int quarter = warp & 3;
        constexpr int HALVES = L::EPW / 4;
        const int half = ew >> 2;
        for (int it = 0; it < my_items && !*reinterpret_cast<volatile int *>(&s_fail); ++it) {
            const int item = (int)blockIdx.x + it * (int)gridDim.x;
            const int tile = item / MT, mt = item - tile * MT;
            const int4 tr = a.tiles[tile];
            const int e = (tr.x < 0 || tr.x >= a.E) ? 0 : tr.x;
            const int b = it % ACC;
            constexpr int NCH = DOWN ? NT / (16 * HALVES) : 1;
            int msl[NCH];
            float mw[NCH];
            if (DOWN) down_epi_meta<NCH>(a, tr, 16 * half, 16 * HALVES, lane, msl, mw);
            if (!mbar_wait_bounded(accf + b, (unsigned)((it / ACC) & 1))) {
                if (lane == 0) atomicOr(a.err, timeout_err);
                break;
            }
            tc_fence_after();
            const int row = mt * TC_M + quarter * 32 + lane;
            const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16);
            if (!DOWN) {
                const float bgr = a.bg ? a.bg[(size_t)e * a.f + row] : 0.f, bur = a.bu ? a.bu[(size_t)e * a.f + row] : 0.f;
                const int hrow = a.h_kperm ? kperm64(row) : row;
                for (int c0 = 16 * half; c0 < tr.z; c0 += 16 * HALVES) {
                    float gv[16], uv[16];
                    tmem_ld16(tl + (uint32_t)((b * 2 + 0) * NT + c0), gv);
                    tmem_ld16(tl + (uint32_t)((b * 2 + 1) * NT + c0), uv);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int n = c0 + jj;
                        if (n < tr.z) a.h[(size_t)(tr.y + n) * a.f + hrow] = f2bf(act_glu(a.act, gv[jj] + bgr, uv[jj] + bur));
                    }
                }
            } else {
                const float bdr = a.bd ? a.bd[(size_t)e * a.d + row] : 0.f;
#pragma unroll
                for (int q = 0; q < NCH; ++q) {
                    const int c0 = 16 * half + q * 16 * HALVES;
                    if (c0 >= tr.z) break;
                    float dv[16];
                    tmem_ld16(tl + (uint32_t)(b * NT + c0), dv);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int slot = __shfl_sync(0xffffffffu, msl[q], jj);
                        const float wsl = __shfl_sync(0xffffffffu, mw[q], jj);
                        if (c0 + jj < tr.z) slot_row(a, slot)[row] = wsl * (dv[jj] + bdr);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive1(acce + b);
        }
        if (DOWN && a.ypeers) __threadfence_system();  // peer stores visible before the signal kernel runs
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)L::TMEM_COLS)
                     : "memory");
    }
}

// Configurations. TMEM-operand kernels (k_experts_tca) wherever their accumulators and A stages fit the 512
// TMEM columns: gate/up tiles of 32 / 64 / 128 / 192 slots (192: one accumulator set of 2 x 192 columns and two
// single-group A stages fill the 512), down tiles of 32 .. 256. Gate/up tiles of 256 need all 512 columns for the
// two accumulators and keep A in shared memory (k_experts_tc). Raw and operand rings are as deep
// as the 227 KB of shared memory allow.
//   tca: (NT, NR, NS, ACC, DOWN, SGK): SGK 64-groups per stage (two halve the per-stage barrier, TMEM-store and
//   MMA-issue latencies per group and fetch 1 KB code rows per copy); down tiles of 256 keep one, as their
//   64 KB activation stages leave no room for a deep raw ring
#define MOEB_TCA_CFGS(X) \
    X(32, 10, 3, 2, false, 2) X(64, 10, 2, 2, false, 2) X(128, 8, 2, 1, false, 2) X(192, 16, 2, 1, false, 1) \
    X(32, 16, 6, 2, true, 2) X(64, 12, 6, 2, true, 2) X(128, 10, 4, 2, true, 2) X(192, 16, 4, 2, true, 1) \
    X(256, 16, 4, 1, true, 1)

TcInfo experts_tc_info(int fmt, int nt, bool down) {
    TcInfo r = {nullptr, 0, 0, false, 1};
#define MOEB_TCA_PICK(NT_, NR_, NS_, ACC_, DOWN_, SGK_)                                                         \
    if (nt == NT_ && down == DOWN_) {                                                                           \
        if (fmt == FMT_FP4) {                                                                                   \
            using L = TAL<FMT_FP4, NT_, NR_, NS_, ACC_, DOWN_, SGK_>;                                            \
            r = {k_experts_tca<FMT_FP4, NT_, NR_, NS_, ACC_, DOWN_, SGK_>, L::THREADS, (size_t)L::SMEM, true, SGK_}; \
        } else {                                                                                                \
            using L = TAL<FMT_Q4, NT_, NR_, NS_, ACC_, DOWN_, SGK_>;                                             \
            r = {k_experts_tca<FMT_Q4, NT_, NR_, NS_, ACC_, DOWN_, SGK_>, L::THREADS, (size_t)L::SMEM, true, SGK_};  \
        }                                                                                                       \
    }
    MOEB_TCA_CFGS(MOEB_TCA_PICK)
#undef MOEB_TCA_PICK
    if (nt == 256 && !down) {
        if (fmt == FMT_FP4) {
            using L = TCL<FMT_FP4, 256, 6, 2, 3, 1, false>;
            r = {k_experts_tc<FMT_FP4, 256, 6, 2, 3, 1, false>, L::THREADS, (size_t)L::SMEM, false, 1};
        } else {
            using L = TCL<FMT_Q4, 256, 6, 2, 3, 1, false>;
            r = {k_experts_tc<FMT_Q4, 256, 6, 2, 3, 1, false>, L::THREADS, (size_t)L::SMEM, false, 1};
        }
    }
    return r;
}

// x rows of the slots in expert-sorted order (the activation operand of the tensor-core gate/up); perm: in the
// 64-group k order of the TMEM-operand kernels (8-byte chunks of 4 k: chunk 4b + a goes to 4a + b)
__global__ void __launch_bounds__(256) k_gather_rows(const uint16_t *__restrict__ x, const int *__restrict__ sorted,
                                                     int TK, int k, int d, int xstride, int perm,
                                                     uint16_t *__restrict__ xs) {
    pdl_launch();
    pdl_wait();
    const int i = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (i >= TK) return;
    if (!perm) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)(sorted[i] / k) * xstride);
        uint4 *dst = reinterpret_cast<uint4 *>(xs + (size_t)i * d);
        for (int c = lane; c < d / 8; c += 32) dst[c] = src[c];
    } else {
        const uint2 *src = reinterpret_cast<const uint2 *>(x + (size_t)(sorted[i] / k) * xstride);
        uint2 *dst = reinterpret_cast<uint2 *>(xs + (size_t)i * d);
        for (int c = lane; c < d / 4; c += 32) {
            const int u = c & 15;
            dst[(c & ~15) | ((u & 3) << 2) | (u >> 2)] = src[c];
        }
    }
}

}  // namespace moeb
