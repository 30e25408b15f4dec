// Grouped expert kernels on the 5th-generation tensor cores (tcgen05, accumulators in TMEM), for high loads
// (tiles of up to NT = 256 slots of one expert: the weights are dequantized once per tile).
//
// A work item is (tile, 128 output rows). D[128 rows][NT slots] = W[128][K] . X[NT][K]^T accumulates in TMEM
// (fp32, lane = row, column = slot). K streams through an NS-deep shared-memory ring, one 64-group per stage:
//   warp 0 (producer, one lane): per stage, 2-D tensor copies of the packed int4 codes and scale|bias words of
//     the 8 row blocks (one group; per projection) and of the tile's activation rows (64 k, NT rows, 128-byte
//     swizzle: the UMMA K-major layout); "full" mbarrier with transaction bytes. No multicast.
//   warps 2..9 (dequant): int4 -> bf16 w = s*q + b (q|0x4300 = 128+q exactly; one HSUB2 and one HFMA2, a single
//     bf16 rounding), written into the stage's A tile in the same swizzled K-major layout; then a proxy fence
//     (generic writes -> tensor-core reads) and one arrival per warp on the stage's "deq" mbarrier.
//   warp 1 (MMA, one lane): waits "deq", issues 4 k-steps of tcgen05.mma (M = 128, N = the tile's slot count
//     rounded up to 16, K = 16, bf16 x bf16 -> fp32) per projection, and tcgen05.commit frees the stage ("empty"); after the last group it commits the
//     item's accumulator ("accf"). With two accumulator sets (down) the next item's MMAs run while the epilogue
//     drains the previous one; gate/up's two projections of 256 columns fill TMEM, so it has one set (the
//     epilogue is a few percent of an item's K loop).
//   warps 10..13 (epilogue): tcgen05.ld 16 columns at a time (warp w reads TMEM lanes 32*(w%4)..+31 = its rows);
//     gate/up: bias + activation -> h in slot-sorted order; down: weight * (acc + bias) -> the slot's fp32 row
//     for the separate combine pass. Then "acce" frees the accumulator set.
// The activations arrive in expert-sorted order (x gathered by k_gather_rows; gate/up writes h sorted), so each
// tile's rows are contiguous for the tensor copy. Weights are dequantized once per tile, so the kernel pays off
// once tiles hold many slots; the dispatcher uses it from 64 slots per expert on.
// Every wait is bounded (timeout -> MOEB_DEVERR_TIMEOUT, the roles stop, in-flight copies and MMAs are drained
// with bounded waits, TMEM is released).
#include "experts_common.cuh"

namespace moeb {

namespace {

constexpr int TC_M = 128;
constexpr int TC_DQW = 8;                       // dequant warps
constexpr int TC_THREADS = 32 * (2 + TC_DQW + 4);  // producer, MMA, dequant, 4 epilogue warps

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

template <int FMT, int NT, int ACC, bool DOWN>
struct TCL {
    static constexpr int NP = DOWN ? 1 : 2;
    static constexpr int SBG = FMT == FMT_FP4 ? 32 : 64;  // scale bytes per (row block, group)
    static constexpr int A_BYTES = TC_M * 128;         // one projection's 128 rows x 64 k, bf16, swizzled
    static constexpr int X_BYTES = NT * 128;           // NT rows x 64 k
    static constexpr int Q_BYTES = 8 * 512;            // packed codes, 8 row blocks x one group
    static constexpr int S_BYTES = 8 * SBG;            // int4 scale|bias words / MXFP4 E8M0 bytes
    static constexpr int STAGE_RAW = NP * A_BYTES + X_BYTES + NP * (Q_BYTES + S_BYTES);
    static constexpr int STAGE = (STAGE_RAW + 1023) / 1024 * 1024;
    static constexpr int TMEM_COLS = ACC * NP * NT;    // ACC accumulator sets
    static_assert(TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM allocation");
};

}  // namespace

template <int FMT, int NT, int NS, int ACC, bool DOWN>
__global__ void __launch_bounds__(TC_THREADS, 1) k_experts_tc(const __grid_constant__ ExpArgs a) {
    using L = TCL<FMT, NT, ACC, DOWN>;
    pdl_launch();
    pdl_wait();
    extern __shared__ __align__(1024) unsigned char tsm_raw[];
    // 1024-byte aligned base for the swizzled tiles
    unsigned char *tsm = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(tsm_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *full = reinterpret_cast<uint64_t *>(tsm + (size_t)NS * L::STAGE);
    uint64_t *deq = full + NS, *empty = deq + NS, *accf = empty + NS, *acce = accf + ACC;
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int RB = DOWN ? (a.d >> 4) : (a.f >> 4);     // 16-row blocks of the output rows
    const int G = DOWN ? (a.f >> 6) : (a.d >> 6);      // 64-groups of K
    const int MT = RB / 8;                             // 128-row work items per tile
    const int n_tiles = *a.ntiles;
    const int n_items = n_tiles * MT;
    const int my_items = (int)blockIdx.x < n_items ? (n_items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(full + i, 1);
            mbar_init(deq + i, TC_DQW);
            mbar_init(empty + i, 1);
        }
        for (int b = 0; b < ACC; ++b) {
            mbar_init(accf + b, 1);
            mbar_init(acce + b, 4);
        }
        mbar_fence_init();
        s_fail = 0;
    }
    if (warp == 1) {  // TMEM: two accumulator sets of NP x NT fp32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"((uint32_t)L::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const int m0 = DOWN ? 2 : 0;  // tensor maps of this kernel's projections
    const unsigned timeout_err = ERR_TIMEOUT;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy(), pol_x = l2_evict_last_policy();  // x is re-read per row tile
            for (int p = 0; p < L::NP; ++p) {
                tmap_prefetch(&a.tmq[m0 + p]);
                tmap_prefetch(&a.tmsb[m0 + p]);
            }
            tmap_prefetch(&a.tmx);
            int k = 0;
            bool ok = true;
            for (int it = 0; it < my_items && ok; ++it) {
                const int item = (int)blockIdx.x + it * (int)gridDim.x;
                const int tile = item / MT, mt = item - tile * MT;
                const int4 tr = a.tiles[tile];
                const int e = (tr.x < 0 || tr.x >= a.E) ? 0 : tr.x;
                const int row0 = e * RB + mt * 8;
                for (int g = 0; g < G; ++g, ++k) {
                    const int s = k % NS;
                    if (k >= NS && !mbar_wait_bounded(empty + s, (unsigned)(((k / NS) - 1) & 1))) {
                        atomicOr(a.err, timeout_err);
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    unsigned char *st = tsm + (size_t)s * L::STAGE;
                    unsigned char *q = st + L::NP * L::A_BYTES + L::X_BYTES;
                    mbar_expect_tx(full + s, (unsigned)(L::X_BYTES + L::NP * (L::Q_BYTES + L::S_BYTES)));
                    tma_load_2d(st + L::NP * L::A_BYTES, &a.tmx, g * 64, tr.y, full + s, pol_x);
                    for (int p = 0; p < L::NP; ++p) {
                        tma_load_2d(q + p * L::Q_BYTES, &a.tmq[m0 + p], g * 64, row0, full + s, pol);
                        tma_load_2d(q + L::NP * L::Q_BYTES + p * L::S_BYTES, &a.tmsb[m0 + p], g * (L::SBG / 4), row0,
                                    full + s, pol);
                    }
                }
            }
            // let the copies this CTA issued land before it can exit (bounded)
            for (int q = k - NS; q < k; ++q)
                if (q >= 0) mbar_wait_bounded(full + q % NS, (unsigned)((q / NS) & 1), 1u << 16);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int k = 0;
            bool ok = true;
            for (int it = 0; it < my_items && ok; ++it) {
                const int b = it % ACC, use = it / ACC;  // accumulator set and how often it was used before
                const int item = (int)blockIdx.x + it * (int)gridDim.x;
                const int nslot = a.tiles[item / MT].z;
                // MMA width: the tile's slots rounded up to 16 (columns past them are never read)
                const uint32_t idesc = idesc_bf16(TC_M, min(NT, max(16, (nslot + 15) & ~15)));
                if (use >= 1 && !mbar_wait_bounded(acce + b, (unsigned)((use - 1) & 1))) {
                    atomicOr(a.err, timeout_err);
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                for (int g = 0; g < G; ++g, ++k) {
                    const int s = k % NS;
                    if (!mbar_wait_bounded(deq + s, (unsigned)((k / NS) & 1))) {
                        atomicOr(a.err, timeout_err);
                        s_fail = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const unsigned char *st = tsm + (size_t)s * L::STAGE;
                    const uint64_t bdesc = sdesc_sw128(smem_u32(st + L::NP * L::A_BYTES));
#pragma unroll
                    for (int p = 0; p < L::NP; ++p) {
                        const uint64_t adesc = sdesc_sw128(smem_u32(st + p * L::A_BYTES));
                        const uint32_t d_tmem = tmem + (uint32_t)((b * L::NP + p) * NT);
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks)  // 16 k = 32 bytes along the swizzled row: +2 in 16-byte units
                            umma_bf16(d_tmem, adesc + 2 * ks, bdesc + 2 * ks, idesc, (g > 0 || ks > 0) ? 1u : 0u);
                    }
                    umma_commit(empty + s);  // the stage is free once these MMAs have read it
                }
                if (ok) umma_commit(accf + b);
            }
            // MMAs still in flight finish before TMEM is released (bounded)
            if (k > 0) mbar_wait_bounded(empty + (k - 1) % NS, (unsigned)(((k - 1) / NS) & 1), 1u << 16);
        }
    } else if (warp < 2 + TC_DQW) {
        // ------------------------------------------------------------ dequant (8 warps, NP of the 8 * NP blocks each)
        const int dw = warp - 2;
        const int gq = lane >> 2, c = lane & 3;
        const uint32_t k128 = 0x43004300u;
        int k = 0;
        for (int it = 0; it < my_items && !*reinterpret_cast<volatile int *>(&s_fail); ++it) {
            bool ok = true;
            for (int g = 0; g < G; ++g, ++k) {
                const int s = k % NS;
                if (!mbar_wait_bounded(full + s, (unsigned)((k / NS) & 1))) {
                    if (lane == 0) atomicOr(a.err, timeout_err);
                    ok = false;
                    break;
                }
                unsigned char *st = tsm + (size_t)s * L::STAGE;
                const unsigned char *q = st + L::NP * L::A_BYTES + L::X_BYTES;
#pragma unroll
                for (int j = 0; j < L::NP; ++j) {
                    const int blk = dw + TC_DQW * j;  // (projection, row block)
                    const int p = blk >> 3, rb = blk & 7;
                    const uint4 w = reinterpret_cast<const uint4 *>(q + p * L::Q_BYTES + rb * 512)[lane];
                    const uint32_t *sbw = reinterpret_cast<const uint32_t *>(q + L::NP * L::Q_BYTES + p * L::S_BYTES + rb * L::SBG);
                    unsigned char *A = st + p * L::A_BYTES;
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {  // rows gq (words .x .y) and gq + 8 (words .z .w)
                        const int r = rb * 16 + gq + 8 * hf;
                        const uint32_t wa = hf ? w.z : w.x, wb = hf ? w.w : w.y;
                        uint32_t out[8];
                        if (FMT == FMT_FP4) {
                            // E2M1 * 2^(S-127) is exact in bf16; elements 16c .. 16c+15 share the scale of half c / 2
                            const uint32_t S = (sbw[gq] >> (8 * (hf * 2 + (c >> 1)))) & 0xFFu;
                            uint32_t lo[4], hi[4];
                            fp4_word(wa, fp4_scale2(S), lo);
                            fp4_word(wb, fp4_scale2(S), hi);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                out[i] = lo[i];
                                out[4 + i] = hi[i];
                            }
                        } else {
                            const uint32_t sbv = sbw[gq * 2 + hf];
                            const uint32_t s2 = (sbv & 0xFFFFu) | (sbv << 16), b2 = (sbv >> 16) | (sbv & 0xFFFF0000u);
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                const uint32_t v = q4pair(i < 4 ? wa : wb, i & 3);  // (128 + q_2p, 128 + q_2p+1)
                                __nv_bfloat162 qv = *reinterpret_cast<const __nv_bfloat162 *>(&v);
                                qv = __hsub2(qv, *reinterpret_cast<const __nv_bfloat162 *>(&k128));
                                const __nv_bfloat162 r2 = __hfma2(qv, *reinterpret_cast<const __nv_bfloat162 *>(&s2),
                                                                  *reinterpret_cast<const __nv_bfloat162 *>(&b2));
                                out[i] = *reinterpret_cast<const uint32_t *>(&r2);
                            }
                        }
                        // elements 16c .. 16c+15 of row r = chunks 2c, 2c+1 (16 B each), swizzled by r % 8
                        uint4 *row = reinterpret_cast<uint4 *>(A + r * 128);
                        row[(2 * c) ^ (r & 7)] = make_uint4(out[0], out[1], out[2], out[3]);
                        row[(2 * c + 1) ^ (r & 7)] = make_uint4(out[4], out[5], out[6], out[7]);
                    }
                }
                fence_async_smem();  // generic-proxy writes of A -> the tensor core's reads
                __syncwarp();
                if (lane == 0) mbar_arrive1(deq + s);
            }
            if (!ok) break;
        }
    } else {
        // ------------------------------------------------------------ epilogue (warps 10..13: rows 32 * (warp % 4) + lane)
        const int quarter = warp & 3;
        for (int it = 0; it < my_items && !*reinterpret_cast<volatile int *>(&s_fail); ++it) {
            const int item = (int)blockIdx.x + it * (int)gridDim.x;
            const int tile = item / MT, mt = item - tile * MT;
            const int4 tr = a.tiles[tile];
            const int e = (tr.x < 0 || tr.x >= a.E) ? 0 : tr.x;
            const int b = it % ACC;
            if (!mbar_wait_bounded(accf + b, (unsigned)((it / ACC) & 1))) {
                if (lane == 0) atomicOr(a.err, timeout_err);
                break;
            }
            tc_fence_after();
            const int row = mt * TC_M + quarter * 32 + lane;  // output row (f for gate/up, d for down)
            const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16);
            if (!DOWN) {
                const float bgr = a.bg ? a.bg[(size_t)e * a.f + row] : 0.f, bur = a.bu ? a.bu[(size_t)e * a.f + row] : 0.f;
                for (int c0 = 0; c0 < tr.z; c0 += 16) {
                    float gv[16], uv[16];
                    tmem_ld16(tl + (uint32_t)((b * 2 + 0) * NT + c0), gv);
                    tmem_ld16(tl + (uint32_t)((b * 2 + 1) * NT + c0), uv);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = c0 + j;
                        if (n < tr.z) a.h[(size_t)(tr.y + n) * a.f + row] = f2bf(act_glu(a.act, gv[j] + bgr, uv[j] + bur));
                    }
                }
            } else {
                const float bdr = a.bd ? a.bd[(size_t)e * a.d + row] : 0.f;
                for (int c0 = 0; c0 < tr.z; c0 += 16) {
                    float dv[16];
                    tmem_ld16(tl + (uint32_t)(b * NT + c0), dv);
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int n = c0 + j;
                        if (n < tr.z) {
                            const int slot = a.sorted[tr.y + n];
                            const int e_raw = a.idx[slot];
                            const float wsl = (e_raw >= 0 && e_raw < a.E) ? a.wts[slot] : 0.f;
                            a.yp[(size_t)slot * a.d + row] = wsl * (dv[j] + bdr);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive1(acce + b);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)L::TMEM_COLS)
                     : "memory");
    }
}

size_t experts_tc_smem(int nt, int ns, int acc, bool down, int fmt) {
    (void)acc;
    const int np = down ? 1 : 2, sbg = fmt == FMT_FP4 ? 32 : 64;
    const size_t raw = (size_t)np * TC_M * 128 + (size_t)nt * 128 + (size_t)np * (8 * 512 + 8 * sbg);
    const size_t stage = (raw + 1023) / 1024 * 1024;
    return 1024 /* alignment slack */ + ns * stage + (3 * ns + 2 * acc) * 8;
}

// x rows of the slots in expert-sorted order (the activation operand of the tensor-core gate/up)
__global__ void __launch_bounds__(256) k_gather_rows(const uint16_t *__restrict__ x, const int *__restrict__ sorted,
                                                     int TK, int k, int d, uint16_t *__restrict__ xs) {
    pdl_launch();
    pdl_wait();
    const int i = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (i >= TK) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)(sorted[i] / k) * d);
    uint4 *dst = reinterpret_cast<uint4 *>(xs + (size_t)i * d);
    for (int c = lane; c < d / 8; c += 32) dst[c] = src[c];
}

// gate/up: tiles of 256 slots with one accumulator set (2 x 256 TMEM columns) or of 128 with two; down: 4 stages,
// two sets
#define MOEB_TC(FMT)                                                                         \
    template __global__ void k_experts_tc<FMT, 256, 3, 1, false>(const __grid_constant__ ExpArgs); \
    template __global__ void k_experts_tc<FMT, 256, 4, 2, true>(const __grid_constant__ ExpArgs);  \
    template __global__ void k_experts_tc<FMT, 128, 3, 2, false>(const __grid_constant__ ExpArgs); \
    template __global__ void k_experts_tc<FMT, 128, 4, 2, true>(const __grid_constant__ ExpArgs);
MOEB_TC(FMT_Q4)
MOEB_TC(FMT_FP4)

}  // namespace moeb
