// Shared device helpers for the moelab_b200 kernels (sm_100a).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define MOEB_DEV __device__ __forceinline__

namespace moeb {

// Error bits written to the workspace error word by device code (read back with moeb_read_error).
enum : uint32_t {
    ERR_EXPERT_ID = 1u,  // an expert id outside [0, E): the slot contributes nothing
    ERR_TIMEOUT = 2u,    // a bounded wait gave up
};

// Row stride (floats) of the per-64-group activation sums: padded to 4 so rows stay 16-byte aligned for TMA.
__host__ __device__ __forceinline__ int xsum_stride(int d) { return ((d / 64 + 3) / 4) * 4; }

MOEB_DEV float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
MOEB_DEV float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
MOEB_DEV float bf2f(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }
MOEB_DEV uint16_t f2bf(float f) {
    __nv_bfloat16 b = __float2bfloat16_rn(f);
    return *reinterpret_cast<uint16_t *>(&b);
}
MOEB_DEV uint32_t pack_bf2(float lo, float hi) {
    return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}

// Programmatic dependent launch: wait for the preceding grid's results / let the next grid launch early.
MOEB_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MOEB_DEV void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Streaming loads of expert weights (read once per call): keep them out of L1.
MOEB_DEV uint2 ld_stream_u2(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
MOEB_DEV uint32_t ld_stream_u32(const void *p) {
    uint32_t r;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}
MOEB_DEV uint4 ld_stream_u4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// Warp-level bf16 tensor-core MMA, fp32 accumulate: D = A(16x16) * B(16x8) + C.
MOEB_DEV void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// bf16x2 (128 + q_lo, 128 + q_hi) from the nibble pair (p, p + 4) of a packed int4 word: q | 0x4300 read as
// bf16 is exactly 128 + q, so one lop3 turns two codes into two exact MMA operands.
MOEB_DEV uint32_t q4pair(uint32_t w, int p) {
    uint32_t t = w >> (4 * p), r;
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(r) : "r"(t), "r"(0x000F000Fu), "r"(0x43004300u));
    return r;
}

// Ampere-style asynchronous global->shared copies (per lane, no register staging). A false predicate copies
// nothing and zero-fills the destination; the source must still be a valid address.
MOEB_DEV void cp_async16(void *smem, const void *gmem, bool pred = true) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(pred ? 16 : 0) : "memory");
}
MOEB_DEV void cp_async8(void *smem, const void *gmem, bool pred = true) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(s), "l"(gmem), "r"(pred ? 8 : 0) : "memory");
}
MOEB_DEV void cp_async4(void *smem, const void *gmem, bool pred = true) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(s), "l"(gmem), "r"(pred ? 4 : 0) : "memory");
}
MOEB_DEV void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
MOEB_DEV void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ---- TMA bulk copies (cp.async.bulk, no multicast) completing on an mbarrier
// Device-scope acquire-release add: the last-arriver hand-offs use it in place of fence + atomic + fence (the
// release covers the CTA's earlier writes through the preceding __syncthreads, the acquire the other CTAs' ones).
MOEB_DEV unsigned atom_add_acq_rel_gpu(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
MOEB_DEV unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
MOEB_DEV void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
MOEB_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
MOEB_DEV void mbar_expect_tx(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
MOEB_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
MOEB_DEV bool mbar_try_wait(uint64_t *bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after `limit` polls (each poll already blocks for a hardware-defined interval).
MOEB_DEV bool mbar_wait_bounded(uint64_t *bar, unsigned parity, unsigned limit = 1u << 22) {
    for (unsigned i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
MOEB_DEV uint64_t l2_evict_last_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
MOEB_DEV uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// global -> this CTA's shared memory, `bytes` a multiple of 16, both addresses 16-byte aligned
MOEB_DEV void tma_load_1d(void *dst, const void *src, unsigned bytes, uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

MOEB_DEV void tma_load_1d(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// 3-D tiled tensor copy global -> this CTA's shared memory (no multicast); box and strides come from the
// tensor map (a __grid_constant__ kernel parameter). Coordinates are element indices, innermost first; the
// innermost coordinate is always 0 here (16-byte aligned). Out-of-range rows read as zero.
MOEB_DEV void tma_load_3d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
MOEB_DEV void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
MOEB_DEV void tmap_prefetch(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- cross-GPU signalling (expert-parallel exchange over peer memory)
// Slot id meaning "no work here" (padding of a capacity block): skipped by the tile builder, not an error.
constexpr int SLOT_SKIP = -2147483647 - 1;

MOEB_DEV uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
MOEB_DEV unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
MOEB_DEV void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait until *flag == want (acquire, system scope). Gives up after limit_ns of wall time (0: 2 s) - a
// peer that never signals -, records ERR_TIMEOUT and returns false; the caller then carries on with whatever data
// is there.
MOEB_DEV bool wait_flag_sys(const unsigned *flag, unsigned want, unsigned *err, uint64_t limit_ns = 0) {
    if (ld_acquire_sys(flag) == want) return true;
    const uint64_t lim = limit_ns ? limit_ns : 2000000000ull;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(flag) != want) {
        if (globaltimer_ns() - t0 > lim) {
            atomicOr(err, ERR_TIMEOUT);
            return false;
        }
        __nanosleep(128);
    }
    return true;
}

MOEB_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

MOEB_DEV float act_glu(int act, float g, float u) {
    if (act == 1) return 0.5f * g * (1.f + tanhf(0.7978845608028654f * (g + 0.044715f * g * g * g))) * u;
    if (act == 2) {
        g = fminf(g, 7.0f);
        u = fminf(fmaxf(u, -7.0f), 7.0f);
        return g / (1.f + expf(-1.702f * g)) * (u + 1.f);
    }
    return g / (1.f + expf(-g)) * u;
}

}  // namespace moeb
