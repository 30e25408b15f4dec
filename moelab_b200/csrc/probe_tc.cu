// Measurement probes (not on any layer path): how fast one SM's tensor core takes the MMA shapes the expert
// kernels issue, and what limits a single issuing thread. One CTA per SM (120 KB of shared memory keeps it
// alone); `issuers` warps each have one thread issue back-to-back tcgen05.mma of M = 128, K = 16, N = n
// (kind::f16, A from TMEM, B from shared memory) into their own accumulator, `per_stage` MMAs (unrolled)
// between optional waits on an mbarrier phase that has already completed (the cost a pipelined kernel pays to
// learn that its operands are ready). Cycles per MMA = clock64 span of the slowest issuer / MMAs issued by the
// CTA, averaged over the SMs; TFLOP/s from CUDA events around the launch. A second probe times mma.sync
// m16n8k16 (bf16 -> fp32) over independent chains for comparison.
// Every wait is bounded; a timeout is reported as MOEB_ELAUNCH. The operands are zeros, or (data != 0) random bf16
// values of magnitude 0.5 .. 1 in both A (TMEM) and B (shared memory), to see whether the MMA rate depends on them.
// side != 0: four more warps run beside the MMAs, as the dequant (1: tcgen05.st 16x256b.x4 then wait::st) or
// epilogue warps (2: tcgen05.ld 32x32b.x16 then wait::ld) of the expert kernels do, on TMEM columns the MMAs do not
// touch, or (3) integer ALU work in 8 independent chains (competing with the issuing threads for issue slots);
// they stop when the issuers are done (bounded) and report how many operations they completed.
#include <cstdint>
#include <cuda_runtime.h>

#include "common.cuh"
#include "moelab_b200.h"

namespace moeb {
namespace {

MOEB_DEV uint64_t probe_desc_sw128(uint32_t saddr) {  // K-major, 128-byte swizzle, 8-row groups 1024 B apart
    uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}
MOEB_DEV uint32_t probe_idesc(int m, int n) {  // kind::f16: fp32 accumulate, bf16 A and B, K-major
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
MOEB_DEV void probe_mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

constexpr int PROBE_SMEM = 120 * 1024;
constexpr int PROBE_A_COL = 384;  // A operand columns [384, 416); accumulators below

MOEB_DEV uint32_t probe_rand_bf16x2(uint32_t i) {  // two bf16 of magnitude [0.5, 1) with random signs
    uint32_t h = i * 2654435761u;
    h ^= h >> 13;
    h *= 0x5bd1e995u;
    h ^= h >> 15;
    const uint32_t lo = 0x3F00u | (h & 0x7Fu) | ((h >> 7) & 1u) << 15;
    const uint32_t hi = 0x3F00u | ((h >> 8) & 0x7Fu) | ((h >> 15) & 1u) << 15;
    return lo | (hi << 16);
}

template <int PER>
__global__ void __launch_bounds__(256, 1) k_probe_tc(int n, int issuers, int wait, int stages, int dstride, int data,
                                                    int side, unsigned long long *cyc, unsigned *err,
                                                    unsigned long long *side_ops) {
    extern __shared__ __align__(1024) unsigned char psm[];
    __shared__ uint64_t ready, done[4];
    __shared__ uint32_t s_tmem;
    __shared__ int s_done;
    unsigned char *B = psm + ((1024 - (smem_u32(psm) & 1023)) & 1023);  // 32 KB of B rows, 1024-aligned
    for (int i = threadIdx.x; i < 32768 / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(B)[i] = data ? make_uint4(probe_rand_bf16x2(4 * i), probe_rand_bf16x2(4 * i + 1),
                                                            probe_rand_bf16x2(4 * i + 2), probe_rand_bf16x2(4 * i + 3))
                                               : make_uint4(0, 0, 0, 0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(&ready, 1);
        for (int i = 0; i < 4; ++i) mbar_init(done + i, 1);
        mbar_fence_init();
        mbar_arrive(&ready);  // phase 0 complete: every later wait on it succeeds at once
        s_done = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(512u)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;
    if (data && warp < 4) {  // A columns: each warp its TMEM lane quarter, two 16-lane x 32-column stores
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t v[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) v[q] = probe_rand_bf16x2((uint32_t)((threadIdx.x * 2 + h) * 16 + q) + 77777u);
            const uint32_t ta = tmem + ((uint32_t)(warp * 32 + h * 16) << 16) + PROBE_A_COL;
            asm volatile(
                "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                "%14, %15, %16};" ::"r"(ta),
                "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
                "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
                : "memory");
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();  // every thread of the CTA: the A stores are complete before any MMA
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp < issuers && lane == 0) {
        const uint32_t id = probe_idesc(128, n);
        const uint64_t bd = probe_desc_sw128(smem_u32(B));
        const uint32_t d = tmem + (uint32_t)(warp * dstride);
        bool ok = true;
        const long long t0 = clock64();
        for (int k = 0; k < stages && ok; ++k) {
            if (wait) ok = mbar_wait_bounded(&ready, 0);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int m = 0; m < PER; ++m)
                probe_mma_ts(d, tmem + PROBE_A_COL + (m & 3) * 8, bd + 2 * (m & 3), id, (k || m) ? 1u : 0u);
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(done + warp))
                     : "memory");
        if (!mbar_wait_bounded(done + warp, 0)) ok = false;
        const long long t1 = clock64();
        if (!ok) atomicOr(err, ERR_TIMEOUT);
        cyc[4 * blockIdx.x + warp] = (unsigned long long)(t1 - t0);
        atomicAdd(&s_done, 1);
    }
    if (side && warp >= 4) {  // TMEM traffic beside the MMAs: lanes of quarter warp % 4, columns 448 .. 511
        const uint32_t base = tmem + ((uint32_t)((warp & 3) * 32) << 16) + 448;
        unsigned long long ops = 0;
        uint32_t v[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) v[q] = (uint32_t)(lane * 16 + q);
        while (*reinterpret_cast<volatile int *>(&s_done) < issuers && ops < (1ull << 22)) {
            if (side == 1) {
                asm volatile(
                    "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                    "%13, %14, %15, %16};" ::"r"(base + (uint32_t)((ops & 1) * 16 << 16) + (uint32_t)((ops >> 1 & 1) * 32)),
                    "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
                    "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
                    : "memory");
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            } else if (side == 3) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const uint32_t x = v[q];
                    v[q] = ((x ^ (x >> 3)) + (x << 5)) ^ (v[q + 8] >> 1);
                    v[q + 8] = (v[q + 8] & 0x0F0F0F0Fu) | (x << 4);
                }
            } else {
                uint32_t r[16];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                    "[%16];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                      "=r"(r[15])
                    : "r"(base + (uint32_t)((ops & 3) * 16)));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                v[0] += r[0] ^ r[15];
            }
            ++ops;
        }
        if (lane == 0) atomicAdd(side_ops, ops);
        if (v[0] == 0xFFFFFFFFu && lane == 99) side_ops[1] = v[0];  // keeps the loads live; never true
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
    }
}

__global__ void __launch_bounds__(1024, 1) k_probe_mma_sync(int iters, float *sink) {
    float c[4][4] = {};
    const uint32_t a0 = threadIdx.x, a1 = threadIdx.x * 3u, a2 = threadIdx.x * 5u, a3 = threadIdx.x * 7u;
    const uint32_t b0 = threadIdx.x * 11u, b1 = threadIdx.x * 13u;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            asm volatile(
                "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%0,%1,%2,%3};"
                : "+f"(c[j][0]), "+f"(c[j][1]), "+f"(c[j][2]), "+f"(c[j][3])
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
    float s = 0.f;
    for (int j = 0; j < 4; ++j)
        for (int i = 0; i < 4; ++i) s += c[j][i];
    if (s == 12345.f) sink[threadIdx.x] = s;  // keeps the chains live; never true for these operands
}

int sm_count_of_current() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

}  // namespace
}  // namespace moeb

using namespace moeb;

extern "C" int moeb_probe_tc_issue(int n, int issuers, int per_stage, int wait, int data, int side,
                                   int mmas_per_issuer, double *cycles_per_mma, double *tflops,
                                   double *side_cycles_per_op) {
    if (n < 16 || n > 256 || n % 16 || issuers < 1 || issuers > 4 || mmas_per_issuer < per_stage ||
        (per_stage != 4 && per_stage != 8 && per_stage != 16) || !cycles_per_mma || !tflops)
        return MOEB_EINVAL;
    const int dstride = n <= 64 ? 64 : n <= 128 ? 128 : 256;  // each issuer's accumulator, below the A columns
    if (issuers * dstride > PROBE_A_COL) return MOEB_EINVAL;
    const int sms = sm_count_of_current(), stages = mmas_per_issuer / per_stage;
    if (side < 0 || side > 3) return MOEB_EINVAL;
    void (*fn)(int, int, int, int, int, int, int, unsigned long long *, unsigned *, unsigned long long *) =
        per_stage == 4 ? k_probe_tc<4> : per_stage == 8 ? k_probe_tc<8> : k_probe_tc<16>;
    if (cudaFuncSetAttribute((const void *)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, PROBE_SMEM) != cudaSuccess)
        return MOEB_ELAUNCH;
    unsigned long long *cyc = nullptr;
    unsigned *err = nullptr;
    if (cudaMalloc(&cyc, (size_t)(4 * sms + 2) * sizeof(unsigned long long)) != cudaSuccess) return MOEB_ELAUNCH;
    unsigned long long *ops = cyc + 4 * sms;
    if (cudaMalloc(&err, sizeof(unsigned)) != cudaSuccess) {
        cudaFree(cyc);
        return MOEB_ELAUNCH;
    }
    cudaMemset(cyc, 0, (size_t)(4 * sms + 2) * sizeof(unsigned long long));
    cudaMemset(err, 0, sizeof(unsigned));
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    fn<<<sms, 256, PROBE_SMEM>>>(n, issuers, wait, per_stage, dstride, data, side, cyc, err, ops);  // warm-up
    cudaMemsetAsync(ops, 0, 2 * sizeof(unsigned long long));
    cudaEventRecord(e0);
    fn<<<sms, 256, PROBE_SMEM>>>(n, issuers, wait, stages, dstride, data, side, cyc, err, ops);
    cudaEventRecord(e1);
    int rc = cudaEventSynchronize(e1) == cudaSuccess ? MOEB_OK : MOEB_ELAUNCH;
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    unsigned herr = 0;
    unsigned long long *h = new unsigned long long[(size_t)4 * sms + 2];
    if (cudaMemcpy(h, cyc, (size_t)(4 * sms + 2) * sizeof(unsigned long long), cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(&herr, err, sizeof(unsigned), cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = MOEB_ELAUNCH;
    if (herr) rc = MOEB_ELAUNCH;
    double span = 0.0;
    for (int s = 0; s < sms; ++s) {
        unsigned long long m = 0;
        for (int i = 0; i < issuers; ++i) m = h[4 * s + i] > m ? h[4 * s + i] : m;
        span += (double)m;
    }
    const double side_total = (double)h[4 * sms];
    delete[] h;
    const double mmas = (double)stages * per_stage * issuers;
    *cycles_per_mma = span / sms / mmas;
    if (side_cycles_per_op) *side_cycles_per_op = side && side_total > 0 ? span / (side_total / 4.0) : 0.0;
    *tflops = 2.0 * 128 * n * 16 * mmas * sms / (ms * 1e-3) / 1e12;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(cyc);
    cudaFree(err);
    return rc;
}

extern "C" int moeb_probe_mma_sync(int warps_per_sm, int iters, double *tflops) {
    if (warps_per_sm < 1 || warps_per_sm > 32 || iters < 1 || !tflops) return MOEB_EINVAL;
    const int sms = sm_count_of_current();
    float *sink = nullptr;
    if (cudaMalloc(&sink, 1024 * sizeof(float)) != cudaSuccess) return MOEB_ELAUNCH;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    k_probe_mma_sync<<<sms, 32 * warps_per_sm>>>(iters / 10 + 1, sink);
    cudaEventRecord(e0);
    k_probe_mma_sync<<<sms, 32 * warps_per_sm>>>(iters, sink);
    cudaEventRecord(e1);
    const int rc = cudaEventSynchronize(e1) == cudaSuccess ? MOEB_OK : MOEB_ELAUNCH;
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    *tflops = 2.0 * 16 * 8 * 16 * 4.0 * iters * warps_per_sm * sms / (ms * 1e-3) / 1e12;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(sink);
    return rc;
}
