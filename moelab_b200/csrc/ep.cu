// Expert parallelism: the device steps around the two all-to-all exchanges of an expert-parallel MoE layer.
// P ranks (one per GPU) each own E/P consecutive experts; every rank routes its own tokens.
//
//   k_ep_plan    (1 CTA)    stable counting sort of the T*k slots by owning rank: per-rank send counts and the
//                           send-buffer row of every slot (slot order kept inside a rank, so the receiver sees
//                           its rows grouped by source rank and, inside one source, in token order).
//   k_ep_pack    (warp/slot) gathers x of each slot's token into its send row and appends the 16-byte tail
//                           {local expert id, weight bits, 0, 0}: one all-to-all moves rows and routing together.
//   k_ep_combine (CTA/token) y[t] = sum_j back[slot_pos[t*k + j]] in fixed j order (+ residual), where back
//                           holds the owners' weighted fp32 slot outputs returned by the second all-to-all. The
//                           order and rounding are those of the single-GPU combine, so results match it bit for
//                           bit when both sides run the same expert kernels.
#include "common.cuh"
#include "kernels.h"

namespace moeb {

namespace {
constexpr int PLAN_THREADS = 1024;
constexpr int PLAN_MAXP = 32;
}  // namespace

__global__ void __launch_bounds__(PLAN_THREADS) k_ep_plan(EPArgs a) {
    pdl_launch();
    pdl_wait();
    __shared__ int base[PLAN_MAXP];                      // running count per owner over finished chunks
    __shared__ int wcnt[PLAN_THREADS / 32][PLAN_MAXP];   // per-warp counts of the current chunk, then offsets
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int TK = a.T * a.k, P = a.P, El = a.E / a.P;
    if (tid < P) base[tid] = 0;
    if (a.C > 0 && tid == 0) {  // peer-memory exchange: a new layer call (every rank counts the same calls)
        unsigned *ep = reinterpret_cast<unsigned *>(a.self + p2p_layout(P, a.C, a.d).epoch);
        *ep = *ep + 1u;
    }
    for (int c0 = 0; c0 < TK; c0 += PLAN_THREADS) {
        if (lane < P) wcnt[warp][lane] = 0;
        __syncthreads();  // zeroed counts (and, first time, base) visible
        const int s = c0 + tid;
        int owner = -1;
        if (s < TK) {
            const int e = a.idx[s];
            if (e >= 0 && e < a.E) owner = e / El;
            else atomicOr(a.err, ERR_EXPERT_ID);
        }
        const unsigned same = __match_any_sync(0xffffffffu, owner);
        const int rank_w = __popc(same & ((1u << lane) - 1u));
        if (owner >= 0 && rank_w == 0) wcnt[warp][owner] = __popc(same);
        __syncthreads();
        if (tid < P) {  // exclusive scan over the warps, per owner, continuing from earlier chunks
            int run = base[tid];
            for (int w = 0; w < PLAN_THREADS / 32; ++w) {
                const int c = wcnt[w][tid];
                wcnt[w][tid] = run;
                run += c;
            }
            base[tid] = run;
        }
        __syncthreads();
        if (s < TK) a.slot_pos[s] = owner >= 0 ? wcnt[warp][owner] + rank_w : -1;  // rank inside the owner
        __syncthreads();  // wcnt is rewritten by the next chunk
    }
    __syncthreads();
    // base[] now holds the totals: exclusive scan over the owners, then shift every slot by its owner's offset
    __shared__ int off[PLAN_MAXP];
    if (tid == 0) {  // packed send buffer: owner blocks back to back; peer exchange: fixed blocks of C rows
        int run = 0;
        for (int p = 0; p < P; ++p) {
            off[p] = a.C > 0 ? p * a.Cs : run;
            run += base[p];
        }
    }
    __syncthreads();
    if (tid < P) a.send_counts[tid] = base[tid];
    for (int s = tid; s < TK; s += PLAN_THREADS) {  // the same thread wrote slot_pos[s] above
        const int pos = a.slot_pos[s];
        if (pos >= 0) a.slot_pos[s] = pos + off[a.idx[s] / El];
    }
}

// grid ceil(T*k / 8), block 256: one warp per slot
__global__ void __launch_bounds__(256) k_ep_pack(EPArgs a) {
    pdl_launch();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int s = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (s >= a.T * a.k) return;
    const int pos = a.slot_pos[s];
    if (pos < 0) return;
    const int d = a.d, El = a.E / a.P;
    const uint4 *src = reinterpret_cast<const uint4 *>(a.x + (size_t)(s / a.k) * d);
    uint4 *dst = reinterpret_cast<uint4 *>(a.rows + (size_t)pos * (d + 8));
    for (int i = lane; i < d / 8; i += 32) dst[i] = src[i];
    if (lane == 0) {
        const int e = a.idx[s];
        dst[d / 8] = make_uint4((unsigned)(e % El), __float_as_uint(a.wts[s]), 0u, 0u);
    }
}

// Peer-memory dispatch: grid ceil(T*k / 8), block 256, warp per slot. The slot's row goes straight into the
// owner's exchange buffer (source block `me`, row slot_pos % C); the last CTA to finish then publishes, per
// owner, the row count and the epoch flag (system-scope release after a system-scope fence).
__global__ void __launch_bounds__(256) k_ep_send(EPArgs a) {
    pdl_launch();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int s = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int d = a.d, El = a.E / a.P, Cs = a.Cs;
    const P2PLayout L = p2p_layout(a.P, a.C, d);
    if (s < a.T * a.k) {
        const int pos = a.slot_pos[s];
        if (pos >= 0) {
            const int dst = pos / Cs, row = pos - dst * Cs;
            const uint4 *src = reinterpret_cast<const uint4 *>(a.x + (size_t)(s / a.k) * d);
            uint4 *out = reinterpret_cast<uint4 *>(a.peers[dst] + L.rows + ((size_t)a.me * Cs + row) * (d + 8) * 2);
            for (int i = lane; i < d / 8; i += 32) out[i] = src[i];
            if (lane == 0) out[d / 8] = make_uint4((unsigned)(a.idx[s] % El), __float_as_uint(a.wts[s]), 0u, 0u);
        }
    }
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();  // this CTA's row stores (ordered by the barrier) before the counter
        unsigned *ctr = reinterpret_cast<unsigned *>(a.self + L.ctr);
        s_last = atomicAdd(ctr, 1u) == gridDim.x - 1;
        if (s_last) {
            *ctr = 0u;
            __threadfence_system();
        }
    }
    __syncthreads();
    if (!s_last) return;
    const unsigned ep = *reinterpret_cast<const unsigned *>(a.self + L.epoch);
    for (int dst = threadIdx.x; dst < a.P; dst += blockDim.x) {
        reinterpret_cast<int *>(a.peers[dst] + L.rcnt)[a.me] = a.send_counts[dst];
        __threadfence_system();
        st_release_sys(reinterpret_cast<unsigned *>(a.peers[dst] + L.rflag) + a.me, ep);
    }
}

// Peer-memory return: one warp after the expert kernels wrote their rows into the owners' return blocks (each
// writing warp fenced at system scope): tell every owner that this rank's block is complete.
__global__ void k_ep_signal(unsigned char *const *peers, unsigned char *self, int P, int C, int d, int me) {
    pdl_launch();
    pdl_wait();
    const P2PLayout L = p2p_layout(P, C, d);
    const unsigned ep = *reinterpret_cast<const unsigned *>(self + L.epoch);
    __threadfence_system();
    for (int dst = threadIdx.x; dst < P; dst += blockDim.x)
        st_release_sys(reinterpret_cast<unsigned *>(peers[dst] + L.bflag) + me, ep);
}

// Peer-memory combine: grid ceil(T * d / 4 / 128), block 128. Waits until every expert rank holding one of the
// token's slots has signalled, then y[t] = sum_j back[slot_pos[t*k + j]] (fixed j order) + residual.
__global__ void __launch_bounds__(128) k_ep_combine_p2p(const unsigned char *self, const int *__restrict__ slot_pos,
                                                        int P, int C, int T, int d, int k,
                                                        const uint16_t *__restrict__ residual,
                                                        uint16_t *__restrict__ y, unsigned *err) {
    pdl_launch();
    pdl_wait();
    const P2PLayout L = p2p_layout(P, C, d);
    const unsigned ep = *reinterpret_cast<const unsigned *>(self + L.epoch);
    const unsigned *bflag = reinterpret_cast<const unsigned *>(self + L.bflag);
    const uint64_t lim = *reinterpret_cast<const unsigned long long *>(self + L.wait);
    __shared__ int ok;
    if (threadIdx.x < 32) {  // one warp waits for all P expert ranks (P <= 32)
        const bool done = threadIdx.x >= P || wait_flag_sys(bflag + threadIdx.x, ep, err, lim);
        (void)done;
        __syncwarp();
        if (threadIdx.x == 0) ok = 1;
    }
    __syncthreads();
    (void)ok;
    const float *back = reinterpret_cast<const float *>(self + L.back);
    const int q = d / 4;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)T * q) return;
    const int t = (int)(i / q), c = (int)(i - (long)t * q);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
        const int pos = slot_pos[(size_t)t * k + j];
        if (pos < 0) continue;
        const float4 v = __ldcs(reinterpret_cast<const float4 *>(back + (size_t)pos * d) + c);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    if (residual) {
        const uint2 r = *reinterpret_cast<const uint2 *>(residual + (size_t)t * d + 4 * c);
        acc.x += bf16lo(r.x);
        acc.y += bf16hi(r.x);
        acc.z += bf16lo(r.y);
        acc.w += bf16hi(r.y);
    }
    *reinterpret_cast<uint2 *>(y + (size_t)t * d + 4 * c) = make_uint2(pack_bf2(acc.x, acc.y), pack_bf2(acc.z, acc.w));
}

// grid T, block 256: one CTA per token, 4 columns per thread per step
__global__ void __launch_bounds__(256) k_ep_combine(const float *__restrict__ back, const int *__restrict__ slot_pos,
                                                    int T, int d, int k, const uint16_t *__restrict__ residual,
                                                    uint16_t *__restrict__ y) {
    pdl_launch();
    pdl_wait();
    __shared__ int pos[32];
    const int t = blockIdx.x;
    if (threadIdx.x < k) pos[threadIdx.x] = slot_pos[(size_t)t * k + threadIdx.x];
    __syncthreads();
    for (int c = threadIdx.x; c < d / 4; c += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < k; ++j) {
            if (pos[j] < 0) continue;
            const float4 v = __ldcs(reinterpret_cast<const float4 *>(back + (size_t)pos[j] * d) + c);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        if (residual) {
            const uint2 r = *reinterpret_cast<const uint2 *>(residual + (size_t)t * d + 4 * c);
            acc.x += bf16lo(r.x);
            acc.y += bf16hi(r.x);
            acc.z += bf16lo(r.y);
            acc.w += bf16hi(r.y);
        }
        *reinterpret_cast<uint2 *>(y + (size_t)t * d + 4 * c) = make_uint2(pack_bf2(acc.x, acc.y), pack_bf2(acc.z, acc.w));
    }
}

// grid ceil(T * d / 4 / 128), block 128: one thread per (token, 4 columns) so every slot row is loaded by many
// CTAs at once. y[t] = sum_j yp[t*k + j] (fixed j order) + residual, rounded once to bf16: the combine of the
// grouped kernels when down writes only the weighted slot rows (same order and rounding as the fused one).
__global__ void __launch_bounds__(128) k_combine(const float *__restrict__ yp, int T, int d, int k,
                                                 const uint16_t *__restrict__ residual, uint16_t *__restrict__ y) {
    pdl_launch();
    pdl_wait();
    const int q = d / 4;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)T * q) return;
    const int t = (int)(i / q), c = (int)(i - (long)t * q);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
        const float4 v = __ldcs(reinterpret_cast<const float4 *>(yp + ((size_t)t * k + j) * d) + c);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    if (residual) {
        const uint2 r = *reinterpret_cast<const uint2 *>(residual + (size_t)t * d + 4 * c);
        acc.x += bf16lo(r.x);
        acc.y += bf16hi(r.x);
        acc.z += bf16lo(r.y);
        acc.w += bf16hi(r.y);
    }
    *reinterpret_cast<uint2 *>(y + (size_t)t * d + 4 * c) = make_uint2(pack_bf2(acc.x, acc.y), pack_bf2(acc.z, acc.w));
}

}  // namespace moeb
