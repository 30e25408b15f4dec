// Router device pieces shared by the router kernel (route.cu) and the fused decode kernel (decode.cu).
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace moeb {

// per-64-group sums of one token row (fp32); warp-cooperative
__device__ __forceinline__ void row_group_sums(const uint16_t *__restrict__ xr, int d, float *__restrict__ out,
                                               int lane) {
    for (int g = lane; g < d / 64; g += 32) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint4 u = *reinterpret_cast<const uint4 *>(xr + g * 64 + 8 * i);
            s += bf16lo(u.x) + bf16hi(u.x) + bf16lo(u.y) + bf16hi(u.y) + bf16lo(u.z) + bf16hi(u.z) + bf16lo(u.w) +
                 bf16hi(u.w);
        }
        out[g] = s;
    }
}

// fp32 -> unsigned with the same order (for the warp max reductions); -0 is folded into +0 by the caller
__device__ __forceinline__ unsigned fkey(float f) {
    const unsigned u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Top-k of token t from the fp32 logits in a.logits; writes the token's k + ns slots (routed ids / weights, then
// the shared experts) to idx_out / wts_out [t * (k + ns) + j].
// srow: the token's logits in shared memory (null: a.logits row t, read through L2).
template <int JMAX>
__device__ void topk_token_to(const RouterArgs &a, int t, int lane, int *idx_out, float *wts_out,
                              const float *srow = nullptr) {
    const int E = a.E, k = a.k;
    float v[JMAX];
    float m0 = -INFINITY;
#pragma unroll
    for (int j = 0; j < JMAX; ++j) {
        const int e = j * 32 + lane;
        float l = e < E ? (srow ? srow[e] : __ldcg(a.logits + (size_t)t * E + e)) : -INFINITY;
        v[j] = isnan(l) ? -INFINITY : l + 0.f;  // NaN = -inf; -0 -> +0 (equal values compare as keys too)
        m0 = fmaxf(m0, v[j]);
    }
    m0 = fkey_inv(__reduce_max_sync(0xffffffffu, fkey(m0)));
    float den = 0.f;
    if (!a.norm) {
#pragma unroll
        for (int j = 0; j < JMAX; ++j) den += v[j] == -INFINITY ? 0.f : expf(v[j] - m0);
        den = warp_sum(den);
    }
    float myv = -INFINITY, top0 = -INFINITY;
    int myi = 0;
    for (int r = 0; r < k; ++r) {
        // the largest remaining value (one warp max on order-preserving keys), lowest id among equal ones
        float b = -INFINITY;
        unsigned bi = 0xffffffffu;
#pragma unroll
        for (int j = 0; j < JMAX; ++j)
            if (v[j] > b) { b = v[j]; bi = (unsigned)(j * 32 + lane); }
        const unsigned kb = fkey(b), km = __reduce_max_sync(0xffffffffu, kb);
        float m = fkey_inv(km);
        unsigned sel = __reduce_min_sync(0xffffffffu, kb == km ? bi : 0xffffffffu);
        if (sel == 0xffffffffu) {  // fewer than k values above -inf: lowest unused id, weight 0
            unsigned cand = 0;
            while (__any_sync(0xffffffffu, lane < r && (unsigned)myi == cand)) ++cand;
            sel = cand;
            m = -INFINITY;
        } else if ((int)(sel & 31u) == lane) {
#pragma unroll
            for (int j = 0; j < JMAX; ++j)
                if (j == (int)(sel >> 5)) v[j] = -INFINITY;
        }
        if (lane == r) { myv = m; myi = (int)sel; }
        if (r == 0) top0 = m;
    }
    float s = 0.f;
    if (a.norm) {
        for (int r = 0; r < k; ++r) s += expf(__shfl_sync(0xffffffffu, myv, r) - top0);
    } else {
        s = den;
    }
    const float off = a.norm ? top0 : m0;
    const int ks = k + a.ns;
    if (lane < k) {
        idx_out[(size_t)t * ks + lane] = myi;
        wts_out[(size_t)t * ks + lane] = expf(myv - off) / s * a.scale;
    } else if (lane < ks) {  // always-on shared experts after the routed ones (summed last, weight 1)
        idx_out[(size_t)t * ks + lane] = E + (lane - k);
        wts_out[(size_t)t * ks + lane] = 1.f;
    }
}

template <int JMAX>
__device__ __forceinline__ void topk_token(const RouterArgs &a, int t, int lane) {
    topk_token_to<JMAX>(a, t, lane, a.idx, a.wts);
}

// Top-k of every token from the logits in shared memory (lg [T][E], NaN already -inf, -0 already +0), by rank:
// expert e's rank is the number of experts with a larger value or an equal value and a lower id, so the k experts
// of rank < k in rank order are exactly router.py's selection (largest first, lowest id on ties, the lowest unused
// ids when fewer than k are finite). The weights repeat topk_token_to's arithmetic operation for operation.
// T tokens (rows of lg, each padded to E rounded up to 16 with -inf); sel: [T][k] scratch; idx_out / wts_out:
// the tokens' [T][k + ns] slots. Every thread of the CTA calls it (blockDim.x a multiple of 32).
__device__ __forceinline__ void topk_rank(const RouterArgs &r, int T, const float *lg, int *sel, int *idx_out,
                                          float *wts_out) {
    const int E = r.E, k = r.k, ks = k + r.ns;
    // four threads per (token, expert), each comparing a quarter of the row (E4 = E rounded up to 16, the row padded
    // with -inf entries that never outrank a real one: equal values lose to lower ids, and padding ids are larger)
    const int E4 = (E + 15) & ~15, q4 = E4 / 4;
    for (int base = 0; base < T * E; base += blockDim.x / 4) {
        const int pr = base + (int)threadIdx.x / 4, sub = threadIdx.x & 3;
        const bool act_ = pr < T * E;
        const int t = act_ ? pr / E : 0, e = act_ ? pr - t * E : 0;
        const float *row = lg + (size_t)t * E4;
        const float v = row[e];
        int rank = 0;
        const float4 *r4 = reinterpret_cast<const float4 *>(row + sub * q4);
        for (int j = 0; j < q4 / 4; ++j) {
            const float4 o = r4[j];
            const int e2 = sub * q4 + 4 * j;
            rank += (o.x > v || (o.x == v && e2 < e)) + (o.y > v || (o.y == v && e2 + 1 < e)) +
                    (o.z > v || (o.z == v && e2 + 2 < e)) + (o.w > v || (o.w == v && e2 + 3 < e));
        }
        rank += __shfl_xor_sync(0xffffffffu, rank, 1);
        rank += __shfl_xor_sync(0xffffffffu, rank, 2);
        if (act_ && sub == 0 && rank < k) sel[t * k + rank] = e;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int t = warp; t < T; t += nw) {
        const float *row = lg + (size_t)t * E4;
        float m0 = -INFINITY;
        for (int e = lane; e < E; e += 32) m0 = fmaxf(m0, row[e]);
        m0 = fkey_inv(__reduce_max_sync(0xffffffffu, fkey(m0)));
        float den = 0.f;
        if (!r.norm) {
            for (int e = lane; e < E; e += 32) den += row[e] == -INFINITY ? 0.f : expf(row[e] - m0);
            den = warp_sum(den);
        }
        const int myi = lane < k ? sel[t * k + lane] : 0;
        const float myv = lane < k ? row[myi] : -INFINITY;
        const float top0 = row[sel[t * k]];
        float s = 0.f;
        if (r.norm) {
            for (int q = 0; q < k; ++q) s += expf(__shfl_sync(0xffffffffu, myv, q) - top0);
        } else {
            s = den;
        }
        const float off = r.norm ? top0 : m0;
        if (lane < k) {
            idx_out[(size_t)t * ks + lane] = myi;
            wts_out[(size_t)t * ks + lane] = expf(myv - off) / s * r.scale;
        } else if (lane < ks) {
            idx_out[(size_t)t * ks + lane] = E + (lane - k);
            wts_out[(size_t)t * ks + lane] = 1.f;
        }
    }
}



}  // namespace moeb
