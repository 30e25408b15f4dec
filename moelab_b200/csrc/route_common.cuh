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

template <int JMAX>
__device__ void topk_token(const RouterArgs &a, int t, int lane) {
    const int E = a.E, k = a.k;
    float v[JMAX];
    float m0 = -INFINITY;
#pragma unroll
    for (int j = 0; j < JMAX; ++j) {
        const int e = j * 32 + lane;
        float l = e < E ? __ldcg(a.logits + (size_t)t * E + e) : -INFINITY;
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
        a.idx[(size_t)t * ks + lane] = myi;
        a.wts[(size_t)t * ks + lane] = expf(myv - off) / s * a.scale;
    } else if (lane < ks) {  // always-on shared experts after the routed ones (summed last, weight 1)
        a.idx[(size_t)t * ks + lane] = E + (lane - k);
        a.wts[(size_t)t * ks + lane] = 1.f;
    }
}


}  // namespace moeb
