// Weight formats: int4 affine g64 and MXFP4, quantized on the GPU into the B200 layout.
//
// int4 (reference state: moelab/variants/mlx/metal_q4_moe.py:32-39, W_BITS 4.5):
//   qw  uint32 [rows][K/8]   word j holds elements 8j..8j+7; nibble p (p < 4) = element 8j+2p,
//                            nibble p+4 = element 8j+2p+1, so `(w >> 4p) & 0x000F000F` yields the
//                            consecutive pair (8j+2p, 8j+2p+1) as two bf16 lanes (see q4pair).
//   sb  uint32 [rows][K/64]  bf16 scale in the low half, bf16 bias in the high half (one load per group).
// MXFP4 (metal_mxfp4_moe.py:1-12, :448-455, W_BITS 4.25):
//   qw  uint32 [rows][K/8]   same nibble interleave, E2M1 codes (sign bit 3, exponent bits 1-2, mantissa 0)
//   sc  uint8  [rows][K/32]  E8M0 scale bytes
// The quantizers follow the CPU oracle (oracle/moe_oracle.c) operation for operation, so GPU and CPU agree
// bit for bit on the packed tensors.
#include "common.cuh"

namespace moeb {

__device__ __forceinline__ uint32_t interleave_word(uint32_t nat) {
    // natural nibble order (element i at nibble i) -> B200 order (pairs split across the half-words)
    uint32_t r = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        r |= ((nat >> (8 * p)) & 0xfu) << (4 * p);
        r |= ((nat >> (8 * p + 4)) & 0xfu) << (4 * (p + 4));
    }
    return r;
}

__device__ __forceinline__ uint32_t deinterleave_word(uint32_t w) {
    uint32_t r = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        r |= ((w >> (4 * p)) & 0xfu) << (8 * p);
        r |= ((w >> (4 * (p + 4))) & 0xfu) << (8 * p + 4);
    }
    return r;
}

// One thread per (row, 64-group).
__global__ void k_q4_quantize(const uint16_t *__restrict__ w, long rows, long K, uint32_t *__restrict__ qw,
                              uint32_t *__restrict__ sb) {
    const long ng = K / 64;
    const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * ng) return;
    const long r = gid / ng, g = gid - r * ng;
    const uint16_t *src = w + r * K + g * 64;
    float v[64];
    float wmax = -INFINITY, wmin = INFINITY;
#pragma unroll
    for (int i = 0; i < 64; i += 8) {
        uint4 u = *reinterpret_cast<const uint4 *>(src + i);
        uint32_t ww[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[i + 2 * j] = bf16lo(ww[j]);
            v[i + 2 * j + 1] = bf16hi(ww[j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 64; ++i) {
        wmax = v[i] > wmax ? v[i] : wmax;
        wmin = v[i] < wmin ? v[i] : wmin;
    }
    const bool mask = fabsf(wmin) > fabsf(wmax);
    float scale = __fdiv_rn(__fsub_rn(wmax, wmin), 15.0f);
    scale = scale > 1e-7f ? scale : 1e-7f;
    scale = mask ? scale : -scale;
    const float edge = mask ? wmin : wmax;
    const float q0 = rintf(__fdiv_rn(edge, scale));
    float bias = 0.0f;
    if (q0 != 0.0f) {
        scale = __fdiv_rn(edge, q0);
        bias = edge;
    }
    uint32_t *dst = qw + r * (K / 8) + g * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t nat = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float q = rintf(__fdiv_rn(__fsub_rn(v[8 * j + i], bias), scale));
            q = q < 0.0f ? 0.0f : (q > 15.0f ? 15.0f : q);
            nat |= ((uint32_t)q & 0xfu) << (4 * i);
        }
        dst[j] = interleave_word(nat);
    }
    sb[r * ng + g] = (uint32_t)f2bf(scale) | ((uint32_t)f2bf(bias) << 16);
}

// fp32 dequant in natural element order: w = fmaf(scale, q, bias). One thread per packed word.
__global__ void k_q4_dequant(const uint32_t *__restrict__ qw, const uint32_t *__restrict__ sb, long rows, long K,
                             float *__restrict__ out) {
    const long nw = K / 8;
    const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * nw) return;
    const long r = gid / nw, j = gid - r * nw;
    const uint32_t nat = deinterleave_word(qw[gid]);
    const uint32_t s_b = sb[r * (K / 64) + j / 8];
    const float s = bf16lo(s_b), b = bf16hi(s_b);
    float4 o0, o1;
    float *o = reinterpret_cast<float *>(&o0);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = __fmaf_rn(s, (float)((nat >> (4 * i)) & 0xfu), b);
    o = reinterpret_cast<float *>(&o1);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = __fmaf_rn(s, (float)((nat >> (4 * (i + 4))) & 0xfu), b);
    float4 *dst = reinterpret_cast<float4 *>(out + r * K + j * 8);
    dst[0] = o0;
    dst[1] = o1;
}

// mlx state (natural nibble order, separate bf16 scales / biases) -> B200 layout. One thread per word.
__global__ void k_q4_from_mlx(const uint32_t *__restrict__ wq, const uint16_t *__restrict__ scales,
                              const uint16_t *__restrict__ biases, long rows, long K, uint32_t *__restrict__ qw,
                              uint32_t *__restrict__ sb) {
    const long nw = K / 8;
    const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * nw) return;
    qw[gid] = interleave_word(wq[gid]);
    const long r = gid / nw, j = gid - r * nw;
    if ((j & 7) == 0) {
        const long gi = r * (K / 64) + j / 8;
        sb[gi] = (uint32_t)scales[gi] | ((uint32_t)biases[gi] << 16);
    }
}

// ------------------------------------------------------------------ MXFP4
__device__ __forceinline__ uint32_t e2m1_round(float v) {
    const uint32_t sign = signbit(v) ? 8u : 0u;
    const float a = fabsf(v);
    uint32_t c;
    if (!(a == a)) c = 7;
    else if (a <= 0.25f) c = 0;
    else if (a < 0.75f) c = 1;
    else if (a <= 1.25f) c = 2;
    else if (a < 1.75f) c = 3;
    else if (a <= 2.5f) c = 4;
    else if (a < 3.5f) c = 5;
    else if (a <= 5.0f) c = 6;
    else c = 7;
    return sign | c;
}

// One thread per (row, 32-group).
__global__ void k_fp4_quantize(const uint16_t *__restrict__ w, long rows, long K, uint32_t *__restrict__ qw,
                               uint8_t *__restrict__ sc) {
    const long ng = K / 32;
    const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * ng) return;
    const long r = gid / ng, g = gid - r * ng;
    const uint16_t *src = w + r * K + g * 32;
    float v[32];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        v[i] = bf2f(src[i]);
        const float a = fabsf(v[i]);
        amax = a > amax ? a : amax;
    }
    int e;
    if (amax == 0.0f) e = -127;
    else {
        int ex;
        frexpf(amax, &ex);
        e = ex - 1 - 2;
    }
    e = e < -127 ? -127 : (e > 127 ? 127 : e);
    const float inv = ldexpf(1.0f, -e);
    uint32_t *dst = qw + r * (K / 8) + g * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t nat = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) nat |= e2m1_round(__fmul_rn(v[8 * j + i], inv)) << (4 * i);
        dst[j] = interleave_word(nat);
    }
    sc[r * ng + g] = (uint8_t)(e + 127);
}

__device__ __forceinline__ float e2m1_value(uint32_t c) {
    const float m = (c & 7u) < 2 ? 0.5f * (float)(c & 7u)
                                 : ldexpf(1.0f + 0.5f * (float)(c & 1u), (int)((c & 7u) >> 1) - 1);
    return (c & 8u) ? -m : m;
}

__global__ void k_fp4_dequant(const uint32_t *__restrict__ qw, const uint8_t *__restrict__ sc, long rows, long K,
                              float *__restrict__ out) {
    const long nw = K / 8;
    const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * nw) return;
    const long r = gid / nw, j = gid - r * nw;
    const uint32_t nat = deinterleave_word(qw[gid]);
    const int ex = (int)sc[r * (K / 32) + j / 4] - 127;
    float *dst = out + r * K + j * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = ldexpf(e2m1_value((nat >> (4 * i)) & 0xfu), ex);
}

__global__ void k_fp4_from_mlx(const uint32_t *__restrict__ wq, const uint8_t *__restrict__ scales, long rows,
                               long K, uint32_t *__restrict__ qw, uint8_t *__restrict__ sc) {
    const long nw = K / 8;
    const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * nw) return;
    qw[gid] = interleave_word(wq[gid]);
    const long r = gid / nw, j = gid - r * nw;
    if ((j & 3) == 0) sc[r * (K / 32) + j / 4] = scales[r * (K / 32) + j / 4];
}

}  // namespace moeb
