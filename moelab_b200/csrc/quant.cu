// Weight formats: int4 affine g64 and MXFP4, quantized on the GPU into the B200 layout.
//
// Reference state (moelab/variants/mlx/metal_q4_moe.py:32-39, W_BITS 4.5; metal_mxfp4_moe.py:448-455, W_BITS
// 4.25): uint32 [rows][K/8] with element 8j+i at bits 4i of word j, scales (and biases) per group.
//
// B200 layout ("fragment-major"): rows are taken in blocks of 16 (rows never straddle experts since
// N % 16 == 0) and K in groups of 64. Each (row block, group) is one contiguous 512-byte block holding, for
// warp lane L = 4*gq + c, the uint4 {row gq: word 2c, word 2c+1; row gq+8: word 2c, word 2c+1} - exactly the
// m16n8k16 A fragments of that lane for the 4 k-steps of the group (the k permutation is described in
// experts.cu). A warp therefore reads a whole A operand with one coalesced 16-byte load per lane. Inside
// each word the nibbles are interleaved: nibble p (p < 4) = element 2p, nibble p+4 = element 2p+1, so
// `(w >> 4p) & 0x000F000F` yields the consecutive pair (2p, 2p+1) as two bf16 lanes (q4pair).
//   int4  q  uint32 [E*N/16][K/64][32][4]
//         sb uint32 [E*N/16][K/64][8][2]  (gq, upper) -> bf16 scale | bf16 bias << 16
//   MXFP4 q  same as int4 (E2M1 codes: sign bit 3, exponent bits 1-2, mantissa bit 0)
//         sc uint8  [E*N/16][K/64][8][2][2] (gq, upper, 32-half) -> E8M0 byte
// The quantizers follow the CPU oracle (oracle/moe_oracle.c) operation for operation, so GPU and CPU agree
// bit for bit on the codes, scales and biases.
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

// word index of (row, k-word j) in the fragment-major layout
__device__ __forceinline__ long fm_word(long row, long j, long K) {
    const long rb = row >> 4, rr = row & 15, g = j >> 3, jj = j & 7;
    const long lane = (rr & 7) * 4 + (jj >> 1);
    return ((rb * (K / 64) + g) * 32 + lane) * 4 + (rr >> 3) * 2 + (jj & 1);
}
// index of (row, 64-group g) in the scale|bias array
__device__ __forceinline__ long fm_sb(long row, long g, long K) {
    const long rb = row >> 4, rr = row & 15;
    return ((rb * (K / 64) + g) * 8 + (rr & 7)) * 2 + (rr >> 3);
}
// index of (row, 32-group h) in the MXFP4 scale-byte array
__device__ __forceinline__ long fm_sc(long row, long h, long K) {
    const long rb = row >> 4, rr = row & 15;
    return (((rb * (K / 64) + (h >> 1)) * 8 + (rr & 7)) * 2 + (rr >> 3)) * 2 + (h & 1);
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
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t nat = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float q = rintf(__fdiv_rn(__fsub_rn(v[8 * j + i], bias), scale));
            q = q < 0.0f ? 0.0f : (q > 15.0f ? 15.0f : q);
            nat |= ((uint32_t)q & 0xfu) << (4 * i);
        }
        qw[fm_word(r, g * 8 + j, K)] = interleave_word(nat);
    }
    sb[fm_sb(r, g, K)] = (uint32_t)f2bf(scale) | ((uint32_t)f2bf(bias) << 16);
}

// fp32 dequant in natural element order: w = fmaf(scale, q, bias). One thread per packed word.
__global__ void k_q4_dequant(const uint32_t *__restrict__ qw, const uint32_t *__restrict__ sb, long rows, long K,
                             float *__restrict__ out) {
    const long nw = K / 8;
    const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * nw) return;
    const long r = gid / nw, j = gid - r * nw;
    const uint32_t nat = deinterleave_word(qw[fm_word(r, j, K)]);
    const uint32_t s_b = sb[fm_sb(r, j / 8, K)];
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
    const long r = gid / nw, j = gid - r * nw;
    qw[fm_word(r, j, K)] = interleave_word(wq[gid]);
    if ((j & 7) == 0) {
        const long gi = r * (K / 64) + j / 8;
        sb[fm_sb(r, j / 8, K)] = (uint32_t)scales[gi] | ((uint32_t)biases[gi] << 16);
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
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t nat = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) nat |= e2m1_round(__fmul_rn(v[8 * j + i], inv)) << (4 * i);
        qw[fm_word(r, g * 4 + j, K)] = interleave_word(nat);
    }
    sc[fm_sc(r, g, K)] = (uint8_t)(e + 127);
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
    const uint32_t nat = deinterleave_word(qw[fm_word(r, j, K)]);
    const int ex = (int)sc[fm_sc(r, j / 4, K)] - 127;
    float *dst = out + r * K + j * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = ldexpf(e2m1_value((nat >> (4 * i)) & 0xfu), ex);
}

__global__ void k_fp4_from_mlx(const uint32_t *__restrict__ wq, const uint8_t *__restrict__ scales, long rows,
                               long K, uint32_t *__restrict__ qw, uint8_t *__restrict__ sc) {
    const long nw = K / 8;
    const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * nw) return;
    const long r = gid / nw, j = gid - r * nw;
    qw[fm_word(r, j, K)] = interleave_word(wq[gid]);
    if ((j & 3) == 0) sc[fm_sc(r, j / 4, K)] = scales[r * (K / 32) + j / 4];
}

}  // namespace moeb
