// xpack.cuh -- activation packing for the integer-dot GEMV kernels.
//
// Every K-quant GEMV here computes its dot products with dp4a on int8
// operands.  The activation vector x is therefore handed to the GEMV as an
// "x-pack" with three regions:
//
//   limbs  int8   NL bytes per element, in GEMV lane order (below)
//   gsum   float  [B][nb][8]   sum over each 32-weight group of x as packed
//   scale  float  [B][nb]      value of one unit of limb 0
//
// with nb = K/256 super-blocks.  For F32 activations NL = 3 or 4: each
// 256-block is scaled by the largest power of two 2^s that keeps |x| * 2^s
// inside the balanced NL-limb range, rounded to an integer xi and split into
// signed bytes xi = l0 + 256*l1 + 65536*l2 (+ 2^24*l3).  Every element keeps
// 23 (NL = 3) or 30 (NL = 4) bits relative to the block maximum and the dot
// products are exact integers.  The rounding of x is then the only error
// against an FP64 dot: for N(0,1) activations and the benchmark's weights its
// standard deviation is about 2.3e-5 at K = 5120 with three limbs and 4e-5 at
// K = 17408, so wide projections use four limbs (about 2^-7 of that).  For
// Q8_K activations NL = 1: the limb is the Q8_K byte itself, scale is the
// Q8_K d and gsum comes from the Q8_K bsums, exactly the quantities the
// reference's Q5_K x Q8_K kernel uses (src/driver.cpp:3660-3885).
//
// Limb order.  A GEMV lane owns (super-block b, pair of groups p) and reads,
// for each of 8 words i (weights 4i..4i+3 of groups 2p and 2p+1), the NL limb
// words of group 2p then of group 2p+1.  Those 8*2*NL u32 form 4*NL 16-byte
// quads q (words 0-3 -> quads [0, 2NL), words 4-7 -> quads [2NL, 4NL)).  The
// quads are stored quad-major over a group of 4 super-blocks:
//     offset = (((b/4) * 4NL + q) * 4 + b%4) * 4 + p) * 16
// so the 16 lanes (b%4, p) of a GEMV warp that read quad q at the same time
// touch 256 contiguous bytes.
#pragma once

#include "common.cuh"

namespace q38 {

constexpr int kQK = 256;

__host__ __device__ constexpr uint32_t xpack_record_bytes(int nl) { return 64u * static_cast<uint32_t>(nl); }
// The quad-major order interleaves groups of 4 super-blocks, so a row's limb
// region always spans a whole number of such groups.
__host__ __device__ constexpr uint32_t xpack_nb4(uint32_t nb) { return (nb + 3u) & ~3u; }
__host__ __device__ constexpr size_t xpack_row_limb_bytes(int nl, uint32_t nb) {
    return static_cast<size_t>(xpack_nb4(nb)) * 4u * xpack_record_bytes(nl);
}
__host__ __device__ constexpr size_t xpack_limb_bytes(int nl, uint32_t nb, uint32_t batch) {
    return static_cast<size_t>(batch) * xpack_row_limb_bytes(nl, nb);
}

// Byte offset of limb `limb` of element j (0..255) of super-block b inside the
// limb region of one batch row.
__device__ __forceinline__ uint32_t xpack_offset(uint32_t b, uint32_t j, uint32_t limb, int nl) {
    const uint32_t g = j >> 5, l = j & 31u;
    const uint32_t p = g >> 1, grp = g & 1u, i = l >> 2, m = l & 3u;
    const uint32_t word = (i * 2u + grp) * static_cast<uint32_t>(nl) + limb;  // u32 index within the record
    const uint32_t q = word >> 2, wq = word & 3u;
    const uint32_t quad = (((b >> 2) * 4u * static_cast<uint32_t>(nl) + q) * 4u + (b & 3u)) * 4u + p;
    return quad * 16u + wq * 4u + m;
}

// Exact value sum_k 256^k * t[k] of NL limb dot products (|t[k]| < 2^26), in
// fp64: exact for NL <= 4.
template <int NL>
__device__ __forceinline__ double limb_value(const int (&t)[NL]) {
    double v = static_cast<double>(t[NL - 1]);
#pragma unroll
    for (int k = NL - 2; k >= 0; --k) v = __fma_rn(v, 256.0, static_cast<double>(t[k]));
    return v;
}

// Integer bits kept per activation, relative to the largest power of two at or
// above its 256-block's maximum: 23 for three limbs, 30 for four.
template <int NL>
__host__ __device__ constexpr int xpack_bits() {
    return NL == 3 ? 23 : 30;
}
// Largest positive integer the balanced NL-limb form holds (0x7f..7f).
template <int NL>
__host__ __device__ constexpr double xpack_limit() {
    return NL == 3 ? 8355711.0 : 2139062143.0;
}

// Scale of a block whose largest magnitude is amax (> 0, finite): the shift s
// that gives amax * 2^s xpack_bits<NL> integer bits inside the balanced range
// (frexp semantics, one step down when rounding would exceed the limit), and
// unit = 2^-s (0 when 2^-s is below the smallest subnormal).  *mul = 2^s when
// both 2^s and 2^-s are normal floats, else 0 (then s > 126: amax is tiny).
// Everything comes from the float's bits -- no frexpf/ldexpf: a subnormal amax
// is first scaled by 2^64 (exact), and 2^s beyond the normal range is applied
// as 2^126 * 2^(s - 126), both factors exact.
template <int NL>
__device__ __forceinline__ int xpack_shift(float amax, float* mul, float* unit) {
    const int ebits = (__float_as_int(amax) >> 23) & 0xff;
    const int e = ebits != 0 ? ebits - 126  // amax = m * 2^e, m in [0.5, 1)
                             : ((__float_as_int(amax * 0x1p64f) >> 23) & 0xff) - 126 - 64;
    int s = xpack_bits<NL>() - e;
    const bool fast = s >= -125 && s <= 126;
    const float scaled = fast ? amax * __int_as_float((s + 127) << 23)
                              : amax * 0x1p126f * __int_as_float((s - 126 + 127) << 23);
    if (static_cast<double>(scaled) > xpack_limit<NL>()) s -= 1;
    if (fast) {
        *mul = __int_as_float((s + 127) << 23);
        *unit = __int_as_float((127 - s) << 23);
    } else {
        *mul = 0.0f;
        *unit = s <= 149 ? __int_as_float(1 << (149 - s)) : 0.0f;  // subnormal 2^-s
    }
    return s;
}
// round(v * 2^s) with the scale from xpack_shift (s > 126 when mul is 0; every
// product is exact, so this is ldexpf(v, s) rounded to the nearest integer).
__device__ __forceinline__ int xpack_scale_round(float v, int s, float mul) {
    return __float2int_rn(mul != 0.0f ? v * mul : v * 0x1p126f * __int_as_float((s - 126 + 127) << 23));
}

// One CTA of 256 threads per (super-block, batch row), NL = 3 or 4.  Also the
// place where a producer kernel (RMSNorm, SiLU*up, gated norm) would emit its
// output.
template <int NL>
__global__ void __launch_bounds__(256) xpack_f32_kernel(const float* __restrict__ x, uint32_t K,
                                                        uint8_t* __restrict__ limbs, float* __restrict__ gsum,
                                                        float* __restrict__ scale) {
    static_assert(NL == 3 || NL == 4, "f32 activations use three or four limbs");
    pdl_wait();
    const uint32_t nb = K / kQK;
    const uint32_t b = blockIdx.x, t = blockIdx.y, j = threadIdx.x;
    if (b >= nb) {  // a grid wider than K: zero padding blocks of a K-sliced projection
        uint8_t* row = limbs + static_cast<size_t>(t) * xpack_row_limb_bytes(NL, gridDim.x);
#pragma unroll
        for (int k = 0; k < NL; ++k) row[xpack_offset(b, j, static_cast<uint32_t>(k), NL)] = 0;
        if ((j & 31u) == 0) gsum[(static_cast<size_t>(t) * gridDim.x + b) * 8u + (j >> 5)] = 0.0f;
        if (j == 0) scale[static_cast<size_t>(t) * gridDim.x + b] = 0.0f;
        pdl_launch_dependents();
        return;
    }
    const float v = x[static_cast<size_t>(t) * K + static_cast<size_t>(b) * kQK + j];

    __shared__ float wmax[8];
    float a = fabsf(v);
    if (!(a <= 3.0e38f)) a = INFINITY;  // NaN/inf poison the whole block
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if ((j & 31u) == 0) wmax[j >> 5] = a;
    __syncthreads();
    float amax = wmax[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) amax = fmaxf(amax, wmax[w]);

    int xi = 0;
    float unit = 0.0f;  // value of one integer step
    if (amax == INFINITY) {
        unit = __int_as_float(0x7fc00000);  // NaN: every dot touching this block becomes NaN
    } else if (amax > 0.0f) {
        // Largest power-of-two scale that keeps every element inside the
        // balanced NL-limb range.
        float mul;
        const int s = xpack_shift<NL>(amax, &mul, &unit);
        xi = xpack_scale_round(v, s, mul);
    }
    const uint32_t nbp = gridDim.x;  // packed blocks per row (nb, or more with padding)
    uint8_t* row = limbs + static_cast<size_t>(t) * xpack_row_limb_bytes(NL, nbp);
    int r = xi;
#pragma unroll
    for (int k = 0; k < NL; ++k) {
        const int l = ((r + 128) & 255) - 128;  // balanced byte
        row[xpack_offset(b, j, static_cast<uint32_t>(k), NL)] = static_cast<uint8_t>(l);
        r = (r - l) >> 8;
    }

    double gs = static_cast<double>(xi);  // exact: |sum of 32| < 2^36
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) gs += __shfl_xor_sync(0xffffffffu, gs, o);
    if ((j & 31u) == 0)
        gsum[(static_cast<size_t>(t) * nbp + b) * 8u + (j >> 5)] = static_cast<float>(gs * static_cast<double>(unit));
    if (j == 0) scale[static_cast<size_t>(t) * nbp + b] = unit;
    pdl_launch_dependents();
}

// Balanced base-256 limbs of eight quantised values (|xi| inside the NL-limb
// range): lw[h][k] holds limb k of values 4h..4h+3, byte i for value 4h+i.
// The balanced digits of xi are the bytes of xi + 0x80..80 with 128 taken off
// each (one add and one xor give all limbs of a value), then 4x4 byte
// transposes.  Returns the exact sum of the eight values, from the limb sums.
template <int NL>
__device__ __forceinline__ double xpack_limbs8(const int (&xi)[8], uint32_t (&lw)[2][4]) {
    constexpr uint32_t kBias = NL == 3 ? 0x00808080u : 0x80808080u;
    uint32_t dg[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) dg[t] = (static_cast<uint32_t>(xi[t]) + kBias) ^ kBias;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t lo01 = __byte_perm(dg[4 * h], dg[4 * h + 1], 0x5140u);
        const uint32_t hi01 = __byte_perm(dg[4 * h], dg[4 * h + 1], 0x7362u);
        const uint32_t lo23 = __byte_perm(dg[4 * h + 2], dg[4 * h + 3], 0x5140u);
        const uint32_t hi23 = __byte_perm(dg[4 * h + 2], dg[4 * h + 3], 0x7362u);
        lw[h][0] = __byte_perm(lo01, lo23, 0x5410u);
        lw[h][1] = __byte_perm(lo01, lo23, 0x7632u);
        lw[h][2] = __byte_perm(hi01, hi23, 0x5410u);
        lw[h][3] = __byte_perm(hi01, hi23, 0x7632u);
    }
    double gs = 0.0;
#pragma unroll
    for (int k = NL - 1; k >= 0; --k)
        gs = __fma_rn(gs, 256.0,
                      static_cast<double>(__dp4a(static_cast<int>(lw[0][k]), 0x01010101,
                                                 __dp4a(static_cast<int>(lw[1][k]), 0x01010101, 0))));
    return gs;
}

// Pack super-block b of a row with one warp: lane l holds elements 8l..8l+7
// in v.  Same arithmetic as xpack_f32_kernel<NL> (largest power-of-two scale
// inside the balanced NL-limb range, round to nearest even, balanced limbs,
// exact group sums), so both produce identical bytes.  limbs/gsum/scale point
// at the row's regions (shared or global memory).
template <int NL>
__device__ __forceinline__ void pack_block_warp(const float (&v)[8], uint32_t b, uint32_t lane, uint8_t* limbs,
                                                float* gsum, float* scale) {
    float a = 0.0f;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        float ab = fabsf(v[t]);
        if (!(ab <= 3.0e38f)) ab = INFINITY;
        a = fmaxf(a, ab);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    int sh = 0;
    float unit = 0.0f, mul = 0.0f;
    const bool poison = a == INFINITY;
    if (poison) {
        unit = __int_as_float(0x7fc00000);
    } else if (a > 0.0f) {
        sh = xpack_shift<NL>(a, &mul, &unit);
    }
    int xi[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) xi[t] = (poison || a == 0.0f) ? 0 : xpack_scale_round(v[t], sh, mul);
    uint32_t lw[2][4];
    double gs = xpack_limbs8<NL>(xi, lw);
    // element j = 8*lane + t: group g = lane/4, word i = 2*(lane%4) + t/4
    const uint32_t g = lane >> 2, p = g >> 1, grp = g & 1u;
#pragma unroll
    for (int hw = 0; hw < 2; ++hw) {
        const uint32_t i = 2u * (lane & 3u) + hw;
#pragma unroll
        for (int k = 0; k < NL; ++k) {
            const uint32_t word = (i * 2u + grp) * NL + k;
            const uint32_t q = word >> 2, wq = word & 3u;
            const uint32_t quad = (((b >> 2) * 4u * NL + q) * 4u + (b & 3u)) * 4u + p;
            *reinterpret_cast<uint32_t*>(limbs + quad * 16u + wq * 4u) = lw[hw][k];
        }
    }
    gs += __shfl_xor_sync(0xffffffffu, gs, 1);
    gs += __shfl_xor_sync(0xffffffffu, gs, 2);
    if ((lane & 3u) == 0) gsum[b * 8u + g] = static_cast<float>(gs * static_cast<double>(unit));
    if (lane == 0) scale[b] = unit;
}

// Q8_K blocks (f32 d | int8 qs[256] | int16 bsums[16], 292 B) -> x-pack, NL=1.
__global__ void __launch_bounds__(256) xpack_q8k_kernel(const uint8_t* __restrict__ q8, uint32_t nb,
                                                        uint8_t* __restrict__ limbs, float* __restrict__ gsum,
                                                        float* __restrict__ scale) {
    pdl_wait();
    const uint32_t b = blockIdx.x, t = blockIdx.y, j = threadIdx.x;
    const uint8_t* src = q8 + (static_cast<size_t>(t) * nb + b) * 292u;
    float d;
    memcpy(&d, src, 4);
    uint8_t* row = limbs + static_cast<size_t>(t) * xpack_row_limb_bytes(1, nb);
    row[xpack_offset(b, j, 0, 1)] = src[4 + j];
    if (j < 8) {
        int16_t s0, s1;
        memcpy(&s0, src + 260 + 4 * j, 2);
        memcpy(&s1, src + 262 + 4 * j, 2);
        gsum[(static_cast<size_t>(t) * nb + b) * 8u + j] = d * static_cast<float>(s0 + s1);
    }
    if (j == 0) scale[static_cast<size_t>(t) * nb + b] = d;
    pdl_launch_dependents();
}

}  // namespace q38
