// q81.cuh -- Q8_1 activations and the IQ4_XS x Q8_1 GEMV (the variant the
// reference built and set aside as slower than F32 activations,
// src/driver.cpp:2641-2875, README "IQ4_XS x Q8_1").
//
// Q8_1 block (36 B per 32 values, src/quant.cpp:264-313): d fp16 | s fp16 |
// int8 qs[32], with d = amax / 127, q = clamp(round(x / d), -127, 127) and
// s = d * sum(q).  quantize_q8_1_kernel restates quantize_q8_1_cpu for one warp
// per block (lane j holds value j): the same float operations in the same
// order (the division, the reciprocal, the product, round-half-away, the
// fp16 conversions with round-to-nearest-even), so the blocks are bit-exact.
//
// IQ4_XS x Q8_1: IQ4_XS groups of 32 weights (scale ls - 32) line up with the
// Q8_1 blocks, so each group is one exact integer dot (codebook int8 x q8 by
// dp4a) times d_w * (ls - 32) * d_x, summed in FP64 over the row; one warp per
// row, lanes over groups.
#pragma once

#include "gemv_kq.cuh"

namespace q38 {

constexpr uint32_t kQ81Bytes = 36;

__global__ void __launch_bounds__(256) quantize_q8_1_kernel(const float* __restrict__ x, uint32_t nblocks,
                                                            uint8_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t b = blockIdx.x * 8u + (threadIdx.x >> 5);
    if (b >= nblocks) return;  // warp-uniform
    const float v = __ldcg(x + static_cast<size_t>(b) * 32u + lane);
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    int q = static_cast<int>(roundf(v * id));
    q = max(-127, min(127, q));
    int sum = q;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    uint8_t* blk = out + static_cast<size_t>(b) * kQ81Bytes;
    blk[4u + lane] = static_cast<uint8_t>(static_cast<int8_t>(q));
    if (lane == 0) {
        const float s = static_cast<float>(sum) * d;
        const uint16_t dh = __half_as_ushort(__float2half_rn(d)), sh = __half_as_ushort(__float2half_rn(s));
        *reinterpret_cast<uint32_t*>(blk) = static_cast<uint32_t>(dh) | (static_cast<uint32_t>(sh) << 16);
    }
}

__global__ void __launch_bounds__(256) iq4xs_q81_gemv_kernel(const uint8_t* __restrict__ w,
                                                             const uint8_t* __restrict__ xq, float* __restrict__ y,
                                                             uint32_t nb, uint32_t rows) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t row = blockIdx.x * 8u + (threadIdx.x >> 5);
    if (row >= rows) return;  // warp-uniform
    const uint8_t* wr = w + static_cast<size_t>(row) * nb * 136u;
    double acc = 0.0;
    for (uint32_t g = lane; g < nb * 8u; g += 32u) {
        const uint32_t b = g >> 3, j = g & 7u;
        const uint8_t* blk = wr + static_cast<size_t>(b) * 136u;
        const uint32_t head = __ldg(reinterpret_cast<const uint32_t*>(blk));  // d | scales_h
        const uint32_t sl = __ldg(blk + 4u + (j >> 1));
        const int ls = static_cast<int>(((sl >> (4u * (j & 1u))) & 15u) | (((head >> (16u + 2u * j)) & 3u) << 4));
        const float dw = half_bits_to_float(head);
        const uint32_t* qs = reinterpret_cast<const uint32_t*>(blk + 8u + 16u * j);
        const uint8_t* xb = xq + static_cast<size_t>(g) * kQ81Bytes;  // Q8_1 block g of the row
        const float dx = half_bits_to_float(__ldcg(reinterpret_cast<const uint32_t*>(xb)));
        const uint32_t* x8 = reinterpret_cast<const uint32_t*>(xb + 4u);
        int sumi = 0;
#pragma unroll
        for (uint32_t i = 0; i < 4u; ++i) {
            const uint32_t q = __ldg(qs + i);
            sumi = dp4a(iq4nl_lookup4(q & 0x0f0f0f0fu), __ldcg(x8 + i), sumi);
            sumi = dp4a(iq4nl_lookup4((q >> 4) & 0x0f0f0f0fu), __ldcg(x8 + 4u + i), sumi);
        }
        acc = fma(static_cast<double>(sumi), static_cast<double>(dw * static_cast<float>(ls - 32)) *
                                                static_cast<double>(dx),
                  acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[row] = static_cast<float>(acc);
}

}  // namespace q38
