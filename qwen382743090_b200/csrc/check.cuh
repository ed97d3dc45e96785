// check.cuh -- reference rows for the smoke entries' checks, on the device.
//
// The reference checks each GPU GEMV against a CPU dequantisation and an FP64
// dot of the first rows (src/driver.cpp:6946-6965).  The C++ host facade does
// the same check here instead, with plain code independent of the fast
// kernels: one thread per weight of a super-block, the block formats of
// quant.cpp restated with its float operation order (products and differences
// as separate IEEE operations, never contracted), and an FP64 dot in a fixed
// order.  The dequantised weights are bit-exact to the CPU functions; the dot
// differs from a sequential FP64 sum only by its summation order.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace q38 {

struct CheckArgs {
    uint32_t type, layout;  // GGML type; 0 = GGUF blocks, 1 = Q5_K SoA planes
    const uint8_t* w;       // blocks, or the META plane
    const uint8_t* aux0;    // QH plane (layout 1)
    const uint8_t* aux1;    // QS plane (layout 1)
    uint32_t cols;
    const float* x;  // f32 [cols] or null
    double* y;       // FP64 [rows] (with x)
    float* deq;      // f32 [rows][cols] or null
};

__device__ __forceinline__ float ck_half(const uint8_t* p) {
    return __half2float(__ushort_as_half(static_cast<uint16_t>(p[0] | (p[1] << 8))));
}

// get_scale_min_k4 (src/quant.cpp:89-97).
__device__ __forceinline__ void ck_scale_min(int j, const uint8_t* s, int& sc, int& mn) {
    if (j < 4) {
        sc = s[j] & 63;
        mn = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// Weight n (0..255) of super-block b of `row`.
__device__ float ck_weight(const CheckArgs& a, uint32_t row, uint32_t b, int n) {
    const size_t blk = static_cast<size_t>(row) * (a.cols / 256u) + b;
    const int g = n >> 5, l = n & 31;
    if (a.layout == 1) {  // Q5_K SoA: META20 | QH32 | QS128 planes (src/quant.cpp:425-463)
        const uint8_t* meta = a.w + blk * 20u;
        const uint8_t* qh = a.aux0 + blk * 32u;
        const uint8_t* qs = a.aux1 + blk * 128u;
        const float ds = __fmul_rn(ck_half(meta), static_cast<float>(meta[4 + 2 * g]));
        const float dm = __fmul_rn(ck_half(meta + 2), static_cast<float>(meta[5 + 2 * g]));
        const uint8_t byte = qs[(g >> 1) * 32 + l];
        int q = (g & 1) ? (byte >> 4) : (byte & 15);
        if (qh[l] & (1u << g)) q += 16;
        return __fsub_rn(__fmul_rn(ds, static_cast<float>(q)), dm);
    }
    switch (a.type) {
        case 12: {  // Q4_K, 144 B (src/quant.cpp:99-136)
            const uint8_t* p = a.w + blk * 144u;
            int sc, mn;
            ck_scale_min(g, p + 4, sc, mn);
            const float ds = __fmul_rn(ck_half(p), static_cast<float>(sc));
            const float dm = __fmul_rn(ck_half(p + 2), static_cast<float>(mn));
            const uint8_t byte = p[16 + (g >> 1) * 32 + l];
            const int q = (g & 1) ? (byte >> 4) : (byte & 15);
            return __fsub_rn(__fmul_rn(ds, static_cast<float>(q)), dm);
        }
        case 13: {  // Q5_K, 176 B (src/quant.cpp:138-183)
            const uint8_t* p = a.w + blk * 176u;
            int sc, mn;
            ck_scale_min(g, p + 4, sc, mn);
            const float ds = __fmul_rn(ck_half(p), static_cast<float>(sc));
            const float dm = __fmul_rn(ck_half(p + 2), static_cast<float>(mn));
            const uint8_t byte = p[48 + (g >> 1) * 32 + l];
            int q = (g & 1) ? (byte >> 4) : (byte & 15);
            if (p[16 + l] & (1u << g)) q += 16;
            return __fsub_rn(__fmul_rn(ds, static_cast<float>(q)), dm);
        }
        case 14: {  // Q6_K, 210 B (src/quant.cpp:186-249)
            const uint8_t* p = a.w + blk * 210u;
            const int h = n >> 7, r = n & 127, t = r >> 5, lr = r & 31;
            const uint8_t lb = p[64 * h + lr + 32 * (t & 1)];
            const int lo = t < 2 ? (lb & 15) : (lb >> 4);
            const int hi = (p[128 + 32 * h + lr] >> (2 * t)) & 3;
            const int q = (lo | (hi << 4)) - 32;
            const int8_t sc = static_cast<int8_t>(p[192 + 8 * h + 2 * t + lr / 16]);
            return __fmul_rn(__fmul_rn(ck_half(p + 208), static_cast<float>(sc)), static_cast<float>(q));
        }
        case 23: {  // IQ4_XS, 136 B (src/quant.cpp:465-503), the IQ4_NL codebook of :468-471
            const uint8_t* p = a.w + blk * 136u;
            const int8_t kv[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
            const int sh = p[2] | (p[3] << 8);
            const int ls = ((p[4 + (g >> 1)] >> (4 * (g & 1))) & 15) | (((sh >> (2 * g)) & 3) << 4);
            const float dl = __fmul_rn(ck_half(p), static_cast<float>(ls - 32));
            const uint8_t byte = p[8 + 16 * g + (l & 15)];
            return __fmul_rn(dl, static_cast<float>(kv[l < 16 ? (byte & 15) : (byte >> 4)]));
        }
        default:
            return 0.0f;
    }
}

// One CTA of 256 threads per row: every super-block dequantised one weight
// per thread (written to deq when given), products summed in FP64 by a fixed
// tree, super-blocks added in order.
__global__ void __launch_bounds__(256) check_rows_kernel(const CheckArgs a) {
    __shared__ double red[256];
    const uint32_t row = blockIdx.x, n = threadIdx.x, nb = a.cols / 256u;
    double acc = 0.0;
    for (uint32_t b = 0; b < nb; ++b) {
        const float w = ck_weight(a, row, b, static_cast<int>(n));
        if (a.deq) a.deq[static_cast<size_t>(row) * a.cols + b * 256u + n] = w;
        if (!a.x) continue;
        red[n] = static_cast<double>(w) * static_cast<double>(a.x[b * 256u + n]);
        __syncthreads();
        for (uint32_t s = 128; s > 0; s >>= 1) {
            if (n < s) red[n] += red[n + s];
            __syncthreads();
        }
        if (n == 0) acc += red[0];
        __syncthreads();
    }
    if (n == 0 && a.x && a.y) a.y[row] = acc;
}

}  // namespace q38
