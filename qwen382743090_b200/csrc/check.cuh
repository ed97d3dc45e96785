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

// ---- decoder-layer reference values -----------------------------------------
// The reference's CPU checks of its layer kernels (src/driver.cpp:8090-8242,
// 8365-8393 and 11255-11301) restated for one device thread per output: FP64
// arithmetic in the same order, every stored value rounded to float where
// the reference stores a float, each sum accumulated sequentially by one
// thread.  Only the double-precision exp / log1p / sqrt of the device's math
// library differ from the host's, by at most an ulp of the double.

// conv4 + SiLU + state roll, one thread per channel (src/driver.cpp:8090-8107).
__global__ void check_conv4_kernel(const float* __restrict__ qkv, const float* __restrict__ w,
                                   const float* __restrict__ st_in, float* out, float* st_out, uint32_t C) {
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const float x0 = st_in[c], x1 = st_in[C + c], x2 = st_in[2u * C + c], x3 = qkv[c];
    const float* wc = w + 4u * c;
    const double raw = __dadd_rn(__dadd_rn(__dadd_rn(__dmul_rn(x0, wc[0]), __dmul_rn(x1, wc[1])),
                                           __dmul_rn(x2, wc[2])),
                                 __dmul_rn(x3, wc[3]));
    out[c] = static_cast<float>(__ddiv_rn(raw, __dadd_rn(1.0, exp(-raw))));
    st_out[c] = x1;
    st_out[C + c] = x2;
    st_out[2u * C + c] = x3;
}

// Per head x * (1 / sqrt(sum x^2 + eps)) (src/driver.cpp:8109-8140); one
// thread per head for the sum, then one per element.
__global__ void check_l2norm_kernel(const float* __restrict__ x, uint32_t dim, float eps, float* y) {
    __shared__ double inv;
    const float* xh = x + static_cast<size_t>(blockIdx.x) * dim;
    if (threadIdx.x == 0) {
        double ss = 0.0;
        for (uint32_t i = 0; i < dim; ++i) ss = __dadd_rn(ss, __dmul_rn(xh[i], xh[i]));
        inv = __ddiv_rn(1.0, sqrt(__dadd_rn(ss, static_cast<double>(eps))));
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < dim; i += blockDim.x)
        y[static_cast<size_t>(blockIdx.x) * dim + i] = static_cast<float>(__dmul_rn(xh[i], inv));
}

// beta = sigmoid(b), gate = softplus(a + dt_bias) * A with the softplus
// branches at +-20 (src/driver.cpp:8142-8159).
__global__ void check_beta_gate_kernel(const float* b, const float* a, const float* dt, const float* A, uint32_t n,
                                       float* beta, float* gate) {
    const uint32_t h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h >= n) return;
    beta[h] = static_cast<float>(__ddiv_rn(1.0, __dadd_rn(1.0, exp(-static_cast<double>(b[h])))));
    const double v = __dadd_rn(a[h], dt[h]);
    const double sp = v > 20.0 ? v : (v < -20.0 ? exp(v) : log1p(exp(v)));
    gate[h] = static_cast<float>(__dmul_rn(sp, A[h]));
}

// One Gated DeltaNet step, one thread per (value head, column): state
// [H][col][row], q/k head h % Hq, decay e^g (src/driver.cpp:11255-11301).
__global__ void check_gdn_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                                 const float* __restrict__ g, const float* __restrict__ beta,
                                 const float* __restrict__ st_in, float* out, float* st_out, uint32_t Hq, uint32_t Hv,
                                 uint32_t D) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= Hv * D) return;
    const uint32_t h = i / D, c = i % D;
    const float* qh = q + static_cast<size_t>(h % Hq) * D;
    const float* kh = k + static_cast<size_t>(h % Hq) * D;
    const double G = exp(static_cast<double>(g[h])), B = beta[h];
    const double scale = __ddiv_rn(1.0, sqrt(static_cast<double>(D)));
    const size_t base = (static_cast<size_t>(h) * D + c) * D;
    double kv = 0.0;
    for (uint32_t r = 0; r < D; ++r) kv = __dadd_rn(kv, __dmul_rn(st_in[base + r], kh[r]));
    const double delta = __dmul_rn(__dsub_rn(v[i], __dmul_rn(G, kv)), B);
    double o = 0.0;
    for (uint32_t r = 0; r < D; ++r) {
        const double u = __dadd_rn(__dmul_rn(G, st_in[base + r]), __dmul_rn(kh[r], delta));
        st_out[base + r] = static_cast<float>(u);
        o = __dadd_rn(o, __dmul_rn(u, qh[r]));
    }
    out[i] = static_cast<float>(__dmul_rn(o, scale));
}

// Per head o * (1 / sqrt(mean(o^2) + eps)) * w * SiLU(z) (src/driver.cpp:
// 8216-8242), or with z null the whole-row RMSNorm x * inv * w of
// src/driver.cpp:8365-8381 (one "head" of n values).
__global__ void check_rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                     const float* __restrict__ z, uint32_t dim, float eps, float* y) {
    __shared__ double inv;
    const size_t off = static_cast<size_t>(blockIdx.x) * dim;
    if (threadIdx.x == 0) {
        double ss = 0.0;
        for (uint32_t i = 0; i < dim; ++i) ss = __dadd_rn(ss, __dmul_rn(x[off + i], x[off + i]));
        inv = __ddiv_rn(1.0, sqrt(__dadd_rn(__ddiv_rn(ss, static_cast<double>(dim)), static_cast<double>(eps))));
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < dim; i += blockDim.x) {
        double r = __dmul_rn(__dmul_rn(x[off + i], inv), w[i]);
        if (z) {
            const double zv = z[off + i];
            r = __dmul_rn(r, __ddiv_rn(zv, __dadd_rn(1.0, exp(-zv))));
        }
        y[off + i] = static_cast<float>(r);
    }
}

// SiLU(g) * u (src/driver.cpp:8383-8393).
__global__ void check_silu_mul_kernel(const float* g, const float* u, uint32_t n, float* y) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const double gv = g[i];
    y[i] = static_cast<float>(__dmul_rn(__ddiv_rn(gv, __dadd_rn(1.0, exp(-gv))), u[i]));
}

}  // namespace q38
