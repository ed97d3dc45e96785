// gemv_common.cuh -- pieces shared by the GEMV kernels: the deterministic
// boundary combine of row groups split between consumer warps, activation
// x-packs staged in shared memory (packed in-CTA from f32, optionally after
// RMSNorm), the fixed-order inverse RMS and the output epilogue.
#pragma once

#include "gemv_q5k.cuh"
#include "layer.cuh"

namespace q38 {

constexpr uint32_t kL2PrefetchPiece = 2048;
// Activations are staged in shared memory when they fit next to a kernel's
// ring and still leave room for the next kernel's CTA (PDL co-residency).
constexpr size_t kSmemBudget = 112u * 1024u;

// Partial sums of row groups (pairs or quads, R rows) split between
// consumers (C consumers, two entries each), combined after the main loop in
// consumer order.
template <int C, int R = 2>
struct PairBoundary {
    int pair[C * 2];
    double v[C * 2][R];
};
// Bytes of the activation x-pack for one row of nb super-blocks.
__host__ __device__ constexpr uint32_t xpack_smem_bytes(uint32_t nb, int nl) {
    return static_cast<uint32_t>(xpack_row_limb_bytes(nl, nb)) + nb * 32u + xpack_nb4(nb) * 4u;
}
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Integer dots of one 4-word chunk (16 weights of each group of pair p) of
// both rows with the chunk's activation limbs: a = group 2p, b = group 2p+1.
template <int NL>
__device__ __forceinline__ void q5_chunk_dot(uint4 q0, uint4 h0, uint4 q1, uint4 h1, const uint32_t (&xl)[8 * NL],
                                             uint32_t rot_lo, uint32_t rot_hi, int (&a0)[NL], int (&b0)[NL],
                                             int (&a1)[NL], int (&b1)[NL]) {
    const uint32_t qw0[4] = {q0.x, q0.y, q0.z, q0.w}, hw0[4] = {h0.x, h0.y, h0.z, h0.w};
    const uint32_t qw1[4] = {q1.x, q1.y, q1.z, q1.w}, hw1[4] = {h1.x, h1.y, h1.z, h1.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t lo0, hi0, lo1, hi1;
        q5_decode(qw0[i], hw0[i], rot_lo, rot_hi, lo0, hi0);
        q5_decode(qw1[i], hw1[i], rot_lo, rot_hi, lo1, hi1);
#pragma unroll
        for (int k = 0; k < NL; ++k) {
            a0[k] = dp4a(lo0, xl[(i * 2 + 0) * NL + k], a0[k]);
            b0[k] = dp4a(hi0, xl[(i * 2 + 1) * NL + k], b0[k]);
            a1[k] = dp4a(lo1, xl[(i * 2 + 0) * NL + k], a1[k]);
            b1[k] = dp4a(hi1, xl[(i * 2 + 1) * NL + k], b1[k]);
        }
    }
}

// Output row value, plus the residual when one is given (y may alias res:
// each row is read and written by the same thread).
__device__ __forceinline__ float gemv_out(double v, const float* res, uint32_t row) {
    return static_cast<float>(res ? v + static_cast<double>(res[row]) : v);
}

template <int NL, bool XS>
__device__ __forceinline__ uint4 xpack_load_quad(const uint8_t* p) {
    if constexpr (XS) return *reinterpret_cast<const uint4*>(p);
    else return __ldcg(reinterpret_cast<const uint4*>(p));
}

// Pack one row of f32 activations (nb super-blocks) into the three-limb
// x-pack layout in shared memory, one warp per super-block.  With nw given the
// packed values are the RMSNorm output x * inv * nw.
__device__ __forceinline__ void pack_x_f32_smem(const float* __restrict__ x, uint32_t nb, uint8_t* xs, float* gsum,
                                              float* scale, uint32_t warp, uint32_t lane, uint32_t nwarps,
                                              const float* __restrict__ nw = nullptr, float inv = 1.0f) {
    for (uint32_t b = warp; b < nb; b += nwarps) {
        const float4 v0 = __ldcg(reinterpret_cast<const float4*>(x + b * 256u + lane * 8u));
        const float4 v1 = __ldcg(reinterpret_cast<const float4*>(x + b * 256u + lane * 8u + 4u));
        float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        if (nw) {
            const float4 w0 = __ldg(reinterpret_cast<const float4*>(nw + b * 256u + lane * 8u));
            const float4 w1 = __ldg(reinterpret_cast<const float4*>(nw + b * 256u + lane * 8u + 4u));
            const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int t = 0; t < 8; ++t) v[t] = v[t] * inv * w[t];
        }
        pack_block_warp<3>(v, b, lane, xs, gsum, scale);
    }
}

// 1 / sqrt(mean(x^2) + eps) of one f32 row of nb super-blocks, the same bits
// for any block size: per super-block a fixed-order fp32 lane sum and an fp64
// butterfly, then one thread adds the blocks in order.  blk holds nb doubles
// of shared memory; every thread gets the result.
__device__ __forceinline__ float row_inv_rms(const float* __restrict__ x, uint32_t nb, float eps, double* blk,
                                             float* inv_out, uint32_t warp, uint32_t lane, uint32_t nwarps) {
    for (uint32_t b = warp; b < nb; b += nwarps) {
        const float4 v0 = __ldcg(reinterpret_cast<const float4*>(x + b * 256u + lane * 8u));
        const float4 v1 = __ldcg(reinterpret_cast<const float4*>(x + b * 256u + lane * 8u + 4u));
        float s = v0.x * v0.x;
        s = fmaf(v0.y, v0.y, s); s = fmaf(v0.z, v0.z, s); s = fmaf(v0.w, v0.w, s);
        s = fmaf(v1.x, v1.x, s); s = fmaf(v1.y, v1.y, s); s = fmaf(v1.z, v1.z, s); s = fmaf(v1.w, v1.w, s);
        double d = s;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (lane == 0) blk[b] = d;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (uint32_t b = 0; b < nb; ++b) t += blk[b];
        *inv_out = static_cast<float>(1.0 / sqrt(t / (256.0 * nb) + static_cast<double>(eps)));
    }
    __syncthreads();
    return *inv_out;
}

// n floats from src to dst by the SMs, for the vectors of a host-buffer GEMV:
// src or dst is page-locked host memory read or written over the bus
// (volatile loads: nothing of it stays cached on the device).  For a few KB
// this is far quicker than a copy-engine transfer and chains to the GEMV
// with PDL.
__global__ void __launch_bounds__(256) copy_f32_kernel(const float* src, float* dst, uint32_t n) {
    pdl_launch_dependents();
    pdl_wait();
    for (uint32_t i = blockIdx.x * 256u + threadIdx.x; i < n; i += gridDim.x * 256u) dst[i] = __ldcv(src + i);
}
// The same with 16-byte accesses (src and dst 16-byte aligned, n4 = n / 4):
// a quarter of the bus requests, which set the time of a host read.
__global__ void __launch_bounds__(256) copy_f32x4_kernel(const float4* src, float4* dst, uint32_t n4) {
    pdl_launch_dependents();
    pdl_wait();
    for (uint32_t i = blockIdx.x * 256u + threadIdx.x; i < n4; i += gridDim.x * 256u) dst[i] = __ldcv(src + i);
}

// Largest row the fused RMSNorm handles (super-blocks).
constexpr uint32_t kNormMaxBlocks = 128;

}  // namespace q38
