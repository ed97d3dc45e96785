// gemv_kq.cuh -- K-quant GEMV over the GGUF-native row-major layout (Q38PACK
// layout 0): Q4_K, Q5_K, Q6_K and IQ4_XS weights with F32 (three limbs) or
// Q8_K (one limb) activations.  Same mathematics as the reference kernels
//   q38_q4k_gemv_f32          src/driver.cpp:1852-2021
//   q38_q5k_gemv_f32          src/driver.cpp:3248-3453
//   q38_q6k_gemv_f32_scalar   src/driver.cpp:1315-1473
//   q38_iq4xs_gemv_f32_prmt   src/driver.cpp:2877-3120
//   q38_q5k_q8k_dp4a_gemv     src/driver.cpp:3660-3885
// and the block formats of src/quant.cpp (Q4_K :99-136, Q5_K :138-183,
// Q6_K :186-249, IQ4_XS :465-503).
//
// Structure (shared with the tiled Q5_K kernel of gemv_tiled.cuh):
//  * a tile is 2 rows x 4 super-blocks; in layout 0 that is two row segments
//    of 4 blocks, each fetched by one 1-D bulk TMA copy into the consumer's
//    private shared-memory ring slot.  Q6_K (210-byte blocks) and IQ4_XS
//    (136-byte blocks) segments need not start on 16 bytes, so their copies
//    cover the enclosing 16-byte-aligned span and the consumer reads from the
//    offset inside it;
//  * 2*W consumers (half-warps) per CTA each own a contiguous run of the CTA's
//    tiles, prefetched into L2 at kernel entry before the PDL dependency wait;
//  * lane (s, p) of a consumer decodes super-block s, group pair p of both
//    rows, so each activation word it loads serves two rows; integer dp4a
//    dots against the x-pack limbs, integer group scales, fp32 per-lane sums,
//    fp64 reductions and a deterministic boundary combine.
//
// Memory contract: a Q6_K or IQ4_XS tensor must be readable up to the next
// 16-byte boundary after its last byte (true for every tensor inside a
// Q38PACK file mapping and for q38_alloc'd buffers).
#pragma once

#include "gemv_common.cuh"

namespace q38 {

template <int T>
struct KqType;
template <>
struct KqType<12> {  // Q4_K: d, dmin | scales[12] | qs[128]
    static constexpr uint32_t kBlock = 144, kWarps = 16;
    static constexpr bool kUnaligned = false;
};
template <>
struct KqType<13> {  // Q5_K: d, dmin | scales[12] | qh[32] | qs[128]
    static constexpr uint32_t kBlock = 176, kWarps = 12;
    static constexpr bool kUnaligned = false;
};
template <>
struct KqType<14> {  // Q6_K: ql[128] | qh[64] | int8 scales[16] | d
    static constexpr uint32_t kBlock = 210, kWarps = 12;
    static constexpr bool kUnaligned = true;
};
template <>
struct KqType<23> {  // IQ4_XS: d | scales_h | scales_l[4] | qs[128]
    static constexpr uint32_t kBlock = 136, kWarps = 12;
    static constexpr bool kUnaligned = true;
};

constexpr uint32_t kKqDepth = 2;

template <int T>
__host__ __device__ constexpr uint32_t kq_seg_stride() {
    return KqType<T>::kUnaligned ? ((4u * KqType<T>::kBlock + 15u + 15u) & ~15u) : 4u * KqType<T>::kBlock;
}
template <int T, int W = KqType<T>::kWarps>
__host__ __device__ constexpr size_t kq_ring_bytes() {
    return static_cast<size_t>(2u * W) * kKqDepth * 2u * kq_seg_stride<T>();
}
template <int T, int W = KqType<T>::kWarps>
__host__ __device__ constexpr size_t kq_fixed_bytes() {
    constexpr uint32_t C = 2u * W;
    return kq_ring_bytes<T, W>() + C * kKqDepth * 8u + 8u + sizeof(PairBoundary<C>) + 256u;
}
template <int T, int W = KqType<T>::kWarps>
__host__ __device__ constexpr size_t kq_smem_bytes(uint32_t nb, int nl, bool xsmem) {
    return kq_fixed_bytes<T, W>() + (xsmem ? xpack_smem_bytes(nb, nl) : 0u);
}

// ---- per-type pieces ---------------------------------------------------------

// 16 bytes at a 2-byte-aligned shared-memory address: five aligned words and a
// funnel shift (the shift is 0 or 16 bits).
__device__ __forceinline__ void lds16_unaligned(const uint8_t* p, uint32_t (&o)[4]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    const uint32_t sh = 8u * static_cast<uint32_t>(a & 3u);
    uint32_t v[5];
#pragma unroll
    for (int k = 0; k < 5; ++k) v[k] = w[k];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = __funnelshift_r(v[k], v[k + 1], sh);
}
__device__ __forceinline__ uint32_t lds4_unaligned(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    return __funnelshift_r(w[0], w[1], 8u * static_cast<uint32_t>(a & 3u));
}

// get_scale_min_k4 (src/quant.cpp:89-97) for groups 2p and 2p+1 of a Q4_K /
// Q5_K header {d|dmin, scales[0..3], scales[4..7], scales[8..11]}.
__device__ __forceinline__ void kq_scale_min_pair(uint4 hd, uint32_t p, int& sa, int& sb, int& ma, int& mb) {
    const uint32_t q = (p & 1u) * 16u;
    const uint32_t y = hd.y >> q, z = hd.z >> q, w = hd.w >> q;
    if (p < 2u) {
        sa = static_cast<int>(y & 63u);
        sb = static_cast<int>((y >> 8) & 63u);
        ma = static_cast<int>(z & 63u);
        mb = static_cast<int>((z >> 8) & 63u);
    } else {
        sa = static_cast<int>((w & 15u) | (((y >> 6) & 3u) << 4));
        sb = static_cast<int>(((w >> 8) & 15u) | (((y >> 14) & 3u) << 4));
        ma = static_cast<int>(((w >> 4) & 15u) | (((z >> 6) & 3u) << 4));
        mb = static_cast<int>(((w >> 12) & 15u) | (((z >> 14) & 3u) << 4));
    }
}

// IQ4_XS codebook (src/quant.cpp:468-471) as four words of int8 bytes.
__host__ __device__ constexpr uint32_t iq4nl_word(int a, int b, int c, int d) {
    return (static_cast<uint32_t>(a) & 255u) | ((static_cast<uint32_t>(b) & 255u) << 8) |
           ((static_cast<uint32_t>(c) & 255u) << 16) | ((static_cast<uint32_t>(d) & 255u) << 24);
}
constexpr uint32_t kIq4T0 = iq4nl_word(-127, -104, -83, -65);
constexpr uint32_t kIq4T1 = iq4nl_word(-49, -35, -22, -10);
constexpr uint32_t kIq4T2 = iq4nl_word(1, 13, 25, 38);
constexpr uint32_t kIq4T3 = iq4nl_word(53, 69, 89, 113);

// Four 4-bit codes (one per byte of idx, each 0..15) -> four int8 codebook
// values.  The codes are packed into a byte_perm selector; each half of the
// codebook is looked up with the low three bits and bit 3 picks the half.
__device__ __forceinline__ uint32_t iq4nl_lookup4(uint32_t idx) {
    const uint32_t x = idx | (idx >> 4);
    const uint32_t sel = __byte_perm(x, 0u, 0x0020u);  // nibble k = code of byte k
    const uint32_t s7 = sel & 0x7777u;
    const uint32_t lo = __byte_perm(kIq4T0, kIq4T1, s7);
    const uint32_t hi = __byte_perm(kIq4T2, kIq4T3, s7);
    return __byte_perm(lo, hi, ((sel >> 1) & 0x4444u) | 0x3210u);
}

// Activation words of half c (words 4c..4c+3 of groups 2p, 2p+1) for one lane.
template <int NL, bool XS>
__device__ __forceinline__ void kq_load_x(const uint8_t* xq, uint32_t c, uint32_t (&xl)[8 * NL]) {
#pragma unroll
    for (int j = 0; j < 2 * NL; ++j) {
        const uint4 v = xpack_load_quad<NL, XS>(xq + (2u * NL * c + j) * 256u);
        xl[4 * j + 0] = v.x;
        xl[4 * j + 1] = v.y;
        xl[4 * j + 2] = v.z;
        xl[4 * j + 3] = v.w;
    }
}

// Partial dot of super-block s, group pair p of both rows of a tile.
// b0/b1: the block in shared memory (row 0 / row 1), xq: the lane's quad 0 of
// this 4-block activation group, X: x group sums of groups 2p/2p+1, es: the
// activation unit of the block.  The integer dots are exact; the block scale
// and the lane sums are fp64, so over K = 17408 the result stays within a few
// 1e-5 of the FP64 dot (fp32 here would add ~8e-5 of rounding).
template <int T, int NL, bool XS>
__device__ __forceinline__ void kq_block_dot(const uint8_t* b0, const uint8_t* b1, const uint8_t* xq, uint32_t p,
                                             uint32_t c0, float2 X, float es, double& acc0, double& acc1) {
    if constexpr (T == 12 || T == 13) {
        constexpr uint32_t kQs = T == 13 ? 48u : 16u;
        const uint32_t rot_lo = (4u - 2u * p) & 31u, rot_hi = (3u - 2u * p) & 31u;
        int a0[NL], bb0[NL], a1[NL], bb1[NL];
#pragma unroll
        for (int k = 0; k < NL; ++k) a0[k] = bb0[k] = a1[k] = bb1[k] = 0;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const uint32_t c = half ? (c0 ^ 1u) : c0;
            const uint4 q0 = *reinterpret_cast<const uint4*>(b0 + kQs + 32u * p + 16u * c);
            const uint4 q1 = *reinterpret_cast<const uint4*>(b1 + kQs + 32u * p + 16u * c);
            uint4 h0 = make_uint4(0u, 0u, 0u, 0u), h1 = h0;
            if constexpr (T == 13) {
                h0 = *reinterpret_cast<const uint4*>(b0 + 16u + 16u * c);
                h1 = *reinterpret_cast<const uint4*>(b1 + 16u + 16u * c);
            }
            uint32_t xl[8 * NL];
            kq_load_x<NL, XS>(xq, c, xl);
            if constexpr (T == 13) {
                q5_chunk_dot<NL>(q0, h0, q1, h1, xl, rot_lo, rot_hi, a0, bb0, a1, bb1);
            } else {
                const uint32_t qw0[4] = {q0.x, q0.y, q0.z, q0.w}, qw1[4] = {q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t lo0 = qw0[i] & 0x0f0f0f0fu, hi0 = (qw0[i] >> 4) & 0x0f0f0f0fu;
                    const uint32_t lo1 = qw1[i] & 0x0f0f0f0fu, hi1 = (qw1[i] >> 4) & 0x0f0f0f0fu;
#pragma unroll
                    for (int k = 0; k < NL; ++k) {
                        a0[k] = dp4a(lo0, xl[(i * 2 + 0) * NL + k], a0[k]);
                        bb0[k] = dp4a(hi0, xl[(i * 2 + 1) * NL + k], bb0[k]);
                        a1[k] = dp4a(lo1, xl[(i * 2 + 0) * NL + k], a1[k]);
                        bb1[k] = dp4a(hi1, xl[(i * 2 + 1) * NL + k], bb1[k]);
                    }
                }
            }
        }
        const uint4 hd0 = *reinterpret_cast<const uint4*>(b0);
        const uint4 hd1 = *reinterpret_cast<const uint4*>(b1);
        int sa, sb, ma, mb;
        int t[NL];
        kq_scale_min_pair(hd0, p, sa, sb, ma, mb);
#pragma unroll
        for (int k = 0; k < NL; ++k) t[k] = sa * a0[k] + sb * bb0[k];
        float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&hd0.x));
        acc0 += __fma_rn(static_cast<double>(dm.x * es), limb_value<NL>(t),
                    -static_cast<double>(dm.y) * __fma_rn(static_cast<double>(ma), static_cast<double>(X.x), static_cast<double>(mb) * static_cast<double>(X.y)));
        kq_scale_min_pair(hd1, p, sa, sb, ma, mb);
#pragma unroll
        for (int k = 0; k < NL; ++k) t[k] = sa * a1[k] + sb * bb1[k];
        dm = __half22float2(*reinterpret_cast<const __half2*>(&hd1.x));
        acc1 += __fma_rn(static_cast<double>(dm.x * es), limb_value<NL>(t),
                    -static_cast<double>(dm.y) * __fma_rn(static_cast<double>(ma), static_cast<double>(X.x), static_cast<double>(mb) * static_cast<double>(X.y)));
    } else if constexpr (T == 14) {
        // Group g = 4n + t of the block: weights 32g + l (l < 32) take the
        // nibble t>>1 of ql[64n + 32(t&1) + l] and bits 2t..2t+1 of qh[32n + l];
        // scale sc[8n + 2t + l/16].  Lane p: n = p>>1, t = 2(p&1) and 2(p&1)+1.
        const uint32_t n = p >> 1, sh = 4u * (p & 1u);
        int t0[NL], t1[NL];
#pragma unroll
        for (int k = 0; k < NL; ++k) t0[k] = t1[k] = 0;
        const uint32_t sc0 = lds4_unaligned(b0 + 192u + 4u * p);
        const uint32_t sc1 = lds4_unaligned(b1 + 192u + 4u * p);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const uint32_t c = half ? (c0 ^ 1u) : c0;
            uint32_t la0[4], lb0[4], qh0[4], la1[4], lb1[4], qh1[4];
            lds16_unaligned(b0 + 64u * n + 16u * c, la0);
            lds16_unaligned(b0 + 64u * n + 32u + 16u * c, lb0);
            lds16_unaligned(b0 + 128u + 32u * n + 16u * c, qh0);
            lds16_unaligned(b1 + 64u * n + 16u * c, la1);
            lds16_unaligned(b1 + 64u * n + 32u + 16u * c, lb1);
            lds16_unaligned(b1 + 128u + 32u * n + 16u * c, qh1);
            uint32_t xl[8 * NL];
            kq_load_x<NL, XS>(xq, c, xl);
            int a0[NL], bb0[NL], a1[NL], bb1[NL];
#pragma unroll
            for (int k = 0; k < NL; ++k) a0[k] = bb0[k] = a1[k] = bb1[k] = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t wa0 = __vsub4(((la0[i] >> sh) & 0x0f0f0f0fu) | (((qh0[i] >> sh) & 0x03030303u) << 4),
                                             0x20202020u);
                const uint32_t wb0 = __vsub4(
                    ((lb0[i] >> sh) & 0x0f0f0f0fu) | (((qh0[i] >> (sh + 2u)) & 0x03030303u) << 4), 0x20202020u);
                const uint32_t wa1 = __vsub4(((la1[i] >> sh) & 0x0f0f0f0fu) | (((qh1[i] >> sh) & 0x03030303u) << 4),
                                             0x20202020u);
                const uint32_t wb1 = __vsub4(
                    ((lb1[i] >> sh) & 0x0f0f0f0fu) | (((qh1[i] >> (sh + 2u)) & 0x03030303u) << 4), 0x20202020u);
#pragma unroll
                for (int k = 0; k < NL; ++k) {
                    a0[k] = dp4a(wa0, xl[(i * 2 + 0) * NL + k], a0[k]);
                    bb0[k] = dp4a(wb0, xl[(i * 2 + 1) * NL + k], bb0[k]);
                    a1[k] = dp4a(wa1, xl[(i * 2 + 0) * NL + k], a1[k]);
                    bb1[k] = dp4a(wb1, xl[(i * 2 + 1) * NL + k], bb1[k]);
                }
            }
            // sc bytes at 4p: [group 2p half 0, half 1, group 2p+1 half 0, half 1]
            const int sa0 = static_cast<int8_t>((sc0 >> (8u * c)) & 255u);
            const int sb0 = static_cast<int8_t>((sc0 >> (8u * c + 16u)) & 255u);
            const int sa1 = static_cast<int8_t>((sc1 >> (8u * c)) & 255u);
            const int sb1 = static_cast<int8_t>((sc1 >> (8u * c + 16u)) & 255u);
#pragma unroll
            for (int k = 0; k < NL; ++k) {
                t0[k] += sa0 * a0[k] + sb0 * bb0[k];
                t1[k] += sa1 * a1[k] + sb1 * bb1[k];
            }
        }
        const float d0 = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(b0 + 208u)));
        const float d1 = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(b1 + 208u)));
        acc0 = __fma_rn(static_cast<double>(d0 * es), limb_value<NL>(t0), acc0);
        acc1 = __fma_rn(static_cast<double>(d1 * es), limb_value<NL>(t1), acc1);
        (void)X;
    } else {
        static_assert(T == 23, "unsupported K-quant type");
        // Group g: 16 bytes at 8 + 16g; byte j holds weight j (low nibble) and
        // weight 16 + j (high nibble); scale ls = 6 bits from scales_l/scales_h.
        const uint2 hd0 = *reinterpret_cast<const uint2*>(b0);
        const uint2 hd1 = *reinterpret_cast<const uint2*>(b1);
        uint32_t qa0[4], qb0[4], qa1[4], qb1[4];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint2 u0 = *reinterpret_cast<const uint2*>(b0 + 8u + 32u * p + 8u * k);
            const uint2 v0 = *reinterpret_cast<const uint2*>(b0 + 24u + 32u * p + 8u * k);
            const uint2 u1 = *reinterpret_cast<const uint2*>(b1 + 8u + 32u * p + 8u * k);
            const uint2 v1 = *reinterpret_cast<const uint2*>(b1 + 24u + 32u * p + 8u * k);
            qa0[2 * k] = u0.x; qa0[2 * k + 1] = u0.y;
            qb0[2 * k] = v0.x; qb0[2 * k + 1] = v0.y;
            qa1[2 * k] = u1.x; qa1[2 * k + 1] = u1.y;
            qb1[2 * k] = v1.x; qb1[2 * k + 1] = v1.y;
        }
        int t0[NL], t1[NL];
#pragma unroll
        for (int k = 0; k < NL; ++k) t0[k] = t1[k] = 0;
        auto ls = [p](uint2 hd, int& la, int& lb) {
            const uint32_t sh = hd.x >> 16, sl = (hd.y >> (8u * p)) & 255u;
            la = static_cast<int>((sl & 15u) | (((sh >> (4u * p)) & 3u) << 4)) - 32;
            lb = static_cast<int>((sl >> 4) | (((sh >> (4u * p + 2u)) & 3u) << 4)) - 32;
        };
        int la0, lb0, la1, lb1;
        ls(hd0, la0, lb0);
        ls(hd1, la1, lb1);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const uint32_t c = half ? (c0 ^ 1u) : c0;  // words 4c..4c+3 = nibble c of the 4 qs words
            uint32_t xl[8 * NL];
            kq_load_x<NL, XS>(xq, c, xl);
            int a0[NL], bb0[NL], a1[NL], bb1[NL];
#pragma unroll
            for (int k = 0; k < NL; ++k) a0[k] = bb0[k] = a1[k] = bb1[k] = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t wa0 = iq4nl_lookup4((qa0[i] >> (4u * c)) & 0x0f0f0f0fu);
                const uint32_t wb0 = iq4nl_lookup4((qb0[i] >> (4u * c)) & 0x0f0f0f0fu);
                const uint32_t wa1 = iq4nl_lookup4((qa1[i] >> (4u * c)) & 0x0f0f0f0fu);
                const uint32_t wb1 = iq4nl_lookup4((qb1[i] >> (4u * c)) & 0x0f0f0f0fu);
#pragma unroll
                for (int k = 0; k < NL; ++k) {
                    a0[k] = dp4a(wa0, xl[(i * 2 + 0) * NL + k], a0[k]);
                    bb0[k] = dp4a(wb0, xl[(i * 2 + 1) * NL + k], bb0[k]);
                    a1[k] = dp4a(wa1, xl[(i * 2 + 0) * NL + k], a1[k]);
                    bb1[k] = dp4a(wb1, xl[(i * 2 + 1) * NL + k], bb1[k]);
                }
            }
#pragma unroll
            for (int k = 0; k < NL; ++k) {
                t0[k] += la0 * a0[k] + lb0 * bb0[k];
                t1[k] += la1 * a1[k] + lb1 * bb1[k];
            }
        }
        const float d0 = __half2float(__ushort_as_half(static_cast<unsigned short>(hd0.x & 0xffffu)));
        const float d1 = __half2float(__ushort_as_half(static_cast<unsigned short>(hd1.x & 0xffffu)));
        acc0 = __fma_rn(static_cast<double>(d0 * es), limb_value<NL>(t0), acc0);
        acc1 = __fma_rn(static_cast<double>(d1 * es), limb_value<NL>(t1), acc1);
        (void)X;
    }
}

// XM: 0 = x-pack read through L1, 1 = x-pack copied into shared memory,
// 2 = f32 x packed into shared memory by this CTA (xlimbs = the f32 vector),
// 3 = the same after RMSNorm (xgsum = the norm weight, eps its epsilon).
template <int T, int NL, int XM, int WARPS = KqType<T>::kWarps, int MINB = 2>
__global__ void __launch_bounds__(WARPS * 32, MINB)
    gemv_kq_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xlimbs,
                   const float* __restrict__ xgsum, const float* __restrict__ xscale, float* y,
                   const float* res, uint32_t rows, uint32_t nb, float eps) {
    using Ty = KqType<T>;
    constexpr uint32_t W = WARPS, C = 2u * W, S = kq_seg_stride<T>(), SLOT = 2u * S, D = kKqDepth;
    constexpr size_t RING = kq_ring_bytes<T, W>();
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + RING);
    uint64_t* xbar = bars + C * D;
    PairBoundary<C>* bnd = reinterpret_cast<PairBoundary<C>*>(xbar + 1);
    uint8_t* xs = reinterpret_cast<uint8_t*>(bnd + 1);
    xs += (128u - (reinterpret_cast<uintptr_t>(xs) & 127u)) & 127u;

    if (threadIdx.x == 0) pdl_launch_dependents();

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t h = lane >> 4, cons = 2u * warp + h, l16 = lane & 15u;
    const uint32_t hmask = h ? 0xffff0000u : 0x0000ffffu;
    const uint32_t npairs = (rows + 1u) >> 1;
    const uint32_t nkc = (nb + 3u) >> 2;
    const size_t rowbytes = static_cast<size_t>(nb) * Ty::kBlock;
    const uint32_t p0 = static_cast<uint32_t>(static_cast<uint64_t>(npairs) * blockIdx.x / gridDim.x);
    const uint32_t p1 = static_cast<uint32_t>(static_cast<uint64_t>(npairs) * (blockIdx.x + 1) / gridDim.x);
    const uint32_t Tn = (p1 - p0) * nkc;
    const uint32_t base = Tn / C, rem = Tn % C;
    const uint32_t len = base + (cons < rem ? 1u : 0u);
    const uint32_t chunk0 = cons * base + min(cons, rem);
    uint8_t* ring = smem + static_cast<size_t>(cons) * D * SLOT;
    uint64_t* full = bars + cons * D;

    // Source span of segment r (0/1) of tile i of this consumer.
    auto seg_src = [&](uint32_t i, uint32_t r, uint32_t& nblk) -> const uint8_t* {
        const uint32_t g = chunk0 + i, pr = p0 + g / nkc, kc = g - (g / nkc) * nkc;
        nblk = min(4u, nb - 4u * kc);
        return w + static_cast<size_t>(2u * pr + r) * rowbytes + static_cast<size_t>(kc) * 4u * Ty::kBlock;
    };
    auto issue = [&](uint32_t i, uint32_t slot) {
        const uint32_t g = chunk0 + i, pr = p0 + g / nkc;
        const bool two = 2u * pr + 1u < rows;
        uint32_t nblk;
        const uint8_t* s0 = seg_src(i, 0, nblk);
        const uintptr_t a0 = reinterpret_cast<uintptr_t>(s0) & ~uintptr_t(15);
        const uint32_t n0 = (static_cast<uint32_t>(reinterpret_cast<uintptr_t>(s0) & 15u) + nblk * Ty::kBlock + 15u) & ~15u;
        uint32_t n1 = 0;
        uintptr_t a1 = 0;
        if (two) {
            const uint8_t* s1 = s0 + rowbytes;
            a1 = reinterpret_cast<uintptr_t>(s1) & ~uintptr_t(15);
            n1 = (static_cast<uint32_t>(reinterpret_cast<uintptr_t>(s1) & 15u) + nblk * Ty::kBlock + 15u) & ~15u;
        }
        uint8_t* dst = ring + slot * SLOT;
        mbar_arrive_expect_tx(&full[slot], n0 + n1);
        tma_load_1d(dst, reinterpret_cast<const void*>(a0), n0, &full[slot]);
        if (two) tma_load_1d(dst + S, reinterpret_cast<const void*>(a1), n1, &full[slot]);
    };

    if (l16 == 0) {
        // L2 prefetch of every row segment of this consumer's run.
        uint32_t i = 0;
        while (i < len) {
            const uint32_t g = chunk0 + i, pr = p0 + g / nkc, kc = g - (g / nkc) * nkc;
            const uint32_t run = min(nkc - kc, len - i);  // tiles of this row pair in the run
            for (uint32_t r = 0; r < 2u && 2u * pr + r < rows; ++r) {
                const uint8_t* s = w + static_cast<size_t>(2u * pr + r) * rowbytes + static_cast<size_t>(kc) * 4u * Ty::kBlock;
                const size_t bytes = min(static_cast<size_t>(run) * 4u * Ty::kBlock,
                                         rowbytes - static_cast<size_t>(kc) * 4u * Ty::kBlock);
                const uintptr_t a = reinterpret_cast<uintptr_t>(s) & ~uintptr_t(15);
                const size_t span = ((reinterpret_cast<uintptr_t>(s) & 15u) + bytes + 15u) & ~size_t(15);
                for (size_t off = 0; off < span; off += kL2PrefetchPiece) {
                    const size_t left = span - off;
                    prefetch_l2(reinterpret_cast<const void*>(a + off),
                                static_cast<uint32_t>(left < kL2PrefetchPiece ? left : kL2PrefetchPiece));
                }
            }
            i += run;
        }
        for (uint32_t k = 0; k < D; ++k) mbar_init(&full[k], 1);
        if (XM == 1 && cons == 0) mbar_init(xbar, 1);
        fence_mbar_init();
        for (uint32_t k = 0; k < D && k < len; ++k) issue(k, k);
    }
    if (threadIdx.x < 2u * C) bnd->pair[threadIdx.x] = -1;
    __syncthreads();

    pdl_wait();
    constexpr bool XS = XM != 0;
    const uint32_t lbytes = static_cast<uint32_t>(xpack_row_limb_bytes(NL, nb));
    const uint8_t* xl_base;
    const float2* xg2;
    const float* xsc;
    if constexpr (XM >= 2) {
        static_assert(NL == 3, "f32 activations pack into three limbs");
        const float* xf = reinterpret_cast<const float*>(xlimbs);
        float inv = 1.0f;
        if constexpr (XM == 3) {
            __shared__ double blk[kNormMaxBlocks];
            __shared__ float inv_s;
            inv = row_inv_rms(xf, nb, eps, blk, &inv_s, warp, lane, W);
        }
        pack_x_f32_smem(xf, nb, xs, reinterpret_cast<float*>(xs + lbytes), reinterpret_cast<float*>(xs + lbytes + nb * 32u),
                      warp, lane, W, XM == 3 ? xgsum : nullptr, inv);
        xl_base = xs;
        xg2 = reinterpret_cast<const float2*>(xs + lbytes);
        xsc = reinterpret_cast<const float*>(xs + lbytes + nb * 32u);
    } else if constexpr (XM == 1) {
        if (threadIdx.x == 0) {
            const uint32_t scb = xpack_nb4(nb) * 4u;
            mbar_arrive_expect_tx(xbar, lbytes + nb * 32u + scb);
            tma_load_1d(xs, xlimbs, lbytes, xbar);
            tma_load_1d(xs + lbytes, xgsum, nb * 32u, xbar);
            tma_load_1d(xs + lbytes + nb * 32u, xscale, scb, xbar);
        }
        xl_base = xs;
        xg2 = reinterpret_cast<const float2*>(xs + lbytes);
        xsc = reinterpret_cast<const float*>(xs + lbytes + nb * 32u);
    } else {
        for (uint32_t off = threadIdx.x * 128u; off < lbytes; off += W * 32u * 128u) prefetch_l1(xlimbs + off);
        xl_base = xlimbs;
        xg2 = reinterpret_cast<const float2*>(xgsum);
        xsc = xscale;
    }
    const uint32_t s = (lane >> 2) & 3u, p = lane & 3u;
    const uint32_t c0 = s & 1u;
    const uint8_t* xlane = xl_base + (s * 4u + p) * 16u;
    bool ok = true;
    if constexpr (XM == 1) {
        if (!mbar_wait_spin(xbar, 0, kFaultFullWait)) ok = false;
    }
    if constexpr (XM >= 2) __syncthreads();

    double acc0 = 0.0, acc1 = 0.0;
    uint32_t issued = min(len, D), waited = 0;
    uint32_t pair = chunk0 / nkc, kc = chunk0 - pair * nkc;
    uint32_t kc_first = kc, nflush = 0;
    bool started = false;

    auto flush = [&](bool whole) {
        double v0 = acc0, v1 = acc1;
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) {
            v0 += __shfl_xor_sync(hmask, v0, o);
            v1 += __shfl_xor_sync(hmask, v1, o);
        }
        if (l16 == 0) {
            const uint32_t row = 2u * (p0 + pair);
            if (whole) {
                if (ok && row < rows) y[row] = gemv_out(v0, res, row);
                if (ok && row + 1u < rows) y[row + 1u] = gemv_out(v1, res, row + 1u);
            } else {
                const uint32_t e = cons * 2u + (nflush == 0 ? 0u : 1u);
                bnd->v[e][0] = v0;
                bnd->v[e][1] = v1;
                bnd->pair[e] = static_cast<int>(pair);
            }
        }
        ++nflush;
        acc0 = 0.0;
        acc1 = 0.0;
    };

    const uint32_t len_w = base + (2u * warp < rem ? 1u : 0u);
    for (uint32_t i = 0; i < len_w; ++i) {
        if (i < len) {
            const uint32_t slot = i % D;
            const bool landed = ok && mbar_wait_spin(&full[slot], (i / D) & 1u, kFaultFullWait);
            if (!landed) ok = false;
            started = true;
            const uint32_t nblk = min(4u, nb - 4u * kc);
            if (ok && s < nblk) {
                const uint32_t bcol = kc * 4u + s;
                uint32_t dummy;
                const uint8_t* s0 = seg_src(i, 0, dummy);
                const uint8_t* tb = ring + slot * SLOT;
                const uint32_t d0 = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(s0) & 15u);
                const uint32_t d1 = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(s0 + rowbytes) & 15u);
                const uint8_t* blk0 = tb + d0 + s * Ty::kBlock;
                const uint8_t* blk1 = 2u * (p0 + pair) + 1u < rows ? tb + S + d1 + s * Ty::kBlock : blk0;
                const uint8_t* xq = xlane + static_cast<size_t>(kc) * (4u * NL) * 256u;
                float2 X = make_float2(0.0f, 0.0f);
                if constexpr (T == 12 || T == 13) X = XS ? xg2[bcol * 4u + p] : __ldcg(xg2 + bcol * 4u + p);
                const float es = XS ? xsc[bcol] : __ldcg(xsc + bcol);
                kq_block_dot<T, NL, XS>(blk0, blk1, xq, p, c0, X, es, acc0, acc1);
            }
            __syncwarp(hmask);
            if (ok && l16 == 0 && i + D < len) {
                fence_proxy_async_smem();
                issue(i + D, slot);
                issued = i + D + 1u;
            }
            if (landed) waited = i + 1u;
            if (++kc == nkc) {
                flush(kc_first == 0);
                kc = 0;
                kc_first = 0;
                ++pair;
                started = false;
            }
        }
    }
    if (started) flush(false);
    if (!ok && l16 == 0) {
        for (uint32_t i = waited; i < issued; ++i)
            if (!mbar_wait(&full[i % D], (i / D) & 1u, kFaultDrain)) break;
    }

    __syncthreads();
    if (threadIdx.x < 2u * C && ok) {
        const uint32_t e = threadIdx.x;
        const int pr = bnd->pair[e];
        if (pr >= 0) {
            int prev = e >= 1 ? bnd->pair[e - 1] : -1;
            if (prev == -1 && e >= 2) prev = bnd->pair[e - 2];
            if (prev != pr) {
                double v0 = bnd->v[e][0], v1 = bnd->v[e][1];
                for (uint32_t q = e + 1u; q < 2u * C; ++q) {
                    const int pq = bnd->pair[q];
                    if (pq == -1) continue;
                    if (pq != pr) break;
                    v0 += bnd->v[q][0];
                    v1 += bnd->v[q][1];
                }
                const uint32_t row = 2u * (p0 + static_cast<uint32_t>(pr));
                if (row < rows) y[row] = gemv_out(v0, res, row);
                if (row + 1u < rows) y[row + 1u] = gemv_out(v1, res, row + 1u);
            }
        }
    }
}

}  // namespace q38
