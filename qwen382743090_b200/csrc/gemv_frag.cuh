// gemv_frag.cuh -- batch-1 K-quant GEMV on the tensor cores over the B200
// fragment-ordered tile layout (Q38PACK layout 2), for Q5_K and Q4_K.  Same
// mathematics as the reference's q38_q5k_sm86_soa_gemv_vec
// (src/driver.cpp:3887-4138) and q38_q4k_gemv_f32 (:1857):
//   y[r] = sum_b d_b * sum_g sc_g * <q_g, x_g> - dmin_b * sum_g m_g * sum(x_g).
//
// Layout 2.  A tile is 8 weight rows x 2 super-blocks, stored so that every
// lane of a warp reads its own mma fragments with 128-bit, conflict-free
// shared-memory loads (lane = 4*g + t: row g, position chunk t):
//   QS [2048 B] [s][c][lane][16]: for row g of block s and group pairs 2c and
//               2c+1, the bytes of positions 8t..8t+3 (word Q0) and 8t+4..8t+7
//               (word Q1) of each pair.  A byte holds the even group's weight
//               in its low nibble (Q5_K: the low 4 bits) and the odd group's in
//               its high nibble (Q5_K: the TOP 4 bits, w_odd >> 1).
//   QH [ 512 B] (Q5_K only) [lane][16]: one byte per position (block 0 then
//               block 1), bit 2p+1 = fifth bit of the even group of pair p and
//               bit 2p = lowest bit of the odd group.
//   SC [ 256 B] [s][g][16]: the eight 6-bit scales, then the eight 6-bit mins.
//   DM [  64 B] [s][g][4]: d, dmin (fp16).
// Q5_K tiles are 2880 bytes, Q4_K tiles 2368 bytes (no QH).  Tiles are stored
// row-octet-major, tile (o, kc) at (o * nb/2 + kc) * tile_bytes; rows pad to a
// multiple of 8 with zero rows (d = dmin = 0) and nb must be even.  The bytes
// are a permutation of each block's bits (plus the expanded 6-bit scales), so
// the dequantised weights are exactly GGML's.
//
// Kernel.  One mma.sync.m16n8k32 (u8 x s8 -> s32) per (8 rows, group pair):
// A rows 0..7 are the even group of rows 0..7 and A rows 8..15 the odd group
// scaled by 8 (Q5_K) or 16 (Q4_K), decoded in registers with two to three
// logic operations per 4 weights:
//   Q5_K: R = rotl(qh, 3 - 2p); even = (q & 0x0f..) | (R & 0x10..);
//         odd8 = (q & 0xf0..) | (R & 0x08..)  = 8 * w_odd
//   Q4_K: even = q & 0x0f..;  odd16 = q & 0xf0..  = 16 * w_odd
// B columns 2l and 2l+1 are activation limb l of the even and of the odd group
// (x-fragments below).  The mma k index maps to group positions as
// k = 4t + j -> 8t + j and k = 16 + 4t + j -> 8t + 4 + j for both operands.
// Lane (g, t) keeps C[g][2t] (even group x limb t) and C[g+8][2t+1] (odd group
// x limb t), multiplies them by the 6-bit group scales in int32 (exact) and
// sums the 8 groups of a super-block; the block scale d * unit * 256^t / 8 and
// its share (pair t) of the dmin * m * sum(x) term are applied in fp64 / fp32,
// and the four lanes of a row are summed at the end of the row octet.
//
// Pipeline: each warp owns a contiguous run of its CTA's tiles and a private
// ring of DEPTH 1-D bulk-copy slots (no multicast).  The ring is filled before
// the grid dependency resolves (PDL); a landed tile is copied to registers and
// its slot refilled at once, so the copies stay in flight while the warp
// computes.  Row octets split between warps are summed afterwards in warp
// order (deterministic).
#pragma once

#include "gemv_common.cuh"
#include "gemv_kq.cuh"  // the IQ4_XS codebook words

namespace q38 {

constexpr uint32_t kF8Rows = 8;
constexpr uint32_t kF8Blocks = 2;
constexpr uint32_t kF8QsBytes = 2048;
constexpr uint32_t kF8QhBytes = 512;
constexpr uint32_t kF8PackPerWarp = 4;  // XM 2: super-blocks each warp packs (nb <= 4 * warps)

template <uint32_t T>
struct FragTile;
template <>
struct FragTile<13> {  // Q5_K
    static constexpr uint32_t kQh = kF8QsBytes, kSc = kF8QsBytes + kF8QhBytes, kDm = kSc + 256u, kBytes = kDm + 64u;
    static constexpr uint32_t kOddShift = 0;  // odd group counted x8
};
template <>
struct FragTile<12> {  // Q4_K
    static constexpr uint32_t kQh = 0, kSc = kF8QsBytes, kDm = kSc + 256u, kBytes = kDm + 64u;
    static constexpr uint32_t kOddShift = 1;  // odd group counted x16
};
// Q6_K: LO [s][lane][32 B] | HI [s][lane][16 B] | SC [s][row][16] int8 | D [s][row] f16.
// Lane (g, t) holds, for each 16-weight group pair j (groups 2j, 2j+1) of row g,
// positions 4t..4t+3: LO word j byte k = low nibble of the even group's code at
// position 4t+k | the odd group's << 4; HI words E_a, E_b, O_a, O_b (even groups
// of pairs 0-3 / 4-7, odd groups of pairs 0-3 / 4-7): byte k, bits 2(j&3)..+1 =
// the code's top two bits.  The same 210 bytes per row and super-block as GGUF.
template <>
struct FragTile<14> {
    static constexpr uint32_t kLo = 0, kHi = 2048u, kSc = 3072u, kD = 3328u, kBytes = 3360u;
};
// IQ4_XS: QS [s][c][lane][16] | SC [s][row][8] int8 (the group scale ls - 32) |
// D [s][row] f16.  Lane (g, t)'s 16 bytes hold, for group pairs 2c and 2c+1
// (32-weight groups 2p, 2p+1), two words per pair: positions 8t..8t+3 and
// 8t+4..8t+7, each with the even group's four 4-bit codes in its low 16 bits
// and the odd group's in its high 16 bits (ready-made byte_perm selectors).
// A code c is stored rotated, iq4_tile_code(c) = (c & 1) << 3 | c >> 1, so
// that selector slot i holds codebook entries 2i and 2i + 1, which share a
// sign (iq4_codes8).
template <>
struct FragTile<23> {
    static constexpr uint32_t kSc = kF8QsBytes, kD = kSc + 128u, kBytes = kD + 32u;
};
static_assert(FragTile<13>::kBytes == 2880 && FragTile<12>::kBytes == 2368 && FragTile<14>::kBytes == 3360 &&
                  FragTile<23>::kBytes == 2208,
              "tile sizes");

__host__ __device__ constexpr uint32_t frag_tile_bytes(uint32_t type) {
    return type == 13u ? FragTile<13>::kBytes
           : type == 12u ? FragTile<12>::kBytes
           : type == 14u ? FragTile<14>::kBytes
           : type == 23u ? FragTile<23>::kBytes
                         : 0u;
}
// Bytes of a rows x cols matrix in layout 2 (0 when the shape or type does not fit).
__host__ __device__ constexpr size_t frag_matrix_bytes(uint32_t type, uint32_t rows, uint32_t cols) {
    return (frag_tile_bytes(type) == 0u || rows == 0u || cols == 0u || cols % 512u)
               ? 0u
               : static_cast<size_t>((rows + kF8Rows - 1u) / kF8Rows) * (cols / 512u) * frag_tile_bytes(type);
}

// ---- x-fragments ---------------------------------------------------------------
// One activation row: per super-block 1088 bytes = the limb fragments
// [c][lane][16] (1 KiB; lane (g, t) holds for pairs 2c, 2c+1 the 8 bytes of
// limb g/2 of group 2p + (g & 1) at positions 8t..8t+7), then for each limb t a
// 16-byte record {double unit * 256^t / 8; float sum(x) of group 2t; float
// sum(x) of group 2t+1}.  The limbs are those of the x-pack with NL = 4
// (balanced bytes of round(x / unit), |x / unit| < 2^30).
constexpr uint32_t kXfBlockBytes = 1088;
constexpr uint32_t kXfMetaOff = 1024;
__host__ __device__ constexpr size_t xfrag1_bytes(uint32_t nb) { return static_cast<size_t>(nb) * kXfBlockBytes; }

// Q6 x-fragments (the activation side of the Q6_K tiles, 16-weight groups):
// per super-block 1056 bytes = [j/4][lane][j%4] words (1 KiB; lane (g, t) holds
// for group pair j the 4 bytes of limb g/2 of group 2j + (g & 1) at positions
// 4t..4t+3), then for each limb t the double unit * 256^t / 4.  Same limbs as
// the x-fragments.
constexpr uint32_t kX6BlockBytes = 1056;
constexpr uint32_t kX6MetaOff = 1024;
__host__ __device__ constexpr uint32_t xf_block_bytes(uint32_t type) {
    return type == 14u ? kX6BlockBytes : kXfBlockBytes;
}
__host__ __device__ constexpr size_t xfrag_bytes_t(uint32_t type, uint32_t nb) {
    return static_cast<size_t>(nb) * xf_block_bytes(type);
}

// Producer lane (G, t) holds group G at positions 8t..8t+7; limb k of it is B
// column 2k + (G & 1) of pair G/2, i.e. consumer lane 4 * (2k + (G & 1)) + t.
__device__ __forceinline__ void xfrag_store_limbs(uint8_t* blockp, uint32_t lane, const uint32_t (&lw)[2][4]) {
    const uint32_t G = lane >> 2, t = lane & 3u, p = G >> 1;
    uint8_t* base = blockp + (p >> 1) * 512u + (p & 1u) * 8u;
#pragma unroll
    for (uint32_t k = 0; k < 4u; ++k)
        *reinterpret_cast<uint2*>(base + (4u * (2u * k + (G & 1u)) + t) * 16u) = make_uint2(lw[0][k], lw[1][k]);
}
// The block's records: lane (G, 0) stores its group's sum, lanes 0..3 the
// scaled units.
__device__ __forceinline__ void xfrag_store_meta(uint8_t* blockp, uint32_t lane, double gsum_group, float unit) {
    const uint32_t G = lane >> 2, t = lane & 3u;
    uint8_t* meta = blockp + kXfMetaOff;
    if (t == 0) reinterpret_cast<float*>(meta + (G >> 1) * 16u + 8u)[G & 1u] = static_cast<float>(gsum_group);
    if (lane < 4u)
        *reinterpret_cast<double*>(meta + lane * 16u) =
            static_cast<double>(unit) * static_cast<double>(1u << (8u * lane)) * 0.125;
}

// Quantise one super-block of f32 activations (warp; lane holds elements
// 8*lane..8*lane+7) exactly like pack_block_warp<4>: the lane's limb words
// lw[h][k] (limb k of elements 8*lane+4h .. +3), the block's unit in *unit, and
// the sum of the lane's eight quantised values (returned).
__device__ __forceinline__ double quantize_block_warp4(const float (&v)[8], uint32_t (&lw)[2][4], float* unit_out) {
    constexpr int NL = 4;
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
    *unit_out = unit;
    return xpack_limbs8<NL>(xi, lw);
}

// Quantise one super-block of f32 activations (warp; lane holds elements
// 8*lane..8*lane+7) exactly like pack_block_warp<4> and write x-fragments.
__device__ __forceinline__ void pack_block_warp_frag(const float (&v)[8], uint32_t lane, uint8_t* blockp) {
    constexpr int NL = 4;
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
    xfrag_store_limbs(blockp, lane, lw);
    gs += __shfl_xor_sync(0xffffffffu, gs, 1);
    gs += __shfl_xor_sync(0xffffffffu, gs, 2);
    xfrag_store_meta(blockp, lane, gs * static_cast<double>(unit), unit);
}

// Producer lane L's limb words (elements 8L..8L+7: lw[h][k] = limb k of
// elements 8L+4h..8L+4h+3) and the block's units, in the Q6 x-fragment layout.
__device__ __forceinline__ void x6_store(uint8_t* blockp, uint32_t lane, const uint32_t (&lw)[2][4], float unit) {
    const uint32_t G = lane >> 1, j = G >> 1, par = G & 1u;
#pragma unroll
    for (uint32_t k = 0; k < 4u; ++k)
#pragma unroll
        for (uint32_t h = 0; h < 2u; ++h) {
            const uint32_t t = 2u * (lane & 1u) + h, g = 2u * k + par;
            *reinterpret_cast<uint32_t*>(blockp + (j >> 2) * 512u + (4u * g + t) * 16u + (j & 3u) * 4u) = lw[h][k];
        }
    if (lane < 4u)
        *reinterpret_cast<double*>(blockp + kX6MetaOff + lane * 8u) =
            static_cast<double>(unit) * static_cast<double>(1u << (8u * lane)) * 0.25;
}

// The same quantisation as pack_block_warp_frag, written as Q6 x-fragments:
// producer lane L holds elements 8L..8L+7 = positions 8(L&1)..+7 of 16-group
// L/2, so its half h (positions 4t..4t+3, t = 2(L&1) + h) of limb k goes to
// consumer lane (2k + (L/2 & 1), t) of group pair L/4.
__device__ __forceinline__ void pack_block_warp_x6(const float (&v)[8], uint32_t lane, uint8_t* blockp) {
    constexpr int NL = 4;
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
    (void)xpack_limbs8<NL>(xi, lw);
    x6_store(blockp, lane, lw, unit);
}

// Q8_K activations (f32 d | int8 qs[256] | int16 bsums[16], 292 B) -> Q6
// x-fragments: limb 0 is the Q8_K byte, limbs 1..3 are zero, unit = d.
__global__ void __launch_bounds__(256) x6frag_q8k_kernel(const uint8_t* __restrict__ q8, uint32_t nb, uint32_t B,
                                                         uint8_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t w = blockIdx.x * 8u + (threadIdx.x >> 5);
    if (w >= nb * B) return;  // warp-uniform
    const uint8_t* src = q8 + static_cast<size_t>(w) * 292u;
    const float d = *reinterpret_cast<const float*>(src);
    uint32_t lw[2][4] = {{0u, 0u, 0u, 0u}, {0u, 0u, 0u, 0u}};
#pragma unroll
    for (int k = 0; k < 8; ++k) lw[k >> 2][0] |= static_cast<uint32_t>(src[4u + lane * 8u + k]) << (8u * (k & 3));
    const uint32_t blk = w % nb, b = w / nb;
    x6_store(out + static_cast<size_t>(b) * xfrag_bytes_t(14u, nb) + blk * kX6BlockBytes, lane, lw, d);
}

// f32 activations [B][K] -> Q6 x-fragments [B][xfrag_bytes_t(14, K / 256)].
__global__ void __launch_bounds__(256) x6frag_f32_kernel(const float* __restrict__ x, uint32_t K, uint32_t B,
                                                         uint8_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t nb = K / 256u, lane = threadIdx.x & 31u;
    const uint32_t w = blockIdx.x * 8u + (threadIdx.x >> 5);
    if (w >= nb * B) return;  // warp-uniform
    const uint32_t blk = w % nb, b = w / nb;
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(b) * K + blk * 256u + lane * 8u);
    const float4 v0 = xr[0], v1 = xr[1];
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    pack_block_warp_x6(v, lane, out + static_cast<size_t>(b) * xfrag_bytes_t(14u, nb) + blk * kX6BlockBytes);
}

// f32 activations [B][K] -> x-fragments [B][xfrag1_bytes(K / 256)], one warp
// per (super-block, row).
__global__ void __launch_bounds__(256) xfrag1_f32_kernel(const float* __restrict__ x, uint32_t K, uint32_t B,
                                                         uint8_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t nb = K / 256u, lane = threadIdx.x & 31u;
    const uint32_t w = blockIdx.x * 8u + (threadIdx.x >> 5);
    if (w >= nb * B) return;  // warp-uniform
    const uint32_t blk = w % nb, b = w / nb;
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(b) * K + blk * 256u + lane * 8u);
    const float4 v0 = xr[0], v1 = xr[1];
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    pack_block_warp_frag(v, lane, out + static_cast<size_t>(b) * xfrag1_bytes(nb) + blk * kXfBlockBytes);
}

// f32 activations [K] in page-locked host memory -> x-fragments (Q6 x-fragments
// for T = 14) in device memory, one warp per super-block: the host-buffer GEMV
// packs while it reads x over the bus, so the GEMV that follows runs on
// pre-packed x.  x is read with ld.global.cv: the caller rewrites it between
// calls, and no copy of it may be served from a cache.  EARLY: x was written
// by the host before this launch, not by the kernels it follows (the caller
// promises it), so it is read and quantised before the dependency wait and
// only the stores into `out`, which the previous GEMV may still be reading,
// wait for it; otherwise everything waits (x may be an earlier GEMV's y).
template <uint32_t T, bool EARLY>
__global__ void __launch_bounds__(256) xfrag_host_f32_kernel(const float* x, uint32_t K, uint8_t* __restrict__ out) {
    pdl_launch_dependents();
    if constexpr (!EARLY) pdl_wait();
    const uint32_t nb = K / 256u, lane = threadIdx.x & 31u;
    const uint32_t blk = blockIdx.x * 8u + (threadIdx.x >> 5);
    if (blk >= nb) return;  // warp-uniform
    const float4* xr = reinterpret_cast<const float4*>(x + blk * 256u + lane * 8u);
    const float4 v0 = __ldcv(xr), v1 = __ldcv(xr + 1);
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    uint32_t lw[2][4];
    float unit;
    double gs = quantize_block_warp4(v, lw, &unit);  // the arithmetic of pack_block_warp_frag / _x6
    if constexpr (EARLY) pdl_wait();
    if constexpr (T == 14u) {
        x6_store(out + blk * kX6BlockBytes, lane, lw, unit);
    } else {
        uint8_t* blockp = out + blk * kXfBlockBytes;
        xfrag_store_limbs(blockp, lane, lw);
        gs += __shfl_xor_sync(0xffffffffu, gs, 1);
        gs += __shfl_xor_sync(0xffffffffu, gs, 2);
        xfrag_store_meta(blockp, lane, gs * static_cast<double>(unit), unit);
    }
}

// Q8_K activations (blocks of f32 d | int8 qs[256] | int16 bsums[16], 292 B)
// -> x-fragments: limb 0 is the Q8_K byte, limbs 1..3 are zero, unit = d and
// the group sums are d * (sum of the group's bytes), as in xpack_q8k_kernel.
__global__ void __launch_bounds__(256) xfrag1_q8k_kernel(const uint8_t* __restrict__ q8, uint32_t nb, uint32_t B,
                                                         uint8_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t w = blockIdx.x * 8u + (threadIdx.x >> 5);
    if (w >= nb * B) return;  // warp-uniform
    const uint8_t* src = q8 + static_cast<size_t>(w) * 292u;  // the blocks of row b follow each other
    const float d = *reinterpret_cast<const float*>(src);
    uint32_t lw[2][4] = {{0u, 0u, 0u, 0u}, {0u, 0u, 0u, 0u}};
    int s = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t byte = src[4u + lane * 8u + k];
        lw[k >> 2][0] |= byte << (8u * (k & 3));
        s += static_cast<int8_t>(byte);
    }
    const uint32_t blk = w % nb, b = w / nb;
    uint8_t* blockp = out + static_cast<size_t>(b) * xfrag1_bytes(nb) + blk * kXfBlockBytes;
    xfrag_store_limbs(blockp, lane, lw);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    xfrag_store_meta(blockp, lane, static_cast<double>(d) * static_cast<double>(s), d);
}

// ---- GGUF blocks -> layout 2 on the device ----------------------------------------
// One thread per (row, super-block); tiles must be zeroed first when rows is
// not a multiple of 8.  Q5_K blocks: d, dmin | scales[12] | qh[32] | qs[128]
// (176 B); Q4_K: d, dmin | scales[12] | qs[128] (144 B).  The 6-bit scales and
// mins follow get_scale_min_k4 (src/quant.cpp:89-97).
template <uint32_t T>
__global__ void repack_frag_kernel(const uint8_t* __restrict__ blocks, uint8_t* __restrict__ tiles, uint32_t rows,
                                   uint32_t nb) {
    using F = FragTile<T>;
    constexpr uint32_t kBlk = T == 13u ? 176u : 144u, kQsOff = T == 13u ? 48u : 16u;
    const uint64_t idx = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<uint64_t>(rows) * nb) return;
    const uint32_t r = static_cast<uint32_t>(idx / nb), b = static_cast<uint32_t>(idx % nb);
    const uint32_t o = r >> 3, g = r & 7u, kc = b >> 1, s = b & 1u;
    const uint8_t* src = blocks + idx * kBlk;
    uint8_t* tile = tiles + (static_cast<uint64_t>(o) * (nb / 2u) + kc) * F::kBytes;
    const uint8_t* qs = src + kQsOff;
    for (uint32_t p = 0; p < 4u; ++p) {
        for (uint32_t j = 0; j < 32u; ++j) {
            uint32_t byte = qs[32u * p + j];
            if constexpr (T == 13u) {
                const uint32_t w_odd = (byte >> 4) | (((src[16u + j] >> (2u * p + 1u)) & 1u) << 4);
                byte = (byte & 15u) | ((w_odd >> 1) << 4);
            }
            const uint32_t lane = 4u * g + (j >> 3);
            tile[s * 1024u + (p >> 1) * 512u + lane * 16u + (p & 1u) * 8u + (j & 7u)] = static_cast<uint8_t>(byte);
        }
    }
    if constexpr (T == 13u) {
        for (uint32_t j = 0; j < 32u; ++j) {
            const uint32_t hb = src[16u + j];
            uint32_t nh = 0;
            for (uint32_t p = 0; p < 4u; ++p) {
                const uint32_t w_odd = (qs[32u * p + j] >> 4) | (((hb >> (2u * p + 1u)) & 1u) << 4);
                nh |= ((hb >> (2u * p)) & 1u) << (2u * p + 1u);  // fifth bit of the even group
                nh |= (w_odd & 1u) << (2u * p);                   // lowest bit of the odd group
            }
            const uint32_t lane = 4u * g + (j >> 3);
            tile[F::kQh + lane * 16u + s * 8u + (j & 7u)] = static_cast<uint8_t>(nh);
        }
    }
    uint8_t* sc = tile + F::kSc + s * 128u + g * 16u;
    const uint8_t* q = src + 4;
    for (uint32_t j = 0; j < 8u; ++j) {
        uint8_t scale, mn;
        if (j < 4u) {
            scale = q[j] & 63u;
            mn = q[j + 4u] & 63u;
        } else {
            scale = static_cast<uint8_t>((q[j + 4u] & 15u) | ((q[j - 4u] >> 6) << 4));
            mn = static_cast<uint8_t>((q[j + 4u] >> 4) | ((q[j] >> 6) << 4));
        }
        sc[j] = scale;
        sc[8u + j] = mn;
    }
    uint8_t* dm = tile + F::kDm + s * 32u + g * 4u;
    for (uint32_t k = 0; k < 4u; ++k) dm[k] = src[k];
}

// GGUF Q6_K blocks (ql[128] | qh[64] | int8 scales[16] | d, 210 B; the code
// of element n: low nibble of ql[64h + l + 32(t&1)] (t < 2) or its high nibble,
// plus bits 2t..2t+1 of qh[32h + l] << 4, with h = n/128, t = n%128/32,
// l = n%32, src/quant.cpp's Q6_K dequantisation) -> layout-2 tiles.  One thread
// per (row, super-block); rows past a multiple of 8 must be zeroed first.
__global__ void repack_frag_q6_kernel(const uint8_t* __restrict__ blocks, uint8_t* __restrict__ tiles, uint32_t rows,
                                      uint32_t nb) {
    using F = FragTile<14>;
    const uint64_t idx = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<uint64_t>(rows) * nb) return;
    const uint32_t r = static_cast<uint32_t>(idx / nb), b = static_cast<uint32_t>(idx % nb);
    const uint32_t o = r >> 3, g = r & 7u, kc = b >> 1, s = b & 1u;
    const uint8_t* src = blocks + idx * 210u;
    uint8_t* tile = tiles + (static_cast<uint64_t>(o) * (nb / 2u) + kc) * F::kBytes;
    uint32_t lo[4][8], hi[4][4];
    for (uint32_t t = 0; t < 4u; ++t) {
        for (uint32_t j = 0; j < 8u; ++j) lo[t][j] = 0;
        for (uint32_t j = 0; j < 4u; ++j) hi[t][j] = 0;
    }
    for (uint32_t n = 0; n < 256u; ++n) {
        const uint32_t h = n >> 7, tq = (n & 127u) >> 5, l = n & 31u;
        const uint32_t lb = src[64u * h + l + 32u * (tq & 1u)];
        const uint32_t lo4 = tq < 2u ? (lb & 15u) : (lb >> 4);
        const uint32_t hi2 = (src[128u + 32u * h + l] >> (2u * tq)) & 3u;
        const uint32_t G = n >> 4, pos = n & 15u, j = G >> 1, par = G & 1u, t = pos >> 2, k = pos & 3u;
        lo[t][j] |= lo4 << (8u * k + 4u * par);
        hi[t][2u * par + (j >> 2)] |= hi2 << (8u * k + 2u * (j & 3u));
    }
    for (uint32_t t = 0; t < 4u; ++t) {
        const uint32_t lane = 4u * g + t;
        uint4* lp = reinterpret_cast<uint4*>(tile + F::kLo + s * 1024u + lane * 32u);
        lp[0] = make_uint4(lo[t][0], lo[t][1], lo[t][2], lo[t][3]);
        lp[1] = make_uint4(lo[t][4], lo[t][5], lo[t][6], lo[t][7]);
        *reinterpret_cast<uint4*>(tile + F::kHi + s * 512u + lane * 16u) = make_uint4(hi[t][0], hi[t][1], hi[t][2], hi[t][3]);
    }
    for (uint32_t i = 0; i < 16u; ++i) tile[F::kSc + s * 128u + g * 16u + i] = src[192u + i];
    tile[F::kD + s * 16u + g * 2u] = src[208];
    tile[F::kD + s * 16u + g * 2u + 1u] = src[209];
}

// A 4-bit IQ4_XS code as stored in a tile (FragTile<23>).
__host__ __device__ constexpr uint32_t iq4_tile_code(uint32_t c) { return ((c & 1u) << 3) | (c >> 1); }

// GGUF IQ4_XS blocks (d | scales_h u16 | scales_l[4] | qs[128], 136 B; group g
// code j < 16 in the low nibble of qs[16g + j], code j + 16 in its high
// nibble, scale ls = low nibble of scales_l[g/2] >> 4(g&1) | two bits of
// scales_h << 4, src/quant.cpp's IQ4_XS dequantisation) -> layout-2 tiles.
__global__ void repack_frag_iq4_kernel(const uint8_t* __restrict__ blocks, uint8_t* __restrict__ tiles, uint32_t rows,
                                       uint32_t nb) {
    using F = FragTile<23>;
    const uint64_t idx = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<uint64_t>(rows) * nb) return;
    const uint32_t r = static_cast<uint32_t>(idx / nb), b = static_cast<uint32_t>(idx % nb);
    const uint32_t o = r >> 3, g = r & 7u, kc = b >> 1, s = b & 1u;
    const uint8_t* src = blocks + idx * 136u;
    uint8_t* tile = tiles + (static_cast<uint64_t>(o) * (nb / 2u) + kc) * F::kBytes;
    const uint32_t sh = static_cast<uint32_t>(src[2]) | (static_cast<uint32_t>(src[3]) << 8);
    for (uint32_t G = 0; G < 8u; ++G) {
        const uint32_t ls = ((src[4u + G / 2u] >> (4u * (G & 1u))) & 15u) | (((sh >> (2u * G)) & 3u) << 4);
        tile[F::kSc + s * 64u + g * 8u + G] = static_cast<uint8_t>(static_cast<int8_t>(static_cast<int>(ls) - 32));
    }
    tile[F::kD + s * 16u + g * 2u] = src[0];
    tile[F::kD + s * 16u + g * 2u + 1u] = src[1];
    const uint8_t* qs = src + 8;
    for (uint32_t p = 0; p < 4u; ++p) {          // group pair (groups 2p, 2p+1)
        for (uint32_t t = 0; t < 4u; ++t) {      // lane (g, t): positions 8t..8t+7
            for (uint32_t half = 0; half < 2u; ++half) {
                uint32_t w = 0;
                for (uint32_t k = 0; k < 4u; ++k) {
                    const uint32_t pos = 8u * t + 4u * half + k;
                    for (uint32_t par = 0; par < 2u; ++par) {
                        const uint32_t G = 2u * p + par;
                        const uint32_t byte = qs[16u * G + (pos & 15u)];
                        const uint32_t code = pos < 16u ? (byte & 15u) : (byte >> 4);
                        w |= iq4_tile_code(code) << (16u * par + 4u * k);
                    }
                }
                const uint32_t lane = 4u * g + t;
                *reinterpret_cast<uint32_t*>(tile + s * 1024u + (p >> 1) * 512u + lane * 16u + (p & 1u) * 8u +
                                             half * 4u) = w;
            }
        }
    }
}

// ---- the GEMV --------------------------------------------------------------------
template <uint32_t T, int W, int DEPTH>
__host__ __device__ constexpr size_t frag_fixed_bytes() {
    return static_cast<size_t>(W) * DEPTH * FragTile<T>::kBytes + W * DEPTH * 8 + 8 +
           sizeof(PairBoundary<W, kF8Rows>) + 256;
}
template <uint32_t T, int W, int DEPTH>
__host__ __device__ constexpr size_t frag_smem_bytes(uint32_t nb, bool xsmem) {
    return frag_fixed_bytes<T, W, DEPTH>() + (xsmem ? xfrag_bytes_t(T, nb) : 0u);
}

// Byte I of w, zero-extended (one PRMT).
template <uint32_t I>
__device__ __forceinline__ int byte_u(uint32_t w) {
    return static_cast<int>(__byte_perm(w, 0u, 0x4440u | I));
}
// Exact float of the byte of w chosen by a PRMT selector over the constant
// 2^23 (the bits of 2^23 + byte), minus 2^23: no conversion instruction.
__device__ __forceinline__ float byte_f(uint32_t w, uint32_t sel) {
    return __uint_as_float(__byte_perm(w, 0x4b000000u, sel)) - 8388608.0f;
}

// Weights of one qs word (4 positions of group pair P): even group and the
// odd group scaled by 8 (Q5_K) or 16 (Q4_K).
template <uint32_t T, uint32_t P>
__device__ __forceinline__ void frag_decode(uint32_t q, uint32_t h, uint32_t& even, uint32_t& odd) {
    if constexpr (T == 13u) {
        const uint32_t R = __funnelshift_l(h, h, (3u - 2u * P) & 31u);
        even = (q & 0x0f0f0f0fu) | (R & 0x10101010u);
        odd = (q & 0xf0f0f0f0u) | (R & 0x08080808u);
    } else {
        (void)h;
        even = q & 0x0f0f0f0fu;
        odd = q & 0xf0f0f0f0u;
    }
}

// D = A x B (k = 32), A unsigned weights, B signed activation limbs; returns
// C[g][2t] and C[g+8][2t+1] of this lane.
__device__ __forceinline__ void mma_u8s8_16x8x32(int& c0, int& c3, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
    int c1, c2;
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(c0), "=r"(c1), "=r"(c2), "=r"(c3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
    (void)c1;
    (void)c2;
}

// One lane's share of a landed tile (8 rows x 2 super-blocks at chunk kc)
// added to its running fp64 sum acc (row g, limb t): per block
// (8 * Ae + Ao') * d * unit * 256^t / 8, then minus pair t's share of the min
// term of both blocks.
// The tile's bytes are read from shared memory `tb` into registers first and
// `after_load` runs between (it hands the slot back to the copy engine);
// xb points at the chunk's two x-fragment blocks (XL2: read from L2 with
// ld.cg, else shared memory).
template <uint32_t T, bool XL2, class AfterLoad>
__device__ __forceinline__ void frag_tile_acc(const uint8_t* tb, const uint8_t* xb, uint32_t lane, double& acc,
                                              AfterLoad&& after_load) {
    using F = FragTile<T>;
    const uint32_t g = lane >> 2, t = lane & 3u;
    // PRMT selectors of this lane's two mins (pair t) in word sc.z (t < 2) or
    // sc.w: bytes 2(t&1) and 2(t&1)+1, over the constant 2^23.
    const uint32_t msel_a = 0x7640u | (2u * (t & 1u)), msel_b = 0x7640u | (2u * (t & 1u) + 1u);
    uint4 qh = make_uint4(0u, 0u, 0u, 0u);
    if constexpr (T == 13u) qh = *reinterpret_cast<const uint4*>(tb + F::kQh + lane * 16u);
    uint4 qv[kF8Blocks][2], sc[kF8Blocks];
    uint32_t dmw[kF8Blocks];
#pragma unroll
    for (uint32_t s = 0; s < kF8Blocks; ++s) {
        sc[s] = *reinterpret_cast<const uint4*>(tb + F::kSc + s * 128u + g * 16u);
        dmw[s] = *reinterpret_cast<const uint32_t*>(tb + F::kDm + s * 32u + g * 4u);
#pragma unroll
        for (uint32_t c = 0; c < 2u; ++c) qv[s][c] = *reinterpret_cast<const uint4*>(tb + s * 1024u + c * 512u + lane * 16u);
    }
    after_load();
    float mn = 0.0f;
#pragma unroll
    for (uint32_t s = 0; s < kF8Blocks; ++s) {
        const uint8_t* xbs = xb + s * kXfBlockBytes;
        const uint32_t h0 = s ? qh.z : qh.x, h1 = s ? qh.w : qh.y;
        int Ae = 0, Ao = 0;  // even groups; odd groups (x8 or x16)
#pragma unroll
        for (uint32_t c = 0; c < 2u; ++c) {
            const uint8_t* xp = xbs + c * 512u + lane * 16u;
            const uint4 xv = XL2 ? __ldcg(reinterpret_cast<const uint4*>(xp)) : *reinterpret_cast<const uint4*>(xp);
            const uint32_t scw = c ? sc[s].y : sc[s].x;  // scales of groups 4c..4c+3
            const uint4 q = qv[s][c];
            uint32_t e0, o0w, e1, o1w;
            int d0, d3;
            if (c == 0) {
                frag_decode<T, 0>(q.x, h0, e0, o0w);
                frag_decode<T, 0>(q.y, h1, e1, o1w);
            } else {
                frag_decode<T, 2>(q.x, h0, e0, o0w);
                frag_decode<T, 2>(q.y, h1, e1, o1w);
            }
            mma_u8s8_16x8x32(d0, d3, e0, o0w, e1, o1w, xv.x, xv.y);
            Ae += byte_u<0>(scw) * d0;
            Ao += byte_u<1>(scw) * d3;
            if (c == 0) {
                frag_decode<T, 1>(q.z, h0, e0, o0w);
                frag_decode<T, 1>(q.w, h1, e1, o1w);
            } else {
                frag_decode<T, 3>(q.z, h0, e0, o0w);
                frag_decode<T, 3>(q.w, h1, e1, o1w);
            }
            mma_u8s8_16x8x32(d0, d3, e0, o0w, e1, o1w, xv.z, xv.w);
            Ae += byte_u<2>(scw) * d0;
            Ao += byte_u<3>(scw) * d3;
        }
        // limb t of this row: (8 * Ae + Ao') * d * unit * 256^t / 8, exact
        // in int32 (|.| < 2^30); pair t's share of the min term in fp32
        const int A8 = Ae * 8 + (Ao >> F::kOddShift);
        const uint4 xm = XL2 ? __ldcg(reinterpret_cast<const uint4*>(xbs + kXfMetaOff + t * 16u))
                             : *reinterpret_cast<const uint4*>(xbs + kXfMetaOff + t * 16u);
        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&dmw[s]));
        const double unw = __hiloint2double(static_cast<int>(xm.y), static_cast<int>(xm.x));
        acc = __fma_rn(static_cast<double>(A8), static_cast<double>(dm.x) * unw, acc);
        const uint32_t mw = t < 2u ? sc[s].z : sc[s].w;
        const float pm = fmaf(byte_f(mw, msel_a), __uint_as_float(xm.z), byte_f(mw, msel_b) * __uint_as_float(xm.w));
        mn = fmaf(dm.y, pm, mn);
    }
    acc -= static_cast<double>(mn);
}

// D = A x B (k = 16), A and B signed bytes; returns D[g][2t] and D[g+8][2t+1].
__device__ __forceinline__ void mma_s8s8_16x8x16(int& c0, int& c3, uint32_t a0, uint32_t a1, uint32_t b0) {
    int c1, c2;
    asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};\n"
        : "=r"(c0), "=r"(c1), "=r"(c2), "=r"(c3)
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
    (void)c1;
    (void)c2;
}

// Signed byte k of w.
template <int K>
__device__ __forceinline__ int byte_s(uint32_t w) {
    return static_cast<int>(w << (24 - 8 * K)) >> 24;
}

// One lane's share of a landed Q6_K tile added to its fp64 sum (row g, limb t):
// per super-block and group pair j one mma.sync.m16n8k16.s8 of A rows 0-7 =
// the 8 rows' even group 2j, rows 8-15 = their odd group 2j+1, A bytes
// 4 (q - 32) built as (4q) ^ 0x80 from the LO nibbles and the HI two-bit
// fields; exact int32 group scaling by the int8 scales, then
// (Ae + Ao) * d * unit * 256^t / 4 in fp64.
template <bool XL2, class AfterLoad>
__device__ __forceinline__ void q6_tile_acc(const uint8_t* tb, const uint8_t* xb, uint32_t lane, double& acc,
                                            AfterLoad&& after_load) {
    using F = FragTile<14>;
    const uint32_t g = lane >> 2, t = lane & 3u;
    uint4 lo[kF8Blocks][2], hi[kF8Blocks], sc[kF8Blocks];
    uint32_t dw[kF8Blocks];
#pragma unroll
    for (uint32_t s = 0; s < kF8Blocks; ++s) {
        lo[s][0] = *reinterpret_cast<const uint4*>(tb + F::kLo + s * 1024u + lane * 32u);
        lo[s][1] = *reinterpret_cast<const uint4*>(tb + F::kLo + s * 1024u + lane * 32u + 16u);
        hi[s] = *reinterpret_cast<const uint4*>(tb + F::kHi + s * 512u + lane * 16u);
        sc[s] = *reinterpret_cast<const uint4*>(tb + F::kSc + s * 128u + g * 16u);
        dw[s] = *reinterpret_cast<const uint16_t*>(tb + F::kD + s * 16u + g * 2u);
    }
    after_load();
#pragma unroll
    for (uint32_t s = 0; s < kF8Blocks; ++s) {
        const uint8_t* xbs = xb + s * kX6BlockBytes;
        const uint4 xa = XL2 ? __ldcg(reinterpret_cast<const uint4*>(xbs + lane * 16u))
                             : *reinterpret_cast<const uint4*>(xbs + lane * 16u);
        const uint4 xc = XL2 ? __ldcg(reinterpret_cast<const uint4*>(xbs + 512u + lane * 16u))
                             : *reinterpret_cast<const uint4*>(xbs + 512u + lane * 16u);
        const uint32_t L[8] = {lo[s][0].x, lo[s][0].y, lo[s][0].z, lo[s][0].w,
                               lo[s][1].x, lo[s][1].y, lo[s][1].z, lo[s][1].w};
        const uint32_t X[8] = {xa.x, xa.y, xa.z, xa.w, xc.x, xc.y, xc.z, xc.w};
        const uint32_t S[4] = {sc[s].x, sc[s].y, sc[s].z, sc[s].w};
        int Ae = 0, Ao = 0;
#pragma unroll
        for (uint32_t j = 0; j < 8u; ++j) {
            const uint32_t E = j < 4u ? hi[s].x : hi[s].y, O = j < 4u ? hi[s].z : hi[s].w;
            const uint32_t sh = 6u - 2u * (j & 3u);
            const uint32_t ae = ((L[j] << 2) & 0x3c3c3c3cu) | (((E << sh) & 0xc0c0c0c0u) ^ 0x80808080u);
            const uint32_t ao = ((L[j] >> 2) & 0x3c3c3c3cu) | (((O << sh) & 0xc0c0c0c0u) ^ 0x80808080u);
            int d0, d3;
            mma_s8s8_16x8x16(d0, d3, ae, ao, X[j]);
            const uint32_t sw = S[j >> 1];  // int8 scales of groups 4(j/2) .. 4(j/2)+3
            if (j & 1u) {
                Ae += byte_s<2>(sw) * d0;
                Ao += byte_s<3>(sw) * d3;
            } else {
                Ae += byte_s<0>(sw) * d0;
                Ao += byte_s<1>(sw) * d3;
            }
        }
        const double unw = *reinterpret_cast<const double*>(xbs + kX6MetaOff + t * 8u);
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(dw[s])));
        acc = __fma_rn(static_cast<double>(Ae + Ao), static_cast<double>(d) * unw, acc);
    }
}

// prmt.b32 with the full selector: a selector nibble with bit 3 set gives the
// sign of the selected byte replicated over the result byte (PTX ISA, prmt).
__device__ __forceinline__ uint32_t prmt_b32(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// The IQ4_XS codebook (src/quant.cpp:468-471, kv[0..15]) split for tile codes:
// slot i of L holds kv[2i]; slot i of H holds kv[2i + 1], complemented where
// kv[2i] (and so kv[2i + 1]) is negative, which leaves every H byte positive.
constexpr uint32_t kIq4L0 = iq4nl_word(-127, -83, -49, -22);
constexpr uint32_t kIq4L1 = iq4nl_word(1, 25, 53, 89);
constexpr uint32_t kIq4H0 = iq4nl_word(~-104, ~-65, ~-35, ~-10);
constexpr uint32_t kIq4H1 = iq4nl_word(13, 38, 69, 113);

// One tile word of eight stored codes e (group 2p's four in the low 16 bits,
// group 2p + 1's in the high 16 bits) -> two words of four int8 codebook
// values.  For e = 8h + i the L lookup with selector e gives kv[2i] when h = 0
// and sign(kv[2i]) when h = 1; the H lookup with selector e ^ 8 gives
// sign(H[i]) = 0 when h = 0 and H[i] = kv[2i + 1] ^ sign(kv[2i]) when h = 1.
// Their XOR is kv[2i + h], the entry of the code c = 2i + h, in both cases:
// two byte_perms and one XOR per four codes, no masks.
__device__ __forceinline__ void iq4_codes8(uint32_t q, uint32_t& even, uint32_t& odd) {
    const uint32_t f = q ^ 0x88888888u;
    even = prmt_b32(kIq4L0, kIq4L1, q) ^ prmt_b32(kIq4H0, kIq4H1, f);
    odd = prmt_b32(kIq4L0, kIq4L1, q >> 16) ^ prmt_b32(kIq4H0, kIq4H1, f >> 16);
}

// D = A x B (k = 32), A and B signed bytes; returns D[g][2t] and D[g+8][2t+1].
__device__ __forceinline__ void mma_s8s8_16x8x32(int& c0, int& c3, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
    int c1, c2;
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(c0), "=r"(c1), "=r"(c2), "=r"(c3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
    (void)c1;
    (void)c2;
}

// One lane's share of a landed IQ4_XS tile added to its fp64 sum (row g, limb
// t): the same mma per (8 rows, group pair) as the Q5_K / Q4_K tiles, with the
// codebook values (signed) as A, then the signed group scales, then
// 8 (Ae + Ao) * d * unit * 256^t / 8 against the x-fragments (no min term).
template <bool XL2, class AfterLoad>
__device__ __forceinline__ void iq4_tile_acc(const uint8_t* tb, const uint8_t* xb, uint32_t lane, double& acc,
                                             AfterLoad&& after_load) {
    using F = FragTile<23>;
    const uint32_t g = lane >> 2, t = lane & 3u;
    uint4 qv[kF8Blocks][2];
    uint2 scv[kF8Blocks];
    uint32_t dw[kF8Blocks];
#pragma unroll
    for (uint32_t s = 0; s < kF8Blocks; ++s) {
#pragma unroll
        for (uint32_t c = 0; c < 2u; ++c) qv[s][c] = *reinterpret_cast<const uint4*>(tb + s * 1024u + c * 512u + lane * 16u);
        scv[s] = *reinterpret_cast<const uint2*>(tb + F::kSc + s * 64u + g * 8u);
        dw[s] = *reinterpret_cast<const uint16_t*>(tb + F::kD + s * 16u + g * 2u);
    }
    after_load();
#pragma unroll
    for (uint32_t s = 0; s < kF8Blocks; ++s) {
        const uint8_t* xbs = xb + s * kXfBlockBytes;
        int Ae = 0, Ao = 0;
#pragma unroll
        for (uint32_t c = 0; c < 2u; ++c) {
            const uint8_t* xp = xbs + c * 512u + lane * 16u;
            const uint4 xv = XL2 ? __ldcg(reinterpret_cast<const uint4*>(xp)) : *reinterpret_cast<const uint4*>(xp);
            const uint4 q = qv[s][c];
            const uint32_t sw = c ? scv[s].y : scv[s].x;  // scales of groups 4c..4c+3
            int d0, d3;
            uint32_t a0, a1, a2, a3;
            iq4_codes8(q.x, a0, a1);
            iq4_codes8(q.y, a2, a3);
            mma_s8s8_16x8x32(d0, d3, a0, a1, a2, a3, xv.x, xv.y);
            Ae += byte_s<0>(sw) * d0;
            Ao += byte_s<1>(sw) * d3;
            iq4_codes8(q.z, a0, a1);
            iq4_codes8(q.w, a2, a3);
            mma_s8s8_16x8x32(d0, d3, a0, a1, a2, a3, xv.z, xv.w);
            Ae += byte_s<2>(sw) * d0;
            Ao += byte_s<3>(sw) * d3;
        }
        const double unw = *reinterpret_cast<const double*>(xbs + kXfMetaOff + t * 16u);
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(dw[s])));
        acc = __fma_rn(static_cast<double>((Ae + Ao) * 8), static_cast<double>(d) * unw, acc);
    }
}

// f32 activations [nb * 256] -> x-fragments in shared memory xs, packed by the
// CTA's W warps (warp w takes blocks w, w + W, ...; at most kF8PackPerWarp
// each): every warp loads all of its blocks first (one L2 round trip), then
// packs them.  The caller synchronises the CTA afterwards.
template <int W, uint32_t T = 13>
__device__ __forceinline__ void frag_pack_x_f32(const float* xv, uint32_t nb, uint8_t* xs, uint32_t warp,
                                                uint32_t lane) {
    float4 v0[kF8PackPerWarp], v1[kF8PackPerWarp];
#pragma unroll
    for (uint32_t i = 0; i < kF8PackPerWarp; ++i) {
        const uint32_t b = warp + i * W;
        if (b < nb) {
            v0[i] = __ldcg(reinterpret_cast<const float4*>(xv + b * 256u + lane * 8u));
            v1[i] = __ldcg(reinterpret_cast<const float4*>(xv + b * 256u + lane * 8u + 4u));
        }
    }
#pragma unroll
    for (uint32_t i = 0; i < kF8PackPerWarp; ++i) {
        const uint32_t b = warp + i * W;
        if (b < nb) {
            const float v[8] = {v0[i].x, v0[i].y, v0[i].z, v0[i].w, v1[i].x, v1[i].y, v1[i].z, v1[i].w};
            if constexpr (T == 14u)
                pack_block_warp_x6(v, lane, xs + b * kX6BlockBytes);
            else
                pack_block_warp_frag(v, lane, xs + b * kXfBlockBytes);
        }
    }
}

// Row octets split between warps: the first entry of each run of a CTA's
// boundary table sums the run in warp order and writes the eight rows (row
// octet o0 + pair).  Called by threads 0 .. 2W-1 after a CTA barrier.
template <int W>
__device__ __forceinline__ void frag_boundary_combine(const PairBoundary<W, kF8Rows>* bnd, uint32_t e, uint32_t o0,
                                                      uint32_t rows, float* y, const float* res) {
    constexpr uint32_t R = kF8Rows;
    const int pr = bnd->pair[e];
    if (pr < 0) return;
    int prev = e >= 1 ? bnd->pair[e - 1] : -1;
    if (prev == -1 && e >= 2) prev = bnd->pair[e - 2];
    if (prev == pr) return;
    double v[R];
#pragma unroll
    for (uint32_t r = 0; r < R; ++r) v[r] = bnd->v[e][r];
    for (uint32_t q = e + 1u; q < 2u * W; ++q) {
        const int pq = bnd->pair[q];
        if (pq == -1) continue;
        if (pq != pr) break;
#pragma unroll
        for (uint32_t r = 0; r < R; ++r) v[r] += bnd->v[q][r];
    }
    const uint32_t row = R * (o0 + static_cast<uint32_t>(pr));
    float out[R];
#pragma unroll
    for (uint32_t r = 0; r < R; ++r) out[r] = row + r < rows ? gemv_out(v[r], res, row + r) : 0.0f;
    if ((reinterpret_cast<uintptr_t>(y) & 15u) == 0 && row + R <= rows) {
        *reinterpret_cast<float4*>(y + row) = make_float4(out[0], out[1], out[2], out[3]);
        *reinterpret_cast<float4*>(y + row + 4u) = make_float4(out[4], out[5], out[6], out[7]);
        return;
    }
#pragma unroll
    for (uint32_t r = 0; r < R; ++r)
        if (row + r < rows) y[row + r] = out[r];
}

// Activations come from the previous kernel of a PDL chain, whose CTAs can
// share an SM with this grid's: they are read with L2-only loads (ld.cg), never
// through the non-coherent read-only path, which can return lines cached on
// the SM before the producer wrote them.
// XM 0: x-fragments read from L2; XM 1: copied to shared memory by one
// bulk copy per CTA; XM 2: xf is an f32 vector that every CTA packs into
// x-fragments in shared memory itself (one kernel for an f32 GEMV).  res (may
// alias y) is added to the output when non-null.
//
// The work of one CTA: `cta` of `ncta` CTAs sharing the matrix (row octets
// split evenly), in the dynamic shared memory `smem`.
template <uint32_t T, int XM, int W, int DEPTH>
__device__ __forceinline__ void gemv_frag_cta(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xf, float* y,
                                              const float* res, uint32_t rows, uint32_t nb, uint32_t cta,
                                              uint32_t ncta, uint8_t* smem) {
    using F = FragTile<T>;
    constexpr uint32_t C = W, R = kF8Rows, TB = F::kBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(W) * DEPTH * TB);
    uint64_t* xbar = bars + C * DEPTH;
    PairBoundary<W, R>* bnd = reinterpret_cast<PairBoundary<W, R>*>(xbar + 1);
    uint8_t* xs = reinterpret_cast<uint8_t*>(bnd + 1);
    xs += (128u - (reinterpret_cast<uintptr_t>(xs) & 127u)) & 127u;

    if (threadIdx.x == 0) pdl_launch_dependents();

    const uint32_t cons = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t nocts = (rows + R - 1u) / R, nkc = nb / kF8Blocks;
    // even split of row octets over CTAs, then of the CTA's tiles over warps
    const uint32_t obase = nocts / ncta, orem = nocts % ncta;
    const uint32_t o0 = cta * obase + min(cta, orem);
    const uint32_t o1 = o0 + obase + (cta < orem ? 1u : 0u);
    const uint32_t ntiles = (o1 - o0) * nkc;
    const uint32_t base = ntiles / C, rem = ntiles % C;
    const uint32_t len = base + (cons < rem ? 1u : 0u);
    const uint32_t first = cons * base + min(cons, rem);
    const uint8_t* src = w + (static_cast<size_t>(o0) * nkc + first) * TB;
    uint8_t* ring = smem + static_cast<size_t>(cons) * DEPTH * TB;
    uint64_t* full = bars + cons * DEPTH;
    auto issue = [&](uint32_t k) {
        mbar_arrive_expect_tx(&full[k % DEPTH], TB);
        tma_load_1d(ring + (k % DEPTH) * TB, src + static_cast<size_t>(k) * TB, TB, &full[k % DEPTH]);
    };
    if (lane == 0) {
        for (uint32_t i = 0; i < DEPTH; ++i) mbar_init(&full[i], 1);
        if (XM == 1 && cons == 0) mbar_init(xbar, 1);
        fence_mbar_init();
        for (uint32_t k = 0; k < DEPTH && k < len; ++k) issue(k);
    }
    if (threadIdx.x < 2 * C) bnd->pair[threadIdx.x] = -1;
    __syncthreads();

    pdl_wait();  // x-fragments, y and res belong to the dependency chain
    const uint8_t* xl;
    if constexpr (XM == 2) {
        // the host keeps nb <= kF8PackPerWarp * W for this mode
        frag_pack_x_f32<W, T>(reinterpret_cast<const float*>(xf), nb, xs, cons, lane);
        __syncthreads();
        xl = xs;
    } else if constexpr (XM == 1) {
        if (threadIdx.x == 0) {
            const uint32_t bytes = static_cast<uint32_t>(xfrag_bytes_t(T, nb));
            mbar_arrive_expect_tx(xbar, bytes);
            tma_load_1d(xs, xf, bytes, xbar);
        }
        xl = xs;
    } else {
        xl = xf;
    }
    const uint32_t g = lane >> 2, t = lane & 3u;
    bool ok = true;
    if constexpr (XM == 1) {
        if (!mbar_wait_spin(xbar, 0, kFaultFullWait)) ok = false;
    }

    double acc = 0.0;
    uint32_t issued = min(len, static_cast<uint32_t>(DEPTH)), waited = 0;
    uint32_t oct = first / nkc, kc = first - oct * nkc;
    uint32_t kc_first = kc, nflush = 0;
    bool started = false;

    // an octet's 8 outputs leave as two 16-byte stores when y allows it: a
    // quarter of the stores, which matters when y is page-locked host memory
    const bool y16 = (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
    auto flush = [&](bool whole) {
        double v = acc;  // after the two exchanges every lane of row g holds the same sum
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        const uint32_t row0 = R * (o0 + oct), row = row0 + g;
        if (whole) {
            const float out = row < rows ? gemv_out(v, res, row) : 0.0f;
            const float o1 = __shfl_down_sync(0xffffffffu, out, 4);   // rows g + 1,
            const float o2 = __shfl_down_sync(0xffffffffu, out, 8);   // g + 2
            const float o3 = __shfl_down_sync(0xffffffffu, out, 12);  // and g + 3
            if (ok) {
                if (y16 && row0 + R <= rows) {
                    if ((lane & 15u) == 0u) *reinterpret_cast<float4*>(y + row) = make_float4(out, o1, o2, o3);
                } else if (t == 0 && row < rows) {
                    y[row] = out;
                }
            }
        } else if (t == 0) {
            const uint32_t e = cons * 2u + (nflush == 0 ? 0u : 1u);
            bnd->v[e][g] = v;
            if (g == 0) bnd->pair[e] = static_cast<int>(oct);
        }
        ++nflush;
        acc = 0.0;
    };

    for (uint32_t i = 0; i < len; ++i) {
        const uint32_t slot = i % DEPTH;
        const bool landed =
            __all_sync(0xffffffffu, ok && mbar_wait_spin(&full[slot], (i / DEPTH) & 1u, kFaultFullWait));
        if (!landed) ok = false;
        else waited = i + 1u;
        started = true;
        if (ok) {
            // This lane's share of the tile goes to registers, then the slot is
            // handed straight back to the copy engine.
            auto refill = [&] {
                __syncwarp();
                if (lane == 0 && i + DEPTH < len) {
                    fence_proxy_async_smem();
                    issue(i + DEPTH);
                    issued = i + DEPTH + 1u;
                }
            };
            const uint8_t* xk = xl + static_cast<size_t>(kc) * (kF8Blocks * xf_block_bytes(T));
            if constexpr (T == 14u)
                q6_tile_acc<XM == 0>(ring + slot * TB, xk, lane, acc, refill);
            else if constexpr (T == 23u)
                iq4_tile_acc<XM == 0>(ring + slot * TB, xk, lane, acc, refill);
            else
                frag_tile_acc<T, XM == 0>(ring + slot * TB, xk, lane, acc, refill);
        }
        if (++kc == nkc) {  // octet complete
            flush(kc_first == 0);
            kc = 0;
            kc_first = 0;
            ++oct;
            started = false;
        }
    }
    if (started) flush(false);
    if (!ok && lane == 0) {
        for (uint32_t k = waited; k < issued; ++k)
            if (!mbar_wait(&full[k % DEPTH], (k / DEPTH) & 1u, kFaultDrain)) break;
    }

    // Octets split between warps: the first entry of each run sums it in warp
    // order and writes the eight rows.
    __syncthreads();
    if (threadIdx.x < 2u * C && ok) frag_boundary_combine<W>(bnd, threadIdx.x, o0, rows, y, res);
}

template <uint32_t T, int XM, int W, int DEPTH, int MINB>
__global__ void __launch_bounds__(W * 32, MINB)
    gemv_frag_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xf, float* y, const float* res,
                     uint32_t rows, uint32_t nb) {
    extern __shared__ __align__(128) uint8_t smem[];
    gemv_frag_cta<T, XM, W, DEPTH>(w, xf, y, res, rows, nb, blockIdx.x, gridDim.x, smem);
}

// Two GEMVs over the same x-fragments in one launch -- the decode layer's
// qkv+z (Q5_K) with beta+alpha (Q4_K) and ffn_gate (Q4_K) with ffn_up (Q5_K):
// CTAs [0, split) compute y_a = W_a x, the others y_b = W_b x, each exactly as
// its own gemv_frag_kernel launch would, so the pair costs one dependent
// launch instead of two.
struct FragJob {
    const uint8_t* w;
    float* y;
    uint32_t rows;
};

template <uint32_t TA, uint32_t TB, int XM, int W, int DEPTH>
__global__ void __launch_bounds__(W * 32, 1)
    gemv_frag_pair_kernel(const FragJob a, const FragJob b, const uint8_t* __restrict__ xf, uint32_t nb,
                          uint32_t split) {
    extern __shared__ __align__(128) uint8_t smem[];
    if (blockIdx.x < split)
        gemv_frag_cta<TA, XM, W, DEPTH>(a.w, xf, a.y, nullptr, a.rows, nb, blockIdx.x, split, smem);
    else
        gemv_frag_cta<TB, XM, W, DEPTH>(b.w, xf, b.y, nullptr, b.rows, nb, blockIdx.x - split, gridDim.x - split,
                                        smem);
}

// The same pair when matrix b reads another activation format: CTAs [0,
// split) run W_a over the x-fragments xfa (staged by one bulk copy), the others
// pack f32 x (xb) in the CTA -- the attention block's q|gate|k projection
// (Q5_K) with its v projection (Q6_K tiles, whose 16-weight groups read Q6
// x-fragments), one dependent launch instead of two.
template <uint32_t TA, uint32_t TB, int W, int DEPTH>
__global__ void __launch_bounds__(W * 32, 1)
    gemv_frag_pair_xf_kernel(const FragJob a, const FragJob b, const uint8_t* __restrict__ xfa,
                             const float* __restrict__ xb, uint32_t nb, uint32_t split) {
    extern __shared__ __align__(128) uint8_t smem[];
    if (blockIdx.x < split)
        gemv_frag_cta<TA, 1, W, DEPTH>(a.w, xfa, a.y, nullptr, a.rows, nb, blockIdx.x, split, smem);
    else
        gemv_frag_cta<TB, 2, W, DEPTH>(b.w, reinterpret_cast<const uint8_t*>(xb), b.y, nullptr, b.rows, nb,
                                       blockIdx.x - split, gridDim.x - split, smem);
}

}  // namespace q38
