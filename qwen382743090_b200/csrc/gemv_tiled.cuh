// gemv_tiled.cuh -- Q5_K GEMV over the B200 tiled execution layout (Q38PACK
// layout 2).  Same mathematics as the reference's q38_q5k_sm86_soa_gemv_vec
// (src/driver.cpp:3887-4138) and q38_q5k_q8k_dp4a_gemv (:3660-3885).
//
// Layout 2 (Q5_K).  Rows are grouped in quads (4 rows; a partial last quad is
// padded with all-zero rows) and K in chunks of 4 super-blocks; each (quad,
// chunk) is one contiguous 2880-byte tile
//     QS   [4 rows][4 blocks][128]   at    0
//     QH   [4 rows][4 blocks][32]    at 2048
//     META [4 rows][4 blocks][20]    at 2560   (d, dmin, 8 x {scale, min})
// stored quad-major: tile (quad j, chunk c) at byte (j * nb/4 + c) * 2880.
// The bytes of every block are those of the SoA planes of layout 1, so the
// decoded weights are unchanged; only their order differs.  A CTA that owns a
// contiguous range of quads therefore reads one contiguous byte range.
//
// Kernel structure (sm_100a):
//  * 16 consumers (one per warp) per CTA each own a contiguous run of the CTA's
//    tiles.  In the prologue each consumer asks L2 to prefetch its whole run in
//    2 KB pieces (cp.async.bulk.prefetch.L2) and the CTA triggers the next grid
//    (PDL), so the DRAM stream starts at full width before any dependency
//    resolves; then each consumer keeps 4 single-tile 1-D bulk TMA copies
//    (cp.async.bulk, no multicast) in flight in its private smem ring;
//  * after the dependency resolves the CTA copies the whole x-pack into shared
//    memory with one bulk copy when it fits (else lanes read it through L1);
//  * a lane is (row r, super-block s, group pair p) and decodes 64 weights per
//    tile in registers; the lanes of both rows load the same activation quads
//    in one instruction (broadcast); dot products are dp4a against the x-pack
//    limbs (xpack.cuh) and the 6-bit group scales multiply the integer sums
//    before any conversion;
//  * a lane accumulates in fp64 while its consumer stays on one row pair; the
//    16 lanes of a row reduce with shuffles, and row pairs split between
//    consumers are summed afterwards in consumer order (deterministic);
//  * only x, y and the x-dependent work wait for the predecessor grid.
#pragma once

#include "gemv_q5k.cuh"
#include "layer.cuh"

namespace q38 {

constexpr uint32_t kT2Rows = 4;
constexpr uint32_t kT2Blocks = 4;
constexpr uint32_t kT2TileBytes = kT2Rows * kT2Blocks * 180;  // 2880
constexpr uint32_t kT2QhOff = kT2Rows * kT2Blocks * 128;      // 2048
constexpr uint32_t kT2MetaOff = kT2QhOff + kT2Rows * kT2Blocks * 32;  // 2560
constexpr uint32_t kT2Warps = 16;                     // warps per CTA, each an independent consumer
constexpr uint32_t kT2Threads = kT2Warps * 32;
constexpr uint32_t kT2Depth = 2;                      // private ring slots per consumer
constexpr uint32_t kT2TilesPerSlot = 1;               // tiles per slot, fetched by one bulk copy
constexpr uint32_t kL2PrefetchPiece = 2048;
// Activations are staged in shared memory when they fit next to the ring and
// still leave room for the next kernel's CTA (PDL co-residency).
constexpr size_t kT2SmemBudget = 112u * 1024u;

// Partial sums of row groups (pairs or quads, R rows) split between
// consumers (C consumers, two entries each), combined after the main loop in
// consumer order.
template <int C, int R = 2>
struct PairBoundary {
    int pair[C * 2];
    double v[C * 2][R];
};
template <int W, int DEPTH, int TPS = kT2TilesPerSlot>
__host__ __device__ constexpr size_t t2_ring_bytes() {
    return static_cast<size_t>(W) * DEPTH * TPS * kT2TileBytes;
}
// +256: 128-byte alignment of the activation region
template <int W, int DEPTH, int TPS = kT2TilesPerSlot>
__host__ __device__ constexpr size_t t2_fixed_bytes() {
    return t2_ring_bytes<W, DEPTH, TPS>() + W * DEPTH * 8 + 8 + sizeof(PairBoundary<W, kT2Rows>) + 256;
}
constexpr size_t kT2RingBytes = t2_ring_bytes<kT2Warps, kT2Depth>();  // 92160
constexpr size_t kT2FixedBytes = t2_fixed_bytes<kT2Warps, kT2Depth>();

// Bytes of the activation x-pack for one row of nb super-blocks.
__host__ __device__ constexpr uint32_t t2_xbytes(uint32_t nb, int nl) {
    return static_cast<uint32_t>(xpack_row_limb_bytes(nl, nb)) + nb * 32u + xpack_nb4(nb) * 4u;
}
template <int W, int DEPTH, int TPS = kT2TilesPerSlot>
__host__ __device__ constexpr size_t t2_smem_bytes_t(uint32_t nb, int nl, bool xsmem) {
    return t2_fixed_bytes<W, DEPTH, TPS>() + (xsmem ? t2_xbytes(nb, nl) : 0u);
}
__host__ __device__ constexpr size_t t2_smem_bytes(uint32_t nb, int nl, bool xsmem) {
    return t2_smem_bytes_t<kT2Warps, kT2Depth>(nb, nl, xsmem);
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

// Scale the two group dots of one (row, super-block, pair): the 6-bit group
// scales multiply the integer limb sums exactly (|sc*a| < 2^25 per limb), the
// limbs combine exactly in 64-bit integers and convert to fp64 once; d*es
// multiplies in fp64.  The dmin*m*sum(x) term is a few units in magnitude per
// group and stays in fp32 (its rounding is ~1e-7 of a unit).
template <int NL>
__device__ __forceinline__ double q5_pair_scale(const int (&aa)[NL], const int (&ab)[NL], uint32_t dm, uint32_t scm,
                                                float es, float2 X) {
    const int sca = static_cast<int>(scm & 0xffu), scb = static_cast<int>((scm >> 16) & 0xffu);
    long long f = 0;
#pragma unroll
    for (int k = NL - 1; k >= 0; --k) f = f * 256 + static_cast<long long>(sca * aa[k] + scb * ab[k]);
    const float2 dmf = __half22float2(*reinterpret_cast<const __half2*>(&dm));
    const float mn = fmaf(static_cast<float>((scm >> 8) & 0xffu), X.x, static_cast<float>(scm >> 24) * X.y);
    return __fma_rn(static_cast<double>(dmf.x * es), static_cast<double>(f), static_cast<double>(-dmf.y * mn));
}

// Output row value, plus the residual when one is given (y may alias res:
// each row is read and written by the same thread).
__device__ __forceinline__ float gemv_out(double v, const float* res, uint32_t row) {
    return static_cast<float>(res ? v + static_cast<double>(res[row]) : v);
}

template <int NL, bool XS>
__device__ __forceinline__ uint4 t2_load_quad(const uint8_t* p) {
    if constexpr (XS) return *reinterpret_cast<const uint4*>(p);
    else return __ldg(reinterpret_cast<const uint4*>(p));
}

// Pack one row of f32 activations (nb super-blocks) into the three-limb
// x-pack layout in shared memory, one warp per super-block.  With nw given the
// packed values are the RMSNorm output x * inv * nw.
__device__ __forceinline__ void t2_pack_x_f32(const float* __restrict__ x, uint32_t nb, uint8_t* xs, float* gsum,
                                              float* scale, uint32_t warp, uint32_t lane, uint32_t nwarps,
                                              const float* __restrict__ nw = nullptr, float inv = 1.0f) {
    for (uint32_t b = warp; b < nb; b += nwarps) {
        const float4 v0 = __ldg(reinterpret_cast<const float4*>(x + b * 256u + lane * 8u));
        const float4 v1 = __ldg(reinterpret_cast<const float4*>(x + b * 256u + lane * 8u + 4u));
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
        const float4 v0 = __ldg(reinterpret_cast<const float4*>(x + b * 256u + lane * 8u));
        const float4 v1 = __ldg(reinterpret_cast<const float4*>(x + b * 256u + lane * 8u + 4u));
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

// Largest row the fused RMSNorm handles (super-blocks).
constexpr uint32_t kNormMaxBlocks = 128;

// XM selects where the activations come from: 0 = x-pack read through L1,
// 1 = x-pack copied into shared memory, 2 = f32 x packed into shared memory by
// this CTA (xlimbs then points at the f32 vector; NL must be 3), 3 = the same
// after RMSNorm (xgsum then points at the norm weight, eps is its epsilon).
// With res non-null the kernel writes y = W x + res (y may equal res).
//
// Each of the W warps is one consumer with a private ring of DEPTH slots of
// TPS tiles.  In a tile, lane (h, s, p) = (lane / 16, lane / 4 % 4, lane % 4)
// decodes rows h and h + 2 of the quad for super-block s and group pair p:
// 2 x 64 weights against one set of activation words (the two 16-lane halves
// load the same words in one instruction, a shared-memory broadcast).  The
// whole warp waits on one barrier per slot, so its lanes never diverge.
template <int NL, int XM, int W = kT2Warps, int DEPTH = kT2Depth, int TPS = kT2TilesPerSlot, bool L2PF = false>
__global__ void __launch_bounds__(W * 32, 2)
    gemv_q5k_tiled_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xlimbs,
                          const float* __restrict__ xgsum, const float* __restrict__ xscale, float* y,
                          const float* res, uint32_t rows, uint32_t nb, float eps) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t C = W;  // consumers
    constexpr uint32_t R = kT2Rows;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + t2_ring_bytes<W, DEPTH, TPS>());
    uint64_t* xbar = bars + C * DEPTH;
    PairBoundary<W, R>* bnd = reinterpret_cast<PairBoundary<W, R>*>(xbar + 1);
    uint8_t* xs = reinterpret_cast<uint8_t*>(bnd + 1);  // staged x-pack when XS
    xs += (128u - (reinterpret_cast<uintptr_t>(xs) & 127u)) & 127u;

    if (threadIdx.x == 0) pdl_launch_dependents();

    const uint32_t cons = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t nquads = (rows + R - 1u) / R;
    const uint32_t nkc = nb / kT2Blocks;
    const uint32_t q0 = static_cast<uint32_t>(static_cast<uint64_t>(nquads) * blockIdx.x / gridDim.x);
    const uint32_t q1 = static_cast<uint32_t>(static_cast<uint64_t>(nquads) * (blockIdx.x + 1) / gridDim.x);
    const uint32_t T = (q1 - q0) * nkc;  // tiles of this CTA
    const uint32_t base = T / C, rem = T % C;
    const uint32_t len = base + (cons < rem ? 1u : 0u);
    const uint32_t chunk0 = cons * base + min(cons, rem);
    const uint8_t* src = w + (static_cast<size_t>(q0) * nkc + chunk0) * kT2TileBytes;  // this consumer's tiles
    constexpr uint32_t kSlot = TPS * kT2TileBytes;
    uint8_t* ring = smem + static_cast<size_t>(cons) * DEPTH * kSlot;
    uint64_t* full = bars + cons * DEPTH;
    const uint32_t ncopies = (len + TPS - 1u) / TPS;  // one bulk copy fills a slot with up to TPS tiles
    auto issue = [&](uint32_t k) {
        const uint32_t n = min(TPS, len - k * TPS);
        mbar_arrive_expect_tx(&full[k % DEPTH], n * kT2TileBytes);
        tma_load_1d(ring + (k % DEPTH) * kSlot, src + static_cast<size_t>(k) * kSlot, n * kT2TileBytes,
                    &full[k % DEPTH]);
    };

    if (lane == 0) {
        if constexpr (L2PF) {  // optionally ask L2 for the consumer's whole run
            const size_t bytes = static_cast<size_t>(len) * kT2TileBytes;
            for (size_t off = 0; off < bytes; off += kL2PrefetchPiece) {
                const size_t left = bytes - off;
                prefetch_l2(src + off, static_cast<uint32_t>(left < kL2PrefetchPiece ? left : kL2PrefetchPiece));
            }
        }
        for (uint32_t i = 0; i < DEPTH; ++i) mbar_init(&full[i], 1);
        if (XM == 1 && cons == 0) mbar_init(xbar, 1);
        fence_mbar_init();
        for (uint32_t k = 0; k < DEPTH && k < ncopies; ++k) issue(k);
    }
    if (threadIdx.x < 2 * C) bnd->pair[threadIdx.x] = -1;
    __syncthreads();

    pdl_wait();  // x-pack, y and res belong to the dependency chain
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
            inv = row_inv_rms(xf, nb, eps, blk, &inv_s, cons, lane, W);
        }
        t2_pack_x_f32(xf, nb, xs, reinterpret_cast<float*>(xs + lbytes), reinterpret_cast<float*>(xs + lbytes + nb * 32u),
                      cons, lane, W, XM == 3 ? xgsum : nullptr, inv);
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
        for (uint32_t off = threadIdx.x * 128u; off < lbytes; off += (W * 32u) * 128u) prefetch_l1(xlimbs + off);
        xl_base = xlimbs;
        xg2 = reinterpret_cast<const float2*>(xgsum);
        xsc = xscale;
    }
    const uint32_t hh = lane >> 4, s = (lane >> 2) & 3u, p = lane & 3u;
    const uint32_t rot_lo = (4u - 2u * p) & 31u, rot_hi = (3u - 2u * p) & 31u;
    const uint32_t c0 = s & 1u, c1 = c0 ^ 1u;  // bank-conflict-free order of the 16-byte halves
    const uint8_t* xlane = xl_base + (s * 4u + p) * 16u;
    const uint32_t slot0 = hh * kT2Blocks + s, slot1 = (hh + 2u) * kT2Blocks + s;  // block slots of rows hh, hh+2
    bool ok = true;
    if constexpr (XM == 1) {
        if (!mbar_wait_spin(xbar, 0, kFaultFullWait)) ok = false;
    }
    if constexpr (XM >= 2) __syncthreads();  // packed activations visible to every consumer

    double acc0 = 0.0, acc1 = 0.0;  // rows 4q + hh and 4q + hh + 2
    uint32_t issued = min(ncopies, DEPTH), waited = 0;  // slot copies issued / slot copies landed
    uint32_t quad = chunk0 / nkc, kc = chunk0 - quad * nkc;
    uint32_t kc_first = kc, nflush = 0;
    bool started = false;

    auto flush = [&](bool whole) {
        double v0 = acc0, v1 = acc1;
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) {
            v0 += __shfl_xor_sync(0xffffffffu, v0, o);
            v1 += __shfl_xor_sync(0xffffffffu, v1, o);
        }
        if ((lane & 15u) == 0) {
            const uint32_t row = R * (q0 + quad) + hh;
            if (whole) {
                if (ok && row < rows) y[row] = gemv_out(v0, res, row);
                if (ok && row + 2u < rows) y[row + 2u] = gemv_out(v1, res, row + 2u);
            } else {
                const uint32_t e = cons * 2u + (nflush == 0 ? 0u : 1u);
                bnd->v[e][hh] = v0;
                bnd->v[e][hh + 2u] = v1;
                if (hh == 0) bnd->pair[e] = static_cast<int>(quad);
            }
        }
        ++nflush;
        acc0 = 0.0;
        acc1 = 0.0;
    };

    for (uint32_t i = 0; i < len; ++i) {
        const uint32_t kcopy = i / TPS, j = i - kcopy * TPS, slot = kcopy % DEPTH;
        if (j == 0) {
            const bool landed =
                __all_sync(0xffffffffu, ok && mbar_wait_spin(&full[slot], (kcopy / DEPTH) & 1u, kFaultFullWait));
            if (!landed) ok = false;
            else waited = kcopy + 1u;
        }
        started = true;
        if (ok) {
            const uint32_t bcol = kc * kT2Blocks + s;
            const uint8_t* tb = ring + slot * kSlot + j * kT2TileBytes;
            const uint8_t* qs0 = tb + slot0 * 128u + p * 32u;
            const uint8_t* qs1 = tb + slot1 * 128u + p * 32u;
            const uint8_t* qh0 = tb + kT2QhOff + slot0 * 32u;
            const uint8_t* qh1 = tb + kT2QhOff + slot1 * 32u;
            const uint8_t* xq = xlane + static_cast<size_t>(kc) * (4u * NL) * 256u;
            int a0[NL], b0[NL], a1[NL], b1[NL];
#pragma unroll
            for (int k = 0; k < NL; ++k) a0[k] = b0[k] = a1[k] = b1[k] = 0;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const uint32_t c = half ? c1 : c0;
                const uint4 qa = *reinterpret_cast<const uint4*>(qs0 + 16u * c);
                const uint4 ha = *reinterpret_cast<const uint4*>(qh0 + 16u * c);
                const uint4 qb = *reinterpret_cast<const uint4*>(qs1 + 16u * c);
                const uint4 hb = *reinterpret_cast<const uint4*>(qh1 + 16u * c);
                uint32_t xl[8 * NL];
#pragma unroll
                for (int jj = 0; jj < 2 * NL; ++jj) {
                    const uint4 v = t2_load_quad<NL, XS>(xq + (2u * NL * c + jj) * 256u);
                    xl[4 * jj + 0] = v.x; xl[4 * jj + 1] = v.y; xl[4 * jj + 2] = v.z; xl[4 * jj + 3] = v.w;
                }
                q5_chunk_dot<NL>(qa, ha, qb, hb, xl, rot_lo, rot_hi, a0, b0, a1, b1);
            }
            const float2 X = XS ? xg2[bcol * 4u + p] : __ldg(xg2 + bcol * 4u + p);
            const float es = XS ? xsc[bcol] : __ldg(xsc + bcol);
            const uint8_t* m0 = tb + kT2MetaOff + slot0 * 20u;
            const uint8_t* m1 = tb + kT2MetaOff + slot1 * 20u;
            acc0 += q5_pair_scale<NL>(a0, b0, *reinterpret_cast<const uint32_t*>(m0),
                                      *reinterpret_cast<const uint32_t*>(m0 + 4u + 4u * p), es, X);
            acc1 += q5_pair_scale<NL>(a1, b1, *reinterpret_cast<const uint32_t*>(m1),
                                      *reinterpret_cast<const uint32_t*>(m1 + 4u + 4u * p), es, X);
        }
        // After the last tile of a slot every lane is done with it: refill it
        // with copy kcopy + DEPTH.
        if (j == TPS - 1u || i + 1u == len) {
            __syncwarp();
            if (ok && lane == 0 && kcopy + DEPTH < ncopies) {
                fence_proxy_async_smem();
                issue(kcopy + DEPTH);
                issued = kcopy + DEPTH + 1u;
            }
        }
        if (++kc == nkc) {  // quad complete
            flush(kc_first == 0);
            kc = 0;
            kc_first = 0;
            ++quad;
            started = false;
        }
    }
    if (started) flush(false);  // run ended inside a quad
    // Drain after a fault: copies still in flight must land before exit.
    if (!ok && lane == 0) {
        for (uint32_t k = waited; k < issued; ++k)
            if (!mbar_wait(&full[k % DEPTH], (k / DEPTH) & 1u, kFaultDrain)) break;
    }

    // Quads split between consumers: the first entry of every run of equal
    // quads sums its run in consumer order and writes the four rows.
    __syncthreads();
    if (threadIdx.x < 2u * C && ok) {
        const uint32_t e = threadIdx.x;
        const int pr = bnd->pair[e];
        if (pr >= 0) {
            // A consumer leaves its second slot empty only when its whole run
            // lies inside one quad, so the previous used slot is e-1 or e-2.
            int prev = e >= 1 ? bnd->pair[e - 1] : -1;
            if (prev == -1 && e >= 2) prev = bnd->pair[e - 2];
            if (prev != pr) {
                double v[R];
#pragma unroll
                for (uint32_t r = 0; r < R; ++r) v[r] = bnd->v[e][r];
                for (uint32_t q = e + 1u; q < 2u * C; ++q) {
                    const int pq = bnd->pair[q];
                    if (pq == -1) continue;
                    if (pq != pr) break;
#pragma unroll
                    for (uint32_t r = 0; r < R; ++r) v[r] += bnd->v[q][r];
                }
                const uint32_t row = R * (q0 + static_cast<uint32_t>(pr));
#pragma unroll
                for (uint32_t r = 0; r < R; ++r)
                    if (row + r < rows) y[row + r] = gemv_out(v[r], res, row + r);
            }
        }
    }
}

}  // namespace q38
