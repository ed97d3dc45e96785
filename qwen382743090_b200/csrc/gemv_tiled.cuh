// gemv_tiled.cuh -- Q5_K GEMV over the B200 tiled execution layout (Q38PACK
// layout 2).  Same mathematics as the reference's q38_q5k_sm86_soa_gemv_vec
// (src/driver.cpp:3887-4138) and q38_q5k_q8k_dp4a_gemv (:3660-3885).
//
// Layout 2 (Q5_K).  Rows are grouped in pairs and K in chunks of 4
// super-blocks; each (row pair, chunk) is one contiguous 1440-byte tile
//     QS   [2 rows][4 blocks][128]   at    0
//     QH   [2 rows][4 blocks][32]    at 1024
//     META [2 rows][4 blocks][20]    at 1280   (d, dmin, 8 x {scale, min})
// stored pair-major: tile (pair j, chunk c) at byte (j * nb/4 + c) * 1440.
// The bytes of every block are those of the SoA planes of layout 1, so the
// decoded weights are unchanged; only their order differs.  A CTA that owns a
// contiguous range of row pairs therefore reads one contiguous byte range.
//
// Kernel structure (sm_100a):
//  * 32 consumers (half-warps of 16 warps) per CTA each own a contiguous run of the CTA's
//    tiles.  In the prologue each consumer asks L2 to prefetch its whole run in
//    2 KB pieces (cp.async.bulk.prefetch.L2) and the CTA triggers the next grid
//    (PDL), so the DRAM stream starts at full width before any dependency
//    resolves; then each consumer keeps 2 single-tile 1-D bulk TMA copies
//    (cp.async.bulk, no multicast) in flight in its private smem ring;
//  * after the dependency resolves the CTA copies the whole x-pack into shared
//    memory with one bulk copy when it fits (else lanes read it through L1);
//  * a
//    lane is (super-block s, group pair p) and decodes 2 rows x 64 weights per
//    tile in registers, so every activation word it loads serves both rows;
//    dot products are dp4a against the x-pack limbs (xpack.cuh) and the 6-bit
//    group scales multiply the integer sums before any conversion;
//  * a lane accumulates in fp32 while its consumer stays on one row pair; the
//    16 lanes reduce in fp64 with shuffles, and row pairs split between
//    consumers are summed afterwards in consumer order (deterministic);
//  * only x, y and the x-dependent work wait for the predecessor grid.
#pragma once

#include "gemv_q5k.cuh"

namespace q38 {

constexpr uint32_t kT2Rows = 2;
constexpr uint32_t kT2Blocks = 4;
constexpr uint32_t kT2TileBytes = kT2Rows * kT2Blocks * 180;  // 1440
constexpr uint32_t kT2QhOff = kT2Rows * kT2Blocks * 128;      // 1024
constexpr uint32_t kT2MetaOff = kT2QhOff + kT2Rows * kT2Blocks * 32;  // 1280
constexpr uint32_t kT2Warps = 16;                     // warps per CTA
constexpr uint32_t kT2Consumers = 2 * kT2Warps;       // half-warps, each an independent consumer
constexpr uint32_t kT2Threads = kT2Warps * 32;
constexpr uint32_t kT2Depth = 2;                      // private ring slots per consumer (one tile each)
constexpr uint32_t kL2PrefetchPiece = 2048;
// Activations are staged in shared memory when they fit next to the ring and
// still leave room for the next kernel's CTA (PDL co-residency).
constexpr size_t kT2SmemBudget = 112u * 1024u;

struct T2Boundary {
    int pair[kT2Consumers * 2];
    double v[kT2Consumers * 2][2];
};
constexpr size_t kT2RingBytes = static_cast<size_t>(kT2Consumers) * kT2Depth * kT2TileBytes;  // 92160
constexpr size_t kT2FixedBytes = kT2RingBytes + kT2Consumers * kT2Depth * 8 + 8 + sizeof(T2Boundary) + 256;  // +256: 128-B alignment of the x region

// Bytes of the activation x-pack for one row of nb super-blocks.
__host__ __device__ constexpr uint32_t t2_xbytes(uint32_t nb, int nl) {
    return static_cast<uint32_t>(xpack_row_limb_bytes(nl, nb)) + nb * 32u + xpack_nb4(nb) * 4u;
}
__host__ __device__ constexpr size_t t2_smem_bytes(uint32_t nb, int nl, bool xsmem) {
    return kT2FixedBytes + (xsmem ? t2_xbytes(nb, nl) : 0u);
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
// limbs combine exactly in fp64, then d*es and the dmin*m*sum(x) term.
template <int NL>
__device__ __forceinline__ double q5_pair_scale(const int (&aa)[NL], const int (&ab)[NL], uint32_t dm, uint32_t scm,
                                                float es, float2 X) {
    const int sca = static_cast<int>(scm & 0xffu), scb = static_cast<int>((scm >> 16) & 0xffu);
    int t[NL];
#pragma unroll
    for (int k = 0; k < NL; ++k) t[k] = sca * aa[k] + scb * ab[k];
    const float2 dmf = __half22float2(*reinterpret_cast<const __half2*>(&dm));
    const double mna = static_cast<double>((scm >> 8) & 0xffu), mnb = static_cast<double>(scm >> 24);
    return __fma_rn(static_cast<double>(dmf.x * es), limb_value<NL>(t),
                    -static_cast<double>(dmf.y) *
                        __fma_rn(mna, static_cast<double>(X.x), mnb * static_cast<double>(X.y)));
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
// x-pack layout in shared memory, one warp per super-block.
__device__ __forceinline__ void t2_pack_x_f32(const float* __restrict__ x, uint32_t nb, uint8_t* xs, float* gsum,
                                              float* scale, uint32_t warp, uint32_t lane, uint32_t nwarps) {
    for (uint32_t b = warp; b < nb; b += nwarps) {
        const float4 v0 = __ldg(reinterpret_cast<const float4*>(x + b * 256u + lane * 8u));
        const float4 v1 = __ldg(reinterpret_cast<const float4*>(x + b * 256u + lane * 8u + 4u));
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        pack_block_warp<3>(v, b, lane, xs, gsum, scale);
    }
}

// XM selects where the activations come from: 0 = x-pack read through L1,
// 1 = x-pack copied into shared memory, 2 = f32 x packed into shared memory by
// this CTA (xlimbs then points at the f32 vector; NL must be 3).  With res
// non-null the kernel writes y = W x + res (y may equal res).
template <int NL, int XM>
__global__ void __launch_bounds__(kT2Threads, 2)
    gemv_q5k_tiled_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xlimbs,
                          const float* __restrict__ xgsum, const float* __restrict__ xscale, float* y,
                          const float* res, uint32_t rows, uint32_t nb) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kT2RingBytes);
    uint64_t* xbar = bars + kT2Consumers * kT2Depth;
    T2Boundary* bnd = reinterpret_cast<T2Boundary*>(xbar + 1);
    uint8_t* xs = reinterpret_cast<uint8_t*>(bnd + 1);  // staged x-pack when XS
    xs += (128u - (reinterpret_cast<uintptr_t>(xs) & 127u)) & 127u;

    if (threadIdx.x == 0) pdl_launch_dependents();

    constexpr uint32_t C = kT2Consumers;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t h = lane >> 4, cons = 2u * warp + h, l16 = lane & 15u;
    const uint32_t hmask = h ? 0xffff0000u : 0x0000ffffu;
    const uint32_t npairs = (rows + 1u) >> 1;
    const uint32_t nkc = nb / kT2Blocks;
    const uint32_t p0 = static_cast<uint32_t>(static_cast<uint64_t>(npairs) * blockIdx.x / gridDim.x);
    const uint32_t p1 = static_cast<uint32_t>(static_cast<uint64_t>(npairs) * (blockIdx.x + 1) / gridDim.x);
    const uint32_t T = (p1 - p0) * nkc;  // tiles of this CTA
    const uint32_t base = T / C, rem = T % C;
    const uint32_t len = base + (cons < rem ? 1u : 0u);
    const uint32_t chunk0 = cons * base + min(cons, rem);
    const uint8_t* src = w + (static_cast<size_t>(p0) * nkc + chunk0) * kT2TileBytes;  // this consumer's tiles
    uint8_t* ring = smem + static_cast<size_t>(cons) * kT2Depth * kT2TileBytes;
    uint64_t* full = bars + cons * kT2Depth;

    // Each consumer streams its own contiguous run: ask L2 for all of it now,
    // then keep kT2Depth single-tile bulk copies in flight.
    if (l16 == 0) {
        const size_t bytes = static_cast<size_t>(len) * kT2TileBytes;
        for (size_t off = 0; off < bytes; off += kL2PrefetchPiece) {
            const size_t left = bytes - off;
            prefetch_l2(src + off, static_cast<uint32_t>(left < kL2PrefetchPiece ? left : kL2PrefetchPiece));
        }
        for (uint32_t i = 0; i < kT2Depth; ++i) mbar_init(&full[i], 1);
        if (XM == 1 && cons == 0) mbar_init(xbar, 1);
        fence_mbar_init();
        for (uint32_t i = 0; i < kT2Depth && i < len; ++i) {
            mbar_arrive_expect_tx(&full[i], kT2TileBytes);
            tma_load_1d(ring + i * kT2TileBytes, src + static_cast<size_t>(i) * kT2TileBytes, kT2TileBytes, &full[i]);
        }
    }
    if (threadIdx.x < 2 * C) bnd->pair[threadIdx.x] = -1;
    __syncthreads();

    pdl_wait();  // x-pack and y belong to the dependency chain
    constexpr bool XS = XM != 0;
    const uint32_t lbytes = static_cast<uint32_t>(xpack_row_limb_bytes(NL, nb));
    const uint8_t* xl_base;
    const float2* xg2;
    const float* xsc;
    if constexpr (XM == 2) {
        static_assert(NL == 3, "f32 activations pack into three limbs");
        t2_pack_x_f32(reinterpret_cast<const float*>(xlimbs), nb, xs, reinterpret_cast<float*>(xs + lbytes),
                      reinterpret_cast<float*>(xs + lbytes + nb * 32u), warp, lane, kT2Warps);
        xl_base = xs;
        xg2 = reinterpret_cast<const float2*>(xs + lbytes);
        xsc = reinterpret_cast<const float*>(xs + lbytes + nb * 32u);
    } else if constexpr (XM == 1) {
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(xbar, lbytes + nb * 36u);
            tma_load_1d(xs, xlimbs, lbytes, xbar);
            tma_load_1d(xs + lbytes, xgsum, nb * 32u, xbar);
            tma_load_1d(xs + lbytes + nb * 32u, xscale, nb * 4u, xbar);
        }
        xl_base = xs;
        xg2 = reinterpret_cast<const float2*>(xs + lbytes);
        xsc = reinterpret_cast<const float*>(xs + lbytes + nb * 32u);
    } else {
        for (uint32_t off = threadIdx.x * 128u; off < lbytes; off += kT2Threads * 128u) prefetch_l1(xlimbs + off);
        xl_base = xlimbs;
        xg2 = reinterpret_cast<const float2*>(xgsum);
        xsc = xscale;
    }
    const uint32_t s = (lane >> 2) & 3u, p = lane & 3u;
    const uint32_t rot_lo = (4u - 2u * p) & 31u, rot_hi = (3u - 2u * p) & 31u;
    const uint32_t c0 = s & 1u, c1 = c0 ^ 1u;  // bank-conflict-free order of the 16-byte halves
    const uint8_t* xlane = xl_base + (s * 4u + p) * 16u;
    bool ok = true;
    if constexpr (XM == 1) {
        if (!mbar_wait_spin(xbar, 0, kFaultFullWait)) ok = false;
    }
    if constexpr (XM == 2) __syncthreads();  // packed activations visible to every consumer

    double acc0 = 0.0, acc1 = 0.0;
    uint32_t issued = min(len, kT2Depth), waited = 0;  // tiles copied / tiles consumed by this consumer
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

    // warp-uniform trip count (the other half-warp may own one tile more)
    const uint32_t len_w = base + (2u * warp < rem ? 1u : 0u);
    for (uint32_t i = 0; i < len_w; ++i) {
        if (i < len) {
            const uint32_t slot = i % kT2Depth;
            const bool landed = ok && mbar_wait_spin(&full[slot], (i / kT2Depth) & 1u, kFaultFullWait);
            if (!landed) ok = false;
            started = true;
            if (ok) {
                const uint32_t bcol = kc * kT2Blocks + s;
                const uint8_t* tb = ring + slot * kT2TileBytes;
                const uint8_t* qsp = tb + s * 128u + p * 32u;
                const uint8_t* qhp = tb + kT2QhOff + s * 32u;
                const uint8_t* mp = tb + kT2MetaOff + s * 20u;
                const uint8_t* xq = xlane + static_cast<size_t>(kc) * (4u * NL) * 256u;
                int a0[NL], b0[NL], a1[NL], b1[NL];
#pragma unroll
                for (int k = 0; k < NL; ++k) a0[k] = b0[k] = a1[k] = b1[k] = 0;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const uint32_t c = half ? c1 : c0;
                    const uint4 q0 = *reinterpret_cast<const uint4*>(qsp + 16u * c);
                    const uint4 hq0 = *reinterpret_cast<const uint4*>(qhp + 16u * c);
                    const uint4 q1 = *reinterpret_cast<const uint4*>(qsp + 512u + 16u * c);
                    const uint4 hq1 = *reinterpret_cast<const uint4*>(qhp + 128u + 16u * c);
                    uint32_t xl[8 * NL];
#pragma unroll
                    for (int j = 0; j < 2 * NL; ++j) {
                        const uint4 v = t2_load_quad<NL, XS>(xq + (2u * NL * c + j) * 256u);
                        xl[4 * j + 0] = v.x; xl[4 * j + 1] = v.y; xl[4 * j + 2] = v.z; xl[4 * j + 3] = v.w;
                    }
                    q5_chunk_dot<NL>(q0, hq0, q1, hq1, xl, rot_lo, rot_hi, a0, b0, a1, b1);
                }
                const float2 X = XS ? xg2[bcol * 4u + p] : __ldg(xg2 + bcol * 4u + p);
                const float es = XS ? xsc[bcol] : __ldg(xsc + bcol);
                const uint32_t dm0 = *reinterpret_cast<const uint32_t*>(mp);
                const uint32_t sm0 = *reinterpret_cast<const uint32_t*>(mp + 4u + 4u * p);
                const uint32_t dm1 = *reinterpret_cast<const uint32_t*>(mp + 80u);
                const uint32_t sm1 = *reinterpret_cast<const uint32_t*>(mp + 84u + 4u * p);
                acc0 += q5_pair_scale<NL>(a0, b0, dm0, sm0, es, X);
                acc1 += q5_pair_scale<NL>(a1, b1, dm1, sm1, es, X);
            }
            // Every lane has consumed the slot: refill it with tile i + depth.
            __syncwarp(hmask);
            if (ok && l16 == 0 && i + kT2Depth < len) {
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&full[slot], kT2TileBytes);
                tma_load_1d(ring + slot * kT2TileBytes, src + static_cast<size_t>(i + kT2Depth) * kT2TileBytes,
                            kT2TileBytes, &full[slot]);
                issued = i + kT2Depth + 1u;
            }
            if (landed) waited = i + 1u;
            if (++kc == nkc) {  // row pair complete
                flush(kc_first == 0);
                kc = 0;
                kc_first = 0;
                ++pair;
                started = false;
            }
        }
    }
    if (started) flush(false);  // run ended inside a row pair
    // Drain after a fault: copies still in flight must land before exit.
    if (!ok && l16 == 0) {
        for (uint32_t i = waited; i < issued; ++i)
            if (!mbar_wait(&full[i % kT2Depth], (i / kT2Depth) & 1u, kFaultDrain)) break;
    }

    // Row pairs split between consumers: the first entry of every run of equal
    // pairs sums its run in consumer order and writes the two rows.
    __syncthreads();
    if (threadIdx.x < 2u * C && ok) {
        const uint32_t e = threadIdx.x;
        const int pr = bnd->pair[e];
        if (pr >= 0) {
            // A consumer leaves its second slot empty only when its whole run
            // lies inside one row pair, so the previous used slot is e-1 or e-2.
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
