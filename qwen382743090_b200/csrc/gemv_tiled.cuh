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
//  * 16 consumers (half-warps) per CTA each own a contiguous run of the CTA's
//    tiles.  In the prologue each consumer asks L2 to prefetch its whole run in
//    2 KB pieces (cp.async.bulk.prefetch.L2) and the CTA triggers the next grid
//    (PDL), so the DRAM stream starts at full width before any dependency
//    resolves; then each consumer keeps 2 two-tile 1-D bulk TMA copies
//    (cp.async.bulk, no multicast) in flight in its private smem ring, one
//    barrier wait per copy;
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
constexpr uint32_t kT2Warps = 8;                      // warps per CTA
constexpr uint32_t kT2Consumers = 2 * kT2Warps;       // half-warps, each an independent consumer
constexpr uint32_t kT2Threads = kT2Warps * 32;
constexpr uint32_t kT2TilesPerCopy = 2;               // tiles per bulk copy (one barrier wait per copy)
constexpr uint32_t kT2Depth = 2;                      // private ring slots (copies) per consumer
constexpr uint32_t kT2CopyBytes = kT2TilesPerCopy * kT2TileBytes;  // 2880
constexpr uint32_t kL2PrefetchPiece = 2048;

struct T2Boundary {
    int pair[kT2Consumers * 2];
    double v[kT2Consumers * 2][2];
};
constexpr size_t kT2RingBytes = static_cast<size_t>(kT2Consumers) * kT2Depth * kT2CopyBytes;  // 92160
constexpr size_t kT2SmemBytes = kT2RingBytes + kT2Consumers * kT2Depth * 8 + sizeof(T2Boundary) + 64;

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Integer dot of one row's 64 weights (super-block s, group pair p) with the
// lane's activation limbs: aa = group 2p, ab = group 2p+1, one sum per limb.
template <int NL>
__device__ __forceinline__ void q5_pair_dot(const uint8_t* qsp, const uint8_t* qhp, uint32_t c0, uint32_t c1,
                                            uint32_t rot_lo, uint32_t rot_hi, const uint32_t (&xl)[16 * NL],
                                            int (&aa)[NL], int (&ab)[NL]) {
    const uint4 qa = *reinterpret_cast<const uint4*>(qsp + 16u * c0);
    const uint4 qb = *reinterpret_cast<const uint4*>(qsp + 16u * c1);
    const uint4 ha = *reinterpret_cast<const uint4*>(qhp + 16u * c0);
    const uint4 hb = *reinterpret_cast<const uint4*>(qhp + 16u * c1);
    const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const uint32_t hw[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
#pragma unroll
    for (int k = 0; k < NL; ++k) aa[k] = ab[k] = 0;
#pragma unroll
    for (int i8 = 0; i8 < 8; ++i8) {
        uint32_t lo5, hi5;
        q5_decode(qw[i8], hw[i8], rot_lo, rot_hi, lo5, hi5);
#pragma unroll
        for (int k = 0; k < NL; ++k) {
            aa[k] = dp4a(lo5, xl[(i8 * 2 + 0) * NL + k], aa[k]);
            ab[k] = dp4a(hi5, xl[(i8 * 2 + 1) * NL + k], ab[k]);
        }
    }
}

// Scale the two group dots of one (row, super-block, pair): the 6-bit group
// scales multiply the integer limb sums exactly (|sc*a| < 2^24 per limb), one
// conversion per limb, then d*es and the dmin*m*sum(x) term in fp32.
template <int NL>
__device__ __forceinline__ float q5_pair_scale(const int (&aa)[NL], const int (&ab)[NL], uint32_t dm, uint32_t scm,
                                               float es, float2 X) {
    const int sca = static_cast<int>(scm & 0xffu), scb = static_cast<int>((scm >> 16) & 0xffu);
    float f;
    if constexpr (NL == 1) {
        f = static_cast<float>(sca * aa[0] + scb * ab[0]);
    } else {
        const float t0 = static_cast<float>(sca * aa[0] + scb * ab[0]);
        const float t1 = static_cast<float>(sca * aa[1] + scb * ab[1]);
        const float t2 = static_cast<float>(sca * aa[2] + scb * ab[2]);
        f = fmaf(65536.0f, t2, fmaf(256.0f, t1, t0));
    }
    const float2 dmf = __half22float2(*reinterpret_cast<const __half2*>(&dm));
    const float mna = byte_to_float(scm, 0x7541u), mnb = byte_to_float(scm, 0x7543u);
    return fmaf(dmf.x * es, f, -dmf.y * fmaf(mna, X.x, mnb * X.y));
}

template <int NL, int MINB>
__global__ void __launch_bounds__(kT2Threads, MINB)
    gemv_q5k_tiled_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xlimbs,
                          const float* __restrict__ xgsum, const float* __restrict__ xscale, float* __restrict__ y,
                          uint32_t rows, uint32_t nb) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kT2RingBytes);
    T2Boundary* bnd = reinterpret_cast<T2Boundary*>(bars + kT2Consumers * kT2Depth);

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
    uint8_t* ring = smem + static_cast<size_t>(cons) * kT2Depth * kT2CopyBytes;
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
        fence_mbar_init();
        for (uint32_t c = 0; c < kT2Depth && c * kT2TilesPerCopy < len; ++c) {
            const uint32_t n = min(kT2TilesPerCopy, len - c * kT2TilesPerCopy) * kT2TileBytes;
            mbar_arrive_expect_tx(&full[c], n);
            tma_load_1d(ring + c * kT2CopyBytes, src + static_cast<size_t>(c) * kT2CopyBytes, n, &full[c]);
        }
    }
    if (threadIdx.x < 2 * C) bnd->pair[threadIdx.x] = -1;
    __syncthreads();

    pdl_wait();  // x-pack and y belong to the dependency chain
    // Every consumer reads activation limbs of several K chunks; pull the whole
    // x-pack of this row into L1 at once so no tile waits on an L2 round trip.
    {
        const uint32_t lbytes = nb * 4u * xpack_record_bytes(NL);
        for (uint32_t off = threadIdx.x * 128u; off < lbytes; off += kT2Threads * 128u) prefetch_l1(xlimbs + off);
        if (threadIdx.x < (nb * 32u + 127u) / 128u) prefetch_l1(reinterpret_cast<const uint8_t*>(xgsum) + threadIdx.x * 128u);
        if (threadIdx.x < (nb * 4u + 127u) / 128u) prefetch_l1(reinterpret_cast<const uint8_t*>(xscale) + threadIdx.x * 128u);
    }
    const uint32_t s = (lane >> 2) & 3u, p = lane & 3u;
    const uint32_t rot_lo = (4u - 2u * p) & 31u, rot_hi = (3u - 2u * p) & 31u;
    const uint32_t c0 = s & 1u, c1 = c0 ^ 1u;  // bank-conflict-free order of the 16-byte halves
    const uint8_t* xlane = xlimbs + (s * 4u + p) * 16u;
    const float2* xg2 = reinterpret_cast<const float2*>(xgsum);

    float acc0 = 0.0f, acc1 = 0.0f;
    const uint32_t ncopy = (len + kT2TilesPerCopy - 1u) / kT2TilesPerCopy;
    uint32_t issued = min(ncopy, kT2Depth), waited = 0;  // copies issued / copies consumed by this consumer
    uint32_t pair = chunk0 / nkc, kc = chunk0 - pair * nkc;
    uint32_t kc_first = kc, nflush = 0;
    bool ok = true, started = false;

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
                if (ok && row < rows) y[row] = static_cast<float>(v0);
                if (ok && row + 1u < rows) y[row + 1u] = static_cast<float>(v1);
            } else {
                const uint32_t e = cons * 2u + (nflush == 0 ? 0u : 1u);
                bnd->v[e][0] = v0;
                bnd->v[e][1] = v1;
                bnd->pair[e] = static_cast<int>(pair);
            }
        }
        ++nflush;
        acc0 = 0.0f;
        acc1 = 0.0f;
    };

    // warp-uniform trip count (the other half-warp may own one copy more)
    const uint32_t len_w = base + (2u * warp < rem ? 1u : 0u);
    const uint32_t ncopy_w = (len_w + kT2TilesPerCopy - 1u) / kT2TilesPerCopy;
    for (uint32_t ci = 0; ci < ncopy_w; ++ci) {
        if (ci < ncopy) {
            const uint32_t slot = ci % kT2Depth;
            const bool landed = ok && mbar_wait_spin(&full[slot], (ci / kT2Depth) & 1u, kFaultFullWait);
            if (!landed) ok = false;
            const uint32_t nt = min(kT2TilesPerCopy, len - ci * kT2TilesPerCopy);
            for (uint32_t u = 0; u < kT2TilesPerCopy; ++u) {
                if (u >= nt) break;
                started = true;
                if (ok) {
                    const uint32_t bcol = kc * kT2Blocks + s;
                    uint32_t xl[16 * NL];  // [0, 8NL): half c0, [8NL, 16NL): half c1
                    const uint8_t* xq = xlane + static_cast<size_t>(kc) * (4u * NL) * 256u;
#pragma unroll
                    for (int j = 0; j < 2 * NL; ++j) {
                        const uint4 va = __ldg(reinterpret_cast<const uint4*>(xq + (2u * NL * c0 + j) * 256u));
                        const uint4 vb = __ldg(reinterpret_cast<const uint4*>(xq + (2u * NL * c1 + j) * 256u));
                        xl[4 * j + 0] = va.x; xl[4 * j + 1] = va.y; xl[4 * j + 2] = va.z; xl[4 * j + 3] = va.w;
                        xl[8 * NL + 4 * j + 0] = vb.x; xl[8 * NL + 4 * j + 1] = vb.y;
                        xl[8 * NL + 4 * j + 2] = vb.z; xl[8 * NL + 4 * j + 3] = vb.w;
                    }
                    const float2 X = __ldg(xg2 + bcol * 4u + p);
                    const float es = __ldg(xscale + bcol);
                    const uint8_t* tb = ring + slot * kT2CopyBytes + u * kT2TileBytes;
                    const uint8_t* qs0 = tb + s * 128u + p * 32u;
                    const uint8_t* qh0 = tb + kT2QhOff + s * 32u;
                    const uint8_t* m0 = tb + kT2MetaOff + s * 20u;
                    const uint32_t dm0 = *reinterpret_cast<const uint32_t*>(m0);
                    const uint32_t sm0 = *reinterpret_cast<const uint32_t*>(m0 + 4u + 4u * p);
                    const uint32_t dm1 = *reinterpret_cast<const uint32_t*>(m0 + 80u);
                    const uint32_t sm1 = *reinterpret_cast<const uint32_t*>(m0 + 84u + 4u * p);
                    int a0[NL], b0[NL], a1[NL], b1[NL];
                    q5_pair_dot<NL>(qs0, qh0, c0, c1, rot_lo, rot_hi, xl, a0, b0);
                    q5_pair_dot<NL>(qs0 + 512u, qh0 + 128u, c0, c1, rot_lo, rot_hi, xl, a1, b1);
                    acc0 += q5_pair_scale<NL>(a0, b0, dm0, sm0, es, X);
                    acc1 += q5_pair_scale<NL>(a1, b1, dm1, sm1, es, X);
                }
                if (++kc == nkc) {  // row pair complete
                    flush(kc_first == 0);
                    kc = 0;
                    kc_first = 0;
                    ++pair;
                    started = false;
                }
            }
            // Every lane has consumed the slot: refill it with copy ci + depth.
            __syncwarp(hmask);
            const uint32_t nx = ci + kT2Depth;
            if (ok && l16 == 0 && nx < ncopy) {
                const uint32_t n = min(kT2TilesPerCopy, len - nx * kT2TilesPerCopy) * kT2TileBytes;
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&full[slot], n);
                tma_load_1d(ring + slot * kT2CopyBytes, src + static_cast<size_t>(nx) * kT2CopyBytes, n, &full[slot]);
                issued = nx + 1u;
            }
            if (landed) waited = ci + 1u;
        }
    }
    if (started) flush(false);  // run ended inside a row pair
    // Drain after a fault: copies still in flight must land before exit.
    if (!ok && l16 == 0) {
        for (uint32_t c = waited; c < issued; ++c)
            if (!mbar_wait(&full[c % kT2Depth], (c / kT2Depth) & 1u, kFaultDrain)) break;
    }

    // Row pairs split between consumers: the first entry of every run of equal
    // pairs sums its run in consumer order and writes the two rows.
    __syncthreads();
    if (threadIdx.x < 2u * C && ok) {
        const uint32_t e = threadIdx.x;
        const int pr = bnd->pair[e];
        if (pr >= 0) {
            int prev = -1;
            for (int q = static_cast<int>(e) - 1; q >= 0; --q) {
                if (bnd->pair[q] != -1) {
                    prev = bnd->pair[q];
                    break;
                }
            }
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
                if (row < rows) y[row] = static_cast<float>(v0);
                if (row + 1u < rows) y[row + 1u] = static_cast<float>(v1);
            }
        }
    }
}

}  // namespace q38
