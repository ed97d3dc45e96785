// gemv_q5k.cuh -- Q5_K dequant-GEMV for sm_100a over the META/QH/QS SoA planes.
//
// Replaces the reference kernel q38_q5k_sm86_soa_gemv_vec
// (src/driver.cpp:3887-4138; host run_q5k_sm86_gemv_smoke :6800-7019) and its
// Q8_K variant q38_q5k_q8k_dp4a_gemv (:3660-3885).  Same mathematics:
//   y[r] = sum_b sum_g  d*sc_g * sum_j q_j x_j  -  dmin*m_g * sum_j x_j
// with q_j = low/high nibble of qs[(g/2)*32 + j] plus 16 * bit g of qh[j].
//
// B200 structure (not the reference's one-warp-per-row loop):
//  * persistent grid, one CTA per SM pair slot, each CTA owning a contiguous
//    range of row pairs (balanced to within one pair);
//  * one producer thread streams tiles of 4 rows x 4 super-blocks from the
//    three planes with 2-D TMA (cp.async.bulk.tensor, no multicast) into a
//    32-slot shared-memory ring guarded by mbarriers (bounded waits);
//  * 8 consumer warps decode in registers: lane = (row pair hh, super-block s,
//    pair of groups p); every lane handles 2 rows x 64 weights per tile, so
//    each activation word it loads serves two rows;
//  * dot products are exact dp4a integer sums against the x-pack limbs
//    (xpack.cuh); scales are applied once per 32-weight group;
//  * deterministic reduction with warp shuffles, no atomics;
//  * programmatic dependent launch: the weight stream starts before the
//    predecessor kernel has finished, only x and y wait for it.
#pragma once

#include "xpack.cuh"

namespace q38 {

constexpr int kTileRows = 4;         // rows per TMA tile
constexpr int kTileBlocks = 4;       // super-blocks per TMA tile
constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;
constexpr int kRingSlots = 32;

// Per-slot layout: QS [4][512] | QH [4][128] | META [4][80] (+ pad to 128 B).
constexpr uint32_t kSoaQsBytes = kTileRows * kTileBlocks * 128;   // 2048
constexpr uint32_t kSoaQhBytes = kTileRows * kTileBlocks * 32;    // 512
constexpr uint32_t kSoaMetaBytes = kTileRows * kTileBlocks * 20;  // 320
constexpr uint32_t kSoaSlotBytes = 2944;                          // 2880 rounded to 128
constexpr uint32_t kSoaTileBytes = kSoaQsBytes + kSoaQhBytes + kSoaMetaBytes;
constexpr size_t kSoaSmemBytes = static_cast<size_t>(kRingSlots) * kSoaSlotBytes + 2 * kRingSlots * 8 + 128;

struct Q5kSoaMaps {
    CUtensorMap meta4, qh4, qs4;  // 4-row boxes
    CUtensorMap meta2, qh2, qs2;  // 2-row boxes (odd row pair at the end of a CTA range)
};

// Decode the 4 weights of one qs/qh word pair into 5-bit bytes.
//   lo: group 2p  -> low nibbles,  high bit = bit 2p   of each qh byte
//   hi: group 2p+1-> high nibbles, high bit = bit 2p+1 of each qh byte
// Rotations move bit k of every byte to bit 4 at once (see the index proof in
// the kernel comment); 7 integer ops per 8 weights.
__device__ __forceinline__ void q5_decode(uint32_t qs, uint32_t qh, uint32_t rot_lo, uint32_t rot_hi,
                                          uint32_t& lo5, uint32_t& hi5) {
    lo5 = (qs & 0x0f0f0f0fu) | (rotl(qh, rot_lo) & 0x10101010u);
    hi5 = ((qs >> 4) & 0x0f0f0f0fu) | (rotl(qh, rot_hi) & 0x10101010u);
}

// Combine NL limb accumulators into the integer dot as a float.
template <int NL>
__device__ __forceinline__ float limb_combine(const int (&a)[NL]) {
    if constexpr (NL == 1) {
        return static_cast<float>(a[0]);
    } else {
        const int a01 = a[0] + (a[1] << 8);  // |a01| < 2^25, exact
        return fmaf(65536.0f, static_cast<float>(a[2]), static_cast<float>(a01));
    }
}

template <int NL>
__global__ void __launch_bounds__(kGemvThreads, 2)
    gemv_q5k_soa_kernel(const __grid_constant__ Q5kSoaMaps maps, const uint8_t* __restrict__ xlimbs,
                        const float* __restrict__ xgsum, const float* __restrict__ xscale,
                        float* __restrict__ y, uint32_t rows, uint32_t nb) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRingSlots * kSoaSlotBytes);
    uint64_t* empty = full + kRingSlots;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t npairs = (rows + 1u) >> 1;
    const uint32_t p0 = static_cast<uint32_t>(static_cast<uint64_t>(npairs) * blockIdx.x / gridDim.x);
    const uint32_t p1 = static_cast<uint32_t>(static_cast<uint64_t>(npairs) * (blockIdx.x + 1) / gridDim.x);
    const uint32_t row0 = 2u * p0;
    const uint32_t nrt = (p1 - p0 + 1u) >> 1;  // row tiles (last may hold one pair)
    const uint32_t nkc = nb / kTileBlocks;
    const bool last_half = ((p1 - p0) & 1u) != 0;  // final tile holds only 2 rows

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRingSlots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    // Tile order: groups of kConsumerWarps row tiles; inside a group the
    // k-chunk is the outer loop so every warp streams its own row tile in
    // parallel.  Tile t lands in slot t % kRingSlots.
    if (warp == kConsumerWarps) {
        if (lane == 0) {
            prefetch_tmap(&maps.qs4);
            prefetch_tmap(&maps.qh4);
            prefetch_tmap(&maps.meta4);
            uint32_t t = 0;
            bool ok = true;
            for (uint32_t g0 = 0; g0 < nrt && ok; g0 += kConsumerWarps) {
                const uint32_t gsize = min(static_cast<uint32_t>(kConsumerWarps), nrt - g0);
                for (uint32_t kc = 0; kc < nkc && ok; ++kc) {
                    for (uint32_t w = 0; w < gsize; ++w, ++t) {
                        const uint32_t slot = t % kRingSlots;
                        if (t >= kRingSlots) {
                            if (!mbar_wait(&empty[slot], ((t / kRingSlots) - 1u) & 1u, kFaultEmptyWait)) {
                                ok = false;
                                break;
                            }
                        }
                        const uint32_t rt = g0 + w;
                        const bool half = last_half && rt == nrt - 1u;
                        const int32_t r = static_cast<int32_t>(row0 + rt * kTileRows);
                        uint8_t* dst = ring + slot * kSoaSlotBytes;
                        const uint32_t bytes = half ? kSoaTileBytes / 2 : kSoaTileBytes;
                        mbar_arrive_expect_tx(&full[slot], bytes);
                        // inner coordinates in map elements: qs/qh as u64, meta as u32
                        tma_load_2d(dst, half ? &maps.qs2 : &maps.qs4, static_cast<int32_t>(kc * 64), r, &full[slot]);
                        tma_load_2d(dst + kSoaQsBytes, half ? &maps.qh2 : &maps.qh4, static_cast<int32_t>(kc * 16), r,
                                    &full[slot]);
                        tma_load_2d(dst + kSoaQsBytes + kSoaQhBytes, half ? &maps.meta2 : &maps.meta4,
                                    static_cast<int32_t>(kc * 20), r, &full[slot]);
                    }
                }
            }
            pdl_launch_dependents();
            // Drain: every issued copy must land before the CTA may exit.
            const uint32_t issued = t;
            const uint32_t first = issued > kRingSlots ? issued - kRingSlots : 0u;
            for (uint32_t u = first; u < issued; ++u) {
                if (!mbar_wait(&full[u % kRingSlots], (u / kRingSlots) & 1u, kFaultDrain)) break;
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    pdl_wait();  // x-pack and y belong to the dependency chain
    const uint32_t hh = lane >> 4, s = (lane >> 2) & 3u, p = lane & 3u;
    const uint32_t rot_lo = (4u - 2u * p) & 31u, rot_hi = (3u - 2u * p) & 31u;
    const uint32_t swap = s & 1u;  // bank-conflict-free order of the two 16-B qs halves

    uint32_t t = 0;
    bool ok = true;
    for (uint32_t g0 = 0; g0 < nrt; g0 += kConsumerWarps) {
        const uint32_t gsize = min(static_cast<uint32_t>(kConsumerWarps), nrt - g0);
        const uint32_t rt = g0 + warp;
        if (warp < gsize) {
            float acc0 = 0.0f, acc1 = 0.0f;
            for (uint32_t kc = 0; kc < nkc; ++kc) {
                const uint32_t tt = t + kc * gsize + warp;
                const uint32_t slot = tt % kRingSlots;
                if (ok && !mbar_wait(&full[slot], (tt / kRingSlots) & 1u, kFaultFullWait)) ok = false;
                if (ok) {
                    const uint8_t* base = ring + slot * kSoaSlotBytes;
                    const uint32_t bcol = kc * kTileBlocks + s;
                    // activation limbs for (bcol, p): 8 words x 2 groups x NL
                    const uint4* xr = reinterpret_cast<const uint4*>(
                        xlimbs + (static_cast<size_t>(bcol) * 4u + p) * xpack_record_bytes(NL));
                    uint32_t xl[16 * NL];
#pragma unroll
                    for (int k = 0; k < 4 * NL; ++k) {
                        const uint4 v = __ldg(xr + k);
                        xl[4 * k + 0] = v.x;
                        xl[4 * k + 1] = v.y;
                        xl[4 * k + 2] = v.z;
                        xl[4 * k + 3] = v.w;
                    }
                    const float2 X = __ldg(reinterpret_cast<const float2*>(xgsum) + bcol * 4u + p);
                    const float es = __ldg(xscale + bcol);
#pragma unroll
                    for (int rr = 0; rr < 2; ++rr) {
                        const uint32_t row = 2u * hh + rr;
                        const uint8_t* qsp = base + row * 512u + s * 128u + p * 32u;
                        const uint8_t* qhp = base + kSoaQsBytes + row * 128u + s * 32u;
                        const uint8_t* mp = base + kSoaQsBytes + kSoaQhBytes + row * 80u + s * 20u;
                        const uint4 qa = *reinterpret_cast<const uint4*>(qsp + 16u * swap);
                        const uint4 qb = *reinterpret_cast<const uint4*>(qsp + 16u * (1u - swap));
                        const uint4 ha = *reinterpret_cast<const uint4*>(qhp);
                        const uint4 hb = *reinterpret_cast<const uint4*>(qhp + 16u);
                        const uint32_t qw[8] = {swap ? qb.x : qa.x, swap ? qb.y : qa.y, swap ? qb.z : qa.z,
                                                swap ? qb.w : qa.w, swap ? qa.x : qb.x, swap ? qa.y : qb.y,
                                                swap ? qa.z : qb.z, swap ? qa.w : qb.w};
                        const uint32_t hw[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
                        int aa[NL], ab[NL];
#pragma unroll
                        for (int k = 0; k < NL; ++k) aa[k] = ab[k] = 0;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            uint32_t lo5, hi5;
                            q5_decode(qw[i], hw[i], rot_lo, rot_hi, lo5, hi5);
#pragma unroll
                            for (int k = 0; k < NL; ++k) {
                                aa[k] = dp4a(lo5, xl[(i * 2 + 0) * NL + k], aa[k]);
                                ab[k] = dp4a(hi5, xl[(i * 2 + 1) * NL + k], ab[k]);
                            }
                        }
                        const uint32_t dm = *reinterpret_cast<const uint32_t*>(mp);
                        const uint32_t scm = *reinterpret_cast<const uint32_t*>(mp + 4u + 4u * p);
                        const float dd = half_bits_to_float(dm) * es;
                        const float dmin = half_bits_to_float(dm >> 16);
                        float a = 0.0f;
                        a = fmaf(dd * static_cast<float>(scm & 0xffu), limb_combine<NL>(aa), a);
                        a = fmaf(-dmin * static_cast<float>((scm >> 8) & 0xffu), X.x, a);
                        a = fmaf(dd * static_cast<float>((scm >> 16) & 0xffu), limb_combine<NL>(ab), a);
                        a = fmaf(-dmin * static_cast<float>(scm >> 24), X.y, a);
                        if (rr == 0) acc0 += a; else acc1 += a;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
            // reduce over (s, p): lanes differing in bits 0..3
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) {
                acc0 += __shfl_xor_sync(0xffffffffu, acc0, o);
                acc1 += __shfl_xor_sync(0xffffffffu, acc1, o);
            }
            if ((lane & 15u) == 0 && ok) {
                const uint32_t r = row0 + rt * kTileRows + 2u * hh;
                const uint32_t rend = min(2u * p1, rows);
                if (r < rend) y[r] = acc0;
                if (r + 1u < rend) y[r + 1u] = acc1;
            }
        }
        t += nkc * gsize;
    }
}

}  // namespace q38
