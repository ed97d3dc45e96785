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
//  * each lane accumulates its (row, super-block, pair) terms in fp64 and the
//    16 lanes of a row reduce with fp64 warp shuffles: deterministic, no
//    atomics, and no long fp32 accumulation chain;
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

// Per-lane partial sums of one CTA's boundary row tiles, combined after all
// consumer warps finish (fixed order -> deterministic).
struct BoundaryPartials {
    int rt[kConsumerWarps * 2];
    double v[kConsumerWarps * 2][4];
};
constexpr size_t kSoaSmemBytes2 = kSoaSmemBytes + sizeof(BoundaryPartials) + 16;

template <int NL, int MINB>
__global__ void __launch_bounds__(kGemvThreads, MINB)
    gemv_q5k_soa_kernel(const __grid_constant__ Q5kSoaMaps maps, const uint8_t* __restrict__ xlimbs,
                        const float* __restrict__ xgsum, const float* __restrict__ xscale,
                        float* __restrict__ y, uint32_t rows, uint32_t nb) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRingSlots * kSoaSlotBytes);
    uint64_t* empty = full + kRingSlots;
    BoundaryPartials* bnd = reinterpret_cast<BoundaryPartials*>(empty + kRingSlots);

    constexpr uint32_t W = kConsumerWarps;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t npairs = (rows + 1u) >> 1;
    const uint32_t p0 = static_cast<uint32_t>(static_cast<uint64_t>(npairs) * blockIdx.x / gridDim.x);
    const uint32_t p1 = static_cast<uint32_t>(static_cast<uint64_t>(npairs) * (blockIdx.x + 1) / gridDim.x);
    const uint32_t row0 = 2u * p0;
    const uint32_t rend = min(2u * p1, rows);
    const uint32_t nrt = (p1 - p0 + 1u) >> 1;       // row tiles (last may hold one pair)
    const bool last_half = ((p1 - p0) & 1u) != 0;   // final tile holds only 2 rows
    const uint32_t nkc = nb / kTileBlocks;
    const uint32_t T = nrt * nkc;                   // tiles, row-tile-major
    // Warp w consumes the contiguous tile chunk [c0, c0 + len); tile i of that
    // chunk is the (i*W + w)-th tile the producer issues.
    const uint32_t base = T / W, rem = T % W;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRingSlots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        fence_mbar_init();
    }
    if (threadIdx.x < 2 * W) bnd->rt[threadIdx.x] = -1;
    __syncthreads();

    if (warp == W) {
        // ---------------- producer: one thread streams every tile ----------------
        if (lane == 0) {
            prefetch_tmap(&maps.qs4);
            prefetch_tmap(&maps.qh4);
            prefetch_tmap(&maps.meta4);
            uint32_t seq = 0;
            for (; seq < T; ++seq) {
                const uint32_t w = seq % W, i = seq / W;
                const uint32_t tile = w * base + min(w, rem) + i;
                const uint32_t rt = tile / nkc, kc = tile - rt * nkc;
                const uint32_t slot = seq % kRingSlots;
                if (seq >= kRingSlots &&
                    !mbar_wait(&empty[slot], ((seq / kRingSlots) - 1u) & 1u, kFaultEmptyWait))
                    break;
                const bool half = last_half && rt == nrt - 1u;
                const int32_t r = static_cast<int32_t>(row0 + rt * kTileRows);
                uint8_t* dst = ring + slot * kSoaSlotBytes;
                mbar_arrive_expect_tx(&full[slot], half ? kSoaTileBytes / 2 : kSoaTileBytes);
                // inner coordinates in tensor-map elements: qs/qh as u64, meta as u32
                tma_load_2d(dst, half ? &maps.qs2 : &maps.qs4, static_cast<int32_t>(kc * 64), r, &full[slot]);
                tma_load_2d(dst + kSoaQsBytes, half ? &maps.qh2 : &maps.qh4, static_cast<int32_t>(kc * 16), r,
                            &full[slot]);
                tma_load_2d(dst + kSoaQsBytes + kSoaQhBytes, half ? &maps.meta2 : &maps.meta4,
                            static_cast<int32_t>(kc * 20), r, &full[slot]);
            }
            pdl_launch_dependents();
            // Drain: every issued copy must land before the CTA may exit.
            const uint32_t first = seq > kRingSlots ? seq - kRingSlots : 0u;
            for (uint32_t u = first; u < seq; ++u)
                if (!mbar_wait(&full[u % kRingSlots], (u / kRingSlots) & 1u, kFaultDrain)) break;
        }
        return;
    }

    // ---------------- consumers ----------------
    pdl_wait();  // x-pack and y belong to the dependency chain
    const uint32_t hh = lane >> 4, s = (lane >> 2) & 3u, p = lane & 3u;
    const uint32_t rot_lo = (4u - 2u * p) & 31u, rot_hi = (3u - 2u * p) & 31u;
    // Lanes with odd s read the second 16-byte half of their 32-byte qs run
    // first (bank-conflict-free quarter warps); the activation quads are
    // fetched in the same order, so no select is needed.
    const uint32_t c0 = s & 1u, c1 = c0 ^ 1u;
    const uint32_t len = base + (warp < rem ? 1u : 0u);
    const uint32_t chunk0 = warp * base + min(warp, rem);
    const uint8_t* xrow = xlimbs + (s * 4u + p) * 16u;  // lane's column inside a quad group
    const float2* xg2 = reinterpret_cast<const float2*>(xgsum);

    double acc0 = 0.0, acc1 = 0.0;  // fp64 row partials of this lane
    uint32_t cur_rt = 0xffffffffu, kc_first = 0, nflush = 0;
    bool ok = true;

    auto flush = [&](uint32_t rt, uint32_t kc_last) {
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) {
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, o);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, o);
        }
        const bool whole = kc_first == 0 && kc_last == nkc - 1u;
        if ((lane & 15u) == 0) {
            if (whole) {
                const uint32_t r = row0 + rt * kTileRows + 2u * hh;
                if (ok && r < rend) y[r] = static_cast<float>(acc0);
                if (ok && r + 1u < rend) y[r + 1u] = static_cast<float>(acc1);
            } else {
                const uint32_t e = warp * 2u + (nflush == 0 ? 0u : 1u);
                bnd->v[e][2 * hh] = acc0;
                bnd->v[e][2 * hh + 1] = acc1;
                if (hh == 0) bnd->rt[e] = static_cast<int>(rt);
            }
        }
        ++nflush;
        acc0 = 0.0;
        acc1 = 0.0;
    };

    for (uint32_t i = 0; i < len; ++i) {
        const uint32_t seq = i * W + warp;
        const uint32_t tile = chunk0 + i;
        const uint32_t rt = tile / nkc, kc = tile - rt * nkc;
        if (rt != cur_rt) {
            if (cur_rt != 0xffffffffu) flush(cur_rt, nkc - 1u);
            cur_rt = rt;
            kc_first = kc;
        }
        const uint32_t slot = seq % kRingSlots;
        const uint32_t bcol = kc * kTileBlocks + s;
        // activation quads and group sums do not depend on the tile's arrival
        // xl[0, 8NL): words of the half read first (c0), xl[8NL, 16NL): the other
        uint32_t xl[16 * NL];
        const uint8_t* xq = xrow + static_cast<size_t>(kc) * (4u * NL) * 256u;
#pragma unroll
        for (int j = 0; j < 2 * NL; ++j) {
            const uint4 va = __ldcg(reinterpret_cast<const uint4*>(xq + (2u * NL * c0 + j) * 256u));
            const uint4 vb = __ldcg(reinterpret_cast<const uint4*>(xq + (2u * NL * c1 + j) * 256u));
            xl[4 * j + 0] = va.x; xl[4 * j + 1] = va.y; xl[4 * j + 2] = va.z; xl[4 * j + 3] = va.w;
            xl[8 * NL + 4 * j + 0] = vb.x; xl[8 * NL + 4 * j + 1] = vb.y;
            xl[8 * NL + 4 * j + 2] = vb.z; xl[8 * NL + 4 * j + 3] = vb.w;
        }
        const float2 X = __ldcg(xg2 + bcol * 4u + p);
        const float es = __ldcg(xscale + bcol);

        if (ok && !mbar_wait(&full[slot], (seq / kRingSlots) & 1u, kFaultFullWait)) ok = false;
        if (ok) {
            const uint8_t* tb = ring + slot * kSoaSlotBytes;
            uint4 qA[2], qB[2], hA[2], hB[2];
            uint32_t dm[2], scm[2];
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const uint32_t row = 2u * hh + rr;
                const uint8_t* qsp = tb + row * 512u + s * 128u + p * 32u;
                const uint8_t* qhp = tb + kSoaQsBytes + row * 128u + s * 32u;
                const uint8_t* mp = tb + kSoaQsBytes + kSoaQhBytes + row * 80u + s * 20u;
                qA[rr] = *reinterpret_cast<const uint4*>(qsp + 16u * c0);
                qB[rr] = *reinterpret_cast<const uint4*>(qsp + 16u * c1);
                hA[rr] = *reinterpret_cast<const uint4*>(qhp + 16u * c0);
                hB[rr] = *reinterpret_cast<const uint4*>(qhp + 16u * c1);
                dm[rr] = *reinterpret_cast<const uint32_t*>(mp);
                scm[rr] = *reinterpret_cast<const uint32_t*>(mp + 4u + 4u * p);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);  // slot data now lives in registers
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const uint32_t qw[8] = {qA[rr].x, qA[rr].y, qA[rr].z, qA[rr].w, qB[rr].x, qB[rr].y, qB[rr].z, qB[rr].w};
                const uint32_t hw[8] = {hA[rr].x, hA[rr].y, hA[rr].z, hA[rr].w, hB[rr].x, hB[rr].y, hB[rr].z, hB[rr].w};
                int aa[NL], ab[NL];
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
                const double fa = limb_value<NL>(aa), fb = limb_value<NL>(ab);
                const float2 dmf = __half22float2(*reinterpret_cast<const __half2*>(&dm[rr]));
                const double sca = static_cast<double>(scm[rr] & 0xffu), mna = static_cast<double>((scm[rr] >> 8) & 0xffu);
                const double scb = static_cast<double>((scm[rr] >> 16) & 0xffu), mnb = static_cast<double>(scm[rr] >> 24);
                double a = static_cast<double>(dmf.x * es) * __fma_rn(sca, fa, scb * fb);
                a = __fma_rn(-static_cast<double>(dmf.y),
                             __fma_rn(mna, static_cast<double>(X.x), mnb * static_cast<double>(X.y)), a);
                if (rr == 0) acc0 += a; else acc1 += a;
            }
        } else {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
    }
    if (cur_rt != 0xffffffffu) {
        const uint32_t last_tile = chunk0 + len - 1u;
        flush(cur_rt, last_tile - cur_rt * nkc);
    }

    // Row tiles shared by several warps: combine in warp order.
    asm volatile("bar.sync 1, %0;" ::"r"(W * 32u) : "memory");
    if (threadIdx.x == 0 && ok) {
        int cur = -1;
        double v[4] = {0.0, 0.0, 0.0, 0.0};
        for (uint32_t e = 0; e <= 2u * W; ++e) {
            const int r = e < 2u * W ? bnd->rt[e] : -2;
            if (r == -1) continue;
            if (r != cur) {
                if (cur >= 0) {
                    const uint32_t rbase = row0 + static_cast<uint32_t>(cur) * kTileRows;
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        if (rbase + k < rend) y[rbase + k] = static_cast<float>(v[k]);
                }
                cur = r;
                if (r >= 0)
                    for (int k = 0; k < 4; ++k) v[k] = bnd->v[e][k];
            } else {
                for (int k = 0; k < 4; ++k) v[k] += bnd->v[e][k];
            }
        }
    }
}

}  // namespace q38
