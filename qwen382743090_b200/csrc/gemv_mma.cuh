// gemv_mma.cuh -- batched K-quant GEMM (Y[b][r] = sum_k W[r][k] X[b][k], batch
// 2..8 with f32 activations) over layout 2 (Q5_K and Q4_K fragment tiles,
// gemv_frag.cuh) on the tensor cores: the multi-token verify / prefill path.
// Same mathematics as the batch-1 GEMV (the reference's
// q38_q5k_sm86_soa_gemv_vec, src/driver.cpp:3887-4138, per activation row).
//
// One mma.sync.m16n8k32 (s8 x u8 -> s32) per (32-weight group, tile): the A
// operand is the activations -- 16 rows (batch b, limb l) x the group's 32
// elements, identical for every weight row, read as ready-made fragments from
// an "x-fragment" buffer -- and the B operand is the tile's 8 weight rows x 32
// weights decoded in registers exactly as in the GEMV (lane (g, t) reads its
// own words of row g; one word gives 4 weights of the even group and 4 of the
// odd group, the latter scaled by 8 or 16).  Both operands map the mma k index
// to group positions as k = 4t + j -> 8t + j, k = 16 + 4t + j -> 8t + 4 + j.
// The group's int32 tile is multiplied by the 6-bit group scale in integer
// arithmetic (exact), a super-block's 8 groups are summed in int32, and the
// block scale d * unit(b) * 256^l and the dmin * m * sum(x) term are applied
// in fp64 once per super-block.
//
// Work: warps are consumers with private rings of tile slots; each consumer
// owns a contiguous run of the CTA's (row octet, chunk) tiles; octets split
// between consumers are combined after the main loop in consumer order.
#pragma once

#include "gemv_frag.cuh"

namespace q38 {

constexpr uint32_t kMmaWarps = 8;
constexpr uint32_t kMmaDepth = 4;
constexpr uint32_t kMmaMaxBatch = 16;

// Bytes of the x-fragment buffer: per 32-element group and 16-row m-tile a
// 512-byte block (lane t's 16 bytes = its four A registers), then group sums
// float[B][groups] and units float[B][nb].
__host__ __device__ constexpr size_t xfrag_limb_bytes(uint32_t nb, uint32_t mtiles) {
    return static_cast<size_t>(nb) * 8u * mtiles * 512u;
}

// mma k index of group position P (shared with the weight fragments).
__host__ __device__ constexpr uint32_t frag_kslot(uint32_t P) {
    return 4u * (P >> 3) + (P & 3u) + 16u * ((P >> 2) & 1u);
}

// Offset of (m = b * NL + l, k) of group G inside the fragment region.
__device__ __forceinline__ uint32_t xfrag_offset(uint32_t G, uint32_t m, uint32_t k, uint32_t mtiles) {
    const uint32_t mt = m >> 4, mm = m & 15u;
    const uint32_t gid = mm & 7u, hi = mm >> 3, q = (k & 15u) >> 2, kh = k >> 4;
    const uint32_t lane = gid * 4u + q, reg = kh * 2u + hi;
    return ((G * mtiles + mt) * 32u + lane) * 16u + reg * 4u + (k & 3u);
}

// x f32 [B][K] -> x-fragments.  One warp per (super-block, batch row), the
// arithmetic of pack_block_warp<NL> (so the limbs equal the GEMV's).
template <int NL>
__global__ void __launch_bounds__(256) xfrag_f32_kernel(const float* __restrict__ x, uint32_t K, uint32_t B,
                                                        uint32_t mtiles, uint8_t* __restrict__ frag,
                                                        float* __restrict__ gsum, float* __restrict__ unit_out) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t nb = K / 256u, lane = threadIdx.x & 31u;
    const uint32_t w = blockIdx.x * 8u + (threadIdx.x >> 5);
    if (w >= nb * B) return;  // warp-uniform
    const uint32_t blk = w % nb, b = w / nb;
    const float* xr = x + static_cast<size_t>(b) * K + blk * 256u + lane * 8u;
    float v[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = xr[t];
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
    double gs = 0.0;
    const uint32_t g = lane >> 2;  // group of this lane's 8 elements
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const int xi = (poison || a == 0.0f) ? 0 : xpack_scale_round(v[t], sh, mul);
        gs += static_cast<double>(xi);
        int r = xi;
        const uint32_t k = frag_kslot((lane & 3u) * 8u + t);  // mma k of the element
#pragma unroll
        for (int l = 0; l < NL; ++l) {
            const int byte = ((r + 128) & 255) - 128;
            frag[xfrag_offset(blk * 8u + g, b * NL + l, k, mtiles)] = static_cast<uint8_t>(byte);
            r = (r - byte) >> 8;
        }
    }
    gs += __shfl_xor_sync(0xffffffffu, gs, 1);
    gs += __shfl_xor_sync(0xffffffffu, gs, 2);
    if ((lane & 3u) == 0) gsum[static_cast<size_t>(b) * nb * 8u + blk * 8u + g] = static_cast<float>(gs * unit);
    if (lane == 0) unit_out[static_cast<size_t>(b) * nb + blk] = unit;
}

// D = A x B (k = 32), A signed activation limbs, B unsigned weights.
__device__ __forceinline__ void mma_s8u8(int (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "r"(0));
}

template <int C, int MT>
struct MmaBoundary {
    int pair[C * 2];
    double v[C * 2][MT * 16][8];  // partial tiles of octets split between consumers
    double tmp[C][MT * 16][8];    // per-consumer staging of whole octets
};

template <uint32_t T, int MT>
__host__ __device__ constexpr size_t mma_smem_bytes() {
    return static_cast<size_t>(kMmaWarps) * kMmaDepth * FragTile<T>::kBytes + kMmaWarps * kMmaDepth * 8u +
           sizeof(MmaBoundary<kMmaWarps, MT>) + 256u;
}

// Decode pair p (runtime) of one word pair.
template <uint32_t T>
__device__ __forceinline__ void frag_decode_rt(uint32_t p, uint32_t q0, uint32_t q1, uint32_t h0, uint32_t h1,
                                               uint32_t& e0, uint32_t& o0, uint32_t& e1, uint32_t& o1) {
    switch (p) {
        case 0: frag_decode<T, 0>(q0, h0, e0, o0); frag_decode<T, 0>(q1, h1, e1, o1); break;
        case 1: frag_decode<T, 1>(q0, h0, e0, o0); frag_decode<T, 1>(q1, h1, e1, o1); break;
        case 2: frag_decode<T, 2>(q0, h0, e0, o0); frag_decode<T, 2>(q1, h1, e1, o1); break;
        default: frag_decode<T, 3>(q0, h0, e0, o0); frag_decode<T, 3>(q1, h1, e1, o1); break;
    }
}

// MT m-tiles of 16 (batch, limb) rows: B * NL <= 16 * MT.
template <uint32_t T, int NL, int MT>
__global__ void __launch_bounds__(kMmaWarps * 32, 1)
    gemm_frag_mma_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xfrag,
                         const float* __restrict__ xgsum, const float* __restrict__ xunit, float* __restrict__ y,
                         uint32_t rows, uint32_t nb, uint32_t B) {
    using F = FragTile<T>;
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t W = kMmaWarps, D = kMmaDepth, TB = F::kBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(W) * D * TB);
    MmaBoundary<W, MT>* bnd = reinterpret_cast<MmaBoundary<W, MT>*>(bars + W * D);
    if (threadIdx.x == 0) pdl_launch_dependents();

    const uint32_t cons = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t gid = lane >> 2, q = lane & 3u;
    const uint32_t nocts = (rows + 7u) / 8u, nkc = nb / 2u;
    const uint32_t obase = nocts / gridDim.x, orem = nocts % gridDim.x;
    const uint32_t o0 = blockIdx.x * obase + min(blockIdx.x, orem);
    const uint32_t o1 = o0 + obase + (blockIdx.x < orem ? 1u : 0u);
    const uint32_t ntiles = (o1 - o0) * nkc;
    const uint32_t base = ntiles / W, rem = ntiles % W;
    const uint32_t len = base + (cons < rem ? 1u : 0u);
    const uint32_t step0 = cons * base + min(cons, rem);
    const uint8_t* src = w + (static_cast<size_t>(o0) * nkc + step0) * TB;
    uint8_t* ring = smem + static_cast<size_t>(cons) * D * TB;
    uint64_t* full = bars + cons * D;
    auto issue = [&](uint32_t i) {
        mbar_arrive_expect_tx(&full[i % D], TB);
        tma_load_1d(ring + (i % D) * TB, src + static_cast<size_t>(i) * TB, TB, &full[i % D]);
    };
    if (lane == 0) {
        for (uint32_t i = 0; i < D; ++i) mbar_init(&full[i], 1);
        fence_mbar_init();
        for (uint32_t i = 0; i < D && i < len; ++i) issue(i);
    }
    if (threadIdx.x < 2u * W) bnd->pair[threadIdx.x] = -1;
    __syncthreads();
    pdl_wait();

    // This lane's B-fragment row is weight row gid of the octet; its C entries
    // belong to weight rows 2q and 2q+1 and activation rows gid, gid+8.
    double acc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][e] = 0.0;
    bool ok = true;
    uint32_t waited = 0, issued = min(len, D);
    uint32_t oct = step0 / nkc, kc = step0 % nkc, kc_first = kc, nflush = 0;
    bool started = false;
    const uint32_t mrow[2] = {gid, gid + 8u};

    auto flush = [&](bool whole) {
        const uint32_t e = cons * 2u + (nflush == 0 ? 0u : 1u);
        double(*tile)[8] = whole ? bnd->tmp[cons] : bnd->v[e];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j) tile[mt * 16 + mrow[j >> 1]][2u * q + (j & 1u)] = acc[mt][j];
        __syncwarp();
        if (whole) {
            for (uint32_t t = lane; t < B * 8u; t += 32u) {
                const uint32_t b = t / 8u, r = t % 8u, row = 8u * (o0 + oct) + r;
                double s = 0.0;
                for (int l = 0; l < NL; ++l) s += tile[b * NL + l][r];
                if (ok && row < rows) y[static_cast<size_t>(b) * rows + row] = static_cast<float>(s);
            }
            __syncwarp();
        } else if (lane == 0) {
            bnd->pair[e] = static_cast<int>(oct);
        }
        ++nflush;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[mt][j] = 0.0;
    };

    for (uint32_t i = 0; i < len; ++i) {
        const uint32_t slot = i % D;
        const bool landed = __all_sync(0xffffffffu, ok && mbar_wait_spin(&full[slot], (i / D) & 1u, kFaultFullWait));
        if (!landed) ok = false;
        else waited = i + 1u;
        started = true;
        if (ok) {
            const uint8_t* tb = ring + slot * TB;
            uint4 qh = make_uint4(0u, 0u, 0u, 0u);
            if constexpr (T == 13u) qh = *reinterpret_cast<const uint4*>(tb + F::kQh + lane * 16u);
#pragma unroll 1
            for (uint32_t s = 0; s < 2u; ++s) {
                const uint32_t blk = kc * 2u + s;
                // scales / mins of the C rows 2q and 2q+1
                const uint4 sc0 = *reinterpret_cast<const uint4*>(tb + F::kSc + s * 128u + (2u * q) * 16u);
                const uint4 sc1 = *reinterpret_cast<const uint4*>(tb + F::kSc + s * 128u + (2u * q + 1u) * 16u);
                const uint32_t h0 = s ? qh.z : qh.x, h1 = s ? qh.w : qh.y;
                int ae[MT][4], ao[MT][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) ae[mt][j] = ao[mt][j] = 0;
#pragma unroll 1
                for (uint32_t p = 0; p < 4u; ++p) {
                    const uint2 qw = *reinterpret_cast<const uint2*>(tb + s * 1024u + (p >> 1) * 512u + lane * 16u +
                                                                     (p & 1u) * 8u);
                    uint32_t e0, od0, e1, od1;
                    frag_decode_rt<T>(p, qw.x, qw.y, h0, h1, e0, od0, e1, od1);
                    const uint32_t s0 = (p < 2u ? sc0.x : sc0.y) >> (16u * (p & 1u));
                    const uint32_t s1 = (p < 2u ? sc1.x : sc1.y) >> (16u * (p & 1u));
                    const int se0 = static_cast<int>(s0 & 0xffu), so0 = static_cast<int>((s0 >> 8) & 0xffu);
                    const int se1 = static_cast<int>(s1 & 0xffu), so1 = static_cast<int>((s1 >> 8) & 0xffu);
                    const uint32_t ge = blk * 8u + 2u * p;  // global group of the even weights
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const uint4 fa = __ldcg(reinterpret_cast<const uint4*>(xfrag + ((ge * MT + mt) * 32u + lane) * 16u));
                        const uint4 fb =
                            __ldcg(reinterpret_cast<const uint4*>(xfrag + (((ge + 1u) * MT + mt) * 32u + lane) * 16u));
                        int de[4], dd[4];
                        mma_s8u8(de, fa, e0, e1);
                        mma_s8u8(dd, fb, od0, od1);
                        ae[mt][0] += se0 * de[0];
                        ae[mt][1] += se1 * de[1];
                        ae[mt][2] += se0 * de[2];
                        ae[mt][3] += se1 * de[3];
                        ao[mt][0] += so0 * dd[0];
                        ao[mt][1] += so1 * dd[1];
                        ao[mt][2] += so0 * dd[2];
                        ao[mt][3] += so1 * dd[3];
                    }
                }
                // super-block scales: d, dmin of rows 2q, 2q+1; unit and group sums of each activation row
                const uint32_t dmw0 = *reinterpret_cast<const uint32_t*>(tb + F::kDm + s * 32u + (2u * q) * 4u);
                const uint32_t dmw1 = *reinterpret_cast<const uint32_t*>(tb + F::kDm + s * 32u + (2u * q + 1u) * 4u);
                const float2 dm0 = __half22float2(*reinterpret_cast<const __half2*>(&dmw0));
                const float2 dm1 = __half22float2(*reinterpret_cast<const __half2*>(&dmw1));
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t m = mt * 16u + mrow[j >> 1];
                        const uint32_t b = m / NL, l = m % NL;
                        if (b >= B) continue;
                        const float2 dm = (j & 1) ? dm1 : dm0;
                        const double un = static_cast<double>(__ldcg(xunit + static_cast<size_t>(b) * nb + blk));
                        const int a8 = ae[mt][j] * 8 + (ao[mt][j] >> F::kOddShift);  // x8, exact
                        double v = static_cast<double>(a8) * static_cast<double>(dm.x) * un *
                                   static_cast<double>(1u << (8u * l)) * 0.125;
                        if (l == 0) {  // the min term, once per (activation row, weight row)
                            const uint4 sm = (j & 1) ? sc1 : sc0;
                            const float* X = xgsum + static_cast<size_t>(b) * nb * 8u + blk * 8u;
                            const uint32_t mins[2] = {sm.z, sm.w};
                            float mn = 0.0f;
#pragma unroll
                            for (int gg = 0; gg < 8; ++gg)
                                mn = fmaf(static_cast<float>((mins[gg >> 2] >> (8 * (gg & 3))) & 0xffu), __ldcg(X + gg),
                                          mn);
                            v -= static_cast<double>(dm.y * mn);
                        }
                        acc[mt][j] += v;
                    }
            }
        }
        __syncwarp();
        if (ok && lane == 0 && i + D < len) {
            fence_proxy_async_smem();
            issue(i + D);
            issued = i + D + 1u;
        }
        if (++kc == nkc) {
            flush(kc_first == 0);
            kc = 0;
            kc_first = 0;
            ++oct;
            started = false;
        }
    }
    if (started) flush(false);
    if (!ok && lane == 0) {
        for (uint32_t i = waited; i < issued; ++i)
            if (!mbar_wait(&full[i % D], (i / D) & 1u, kFaultDrain)) break;
    }
    __syncthreads();
    // octets split between consumers: the first entry of each run sums it
    if (threadIdx.x < 2u * W && ok) {
        const uint32_t e = threadIdx.x;
        const int pr = bnd->pair[e];
        if (pr >= 0) {
            int prev = e >= 1 ? bnd->pair[e - 1] : -1;
            if (prev == -1 && e >= 2) prev = bnd->pair[e - 2];
            if (prev != pr) {
                for (uint32_t t = 0; t < B * 8u; ++t) {
                    const uint32_t b = t / 8u, r = t % 8u, row = 8u * (o0 + static_cast<uint32_t>(pr)) + r;
                    double s = 0.0;
                    for (uint32_t qq = e; qq < 2u * W; ++qq) {
                        const int pq = bnd->pair[qq];
                        if (pq == -1) continue;
                        if (pq != pr) break;
                        for (int l = 0; l < NL; ++l) s += bnd->v[qq][b * NL + l][r];
                    }
                    if (row < rows) y[static_cast<size_t>(b) * rows + row] = static_cast<float>(s);
                }
            }
        }
    }
}

}  // namespace q38
