// gemv_mma.cuh -- batched Q5_K GEMM (Y[b][r] = sum_k W[r][k] X[b][k], batch
// 2..10 with f32 activations, up to 16 with Q8_K) over the B200 tiled layout
// on the tensor cores: the multi-token verify / prefill path.  Same
// mathematics as the batch-1 GEMV (the reference's q38_q5k_sm86_soa_gemv_vec,
// src/driver.cpp:3887-4138, per activation row).
//
// One mma.sync.m16n8k32 (int8 x int8 -> int32) per (32-weight group, 8 weight
// rows): the A operand is the activations -- 16 rows (batch b, limb l) x the
// group's 32 elements, identical for every weight row, read as ready-made
// fragments from an "x-fragment" buffer -- and the B operand is 8 weight rows
// x 32 weights decoded in registers (the same 5-bit decode as the GEMV; one
// qs/qh word pair yields 4 weights of each group of a pair, i.e. both groups'
// fragments).  The group's int32 tile is multiplied by the 6-bit group scale
// in integer arithmetic (exact), a super-block's 8 groups are summed in int32,
// and the block scale d * unit(b) * 256^l and the dmin * m * sum(x) term are
// applied in fp64 once per super-block.  mma.sync takes both operands from
// registers, so the decoded weights never leave the register file; for batch
// <= 16 the tensor pipe is far from its limit and the kernel is bound by
// weight streaming and decode, like the GEMV.
//
// Work: warps are consumers with private rings of 2-tile slots (tiles (2J, kc)
// and (2J+1, kc): 8 rows x 4 super-blocks); each consumer owns a contiguous
// run of the CTA's (quad pair, chunk) steps; quad pairs split between
// consumers are combined after the main loop in consumer order.
#pragma once

#include "gemv_tiled.cuh"

namespace q38 {

constexpr uint32_t kMmaWarps = 8;
constexpr uint32_t kMmaDepth = 2;
constexpr uint32_t kMmaSlot = 2u * kT2TileBytes;  // two quads at the same chunk
constexpr uint32_t kMmaMaxBatch = 16;

// Bytes of the x-fragment buffer: per 32-element group and 16-row m-tile a
// 512-byte block (lane t's 16 bytes = its four A registers), then group sums
// float[B][groups] and units float[B][nb].
__host__ __device__ constexpr size_t xfrag_limb_bytes(uint32_t nb, uint32_t mtiles) {
    return static_cast<size_t>(nb) * 8u * mtiles * 512u;
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
    float unit = 0.0f;
    const bool poison = a == INFINITY;
    if (poison) {
        unit = __int_as_float(0x7fc00000);
    } else if (a > 0.0f) {
        int e;
        frexpf(a, &e);
        sh = xpack_bits<NL>() - e;
        if (static_cast<double>(ldexpf(a, sh)) > xpack_limit<NL>()) sh -= 1;
        unit = ldexpf(1.0f, -sh);
    }
    double gs = 0.0;
    const uint32_t g = lane >> 2;  // group of this lane's 8 elements
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const int xi = (poison || a == 0.0f) ? 0 : __float2int_rn(ldexpf(v[t], sh));
        gs += static_cast<double>(xi);
        int r = xi;
        const uint32_t k = (lane & 3u) * 8u + t;  // element inside the group
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

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

template <int C, int MT>
struct MmaBoundary {
    int pair[C * 2];
    double v[C * 2][MT * 16][8];  // partial tiles of quad pairs split between consumers
    double tmp[C][MT * 16][8];    // per-consumer staging of whole quad pairs
};

template <int NL, int MT>
__host__ __device__ constexpr size_t mma_smem_bytes() {
    return static_cast<size_t>(kMmaWarps) * kMmaDepth * kMmaSlot + kMmaWarps * kMmaDepth * 8u +
           sizeof(MmaBoundary<kMmaWarps, MT>) + 256u;
}

// MT m-tiles of 16 (batch, limb) rows: B * NL <= 16 * MT.
template <int NL, int MT>
__global__ void __launch_bounds__(kMmaWarps * 32, 1)
    gemm_q5k_tiled_mma_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xfrag,
                              const float* __restrict__ xgsum, const float* __restrict__ xunit, float* __restrict__ y,
                              uint32_t rows, uint32_t nb, uint32_t B) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t W = kMmaWarps, D = kMmaDepth;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(W) * D * kMmaSlot);
    MmaBoundary<W, MT>* bnd = reinterpret_cast<MmaBoundary<W, MT>*>(bars + W * D);
    if (threadIdx.x == 0) pdl_launch_dependents();

    const uint32_t cons = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t gid = lane >> 2, q = lane & 3u;
    const uint32_t nquads = (rows + 3u) / 4u, npairs = (nquads + 1u) / 2u;
    const uint32_t nkc = nb / 4u;
    const uint32_t p0 = static_cast<uint32_t>(static_cast<uint64_t>(npairs) * blockIdx.x / gridDim.x);
    const uint32_t p1 = static_cast<uint32_t>(static_cast<uint64_t>(npairs) * (blockIdx.x + 1) / gridDim.x);
    const uint32_t T = (p1 - p0) * nkc;
    const uint32_t base = T / W, rem = T % W;
    const uint32_t len = base + (cons < rem ? 1u : 0u);
    const uint32_t step0 = cons * base + min(cons, rem);
    uint8_t* ring = smem + static_cast<size_t>(cons) * D * kMmaSlot;
    uint64_t* full = bars + cons * D;

    auto issue = [&](uint32_t i) {
        const uint32_t st = step0 + i, J = p0 + st / nkc, kc = st % nkc;
        const uint32_t qa = 2u * J, qb = qa + 1u;
        uint8_t* dst = ring + (i % D) * kMmaSlot;
        const uint32_t bytes = (qb < nquads ? 2u : 1u) * kT2TileBytes;
        mbar_arrive_expect_tx(&full[i % D], bytes);
        tma_load_1d(dst, w + (static_cast<size_t>(qa) * nkc + kc) * kT2TileBytes, kT2TileBytes, &full[i % D]);
        if (qb < nquads)
            tma_load_1d(dst + kT2TileBytes, w + (static_cast<size_t>(qb) * nkc + kc) * kT2TileBytes, kT2TileBytes,
                        &full[i % D]);
    };
    if (lane == 0) {
        for (uint32_t i = 0; i < D; ++i) mbar_init(&full[i], 1);
        fence_mbar_init();
        for (uint32_t i = 0; i < D && i < len; ++i) issue(i);
    }
    if (threadIdx.x < 2u * W) bnd->pair[threadIdx.x] = -1;
    __syncthreads();
    pdl_wait();

    // This lane's B-fragment row n = gid: quad n/4 of the pair, row n%4; its C
    // entries belong to weight rows 2q and 2q+1 and activation rows gid, gid+8.
    const uint32_t brow = gid & 3u, bquad = gid >> 2;
    const uint32_t rot_lo_base = 4u, rot_hi_base = 3u;
    double acc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][e] = 0.0;
    bool ok = true;
    uint32_t waited = 0, issued = min(len, D);
    uint32_t pair = step0 / nkc, kc = step0 % nkc, kc_first = kc, nflush = 0;
    bool started = false;
    // activation row m of entry e (rows gid, gid, gid+8, gid+8) and its limb weight
    const uint32_t mrow[2] = {gid, gid + 8u};

    auto flush = [&](bool whole) {
        // Stage this consumer's 16*MT x 8 partial tile in its boundary slot,
        // then sum limbs per (batch, row).
        const uint32_t e = cons * 2u + (nflush == 0 ? 0u : 1u);
        double(*tile)[8] = whole ? bnd->tmp[cons] : bnd->v[e];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j) tile[mt * 16 + mrow[j >> 1]][2u * q + (j & 1u)] = acc[mt][j];
        __syncwarp();
        if (whole) {
            for (uint32_t t = lane; t < B * 8u; t += 32u) {
                const uint32_t b = t / 8u, r = t % 8u, row = 8u * (p0 + pair) + r;
                double s = 0.0;
                for (int l = 0; l < NL; ++l) s += tile[b * NL + l][r];
                if (ok && row < rows) y[static_cast<size_t>(b) * rows + row] = static_cast<float>(s);
            }
            __syncwarp();
        } else if (lane == 0) {
            bnd->pair[e] = static_cast<int>(pair);
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
            const uint8_t* tb = ring + slot * kMmaSlot;
            const uint8_t* tq = tb + bquad * kT2TileBytes;  // this lane's quad (B operand rows)
            const bool bvalid = 4u * (2u * (p0 + pair) + bquad) < rows || bquad == 0;
#pragma unroll 1
            for (uint32_t s = 0; s < 4u; ++s) {
                const uint32_t blk = kc * 4u + s;
                int ai[MT][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) ai[mt][j] = 0;
                // META of the C rows 2q, 2q+1 (quad 0 for q < 2, else quad 1)
                const uint8_t* mq = tb + (q >> 1) * kT2TileBytes + kT2MetaOff;
                const uint8_t* m0 = mq + (((2u * q) & 3u) * 4u + s) * 20u;
                const uint8_t* m1 = mq + (((2u * q + 1u) & 3u) * 4u + s) * 20u;
#pragma unroll
                for (uint32_t p = 0; p < 4u; ++p) {
                    const uint8_t* qs = tq + (brow * 4u + s) * 128u + 32u * p;
                    const uint8_t* qh = tq + kT2QhOff + (brow * 4u + s) * 32u;
                    const uint32_t w0 = bvalid ? *reinterpret_cast<const uint32_t*>(qs + 4u * q) : 0u;
                    const uint32_t w1 = bvalid ? *reinterpret_cast<const uint32_t*>(qs + 16u + 4u * q) : 0u;
                    const uint32_t h0 = bvalid ? *reinterpret_cast<const uint32_t*>(qh + 4u * q) : 0u;
                    const uint32_t h1 = bvalid ? *reinterpret_cast<const uint32_t*>(qh + 16u + 4u * q) : 0u;
                    const uint32_t rl = (rot_lo_base - 2u * p) & 31u, rh = (rot_hi_base - 2u * p) & 31u;
                    uint32_t lo0, hi0, lo1, hi1;
                    q5_decode(w0, h0, rl, rh, lo0, hi0);
                    q5_decode(w1, h1, rl, rh, lo1, hi1);
                    const uint32_t ga = blk * 8u + 2u * p;  // global group of lo*, ga + 1 of hi*
                    const int sa0 = m0[4u + 4u * p], sb0 = m0[6u + 4u * p];  // scales of rows 2q, groups 2p/2p+1
                    const int sa1 = m1[4u + 4u * p], sb1 = m1[6u + 4u * p];
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const uint4 fa = __ldg(reinterpret_cast<const uint4*>(xfrag + ((ga * MT + mt) * 32u + lane) * 16u));
                        const uint4 fb =
                            __ldg(reinterpret_cast<const uint4*>(xfrag + (((ga + 1u) * MT + mt) * 32u + lane) * 16u));
                        int da[4], db[4];
                        mma_s8(da, fa, lo0, lo1);
                        mma_s8(db, fb, hi0, hi1);
                        ai[mt][0] += sa0 * da[0] + sb0 * db[0];
                        ai[mt][1] += sa1 * da[1] + sb1 * db[1];
                        ai[mt][2] += sa0 * da[2] + sb0 * db[2];
                        ai[mt][3] += sa1 * da[3] + sb1 * db[3];
                    }
                }
                // super-block scales: d, dmin of rows 2q, 2q+1; unit and group sums of each activation row
                const float2 dm0 = __half22float2(*reinterpret_cast<const __half2*>(m0));
                const float2 dm1 = __half22float2(*reinterpret_cast<const __half2*>(m1));
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t m = mt * 16u + mrow[j >> 1];
                        const uint32_t b = m / NL, l = m % NL;
                        if (b >= B) continue;
                        const float2 dm = (j & 1) ? dm1 : dm0;
                        const double un = static_cast<double>(__ldg(xunit + static_cast<size_t>(b) * nb + blk));
                        double v = static_cast<double>(ai[mt][j]) * static_cast<double>(dm.x) * un *
                                   static_cast<double>(1u << (8u * l));
                        if (l == 0) {  // the min term, once per (activation row, weight row)
                            const uint8_t* mm = (j & 1) ? m1 : m0;
                            const float* X = xgsum + static_cast<size_t>(b) * nb * 8u + blk * 8u;
                            float mn = 0.0f;
#pragma unroll
                            for (int g = 0; g < 8; ++g) mn = fmaf(static_cast<float>(mm[5 + 2 * g]), __ldg(X + g), mn);
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
            ++pair;
            started = false;
        }
    }
    if (started) flush(false);
    if (!ok && lane == 0) {
        for (uint32_t i = waited; i < issued; ++i)
            if (!mbar_wait(&full[i % D], (i / D) & 1u, kFaultDrain)) break;
    }
    __syncthreads();
    // quad pairs split between consumers: the first entry of each run sums it
    if (threadIdx.x < 2u * W && ok) {
        const uint32_t e = threadIdx.x;
        const int pr = bnd->pair[e];
        if (pr >= 0) {
            int prev = e >= 1 ? bnd->pair[e - 1] : -1;
            if (prev == -1 && e >= 2) prev = bnd->pair[e - 2];
            if (prev != pr) {
                for (uint32_t t = 0; t < B * 8u; ++t) {
                    const uint32_t b = t / 8u, r = t % 8u, row = 8u * (p0 + static_cast<uint32_t>(pr)) + r;
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
