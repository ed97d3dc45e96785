// gemm_frag.cuh -- batched K-quant GEMM Y[b][r] = sum_k W[r][k] X[b][k] for
// up to 8 activation rows (the multi-token verify / prefill path) over the
// B200 fragment tiles of layout 2 (Q5_K and Q4_K, gemv_frag.cuh).
//
// It is the batch-1 tile kernel (gemv_frag_cta) with the batch rows folded
// into the tile loop: a warp decodes each landed tile's weights into mma A
// fragments once -- and extracts the tile's group scales, d / dmin and min
// selectors once -- then, for all batch rows together, runs the same two
// mma.sync.m16n8k32 per (8 rows, group pair) against each row's x-fragments
// and the same exact int32 group scaling and fp64 block epilogue into the
// row's own accumulator.  The weights are streamed from HBM once per call
// whatever the batch, which is the point of the batched path; per batch row
// the arithmetic and its order are those of the batch-1 kernel, so row b of Y
// is bit-identical to the single-row GEMV of X[b] on the same CTA split.
//
// x-fragments of all rows are staged in shared memory by bulk copies after the
// dependency wait, one mbarrier per chunk of 2 super-blocks (XM 1), when they
// fit next to the rings, else read from L2 with ld.cg (XM 0).  Rows of the
// CTA's share split between warps are combined per batch row in warp order,
// as in the GEMV.
#pragma once

#include "gemv_frag.cuh"

namespace q38 {

constexpr uint32_t kGemmMaxBatch = 8;
constexpr uint32_t kGemmMaxChunks = 64;  // x staged in shared memory (XM 1) for K <= 64 * 512

template <uint32_t T, int W, int DEPTH, int NB>
__host__ __device__ constexpr size_t gemm_frag_fixed_bytes() {
    return static_cast<size_t>(W) * DEPTH * FragTile<T>::kBytes + W * DEPTH * 8 + kGemmMaxChunks * 8 +
           NB * sizeof(PairBoundary<W, kF8Rows>) + 256;
}
template <uint32_t T, int W, int DEPTH, int NB>
__host__ __device__ constexpr size_t gemm_frag_smem_bytes(uint32_t nb, bool xsmem) {
    return gemm_frag_fixed_bytes<T, W, DEPTH, NB>() + (xsmem ? NB * xfrag1_bytes(nb) : 0u);
}

// The tile's words in registers (one lane's share) and what the batch rows share.
template <uint32_t T>
struct GemmTileRegs {
    uint32_t ev[kF8Blocks][2][2], od[kF8Blocks][2][2];  // A fragments: [s][c][half] even / odd words, 2 rows each
    uint32_t ev1[kF8Blocks][2][2], od1[kF8Blocks][2][2];
    int sc[kF8Blocks][2][4];                             // 6-bit group scales of the lane's row
    double dmx[kF8Blocks];                               // d as double
    float dmy[kF8Blocks], mna[kF8Blocks], mnb[kF8Blocks];  // dmin; the two mins of pair t
};

template <uint32_t T>
__device__ __forceinline__ void gemm_tile_decode(const uint8_t* tb, uint32_t lane, GemmTileRegs<T>& r) {
    using F = FragTile<T>;
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t msel_a = 0x7640u | (2u * (t & 1u)), msel_b = 0x7640u | (2u * (t & 1u) + 1u);
    uint4 qh = make_uint4(0u, 0u, 0u, 0u);
    if constexpr (T == 13u) qh = *reinterpret_cast<const uint4*>(tb + F::kQh + lane * 16u);
#pragma unroll
    for (uint32_t s = 0; s < kF8Blocks; ++s) {
        const uint4 scw = *reinterpret_cast<const uint4*>(tb + F::kSc + s * 128u + g * 16u);
        const uint32_t dmw = *reinterpret_cast<const uint32_t*>(tb + F::kDm + s * 32u + g * 4u);
        const uint32_t h0 = s ? qh.z : qh.x, h1 = s ? qh.w : qh.y;
#pragma unroll
        for (uint32_t c = 0; c < 2u; ++c) {
            const uint4 q = *reinterpret_cast<const uint4*>(tb + s * 1024u + c * 512u + lane * 16u);
            if (c == 0) {
                frag_decode<T, 0>(q.x, h0, r.ev[s][c][0], r.od[s][c][0]);
                frag_decode<T, 0>(q.y, h1, r.ev1[s][c][0], r.od1[s][c][0]);
                frag_decode<T, 1>(q.z, h0, r.ev[s][c][1], r.od[s][c][1]);
                frag_decode<T, 1>(q.w, h1, r.ev1[s][c][1], r.od1[s][c][1]);
            } else {
                frag_decode<T, 2>(q.x, h0, r.ev[s][c][0], r.od[s][c][0]);
                frag_decode<T, 2>(q.y, h1, r.ev1[s][c][0], r.od1[s][c][0]);
                frag_decode<T, 3>(q.z, h0, r.ev[s][c][1], r.od[s][c][1]);
                frag_decode<T, 3>(q.w, h1, r.ev1[s][c][1], r.od1[s][c][1]);
            }
            const uint32_t sw = c ? scw.y : scw.x;
            r.sc[s][c][0] = byte_u<0>(sw);
            r.sc[s][c][1] = byte_u<1>(sw);
            r.sc[s][c][2] = byte_u<2>(sw);
            r.sc[s][c][3] = byte_u<3>(sw);
        }
        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&dmw));
        r.dmx[s] = static_cast<double>(dm.x);
        r.dmy[s] = dm.y;
        const uint32_t mw = t < 2u ? scw.z : scw.w;
        r.mna[s] = byte_f(mw, msel_a);
        r.mnb[s] = byte_f(mw, msel_b);
    }
}


// Batch rows [B0, B0 + RG)'s shares of a decoded tile, each added to its
// running fp64 sum in the batch-1 kernel's order (frag_tile_acc).  The rows
// are interleaved -- the RG rows' mma of one (super-block, group pair) issue
// back to back -- so a warp has RG independent dependency chains in flight.  Row b
// reads its x-fragments at xb + xrow[b] (rows past the batch point at a real
// row and are computed but never stored, so the loop has no branch).
template <uint32_t T, int NB, int B0, int RG, bool XL2>
__device__ __forceinline__ void gemm_tile_rows(const GemmTileRegs<T>& r, const uint8_t* xb, const uint32_t (&xrow)[NB],
                                               uint32_t lane, double (&acc)[NB]) {
    using F = FragTile<T>;
    const uint32_t t = lane & 3u;
    float mn[NB];
#pragma unroll
    for (int b = B0; b < B0 + RG; ++b) mn[b] = 0.0f;
#pragma unroll
    for (uint32_t s = 0; s < kF8Blocks; ++s) {
        int Ae[NB], Ao[NB];
#pragma unroll
        for (int b = B0; b < B0 + RG; ++b) Ae[b] = Ao[b] = 0;
#pragma unroll
        for (uint32_t c = 0; c < 2u; ++c) {
#pragma unroll
            for (int b = B0; b < B0 + RG; ++b) {
                const uint8_t* xp = xb + xrow[b] + s * kXfBlockBytes + c * 512u + lane * 16u;
                const uint4 xv = XL2 ? __ldcg(reinterpret_cast<const uint4*>(xp)) : *reinterpret_cast<const uint4*>(xp);
                int d0, d3;
                mma_u8s8_16x8x32(d0, d3, r.ev[s][c][0], r.od[s][c][0], r.ev1[s][c][0], r.od1[s][c][0], xv.x, xv.y);
                Ae[b] += r.sc[s][c][0] * d0;
                Ao[b] += r.sc[s][c][1] * d3;
                mma_u8s8_16x8x32(d0, d3, r.ev[s][c][1], r.od[s][c][1], r.ev1[s][c][1], r.od1[s][c][1], xv.z, xv.w);
                Ae[b] += r.sc[s][c][2] * d0;
                Ao[b] += r.sc[s][c][3] * d3;
            }
        }
#pragma unroll
        for (int b = B0; b < B0 + RG; ++b) {
            const uint8_t* xm_p = xb + xrow[b] + s * kXfBlockBytes + kXfMetaOff + t * 16u;
            const uint4 xm = XL2 ? __ldcg(reinterpret_cast<const uint4*>(xm_p)) : *reinterpret_cast<const uint4*>(xm_p);
            const int A8 = Ae[b] * 8 + (Ao[b] >> F::kOddShift);
            const double unw = __hiloint2double(static_cast<int>(xm.y), static_cast<int>(xm.x));
            acc[b] = __fma_rn(static_cast<double>(A8), r.dmx[s] * unw, acc[b]);
            const float pm = fmaf(r.mna[s], __uint_as_float(xm.z), r.mnb[s] * __uint_as_float(xm.w));
            mn[b] = fmaf(r.dmy[s], pm, mn[b]);
        }
    }
#pragma unroll
    for (int b = B0; b < B0 + RG; ++b) acc[b] -= static_cast<double>(mn[b]);
}

// xf: x-fragments of the batch rows, row b at xf + b * xf_stride bytes; y row b
// at y + b * y_stride floats; rows >= batch of the NB are computed on a copy
// of row batch - 1 and not stored.  XM 1 stages the rows' x-fragments in
// shared memory chunk by chunk (2 super-blocks of every row per mbarrier), so
// a warp starts on its first tile once that tile's chunk has landed.  The
// rows run in two interleaved groups (RG, then NB - RG) when NB > RG.
template <uint32_t T, int XM, int W, int DEPTH, int NB, int RG>
__global__ void __launch_bounds__(W * 32, 1)
    gemm_frag_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xf, uint32_t xf_stride, float* y,
                     uint32_t y_stride, uint32_t rows, uint32_t nb, uint32_t batch) {
    extern __shared__ __align__(128) uint8_t smem[];
    using F = FragTile<T>;
    constexpr uint32_t C = W, R = kF8Rows, TB = F::kBytes, XC = kF8Blocks * kXfBlockBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(W) * DEPTH * TB);
    uint64_t* xbar = bars + C * DEPTH;
    PairBoundary<W, R>* bnd = reinterpret_cast<PairBoundary<W, R>*>(xbar + kGemmMaxChunks);
    uint8_t* xs = reinterpret_cast<uint8_t*>(bnd + NB);
    xs += (128u - (reinterpret_cast<uintptr_t>(xs) & 127u)) & 127u;
    const uint32_t xbytes = static_cast<uint32_t>(xfrag1_bytes(nb));

    if (threadIdx.x == 0) pdl_launch_dependents();
    const uint32_t cta = blockIdx.x, ncta = gridDim.x;
    const uint32_t cons = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t nocts = (rows + R - 1u) / R, nkc = nb / kF8Blocks;
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
        if (XM == 1 && cons == 0)
            for (uint32_t k = 0; k < nkc; ++k) mbar_init(&xbar[k], 1);
        fence_mbar_init();
        for (uint32_t k = 0; k < DEPTH && k < len; ++k) issue(k);
    }
    for (uint32_t i = threadIdx.x; i < 2u * C * NB; i += blockDim.x) bnd[i / (2u * C)].pair[i % (2u * C)] = -1;
    __syncthreads();

    pdl_wait();  // x-fragments and y belong to the dependency chain
    if constexpr (XM == 1) {
        // warp 0 stages chunk k of every row: lane b < batch copies row b
        if (cons == 0) {
            for (uint32_t k = 0; k < nkc; ++k) {
                if (lane == 0) mbar_arrive_expect_tx(&xbar[k], XC * batch);
                __syncwarp();
                if (lane < batch)
                    tma_load_1d(xs + lane * xbytes + k * XC, xf + static_cast<size_t>(lane) * xf_stride + k * XC, XC,
                                &xbar[k]);
            }
        }
    }
    const uint32_t g = lane >> 2, t = lane & 3u;
    uint32_t xrow[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        const uint32_t bb = min(static_cast<uint32_t>(b), batch - 1u);
        xrow[b] = XM == 1 ? bb * xbytes : bb * xf_stride;
    }
    const uint8_t* xbase = XM == 1 ? xs : xf;
    double acc[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = 0.0;
    bool ok = true;
    uint32_t issued = min(len, static_cast<uint32_t>(DEPTH)), waited = 0;
    uint32_t oct = first / nkc, kc = first - oct * nkc;
    uint32_t kc_first = kc, nflush = 0;
    bool started = false;

    auto flush = [&](bool whole) {
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            double v = acc[b];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            if (t == 0 && static_cast<uint32_t>(b) < batch) {
                const uint32_t row = R * (o0 + oct) + g;
                if (whole) {
                    if (ok && row < rows) y[static_cast<size_t>(b) * y_stride + row] = static_cast<float>(v);
                } else {
                    const uint32_t e = cons * 2u + (nflush == 0 ? 0u : 1u);
                    bnd[b].v[e][g] = v;
                    if (g == 0) bnd[b].pair[e] = static_cast<int>(oct);
                }
            }
            acc[b] = 0.0;
        }
        ++nflush;
    };

    for (uint32_t i = 0; i < len; ++i) {
        const uint32_t slot = i % DEPTH;
        bool landed = ok && mbar_wait_spin(&full[slot], (i / DEPTH) & 1u, kFaultFullWait);
        if (XM == 1 && landed) landed = mbar_wait_spin(&xbar[kc], 0u, kFaultFullWait);
        landed = __all_sync(0xffffffffu, landed);
        if (!landed) ok = false;
        else waited = i + 1u;
        started = true;
        if (ok) {
            GemmTileRegs<T> r;
            gemm_tile_decode<T>(ring + slot * TB, lane, r);
            __syncwarp();
            if (lane == 0 && i + DEPTH < len) {
                fence_proxy_async_smem();
                issue(i + DEPTH);
                issued = i + DEPTH + 1u;
            }
            gemm_tile_rows<T, NB, 0, RG, XM == 0>(r, xbase + static_cast<size_t>(kc) * XC, xrow, lane, acc);
            if constexpr (NB > RG)
                gemm_tile_rows<T, NB, RG, NB - RG, XM == 0>(r, xbase + static_cast<size_t>(kc) * XC, xrow, lane, acc);
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
        for (uint32_t k = waited; k < issued; ++k)
            if (!mbar_wait(&full[k % DEPTH], (k / DEPTH) & 1u, kFaultDrain)) break;
    }
    if constexpr (XM == 1) {
        // every staged chunk lands before the CTA exits, used or not
        if (cons == 0 && lane == 0)
            for (uint32_t k = 0; k < nkc; ++k)
                if (!mbar_wait(&xbar[k], 0u, kFaultDrain)) break;
    }
    __syncthreads();
    if (threadIdx.x < 2u * C && ok)
        for (uint32_t b = 0; b < batch && b < static_cast<uint32_t>(NB); ++b)
            frag_boundary_combine<W>(bnd + b, threadIdx.x, o0, rows, y + static_cast<size_t>(b) * y_stride, nullptr);
}

}  // namespace q38
