// gemv_soa_frag.cuh -- Q5_K GEMV straight from the reference's SoA planes
// (Q38PACK layout 1: META20 / QH32 / QS128 per super-block in three row-major
// planes, tools/gguf_to_q38pack.py:240-300), with the structure of the
// fragment-tile kernel (gemv_frag.cuh) instead of the reference's
// warp-per-row loop (q38_q5k_sm86_soa_gemv_vec, src/driver.cpp:3887-4138).
//
// A tile is 8 rows x 4 super-blocks: six 2-D TMA boxes of 8 rows -- QS one
// 8 x 128 B box per super-block and QH one 8 x 128 B box, both with the
// 128-byte swizzle (a row's 16-byte chunks XOR-permuted by the row index, so
// the 8 rows a warp reads at the same offset fall in different banks), and
// META one 8 x 80 B box (80 B is the smallest META box whose width is a
// multiple of 16 bytes, hence 4 super-blocks).  Each consumer warp
// owns a ring of DEPTH tile slots and issues its own copies before the PDL
// wait; its lane (g, t) reads row g's bytes 8t..8t+7 of every group pair and
// builds the same mma.sync.m16n8k32 A fragments as the tiled layout (even
// group: its 5-bit weights; odd group: its weights times 8, the fifth bit
// moved into bit 7), so the integer sums, the group scaling and the fp64
// block epilogue are those of gemv_frag_cta, against the same x-fragments.
// Rows of the last octet past `rows` are zero-filled by the copies and never
// stored.
#pragma once

#include "gemv_frag.cuh"

namespace q38 {

constexpr uint32_t kSfRows = 8, kSfBlocks = 4;
constexpr uint32_t kSfQs = kSfRows * kSfBlocks * 128;   // 4 x [8 rows][128 B], swizzled
constexpr uint32_t kSfQh = kSfRows * kSfBlocks * 32;    // [8 rows][128 B], swizzled
constexpr uint32_t kSfMeta = kSfRows * kSfBlocks * 20;  // [8 rows][80 B]
constexpr uint32_t kSfTxBytes = kSfQs + kSfQh + kSfMeta;  // 5760 bytes landed per tile
constexpr uint32_t kSfTile = 6144;                        // slot: swizzled boxes start on 1 KiB

// 8-row boxes of the three planes (uint32 elements; QS and QH 128-byte swizzled).
struct SoaFragMaps {
    CUtensorMap qs, qh, meta;
};

template <int W, int DEPTH>
__host__ __device__ constexpr size_t soa_frag_fixed_bytes() {
    return 1024 + static_cast<size_t>(W) * DEPTH * kSfTile + W * DEPTH * 8 + 8 + sizeof(PairBoundary<W, kF8Rows>) +
           256;
}

// Byte offset of row g's 16-byte chunk c in an 8 x 128 B box written with the
// 128-byte swizzle (chunk index XOR row index).
__device__ __forceinline__ uint32_t sw128(uint32_t g, uint32_t c) { return g * 128u + ((c ^ g) << 4); }
template <int W, int DEPTH>
__host__ __device__ constexpr size_t soa_frag_smem_bytes(uint32_t nb, bool xsmem) {
    return soa_frag_fixed_bytes<W, DEPTH>() + (xsmem ? xfrag1_bytes(nb) : 0u);
}

// Pair p's 5-bit weights of four positions as mma A bytes: the even group
// (2p) as is, the odd group (2p+1) times 8.  q: QS word (low nibble = group
// 2p, high nibble = group 2p+1); h: the QH bytes of the same positions (bit
// 2p / 2p+1 = the fifth bits).
template <uint32_t P>
__device__ __forceinline__ void soa_decode(uint32_t q, uint32_t h, uint32_t& even, uint32_t& odd) {
    even = (q & 0x0f0f0f0fu) | (rotl(h, (4u - 2u * P) & 31u) & 0x10101010u);
    odd = ((q & 0xf0f0f0f0u) >> 1) | (rotl(h, (6u - 2u * P) & 31u) & 0x80808080u);
}

// One lane's share of a landed tile added to its fp64 sum (row g, limb t):
// the four super-blocks in order, each exactly as frag_tile_acc does one.
// tb: the tile's slot; xb: the x-fragments of its first super-block.
template <bool XL2, class AfterLoad>
__device__ __forceinline__ void soa_tile_acc(const uint8_t* tb, const uint8_t* xb, uint32_t lane, double& acc,
                                             AfterLoad&& after_load) {
    const uint32_t g = lane >> 2, t = lane & 3u;
    uint2 qv[kSfBlocks][4];
    uint2 hv[kSfBlocks];
    uint32_t dmw[kSfBlocks], scw[kSfBlocks][4];
#pragma unroll
    for (uint32_t s = 0; s < kSfBlocks; ++s) {
#pragma unroll
        for (uint32_t p = 0; p < 4u; ++p)
            qv[s][p] = *reinterpret_cast<const uint2*>(tb + s * 1024u + sw128(g, 2u * p + (t >> 1)) + (t & 1u) * 8u);
        hv[s] = *reinterpret_cast<const uint2*>(tb + kSfQs + sw128(g, 2u * s + (t >> 1)) + (t & 1u) * 8u);
        const uint32_t* m = reinterpret_cast<const uint32_t*>(tb + kSfQs + kSfQh + g * 80u + s * 20u);
        dmw[s] = m[0];
#pragma unroll
        for (uint32_t k = 0; k < 4u; ++k) scw[s][k] = m[1 + k];  // sc, mn of groups 2k and 2k+1
    }
    after_load();
    float mn = 0.0f;
#pragma unroll
    for (uint32_t s = 0; s < kSfBlocks; ++s) {
        const uint8_t* xbs = xb + s * kXfBlockBytes;
        int Ae = 0, Ao = 0;
#pragma unroll
        for (uint32_t c = 0; c < 2u; ++c) {
            const uint8_t* xp = xbs + c * 512u + lane * 16u;
            const uint4 xv = XL2 ? __ldcg(reinterpret_cast<const uint4*>(xp)) : *reinterpret_cast<const uint4*>(xp);
            uint32_t e0, o0, e1, o1;
            int d0, d3;
            const uint2 qa = qv[s][2u * c], qb = qv[s][2u * c + 1u];
            const uint32_t wa = scw[s][2u * c], wb = scw[s][2u * c + 1u];
            if (c == 0) {
                soa_decode<0>(qa.x, hv[s].x, e0, o0);
                soa_decode<0>(qa.y, hv[s].y, e1, o1);
            } else {
                soa_decode<2>(qa.x, hv[s].x, e0, o0);
                soa_decode<2>(qa.y, hv[s].y, e1, o1);
            }
            mma_u8s8_16x8x32(d0, d3, e0, o0, e1, o1, xv.x, xv.y);
            Ae += byte_u<0>(wa) * d0;  // scale of group 4c
            Ao += byte_u<2>(wa) * d3;  // scale of group 4c+1
            if (c == 0) {
                soa_decode<1>(qb.x, hv[s].x, e0, o0);
                soa_decode<1>(qb.y, hv[s].y, e1, o1);
            } else {
                soa_decode<3>(qb.x, hv[s].x, e0, o0);
                soa_decode<3>(qb.y, hv[s].y, e1, o1);
            }
            mma_u8s8_16x8x32(d0, d3, e0, o0, e1, o1, xv.z, xv.w);
            Ae += byte_u<0>(wb) * d0;  // group 4c+2
            Ao += byte_u<2>(wb) * d3;  // group 4c+3
        }
        const int A8 = Ae * 8 + Ao;
        const uint4 xm = XL2 ? __ldcg(reinterpret_cast<const uint4*>(xbs + kXfMetaOff + t * 16u))
                             : *reinterpret_cast<const uint4*>(xbs + kXfMetaOff + t * 16u);
        const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&dmw[s]));
        const double unw = __hiloint2double(static_cast<int>(xm.y), static_cast<int>(xm.x));
        acc = __fma_rn(static_cast<double>(A8), static_cast<double>(dm.x) * unw, acc);
        // pair t's mins: groups 2t and 2t+1 = bytes 1 and 3 of META word t
        const uint32_t mw = scw[s][t];
        const float pm = fmaf(static_cast<float>(byte_u<1>(mw)), __uint_as_float(xm.z),
                              static_cast<float>(byte_u<3>(mw)) * __uint_as_float(xm.w));
        mn = fmaf(dm.y, pm, mn);
    }
    acc -= static_cast<double>(mn);
}

// XM 1: x-fragments copied to shared memory by one bulk copy per CTA; XM 2:
// xf is f32 x, packed into x-fragments by every CTA (nb <= kF8PackPerWarp * W).
// One CTA's work: row octets split evenly over the grid, its tiles (octet,
// 4-block chunk; chunk fastest) split evenly over the W warps.
template <int XM, int W, int DEPTH, int MINB>
__global__ void __launch_bounds__(W * 32, MINB)
    gemv_soa_frag_kernel(const __grid_constant__ SoaFragMaps maps, const uint8_t* __restrict__ xf, float* y,
                         uint32_t rows, uint32_t nb) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t C = W, R = kF8Rows, TB = kSfTile;
    uint8_t* tiles = smem + ((1024u - (reinterpret_cast<uintptr_t>(smem) & 1023u)) & 1023u);
    uint64_t* bars = reinterpret_cast<uint64_t*>(tiles + static_cast<size_t>(W) * DEPTH * TB);
    uint64_t* xbar = bars + C * DEPTH;
    PairBoundary<W, R>* bnd = reinterpret_cast<PairBoundary<W, R>*>(xbar + 1);
    uint8_t* xs = reinterpret_cast<uint8_t*>(bnd + 1);
    xs += (128u - (reinterpret_cast<uintptr_t>(xs) & 127u)) & 127u;

    if (threadIdx.x == 0) pdl_launch_dependents();
    const uint32_t cta = blockIdx.x, ncta = gridDim.x;
    const uint32_t cons = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t nocts = (rows + R - 1u) / R, nkc = nb / kSfBlocks;
    const uint32_t obase = nocts / ncta, orem = nocts % ncta;
    const uint32_t o0 = cta * obase + min(cta, orem);
    const uint32_t o1 = o0 + obase + (cta < orem ? 1u : 0u);
    const uint32_t ntiles = (o1 - o0) * nkc;
    const uint32_t base = ntiles / C, rem = ntiles % C;
    const uint32_t len = base + (cons < rem ? 1u : 0u);
    const uint32_t first = cons * base + min(cons, rem);
    uint8_t* ring = tiles + static_cast<size_t>(cons) * DEPTH * TB;
    uint64_t* full = bars + cons * DEPTH;
    auto issue = [&](uint32_t k) {
        const uint32_t tile = first + k, oc = o0 + tile / nkc, kc = tile % nkc;
        uint8_t* dst = ring + (k % DEPTH) * TB;
        const int32_t r = static_cast<int32_t>(oc * R);
        mbar_arrive_expect_tx(&full[k % DEPTH], kSfTxBytes);
        for (uint32_t s = 0; s < kSfBlocks; ++s)
            tma_load_2d(dst + s * 1024u, &maps.qs, static_cast<int32_t>((kc * kSfBlocks + s) * 32u), r,
                        &full[k % DEPTH]);
        tma_load_2d(dst + kSfQs, &maps.qh, static_cast<int32_t>(kc * 32u), r, &full[k % DEPTH]);
        tma_load_2d(dst + kSfQs + kSfQh, &maps.meta, static_cast<int32_t>(kc * 20u), r, &full[k % DEPTH]);
    };
    if (lane == 0) {
        for (uint32_t i = 0; i < DEPTH; ++i) mbar_init(&full[i], 1);
        if (XM == 1 && cons == 0) mbar_init(xbar, 1);
        fence_mbar_init();
        for (uint32_t k = 0; k < DEPTH && k < len; ++k) issue(k);
    }
    if (threadIdx.x < 2 * C) bnd->pair[threadIdx.x] = -1;
    __syncthreads();

    pdl_wait();  // x and y belong to the dependency chain
    if constexpr (XM == 2) {
        frag_pack_x_f32<W>(reinterpret_cast<const float*>(xf), nb, xs, cons, lane);
        __syncthreads();
    } else {
        if (threadIdx.x == 0) {
            const uint32_t bytes = static_cast<uint32_t>(xfrag1_bytes(nb));
            mbar_arrive_expect_tx(xbar, bytes);
            tma_load_1d(xs, xf, bytes, xbar);
        }
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

    // an octet's 8 outputs leave as two 16-byte stores when y allows it
    const bool y16 = (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
    auto flush = [&](bool whole) {
        double v = acc;  // after the two exchanges every lane of row g holds the same sum
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        const uint32_t row0 = R * (o0 + oct), row = row0 + g;
        if (whole) {
            const float out = static_cast<float>(v);
            const float o1 = __shfl_down_sync(0xffffffffu, out, 4);
            const float o2 = __shfl_down_sync(0xffffffffu, out, 8);
            const float o3 = __shfl_down_sync(0xffffffffu, out, 12);
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
            soa_tile_acc<false>(ring + slot * TB, xs + static_cast<size_t>(kc) * (kSfBlocks * kXfBlockBytes), lane,
                                acc, [&] {
                                    __syncwarp();
                                    if (lane == 0 && i + DEPTH < len) {
                                        fence_proxy_async_smem();
                                        issue(i + DEPTH);
                                        issued = i + DEPTH + 1u;
                                    }
                                });
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
    __syncthreads();
    if (threadIdx.x < 2u * C && ok) frag_boundary_combine<W>(bnd, threadIdx.x, o0, rows, y, nullptr);
}

}  // namespace q38
