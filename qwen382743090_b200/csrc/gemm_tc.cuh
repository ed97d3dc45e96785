// gemm_tc.cuh -- batched (multi-token verify / prefill) Q5_K / Q4_K GEMM on the
// fifth-generation tensor cores: tcgen05.mma kind::i8 with the accumulators in
// tensor memory (TMEM), over the B200 fragment tiles (Q38PACK layout 2).
//
//   Y[b][r] = sum_s d_rs * sum_g sc_rsg * <q_rsg, x_bsg> - dmin_rs * sum_g m_rsg * sum(x_bsg)
//
// the same mathematics as the reference's batch-1 kernels (q38_q5k_sm86_soa_gemv_vec,
// src/driver.cpp:3887-4138; q38_q4k_gemv_f32, :1857), here for up to 8 activation
// rows at once.
//
// Operands.  For one super-block s the CTA holds, in shared memory:
//   A = the 5-bit (Q5_K) / 4-bit (Q4_K) weight codes of 128 rows x 256 positions,
//       one unsigned byte each (odd groups x8 / x16, as the tiles store them),
//       decoded from the landed tiles by the CTA's warps;
//   B = the activation limbs: the exact integer round(x / unit) of every
//       activation row b split into four balanced signed bytes l (the x-pack
//       limbs), as N = 4 x slots columns n = 4b + l, written by xtc_pack_kernel
//       and landed by one bulk copy per K chunk.
// Both are K-major with no swizzle: 8-row x 16-byte core matrices, LBO = the step
// between core matrices along K, SBO = the step between 8-row groups.  One
// tcgen05.mma (M = 128, N, K = 32) per 32-weight group g writes the group's
// exact int32 dot products D_g[r][n] = <q_rg, limb_l(x_bg)> to its own N TMEM
// columns, so the group scale is applied afterwards in int32, exactly:
//   A8[r][b][l] = 8 sum_{g even} sc_g D_g + (sum_{g odd} sc_g D_g) >> oddshift.
// Eight groups x N columns per super-block, two super-blocks in flight: 16 N
// TMEM columns (512 for 8 rows, 256 for 4).
//
// Epilogue (12 warps): epilogue warp e reads TMEM lanes 32 (e % 4) .. +31 (its
// rows) for activation rows b = e / 4 + 3 j with tcgen05.ld 32x32b, applies the
// group scales in int32, joins the four limbs exactly in int64
// (sum_l A8_l 256^l), then applies d * unit / 8 in fp64; the dmin * m * sum(x)
// term is summed in fp32 and subtracted once per K chunk.
//
// Work split: a CTA owns 16 row octets (128 rows, the UMMA M) and a contiguous
// range of K chunks (2 super-blocks, one tile per octet); when there are fewer
// row blocks than SMs the K range is split into S slices, each CTA writes its
// fp64 partials to a workspace and the last CTA of a row block (counter in the
// workspace, zeroed by the pack kernel) adds them in slice order: deterministic.
//
// Pipeline (one CTA per SM, ~200 KB of shared memory, 16 N TMEM columns),
// warp-specialised so that decode, MMA and epilogue of neighbouring
// super-blocks overlap:
//   warps 0-7   decode super-block i (two octets each) into A[i % 2] and the
//               side buffer (scales, d / dmin, the x records), then arrive
//               a_full[i % 2] (and tile_empty after a chunk's second half);
//   warp 20     (one thread) waits a_full, the x stage and tmem_empty, issues
//               the 8 MMAs of i into TMEM stage i % 2 and commits them to
//               mma_done[i % 2] (plus x_empty after a chunk's last MMAs);
//   warps 8-19  wait mma_done, read TMEM stage i % 2, arrive tmem_empty;
//   warps 21-22 (one thread each) issue the tile copies (2 stages of 16 tiles,
//               the first two before the PDL wait) and the x copies (2 stages)
//               as soon as a stage is empty.  A bulk copy occupies the
//               issuing thread for tens of nanoseconds, so no thread on the
//               decode -> MMA -> epilogue path issues one.
// mma_done and x_empty also take a plain arrival of the control thread, which
// publishes what it acquired from the decoders (the side buffer) to the
// epilogue and the producers.  A parity wait is only safe if the barrier
// cannot complete two phases past the one awaited: each barrier's next phase
// here needs the waiting thread's own later progress.
// Every wait is bounded (the fault word records the site); TMEM is freed on
// every path after the last MMA has completed.
#pragma once

#include "gemv_frag.cuh"

namespace q38 {

constexpr uint32_t kTcRows = 128;                 // rows per CTA = TMEM lanes = UMMA M
constexpr uint32_t kTcOcts = kTcRows / kF8Rows;   // 16 row octets
constexpr uint32_t kTcDecWarps = 8;               // warps 0-7: tile copies + decode (2 octets each)
constexpr uint32_t kTcEpiWarps = 12;              // warps 8-19: TMEM read-back + scales (3 per lane quarter)
constexpr uint32_t kTcCtlWarp = kTcDecWarps + kTcEpiWarps;  // warp 20: MMA issue
constexpr uint32_t kTcProdWarp = kTcCtlWarp + 1u;  // warps 21, 22: tile and x copies (lane 0)
constexpr uint32_t kTcThreads = (kTcProdWarp + 2u) * 32u;
constexpr uint32_t kTcTileStages = 2;
constexpr uint32_t kTcXStages = 2;
constexpr uint32_t kTcSideBufs = 4;
constexpr uint32_t kTcABytes = kTcRows * 256u;    // one super-block of A: 32 KiB
constexpr uint32_t kTcMetaBytes = 64u;            // per activation row and super-block
constexpr uint32_t kTcMaxBatch = 8;

// Activation slots (UMMA N = 4 x slots): 4 for up to 4 rows, 8 for up to 8.
__host__ __device__ constexpr uint32_t tc_slots(uint32_t batch) { return batch <= 4u ? 4u : 8u; }
// Bytes of one super-block of packed activations: N x 256 limb bytes, then one
// 64-byte record per slot {double unit * 256^l / 8 [4]; float sum(x_g) [8]}.
__host__ __device__ constexpr uint32_t tc_xsb_bytes(uint32_t slots) { return slots * (1024u + kTcMetaBytes); }

template <uint32_t T, uint32_t SLOTS>
struct TcCfg {
    static constexpr uint32_t TB = FragTile<T>::kBytes;
    static constexpr uint32_t N = 4u * SLOTS;
    static constexpr uint32_t XSB = tc_xsb_bytes(SLOTS);
    static constexpr uint32_t LBOB = (N / 8u) * 128u;  // B: step between 16-byte K chunks
    static constexpr uint32_t kA = 0;  // two super-block buffers
    static constexpr uint32_t kTiles = 2u * kTcABytes;
    static constexpr uint32_t kX = kTiles + kTcTileStages * kTcOcts * TB;
    static constexpr uint32_t kSide = kX + kTcXStages * 2u * XSB;
    // per super-block: 16 scale/min bytes and d, dmin per row, then the slots' x records
    static constexpr uint32_t kSideRec = kTcRows * 20u;
    static constexpr uint32_t kSideBytes = kSideRec + SLOTS * kTcMetaBytes;
    static constexpr uint32_t kBars = kSide + kTcSideBufs * kSideBytes;
    static constexpr uint32_t kSmem = kBars + 128u;
    static constexpr uint32_t kTmemCols = 16u * N;  // 2 super-blocks x 8 groups x N
    static_assert(kTiles % 1024u == 0 && kX % 16u == 0 && XSB % 16u == 0 && kSide % 16u == 0 && kBars % 16u == 0,
                  "shared-memory carve alignment");
    static_assert(kTmemCols == 256u || kTmemCols == 512u, "TMEM allocation is a power of two");
};

// ---- tcgen05 building blocks ------------------------------------------------
// Shared-memory matrix descriptor, K-major, no swizzle (layout type 0), the
// sm_100 descriptor version 1 at bits 46-47; addresses and offsets >> 4.
__host__ __device__ constexpr uint64_t umma_smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3fffu) | (static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::i8: D s32 (bits 4-5 = 2), A unsigned 8-bit
// (bits 7-9 = 0), B signed 8-bit (bits 10-12 = 1), both K-major, N >> 3 at
// bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_u8s8(uint32_t m, uint32_t n) {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] = A x B (enable_d = 0) or D += A x B; one thread issues it.
__device__ __forceinline__ void umma_u8s8(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t enable_d) {
    const uint32_t mask = 0u;  // no output lane disabled
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(dtmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(enable_d), "r"(mask)
        : "memory");
}
// Arrive (once) on bar when every earlier tcgen05.mma of this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// Four consecutive 32-bit TMEM columns of this thread's lane (warp-wide).
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(taddr));
}
// tcgen05.wait::ld with eight loaded registers as operands, so that no use of
// them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld8(uint32_t (&r)[8]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])
                 :
                 : "memory");
}

// ---- activations: f32 rows -> UMMA B limbs + per-super-block records ----------
// One warp per (super-block, slot); rows b >= nbatch are zero.  The counters of
// the split-K combine are zeroed here (this kernel runs right before the GEMM).
template <uint32_t SLOTS>
__global__ void __launch_bounds__(256) xtc_pack_kernel(const float* __restrict__ x, uint32_t K, uint32_t nbatch,
                                                      uint8_t* __restrict__ xu, uint32_t* __restrict__ cnt,
                                                      uint32_t ncnt) {
    constexpr uint32_t N = 4u * SLOTS, XSB = tc_xsb_bytes(SLOTS), LBOB = (N / 8u) * 128u;
    pdl_wait();  // x comes from the stream's previous work; xu and cnt may still be read by the previous GEMM
    if (threadIdx.x == 0) pdl_launch_dependents();
    if (blockIdx.x == 0)
        for (uint32_t i = threadIdx.x; i < ncnt; i += blockDim.x) cnt[i] = 0u;
    const uint32_t nb = K / 256u;
    const uint32_t gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31u;
    if (gw >= nb * SLOTS) return;
    const uint32_t s = gw / SLOTS, b = gw % SLOTS;
    uint8_t* sbp = xu + static_cast<size_t>(s) * XSB;
    uint32_t lw[2][4] = {{0u, 0u, 0u, 0u}, {0u, 0u, 0u, 0u}};
    double gs = 0.0;
    float unit = 0.0f;
    if (b < nbatch) {
        const float* xp = x + static_cast<size_t>(b) * K + s * 256u + lane * 8u;
        const float4 a0 = __ldcg(reinterpret_cast<const float4*>(xp));
        const float4 a1 = __ldcg(reinterpret_cast<const float4*>(xp + 4));
        const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        gs = quantize_block_warp4(v, lw, &unit);
    }
    // element (n = 4b + l, k = 8 lane + 4h + j) = byte j of lw[h][l]
#pragma unroll
    for (uint32_t l = 0; l < 4u; ++l) {
        const uint32_t n = 4u * b + l;
        *reinterpret_cast<uint2*>(sbp + (lane >> 1) * LBOB + (n >> 3) * 128u + (n & 7u) * 16u + (lane & 1u) * 8u) =
            make_uint2(lw[0][l], lw[1][l]);
    }
    gs += __shfl_xor_sync(0xffffffffu, gs, 1);
    gs += __shfl_xor_sync(0xffffffffu, gs, 2);
    uint8_t* meta = sbp + N * 256u + b * kTcMetaBytes;
    if (lane < 4u)
        reinterpret_cast<double*>(meta)[lane] =
            static_cast<double>(unit) * static_cast<double>(1u << (8u * lane)) * 0.125;
    if ((lane & 3u) == 0u) reinterpret_cast<float*>(meta + 32u)[lane >> 2] = static_cast<float>(gs * static_cast<double>(unit));
}

// ---- the GEMM ------------------------------------------------------------------
// Warp `oct` decodes super-block `half` of its landed tile tb into A (rows
// 8 oct .. 8 oct + 7) and copies the rows' scales and d / dmin to the side buffer.
// Lane (g, t) holds positions 8t .. 8t+7 of each group: core matrix (K chunk
// 2G + t/2, row octet oct), bytes 16 g + 8 (t & 1).
template <uint32_t T>
__device__ __forceinline__ void tc_decode(const uint8_t* tb, uint32_t half, uint8_t* As, uint8_t* side, uint32_t oct,
                                          uint32_t lane) {
    static_assert(kTcRows * 20u % 16u == 0u, "side buffer records");
    using F = FragTile<T>;
    const uint32_t g = lane >> 2, t = lane & 3u;
    uint32_t h0 = 0u, h1 = 0u;
    if constexpr (T == 13u) {
        const uint4 qh = *reinterpret_cast<const uint4*>(tb + F::kQh + lane * 16u);
        h0 = half ? qh.z : qh.x;
        h1 = half ? qh.w : qh.y;
    }
    const uint4 qa = *reinterpret_cast<const uint4*>(tb + half * 1024u + lane * 16u);         // pairs 0, 1
    const uint4 qb = *reinterpret_cast<const uint4*>(tb + half * 1024u + 512u + lane * 16u);  // pairs 2, 3
    uint8_t* base = As + oct * 128u + g * 16u + (t & 1u) * 8u + (t >> 1) * 2048u;  // + 4096 per group
    uint32_t e0, o0, e1, o1;
    frag_decode<T, 0>(qa.x, h0, e0, o0);
    frag_decode<T, 0>(qa.y, h1, e1, o1);
    *reinterpret_cast<uint2*>(base + 0u * 4096u) = make_uint2(e0, e1);
    *reinterpret_cast<uint2*>(base + 1u * 4096u) = make_uint2(o0, o1);
    frag_decode<T, 1>(qa.z, h0, e0, o0);
    frag_decode<T, 1>(qa.w, h1, e1, o1);
    *reinterpret_cast<uint2*>(base + 2u * 4096u) = make_uint2(e0, e1);
    *reinterpret_cast<uint2*>(base + 3u * 4096u) = make_uint2(o0, o1);
    frag_decode<T, 2>(qb.x, h0, e0, o0);
    frag_decode<T, 2>(qb.y, h1, e1, o1);
    *reinterpret_cast<uint2*>(base + 4u * 4096u) = make_uint2(e0, e1);
    *reinterpret_cast<uint2*>(base + 5u * 4096u) = make_uint2(o0, o1);
    frag_decode<T, 3>(qb.z, h0, e0, o0);
    frag_decode<T, 3>(qb.w, h1, e1, o1);
    *reinterpret_cast<uint2*>(base + 6u * 4096u) = make_uint2(e0, e1);
    *reinterpret_cast<uint2*>(base + 7u * 4096u) = make_uint2(o0, o1);
    if (t == 0u) {
        const uint32_t r = oct * kF8Rows + g;
        *reinterpret_cast<uint4*>(side + r * 16u) = *reinterpret_cast<const uint4*>(tb + F::kSc + half * 128u + g * 16u);
        *reinterpret_cast<uint32_t*>(side + kTcRows * 16u + r * 4u) =
            *reinterpret_cast<const uint32_t*>(tb + F::kDm + half * 32u + g * 4u);
    }
}

// w: layout-2 tiles; xu: xtc_pack_kernel's output; y: [nbatch][rows];
// part / cnt: split-K workspace (S > 1).  Grid = (row blocks) x S.
template <uint32_t T, uint32_t SLOTS>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ xu, float* __restrict__ y,
                   double* __restrict__ part, uint32_t* __restrict__ cnt, uint32_t rows, uint32_t nb,
                   uint32_t nbatch, uint32_t S) {
    using C = TcCfg<T, SLOTS>;
    using F = FragTile<T>;
    constexpr uint32_t N = C::N, TB = C::TB, XSB = C::XSB, NJ = (SLOTS + 2u) / 3u;  // activation rows per thread
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* sA = smem + C::kA;
    uint8_t* sT = smem + C::kTiles;
    uint8_t* sX = smem + C::kX;
    uint8_t* sSide = smem + C::kSide;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBars);
    uint64_t* tile_full = bars;        // [2] one arrival per octet
    uint64_t* x_full = bars + 2;       // [2] control thread
    uint64_t* a_full = bars + 4;       // [2] every decoder thread
    uint64_t* mma_done = bars + 6;     // [2] the commit + the control thread
    uint64_t* tmem_empty = bars + 8;   // [2] every epilogue thread
    uint64_t* tile_empty = bars + 10;  // [2] every decoder thread, after a chunk's second half
    uint64_t* x_empty = bars + 12;     // [2] the commit of a chunk's last MMAs + the control thread
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 14);
    volatile uint32_t* sfail = tslot + 1;
    volatile uint32_t* slast = tslot + 2;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t nkc = nb / 2u, nocts = (rows + kF8Rows - 1u) / kF8Rows;
    const uint32_t rb = blockIdx.x / S, sl = blockIdx.x % S;
    const uint32_t o0 = rb * kTcOcts, octs = min(kTcOcts, nocts - o0);
    const uint32_t cbase = nkc / S, crem = nkc % S;
    const uint32_t c0 = sl * cbase + min(sl, crem), nch = cbase + (sl < crem ? 1u : 0u);
    const uint32_t nsb = 2u * nch;

    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < 2u; ++i) {
            mbar_init(&tile_full[i], octs);
            mbar_init(&x_full[i], 1);
            mbar_init(&a_full[i], kTcDecWarps * 32u);
            mbar_init(&mma_done[i], 2);  // the MMAs' commit + the control thread's release
            mbar_init(&tmem_empty[i], kTcEpiWarps * 32u);
            mbar_init(&tile_empty[i], kTcDecWarps * 32u);
            mbar_init(&x_empty[i], 2);
        }
        *sfail = 0u;
        *slast = 0u;
        fence_mbar_init();
    }
    if (warp == kTcCtlWarp) {
        tmem_alloc(tslot, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    // bounded wait; false (and the CTA's failure flag set) when it gave up or
    // another role already failed, so every role leaves its loop
    auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        if (*sfail) return false;
        if (mbar_wait_spin(bar, parity, kFaultFullWait)) return true;
        *sfail = 1u;
        return false;
    };
    // Parity waits are safe only if the barrier cannot complete two phases past
    // the one waited for; every wait below is on a barrier whose next phase
    // needs this thread's own later progress.
    // the same for a whole warp: every lane leaves together
    auto wait_warp = [&](uint64_t* bar, uint32_t parity) -> bool {
        return __all_sync(0xffffffffu, wait(bar, parity));
    };

    // per-thread copy bookkeeping (for the drain on a failed wait)
    uint32_t t_issued = 0, x_issued = 0, mma_issued = 0;
    const uint32_t oa = 2u * warp, ob = 2u * warp + 1u;  // a decoder warp's octets
    // producer warp p (0 or 1) copies the tiles of octets 8p .. 8p + 7
    const uint32_t pw = warp - kTcProdWarp, pbeg = 8u * pw, pend = min(8u * pw + 8u, octs);
    auto issue_tiles = [&](uint32_t k) {
        uint64_t* bar = &tile_full[k % kTcTileStages];
        uint8_t* dst = sT + (k % kTcTileStages) * (kTcOcts * TB);
        for (uint32_t o = pbeg; o < pend; ++o) {
            mbar_arrive_expect_tx(bar, TB);
            tma_load_1d(dst + o * TB, w + ((static_cast<size_t>(o0) + o) * nkc + c0 + k) * TB, TB, bar);
        }
        t_issued = k + 1u;
    };
    auto issue_x = [&](uint32_t k) {
        uint64_t* bar = &x_full[k % kTcXStages];
        mbar_arrive_expect_tx(bar, 2u * XSB);
        tma_load_1d(sX + (k % kTcXStages) * 2u * XSB, xu + static_cast<size_t>(c0 + k) * 2u * XSB, 2u * XSB, bar);
        x_issued = k + 1u;
    };

    double acc[NJ];
    float mn[NJ];
#pragma unroll
    for (uint32_t j = 0; j < NJ; ++j) {
        acc[j] = 0.0;
        mn[j] = 0.0f;
    }
    // epilogue warp e = warp - 8: TMEM lane quarter e % 4, activation rows e / 4 + 3 j
    const uint32_t q4 = warp & 3u, row = 32u * q4 + lane, bsel = (warp - kTcDecWarps) >> 2;

    if (warp < kTcDecWarps) {
        // ---- decoders: tiles -> A[i % 2] and the side buffer of super-block i ----
        for (uint32_t i = 0; i < nsb; ++i) {
            const uint32_t k = i >> 1, half = i & 1u;
            if (half == 0u && !wait_warp(&tile_full[k % kTcTileStages], (k / kTcTileStages) & 1u)) break;
            if (half == 0u && !wait_warp(&x_full[k % kTcXStages], (k / kTcXStages) & 1u)) break;
            // A[i % 2] was read by the MMAs of i - 2; side[i % 4] by the epilogue of
            // i - 4, which finished before those MMAs were issued
            if (i >= 2u && !wait_warp(&mma_done[i & 1u], ((i - 2u) >> 1) & 1u)) break;
            uint8_t* side = sSide + (i % kTcSideBufs) * C::kSideBytes;
            const uint8_t* stage = sT + (k % kTcTileStages) * (kTcOcts * TB);
            uint8_t* As = sA + (i & 1u) * kTcABytes;
            if (oa < octs) tc_decode<T>(stage + oa * TB, half, As, side, oa, lane);
            if (ob < octs) tc_decode<T>(stage + ob * TB, half, As, side, ob, lane);
            if (threadIdx.x < SLOTS * kTcMetaBytes / 16u)  // this super-block's x records
                reinterpret_cast<uint4*>(side + C::kSideRec)[threadIdx.x] = reinterpret_cast<const uint4*>(
                    sX + (k % kTcXStages) * 2u * XSB + half * XSB + N * 256u)[threadIdx.x];
            fence_proxy_async_smem();  // A is read by the tensor cores (async proxy)
            mbar_arrive(&a_full[i & 1u]);
            if (half == 1u) mbar_arrive(&tile_empty[k % kTcTileStages]);  // chunk k's stage is read
        }
    } else if (warp < kTcCtlWarp) {
        // ---- epilogue: TMEM stage i % 2 -> group scales (int32) -> fp64 sums ----
        pdl_wait();  // y and the split-K partials belong to the dependency chain
        for (uint32_t i = 0; i < nsb; ++i) {
            const uint32_t half = i & 1u;
            // warp-uniform for the .sync.aligned loads; the control thread's
            // arrival on mma_done also publishes the decoders' side buffer
            if (!wait_warp(&mma_done[i & 1u], (i >> 1) & 1u)) break;
            tc_fence_after();
            const uint8_t* side = sSide + (i % kTcSideBufs) * C::kSideBytes;
            const uint4 sc = *reinterpret_cast<const uint4*>(side + row * 16u);
            const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(side + kTcRows * 16u + row * 4u));
            const uint8_t* xrec = side + C::kSideRec;
            const uint32_t taddr = tmem + ((32u * q4) << 16) + (i & 1u) * 8u * N;
            // the row's eight mins as floats, shared by its activation rows
            float mf[8];
#pragma unroll
            for (uint32_t g = 0; g < 8u; ++g) mf[g] = byte_f(g < 4u ? sc.z : sc.w, 0x7640u | (g & 3u));
#pragma unroll
            for (uint32_t j = 0; j < NJ; ++j) {
                const uint32_t b = bsel + 3u * j;
                if (b >= nbatch) continue;  // warp-uniform
                uint32_t D[4][8];           // D[l][G]
#pragma unroll
                for (uint32_t G = 0; G < 8u; ++G) tmem_ld4(taddr + G * N + 4u * b, D[0][G], D[1][G], D[2][G], D[3][G]);
#pragma unroll
                for (uint32_t l = 0; l < 4u; ++l) tmem_wait_ld8(D[l]);
                const uint8_t* meta = xrec + b * kTcMetaBytes;
                const double unw0 = *reinterpret_cast<const double*>(meta);  // unit / 8 (limb 0)
                const float4 xa = *reinterpret_cast<const float4*>(meta + 32u);
                const float4 xb = *reinterpret_cast<const float4*>(meta + 48u);
                const float xsum[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
                // sum over the limbs l of A8_l 256^l in int64 (|A8_l| < 2^30), exact
                long long A = 0;
#pragma unroll
                for (uint32_t l = 0; l < 4u; ++l) {
                    int Ae = 0, Ao = 0;
                    Ae += byte_u<0>(sc.x) * static_cast<int>(D[l][0]);
                    Ao += byte_u<1>(sc.x) * static_cast<int>(D[l][1]);
                    Ae += byte_u<2>(sc.x) * static_cast<int>(D[l][2]);
                    Ao += byte_u<3>(sc.x) * static_cast<int>(D[l][3]);
                    Ae += byte_u<0>(sc.y) * static_cast<int>(D[l][4]);
                    Ao += byte_u<1>(sc.y) * static_cast<int>(D[l][5]);
                    Ae += byte_u<2>(sc.y) * static_cast<int>(D[l][6]);
                    Ao += byte_u<3>(sc.y) * static_cast<int>(D[l][7]);
                    const int A8 = Ae * 8 + (Ao >> F::kOddShift);
                    A += static_cast<long long>(A8) * (1ll << (8u * l));
                }
                acc[j] = __fma_rn(static_cast<double>(A), static_cast<double>(dm.x) * unw0, acc[j]);
                // the min term: dmin * sum_g m_g sum(x_g), subtracted once per chunk
                float pm = mf[0] * xsum[0];
#pragma unroll
                for (uint32_t g = 1; g < 8u; ++g) pm = fmaf(mf[g], xsum[g], pm);
                mn[j] = fmaf(dm.y, pm, mn[j]);
                if (half) {
                    acc[j] -= static_cast<double>(mn[j]);
                    mn[j] = 0.0f;
                }
            }
            tc_fence_before();
            mbar_arrive(&tmem_empty[i & 1u]);
        }
    } else if (warp == kTcCtlWarp && lane == 0u) {
        // ---- control: the MMAs (one thread) ----
        pdl_launch_dependents();
        const uint32_t idesc = umma_idesc_u8s8(kTcRows, N);
        for (uint32_t i = 0; i < nsb; ++i) {
            const uint32_t k = i >> 1, half = i & 1u;
            if (!wait(&a_full[i & 1u], (i >> 1) & 1u)) break;
            if (half == 0u && !wait(&x_full[k % kTcXStages], (k / kTcXStages) & 1u)) break;
            if (i >= 2u && !wait(&tmem_empty[i & 1u], ((i - 2u) >> 1) & 1u)) break;
            tc_fence_after();
            const uint32_t a_base = smem_u32(sA + (i & 1u) * kTcABytes);
            const uint32_t b_base = smem_u32(sX + (k % kTcXStages) * 2u * XSB + half * XSB);
            const uint32_t d_base = tmem + (i & 1u) * 8u * N;
#pragma unroll
            for (uint32_t G = 0; G < 8u; ++G)
                umma_u8s8(d_base + G * N, umma_smem_desc(a_base + G * 4096u, 2048u, 128u),
                          umma_smem_desc(b_base + G * 2u * C::LBOB, C::LBOB, 128u), idesc, 0u);
            umma_commit(&mma_done[i & 1u]);
            mbar_arrive(&mma_done[i & 1u]);  // release: what this thread acquired from the decoders
            if (half == 1u) {
                // chunk k's x stage is free once its last MMAs completed (its records were copied at decode)
                umma_commit(&x_empty[k % kTcXStages]);
                mbar_arrive(&x_empty[k % kTcXStages]);
            }
            mma_issued = i + 1u;
        }
    } else if (warp >= kTcProdWarp && lane == 0u) {
        // ---- producers: tile copies (both warps) and x copies (the first), off the critical path ----
        for (uint32_t k = 0; k < kTcTileStages && k < nch; ++k) issue_tiles(k);  // before the PDL wait
        if (pw == 0u) {
            pdl_wait();  // the packed activations come from the previous kernel
            for (uint32_t k = 0; k < kTcXStages && k < nch; ++k) issue_x(k);
        }
        for (uint32_t k = kTcTileStages; k < nch; ++k) {
            if (!wait(&tile_empty[k % kTcTileStages], ((k - kTcTileStages) / kTcTileStages) & 1u)) break;
            issue_tiles(k);
            if (pw == 0u && k >= kTcXStages) {
                if (!wait(&x_empty[k % kTcXStages], ((k - kTcXStages) / kTcXStages) & 1u)) break;
                issue_x(k);
            }
        }
    }

    // ---- teardown: every MMA complete, every copy landed, TMEM freed ----
    __syncthreads();
    const bool ok = *sfail == 0u;
    if (!ok && lane == 0u) {
        if (warp == kTcCtlWarp && mma_issued)
            (void)mbar_wait(&mma_done[(mma_issued - 1u) & 1u], ((mma_issued - 1u) >> 1) & 1u, kFaultDrain);
        for (uint32_t k = 0; k < t_issued; ++k)
            if (!mbar_wait(&tile_full[k % kTcTileStages], (k / kTcTileStages) & 1u, kFaultDrain)) break;
        for (uint32_t k = 0; k < x_issued; ++k)
            if (!mbar_wait(&x_full[k % kTcXStages], (k / kTcXStages) & 1u, kFaultDrain)) break;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTcCtlWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
    if (warp < kTcDecWarps || warp == kTcCtlWarp) {
        if (S == 1u) return;
    }

    // ---- output (epilogue warps): (l0 + l1) + (l2 + l3) per row and activation row ----
    const bool epi = warp >= kTcDecWarps && warp < kTcCtlWarp;
    const uint32_t grow = o0 * kF8Rows + row;
    const bool rvalid = epi && row < octs * kF8Rows && grow < rows;
    if (S == 1u) {
#pragma unroll
        for (uint32_t j = 0; j < NJ; ++j) {
            const uint32_t b = bsel + 3u * j;
            if (ok && rvalid && b < nbatch) y[static_cast<size_t>(b) * rows + grow] = static_cast<float>(acc[j]);
        }
        return;
    }
    const uint32_t nrb = (nocts + kTcOcts - 1u) / kTcOcts;
    const size_t rowsp = static_cast<size_t>(nrb) * kTcRows;
#pragma unroll
    for (uint32_t j = 0; j < NJ; ++j) {
        const uint32_t b = bsel + 3u * j;
        if (rvalid && b < nbatch) part[(static_cast<size_t>(sl) * SLOTS + b) * rowsp + grow] = acc[j];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == kTcDecWarps * 32u) *slast = (atomicAdd(&cnt[rb], 1u) == S - 1u) ? 1u : 0u;  // after its PDL wait
    __syncthreads();
    if (*slast == 0u) return;
    __threadfence();
    // the last CTA of the row block adds the slices in order
#pragma unroll
    for (uint32_t j = 0; j < NJ; ++j) {
        const uint32_t b = bsel + 3u * j;
        if (!rvalid || b >= nbatch) continue;
        double v = __ldcg(part + static_cast<size_t>(b) * rowsp + grow);
        for (uint32_t u = 1; u < S; ++u) v += __ldcg(part + (static_cast<size_t>(u) * SLOTS + b) * rowsp + grow);
        y[static_cast<size_t>(b) * rows + grow] = static_cast<float>(v);
    }
}

}  // namespace q38
