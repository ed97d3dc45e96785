// engine_kernels.cuh -- device kernels of the decode engine beyond the GEMVs
// and the recurrent core: seeded synthetic weights, the on-device repack into
// the B200 tiled layout, producers that emit x-packs (RMSNorm, SiLU*up), the
// token embedding, full-attention prep and split-K decode attention, and the
// greedy argmax.  The reference has no full-model decode (src/runtime.cpp:74-76);
// the attention layer follows the geometry the reference records for the
// real model (README.md:1160-1175): 24 query heads of 256 with a 256-wide
// output gate each, 4 KV heads, fp16 KV cache.
#pragma once

#include "gemv_frag.cuh"
#include "layer.cuh"
#include "xpack.cuh"

namespace q38 {

// ---- seeded synthetic data ------------------------------------------------------
// splitmix64 (Steele, Lea, Flood 2014) as a counter-based generator: value i
// of stream s is mix(s + (i+1) * golden).
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
struct Rng {
    uint64_t s;
    __device__ explicit Rng(uint64_t stream) : s(mix64(stream)) {}
    __device__ uint64_t next() {
        s += 0x9e3779b97f4a7c15ull;
        return mix64(s);
    }
    __device__ double uniform() { return (static_cast<double>(next() >> 11) + 0.5) * 0x1.0p-53; }  // (0,1)
    __device__ double normal() {  // Box-Muller
        const double u1 = uniform(), u2 = uniform();
        return sqrt(-2.0 * log(u1)) * cospi(2.0 * u2);
    }
};

__device__ __forceinline__ uint16_t half_scale(Rng& r) {
    return __half_as_ushort(__float2half_rn(static_cast<float>(fabs(r.normal()) * 0x1.0p-8)));
}

// One GGUF block per thread (layout 0) of type 12/13/14/23 with the benchmark
// distributions: d, dmin = fp16(|N(0,1)| 2^-8); 6-bit scales and mins uniform,
// packed with the inverse of get_scale_min_k4; quant bytes uniform; Q6_K int8
// scales uniform; IQ4_XS scale bits uniform.
//
// The bytes of a block depend only on (seed, global block index), so a shard
// of a matrix is generated directly: local block (i, b) of a rows x nb matrix
// is global block row_map[i] * nb_g + kb_map[b] (identity maps when null); a
// negative kb_map entry makes an all-zero padding block.
__global__ void synth_blocks_kernel(uint32_t type, uint8_t* __restrict__ out, uint32_t rows, uint32_t nb,
                                    const uint32_t* __restrict__ row_map, const int32_t* __restrict__ kb_map,
                                    uint32_t nb_g, uint64_t seed) {
    const uint64_t blk = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (blk >= static_cast<uint64_t>(rows) * nb) return;
    const uint32_t bb = type == 12 ? 144u : type == 13 ? 176u : type == 14 ? 210u : 136u;
    uint8_t* o = out + blk * bb;
    const uint32_t i = static_cast<uint32_t>(blk / nb), b = static_cast<uint32_t>(blk % nb);
    const int32_t gb = kb_map ? kb_map[b] : static_cast<int32_t>(b);
    if (gb < 0) {
        for (uint32_t k = 0; k < bb; ++k) o[k] = 0;
        return;
    }
    const uint64_t gblk = static_cast<uint64_t>(row_map ? row_map[i] : i) * nb_g + static_cast<uint32_t>(gb);
    Rng r(seed * 0x2545f4914f6cdd1dull + gblk);
    auto fill = [&](uint32_t from, uint32_t to) {
        for (uint32_t k0 = from; k0 < to; k0 += 8) {
            const uint64_t v = r.next();
            for (uint32_t k = 0; k < 8 && k0 + k < to; ++k) o[k0 + k] = static_cast<uint8_t>(v >> (8 * k));
        }
    };
    if (type == 12 || type == 13) {
        const uint16_t d = half_scale(r), dm = half_scale(r);
        o[0] = d & 255u; o[1] = d >> 8; o[2] = dm & 255u; o[3] = dm >> 8;
        uint8_t sc[8], mn[8];
        const uint64_t v = r.next(), w = r.next();
        for (int j = 0; j < 8; ++j) {
            sc[j] = static_cast<uint8_t>((v >> (6 * j)) & 63u);
            mn[j] = static_cast<uint8_t>((w >> (6 * j)) & 63u);
        }
        for (int j = 0; j < 4; ++j) {
            o[4 + j] = static_cast<uint8_t>((sc[j] & 63u) | ((sc[4 + j] >> 4) << 6));
            o[8 + j] = static_cast<uint8_t>((mn[j] & 63u) | ((mn[4 + j] >> 4) << 6));
            o[12 + j] = static_cast<uint8_t>((sc[4 + j] & 15u) | ((mn[4 + j] & 15u) << 4));
        }
        fill(16, bb);
    } else if (type == 14) {
        fill(0, 208);
        const uint16_t d = half_scale(r);
        o[208] = d & 255u;
        o[209] = d >> 8;
    } else {
        const uint16_t d = half_scale(r);
        o[0] = d & 255u;
        o[1] = d >> 8;
        fill(2, 136);
    }
}

// f32 values mean + std * N(0,1), or -exp(N(0,1)) (ssm_a) when neg_exp.
// Element i is global element map(i): chunk_map[i / chunk] * chunk + i % chunk
// (identity when chunk_map is null), so shards match the whole tensor.
__global__ void synth_f32_kernel(float* __restrict__ out, uint64_t n, uint64_t seed, float mean, float stdev,
                                 int neg_exp, const uint32_t* __restrict__ chunk_map, uint32_t chunk) {
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint64_t gi = chunk_map ? static_cast<uint64_t>(chunk_map[i / chunk]) * chunk + i % chunk : i;
    Rng r(seed * 0x9e3779b97f4a7c15ull + gi);
    const double z = r.normal();
    out[i] = neg_exp ? static_cast<float>(-exp(z)) : static_cast<float>(mean + stdev * z);
}

// fp16 values std * N(0,1) (seeded KV cache contents).
__global__ void synth_f16_kernel(uint16_t* __restrict__ out, uint64_t n, uint64_t seed, float stdev) {
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    Rng r(seed * 0x9e3779b97f4a7c15ull + i);
    out[i] = __half_as_ushort(__float2half_rn(static_cast<float>(stdev * r.normal())));
}

// ---- activation producers ---------------------------------------------------------
// Warps 0 and 1 of a CTA pack super-block b of a normalised row from the
// lane's eight values x0|x1 (elements b*256 + lane*8 ...): v = x * inv * w;
// warp 0 writes the x-fragments (frag non-null) and the f32 copy (y non-null),
// warp 1 the NL-limb x-pack (limbs non-null), in parallel.
template <int NL>
__device__ __forceinline__ void norm_pack_block(const float4& x0, const float4& x1, const float4& w0, const float4& w1,
                                                float inv, uint32_t warp, uint32_t lane, uint32_t b, float* y,
                                                uint8_t* limbs, float* gsum, float* scale, uint8_t* frag) {
    float v[8] = {x0.x * inv * w0.x, x0.y * inv * w0.y, x0.z * inv * w0.z, x0.w * inv * w0.w,
                  x1.x * inv * w1.x, x1.y * inv * w1.y, x1.z * inv * w1.z, x1.w * inv * w1.w};
    if (warp == 0) {
        if (y) {
#pragma unroll
            for (int t = 0; t < 8; ++t) y[b * 256u + lane * 8u + t] = v[t];
        }
        if (frag) pack_block_warp_frag(v, lane, frag + b * kXfBlockBytes);
    } else if (warp == 1 && limbs) {
        pack_block_warp<NL>(v, b, lane, limbs, gsum, scale);
    }
}

// RMSNorm of one row of n (n % 256 == 0, n <= 32768) written straight into an
// NL-limb x-pack (limbs non-null), into x-fragments (frag non-null) and, when
// y is non-null, as f32.  One CTA of 256 threads per super-block: every CTA
// computes the same inverse RMS (row_inv_rms has a fixed order), then packs
// its own super-block.  The same products as the GEMVs' fused RMSNorm
// (XM = 3), so both paths give identical bits.
template <int NL>
__global__ void __launch_bounds__(256) rmsnorm_xpack_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                            uint32_t n, float eps, float* __restrict__ y,
                                                            uint8_t* __restrict__ limbs, float* __restrict__ gsum,
                                                            float* __restrict__ scale, uint8_t* __restrict__ frag) {
    constexpr uint32_t kPer = 4;  // super-blocks per warp loaded up front (32 per CTA)
    __shared__ double blk[kNormMaxBlocks];
    __shared__ float inv_s;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nb = n / 256u;
    const uint32_t b = blockIdx.x, base = b * 256u + lane * 8u;
    // Every load first (one L2 round trip): this CTA's block of x and w for
    // the packing warps, and the warp's share of x for the sum of squares.
    float4 pv0 = make_float4(0.f, 0.f, 0.f, 0.f), pv1 = pv0, pw0 = pv0, pw1 = pv0;
    if (warp < 2u) {
        pv0 = __ldcg(reinterpret_cast<const float4*>(x + base));
        pv1 = __ldcg(reinterpret_cast<const float4*>(x + base + 4u));
        pw0 = *reinterpret_cast<const float4*>(w + base);
        pw1 = *reinterpret_cast<const float4*>(w + base + 4u);
    }
    float4 r0[kPer], r1[kPer];
#pragma unroll
    for (uint32_t i = 0; i < kPer; ++i) {
        const uint32_t bb = warp + 8u * i;
        if (bb < nb) {
            r0[i] = __ldcg(reinterpret_cast<const float4*>(x + bb * 256u + lane * 8u));
            r1[i] = __ldcg(reinterpret_cast<const float4*>(x + bb * 256u + lane * 8u + 4u));
        }
    }
    // Same per-block order as row_inv_rms: fp32 lane sums, fp64 butterfly,
    // then the blocks added in order by one thread.
#pragma unroll
    for (uint32_t i = 0; i < kPer; ++i) {
        const uint32_t bb = warp + 8u * i;
        if (bb < nb) {
            const float4 v0 = r0[i], v1 = r1[i];
            float s = v0.x * v0.x;
            s = fmaf(v0.y, v0.y, s); s = fmaf(v0.z, v0.z, s); s = fmaf(v0.w, v0.w, s);
            s = fmaf(v1.x, v1.x, s); s = fmaf(v1.y, v1.y, s); s = fmaf(v1.z, v1.z, s); s = fmaf(v1.w, v1.w, s);
            double d = s;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            if (lane == 0) blk[bb] = d;
        }
    }
    for (uint32_t bb = warp + 8u * kPer; bb < nb; bb += 8u) {  // rows longer than 32 super-blocks
        const float4 v0 = __ldcg(reinterpret_cast<const float4*>(x + bb * 256u + lane * 8u));
        const float4 v1 = __ldcg(reinterpret_cast<const float4*>(x + bb * 256u + lane * 8u + 4u));
        float s = v0.x * v0.x;
        s = fmaf(v0.y, v0.y, s); s = fmaf(v0.z, v0.z, s); s = fmaf(v0.w, v0.w, s);
        s = fmaf(v1.x, v1.x, s); s = fmaf(v1.y, v1.y, s); s = fmaf(v1.z, v1.z, s); s = fmaf(v1.w, v1.w, s);
        double d = s;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (lane == 0) blk[bb] = d;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (uint32_t bb = 0; bb < nb; ++bb) t += blk[bb];
        inv_s = static_cast<float>(1.0 / sqrt(t / (256.0 * nb) + static_cast<double>(eps)));
    }
    __syncthreads();
    if (warp >= 2u) return;
    norm_pack_block<NL>(pv0, pv1, pw0, pw1, inv_s, warp, lane, b, y, limbs, gsum, scale, frag);
}

// SiLU(g) * u (the ffn_down input) as x-fragments, zero-padded from n to
// nb_pack super-blocks; one warp per super-block.
__global__ void __launch_bounds__(256) silu_mul_xfrag_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                                             uint32_t n, uint32_t nb_pack, uint8_t* __restrict__ frag) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31u, b = blockIdx.x * 8u + (threadIdx.x >> 5);
    if (b >= nb_pack) return;  // warp-uniform
    const uint32_t base = b * 256u + lane * 8u;
    float v[8];
    const bool pad = b >= n / 256u;  // zero padding block of a K-sliced projection
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = pad ? 0.0f : silu_f(__ldcg(g + base + t)) * __ldcg(u + base + t);
    pack_block_warp_frag(v, lane, frag + b * kXfBlockBytes);
}

// f32 vector of n as x-fragments, zero-padded to nb_pack super-blocks; one
// warp per super-block.
__global__ void __launch_bounds__(256) f32_xfrag_pad_kernel(const float* __restrict__ x, uint32_t n, uint32_t nb_pack,
                                                            uint8_t* __restrict__ frag) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31u, b = blockIdx.x * 8u + (threadIdx.x >> 5);
    if (b >= nb_pack) return;  // warp-uniform
    const uint32_t base = b * 256u + lane * 8u;
    float v[8];
    const bool pad = b >= n / 256u;
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = pad ? 0.0f : __ldcg(x + base + t);
    pack_block_warp_frag(v, lane, frag + b * kXfBlockBytes);
}

// ---- tensor-parallel exchange: the all-reduce fused with the next RMSNorm ----------
// After a row-parallel projection (ssm_out, wo, ffn_down) every rank holds a
// partial of the residual update; this kernel sums the partials of all ranks
// into the residual and normalises and packs the result for the next
// projection, replacing an all-reduce plus the RMSNorm kernel.
//
// Every rank owns an exchange region that all ranks map (CUDA IPC): slots
// [parity][sender][n/2] of 16-byte units {x[2i], epoch, x[2i+1], epoch}.  A
// sender writes each unit with one 16-byte store straight into the receiver's
// region; the receiver accepts each 8-byte half only when its epoch word equals
// the exchange's epoch, so data and flag travel together and no fence or
// separate signal is needed.  Each rank reads only its own region.
//
// The epoch of an exchange is (step << 9) + instance + 1: `step` counts decode
// steps (tp_step_kernel bumps it once per step) and `instance` numbers the
// exchanges of a step, two per layer.  The slot parity alternates with the
// instance.  A rank cannot finish exchange k+1 before every peer has started
// it, and a peer starts k+1 only after its exchange k has completed (every
// kernel of the chain waits for its predecessor), so no rank writes a slot of
// parity k & 1 again while a peer may still read it.
//
// CTA b (one per super-block, 256 threads) reads only super-block b of every
// rank's partial and forms x_out = x_in + partial(rank 0) + partial(rank 1)
// + ... element by element -- the same order, hence the same bits, on every
// rank.  The inverse RMS needs the whole row: each CTA publishes its block's
// sum of squares (the per-block order of row_inv_rms) in scratch of this
// rank's own region, tagged with the epoch, and polls, bounded, until all nb
// carry it, then adds them in block order.  Reading one block per rank instead of the whole row
// per rank keeps the cost nearly flat in the rank count.  Every poll is bounded: a partial that
// never arrives records kFaultPeerWait and the kernel finishes; once the fault
// word is set, later exchanges skip their waits.
constexpr uint32_t kMaxTp = 8;
constexpr uint32_t kTpWarps = 8;             // 256 threads: one element of the CTA's super-block each
constexpr uint32_t kTpScratch = 16u * kNormMaxBlocks;  // per-region local scratch: the block sums
constexpr uint32_t kTpSpinLimit = 1u << 21;  // polls of one unit (L2 round trips: about a second)

// Slots, then kTpScratch bytes only this rank touches: the CTAs' block sums
// of squares, one 16-byte unit {low word, epoch, high word, epoch} each.
__host__ __device__ constexpr size_t tp_slots_bytes(uint32_t n) { return 2ull * kMaxTp * (n / 2u) * 16u; }
__host__ __device__ constexpr size_t tp_exchange_bytes(uint32_t n) { return tp_slots_bytes(n) + kTpScratch; }

struct TpReduceArgs {
    const float* x_in;
    float* x_out;           // a different buffer from x_in (the entry point checks)
    const float* part;      // this rank's partial (n floats)
    uint4* region[kMaxTp];  // every rank's exchange region as mapped in this process
    const uint32_t* step;   // decode steps taken
    const float* norm_w;    // next RMSNorm weight; null: x_out only
    uint8_t* frag;          // x-fragments of the normalised row
    uint8_t* limbs;         // four-limb x-pack of it (null: none)
    float* y;               // the normalised row as f32 (null: none)
    float* gsum;
    float* scale;
    uint32_t n, rank, size, instance;
    float eps;
};

__device__ __forceinline__ void st_volatile_u4(uint4* p, uint4 v) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint4 ld_volatile_u4(const uint4* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

// Poll unit *p (first read v) until both halves carry epoch E, at most
// kTpSpinLimit times; a timeout records the fault and ends this thread's waits.
__device__ __forceinline__ uint4 tp_unit_wait(const uint4* p, uint4 v, uint32_t E, bool& wait) {
    for (uint32_t i = 0; wait && (v.y != E || v.w != E); ++i) {
        if (i == kTpSpinLimit) {
            record_fault(kFaultPeerWait);
            wait = false;
            break;
        }
        v = ld_volatile_u4(p);
    }
    return v;
}

template <int NL>
__global__ void __launch_bounds__(kTpWarps * 32, 1) tp_reduce_norm_kernel(const __grid_constant__ TpReduceArgs a) {
    __shared__ __align__(16) float sv[kMaxTp][256];  // block b of every rank's partial
    __shared__ __align__(16) float xb[256];
    __shared__ double bs[kNormMaxBlocks];
    __shared__ float inv_s;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t t = threadIdx.x, warp = t >> 5, lane = t & 31u, nb = a.n / 256u, b = blockIdx.x;
    const uint32_t E = (*a.step << 9) + a.instance + 1u, par = a.instance & 1u;
    const size_t units = a.n / 2u;
    bool wait = *static_cast<volatile uint32_t*>(&g_q38_fault) == 0u;
    uint4* blksum = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.region[a.rank]) + tp_slots_bytes(a.n));
    // 1. this CTA's super-block of the partial to every peer (128 units)
    {
        const uint32_t u = t & 127u;
        const float2 p = __ldcg(reinterpret_cast<const float2*>(a.part + b * 256u + 2u * u));
        const uint4 v = make_uint4(__float_as_uint(p.x), E, __float_as_uint(p.y), E);
        for (uint32_t j = t >> 7; j < a.size; j += kTpWarps * 32u / 128u)
            if (j != a.rank)
                st_volatile_u4(a.region[j] + (static_cast<size_t>(par) * kMaxTp + a.rank) * units + b * 128u + u, v);
    }
    // 2. super-block b of every rank's partial into shared memory: all loads
    // issued first, then each polled (bounded) until its epoch matches.
    {
        const uint4* mine = a.region[a.rank] + static_cast<size_t>(par) * kMaxTp * units + b * 128u;
        constexpr uint32_t kPerThread = kMaxTp * 128u / (kTpWarps * 32u);
        uint4 v[kPerThread];
#pragma unroll
        for (uint32_t k = 0; k < kPerThread; ++k) {
            const uint32_t idx = t + k * kTpWarps * 32u, j = idx >> 7, u = idx & 127u;
            if (j < a.size && j != a.rank) v[k] = ld_volatile_u4(mine + static_cast<size_t>(j) * units + u);
        }
#pragma unroll
        for (uint32_t k = 0; k < kPerThread; ++k) {
            const uint32_t idx = t + k * kTpWarps * 32u, j = idx >> 7, u = idx & 127u;
            if (j >= a.size) continue;
            float2 p;
            if (j == a.rank) {
                p = __ldcg(reinterpret_cast<const float2*>(a.part + b * 256u + 2u * u));
            } else {
                const uint4 r = tp_unit_wait(mine + static_cast<size_t>(j) * units + u, v[k], E, wait);
                p = make_float2(__uint_as_float(r.x), __uint_as_float(r.z));
            }
            *reinterpret_cast<float2*>(&sv[j][2u * u]) = p;
        }
    }
    __syncthreads();
    // 3. x_out of the block: x_in + partial(rank 0) + partial(rank 1) + ...
    {
        float acc = __ldcg(a.x_in + b * 256u + t);
        for (uint32_t j = 0; j < a.size; ++j) acc += sv[j][t];
        xb[t] = acc;
        a.x_out[b * 256u + t] = acc;
    }
    __syncthreads();
    // 4. the block's sum of squares (row_inv_rms's per-block order), published
    // to this rank's scratch with the epoch in both halves; every CTA polls
    // all nb of them (no atomics: data and flag travel together).
    if (warp == 0) {
        const float4 v0 = *reinterpret_cast<const float4*>(xb + lane * 8u);
        const float4 v1 = *reinterpret_cast<const float4*>(xb + lane * 8u + 4u);
        float sq = v0.x * v0.x;
        sq = fmaf(v0.y, v0.y, sq); sq = fmaf(v0.z, v0.z, sq); sq = fmaf(v0.w, v0.w, sq);
        sq = fmaf(v1.x, v1.x, sq); sq = fmaf(v1.y, v1.y, sq); sq = fmaf(v1.z, v1.z, sq); sq = fmaf(v1.w, v1.w, sq);
        double d = sq;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (lane == 0) {
            const unsigned long long bits = static_cast<unsigned long long>(__double_as_longlong(d));
            st_volatile_u4(blksum + b, make_uint4(static_cast<uint32_t>(bits), E, static_cast<uint32_t>(bits >> 32), E));
        }
        // every block's sum, polled (bounded) by the warp's lanes at once
        for (uint32_t bb = lane; bb < nb; bb += 32u) {
            const uint4 r = tp_unit_wait(blksum + bb, ld_volatile_u4(blksum + bb), E, wait);
            bs[bb] = __longlong_as_double(static_cast<long long>((static_cast<unsigned long long>(r.z) << 32) | r.x));
        }
        __syncwarp();
        if (lane == 0) {
            double tot = 0.0;
            for (uint32_t bb = 0; bb < nb; ++bb) tot += bs[bb];
            inv_s = static_cast<float>(1.0 / sqrt(tot / (256.0 * nb) + static_cast<double>(a.eps)));
        }
    }
    __syncthreads();
    if (!a.norm_w || warp >= 2u) return;
    const float4 x0 = *reinterpret_cast<const float4*>(xb + lane * 8u);
    const float4 x1 = *reinterpret_cast<const float4*>(xb + lane * 8u + 4u);
    const float4 w0 = *reinterpret_cast<const float4*>(a.norm_w + b * 256u + lane * 8u);
    const float4 w1 = *reinterpret_cast<const float4*>(a.norm_w + b * 256u + lane * 8u + 4u);
    norm_pack_block<NL>(x0, x1, w0, w1, inv_s, warp, lane, b, a.y, a.limbs, a.gsum, a.scale, a.frag);
}

// One decode step begins: the exchange epochs move on.
__global__ void tp_step_kernel(uint32_t* step) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) *step += 1u;
}

// ---- Q8_K activations on the device ---------------------------------------------------
// quantize_q8_k_cpu (src/quant.cpp:336-389) restated for one warp per block of
// 256 (lane holds values 8 lane .. 8 lane + 7): the scale comes from the value
// of largest magnitude (the first of equal ones), iscale = -127 / vmax,
// d = 1 / iscale, q = round(iscale * v) by the 1.5 * 2^23 magic add
// (src/quant.cpp:253-259) capped at 127, and the sums of each 16 values.
// Every product, sum and quotient is a separate IEEE operation, as on the
// CPU, so the 292-byte blocks are bit-exact.
__device__ __forceinline__ void q8k_quantize_block_warp(const float (&v)[8], uint32_t lane, uint8_t* blk) {
    float amax = 0.0f, vmax = 0.0f;
    uint32_t at = 0xffffffffu;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const float a = fabsf(v[t]);
        if (a > amax) {
            amax = a;
            vmax = v[t];
            at = lane * 8u + t;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {  // larger magnitude wins; on a tie the earlier index
        const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
        const float ov = __shfl_xor_sync(0xffffffffu, vmax, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, at, o);
        if (oa > amax || (oa == amax && oi < at)) {
            amax = oa;
            vmax = ov;
            at = oi;
        }
    }
    uint32_t w0 = 0u, w1 = 0u;
    int sum = 0;
    float d = 0.0f;
    if (amax != 0.0f) {
        const float iscale = __fdiv_rn(-127.0f, vmax);
        d = __fdiv_rn(1.0f, iscale);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const float m = __fadd_rn(__fmul_rn(iscale, v[t]), 12582912.0f);
            int q = (__float_as_int(m) & 0x007fffff) - 0x00400000;
            q = q > 127 ? 127 : q;
            sum += q;
            const uint32_t byte = static_cast<uint32_t>(q) & 255u;
            if (t < 4) w0 |= byte << (8 * t);
            else w1 |= byte << (8 * (t - 4));
        }
    }
    if (lane == 0) *reinterpret_cast<float*>(blk) = d;
    *reinterpret_cast<uint32_t*>(blk + 4 + lane * 8u) = w0;
    *reinterpret_cast<uint32_t*>(blk + 8 + lane * 8u) = w1;
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);  // lanes 2k, 2k+1: values 16k .. 16k + 15
    if ((lane & 1u) == 0) *reinterpret_cast<int16_t*>(blk + 260 + lane) = static_cast<int16_t>(sum);
}

// f32 [cols] -> Q8_K blocks [cols / 256][292], one warp per block.
__global__ void __launch_bounds__(256) quantize_q8k_kernel(const float* __restrict__ x, uint32_t nb,
                                                           uint8_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t lane = threadIdx.x & 31u, b = blockIdx.x * 8u + (threadIdx.x >> 5);
    if (b >= nb) return;  // warp-uniform
    const float4 v0 = __ldcg(reinterpret_cast<const float4*>(x + b * 256u + lane * 8u));
    const float4 v1 = __ldcg(reinterpret_cast<const float4*>(x + b * 256u + lane * 8u + 4u));
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    q8k_quantize_block_warp(v, lane, out + static_cast<size_t>(b) * 292u);
}

// RMSNorm of one row (n % 256 == 0, n <= 32768) straight into Q8_K blocks, one
// CTA per super-block: the inverse RMS of row_inv_rms (the order of the decode
// engine's norm kernel) and v = x * inv * w, then warp 0 quantises the block;
// y (f32, may be null) receives the normalised values that were quantised.
__global__ void __launch_bounds__(256) rmsnorm_q8k_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                          uint32_t n, float eps, float* __restrict__ y,
                                                          uint8_t* __restrict__ out) {
    __shared__ double blk[kNormMaxBlocks];
    __shared__ float inv_s;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, b = blockIdx.x;
    const float inv = row_inv_rms(x, n / 256u, eps, blk, &inv_s, warp, lane, 8u);
    if (warp != 0) return;
    const uint32_t base = b * 256u + lane * 8u;
    const float4 x0 = __ldcg(reinterpret_cast<const float4*>(x + base));
    const float4 x1 = __ldcg(reinterpret_cast<const float4*>(x + base + 4u));
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + base));
    const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + base + 4u));
    const float v[8] = {x0.x * inv * w0.x, x0.y * inv * w0.y, x0.z * inv * w0.z, x0.w * inv * w0.w,
                        x1.x * inv * w1.x, x1.y * inv * w1.y, x1.z * inv * w1.z, x1.w * inv * w1.w};
    if (y) {
#pragma unroll
        for (int t = 0; t < 8; ++t) y[base + t] = v[t];
    }
    q8k_quantize_block_warp(v, lane, out + static_cast<size_t>(b) * 292u);
}

// ---- embedding ----------------------------------------------------------------------
// out[hidden] = dequantised Q6_K row `*token` of the table (dequantize_q6_k_block_cpu,
// src/quant.cpp:186-249, with its float operation order).
// A token outside [0, vocab) reads row 0.
__global__ void __launch_bounds__(256) embed_q6k_kernel(const uint8_t* __restrict__ table, const int* __restrict__ token,
                                                        uint32_t vocab, uint32_t hidden, float* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t nb = hidden / 256u, j = threadIdx.x;
    const int tok = *token;
    const uint32_t id = tok >= 0 && static_cast<uint32_t>(tok) < vocab ? static_cast<uint32_t>(tok) : 0u;
    const uint8_t* row = table + static_cast<uint64_t>(id) * nb * 210u;
    const uint32_t n = j >> 7, rr = j & 127u, t = rr >> 5, l = rr & 31u;
    for (uint32_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * 210u;
        const uint32_t ql = blk[64u * n + l + 32u * (t & 1u)];
        const uint32_t qh = blk[128u + 32u * n + l];
        const int q = static_cast<int>(((ql >> (4u * (t >> 1))) & 15u) | (((qh >> (2u * t)) & 3u) << 4)) - 32;
        const int sc = static_cast<int8_t>(blk[192u + 8u * n + (l >> 4) + 2u * t]);
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[208] | (blk[209] << 8))));
        out[b * 256u + j] = d * static_cast<float>(sc) * static_cast<float>(q);
    }
}

// ---- full attention ---------------------------------------------------------------
constexpr uint32_t kAttnDim = 256;

// Per head RMSNorm (weight [256]) then NeoX RoPE on the first rope_dim dims at
// position *pos.  CTAs [0, Hq): query heads of qg ([Hq][q 256 | gate 256]) ->
// q [Hq][256]; CTAs [Hq, Hq+Hkv): key heads -> K cache; the value heads are
// copied to the V cache.  Caches are [Hkv][ctx][256] fp16.
__global__ void __launch_bounds__(kAttnDim) attn_prep_kernel(const float* __restrict__ qg, const float* __restrict__ kin,
                                                             const float* __restrict__ vin, const float* __restrict__ qnw,
                                                             const float* __restrict__ knw, const int* __restrict__ pos,
                                                             float* __restrict__ q, __half* __restrict__ kc,
                                                             __half* __restrict__ vc, uint32_t Hq, uint32_t ctx,
                                                             uint32_t rope_dim, float theta, float eps) {
    __shared__ double red[33];
    __shared__ float sv[kAttnDim];
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t hb = blockIdx.x, t = threadIdx.x;
    const bool isq = hb < Hq;
    const uint32_t kvh = hb - Hq;
    const int p = *pos;
    const float x = isq ? qg[hb * 2u * kAttnDim + t] : kin[kvh * kAttnDim + t];
    const double ss = block_sum(static_cast<double>(x) * x, red);
    const float inv = static_cast<float>(1.0 / sqrt(ss / kAttnDim + static_cast<double>(eps)));
    const float xn = x * inv * (isq ? qnw[t] : knw[t]);
    sv[t] = xn;
    __syncthreads();
    float r = xn;
    const uint32_t half = rope_dim / 2u;
    if (t < rope_dim) {
        const uint32_t i = t < half ? t : t - half;
        const double ang = static_cast<double>(p) * pow(static_cast<double>(theta), -2.0 * i / rope_dim);
        const double c = cos(ang), s = sin(ang);
        const double a = sv[i], b = sv[i + half];
        r = static_cast<float>(t < half ? a * c - b * s : b * c + a * s);
    }
    if (isq) {
        q[hb * kAttnDim + t] = r;
    } else if (p >= 0 && static_cast<uint32_t>(p) < ctx) {  // a full cache is never written past its end
        const size_t off = (static_cast<size_t>(kvh) * ctx + static_cast<size_t>(p)) * kAttnDim + t;
        kc[off] = __float2half_rn(r);
        vc[off] = __float2half_rn(vin[kvh * kAttnDim + t]);
    }
}

struct AttnArgs {
    const float* q;      // [Hq][256], normed and roped
    const float* qg;     // [Hq][q 256 | gate 256]: the gate half is read
    const __half* kc;    // [Hkv][ctx][256]
    const __half* vc;
    const int* pos;      // tokens 0..*pos are attended
    float* part_o;       // [Hq][S][256]
    float* part_ml;      // [Hq][S][2]
    float* out;          // [Hq][256] = softmax(q K^T / 16) V * sigmoid(gate)
    uint32_t Hq, Hkv, ctx;
    uint32_t splits;     // CTAs per KV head (<= kAttnSplits)
    uint8_t* xf;         // non-null: out also as x-fragments for the output projection
};                       // (head h = super-block h; its K is Hq * 256)

constexpr uint32_t kAttnSplits = 64;  // largest split count (scratch sizing)
constexpr uint32_t kAttnMaxGroup = 8;

// Grid (Hkv, splits), kAttnWarps warps.  CTA (g, s) takes a contiguous slice
// of the tokens for the G = Hq/Hkv query heads of KV head g, in chunks of up
// to kAttnChunk tokens whose K and V rows (contiguous in the cache) are
// copied into shared memory by two 1-D bulk copies (no multicast); scoring
// starts as soon as the K copy lands.
//  * Scores: a warp takes 8 tokens and two heads per pass; lane l holds dims
//    8l..8l+7, so it forms 16 partial dot products (8 tokens x 2 heads); a
//    reduce-scatter over lane bits 4..1 (15 shuffles) plus one exchange with
//    the neighbour lane leaves the full product of combination l/2 in lanes l
//    and l^1: one shuffle per score instead of a 5-step butterfly per score.
//  * Softmax: one warp per head finds the chunk's maximum, turns the scores
//    into exp(s - m) and keeps the running (m, l) of the CTA; every warp
//    rescales its partial output once per chunk.
//  * P V: warp w adds tokens w, w + W, ... into its 8 dims x G heads.
// The warps' partial outputs are summed (same running maximum) and the CTA
// writes a partial (m, l, o) for attn_combine_kernel.
constexpr uint32_t kAttnChunk = 128;
constexpr uint32_t kAttnWarps = 16;

// The warps' partial outputs reuse the K/V chunk buffers after the last chunk.
template <int G>
__host__ __device__ constexpr size_t attn_smem_bytes() {
    static_assert(kAttnWarps * G * kAttnDim * 4u <= 2u * kAttnChunk * kAttnDim * 2u, "partials fit the chunk buffers");
    return 2u * kAttnChunk * kAttnDim * 2u            // K and V chunks (fp16), later the per-warp partial outputs
           + G * kAttnChunk * 4u                      // scores / probabilities
           + G * kAttnDim * 4u                        // q of the group's heads, scaled
           + 4u * G * 4u                              // running m, l, chunk rescale
           + 2u * 8u + 128u;                          // two mbarriers + alignment
}

// Exact float value of two halves.
__device__ __forceinline__ void half8_to_float(const uint4 v, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 t = __half22float2(h[k]);
        f[2 * k] = t.x;
        f[2 * k + 1] = t.y;
    }
}

template <int G>
__global__ void __launch_bounds__(kAttnWarps * 32, 1) attn_decode_kernel(const AttnArgs a) {
    static_assert(G >= 1 && G <= kAttnWarps, "one softmax warp per head");
    constexpr uint32_t W = kAttnWarps, NP = (G + 1) / 2;  // passes of two heads
    extern __shared__ __align__(128) uint8_t smem_raw[];
    __half* ks = reinterpret_cast<__half*>(smem_raw);
    __half* vs = ks + kAttnChunk * kAttnDim;
    float* sc = reinterpret_cast<float*>(vs + kAttnChunk * kAttnDim);  // [G][kAttnChunk]
    float* qs = sc + G * kAttnChunk;                                   // [G][256] q / 16
    float* st = qs + G * kAttnDim;                                     // [G] m, [G] l, [G] rescale
    float* so = reinterpret_cast<float*>(smem_raw);                    // [W][G][256] after the chunks
    uint64_t* bars = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(st + 4u * G) + 7u) & ~static_cast<uintptr_t>(7u));
    const uint32_t g = blockIdx.x, sidx = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
    }
    if (threadIdx.x < G) {
        st[threadIdx.x] = -INFINITY;
        st[G + threadIdx.x] = 0.0f;
    }
    pdl_launch_dependents();
    pdl_wait();
    // q of the group's heads, pre-scaled by 1/sqrt(256)
    for (uint32_t e = threadIdx.x; e < G * kAttnDim; e += W * 32u)
        qs[e] = a.q[g * G * kAttnDim + e] * 0.0625f;
    __syncthreads();
    const uint32_t T = static_cast<uint32_t>(*a.pos) + 1u;
    const uint32_t S = a.splits;
    const uint32_t span = (T + S - 1u) / S;
    const uint32_t t0 = min(T, sidx * span), t1 = min(T, t0 + span);
    float o[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
        for (int d = 0; d < 8; ++d) o[h][d] = 0.0f;
    const __half* kb = a.kc + static_cast<size_t>(g) * a.ctx * kAttnDim;
    const __half* vb = a.vc + static_cast<size_t>(g) * a.ctx * kAttnDim;
    bool ok = true;
    uint32_t phase = 0;
    for (uint32_t c0 = t0; c0 < t1; c0 += kAttnChunk, phase ^= 1u) {
        const uint32_t n = min(kAttnChunk, t1 - c0);
        if (threadIdx.x == 0) {
            const uint32_t bytes = n * kAttnDim * 2u;
            mbar_arrive_expect_tx(&bars[0], bytes);
            tma_load_1d(ks, kb + static_cast<size_t>(c0) * kAttnDim, bytes, &bars[0]);
            mbar_arrive_expect_tx(&bars[1], bytes);
            tma_load_1d(vs, vb + static_cast<size_t>(c0) * kAttnDim, bytes, &bars[1]);
        }
        if (!__syncthreads_and(mbar_wait_spin(&bars[0], phase, kFaultFullWait))) {
            ok = false;  // uniform over the CTA
            break;
        }
        // ---- scores: 8 tokens x 2 heads per warp pass, reduce-scattered over the lanes
        for (uint32_t tb = warp * 8u; tb < n; tb += W * 8u) {
#pragma unroll
            for (uint32_t hp = 0; hp < NP; ++hp) {
                const uint32_t ha = 2u * hp, hb = 2u * hp + 1u < static_cast<uint32_t>(G) ? 2u * hp + 1u : 2u * hp;
                float qa[8], qb[8];
                {
                    const float4 a0 = *reinterpret_cast<const float4*>(qs + ha * kAttnDim + lane * 8u);
                    const float4 a1 = *reinterpret_cast<const float4*>(qs + ha * kAttnDim + lane * 8u + 4u);
                    const float4 b0 = *reinterpret_cast<const float4*>(qs + hb * kAttnDim + lane * 8u);
                    const float4 b1 = *reinterpret_cast<const float4*>(qs + hb * kAttnDim + lane * 8u + 4u);
                    qa[0] = a0.x; qa[1] = a0.y; qa[2] = a0.z; qa[3] = a0.w; qa[4] = a1.x; qa[5] = a1.y; qa[6] = a1.z; qa[7] = a1.w;
                    qb[0] = b0.x; qb[1] = b0.y; qb[2] = b0.z; qb[3] = b0.w; qb[4] = b1.x; qb[5] = b1.y; qb[6] = b1.z; qb[7] = b1.w;
                }
                float v[16];
#pragma unroll
                for (uint32_t j = 0; j < 8u; ++j) {
                    float kf[8];
                    const uint32_t t = tb + j < n ? tb + j : n - 1u;  // a valid row; its score is dropped
                    half8_to_float(*reinterpret_cast<const uint4*>(ks + t * kAttnDim + lane * 8u), kf);
                    float da = 0.0f, db = 0.0f;
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        da = fmaf(qa[e], kf[e], da);
                        db = fmaf(qb[e], kf[e], db);
                    }
                    v[2u * j] = da;
                    v[2u * j + 1u] = db;
                }
#pragma unroll
                for (uint32_t len = 16u, off = 16u; off > 1u; len >>= 1, off >>= 1) {
                    const bool up = (lane & off) != 0u;
#pragma unroll
                    for (uint32_t i = 0; i < len / 2u; ++i) {
                        const float send = up ? v[i] : v[i + len / 2u];
                        const float keep = up ? v[i + len / 2u] : v[i];
                        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                    }
                }
                v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);  // lanes 2c and 2c+1 hold combination c
                const uint32_t c = lane >> 1, j = c >> 1, h = 2u * hp + (c & 1u);
                if ((lane & 1u) == 0u && tb + j < n && h < static_cast<uint32_t>(G)) sc[h * kAttnChunk + tb + j] = v[0];
            }
        }
        __syncthreads();
        // ---- softmax statistics: warp h owns head h
        if (warp < static_cast<uint32_t>(G)) {
            const uint32_t h = warp;
            float mx = -INFINITY;
            for (uint32_t t = lane; t < n; t += 32u) mx = fmaxf(mx, sc[h * kAttnChunk + t]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mold = st[h], mnew = fmaxf(mold, mx);
            float sum = 0.0f;
            for (uint32_t t = lane; t < n; t += 32u) {
                const float p = expf(sc[h * kAttnChunk + t] - mnew);
                sc[h * kAttnChunk + t] = p;
                sum += p;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            if (lane == 0) {
                const float r = mold == -INFINITY ? 0.0f : expf(mold - mnew);
                st[h] = mnew;
                st[G + h] = fmaf(st[G + h], r, sum);
                st[2u * G + h] = r;
            }
        }
        __syncthreads();
        // ---- P V
        if (!__syncthreads_and(mbar_wait_spin(&bars[1], phase, kFaultFullWait))) {
            ok = false;
            break;
        }
#pragma unroll
        for (int h = 0; h < G; ++h) {
            const float r = st[2u * G + h];
#pragma unroll
            for (int d = 0; d < 8; ++d) o[h][d] *= r;
        }
        for (uint32_t t = warp; t < n; t += W) {
            float vf[8];
            half8_to_float(*reinterpret_cast<const uint4*>(vs + t * kAttnDim + lane * 8u), vf);
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float p = sc[h * kAttnChunk + t];
#pragma unroll
                for (int d = 0; d < 8; ++d) o[h][d] = fmaf(p, vf[d], o[h][d]);
            }
        }
        __syncthreads();  // the chunk buffers are reused by the next copy
    }
    if (!ok) {  // a copy did not land in time: wait (bounded) for both before reusing the buffers
        if (threadIdx.x == 0) {
            mbar_wait(&bars[0], phase, kFaultDrain);
            mbar_wait(&bars[1], phase, kFaultDrain);
        }
        __syncthreads();
    }
    // ---- sum the warps' partial outputs (one running maximum per head)
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
        for (int d = 0; d < 8; ++d) so[(warp * G + h) * kAttnDim + lane * 8u + d] = o[h][d];
    __syncthreads();
    for (uint32_t e = threadIdx.x; e < G * kAttnDim; e += W * 32u) {
        const uint32_t h = e / kAttnDim, d = e % kAttnDim;
        float acc = 0.0f;
        for (uint32_t w = 0; w < W; ++w) acc += so[(w * G + h) * kAttnDim + d];
        const uint32_t hq = g * G + h;
        a.part_o[(static_cast<size_t>(hq) * kAttnSplits + sidx) * kAttnDim + d] = acc;
        if (d == 0) {
            a.part_ml[(hq * kAttnSplits + sidx) * 2u] = ok ? st[h] : -INFINITY;
            a.part_ml[(hq * kAttnSplits + sidx) * 2u + 1u] = ok ? st[G + h] : 0.0f;
        }
    }
}

// Combine the per-split partials of every query head in split order and apply
// the output gate.  Grid Hq, 256 threads (one per output dimension); with
// a.xf, warp 0 then packs the head into x-fragments exactly as
// f32_xfrag_pad_kernel would from out (one launch fewer before the output
// projection).
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnArgs a) {
    __shared__ float fw[kAttnSplits];
    __shared__ float den;
    __shared__ __align__(16) float so[kAttnDim];
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t hq = blockIdx.x, d = threadIdx.x, S = a.splits;
    if (d < 32) {
        float M = -INFINITY;
        for (uint32_t sp = d; sp < S; sp += 32) M = fmaxf(M, a.part_ml[(hq * kAttnSplits + sp) * 2u]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        for (uint32_t sp = d; sp < S; sp += 32) {
            const float ms = a.part_ml[(hq * kAttnSplits + sp) * 2u];
            fw[sp] = ms == -INFINITY ? 0.0f : expf(ms - M);
        }
        __syncwarp();
        if (d == 0) {
            float L = 0.0f;
            for (uint32_t sp = 0; sp < S; ++sp) L = fmaf(fw[sp], a.part_ml[(hq * kAttnSplits + sp) * 2u + 1u], L);
            den = L;
        }
    }
    __syncthreads();
    float num = 0.0f;
    for (uint32_t sp = 0; sp < S; ++sp)
        num = fmaf(fw[sp], a.part_o[(static_cast<size_t>(hq) * kAttnSplits + sp) * kAttnDim + d], num);
    const float gate = a.qg[hq * 2u * kAttnDim + kAttnDim + d];
    const float o = num / den * (1.0f / (1.0f + expf(-gate)));
    a.out[hq * kAttnDim + d] = o;
    if (a.xf == nullptr) return;  // CTA-uniform
    so[d] = o;
    __syncthreads();
    if (d < 32) {
        const float4 v0 = *reinterpret_cast<const float4*>(so + d * 8u);
        const float4 v1 = *reinterpret_cast<const float4*>(so + d * 8u + 4u);
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        pack_block_warp_frag(v, d, a.xf + static_cast<size_t>(hq) * kXfBlockBytes);
    }
}

// ---- greedy sampling ----------------------------------------------------------------
// token = argmax(logits) (lowest index on ties), then *pos += 1.  Grid of
// kArgmaxCtas CTAs; the last CTA to finish reduces the per-CTA winners in
// CTA order.
constexpr uint32_t kArgmaxCtas = 148;
// Orderable 64-bit key of (value, index): larger value first, then lower index.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<unsigned long long>(u) << 32) | (0xffffffffu - idx);
}

// With key non-null (tensor parallel: logits are this rank's vocab slice
// starting at index base) the winner is written as a key for a max
// all-reduce instead of updating token and pos.
__global__ void __launch_bounds__(256) argmax_kernel(const float* __restrict__ logits, uint32_t n,
                                                     float* __restrict__ part_v, uint32_t* __restrict__ part_i,
                                                     unsigned* counter, int* token, int* pos,
                                                     unsigned long long* key, uint32_t base) {
    __shared__ float sv[256];
    __shared__ uint32_t si[256];
    __shared__ unsigned ticket;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t per = (n + gridDim.x - 1u) / gridDim.x;
    const uint32_t lo = blockIdx.x * per, hi = min(n, lo + per);
    float bv = -INFINITY;
    uint32_t bi = 0xffffffffu;
    for (uint32_t i = lo + threadIdx.x; i < hi; i += 256u) {
        const float v = logits[i];
        if (v > bv || (v == bv && i < bi)) {
            bv = v;
            bi = i;
        }
    }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (uint32_t s = 128; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            const float v = sv[threadIdx.x + s];
            const uint32_t i = si[threadIdx.x + s];
            if (v > sv[threadIdx.x] || (v == sv[threadIdx.x] && i < si[threadIdx.x])) {
                sv[threadIdx.x] = v;
                si[threadIdx.x] = i;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        part_v[blockIdx.x] = sv[0];
        part_i[blockIdx.x] = si[0];
        __threadfence();
        ticket = atomicAdd(counter, 1u);
    }
    __syncthreads();
    if (ticket != gridDim.x - 1u) return;  // CTA-uniform
    __threadfence();
    // The last CTA: the CTAs' winners, one per thread, reduced as a tree (the
    // winner is the maximum under (larger value, then lower index), so it does
    // not depend on the order); index 0xffffffff marks a slice without a
    // comparable value.
    float v = -INFINITY;
    uint32_t idx = 0xffffffffu;
    for (uint32_t c = threadIdx.x; c < gridDim.x; c += 256u) {
        const float cv = __ldcg(part_v + c);
        const uint32_t ci = __ldcg(part_i + c);
        if (ci != 0xffffffffu && (idx == 0xffffffffu || cv > v || (cv == v && ci < idx))) {
            v = cv;
            idx = ci;
        }
    }
    sv[threadIdx.x] = v;
    si[threadIdx.x] = idx;
    __syncthreads();
    for (uint32_t st = 128; st > 0; st >>= 1) {
        if (threadIdx.x < st) {
            const float ov = sv[threadIdx.x + st];
            const uint32_t oi = si[threadIdx.x + st];
            const uint32_t mi = si[threadIdx.x];
            if (oi != 0xffffffffu && (mi == 0xffffffffu || ov > sv[threadIdx.x] || (ov == sv[threadIdx.x] && oi < mi))) {
                sv[threadIdx.x] = ov;
                si[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x != 0) return;
    v = sv[0];
    idx = si[0];
    *counter = 0u;
    if (key) {
        *key = idx == 0xffffffffu ? 0ull : argmax_key(v, base + idx);
        return;
    }
    *token = idx == 0xffffffffu ? 0 : static_cast<int>(idx);
    *pos = *pos + 1;
}

// token = index of the all-reduced key; pos += 1.
__global__ void token_from_key_kernel(const unsigned long long* key, int* token, int* pos) {
    pdl_launch_dependents();
    pdl_wait();
    *token = static_cast<int>(0xffffffffu - static_cast<uint32_t>(*key & 0xffffffffull));
    *pos = *pos + 1;
}

// ---- loading a Q38PACK ------------------------------------------------------------
// Weights come from a pack as GGUF blocks (layout 0), the reference's Q5_K SoA
// planes (layout 1) or B200 fragment tiles (layout 2).  The loader uploads the
// row window of each source tensor that this rank's shard touches, turns it
// into GGUF blocks on the device (soa_q5k_to_gguf_kernel, unfrag_kernel),
// gathers the shard's rows and super-blocks (gather_blocks_kernel) and, for
// layout-2 weights, re-tiles the shard (repack_frag_kernel).

// Q5_K SoA records (META20 = d, dmin | 8 x (scale, min) bytes; QH32; QS128,
// three planes of n records, tools/gguf_to_q38pack.py:240-300) -> 176-byte
// GGUF blocks.
__global__ void soa_q5k_to_gguf_kernel(const uint8_t* __restrict__ meta, const uint8_t* __restrict__ qh,
                                       const uint8_t* __restrict__ qs, uint64_t n, uint8_t* __restrict__ out) {
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint8_t* m = meta + i * 20u;
    uint8_t* o = out + i * 176u;
    for (int k = 0; k < 4; ++k) o[k] = m[k];
    for (int j = 0; j < 4; ++j) {
        const uint32_t sc = m[4 + 2 * j], mn = m[5 + 2 * j], sc4 = m[12 + 2 * j], mn4 = m[13 + 2 * j];
        o[4 + j] = static_cast<uint8_t>((sc & 63u) | ((sc4 >> 4) << 6));
        o[8 + j] = static_cast<uint8_t>((mn & 63u) | ((mn4 >> 4) << 6));
        o[12 + j] = static_cast<uint8_t>((sc4 & 15u) | ((mn4 & 15u) << 4));
    }
    for (int k = 0; k < 32; ++k) o[16 + k] = qh[i * 32u + k];
    for (int k = 0; k < 128; ++k) o[48 + k] = qs[i * 128u + k];
}

// Layout-2 tiles of `rows` rows (the first at a tile boundary) x nb
// super-blocks -> row-major GGUF blocks; the inverse of repack_frag_kernel.
template <uint32_t T>
__global__ void unfrag_kernel(const uint8_t* __restrict__ tiles, uint8_t* __restrict__ blocks, uint32_t rows,
                              uint32_t nb) {
    using F = FragTile<T>;
    constexpr uint32_t kBlk = T == 13u ? 176u : 144u, kQsOff = T == 13u ? 48u : 16u;
    const uint64_t idx = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<uint64_t>(rows) * nb) return;
    const uint32_t r = static_cast<uint32_t>(idx / nb), b = static_cast<uint32_t>(idx % nb);
    const uint32_t o = r >> 3, g = r & 7u, kc = b >> 1, s = b & 1u;
    const uint8_t* tile = tiles + (static_cast<uint64_t>(o) * (nb / 2u) + kc) * F::kBytes;
    uint8_t* dst = blocks + idx * kBlk;
    const uint8_t* dm = tile + F::kDm + s * 32u + g * 4u;
    for (uint32_t k = 0; k < 4u; ++k) dst[k] = dm[k];
    const uint8_t* sc = tile + F::kSc + s * 128u + g * 16u;  // 8 scales, then 8 mins
    for (uint32_t j = 0; j < 4u; ++j) {
        dst[4u + j] = static_cast<uint8_t>((sc[j] & 63u) | ((sc[4u + j] >> 4) << 6));
        dst[8u + j] = static_cast<uint8_t>((sc[8u + j] & 63u) | ((sc[12u + j] >> 4) << 6));
        dst[12u + j] = static_cast<uint8_t>((sc[4u + j] & 15u) | ((sc[12u + j] & 15u) << 4));
    }
    uint8_t qh[32];
    for (uint32_t j = 0; j < 32u; ++j) qh[j] = 0;
    for (uint32_t p = 0; p < 4u; ++p) {
        for (uint32_t j = 0; j < 32u; ++j) {
            const uint32_t lane = 4u * g + (j >> 3);
            const uint32_t byte = tile[s * 1024u + (p >> 1) * 512u + lane * 16u + (p & 1u) * 8u + (j & 7u)];
            if constexpr (T == 13u) {
                const uint32_t nh = tile[F::kQh + lane * 16u + s * 8u + (j & 7u)];
                const uint32_t e5 = (byte & 15u) | (((nh >> (2u * p + 1u)) & 1u) << 4);
                const uint32_t o5 = ((byte >> 4) << 1) | ((nh >> (2u * p)) & 1u);
                dst[kQsOff + 32u * p + j] = static_cast<uint8_t>((e5 & 15u) | ((o5 & 15u) << 4));
                qh[j] = static_cast<uint8_t>(qh[j] | ((e5 >> 4) << (2u * p)) | ((o5 >> 4) << (2u * p + 1u)));
            } else {
                dst[kQsOff + 32u * p + j] = static_cast<uint8_t>(byte);
            }
        }
    }
    if constexpr (T == 13u)
        for (uint32_t j = 0; j < 32u; ++j) dst[16u + j] = qh[j];
}

// Global rows of a matrix stored as two tensors (rows [0, split) in the
// first, the rest in the second; one tensor: split = its rows); a segment
// holds the GGUF blocks of rows [lo, hi) of its tensor, p = row lo.
struct GatherSeg {
    const uint8_t* p;
    uint32_t lo, hi;
};

// Local block (i, b) of a rows x nb shard = global block (row_map[i],
// kb_map[b]) (identity maps when null; kb_map -1 = zero padding).  A global
// row outside the uploaded segments sets *err and writes zeros.
__global__ void gather_blocks_kernel(uint32_t bb, uint8_t* __restrict__ out, uint32_t rows, uint32_t nb,
                                     const uint32_t* __restrict__ row_map, const int32_t* __restrict__ kb_map,
                                     uint32_t nb_g, GatherSeg a, GatherSeg c, uint32_t split, unsigned* err) {
    const uint64_t blk = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (blk >= static_cast<uint64_t>(rows) * nb) return;
    const uint32_t i = static_cast<uint32_t>(blk / nb), b = static_cast<uint32_t>(blk % nb);
    const int32_t gb = kb_map ? kb_map[b] : static_cast<int32_t>(b);
    const uint8_t* src = nullptr;
    if (gb >= 0) {
        const uint32_t gr = row_map ? row_map[i] : i;
        const bool first = gr < split;
        const uint32_t r = first ? gr : gr - split, lo = first ? a.lo : c.lo, hi = first ? a.hi : c.hi;
        const uint8_t* base = first ? a.p : c.p;
        if (base && r >= lo && r < hi && static_cast<uint32_t>(gb) < nb_g)
            src = base + (static_cast<uint64_t>(r - lo) * nb_g + static_cast<uint32_t>(gb)) * bb;
        else
            atomicOr(err, 1u);
    }
    uint8_t* o = out + blk * bb;
    for (uint32_t k = 0; k < bb; ++k) o[k] = src ? src[k] : 0u;
}

// out[i] = src[g(i)], g(i) = chunk_map[i / chunk] * chunk + i % chunk
// (identity when chunk_map is null); g(i) >= src_n sets *err and writes 0.
__global__ void gather_f32_kernel(float* __restrict__ out, uint64_t n, const float* __restrict__ src, uint64_t src_n,
                                  const uint32_t* __restrict__ chunk_map, uint32_t chunk, unsigned* err) {
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint64_t gi = chunk_map ? static_cast<uint64_t>(chunk_map[i / chunk]) * chunk + i % chunk : i;
    if (gi < src_n) {
        out[i] = src[gi];
    } else {
        out[i] = 0.0f;
        atomicOr(err, 2u);
    }
}

}  // namespace q38
