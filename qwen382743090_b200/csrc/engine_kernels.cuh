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
    __shared__ double blk[kNormMaxBlocks];
    __shared__ float inv_s;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nb = n / 256u;
    const float inv = row_inv_rms(x, nb, eps, blk, &inv_s, warp, lane, blockDim.x >> 5);
    if (warp != 0) return;
    const uint32_t b = blockIdx.x, base = b * 256u + lane * 8u;
    float v[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = x[base + t] * inv * w[base + t];
    if (y) {
#pragma unroll
        for (int t = 0; t < 8; ++t) y[base + t] = v[t];
    }
    if (limbs) pack_block_warp<NL>(v, b, lane, limbs, gsum, scale);
    if (frag) pack_block_warp_frag(v, lane, frag + b * kXfBlockBytes);
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
    for (int t = 0; t < 8; ++t) v[t] = pad ? 0.0f : silu_f(g[base + t]) * u[base + t];
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
    for (int t = 0; t < 8; ++t) v[t] = pad ? 0.0f : x[base + t];
    pack_block_warp_frag(v, lane, frag + b * kXfBlockBytes);
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
};

constexpr uint32_t kAttnSplits = 64;  // largest split count (scratch sizing)
constexpr uint32_t kAttnMaxGroup = 8;

// Grid (Hkv, splits), 256 threads.  CTA (g, s) takes a contiguous slice of the
// tokens for the G = Hq/Hkv query heads of KV head g; warps take every 8th
// token (four at a time, loads first) with an online softmax; the CTA merges
// its warps and writes a partial (m, l, o) for attn_combine_kernel.
template <int G>
__global__ void __launch_bounds__(256) attn_decode_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) float sm[];  // [8 warps][G][256] then [8][G][2]
    const uint32_t g = blockIdx.x, sidx = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t T = static_cast<uint32_t>(*a.pos) + 1u;
    const uint32_t S = a.splits;
    const uint32_t chunk = (T + S - 1u) / S;
    const uint32_t t0 = min(T, sidx * chunk), t1 = min(T, t0 + chunk);
    // q of the group's heads, pre-scaled by 1/sqrt(256), lane owns dims 8l..8l+7
    float qr[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        const float4* qp = reinterpret_cast<const float4*>(a.q + (g * G + h) * kAttnDim + lane * 8u);
        const float4 u = qp[0], v = qp[1];
        qr[h][0] = u.x * 0.0625f; qr[h][1] = u.y * 0.0625f; qr[h][2] = u.z * 0.0625f; qr[h][3] = u.w * 0.0625f;
        qr[h][4] = v.x * 0.0625f; qr[h][5] = v.y * 0.0625f; qr[h][6] = v.z * 0.0625f; qr[h][7] = v.w * 0.0625f;
    }
    float m[G], l[G], o[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.0f;
#pragma unroll
        for (int d = 0; d < 8; ++d) o[h][d] = 0.0f;
    }
    const __half* kb = a.kc + static_cast<size_t>(g) * a.ctx * kAttnDim + lane * 8u;
    const __half* vb = a.vc + static_cast<size_t>(g) * a.ctx * kAttnDim + lane * 8u;
    constexpr uint32_t U = 4;  // tokens per warp whose K/V rows are loaded together
    for (uint32_t tb = t0 + warp; tb < t1; tb += 8u * U) {
        uint4 kr[U], vr[U];
#pragma unroll
        for (uint32_t u = 0; u < U; ++u) {
            const uint32_t t = tb + 8u * u;
            if (t < t1) {
                kr[u] = *reinterpret_cast<const uint4*>(kb + static_cast<size_t>(t) * kAttnDim);
                vr[u] = *reinterpret_cast<const uint4*>(vb + static_cast<size_t>(t) * kAttnDim);
            }
        }
#pragma unroll
        for (uint32_t u = 0; u < U; ++u) {
            if (tb + 8u * u >= t1) break;  // warp-uniform
            const __half2* kh = reinterpret_cast<const __half2*>(&kr[u]);
            const __half2* vh = reinterpret_cast<const __half2*>(&vr[u]);
            float kf[8], vf[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 kk = __half22float2(kh[k]), vv = __half22float2(vh[k]);
                kf[2 * k] = kk.x; kf[2 * k + 1] = kk.y;
                vf[2 * k] = vv.x; vf[2 * k + 1] = vv.y;
            }
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float sdot = 0.0f;
#pragma unroll
                for (int d = 0; d < 8; ++d) sdot = fmaf(qr[h][d], kf[d], sdot);
                sdot = warp_sum(sdot);
                const float mn = fmaxf(m[h], sdot);
                const float corr = expf(m[h] - mn), pexp = expf(sdot - mn);
                l[h] = fmaf(l[h], corr, pexp);
#pragma unroll
                for (int d = 0; d < 8; ++d) o[h][d] = fmaf(o[h][d], corr, pexp * vf[d]);
                m[h] = mn;
            }
        }
    }
    // merge the 8 warps of the CTA
    float* so = sm;
    float* sml = sm + 8u * G * kAttnDim;
#pragma unroll
    for (int h = 0; h < G; ++h) {
#pragma unroll
        for (int d = 0; d < 8; ++d) so[(warp * G + h) * kAttnDim + lane * 8u + d] = o[h][d];
        if (lane == 0) {
            sml[(warp * G + h) * 2u] = m[h];
            sml[(warp * G + h) * 2u + 1u] = l[h];
        }
    }
    __syncthreads();
    for (uint32_t e = threadIdx.x; e < G * kAttnDim; e += 256u) {
        const uint32_t h = e / kAttnDim, d = e % kAttnDim;
        float M = -INFINITY;
        for (uint32_t w = 0; w < 8; ++w) M = fmaxf(M, sml[(w * G + h) * 2u]);
        float acc = 0.0f, L = 0.0f;
        for (uint32_t w = 0; w < 8; ++w) {
            const float mw = sml[(w * G + h) * 2u];
            const float f = mw == -INFINITY ? 0.0f : expf(mw - M);
            acc = fmaf(f, so[(w * G + h) * kAttnDim + d], acc);
            L = fmaf(f, sml[(w * G + h) * 2u + 1u], L);
        }
        const uint32_t hq = g * G + h;
        a.part_o[(static_cast<size_t>(hq) * kAttnSplits + sidx) * kAttnDim + d] = acc;
        if (d == 0) {
            a.part_ml[(hq * kAttnSplits + sidx) * 2u] = M;
            a.part_ml[(hq * kAttnSplits + sidx) * 2u + 1u] = L;
        }
    }
}

// Combine the per-split partials of every query head in split order and apply
// the output gate.  Grid Hq, 256 threads (one per output dimension).
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnArgs a) {
    __shared__ float fw[kAttnSplits];
    __shared__ float den;
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
    a.out[hq * kAttnDim + d] = num / den * (1.0f / (1.0f + expf(-gate)));
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
    if (ticket != gridDim.x - 1u || threadIdx.x != 0) return;
    __threadfence();
    float v = -INFINITY;
    uint32_t idx = 0xffffffffu;
    for (uint32_t c = 0; c < gridDim.x; ++c) {
        const float cv = __ldcg(part_v + c);
        const uint32_t ci = __ldcg(part_i + c);
        if (ci == 0xffffffffu) continue;  // slice without a comparable value
        if (idx == 0xffffffffu || cv > v || (cv == v && ci < idx)) {
            v = cv;
            idx = ci;
        }
    }
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

}  // namespace q38
