// layer.cuh -- pointwise and recurrent kernels of the hybrid Qwen decoder
// layer (batch-1 decode), replacing the reference's sm_86 PTX entries:
//   q38_sumsq + q38_rmsnorm_apply      src/driver.cpp:240-324
//   q38_conv4_silu_roll                src/driver.cpp:759-837
//   q38_qk_l2norm_128                  src/driver.cpp:839-946
//   q38_beta_gate_48                   src/driver.cpp:948-1017
//   q38_gdn_ar_128                     src/driver.cpp:555-752
//   q38_gated_rmsnorm_silu_128         src/driver.cpp:1025-1143
//   q38_add_residual_f32, q38_ffn_silu_mul_f32   src/driver.cpp:1145-1228
// with the mathematics of the reference's CPU composition check
// (src/driver.cpp:8090-8242, 8365-8393, 11255-11301).
//
// Every reduction is a fixed-order tree (fp32 lanes, fp64 across warps), so
// results are deterministic.  gdn_fused_kernel runs conv+SiLU+roll, the q/k
// L2 norm, beta/gate, the state update and the gated RMSNorm of one value head
// in one cluster of 4 CTAs: the decode path launches it instead of five
// kernels.
#pragma once

#include "common.cuh"

namespace q38 {

constexpr uint32_t kGdnDim = 128;  // S_v = S_k = 128 (head dimension of the GDN state)

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

// Sum over the block (blockDim.x a multiple of 32, at most 1024) in fp64.
// `red` is 33 doubles of shared memory; every thread gets the total.
__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, nw = blockDim.x >> 5;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        double t = lane < nw ? red[lane] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (lane == 0) red[32] = t;
    }
    __syncthreads();
    const double r = red[32];
    __syncthreads();  // red may be reused right after
    return r;
}

// Warp-wide fp32 sum (fixed butterfly order).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// y = x * rsqrt(mean(x^2) + eps) * w, one CTA per row of n.
__global__ void __launch_bounds__(1024) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                       float* __restrict__ y, uint32_t n, float eps) {
    __shared__ double red[33];
    pdl_launch_dependents();
    pdl_wait();
    const float* xr = x + static_cast<size_t>(blockIdx.x) * n;
    float* yr = y + static_cast<size_t>(blockIdx.x) * n;
    float ss = 0.0f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    const double tot = block_sum(static_cast<double>(ss), red);
    const float inv = static_cast<float>(1.0 / sqrt(tot / static_cast<double>(n) + static_cast<double>(eps)));
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) yr[i] = xr[i] * inv * w[i];
}

// Causal depthwise conv (kernel 4) + SiLU and roll of the [3][C] state
// (oldest first); weight [C][4].  One thread per channel, so state_in may
// equal state_out.
__global__ void conv4_silu_roll_kernel(const float* __restrict__ qkv, const float* __restrict__ weight,
                                       const float* state_in, float* __restrict__ out, float* state_out,
                                       uint32_t C) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const float x0 = state_in[c], x1 = state_in[C + c], x2 = state_in[2u * C + c], x3 = qkv[c];
    const float4 w = *reinterpret_cast<const float4*>(weight + 4u * c);
    const float raw = fmaf(x3, w.w, fmaf(x2, w.z, fmaf(x1, w.y, x0 * w.x)));
    out[c] = silu_f(raw);
    state_out[c] = x1;
    state_out[C + c] = x2;
    state_out[2u * C + c] = x3;
}

// Per-head L2 norm of q (conv[0, H*D)) and k (conv[H*D, 2H*D)): x * rsqrt(sum x^2 + eps).
__global__ void __launch_bounds__(kGdnDim) qk_l2norm_kernel(const float* __restrict__ conv, float* __restrict__ q,
                                                            float* __restrict__ k, uint32_t H, float eps) {
    __shared__ double red[33];
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t b = blockIdx.x, t = threadIdx.x;
    const float v = conv[static_cast<size_t>(b) * kGdnDim + t];
    const double ss = block_sum(static_cast<double>(v) * v, red);
    const float inv = static_cast<float>(1.0 / sqrt(ss + static_cast<double>(eps)));
    float* dst = b < H ? q + static_cast<size_t>(b) * kGdnDim : k + static_cast<size_t>(b - H) * kGdnDim;
    dst[t] = v * inv;
}

// beta = sigmoid(b); g = softplus(a + dt) * A with softplus linear above 20
// and exp below -20 (src/driver.cpp:8142-8159).
__device__ __forceinline__ void beta_gate_one(float b, float a, float dt, float A, float& beta, float& g) {
    beta = static_cast<float>(1.0 / (1.0 + exp(-static_cast<double>(b))));
    const double v = static_cast<double>(a) + static_cast<double>(dt);
    const double sp = v > 20.0 ? v : (v < -20.0 ? exp(v) : log1p(exp(v)));
    g = static_cast<float>(sp * static_cast<double>(A));
}

__global__ void beta_gate_kernel(const float* __restrict__ braw, const float* __restrict__ araw,
                                 const float* __restrict__ dt, const float* __restrict__ A, float* __restrict__ beta,
                                 float* __restrict__ g, uint32_t n) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h < n) beta_gate_one(braw[h], araw[h], dt[h], A[h], beta[h], g[h]);
}

// One Gated DeltaNet step for 8 state columns per warp of value head h:
//   G = e^g[h];  kv_c = S[h][c] . k;  delta_c = (v_c - G kv_c) beta[h];
//   S'[h][c] = G S[h][c] + k delta_c;  o_c = (S'[h][c] . q) * scale
// with q/k = head h % Hq.  Lane l holds elements 4l..4l+3 of a 128-vector.
// A warp loads all its rows before writing any, so S_in may equal S_out.
template <int COLS>
__device__ __forceinline__ void gdn_columns(const float* __restrict__ s_in, float* s_out, uint32_t col0, float4 qv,
                                            float4 kv4, const float* __restrict__ v, float G, float B, float scale,
                                            float* o) {
    const uint32_t lane = threadIdx.x & 31u;
    float4 s[COLS];
#pragma unroll
    for (int j = 0; j < COLS; ++j)
        s[j] = *reinterpret_cast<const float4*>(s_in + static_cast<size_t>(col0 + j) * kGdnDim + 4u * lane);
#pragma unroll
    for (int j = 0; j < COLS; ++j) {
        const float kv = warp_sum(s[j].x * kv4.x + s[j].y * kv4.y + s[j].z * kv4.z + s[j].w * kv4.w);
        const float delta = (v[col0 + j] - G * kv) * B;
        float4 u;
        u.x = fmaf(G, s[j].x, kv4.x * delta);
        u.y = fmaf(G, s[j].y, kv4.y * delta);
        u.z = fmaf(G, s[j].z, kv4.z * delta);
        u.w = fmaf(G, s[j].w, kv4.w * delta);
        *reinterpret_cast<float4*>(s_out + static_cast<size_t>(col0 + j) * kGdnDim + 4u * lane) = u;
        const float oc = warp_sum(u.x * qv.x + u.y * qv.y + u.z * qv.z + u.w * qv.w);
        if (lane == 0) o[col0 + j] = oc * scale;
    }
}

// Grid (Hv, 128 / (8 * kGdnStepCols)): 8 warps x kGdnStepCols columns per CTA.
// One column per warp: every state column's load is in flight at once and the
// two warp reductions per column do not queue behind other columns (4 columns
// per warp over 192 CTAs measured 3.9 us for the 48-head step).
constexpr uint32_t kGdnStepCols = 1;
__global__ void __launch_bounds__(256) gdn_step_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                       const float* __restrict__ v, const float* __restrict__ g,
                                                       const float* __restrict__ beta, const float* s_in,
                                                       float* __restrict__ out, float* s_out, uint32_t Hq,
                                                       float scale) {
    pdl_launch_dependents();
    const uint32_t h = blockIdx.x, lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const size_t hs = static_cast<size_t>(h) * kGdnDim * kGdnDim;
    pdl_wait();
    const uint32_t qh = h % Hq;
    const float4 qv = *reinterpret_cast<const float4*>(q + qh * kGdnDim + 4u * lane);
    const float4 kv4 = *reinterpret_cast<const float4*>(k + qh * kGdnDim + 4u * lane);
    const float G = expf(g[h]), B = beta[h];
    gdn_columns<kGdnStepCols>(s_in + hs, s_out + hs, (blockIdx.y * 8u + warp) * kGdnStepCols, qv, kv4,
                              v + h * kGdnDim, G, B, scale, out + h * kGdnDim);
}

// Per head: o * rsqrt(mean(o^2) + eps) * w[D] * SiLU(z).
__global__ void __launch_bounds__(kGdnDim) gated_rmsnorm_silu_kernel(const float* __restrict__ o,
                                                                     const float* __restrict__ w,
                                                                     const float* __restrict__ z,
                                                                     float* __restrict__ y, float eps) {
    __shared__ double red[33];
    pdl_launch_dependents();
    pdl_wait();
    const size_t i = static_cast<size_t>(blockIdx.x) * kGdnDim + threadIdx.x;
    const float ov = o[i];
    const double ss = block_sum(static_cast<double>(ov) * ov, red);
    const float inv = static_cast<float>(1.0 / sqrt(ss / kGdnDim + static_cast<double>(eps)));
    y[i] = ov * inv * w[threadIdx.x] * silu_f(z[i]);
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ y,
                           uint32_t n) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = a[i] + b[i];
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ y,
                                uint32_t n) {
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = silu_f(g[i]) * u[i];
}

// ---- fused recurrent core: conv + norms + gates + GDN step + gated norm ------

struct GdnFusedArgs {
    const float* qkv;        // [2*Hq*D + Hv*D] output of the qkv projection
    const float* conv_w;     // [C][4]
    const float* conv_in;    // [3][C]
    float* conv_out;         // [3][C], a different buffer from conv_in
    const float* beta_raw;   // [Hv]
    const float* alpha_raw;  // [Hv]
    const float* dt_bias;    // [Hv]
    const float* ssm_a;      // [Hv]
    const float* s_in;       // [Hv][D][D]
    float* s_out;            // [Hv][D][D], may equal s_in
    const float* z;          // [Hv*D]
    const float* norm_w;     // [D]
    float* y;                // [Hv*D] gated-norm output (input of ssm_out)
    uint32_t Hq, Hv;
    float eps;    // q/k L2-norm and gated RMSNorm epsilon (rms_eps)
    float scale;  // 1/sqrt(D)
    const int* parity;  // optional: when *parity is odd, conv_in and conv_out swap roles
};

// A cluster of kGdnSplit CTAs (kGdnFusedThreads each) per value head h; CTA r
// of the cluster owns state columns [32r, 32r + 32) (2 per warp).  Channels: q/k
// of head h % Hq and v of head h; every CTA recomputes the head's conv and
// norms, and rank 0 of the clusters with h < Hq (q/k) or of every head (v)
// writes the rolled conv state, so it must be double-buffered (conv_in !=
// conv_out).  The gated RMSNorm's sum of squares meets across the cluster in
// distributed shared memory: each CTA's warp sum of its 32 outputs goes to
// every CTA of the cluster, then all add the four in the order of a
// 128-thread block reduction, so the outputs are those of one CTA per head.
constexpr uint32_t kGdnSplit = 4;
constexpr uint32_t kGdnFusedThreads = 512;  // 16 warps x 2 state columns

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void st_cluster_f64(const void* local, uint32_t rank, double v) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(remote), "d"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kGdnFusedThreads) gdn_fused_kernel(const GdnFusedArgs a) {
    constexpr uint32_t D = kGdnDim;
    __shared__ __align__(128) float sst[32 * D];  // this CTA's 32 state columns (16 KB)
    __shared__ __align__(16) float cv[3 * D];     // q | k | v after conv+SiLU (q, k then normalised)
    __shared__ __align__(16) float o[D];
    __shared__ double red[2];
    __shared__ double part[kGdnSplit];  // the cluster's per-CTA sums of squares, by rank
    __shared__ float gb[2];
    __shared__ __align__(8) uint64_t sbar;
    const uint32_t r = cluster_ctarank(), h = blockIdx.x / kGdnSplit;
    const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
    const uint32_t qh = h % a.Hq, C = 2u * a.Hq * D + a.Hv * D;
    const float* conv_in = a.conv_in;
    float* conv_out = a.conv_out;
    const float* s_in = a.s_in + (static_cast<size_t>(h) * D + r * 32u) * D;
    float* s_out = a.s_out + (static_cast<size_t>(h) * D + r * 32u) * D;
    // The state is read before the dependency wait only as an L2 hint; its
    // copy into shared memory starts right after the wait and lands while the
    // conv and the norms run.
    if (t < 8) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(s_in + t * 4u * D), "r"(2048u) : "memory");
    if (t == 0) {
        mbar_init(&sbar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();
    if (t == 0) {
        mbar_arrive_expect_tx(&sbar, 32u * D * 4u);
        tma_load_1d(sst, s_in, 32u * D * 4u, &sbar);
    }
    if (a.parity && (*a.parity & 1)) {  // ping-pong by decode position
        conv_in = a.conv_out;
        conv_out = const_cast<float*>(a.conv_in);
    }
    const uint32_t c_out = r * 32u + lane;
    float zc = 0.0f, nwc = 0.0f;
    if (warp == 7) {  // the gated norm's inputs, early
        zc = a.z[static_cast<size_t>(h) * D + c_out];
        nwc = a.norm_w[c_out];
    }
    for (uint32_t c = t; c < 3u * D; c += blockDim.x) {
        const uint32_t part3 = c / D, i = c % D;
        const uint32_t ch = part3 == 0 ? qh * D + i : (part3 == 1 ? a.Hq * D + qh * D + i : 2u * a.Hq * D + h * D + i);
        const float x0 = conv_in[ch], x1 = conv_in[C + ch], x2 = conv_in[2u * C + ch], x3 = a.qkv[ch];
        const float4 w = *reinterpret_cast<const float4*>(a.conv_w + 4u * ch);
        cv[c] = silu_f(fmaf(x3, w.w, fmaf(x2, w.z, fmaf(x1, w.y, x0 * w.x))));
        if (r == 0 && (part3 == 2 || h < a.Hq)) {
            conv_out[ch] = x1;
            conv_out[C + ch] = x2;
            conv_out[2u * C + ch] = x3;
        }
    }
    if (t == kGdnFusedThreads - 32u) {  // the gates on the last warp, beside the norms of warps 0 and 1
        float beta, g;
        beta_gate_one(a.beta_raw[h], a.alpha_raw[h], a.dt_bias[h], a.ssm_a[h], beta, g);
        gb[0] = expf(g);
        gb[1] = beta;
    }
    __syncthreads();
    // L2 norms of q (warp 0) and k (warp 1), fp64 lane partials; the inverse
    // norm is formed once per head.
    if (warp < 2) {
        const float4 v4 = *reinterpret_cast<const float4*>(cv + warp * D + 4u * lane);
        double ss = static_cast<double>(v4.x) * v4.x + static_cast<double>(v4.y) * v4.y +
                    static_cast<double>(v4.z) * v4.z + static_cast<double>(v4.w) * v4.w;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (lane == 0) red[warp] = static_cast<float>(1.0 / sqrt(ss + static_cast<double>(a.eps)));
    }
    __syncthreads();
    if (t < 2 * D) cv[t] *= static_cast<float>(red[t / D]);
    __syncthreads();
    const float4 qv = *reinterpret_cast<const float4*>(cv + 4u * lane);
    const float4 kv4 = *reinterpret_cast<const float4*>(cv + D + 4u * lane);
    const bool landed = __all_sync(0xffffffffu, mbar_wait(&sbar, 0, kFaultFullWait));
    if (landed) gdn_columns<2>(sst, s_out, warp * 2u, qv, kv4, cv + 2u * D + r * 32u, gb[0], gb[1], a.scale, o + r * 32u);
    __syncthreads();
    if (warp == 7) {
        const float ov = o[c_out];
        double ss = static_cast<double>(ov) * ov;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (lane < kGdnSplit) st_cluster_f64(&part[r], lane, ss);  // to every CTA of the cluster
    }
    cluster_sync_all();
    if (warp == 7 && landed) {
        // the order of a butterfly over 4 warp sums: (p0 + p2) + (p1 + p3)
        const double tot = (part[0] + part[2]) + (part[1] + part[3]);
        const float inv = static_cast<float>(1.0 / sqrt(tot / D + static_cast<double>(a.eps)));
        a.y[static_cast<size_t>(h) * D + c_out] = o[c_out] * inv * nwc * silu_f(zc);
    }
}

}  // namespace q38
