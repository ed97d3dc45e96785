// engine.cuh -- batch-1 greedy decode engine of the synthetic hybrid Qwen
// model (host side; included by q38rt.cu after the C ABI helpers).
//
// The reference stops at one recurrent layer (run_qwen35_layer0_full,
// src/driver.cpp:7025-8631; native decode is disabled, src/runtime.cpp:74-76).
// This engine runs the whole model on one device: token embedding, n_layers
// layers with full attention every attn_every-th layer (layers 3, 7, ..., 63
// for the 64-layer topology, src/layer_topology.cpp:152-173), final RMSNorm,
// the Q6_K lm_head and a greedy argmax, all without a host round trip, so one
// decode step is one replayable CUDA graph.
//
// Weights are seeded synthetic tensors generated on the device.  All tensors
// live in one arena (256-byte aligned offsets).  Same-type neighbours that
// read the same activations are stored as one matrix: the Q5_K qkv and z
// projections (10240 + 6144 rows) and the Q4_K beta and alpha projections
// (48 + 48 rows), so each pair is one GEMV launch.
//
// Per recurrent layer the launch chain is: RMSNorm->x-pack, qkvz GEMV, beta/alpha
// GEMV, fused recurrent core, ssm_out GEMV (+ residual), RMSNorm->x-pack,
// ffn_gate GEMV, ffn_up GEMV, SiLU*up->x-pack, ffn_down GEMV (+ residual).
#pragma once

#include <algorithm>
#include <memory>
#include <string>
#include <vector>

#include "engine_kernels.cuh"

namespace {

struct GemvW {
    q38_weight_desc d{};
    uint64_t bytes = 0;   // bytes as stored
    uint64_t algo = 0;    // bytes in the GGUF block size (176/144/210/136 per 256)
};

struct LayerW {
    bool attn = false;
    float* attn_norm = nullptr;
    float* post_norm = nullptr;
    // recurrent
    GemvW qkvz, ba, ssm_out;
    float *conv_w = nullptr, *dt = nullptr, *ssm_a = nullptr, *ssm_norm = nullptr;
    float* conv_state[2] = {nullptr, nullptr};
    float* ssm_state = nullptr;
    // attention
    GemvW wq, wk, wv, wo;
    float *q_norm = nullptr, *k_norm = nullptr;
    __half *kc = nullptr, *vc = nullptr;
    // ffn
    GemvW gate, up, down;
};

uint32_t block_bytes(uint32_t type) {
    switch (type) {
        case Q38_TYPE_Q4_K: return 144;
        case Q38_TYPE_Q5_K: return 176;
        case Q38_TYPE_Q6_K: return 210;
        case Q38_TYPE_IQ4_XS: return 136;
        default: return 0;
    }
}

}  // namespace

struct q38_model {
    q38_model_config cfg{};
    int device = 0;
    int sm_count = 148;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0, arena_used = 0;
    uint8_t* tmp = nullptr;  // layout-0 staging for the on-device repack
    size_t tmp_bytes = 0;
    std::vector<LayerW> layers;
    GemvW embd, lm_head;
    float* out_norm = nullptr;
    // activations and scratch
    float *x = nullptr, *qkvz = nullptr, *ba = nullptr, *ygdn = nullptr, *qg = nullptr, *kv_k = nullptr,
          *kv_v = nullptr, *qr = nullptr, *ao = nullptr, *g = nullptr, *u = nullptr, *logits = nullptr;
    uint8_t *xp = nullptr, *xp4 = nullptr;
    float *part_o = nullptr, *part_ml = nullptr, *am_v = nullptr;
    uint32_t* am_i = nullptr;
    unsigned* counters = nullptr;  // [8]: argmax ticket
    int *d_token = nullptr, *d_pos = nullptr;
    uint64_t step_bytes = 0;   // algorithmic weight bytes streamed per decode step
    cudaGraphExec_t graph = nullptr;
    uint32_t graph_steps = 0;
};

namespace {

int model_alloc(q38_model* m, size_t bytes, void** out) {
    const size_t off = (m->arena_used + 255u) & ~size_t(255);
    if (off + bytes > m->arena_bytes) return fail(Q38_ERR_NOMEM, "model arena exhausted (%zu + %zu > %zu)", off, bytes, m->arena_bytes);
    *out = m->arena + off;
    m->arena_used = off + bytes;
    return Q38_OK;
}

uint64_t gemv_stored_bytes(uint32_t type, uint32_t layout, uint32_t rows, uint32_t cols) {
    if (layout == Q38_LAYOUT_B200_TILED)
        return static_cast<uint64_t>((rows + q38::kT2Rows - 1u) / q38::kT2Rows) * (cols / 1024u) * q38::kT2TileBytes;
    return static_cast<uint64_t>(rows) * (cols / 256u) * block_bytes(type);
}

// Bytes the arena needs for the whole model (weights, state, scratch).
size_t model_arena_bytes(const q38_model_config& c) {
    size_t b = 0;
    auto add = [&](size_t n) { b += (n + 255u) & ~size_t(255); };
    const uint32_t H = c.hidden, F = c.ffn, D = 128u, Hq = c.gdn_qk_heads, Hv = c.gdn_v_heads;
    const uint32_t C = 2u * Hq * D + Hv * D;
    for (uint32_t L = 0; L < c.n_layers; ++L) {
        const bool attn = (L % c.attn_every) == c.attn_every - 1u;
        add(4u * H);
        add(4u * H);
        if (!attn) {
            add(gemv_stored_bytes(13, 2, C + Hv * D, H));
            add(gemv_stored_bytes(12, 0, 2u * Hv, H));
            add(gemv_stored_bytes(13, 2, H, Hv * D));
            add(16u * C);
            add(4u * Hv);
            add(4u * Hv);
            add(4u * D);
            add(12u * C);
            add(12u * C);
            add(4ull * Hv * D * D);
        } else {
            const uint32_t AQ = c.attn_q_heads, AK = c.attn_kv_heads, AD = q38::kAttnDim;
            add(gemv_stored_bytes(13, 2, 2u * AQ * AD, H));
            add(gemv_stored_bytes(13, 2, AK * AD, H));
            add(gemv_stored_bytes(14, 0, AK * AD, H));
            add(gemv_stored_bytes(13, 2, H, AQ * AD));
            add(4u * AD);
            add(4u * AD);
            add(2ull * AK * c.ctx * AD);
            add(2ull * AK * c.ctx * AD);
        }
        add(gemv_stored_bytes(12, 0, F, H));
        add(gemv_stored_bytes(13, 2, F, H));
        add(gemv_stored_bytes(13, 2, H, F));
    }
    add(gemv_stored_bytes(14, 0, c.vocab, H));
    add(gemv_stored_bytes(14, 0, c.vocab, H));
    add(4u * H);
    // scratch
    const uint32_t AQ = c.attn_q_heads, AD = q38::kAttnDim;
    for (size_t n : {size_t(4u * H), size_t(4u * (C + Hv * D)), size_t(4u * 2u * Hv), size_t(4u * Hv * D),
                     size_t(4u * 2u * AQ * AD), size_t(4u * c.attn_kv_heads * AD), size_t(4u * c.attn_kv_heads * AD),
                     size_t(4u * AQ * AD), size_t(4u * AQ * AD), size_t(4u * F), size_t(4u * F), size_t(4u * c.vocab),
                     q38_xpack_bytes(3, H, 1) + q38_xpack_bytes(3, Hv * D, 1) + q38_xpack_bytes(3, AQ * AD, 1),
                     q38_xpack_bytes(4, F, 1), size_t(4u) * AQ * q38::kAttnSplits * AD,
                     size_t(8u) * AQ * q38::kAttnSplits, size_t(4u * q38::kArgmaxCtas), size_t(4u * q38::kArgmaxCtas),
                     size_t(64), size_t(16)})
        add(n);
    return b + 4096u;
}

int synth_gemv(q38_model* m, GemvW* w, uint32_t type, uint32_t layout, uint32_t rows, uint32_t cols, uint64_t seed,
               cudaStream_t s) {
    void* p = nullptr;
    w->bytes = gemv_stored_bytes(type, layout, rows, cols);
    w->algo = static_cast<uint64_t>(rows) * (cols / 256u) * block_bytes(type);
    if (int rc = model_alloc(m, w->bytes, &p)) return rc;
    const uint64_t nblocks = static_cast<uint64_t>(rows) * (cols / 256u);
    const uint32_t grid = static_cast<uint32_t>((nblocks + 255u) / 256u);
    if (layout == Q38_LAYOUT_GGUF_NATIVE) {
        q38::synth_blocks_kernel<<<grid, 256, 0, s>>>(type, static_cast<uint8_t*>(p), nblocks, seed);
    } else {
        const size_t need = nblocks * 176u;
        if (need > m->tmp_bytes) return fail(Q38_ERR_INVALID, "repack staging too small");
        q38::synth_blocks_kernel<<<grid, 256, 0, s>>>(type, m->tmp, nblocks, seed);
        if (rows % q38::kT2Rows) Q38_CUDA(cudaMemsetAsync(p, 0, w->bytes, s), "cudaMemsetAsync(pad rows)");
        q38::repack_q5k_tiled_kernel<<<grid, 256, 0, s>>>(m->tmp, static_cast<uint8_t*>(p), rows, cols / 256u);
    }
    Q38_CUDA(cudaGetLastError(), "launch synthetic weight kernels");
    w->d = q38_weight_desc{type, layout, rows, cols, static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(p)), 0, 0};
    return Q38_OK;
}

int synth_vec(q38_model* m, float** out, uint64_t n, uint64_t seed, float mean, float stdev, int neg_exp,
              cudaStream_t s) {
    void* p = nullptr;
    if (int rc = model_alloc(m, 4u * n, &p)) return rc;
    *out = static_cast<float*>(p);
    q38::synth_f32_kernel<<<static_cast<uint32_t>((n + 255u) / 256u), 256, 0, s>>>(*out, n, seed, mean, stdev, neg_exp);
    Q38_CUDA(cudaGetLastError(), "launch synth_f32");
    return Q38_OK;
}

template <class T>
int scratch(q38_model* m, T** out, size_t bytes) {
    void* p = nullptr;
    if (int rc = model_alloc(m, bytes, &p)) return rc;
    *out = static_cast<T*>(p);
    return Q38_OK;
}

q38_devptr dp(const void* p) { return static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(p)); }

// y (+ res) = W x with x already packed at xp (nl limbs).
int gemv_xp(q38_model* m, const GemvW& w, const uint8_t* xp, uint32_t nl, float* y, const float* res,
            cudaStream_t s) {
    const XPackView v = xpack_view(const_cast<uint8_t*>(xp), nl, w.d.cols / 256u, 1);
    if (w.d.layout == Q38_LAYOUT_B200_TILED)
        return launch_tiled_packed(w.d.data, v, nl, y, w.d.cols, w.d.rows, s, XF32(), res);
    (void)m;
    return launch_kq(w.d.ggml_type, w.d.data, v, nl, y, w.d.cols, w.d.rows, s, XF32(), res);
}

// y (+ res) = W x with f32 x packed inside every CTA, after RMSNorm with
// weight nw when nw is given.
int gemv_inline(const GemvW& w, const float* x, float* y, const float* res, cudaStream_t s,
                const float* nw = nullptr, float eps = 0.0f) {
    const XF32 xf = nw ? XF32(x, nw, eps) : XF32(x);
    if (w.d.layout == Q38_LAYOUT_B200_TILED)
        return launch_tiled_packed(w.d.data, XPackView{}, 3, y, w.d.cols, w.d.rows, s, xf, res);
    return launch_kq(w.d.ggml_type, w.d.data, XPackView{}, 3, y, w.d.cols, w.d.rows, s, xf, res);
}

// RMSNorm of x written as a three-limb x-pack (one CTA per super-block).
int norm_pack(q38_model* m, const float* x, const float* w, uint32_t n, uint8_t* xp, cudaStream_t s) {
    const XPackView v = xpack_view(xp, 3, n / 256u, 1);
    return launch_pdl(q38::rmsnorm_xpack_kernel<3>, dim3(n / 256u), dim3(256), 0, s, "launch rmsnorm_xpack", x, w, n,
                      m->cfg.rms_eps, static_cast<float*>(nullptr), v.limbs, v.gsum, v.scale);
}

// Three-limb x-pack of an f32 vector of n (one CTA per super-block).
int pack_f32(const float* x, uint32_t n, uint8_t* xp, cudaStream_t s) {
    const XPackView v = xpack_view(xp, 3, n / 256u, 1);
    return launch_pdl(q38::xpack_f32_kernel<3>, dim3(n / 256u, 1), dim3(256), 0, s, "launch xpack_f32", x, n, v.limbs,
                      v.gsum, v.scale);
}

int layer_forward(q38_model* m, uint32_t L, float* x, cudaStream_t s) {
    const q38_model_config& c = m->cfg;
    LayerW& w = m->layers[L];
    const uint32_t D = 128u, Hq = c.gdn_qk_heads, Hv = c.gdn_v_heads;
    if (int rc = norm_pack(m, x, w.attn_norm, c.hidden, m->xp, s)) return rc;
    if (!w.attn) {
        if (int rc = gemv_xp(m, w.qkvz, m->xp, 3, m->qkvz, nullptr, s)) return rc;
        if (int rc = gemv_xp(m, w.ba, m->xp, 3, m->ba, nullptr, s)) return rc;
        q38::GdnFusedArgs a{};
        a.qkv = m->qkvz;
        a.conv_w = w.conv_w;
        a.conv_in = w.conv_state[0];
        a.conv_out = w.conv_state[1];
        a.beta_raw = m->ba;
        a.alpha_raw = m->ba + Hv;
        a.dt_bias = w.dt;
        a.ssm_a = w.ssm_a;
        a.s_in = w.ssm_state;
        a.s_out = w.ssm_state;
        a.z = m->qkvz + 2u * Hq * D + Hv * D;
        a.norm_w = w.ssm_norm;
        a.y = m->ygdn;
        a.Hq = Hq;
        a.Hv = Hv;
        a.eps = c.rms_eps;
        a.scale = 1.0f / sqrtf(static_cast<float>(D));
        a.parity = m->d_pos;
        if (int rc = launch_pdl(q38::gdn_fused_kernel, dim3(Hv), dim3(512), 0, s, "launch gdn_fused", a)) return rc;
        if (int rc = pack_f32(m->ygdn, Hv * D, m->xp, s)) return rc;
        if (int rc = gemv_xp(m, w.ssm_out, m->xp, 3, x, x, s)) return rc;
    } else {
        const uint32_t AQ = c.attn_q_heads, AK = c.attn_kv_heads;
        if (int rc = gemv_xp(m, w.wq, m->xp, 3, m->qg, nullptr, s)) return rc;
        if (int rc = gemv_xp(m, w.wk, m->xp, 3, m->kv_k, nullptr, s)) return rc;
        if (int rc = gemv_xp(m, w.wv, m->xp, 3, m->kv_v, nullptr, s)) return rc;
        if (int rc = launch_pdl(q38::attn_prep_kernel, dim3(AQ + AK), dim3(q38::kAttnDim), 0, s, "launch attn_prep",
                                static_cast<const float*>(m->qg), static_cast<const float*>(m->kv_k),
                                static_cast<const float*>(m->kv_v), static_cast<const float*>(w.q_norm),
                                static_cast<const float*>(w.k_norm), static_cast<const int*>(m->d_pos), m->qr, w.kc,
                                w.vc, AQ, c.ctx, c.rope_dim, c.rope_theta, c.rms_eps))
            return rc;
        q38::AttnArgs a{};
        a.q = m->qr;
        a.qg = m->qg;
        a.kc = w.kc;
        a.vc = w.vc;
        a.pos = m->d_pos;
        a.part_o = m->part_o;
        a.part_ml = m->part_ml;
        a.out = m->ao;
        a.Hq = AQ;
        a.Hkv = AK;
        a.ctx = c.ctx;
        a.splits = std::max(1u, std::min<uint32_t>(q38::kAttnSplits, static_cast<uint32_t>(m->sm_count) / AK));
        const size_t smem = 8u * (AQ / AK) * (q38::kAttnDim + 2u) * 4u;
        if (AQ / AK != 6) return fail(Q38_ERR_UNSUPPORTED, "attention group size %u (only 6 is built)", AQ / AK);
        if (int rc = ensure_smem_attr<q38::attn_decode_kernel<6>>(m->device, smem)) return rc;
        if (int rc = launch_pdl(q38::attn_decode_kernel<6>, dim3(AK, a.splits), dim3(256), smem, s,
                                "launch attn_decode", a))
            return rc;
        if (int rc = launch_pdl(q38::attn_combine_kernel, dim3(AQ), dim3(q38::kAttnDim), 0, s, "launch attn_combine",
                                a))
            return rc;
        if (int rc = pack_f32(m->ao, AQ * q38::kAttnDim, m->xp, s)) return rc;
        if (int rc = gemv_xp(m, w.wo, m->xp, 3, x, x, s)) return rc;
    }
    if (int rc = norm_pack(m, x, w.post_norm, c.hidden, m->xp, s)) return rc;
    if (int rc = gemv_xp(m, w.gate, m->xp, 3, m->g, nullptr, s)) return rc;
    if (int rc = gemv_xp(m, w.up, m->xp, 3, m->u, nullptr, s)) return rc;
    {
        const XPackView v = xpack_view(m->xp4, 4, c.ffn / 256u, 1);
        if (int rc = launch_pdl(q38::silu_mul_xpack_kernel<4>, dim3((c.ffn / 256u + 7u) / 8u), dim3(256), 0, s,
                                "launch silu_mul_xpack", static_cast<const float*>(m->g),
                                static_cast<const float*>(m->u), c.ffn, static_cast<float*>(nullptr), v.limbs, v.gsum,
                                v.scale))
            return rc;
    }
    return gemv_xp(m, w.down, m->xp4, 4, x, x, s);
}

int model_step(q38_model* m, cudaStream_t s) {
    const q38_model_config& c = m->cfg;
    if (int rc = launch_pdl(q38::embed_q6k_kernel, dim3(1), dim3(256), 0, s, "launch embed",
                            static_cast<const uint8_t*>(dptr<uint8_t>(m->embd.d.data)),
                            static_cast<const int*>(m->d_token), c.vocab, c.hidden, m->x))
        return rc;
    for (uint32_t L = 0; L < c.n_layers; ++L)
        if (int rc = layer_forward(m, L, m->x, s)) return rc;
    if (int rc = norm_pack(m, m->x, m->out_norm, c.hidden, m->xp, s)) return rc;
    if (int rc = gemv_xp(m, m->lm_head, m->xp, 3, m->logits, nullptr, s)) return rc;
    return launch_pdl(q38::argmax_kernel, dim3(q38::kArgmaxCtas), dim3(256), 0, s, "launch argmax",
                      static_cast<const float*>(m->logits), c.vocab, m->am_v, m->am_i, m->counters + 8, m->d_token,
                      m->d_pos);
}

int check_model_config(const q38_model_config* c) {
    if (!c || c->n_layers == 0 || c->attn_every == 0 || c->hidden == 0 || c->hidden % 1024u || c->ffn % 1024u ||
        c->ffn == 0 || c->vocab == 0 || c->gdn_qk_heads == 0 || c->gdn_v_heads % c->gdn_qk_heads || c->ctx == 0 ||
        c->attn_kv_heads == 0 || c->attn_q_heads % c->attn_kv_heads || c->rope_dim > q38::kAttnDim ||
        c->rope_dim % 2u)
        return fail(Q38_ERR_INVALID, "q38_model_config: inconsistent dimensions");
    if ((c->gdn_v_heads * 128u) % 1024u || (c->attn_q_heads * q38::kAttnDim) % 1024u)
        return fail(Q38_ERR_UNSUPPORTED, "projection inputs must be multiples of 1024");
    if (c->attn_q_heads > q38::kAttnMaxGroup * c->attn_kv_heads * 8u)
        return fail(Q38_ERR_UNSUPPORTED, "too many query heads");
    return Q38_OK;
}

}  // namespace

extern "C" {

int q38_model_create(const q38_model_config* cfg, q38_model** out) {
    if (!out) return fail(Q38_ERR_INVALID, "q38_model_create: out is null");
    *out = nullptr;
    if (int rc = check_model_config(cfg)) return rc;
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    auto m = std::make_unique<q38_model>();
    m->cfg = *cfg;
    m->device = dev;
    m->sm_count = st->sm_count;
    const q38_model_config& c = m->cfg;
    m->arena_bytes = model_arena_bytes(c);
    Q38_CUDA(cudaMalloc(&m->arena, m->arena_bytes), "cudaMalloc(model arena)");
    const uint32_t H = c.hidden, F = c.ffn, D = 128u, Hq = c.gdn_qk_heads, Hv = c.gdn_v_heads;
    const uint32_t C = 2u * Hq * D + Hv * D;
    m->tmp_bytes = static_cast<size_t>(std::max({C + Hv * D, F, H, 2u * c.attn_q_heads * q38::kAttnDim})) *
                   std::max(H, F) / 256u * 176u;
    if (cudaMalloc(&m->tmp, m->tmp_bytes) != cudaSuccess) {
        cudaFree(m->arena);
        return fail(Q38_ERR_NOMEM, "cudaMalloc(repack staging)");
    }
    cudaStream_t s = nullptr;
    uint64_t seed = c.seed * 1000003ull;
    auto next_seed = [&]() { return ++seed; };
    int rc = Q38_OK;
    m->layers.resize(c.n_layers);
    for (uint32_t L = 0; L < c.n_layers && rc == Q38_OK; ++L) {
        LayerW& w = m->layers[L];
        w.attn = (L % c.attn_every) == c.attn_every - 1u;
        rc = rc ? rc : synth_vec(m.get(), &w.attn_norm, H, next_seed(), 1.0f, 0.1f, 0, s);
        rc = rc ? rc : synth_vec(m.get(), &w.post_norm, H, next_seed(), 1.0f, 0.1f, 0, s);
        if (!w.attn) {
            rc = rc ? rc : synth_gemv(m.get(), &w.qkvz, 13, 2, C + Hv * D, H, next_seed(), s);
            rc = rc ? rc : synth_gemv(m.get(), &w.ba, 12, 0, 2u * Hv, H, next_seed(), s);
            rc = rc ? rc : synth_gemv(m.get(), &w.ssm_out, 13, 2, H, Hv * D, next_seed(), s);
            rc = rc ? rc : synth_vec(m.get(), &w.conv_w, 4ull * C, next_seed(), 0.0f, 0.5f, 0, s);
            rc = rc ? rc : synth_vec(m.get(), &w.dt, Hv, next_seed(), 0.0f, 1.0f, 0, s);
            rc = rc ? rc : synth_vec(m.get(), &w.ssm_a, Hv, next_seed(), 0.0f, 1.0f, 1, s);
            rc = rc ? rc : synth_vec(m.get(), &w.ssm_norm, D, next_seed(), 1.0f, 0.1f, 0, s);
            rc = rc ? rc : synth_vec(m.get(), &w.conv_state[0], 3ull * C, next_seed(), 0.0f, 1.0f, 0, s);
            rc = rc ? rc : scratch(m.get(), &w.conv_state[1], 12ull * C);
            rc = rc ? rc : synth_vec(m.get(), &w.ssm_state, static_cast<uint64_t>(Hv) * D * D, next_seed(), 0.0f,
                                     0.02f, 0, s);
        } else {
            const uint32_t AQ = c.attn_q_heads, AK = c.attn_kv_heads, AD = q38::kAttnDim;
            rc = rc ? rc : synth_gemv(m.get(), &w.wq, 13, 2, 2u * AQ * AD, H, next_seed(), s);
            rc = rc ? rc : synth_gemv(m.get(), &w.wk, 13, 2, AK * AD, H, next_seed(), s);
            rc = rc ? rc : synth_gemv(m.get(), &w.wv, 14, 0, AK * AD, H, next_seed(), s);
            rc = rc ? rc : synth_gemv(m.get(), &w.wo, 13, 2, H, AQ * AD, next_seed(), s);
            rc = rc ? rc : synth_vec(m.get(), &w.q_norm, AD, next_seed(), 1.0f, 0.1f, 0, s);
            rc = rc ? rc : synth_vec(m.get(), &w.k_norm, AD, next_seed(), 1.0f, 0.1f, 0, s);
            rc = rc ? rc : scratch(m.get(), &w.kc, 2ull * AK * c.ctx * AD);
            rc = rc ? rc : scratch(m.get(), &w.vc, 2ull * AK * c.ctx * AD);
        }
        rc = rc ? rc : synth_gemv(m.get(), &w.gate, 12, 0, F, H, next_seed(), s);
        rc = rc ? rc : synth_gemv(m.get(), &w.up, 13, 2, F, H, next_seed(), s);
        rc = rc ? rc : synth_gemv(m.get(), &w.down, 13, 2, H, F, next_seed(), s);
    }
    rc = rc ? rc : synth_gemv(m.get(), &m->embd, 14, 0, c.vocab, H, next_seed(), s);
    rc = rc ? rc : synth_gemv(m.get(), &m->lm_head, 14, 0, c.vocab, H, next_seed(), s);
    rc = rc ? rc : synth_vec(m.get(), &m->out_norm, H, next_seed(), 1.0f, 0.1f, 0, s);
    const uint32_t AQ = c.attn_q_heads, AD = q38::kAttnDim;
    rc = rc ? rc : scratch(m.get(), &m->x, 4u * H);
    rc = rc ? rc : scratch(m.get(), &m->qkvz, 4u * (C + Hv * D));
    rc = rc ? rc : scratch(m.get(), &m->ba, 4u * 2u * Hv);
    rc = rc ? rc : scratch(m.get(), &m->ygdn, 4u * Hv * D);
    rc = rc ? rc : scratch(m.get(), &m->qg, 4u * 2u * AQ * AD);
    rc = rc ? rc : scratch(m.get(), &m->kv_k, 4u * c.attn_kv_heads * AD);
    rc = rc ? rc : scratch(m.get(), &m->kv_v, 4u * c.attn_kv_heads * AD);
    rc = rc ? rc : scratch(m.get(), &m->qr, 4u * AQ * AD);
    rc = rc ? rc : scratch(m.get(), &m->ao, 4u * AQ * AD);
    rc = rc ? rc : scratch(m.get(), &m->g, 4u * F);
    rc = rc ? rc : scratch(m.get(), &m->u, 4u * F);
    rc = rc ? rc : scratch(m.get(), &m->logits, 4u * c.vocab);
    rc = rc ? rc : scratch(m.get(), &m->xp, std::max({q38_xpack_bytes(3, H, 1), q38_xpack_bytes(3, Hv * D, 1),
                                                       q38_xpack_bytes(3, AQ * AD, 1)}));
    rc = rc ? rc : scratch(m.get(), &m->xp4, q38_xpack_bytes(4, F, 1));
    rc = rc ? rc : scratch(m.get(), &m->part_o, size_t(4u) * AQ * q38::kAttnSplits * AD);
    rc = rc ? rc : scratch(m.get(), &m->part_ml, size_t(8u) * AQ * q38::kAttnSplits);
    rc = rc ? rc : scratch(m.get(), &m->am_v, 4u * q38::kArgmaxCtas);
    rc = rc ? rc : scratch(m.get(), &m->am_i, 4u * q38::kArgmaxCtas);
    rc = rc ? rc : scratch(m.get(), &m->counters, 64);
    rc = rc ? rc : scratch(m.get(), &m->d_token, 8);
    rc = rc ? rc : scratch(m.get(), &m->d_pos, 8);
    if (rc == Q38_OK) {
        if (cudaMemsetAsync(m->counters, 0, 64, s) != cudaSuccess || cudaMemsetAsync(m->d_token, 0, 8, s) != cudaSuccess ||
            cudaMemsetAsync(m->d_pos, 0, 8, s) != cudaSuccess)
            rc = fail(Q38_ERR_CUDA, "cudaMemsetAsync(model scratch)");
    }
    if (rc == Q38_OK) {
        const cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) rc = cuda_fail(e, "synthetic model generation");
    }
    cudaFree(m->tmp);
    m->tmp = nullptr;
    if (rc != Q38_OK) {
        cudaFree(m->arena);
        return rc;
    }
    uint64_t bytes = m->embd.algo / c.vocab + m->lm_head.algo;
    for (const LayerW& w : m->layers) {
        for (const GemvW* g : {&w.qkvz, &w.ba, &w.ssm_out, &w.wq, &w.wk, &w.wv, &w.wo, &w.gate, &w.up, &w.down})
            bytes += g->algo;
    }
    m->step_bytes = bytes;
    *out = m.release();
    return Q38_OK;
}

int q38_model_destroy(q38_model* m) {
    if (!m) return Q38_OK;
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->arena) cudaFree(m->arena);
    delete m;
    return Q38_OK;
}

int q38_model_info(const q38_model* m, q38_model_stats* out) {
    if (!m || !out) return fail(Q38_ERR_INVALID, "q38_model_info: null argument");
    out->weight_bytes_per_step = m->step_bytes;
    out->arena_bytes = m->arena_used;
    uint64_t state = 0;
    for (const LayerW& w : m->layers) {
        if (w.attn) continue;
        state += 4ull * m->cfg.gdn_v_heads * 128u * 128u;
    }
    out->state_bytes_per_step = 2u * state;
    return Q38_OK;
}

int q38_model_set_position(q38_model* m, int32_t token, int32_t pos, uint64_t kv_seed) {
    if (!m || pos < 0 || static_cast<uint32_t>(pos) >= m->cfg.ctx)
        return fail(Q38_ERR_INVALID, "q38_model_set_position: position outside the cache");
    const q38_model_config& c = m->cfg;
    for (uint32_t L = 0; L < c.n_layers; ++L) {
        LayerW& w = m->layers[L];
        if (!w.attn || pos == 0) continue;
        const uint64_t n = static_cast<uint64_t>(pos) * q38::kAttnDim;
        for (uint32_t h = 0; h < c.attn_kv_heads; ++h) {
            const uint64_t off = static_cast<uint64_t>(h) * c.ctx * q38::kAttnDim;
            q38::synth_f16_kernel<<<static_cast<uint32_t>((n + 255u) / 256u), 256>>>(
                reinterpret_cast<uint16_t*>(w.kc + off), n, kv_seed * 131u + L * 8u + h, 1.0f);
            q38::synth_f16_kernel<<<static_cast<uint32_t>((n + 255u) / 256u), 256>>>(
                reinterpret_cast<uint16_t*>(w.vc + off), n, kv_seed * 137u + L * 8u + h + 4u, 1.0f);
        }
    }
    Q38_CUDA(cudaGetLastError(), "launch KV fill");
    Q38_CUDA(cudaMemcpy(m->d_token, &token, 4, cudaMemcpyHostToDevice), "set token");
    Q38_CUDA(cudaMemcpy(m->d_pos, &pos, 4, cudaMemcpyHostToDevice), "set position");
    Q38_CUDA(cudaDeviceSynchronize(), "q38_model_set_position");
    return Q38_OK;
}

int q38_model_get_position(q38_model* m, int32_t* token, int32_t* pos) {
    if (!m || !token || !pos) return fail(Q38_ERR_INVALID, "q38_model_get_position: null argument");
    Q38_CUDA(cudaMemcpy(token, m->d_token, 4, cudaMemcpyDeviceToHost), "read token");
    Q38_CUDA(cudaMemcpy(pos, m->d_pos, 4, cudaMemcpyDeviceToHost), "read position");
    return Q38_OK;
}

int q38_model_step(q38_model* m, q38_stream stream) {
    if (!m) return fail(Q38_ERR_INVALID, "q38_model_step: model is null");
    return model_step(m, as_stream(stream));
}

int q38_model_layer(q38_model* m, uint32_t layer, q38_devptr x, q38_stream stream) {
    if (!m || !x || layer >= m->cfg.n_layers) return fail(Q38_ERR_INVALID, "q38_model_layer: bad arguments");
    return layer_forward(m, layer, dptr<float>(x), as_stream(stream));
}

int q38_model_capture(q38_model* m, uint32_t steps, q38_stream stream) {
    if (!m || steps == 0 || !stream) return fail(Q38_ERR_INVALID, "q38_model_capture: needs a model, steps > 0 and a non-default stream");
    cudaStream_t s = as_stream(stream);
    if (m->graph) {
        cudaGraphExecDestroy(m->graph);
        m->graph = nullptr;
    }
    Q38_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    int rc = Q38_OK;
    for (uint32_t i = 0; i < steps && rc == Q38_OK; ++i) rc = model_step(m, s);
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(s, &g);
    if (rc != Q38_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    const cudaError_t ei = cudaGraphInstantiate(&m->graph, g, 0);
    cudaGraphDestroy(g);
    if (ei != cudaSuccess) return cuda_fail(ei, "cudaGraphInstantiate");
    m->graph_steps = steps;
    return Q38_OK;
}

int q38_model_replay(q38_model* m, q38_stream stream) {
    if (!m || !m->graph) return fail(Q38_ERR_INVALID, "q38_model_replay: no captured graph");
    Q38_CUDA(cudaGraphLaunch(m->graph, as_stream(stream)), "cudaGraphLaunch");
    return Q38_OK;
}

int q38_model_tensor(const q38_model* m, const char* name, q38_weight_desc* out) {
    if (!m || !name || !out) return fail(Q38_ERR_INVALID, "q38_model_tensor: null argument");
    std::string n(name);
    auto vec = [&](const void* p, uint32_t count) {
        *out = q38_weight_desc{Q38_TYPE_F32, Q38_LAYOUT_GGUF_NATIVE, 1, count, dp(p), 0, 0};
        return Q38_OK;
    };
    const q38_model_config& c = m->cfg;
    if (n == "token_embd") { *out = m->embd.d; return Q38_OK; }
    if (n == "output") { *out = m->lm_head.d; return Q38_OK; }
    if (n == "output_norm") return vec(m->out_norm, c.hidden);
    if (n == "x") return vec(m->x, c.hidden);
    if (n == "logits") return vec(m->logits, c.vocab);
    unsigned L = 0;
    char field[64] = {0};
    if (sscanf(name, "blk.%u.%63s", &L, field) != 2 || L >= c.n_layers)
        return fail(Q38_ERR_INVALID, "unknown tensor '%s'", name);
    const LayerW& w = m->layers[L];
    const std::string f(field);
    const uint32_t D = 128u, C = 2u * c.gdn_qk_heads * D + c.gdn_v_heads * D;
    if (f == "attn_norm") return vec(w.attn_norm, c.hidden);
    if (f == "post_attention_norm") return vec(w.post_norm, c.hidden);
    if (f == "ffn_gate") { *out = w.gate.d; return Q38_OK; }
    if (f == "ffn_up") { *out = w.up.d; return Q38_OK; }
    if (f == "ffn_down") { *out = w.down.d; return Q38_OK; }
    if (!w.attn) {
        if (f == "attn_qkvz") { *out = w.qkvz.d; return Q38_OK; }
        if (f == "ssm_ba") { *out = w.ba.d; return Q38_OK; }
        if (f == "ssm_out") { *out = w.ssm_out.d; return Q38_OK; }
        if (f == "ssm_conv1d") return vec(w.conv_w, 4u * C);
        if (f == "ssm_dt") return vec(w.dt, c.gdn_v_heads);
        if (f == "ssm_a") return vec(w.ssm_a, c.gdn_v_heads);
        if (f == "ssm_norm") return vec(w.ssm_norm, D);
        if (f == "conv_state0") return vec(w.conv_state[0], 3u * C);
        if (f == "conv_state1") return vec(w.conv_state[1], 3u * C);
        if (f == "ssm_state") return vec(w.ssm_state, c.gdn_v_heads * D * D);
    } else {
        if (f == "attn_q") { *out = w.wq.d; return Q38_OK; }
        if (f == "attn_k") { *out = w.wk.d; return Q38_OK; }
        if (f == "attn_v") { *out = w.wv.d; return Q38_OK; }
        if (f == "attn_output") { *out = w.wo.d; return Q38_OK; }
        if (f == "attn_q_norm") return vec(w.q_norm, q38::kAttnDim);
        if (f == "attn_k_norm") return vec(w.k_norm, q38::kAttnDim);
        if (f == "k_cache") return vec(w.kc, c.attn_kv_heads * c.ctx * q38::kAttnDim / 2u);
        if (f == "v_cache") return vec(w.vc, c.attn_kv_heads * c.ctx * q38::kAttnDim / 2u);
    }
    return fail(Q38_ERR_INVALID, "unknown tensor '%s'", name);
}

}  // extern "C"
