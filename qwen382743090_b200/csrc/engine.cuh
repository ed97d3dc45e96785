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
    uint64_t algo = 0;    // bytes in the GGUF block size (176/144/210/136 per 256), padding excluded
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
    GemvW wqk;  // wq and wk as one layout-2 matrix when their tiles are adjacent (else rows == 0)
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

// The slice of the model one tensor-parallel rank holds.
struct Shard {
    uint32_t rank = 0, size = 1;
    // Gated DeltaNet: q/k heads [qk0, qk0 + hq); value heads in local order
    // t * hq + j -> global qk0 + j + t * Hq (so local head j uses local q/k head j % hq).
    uint32_t hq = 0, hv = 0, qk0 = 0;
    std::vector<uint32_t> vheads;
    // ffn rows [f0, f1)
    uint32_t f0 = 0, f1 = 0;
    // attention: query heads [aq0, aq0 + aq), KV heads [ak0, ak0 + ak)
    uint32_t aq = 0, ak = 0, aq0 = 0, ak0 = 0;
    // lm_head vocab rows [v0, v1)
    uint32_t v0 = 0, v1 = 0;
};

int make_shard(const q38_model_config& c, Shard* sh) {
    const uint32_t N = c.tp_size ? c.tp_size : 1u, r = c.tp_rank;
    if (r >= N) return fail(Q38_ERR_INVALID, "tp_rank %u outside tp_size %u", r, N);
    const uint32_t Hq = c.gdn_qk_heads, Hv = c.gdn_v_heads, AQ = c.attn_q_heads, AK = c.attn_kv_heads;
    if (Hq % N || (N > 1 && (Hq / N) % 2u) || AQ % N)
        return fail(Q38_ERR_UNSUPPORTED, "tp_size %u does not divide the heads (q/k %u, query %u)", N, Hq, AQ);
    sh->rank = r;
    sh->size = N;
    sh->hq = Hq / N;
    sh->qk0 = r * sh->hq;
    sh->hv = Hv / N;
    sh->vheads.clear();
    for (uint32_t t = 0; t < Hv / Hq; ++t)
        for (uint32_t j = 0; j < sh->hq; ++j) sh->vheads.push_back(sh->qk0 + j + t * Hq);
    const uint32_t fb = c.ffn / 256u, base = fb / N, rem = fb % N;
    sh->f0 = 256u * (r * base + std::min(r, rem));
    sh->f1 = sh->f0 + 256u * (base + (r < rem ? 1u : 0u));
    sh->aq = AQ / N;
    sh->aq0 = r * sh->aq;
    const uint32_t G = AQ / AK;
    if (AK % N == 0) {
        sh->ak = AK / N;
        sh->ak0 = r * sh->ak;
    } else {
        sh->ak = 1;
        sh->ak0 = sh->aq0 / G;
        if ((sh->aq0 + sh->aq - 1u) / G != sh->ak0)
            return fail(Q38_ERR_UNSUPPORTED, "tp_size %u splits a KV group", N);
    }
    sh->v0 = static_cast<uint32_t>(static_cast<uint64_t>(c.vocab) * r / N);
    sh->v1 = static_cast<uint32_t>(static_cast<uint64_t>(c.vocab) * (r + 1) / N);
    return Q38_OK;
}

// K padded to the tiled layout's 4-super-block chunks.
uint32_t pad_k(uint32_t k) { return (k + 1023u) & ~1023u; }

}  // namespace

struct q38_model {
    q38_model_config cfg{};
    Shard sh;
    q38_comm* comm = nullptr;
    int device = 0;
    int sm_count = 148;
    bool dry = false;        // sizing pass: allocate nothing, generate nothing
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0, arena_used = 0;
    uint8_t* tmp = nullptr;  // layout-0 staging for the on-device repack
    size_t tmp_bytes = 0, tmp_need = 0;
    uint32_t* maps = nullptr;  // device staging of row / block maps
    const q38_pack* pack = nullptr;  // weight source while building (null: seeded weights)
    uint8_t* stage = nullptr;        // pack uploads and their GGUF conversion
    size_t stage_bytes = 0, stage_need = 0;
    unsigned* load_err = nullptr;    // gather outside the uploaded rows (device word)
    std::vector<LayerW> layers;
    GemvW embd, lm_head;
    float* out_norm = nullptr;
    // activations and scratch
    float *x = nullptr, *xn = nullptr, *qkvz = nullptr, *ba = nullptr, *ygdn = nullptr, *qg = nullptr, *kv_k = nullptr,
          *kv_v = nullptr, *qr = nullptr, *ao = nullptr, *g = nullptr, *u = nullptr, *logits = nullptr;
    uint8_t *xp = nullptr, *xf = nullptr;  // x-pack (layout-0 GEMVs), x-fragments (layout 2)
    float *part_o = nullptr, *part_ml = nullptr, *am_v = nullptr;
    uint32_t* am_i = nullptr;
    unsigned* counters = nullptr;  // [8]: argmax ticket
    unsigned long long* key = nullptr;  // tensor-parallel argmax key
    // tensor-parallel exchange (tp_size > 1)
    float *part = nullptr, *xalt = nullptr;  // row-parallel partial; second residual buffer
    uint32_t* tp_step = nullptr;             // decode steps taken (exchange epochs)
    uint8_t* xchg = nullptr;                 // this rank's exchange region (own cudaMalloc, IPC-exported)
    void* xchg_peer[q38::kMaxTp] = {};       // every rank's region as mapped here
    int *d_token = nullptr, *d_pos = nullptr;
    uint64_t step_bytes = 0;   // algorithmic weight bytes this rank streams per decode step
    cudaGraphExec_t graph = nullptr;
    uint32_t graph_steps = 0;
};

namespace {

constexpr size_t kMapWords = 1u << 18;  // staging for maps (256K entries: a vocab slice of rows)

int model_alloc(q38_model* m, size_t bytes, void** out) {
    const size_t off = (m->arena_used + 255u) & ~size_t(255);
    m->arena_used = off + bytes;
    if (m->dry) {
        *out = nullptr;
        return Q38_OK;
    }
    if (m->arena_used > m->arena_bytes)
        return fail(Q38_ERR_NOMEM, "model arena exhausted (%zu > %zu)", m->arena_used, m->arena_bytes);
    *out = m->arena + off;
    return Q38_OK;
}

uint64_t gemv_stored_bytes(uint32_t type, uint32_t layout, uint32_t rows, uint32_t cols) {
    if (layout == Q38_LAYOUT_B200_TILED) return q38::frag_matrix_bytes(type, rows, cols);
    return static_cast<uint64_t>(rows) * (cols / 256u) * block_bytes(type);
}

// Copy a host map to the device staging area (maps are consumed by the next
// kernel on the same stream before the next copy).
int put_map(q38_model* m, const std::vector<uint32_t>& v, const uint32_t** out, cudaStream_t s) {
    *out = nullptr;
    if (v.empty() || m->dry) return Q38_OK;
    if (v.size() > kMapWords) return fail(Q38_ERR_INVALID, "map too large");
    Q38_CUDA(cudaMemcpyAsync(m->maps, v.data(), v.size() * 4u, cudaMemcpyHostToDevice, s), "copy map");
    Q38_CUDA(cudaStreamSynchronize(s), "copy map");
    *out = m->maps;
    return Q38_OK;
}

// Size and place the shard of a weight in the arena (the same in the sizing
// and the real pass); *p is its address (null in the sizing pass).
int place_gemv(q38_model* m, GemvW* w, uint32_t type, uint32_t layout, uint32_t rows, uint32_t cols,
               const std::vector<int32_t>& kb_map, void** p) {
    w->bytes = gemv_stored_bytes(type, layout, rows, cols);
    uint32_t real_blocks = cols / 256u;
    if (!kb_map.empty()) {
        real_blocks = 0;
        for (int32_t v : kb_map) real_blocks += v >= 0 ? 1u : 0u;
    }
    w->algo = static_cast<uint64_t>(rows) * real_blocks * block_bytes(type);
    if (int rc = model_alloc(m, w->bytes, p)) return rc;
    w->d = q38_weight_desc{type, layout, rows, cols, static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(*p)), 0, 0};
    const uint64_t nblocks = static_cast<uint64_t>(rows) * (cols / 256u);
    if (layout != Q38_LAYOUT_GGUF_NATIVE) m->tmp_need = std::max<size_t>(m->tmp_need, nblocks * block_bytes(type));
    if (layout != Q38_LAYOUT_GGUF_NATIVE && !m->dry && nblocks * block_bytes(type) > m->tmp_bytes)
        return fail(Q38_ERR_INVALID, "repack staging too small");
    return Q38_OK;
}

// The row map, then the block map, in the device map staging.
int put_maps(q38_model* m, const std::vector<uint32_t>& row_map, const std::vector<int32_t>& kb_map,
             const uint32_t** rmap, const int32_t** kmap, cudaStream_t s) {
    std::vector<uint32_t> both(row_map);
    const size_t kb_off = both.size();
    for (int32_t v : kb_map) both.push_back(static_cast<uint32_t>(v));
    const uint32_t* dmap = nullptr;
    if (int rc = put_map(m, both, &dmap, s)) return rc;
    *rmap = row_map.empty() ? nullptr : dmap;
    *kmap = kb_map.empty() ? nullptr : reinterpret_cast<const int32_t*>(dmap + kb_off);
    return Q38_OK;
}

// The shard's GGUF blocks are in place (the arena for layout 0, m->tmp for
// layout 2): tile them into the arena, then wait (the staging is reused next).
int finish_gemv(q38_model* m, const GemvW& w, cudaStream_t s) {
    if (w.d.layout != Q38_LAYOUT_GGUF_NATIVE) {
        const uint32_t rows = w.d.rows, nb = w.d.cols / 256u;
        const uint32_t grid = static_cast<uint32_t>((static_cast<uint64_t>(rows) * nb + 255u) / 256u);
        uint8_t* p = dptr<uint8_t>(w.d.data);
        if (rows % q38::kF8Rows) Q38_CUDA(cudaMemsetAsync(p, 0, w.bytes, s), "cudaMemsetAsync(pad rows)");
        if (w.d.ggml_type == Q38_TYPE_Q5_K)
            q38::repack_frag_kernel<13><<<grid, 256, 0, s>>>(m->tmp, p, rows, nb);
        else if (w.d.ggml_type == Q38_TYPE_Q6_K)
            q38::repack_frag_q6_kernel<<<grid, 256, 0, s>>>(m->tmp, p, rows, nb);
        else if (w.d.ggml_type == Q38_TYPE_IQ4_XS)
            q38::repack_frag_iq4_kernel<<<grid, 256, 0, s>>>(m->tmp, p, rows, nb);
        else
            q38::repack_frag_kernel<12><<<grid, 256, 0, s>>>(m->tmp, p, rows, nb);
    }
    Q38_CUDA(cudaGetLastError(), "launch weight kernels");
    Q38_CUDA(cudaStreamSynchronize(s), "weights");
    return Q38_OK;
}

// A rows x cols shard of a global rows_g x cols_g matrix: local row i is global
// row row_map[i] (identity when empty); local super-block b is global block
// kb_map[b] (identity when empty, -1 = zero padding).  cols is the local K
// (padded for layout 2).
int synth_gemv(q38_model* m, GemvW* w, uint32_t type, uint32_t layout, uint32_t rows, uint32_t cols,
               uint32_t cols_g, const std::vector<uint32_t>& row_map, const std::vector<int32_t>& kb_map,
               uint64_t seed, cudaStream_t s) {
    void* p = nullptr;
    if (int rc = place_gemv(m, w, type, layout, rows, cols, kb_map, &p)) return rc;
    if (m->dry) return Q38_OK;
    const uint32_t* rmap = nullptr;
    const int32_t* kmap = nullptr;
    if (int rc = put_maps(m, row_map, kb_map, &rmap, &kmap, s)) return rc;
    const uint64_t nblocks = static_cast<uint64_t>(rows) * (cols / 256u);
    const uint32_t grid = static_cast<uint32_t>((nblocks + 255u) / 256u);
    uint8_t* dst = layout == Q38_LAYOUT_GGUF_NATIVE ? static_cast<uint8_t*>(p) : m->tmp;
    q38::synth_blocks_kernel<<<grid, 256, 0, s>>>(type, dst, rows, cols / 256u, rmap, kmap, cols_g / 256u, seed);
    return finish_gemv(m, *w, s);
}

// n f32 values; element i is global element chunk_map[i / chunk] * chunk + i % chunk.
int synth_vec(q38_model* m, float** out, uint64_t n, uint64_t seed, float mean, float stdev, int neg_exp,
              cudaStream_t s, const std::vector<uint32_t>& chunk_map = {}, uint32_t chunk = 1) {
    void* p = nullptr;
    if (int rc = model_alloc(m, 4u * n, &p)) return rc;
    *out = static_cast<float*>(p);
    if (m->dry) return Q38_OK;
    const uint32_t* dmap = nullptr;
    if (int rc = put_map(m, chunk_map, &dmap, s)) return rc;
    q38::synth_f32_kernel<<<static_cast<uint32_t>((n + 255u) / 256u), 256, 0, s>>>(*out, n, seed, mean, stdev, neg_exp,
                                                                                  dmap, chunk);
    Q38_CUDA(cudaGetLastError(), "launch synth_f32");
    Q38_CUDA(cudaStreamSynchronize(s), "synthetic vector");
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

std::vector<uint32_t> iota_rows(uint32_t first, uint32_t n) {
    std::vector<uint32_t> v(n);
    for (uint32_t i = 0; i < n; ++i) v[i] = first + i;
    return v;
}

// Global rows of 128-row heads, in the order given.
std::vector<uint32_t> head_rows(const std::vector<uint32_t>& heads, uint32_t first_row, uint32_t head_dim) {
    std::vector<uint32_t> v;
    v.reserve(heads.size() * head_dim);
    for (uint32_t h : heads)
        for (uint32_t i = 0; i < head_dim; ++i) v.push_back(first_row + h * head_dim + i);
    return v;
}

// K blocks of a row-parallel shard padded to whole 4-block chunks.
std::vector<int32_t> pad_blocks(std::vector<int32_t> kb) {
    while (kb.size() % 4u) kb.push_back(-1);
    return kb;
}

// ---- weights from a Q38PACK ------------------------------------------------------
const q38_tensor_record* pack_tensor(const q38_model* m, const std::string& name) {
    for (const q38_tensor_record& t : m->pack->tensors)
        if (name == t.name) return &t;
    return nullptr;
}

uint64_t stage_align(uint64_t v) { return (v + 255u) & ~uint64_t(255); }

int pack_copy(q38_model* m, uint8_t* dst, uint64_t file_off, uint64_t bytes, cudaStream_t s) {
    if (bytes == 0) return Q38_OK;
    if (file_off > m->pack->size || bytes > m->pack->size - file_off)
        return fail(Q38_ERR_INVALID, "q38pack: tensor bytes outside the file");
    Q38_CUDA(cudaMemcpyAsync(dst, m->pack->map + file_off, bytes, cudaMemcpyHostToDevice, s), "upload pack rows");
    return Q38_OK;
}

// f32 vector of n (this rank's elements, chunk-mapped as in synth_vec) from the
// f32 pack tensor `name` of n_g elements.
int load_vec(q38_model* m, float** out, uint64_t n, const std::string& name, uint64_t n_g, cudaStream_t s,
             const std::vector<uint32_t>& chunk_map, uint32_t chunk) {
    void* p = nullptr;
    if (int rc = model_alloc(m, 4u * n, &p)) return rc;
    *out = static_cast<float*>(p);
    const q38_tensor_record* t = pack_tensor(m, name);
    if (!t) return fail(Q38_ERR_INVALID, "q38pack: no tensor '%s'", name.c_str());
    uint64_t count = 1;
    for (uint32_t d = 0; d < t->ndim; ++d) count *= t->dims[d];
    if (t->ggml_type != Q38_TYPE_F32 || t->layout != Q38_LAYOUT_GGUF_NATIVE || count != n_g ||
        t->stored_bytes < 4u * n_g)
        return fail(Q38_ERR_INVALID, "q38pack: tensor '%s' is not f32[%llu]", name.c_str(),
                    static_cast<unsigned long long>(n_g));
    m->stage_need = std::max<size_t>(m->stage_need, 4u * n_g);
    if (m->dry) return Q38_OK;
    if (int rc = pack_copy(m, m->stage, t->data_offset, 4u * n_g, s)) return rc;
    const uint32_t* dmap = nullptr;
    if (int rc = put_map(m, chunk_map, &dmap, s)) return rc;
    q38::gather_f32_kernel<<<static_cast<uint32_t>((n + 255u) / 256u), 256, 0, s>>>(
        *out, n, reinterpret_cast<const float*>(m->stage), n_g, dmap, chunk, m->load_err);
    Q38_CUDA(cudaGetLastError(), "launch gather_f32");
    Q38_CUDA(cudaStreamSynchronize(s), "pack vector");
    return Q38_OK;
}

// One source tensor of a weight and the window of its rows the shard reads.
struct PackSrc {
    const q38_tensor_record* t = nullptr;
    uint32_t rows = 0, lo = 0, hi = 0;
    uint64_t raw_off = 0, raw_bytes = 0, gguf_off = 0;
};

// The shard of a weight whose global matrix is pack tensor na (rows
// [0, rows_a)) followed by nb2's rows (empty: none).  Only the row window the
// shard reads is uploaded; layout-1 and layout-2 windows are converted to
// GGUF blocks on the device before the gather.
int load_gemv(q38_model* m, GemvW* w, uint32_t type, uint32_t layout, uint32_t rows, uint32_t cols,
              uint32_t cols_g, const std::vector<uint32_t>& row_map, const std::vector<int32_t>& kb_map,
              const std::string& na, const std::string& nb2, cudaStream_t s) {
    void* p = nullptr;
    if (int rc = place_gemv(m, w, type, layout, rows, cols, kb_map, &p)) return rc;
    const uint32_t bb = block_bytes(type), nb_g = cols_g / 256u;
    PackSrc src[2];
    const std::string* names[2] = {&na, &nb2};
    for (int k = 0; k < 2; ++k) {
        if (names[k]->empty()) continue;
        const q38_tensor_record* t = pack_tensor(m, *names[k]);
        if (!t) return fail(Q38_ERR_INVALID, "q38pack: no tensor '%s'", names[k]->c_str());
        if (t->ggml_type != type || t->ndim < 2 || t->dims[0] != cols_g || t->dims[1] == 0 || t->dims[1] > 0xffffffffull)
            return fail(Q38_ERR_INVALID, "q38pack: tensor '%s' is type %u [%llu x %llu], the model needs type %u with %u columns",
                        t->name, t->ggml_type, static_cast<unsigned long long>(t->dims[1]),
                        static_cast<unsigned long long>(t->dims[0]), type, cols_g);
        const uint64_t rows_t = t->dims[1], blocks = rows_t * nb_g;
        if (t->layout == Q38_LAYOUT_SM86_Q5K_SOA) {
            if (type != Q38_TYPE_Q5_K || t->data_offset + blocks * 20u > t->aux0_offset ||
                t->aux0_offset + blocks * 32u > t->aux1_offset || t->aux1_offset + blocks * 128u > t->data_offset + t->stored_bytes)
                return fail(Q38_ERR_INVALID, "q38pack: SoA planes of '%s' do not hold its blocks", t->name);
        } else if (t->layout == Q38_LAYOUT_GGUF_NATIVE) {
            if (t->stored_bytes < blocks * bb) return fail(Q38_ERR_INVALID, "q38pack: tensor '%s' is truncated", t->name);
        } else if (t->layout != Q38_LAYOUT_B200_TILED) {
            return fail(Q38_ERR_UNSUPPORTED, "q38pack: layout %u of '%s'", t->layout, t->name);
        }
        src[k].t = t;
        src[k].rows = static_cast<uint32_t>(rows_t);
        src[k].lo = src[k].rows;
        src[k].hi = 0;
    }
    const uint32_t split = src[0].rows, total = split + src[1].rows;
    for (uint32_t i = 0; i < rows; ++i) {
        const uint32_t g = row_map.empty() ? i : row_map[i];
        if (g >= total) return fail(Q38_ERR_INVALID, "q38pack: row %u outside '%s' (%u rows)", g, na.c_str(), total);
        PackSrc& e = src[g < split ? 0 : 1];
        const uint32_t r = g < split ? g : g - split;
        e.lo = std::min(e.lo, r);
        e.hi = std::max(e.hi, r + 1u);
    }
    for (int32_t v : kb_map)
        if (v >= static_cast<int32_t>(nb_g)) return fail(Q38_ERR_INVALID, "q38pack: block map outside '%s'", na.c_str());
    uint64_t off = 0;
    for (PackSrc& e : src) {
        if (!e.t || e.lo >= e.hi) {
            e.t = nullptr;
            continue;
        }
        if (e.t->layout == Q38_LAYOUT_B200_TILED) {  // whole tiles of 8 rows
            e.lo &= ~7u;
            e.hi = std::min(e.rows, (e.hi + 7u) & ~7u);
        }
        const uint64_t n = e.hi - e.lo;
        e.raw_bytes = e.t->layout == Q38_LAYOUT_SM86_Q5K_SOA ? 3u * 256u + n * nb_g * (20u + 32u + 128u)
                      : e.t->layout == Q38_LAYOUT_B200_TILED ? (n + 7u) / 8u * (nb_g / 2u) * q38::frag_tile_bytes(type)
                                                             : 0u;
        e.raw_off = stage_align(off);
        off = e.raw_off + e.raw_bytes;
        e.gguf_off = stage_align(off);
        off = e.gguf_off + n * nb_g * bb;
    }
    m->stage_need = std::max<size_t>(m->stage_need, off);
    if (m->dry) return Q38_OK;
    if (off > m->stage_bytes) return fail(Q38_ERR_INVALID, "pack staging too small");
    q38::GatherSeg seg[2] = {{nullptr, 0, 0}, {nullptr, 0, 0}};
    for (int k = 0; k < 2; ++k) {
        const PackSrc& e = src[k];
        if (!e.t) continue;
        const uint64_t n = e.hi - e.lo, nblk = n * nb_g;
        uint8_t* raw = m->stage + e.raw_off;
        uint8_t* gg = m->stage + e.gguf_off;
        const uint32_t grid = static_cast<uint32_t>((nblk + 255u) / 256u);
        if (e.t->layout == Q38_LAYOUT_GGUF_NATIVE) {
            if (int rc = pack_copy(m, gg, e.t->data_offset + e.lo * uint64_t(nb_g) * bb, nblk * bb, s)) return rc;
        } else if (e.t->layout == Q38_LAYOUT_SM86_Q5K_SOA) {
            const uint64_t first = e.lo * uint64_t(nb_g);
            uint8_t* meta = raw;
            uint8_t* qh = raw + stage_align(nblk * 20u);
            uint8_t* qs = qh + stage_align(nblk * 32u);
            if (int rc = pack_copy(m, meta, e.t->data_offset + first * 20u, nblk * 20u, s)) return rc;
            if (int rc = pack_copy(m, qh, e.t->aux0_offset + first * 32u, nblk * 32u, s)) return rc;
            if (int rc = pack_copy(m, qs, e.t->aux1_offset + first * 128u, nblk * 128u, s)) return rc;
            q38::soa_q5k_to_gguf_kernel<<<grid, 256, 0, s>>>(meta, qh, qs, nblk, gg);
        } else {
            const uint64_t tb = q38::frag_tile_bytes(type), per_oct = (nb_g / 2u) * tb;
            if (int rc = pack_copy(m, raw, e.t->data_offset + (e.lo / 8u) * per_oct, e.raw_bytes, s)) return rc;
            if (type == Q38_TYPE_Q5_K)
                q38::unfrag_kernel<13><<<grid, 256, 0, s>>>(raw, gg, static_cast<uint32_t>(n), nb_g);
            else
                q38::unfrag_kernel<12><<<grid, 256, 0, s>>>(raw, gg, static_cast<uint32_t>(n), nb_g);
        }
        seg[k] = q38::GatherSeg{gg, e.lo, e.hi};
    }
    const uint32_t* rmap = nullptr;
    const int32_t* kmap = nullptr;
    if (int rc = put_maps(m, row_map, kb_map, &rmap, &kmap, s)) return rc;
    const uint64_t nblocks = static_cast<uint64_t>(rows) * (cols / 256u);
    uint8_t* dst = layout == Q38_LAYOUT_GGUF_NATIVE ? static_cast<uint8_t*>(p) : m->tmp;
    q38::gather_blocks_kernel<<<static_cast<uint32_t>((nblocks + 255u) / 256u), 256, 0, s>>>(
        bb, dst, rows, cols / 256u, rmap, kmap, nb_g, seg[0], seg[1], split, m->load_err);
    return finish_gemv(m, *w, s);
}

// Seeded (m->pack null) or loaded: the weight's global matrix is the pack
// tensor(s) named, or the seeded matrix of `seed`.
int make_gemv(q38_model* m, GemvW* w, uint32_t type, uint32_t layout, uint32_t rows, uint32_t cols, uint32_t cols_g,
              const std::vector<uint32_t>& row_map, const std::vector<int32_t>& kb_map, uint64_t seed,
              cudaStream_t s, const std::string& na, const std::string& nb2 = std::string()) {
    if (m->pack) return load_gemv(m, w, type, layout, rows, cols, cols_g, row_map, kb_map, na, nb2, s);
    return synth_gemv(m, w, type, layout, rows, cols, cols_g, row_map, kb_map, seed, s);
}

int make_vec(q38_model* m, float** out, uint64_t n, const std::string& name, uint64_t n_g, uint64_t seed, float mean,
             float stdev, int neg_exp, cudaStream_t s, const std::vector<uint32_t>& chunk_map = {}, uint32_t chunk = 1) {
    if (m->pack) return load_vec(m, out, n, name, n_g, s, chunk_map, chunk);
    return synth_vec(m, out, n, seed, mean, stdev, neg_exp, s, chunk_map, chunk);
}

// Generate (or size, in the dry pass) every tensor of this rank's shard.
int build_model(q38_model* m, cudaStream_t s) {
    const q38_model_config& c = m->cfg;
    const Shard& sh = m->sh;
    const bool tp = sh.size > 1;
    const uint32_t H = c.hidden, F = c.ffn, D = 128u, Hq = c.gdn_qk_heads, Hv = c.gdn_v_heads;
    const uint32_t C = 2u * Hq * D + Hv * D;       // global conv channels (q | k | v)
    const uint32_t Cl = 2u * sh.hq * D + sh.hv * D;  // local
    const uint32_t AQ = c.attn_q_heads, AD = q38::kAttnDim;
    const uint32_t Fl = sh.f1 - sh.f0;
    const uint32_t gate_t = c.ffn_gate_type == Q38_TYPE_IQ4_XS ? Q38_TYPE_IQ4_XS : Q38_TYPE_Q4_K;
    uint64_t seed = c.seed * 1000003ull;
    auto next_seed = [&]() { return ++seed; };
    const std::vector<uint32_t> none;
    const std::vector<int32_t> nokb;

    // local q/k heads (global ids) and conv channel map
    std::vector<uint32_t> qk_heads = iota_rows(sh.qk0, sh.hq);
    std::vector<uint32_t> ch_map;
    if (tp) {
        for (uint32_t v : head_rows(qk_heads, 0, D)) ch_map.push_back(v);
        for (uint32_t v : head_rows(qk_heads, Hq * D, D)) ch_map.push_back(v);
        for (uint32_t v : head_rows(sh.vheads, 2u * Hq * D, D)) ch_map.push_back(v);
    }
    std::vector<uint32_t> qkvz_rows, ba_rows, conv_state_map;
    std::vector<int32_t> out_kb;
    if (tp) {
        qkvz_rows = ch_map;
        for (uint32_t v : head_rows(sh.vheads, C, D)) qkvz_rows.push_back(v);  // z
        for (uint32_t h : sh.vheads) ba_rows.push_back(h);
        for (uint32_t h : sh.vheads) ba_rows.push_back(Hv + h);
        for (uint32_t j = 0; j < sh.hv; j += 2) out_kb.push_back(static_cast<int32_t>(sh.vheads[j] / 2u));
        out_kb = pad_blocks(out_kb);
        for (uint32_t row = 0; row < 3; ++row)
            for (uint32_t ch : ch_map) conv_state_map.push_back(row * C + ch);
    }
    std::vector<uint32_t> conv_w_map;  // [C][4] elements: chunks of 4
    if (tp) conv_w_map = ch_map;
    const uint32_t out_k = tp ? static_cast<uint32_t>(out_kb.size()) * 256u : Hv * D;
    std::vector<int32_t> wo_kb;
    if (tp) {
        for (uint32_t j = 0; j < sh.aq; ++j) wo_kb.push_back(static_cast<int32_t>(sh.aq0 + j));
        wo_kb = pad_blocks(wo_kb);
    }
    const uint32_t wo_k = tp ? static_cast<uint32_t>(wo_kb.size()) * 256u : AQ * AD;
    std::vector<int32_t> down_kb;
    if (tp) {
        for (uint32_t b = sh.f0 / 256u; b < sh.f1 / 256u; ++b) down_kb.push_back(static_cast<int32_t>(b));
        down_kb = pad_blocks(down_kb);
    }
    const uint32_t down_k = tp ? static_cast<uint32_t>(down_kb.size()) * 256u : F;

    int rc = Q38_OK;
    m->layers.assign(c.n_layers, LayerW{});
    for (uint32_t L = 0; L < c.n_layers && rc == Q38_OK; ++L) {
        LayerW& w = m->layers[L];
        w.attn = (L % c.attn_every) == c.attn_every - 1u;
        const std::string b = "blk." + std::to_string(L) + ".";
        rc = rc ? rc : make_vec(m, &w.attn_norm, H, b + "attn_norm.weight", H, next_seed(), 1.0f, 0.1f, 0, s);
        rc = rc ? rc : make_vec(m, &w.post_norm, H, b + "post_attention_norm.weight", H, next_seed(), 1.0f, 0.1f, 0, s);
        if (!w.attn) {
            rc = rc ? rc : make_gemv(m, &w.qkvz, 13, 2, Cl + sh.hv * D, H, H, qkvz_rows, nokb, next_seed(), s,
                                     b + "attn_qkv.weight", b + "attn_gate.weight");
            rc = rc ? rc : make_gemv(m, &w.ba, 12, 2, 2u * sh.hv, H, H, ba_rows, nokb, next_seed(), s,
                                     b + "ssm_beta.weight", b + "ssm_alpha.weight");
            rc = rc ? rc : make_gemv(m, &w.ssm_out, 13, 2, H, out_k, Hv * D, none, out_kb, next_seed(), s,
                                     b + "ssm_out.weight");
            rc = rc ? rc : make_vec(m, &w.conv_w, 4ull * Cl, b + "ssm_conv1d.weight", 4ull * C, next_seed(), 0.0f, 0.5f,
                                    0, s, conv_w_map, 4);
            rc = rc ? rc : make_vec(m, &w.dt, sh.hv, b + "ssm_dt.bias", Hv, next_seed(), 0.0f, 1.0f, 0, s,
                                    tp ? sh.vheads : none, 1);
            rc = rc ? rc : make_vec(m, &w.ssm_a, sh.hv, b + "ssm_a", Hv, next_seed(), 0.0f, 1.0f, 1, s,
                                    tp ? sh.vheads : none, 1);
            rc = rc ? rc : make_vec(m, &w.ssm_norm, D, b + "ssm_norm.weight", D, next_seed(), 1.0f, 0.1f, 0, s);
            rc = rc ? rc : synth_vec(m, &w.conv_state[0], 3ull * Cl, next_seed(), 0.0f, 1.0f, 0, s, conv_state_map, 1);
            rc = rc ? rc : scratch(m, &w.conv_state[1], 12ull * Cl);
            rc = rc ? rc : synth_vec(m, &w.ssm_state, static_cast<uint64_t>(sh.hv) * D * D, next_seed(), 0.0f, 0.02f,
                                     0, s, tp ? sh.vheads : none, D * D);
        } else {
            rc = rc ? rc : make_gemv(m, &w.wq, 13, 2, 2u * sh.aq * AD, H, H,
                                     tp ? iota_rows(2u * sh.aq0 * AD, 2u * sh.aq * AD) : none, nokb, next_seed(), s,
                                     b + "attn_q.weight");
            rc = rc ? rc : make_gemv(m, &w.wk, 13, 2, sh.ak * AD, H, H, tp ? iota_rows(sh.ak0 * AD, sh.ak * AD) : none,
                                     nokb, next_seed(), s, b + "attn_k.weight");
            // wq's tiles end where wk's begin (whole row octets, 256-byte sizes), so
            // the pair is one matrix of rows q|gate then k for a single GEMV.
            if (rc == Q38_OK && w.wq.d.rows % q38::kF8Rows == 0 && w.wk.d.data == w.wq.d.data + w.wq.bytes) {
                w.wqk = w.wq;
                w.wqk.d.rows = w.wq.d.rows + w.wk.d.rows;
                w.wqk.bytes = w.wq.bytes + w.wk.bytes;
                w.wqk.algo = w.wq.algo + w.wk.algo;
            }
            rc = rc ? rc : make_gemv(m, &w.wv, 14, 2, sh.ak * AD, H, H, tp ? iota_rows(sh.ak0 * AD, sh.ak * AD) : none,
                                     nokb, next_seed(), s, b + "attn_v.weight");
            rc = rc ? rc : make_gemv(m, &w.wo, 13, 2, H, wo_k, AQ * AD, none, wo_kb, next_seed(), s,
                                     b + "attn_output.weight");
            rc = rc ? rc : make_vec(m, &w.q_norm, AD, b + "attn_q_norm.weight", AD, next_seed(), 1.0f, 0.1f, 0, s);
            rc = rc ? rc : make_vec(m, &w.k_norm, AD, b + "attn_k_norm.weight", AD, next_seed(), 1.0f, 0.1f, 0, s);
            rc = rc ? rc : scratch(m, &w.kc, 2ull * sh.ak * c.ctx * AD);
            rc = rc ? rc : scratch(m, &w.vc, 2ull * sh.ak * c.ctx * AD);
        }
        const std::vector<uint32_t> frows = tp ? iota_rows(sh.f0, Fl) : none;
        rc = rc ? rc : make_gemv(m, &w.gate, gate_t, 2, Fl, H, H, frows, nokb, next_seed(), s, b + "ffn_gate.weight");
        rc = rc ? rc : make_gemv(m, &w.up, 13, 2, Fl, H, H, frows, nokb, next_seed(), s, b + "ffn_up.weight");
        rc = rc ? rc : make_gemv(m, &w.down, 13, 2, H, down_k, F, none, down_kb, next_seed(), s, b + "ffn_down.weight");
    }
    rc = rc ? rc : make_gemv(m, &m->embd, 14, 0, c.vocab, H, H, none, nokb, next_seed(), s, "token_embd.weight");
    rc = rc ? rc : make_gemv(m, &m->lm_head, 14, 2, sh.v1 - sh.v0, H, H, tp ? iota_rows(sh.v0, sh.v1 - sh.v0) : none,
                             nokb, next_seed(), s, "output.weight");
    rc = rc ? rc : make_vec(m, &m->out_norm, H, "output_norm.weight", H, next_seed(), 1.0f, 0.1f, 0, s);
    const size_t xp_bytes = q38_xpack_bytes(4, H, 1);
    const size_t xf_bytes = q38::xfrag1_bytes(std::max({H, out_k, wo_k, down_k}) / 256u);
    rc = rc ? rc : scratch(m, &m->x, 4u * H);
    rc = rc ? rc : scratch(m, &m->xn, 4u * H);
    rc = rc ? rc : scratch(m, &m->qkvz, 4u * (Cl + sh.hv * D));
    rc = rc ? rc : scratch(m, &m->ba, 4u * 2u * sh.hv);
    rc = rc ? rc : scratch(m, &m->ygdn, 4u * sh.hv * D);
    rc = rc ? rc : scratch(m, &m->qg, 4u * 2u * sh.aq * AD);
    rc = rc ? rc : scratch(m, &m->kv_k, 4u * sh.ak * AD);
    rc = rc ? rc : scratch(m, &m->kv_v, 4u * sh.ak * AD);
    rc = rc ? rc : scratch(m, &m->qr, 4u * sh.aq * AD);
    rc = rc ? rc : scratch(m, &m->ao, 4u * sh.aq * AD);
    rc = rc ? rc : scratch(m, &m->g, 4u * Fl);
    rc = rc ? rc : scratch(m, &m->u, 4u * Fl);
    rc = rc ? rc : scratch(m, &m->logits, 4u * (sh.v1 - sh.v0));
    rc = rc ? rc : scratch(m, &m->xp, xp_bytes);
    rc = rc ? rc : scratch(m, &m->xf, xf_bytes);
    rc = rc ? rc : scratch(m, &m->part_o, size_t(4u) * sh.aq * q38::kAttnSplits * AD);
    rc = rc ? rc : scratch(m, &m->part_ml, size_t(8u) * sh.aq * q38::kAttnSplits);
    rc = rc ? rc : scratch(m, &m->am_v, 4u * q38::kArgmaxCtas);
    rc = rc ? rc : scratch(m, &m->am_i, 4u * q38::kArgmaxCtas);
    rc = rc ? rc : scratch(m, &m->counters, 64);
    rc = rc ? rc : scratch(m, &m->key, 64);
    rc = rc ? rc : scratch(m, &m->d_token, 8);
    rc = rc ? rc : scratch(m, &m->d_pos, 8);
    if (tp) {
        rc = rc ? rc : scratch(m, &m->part, 4u * H);
        rc = rc ? rc : scratch(m, &m->xalt, 4u * H);
        rc = rc ? rc : scratch(m, &m->tp_step, 64);
    }
    return rc;
}

// y (+ res) = W x with x already packed: layout-2 weights read the
// x-fragments m->xf, layout-0 weights (the Q6_K attention v and vocabulary
// projections) the four-limb x-pack m->xp.  Four limbs (30-bit x): with
// 23-bit x, 4 of the 151936 vocabulary rows exceeded the GEMV tolerance.
int gemv_x(q38_model* m, const GemvW& w, float* y, const float* res, cudaStream_t s) {
    if (w.d.layout == Q38_LAYOUT_B200_TILED)
        return launch_frag(w.d.ggml_type, w.d.data, m->xf, y, w.d.cols, w.d.rows, s, res);
    const XPackView v = xpack_view(m->xp, 4, w.d.cols / 256u, 1);
    return launch_kq(w.d.ggml_type, w.d.data, v, 4, y, w.d.cols, w.d.rows, s, XF32(), res);
}

// Two GEMVs over the current x-fragments (y_a = W_a x, y_b = W_b x): one
// launch when both are layout 2 of the same K and a pair kernel exists,
// else two.
int gemv_pair(q38_model* m, const GemvW& wa, float* ya, const GemvW& wb, float* yb, cudaStream_t s) {
    if (wa.d.layout == Q38_LAYOUT_B200_TILED && wb.d.layout == Q38_LAYOUT_B200_TILED && wa.d.cols == wb.d.cols) {
        const int rc = launch_frag_pair(wa.d.ggml_type, wa.d.data, wa.d.rows, ya, wb.d.ggml_type, wb.d.data,
                                        wb.d.rows, yb, m->xf, wa.d.cols, s);
        if (rc != Q38_ERR_UNSUPPORTED) return rc;
    }
    if (int rc = gemv_x(m, wa, ya, nullptr, s)) return rc;
    return gemv_x(m, wb, yb, nullptr, s);
}

// RMSNorm of x written as x-fragments and, when with_xpack, also as the
// four-limb x-pack for layout-0 consumers (one CTA per super-block).
int norm_pack(q38_model* m, const float* x, const float* w, uint32_t n, bool with_xpack, cudaStream_t s,
              float* y = nullptr) {
    const XPackView v = xpack_view(m->xp, 4, n / 256u, 1);
    return launch_pdl(q38::rmsnorm_xpack_kernel<4>, dim3(n / 256u), dim3(256), 0, s, "launch rmsnorm_xpack", x, w, n,
                      m->cfg.rms_eps, y, with_xpack ? v.limbs : nullptr, v.gsum, v.scale, m->xf);
}

// x-fragments of an f32 vector of n, zero-padded to n_pack (8 super-blocks per CTA).
int pack_f32(q38_model* m, const float* x, uint32_t n, uint32_t n_pack, cudaStream_t s) {
    const uint32_t nbp = n_pack / 256u;
    return launch_pdl(q38::f32_xfrag_pad_kernel, dim3((nbp + 7u) / 8u), dim3(256), 0, s, "launch f32_xfrag", x, n, nbp,
                      m->xf);
}

// Tensor-parallel exchange `instance` of this step: x_out = x_in + every
// rank's row-parallel partial (m->part here), then RMSNorm by norm_w (null:
// none) into the x-fragments and, when with_xpack, the four-limb x-pack.
int tp_reduce_norm(q38_model* m, const float* x_in, float* x_out, const float* norm_w, bool with_xpack,
                   uint32_t instance, cudaStream_t s, float* y = nullptr) {
    if (!m->xchg) return fail(Q38_ERR_INVALID, "tensor-parallel model has no communicator (q38_model_set_comm)");
    const uint32_t H = m->cfg.hidden;
    q38::TpReduceArgs a{};
    a.x_in = x_in;
    a.x_out = x_out;
    a.part = m->part;
    for (uint32_t r = 0; r < m->sh.size; ++r) a.region[r] = static_cast<uint4*>(m->xchg_peer[r]);
    a.step = m->tp_step;
    a.norm_w = norm_w;
    a.frag = m->xf;
    const XPackView v = xpack_view(m->xp, 4, H / 256u, 1);
    a.limbs = with_xpack ? v.limbs : nullptr;
    a.y = y;
    a.gsum = v.gsum;
    a.scale = v.scale;
    a.n = H;
    a.rank = m->sh.rank;
    a.size = m->sh.size;
    a.instance = instance;
    a.eps = m->cfg.rms_eps;
    return launch_pdl(q38::tp_reduce_norm_kernel<4>, dim3(H / 256u), dim3(q38::kTpWarps * 32u), 0, s,
                      "launch tp_reduce_norm", a);
}

int tp_next_step(q38_model* m, cudaStream_t s) {
    return launch_pdl(q38::tp_step_kernel, dim3(1), dim3(32), 0, s, "launch tp_step", m->tp_step);
}

template <int G>
int launch_attn(q38_model* m, const q38::AttnArgs& a, cudaStream_t s) {
    const size_t smem = q38::attn_smem_bytes<G>();
    if (int rc = ensure_smem_attr<q38::attn_decode_kernel<G>>(m->device, smem)) return rc;
    return launch_pdl(q38::attn_decode_kernel<G>, dim3(a.Hkv, a.splits), dim3(q38::kAttnWarps * 32u), smem, s,
                      "launch attn_decode", a);
}

// One layer on the residual x (updated in place).  At tp_size 1 the layer
// starts with its RMSNorm and the row-parallel GEMVs add the residual into x.
// At tp_size > 1 they write this rank's partial to m->part and the layer's two
// exchanges (instances 2L and 2L+1 of the step) add every rank's partial to
// the residual: the first normalises for the FFN, the second for the next
// consumer (next_norm, null: none; with the x-pack when next_xpack).  in_packed:
// the attention-norm x-fragments (and x-pack) of x are in place already (the
// previous layer's second exchange made them).
// What a layer's input RMSNorm must also write besides the x-fragments: the
// x-pack for a layout-0 attention v, f32 for a Q6_K-tiled one (Q6 x-fragments
// packed in its CTAs).
bool norm_xpack(const LayerW& w) { return w.attn && w.wv.d.layout == Q38_LAYOUT_GGUF_NATIVE; }
float* norm_f32(q38_model* m, const LayerW& w) {
    return w.attn && w.wv.d.layout == Q38_LAYOUT_B200_TILED ? m->xn : nullptr;
}

int layer_forward(q38_model* m, uint32_t L, float* x, cudaStream_t s, bool in_packed = false,
                  const float* next_norm = nullptr, bool next_xpack = false, float* next_y = nullptr) {
    const q38_model_config& c = m->cfg;
    const Shard& sh = m->sh;
    LayerW& w = m->layers[L];
    const uint32_t D = 128u;
    const bool tp = sh.size > 1;
    const float* res = tp ? nullptr : x;
    float* yrow = tp ? m->part : x;  // row-parallel projection output
    // The norm and packing kernels stay separate from the GEMVs: in the PDL
    // chain they run while the next GEMV's CTAs already stream their first
    // weight tiles, which costs less than packing inside every GEMV CTA
    // (measured: 5.44 vs 5.97 ms per token with the in-CTA variants).
    if (!(tp && in_packed))
        if (int rc = norm_pack(m, x, w.attn_norm, c.hidden, norm_xpack(w), s, norm_f32(m, w))) return rc;
    if (!w.attn) {
        if (int rc = gemv_pair(m, w.qkvz, m->qkvz, w.ba, m->ba, s)) return rc;
        q38::GdnFusedArgs a{};
        a.qkv = m->qkvz;
        a.conv_w = w.conv_w;
        a.conv_in = w.conv_state[0];
        a.conv_out = w.conv_state[1];
        a.beta_raw = m->ba;
        a.alpha_raw = m->ba + sh.hv;
        a.dt_bias = w.dt;
        a.ssm_a = w.ssm_a;
        a.s_in = w.ssm_state;
        a.s_out = w.ssm_state;
        a.z = m->qkvz + 2u * sh.hq * D + sh.hv * D;
        a.norm_w = w.ssm_norm;
        a.y = m->ygdn;
        a.Hq = sh.hq;
        a.Hv = sh.hv;
        a.eps = c.rms_eps;
        a.scale = 1.0f / sqrtf(static_cast<float>(D));
        a.parity = m->d_pos;
        if (int rc = launch_pdl_cluster(q38::gdn_fused_kernel, dim3(sh.hv * q38::kGdnSplit), dim3(q38::kGdnFusedThreads),
                                        q38::kGdnSplit,
                                        0, s, "launch gdn_fused", a))
            return rc;
        if (int rc = pack_f32(m, m->ygdn, sh.hv * D, w.ssm_out.d.cols, s)) return rc;
        if (int rc = gemv_x(m, w.ssm_out, yrow, res, s)) return rc;
    } else {
        bool v_done = false;
        if (w.wqk.d.rows != 0 && m->kv_k == m->qg + w.wq.d.rows) {  // one GEMV writes q|gate then k
            // with v in Q6_K tiles: the same launch, its CTAs packing the f32 input
            if (w.wqk.d.layout == Q38_LAYOUT_B200_TILED && w.wv.d.layout == Q38_LAYOUT_B200_TILED &&
                w.wqk.d.cols == w.wv.d.cols) {
                const int rc = launch_frag_pair_xf(w.wqk.d.ggml_type, w.wqk.d.data, w.wqk.d.rows, m->qg,
                                                   w.wv.d.ggml_type, w.wv.d.data, w.wv.d.rows, m->kv_v, m->xf,
                                                   m->xn, w.wqk.d.cols, s);
                if (rc != Q38_ERR_UNSUPPORTED) {
                    if (rc) return rc;
                    v_done = true;
                }
            }
            if (!v_done)
                if (int rc = gemv_x(m, w.wqk, m->qg, nullptr, s)) return rc;
        } else {
            if (int rc = gemv_x(m, w.wq, m->qg, nullptr, s)) return rc;
            if (int rc = gemv_x(m, w.wk, m->kv_k, nullptr, s)) return rc;
        }
        if (!v_done) {
            const int rc = w.wv.d.layout == Q38_LAYOUT_B200_TILED
                               ? launch_frag(w.wv.d.ggml_type, w.wv.d.data, reinterpret_cast<const uint8_t*>(m->xn),
                                             m->kv_v, w.wv.d.cols, w.wv.d.rows, s, nullptr, true)
                               : gemv_x(m, w.wv, m->kv_v, nullptr, s);
            if (rc) return rc;
        }
        if (int rc = launch_pdl(q38::attn_prep_kernel, dim3(sh.aq + sh.ak), dim3(q38::kAttnDim), 0, s,
                                "launch attn_prep", static_cast<const float*>(m->qg),
                                static_cast<const float*>(m->kv_k), static_cast<const float*>(m->kv_v),
                                static_cast<const float*>(w.q_norm), static_cast<const float*>(w.k_norm),
                                static_cast<const int*>(m->d_pos), m->qr, w.kc, w.vc, sh.aq, c.ctx, c.rope_dim,
                                c.rope_theta, c.rms_eps))
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
        a.Hq = sh.aq;
        a.Hkv = sh.ak;
        a.ctx = c.ctx;
        a.splits = std::max(1u, std::min<uint32_t>(q38::kAttnSplits, static_cast<uint32_t>(m->sm_count) / sh.ak));
        const uint32_t G = sh.aq / sh.ak;
        int rc = G == 6 ? launch_attn<6>(m, a, s)
                 : G == 3 ? launch_attn<3>(m, a, s)
                          : fail(Q38_ERR_UNSUPPORTED, "attention group size %u (6 and 3 are built)", G);
        if (rc) return rc;
        // a layout-2 output projection reads x-fragments: the combine packs them
        // (a K padded past the heads, as in 8-way shards, keeps the pack kernel)
        const bool pack_in_combine = w.wo.d.layout == Q38_LAYOUT_B200_TILED && w.wo.d.cols == sh.aq * q38::kAttnDim;
        if (pack_in_combine) a.xf = m->xf;
        if (int rc2 = launch_pdl(q38::attn_combine_kernel, dim3(sh.aq), dim3(q38::kAttnDim), 0, s,
                                 "launch attn_combine", a))
            return rc2;
        if (!pack_in_combine)
            if (int rc2 = pack_f32(m, m->ao, sh.aq * q38::kAttnDim, w.wo.d.cols, s)) return rc2;
        if (int rc2 = gemv_x(m, w.wo, yrow, res, s)) return rc2;
    }
    const bool gate_xpack = w.gate.d.layout == Q38_LAYOUT_GGUF_NATIVE;  // IQ4_XS gate reads the x-pack
    if (int rc = tp ? tp_reduce_norm(m, x, m->xalt, w.post_norm, gate_xpack, 2u * L, s)
                    : norm_pack(m, x, w.post_norm, c.hidden, gate_xpack, s))
        return rc;
    if (int rc = gemv_pair(m, w.gate, m->g, w.up, m->u, s)) return rc;
    {
        const uint32_t fl = sh.f1 - sh.f0, nbp = w.down.d.cols / 256u;
        if (int rc = launch_pdl(q38::silu_mul_xfrag_kernel, dim3((nbp + 7u) / 8u), dim3(256), 0, s,
                                "launch silu_mul_xfrag", static_cast<const float*>(m->g),
                                static_cast<const float*>(m->u), fl, nbp, m->xf))
            return rc;
    }
    if (int rc = gemv_x(m, w.down, yrow, res, s)) return rc;
    return tp ? tp_reduce_norm(m, m->xalt, x, next_norm, next_xpack, 2u * L + 1u, s, next_y) : Q38_OK;
}

int model_step(q38_model* m, cudaStream_t s) {
    const q38_model_config& c = m->cfg;
    const Shard& sh = m->sh;
    const bool tp = sh.size > 1;
    // The vocabulary projection reads the final RMSNorm as f32 (layout-2 Q6_K
    // tiles pack it in every CTA) or as the x-pack (layout 0).
    const bool head_tiled = m->lm_head.d.layout == Q38_LAYOUT_B200_TILED;
    if (tp)
        if (int rc = tp_next_step(m, s)) return rc;
    if (int rc = launch_pdl(q38::embed_q6k_kernel, dim3(1), dim3(256), 0, s, "launch embed",
                            static_cast<const uint8_t*>(dptr<uint8_t>(m->embd.d.data)),
                            static_cast<const int*>(m->d_token), c.vocab, c.hidden, m->x))
        return rc;
    if (!tp) {
        for (uint32_t L = 0; L < c.n_layers; ++L)
            if (int rc = layer_forward(m, L, m->x, s)) return rc;
        if (int rc = norm_pack(m, m->x, m->out_norm, c.hidden, !head_tiled, s, head_tiled ? m->xn : nullptr)) return rc;
    } else {
        // Each layer's last exchange normalises for the next layer (or the output norm).
        if (int rc = norm_pack(m, m->x, m->layers[0].attn_norm, c.hidden, norm_xpack(m->layers[0]), s,
                               norm_f32(m, m->layers[0])))
            return rc;
        for (uint32_t L = 0; L < c.n_layers; ++L) {
            const bool last = L + 1u == c.n_layers;
            const float* nn = last ? m->out_norm : m->layers[L + 1u].attn_norm;
            const bool nx = last ? !head_tiled : norm_xpack(m->layers[L + 1u]);
            float* ny = last ? (head_tiled ? m->xn : nullptr) : norm_f32(m, m->layers[L + 1u]);
            if (int rc = layer_forward(m, L, m->x, s, true, nn, nx, ny)) return rc;
        }
    }
    if (head_tiled) {
        if (int rc = launch_frag(m->lm_head.d.ggml_type, m->lm_head.d.data, reinterpret_cast<const uint8_t*>(m->xn),
                                 m->logits, m->lm_head.d.cols, m->lm_head.d.rows, s, nullptr, true))
            return rc;
    } else if (int rc = gemv_x(m, m->lm_head, m->logits, nullptr, s)) {
        return rc;
    }
    if (sh.size == 1)
        return launch_pdl(q38::argmax_kernel, dim3(q38::kArgmaxCtas), dim3(256), 0, s, "launch argmax",
                          static_cast<const float*>(m->logits), c.vocab, m->am_v, m->am_i, m->counters + 8, m->d_token,
                          m->d_pos, static_cast<unsigned long long*>(nullptr), 0u);
    if (int rc = launch_pdl(q38::argmax_kernel, dim3(q38::kArgmaxCtas), dim3(256), 0, s, "launch argmax",
                            static_cast<const float*>(m->logits), sh.v1 - sh.v0, m->am_v, m->am_i, m->counters + 8,
                            m->d_token, m->d_pos, m->key, sh.v0))
        return rc;
    if (!m->comm) return fail(Q38_ERR_INVALID, "tensor-parallel model has no communicator (q38_model_set_comm)");
    if (int r = g_nccl.allReduce(m->key, m->key, 1, kNcclUint64, kNcclMax, m->comm->comm, s))
        return nccl_fail(r, "ncclAllReduce(argmax)");
    return launch_pdl(q38::token_from_key_kernel, dim3(1), dim3(1), 0, s, "launch token_from_key",
                      static_cast<const unsigned long long*>(m->key), m->d_token, m->d_pos);
}

int check_model_config(const q38_model_config* c) {
    if (!c || c->n_layers == 0 || c->attn_every == 0 || c->hidden == 0 || c->hidden % 1024u || c->ffn % 1024u ||
        c->ffn == 0 || c->vocab == 0 || c->gdn_qk_heads == 0 || c->gdn_v_heads % c->gdn_qk_heads || c->ctx == 0 ||
        c->attn_kv_heads == 0 || c->attn_q_heads % c->attn_kv_heads || c->rope_dim > q38::kAttnDim ||
        c->rope_dim % 2u)
        return fail(Q38_ERR_INVALID, "q38_model_config: inconsistent dimensions");
    if ((c->gdn_v_heads * 128u) % 1024u || (c->attn_q_heads * q38::kAttnDim) % 1024u)
        return fail(Q38_ERR_UNSUPPORTED, "projection inputs must be multiples of 1024");
    if (c->hidden > 256u * q38::kNormMaxBlocks) return fail(Q38_ERR_UNSUPPORTED, "hidden too large");
    if (c->ffn_gate_type != 0 && c->ffn_gate_type != Q38_TYPE_Q4_K && c->ffn_gate_type != Q38_TYPE_IQ4_XS)
        return fail(Q38_ERR_UNSUPPORTED, "ffn_gate_type %u (Q4_K or IQ4_XS)", c->ffn_gate_type);
    return Q38_OK;
}

// One rank's model: seeded weights (pack null) or the pack's.
int model_create(const q38_model_config* cfg, const q38_pack* pack, q38_model** out) {
    if (!out) return fail(Q38_ERR_INVALID, "q38_model_create: out is null");
    *out = nullptr;
    if (int rc = check_model_config(cfg)) return rc;
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    auto m = std::make_unique<q38_model>();
    m->cfg = *cfg;
    if (m->cfg.tp_size == 0) m->cfg.tp_size = 1;
    if (int rc = make_shard(m->cfg, &m->sh)) return rc;
    m->device = dev;
    m->sm_count = st->sm_count;
    m->pack = pack;
    cudaStream_t s = nullptr;
    // sizing pass (the placement plan of this rank's shard), then the real one
    m->dry = true;
    if (int rc = build_model(m.get(), s)) return rc;
    m->dry = false;
    m->arena_bytes = m->arena_used + 4096u;
    m->arena_used = 0;
    m->tmp_bytes = m->tmp_need;
    Q38_CUDA(cudaMalloc(&m->arena, m->arena_bytes), "cudaMalloc(model arena)");
    m->stage_bytes = pack ? (m->stage_need + 255u) & ~size_t(255) : 0;
    if (cudaMalloc(&m->tmp, std::max<size_t>(m->tmp_bytes, 256)) != cudaSuccess ||
        cudaMalloc(&m->maps, kMapWords * 4u) != cudaSuccess ||
        (pack && cudaMalloc(&m->stage, m->stage_bytes + 256u) != cudaSuccess)) {
        cudaFree(m->arena);
        cudaFree(m->tmp);
        cudaFree(m->maps);
        return fail(Q38_ERR_NOMEM, "cudaMalloc(model staging)");
    }
    int rc = Q38_OK;
    if (pack) {
        m->load_err = reinterpret_cast<unsigned*>(m->stage + m->stage_bytes);
        if (cudaMemsetAsync(m->load_err, 0, 4, s) != cudaSuccess) rc = fail(Q38_ERR_CUDA, "cudaMemsetAsync(load flag)");
    }
    rc = rc ? rc : build_model(m.get(), s);
    if (rc == Q38_OK) {
        if (cudaMemsetAsync(m->counters, 0, 64, s) != cudaSuccess || cudaMemsetAsync(m->d_token, 0, 8, s) != cudaSuccess ||
            cudaMemsetAsync(m->d_pos, 0, 8, s) != cudaSuccess ||
            (m->tp_step && cudaMemsetAsync(m->tp_step, 0, 64, s) != cudaSuccess))
            rc = fail(Q38_ERR_CUDA, "cudaMemsetAsync(model scratch)");
    }
    if (rc == Q38_OK) {
        const cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) rc = cuda_fail(e, pack ? "model load" : "synthetic model generation");
    }
    if (rc == Q38_OK && pack) {
        unsigned err = 0;
        const cudaError_t e = cudaMemcpy(&err, m->load_err, 4, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = cuda_fail(e, "read load flag");
        else if (err) rc = fail(Q38_ERR_INVALID, "q38pack: shard gather read outside the uploaded rows (flag %u)", err);
    }
    cudaFree(m->tmp);
    cudaFree(m->maps);
    cudaFree(m->stage);
    m->tmp = nullptr;
    m->maps = nullptr;
    m->stage = nullptr;
    m->load_err = nullptr;
    m->pack = nullptr;
    if (rc != Q38_OK) {
        cudaFree(m->arena);
        return rc;
    }
    const q38_model_config& c = m->cfg;
    uint64_t bytes = m->embd.algo / c.vocab + m->lm_head.algo;
    for (const LayerW& w : m->layers) {
        for (const GemvW* g : {&w.qkvz, &w.ba, &w.ssm_out, &w.wq, &w.wk, &w.wv, &w.wo, &w.gate, &w.up, &w.down})
            bytes += g->algo;
    }
    m->step_bytes = bytes;
    *out = m.release();
    return Q38_OK;
}

}  // namespace

extern "C" {

int q38_model_create(const q38_model_config* cfg, q38_model** out) { return model_create(cfg, nullptr, out); }

int q38_model_create_from_pack(const q38_model_config* cfg, const q38_pack* pack, q38_model** out) {
    if (!pack) return fail(Q38_ERR_INVALID, "q38_model_create_from_pack: pack is null");
    return model_create(cfg, pack, out);
}

int q38_model_shard_info(const q38_model_config* cfg, q38_shard_info* out) {
    if (!cfg || !out) return fail(Q38_ERR_INVALID, "q38_model_shard_info: null argument");
    if (int rc = check_model_config(cfg)) return rc;
    q38_model_config c = *cfg;
    if (c.tp_size == 0) c.tp_size = 1;
    Shard sh;
    if (int rc = make_shard(c, &sh)) return rc;
    if (sh.vheads.size() > 64) return fail(Q38_ERR_UNSUPPORTED, "too many value heads");
    *out = q38_shard_info{};
    out->qk_head0 = sh.qk0;
    out->qk_heads = sh.hq;
    out->v_heads = sh.hv;
    for (size_t i = 0; i < sh.vheads.size(); ++i) out->v_head[i] = sh.vheads[i];
    out->ffn_row0 = sh.f0;
    out->ffn_row1 = sh.f1;
    out->q_head0 = sh.aq0;
    out->q_heads = sh.aq;
    out->kv_head0 = sh.ak0;
    out->kv_heads = sh.ak;
    out->vocab0 = sh.v0;
    out->vocab1 = sh.v1;
    return Q38_OK;
}

int q38_quantize_q8k(q38_devptr x, uint32_t cols, q38_devptr out, q38_stream stream) {
    if (!x || !out || cols == 0 || cols % 256u) return fail(Q38_ERR_INVALID, "q38_quantize_q8k: bad arguments");
    if ((x & 15u) || (out & 3u)) return fail(Q38_ERR_INVALID, "q38_quantize_q8k: x 16-byte, out 4-byte aligned");
    const uint32_t nb = cols / 256u;
    return launch_pdl(q38::quantize_q8k_kernel, dim3((nb + 7u) / 8u), dim3(256), 0, as_stream(stream),
                      "launch quantize_q8k", dptr<const float>(x), nb, dptr<uint8_t>(out));
}

int q38_rmsnorm_q8k(q38_devptr x, q38_devptr w, uint32_t n, float eps, q38_devptr y, q38_devptr out,
                    q38_stream stream) {
    if (!x || !w || !out || n == 0 || n % 256u || n > 256u * q38::kNormMaxBlocks)
        return fail(Q38_ERR_INVALID, "q38_rmsnorm_q8k: bad arguments (n %% 256 == 0, n <= 32768)");
    if ((x & 15u) || (w & 15u) || (y & 15u) || (out & 3u))
        return fail(Q38_ERR_INVALID, "q38_rmsnorm_q8k: x, w, y 16-byte, out 4-byte aligned");
    return launch_pdl(q38::rmsnorm_q8k_kernel, dim3(n / 256u), dim3(256), 0, as_stream(stream), "launch rmsnorm_q8k",
                      dptr<const float>(x), dptr<const float>(w), n, eps, y ? dptr<float>(y) : nullptr,
                      dptr<uint8_t>(out));
}

size_t q38_tp_exchange_bytes(uint32_t n) { return q38::tp_exchange_bytes(n); }

int q38_tp_exchange(const q38_tp_exchange_desc* d, q38_stream stream) {
    if (!d || !d->x_in || !d->x_out || !d->part || !d->step || d->x_in == d->x_out)
        return fail(Q38_ERR_INVALID, "q38_tp_exchange: null or aliased buffers");
    if (d->n == 0 || d->n % 256u || d->n > 256u * q38::kNormMaxBlocks || d->size == 0 || d->size > q38::kMaxTp ||
        d->rank >= d->size || d->instance >= 511u || (d->norm_w && !d->xfrag))
        return fail(Q38_ERR_INVALID,
                    "q38_tp_exchange: bad shape (n %% 256, n <= 32768, rank < size <= 8, instance <= 510)");
    // The kernel reads part as float2, norm_w as float4 and writes the
    // x-fragments with vector stores: refuse pointers a vector access would
    // fault on instead of poisoning the context.
    if ((d->x_in & 3u) || (d->x_out & 3u) || (d->part & 7u) || (d->step & 3u) || (d->norm_w & 15u) ||
        (d->xfrag & 15u))
        return fail(Q38_ERR_INVALID,
                    "q38_tp_exchange: misaligned buffer (x_in, x_out, step 4-byte; part 8-byte; norm_w, xfrag 16-byte)");
    q38::TpReduceArgs a{};
    for (uint32_t r = 0; r < d->size; ++r) {
        if (!d->region[r] || (d->region[r] & 15u)) return fail(Q38_ERR_INVALID, "q38_tp_exchange: region %u", r);
        a.region[r] = dptr<uint4>(d->region[r]);
    }
    a.x_in = dptr<const float>(d->x_in);
    a.x_out = dptr<float>(d->x_out);
    a.part = dptr<const float>(d->part);
    a.step = dptr<const uint32_t>(d->step);
    a.norm_w = d->norm_w ? dptr<const float>(d->norm_w) : nullptr;
    a.frag = d->norm_w ? dptr<uint8_t>(d->xfrag) : nullptr;
    a.n = d->n;
    a.rank = d->rank;
    a.size = d->size;
    a.instance = d->instance;
    a.eps = d->eps;
    return launch_pdl(q38::tp_reduce_norm_kernel<4>, dim3(d->n / 256u), dim3(q38::kTpWarps * 32u), 0,
                      as_stream(stream), "launch tp_reduce_norm", a);
}

int q38_model_set_comm(q38_model* m, q38_comm* comm) {
    if (!m || !comm) return fail(Q38_ERR_INVALID, "q38_model_set_comm: null argument");
    if (static_cast<uint32_t>(comm->size) != m->sh.size || static_cast<uint32_t>(comm->rank) != m->sh.rank)
        return fail(Q38_ERR_INVALID, "communicator rank %d/%d does not match the model shard %u/%u", comm->rank,
                    comm->size, m->sh.rank, m->sh.size);
    if (m->comm) return m->comm == comm ? Q38_OK : fail(Q38_ERR_INVALID, "q38_model_set_comm: communicator already set");
    if (m->sh.size > 1) {
        if (m->sh.size > q38::kMaxTp || 2u * m->cfg.n_layers >= 512u)
            return fail(Q38_ERR_UNSUPPORTED, "tensor-parallel exchange: tp_size <= %u and fewer than 256 layers",
                        q38::kMaxTp);
        const size_t bytes = q38::tp_exchange_bytes(m->cfg.hidden);
        Q38_CUDA(cudaMalloc(&m->xchg, bytes), "cudaMalloc(exchange region)");
        int rc = cudaMemset(m->xchg, 0, bytes) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess
                     ? comm_map_peers(comm, m->xchg, m->xchg_peer)
                     : fail(Q38_ERR_CUDA, "clear exchange region");
        if (rc != Q38_OK) {
            comm_unmap_peers(comm->rank, comm->size, m->xchg_peer);
            cudaFree(m->xchg);
            m->xchg = nullptr;
            return rc;
        }
    }
    m->comm = comm;
    return Q38_OK;
}

int q38_model_destroy(q38_model* m) {
    if (!m) return Q38_OK;
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->xchg) {
        comm_unmap_peers(static_cast<int>(m->sh.rank), static_cast<int>(m->sh.size), m->xchg_peer);
        cudaFree(m->xchg);
    }
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
        state += 4ull * m->sh.hv * 128u * 128u;
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
        for (uint32_t h = 0; h < m->sh.ak; ++h) {
            const uint64_t off = static_cast<uint64_t>(h) * c.ctx * q38::kAttnDim;
            const uint64_t gh = m->sh.ak0 + h;  // global KV head: the same values at any tp_size
            q38::synth_f16_kernel<<<static_cast<uint32_t>((n + 255u) / 256u), 256>>>(
                reinterpret_cast<uint16_t*>(w.kc + off), n, kv_seed * 131u + L * 8u + gh, 1.0f);
            q38::synth_f16_kernel<<<static_cast<uint32_t>((n + 255u) / 256u), 256>>>(
                reinterpret_cast<uint16_t*>(w.vc + off), n, kv_seed * 137u + L * 8u + gh + 4u, 1.0f);
        }
    }
    Q38_CUDA(cudaGetLastError(), "launch KV fill");
    Q38_CUDA(cudaMemcpy(m->d_token, &token, 4, cudaMemcpyHostToDevice), "set token");
    Q38_CUDA(cudaMemcpy(m->d_pos, &pos, 4, cudaMemcpyHostToDevice), "set position");
    Q38_CUDA(cudaDeviceSynchronize(), "q38_model_set_position");
    return Q38_OK;
}

int q38_model_reset(q38_model* m, int32_t token) {
    if (!m || token < 0 || static_cast<uint32_t>(token) >= m->cfg.vocab)
        return fail(Q38_ERR_INVALID, "q38_model_reset: token outside the vocabulary");
    const uint32_t D = 128u, Cl = 2u * m->sh.hq * D + m->sh.hv * D;
    for (const LayerW& w : m->layers) {
        if (w.attn) continue;
        Q38_CUDA(cudaMemset(w.conv_state[0], 0, 12ull * Cl), "reset conv state");
        Q38_CUDA(cudaMemset(w.conv_state[1], 0, 12ull * Cl), "reset conv state");
        Q38_CUDA(cudaMemset(w.ssm_state, 0, 4ull * m->sh.hv * D * D), "reset GDN state");
    }
    const int32_t zero = 0;
    Q38_CUDA(cudaMemcpy(m->d_token, &token, 4, cudaMemcpyHostToDevice), "set token");
    Q38_CUDA(cudaMemcpy(m->d_pos, &zero, 4, cudaMemcpyHostToDevice), "set position");
    Q38_CUDA(cudaDeviceSynchronize(), "q38_model_reset");
    return Q38_OK;
}

int q38_model_set_token(q38_model* m, int32_t token) {
    if (!m || token < 0 || static_cast<uint32_t>(token) >= m->cfg.vocab)
        return fail(Q38_ERR_INVALID, "q38_model_set_token: token outside the vocabulary");
    Q38_CUDA(cudaMemcpy(m->d_token, &token, 4, cudaMemcpyHostToDevice), "set token");
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
    if (m->sh.size > 1)
        if (int rc = tp_next_step(m, as_stream(stream))) return rc;
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
    if (n == "logits") return vec(m->logits, m->sh.v1 - m->sh.v0);
    unsigned L = 0;
    char field[64] = {0};
    if (sscanf(name, "blk.%u.%63s", &L, field) != 2 || L >= c.n_layers)
        return fail(Q38_ERR_INVALID, "unknown tensor '%s'", name);
    const LayerW& w = m->layers[L];
    const std::string f(field);
    const uint32_t D = 128u, C = 2u * m->sh.hq * D + m->sh.hv * D;
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
        if (f == "ssm_dt") return vec(w.dt, m->sh.hv);
        if (f == "ssm_a") return vec(w.ssm_a, m->sh.hv);
        if (f == "ssm_norm") return vec(w.ssm_norm, D);
        if (f == "conv_state0") return vec(w.conv_state[0], 3u * C);
        if (f == "conv_state1") return vec(w.conv_state[1], 3u * C);
        if (f == "ssm_state") return vec(w.ssm_state, m->sh.hv * D * D);
    } else {
        if (f == "attn_q") { *out = w.wq.d; return Q38_OK; }
        if (f == "attn_k") { *out = w.wk.d; return Q38_OK; }
        if (f == "attn_v") { *out = w.wv.d; return Q38_OK; }
        if (f == "attn_output") { *out = w.wo.d; return Q38_OK; }
        if (f == "attn_q_norm") return vec(w.q_norm, q38::kAttnDim);
        if (f == "attn_k_norm") return vec(w.k_norm, q38::kAttnDim);
        if (f == "k_cache") return vec(w.kc, m->sh.ak * c.ctx * q38::kAttnDim / 2u);
        if (f == "v_cache") return vec(w.vc, m->sh.ak * c.ctx * q38::kAttnDim / 2u);
    }
    return fail(Q38_ERR_INVALID, "unknown tensor '%s'", name);
}

}  // extern "C"
