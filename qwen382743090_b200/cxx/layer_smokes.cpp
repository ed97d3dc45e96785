// layer_smokes.cpp -- the decoder-layer methods of q38::NvidiaDriver
// (include/q38/driver.hpp): the layer-0 chains, the recurrent-prep and GDN
// smokes, the Q5_K x Q8_K GEMV smoke and the dequantisation smokes, over the
// C ABI of include/q38rt.h.
//
// Each keeps the reference's contract (src/driver.cpp:7025-12461): the same
// shapes (hidden 5120, qkv 10240 = q 2048 | k 2048 | v 6144, z 6144, 48
// beta/alpha rows, 16 q/k heads and 48 value heads of 128, FFN 17408), the
// same deterministic inputs and recurrent states, the same tolerances and
// Stats fields, and per-stage timings over the same iteration counts.  The
// check runs on the device: the q38_check_* entries restate the reference's
// CPU check loops in FP64 (fed the GPU's own intermediates, as the reference
// feeds its CPU chain) and q38_check_rows gives the FP64 reference rows of the
// quantised projections.
#include <array>
#include <cstring>
#include <memory>
#include <sstream>

#include "../../include/q38/driver.hpp"
#include "facade_util.hpp"

namespace q38 {
namespace {

using facade::bench_ms;
using facade::ck;
using facade::ctx_of;
using facade::DevBuf;
using facade::download;
using facade::download64;
using facade::max_abs_diff;
using facade::max_rel_diff;
using facade::upload;

constexpr std::uint32_t kCols = 5120, kQkvRows = 10240, kZRows = 6144, kSmallRows = 48, kHeadDim = 128;
constexpr std::uint32_t kQkHeads = 16, kValueHeads = 48, kFfnDim = 17408;
constexpr std::uint32_t kKeyDim = kQkHeads * kHeadDim, kValueDim = kValueHeads * kHeadDim;
constexpr std::size_t kGdnState = static_cast<std::size_t>(kValueHeads) * kHeadDim * kHeadDim;

std::size_t soa_bytes(std::size_t rows, std::size_t cols, std::size_t qh, std::size_t qs, const char* what) {
    const std::size_t blocks = rows * (cols / 256u);
    if (qh < blocks * 20 || qs < qh + blocks * 32) throw std::invalid_argument(std::string("invalid ") + what + " Q5_K plane offsets");
    return qs + blocks * 128;
}

// One SoA Q5_K matrix (META | QH | QS at the given offsets) on the device.
struct SoAMat {
    DevBuf buf;
    q38_weight_desc d{};
    SoAMat(q38_ctx* ctx, const std::byte* m, std::size_t qh, std::size_t qs, std::uint32_t rows, std::uint32_t cols,
           const char* what)
        : buf(ctx, soa_bytes(rows, cols, qh, qs, what)) {
        if (!m) throw std::invalid_argument(std::string(what) + " matrix is null");
        upload(buf.get(), m, soa_bytes(rows, cols, qh, qs, what), what);
        d = q38_weight_desc{Q38_TYPE_Q5_K, Q38_LAYOUT_SM86_Q5K_SOA, rows, cols, buf.get(), buf.get() + qh, buf.get() + qs};
    }
    int gemv(q38_devptr x, q38_devptr y) const {
        return q38_q5k_sm86_soa_gemv_vec(d.data, d.aux0, d.aux1, x, y, d.cols, d.rows, nullptr);
    }
};

// One GGUF-native matrix (Q4_K 144 B or IQ4_XS 136 B per 256 weights).
struct NativeMat {
    DevBuf buf;
    q38_weight_desc d{};
    NativeMat(q38_ctx* ctx, const std::byte* m, std::uint32_t type, std::size_t block_bytes, std::uint32_t rows,
              std::uint32_t cols, const char* what)
        : buf(ctx, static_cast<std::size_t>(rows) * (cols / 256u) * block_bytes + 16u) {
        if (!m) throw std::invalid_argument(std::string(what) + " matrix is null");
        upload(buf.get(), m, static_cast<std::size_t>(rows) * (cols / 256u) * block_bytes, what);
        d = q38_weight_desc{type, Q38_LAYOUT_GGUF_NATIVE, rows, cols, buf.get(), 0, 0};
    }
    int gemv(q38_devptr x, q38_devptr y) const {
        return d.ggml_type == Q38_TYPE_Q4_K ? q38_q4k_gemv_f32(d.data, x, y, d.cols, d.rows, nullptr)
                                            : q38_iq4xs_gemv_f32(d.data, x, y, d.cols, d.rows, nullptr);
    }
};

DevBuf f32_buf(q38_ctx* ctx, const float* src, std::size_t n, const char* what) {
    if (!src) throw std::invalid_argument(std::string(what) + " is null");
    DevBuf b(ctx, n * sizeof(float));
    upload(b.get(), src, n * sizeof(float), what);
    return b;
}

// FP64 reference rows of the first nrows rows of a matrix against an f32 x on
// the device; returns them on the host.
std::vector<double> ref_rows(q38_ctx* ctx, const q38_weight_desc& d, std::uint32_t nrows, q38_devptr x) {
    DevBuf y(ctx, nrows * sizeof(double));
    ck(q38_check_rows(&d, nrows, x, y.get(), 0, nullptr), "q38_check_rows");
    return download64(y.get(), nrows, "reference rows");
}

// The decode-time input and recurrent states of the layer-0 chains
// (src/driver.cpp:7316-7342).
struct Layer0Inputs {
    std::vector<float> hidden, conv_state, gdn_state;
    Layer0Inputs() : hidden(facade::smoke_x(kCols)), conv_state(3u * kQkvRows), gdn_state(kGdnState) {
        for (std::uint32_t s = 0; s < 3u; ++s)
            for (std::uint32_t i = 0; i < kQkvRows; ++i) {
                const float fi = static_cast<float>(i), fs = static_cast<float>(s + 1);
                conv_state[static_cast<std::size_t>(s) * kQkvRows + i] =
                    0.08f * std::sin(fi * (0.0029f + 0.0006f * fs)) + 0.03f * std::cos(fi * (0.0017f + 0.0004f * fs));
            }
        for (std::size_t i = 0; i < gdn_state.size(); ++i) {
            const float fi = static_cast<float>(i);
            gdn_state[i] = 0.011f * std::sin(fi * 0.0011f) + 0.005f * std::cos(fi * 0.00073f);
        }
    }
};

// The recurrent layer: weights, activations and the launch chain.  Stages:
// projection (RMSNorm, qkv / z / beta / alpha), prep (conv4 + SiLU + roll,
// q/k norm, beta/gate), GDN, tail (gated norm, ssm_out, residual), FFN
// (post norm, gate / up, SiLU * up, down, residual).
struct Layer0 {
    q38_ctx* ctx;
    float eps;
    DevBuf norm, conv_w, dt, a, ssm_norm, post_norm;
    SoAMat qkv, z;
    NativeMat beta_m, alpha_m;
    std::unique_ptr<SoAMat> ssm_out, up, down;
    std::unique_ptr<NativeMat> gate;
    DevBuf hidden, normed, qkv_y, z_y, beta_raw, alpha_raw, conv, cs_in, cs_out, q, k, beta, gate_v, st_in, st_out,
        gdn_out, gated, ssm_y, residual, ffn_normed, ffn_gate_y, ffn_up_y, ffn_mul, ffn_down_y, layer_out;

    Layer0(q38_ctx* c, float e, const float* norm_weight, const std::byte* qkv_m, std::size_t qkv_qh,
           std::size_t qkv_qs, const std::byte* z_m, std::size_t z_qh, std::size_t z_qs, const std::byte* beta_mat,
           const std::byte* alpha_mat, const float* conv_weight, const float* dt_bias, const float* ssm_a)
        : ctx(c), eps(e), norm(f32_buf(c, norm_weight, kCols, "norm weight")),
          conv_w(f32_buf(c, conv_weight, 4u * kQkvRows, "conv weight")),
          dt(f32_buf(c, dt_bias, kSmallRows, "dt bias")), a(f32_buf(c, ssm_a, kSmallRows, "ssm_a")),
          qkv(c, qkv_m, qkv_qh, qkv_qs, kQkvRows, kCols, "qkv"), z(c, z_m, z_qh, z_qs, kZRows, kCols, "z"),
          beta_m(c, beta_mat, Q38_TYPE_Q4_K, 144, kSmallRows, kCols, "beta"),
          alpha_m(c, alpha_mat, Q38_TYPE_Q4_K, 144, kSmallRows, kCols, "alpha"), hidden(c, kCols * 4u),
          normed(c, kCols * 4u), qkv_y(c, kQkvRows * 4u), z_y(c, kZRows * 4u), beta_raw(c, kSmallRows * 4u),
          alpha_raw(c, kSmallRows * 4u), conv(c, kQkvRows * 4u), cs_in(c, 3u * kQkvRows * 4u),
          cs_out(c, 3u * kQkvRows * 4u), q(c, kKeyDim * 4u), k(c, kKeyDim * 4u), beta(c, kSmallRows * 4u),
          gate_v(c, kSmallRows * 4u), st_in(c, kGdnState * 4u), st_out(c, kGdnState * 4u), gdn_out(c, kValueDim * 4u),
          gated(c, kValueDim * 4u), ssm_y(c, kCols * 4u), residual(c, kCols * 4u), ffn_normed(c, kCols * 4u),
          ffn_gate_y(c, kFfnDim * 4u), ffn_up_y(c, kFfnDim * 4u), ffn_mul(c, kFfnDim * 4u), ffn_down_y(c, kCols * 4u),
          layer_out(c, kCols * 4u) {
        const Layer0Inputs in;
        upload(hidden.get(), in.hidden.data(), kCols * 4u, "hidden");
        upload(cs_in.get(), in.conv_state.data(), in.conv_state.size() * 4u, "conv state");
        upload(st_in.get(), in.gdn_state.data(), in.gdn_state.size() * 4u, "GDN state");
    }
    void add_tail(const float* ssm_norm_weight, const std::byte* m, std::size_t qh, std::size_t qs) {
        ssm_norm = f32_buf(ctx, ssm_norm_weight, kHeadDim, "ssm norm weight");
        ssm_out = std::make_unique<SoAMat>(ctx, m, qh, qs, kCols, kValueDim, "ssm_out");
    }
    void add_ffn(const float* post_norm_weight, const std::byte* gate_m, const std::byte* up_m, std::size_t up_qh,
                 std::size_t up_qs, const std::byte* down_m, std::size_t down_qh, std::size_t down_qs) {
        post_norm = f32_buf(ctx, post_norm_weight, kCols, "post norm weight");
        gate = std::make_unique<NativeMat>(ctx, gate_m, Q38_TYPE_IQ4_XS, 136, kFfnDim, kCols, "ffn_gate");
        up = std::make_unique<SoAMat>(ctx, up_m, up_qh, up_qs, kFfnDim, kCols, "ffn_up");
        down = std::make_unique<SoAMat>(ctx, down_m, down_qh, down_qs, kCols, kFfnDim, "ffn_down");
    }

    void projection() {
        ck(q38_rmsnorm(hidden.get(), norm.get(), normed.get(), kCols, 1, eps, nullptr), "layer RMSNorm");
        ck(qkv.gemv(normed.get(), qkv_y.get()), "qkv projection");
        ck(z.gemv(normed.get(), z_y.get()), "z projection");
        ck(beta_m.gemv(normed.get(), beta_raw.get()), "beta projection");
        ck(alpha_m.gemv(normed.get(), alpha_raw.get()), "alpha projection");
    }
    void prep() {
        ck(q38_conv4_silu_roll(qkv_y.get(), conv_w.get(), cs_in.get(), conv.get(), cs_out.get(), kQkvRows, nullptr),
           "conv4 + SiLU");
        ck(q38_qk_l2norm(conv.get(), q.get(), k.get(), kQkHeads, eps, nullptr), "q/k norm");
        ck(q38_beta_gate(beta_raw.get(), alpha_raw.get(), dt.get(), a.get(), beta.get(), gate_v.get(), kSmallRows,
                         nullptr),
           "beta/gate");
    }
    void gdn() {
        ck(q38_gdn_step(q.get(), k.get(), conv.get() + 4u * 2u * kKeyDim, gate_v.get(), beta.get(), st_in.get(),
                        gdn_out.get(), st_out.get(), kQkHeads, kValueHeads, 1.0f / std::sqrt(128.0f), nullptr),
           "GDN step");
    }
    void tail() {
        ck(q38_gated_rmsnorm_silu(gdn_out.get(), ssm_norm.get(), z_y.get(), gated.get(), kValueHeads, eps, nullptr),
           "gated norm");
        ck(ssm_out->gemv(gated.get(), ssm_y.get()), "ssm_out projection");
        ck(q38_add_residual(ssm_y.get(), hidden.get(), residual.get(), kCols, nullptr), "attention residual");
    }
    void post_norm_stage() {
        ck(q38_rmsnorm(residual.get(), post_norm.get(), ffn_normed.get(), kCols, 1, eps, nullptr), "post norm");
    }
    void ffn_gate() { ck(gate->gemv(ffn_normed.get(), ffn_gate_y.get()), "ffn_gate projection"); }
    void ffn_up() { ck(up->gemv(ffn_normed.get(), ffn_up_y.get()), "ffn_up projection"); }
    void ffn_pointwise() {
        ck(q38_ffn_silu_mul(ffn_gate_y.get(), ffn_up_y.get(), ffn_mul.get(), kFfnDim, nullptr), "SiLU(gate) * up");
    }
    void ffn_down() {
        ck(down->gemv(ffn_mul.get(), ffn_down_y.get()), "ffn_down projection");
        ck(q38_add_residual(ffn_down_y.get(), residual.get(), layer_out.get(), kCols, nullptr), "ffn residual");
    }
    void front() {
        projection();
        prep();
        gdn();
    }
    void attention() {
        front();
        tail();
    }
    void ffn() {
        post_norm_stage();
        ffn_gate();
        ffn_up();
        ffn_pointwise();
        ffn_down();
    }
};

// ---- checks of the front (src/driver.cpp:9620-9690) ----
void check_front(Layer0& L, Layer0RecurrentFrontStats& s, DevBuf& conv_ref, DevBuf& q_ref, DevBuf& k_ref,
                 DevBuf& beta_ref, DevBuf& gate_ref, DevBuf& gdn_ref) {
    q38_ctx* c = L.ctx;
    DevBuf cs_ref(c, 3u * kQkvRows * 4u), st_ref(c, kGdnState * 4u);
    ck(q38_check_conv4(L.qkv_y.get(), L.conv_w.get(), L.cs_in.get(), conv_ref.get(), cs_ref.get(), kQkvRows, nullptr),
       "check conv");
    ck(q38_check_l2norm(conv_ref.get(), kQkHeads, kHeadDim, L.eps, q_ref.get(), nullptr), "check q");
    ck(q38_check_l2norm(conv_ref.get() + 4u * kKeyDim, kQkHeads, kHeadDim, L.eps, k_ref.get(), nullptr), "check k");
    ck(q38_check_beta_gate(L.beta_raw.get(), L.alpha_raw.get(), L.dt.get(), L.a.get(), kSmallRows, beta_ref.get(),
                           gate_ref.get(), nullptr),
       "check beta/gate");
    ck(q38_check_gdn(q_ref.get(), k_ref.get(), conv_ref.get() + 4u * 2u * kKeyDim, gate_ref.get(), beta_ref.get(),
                     L.st_in.get(), gdn_ref.get(), st_ref.get(), kQkHeads, kValueHeads, kHeadDim, nullptr),
       "check GDN");
    const auto g = [](const DevBuf& b, std::size_t n, const char* w) { return download(b.get(), n, w); };
    s.conv_max_abs = max_abs_diff(g(L.conv, kQkvRows, "conv"), g(conv_ref, kQkvRows, "conv ref"));
    s.q_max_abs = max_abs_diff(g(L.q, kKeyDim, "q"), g(q_ref, kKeyDim, "q ref"));
    s.k_max_abs = max_abs_diff(g(L.k, kKeyDim, "k"), g(k_ref, kKeyDim, "k ref"));
    s.beta_max_abs = max_abs_diff(g(L.beta, kSmallRows, "beta"), g(beta_ref, kSmallRows, "beta ref"));
    s.gate_max_abs = max_abs_diff(g(L.gate_v, kSmallRows, "gate"), g(gate_ref, kSmallRows, "gate ref"));
    s.conv_state_max_abs = max_abs_diff(g(L.cs_out, 3u * kQkvRows, "conv state"), g(cs_ref, 3u * kQkvRows, "ref"));
    const auto o = g(L.gdn_out, kValueDim, "GDN out"), o_ref = g(gdn_ref, kValueDim, "GDN out ref");
    const auto st = g(L.st_out, kGdnState, "GDN state"), st_r = g(st_ref, kGdnState, "GDN state ref");
    s.gdn_output_max_abs = max_abs_diff(o, o_ref);
    s.gdn_output_max_rel = max_rel_diff(o, o_ref, 1.0e-6);
    s.gdn_state_max_abs = max_abs_diff(st, st_r);
    s.gdn_state_max_rel = max_rel_diff(st, st_r, 1.0e-6);
    if (s.conv_max_abs > 1.0e-3 || s.q_max_abs > 1.0e-3 || s.k_max_abs > 1.0e-3 || s.beta_max_abs > 1.0e-4 ||
        s.gate_max_abs > 1.0e-3 || s.conv_state_max_abs > 1.0e-6 ||
        (s.gdn_output_max_abs > 2.0e-3 && s.gdn_output_max_rel > 2.0e-3) ||
        (s.gdn_state_max_abs > 1.0e-3 && s.gdn_state_max_rel > 1.0e-3)) {
        std::ostringstream oss;
        oss << "layer0 recurrent front mismatch: conv=" << s.conv_max_abs << " q=" << s.q_max_abs
            << " k=" << s.k_max_abs << " beta=" << s.beta_max_abs << " gate=" << s.gate_max_abs
            << " conv_state=" << s.conv_state_max_abs << " gdn_out_abs=" << s.gdn_output_max_abs
            << " gdn_out_rel=" << s.gdn_output_max_rel << " gdn_state_abs=" << s.gdn_state_max_abs
            << " gdn_state_rel=" << s.gdn_state_max_rel;
        throw std::runtime_error(oss.str());
    }
}

// ---- checks of the attention tail (src/driver.cpp:8244-8300, 8430-8466) ----
void check_tail(Layer0& L, Layer0RecurrentAttentionStats& s, DevBuf& gdn_ref, DevBuf& gated_ref) {
    ck(q38_check_rmsnorm(gdn_ref.get(), L.ssm_norm.get(), L.z_y.get(), kValueHeads, kHeadDim, L.eps, gated_ref.get(),
                         nullptr),
       "check gated norm");
    constexpr std::uint32_t kRows = 8;
    const auto ssm_ref = ref_rows(L.ctx, L.ssm_out->d, kRows, gated_ref.get());
    const auto hid = download(L.hidden.get(), kRows, "hidden");
    const auto ssm = download(L.ssm_y.get(), kRows, "ssm_out"), res = download(L.residual.get(), kRows, "residual");
    s.gated_norm_max_abs =
        max_abs_diff(download(L.gated.get(), kValueDim, "gated"), download(gated_ref.get(), kValueDim, "gated ref"));
    for (std::uint32_t r = 0; r < kRows; ++r) {
        s.ssm_out_max_abs = std::max(s.ssm_out_max_abs, std::abs(static_cast<double>(ssm[r]) - ssm_ref[r]));
        s.residual_max_abs = std::max(
            s.residual_max_abs, std::abs(static_cast<double>(res[r]) - (ssm_ref[r] + static_cast<double>(hid[r]))));
    }
    if (s.gated_norm_max_abs > 2.0e-4 || s.ssm_out_max_abs > 3.0e-3 || s.residual_max_abs > 3.0e-3) {
        std::ostringstream oss;
        oss << "layer0 recurrent attention tail mismatch: gated_norm=" << s.gated_norm_max_abs
            << " ssm_out=" << s.ssm_out_max_abs << " residual=" << s.residual_max_abs;
        throw std::runtime_error(oss.str());
    }
}

// ---- checks of the FFN (src/driver.cpp:8365-8530) ----
void check_ffn(Layer0& L, Layer0FullStats& s) {
    q38_ctx* c = L.ctx;
    DevBuf normed_ref(c, kCols * 4u), mul_ref(c, kFfnDim * 4u);
    ck(q38_check_rmsnorm(L.residual.get(), L.post_norm.get(), 0, 1, kCols, L.eps, normed_ref.get(), nullptr),
       "check post norm");
    ck(q38_check_silu_mul(L.ffn_gate_y.get(), L.ffn_up_y.get(), kFfnDim, mul_ref.get(), nullptr), "check SiLU * up");
    constexpr std::uint32_t kRows = 8;
    const auto down_ref = ref_rows(c, L.down->d, kRows, mul_ref.get());
    const auto res = download(L.residual.get(), kRows, "residual");
    const auto down = download(L.ffn_down_y.get(), kRows, "ffn_down"), out = download(L.layer_out.get(), kRows, "out");
    s.ffn_norm_max_abs =
        max_abs_diff(download(L.ffn_normed.get(), kCols, "ffn normed"), download(normed_ref.get(), kCols, "ref"));
    s.ffn_gate_up_max_abs =
        max_abs_diff(download(L.ffn_mul.get(), kFfnDim, "ffn mul"), download(mul_ref.get(), kFfnDim, "ref"));
    for (std::uint32_t r = 0; r < kRows; ++r) {
        s.ffn_down_max_abs = std::max(s.ffn_down_max_abs, std::abs(static_cast<double>(down[r]) - down_ref[r]));
        s.layer_output_max_abs = std::max(s.layer_output_max_abs,
                                          std::abs(static_cast<double>(out[r]) -
                                                   (down_ref[r] + static_cast<double>(res[r]))));
    }
    if (s.ffn_norm_max_abs > 3.0e-4 || s.ffn_gate_up_max_abs > 3.0e-4 || s.ffn_down_max_abs > 4.0e-3 ||
        s.layer_output_max_abs > 4.0e-3) {
        std::ostringstream oss;
        oss << "layer0 FFN mismatch: norm=" << s.ffn_norm_max_abs << " gate_up=" << s.ffn_gate_up_max_abs
            << " down=" << s.ffn_down_max_abs << " output=" << s.layer_output_max_abs;
        throw std::runtime_error(oss.str());
    }
}

struct FrontTimes {
    double projection, prep, gdn, chain;
};
FrontTimes time_front(Layer0& L) {
    FrontTimes t{};
    t.projection = bench_ms(50, [&] { L.projection(); }, "front projection benchmark");
    t.prep = bench_ms(200, [&] { L.prep(); }, "front prep benchmark");
    t.gdn = bench_ms(200, [&] { L.gdn(); }, "front gdn benchmark");
    t.chain = bench_ms(50, [&] { L.front(); }, "front chain benchmark");
    return t;
}

void sync(const char* what) { ck(q38_stream_synchronize(nullptr), what); }

// The reference's GDN decode-core smoke inputs (src/driver.cpp:11198-11244).
void gdn_smoke_inputs(std::uint32_t D, std::uint32_t Hq, std::uint32_t Hv, std::vector<float>& q, std::vector<float>& k,
                      std::vector<float>& v, std::vector<float>& g, std::vector<float>& beta,
                      std::vector<float>& state) {
    constexpr float kEps = 1.0e-6f;
    q.assign(static_cast<std::size_t>(Hq) * D, 0.0f);
    k.assign(q.size(), 0.0f);
    v.assign(static_cast<std::size_t>(Hv) * D, 0.0f);
    g.assign(Hv, 0.0f);
    beta.assign(Hv, 0.0f);
    state.assign(static_cast<std::size_t>(Hv) * D * D, 0.0f);
    for (std::uint32_t h = 0; h < Hq; ++h) {
        double q_ss = 0.0, k_ss = 0.0;
        for (std::uint32_t i = 0; i < D; ++i) {
            const float fi = static_cast<float>(i), fh = static_cast<float>(h);
            const float qv = std::sin(fi * 0.037f + fh * 0.11f) * 0.8f + std::cos(fi * 0.013f - fh * 0.07f) * 0.2f;
            const float kv = std::cos(fi * 0.029f + fh * 0.09f) * 0.75f - std::sin(fi * 0.017f + fh * 0.05f) * 0.25f;
            q[static_cast<std::size_t>(h) * D + i] = qv;
            k[static_cast<std::size_t>(h) * D + i] = kv;
            q_ss += static_cast<double>(qv) * qv;
            k_ss += static_cast<double>(kv) * kv;
        }
        const double q_inv = 1.0 / std::sqrt(q_ss + kEps), k_inv = 1.0 / std::sqrt(k_ss + kEps);
        for (std::uint32_t i = 0; i < D; ++i) {
            float& qe = q[static_cast<std::size_t>(h) * D + i];
            float& ke = k[static_cast<std::size_t>(h) * D + i];
            qe = static_cast<float>(static_cast<double>(qe) * q_inv);
            ke = static_cast<float>(static_cast<double>(ke) * k_inv);
        }
    }
    for (std::uint32_t h = 0; h < Hv; ++h) {
        g[h] = -0.025f - 0.0015f * static_cast<float>(h % 19);
        beta[h] = 0.20f + 0.012f * static_cast<float>(h % 37);
        for (std::uint32_t col = 0; col < D; ++col) {
            const std::size_t o = static_cast<std::size_t>(h) * D + col;
            const float fidx = static_cast<float>(o);
            v[o] = std::sin(fidx * 0.009f) * 0.7f + std::cos(fidx * 0.004f) * 0.3f;
            const std::size_t base = o * D;
            for (std::uint32_t i = 0; i < D; ++i) {
                const float fs = static_cast<float>(base + i);
                state[base + i] = 0.012f * std::sin(fs * 0.0013f) + 0.006f * std::cos(fs * 0.0007f);
            }
        }
    }
}

}  // namespace

bool NvidiaDriver::run_gdn_ar_smoke(std::uint32_t state_dim, std::uint32_t qk_heads, std::uint32_t value_heads,
                                    GdnArSmokeStats* stats, std::string* error) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        if (state_dim != 128) throw std::invalid_argument("the GDN step is specialised for state_dim=128");
        if (qk_heads == 0 || value_heads == 0 || value_heads % qk_heads != 0)
            throw std::invalid_argument("GDN AR requires non-zero heads and value_heads divisible by qk_heads");
        std::vector<float> q, k, v, g, beta, state;
        gdn_smoke_inputs(state_dim, qk_heads, value_heads, q, k, v, g, beta, state);
        const std::size_t nv = v.size(), ns = state.size();
        DevBuf qd(ctx, q.size() * 4u), kd(ctx, k.size() * 4u), vd(ctx, nv * 4u), gd(ctx, g.size() * 4u),
            bd(ctx, beta.size() * 4u), sin(ctx, ns * 4u), out(ctx, nv * 4u), sout(ctx, ns * 4u), oref(ctx, nv * 4u),
            sref(ctx, ns * 4u);
        upload(qd.get(), q.data(), q.size() * 4u, "q");
        upload(kd.get(), k.data(), k.size() * 4u, "k");
        upload(vd.get(), v.data(), nv * 4u, "v");
        upload(gd.get(), g.data(), g.size() * 4u, "g");
        upload(bd.get(), beta.data(), beta.size() * 4u, "beta");
        upload(sin.get(), state.data(), ns * 4u, "state");
        const float scale = 1.0f / std::sqrt(static_cast<float>(state_dim));
        auto launch = [&] {
            ck(q38_gdn_step(qd.get(), kd.get(), vd.get(), gd.get(), bd.get(), sin.get(), out.get(), sout.get(),
                            qk_heads, value_heads, scale, nullptr),
               "q38_gdn_step");
        };
        launch();
        ck(q38_check_gdn(qd.get(), kd.get(), vd.get(), gd.get(), bd.get(), sin.get(), oref.get(), sref.get(),
                         qk_heads, value_heads, state_dim, nullptr),
           "check GDN");
        sync("GDN AR correctness");
        GdnArSmokeStats local{};
        const auto o = download(out.get(), nv, "out"), o_ref = download(oref.get(), nv, "out ref");
        const auto st = download(sout.get(), ns, "state"), st_ref = download(sref.get(), ns, "state ref");
        bool bad = false;
        for (std::size_t i = 0; i < nv; ++i) {
            const double ae = std::abs(static_cast<double>(o[i]) - o_ref[i]);
            const double re = ae / std::max(1.0e-6, std::abs(static_cast<double>(o_ref[i])));
            local.output_max_abs = std::max(local.output_max_abs, ae);
            local.output_max_rel = std::max(local.output_max_rel, re);
            if (ae > 5.0e-4 && re > 5.0e-4) bad = true;
        }
        for (std::size_t i = 0; i < ns; ++i) {
            const double ae = std::abs(static_cast<double>(st[i]) - st_ref[i]);
            const double re = ae / std::max(1.0e-6, std::abs(static_cast<double>(st_ref[i])));
            local.state_max_abs = std::max(local.state_max_abs, ae);
            local.state_max_rel = std::max(local.state_max_rel, re);
            if (ae > 2.0e-4 && re > 2.0e-4) bad = true;
        }
        if (bad) {
            std::ostringstream oss;
            oss << "GDN AR mismatch: output_abs=" << local.output_max_abs << " output_rel=" << local.output_max_rel
                << " state_abs=" << local.state_max_abs << " state_rel=" << local.state_max_rel;
            throw std::runtime_error(oss.str());
        }
        local.kernel_ms = bench_ms(100, launch, "GDN AR benchmark");
        local.state_bandwidth_gbps = static_cast<double>(ns * 4u * 2u) / (local.kernel_ms / 1000.0) / 1.0e9;
        if (stats) *stats = local;
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

bool NvidiaDriver::run_recurrent_prep_smoke(const float* conv_weight, const float* dt_bias, const float* ssm_a,
                                            RecurrentPrepSmokeStats* stats, std::string* error) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        if (!conv_weight || !dt_bias || !ssm_a) throw std::invalid_argument("recurrent prep received null tensor");
        // src/driver.cpp:10745-10768
        std::vector<float> qkv(kQkvRows), braw(kValueHeads), araw(kValueHeads), st(3u * kQkvRows);
        for (std::uint32_t i = 0; i < kQkvRows; ++i) {
            const float fi = static_cast<float>(i);
            qkv[i] = 0.55f * std::sin(fi * 0.013f) + 0.31f * std::cos(fi * 0.007f);
            for (std::uint32_t s = 0; s < 3u; ++s) {
                const float fs = static_cast<float>(s + 1);
                st[static_cast<std::size_t>(s) * kQkvRows + i] =
                    0.10f * std::sin(fi * (0.003f + 0.001f * fs)) + 0.04f * std::cos(fi * (0.002f + 0.0005f * fs));
            }
        }
        for (std::uint32_t h = 0; h < kValueHeads; ++h) {
            const float fh = static_cast<float>(h);
            braw[h] = 0.2f * std::sin(fh * 0.21f) - 0.05f;
            araw[h] = 0.3f * std::cos(fh * 0.17f) - 0.1f;
        }
        DevBuf qd(ctx, kQkvRows * 4u), sd(ctx, st.size() * 4u), bd(ctx, kValueHeads * 4u), ad(ctx, kValueHeads * 4u);
        upload(qd.get(), qkv.data(), kQkvRows * 4u, "qkv");
        upload(sd.get(), st.data(), st.size() * 4u, "conv state");
        upload(bd.get(), braw.data(), kValueHeads * 4u, "beta raw");
        upload(ad.get(), araw.data(), kValueHeads * 4u, "alpha raw");
        DevBuf w = f32_buf(ctx, conv_weight, 4u * kQkvRows, "conv weight");
        DevBuf dt = f32_buf(ctx, dt_bias, kValueHeads, "dt bias"), A = f32_buf(ctx, ssm_a, kValueHeads, "ssm_a");
        DevBuf conv(ctx, kQkvRows * 4u), so(ctx, st.size() * 4u), q(ctx, kKeyDim * 4u), k(ctx, kKeyDim * 4u),
            beta(ctx, kValueHeads * 4u), gate(ctx, kValueHeads * 4u);
        DevBuf conv_r(ctx, kQkvRows * 4u), so_r(ctx, st.size() * 4u), q_r(ctx, kKeyDim * 4u), k_r(ctx, kKeyDim * 4u),
            beta_r(ctx, kValueHeads * 4u), gate_r(ctx, kValueHeads * 4u);
        constexpr float kEps = 1.0e-6f;
        auto launch_conv = [&] {
            ck(q38_conv4_silu_roll(qd.get(), w.get(), sd.get(), conv.get(), so.get(), kQkvRows, nullptr), "conv");
        };
        auto launch_qk = [&] { ck(q38_qk_l2norm(conv.get(), q.get(), k.get(), kQkHeads, kEps, nullptr), "qk norm"); };
        auto launch_bg = [&] {
            ck(q38_beta_gate(bd.get(), ad.get(), dt.get(), A.get(), beta.get(), gate.get(), kValueHeads, nullptr),
               "beta/gate");
        };
        launch_conv();
        launch_qk();
        launch_bg();
        ck(q38_check_conv4(qd.get(), w.get(), sd.get(), conv_r.get(), so_r.get(), kQkvRows, nullptr), "check conv");
        ck(q38_check_l2norm(conv_r.get(), kQkHeads, kHeadDim, kEps, q_r.get(), nullptr), "check q");
        ck(q38_check_l2norm(conv_r.get() + 4u * kKeyDim, kQkHeads, kHeadDim, kEps, k_r.get(), nullptr), "check k");
        ck(q38_check_beta_gate(bd.get(), ad.get(), dt.get(), A.get(), kValueHeads, beta_r.get(), gate_r.get(), nullptr),
           "check beta/gate");
        sync("recurrent prep correctness");
        RecurrentPrepSmokeStats local{};
        local.conv_max_abs = max_abs_diff(download(conv.get(), kQkvRows, "conv"), download(conv_r.get(), kQkvRows, "r"));
        local.q_max_abs = max_abs_diff(download(q.get(), kKeyDim, "q"), download(q_r.get(), kKeyDim, "r"));
        local.k_max_abs = max_abs_diff(download(k.get(), kKeyDim, "k"), download(k_r.get(), kKeyDim, "r"));
        local.beta_max_abs =
            max_abs_diff(download(beta.get(), kValueHeads, "beta"), download(beta_r.get(), kValueHeads, "r"));
        local.gate_max_abs =
            max_abs_diff(download(gate.get(), kValueHeads, "gate"), download(gate_r.get(), kValueHeads, "r"));
        local.conv_state_max_abs =
            max_abs_diff(download(so.get(), st.size(), "state"), download(so_r.get(), st.size(), "r"));
        if (local.conv_max_abs > 5.0e-4 || local.q_max_abs > 5.0e-4 || local.k_max_abs > 5.0e-4 ||
            local.beta_max_abs > 5.0e-5 || local.gate_max_abs > 5.0e-4 || local.conv_state_max_abs > 1.0e-7) {
            std::ostringstream oss;
            oss << "recurrent prep mismatch: conv=" << local.conv_max_abs << " q=" << local.q_max_abs
                << " k=" << local.k_max_abs << " beta=" << local.beta_max_abs << " gate=" << local.gate_max_abs
                << " state=" << local.conv_state_max_abs;
            throw std::runtime_error(oss.str());
        }
        local.conv_silu_ms = bench_ms(200, launch_conv, "recurrent conv benchmark");
        local.qk_norm_ms = bench_ms(500, launch_qk, "recurrent qk benchmark");
        local.beta_gate_ms = bench_ms(1000, launch_bg, "recurrent beta/gate benchmark");
        local.chain_ms = bench_ms(
            200,
            [&] {
                launch_conv();
                launch_qk();
                launch_bg();
            },
            "recurrent prep chain benchmark");
        if (stats) *stats = local;
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

bool NvidiaDriver::run_qwen35_layer0_recurrent_front(const float* norm_weight, const std::byte* qkv_matrix,
                                                     std::size_t qkv_qh_offset, std::size_t qkv_qs_offset,
                                                     const std::byte* z_matrix, std::size_t z_qh_offset,
                                                     std::size_t z_qs_offset, const std::byte* beta_matrix,
                                                     const std::byte* alpha_matrix, const float* conv_weight,
                                                     const float* dt_bias, const float* ssm_a, float rms_eps,
                                                     Layer0RecurrentFrontStats* stats, std::string* error) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        Layer0 L(ctx, rms_eps, norm_weight, qkv_matrix, qkv_qh_offset, qkv_qs_offset, z_matrix, z_qh_offset,
                 z_qs_offset, beta_matrix, alpha_matrix, conv_weight, dt_bias, ssm_a);
        L.front();
        DevBuf conv_r(ctx, kQkvRows * 4u), q_r(ctx, kKeyDim * 4u), k_r(ctx, kKeyDim * 4u),
            beta_r(ctx, kSmallRows * 4u), gate_r(ctx, kSmallRows * 4u), gdn_r(ctx, kValueDim * 4u);
        Layer0RecurrentFrontStats local{};
        check_front(L, local, conv_r, q_r, k_r, beta_r, gate_r, gdn_r);
        const FrontTimes t = time_front(L);
        local.projection_ms = t.projection;
        local.conv_prep_ms = t.prep;
        local.gdn_ms = t.gdn;
        local.sum_stage_ms = t.projection + t.prep + t.gdn;
        local.chain_ms = t.chain;
        if (stats) *stats = local;
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

bool NvidiaDriver::run_qwen35_layer0_recurrent_attention(
    const float* norm_weight, const std::byte* qkv_matrix, std::size_t qkv_qh_offset, std::size_t qkv_qs_offset,
    const std::byte* z_matrix, std::size_t z_qh_offset, std::size_t z_qs_offset, const std::byte* beta_matrix,
    const std::byte* alpha_matrix, const float* conv_weight, const float* dt_bias, const float* ssm_a,
    const float* ssm_norm_weight, const std::byte* ssm_out_matrix, std::size_t ssm_out_qh_offset,
    std::size_t ssm_out_qs_offset, float rms_eps, Layer0RecurrentAttentionStats* stats, std::string* error) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        Layer0 L(ctx, rms_eps, norm_weight, qkv_matrix, qkv_qh_offset, qkv_qs_offset, z_matrix, z_qh_offset,
                 z_qs_offset, beta_matrix, alpha_matrix, conv_weight, dt_bias, ssm_a);
        L.add_tail(ssm_norm_weight, ssm_out_matrix, ssm_out_qh_offset, ssm_out_qs_offset);
        L.attention();
        DevBuf conv_r(ctx, kQkvRows * 4u), q_r(ctx, kKeyDim * 4u), k_r(ctx, kKeyDim * 4u),
            beta_r(ctx, kSmallRows * 4u), gate_r(ctx, kSmallRows * 4u), gdn_r(ctx, kValueDim * 4u),
            gated_r(ctx, kValueDim * 4u);
        Layer0RecurrentFrontStats front{};
        check_front(L, front, conv_r, q_r, k_r, beta_r, gate_r, gdn_r);
        Layer0RecurrentAttentionStats local{};
        check_tail(L, local, gdn_r, gated_r);
        local.front_ms = time_front(L).chain;
        local.gated_norm_ms = bench_ms(
            200,
            [&] {
                ck(q38_gated_rmsnorm_silu(L.gdn_out.get(), L.ssm_norm.get(), L.z_y.get(), L.gated.get(), kValueHeads,
                                          rms_eps, nullptr),
                   "gated norm");
            },
            "attention gated norm benchmark");
        local.ssm_out_ms = bench_ms(50, [&] { ck(L.ssm_out->gemv(L.gated.get(), L.ssm_y.get()), "ssm_out"); },
                                    "attention ssm_out benchmark");
        local.tail_ms = bench_ms(50, [&] { L.tail(); }, "attention tail benchmark");
        local.sum_stage_ms = local.front_ms + local.tail_ms;
        local.chain_ms = bench_ms(50, [&] { L.attention(); }, "attention full chain benchmark");
        if (stats) *stats = local;
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

bool NvidiaDriver::run_qwen35_layer0_full(const float* norm_weight, const std::byte* qkv_matrix,
                                          std::size_t qkv_qh_offset, std::size_t qkv_qs_offset,
                                          const std::byte* z_matrix, std::size_t z_qh_offset, std::size_t z_qs_offset,
                                          const std::byte* beta_matrix, const std::byte* alpha_matrix,
                                          const float* conv_weight, const float* dt_bias, const float* ssm_a,
                                          const float* ssm_norm_weight, const std::byte* ssm_out_matrix,
                                          std::size_t ssm_out_qh_offset, std::size_t ssm_out_qs_offset,
                                          const float* post_norm_weight, const std::byte* ffn_gate_matrix,
                                          const std::byte* ffn_up_matrix, std::size_t ffn_up_qh_offset,
                                          std::size_t ffn_up_qs_offset, const std::byte* ffn_down_matrix,
                                          std::size_t ffn_down_qh_offset, std::size_t ffn_down_qs_offset,
                                          float rms_eps, Layer0FullStats* stats, std::string* error) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        Layer0 L(ctx, rms_eps, norm_weight, qkv_matrix, qkv_qh_offset, qkv_qs_offset, z_matrix, z_qh_offset,
                 z_qs_offset, beta_matrix, alpha_matrix, conv_weight, dt_bias, ssm_a);
        L.add_tail(ssm_norm_weight, ssm_out_matrix, ssm_out_qh_offset, ssm_out_qs_offset);
        L.add_ffn(post_norm_weight, ffn_gate_matrix, ffn_up_matrix, ffn_up_qh_offset, ffn_up_qs_offset,
                  ffn_down_matrix, ffn_down_qh_offset, ffn_down_qs_offset);
        L.attention();
        L.ffn();
        DevBuf conv_r(ctx, kQkvRows * 4u), q_r(ctx, kKeyDim * 4u), k_r(ctx, kKeyDim * 4u),
            beta_r(ctx, kSmallRows * 4u), gate_r(ctx, kSmallRows * 4u), gdn_r(ctx, kValueDim * 4u),
            gated_r(ctx, kValueDim * 4u);
        Layer0RecurrentFrontStats front{};
        check_front(L, front, conv_r, q_r, k_r, beta_r, gate_r, gdn_r);
        Layer0RecurrentAttentionStats att{};
        check_tail(L, att, gdn_r, gated_r);
        Layer0FullStats local{};
        check_ffn(L, local);
        local.attention_ms = bench_ms(50, [&] { L.attention(); }, "attention full chain benchmark");
        local.post_norm_ms = bench_ms(100, [&] { L.post_norm_stage(); }, "ffn post norm benchmark");
        local.ffn_gate_ms = bench_ms(50, [&] { L.ffn_gate(); }, "ffn gate benchmark");
        local.ffn_up_ms = bench_ms(50, [&] { L.ffn_up(); }, "ffn up benchmark");
        local.ffn_pointwise_ms = bench_ms(200, [&] { L.ffn_pointwise(); }, "ffn pointwise benchmark");
        local.ffn_down_ms = bench_ms(50, [&] { L.ffn_down(); }, "ffn down benchmark");
        local.ffn_ms = bench_ms(50, [&] { L.ffn(); }, "ffn full benchmark");
        local.sum_stage_ms = local.attention_ms + local.ffn_ms;
        local.chain_ms = bench_ms(
            50,
            [&] {
                L.attention();
                L.ffn();
            },
            "full layer benchmark");
        if (stats) *stats = local;
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

bool NvidiaDriver::run_qwen35_layer0_projection_pack(const float* norm_weight, const std::byte* qkv_matrix,
                                                     std::size_t qkv_qh_offset, std::size_t qkv_qs_offset,
                                                     std::uint32_t qkv_rows, const std::byte* gate_matrix,
                                                     std::size_t gate_qh_offset, std::size_t gate_qs_offset,
                                                     std::uint32_t gate_rows, const std::byte* beta_matrix,
                                                     const std::byte* alpha_matrix, std::uint32_t cols,
                                                     std::uint32_t small_rows, float rms_eps,
                                                     Layer0ProjectionPackStats* stats, std::string* error) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        if (cols == 0 || cols % 256u || !qkv_rows || !gate_rows || !small_rows)
            throw std::invalid_argument("layer0 projection pack needs non-zero rows and cols divisible by 256");
        DevBuf norm = f32_buf(ctx, norm_weight, cols, "norm weight");
        SoAMat qkv(ctx, qkv_matrix, qkv_qh_offset, qkv_qs_offset, qkv_rows, cols, "qkv");
        SoAMat gate(ctx, gate_matrix, gate_qh_offset, gate_qs_offset, gate_rows, cols, "gate");
        NativeMat beta(ctx, beta_matrix, Q38_TYPE_Q4_K, 144, small_rows, cols, "beta");
        NativeMat alpha(ctx, alpha_matrix, Q38_TYPE_Q4_K, 144, small_rows, cols, "alpha");
        const std::vector<float> hidden = facade::smoke_x(cols);
        DevBuf x(ctx, cols * 4u), normed(ctx, cols * 4u), normed_r(ctx, cols * 4u), qy(ctx, qkv_rows * 4u),
            gy(ctx, gate_rows * 4u), by(ctx, small_rows * 4u), ay(ctx, small_rows * 4u);
        upload(x.get(), hidden.data(), cols * 4u, "hidden");
        auto launch_norm = [&] { ck(q38_rmsnorm(x.get(), norm.get(), normed.get(), cols, 1, rms_eps, nullptr), "norm"); };
        auto launch_qkv = [&] { ck(qkv.gemv(normed.get(), qy.get()), "qkv"); };
        auto launch_gate = [&] { ck(gate.gemv(normed.get(), gy.get()), "gate"); };
        auto launch_beta = [&] { ck(beta.gemv(normed.get(), by.get()), "beta"); };
        auto launch_alpha = [&] { ck(alpha.gemv(normed.get(), ay.get()), "alpha"); };
        auto chain = [&] {
            launch_norm();
            launch_qkv();
            launch_gate();
            launch_beta();
            launch_alpha();
        };
        chain();
        ck(q38_check_rmsnorm(x.get(), norm.get(), 0, 1, cols, rms_eps, normed_r.get(), nullptr), "check norm");
        Layer0ProjectionPackStats local{};
        // the first rows of each projection against FP64 rows of the reference
        // norm (src/driver.cpp:11961-12100): Q5_K 4 rows at 3e-3, Q4_K 4 at 2e-3
        auto validate = [&](const q38_weight_desc& d, q38_devptr y, double tol, ProjectionErrorStats& out,
                            const char* what) {
            const std::uint32_t n = std::min<std::uint32_t>(d.rows, 4u);
            const auto ref = ref_rows(ctx, d, n, normed_r.get());
            const auto got = download(y, n, what);
            bool bad = false;
            for (std::uint32_t r = 0; r < n; ++r) {
                const double ae = std::abs(static_cast<double>(got[r]) - ref[r]);
                const double re = ae / std::max(1.0e-5, std::abs(ref[r]));
                out.max_abs = std::max(out.max_abs, ae);
                out.max_rel = std::max(out.max_rel, re);
                if (ae > tol && re > tol) bad = true;
            }
            if (bad) {
                std::ostringstream oss;
                oss << "layer0 " << what << " projection mismatch: max_abs=" << out.max_abs << " max_rel=" << out.max_rel;
                throw std::runtime_error(oss.str());
            }
        };
        validate(qkv.d, qy.get(), 3.0e-3, local.qkv, "qkv");
        validate(gate.d, gy.get(), 3.0e-3, local.gate, "gate");
        validate(beta.d, by.get(), 2.0e-3, local.beta, "beta");
        validate(alpha.d, ay.get(), 2.0e-3, local.alpha, "alpha");
        local.rmsnorm_ms = bench_ms(100, launch_norm, "layer0 norm benchmark");
        local.qkv_ms = bench_ms(50, launch_qkv, "layer0 qkv benchmark");
        local.gate_ms = bench_ms(50, launch_gate, "layer0 gate benchmark");
        local.beta_ms = bench_ms(1000, launch_beta, "layer0 beta benchmark");
        local.alpha_ms = bench_ms(1000, launch_alpha, "layer0 alpha benchmark");
        local.chain_ms = bench_ms(50, chain, "layer0 projection chain benchmark");
        if (stats) *stats = local;
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

bool NvidiaDriver::run_qwen35_layer0_gate_smoke(const float* norm_weight, const std::byte* repacked_matrix,
                                                std::size_t qh_offset, std::size_t qs_offset, std::uint32_t cols,
                                                std::uint32_t rows, float rms_eps, std::string* error,
                                                double* max_abs_error, double* max_rel_error, double* rmsnorm_ms,
                                                double* projection_ms, double* chain_ms,
                                                double* projection_original_equiv_gbps) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        if (cols == 0 || rows == 0 || cols % 256u)
            throw std::invalid_argument("layer0 gate smoke needs non-zero rows and cols divisible by 256");
        DevBuf norm = f32_buf(ctx, norm_weight, cols, "norm weight");
        SoAMat m(ctx, repacked_matrix, qh_offset, qs_offset, rows, cols, "gate");
        const std::vector<float> hidden = facade::smoke_x(cols);
        DevBuf x(ctx, cols * 4u), normed(ctx, cols * 4u), normed_r(ctx, cols * 4u), y(ctx, rows * 4u);
        upload(x.get(), hidden.data(), cols * 4u, "hidden");
        auto launch_norm = [&] { ck(q38_rmsnorm(x.get(), norm.get(), normed.get(), cols, 1, rms_eps, nullptr), "norm"); };
        auto launch_proj = [&] { ck(m.gemv(normed.get(), y.get()), "gate projection"); };
        launch_norm();
        launch_proj();
        ck(q38_check_rmsnorm(x.get(), norm.get(), 0, 1, cols, rms_eps, normed_r.get(), nullptr), "check norm");
        const std::uint32_t n = std::min<std::uint32_t>(rows, 8u);
        const auto ref = ref_rows(ctx, m.d, n, normed_r.get());
        const auto got = download(y.get(), n, "gate");
        double ma = 0.0, mr = 0.0;
        bool bad = false;
        for (std::uint32_t r = 0; r < n; ++r) {
            const double ae = std::abs(static_cast<double>(got[r]) - ref[r]);
            const double re = ae / std::max(1.0e-5, std::abs(ref[r]));
            ma = std::max(ma, ae);
            mr = std::max(mr, re);
            if (ae > 2.0e-3 && re > 2.0e-3) bad = true;
        }
        if (bad) throw std::runtime_error("layer0 gate mismatch: max_abs=" + std::to_string(ma));
        const double tn = bench_ms(100, launch_norm, "layer0 gate norm benchmark");
        const double tp = bench_ms(50, launch_proj, "layer0 gate projection benchmark");
        const double tc = bench_ms(
            50,
            [&] {
                launch_norm();
                launch_proj();
            },
            "layer0 gate chain benchmark");
        if (max_abs_error) *max_abs_error = ma;
        if (max_rel_error) *max_rel_error = mr;
        if (rmsnorm_ms) *rmsnorm_ms = tn;
        if (projection_ms) *projection_ms = tp;
        if (chain_ms) *chain_ms = tc;
        if (projection_original_equiv_gbps)
            *projection_original_equiv_gbps =
                static_cast<double>(rows) * (cols / 256u) * 176.0 / (tp / 1000.0) / 1.0e9;
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

}  // namespace q38
