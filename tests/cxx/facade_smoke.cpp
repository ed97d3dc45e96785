// A host program written against the reference's q38::NvidiaDriver and
// q38::PackFile interfaces (include/q38/driver.hpp, include/q38/q38pack.hpp)
// and linked to libq38driver_b200.so: it opens the device and calls every
// method of the facade -- the pattern, VMM and RMSNorm smokes, the GEMV and
// dequantisation smokes on the matrices a manifest lists, the Q8_K and Q8_1
// activation GEMVs, the GDN decode core, and the recurrent-prep and layer-0
// chains on the tensors of a Q38PACK -- printing `<method>_ok: 0|1` lines.
//
//   facade_smoke MANIFEST LAYER_PACK
//
// Manifest lines: `kind path cols rows [off1 off2]`, kind one of q4k, q5k,
// q6k, iq4xs (GGUF blocks), q5k_sm86 (SoA planes, qh and qs offsets) and
// iq4xs_sm86 (SoA planes, scale and qs offsets).  Exit status 0 and a final
// PASS line when every method succeeded.
#include <cstdio>
#include <fstream>
#include <functional>
#include <iostream>
#include <iterator>
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "q38/driver.hpp"
#include "q38/q38pack.hpp"

static std::vector<std::byte> read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    std::vector<char> raw((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    std::vector<std::byte> out(raw.size());
    for (size_t i = 0; i < raw.size(); ++i) out[i] = static_cast<std::byte>(raw[i]);
    return out;
}

struct Mat {
    std::vector<std::byte> bytes;
    uint32_t cols = 0, rows = 0;
    size_t off1 = 0, off2 = 0;
};

int main(int argc, char** argv) {
    if (argc < 3) {
        std::cerr << "usage: facade_smoke MANIFEST LAYER_PACK\n";
        return 2;
    }
    q38::NvidiaDriver d;
    try {
        d.open();
    } catch (const std::exception& e) {
        std::cerr << "open: " << e.what() << "\n";
        return 3;
    }
    std::cout << "device: " << d.device_name() << "\nsm: " << d.sm_major() << d.sm_minor()
              << "\nis_target_sm: " << (d.is_sm86() ? 1 : 0) << "\n";
    std::map<std::string, Mat> m;
    std::ifstream man(argv[1]);
    for (std::string line; std::getline(man, line);) {
        std::istringstream ls(line);
        std::string kind, path;
        Mat x;
        ls >> kind >> path >> x.cols >> x.rows >> x.off1 >> x.off2;
        x.bytes = read_file(path);
        m[kind] = std::move(x);
    }
    bool all = true;
    auto report = [&](const char* name, bool ok, const std::string& err, double a = 0, double r = 0) {
        std::cout << name << "_ok: " << (ok ? 1 : 0) << "\n" << name << "_max_abs: " << a << "\n"
                  << name << "_max_rel: " << r << "\n";
        if (!ok) std::cout << name << "_error: " << err << "\n";
        all = all && ok;
    };
    std::string err;
    double ma = 0, mr = 0, ms = 0, g1 = 0, g2 = 0;
    report("probe_vmm", d.probe_vmm(64u << 20, &err), err);
    report("run_sm86_smoke", d.run_sm86_smoke(&err), err);
    err.clear();
    report("run_rmsnorm_smoke", d.run_rmsnorm_smoke(&err, &ma, &mr), err, ma, mr);
    // GEMV smokes
    using Gemv = bool (q38::NvidiaDriver::*)(const std::byte*, uint32_t, uint32_t, std::string*, double*, double*,
                                            double*, double*);
    const std::pair<const char*, std::pair<const char*, Gemv>> gemvs[] = {
        {"q4k", {"run_q4k_gemv_smoke", &q38::NvidiaDriver::run_q4k_gemv_smoke}},
        {"q5k", {"run_q5k_gemv_smoke", &q38::NvidiaDriver::run_q5k_gemv_smoke}},
        {"q6k", {"run_q6k_gemv_smoke", &q38::NvidiaDriver::run_q6k_gemv_smoke}},
        {"iq4xs", {"run_iq4xs_gemv_smoke", &q38::NvidiaDriver::run_iq4xs_gemv_smoke}},
        {"q5k", {"run_q5k_q8k_gemv_smoke", &q38::NvidiaDriver::run_q5k_q8k_gemv_smoke}},
        {"iq4xs", {"run_iq4xs_q8_1_gemv_smoke", &q38::NvidiaDriver::run_iq4xs_q8_1_gemv_smoke}},
    };
    for (const auto& g : gemvs) {
        const Mat& x = m.at(g.first);
        err.clear();
        ma = mr = ms = g1 = 0;
        const bool ok = (d.*(g.second.second))(x.bytes.data(), x.cols, x.rows, &err, &ma, &mr, &ms, &g1);
        report(g.second.first, ok, err, ma, mr);
        std::cout << g.second.first << "_gbps: " << g1 << "\n";
    }
    {
        const Mat& x = m.at("q5k_sm86");
        err.clear();
        const bool ok = d.run_q5k_sm86_gemv_smoke(x.bytes.data(), x.off1, x.off2, x.cols, x.rows, &err, &ma, &mr, &ms,
                                                  &g1, &g2);
        report("run_q5k_sm86_gemv_smoke", ok, err, ma, mr);
        std::cout << "run_q5k_sm86_gemv_smoke_gbps: " << g1 << "\n";
    }
    {
        const Mat& x = m.at("iq4xs_sm86");
        err.clear();
        const bool ok = d.run_iq4xs_sm86_gemv_smoke(x.bytes.data(), x.off1, x.off2, x.cols, x.rows, &err, &ma, &mr,
                                                    &ms, &g1, &g2);
        report("run_iq4xs_sm86_gemv_smoke", ok, err, ma, mr);
        std::cout << "run_iq4xs_sm86_gemv_smoke_gbps: " << g1 << "\n";
    }
    // dequantisation smokes on the first block of each GGUF matrix
    err.clear();
    report("run_q4k_dequant_smoke", d.run_q4k_dequant_smoke(m.at("q4k").bytes.data(), &err, &ma, &mr), err, ma, mr);
    err.clear();
    report("run_q5k_dequant_smoke", d.run_q5k_dequant_smoke(m.at("q5k").bytes.data(), &err, &ma, &mr), err, ma, mr);
    err.clear();
    uint32_t first_bad = 0;
    report("run_q6k_dequant_smoke", d.run_q6k_dequant_smoke(m.at("q6k").bytes.data(), &err, &ma, &mr, &first_bad),
           err, ma, mr);
    std::cout << "q6k_first_bad_index: " << first_bad << "\n";
    err.clear();
    report("run_iq4xs_dequant_smoke", d.run_iq4xs_dequant_smoke(m.at("iq4xs").bytes.data(), &err, &ma, &mr), err,
           ma, mr);
    // the GDN decode core on the reference's own inputs
    q38::GdnArSmokeStats gs{};
    err.clear();
    report("run_gdn_ar_smoke", d.run_gdn_ar_smoke(128, 16, 48, &gs, &err), err, gs.output_max_abs,
           gs.output_max_rel);
    std::cout << "gdn_kernel_ms: " << gs.kernel_ms << "\ngdn_state_gbps: " << gs.state_bandwidth_gbps << "\n";
    // recurrent prep and the layer-0 chains on a pack's tensors
    q38::PackFile pack;
    pack.open(argv[2]);
    auto T = [&](const char* n) -> const q38::TensorRecord& {
        const auto* t = pack.find_tensor(n);
        if (!t) throw std::runtime_error(std::string("missing ") + n);
        return *t;
    };
    auto F = [&](const char* n) { return reinterpret_cast<const float*>(pack.tensor_data(T(n))); };
    auto B = [&](const char* n) { return pack.tensor_data(T(n)); };
    auto QH = [&](const char* n) { return static_cast<size_t>(T(n).aux0_offset - T(n).data_offset); };
    auto QS = [&](const char* n) { return static_cast<size_t>(T(n).aux1_offset - T(n).data_offset); };
    const char *norm = "blk.0.attn_norm.weight", *qkv = "blk.0.attn_qkv.weight", *z = "blk.0.attn_gate.weight",
               *beta = "blk.0.ssm_beta.weight", *alpha = "blk.0.ssm_alpha.weight", *conv = "blk.0.ssm_conv1d.weight",
               *dt = "blk.0.ssm_dt.bias", *A = "blk.0.ssm_a", *snorm = "blk.0.ssm_norm.weight",
               *sout = "blk.0.ssm_out.weight", *pnorm = "blk.0.post_attention_norm.weight",
               *fg = "blk.0.ffn_gate.weight", *fu = "blk.0.ffn_up.weight", *fd = "blk.0.ffn_down.weight";
    q38::RecurrentPrepSmokeStats ps{};
    err.clear();
    report("run_recurrent_prep_smoke", d.run_recurrent_prep_smoke(F(conv), F(dt), F(A), &ps, &err), err,
           ps.conv_max_abs);
    q38::Layer0ProjectionPackStats pp{};
    err.clear();
    report("run_qwen35_layer0_projection_pack",
           d.run_qwen35_layer0_projection_pack(F(norm), B(qkv), QH(qkv), QS(qkv), 10240, B(z), QH(z), QS(z), 6144,
                                               B(beta), B(alpha), 5120, 48, 1e-6f, &pp, &err),
           err, pp.qkv.max_abs, pp.qkv.max_rel);
    err.clear();
    report("run_qwen35_layer0_gate_smoke",
           d.run_qwen35_layer0_gate_smoke(F(norm), B(z), QH(z), QS(z), 5120, 6144, 1e-6f, &err, &ma, &mr), err, ma,
           mr);
    q38::Layer0RecurrentFrontStats fs{};
    err.clear();
    report("run_qwen35_layer0_recurrent_front",
           d.run_qwen35_layer0_recurrent_front(F(norm), B(qkv), QH(qkv), QS(qkv), B(z), QH(z), QS(z), B(beta),
                                               B(alpha), F(conv), F(dt), F(A), 1e-6f, &fs, &err),
           err, fs.gdn_output_max_abs, fs.gdn_output_max_rel);
    q38::Layer0RecurrentAttentionStats as{};
    err.clear();
    report("run_qwen35_layer0_recurrent_attention",
           d.run_qwen35_layer0_recurrent_attention(F(norm), B(qkv), QH(qkv), QS(qkv), B(z), QH(z), QS(z), B(beta),
                                                   B(alpha), F(conv), F(dt), F(A), F(snorm), B(sout), QH(sout),
                                                   QS(sout), 1e-6f, &as, &err),
           err, as.gated_norm_max_abs);
    q38::Layer0FullStats ls{};
    err.clear();
    report("run_qwen35_layer0_full",
           d.run_qwen35_layer0_full(F(norm), B(qkv), QH(qkv), QS(qkv), B(z), QH(z), QS(z), B(beta), B(alpha),
                                    F(conv), F(dt), F(A), F(snorm), B(sout), QH(sout), QS(sout), F(pnorm), B(fg), B(fu),
                                    QH(fu), QS(fu), B(fd), QH(fd), QS(fd), 1e-6f, &ls, &err),
           err, ls.layer_output_max_abs);
    std::cout << "layer_chain_ms: " << ls.chain_ms << "\n";
    d.close();
    std::cout << (all ? "PASS" : "FAIL") << "\n";
    return all ? 0 : 1;
}
