// q38_layer_cmds.cpp -- the reference's layer, recurrent and probe commands
// (CMakeLists.txt:21-94 there) over q38::Runtime / q38::NvidiaDriver, one
// binary per command, selected at build time by Q38_CMD:
//   1 q38-gpu-smoke             (src/gpu_smoke.cpp)
//   2 q38-rmsnorm-smoke         (src/rmsnorm_smoke.cpp)
//   3 q38-gdn-ar-smoke          (src/gdn_ar_smoke.cpp)
//   4 q38-recurrent-prep        (src/recurrent_prep.cpp)
//   5 q38-q5k-q8k-gemv          (src/q5k_q8k_gemv.cpp)
//   6 q38-q4k-smoke  7 q38-q5k-smoke  8 q38-iq4xs-smoke (dequantisation)
//   9 q38-layer0-projections   10 q38-layer0-gate
//  11 q38-layer0-recurrent-front  12 q38-layer0-recurrent-attention
//  13 q38-layer0-full          14 q38-recurrent-layer
//  15 q38-layer-topology       16 q38-runtime
// Arguments, exit codes and the `key: value` lines with the final PASS line
// follow the reference's mains.
#include <cstdint>
#include <cstring>
#include <iomanip>
#include <iostream>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/q38/runtime.hpp"

#ifndef Q38_CMD
#error "define Q38_CMD"
#endif

namespace {

struct Args {
    std::string model, tensor;
    std::uint32_t layer = 0;
    bool have_layer = false, no_gpu = false, list = false, gpu_smoke = false;
    float rms_eps = 1.0e-6f;
};

Args parse(int argc, char** argv, const char* usage) {
    Args a;
    for (int i = 1; i < argc; ++i) {
        const std::string arg = argv[i];
        if (arg == "--model" && i + 1 < argc) a.model = argv[++i];
        else if (arg == "--tensor" && i + 1 < argc) a.tensor = argv[++i];
        else if (arg == "--rms-eps" && i + 1 < argc) a.rms_eps = std::stof(argv[++i]);
        else if (arg == "--layer" && i + 1 < argc) {
            a.layer = static_cast<std::uint32_t>(std::stoul(argv[++i]));
            a.have_layer = true;
        } else if (arg == "--no-gpu") a.no_gpu = true;
        else if (arg == "--list-tensors") a.list = true;
        else if (arg == "--gpu-smoke") a.gpu_smoke = true;
        else if (arg == "--help") {
            std::cout << usage << "\n";
            std::exit(0);
        } else {
            throw std::runtime_error("unknown argument: " + arg);
        }
    }
    return a;
}

void print_dims(const q38::TensorRecord& t) {
    std::cout << "dims: [";
    for (std::uint32_t i = 0; i < t.ndim; ++i) std::cout << (i ? "," : "") << t.dims[i];
    std::cout << "]\n";
}

// One GGUF Q5_K block (176 B) rebuilt from block b of SoA planes (META20 |
// QH32 | QS128): the inverse of the reference's repack (src/quant.cpp:401-423).
std::vector<std::byte> q5k_block_from_soa(const std::byte* meta, const std::byte* qh, const std::byte* qs) {
    std::vector<std::byte> out(176);
    std::memcpy(out.data(), meta, 4);
    std::uint8_t sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = static_cast<std::uint8_t>(meta[4 + 2 * j]);
        mn[j] = static_cast<std::uint8_t>(meta[5 + 2 * j]);
    }
    std::uint8_t s[12];
    for (int j = 0; j < 4; ++j) {
        s[j] = static_cast<std::uint8_t>((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = static_cast<std::uint8_t>((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = static_cast<std::uint8_t>((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
    std::memcpy(out.data() + 4, s, 12);
    std::memcpy(out.data() + 16, qh, 32);
    std::memcpy(out.data() + 48, qs, 128);
    return out;
}

int dequant_cmd(const char* name, const char* tag, std::uint32_t type, const char* usage, int argc, char** argv,
                const char* default_tensor = nullptr) {
    Args a = parse(argc, argv, usage);
    if (a.tensor.empty() && default_tensor) a.tensor = default_tensor;
    if (a.model.empty()) {
        std::cerr << name << ": --model is required\n";
        return 2;
    }
    try {
        q38::PackFile pack;
        pack.open(a.model);
        const q38::TensorRecord* target = nullptr;
        if (!a.tensor.empty()) target = pack.find_tensor(a.tensor);
        else
            for (const auto& t : pack.tensors())
                if (t.ggml_type == type && t.stored_bytes > 0) {
                    target = &t;
                    break;
                }
        if (!target || target->ggml_type != type) {
            std::cerr << name << ": no GGML_TYPE_" << tag << " (" << type << ") tensor found\n";
            return 3;
        }
        std::cout << "Q38RT real-model " << tag << " dequant smoke\n";
        std::cout << "tensor: " << target->name << "\n";
        std::cout << "stored bytes: " << target->stored_bytes << "\n";
        print_dims(*target);
        q38::NvidiaDriver driver;
        driver.open();
        std::cout << "device: " << driver.device_name() << "\n";
        std::string error;
        double ma = 0.0, mr = 0.0;
        bool ok = false;
        const std::byte* block = pack.tensor_data(*target);
        if (type == 12) ok = driver.run_q4k_dequant_smoke(block, &error, &ma, &mr);
        else if (type == 23) ok = driver.run_iq4xs_dequant_smoke(block, &error, &ma, &mr);
        else if (target->layout == q38::TensorLayout::Sm86Q5KSoA) {
            const auto b = q5k_block_from_soa(block, pack.tensor_aux_data(*target, 0), pack.tensor_aux_data(*target, 1));
            ok = driver.run_q5k_dequant_smoke(b.data(), &error, &ma, &mr);
        } else {
            ok = driver.run_q5k_dequant_smoke(block, &error, &ma, &mr);
        }
        if (!ok) {
            std::cerr << tag << ": FAILED: " << error << "\n";
            return 4;
        }
        std::cout << std::scientific << std::setprecision(6);
        std::cout << "max_abs_error: " << ma << "\n";
        std::cout << "max_rel_error: " << mr << "\n";
        std::string lower = tag;
        for (auto& c : lower) c = static_cast<char>(std::tolower(static_cast<unsigned char>(c)));
        std::cout << lower << ": PASS\n";
        return 0;
    } catch (const std::exception& e) {
        std::cerr << name << ": " << e.what() << "\n";
        return 1;
    }
}

void print_full(const q38::Layer0FullStats& s) {
    std::cout << std::scientific << std::setprecision(6);
    std::cout << "ffn_norm_max_abs_error: " << s.ffn_norm_max_abs << "\n";
    std::cout << "ffn_gate_up_max_abs_error: " << s.ffn_gate_up_max_abs << "\n";
    std::cout << "ffn_down_max_abs_error: " << s.ffn_down_max_abs << "\n";
    std::cout << "layer_output_max_abs_error: " << s.layer_output_max_abs << "\n";
    std::cout << std::fixed << std::setprecision(4);
    std::cout << "attention_ms: " << s.attention_ms << "\n";
    std::cout << "post_norm_ms: " << s.post_norm_ms << "\n";
    std::cout << "ffn_gate_ms: " << s.ffn_gate_ms << "\n";
    std::cout << "ffn_up_ms: " << s.ffn_up_ms << "\n";
    std::cout << "ffn_pointwise_ms: " << s.ffn_pointwise_ms << "\n";
    std::cout << "ffn_down_ms: " << s.ffn_down_ms << "\n";
    std::cout << "ffn_ms: " << s.ffn_ms << "\n";
    std::cout << "sum_stage_ms: " << s.sum_stage_ms << "\n";
    std::cout << "layer_chain_ms: " << s.chain_ms << "\n";
    if (s.chain_ms > 0.0) std::cout << "layer_per_second: " << (1000.0 / s.chain_ms) << "\n";
    std::cout << "shared_workspace: yes\n";
    std::cout << "weight_upload_in_timing: no\n";
    std::cout << "module_jit_in_timing: no\n";
    std::cout << "n_tokens: 1\n";
}

template <class F>
int runtime_cmd(const char* name, const char* usage, int argc, char** argv, bool need_layer, F&& body) {
    const Args a = parse(argc, argv, usage);
    if (a.model.empty() || (need_layer && !a.have_layer)) {
        std::cerr << name << (need_layer ? ": --model and --layer are required\n" : ": --model is required\n");
        return 2;
    }
    try {
        q38::Runtime runtime;
        runtime.load(a.model, true);
        return body(runtime, a);
    } catch (const std::exception& e) {
        std::cerr << name << ": " << e.what() << "\n";
        return 1;
    }
}

}  // namespace

int main(int argc, char** argv) {
    try {
#if Q38_CMD == 1
        (void)parse(argc, argv, "usage: q38-gpu-smoke");
        q38::NvidiaDriver driver;
        driver.open();
        std::cout << "Q38RT GPU smoke\n";
        std::cout << "device: " << driver.device_name() << "\n";
        std::cout << "driver version: " << driver.driver_version() << "\n";
        std::cout << "compute capability: sm_" << driver.sm_major() << driver.sm_minor() << "\n";
        std::cout << std::fixed << std::setprecision(2)
                  << "VRAM: " << static_cast<double>(driver.total_memory()) / (1024.0 * 1024.0 * 1024.0) << " GiB\n";
        std::cout << "VMM: " << (driver.vmm_available() ? "available" : "not available");
        if (driver.vmm_available()) std::cout << " (granularity " << driver.vmm_granularity() << " bytes)";
        std::cout << "\n";
        std::string error;
        if (!driver.run_sm86_smoke(&error)) {
            std::cerr << "smoke: FAILED: " << error << "\n";
            return 2;
        }
        std::cout << "smoke: PASS (C ABI + VMM + sm_100a kernels)\n";
        return 0;
#elif Q38_CMD == 2
        (void)parse(argc, argv, "usage: q38-rmsnorm-smoke");
        q38::NvidiaDriver driver;
        driver.open();
        std::cout << "Q38RT RMSNorm smoke\n";
        std::cout << "device: " << driver.device_name() << "\n";
        std::cout << "compute capability: sm_" << driver.sm_major() << driver.sm_minor() << "\n";
        std::string error;
        double ma = 0.0, mr = 0.0;
        if (!driver.run_rmsnorm_smoke(&error, &ma, &mr)) {
            std::cerr << "rmsnorm: FAILED: " << error << "\n";
            return 2;
        }
        std::cout << std::scientific << std::setprecision(6);
        std::cout << "max_abs_error: " << ma << "\n";
        std::cout << "max_rel_error: " << mr << "\n";
        std::cout << "rmsnorm: PASS\n";
        return 0;
#elif Q38_CMD == 3
        (void)parse(argc, argv, "usage: q38-gdn-ar-smoke");
        q38::NvidiaDriver driver;
        driver.open();
        constexpr std::uint32_t state_dim = 128, qk_heads = 16, value_heads = 48;
        std::cout << "Q38RT Qwen3.8 fused Gated DeltaNet decode core\n";
        std::cout << "device: " << driver.device_name() << "\n";
        std::cout << "state_dim: " << state_dim << "\n";
        std::cout << "qk_heads: " << qk_heads << "\n";
        std::cout << "value_heads: " << value_heads << "\n";
        std::cout << "qk_broadcast: value_head_mod_qk_heads\n";
        std::cout << "state_layout: [H=48][col=128][row=128] transposed-column-major\n";
        std::cout << "kernel_mapping: grid[head,4] x block[256], state slice staged per CTA\n";
        q38::GdnArSmokeStats stats{};
        std::string error;
        if (!driver.run_gdn_ar_smoke(state_dim, qk_heads, value_heads, &stats, &error)) {
            std::cerr << "gdn_ar: FAILED: " << error << "\n";
            return 2;
        }
        std::cout << std::scientific << std::setprecision(6);
        std::cout << "output_max_abs_error: " << stats.output_max_abs << "\n";
        std::cout << "output_max_rel_error: " << stats.output_max_rel << "\n";
        std::cout << "state_max_abs_error: " << stats.state_max_abs << "\n";
        std::cout << "state_max_rel_error: " << stats.state_max_rel << "\n";
        std::cout << std::fixed << std::setprecision(4);
        std::cout << "kernel_ms: " << stats.kernel_ms << "\n";
        std::cout << "state_read_write_bandwidth_GBps: " << stats.state_bandwidth_gbps << "\n";
        std::cout << "n_tokens: 1\n";
        std::cout << "gdn_mode: GDA_scalar_gate_per_value_head\n";
        std::cout << "gdn_ar: PASS\n";
        return 0;
#elif Q38_CMD == 4
        const Args a = parse(argc, argv, "usage: q38-recurrent-prep --model MODEL.q38pack");
        if (a.model.empty()) {
            std::cerr << "q38-recurrent-prep: --model is required\n";
            return 2;
        }
        q38::PackFile pack;
        pack.open(a.model);
        const auto* conv = pack.find_tensor("blk.0.ssm_conv1d.weight");
        const auto* dt = pack.find_tensor("blk.0.ssm_dt.bias");
        const auto* A = pack.find_tensor("blk.0.ssm_a");
        if (!conv || !dt || !A) {
            std::cerr << "q38-recurrent-prep: missing recurrent F32 tensor\n";
            return 3;
        }
        if (conv->ggml_type != 0 || dt->ggml_type != 0 || A->ggml_type != 0) {
            std::cerr << "q38-recurrent-prep: recurrent prep tensors must be F32\n";
            return 4;
        }
        if (conv->ndim < 2 || conv->dims[0] != 4 || conv->dims[1] != 10240 || dt->dims[0] != 48 || A->dims[0] != 48) {
            std::cerr << "q38-recurrent-prep: unexpected tensor shape\n";
            return 5;
        }
        std::cout << "Q38RT Qwen3.8 recurrent prep\n";
        std::cout << "q38pack_version: " << pack.header().version << "\n";
        std::cout << "conv_tensor: " << conv->name << " [4,10240]\n";
        std::cout << "dt_tensor: " << dt->name << " [48]\n";
        std::cout << "a_tensor: " << A->name << " [48]\n";
        std::cout << "qkv_split: q=2048 k=2048 v=6144\n";
        std::cout << "conv_state: 3x10240 + current qkv\n";
        q38::NvidiaDriver driver;
        driver.open();
        std::cout << "device: " << driver.device_name() << "\n";
        q38::RecurrentPrepSmokeStats stats{};
        std::string error;
        if (!driver.run_recurrent_prep_smoke(reinterpret_cast<const float*>(pack.tensor_data(*conv)),
                                             reinterpret_cast<const float*>(pack.tensor_data(*dt)),
                                             reinterpret_cast<const float*>(pack.tensor_data(*A)), &stats, &error)) {
            std::cerr << "recurrent_prep: FAILED: " << error << "\n";
            return 6;
        }
        std::cout << std::scientific << std::setprecision(6);
        std::cout << "conv_max_abs_error: " << stats.conv_max_abs << "\n";
        std::cout << "q_max_abs_error: " << stats.q_max_abs << "\n";
        std::cout << "k_max_abs_error: " << stats.k_max_abs << "\n";
        std::cout << "beta_max_abs_error: " << stats.beta_max_abs << "\n";
        std::cout << "gate_max_abs_error: " << stats.gate_max_abs << "\n";
        std::cout << "conv_state_max_abs_error: " << stats.conv_state_max_abs << "\n";
        std::cout << std::fixed << std::setprecision(4);
        std::cout << "conv_silu_ms: " << stats.conv_silu_ms << "\n";
        std::cout << "qk_norm_ms: " << stats.qk_norm_ms << "\n";
        std::cout << "beta_gate_ms: " << stats.beta_gate_ms << "\n";
        std::cout << "recurrent_prep_chain_ms: " << stats.chain_ms << "\n";
        std::cout << "recurrent_prep: PASS\n";
        return 0;
#elif Q38_CMD == 5
        Args a = parse(argc, argv, "usage: q38-q5k-q8k-gemv --model MODEL.q38pack [--tensor NAME]");
        if (a.tensor.empty()) a.tensor = "blk.0.attn_gate.weight";
        if (a.model.empty()) {
            std::cerr << "q38-q5k-q8k-gemv: --model is required\n";
            return 2;
        }
        q38::PackFile pack;
        pack.open(a.model);
        const auto* t = pack.find_tensor(a.tensor);
        if (!t) {
            std::cerr << "q38-q5k-q8k-gemv: tensor not found: " << a.tensor << "\n";
            return 3;
        }
        if (t->layout != q38::TensorLayout::GgufNative) {
            std::cerr << "q38-q5k-q8k-gemv: this experiment requires GGUF_NATIVE Q5_K; "
                      << "use q38-q5k-sm86-gemv for SM86_Q5K_SOA\n";
            return 11;
        }
        if (t->ggml_type != 13) {
            std::cerr << "q38-q5k-q8k-gemv: tensor is not GGML_TYPE_Q5_K (13), type=" << t->ggml_type << "\n";
            return 4;
        }
        if (t->ndim < 2 || t->dims[0] == 0 || t->dims[1] == 0) {
            std::cerr << "q38-q5k-q8k-gemv: tensor is not a 2-D matrix\n";
            return 5;
        }
        const auto cols = static_cast<std::uint32_t>(t->dims[0]), rows = static_cast<std::uint32_t>(t->dims[1]);
        std::cout << "Q38RT Q5_K x Q8_K DP4A GEMV\n";
        std::cout << "tensor: " << t->name << "\n";
        std::cout << "shape: [" << cols << "," << rows << "]\n";
        std::cout << "stored bytes: " << t->stored_bytes << "\n";
        q38::NvidiaDriver driver;
        driver.open();
        std::cout << "device: " << driver.device_name() << "\n";
        std::string error;
        double ma = 0.0, mr = 0.0, ms = 0.0, gbps = 0.0;
        if (!driver.run_q5k_q8k_gemv_smoke(pack.tensor_data(*t), cols, rows, &error, &ma, &mr, &ms, &gbps)) {
            std::cerr << "q5_k_x_q8_k: FAILED: " << error << "\n";
            return 6;
        }
        std::cout << std::scientific << std::setprecision(6);
        std::cout << "max_abs_error_vs_q8_reference: " << ma << "\n";
        std::cout << "max_rel_error_vs_q8_reference: " << mr << "\n";
        std::cout << std::fixed << std::setprecision(4);
        std::cout << "kernel_ms: " << ms << "\n";
        std::cout << "effective_weight_bandwidth_GBps: " << gbps << "\n";
        std::cout << "activation_quantization_in_timing: no\n";
        std::cout << "kernel_mapping: x-pack limbs in shared memory, dp4a over Q5_K blocks\n";
        std::cout << "dot_instruction: dp4a.u32.s32\n";
        std::cout << "q5_k_x_q8_k: PASS\n";
        return 0;
#elif Q38_CMD == 6
        return dequant_cmd("q38-q4k-smoke", "Q4_K", 12, "usage: q38-q4k-smoke --model MODEL.q38pack", argc, argv);
#elif Q38_CMD == 7
        return dequant_cmd("q38-q5k-smoke", "Q5_K", 13, "usage: q38-q5k-smoke --model MODEL.q38pack", argc, argv);
#elif Q38_CMD == 8
        // default tensor blk.0.ffn_gate.weight (src/iq4xs_smoke.cpp:13)
        return dequant_cmd("q38-iq4xs-smoke", "IQ4_XS", 23,
                           "usage: q38-iq4xs-smoke --model MODEL.q38pack [--tensor NAME]", argc, argv,
                           "blk.0.ffn_gate.weight");
#elif Q38_CMD == 9
        return runtime_cmd("q38-layer0-projections", "usage: q38-layer0-projections --model MODEL.q38pack [--rms-eps 1e-6]",
                           argc, argv, false, [](q38::Runtime& rt, const Args& a) {
                               std::cout << "Q38RT Qwen3.8 layer0 projection pack\n";
                               std::cout << "q38pack_version: " << rt.pack().header().version << "\n";
                               std::cout << "device: " << rt.info().device_name << "\n";
                               q38::Layer0ProjectionPackStats s{};
                               std::string error;
                               if (!rt.run_layer0_projection_pack(a.rms_eps, &s, &error)) {
                                   std::cerr << "layer0_projections: FAILED: " << error << "\n";
                                   return 3;
                               }
                               std::cout << std::scientific << std::setprecision(6);
                               std::cout << "qkv_max_abs_error: " << s.qkv.max_abs << "\n";
                               std::cout << "qkv_max_rel_error: " << s.qkv.max_rel << "\n";
                               std::cout << "gate_max_abs_error: " << s.gate.max_abs << "\n";
                               std::cout << "gate_max_rel_error: " << s.gate.max_rel << "\n";
                               std::cout << "beta_max_abs_error: " << s.beta.max_abs << "\n";
                               std::cout << "alpha_max_abs_error: " << s.alpha.max_abs << "\n";
                               std::cout << std::fixed << std::setprecision(4);
                               std::cout << "rmsnorm_ms: " << s.rmsnorm_ms << "\n";
                               std::cout << "qkv_ms: " << s.qkv_ms << "\n";
                               std::cout << "gate_ms: " << s.gate_ms << "\n";
                               std::cout << "beta_ms: " << s.beta_ms << "\n";
                               std::cout << "alpha_ms: " << s.alpha_ms << "\n";
                               std::cout << "chain_ms: " << s.chain_ms << "\n";
                               std::cout << "layer0_projections: PASS\n";
                               return 0;
                           });
#elif Q38_CMD == 10
        const Args a = parse(argc, argv, "usage: q38-layer0-gate --model MODEL.q38pack [--rms-eps 1e-6]");
        if (a.model.empty()) {
            std::cerr << "q38-layer0-gate: --model is required\n";
            return 2;
        }
        q38::PackFile pack;
        pack.open(a.model);
        const auto* norm = pack.find_tensor("blk.0.attn_norm.weight");
        const auto* gate = pack.find_tensor("blk.0.attn_gate.weight");
        if (!norm || !gate) {
            std::cerr << "q38-layer0-gate: missing blk.0.attn_norm.weight or blk.0.attn_gate.weight\n";
            return 3;
        }
        if (q38::select_projection_kernel(*norm) != q38::ProjectionKernelKind::F32Direct ||
            q38::select_projection_kernel(*gate) != q38::ProjectionKernelKind::Q5KSm86Vectorized) {
            std::cerr << "q38-layer0-gate: norm must be F32 and attn_gate SM86_Q5K_SOA\n";
            return 4;
        }
        const auto cols = static_cast<std::uint32_t>(gate->dims[0]), rows = static_cast<std::uint32_t>(gate->dims[1]);
        std::cout << "Q38RT Qwen3.8 layer0 RMSNorm -> attn_gate\n";
        std::cout << "q38pack_version: " << pack.header().version << "\n";
        std::cout << "norm_tensor: " << norm->name << " [" << norm->dims[0] << "]\n";
        std::cout << "gate_tensor: " << gate->name << " [" << cols << "," << rows << "]\n";
        std::cout << "gate_layout: SM86_Q5K_SOA\n";
        std::cout << "projection_kernel: q5k_sm86_soa_gemv (2-D TMA planes, x-pack limbs)\n";
        std::cout << std::scientific << std::setprecision(6);
        std::cout << "rms_eps: " << a.rms_eps << "\n";
        q38::NvidiaDriver driver;
        driver.open();
        std::cout << "device: " << driver.device_name() << "\n";
        std::string error;
        double ma = 0, mr = 0, tn = 0, tp = 0, tc = 0, gbps = 0;
        if (!driver.run_qwen35_layer0_gate_smoke(
                reinterpret_cast<const float*>(pack.tensor_data(*norm)), pack.tensor_data(*gate),
                static_cast<std::size_t>(gate->aux0_offset - gate->data_offset),
                static_cast<std::size_t>(gate->aux1_offset - gate->data_offset), cols, rows, a.rms_eps, &error, &ma,
                &mr, &tn, &tp, &tc, &gbps)) {
            std::cerr << "layer0_gate: FAILED: " << error << "\n";
            return 5;
        }
        std::cout << std::scientific << std::setprecision(6);
        std::cout << "max_abs_error: " << ma << "\n";
        std::cout << "max_rel_error: " << mr << "\n";
        std::cout << std::fixed << std::setprecision(4);
        std::cout << "rmsnorm_ms: " << tn << "\n";
        std::cout << "attn_gate_projection_ms: " << tp << "\n";
        std::cout << "attn_gate_original_equiv_GBps: " << gbps << "\n";
        std::cout << "chain_ms: " << tc << "\n";
        if (tc > 0.0) std::cout << "chain_equiv_calls_per_second: " << (1000.0 / tc) << "\n";
        std::cout << "layer0_gate: PASS\n";
        return 0;
#elif Q38_CMD == 11
        return runtime_cmd(
            "q38-layer0-recurrent-front", "usage: q38-layer0-recurrent-front --model MODEL.q38pack [--rms-eps 1e-6]",
            argc, argv, false, [](q38::Runtime& rt, const Args& a) {
                std::cout << "Q38RT Qwen3.8 layer0 recurrent front\n";
                std::cout << "q38pack_version: " << rt.pack().header().version << "\n";
                std::cout << "device: " << rt.info().device_name << "\n";
                std::cout << "chain: RMSNorm -> qkv/z/beta/alpha -> conv4+SiLU -> q/k norm -> beta/gate -> GDN\n";
                q38::Layer0RecurrentFrontStats s{};
                std::string error;
                if (!rt.run_layer0_recurrent_front(a.rms_eps, &s, &error)) {
                    std::cerr << "layer0_recurrent_front: FAILED: " << error << "\n";
                    return 3;
                }
                std::cout << std::scientific << std::setprecision(6);
                std::cout << "conv_max_abs_error: " << s.conv_max_abs << "\n";
                std::cout << "q_max_abs_error: " << s.q_max_abs << "\n";
                std::cout << "k_max_abs_error: " << s.k_max_abs << "\n";
                std::cout << "beta_max_abs_error: " << s.beta_max_abs << "\n";
                std::cout << "gate_max_abs_error: " << s.gate_max_abs << "\n";
                std::cout << "conv_state_max_abs_error: " << s.conv_state_max_abs << "\n";
                std::cout << "gdn_output_max_abs_error: " << s.gdn_output_max_abs << "\n";
                std::cout << "gdn_output_max_rel_error: " << s.gdn_output_max_rel << "\n";
                std::cout << "gdn_state_max_abs_error: " << s.gdn_state_max_abs << "\n";
                std::cout << "gdn_state_max_rel_error: " << s.gdn_state_max_rel << "\n";
                std::cout << std::fixed << std::setprecision(4);
                std::cout << "projection_ms: " << s.projection_ms << "\n";
                std::cout << "conv_prep_ms: " << s.conv_prep_ms << "\n";
                std::cout << "gdn_ms: " << s.gdn_ms << "\n";
                std::cout << "sum_stage_ms: " << s.sum_stage_ms << "\n";
                std::cout << "front_chain_ms: " << s.chain_ms << "\n";
                std::cout << "layer0_recurrent_front: PASS\n";
                return 0;
            });
#elif Q38_CMD == 12
        return runtime_cmd(
            "q38-layer0-recurrent-attention",
            "usage: q38-layer0-recurrent-attention --model MODEL.q38pack [--rms-eps 1e-6]", argc, argv, false,
            [](q38::Runtime& rt, const Args& a) {
                std::cout << "Q38RT Qwen3.8 layer0 recurrent attention\n";
                std::cout << "q38pack_version: " << rt.pack().header().version << "\n";
                std::cout << "device: " << rt.info().device_name << "\n";
                q38::Layer0RecurrentAttentionStats s{};
                std::string error;
                if (!rt.run_layer0_recurrent_attention(a.rms_eps, &s, &error)) {
                    std::cerr << "layer0_recurrent_attention: FAILED: " << error << "\n";
                    return 3;
                }
                std::cout << std::scientific << std::setprecision(6);
                std::cout << "gated_norm_max_abs_error: " << s.gated_norm_max_abs << "\n";
                std::cout << "ssm_out_max_abs_error: " << s.ssm_out_max_abs << "\n";
                std::cout << "residual_max_abs_error: " << s.residual_max_abs << "\n";
                std::cout << std::fixed << std::setprecision(4);
                std::cout << "front_ms: " << s.front_ms << "\n";
                std::cout << "gated_norm_ms: " << s.gated_norm_ms << "\n";
                std::cout << "ssm_out_ms: " << s.ssm_out_ms << "\n";
                std::cout << "tail_ms: " << s.tail_ms << "\n";
                std::cout << "sum_stage_ms: " << s.sum_stage_ms << "\n";
                std::cout << "attention_chain_ms: " << s.chain_ms << "\n";
                std::cout << "layer0_recurrent_attention: PASS\n";
                return 0;
            });
#elif Q38_CMD == 13
        return runtime_cmd("q38-layer0-full", "usage: q38-layer0-full --model MODEL.q38pack [--rms-eps 1e-6]", argc,
                           argv, false, [](q38::Runtime& rt, const Args& a) {
                               std::cout << "Q38RT Qwen3.8 complete recurrent layer0\n";
                               std::cout << "q38pack_version: " << rt.pack().header().version << "\n";
                               std::cout << "device: " << rt.info().device_name << "\n";
                               std::cout << "attention:\n";
                               std::cout << "  RMSNorm -> qkv/z/beta/alpha -> conv/GDN\n";
                               std::cout << "  -> gated norm -> ssm_out -> residual\n";
                               std::cout << "ffn:\n";
                               std::cout << "  post_attention_norm\n";
                               std::cout << "  -> gate IQ4XS_PRMT + up Q5K_SM86_VEC\n";
                               std::cout << "  -> SiLU(gate)*up\n";
                               std::cout << "  -> down Q5K_SM86_VEC -> residual\n";
                               q38::Layer0FullStats s{};
                               std::string error;
                               if (!rt.run_layer0_full(a.rms_eps, &s, &error)) {
                                   std::cerr << "layer0_full: FAILED: " << error << "\n";
                                   return 3;
                               }
                               print_full(s);
                               std::cout << "layer0_full: PASS\n";
                               return 0;
                           });
#elif Q38_CMD == 14
        return runtime_cmd("q38-recurrent-layer",
                           "usage: q38-recurrent-layer --model MODEL.q38pack --layer N [--rms-eps 1e-6]", argc, argv,
                           true, [](q38::Runtime& rt, const Args& a) {
                               std::cout << "Q38RT Qwen3.8 recurrent layer\n";
                               std::cout << "q38pack_version: " << rt.pack().header().version << "\n";
                               std::cout << "device: " << rt.info().device_name << "\n";
                               std::cout << "layer: " << a.layer << "\n";
                               std::cout << "layer_kind: "
                                         << q38::qwen35_layer_kind_name(q38::detect_qwen35_layer_kind(rt.pack(), a.layer))
                                         << "\n";
                               q38::Layer0FullStats s{};
                               std::string error;
                               if (!rt.run_recurrent_layer(a.layer, a.rms_eps, &s, &error)) {
                                   std::cerr << "recurrent_layer: FAILED: " << error << "\n";
                                   return 3;
                               }
                               print_full(s);
                               std::cout << "recurrent_layer: PASS\n";
                               return 0;
                           });
#elif Q38_CMD == 15
        const Args a = parse(argc, argv, "usage: q38-layer-topology --model MODEL.q38pack");
        if (a.model.empty()) {
            std::cerr << "q38-layer-topology: --model is required\n";
            return 2;
        }
        q38::PackFile pack;
        pack.open(a.model);
        std::uint32_t max_layer = 0;
        bool any = false;
        for (const auto& t : pack.tensors())
            if (t.name.rfind("blk.", 0) == 0) {
                max_layer = std::max<std::uint32_t>(max_layer, static_cast<std::uint32_t>(std::stoul(t.name.substr(4))));
                any = true;
            }
        std::map<std::string, std::uint32_t> counts;
        std::cout << "Q38RT Qwen3.8 layer topology\n";
        std::cout << "q38pack_version: " << pack.header().version << "\n";
        const std::uint32_t n = any ? max_layer + 1 : 0;
        std::cout << "layers: " << n << "\n";
        for (std::uint32_t L = 0; L < n; ++L) {
            const char* k = q38::qwen35_layer_kind_name(q38::detect_qwen35_layer_kind(pack, L));
            ++counts[k];
            std::cout << "layer[" << L << "]: " << k << "\n";
        }
        for (const auto& kv : counts) std::cout << "count[" << kv.first << "]: " << kv.second << "\n";
        std::cout << "layer_topology: PASS\n";
        return 0;
#elif Q38_CMD == 16
        const Args a = parse(argc, argv,
                             "usage: q38-runtime --model MODEL.q38pack [--no-gpu] [--list-tensors] [--gpu-smoke]");
        if (a.model.empty()) {
            std::cerr << "q38-runtime: --model is required\n";
            return 2;
        }
        q38::Runtime runtime;
        runtime.load(a.model, !a.no_gpu);
        const q38::RuntimeInfo info = runtime.info();
        auto gib = [](double b) { return b / (1024.0 * 1024.0 * 1024.0); };
        std::cout << "Q38 Runtime probe\n";
        std::cout << "model: " << info.model_path << "\n";
        std::cout << "tensors: " << info.tensor_count << "\n";
        std::cout << std::fixed << std::setprecision(2) << "packed: " << gib(static_cast<double>(info.packed_bytes))
                  << " GiB\n";
        std::cout << "driver: " << (info.driver_available ? "available" : "not available") << "\n";
        if (info.driver_available) {
            std::cout << "driver version: " << info.driver_version << "\n";
            std::cout << "device: " << info.device_name << "\n";
            std::cout << "VRAM: " << gib(static_cast<double>(info.device_memory)) << " GiB\n";
            std::cout << "compute capability: sm_" << info.sm_major << info.sm_minor << "\n";
            std::cout << "VMM: " << (info.vmm_available ? "available" : "not available");
            if (info.vmm_available) std::cout << " (granularity " << info.vmm_granularity << " bytes)";
            std::cout << "\n";
        }
        std::cout << "native decode: " << (info.native_decode_ready ? "ready" : "through the q38_model_* engine")
                  << "\n";
        if (a.gpu_smoke) {
            std::string error;
            if (!runtime.gpu_smoke(&error)) {
                std::cerr << "gpu smoke: FAILED: " << error << "\n";
                return 3;
            }
            std::cout << "gpu smoke: PASS (C ABI + VMM + sm_100a kernels)\n";
        }
        if (a.list)
            for (const auto& t : runtime.pack().tensors()) {
                std::cout << t.name << " type=" << t.ggml_type << " dims=[";
                for (std::uint32_t d = 0; d < t.ndim; ++d) std::cout << (d ? "," : "") << t.dims[d];
                std::cout << "] bytes=" << t.stored_bytes
                          << " kernel=" << q38::projection_kernel_name(q38::select_projection_kernel(t)) << "\n";
            }
        return 0;
#else
#error "unknown Q38_CMD"
#endif
    } catch (const std::exception& e) {
        std::cerr << argv[0] << ": " << e.what() << "\n";
        return 1;
    }
}
