// q38-q4k-gemv, q38-q5k-gemv, q38-q6k-gemv, q38-iq4xs-gemv -- the reference's
// GEMV commands over GGUF-native K-quant tensors (src/q4k_gemv.cpp,
// src/q5k_gemv.cpp, src/q6k_gemv.cpp, src/iq4xs_gemv.cpp) in C++ over this
// library: open a Q38PACK, take one GGUF-native matrix of the command's type,
// run the matching q38::NvidiaDriver GEMV smoke on the B200 and print the
// reference's `key: value` lines and PASS line.  One source built four times,
// Q38_KQUANT naming the GGML type (12, 13, 14 or 23).
//
//   q38-<type>-gemv --model MODEL.q38pack [--tensor NAME]
//
// Exit codes follow the reference: 2 usage, 3 tensor not found, 4 wrong type
// or layout, 5 not a matrix, 6 the GEMV smoke failed, 1 anything else.
#include <cstdint>
#include <iomanip>
#include <iostream>
#include <string>

#include "../../include/q38/driver.hpp"
#include "../../include/q38rt.h"

#ifndef Q38_KQUANT
#error "build with -DQ38_KQUANT=12, 13, 14 or 23"
#endif

static_assert(Q38_KQUANT == 12 || Q38_KQUANT == 13 || Q38_KQUANT == 14 || Q38_KQUANT == 23,
              "Q38_KQUANT must be 12, 13, 14 or 23");

namespace {

struct Command {
    const char* exe;          // command name
    const char* type_name;    // GGML type name
    const char* tag;          // prefix of the PASS / FAILED lines
    const char* title;        // first output line
    const char* tensor;       // default tensor
};

constexpr Command command() {
    if constexpr (Q38_KQUANT == 12) {
        return {"q38-q4k-gemv", "Q4_K", "q4_k_gemv", "Q38RT-B200 Q4_K GEMV", "blk.0.ssm_beta.weight"};
    } else if constexpr (Q38_KQUANT == 13) {
        return {"q38-q5k-gemv", "Q5_K", "q5_k_gemv", "Q38RT-B200 Q5_K GEMV", "blk.0.attn_gate.weight"};
    } else if constexpr (Q38_KQUANT == 14) {
        return {"q38-q6k-gemv", "Q6_K", "q6_k_gemv", "Q38RT-B200 Q6_K GEMV", "blk.3.attn_v.weight"};
    } else {
        return {"q38-iq4xs-gemv", "IQ4_XS", "iq4_xs_gemv", "Q38RT-B200 IQ4_XS GEMV", "blk.0.ffn_gate.weight"};
    }
}

bool smoke(q38::NvidiaDriver& d, const std::byte* m, uint32_t cols, uint32_t rows, std::string* err, double* ma,
           double* mr, double* ms, double* gbps) {
    if constexpr (Q38_KQUANT == 12) return d.run_q4k_gemv_smoke(m, cols, rows, err, ma, mr, ms, gbps);
    else if constexpr (Q38_KQUANT == 13) return d.run_q5k_gemv_smoke(m, cols, rows, err, ma, mr, ms, gbps);
    else if constexpr (Q38_KQUANT == 14) return d.run_q6k_gemv_smoke(m, cols, rows, err, ma, mr, ms, gbps);
    else return d.run_iq4xs_gemv_smoke(m, cols, rows, err, ma, mr, ms, gbps);
}

}  // namespace

int main(int argc, char** argv) {
    constexpr Command C = command();
    std::string model, tensor_name = C.tensor;
    for (int i = 1; i < argc; ++i) {
        const std::string arg = argv[i];
        if (arg == "--model" && i + 1 < argc) {
            model = argv[++i];
        } else if (arg == "--tensor" && i + 1 < argc) {
            tensor_name = argv[++i];
        } else if (arg == "--help") {
            std::cout << "usage: " << C.exe << " --model MODEL.q38pack [--tensor NAME]\n";
            return 0;
        } else {
            std::cerr << C.exe << ": unknown argument: " << arg << "\n";
            return 2;
        }
    }
    if (model.empty()) {
        std::cerr << C.exe << ": --model is required\n";
        return 2;
    }
    q38_pack* pack = nullptr;
    if (q38_pack_open(model.c_str(), &pack) != Q38_OK) {
        std::cerr << C.exe << ": " << q38_last_error() << "\n";
        return 1;
    }
    auto quit = [&](int code, const std::string& msg) {
        std::cerr << C.exe << ": " << msg << "\n";
        q38_pack_close(pack);
        return code;
    };
    uint32_t index = 0;
    if (q38_pack_find(pack, tensor_name.c_str(), &index) != Q38_OK) return quit(3, "tensor not found: " + tensor_name);
    q38_tensor_record t{};
    const void* data = nullptr;
    if (q38_pack_tensor(pack, index, &t) != Q38_OK || q38_pack_host_data(pack, index, &data) != Q38_OK)
        return quit(1, q38_last_error());
    if (t.ggml_type != Q38_KQUANT || t.layout != Q38_LAYOUT_GGUF_NATIVE)
        return quit(4, std::string("tensor must be ") + C.type_name + "/GGUF_NATIVE, type=" +
                           std::to_string(t.ggml_type) + " layout=" + std::to_string(t.layout));
    if (t.ndim < 2 || t.dims[0] == 0 || t.dims[1] == 0) return quit(5, "tensor is not a 2-D matrix");
    const auto cols = static_cast<uint32_t>(t.dims[0]);
    const auto rows = static_cast<uint32_t>(t.dims[1]);
    std::cout << C.title << "\n";
    std::cout << "tensor: " << t.name << "\n";
    std::cout << "shape: [" << cols << "," << rows << "]\n";
    std::cout << "stored bytes: " << t.stored_bytes << "\n";
    try {
        q38::NvidiaDriver driver;
        driver.open();
        std::cout << "device: " << driver.device_name() << "\n";
        std::string error;
        double max_abs = 0, max_rel = 0, ms = 0, gbps = 0;
        if (!smoke(driver, static_cast<const std::byte*>(data), cols, rows, &error, &max_abs, &max_rel, &ms, &gbps)) {
            std::cerr << C.tag << ": FAILED: " << error << "\n";
            q38_pack_close(pack);
            return 6;
        }
        std::cout << std::scientific << std::setprecision(6);
        std::cout << "max_abs_error: " << max_abs << "\n";
        std::cout << "max_rel_error: " << max_rel << "\n";
        std::cout << std::fixed << std::setprecision(4);
        std::cout << "kernel_ms: " << ms << "\n";
        std::cout << "effective_weight_bandwidth_GBps: " << gbps << "\n";
        std::cout << C.tag << ": PASS\n";
    } catch (const std::exception& e) {
        return quit(1, e.what());
    }
    q38_pack_close(pack);
    return 0;
}
