// q38-q5k-sm86-gemv -- the reference's command of that name (src/q5k_sm86_gemv.cpp)
// in C++ over this library: open a Q38PACK, take one Q5_K matrix (persisted in
// the SoA layout, or GGUF blocks repacked to it here), run
// q38::NvidiaDriver::run_q5k_sm86_gemv_smoke on the B200 and print the same
// `key: value` lines and PASS line.
//
//   q38-q5k-sm86-gemv --model MODEL.q38pack [--tensor NAME]
//
// Exit codes follow the reference: 2 usage, 3 tensor not found, 4 not Q5_K,
// 5 not a matrix, 6 cols not a multiple of 256, 7 short native payload,
// 8 the GEMV smoke failed, 9 the repack changed decoded weights, 10 a layout
// this command does not take, 1 anything else.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <iomanip>
#include <iostream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/q38/driver.hpp"
#include "../../include/q38rt.h"

namespace {

void ck(int rc, const char* what) {
    if (rc != Q38_OK) throw std::runtime_error(std::string(what) + ": " + q38_last_error());
}

std::size_t align_up(std::size_t v, std::size_t a) { return (v + a - 1) / a * a; }

// The six-bit scale and min of group j from a K-quant header (get_scale_min_k4,
// src/quant.cpp:89-97).
void scale_min(int j, const std::uint8_t* s, std::uint8_t* sc, std::uint8_t* mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = static_cast<std::uint8_t>((s[j + 4] & 15) | ((s[j - 4] >> 6) << 4));
        *mn = static_cast<std::uint8_t>((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

// GGUF Q5_K blocks (176 B) into the SoA planes META20 | QH32 | QS128, each
// plane 128-byte aligned, as the reference's command builds them in memory
// (src/q5k_sm86_gemv.cpp:101-124; the record of src/quant.cpp:401-423).
std::vector<std::uint8_t> repack_soa(const std::uint8_t* src, std::size_t blocks, std::size_t* qh_off,
                                     std::size_t* qs_off) {
    *qh_off = align_up(blocks * 20, 128);
    *qs_off = align_up(*qh_off + blocks * 32, 128);
    std::vector<std::uint8_t> out(*qs_off + blocks * 128, 0);
    for (std::size_t b = 0; b < blocks; ++b) {
        const std::uint8_t* blk = src + b * 176;
        std::uint8_t* meta = out.data() + b * 20;
        std::memcpy(meta, blk, 4);
        for (int g = 0; g < 8; ++g) scale_min(g, blk + 4, meta + 4 + 2 * g, meta + 5 + 2 * g);
        std::memcpy(out.data() + *qh_off + b * 32, blk + 16, 32);
        std::memcpy(out.data() + *qs_off + b * 128, blk + 48, 128);
    }
    return out;
}

// Largest |difference| between the dequantised weights of the first rows of
// the native blocks and of their SoA repack, both dequantised on the device
// by q38_check_rows (the reference compares the two CPU dequantisations of
// the first 64 blocks, src/q5k_sm86_gemv.cpp:126-142).
double repack_decode_error(const std::uint8_t* native, const std::vector<std::uint8_t>& soa, std::size_t qh_off,
                           std::size_t qs_off, std::uint32_t cols, std::uint32_t rows) {
    q38_ctx* ctx = nullptr;
    ck(q38_ctx_open(0, &ctx), "q38_ctx_open");
    const std::uint32_t bpr = cols / 256u;
    const std::uint32_t nrows = std::min<std::uint32_t>(rows, (64u + bpr - 1u) / bpr);
    const std::size_t nb = static_cast<std::size_t>(nrows) * bpr;
    q38_devptr dn = 0, ds = 0, o1 = 0, o2 = 0;
    double worst = 0.0;
    try {
        ck(q38_alloc(ctx, nb * 176, &dn), "q38_alloc");
        ck(q38_alloc(ctx, soa.size(), &ds), "q38_alloc");
        ck(q38_alloc(ctx, nb * 256 * 4, &o1), "q38_alloc");
        ck(q38_alloc(ctx, nb * 256 * 4, &o2), "q38_alloc");
        ck(q38_memcpy_h2d(dn, native, nb * 176, nullptr), "upload native blocks");
        ck(q38_memcpy_h2d(ds, soa.data(), soa.size(), nullptr), "upload SoA planes");
        const q38_weight_desc wn{Q38_TYPE_Q5_K, Q38_LAYOUT_GGUF_NATIVE, rows, cols, dn, 0, 0};
        const q38_weight_desc ws{Q38_TYPE_Q5_K, Q38_LAYOUT_SM86_Q5K_SOA, rows, cols, ds, ds + qh_off, ds + qs_off};
        ck(q38_check_rows(&wn, nrows, 0, 0, o1, nullptr), "dequantise native");
        ck(q38_check_rows(&ws, nrows, 0, 0, o2, nullptr), "dequantise SoA");
        std::vector<float> a(nb * 256), b(nb * 256);
        ck(q38_memcpy_d2h(a.data(), o1, a.size() * 4, nullptr), "download");
        ck(q38_memcpy_d2h(b.data(), o2, b.size() * 4, nullptr), "download");
        ck(q38_stream_synchronize(nullptr), "synchronize");
        for (std::size_t i = 0; i < a.size(); ++i)
            worst = std::max(worst, std::abs(static_cast<double>(a[i]) - static_cast<double>(b[i])));
    } catch (...) {
        for (q38_devptr p : {dn, ds, o1, o2})
            if (p) q38_free(ctx, p);
        q38_ctx_close(ctx);
        throw;
    }
    for (q38_devptr p : {dn, ds, o1, o2}) q38_free(ctx, p);
    q38_ctx_close(ctx);
    return worst;
}

}  // namespace

int main(int argc, char** argv) {
    std::string model, tensor_name = "blk.0.attn_gate.weight";
    for (int i = 1; i < argc; ++i) {
        const std::string arg = argv[i];
        if (arg == "--model" && i + 1 < argc) {
            model = argv[++i];
        } else if (arg == "--tensor" && i + 1 < argc) {
            tensor_name = argv[++i];
        } else if (arg == "--help") {
            std::cout << "usage: q38-q5k-sm86-gemv --model MODEL.q38pack [--tensor NAME]\n";
            return 0;
        } else {
            std::cerr << "q38-q5k-sm86-gemv: unknown argument: " << arg << "\n";
            return 2;
        }
    }
    if (model.empty()) {
        std::cerr << "q38-q5k-sm86-gemv: --model is required\n";
        return 2;
    }
    q38_pack* pack = nullptr;
    try {
        ck(q38_pack_open(model.c_str(), &pack), "q38_pack_open");
        q38_pack_header_info hdr{};
        ck(q38_pack_header(pack, &hdr), "q38_pack_header");
        std::uint32_t index = 0;
        if (q38_pack_find(pack, tensor_name.c_str(), &index) != Q38_OK) {
            std::cerr << "q38-q5k-sm86-gemv: tensor not found: " << tensor_name << "\n";
            q38_pack_close(pack);
            return 3;
        }
        q38_tensor_record t{};
        ck(q38_pack_tensor(pack, index, &t), "q38_pack_tensor");
        auto quit = [&](int code, const std::string& msg) {
            std::cerr << "q38-q5k-sm86-gemv: " << msg << "\n";
            q38_pack_close(pack);
            return code;
        };
        if (t.ggml_type != Q38_TYPE_Q5_K)
            return quit(4, "tensor is not GGML_TYPE_Q5_K (13), type=" + std::to_string(t.ggml_type));
        if (t.ndim < 2 || t.dims[0] == 0 || t.dims[1] == 0) return quit(5, "tensor is not a 2-D matrix");
        const auto cols = static_cast<std::uint32_t>(t.dims[0]);
        const auto rows = static_cast<std::uint32_t>(t.dims[1]);
        if (cols % 256u) return quit(6, "cols must be divisible by 256");
        const std::size_t blocks = static_cast<std::size_t>(rows) * (cols / 256u);
        const std::size_t original_bytes = blocks * 176;
        const void* data = nullptr;
        ck(q38_pack_host_data(pack, index, &data), "q38_pack_host_data");
        const auto* bytes = static_cast<const std::uint8_t*>(data);

        std::vector<std::uint8_t> repacked;
        const std::uint8_t* planes = nullptr;
        std::size_t qh_off = 0, qs_off = 0, repacked_bytes = 0;
        double repack_ms = 0.0, repack_err = 0.0;
        const bool persisted = t.layout == Q38_LAYOUT_SM86_Q5K_SOA;
        if (persisted) {
            planes = bytes;
            qh_off = static_cast<std::size_t>(t.aux0_offset - t.data_offset);
            qs_off = static_cast<std::size_t>(t.aux1_offset - t.data_offset);
            repacked_bytes = static_cast<std::size_t>(t.stored_bytes);
        } else if (t.layout == Q38_LAYOUT_GGUF_NATIVE) {
            if (t.stored_bytes < original_bytes)
                return quit(7, "native tensor storage is smaller than expected Q5_K payload");
            const auto t0 = std::chrono::steady_clock::now();
            repacked = repack_soa(bytes, blocks, &qh_off, &qs_off);
            repack_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
            repack_err = repack_decode_error(bytes, repacked, qh_off, qs_off, cols, rows);
            if (repack_err != 0.0) {
                std::ostringstream msg;
                msg << "repack changed decoded weights, max_abs=" << repack_err;
                return quit(9, msg.str());
            }
            planes = repacked.data();
            repacked_bytes = repacked.size();
        } else {
            return quit(10, "unsupported tensor layout " + std::to_string(t.layout));
        }

        std::cout << "Q38RT B200 Q5_K SoA GEMV\n";
        std::cout << "q38pack_version: " << hdr.version << "\n";
        std::cout << "source_layout: " << (persisted ? "persisted_v2" : "temporary_from_native") << "\n";
        std::cout << "tensor: " << t.name << "\n";
        std::cout << "shape: [" << cols << "," << rows << "]\n";
        std::cout << "original_Q5K_bytes: " << original_bytes << "\n";
        std::cout << "repacked_bytes: " << repacked_bytes << "\n";
        std::cout << std::fixed << std::setprecision(3);
        std::cout << "repack_size_overhead_percent: "
                  << 100.0 * (static_cast<double>(repacked_bytes) - static_cast<double>(original_bytes)) /
                         static_cast<double>(original_bytes)
                  << "\n";
        std::cout << "offline_repack_ms: " << repack_ms << "\n";
        if (persisted) {
            std::cout << "repack_decode_max_abs_error: persisted_at_conversion\n";
        } else {
            std::cout << std::scientific << std::setprecision(6) << "repack_decode_max_abs_error: " << repack_err
                      << "\n" << std::fixed << std::setprecision(3);
        }
        std::cout << "layout: META20_SOA + QH32_SOA + QS128_SOA\n";

        q38::NvidiaDriver driver;
        driver.open();
        std::cout << "device: " << driver.device_name() << "\n";
        std::string error;
        double max_abs = 0, max_rel = 0, ms = 0, orig_gbps = 0, phys_gbps = 0;
        if (!driver.run_q5k_sm86_gemv_smoke(reinterpret_cast<const std::byte*>(planes), qh_off, qs_off, cols, rows,
                                            &error, &max_abs, &max_rel, &ms, &orig_gbps, &phys_gbps)) {
            std::cerr << "q5_k_sm86: FAILED: " << error << "\n";
            q38_pack_close(pack);
            return 8;
        }
        std::cout << std::scientific << std::setprecision(6);
        std::cout << "max_abs_error: " << max_abs << "\n";
        std::cout << "max_rel_error: " << max_rel << "\n";
        std::cout << std::fixed << std::setprecision(4);
        std::cout << "kernel_ms: " << ms << "\n";
        std::cout << "original_equiv_weight_bandwidth_GBps: " << orig_gbps << "\n";
        std::cout << "physical_repacked_bandwidth_GBps: " << phys_gbps << "\n";
        std::cout << "q5_k_sm86: PASS\n";
        q38_pack_close(pack);
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "q38-q5k-sm86-gemv: " << e.what() << "\n";
        if (pack) q38_pack_close(pack);
        return 1;
    }
}
