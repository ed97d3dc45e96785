// ref_shim.cpp -- C entry points around the reference's own CPU quant code.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together
// with src/quant.cpp taken unmodified from the reference tree, into
// oracle/_ref/libq38ref.so.  Tests use it to pin the C restatement in
// oracle/q38_oracle.c and to generate tests/golden/; bench.py uses it as the
// timed CPU baseline ("kind": "reference").  Nothing in the product loads it.
//
// The GEMV helpers reproduce the reference's correctness check, i.e.
// dequantize_*_block_cpu followed by an FP64 dot per row
// (src/driver.cpp:6946-6965 for the SoA layout, :5338-5359 for Q6_K,
// :6739-6755 for Q8_K activations), with the rows split across threads.
#include "q38/quant.hpp"

#include <array>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

using Block = std::array<float, q38::kQ4KValuesPerBlock>;

bool dequant_any(int type, const std::byte* b, Block& out) {
    switch (type) {
    case 12: q38::dequantize_q4_k_block_cpu(b, out); return true;
    case 13: q38::dequantize_q5_k_block_cpu(b, out); return true;
    case 14: q38::dequantize_q6_k_block_cpu(b, out); return true;
    case 15: q38::dequantize_q8_k_block_cpu(b, out); return true;
    case 23: q38::dequantize_iq4_xs_block_cpu(b, out); return true;
    case 1013: q38::dequantize_q5_k_sm86_block_cpu(b, out); return true;
    default: return false;
    }
}

std::size_t block_bytes(int type) {
    switch (type) {
    case 12: return q38::kQ4KBytesPerBlock;
    case 13: return q38::kQ5KBytesPerBlock;
    case 14: return q38::kQ6KBytesPerBlock;
    case 15: return q38::kQ8KBytesPerBlock;
    case 23: return q38::kIQ4XSBytesPerBlock;
    case 1013: return q38::kQ5KSm86BytesPerBlock;
    default: return 0;
    }
}

template <class RowFn>
void split_rows(std::size_t rows, int threads, RowFn fn) {
    if (threads < 1) threads = 1;
    if (static_cast<std::size_t>(threads) > rows) threads = static_cast<int>(rows);
    if (threads <= 1) {
        fn(std::size_t{0}, rows);
        return;
    }
    std::vector<std::thread> pool;
    for (int i = 0; i < threads; ++i) {
        const std::size_t r0 = rows * i / threads, r1 = rows * (i + 1) / threads;
        pool.emplace_back([=] { fn(r0, r1); });
    }
    for (auto& t : pool) t.join();
}

} // namespace

extern "C" {

float q38ref_fp16_to_fp32(std::uint16_t h) { return q38::fp16_to_fp32(h); }
std::uint16_t q38ref_fp32_to_fp16(float f) { return q38::fp32_to_fp16(f); }

// type: GGML id (12, 13, 14, 15 = Q8_K, 23) or 1013 for the 180-B SoA record.
int q38ref_dequant(int type, const std::uint8_t* block, float* out) {
    Block tmp{};
    if (!dequant_any(type, reinterpret_cast<const std::byte*>(block), tmp)) return -1;
    std::memcpy(out, tmp.data(), sizeof(float) * tmp.size());
    return 0;
}

int q38ref_repack_q5k_soa(const std::uint8_t* src176, std::uint8_t* dst180) {
    q38::repack_q5_k_sm86_block(reinterpret_cast<const std::byte*>(src176),
                                reinterpret_cast<std::byte*>(dst180));
    return 0;
}

int q38ref_quantize_q8k(const float* x, std::size_t n, std::uint8_t* out) {
    try {
        const auto v = q38::quantize_q8_k_cpu(x, n);
        std::memcpy(out, v.data(), v.size());
        return 0;
    } catch (...) {
        return -1;
    }
}

int q38ref_quantize_q8_1(const float* x, std::size_t n, std::uint8_t* out) {
    try {
        const auto v = q38::quantize_q8_1_cpu(x, n);
        std::memcpy(out, v.data(), v.size());
        return 0;
    } catch (...) {
        return -1;
    }
}

// y[t*rows + r] = sum_k W[r][k] * x[t*cols + k] in FP64, W given as
// row-major GGUF blocks of `type`.
int q38ref_gemv(int type, const std::uint8_t* w, const float* x, std::size_t rows,
                std::size_t cols, std::size_t batch, double* y, int threads) {
    const std::size_t bb = block_bytes(type);
    if (!bb || type == 15 || type == 1013 || cols % 256 || !w || !x || !y) return -1;
    if (batch == 0) batch = 1;
    const std::size_t nb = cols / 256;
    split_rows(rows, threads, [&](std::size_t r0, std::size_t r1) {
        Block deq{};
        for (std::size_t r = r0; r < r1; ++r) {
            for (std::size_t t = 0; t < batch; ++t) y[t * rows + r] = 0.0;
            for (std::size_t ib = 0; ib < nb; ++ib) {
                dequant_any(type, reinterpret_cast<const std::byte*>(w + (r * nb + ib) * bb), deq);
                for (std::size_t t = 0; t < batch; ++t) {
                    const float* xv = x + t * cols + ib * 256;
                    double acc = 0.0;
                    for (std::size_t j = 0; j < 256; ++j)
                        acc += static_cast<double>(deq[j]) * static_cast<double>(xv[j]);
                    y[t * rows + r] += acc;
                }
            }
        }
    });
    return 0;
}

// Same over the Q5_K SoA planes (META20 / QH32 / QS128), assembling the
// 180-B logical record exactly as src/driver.cpp:6946-6960 does.
int q38ref_gemv_q5k_soa(const std::uint8_t* meta, const std::uint8_t* qh, const std::uint8_t* qs,
                        const float* x, std::size_t rows, std::size_t cols, std::size_t batch,
                        double* y, int threads) {
    if (cols % 256 || !meta || !qh || !qs || !x || !y) return -1;
    if (batch == 0) batch = 1;
    const std::size_t nb = cols / 256;
    split_rows(rows, threads, [&](std::size_t r0, std::size_t r1) {
        Block deq{};
        std::array<std::byte, q38::kQ5KSm86BytesPerBlock> rec{};
        for (std::size_t r = r0; r < r1; ++r) {
            for (std::size_t t = 0; t < batch; ++t) y[t * rows + r] = 0.0;
            for (std::size_t ib = 0; ib < nb; ++ib) {
                const std::size_t bi = r * nb + ib;
                std::memcpy(rec.data(), meta + bi * 20, 20);
                std::memcpy(rec.data() + 20, qh + bi * 32, 32);
                std::memcpy(rec.data() + 52, qs + bi * 128, 128);
                q38::dequantize_q5_k_sm86_block_cpu(rec.data(), deq);
                for (std::size_t t = 0; t < batch; ++t) {
                    const float* xv = x + t * cols + ib * 256;
                    double acc = 0.0;
                    for (std::size_t j = 0; j < 256; ++j)
                        acc += static_cast<double>(deq[j]) * static_cast<double>(xv[j]);
                    y[t * rows + r] += acc;
                }
            }
        }
    });
    return 0;
}

// Weights of `type` times Q8_K activations: both dequantised, FP64 dot.
int q38ref_gemv_q8k(int type, const std::uint8_t* w, const std::uint8_t* xq8, std::size_t rows,
                    std::size_t cols, std::size_t batch, double* y, int threads) {
    const std::size_t bb = block_bytes(type);
    if (!bb || type == 15 || type == 1013 || cols % 256 || !w || !xq8 || !y) return -1;
    if (batch == 0) batch = 1;
    const std::size_t nb = cols / 256;
    split_rows(rows, threads, [&](std::size_t r0, std::size_t r1) {
        Block deq{}, xd{};
        for (std::size_t r = r0; r < r1; ++r) {
            for (std::size_t t = 0; t < batch; ++t) y[t * rows + r] = 0.0;
            for (std::size_t ib = 0; ib < nb; ++ib) {
                dequant_any(type, reinterpret_cast<const std::byte*>(w + (r * nb + ib) * bb), deq);
                for (std::size_t t = 0; t < batch; ++t) {
                    q38::dequantize_q8_k_block_cpu(
                        reinterpret_cast<const std::byte*>(xq8 + (t * nb + ib) * 292), xd);
                    double acc = 0.0;
                    for (std::size_t j = 0; j < 256; ++j)
                        acc += static_cast<double>(deq[j]) * static_cast<double>(xd[j]);
                    y[t * rows + r] += acc;
                }
            }
        }
    });
    return 0;
}

} // extern "C"
