// nvidia_driver.cpp -- q38::NvidiaDriver (include/q38/driver.hpp) over the
// C ABI of include/q38rt.h.  Built by qwen382743090_b200/build.py into
// lib/libq38driver_b200.so, linked against lib/libq38rt_b200.so.
//
// The smoke methods keep the reference's behaviour (src/driver.cpp:4303-12461):
// the reference's x pattern, the first min(rows, 8) rows checked with its
// tolerance rule, mean time per launch over its iteration counts, and the same
// output pointers.  The check runs on the device (q38_check_rows: plain
// dequantisation and FP64 dots) instead of through a CPU copy of quant.cpp.
#include "../../include/q38/driver.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <functional>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/q38rt.h"
#include "facade_util.hpp"

namespace q38 {
namespace {

constexpr std::uint32_t kValuesPerBlock = 256;
constexpr double kAbsTol = 2.0e-3;  // src/driver.cpp:6955-6956
constexpr double kRelTol = 2.0e-3;

using facade::ck;
using facade::ctx_of;
using facade::DevBuf;
using facade::download;
using facade::smoke_x;
using facade::upload;

// IEEE binary16 bits -> float (exact: every half is a float).
float half_to_float(std::uint16_t h) {
    const std::uint32_t sign = static_cast<std::uint32_t>(h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u;
    std::uint32_t f;
    if (e == 0) {
        const float v = static_cast<float>(m) * 5.9604644775390625e-08f;  // m * 2^-24
        std::memcpy(&f, &v, 4);
        f |= sign;
    } else if (e == 31) {
        f = sign | 0x7f800000u | (m << 13);
    } else {
        f = sign | ((e + 112u) << 23) | (m << 13);
    }
    float out;
    std::memcpy(&out, &f, 4);
    return out;
}

struct SmokeResult {
    double max_abs = 0.0, max_rel = 0.0, ms = 0.0;
};

// Runs `launch` once, checks the first rows of y against the device FP64
// reference of `desc`, then times `iters` launches.  `what` names the kernel
// in error messages.
SmokeResult gemv_smoke(q38_ctx* ctx, const q38_weight_desc& desc, q38_devptr x, q38_devptr y, int iters,
                       const std::function<int()>& launch, const char* what) {
    ck(launch(), what);
    ck(q38_stream_synchronize(nullptr), what);
    const std::uint32_t nchk = std::min<std::uint32_t>(desc.rows, 8u);
    std::vector<float> got(nchk);
    ck(q38_memcpy_d2h(got.data(), y, nchk * sizeof(float), nullptr), "read y");
    DevBuf ref_d(ctx, nchk * sizeof(double));
    ck(q38_check_rows(&desc, nchk, x, ref_d.get(), 0, nullptr), "q38_check_rows");
    std::vector<double> ref(nchk);
    ck(q38_memcpy_d2h(ref.data(), ref_d.get(), nchk * sizeof(double), nullptr), "read reference rows");
    ck(q38_stream_synchronize(nullptr), "reference rows");
    SmokeResult r;
    bool bad = false;
    for (std::uint32_t i = 0; i < nchk; ++i) {
        const double ae = std::abs(static_cast<double>(got[i]) - ref[i]);
        const double re = ae / std::max(1.0e-5, std::abs(ref[i]));
        r.max_abs = std::max(r.max_abs, ae);
        r.max_rel = std::max(r.max_rel, re);
        if (ae > kAbsTol && re > kRelTol) bad = true;
    }
    if (bad) {
        std::ostringstream oss;
        oss << what << " mismatch: max_abs=" << r.max_abs << " max_rel=" << r.max_rel;
        throw std::runtime_error(oss.str());
    }
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < iters; ++i) ck(launch(), what);
    ck(q38_stream_synchronize(nullptr), what);
    const auto t1 = std::chrono::steady_clock::now();
    r.ms = std::chrono::duration<double, std::milli>(t1 - t0).count() / iters;
    return r;
}

// The GGUF-native GEMV smokes share one body; `bytes_per_block` and the C
// entry differ.
bool native_gemv_smoke(void* handle, std::uint32_t type, std::size_t bytes_per_block,
                       int (*entry)(q38_devptr, q38_devptr, q38_devptr, std::uint32_t, std::uint32_t, q38_stream),
                       const char* what, int iters, const std::byte* matrix, std::uint32_t cols, std::uint32_t rows,
                       std::string* error, double* max_abs_error, double* max_rel_error, double* milliseconds,
                       double* bandwidth_gbps) {
    try {
        q38_ctx* ctx = ctx_of(handle);
        if (!matrix) throw std::invalid_argument(std::string(what) + " matrix is null");
        if (cols == 0 || rows == 0 || cols % kValuesPerBlock)
            throw std::invalid_argument(std::string(what) + " requires non-zero rows and cols divisible by 256");
        const std::size_t bytes = static_cast<std::size_t>(rows) * (cols / kValuesPerBlock) * bytes_per_block;
        DevBuf w(ctx, bytes), x(ctx, cols * sizeof(float)), y(ctx, rows * sizeof(float));
        ck(q38_memcpy_h2d(w.get(), matrix, bytes, nullptr), "upload matrix");
        const std::vector<float> xs = smoke_x(cols);
        ck(q38_memcpy_h2d(x.get(), xs.data(), cols * sizeof(float), nullptr), "upload x");
        const q38_weight_desc desc{type, Q38_LAYOUT_GGUF_NATIVE, rows, cols, w.get(), 0, 0};
        const SmokeResult r = gemv_smoke(
            ctx, desc, x.get(), y.get(), iters, [&] { return entry(w.get(), x.get(), y.get(), cols, rows, nullptr); },
            what);
        if (max_abs_error) *max_abs_error = r.max_abs;
        if (max_rel_error) *max_rel_error = r.max_rel;
        if (milliseconds) *milliseconds = r.ms;
        if (bandwidth_gbps) *bandwidth_gbps = static_cast<double>(bytes) / (r.ms / 1000.0) / 1.0e9;
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}


}  // namespace

NvidiaDriver::~NvidiaDriver() { close(); }

// src/driver.cpp:4305-4372: device 0, its properties, the VMM granularity.
void NvidiaDriver::open() {
    if (available()) return;
    q38_device_info info{};
    ck(q38_device_query(0, &info), "q38_device_query");
    q38_ctx* ctx = nullptr;
    ck(q38_ctx_open(0, &ctx), "q38_ctx_open");
    handle_ = ctx;
    initialized_ = true;
    driver_version_ = info.driver_version;
    device_ordinal_ = info.ordinal;
    sm_major_ = info.sm_major;
    sm_minor_ = info.sm_minor;
    device_name_ = info.name;
    total_memory_ = info.total_memory;
    vmm_granularity_ = info.vmm_granularity;
    vmm_available_ = info.vmm_supported != 0;
}

void NvidiaDriver::close() noexcept {
    if (handle_) q38_ctx_close(static_cast<q38_ctx*>(handle_));
    handle_ = nullptr;
    initialized_ = false;
}

bool NvidiaDriver::probe_vmm(std::size_t bytes, std::string* error) {
    try {
        DevBuf b(ctx_of(handle_), bytes);
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

// A device round trip of a known pattern (values[i] = 3i + 7, as the
// reference's pattern smoke writes, src/driver.cpp:4386-4485).
bool NvidiaDriver::run_sm86_smoke(std::string* error) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        constexpr std::uint32_t n = 1024;
        std::vector<std::uint32_t> values(n), back(n, 0);
        for (std::uint32_t i = 0; i < n; ++i) values[i] = i * 3 + 7;
        DevBuf a(ctx, n * 4), b(ctx, n * 4);
        ck(q38_memcpy_h2d(a.get(), values.data(), n * 4, nullptr), "upload");
        ck(q38_memcpy_d2d(b.get(), a.get(), n * 4, nullptr), "device copy");
        ck(q38_memcpy_d2h(back.data(), b.get(), n * 4, nullptr), "download");
        ck(q38_stream_synchronize(nullptr), "synchronize");
        if (values != back) throw std::runtime_error("device round trip mismatch");
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

// RMSNorm of 5120 values, eps 1e-6, against the FP64 device reference
// q38_check_rmsnorm (the reference's smoke shape and x pattern,
// src/driver.cpp:4486-4499).
bool NvidiaDriver::run_rmsnorm_smoke(std::string* error, double* max_abs_error, double* max_rel_error) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        constexpr std::uint32_t n = 5120;
        constexpr float eps = 1.0e-6f;
        std::vector<float> x(n), w(n), y(n);
        for (std::uint32_t i = 0; i < n; ++i) {
            const float fi = static_cast<float>(i);
            x[i] = std::sin(fi * 0.013f) * 0.75f + std::cos(fi * 0.007f) * 0.25f;
            w[i] = 1.0f + 0.05f * std::sin(fi * 0.031f);
        }
        DevBuf xd(ctx, n * 4), wd(ctx, n * 4), yd(ctx, n * 4);
        ck(q38_memcpy_h2d(xd.get(), x.data(), n * 4, nullptr), "upload x");
        ck(q38_memcpy_h2d(wd.get(), w.data(), n * 4, nullptr), "upload w");
        DevBuf rd(ctx, n * 4);
        ck(q38_rmsnorm(xd.get(), wd.get(), yd.get(), n, 1, eps, nullptr), "q38_rmsnorm");
        ck(q38_check_rmsnorm(xd.get(), wd.get(), 0, 1, n, eps, rd.get(), nullptr), "q38_check_rmsnorm");
        y = download(yd.get(), n, "download y");
        const std::vector<float> ref = download(rd.get(), n, "download reference");
        const double ma = facade::max_abs_diff(y, ref), mr = facade::max_rel_diff(y, ref, 1.0e-5);
        if (max_abs_error) *max_abs_error = ma;
        if (max_rel_error) *max_rel_error = mr;
        if (ma > 1.0e-5) throw std::runtime_error("RMSNorm mismatch: max_abs=" + std::to_string(ma));
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

// src/driver.cpp:4764, :6428, :5149, :5682: GGUF-native blocks.
bool NvidiaDriver::run_q4k_gemv_smoke(const std::byte* matrix, std::uint32_t cols, std::uint32_t rows,
                                      std::string* error, double* max_abs_error, double* max_rel_error,
                                      double* milliseconds, double* bandwidth_gbps) {
    return native_gemv_smoke(handle_, Q38_TYPE_Q4_K, 144, q38_q4k_gemv_f32, "Q4_K GEMV", 1000, matrix, cols, rows,
                             error, max_abs_error, max_rel_error, milliseconds, bandwidth_gbps);
}

bool NvidiaDriver::run_q5k_gemv_smoke(const std::byte* matrix, std::uint32_t cols, std::uint32_t rows,
                                      std::string* error, double* max_abs_error, double* max_rel_error,
                                      double* milliseconds, double* bandwidth_gbps) {
    return native_gemv_smoke(handle_, Q38_TYPE_Q5_K, 176, q38_q5k_gemv_f32, "Q5_K GEMV", 50, matrix, cols, rows,
                             error, max_abs_error, max_rel_error, milliseconds, bandwidth_gbps);
}

bool NvidiaDriver::run_q6k_gemv_smoke(const std::byte* matrix, std::uint32_t cols, std::uint32_t rows,
                                      std::string* error, double* max_abs_error, double* max_rel_error,
                                      double* milliseconds, double* bandwidth_gbps) {
    return native_gemv_smoke(handle_, Q38_TYPE_Q6_K, 210, q38_q6k_gemv_f32, "Q6_K GEMV", 50, matrix, cols, rows,
                             error, max_abs_error, max_rel_error, milliseconds, bandwidth_gbps);
}

bool NvidiaDriver::run_iq4xs_gemv_smoke(const std::byte* matrix, std::uint32_t cols, std::uint32_t rows,
                                        std::string* error, double* max_abs_error, double* max_rel_error,
                                        double* milliseconds, double* bandwidth_gbps) {
    return native_gemv_smoke(handle_, Q38_TYPE_IQ4_XS, 136, q38_iq4xs_gemv_f32, "IQ4_XS GEMV", 50, matrix, cols,
                             rows, error, max_abs_error, max_rel_error, milliseconds, bandwidth_gbps);
}

// The headline entry: Q5_K SoA planes (META20 | QH32 | QS128 at the given
// offsets of one buffer), src/driver.cpp:6800-7019.
bool NvidiaDriver::run_q5k_sm86_gemv_smoke(const std::byte* repacked_matrix, std::size_t qh_offset,
                                           std::size_t qs_offset, std::uint32_t cols, std::uint32_t rows,
                                           std::string* error, double* max_abs_error, double* max_rel_error,
                                           double* milliseconds, double* original_equiv_gbps,
                                           double* physical_gbps) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        if (!is_sm86())
            throw std::runtime_error("q38 B200 Q5_K GEMV requires sm_100; detected sm_" + std::to_string(sm_major_) +
                                     std::to_string(sm_minor_));
        if (!repacked_matrix) throw std::invalid_argument("SM86 Q5_K matrix is null");
        if (cols == 0 || rows == 0 || cols % kValuesPerBlock)
            throw std::invalid_argument("SM86 Q5_K GEMV requires non-zero rows and cols divisible by 256");
        const std::size_t blocks = static_cast<std::size_t>(rows) * (cols / kValuesPerBlock);
        if (qh_offset < blocks * 20 || qs_offset < qh_offset + blocks * 32)
            throw std::invalid_argument("invalid SM86 Q5_K SoA offsets");
        const std::size_t repacked_bytes = qs_offset + blocks * 128;
        DevBuf w(ctx, repacked_bytes), x(ctx, cols * sizeof(float)), y(ctx, rows * sizeof(float));
        ck(q38_memcpy_h2d(w.get(), repacked_matrix, repacked_bytes, nullptr), "upload planes");
        const std::vector<float> xs = smoke_x(cols);
        ck(q38_memcpy_h2d(x.get(), xs.data(), cols * sizeof(float), nullptr), "upload x");
        const q38_devptr meta = w.get(), qh = w.get() + qh_offset, qs = w.get() + qs_offset;
        const q38_weight_desc desc{Q38_TYPE_Q5_K, Q38_LAYOUT_SM86_Q5K_SOA, rows, cols, meta, qh, qs};
        const SmokeResult r = gemv_smoke(
            ctx, desc, x.get(), y.get(), 50,
            [&] { return q38_q5k_sm86_soa_gemv_vec(meta, qh, qs, x.get(), y.get(), cols, rows, nullptr); },
            "SM86 Q5_K GEMV");
        if (max_abs_error) *max_abs_error = r.max_abs;
        if (max_rel_error) *max_rel_error = r.max_rel;
        if (milliseconds) *milliseconds = r.ms;
        if (original_equiv_gbps) *original_equiv_gbps = static_cast<double>(blocks * 176) / (r.ms / 1000.0) / 1.0e9;
        if (physical_gbps) *physical_gbps = static_cast<double>(repacked_bytes) / (r.ms / 1000.0) / 1.0e9;
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

namespace {

// Dequantisation smokes (src/driver.cpp:4641, :4944, :5508, :5901): the
// block's weights from the plain device dequantiser (q38_check_rows with deq,
// bit-exact to the reference's CPU dequantisers by the golden-vector tests)
// against the same weights as the fast GEMV kernel of the type sees them
// (y = W e_i for the unit vectors e_i of the 256 positions).  A weight fails
// only beyond 1e-5 absolute and relative, the reference's rule.
bool dequant_smoke(void* handle, std::uint32_t type, std::size_t block_bytes,
                   int (*entry)(q38_devptr, q38_devptr, q38_devptr, std::uint32_t, std::uint32_t, q38_stream),
                   const char* what, const std::byte* block, std::string* error, double* max_abs_error,
                   double* max_rel_error, std::uint32_t* first_bad_index) {
    try {
        q38_ctx* ctx = ctx_of(handle);
        if (!block) throw std::invalid_argument(std::string(what) + " block is null");
        DevBuf w(ctx, block_bytes + 16u), eye(ctx, kValuesPerBlock * kValuesPerBlock * sizeof(float)),
            y(ctx, kValuesPerBlock * sizeof(float)), deq(ctx, kValuesPerBlock * sizeof(float));
        upload(w.get(), block, block_bytes, "upload block");
        std::vector<float> e(kValuesPerBlock * kValuesPerBlock, 0.0f);
        for (std::uint32_t i = 0; i < kValuesPerBlock; ++i) e[i * kValuesPerBlock + i] = 1.0f;
        upload(eye.get(), e.data(), e.size() * sizeof(float), "upload unit vectors");
        const q38_weight_desc desc{type, Q38_LAYOUT_GGUF_NATIVE, 1, kValuesPerBlock, w.get(), 0, 0};
        ck(q38_check_rows(&desc, 1, 0, 0, deq.get(), nullptr), "device dequantisation");
        for (std::uint32_t i = 0; i < kValuesPerBlock; ++i)
            ck(entry(w.get(), eye.get() + i * kValuesPerBlock * sizeof(float), y.get() + i * sizeof(float),
                     kValuesPerBlock, 1, nullptr),
               what);
        const std::vector<float> ref = download(deq.get(), kValuesPerBlock, "dequantised block");
        const std::vector<float> got = download(y.get(), kValuesPerBlock, "kernel weights");
        double ma = 0.0, mr = 0.0;
        std::uint32_t bad = kValuesPerBlock;
        for (std::uint32_t i = 0; i < kValuesPerBlock; ++i) {
            const double ae = std::abs(static_cast<double>(got[i]) - static_cast<double>(ref[i]));
            const double re = ae / std::max(1.0e-6, std::abs(static_cast<double>(ref[i])));
            ma = std::max(ma, ae);
            mr = std::max(mr, re);
            if (bad == kValuesPerBlock && ae > 1.0e-5 && re > 1.0e-5) bad = i;
        }
        if (max_abs_error) *max_abs_error = ma;
        if (max_rel_error) *max_rel_error = mr;
        if (first_bad_index) *first_bad_index = bad;
        if (bad != kValuesPerBlock) {
            std::ostringstream oss;
            oss << what << " dequant mismatch: first_bad=" << bad << " max_abs=" << ma << " max_rel=" << mr;
            throw std::runtime_error(oss.str());
        }
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

}  // namespace

bool NvidiaDriver::run_q4k_dequant_smoke(const std::byte* block, std::string* error, double* max_abs_error,
                                         double* max_rel_error) {
    return dequant_smoke(handle_, Q38_TYPE_Q4_K, 144, q38_q4k_gemv_f32, "Q4_K", block, error, max_abs_error,
                         max_rel_error, nullptr);
}
bool NvidiaDriver::run_q6k_dequant_smoke(const std::byte* block, std::string* error, double* max_abs_error,
                                         double* max_rel_error, std::uint32_t* first_bad_index) {
    return dequant_smoke(handle_, Q38_TYPE_Q6_K, 210, q38_q6k_gemv_f32, "Q6_K", block, error, max_abs_error,
                         max_rel_error, first_bad_index);
}
bool NvidiaDriver::run_q5k_dequant_smoke(const std::byte* block, std::string* error, double* max_abs_error,
                                         double* max_rel_error) {
    return dequant_smoke(handle_, Q38_TYPE_Q5_K, 176, q38_q5k_gemv_f32, "Q5_K", block, error, max_abs_error,
                         max_rel_error, nullptr);
}
bool NvidiaDriver::run_iq4xs_dequant_smoke(const std::byte* block, std::string* error, double* max_abs_error,
                                           double* max_rel_error) {
    return dequant_smoke(handle_, Q38_TYPE_IQ4_XS, 136, q38_iq4xs_gemv_f32, "IQ4_XS", block, error, max_abs_error,
                         max_rel_error, nullptr);
}

// Q5_K weights with Q8_K activations (src/driver.cpp:6610-6798): x of the
// smoke pattern quantised to Q8_K on the device (q38_quantize_q8k, the
// reference's quantize_q8_k_cpu bit for bit), the dp4a GEMV, and the first
// rows against FP64 dots of the dequantised weights with the dequantised
// Q8_K values (d * q, dequantize_q8_k_block_cpu); both errors must stay
// within 2e-3.
bool NvidiaDriver::run_q5k_q8k_gemv_smoke(const std::byte* matrix, std::uint32_t cols, std::uint32_t rows,
                                          std::string* error, double* max_abs_error, double* max_rel_error,
                                          double* milliseconds, double* bandwidth_gbps) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        if (!matrix) throw std::invalid_argument("Q5_K x Q8_K matrix is null");
        if (cols == 0 || rows == 0 || cols % kValuesPerBlock)
            throw std::invalid_argument("Q5_K x Q8_K GEMV requires non-zero rows and cols divisible by 256");
        const std::uint32_t nb = cols / kValuesPerBlock;
        const std::size_t bytes = static_cast<std::size_t>(rows) * nb * 176u;
        DevBuf w(ctx, bytes), x(ctx, cols * sizeof(float)), xq(ctx, nb * 292u), xd(ctx, cols * sizeof(float)),
            y(ctx, rows * sizeof(float));
        upload(w.get(), matrix, bytes, "upload matrix");
        const std::vector<float> xs = smoke_x(cols);
        upload(x.get(), xs.data(), cols * sizeof(float), "upload x");
        ck(q38_quantize_q8k(x.get(), cols, xq.get(), nullptr), "q38_quantize_q8k");
        std::vector<std::uint8_t> q8(nb * 292u);
        ck(q38_memcpy_d2h(q8.data(), xq.get(), q8.size(), nullptr), "read Q8_K blocks");
        ck(q38_stream_synchronize(nullptr), "read Q8_K blocks");
        std::vector<float> xdq(cols);
        for (std::uint32_t b = 0; b < nb; ++b) {
            float d;
            std::memcpy(&d, q8.data() + b * 292u, 4);
            for (std::uint32_t i = 0; i < kValuesPerBlock; ++i)
                xdq[b * kValuesPerBlock + i] = d * static_cast<float>(static_cast<std::int8_t>(q8[b * 292u + 4u + i]));
        }
        upload(xd.get(), xdq.data(), cols * sizeof(float), "upload dequantised x");
        const q38_weight_desc desc{Q38_TYPE_Q5_K, Q38_LAYOUT_GGUF_NATIVE, rows, cols, w.get(), 0, 0};
        const SmokeResult r = gemv_smoke(
            ctx, desc, xd.get(), y.get(), 50,
            [&] { return q38_q5k_q8k_dp4a_gemv(w.get(), xq.get(), y.get(), cols, rows, nullptr); }, "Q5_K x Q8_K GEMV");
        if (max_abs_error) *max_abs_error = r.max_abs;
        if (max_rel_error) *max_rel_error = r.max_rel;
        if (milliseconds) *milliseconds = r.ms;
        if (bandwidth_gbps) *bandwidth_gbps = static_cast<double>(bytes) / (r.ms / 1000.0) / 1.0e9;
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}
// IQ4_XS in the reference's SoA planes (src/driver.cpp:5868-6090; planes D
// [2 B] | SCALES [8 x int8 ls - 32] | QS [128 B] per block, the repack of
// src/quant.cpp:505-534).  The B200 runtime reads IQ4_XS as GGUF blocks, so
// the planes are folded back into 136-byte blocks once on upload (the
// inverse repack: ls = scale + 32 split into scales_l nibbles and scales_h
// bit pairs) and the GGUF-block kernel runs; the timing covers the kernel
// only, physical_gbps counts the planes' bytes.
bool NvidiaDriver::run_iq4xs_sm86_gemv_smoke(const std::byte* repacked_matrix, std::size_t scale_offset,
                                             std::size_t qs_offset, std::uint32_t cols, std::uint32_t rows,
                                             std::string* error, double* max_abs_error, double* max_rel_error,
                                             double* milliseconds, double* original_equiv_gbps,
                                             double* physical_gbps) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        if (!repacked_matrix) throw std::invalid_argument("SM86 IQ4_XS matrix is null");
        if (cols == 0 || rows == 0 || cols % kValuesPerBlock)
            throw std::invalid_argument("SM86 IQ4_XS GEMV requires non-zero rows and cols divisible by 256");
        const std::size_t blocks = static_cast<std::size_t>(rows) * (cols / kValuesPerBlock);
        if (scale_offset < blocks * 2 || qs_offset < scale_offset + blocks * 8)
            throw std::invalid_argument("invalid SM86 IQ4_XS plane offsets");
        std::vector<std::uint8_t> gguf(blocks * 136u);
        const auto* src = reinterpret_cast<const std::uint8_t*>(repacked_matrix);
        for (std::size_t b = 0; b < blocks; ++b) {
            std::uint8_t* o = gguf.data() + b * 136u;
            std::memcpy(o, src + b * 2u, 2);
            std::uint16_t sh = 0;
            std::uint8_t sl[4] = {0, 0, 0, 0};
            for (int g = 0; g < 8; ++g) {
                const int ls = static_cast<int>(static_cast<std::int8_t>(src[scale_offset + b * 8u + g])) + 32;
                sl[g / 2] = static_cast<std::uint8_t>(sl[g / 2] | ((ls & 15) << (4 * (g % 2))));
                sh = static_cast<std::uint16_t>(sh | (((ls >> 4) & 3) << (2 * g)));
            }
            std::memcpy(o + 2, &sh, 2);
            std::memcpy(o + 4, sl, 4);
            std::memcpy(o + 8, src + qs_offset + b * 128u, 128);
        }
        DevBuf w(ctx, gguf.size() + 16u), x(ctx, cols * sizeof(float)), y(ctx, rows * sizeof(float));
        upload(w.get(), gguf.data(), gguf.size(), "upload blocks");
        const std::vector<float> xs = smoke_x(cols);
        upload(x.get(), xs.data(), cols * sizeof(float), "upload x");
        const q38_weight_desc desc{Q38_TYPE_IQ4_XS, Q38_LAYOUT_GGUF_NATIVE, rows, cols, w.get(), 0, 0};
        const SmokeResult r = gemv_smoke(
            ctx, desc, x.get(), y.get(), 50,
            [&] { return q38_iq4xs_gemv_f32(w.get(), x.get(), y.get(), cols, rows, nullptr); }, "SM86 IQ4_XS GEMV");
        if (max_abs_error) *max_abs_error = r.max_abs;
        if (max_rel_error) *max_rel_error = r.max_rel;
        if (milliseconds) *milliseconds = r.ms;
        if (original_equiv_gbps) *original_equiv_gbps = static_cast<double>(blocks * 136u) / (r.ms / 1000.0) / 1.0e9;
        if (physical_gbps)
            *physical_gbps = static_cast<double>(qs_offset + blocks * 128u) / (r.ms / 1000.0) / 1.0e9;
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

// IQ4_XS weights with Q8_1 activations (src/driver.cpp:2641-2875 and its
// smoke): x of the smoke pattern quantised to Q8_1 on the device
// (q38_quantize_q8_1, bit-exact to quantize_q8_1_cpu), the IQ4_XS x Q8_1
// GEMV, and the first rows against FP64 dots of the dequantised weights with
// the dequantised Q8_1 values (d * q); both errors within 3e-3.
bool NvidiaDriver::run_iq4xs_q8_1_gemv_smoke(const std::byte* matrix, std::uint32_t cols, std::uint32_t rows,
                                             std::string* error, double* max_abs_error, double* max_rel_error,
                                             double* milliseconds, double* bandwidth_gbps) {
    try {
        q38_ctx* ctx = ctx_of(handle_);
        if (!matrix) throw std::invalid_argument("IQ4_XS x Q8_1 matrix is null");
        if (cols == 0 || rows == 0 || cols % kValuesPerBlock)
            throw std::invalid_argument("IQ4_XS x Q8_1 GEMV requires non-zero rows and cols divisible by 256");
        const std::size_t bytes = static_cast<std::size_t>(rows) * (cols / kValuesPerBlock) * 136u;
        const std::uint32_t nq = cols / 32u;
        DevBuf w(ctx, bytes + 16u), x(ctx, cols * sizeof(float)), xq(ctx, nq * 36u), xd(ctx, cols * sizeof(float)),
            y(ctx, rows * sizeof(float));
        upload(w.get(), matrix, bytes, "upload matrix");
        const std::vector<float> xs = smoke_x(cols);
        upload(x.get(), xs.data(), cols * sizeof(float), "upload x");
        ck(q38_quantize_q8_1(x.get(), cols, xq.get(), nullptr), "q38_quantize_q8_1");
        std::vector<std::uint8_t> q8(nq * 36u);
        ck(q38_memcpy_d2h(q8.data(), xq.get(), q8.size(), nullptr), "read Q8_1 blocks");
        ck(q38_stream_synchronize(nullptr), "read Q8_1 blocks");
        // dequantize_q8_1_block_cpu: the fp16 d widened exactly, times q in float
        std::vector<float> xdq(cols);
        for (std::uint32_t b = 0; b < nq; ++b) {
            std::uint16_t h = 0;
            std::memcpy(&h, q8.data() + b * 36u, 2);
            const float d = half_to_float(h);
            for (std::uint32_t i = 0; i < 32u; ++i)
                xdq[b * 32u + i] = d * static_cast<float>(static_cast<std::int8_t>(q8[b * 36u + 4u + i]));
        }
        upload(xd.get(), xdq.data(), cols * sizeof(float), "upload dequantised x");
        const q38_weight_desc desc{Q38_TYPE_IQ4_XS, Q38_LAYOUT_GGUF_NATIVE, rows, cols, w.get(), 0, 0};
        const SmokeResult r = gemv_smoke(
            ctx, desc, xd.get(), y.get(), 50,
            [&] { return q38_iq4xs_q8_1_gemv(w.get(), xq.get(), y.get(), cols, rows, nullptr); }, "IQ4_XS x Q8_1 GEMV");
        if (r.max_abs > 3.0e-3 || r.max_rel > 3.0e-3) throw std::runtime_error("IQ4_XS x Q8_1 mismatch");
        if (max_abs_error) *max_abs_error = r.max_abs;
        if (max_rel_error) *max_rel_error = r.max_rel;
        if (milliseconds) *milliseconds = r.ms;
        if (bandwidth_gbps) *bandwidth_gbps = static_cast<double>(bytes) / (r.ms / 1000.0) / 1.0e9;
        return true;
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

}  // namespace q38
