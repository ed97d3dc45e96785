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

namespace q38 {
namespace {

constexpr std::uint32_t kValuesPerBlock = 256;
constexpr double kAbsTol = 2.0e-3;  // src/driver.cpp:6955-6956
constexpr double kRelTol = 2.0e-3;

void ck(int rc, const char* what) {
    if (rc != Q38_OK) throw std::runtime_error(std::string(what) + ": " + q38_last_error());
}

q38_ctx* ctx_of(void* handle) {
    if (!handle) throw std::runtime_error("driver is not initialized");
    return static_cast<q38_ctx*>(handle);
}

// Device buffer from q38_alloc (VMM), freed on scope exit.
class DevBuf {
public:
    DevBuf(q38_ctx* ctx, std::size_t bytes) : ctx_(ctx) { ck(q38_alloc(ctx, bytes ? bytes : 1, &ptr_), "q38_alloc"); }
    ~DevBuf() {
        if (ptr_) q38_free(ctx_, ptr_);
    }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    q38_devptr get() const { return ptr_; }

private:
    q38_ctx* ctx_;
    q38_devptr ptr_ = 0;
};

// The activations of the reference's GEMV smokes (src/driver.cpp:4817-4821).
std::vector<float> smoke_x(std::uint32_t cols) {
    std::vector<float> x(cols);
    for (std::uint32_t i = 0; i < cols; ++i) {
        const float fi = static_cast<float>(i);
        x[i] = std::sin(fi * 0.017f) * 0.65f + std::cos(fi * 0.011f) * 0.35f;
    }
    return x;
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

bool not_provided(std::string* error, const char* method, const char* instead) {
    if (error) *error = std::string(method) + " is not provided by the B200 facade; use " + instead;
    return false;
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

// RMSNorm of 5120 values, eps 1e-6, against an FP64 host reference (the
// reference's smoke shape and x pattern, src/driver.cpp:4486-4499).
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
        ck(q38_rmsnorm(xd.get(), wd.get(), yd.get(), n, 1, eps, nullptr), "q38_rmsnorm");
        ck(q38_memcpy_d2h(y.data(), yd.get(), n * 4, nullptr), "download y");
        ck(q38_stream_synchronize(nullptr), "synchronize");
        double ss = 0.0;
        for (float v : x) ss += static_cast<double>(v) * v;
        const double inv = 1.0 / std::sqrt(ss / n + static_cast<double>(eps));
        double ma = 0.0, mr = 0.0;
        for (std::uint32_t i = 0; i < n; ++i) {
            const double ref = static_cast<double>(x[i]) * inv * static_cast<double>(w[i]);
            const double ae = std::abs(static_cast<double>(y[i]) - ref);
            ma = std::max(ma, ae);
            mr = std::max(mr, ae / std::max(1.0e-5, std::abs(ref)));
        }
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

bool NvidiaDriver::run_q4k_dequant_smoke(const std::byte*, std::string* error, double*, double*) {
    return not_provided(error, "run_q4k_dequant_smoke", "q38_check_rows (deq) or run_q4k_gemv_smoke");
}
bool NvidiaDriver::run_q6k_dequant_smoke(const std::byte*, std::string* error, double*, double*, std::uint32_t*) {
    return not_provided(error, "run_q6k_dequant_smoke", "q38_check_rows (deq) or run_q6k_gemv_smoke");
}
bool NvidiaDriver::run_q5k_dequant_smoke(const std::byte*, std::string* error, double*, double*) {
    return not_provided(error, "run_q5k_dequant_smoke", "q38_check_rows (deq) or run_q5k_gemv_smoke");
}
bool NvidiaDriver::run_iq4xs_dequant_smoke(const std::byte*, std::string* error, double*, double*) {
    return not_provided(error, "run_iq4xs_dequant_smoke", "q38_check_rows (deq) or run_iq4xs_gemv_smoke");
}
bool NvidiaDriver::run_iq4xs_sm86_gemv_smoke(const std::byte*, std::size_t, std::size_t, std::uint32_t,
                                             std::uint32_t, std::string* error, double*, double*, double*, double*,
                                             double*) {
    return not_provided(error, "run_iq4xs_sm86_gemv_smoke", "run_iq4xs_gemv_smoke (q38_iq4xs_gemv_f32)");
}
bool NvidiaDriver::run_iq4xs_q8_1_gemv_smoke(const std::byte*, std::uint32_t, std::uint32_t, std::string* error,
                                             double*, double*, double*, double*) {
    return not_provided(error, "run_iq4xs_q8_1_gemv_smoke", "run_iq4xs_gemv_smoke (the Q8_1 path was rejected)");
}
bool NvidiaDriver::run_q5k_q8k_gemv_smoke(const std::byte*, std::uint32_t, std::uint32_t, std::string* error,
                                          double*, double*, double*, double*) {
    return not_provided(error, "run_q5k_q8k_gemv_smoke", "q38_q5k_q8k_dp4a_gemv or q38_gemv_q8k");
}
bool NvidiaDriver::run_qwen35_layer0_full(const float*, const std::byte*, std::size_t, std::size_t,
                                          const std::byte*, std::size_t, std::size_t, const std::byte*,
                                          const std::byte*, const float*, const float*, const float*, const float*,
                                          const std::byte*, std::size_t, std::size_t, const float*,
                                          const std::byte*, const std::byte*, std::size_t, std::size_t,
                                          const std::byte*, std::size_t, std::size_t, float, Layer0FullStats*,
                                          std::string* error) {
    return not_provided(error, "run_qwen35_layer0_full", "the q38_* layer entries or q38_model_layer");
}
bool NvidiaDriver::run_qwen35_layer0_recurrent_attention(const float*, const std::byte*, std::size_t, std::size_t,
                                                         const std::byte*, std::size_t, std::size_t,
                                                         const std::byte*, const std::byte*, const float*,
                                                         const float*, const float*, const float*,
                                                         const std::byte*, std::size_t, std::size_t, float,
                                                         Layer0RecurrentAttentionStats*, std::string* error) {
    return not_provided(error, "run_qwen35_layer0_recurrent_attention", "the q38_* layer entries or q38_gdn_fused");
}
bool NvidiaDriver::run_qwen35_layer0_recurrent_front(const float*, const std::byte*, std::size_t, std::size_t,
                                                     const std::byte*, std::size_t, std::size_t, const std::byte*,
                                                     const std::byte*, const float*, const float*, const float*,
                                                     float, Layer0RecurrentFrontStats*, std::string* error) {
    return not_provided(error, "run_qwen35_layer0_recurrent_front", "the q38_* layer entries or q38_gdn_fused");
}
bool NvidiaDriver::run_recurrent_prep_smoke(const float*, const float*, const float*, RecurrentPrepSmokeStats*,
                                            std::string* error) {
    return not_provided(error, "run_recurrent_prep_smoke", "q38_conv4_silu_roll, q38_qk_l2norm, q38_beta_gate");
}
bool NvidiaDriver::run_gdn_ar_smoke(std::uint32_t, std::uint32_t, std::uint32_t, GdnArSmokeStats*,
                                    std::string* error) {
    return not_provided(error, "run_gdn_ar_smoke", "q38_gdn_step");
}
bool NvidiaDriver::run_qwen35_layer0_projection_pack(const float*, const std::byte*, std::size_t, std::size_t,
                                                     std::uint32_t, const std::byte*, std::size_t, std::size_t,
                                                     std::uint32_t, const std::byte*, const std::byte*,
                                                     std::uint32_t, std::uint32_t, float,
                                                     Layer0ProjectionPackStats*, std::string* error) {
    return not_provided(error, "run_qwen35_layer0_projection_pack", "q38_rmsnorm + q38_gemv_f32");
}
bool NvidiaDriver::run_qwen35_layer0_gate_smoke(const float*, const std::byte*, std::size_t, std::size_t,
                                                std::uint32_t, std::uint32_t, float, std::string* error, double*,
                                                double*, double*, double*, double*, double*) {
    return not_provided(error, "run_qwen35_layer0_gate_smoke", "q38_rmsnorm + q38_q5k_sm86_soa_gemv_vec");
}

}  // namespace q38
