// facade_util.hpp -- helpers shared by the sources of libq38driver_b200.so
// (the q38::NvidiaDriver / q38::Runtime facade over include/q38rt.h).
#pragma once

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/q38rt.h"

namespace q38 {
namespace facade {

// Throws with the library's last error when a C entry fails.
inline void ck(int rc, const char* what) {
    if (rc != Q38_OK) throw std::runtime_error(std::string(what) + ": " + q38_last_error());
}

inline q38_ctx* ctx_of(void* handle) {
    if (!handle) throw std::runtime_error("driver is not initialized");
    return static_cast<q38_ctx*>(handle);
}

// Device buffer from q38_alloc (VMM), freed on scope exit.
class DevBuf {
public:
    DevBuf() = default;
    DevBuf(q38_ctx* ctx, std::size_t bytes) : ctx_(ctx) { ck(q38_alloc(ctx, bytes ? bytes : 1, &ptr_), "q38_alloc"); }
    ~DevBuf() {
        if (ptr_) q38_free(ctx_, ptr_);
    }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : ctx_(o.ctx_), ptr_(o.ptr_) { o.ptr_ = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        if (this != &o) {
            if (ptr_) q38_free(ctx_, ptr_);
            ctx_ = o.ctx_;
            ptr_ = o.ptr_;
            o.ptr_ = 0;
        }
        return *this;
    }
    q38_devptr get() const { return ptr_; }

private:
    q38_ctx* ctx_ = nullptr;
    q38_devptr ptr_ = 0;
};

inline void upload(q38_devptr dst, const void* src, std::size_t bytes, const char* what) {
    ck(q38_memcpy_h2d(dst, src, bytes, nullptr), what);
}

inline std::vector<float> download(q38_devptr src, std::size_t n, const char* what) {
    std::vector<float> v(n);
    ck(q38_memcpy_d2h(v.data(), src, n * sizeof(float), nullptr), what);
    ck(q38_stream_synchronize(nullptr), what);
    return v;
}

inline std::vector<double> download64(q38_devptr src, std::size_t n, const char* what) {
    std::vector<double> v(n);
    ck(q38_memcpy_d2h(v.data(), src, n * sizeof(double), nullptr), what);
    ck(q38_stream_synchronize(nullptr), what);
    return v;
}

// max |a - b| over two equally long vectors.
inline double max_abs_diff(const std::vector<float>& a, const std::vector<float>& b) {
    double m = 0.0;
    for (std::size_t i = 0; i < a.size() && i < b.size(); ++i)
        m = std::max(m, std::abs(static_cast<double>(a[i]) - static_cast<double>(b[i])));
    return m;
}

// max |a - b| / max(floor, |b|).
inline double max_rel_diff(const std::vector<float>& a, const std::vector<float>& b, double floor) {
    double m = 0.0;
    for (std::size_t i = 0; i < a.size() && i < b.size(); ++i) {
        const double e = std::abs(static_cast<double>(a[i]) - static_cast<double>(b[i]));
        m = std::max(m, e / std::max(floor, std::abs(static_cast<double>(b[i]))));
    }
    return m;
}

// Mean wall time of `iters` launches of fn on the default stream, with a
// synchronisation after the last (the reference's bench lambdas).
template <class F>
double bench_ms(int iters, F&& fn, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < iters; ++i) fn();
    ck(q38_stream_synchronize(nullptr), what);
    const auto t1 = std::chrono::steady_clock::now();
    return std::chrono::duration<double, std::milli>(t1 - t0).count() / static_cast<double>(iters);
}

// The activations of the reference's GEMV smokes and its decode-layer input
// (src/driver.cpp:4817-4821, :7321-7326).
inline std::vector<float> smoke_x(std::uint32_t cols) {
    std::vector<float> x(cols);
    for (std::uint32_t i = 0; i < cols; ++i) {
        const float fi = static_cast<float>(i);
        x[i] = std::sin(fi * 0.017f) * 0.65f + std::cos(fi * 0.011f) * 0.35f;
    }
    return x;
}

}  // namespace facade
}  // namespace q38
