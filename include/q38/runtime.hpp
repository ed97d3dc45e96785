// q38/runtime.hpp -- model runtime with the interface of the reference's
// q38::Runtime (rffanlab/qwen382743090, include/q38/runtime.hpp): a Q38PACK
// opened through q38::PackFile, the projection-kernel dispatch contract
// select_projection_kernel, and the layer chains of q38::NvidiaDriver run on a
// pack's real tensors.  Implemented in qwen382743090_b200/cxx/runtime.cpp.
//
// Dispatch (the reference's table, src/runtime.cpp:42-64, plus the B200
// layout): F32 GGUF -> F32Direct, Q4_K GGUF -> Q4KNative, Q5_K SoA ->
// Q5KSm86Vectorized, Q6_K GGUF -> Q6KNative, IQ4_XS GGUF -> IQ4XSPrmt, and
// Q5_K / Q4_K in layout 2 -> Q5KB200Tiled / Q4KB200Tiled (the tensor-core
// kernels); anything else is Unsupported.
#pragma once

#include <filesystem>
#include <string>
#include <vector>

#include "q38/driver.hpp"
#include "q38/q38pack.hpp"

namespace q38 {

enum class Qwen35LayerKind {
    Missing = 0,
    Recurrent,
    FullAttention,
};

const char* qwen35_layer_kind_name(Qwen35LayerKind kind) noexcept;
Qwen35LayerKind detect_qwen35_layer_kind(const PackFile& pack, std::uint32_t layer) noexcept;

enum class ProjectionKernelKind {
    Unsupported = 0,
    F32Direct,
    Q4KNative,
    Q5KSm86Vectorized,
    Q6KNative,
    IQ4XSPrmt,
    Q5KB200Tiled,
    Q4KB200Tiled,
};

const char* projection_kernel_name(ProjectionKernelKind kind) noexcept;
ProjectionKernelKind select_projection_kernel(const TensorRecord& tensor) noexcept;

struct RuntimeInfo {
    std::string model_path;
    std::uint32_t tensor_count{};
    std::uint64_t packed_bytes{};
    bool driver_available{};
    int driver_version{};
    std::string device_name;
    std::size_t device_memory{};
    int sm_major{};
    int sm_minor{};
    bool vmm_available{};
    std::size_t vmm_granularity{};
    bool native_decode_ready{};
};

class Runtime {
public:
    void load(const std::filesystem::path& model_path, bool require_gpu = true);
    [[nodiscard]] RuntimeInfo info() const;
    [[nodiscard]] const PackFile& pack() const noexcept { return pack_; }
    bool gpu_smoke(std::string* error = nullptr) { return driver_.run_sm86_smoke(error); }
    bool run_layer0_projection_pack(float rms_eps = 1.0e-6f, Layer0ProjectionPackStats* stats = nullptr,
                                    std::string* error = nullptr);
    bool run_layer0_recurrent_front(float rms_eps = 1.0e-6f, Layer0RecurrentFrontStats* stats = nullptr,
                                    std::string* error = nullptr);
    bool run_layer0_recurrent_attention(float rms_eps = 1.0e-6f, Layer0RecurrentAttentionStats* stats = nullptr,
                                        std::string* error = nullptr);
    bool run_layer0_full(float rms_eps = 1.0e-6f, Layer0FullStats* stats = nullptr, std::string* error = nullptr);
    bool run_recurrent_layer(std::uint32_t layer, float rms_eps = 1.0e-6f, Layer0FullStats* stats = nullptr,
                             std::string* error = nullptr);

private:
    std::filesystem::path model_path_;
    PackFile pack_;
    NvidiaDriver driver_;
    bool native_decode_ready_{false};
};

}  // namespace q38
