// q38/q38pack.hpp -- the Q38PACK container reader with the interface of the
// reference's q38::PackFile (rffanlab/qwen382743090, include/q38/q38pack.hpp):
// the same constants, enums, header and tensor-record structs and methods, so
// host code written against the reference (its q38-* mains, q38::Runtime)
// compiles against this header.  Implemented in
// qwen382743090_b200/cxx/runtime.cpp over the library's mmap reader
// (q38_pack_* in include/q38rt.h), which also reads version 3 packs and the
// B200 tiled layout (TensorLayout::B200Tiled).
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <filesystem>
#include <string>
#include <string_view>
#include <vector>

namespace q38 {

inline constexpr std::array<char, 8> kPackMagic{'Q', '3', '8', 'P', 'A', 'C', 'K', '\0'};
inline constexpr std::uint32_t kPackVersion = 3;  // the reference writes 2; 3 adds layout 2
inline constexpr std::uint32_t kPackMinVersion = 1;
inline constexpr std::uint32_t kPackHeaderBytes = 256;
inline constexpr std::uint32_t kTensorEntryBytes = 256;

enum class TensorRole : std::uint32_t {
    Unknown = 0,
    TokenEmbedding = 1,
    OutputNorm = 2,
    Output = 3,
    Attention = 4,
    DeltaNet = 5,
    FeedForward = 6,
    Norm = 7,
    Mtp = 8,
};

enum class TensorLayout : std::uint32_t {
    GgufNative = 0,
    Sm86Q5KSoA = 1,
    B200Tiled = 2,  // fragment tiles of 8 rows x 2 super-blocks (Q5_K, Q4_K)
};

struct PackHeader {
    std::array<char, 8> magic{};
    std::uint32_t version{};
    std::uint32_t header_bytes{};
    std::uint32_t flags{};
    std::uint32_t tensor_count{};
    std::uint32_t alignment{};
    std::uint32_t reserved0{};
    std::uint64_t directory_offset{};
    std::uint64_t directory_bytes{};
    std::uint64_t manifest_offset{};
    std::uint64_t manifest_bytes{};
    std::uint64_t raw_gguf_meta_offset{};
    std::uint64_t raw_gguf_meta_bytes{};
    std::uint64_t data_offset{};
    std::uint64_t data_bytes{};
    std::uint64_t source_file_size{};
    std::uint64_t source_data_offset{};
};

struct TensorRecord {
    std::string name;
    std::uint32_t ndim{};
    std::uint32_t ggml_type{};
    std::array<std::uint64_t, 4> dims{};
    std::uint64_t data_offset{};
    std::uint64_t stored_bytes{};
    std::uint64_t source_offset{};
    TensorRole role{TensorRole::Unknown};
    std::uint32_t flags{};
    TensorLayout layout{TensorLayout::GgufNative};
    std::uint32_t layout_flags{};
    std::uint64_t aux0_offset{};
    std::uint64_t aux1_offset{};
};

class PackFile {
public:
    PackFile() = default;
    ~PackFile();
    PackFile(const PackFile&) = delete;
    PackFile& operator=(const PackFile&) = delete;
    PackFile(PackFile&& other) noexcept;
    PackFile& operator=(PackFile&& other) noexcept;

    // Throws std::runtime_error on a missing, truncated or malformed pack.
    void open(const std::filesystem::path& path);
    void close() noexcept;

    [[nodiscard]] bool is_open() const noexcept { return handle_ != nullptr; }
    [[nodiscard]] const PackHeader& header() const noexcept { return header_; }
    [[nodiscard]] const std::vector<TensorRecord>& tensors() const noexcept { return tensors_; }
    [[nodiscard]] std::string_view manifest_json() const noexcept { return manifest_; }
    [[nodiscard]] const TensorRecord* find_tensor(std::string_view name) const noexcept;
    // Host address of the tensor's bytes in the mapping (layout 1: the META
    // plane; tensor_aux_data(t, 0 / 1) the QH / QS planes).
    [[nodiscard]] const std::byte* tensor_data(const TensorRecord& tensor) const;
    [[nodiscard]] const std::byte* tensor_aux_data(const TensorRecord& tensor, int index) const;
    // The library's reader handle (q38_pack*), for q38_pack_plan / upload.
    [[nodiscard]] void* native_handle() const noexcept { return handle_; }

private:
    void* handle_{nullptr};
    PackHeader header_{};
    std::vector<TensorRecord> tensors_;
    std::string manifest_;
};

}  // namespace q38
