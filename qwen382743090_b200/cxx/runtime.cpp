// runtime.cpp -- q38::PackFile (include/q38/q38pack.hpp) over the library's
// Q38PACK reader and q38::Runtime (include/q38/runtime.hpp) over PackFile and
// q38::NvidiaDriver, with the reference's dispatch contract and tensor
// requirements (src/runtime.cpp:1-620).
#include "../../include/q38/runtime.hpp"

#include <cstring>
#include <fstream>
#include <stdexcept>

#include "../../include/q38rt.h"

namespace q38 {

// ---- PackFile -----------------------------------------------------------------
PackFile::~PackFile() { close(); }

PackFile::PackFile(PackFile&& o) noexcept
    : handle_(o.handle_), header_(o.header_), tensors_(std::move(o.tensors_)), manifest_(std::move(o.manifest_)) {
    o.handle_ = nullptr;
}

PackFile& PackFile::operator=(PackFile&& o) noexcept {
    if (this != &o) {
        close();
        handle_ = o.handle_;
        header_ = o.header_;
        tensors_ = std::move(o.tensors_);
        manifest_ = std::move(o.manifest_);
        o.handle_ = nullptr;
    }
    return *this;
}

void PackFile::open(const std::filesystem::path& path) {
    close();
    q38_pack* p = nullptr;
    if (q38_pack_open(path.c_str(), &p) != Q38_OK)
        throw std::runtime_error("Q38PACK open failed: " + std::string(q38_last_error()));
    handle_ = p;
    q38_pack_header_info h{};
    if (q38_pack_header(p, &h) != Q38_OK) {
        close();
        throw std::runtime_error("Q38PACK header: " + std::string(q38_last_error()));
    }
    header_ = PackHeader{};
    header_.magic = kPackMagic;
    header_.version = h.version;
    header_.header_bytes = h.header_bytes;
    header_.flags = h.flags;
    header_.tensor_count = h.tensor_count;
    header_.alignment = h.alignment;
    header_.directory_offset = h.directory_offset;
    header_.directory_bytes = h.directory_bytes;
    header_.manifest_offset = h.manifest_offset;
    header_.manifest_bytes = h.manifest_bytes;
    header_.raw_gguf_meta_offset = h.raw_gguf_meta_offset;
    header_.raw_gguf_meta_bytes = h.raw_gguf_meta_bytes;
    header_.data_offset = h.data_offset;
    header_.data_bytes = h.data_bytes;
    header_.source_file_size = h.source_file_size;
    header_.source_data_offset = h.source_data_offset;
    tensors_.clear();
    tensors_.reserve(h.tensor_count);
    for (std::uint32_t i = 0; i < h.tensor_count; ++i) {
        q38_tensor_record r{};
        if (q38_pack_tensor(p, i, &r) != Q38_OK) {
            close();
            throw std::runtime_error("Q38PACK tensor record: " + std::string(q38_last_error()));
        }
        TensorRecord t;
        t.name = r.name;
        t.ndim = r.ndim;
        t.ggml_type = r.ggml_type;
        for (int d = 0; d < 4; ++d) t.dims[d] = r.dims[d];
        t.data_offset = r.data_offset;
        t.stored_bytes = r.stored_bytes;
        t.source_offset = r.source_offset;
        t.role = static_cast<TensorRole>(r.role);
        t.flags = r.flags;
        t.layout = static_cast<TensorLayout>(r.layout);
        t.layout_flags = r.layout_flags;
        t.aux0_offset = r.aux0_offset;
        t.aux1_offset = r.aux1_offset;
        tensors_.push_back(std::move(t));
    }
    manifest_.clear();
    if (h.manifest_bytes) {
        std::ifstream f(path, std::ios::binary);
        manifest_.resize(h.manifest_bytes);
        f.seekg(static_cast<std::streamoff>(h.manifest_offset));
        if (!f.read(manifest_.data(), static_cast<std::streamsize>(h.manifest_bytes))) {
            close();
            throw std::runtime_error("Q38PACK manifest is truncated");
        }
    }
}

void PackFile::close() noexcept {
    if (handle_) q38_pack_close(static_cast<q38_pack*>(handle_));
    handle_ = nullptr;
    tensors_.clear();
    manifest_.clear();
}

const TensorRecord* PackFile::find_tensor(std::string_view name) const noexcept {
    for (const auto& t : tensors_)
        if (t.name == name) return &t;
    return nullptr;
}

const std::byte* PackFile::tensor_data(const TensorRecord& tensor) const {
    if (!handle_) throw std::runtime_error("Q38PACK is not open");
    if (tensors_.empty() || &tensor < tensors_.data() || &tensor >= tensors_.data() + tensors_.size())
        throw std::invalid_argument("tensor record does not belong to this pack");
    const void* p = nullptr;
    const auto index = static_cast<std::uint32_t>(&tensor - tensors_.data());
    if (q38_pack_host_data(static_cast<const q38_pack*>(handle_), index, &p) != Q38_OK)
        throw std::runtime_error("Q38PACK tensor data: " + std::string(q38_last_error()));
    return static_cast<const std::byte*>(p);
}

const std::byte* PackFile::tensor_aux_data(const TensorRecord& tensor, int index) const {
    if (tensor.layout != TensorLayout::Sm86Q5KSoA || (index != 0 && index != 1))
        throw std::invalid_argument("only SM86 Q5_K SoA tensors have aux planes 0 and 1");
    const std::uint64_t off = index == 0 ? tensor.aux0_offset : tensor.aux1_offset;
    return tensor_data(tensor) + (off - tensor.data_offset);
}

// ---- dispatch -------------------------------------------------------------------
const char* qwen35_layer_kind_name(Qwen35LayerKind kind) noexcept {
    switch (kind) {
        case Qwen35LayerKind::Recurrent: return "RECURRENT";
        case Qwen35LayerKind::FullAttention: return "FULL_ATTENTION";
        default: return "MISSING";
    }
}

Qwen35LayerKind detect_qwen35_layer_kind(const PackFile& pack, std::uint32_t layer) noexcept {
    const std::string p = "blk." + std::to_string(layer) + ".";
    if (pack.find_tensor(p + "ssm_conv1d.weight")) return Qwen35LayerKind::Recurrent;
    if (pack.find_tensor(p + "attn_q.weight") || pack.find_tensor(p + "attn_k.weight") ||
        pack.find_tensor(p + "attn_v.weight") || pack.find_tensor(p + "attn_output.weight"))
        return Qwen35LayerKind::FullAttention;
    return Qwen35LayerKind::Missing;
}

const char* projection_kernel_name(ProjectionKernelKind kind) noexcept {
    switch (kind) {
        case ProjectionKernelKind::F32Direct: return "F32_DIRECT";
        case ProjectionKernelKind::Q4KNative: return "Q4K_NATIVE";
        case ProjectionKernelKind::Q5KSm86Vectorized: return "Q5K_SM86_VEC";
        case ProjectionKernelKind::Q6KNative: return "Q6K_NATIVE_VEC";
        case ProjectionKernelKind::IQ4XSPrmt: return "IQ4XS_PRMT";
        case ProjectionKernelKind::Q5KB200Tiled: return "Q5K_B200_TILED";
        case ProjectionKernelKind::Q4KB200Tiled: return "Q4K_B200_TILED";
        default: return "UNSUPPORTED";
    }
}

ProjectionKernelKind select_projection_kernel(const TensorRecord& t) noexcept {
    const bool gguf = t.layout == TensorLayout::GgufNative;
    if (t.ggml_type == Q38_TYPE_F32 && gguf) return ProjectionKernelKind::F32Direct;
    if (t.ggml_type == Q38_TYPE_Q4_K && gguf) return ProjectionKernelKind::Q4KNative;
    if (t.ggml_type == Q38_TYPE_Q5_K && t.layout == TensorLayout::Sm86Q5KSoA)
        return ProjectionKernelKind::Q5KSm86Vectorized;
    if (t.ggml_type == Q38_TYPE_Q6_K && gguf) return ProjectionKernelKind::Q6KNative;
    if (t.ggml_type == Q38_TYPE_IQ4_XS && gguf) return ProjectionKernelKind::IQ4XSPrmt;
    if (t.ggml_type == Q38_TYPE_Q5_K && t.layout == TensorLayout::B200Tiled) return ProjectionKernelKind::Q5KB200Tiled;
    if (t.ggml_type == Q38_TYPE_Q4_K && t.layout == TensorLayout::B200Tiled) return ProjectionKernelKind::Q4KB200Tiled;
    return ProjectionKernelKind::Unsupported;
}

// ---- Runtime ----------------------------------------------------------------------
void Runtime::load(const std::filesystem::path& model_path, bool require_gpu) {
    model_path_ = model_path;
    pack_.open(model_path);
    if (require_gpu) {
        driver_.open();
    } else {
        try {
            driver_.open();
        } catch (...) {
        }
    }
    native_decode_ready_ = false;  // decode runs through the q38_model_* engine, not this pack path
}

RuntimeInfo Runtime::info() const {
    RuntimeInfo r;
    r.model_path = model_path_.string();
    r.tensor_count = static_cast<std::uint32_t>(pack_.tensors().size());
    for (const auto& t : pack_.tensors()) r.packed_bytes += t.stored_bytes;
    r.driver_available = driver_.available();
    r.driver_version = driver_.driver_version();
    r.device_name = driver_.device_name();
    r.device_memory = driver_.total_memory();
    r.sm_major = driver_.sm_major();
    r.sm_minor = driver_.sm_minor();
    r.vmm_available = driver_.vmm_available();
    r.vmm_granularity = driver_.vmm_granularity();
    r.native_decode_ready = native_decode_ready_;
    return r;
}

namespace {

// The tensors of one recurrent layer, checked against the reference's
// dispatch and shape requirements (src/runtime.cpp:368-460).
struct LayerTensors {
    const TensorRecord *norm{}, *qkv{}, *z{}, *beta{}, *alpha{}, *conv{}, *dt{}, *a{}, *ssm_norm{}, *ssm_out{},
        *post_norm{}, *ffn_gate{}, *ffn_up{}, *ffn_down{};
};

enum class Part { Projections, Front, Attention, Full };

LayerTensors layer_tensors(const PackFile& pack, std::uint32_t layer, Part part) {
    const std::string p = "blk." + std::to_string(layer) + ".";
    auto req = [&](const char* s) -> const TensorRecord* {
        const TensorRecord* t = pack.find_tensor(p + s);
        if (!t) throw std::runtime_error("missing tensor: " + p + s);
        return t;
    };
    auto kind = [](const TensorRecord* t, ProjectionKernelKind k) {
        if (select_projection_kernel(*t) != k)
            throw std::runtime_error(t->name + " must use " + projection_kernel_name(k) + " (has " +
                                     projection_kernel_name(select_projection_kernel(*t)) + ")");
    };
    auto dims = [](const TensorRecord* t, std::uint64_t d0, std::uint64_t d1) {
        if (t->dims[0] != d0 || (d1 && t->dims[1] != d1))
            throw std::runtime_error(t->name + " has an unexpected shape for the hidden-5120 layer");
    };
    LayerTensors L;
    L.norm = req("attn_norm.weight");
    L.qkv = req("attn_qkv.weight");
    L.z = req("attn_gate.weight");
    L.beta = req("ssm_beta.weight");
    L.alpha = req("ssm_alpha.weight");
    kind(L.norm, ProjectionKernelKind::F32Direct);
    kind(L.qkv, ProjectionKernelKind::Q5KSm86Vectorized);
    kind(L.z, ProjectionKernelKind::Q5KSm86Vectorized);
    kind(L.beta, ProjectionKernelKind::Q4KNative);
    kind(L.alpha, ProjectionKernelKind::Q4KNative);
    if (part == Part::Projections) return L;
    dims(L.norm, 5120, 0);
    dims(L.qkv, 5120, 10240);
    dims(L.z, 5120, 6144);
    dims(L.beta, 5120, 48);
    dims(L.alpha, 5120, 48);
    L.conv = req("ssm_conv1d.weight");
    L.dt = req("ssm_dt.bias");
    L.a = req("ssm_a");
    for (const TensorRecord* t : {L.conv, L.dt, L.a}) kind(t, ProjectionKernelKind::F32Direct);
    dims(L.conv, 4, 10240);
    dims(L.dt, 48, 0);
    dims(L.a, 48, 0);
    if (part == Part::Front) return L;
    L.ssm_norm = req("ssm_norm.weight");
    L.ssm_out = req("ssm_out.weight");
    kind(L.ssm_norm, ProjectionKernelKind::F32Direct);
    kind(L.ssm_out, ProjectionKernelKind::Q5KSm86Vectorized);
    dims(L.ssm_norm, 128, 0);
    dims(L.ssm_out, 6144, 5120);
    if (part == Part::Attention) return L;
    L.post_norm = req("post_attention_norm.weight");
    L.ffn_gate = req("ffn_gate.weight");
    L.ffn_up = req("ffn_up.weight");
    L.ffn_down = req("ffn_down.weight");
    kind(L.post_norm, ProjectionKernelKind::F32Direct);
    kind(L.ffn_gate, ProjectionKernelKind::IQ4XSPrmt);
    kind(L.ffn_up, ProjectionKernelKind::Q5KSm86Vectorized);
    kind(L.ffn_down, ProjectionKernelKind::Q5KSm86Vectorized);
    dims(L.post_norm, 5120, 0);
    dims(L.ffn_gate, 5120, 17408);
    dims(L.ffn_up, 5120, 17408);
    dims(L.ffn_down, 17408, 5120);
    return L;
}

std::size_t qh_off(const TensorRecord* t) { return static_cast<std::size_t>(t->aux0_offset - t->data_offset); }
std::size_t qs_off(const TensorRecord* t) { return static_cast<std::size_t>(t->aux1_offset - t->data_offset); }
const float* f32(const PackFile& p, const TensorRecord* t) { return reinterpret_cast<const float*>(p.tensor_data(*t)); }

}  // namespace

bool Runtime::run_layer0_projection_pack(float rms_eps, Layer0ProjectionPackStats* stats, std::string* error) {
    try {
        if (!driver_.available()) throw std::runtime_error("layer0 projection pack requires an initialized GPU driver");
        const LayerTensors L = layer_tensors(pack_, 0, Part::Projections);
        const auto cols = static_cast<std::uint32_t>(L.norm->dims[0]);
        if (L.qkv->dims[0] != cols || L.z->dims[0] != cols || L.beta->dims[0] != cols || L.alpha->dims[0] != cols)
            throw std::runtime_error("layer0 projection pack input dimensions do not match");
        if (L.beta->dims[1] != L.alpha->dims[1]) throw std::runtime_error("layer0 alpha/beta output dimensions do not match");
        return driver_.run_qwen35_layer0_projection_pack(
            f32(pack_, L.norm), pack_.tensor_data(*L.qkv), qh_off(L.qkv), qs_off(L.qkv),
            static_cast<std::uint32_t>(L.qkv->dims[1]), pack_.tensor_data(*L.z), qh_off(L.z), qs_off(L.z),
            static_cast<std::uint32_t>(L.z->dims[1]), pack_.tensor_data(*L.beta), pack_.tensor_data(*L.alpha), cols,
            static_cast<std::uint32_t>(L.beta->dims[1]), rms_eps, stats, error);
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

bool Runtime::run_layer0_recurrent_front(float rms_eps, Layer0RecurrentFrontStats* stats, std::string* error) {
    try {
        if (!driver_.available()) throw std::runtime_error("layer0 recurrent front requires an initialized GPU driver");
        const LayerTensors L = layer_tensors(pack_, 0, Part::Front);
        return driver_.run_qwen35_layer0_recurrent_front(
            f32(pack_, L.norm), pack_.tensor_data(*L.qkv), qh_off(L.qkv), qs_off(L.qkv), pack_.tensor_data(*L.z),
            qh_off(L.z), qs_off(L.z), pack_.tensor_data(*L.beta), pack_.tensor_data(*L.alpha), f32(pack_, L.conv),
            f32(pack_, L.dt), f32(pack_, L.a), rms_eps, stats, error);
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

bool Runtime::run_layer0_recurrent_attention(float rms_eps, Layer0RecurrentAttentionStats* stats,
                                             std::string* error) {
    try {
        if (!driver_.available())
            throw std::runtime_error("layer0 recurrent attention requires an initialized GPU driver");
        const LayerTensors L = layer_tensors(pack_, 0, Part::Attention);
        return driver_.run_qwen35_layer0_recurrent_attention(
            f32(pack_, L.norm), pack_.tensor_data(*L.qkv), qh_off(L.qkv), qs_off(L.qkv), pack_.tensor_data(*L.z),
            qh_off(L.z), qs_off(L.z), pack_.tensor_data(*L.beta), pack_.tensor_data(*L.alpha), f32(pack_, L.conv),
            f32(pack_, L.dt), f32(pack_, L.a), f32(pack_, L.ssm_norm), pack_.tensor_data(*L.ssm_out), qh_off(L.ssm_out),
            qs_off(L.ssm_out), rms_eps, stats, error);
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

bool Runtime::run_layer0_full(float rms_eps, Layer0FullStats* stats, std::string* error) {
    return run_recurrent_layer(0, rms_eps, stats, error);
}

// The driver's layer chain is specialised by shape, not by layer index, so
// every recurrent layer runs through it with its own tensors
// (src/runtime.cpp:462-600).
bool Runtime::run_recurrent_layer(std::uint32_t layer, float rms_eps, Layer0FullStats* stats, std::string* error) {
    try {
        if (!driver_.available()) throw std::runtime_error("recurrent layer requires an initialized GPU driver");
        if (detect_qwen35_layer_kind(pack_, layer) != Qwen35LayerKind::Recurrent)
            throw std::runtime_error("requested layer is not a recurrent Qwen3.8 layer");
        const LayerTensors L = layer_tensors(pack_, layer, Part::Full);
        return driver_.run_qwen35_layer0_full(
            f32(pack_, L.norm), pack_.tensor_data(*L.qkv), qh_off(L.qkv), qs_off(L.qkv), pack_.tensor_data(*L.z),
            qh_off(L.z), qs_off(L.z), pack_.tensor_data(*L.beta), pack_.tensor_data(*L.alpha), f32(pack_, L.conv),
            f32(pack_, L.dt), f32(pack_, L.a), f32(pack_, L.ssm_norm), pack_.tensor_data(*L.ssm_out), qh_off(L.ssm_out),
            qs_off(L.ssm_out), f32(pack_, L.post_norm), pack_.tensor_data(*L.ffn_gate), pack_.tensor_data(*L.ffn_up),
            qh_off(L.ffn_up), qs_off(L.ffn_up), pack_.tensor_data(*L.ffn_down), qh_off(L.ffn_down),
            qs_off(L.ffn_down), rms_eps, stats, error);
    } catch (const std::exception& e) {
        if (error) *error = e.what();
        return false;
    }
}

}  // namespace q38
