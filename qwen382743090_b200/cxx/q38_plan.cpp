// q38-plan -- the reference's placement-plan command (src/plan.cpp:64-162) in
// C++ over this library's Q38PACK reader and PlacementPlan (q38_pack_plan):
// the pack's tensors at 256-byte aligned offsets of one virtual range rounded
// up to the GPU page, with totals by role, execution layout and tensor type.
// Host only: it needs no GPU.
//
//   q38-plan --model MODEL.q38pack [--page-bytes N] [--list]
#include <cinttypes>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <string>
#include <vector>

#include "../../include/q38rt.h"

namespace {

const char* role_name(uint32_t r) {
    static const char* kNames[] = {"unknown", "embedding", "output_norm", "output", "attention",
                                   "deltanet", "ffn", "norm", "mtp"};
    return r < sizeof(kNames) / sizeof(kNames[0]) ? kNames[r] : "unknown";
}

const char* layout_name(uint32_t l) {
    switch (l) {
        case Q38_LAYOUT_GGUF_NATIVE: return "GGUF_NATIVE";
        case Q38_LAYOUT_SM86_Q5K_SOA: return "SM86_Q5K_SOA";
        case Q38_LAYOUT_B200_TILED: return "B200_TILED";
        default: return "UNKNOWN";
    }
}

const char* type_name(uint32_t t) {
    switch (t) {
        case 0: return "F32";
        case 1: return "F16";
        case 12: return "Q4_K";
        case 13: return "Q5_K";
        case 14: return "Q6_K";
        case 15: return "Q8_K";
        case 23: return "IQ4_XS";
        default: return "UNKNOWN";
    }
}

constexpr double kGiB = 1024.0 * 1024.0 * 1024.0;

struct Tally {
    uint64_t bytes = 0;
    uint32_t count = 0;
};

}  // namespace

int main(int argc, char** argv) {
    std::string model;
    uint64_t page_bytes = 2u << 20;
    bool list = false;
    for (int i = 1; i < argc; ++i) {
        const std::string arg = argv[i];
        if (arg == "--model" && i + 1 < argc) {
            model = argv[++i];
        } else if (arg == "--page-bytes" && i + 1 < argc) {
            page_bytes = std::strtoull(argv[++i], nullptr, 10);
        } else if (arg == "--list") {
            list = true;
        } else if (arg == "--help") {
            std::printf("usage: q38-plan --model MODEL.q38pack [--page-bytes N] [--list]\n");
            return 0;
        } else {
            std::fprintf(stderr, "q38-plan: unknown argument: %s\n", arg.c_str());
            return 2;
        }
    }
    if (model.empty()) {
        std::fprintf(stderr, "q38-plan: --model is required\n");
        return 2;
    }
    q38_pack* pack = nullptr;
    if (q38_pack_open(model.c_str(), &pack) != Q38_OK) {
        std::fprintf(stderr, "q38-plan: %s\n", q38_last_error());
        return 1;
    }
    q38_pack_header_info hdr{};
    q38_plan_stats st{};
    std::vector<uint64_t> offsets;
    int rc = q38_pack_header(pack, &hdr);
    if (rc == Q38_OK) {
        offsets.resize(hdr.tensor_count);
        rc = q38_pack_plan(pack, page_bytes, &st, offsets.data());
    }
    std::vector<q38_tensor_record> tensors(rc == Q38_OK ? hdr.tensor_count : 0);
    for (uint32_t i = 0; rc == Q38_OK && i < hdr.tensor_count; ++i) rc = q38_pack_tensor(pack, i, &tensors[i]);
    if (rc != Q38_OK) {
        std::fprintf(stderr, "q38-plan: %s\n", q38_last_error());
        q38_pack_close(pack);
        return 1;
    }
    std::map<uint32_t, Tally> by_role, by_layout, by_type;
    for (const q38_tensor_record& t : tensors) {
        by_role[t.role].bytes += t.stored_bytes;
        by_layout[t.layout].bytes += t.stored_bytes;
        ++by_layout[t.layout].count;
        by_type[t.ggml_type].bytes += t.stored_bytes;
        ++by_type[t.ggml_type].count;
    }
    std::printf("Q38 GPU placement plan\n");
    std::printf("Q38PACK version: %u\n", hdr.version);
    std::printf("GPU page: %" PRIu64 " bytes\n", st.page_bytes);
    std::printf("tensors: %u\n", hdr.tensor_count);
    std::printf("payload: %.3f GiB\n", st.tensor_payload_bytes / kGiB);
    std::printf("reserved VA: %.3f GiB\n", st.reserved_va_bytes / kGiB);
    std::printf("page padding: %.3f GiB\n", st.page_padding_bytes / kGiB);
    std::printf("pages: %" PRIu64 "\n", st.page_count);
    for (const auto& [r, t] : by_role) std::printf("role[%s]: %.3f GiB\n", role_name(r), t.bytes / kGiB);
    std::printf("execution layouts:\n");
    for (const auto& [l, t] : by_layout)
        std::printf("  layout[%u/%s]: %u tensors, %.3f GiB\n", l, layout_name(l), t.count, t.bytes / kGiB);
    std::printf("tensor types (physical stored bytes):\n");
    for (const auto& [ty, t] : by_type)
        std::printf("  type[%u/%s]: %u tensors, %.3f GiB\n", ty, type_name(ty), t.count, t.bytes / kGiB);
    if (list) {
        for (size_t i = 0; i < tensors.size(); ++i) {
            const q38_tensor_record& t = tensors[i];
            std::printf("%s role=%s va=0x%" PRIx64 " page_off=%" PRIu64 " bytes=%" PRIu64 " layout=%s\n", t.name,
                        role_name(t.role), offsets[i], offsets[i] % st.page_bytes, t.stored_bytes,
                        layout_name(t.layout));
        }
    }
    q38_pack_close(pack);
    return 0;
}
