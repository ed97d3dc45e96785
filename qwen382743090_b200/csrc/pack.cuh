// pack.cuh -- Q38PACK reader, GPU placement plan and resident upload (host
// side; included by q38rt.cu after the C ABI helpers).
//
// Format (docs of the reference: docs/Q38PACK.md; reader src/q38pack.cpp:56-167;
// header field offsets :96-113, directory entry :131-146): a 256-byte
// little-endian header, tensor_count 256-byte directory entries, a JSON
// manifest, the source GGUF metadata, then tensor payloads.  Versions 1 and 2
// are the reference's; version 3 is this library's and adds execution layout 2
// (B200 fragment tiles of 8 rows x 2 super-blocks for Q5_K and Q4_K,
// gemv_frag.cuh).  A reference
// reader rejects version 3 (it accepts 1..2), so a v3 pack never reaches a
// kernel that cannot run it.
//
// The placement plan is PlacementPlan::build (src/placement.cpp:23-60): tensors
// in directory order at 256-byte aligned offsets of one virtual range rounded
// up to the GPU page.  q38_pack_upload maps that range once through VMM and
// copies every payload to its planned offset, so the whole model is resident
// at fixed device addresses.
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace {

constexpr char kPackMagic[8] = {'Q', '3', '8', 'P', 'A', 'C', 'K', '\0'};
constexpr uint32_t kPackHeaderBytes = 256, kPackEntryBytes = 256, kPackMaxVersion = 3;

template <class T>
T rd(const uint8_t* p) {
    T v;
    memcpy(&v, p, sizeof(T));
    return v;
}

uint64_t plan_align(uint64_t v, uint64_t a) { return (v + a - 1u) & ~(a - 1u); }

}  // namespace

struct q38_pack {
    int fd = -1;
    size_t size = 0;
    const uint8_t* map = nullptr;
    q38_pack_header_info hdr{};
    std::vector<q38_tensor_record> tensors;
};

namespace {

int pack_range(const q38_pack* p, uint64_t off, uint64_t bytes, const char* what) {
    if (off > p->size || bytes > p->size - off)
        return fail(Q38_ERR_INVALID, "q38pack: %s outside the file", what);
    return Q38_OK;
}

int pack_parse(q38_pack* p) {
    const uint8_t* b = p->map;
    if (memcmp(b, kPackMagic, 8) != 0) return fail(Q38_ERR_INVALID, "q38pack: bad magic");
    q38_pack_header_info& h = p->hdr;
    h.version = rd<uint32_t>(b + 8);
    h.header_bytes = rd<uint32_t>(b + 12);
    h.flags = rd<uint32_t>(b + 16);
    h.tensor_count = rd<uint32_t>(b + 20);
    h.alignment = rd<uint32_t>(b + 24);
    h.directory_offset = rd<uint64_t>(b + 32);
    h.directory_bytes = rd<uint64_t>(b + 40);
    h.manifest_offset = rd<uint64_t>(b + 48);
    h.manifest_bytes = rd<uint64_t>(b + 56);
    h.raw_gguf_meta_offset = rd<uint64_t>(b + 64);
    h.raw_gguf_meta_bytes = rd<uint64_t>(b + 72);
    h.data_offset = rd<uint64_t>(b + 80);
    h.data_bytes = rd<uint64_t>(b + 88);
    h.source_file_size = rd<uint64_t>(b + 96);
    h.source_data_offset = rd<uint64_t>(b + 104);
    if (h.version < 1 || h.version > kPackMaxVersion || h.header_bytes != kPackHeaderBytes)
        return fail(Q38_ERR_UNSUPPORTED, "q38pack: unsupported version %u / header %u", h.version, h.header_bytes);
    if (h.directory_bytes != static_cast<uint64_t>(h.tensor_count) * kPackEntryBytes)
        return fail(Q38_ERR_INVALID, "q38pack: malformed directory size");
    if (int rc = pack_range(p, h.directory_offset, h.directory_bytes, "directory")) return rc;
    if (int rc = pack_range(p, h.manifest_offset, h.manifest_bytes, "manifest")) return rc;
    if (int rc = pack_range(p, h.raw_gguf_meta_offset, h.raw_gguf_meta_bytes, "raw GGUF metadata")) return rc;
    if (int rc = pack_range(p, h.data_offset, h.data_bytes, "tensor data")) return rc;
    p->tensors.assign(h.tensor_count, q38_tensor_record{});
    for (uint32_t i = 0; i < h.tensor_count; ++i) {
        const uint8_t* e = b + h.directory_offset + static_cast<uint64_t>(i) * kPackEntryBytes;
        q38_tensor_record& t = p->tensors[i];
        size_t n = 0;
        while (n < 160 && e[n] != 0) ++n;
        memcpy(t.name, e, n);
        t.name[n] = '\0';
        t.ndim = rd<uint32_t>(e + 160);
        t.ggml_type = rd<uint32_t>(e + 164);
        if (t.ndim > 4) return fail(Q38_ERR_INVALID, "q38pack: tensor '%s' has more than 4 dimensions", t.name);
        for (int d = 0; d < 4; ++d) t.dims[d] = rd<uint64_t>(e + 168 + 8 * d);
        t.data_offset = rd<uint64_t>(e + 200);
        t.stored_bytes = rd<uint64_t>(e + 208);
        t.source_offset = rd<uint64_t>(e + 216);
        t.role = rd<uint32_t>(e + 224);
        t.flags = rd<uint32_t>(e + 228);
        if (h.version >= 2) {
            t.layout = rd<uint32_t>(e + 232);
            t.layout_flags = rd<uint32_t>(e + 236);
            t.aux0_offset = rd<uint64_t>(e + 240);
            t.aux1_offset = rd<uint64_t>(e + 248);
        }
        if (int rc = pack_range(p, t.data_offset, t.stored_bytes, "tensor")) return rc;
        if (t.data_offset < h.data_offset) return fail(Q38_ERR_INVALID, "q38pack: tensor '%s' outside the data area", t.name);
        const uint64_t end = t.data_offset + t.stored_bytes;
        if (t.layout == Q38_LAYOUT_SM86_Q5K_SOA) {
            if (!(t.data_offset <= t.aux0_offset && t.aux0_offset <= t.aux1_offset && t.aux1_offset < end))
                return fail(Q38_ERR_INVALID, "q38pack: invalid SoA plane offsets of '%s'", t.name);
        } else if (t.layout == Q38_LAYOUT_B200_TILED) {
            if (h.version < 3 || (t.ggml_type != Q38_TYPE_Q5_K && t.ggml_type != Q38_TYPE_Q4_K) || t.dims[0] % 512u)
                return fail(Q38_ERR_INVALID, "q38pack: invalid tiled tensor '%s'", t.name);
            if (t.stored_bytes < q38_tiled_bytes(t.ggml_type, static_cast<uint32_t>(t.dims[0]), static_cast<uint32_t>(t.dims[1])))
                return fail(Q38_ERR_INVALID, "q38pack: tiled tensor '%s' is truncated", t.name);
        } else if (t.layout != Q38_LAYOUT_GGUF_NATIVE) {
            return fail(Q38_ERR_UNSUPPORTED, "q38pack: unknown execution layout %u of '%s'", t.layout, t.name);
        }
    }
    return Q38_OK;
}

}  // namespace

extern "C" {

int q38_pack_open(const char* path, q38_pack** out) {
    if (!path || !out) return fail(Q38_ERR_INVALID, "q38_pack_open: null argument");
    *out = nullptr;
    auto p = std::make_unique<q38_pack>();
    p->fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (p->fd < 0) return fail(Q38_ERR_INVALID, "q38pack: unable to open %s", path);
    struct stat st {};
    if (::fstat(p->fd, &st) != 0 || st.st_size < static_cast<off_t>(kPackHeaderBytes)) {
        ::close(p->fd);
        return fail(Q38_ERR_INVALID, "q38pack: invalid or too-small file %s", path);
    }
    p->size = static_cast<size_t>(st.st_size);
    void* m = ::mmap(nullptr, p->size, PROT_READ, MAP_PRIVATE, p->fd, 0);
    if (m == MAP_FAILED) {
        ::close(p->fd);
        return fail(Q38_ERR_INVALID, "q38pack: mmap failed");
    }
    p->map = static_cast<const uint8_t*>(m);
    if (int rc = pack_parse(p.get())) {
        ::munmap(const_cast<uint8_t*>(p->map), p->size);
        ::close(p->fd);
        return rc;
    }
    *out = p.release();
    return Q38_OK;
}

int q38_pack_close(q38_pack* p) {
    if (!p) return Q38_OK;
    if (p->map) ::munmap(const_cast<uint8_t*>(p->map), p->size);
    if (p->fd >= 0) ::close(p->fd);
    delete p;
    return Q38_OK;
}

int q38_pack_header(const q38_pack* p, q38_pack_header_info* out) {
    if (!p || !out) return fail(Q38_ERR_INVALID, "q38_pack_header: null argument");
    *out = p->hdr;
    return Q38_OK;
}

int q38_pack_tensor(const q38_pack* p, uint32_t index, q38_tensor_record* out) {
    if (!p || !out || index >= p->tensors.size()) return fail(Q38_ERR_INVALID, "q38_pack_tensor: bad index");
    *out = p->tensors[index];
    return Q38_OK;
}

int q38_pack_find(const q38_pack* p, const char* name, uint32_t* index) {
    if (!p || !name || !index) return fail(Q38_ERR_INVALID, "q38_pack_find: null argument");
    for (size_t i = 0; i < p->tensors.size(); ++i)
        if (strcmp(p->tensors[i].name, name) == 0) {
            *index = static_cast<uint32_t>(i);
            return Q38_OK;
        }
    return fail(Q38_ERR_INVALID, "q38pack: no tensor '%s'", name);
}

int q38_pack_host_data(const q38_pack* p, uint32_t index, const void** data) {
    if (!p || !data || index >= p->tensors.size()) return fail(Q38_ERR_INVALID, "q38_pack_host_data: bad index");
    *data = p->map + p->tensors[index].data_offset;
    return Q38_OK;
}

int q38_pack_plan(const q38_pack* p, uint64_t page_bytes, q38_plan_stats* stats, uint64_t* va_offsets) {
    if (!p || !stats) return fail(Q38_ERR_INVALID, "q38_pack_plan: null argument");
    if (page_bytes == 0 || (page_bytes & (page_bytes - 1u)))
        return fail(Q38_ERR_INVALID, "GPU page size must be a positive power of two");
    uint64_t cursor = 0, payload = 0;
    for (size_t i = 0; i < p->tensors.size(); ++i) {
        cursor = plan_align(cursor, 256u);
        if (va_offsets) va_offsets[i] = cursor;
        cursor += p->tensors[i].stored_bytes;
        payload += p->tensors[i].stored_bytes;
    }
    stats->page_bytes = page_bytes;
    stats->tensor_payload_bytes = payload;
    stats->reserved_va_bytes = plan_align(cursor, page_bytes);
    stats->page_padding_bytes = stats->reserved_va_bytes >= payload ? stats->reserved_va_bytes - payload : 0;
    stats->page_count = stats->reserved_va_bytes / page_bytes;
    return Q38_OK;
}

int q38_pack_upload(const q38_pack* p, q38_ctx* ctx, uint64_t page_bytes, q38_devptr* base) {
    if (!p || !ctx || !base) return fail(Q38_ERR_INVALID, "q38_pack_upload: null argument");
    q38_plan_stats st{};
    std::vector<uint64_t> va(p->tensors.size());
    if (int rc = q38_pack_plan(p, page_bytes, &st, va.data())) return rc;
    q38_devptr b = 0;
    if (int rc = q38_alloc(ctx, std::max<uint64_t>(st.reserved_va_bytes, 1u), &b)) return rc;
    for (size_t i = 0; i < p->tensors.size(); ++i) {
        const q38_tensor_record& t = p->tensors[i];
        if (t.stored_bytes == 0) continue;
        const cudaError_t e = cudaMemcpy(dptr<void>(b + va[i]), p->map + t.data_offset, t.stored_bytes,
                                         cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            q38_free(ctx, b);
            return cuda_fail(e, "q38_pack_upload");
        }
    }
    *base = b;
    return Q38_OK;
}

int q38_pack_weight_desc(const q38_pack* p, uint32_t index, q38_devptr base, q38_weight_desc* out) {
    if (!p || !out || index >= p->tensors.size()) return fail(Q38_ERR_INVALID, "q38_pack_weight_desc: bad index");
    q38_plan_stats st{};
    std::vector<uint64_t> va(p->tensors.size());
    if (int rc = q38_pack_plan(p, 1u << 21, &st, va.data())) return rc;
    const q38_tensor_record& t = p->tensors[index];
    const q38_devptr d = base + va[index];
    *out = q38_weight_desc{t.ggml_type, t.layout, static_cast<uint32_t>(t.dims[1]), static_cast<uint32_t>(t.dims[0]),
                           d, 0, 0};
    if (t.layout == Q38_LAYOUT_SM86_Q5K_SOA) {
        out->aux0 = d + (t.aux0_offset - t.data_offset);
        out->aux1 = d + (t.aux1_offset - t.data_offset);
    }
    return Q38_OK;
}

}  // extern "C"
