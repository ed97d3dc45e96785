// q38rt.cu -- C ABI of the Q38RT B200 runtime (declared in include/q38rt.h).
//
// The whole device side is one CUDA translation unit: this file includes
// every kernel header, so module-scope __device__ state (the fault word) is
// defined once and no relocatable-device-code link step is needed.  The CUDA
// runtime is linked statically and the driver is reached through
// cudaGetDriverEntryPoint, so the library loads on machines without a GPU
// driver (its calls then fail with Q38_ERR_NO_DEVICE).
#include <dlfcn.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/q38rt.h"
#include "common.cuh"
#include "check.cuh"
#include "gemv_q5k.cuh"
#include "gemv_kq.cuh"
#include "gemv_frag.cuh"
#include "gemm_frag.cuh"
#include "gemm_tc.cuh"
#include "gemv_soa_frag.cuh"
#include "q81.cuh"
#include "layer.cuh"
#include "xpack.cuh"

// ---- fixed x-pack scratch of q38_q5k_sm86_soa_gemv_vec_noalloc -------------------
// The no-allocation entry point packs x here instead of into the cudaMalloc'd
// workspace.  Sized for kNoAllocMaxCols activations with four limbs (the same
// region layout as q38_xpack_bytes); every byte the GEMV reads is written by
// the pack kernel first, so nothing in it has to start at zero.  One copy
// exists per device (module-scope __device__ memory is per device).
constexpr uint32_t kNoAllocMaxCols = 32768;  // above the widest projection input (ffn_down, 17408)
constexpr size_t round_up_256(size_t b) { return (b + 255u) & ~size_t(255); }
constexpr size_t kNoAllocXpackBytes = round_up_256(q38::xpack_limb_bytes(4, kNoAllocMaxCols / 256u, 1)) +
                                      round_up_256(static_cast<size_t>(kNoAllocMaxCols / 256u) * 32u) +
                                      round_up_256(static_cast<size_t>(kNoAllocMaxCols / 256u) * 4u);
static_assert(kNoAllocXpackBytes == 135680, "no-alloc scratch is 132.5 KiB");
static __device__ __align__(256) uint8_t g_noalloc_xpack[kNoAllocXpackBytes];

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    const int code = (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) ? Q38_ERR_NO_DEVICE
                     : (e == cudaErrorMemoryAllocation)                             ? Q38_ERR_NOMEM
                                                                                    : Q38_ERR_CUDA;
    return fail(code, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define Q38_CUDA(call, what)                                      \
    do {                                                          \
        cudaError_t e_ = (call);                                  \
        if (e_ != cudaSuccess) return cuda_fail(e_, (what));      \
    } while (0)

cudaStream_t as_stream(q38_stream s) { return reinterpret_cast<cudaStream_t>(s); }
template <class T>
T* dptr(q38_devptr p) {
    return reinterpret_cast<T*>(static_cast<uintptr_t>(p));
}

// ---- driver entry points (resolved through the runtime, no -lcuda) ---------
struct DriverApi {
    bool ok = false;
    CUresult (*tensorMapEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                     const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                     CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill) = nullptr;
    CUresult (*memGetAllocationGranularity)(size_t*, const CUmemAllocationProp*,
                                            CUmemAllocationGranularity_flags) = nullptr;
    CUresult (*memCreate)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*,
                          unsigned long long) = nullptr;
    CUresult (*memRelease)(CUmemGenericAllocationHandle) = nullptr;
    CUresult (*memAddressReserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long) = nullptr;
    CUresult (*memAddressFree)(CUdeviceptr, size_t) = nullptr;
    CUresult (*memMap)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long) = nullptr;
    CUresult (*memUnmap)(CUdeviceptr, size_t) = nullptr;
    CUresult (*memSetAccess)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t) = nullptr;
    CUresult (*getErrorString)(CUresult, const char**) = nullptr;
};

std::mutex g_mu;
DriverApi g_drv;

template <class F>
bool resolve(const char* name, F& fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || !p ||
        q != cudaDriverEntryPointSuccess)
        return false;
    fn = reinterpret_cast<F>(p);
    return true;
}

int driver_api(DriverApi** out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_drv.ok) {
        int n = 0;
        cudaError_t e = cudaGetDeviceCount(&n);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
        bool ok = resolve("cuTensorMapEncodeTiled", g_drv.tensorMapEncodeTiled) &&
                  resolve("cuMemGetAllocationGranularity", g_drv.memGetAllocationGranularity) &&
                  resolve("cuMemCreate", g_drv.memCreate) && resolve("cuMemRelease", g_drv.memRelease) &&
                  resolve("cuMemAddressReserve", g_drv.memAddressReserve) &&
                  resolve("cuMemAddressFree", g_drv.memAddressFree) && resolve("cuMemMap", g_drv.memMap) &&
                  resolve("cuMemUnmap", g_drv.memUnmap) && resolve("cuMemSetAccess", g_drv.memSetAccess) &&
                  resolve("cuGetErrorString", g_drv.getErrorString);
        if (!ok) return fail(Q38_ERR_NO_DEVICE, "CUDA driver entry points unavailable");
        g_drv.ok = true;
    }
    *out = &g_drv;
    return Q38_OK;
}

int cu_fail(CUresult r, const char* what) {
    const char* msg = "unknown";
    if (g_drv.getErrorString) g_drv.getErrorString(r, &msg);
    return fail(r == CUDA_ERROR_OUT_OF_MEMORY ? Q38_ERR_NOMEM : Q38_ERR_CUDA, "%s: CUresult %d (%s)", what,
                static_cast<int>(r), msg);
}

// ---- per-device state -----------------------------------------------------
struct DeviceState {
    bool probed = false;
    int sm_major = 0, sm_minor = 0, sm_count = 0;
    void* workspace = nullptr;  // x-pack scratch for the drop-in launchers
    size_t workspace_bytes = 0;
    void* io = nullptr;  // device staging of the host-buffer GEMV's x and y
    size_t io_bytes = 0;
    void* noalloc_xpack = nullptr;  // this device's address of g_noalloc_xpack
    bool attrs_set = false;
};
std::deque<DeviceState> g_dev;  // deque: growing it keeps earlier DeviceState* valid

int current_device(int* dev, DeviceState** st) {
    Q38_CUDA(cudaGetDevice(dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_dev.size() <= static_cast<size_t>(*dev)) g_dev.resize(*dev + 1);
    DeviceState& s = g_dev[*dev];
    if (!s.probed) {
        cudaDeviceProp prop{};
        Q38_CUDA(cudaGetDeviceProperties(&prop, *dev), "cudaGetDeviceProperties");
        s.sm_major = prop.major;
        s.sm_minor = prop.minor;
        s.sm_count = prop.multiProcessorCount;
        s.probed = true;
    }
    *st = &s;
    if (s.sm_major != 10)
        return fail(Q38_ERR_UNSUPPORTED, "Q38RT B200 kernels need sm_100; device %d is sm_%d%d", *dev, s.sm_major,
                    s.sm_minor);
    return Q38_OK;
}

// Grow a per-device scratch buffer to at least `bytes` (powers of two, 1 MiB
// at least); the old contents are not kept.
int ensure_buffer(void** buf, size_t* have, size_t bytes, const char* what, void** out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (*have < bytes) {
        if (*buf) cudaFree(*buf);
        *buf = nullptr;
        *have = 0;
        size_t want = 1;
        while (want < bytes) want <<= 1;
        if (want < (1u << 20)) want = 1u << 20;
        Q38_CUDA(cudaMalloc(buf, want), what);
        *have = want;
    }
    *out = *buf;
    return Q38_OK;
}

int ensure_workspace(DeviceState* st, size_t bytes, void** out) {
    return ensure_buffer(&st->workspace, &st->workspace_bytes, bytes, "cudaMalloc(x-pack workspace)", out);
}

// Address of g_noalloc_xpack on the current device, looked up once per device
// (the caller made that device current through current_device and passes its state).
int noalloc_scratch(DeviceState* st, void** out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!st->noalloc_xpack) {
        void* p = nullptr;
        Q38_CUDA(cudaGetSymbolAddress(&p, g_noalloc_xpack), "cudaGetSymbolAddress(no-alloc x-pack scratch)");
        st->noalloc_xpack = p;
    }
    *out = st->noalloc_xpack;
    return Q38_OK;
}

// ---- tensor maps ------------------------------------------------------------
int encode_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint32_t elem_bytes, uint64_t inner_elems,
              uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
    DriverApi* d = nullptr;
    if (int rc = driver_api(&d)) return rc;
    const cuuint64_t dims[2] = {inner_elems, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    (void)elem_bytes;
    CUresult r = d->tensorMapEncodeTiled(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                                         CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cu_fail(r, "cuTensorMapEncodeTiled");
    return Q38_OK;
}

struct MapKey {
    uint64_t a, b, c;
    uint32_t rows, cols;
    bool operator==(const MapKey& o) const {
        return a == o.a && b == o.b && c == o.c && rows == o.rows && cols == o.cols;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey& k) const {
        uint64_t h = k.a * 0x9e3779b97f4a7c15ull ^ (k.b + 0x632be59bd9b4e019ull) * 31 ^ k.c * 131 ^
                     (static_cast<uint64_t>(k.rows) << 32 | k.cols);
        return static_cast<size_t>(h ^ (h >> 29));
    }
};
std::unordered_map<MapKey, q38::Q5kSoaMaps, MapKeyHash> g_soa_maps;

int soa_maps(q38_devptr meta, q38_devptr qh, q38_devptr qs, uint32_t rows, uint32_t cols, q38::Q5kSoaMaps* out) {
    const MapKey key{meta, qh, qs, rows, cols};
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_soa_maps.find(key);
        if (it != g_soa_maps.end()) {
            *out = it->second;
            return Q38_OK;
        }
    }
    const uint64_t nb = cols / 256u;
    q38::Q5kSoaMaps m{};
    const int box_rows[2] = {4, 2};
    for (int v = 0; v < 2; ++v) {
        CUtensorMap* mm = v == 0 ? &m.meta4 : &m.meta2;
        CUtensorMap* mh = v == 0 ? &m.qh4 : &m.qh2;
        CUtensorMap* ms = v == 0 ? &m.qs4 : &m.qs2;
        if (int rc = encode_2d(mm, dptr<void>(meta), CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, nb * 5, rows, nb * 20,
                               q38::kTileBlocks * 5, box_rows[v]))
            return rc;
        if (int rc = encode_2d(mh, dptr<void>(qh), CU_TENSOR_MAP_DATA_TYPE_UINT64, 8, nb * 4, rows, nb * 32,
                               q38::kTileBlocks * 4, box_rows[v]))
            return rc;
        if (int rc = encode_2d(ms, dptr<void>(qs), CU_TENSOR_MAP_DATA_TYPE_UINT64, 8, nb * 16, rows, nb * 128,
                               q38::kTileBlocks * 16, box_rows[v]))
            return rc;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_soa_maps.size() > 4096) g_soa_maps.clear();
    g_soa_maps.emplace(key, m);
    *out = m;
    return Q38_OK;
}

// cudaFuncSetAttribute(max dynamic shared memory) once per (kernel, device).
template <auto Kernel>
int ensure_smem_attr(int dev, size_t bytes) {
    static std::atomic<uint64_t> done{0};
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return Q38_OK;
    Q38_CUDA(cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
             "cudaFuncSetAttribute(max dynamic shared memory)");
    done.fetch_or(bit, std::memory_order_acq_rel);
    return Q38_OK;
}

// ---- launch helpers -----------------------------------------------------------
template <class... KArgs, class... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const char* what,
               Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q38_CUDA(cudaLaunchKernelEx(&cfg, kernel, args...), what);
    return Q38_OK;
}

// launch_pdl with thread-block clusters of cluster_x CTAs along x.
template <class... KArgs, class... Args>
int launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, unsigned cluster_x, size_t smem,
                       cudaStream_t stream, const char* what, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    Q38_CUDA(cudaLaunchKernelEx(&cfg, kernel, args...), what);
    return Q38_OK;
}

int gemv_ctas_per_sm() {
    static int v = [] {
        const char* e = getenv("Q38_GEMV_CTAS_PER_SM");
        int n = e ? atoi(e) : 1;
        return n < 1 ? 1 : (n > 2 ? 2 : n);
    }();
    return v;
}

struct XPackView {
    uint8_t* limbs;
    float* gsum;
    float* scale;
};

XPackView xpack_view(void* base, uint32_t nl, uint32_t nb, uint32_t batch) {
    uint8_t* p = static_cast<uint8_t*>(base);
    XPackView v{};
    v.limbs = p;
    size_t off = (q38::xpack_limb_bytes(static_cast<int>(nl), nb, batch) + 255u) & ~size_t(255);
    v.gsum = reinterpret_cast<float*>(p + off);
    off += (static_cast<size_t>(batch) * nb * 8u * 4u + 255u) & ~size_t(255);
    v.scale = reinterpret_cast<float*>(p + off);
    return v;
}

// Limbs used when f32 x is packed ahead of a GEMV: three (23-bit
// activations) up to K = 6144, four (30-bit) above, where the rounding of x
// would otherwise approach the 1e-4 absolute tolerance on near-zero rows.
uint32_t f32_limbs(uint32_t cols) { return cols <= 6144u ? 3u : 4u; }

int check_soa_args(q38_devptr meta, q38_devptr qh, q38_devptr qs, uint32_t cols, uint32_t rows) {
    if (rows == 0 || cols == 0 || cols % 256u)
        return fail(Q38_ERR_INVALID, "Q5_K SoA GEMV needs rows > 0 and cols a positive multiple of 256 (got %u x %u)",
                    rows, cols);
    if ((cols / 256u) % 4u)
        return fail(Q38_ERR_UNSUPPORTED, "Q5_K SoA GEMV tiles 4 super-blocks: cols must be a multiple of 1024 (got %u)",
                    cols);
    if ((meta | qh | qs) & 15u) return fail(Q38_ERR_INVALID, "Q5_K SoA planes must be 16-byte aligned");
    if (!meta || !qh || !qs) return fail(Q38_ERR_INVALID, "Q5_K SoA plane pointer is null");
    return Q38_OK;
}

int launch_soa_packed(q38_devptr meta, q38_devptr qh, q38_devptr qs, const XPackView& xv, uint32_t nl, float* y,
                      uint32_t cols, uint32_t rows, cudaStream_t stream) {
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    q38::Q5kSoaMaps maps{};
    if (int rc = soa_maps(meta, qh, qs, rows, cols, &maps)) return rc;
    if (!st->attrs_set) {
        const int smem = static_cast<int>(q38::kSoaSmemBytes2);
        Q38_CUDA(cudaFuncSetAttribute(q38::gemv_q5k_soa_kernel<3, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                 "cudaFuncSetAttribute");
        Q38_CUDA(cudaFuncSetAttribute(q38::gemv_q5k_soa_kernel<3, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                 "cudaFuncSetAttribute");
        Q38_CUDA(cudaFuncSetAttribute(q38::gemv_q5k_soa_kernel<1, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                 "cudaFuncSetAttribute");
        Q38_CUDA(cudaFuncSetAttribute(q38::gemv_q5k_soa_kernel<1, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                 "cudaFuncSetAttribute");
        st->attrs_set = true;
    }
    const int per_sm = gemv_ctas_per_sm();
    const uint32_t npairs = (rows + 1u) / 2u;
    uint32_t grid = static_cast<uint32_t>(st->sm_count * per_sm);
    if (grid > npairs) grid = npairs;
    const uint32_t nb = cols / 256u;
    const uint8_t* xl = xv.limbs;
    const float* gs = xv.gsum;
    const float* sc = xv.scale;
    const dim3 g(grid), b(q38::kGemvThreads);
    const size_t smem = q38::kSoaSmemBytes2;
    if (nl == 4) {
        if (int rc = ensure_smem_attr<q38::gemv_q5k_soa_kernel<4, 1>>(dev, smem)) return rc;
        if (int rc = ensure_smem_attr<q38::gemv_q5k_soa_kernel<4, 2>>(dev, smem)) return rc;
        if (per_sm == 2)
            return launch_pdl(q38::gemv_q5k_soa_kernel<4, 2>, g, b, smem, stream, "launch gemv_q5k_soa<4,2>", maps,
                              xl, gs, sc, y, rows, nb);
        return launch_pdl(q38::gemv_q5k_soa_kernel<4, 1>, g, b, smem, stream, "launch gemv_q5k_soa<4,1>", maps, xl,
                          gs, sc, y, rows, nb);
    }
    if (nl == 3) {
        if (per_sm == 2)
            return launch_pdl(q38::gemv_q5k_soa_kernel<3, 2>, g, b, smem, stream, "launch gemv_q5k_soa<3,2>", maps,
                              xl, gs, sc, y, rows, nb);
        return launch_pdl(q38::gemv_q5k_soa_kernel<3, 1>, g, b, smem, stream, "launch gemv_q5k_soa<3,1>", maps, xl,
                          gs, sc, y, rows, nb);
    }
    if (per_sm == 2)
        return launch_pdl(q38::gemv_q5k_soa_kernel<1, 2>, g, b, smem, stream, "launch gemv_q5k_soa<1,2>", maps, xl,
                          gs, sc, y, rows, nb);
    return launch_pdl(q38::gemv_q5k_soa_kernel<1, 1>, g, b, smem, stream, "launch gemv_q5k_soa<1,1>", maps, xl, gs,
                      sc, y, rows, nb);
}

constexpr size_t kChainlessSmemMaxSoa = 227u * 1024u;
std::unordered_map<MapKey, q38::SoaFragMaps, MapKeyHash> g_soa_frag_maps;

// 8-row boxes of the SoA planes for gemv_soa_frag_kernel (uint32 elements):
// QS one super-block (32 words) and QH four (32 words), both with the 128-byte
// swizzle; META 20 words = 4 super-blocks.
int soa_frag_maps(q38_devptr meta, q38_devptr qh, q38_devptr qs, uint32_t rows, uint32_t cols, q38::SoaFragMaps* out) {
    const MapKey key{meta, qh, qs, rows, cols};
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_soa_frag_maps.find(key);
        if (it != g_soa_frag_maps.end()) {
            *out = it->second;
            return Q38_OK;
        }
    }
    const uint64_t nb = cols / 256u;
    q38::SoaFragMaps m{};
    if (int rc = encode_2d(&m.qs, dptr<void>(qs), CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, nb * 32, rows, nb * 128, 32,
                           q38::kSfRows, CU_TENSOR_MAP_SWIZZLE_128B))  // one super-block: 8 x 128 B
        return rc;
    if (int rc = encode_2d(&m.qh, dptr<void>(qh), CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, nb * 8, rows, nb * 32,
                           q38::kSfBlocks * 8, q38::kSfRows, CU_TENSOR_MAP_SWIZZLE_128B))  // 4 super-blocks: 8 x 128 B
        return rc;
    if (int rc = encode_2d(&m.meta, dptr<void>(meta), CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, nb * 5, rows, nb * 20,
                           q38::kSfBlocks * 5, q38::kSfRows))
        return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_soa_frag_maps.size() > 4096) g_soa_frag_maps.clear();
    g_soa_frag_maps.emplace(key, m);
    *out = m;
    return Q38_OK;
}

// 12 warps with 2-slot rings, one CTA per SM: measured on B200 against 8 / 16
// warps, 1- / 3-slot rings and two 8-warp CTAs per SM, all within 10 % and
// none faster (8.8 us at 6144 x 5120, 16.2 us at 17408 x 5120).  Nor two
// 12-warp CTAs per SM with 1-slot rings, the tile read two super-blocks at a
// time to fit 80 registers (8.82 against 8.72 us at 6144 x 5120).
constexpr int kSfWarps = 12, kSfDepth = 2;

// The SoA-plane GEMV with the fragment-tile structure: x is f32 packed in
// every CTA (inline_x) or x-fragments (16-byte aligned).
int launch_soa_frag(q38_devptr meta, q38_devptr qh, q38_devptr qs, const void* x, bool inline_x, float* y,
                    uint32_t cols, uint32_t rows, cudaStream_t stream) {
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    q38::SoaFragMaps maps{};
    if (int rc = soa_frag_maps(meta, qh, qs, rows, cols, &maps)) return rc;
    const uint32_t nb = cols / 256u;
    const dim3 g(std::min<uint32_t>(static_cast<uint32_t>(st->sm_count), (rows + 7u) / 8u));
    const size_t smem = q38::soa_frag_smem_bytes<kSfWarps, kSfDepth>(nb, true);
    if (smem > kChainlessSmemMaxSoa) return fail(Q38_ERR_UNSUPPORTED, "SoA GEMV: cols %u too large", cols);
    if (inline_x) {
        constexpr auto k = q38::gemv_soa_frag_kernel<2, kSfWarps, kSfDepth, 1>;
        if (int rc = ensure_smem_attr<k>(dev, kChainlessSmemMaxSoa)) return rc;
        return launch_pdl(k, g, dim3(kSfWarps * 32), smem, stream, "launch gemv_soa_frag", maps,
                          static_cast<const uint8_t*>(x), y, rows, nb);
    }
    constexpr auto k = q38::gemv_soa_frag_kernel<1, kSfWarps, kSfDepth, 1>;
    if (int rc = ensure_smem_attr<k>(dev, kChainlessSmemMaxSoa)) return rc;
    return launch_pdl(k, g, dim3(kSfWarps * 32), smem, stream, "launch gemv_soa_frag", maps,
                      static_cast<const uint8_t*>(x), y, rows, nb);
}

// Whether the fragment-structured SoA GEMV takes these columns (its x-fragments
// fit beside the rings), and whether it packs f32 x in every CTA (one launch).
bool soa_frag_fits(uint32_t cols) {
    return q38::soa_frag_smem_bytes<kSfWarps, kSfDepth>(cols / 256u, true) <= kChainlessSmemMaxSoa;
}
bool soa_inline_x(uint32_t cols, q38_devptr x) {
    return (x & 15u) == 0 && cols / 256u <= q38::kF8PackPerWarp * static_cast<uint32_t>(kSfWarps) &&
           soa_frag_fits(cols);
}

// f32 activations for the GEMVs' in-CTA packing: x alone, or x with the
// RMSNorm weight and epsilon to apply first.
struct XF32 {
    const float* x = nullptr;
    const float* nw = nullptr;
    float eps = 0.0f;
    XF32() = default;
    XF32(const float* p) : x(p) {}  // NOLINT: implicit on purpose
    XF32(const float* p, const float* w, float e) : x(p), nw(w), eps(e) {}
};

// Dynamic shared memory a layout-2 GEMV CTA may use (one CTA per SM), and
// the tile count from which the 16-warp configuration runs.
constexpr size_t kFragSmemMax = 200u * 1024u;
// A kernel that needs no co-resident next launch may take the SM's whole
// shared memory (the batched GEMM).
constexpr size_t kChainlessSmemMax = 227u * 1024u;
constexpr uint64_t kFragBigTiles = 12000;

template <uint32_t T, int XM, int W, int D, int MINB = 1>
int launch_frag_kernel(int dev, dim3 g, size_t smem, cudaStream_t stream, const uint8_t* wp, const uint8_t* xf,
                       float* y, const float* res, uint32_t rows, uint32_t nb) {
    constexpr auto kernel = q38::gemv_frag_kernel<T, XM, W, D, MINB>;
    if (int rc = ensure_smem_attr<kernel>(dev, kFragSmemMax)) return rc;
    return launch_pdl(kernel, g, dim3(W * 32), smem, stream, "launch gemv_frag", wp, xf, y, res, rows, nb);
}

// One CTA per SM of W consumer warps with 2 ring slots each (measured best on
// B200: more resident warps beat a co-resident next launch).  x-fragments are
// staged in shared memory (XM 1) or packed there from f32 (XM 2) when they fit,
// otherwise read through L1 (XM 0).  XM 2 with 12 warps keeps the registers of
// two CTAs per SM when their shared memory fits too: the next launch's CTA then
// streams its first tiles during this one's tail, which pays once the packing
// is on the critical path (6.2 vs 6.7 us on y[6144] = W[6144x5120] x).
template <uint32_t T, int W>
int launch_frag_w(int dev, dim3 g, const uint8_t* wp, const uint8_t* xf, float* y, uint32_t nb, uint32_t rows,
                  cudaStream_t stream, const float* res, bool f32_x) {
    const size_t with_x = q38::frag_smem_bytes<T, W, 2>(nb, true);
    if (f32_x) {
        if (with_x > kFragSmemMax || nb > q38::kF8PackPerWarp * W)
            return fail(Q38_ERR_UNSUPPORTED, "in-CTA x-fragment packing needs a smaller K");
        if (W == 12 && 2u * (with_x + 1024u) <= 228u * 1024u)
            return launch_frag_kernel<T, 2, W, 2, 2>(dev, g, with_x, stream, wp, xf, y, res, rows, nb);
        return launch_frag_kernel<T, 2, W, 2>(dev, g, with_x, stream, wp, xf, y, res, rows, nb);
    }
    if (with_x <= kFragSmemMax) return launch_frag_kernel<T, 1, W, 2>(dev, g, with_x, stream, wp, xf, y, res, rows, nb);
    return launch_frag_kernel<T, 0, W, 2>(dev, g, q38::frag_smem_bytes<T, W, 2>(nb, false), stream, wp, xf, y, res,
                                          rows, nb);
}

// Layout-2 GEMV y (+ res) = W x with x given as x-fragments (xfrag1 layout),
// or, with f32_x, as an f32 vector packed by every CTA (XM 2).  Matrices below
// kFragBigTiles tiles run 12 warps per CTA, larger ones 16.
template <uint32_t T>
int launch_frag_t(int dev, int sm_count, const uint8_t* wp, const uint8_t* xf, float* y, uint32_t cols, uint32_t rows,
                  cudaStream_t stream, const float* res, bool f32_x) {
    const uint32_t nb = cols / 256u;
    const uint32_t nocts = (rows + q38::kF8Rows - 1u) / q38::kF8Rows;
    const dim3 g(std::min<uint32_t>(static_cast<uint32_t>(sm_count), nocts));
    if (static_cast<uint64_t>(nocts) * (nb / 2u) < kFragBigTiles)
        return launch_frag_w<T, 12>(dev, g, wp, xf, y, nb, rows, stream, res, f32_x);
    return launch_frag_w<T, 16>(dev, g, wp, xf, y, nb, rows, stream, res, f32_x);
}

int launch_frag(uint32_t type, q38_devptr w, const uint8_t* xf, float* y, uint32_t cols, uint32_t rows,
                cudaStream_t stream, const float* res = nullptr, bool f32_x = false) {
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    const uint8_t* wp = dptr<const uint8_t>(w);
    if (type == Q38_TYPE_Q5_K) return launch_frag_t<13>(dev, st->sm_count, wp, xf, y, cols, rows, stream, res, f32_x);
    if (type == Q38_TYPE_Q6_K) return launch_frag_t<14>(dev, st->sm_count, wp, xf, y, cols, rows, stream, res, f32_x);
    if (type == Q38_TYPE_IQ4_XS)
        return launch_frag_t<23>(dev, st->sm_count, wp, xf, y, cols, rows, stream, res, f32_x);
    return launch_frag_t<12>(dev, st->sm_count, wp, xf, y, cols, rows, stream, res, f32_x);
}

// Two layout-2 GEMVs of the same K over the same x-fragments in one launch
// (gemv_frag_pair_kernel): one CTA per SM, split between the matrices in
// proportion to their tiles, x-fragments staged in shared memory.  Returns
// Q38_ERR_UNSUPPORTED when the pair has no pair kernel (the caller then runs
// two launches).
template <uint32_t TA, uint32_t TB, int W>
int launch_frag_pair_w(int dev, uint32_t ncta, uint32_t split, const q38::FragJob& a, const q38::FragJob& b,
                       const uint8_t* xf, uint32_t nb, cudaStream_t stream) {
    const size_t smem = std::max(q38::frag_smem_bytes<TA, W, 2>(nb, true), q38::frag_smem_bytes<TB, W, 2>(nb, true));
    if (smem > kFragSmemMax) return Q38_ERR_UNSUPPORTED;
    constexpr auto kernel = q38::gemv_frag_pair_kernel<TA, TB, 1, W, 2>;
    if (int rc = ensure_smem_attr<kernel>(dev, kFragSmemMax)) return rc;
    return launch_pdl(kernel, dim3(ncta), dim3(W * 32), smem, stream, "launch gemv_frag_pair", a, b, xf, nb, split);
}

template <uint32_t TA, uint32_t TB>
int launch_frag_pair_t(int dev, uint32_t ncta, uint32_t split, bool big, const q38::FragJob& a,
                       const q38::FragJob& b, const uint8_t* xf, uint32_t nb, cudaStream_t stream) {
    return big ? launch_frag_pair_w<TA, TB, 16>(dev, ncta, split, a, b, xf, nb, stream)
               : launch_frag_pair_w<TA, TB, 12>(dev, ncta, split, a, b, xf, nb, stream);
}

int launch_frag_pair(uint32_t ta, q38_devptr wa, uint32_t rows_a, float* ya, uint32_t tb, q38_devptr wb,
                     uint32_t rows_b, float* yb, const uint8_t* xf, uint32_t cols, cudaStream_t stream) {
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    const uint32_t nb = cols / 256u;
    const uint32_t octs_a = (rows_a + q38::kF8Rows - 1u) / q38::kF8Rows;
    const uint32_t octs_b = (rows_b + q38::kF8Rows - 1u) / q38::kF8Rows;
    const uint32_t ncta = std::min<uint32_t>(static_cast<uint32_t>(st->sm_count), octs_a + octs_b);
    if (ncta < 2) return Q38_ERR_UNSUPPORTED;
    const double share = static_cast<double>(octs_a) / static_cast<double>(octs_a + octs_b);
    uint32_t split = static_cast<uint32_t>(share * ncta + 0.5);
    // every CTA gets at least one row octet of its matrix
    split = std::max(split, std::max(1u, ncta > octs_b ? ncta - octs_b : 1u));
    split = std::min(split, std::min(octs_a, ncta - 1u));
    const bool big = static_cast<uint64_t>(octs_a + octs_b) * (nb / 2u) >= kFragBigTiles;
    const q38::FragJob a{dptr<const uint8_t>(wa), ya, rows_a}, b{dptr<const uint8_t>(wb), yb, rows_b};
    if (ta == Q38_TYPE_Q5_K && tb == Q38_TYPE_Q4_K)
        return launch_frag_pair_t<13, 12>(dev, ncta, split, big, a, b, xf, nb, stream);
    if (ta == Q38_TYPE_Q4_K && tb == Q38_TYPE_Q5_K)
        return launch_frag_pair_t<12, 13>(dev, ncta, split, big, a, b, xf, nb, stream);
    if (ta == Q38_TYPE_IQ4_XS && tb == Q38_TYPE_Q5_K)  // the reference model's ffn_gate with ffn_up
        return launch_frag_pair_t<23, 13>(dev, ncta, split, big, a, b, xf, nb, stream);
    return Q38_ERR_UNSUPPORTED;
}

template <int W>
int launch_frag_pair_xf_w(int dev, uint32_t ncta, uint32_t split, const q38::FragJob& a, const q38::FragJob& b,
                          const uint8_t* xfa, const float* xb, uint32_t nb, cudaStream_t stream) {
    const size_t smem = std::max(q38::frag_smem_bytes<13, W, 2>(nb, true), q38::frag_smem_bytes<14, W, 2>(nb, true));
    if (smem > kFragSmemMax || nb > q38::kF8PackPerWarp * static_cast<uint32_t>(W)) return Q38_ERR_UNSUPPORTED;
    constexpr auto kernel = q38::gemv_frag_pair_xf_kernel<13, 14, W, 2>;
    if (int rc = ensure_smem_attr<kernel>(dev, kFragSmemMax)) return rc;
    return launch_pdl(kernel, dim3(ncta), dim3(W * 32), smem, stream, "launch gemv_frag_pair_xf", a, b, xfa, xb, nb,
                      split);
}

// A Q5_K layout-2 GEMV over x-fragments xfa with a Q6_K layout-2 GEMV over f32
// x (the same activations, xb, packed in its CTAs) of the same K in one
// launch (gemv_frag_pair_xf_kernel); CTAs split in proportion to the two
// matrices' tile bytes.  Q38_ERR_UNSUPPORTED for other pairs or shapes (the
// caller then runs two launches).
int launch_frag_pair_xf(uint32_t ta, q38_devptr wa, uint32_t rows_a, float* ya, uint32_t tb, q38_devptr wb,
                        uint32_t rows_b, float* yb, const uint8_t* xfa, const float* xb, uint32_t cols,
                        cudaStream_t stream) {
    if (ta != Q38_TYPE_Q5_K || tb != Q38_TYPE_Q6_K || (reinterpret_cast<uintptr_t>(xb) & 15u))
        return Q38_ERR_UNSUPPORTED;
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    const uint32_t nb = cols / 256u;
    const uint32_t octs_a = (rows_a + q38::kF8Rows - 1u) / q38::kF8Rows;
    const uint32_t octs_b = (rows_b + q38::kF8Rows - 1u) / q38::kF8Rows;
    const uint32_t ncta = std::min<uint32_t>(static_cast<uint32_t>(st->sm_count), octs_a + octs_b);
    if (ncta < 2) return Q38_ERR_UNSUPPORTED;
    const double ba = static_cast<double>(octs_a) * q38::FragTile<13>::kBytes;
    const double bb = static_cast<double>(octs_b) * q38::FragTile<14>::kBytes;
    uint32_t split = static_cast<uint32_t>(ba / (ba + bb) * ncta + 0.5);
    split = std::max(split, std::max(1u, ncta > octs_b ? ncta - octs_b : 1u));
    split = std::min(split, std::min(octs_a, ncta - 1u));
    const bool big = static_cast<uint64_t>(octs_a + octs_b) * (nb / 2u) >= kFragBigTiles;
    const q38::FragJob a{dptr<const uint8_t>(wa), ya, rows_a}, b{dptr<const uint8_t>(wb), yb, rows_b};
    return big ? launch_frag_pair_xf_w<16>(dev, ncta, split, a, b, xfa, xb, nb, stream)
               : launch_frag_pair_xf_w<12>(dev, ncta, split, a, b, xfa, xb, nb, stream);
}

// Whether the f32 GEMV over layout 2 packs x inside every CTA (one kernel):
// the x-fragments fit next to the 16-warp ring and each of 12 warps packs at
// most kF8PackPerWarp super-blocks.
bool frag_inline_x(uint32_t type, uint32_t cols) {
    const uint32_t nb = cols / 256u;
    if (nb > q38::kF8PackPerWarp * 12u) return false;
    return type == Q38_TYPE_Q5_K   ? q38::frag_smem_bytes<13, 16, 2>(nb, true) <= kFragSmemMax
           : type == Q38_TYPE_Q6_K ? q38::frag_smem_bytes<14, 16, 2>(nb, true) <= kFragSmemMax
           : type == Q38_TYPE_IQ4_XS ? q38::frag_smem_bytes<23, 16, 2>(nb, true) <= kFragSmemMax
                                   : q38::frag_smem_bytes<12, 16, 2>(nb, true) <= kFragSmemMax;
}

// Layout 2 holds Q5_K, Q4_K, Q6_K and IQ4_XS matrices with cols a multiple of 512.
int check_frag_args(uint32_t type, q38_devptr w, uint32_t cols, uint32_t rows) {
    if (type != Q38_TYPE_Q5_K && type != Q38_TYPE_Q4_K && type != Q38_TYPE_Q6_K && type != Q38_TYPE_IQ4_XS)
        return fail(Q38_ERR_UNSUPPORTED, "layout 2 holds Q5_K, Q4_K, Q6_K and IQ4_XS matrices (got type %u)", type);
    if (rows == 0 || cols == 0 || cols % 512u)
        return fail(Q38_ERR_INVALID, "layout-2 GEMV needs rows > 0 and cols a positive multiple of 512 (got %u x %u)",
                    rows, cols);
    if (!w) return fail(Q38_ERR_INVALID, "layout-2 weight pointer is null");
    if (w & 15u) return fail(Q38_ERR_INVALID, "layout-2 weights must be 16-byte aligned");
    return Q38_OK;
}

// cudaFuncSetAttribute(max dynamic shared memory) for a kernel passed by value.
template <class K>
int ensure_smem_attr_dyn(K kernel, int dev, size_t bytes) {
    (void)dev;
    Q38_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
             "cudaFuncSetAttribute(max dynamic shared memory)");
    return Q38_OK;
}

template <int T, int NL, int XM>
int launch_kq_kernel(int dev, dim3 g, size_t smem, cudaStream_t stream, const uint8_t* wp, const uint8_t* xl,
                     const float* gs, const float* sc, float* y, const float* res, uint32_t rows, uint32_t nb,
                     float eps = 0.0f) {
    if (int rc = ensure_smem_attr<q38::gemv_kq_kernel<T, NL, XM>>(dev, q38::kSmemBudget + 1024)) return rc;
    return launch_pdl(q38::gemv_kq_kernel<T, NL, XM>, g, dim3(q38::KqType<T>::kWarps * 32u), smem, stream,
                      "launch gemv_kq", wp, xl, gs, sc, y, res, rows, nb, eps);
}

// Very large Q6_K matrices (the vocabulary projection) run one CTA of 20
// warps per SM: the Q6_K decode is compute-heavy and gains from more resident
// warps (measured 247 -> 217 us on a 151936 x 5120 lm_head).
constexpr uint32_t kKqWideRows = 32768;
constexpr int kKqWideWarps = 20;

template <int T, int NL, int XM>
int launch_kq_wide(int dev, int sm_count, const uint8_t* wp, const XPackView& xv, float* y, uint32_t nb,
                   uint32_t rows, cudaStream_t stream, const float* res) {
    constexpr auto kernel = q38::gemv_kq_kernel<T, NL, XM, kKqWideWarps, 1>;
    const size_t smem = q38::kq_smem_bytes<T, kKqWideWarps>(nb, NL, XM == 1);
    if (int rc = ensure_smem_attr<kernel>(dev, 200u * 1024u)) return rc;
    const dim3 g(std::min<uint32_t>(static_cast<uint32_t>(sm_count), (rows + 1u) / 2u));
    return launch_pdl(kernel, g, dim3(kKqWideWarps * 32u), smem, stream, "launch gemv_kq (wide)", wp, xv.limbs,
                      xv.gsum, xv.scale, y, res, rows, nb, 0.0f);
}

// Layout-0 K-quant GEMV.  xf32 != nullptr: f32 x packed inside every CTA
// (needs kq_smem_bytes(nb, 3, true) within the budget); else the x-pack xv.
template <int T>
int launch_kq_t(int dev, int sm_count, const uint8_t* wp, const XPackView& xv, uint32_t nl, float* y, uint32_t nb,
                uint32_t rows, cudaStream_t stream, const XF32& xf, const float* res) {
    const bool xsmem = q38::kq_smem_bytes<T>(nb, static_cast<int>(nl), true) <= q38::kSmemBudget;
    const size_t smem = q38::kq_smem_bytes<T>(nb, static_cast<int>(nl), xsmem);
    const uint32_t npairs = (rows + 1u) / 2u;
    const dim3 g(std::min<uint32_t>(static_cast<uint32_t>(sm_count), npairs));
    if (xf.x) {
        if (!xsmem) return fail(Q38_ERR_UNSUPPORTED, "in-CTA activation packing: cols %u too large", nb * 256u);
        const uint8_t* xb = reinterpret_cast<const uint8_t*>(xf.x);
        if (xf.nw)
            return launch_kq_kernel<T, 3, 3>(dev, g, smem, stream, wp, xb, xf.nw, nullptr, y, res, rows, nb, xf.eps);
        return launch_kq_kernel<T, 3, 2>(dev, g, smem, stream, wp, xb, nullptr, nullptr, y, res, rows, nb);
    }
    if constexpr (T == 14) {
        if (rows >= kKqWideRows && nl == 4 && q38::kq_smem_bytes<T, kKqWideWarps>(nb, 4, true) <= 200u * 1024u)
            return launch_kq_wide<T, 4, 1>(dev, sm_count, wp, xv, y, nb, rows, stream, res);
        if (rows >= kKqWideRows && nl == 3 && q38::kq_smem_bytes<T, kKqWideWarps>(nb, 3, true) <= 200u * 1024u)
            return launch_kq_wide<T, 3, 1>(dev, sm_count, wp, xv, y, nb, rows, stream, res);
    }
    if (nl == 4)
        return xsmem ? launch_kq_kernel<T, 4, 1>(dev, g, smem, stream, wp, xv.limbs, xv.gsum, xv.scale, y, res, rows, nb)
                     : launch_kq_kernel<T, 4, 0>(dev, g, smem, stream, wp, xv.limbs, xv.gsum, xv.scale, y, res, rows, nb);
    if (nl == 3)
        return xsmem ? launch_kq_kernel<T, 3, 1>(dev, g, smem, stream, wp, xv.limbs, xv.gsum, xv.scale, y, res, rows, nb)
                     : launch_kq_kernel<T, 3, 0>(dev, g, smem, stream, wp, xv.limbs, xv.gsum, xv.scale, y, res, rows, nb);
    return xsmem ? launch_kq_kernel<T, 1, 1>(dev, g, smem, stream, wp, xv.limbs, xv.gsum, xv.scale, y, res, rows, nb)
                 : launch_kq_kernel<T, 1, 0>(dev, g, smem, stream, wp, xv.limbs, xv.gsum, xv.scale, y, res, rows, nb);
}

bool kq_type_supported(uint32_t t) {
    return t == Q38_TYPE_Q4_K || t == Q38_TYPE_Q5_K || t == Q38_TYPE_Q6_K || t == Q38_TYPE_IQ4_XS;
}

// True when f32 x of `cols` can be packed inside every CTA of the layout-0 kernel.
bool kq_inline_x(uint32_t type, uint32_t cols) {
    const uint32_t nb = cols / 256u;
    switch (type) {
        case Q38_TYPE_Q4_K: return q38::kq_smem_bytes<12>(nb, 3, true) <= q38::kSmemBudget;
        case Q38_TYPE_Q5_K: return q38::kq_smem_bytes<13>(nb, 3, true) <= q38::kSmemBudget;
        case Q38_TYPE_Q6_K: return q38::kq_smem_bytes<14>(nb, 3, true) <= q38::kSmemBudget;
        case Q38_TYPE_IQ4_XS: return q38::kq_smem_bytes<23>(nb, 3, true) <= q38::kSmemBudget;
        default: return false;
    }
}

int check_kq_args(uint32_t type, q38_devptr w, uint32_t cols, uint32_t rows) {
    if (!kq_type_supported(type)) return fail(Q38_ERR_UNSUPPORTED, "ggml type %u has no layout-0 GEMV", type);
    if (rows == 0 || cols == 0 || cols % 256u)
        return fail(Q38_ERR_INVALID, "GEMV needs rows > 0 and cols a positive multiple of 256 (got %u x %u)", rows,
                    cols);
    if (!w) return fail(Q38_ERR_INVALID, "weight pointer is null");
    if (w & 15u) return fail(Q38_ERR_INVALID, "weights must be 16-byte aligned");
    return Q38_OK;
}

int launch_kq(uint32_t type, q38_devptr w, const XPackView& xv, uint32_t nl, float* y, uint32_t cols, uint32_t rows,
              cudaStream_t stream, const XF32& xf = XF32(), const float* res = nullptr) {
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    const uint8_t* wp = dptr<const uint8_t>(w);
    const uint32_t nb = cols / 256u;
    switch (type) {
        case Q38_TYPE_Q4_K: return launch_kq_t<12>(dev, st->sm_count, wp, xv, nl, y, nb, rows, stream, xf, res);
        case Q38_TYPE_Q5_K: return launch_kq_t<13>(dev, st->sm_count, wp, xv, nl, y, nb, rows, stream, xf, res);
        case Q38_TYPE_Q6_K: return launch_kq_t<14>(dev, st->sm_count, wp, xv, nl, y, nb, rows, stream, xf, res);
        case Q38_TYPE_IQ4_XS: return launch_kq_t<23>(dev, st->sm_count, wp, xv, nl, y, nb, rows, stream, xf, res);
        default: return fail(Q38_ERR_UNSUPPORTED, "ggml type %u has no layout-0 GEMV", type);
    }
}

// f32 x through the per-device workspace: x-pack kernel, then the GEMV.
int kq_f32_via_workspace(uint32_t type, q38_devptr w, q38_devptr x, float* y, uint32_t cols, uint32_t rows,
                         q38_stream stream) {
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    void* ws = nullptr;
    const uint32_t nl = f32_limbs(cols);
    if (int rc = ensure_workspace(st, q38_xpack_bytes(nl, cols, 1), &ws)) return rc;
    const q38_devptr wsp = static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(ws));
    if (int rc = q38_xpack_f32_limbs(x, cols, 1, nl, wsp, stream)) return rc;
    return launch_kq(type, w, xpack_view(ws, nl, cols / 256u, 1), nl, y, cols, rows, as_stream(stream));
}

struct VmmAlloc {
    CUmemGenericAllocationHandle handle;
    size_t bytes;
};

}  // namespace

struct q38_ctx {
    int device = 0;
    size_t granularity = 0;
    std::unordered_map<uint64_t, VmmAlloc> allocs;
};

extern "C" {

const char* q38_last_error(void) { return g_last_error.c_str(); }

const char* q38_version(void) { return "q38rt-b200 0.1 sm_100a"; }

int q38_device_count(int* count) {
    if (!count) return fail(Q38_ERR_INVALID, "count is null");
    *count = 0;
    Q38_CUDA(cudaGetDeviceCount(count), "cudaGetDeviceCount");
    return Q38_OK;
}

int q38_device_query(int device, q38_device_info* info) {
    if (!info) return fail(Q38_ERR_INVALID, "info is null");
    memset(info, 0, sizeof(*info));
    cudaDeviceProp prop{};
    Q38_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    info->ordinal = device;
    info->sm_major = prop.major;
    info->sm_minor = prop.minor;
    info->sm_count = prop.multiProcessorCount;
    info->total_memory = prop.totalGlobalMem;
    info->l2_bytes = static_cast<size_t>(prop.l2CacheSize);
    snprintf(info->name, sizeof(info->name), "%s", prop.name);
    int drv = 0;
    cudaDriverGetVersion(&drv);
    info->driver_version = drv;
    DriverApi* d = nullptr;
    if (driver_api(&d) == Q38_OK) {
        CUmemAllocationProp p{};
        p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
        p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        p.location.id = device;
        size_t g = 0;
        if (d->memGetAllocationGranularity(&g, &p, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) == CUDA_SUCCESS) {
            info->vmm_granularity = g;
            info->vmm_supported = 1;
        }
    }
    return Q38_OK;
}

int q38_scratch_bytes(int device, size_t* bytes) {
    if (!bytes || device < 0) return fail(Q38_ERR_INVALID, "q38_scratch_bytes: bad arguments");
    std::lock_guard<std::mutex> lk(g_mu);
    *bytes = static_cast<size_t>(device) < g_dev.size()
                 ? g_dev[device].workspace_bytes + g_dev[device].io_bytes
                 : 0u;
    return Q38_OK;
}

int q38_ctx_open(int device, q38_ctx** out) {
    if (!out) return fail(Q38_ERR_INVALID, "out is null");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= n) return fail(Q38_ERR_NO_DEVICE, "device %d out of range (count %d)", device, n);
    Q38_CUDA(cudaSetDevice(device), "cudaSetDevice");
    Q38_CUDA(cudaFree(nullptr), "context init");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    q38_device_info info{};
    if (int rc = q38_device_query(device, &info)) return rc;
    auto* c = new q38_ctx();
    c->device = device;
    c->granularity = info.vmm_granularity ? info.vmm_granularity : (2u << 20);
    *out = c;
    return Q38_OK;
}

int q38_ctx_close(q38_ctx* ctx) {
    if (!ctx) return Q38_OK;
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    DriverApi* d = nullptr;
    if (driver_api(&d) == Q38_OK) {
        for (auto& kv : ctx->allocs) {
            d->memUnmap(static_cast<CUdeviceptr>(kv.first), kv.second.bytes);
            d->memAddressFree(static_cast<CUdeviceptr>(kv.first), kv.second.bytes);
            d->memRelease(kv.second.handle);
        }
    }
    delete ctx;
    return Q38_OK;
}

int q38_alloc(q38_ctx* ctx, size_t bytes, q38_devptr* out) {
    if (!ctx || !out || bytes == 0) return fail(Q38_ERR_INVALID, "q38_alloc: bad arguments");
    DriverApi* d = nullptr;
    if (int rc = driver_api(&d)) return rc;
    const size_t g = ctx->granularity;
    const size_t size = (bytes + g - 1) / g * g;
    CUmemAllocationProp prop{};
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = ctx->device;
    CUmemGenericAllocationHandle h{};
    CUresult r = d->memCreate(&h, size, &prop, 0);
    if (r != CUDA_SUCCESS) return cu_fail(r, "cuMemCreate");
    CUdeviceptr va = 0;
    r = d->memAddressReserve(&va, size, g, 0, 0);
    if (r != CUDA_SUCCESS) {
        d->memRelease(h);
        return cu_fail(r, "cuMemAddressReserve");
    }
    r = d->memMap(va, size, 0, h, 0);
    if (r != CUDA_SUCCESS) {
        d->memAddressFree(va, size);
        d->memRelease(h);
        return cu_fail(r, "cuMemMap");
    }
    CUmemAccessDesc acc{};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = ctx->device;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    r = d->memSetAccess(va, size, &acc, 1);
    if (r != CUDA_SUCCESS) {
        d->memUnmap(va, size);
        d->memAddressFree(va, size);
        d->memRelease(h);
        return cu_fail(r, "cuMemSetAccess");
    }
    ctx->allocs[static_cast<uint64_t>(va)] = VmmAlloc{h, size};
    *out = static_cast<q38_devptr>(va);
    return Q38_OK;
}

int q38_free(q38_ctx* ctx, q38_devptr ptr) {
    if (!ctx) return fail(Q38_ERR_INVALID, "q38_free: ctx is null");
    auto it = ctx->allocs.find(ptr);
    if (it == ctx->allocs.end()) return fail(Q38_ERR_INVALID, "q38_free: pointer not owned by this context");
    DriverApi* d = nullptr;
    if (int rc = driver_api(&d)) return rc;
    cudaDeviceSynchronize();
    d->memUnmap(static_cast<CUdeviceptr>(ptr), it->second.bytes);
    d->memAddressFree(static_cast<CUdeviceptr>(ptr), it->second.bytes);
    d->memRelease(it->second.handle);
    ctx->allocs.erase(it);
    return Q38_OK;
}

int q38_memcpy_h2d(q38_devptr dst, const void* src, size_t bytes, q38_stream stream) {
    Q38_CUDA(cudaMemcpyAsync(dptr<void>(dst), src, bytes, cudaMemcpyHostToDevice, as_stream(stream)),
             "cudaMemcpyAsync(H2D)");
    return Q38_OK;
}

int q38_memcpy_d2h(void* dst, q38_devptr src, size_t bytes, q38_stream stream) {
    Q38_CUDA(cudaMemcpyAsync(dst, dptr<void>(src), bytes, cudaMemcpyDeviceToHost, as_stream(stream)),
             "cudaMemcpyAsync(D2H)");
    return Q38_OK;
}

int q38_memcpy_d2d(q38_devptr dst, q38_devptr src, size_t bytes, q38_stream stream) {
    Q38_CUDA(cudaMemcpyAsync(dptr<void>(dst), dptr<void>(src), bytes, cudaMemcpyDeviceToDevice, as_stream(stream)),
             "cudaMemcpyAsync(D2D)");
    return Q38_OK;
}

int q38_memset_d8(q38_devptr dst, uint8_t value, size_t bytes, q38_stream stream) {
    Q38_CUDA(cudaMemsetAsync(dptr<void>(dst), value, bytes, as_stream(stream)), "cudaMemsetAsync");
    return Q38_OK;
}

int q38_stream_synchronize(q38_stream stream) {
    Q38_CUDA(cudaStreamSynchronize(as_stream(stream)), "cudaStreamSynchronize");
    return Q38_OK;
}

int q38_fault_status(uint32_t* site) {
    if (!site) return fail(Q38_ERR_INVALID, "site is null");
    Q38_CUDA(cudaMemcpyFromSymbol(site, q38::g_q38_fault, sizeof(uint32_t)), "read fault word");
    return Q38_OK;
}

int q38_fault_clear(void) {
    const uint32_t zero = 0;
    Q38_CUDA(cudaMemcpyToSymbol(q38::g_q38_fault, &zero, sizeof(uint32_t)), "clear fault word");
    return Q38_OK;
}

size_t q38_xpack_bytes(uint32_t nl, uint32_t cols, uint32_t batch) {
    if ((nl != 1 && nl != 3 && nl != 4) || cols % 256u) return 0;
    const uint32_t nb = cols / 256u;
    size_t b = (q38::xpack_limb_bytes(static_cast<int>(nl), nb, batch) + 255u) & ~size_t(255);
    b += (static_cast<size_t>(batch) * nb * 32u + 255u) & ~size_t(255);
    b += (static_cast<size_t>(batch) * nb * 4u + 255u) & ~size_t(255);
    return b;
}

int q38_xpack_f32_limbs(q38_devptr x, uint32_t cols, uint32_t batch, uint32_t nl, q38_devptr xpack,
                        q38_stream stream) {
    if (!x || !xpack || cols == 0 || cols % 256u || batch == 0)
        return fail(Q38_ERR_INVALID, "q38_xpack_f32: bad arguments");
    if (nl != 3 && nl != 4) return fail(Q38_ERR_INVALID, "q38_xpack_f32_limbs: nl must be 3 or 4 (got %u)", nl);
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    const uint32_t nb = cols / 256u;
    XPackView v = xpack_view(dptr<void>(xpack), nl, nb, batch);
    if (nl == 4)
        return launch_pdl(q38::xpack_f32_kernel<4>, dim3(nb, batch), dim3(256), 0, as_stream(stream),
                          "launch xpack_f32<4>", static_cast<const float*>(dptr<float>(x)), cols, v.limbs, v.gsum,
                          v.scale);
    return launch_pdl(q38::xpack_f32_kernel<3>, dim3(nb, batch), dim3(256), 0, as_stream(stream), "launch xpack_f32<3>",
                      static_cast<const float*>(dptr<float>(x)), cols, v.limbs, v.gsum, v.scale);
}

int q38_xpack_f32(q38_devptr x, uint32_t cols, uint32_t batch, q38_devptr xpack, q38_stream stream) {
    return q38_xpack_f32_limbs(x, cols, batch, 3, xpack, stream);
}

int q38_xpack_q8k(q38_devptr xq8, uint32_t cols, uint32_t batch, q38_devptr xpack, q38_stream stream) {
    if (!xq8 || !xpack || cols == 0 || cols % 256u || batch == 0)
        return fail(Q38_ERR_INVALID, "q38_xpack_q8k: bad arguments");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    const uint32_t nb = cols / 256u;
    XPackView v = xpack_view(dptr<void>(xpack), 1, nb, batch);
    return launch_pdl(q38::xpack_q8k_kernel, dim3(nb, batch), dim3(256), 0, as_stream(stream), "launch xpack_q8k",
                      static_cast<const uint8_t*>(dptr<uint8_t>(xq8)), nb, v.limbs, v.gsum, v.scale);
}

int q38_gemv_packed(const q38_weight_desc* w, q38_devptr xpack, uint32_t nl, uint32_t batch, q38_devptr y,
                    q38_stream stream) {
    if (!w || !xpack || !y) return fail(Q38_ERR_INVALID, "q38_gemv_packed: null argument");
    if (nl != 1 && nl != 3 && nl != 4) return fail(Q38_ERR_INVALID, "q38_gemv_packed: nl must be 1, 3 or 4");
    if (batch != 1) return fail(Q38_ERR_UNSUPPORTED, "q38_gemv_packed: batch %u not supported yet", batch);
    if (xpack & 15u) return fail(Q38_ERR_INVALID, "q38_gemv_packed: x-pack must be 16-byte aligned");
    if (w->layout == Q38_LAYOUT_GGUF_NATIVE && kq_type_supported(w->ggml_type)) {
        if (int rc = check_kq_args(w->ggml_type, w->data, w->cols, w->rows)) return rc;
        return launch_kq(w->ggml_type, w->data, xpack_view(dptr<void>(xpack), nl, w->cols / 256u, batch), nl,
                         dptr<float>(y), w->cols, w->rows, as_stream(stream));
    }
    if (w->ggml_type == Q38_TYPE_Q5_K && w->layout == Q38_LAYOUT_SM86_Q5K_SOA) {
        if (int rc = check_soa_args(w->data, w->aux0, w->aux1, w->cols, w->rows)) return rc;
        XPackView v = xpack_view(dptr<void>(xpack), nl, w->cols / 256u, batch);
        return launch_soa_packed(w->data, w->aux0, w->aux1, v, nl, dptr<float>(y), w->cols, w->rows,
                                 as_stream(stream));
    }
    if (w->layout == Q38_LAYOUT_B200_TILED)
        return fail(Q38_ERR_UNSUPPORTED, "q38_gemv_packed: layout-2 weights take x-fragments (q38_gemv_xfrag)");
    return fail(Q38_ERR_UNSUPPORTED, "q38_gemv_packed: type %u layout %u not supported", w->ggml_type, w->layout);
}

size_t q38_xfrag_bytes(uint32_t cols, uint32_t batch) {
    if (cols == 0 || cols % 256u || batch == 0) return 0;
    return q38::xfrag1_bytes(cols / 256u) * batch;
}

int q38_xfrag_f32(q38_devptr x, uint32_t cols, uint32_t batch, q38_devptr xfrag, q38_stream stream) {
    if (!x || !xfrag || cols == 0 || cols % 256u || batch == 0)
        return fail(Q38_ERR_INVALID, "q38_xfrag_f32: bad arguments");
    if ((x | xfrag) & 15u) return fail(Q38_ERR_INVALID, "q38_xfrag_f32: x and xfrag must be 16-byte aligned");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    const uint32_t warps = cols / 256u * batch;
    return launch_pdl(q38::xfrag1_f32_kernel, dim3((warps + 7u) / 8u), dim3(256), 0, as_stream(stream),
                      "launch xfrag1_f32", dptr<const float>(x), cols, batch, dptr<uint8_t>(xfrag));
}

int q38_xfrag_q8k(q38_devptr xq8, uint32_t cols, uint32_t batch, q38_devptr xfrag, q38_stream stream) {
    if (!xq8 || !xfrag || cols == 0 || cols % 256u || batch == 0)
        return fail(Q38_ERR_INVALID, "q38_xfrag_q8k: bad arguments");
    if ((xq8 & 3u) || (xfrag & 15u))
        return fail(Q38_ERR_INVALID, "q38_xfrag_q8k: xq8 must be 4-byte and xfrag 16-byte aligned");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    const uint32_t nb = cols / 256u, warps = nb * batch;
    return launch_pdl(q38::xfrag1_q8k_kernel, dim3((warps + 7u) / 8u), dim3(256), 0, as_stream(stream),
                      "launch xfrag1_q8k", dptr<const uint8_t>(xq8), nb, batch, dptr<uint8_t>(xfrag));
}

int q38_gemv_xfrag(const q38_weight_desc* w, q38_devptr xfrag, q38_devptr y, q38_stream stream) {
    if (!w || !xfrag || !y) return fail(Q38_ERR_INVALID, "q38_gemv_xfrag: null argument");
    if (w->layout != Q38_LAYOUT_B200_TILED)
        return fail(Q38_ERR_UNSUPPORTED, "q38_gemv_xfrag: layout %u (x-fragments feed layout 2)", w->layout);
    if (xfrag & 15u) return fail(Q38_ERR_INVALID, "q38_gemv_xfrag: x-fragments must be 16-byte aligned");
    if (int rc = check_frag_args(w->ggml_type, w->data, w->cols, w->rows)) return rc;
    if (w->ggml_type == Q38_TYPE_Q6_K)
        return fail(Q38_ERR_UNSUPPORTED,
                    "q38_gemv_xfrag: Q6_K tiles read 16-weight-group activations; use q38_gemv_f32 or q38_gemv_q8k");
    return launch_frag(w->ggml_type, w->data, dptr<uint8_t>(xfrag), dptr<float>(y), w->cols, w->rows,
                       as_stream(stream));
}

int q38_q5k_sm86_soa_gemv_vec(q38_devptr meta, q38_devptr qh, q38_devptr qs, q38_devptr x, q38_devptr y,
                              uint32_t cols, uint32_t rows, q38_stream stream) {
    if (int rc = check_soa_args(meta, qh, qs, cols, rows)) return rc;
    if (!x || !y) return fail(Q38_ERR_INVALID, "x or y is null");
    if (soa_inline_x(cols, x))  // one kernel: x packed into x-fragments by every CTA
        return launch_soa_frag(meta, qh, qs, dptr<void>(x), true, dptr<float>(y), cols, rows, as_stream(stream));
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    void* ws = nullptr;
    if ((x & 15u) == 0 && soa_frag_fits(cols)) {  // x-fragments into the workspace, then the GEMV
        if (int rc = ensure_workspace(st, q38::xfrag1_bytes(cols / 256u), &ws)) return rc;
        if (int rc = q38_xfrag_f32(x, cols, 1, static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(ws)), stream))
            return rc;
        return launch_soa_frag(meta, qh, qs, ws, false, dptr<float>(y), cols, rows, as_stream(stream));
    }
    const uint32_t nl = f32_limbs(cols);  // x not 16-byte aligned, or K too long: the x-pack path
    if (int rc = ensure_workspace(st, q38_xpack_bytes(nl, cols, 1), &ws)) return rc;
    const q38_devptr wsp = static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(ws));
    if (int rc = q38_xpack_f32_limbs(x, cols, 1, nl, wsp, stream)) return rc;
    XPackView v = xpack_view(ws, nl, cols / 256u, 1);
    return launch_soa_packed(meta, qh, qs, v, nl, dptr<float>(y), cols, rows, as_stream(stream));
}

// Layout-2 GEMV with f32 x: x-fragments into the workspace, then the GEMV.
static int frag_gemv_f32(uint32_t type, q38_devptr w, q38_devptr x, q38_devptr y, uint32_t cols, uint32_t rows,
                         q38_stream stream) {
    if (int rc = check_frag_args(type, w, cols, rows)) return rc;
    if (!x || !y) return fail(Q38_ERR_INVALID, "x or y is null");
    if (x & 15u) return fail(Q38_ERR_INVALID, "x must be 16-byte aligned");
    if (frag_inline_x(type, cols))  // one kernel: x packed into x-fragments by every CTA
        return launch_frag(type, w, dptr<const uint8_t>(x), dptr<float>(y), cols, rows, as_stream(stream), nullptr,
                           true);
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    void* ws = nullptr;
    if (int rc = ensure_workspace(st, q38::xfrag_bytes_t(type, cols / 256u), &ws)) return rc;
    const q38_devptr wsp = static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(ws));
    if (type == Q38_TYPE_Q6_K) {  // Q6 x-fragments (16-weight groups)
        const uint32_t warps = cols / 256u;
        if (int rc = launch_pdl(q38::x6frag_f32_kernel, dim3((warps + 7u) / 8u), dim3(256), 0, as_stream(stream),
                                "launch x6frag_f32", dptr<const float>(x), cols, 1u, static_cast<uint8_t*>(ws)))
            return rc;
    } else if (int rc = q38_xfrag_f32(x, cols, 1, wsp, stream)) {
        return rc;
    }
    return launch_frag(type, w, static_cast<const uint8_t*>(ws), dptr<float>(y), cols, rows, as_stream(stream));
}

int q38_q5k_tiled_gemv(q38_devptr w, q38_devptr x, q38_devptr y, uint32_t cols, uint32_t rows, q38_stream stream) {
    return frag_gemv_f32(Q38_TYPE_Q5_K, w, x, y, cols, rows, stream);
}

int q38_q5k_sm86_soa_gemv_vec_noalloc(q38_devptr meta, q38_devptr qh, q38_devptr qs, q38_devptr x, q38_devptr y,
                                      uint32_t cols, uint32_t rows, q38_stream stream) {
    if (int rc = check_soa_args(meta, qh, qs, cols, rows)) return rc;
    if (!x || !y) return fail(Q38_ERR_INVALID, "x or y is null");
    if (cols > kNoAllocMaxCols)
        return fail(Q38_ERR_INVALID,
                    "q38_q5k_sm86_soa_gemv_vec_noalloc: cols %u exceeds the fixed x-pack scratch (at most %u columns, "
                    "%zu bytes); use q38_q5k_sm86_soa_gemv_vec",
                    cols, kNoAllocMaxCols, kNoAllocXpackBytes);
    // the kernels and activation paths of q38_q5k_sm86_soa_gemv_vec, so the
    // results are the same bits; the fixed scratch stands in for the workspace
    if (soa_inline_x(cols, x))  // needs no scratch at all
        return launch_soa_frag(meta, qh, qs, dptr<void>(x), true, dptr<float>(y), cols, rows, as_stream(stream));
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    void* ws = nullptr;
    if (int rc = noalloc_scratch(st, &ws)) return rc;
    const q38_devptr wsp = static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(ws));
    if ((x & 15u) == 0 && soa_frag_fits(cols)) {
        static_assert(q38::xfrag1_bytes(kNoAllocMaxCols / 256u) <= kNoAllocXpackBytes ||
                          q38::soa_frag_fixed_bytes<kSfWarps, kSfDepth>() + q38::xfrag1_bytes(kNoAllocXpackBytes / 1088u) >
                              kChainlessSmemMaxSoa,
                      "x-fragments of every width the fragment SoA kernel takes fit in the no-alloc scratch");
        if (int rc = q38_xfrag_f32(x, cols, 1, wsp, stream)) return rc;
        return launch_soa_frag(meta, qh, qs, ws, false, dptr<float>(y), cols, rows, as_stream(stream));
    }
    const uint32_t nl = f32_limbs(cols);
    if (int rc = q38_xpack_f32_limbs(x, cols, 1, nl, wsp, stream)) return rc;
    XPackView v = xpack_view(ws, nl, cols / 256u, 1);
    return launch_soa_packed(meta, qh, qs, v, nl, dptr<float>(y), cols, rows, as_stream(stream));
}

int q38_gemv_f32(const q38_weight_desc* w, q38_devptr x, q38_devptr y, q38_stream stream) {
    if (!w || !x || !y) return fail(Q38_ERR_INVALID, "q38_gemv_f32: null argument");
    if (x & 15u) return fail(Q38_ERR_INVALID, "q38_gemv_f32: x must be 16-byte aligned");
    if (w->layout == Q38_LAYOUT_SM86_Q5K_SOA && w->ggml_type == Q38_TYPE_Q5_K)
        return q38_q5k_sm86_soa_gemv_vec(w->data, w->aux0, w->aux1, x, y, w->cols, w->rows, stream);
    if (w->layout == Q38_LAYOUT_B200_TILED)
        return frag_gemv_f32(w->ggml_type, w->data, x, y, w->cols, w->rows, stream);
    if (w->layout != Q38_LAYOUT_GGUF_NATIVE)
        return fail(Q38_ERR_UNSUPPORTED, "q38_gemv_f32: type %u layout %u not supported", w->ggml_type, w->layout);
    if (int rc = check_kq_args(w->ggml_type, w->data, w->cols, w->rows)) return rc;
    if (kq_inline_x(w->ggml_type, w->cols))
        return launch_kq(w->ggml_type, w->data, XPackView{}, 3, dptr<float>(y), w->cols, w->rows, as_stream(stream),
                         dptr<float>(x));
    return kq_f32_via_workspace(w->ggml_type, w->data, x, dptr<float>(y), w->cols, w->rows, stream);
}

int q38_gemv_xfrag_pair(const q38_weight_desc* wa, const q38_weight_desc* wb, q38_devptr xfrag, q38_devptr ya,
                        q38_devptr yb, q38_stream stream) {
    if (!wa || !wb || !xfrag || !ya || !yb) return fail(Q38_ERR_INVALID, "q38_gemv_xfrag_pair: null argument");
    if (wa->layout != Q38_LAYOUT_B200_TILED || wb->layout != Q38_LAYOUT_B200_TILED || wa->cols != wb->cols)
        return fail(Q38_ERR_INVALID, "q38_gemv_xfrag_pair: two layout-2 matrices of the same cols");
    if (int rc = check_frag_args(wa->ggml_type, wa->data, wa->cols, wa->rows)) return rc;
    if (int rc = check_frag_args(wb->ggml_type, wb->data, wb->cols, wb->rows)) return rc;
    if ((xfrag | ya | yb) & 15u) return fail(Q38_ERR_INVALID, "q38_gemv_xfrag_pair: buffers must be 16-byte aligned");
    const int rc = launch_frag_pair(wa->ggml_type, wa->data, wa->rows, dptr<float>(ya), wb->ggml_type, wb->data,
                                    wb->rows, dptr<float>(yb), dptr<const uint8_t>(xfrag), wa->cols, as_stream(stream));
    if (rc == Q38_ERR_UNSUPPORTED)
        return fail(Q38_ERR_UNSUPPORTED,
                    "q38_gemv_xfrag_pair: pairs are Q5_K with Q4_K (either order) or IQ4_XS then Q5_K, K <= 6144");
    return rc;
}

int q38_check_rows(const q38_weight_desc* w, uint32_t nrows, q38_devptr x, q38_devptr y64, q38_devptr deq,
                   q38_stream stream) {
    if (!w || !w->data || nrows == 0 || nrows > w->rows || w->cols == 0 || w->cols % 256u || (!x && !deq) ||
        (x && !y64))
        return fail(Q38_ERR_INVALID, "q38_check_rows: bad arguments");
    const bool soa = w->layout == Q38_LAYOUT_SM86_Q5K_SOA && w->ggml_type == Q38_TYPE_Q5_K;
    const bool native = w->layout == Q38_LAYOUT_GGUF_NATIVE &&
                        (w->ggml_type == Q38_TYPE_Q4_K || w->ggml_type == Q38_TYPE_Q5_K ||
                         w->ggml_type == Q38_TYPE_Q6_K || w->ggml_type == Q38_TYPE_IQ4_XS);
    if (!soa && !native) return fail(Q38_ERR_UNSUPPORTED, "q38_check_rows: type %u layout %u", w->ggml_type, w->layout);
    if (soa && (!w->aux0 || !w->aux1)) return fail(Q38_ERR_INVALID, "q38_check_rows: SoA planes missing");
    q38::CheckArgs a{};
    a.type = w->ggml_type;
    a.layout = soa ? 1u : 0u;
    a.w = dptr<const uint8_t>(w->data);
    a.aux0 = soa ? dptr<const uint8_t>(w->aux0) : nullptr;
    a.aux1 = soa ? dptr<const uint8_t>(w->aux1) : nullptr;
    a.cols = w->cols;
    a.x = x ? dptr<const float>(x) : nullptr;
    a.y = y64 ? dptr<double>(y64) : nullptr;
    a.deq = deq ? dptr<float>(deq) : nullptr;
    q38::check_rows_kernel<<<nrows, 256, 0, as_stream(stream)>>>(a);
    Q38_CUDA(cudaGetLastError(), "launch check_rows");
    return Q38_OK;
}

int q38_check_conv4(q38_devptr qkv, q38_devptr weight, q38_devptr state_in, q38_devptr conv_out,
                    q38_devptr state_out, uint32_t channels, q38_stream stream) {
    if (!qkv || !weight || !state_in || !conv_out || !state_out || channels == 0 || state_in == state_out)
        return fail(Q38_ERR_INVALID, "q38_check_conv4: bad arguments");
    q38::check_conv4_kernel<<<(channels + 255u) / 256u, 256, 0, as_stream(stream)>>>(
        dptr<const float>(qkv), dptr<const float>(weight), dptr<const float>(state_in), dptr<float>(conv_out),
        dptr<float>(state_out), channels);
    Q38_CUDA(cudaGetLastError(), "launch check_conv4");
    return Q38_OK;
}

int q38_check_l2norm(q38_devptr x, uint32_t heads, uint32_t dim, float eps, q38_devptr y, q38_stream stream) {
    if (!x || !y || heads == 0 || dim == 0) return fail(Q38_ERR_INVALID, "q38_check_l2norm: bad arguments");
    q38::check_l2norm_kernel<<<heads, 128, 0, as_stream(stream)>>>(dptr<const float>(x), dim, eps, dptr<float>(y));
    Q38_CUDA(cudaGetLastError(), "launch check_l2norm");
    return Q38_OK;
}

int q38_check_beta_gate(q38_devptr beta_raw, q38_devptr alpha_raw, q38_devptr dt_bias, q38_devptr ssm_a, uint32_t n,
                        q38_devptr beta, q38_devptr gate, q38_stream stream) {
    if (!beta_raw || !alpha_raw || !dt_bias || !ssm_a || !beta || !gate || n == 0)
        return fail(Q38_ERR_INVALID, "q38_check_beta_gate: bad arguments");
    q38::check_beta_gate_kernel<<<(n + 127u) / 128u, 128, 0, as_stream(stream)>>>(
        dptr<const float>(beta_raw), dptr<const float>(alpha_raw), dptr<const float>(dt_bias),
        dptr<const float>(ssm_a), n, dptr<float>(beta), dptr<float>(gate));
    Q38_CUDA(cudaGetLastError(), "launch check_beta_gate");
    return Q38_OK;
}

int q38_check_gdn(q38_devptr q, q38_devptr k, q38_devptr v, q38_devptr gate, q38_devptr beta, q38_devptr state_in,
                  q38_devptr out, q38_devptr state_out, uint32_t qk_heads, uint32_t value_heads, uint32_t dim,
                  q38_stream stream) {
    if (!q || !k || !v || !gate || !beta || !state_in || !out || !state_out || qk_heads == 0 || dim == 0 ||
        value_heads == 0 || value_heads % qk_heads || state_in == state_out)
        return fail(Q38_ERR_INVALID, "q38_check_gdn: bad arguments (separate state buffers, Hv %% Hq == 0)");
    const uint32_t n = value_heads * dim;
    q38::check_gdn_kernel<<<(n + 127u) / 128u, 128, 0, as_stream(stream)>>>(
        dptr<const float>(q), dptr<const float>(k), dptr<const float>(v), dptr<const float>(gate),
        dptr<const float>(beta), dptr<const float>(state_in), dptr<float>(out), dptr<float>(state_out), qk_heads,
        value_heads, dim);
    Q38_CUDA(cudaGetLastError(), "launch check_gdn");
    return Q38_OK;
}

int q38_check_rmsnorm(q38_devptr x, q38_devptr w, q38_devptr z, uint32_t groups, uint32_t dim, float eps, q38_devptr y,
                      q38_stream stream) {
    if (!x || !w || !y || groups == 0 || dim == 0) return fail(Q38_ERR_INVALID, "q38_check_rmsnorm: bad arguments");
    q38::check_rmsnorm_kernel<<<groups, 256, 0, as_stream(stream)>>>(
        dptr<const float>(x), dptr<const float>(w), z ? dptr<const float>(z) : nullptr, dim, eps, dptr<float>(y));
    Q38_CUDA(cudaGetLastError(), "launch check_rmsnorm");
    return Q38_OK;
}

int q38_check_silu_mul(q38_devptr gate, q38_devptr up, uint32_t n, q38_devptr y, q38_stream stream) {
    if (!gate || !up || !y || n == 0) return fail(Q38_ERR_INVALID, "q38_check_silu_mul: bad arguments");
    q38::check_silu_mul_kernel<<<(n + 255u) / 256u, 256, 0, as_stream(stream)>>>(
        dptr<const float>(gate), dptr<const float>(up), n, dptr<float>(y));
    Q38_CUDA(cudaGetLastError(), "launch check_silu_mul");
    return Q38_OK;
}

int q38_quantize_q8_1(q38_devptr x, uint32_t cols, q38_devptr out, q38_stream stream) {
    if (!x || !out || cols == 0 || cols % 32u) return fail(Q38_ERR_INVALID, "q38_quantize_q8_1: cols %% 32 == 0");
    if ((x & 3u) || (out & 3u)) return fail(Q38_ERR_INVALID, "q38_quantize_q8_1: x and out 4-byte aligned");
    const uint32_t nb = cols / 32u;
    return launch_pdl(q38::quantize_q8_1_kernel, dim3((nb + 7u) / 8u), dim3(256), 0, as_stream(stream),
                      "launch quantize_q8_1", dptr<const float>(x), nb, dptr<uint8_t>(out));
}

int q38_iq4xs_q8_1_gemv(q38_devptr w, q38_devptr xq81, q38_devptr y, uint32_t cols, uint32_t rows,
                        q38_stream stream) {
    if (!w || !xq81 || !y || rows == 0 || cols == 0 || cols % 256u)
        return fail(Q38_ERR_INVALID, "q38_iq4xs_q8_1_gemv: rows > 0 and cols a positive multiple of 256");
    if ((w & 3u) || (xq81 & 3u) || (y & 3u)) return fail(Q38_ERR_INVALID, "q38_iq4xs_q8_1_gemv: 4-byte alignment");
    return launch_pdl(q38::iq4xs_q81_gemv_kernel, dim3((rows + 7u) / 8u), dim3(256), 0, as_stream(stream),
                      "launch iq4xs_q81_gemv", dptr<const uint8_t>(w), dptr<const uint8_t>(xq81), dptr<float>(y),
                      cols / 256u, rows);
}

// The device address of page-locked host memory (cudaHostAlloc'd or
// cudaHostRegister'ed); pageable memory is rejected.
static int host_device_ptr(const void* p, const char* what, void** dev) {
    cudaPointerAttributes a{};
    const cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess || a.type != cudaMemoryTypeHost || !a.devicePointer) {
        cudaGetLastError();
        return fail(Q38_ERR_INVALID, "%s must be page-locked host memory (cudaHostAlloc or cudaHostRegister)", what);
    }
    *dev = a.devicePointer;
    return Q38_OK;
}

static int gemv_f32_host(const q38_weight_desc* w, const float* x, float* y, q38_stream stream, bool early) {
    if (!w || !x || !y) return fail(Q38_ERR_INVALID, "q38_gemv_f32_host: null argument");
    void *xh = nullptr, *yh = nullptr;
    if (int rc = host_device_ptr(x, "q38_gemv_f32_host: x", &xh)) return rc;
    if (int rc = host_device_ptr(y, "q38_gemv_f32_host: y", &yh)) return rc;
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    const size_t xb = (std::max(static_cast<size_t>(w->cols) * 4u, q38::xfrag_bytes_t(Q38_TYPE_Q5_K, w->cols / 256u)) +
                       255u) & ~size_t(255);  // f32 x, or (Q6) x-fragments of it
    void* io = nullptr;
    if (int rc = ensure_buffer(&st->io, &st->io_bytes, xb + static_cast<size_t>(w->rows) * 4u,
                               "cudaMalloc(host GEMV staging)", &io))
        return rc;
    float* xs = static_cast<float*>(io);
    float* ys = reinterpret_cast<float*>(static_cast<uint8_t*>(io) + xb);
    cudaStream_t s = as_stream(stream);
    auto copy = [&](const float* src, float* dst, uint32_t n, const char* what) {
        if (n % 4u == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
            const uint32_t ctas = std::min<uint32_t>((n / 4u + 255u) / 256u, static_cast<uint32_t>(st->sm_count));
            return launch_pdl(q38::copy_f32x4_kernel, dim3(ctas), dim3(256), 0, s, what,
                              reinterpret_cast<const float4*>(src), reinterpret_cast<float4*>(dst), n / 4u);
        }
        const uint32_t ctas = std::min<uint32_t>((n + 255u) / 256u, static_cast<uint32_t>(st->sm_count));
        return launch_pdl(q38::copy_f32_kernel, dim3(ctas), dim3(256), 0, s, what, src, dst, n);
    };
    if (w->layout == Q38_LAYOUT_B200_TILED && (reinterpret_cast<uintptr_t>(xh) & 15u) == 0) {
        // Layout 2: x is packed into (Q6) x-fragments while it is read over the
        // bus, the GEMV runs on them pre-packed, and it stores every output
        // once, straight into the page-locked y (two kernels in all).
        if (int rc = check_frag_args(w->ggml_type, w->data, w->cols, w->rows)) return rc;
        const uint32_t nb = w->cols / 256u;
        const uint32_t T = w->ggml_type;
        const auto pack = T == Q38_TYPE_Q6_K ? (early ? q38::xfrag_host_f32_kernel<14, true>
                                                     : q38::xfrag_host_f32_kernel<14, false>)
                                             : (early ? q38::xfrag_host_f32_kernel<13, true>
                                                     : q38::xfrag_host_f32_kernel<13, false>);
        if (int rc = launch_pdl(pack, dim3((nb + 7u) / 8u), dim3(256), 0, s, "launch xfrag_host_f32",
                                static_cast<const float*>(xh), w->cols, static_cast<uint8_t*>(io)))
            return rc;
        return launch_frag(T, w->data, static_cast<const uint8_t*>(io), static_cast<float*>(yh), w->cols, w->rows, s);
    }
    if (int rc = copy(static_cast<const float*>(xh), xs, w->cols, "launch copy_f32 (x in)")) return rc;
    const q38_devptr xsd = static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(xs));
    if (int rc = q38_gemv_f32(w, xsd, static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(ys)), stream)) return rc;
    return copy(ys, static_cast<float*>(yh), w->rows, "launch copy_f32 (y out)");
}

int q38_gemv_f32_host(const q38_weight_desc* w, const float* x, float* y, q38_stream stream) {
    return gemv_f32_host(w, x, y, stream, false);
}

int q38_gemv_f32_host_fed(const q38_weight_desc* w, const float* x, float* y, q38_stream stream) {
    return gemv_f32_host(w, x, y, stream, true);
}

int q38_gemv_q8k(const q38_weight_desc* w, q38_devptr xq8, q38_devptr y, q38_stream stream) {
    if (!w || !xq8 || !y) return fail(Q38_ERR_INVALID, "q38_gemv_q8k: null argument");
    if (w->layout == Q38_LAYOUT_SM86_Q5K_SOA && w->ggml_type == Q38_TYPE_Q5_K)
        return q38_q5k_sm86_soa_q8k_gemv(w->data, w->aux0, w->aux1, xq8, y, w->cols, w->rows, stream);
    if (w->layout == Q38_LAYOUT_B200_TILED) {
        if (int rc = check_frag_args(w->ggml_type, w->data, w->cols, w->rows)) return rc;
        int dev = 0;
        DeviceState* st = nullptr;
        if (int rc = current_device(&dev, &st)) return rc;
        void* ws = nullptr;
        if (int rc = ensure_workspace(st, q38::xfrag_bytes_t(w->ggml_type, w->cols / 256u), &ws)) return rc;
        const q38_devptr wsp = static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(ws));
        if (w->ggml_type == Q38_TYPE_Q6_K) {
            if (xq8 & 3u) return fail(Q38_ERR_INVALID, "q38_gemv_q8k: Q8_K blocks must be 4-byte aligned");
            const uint32_t nb = w->cols / 256u;
            if (int rc = launch_pdl(q38::x6frag_q8k_kernel, dim3((nb + 7u) / 8u), dim3(256), 0, as_stream(stream),
                                    "launch x6frag_q8k", dptr<const uint8_t>(xq8), nb, 1u, static_cast<uint8_t*>(ws)))
                return rc;
            if (y & 3u) return fail(Q38_ERR_INVALID, "q38_gemv_q8k: y must be 4-byte aligned");
            return launch_frag(w->ggml_type, w->data, static_cast<const uint8_t*>(ws), dptr<float>(y), w->cols,
                               w->rows, as_stream(stream));
        }
        if (int rc = q38_xfrag_q8k(xq8, w->cols, 1, wsp, stream)) return rc;
        return q38_gemv_xfrag(w, wsp, y, stream);
    }
    if (w->layout == Q38_LAYOUT_GGUF_NATIVE) {
        if (int rc = check_kq_args(w->ggml_type, w->data, w->cols, w->rows)) return rc;
    } else {
        return fail(Q38_ERR_UNSUPPORTED, "q38_gemv_q8k: type %u layout %u not supported", w->ggml_type, w->layout);
    }
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    void* ws = nullptr;
    if (int rc = ensure_workspace(st, q38_xpack_bytes(1, w->cols, 1), &ws)) return rc;
    const q38_devptr wsp = static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(ws));
    if (int rc = q38_xpack_q8k(xq8, w->cols, 1, wsp, stream)) return rc;
    return q38_gemv_packed(w, wsp, 1, 1, y, stream);
}

static int kq_f32_entry(uint32_t type, q38_devptr w, q38_devptr x, q38_devptr y, uint32_t cols, uint32_t rows,
                        q38_stream stream) {
    const q38_weight_desc d{type, Q38_LAYOUT_GGUF_NATIVE, rows, cols, w, 0, 0};
    return q38_gemv_f32(&d, x, y, stream);
}

int q38_q4k_gemv_f32(q38_devptr w, q38_devptr x, q38_devptr y, uint32_t cols, uint32_t rows, q38_stream stream) {
    return kq_f32_entry(Q38_TYPE_Q4_K, w, x, y, cols, rows, stream);
}
int q38_q5k_gemv_f32(q38_devptr w, q38_devptr x, q38_devptr y, uint32_t cols, uint32_t rows, q38_stream stream) {
    return kq_f32_entry(Q38_TYPE_Q5_K, w, x, y, cols, rows, stream);
}
int q38_q6k_gemv_f32(q38_devptr w, q38_devptr x, q38_devptr y, uint32_t cols, uint32_t rows, q38_stream stream) {
    return kq_f32_entry(Q38_TYPE_Q6_K, w, x, y, cols, rows, stream);
}
int q38_iq4xs_gemv_f32(q38_devptr w, q38_devptr x, q38_devptr y, uint32_t cols, uint32_t rows, q38_stream stream) {
    return kq_f32_entry(Q38_TYPE_IQ4_XS, w, x, y, cols, rows, stream);
}
int q38_q5k_q8k_dp4a_gemv(q38_devptr w, q38_devptr xq8, q38_devptr y, uint32_t cols, uint32_t rows,
                          q38_stream stream) {
    const q38_weight_desc d{Q38_TYPE_Q5_K, Q38_LAYOUT_GGUF_NATIVE, rows, cols, w, 0, 0};
    return q38_gemv_q8k(&d, xq8, y, stream);
}

// ---------------------------------------------------------------- layer ops

static bool aligned16(q38_devptr p) { return (p & 15u) == 0; }

int q38_rmsnorm(q38_devptr x, q38_devptr w, q38_devptr y, uint32_t n, uint32_t rows, float eps, q38_stream stream) {
    if (!x || !w || !y || n == 0 || rows == 0) return fail(Q38_ERR_INVALID, "q38_rmsnorm: bad arguments");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    return launch_pdl(q38::rmsnorm_kernel, dim3(rows), dim3(1024), 0, as_stream(stream), "launch rmsnorm",
                      dptr<const float>(x), dptr<const float>(w), dptr<float>(y), n, eps);
}

int q38_conv4_silu_roll(q38_devptr qkv, q38_devptr weight, q38_devptr state_in, q38_devptr conv_out,
                        q38_devptr state_out, uint32_t channels, q38_stream stream) {
    if (!qkv || !weight || !state_in || !conv_out || !state_out || channels == 0)
        return fail(Q38_ERR_INVALID, "q38_conv4_silu_roll: bad arguments");
    if (!aligned16(weight)) return fail(Q38_ERR_INVALID, "q38_conv4_silu_roll: weight must be 16-byte aligned");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    return launch_pdl(q38::conv4_silu_roll_kernel, dim3((channels + 255u) / 256u), dim3(256), 0, as_stream(stream),
                      "launch conv4_silu_roll", dptr<const float>(qkv), dptr<const float>(weight),
                      dptr<const float>(state_in), dptr<float>(conv_out), dptr<float>(state_out), channels);
}

int q38_qk_l2norm(q38_devptr conv, q38_devptr q, q38_devptr k, uint32_t qk_heads, float eps, q38_stream stream) {
    if (!conv || !q || !k || qk_heads == 0) return fail(Q38_ERR_INVALID, "q38_qk_l2norm: bad arguments");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    return launch_pdl(q38::qk_l2norm_kernel, dim3(2u * qk_heads), dim3(q38::kGdnDim), 0, as_stream(stream),
                      "launch qk_l2norm", dptr<const float>(conv), dptr<float>(q), dptr<float>(k), qk_heads, eps);
}

int q38_beta_gate(q38_devptr beta_raw, q38_devptr alpha_raw, q38_devptr dt_bias, q38_devptr ssm_a,
                  q38_devptr beta_out, q38_devptr gate_out, uint32_t heads, q38_stream stream) {
    if (!beta_raw || !alpha_raw || !dt_bias || !ssm_a || !beta_out || !gate_out || heads == 0)
        return fail(Q38_ERR_INVALID, "q38_beta_gate: bad arguments");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    return launch_pdl(q38::beta_gate_kernel, dim3((heads + 127u) / 128u), dim3(128), 0, as_stream(stream),
                      "launch beta_gate", dptr<const float>(beta_raw), dptr<const float>(alpha_raw),
                      dptr<const float>(dt_bias), dptr<const float>(ssm_a), dptr<float>(beta_out),
                      dptr<float>(gate_out), heads);
}

int q38_gdn_step(q38_devptr q, q38_devptr k, q38_devptr v, q38_devptr g, q38_devptr beta, q38_devptr state_in,
                 q38_devptr out, q38_devptr state_out, uint32_t qk_heads, uint32_t value_heads, float scale,
                 q38_stream stream) {
    if (!q || !k || !v || !g || !beta || !state_in || !out || !state_out || qk_heads == 0 || value_heads == 0)
        return fail(Q38_ERR_INVALID, "q38_gdn_step: bad arguments");
    if (!aligned16(q) || !aligned16(k) || !aligned16(state_in) || !aligned16(state_out))
        return fail(Q38_ERR_INVALID, "q38_gdn_step: q, k and the states must be 16-byte aligned");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    return launch_pdl(q38::gdn_step_kernel, dim3(value_heads, q38::kGdnDim / (8u * q38::kGdnStepCols)), dim3(256), 0,
                      as_stream(stream),
                      "launch gdn_step", dptr<const float>(q), dptr<const float>(k), dptr<const float>(v),
                      dptr<const float>(g), dptr<const float>(beta), dptr<const float>(state_in), dptr<float>(out),
                      dptr<float>(state_out), qk_heads, scale);
}

int q38_gated_rmsnorm_silu(q38_devptr input, q38_devptr weight, q38_devptr z, q38_devptr out, uint32_t heads,
                           float eps, q38_stream stream) {
    if (!input || !weight || !z || !out || heads == 0) return fail(Q38_ERR_INVALID, "q38_gated_rmsnorm_silu: bad arguments");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    return launch_pdl(q38::gated_rmsnorm_silu_kernel, dim3(heads), dim3(q38::kGdnDim), 0, as_stream(stream),
                      "launch gated_rmsnorm_silu", dptr<const float>(input), dptr<const float>(weight),
                      dptr<const float>(z), dptr<float>(out), eps);
}

int q38_add_residual(q38_devptr x, q38_devptr residual, q38_devptr out, uint32_t n, q38_stream stream) {
    if (!x || !residual || !out || n == 0) return fail(Q38_ERR_INVALID, "q38_add_residual: bad arguments");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    return launch_pdl(q38::add_kernel, dim3((n + 255u) / 256u), dim3(256), 0, as_stream(stream), "launch add",
                      dptr<const float>(x), dptr<const float>(residual), dptr<float>(out), n);
}

int q38_ffn_silu_mul(q38_devptr gate, q38_devptr up, q38_devptr out, uint32_t n, q38_stream stream) {
    if (!gate || !up || !out || n == 0) return fail(Q38_ERR_INVALID, "q38_ffn_silu_mul: bad arguments");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    return launch_pdl(q38::silu_mul_kernel, dim3((n + 255u) / 256u), dim3(256), 0, as_stream(stream),
                      "launch silu_mul", dptr<const float>(gate), dptr<const float>(up), dptr<float>(out), n);
}

int q38_gdn_fused(const q38_gdn_fused_args* a, q38_stream stream) {
    if (!a || !a->qkv || !a->conv_w || !a->conv_in || !a->conv_out || !a->beta_raw || !a->alpha_raw || !a->dt_bias ||
        !a->ssm_a || !a->state_in || !a->state_out || !a->z || !a->norm_w || !a->out || a->qk_heads == 0 ||
        a->value_heads == 0)
        return fail(Q38_ERR_INVALID, "q38_gdn_fused: bad arguments");
    if (a->conv_in == a->conv_out)
        return fail(Q38_ERR_INVALID, "q38_gdn_fused: conv_in and conv_out must be different buffers");
    if (!aligned16(a->conv_w) || !aligned16(a->state_in) || !aligned16(a->state_out))
        return fail(Q38_ERR_INVALID, "q38_gdn_fused: conv weights and states must be 16-byte aligned");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    q38::GdnFusedArgs k{};
    k.qkv = dptr<const float>(a->qkv);
    k.conv_w = dptr<const float>(a->conv_w);
    k.conv_in = dptr<const float>(a->conv_in);
    k.conv_out = dptr<float>(a->conv_out);
    k.beta_raw = dptr<const float>(a->beta_raw);
    k.alpha_raw = dptr<const float>(a->alpha_raw);
    k.dt_bias = dptr<const float>(a->dt_bias);
    k.ssm_a = dptr<const float>(a->ssm_a);
    k.s_in = dptr<const float>(a->state_in);
    k.s_out = dptr<float>(a->state_out);
    k.z = dptr<const float>(a->z);
    k.norm_w = dptr<const float>(a->norm_w);
    k.y = dptr<float>(a->out);
    k.Hq = a->qk_heads;
    k.Hv = a->value_heads;
    k.eps = a->eps;
    k.scale = a->scale;
    k.parity = nullptr;
    return launch_pdl_cluster(q38::gdn_fused_kernel, dim3(a->value_heads * q38::kGdnSplit), dim3(q38::kGdnFusedThreads),
                              q38::kGdnSplit, 0, as_stream(stream), "launch gdn_fused", k);
}

// Batched layout-2 GEMM of up to kGemmMaxBatch rows (gemm_frag_kernel): x-fragments
// of the rows staged in shared memory when they fit (XM 1), else read from L2.
extern "C++" {
template <uint32_t T, int NB, int W, int D, int RG>
int launch_gemm_nb(int dev, const DeviceState* st, const q38_weight_desc* w, const uint8_t* xf, float* y,
                   uint32_t batch, cudaStream_t s) {
    const uint32_t nb = w->cols / 256u, rows = w->rows;
    const dim3 g(std::min<uint32_t>(static_cast<uint32_t>(st->sm_count), (rows + 7u) / 8u));
    const uint32_t xstride = static_cast<uint32_t>(q38::xfrag1_bytes(nb));
    const size_t s1 = q38::gemm_frag_smem_bytes<T, W, D, NB>(nb, true);
    if (s1 <= kChainlessSmemMax && nb / 2u <= q38::kGemmMaxChunks) {
        constexpr auto k = q38::gemm_frag_kernel<T, 1, W, D, NB, RG>;
        if (int rc = ensure_smem_attr<k>(dev, kChainlessSmemMax)) return rc;
        return launch_pdl(k, g, dim3(W * 32), s1, s, "launch gemm_frag", dptr<const uint8_t>(w->data), xf, xstride, y,
                          rows, rows, nb, batch);
    }
    const size_t s0 = q38::gemm_frag_smem_bytes<T, W, D, NB>(nb, false);
    constexpr auto k = q38::gemm_frag_kernel<T, 0, W, D, NB, RG>;
    if (int rc = ensure_smem_attr<k>(dev, kChainlessSmemMax)) return rc;
    return launch_pdl(k, g, dim3(W * 32), s0, s, "launch gemm_frag", dptr<const uint8_t>(w->data), xf, xstride, y,
                      rows, rows, nb, batch);
}

// Measured on B200 at 6144 x 5120 Q5_K (kernel alone, CUDA graph): batch 2 in
// 8.1 us (12 warps, 2-deep rings), batch 4 in 11.5 us (12 warps, 2-deep
// rings, the 4 rows interleaved), batch 8 in 20.6 us (8 warps of 8 interleaved
// rows, 1-deep rings: the 8 rows' x-fragments take 174 KB of shared memory).
template <uint32_t T>
int launch_gemm_t(int dev, const DeviceState* st, const q38_weight_desc* w, const uint8_t* xf, float* y,
                  uint32_t batch, cudaStream_t s) {
    if (batch <= 2) return launch_gemm_nb<T, 2, 12, 2, 2>(dev, st, w, xf, y, batch, s);
    if (batch <= 4) return launch_gemm_nb<T, 4, 12, 2, 4>(dev, st, w, xf, y, batch, s);
    return launch_gemm_nb<T, 8, 8, 1, 8>(dev, st, w, xf, y, batch, s);
}
}  // extern "C++"

int q38_gemm_f32(const q38_weight_desc* w, q38_devptr x, uint32_t batch, q38_devptr y, q38_stream stream) {
    if (!w || !x || !y || batch == 0) return fail(Q38_ERR_INVALID, "q38_gemm_f32: bad arguments");
    if (x & 15u) return fail(Q38_ERR_INVALID, "q38_gemm_f32: x must be 16-byte aligned");
    const uint32_t rows = w->rows, cols = w->cols;
    if (batch == 1) return q38_gemv_f32(w, x, y, stream);
    if (w->layout == Q38_LAYOUT_B200_TILED && w->ggml_type != Q38_TYPE_Q6_K) {
        if (int rc = check_frag_args(w->ggml_type, w->data, cols, rows)) return rc;
        if (y & 3u) return fail(Q38_ERR_INVALID, "q38_gemm_f32: y must be 4-byte aligned");
        int dev = 0;
        DeviceState* st = nullptr;
        if (int rc = current_device(&dev, &st)) return rc;
        const size_t xrow = q38::xfrag1_bytes(cols / 256u);
        void* ws = nullptr;
        if (int rc = ensure_workspace(st, xrow * std::min(batch, q38::kGemmMaxBatch), &ws)) return rc;
        const q38_devptr wsp = static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(ws));
        cudaStream_t s = as_stream(stream);
        for (uint32_t b0 = 0; b0 < batch; b0 += q38::kGemmMaxBatch) {
            const uint32_t nbatch = std::min(q38::kGemmMaxBatch, batch - b0);
            if (int rc = q38_xfrag_f32(x + static_cast<q38_devptr>(b0) * cols * 4u, cols, nbatch, wsp, stream))
                return rc;
            float* yb = dptr<float>(y) + static_cast<size_t>(b0) * rows;
            const int rc = w->ggml_type == Q38_TYPE_Q5_K
                               ? launch_gemm_t<13>(dev, st, w, static_cast<const uint8_t*>(ws), yb, nbatch, s)
                               : launch_gemm_t<12>(dev, st, w, static_cast<const uint8_t*>(ws), yb, nbatch, s);
            if (rc) return rc;
        }
        return Q38_OK;
    }
    // other types and layouts: one GEMV per activation row
    for (uint32_t b = 0; b < batch; ++b)
        if (int rc = q38_gemv_f32(w, x + static_cast<q38_devptr>(b) * cols * 4u, y + static_cast<q38_devptr>(b) * rows * 4u,
                                  stream))
            return rc;
    return Q38_OK;
}

extern "C++" {
// Split of a rows x cols layout-2 GEMM over the tcgen05 kernel's CTAs: row
// blocks of 128 rows, each K range cut into S slices so that about one CTA
// runs per SM (S = 1 when the row blocks alone fill the GPU).
struct TcPlan {
    uint32_t nrb, S, nb;
    size_t xu_bytes, cnt_off, part_off, ws_bytes;
};
TcPlan tc_plan(const DeviceState* st, uint32_t rows, uint32_t cols, uint32_t slots) {
    TcPlan p{};
    p.nb = cols / 256u;
    const uint32_t nkc = p.nb / 2u, nocts = (rows + 7u) / 8u;
    p.nrb = (nocts + q38::kTcOcts - 1u) / q38::kTcOcts;
    p.S = std::max(1u, std::min(nkc, static_cast<uint32_t>(st->sm_count) / p.nrb));
    p.xu_bytes = static_cast<size_t>(p.nb) * q38::tc_xsb_bytes(slots);
    p.cnt_off = (p.xu_bytes + 255u) & ~static_cast<size_t>(255u);
    p.part_off = p.cnt_off + ((static_cast<size_t>(p.nrb) * 4u + 255u) & ~static_cast<size_t>(255u));
    p.ws_bytes = p.part_off + (p.S > 1u ? static_cast<size_t>(p.S) * slots * p.nrb * q38::kTcRows * 8u : 0u);
    return p;
}

template <uint32_t T, uint32_t SLOTS>
int launch_gemm_tc(int dev, const TcPlan& p, const q38_weight_desc* w, const float* x, uint8_t* ws, float* y,
                   uint32_t nbatch, cudaStream_t s) {
    using C = q38::TcCfg<T, SLOTS>;
    uint32_t* cnt = reinterpret_cast<uint32_t*>(ws + p.cnt_off);
    double* part = reinterpret_cast<double*>(ws + p.part_off);
    const uint32_t pack_warps = p.nb * SLOTS;
    if (int rc = launch_pdl(q38::xtc_pack_kernel<SLOTS>, dim3((pack_warps + 7u) / 8u), dim3(256), 0, s,
                            "launch xtc_pack", x, w->cols, nbatch, ws, cnt, p.nrb))
        return rc;
    constexpr auto k = q38::gemm_tc_kernel<T, SLOTS>;
    if (int rc = ensure_smem_attr<k>(dev, C::kSmem)) return rc;
    return launch_pdl(k, dim3(p.nrb * p.S), dim3(q38::kTcThreads), C::kSmem, s, "launch gemm_tc",
                      dptr<const uint8_t>(w->data), static_cast<const uint8_t*>(ws), y, part, cnt, w->rows, p.nb,
                      nbatch, p.S);
}
}  // extern "C++"

int q38_gemm_f32_tc(const q38_weight_desc* w, q38_devptr x, uint32_t batch, q38_devptr y, q38_stream stream) {
    if (!w || !x || !y || batch == 0) return fail(Q38_ERR_INVALID, "q38_gemm_f32_tc: bad arguments");
    if (x & 15u) return fail(Q38_ERR_INVALID, "q38_gemm_f32_tc: x must be 16-byte aligned");
    if (y & 3u) return fail(Q38_ERR_INVALID, "q38_gemm_f32_tc: y must be 4-byte aligned");
    if (w->layout != Q38_LAYOUT_B200_TILED || (w->ggml_type != Q38_TYPE_Q5_K && w->ggml_type != Q38_TYPE_Q4_K))
        return fail(Q38_ERR_UNSUPPORTED, "q38_gemm_f32_tc: Q5_K or Q4_K weights in layout 2 only");
    const uint32_t rows = w->rows, cols = w->cols;
    if (int rc = check_frag_args(w->ggml_type, w->data, cols, rows)) return rc;
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    const uint32_t first = std::min(batch, q38::kTcMaxBatch);
    const TcPlan p = tc_plan(st, rows, cols, q38::tc_slots(first));
    void* ws = nullptr;
    if (int rc = ensure_workspace(st, std::max(p.ws_bytes, tc_plan(st, rows, cols, 8u).ws_bytes), &ws)) return rc;
    cudaStream_t s = as_stream(stream);
    for (uint32_t b0 = 0; b0 < batch; b0 += q38::kTcMaxBatch) {
        const uint32_t nbatch = std::min(q38::kTcMaxBatch, batch - b0);
        const float* xb = dptr<const float>(x) + static_cast<size_t>(b0) * cols;
        float* yb = dptr<float>(y) + static_cast<size_t>(b0) * rows;
        const uint32_t slots = q38::tc_slots(nbatch);
        const TcPlan pb = tc_plan(st, rows, cols, slots);
        uint8_t* wsb = static_cast<uint8_t*>(ws);
        int rc;
        if (w->ggml_type == Q38_TYPE_Q5_K)
            rc = slots == 4u ? launch_gemm_tc<13, 4>(dev, pb, w, xb, wsb, yb, nbatch, s)
                             : launch_gemm_tc<13, 8>(dev, pb, w, xb, wsb, yb, nbatch, s);
        else
            rc = slots == 4u ? launch_gemm_tc<12, 4>(dev, pb, w, xb, wsb, yb, nbatch, s)
                             : launch_gemm_tc<12, 8>(dev, pb, w, xb, wsb, yb, nbatch, s);
        if (rc) return rc;
    }
    return Q38_OK;
}

size_t q38_q5k_tiled_bytes(uint32_t cols, uint32_t rows) { return q38::frag_matrix_bytes(Q38_TYPE_Q5_K, rows, cols); }

int q38_repack_tiled(uint32_t ggml_type, q38_devptr blocks, uint32_t cols, uint32_t rows, q38_devptr tiles,
                     q38_stream stream) {
    if (int rc = check_frag_args(ggml_type, tiles, cols, rows)) return rc;
    if (!blocks) return fail(Q38_ERR_INVALID, "q38_repack_tiled: blocks is null");
    const uint32_t nb = cols / 256u;
    const uint64_t n = static_cast<uint64_t>(rows) * nb;
    const uint32_t grid = static_cast<uint32_t>((n + 255u) / 256u);
    cudaStream_t s = as_stream(stream);
    if (rows % q38::kF8Rows)
        Q38_CUDA(cudaMemsetAsync(dptr<void>(tiles), 0, q38::frag_matrix_bytes(ggml_type, rows, cols), s),
                 "cudaMemsetAsync(pad rows)");
    if (ggml_type == Q38_TYPE_Q5_K)
        q38::repack_frag_kernel<13><<<grid, 256, 0, s>>>(dptr<const uint8_t>(blocks), dptr<uint8_t>(tiles), rows, nb);
    else if (ggml_type == Q38_TYPE_Q4_K)
        q38::repack_frag_kernel<12><<<grid, 256, 0, s>>>(dptr<const uint8_t>(blocks), dptr<uint8_t>(tiles), rows, nb);
    else if (ggml_type == Q38_TYPE_IQ4_XS)
        q38::repack_frag_iq4_kernel<<<grid, 256, 0, s>>>(dptr<const uint8_t>(blocks), dptr<uint8_t>(tiles), rows, nb);
    else
        q38::repack_frag_q6_kernel<<<grid, 256, 0, s>>>(dptr<const uint8_t>(blocks), dptr<uint8_t>(tiles), rows, nb);
    Q38_CUDA(cudaGetLastError(), "launch repack to layout 2");
    return Q38_OK;
}

size_t q38_tiled_bytes(uint32_t ggml_type, uint32_t cols, uint32_t rows) {
    return q38::frag_matrix_bytes(ggml_type, rows, cols);
}

int q38_q5k_sm86_soa_q8k_gemv(q38_devptr meta, q38_devptr qh, q38_devptr qs, q38_devptr xq8, q38_devptr y,
                              uint32_t cols, uint32_t rows, q38_stream stream) {
    if (int rc = check_soa_args(meta, qh, qs, cols, rows)) return rc;
    if (!xq8 || !y) return fail(Q38_ERR_INVALID, "xq8 or y is null");
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    void* ws = nullptr;
    if ((xq8 & 3u) == 0 && soa_frag_fits(cols)) {
        // Q8_K blocks -> x-fragments (limb 0 = the int8 values, unit = d), then
        // the fragment-tile GEMV on the planes with them staged per CTA
        if (int rc = ensure_workspace(st, q38::xfrag1_bytes(cols / 256u), &ws)) return rc;
        if (int rc = q38_xfrag_q8k(xq8, cols, 1, static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(ws)), stream))
            return rc;
        return launch_soa_frag(meta, qh, qs, ws, false, dptr<float>(y), cols, rows, as_stream(stream));
    }
    if (int rc = ensure_workspace(st, q38_xpack_bytes(1, cols, 1), &ws)) return rc;
    const q38_devptr wsp = static_cast<q38_devptr>(reinterpret_cast<uintptr_t>(ws));
    if (int rc = q38_xpack_q8k(xq8, cols, 1, wsp, stream)) return rc;
    XPackView v = xpack_view(ws, 1, cols / 256u, 1);
    return launch_soa_packed(meta, qh, qs, v, 1, dptr<float>(y), cols, rows, as_stream(stream));
}

}  // extern "C"

// ---- NCCL, loaded at run time -------------------------------------------------
// The library reaches NCCL through dlopen so that it needs neither NCCL's
// headers nor a link dependency (the process usually has the NCCL that
// PyTorch loaded already; Q38_NCCL_LIB names another).  Only the few calls
// below are used; their types follow nccl.h.
namespace {
typedef struct ncclComm* ncclComm_t;
struct NcclUniqueId {
    char internal[128];
};
enum { kNcclSuccess = 0, kNcclUint8 = 1, kNcclUint64 = 5, kNcclFloat32 = 7, kNcclSum = 0, kNcclMax = 2 };
struct NcclApi {
    bool ok = false;
    int (*getUniqueId)(NcclUniqueId*) = nullptr;
    int (*commInitRank)(ncclComm_t*, int, NcclUniqueId, int) = nullptr;
    int (*commDestroy)(ncclComm_t) = nullptr;
    int (*allReduce)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t) = nullptr;
    int (*allGather)(const void*, void*, size_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*getErrorString)(int) = nullptr;
};
NcclApi g_nccl;

int nccl_api(NcclApi** out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_nccl.ok) {
        const char* path = getenv("Q38_NCCL_LIB");
        void* h = dlopen(path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen(path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return fail(Q38_ERR_UNSUPPORTED, "NCCL not found (%s)", dlerror());
        g_nccl.getUniqueId = reinterpret_cast<int (*)(NcclUniqueId*)>(dlsym(h, "ncclGetUniqueId"));
        g_nccl.commInitRank = reinterpret_cast<int (*)(ncclComm_t*, int, NcclUniqueId, int)>(dlsym(h, "ncclCommInitRank"));
        g_nccl.commDestroy = reinterpret_cast<int (*)(ncclComm_t)>(dlsym(h, "ncclCommDestroy"));
        g_nccl.allReduce = reinterpret_cast<int (*)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t)>(
            dlsym(h, "ncclAllReduce"));
        g_nccl.allGather = reinterpret_cast<int (*)(const void*, void*, size_t, int, ncclComm_t, cudaStream_t)>(
            dlsym(h, "ncclAllGather"));
        g_nccl.getErrorString = reinterpret_cast<const char* (*)(int)>(dlsym(h, "ncclGetErrorString"));
        if (!g_nccl.getUniqueId || !g_nccl.commInitRank || !g_nccl.commDestroy || !g_nccl.allReduce ||
            !g_nccl.allGather || !g_nccl.getErrorString)
            return fail(Q38_ERR_UNSUPPORTED, "NCCL library lacks the needed entry points");
        g_nccl.ok = true;
    }
    *out = &g_nccl;
    return Q38_OK;
}

int nccl_fail(int r, const char* what) {
    return fail(Q38_ERR_CUDA, "%s: NCCL error %d (%s)", what, r, g_nccl.getErrorString ? g_nccl.getErrorString(r) : "?");
}
}  // namespace

struct q38_comm {
    ncclComm_t comm = nullptr;
    int rank = 0, size = 1, device = 0;
};

namespace {

// Collective over the communicator: every rank exports `base` (a cudaMalloc
// allocation on its device) through CUDA IPC and maps every other rank's;
// peers[r] is rank r's allocation as seen from this process (peers[rank] =
// base).  The handles travel by one NCCL all-gather.
int comm_map_peers(q38_comm* c, void* base, void** peers) {
    constexpr size_t kH = sizeof(cudaIpcMemHandle_t);
    cudaIpcMemHandle_t h{};
    Q38_CUDA(cudaIpcGetMemHandle(&h, base), "cudaIpcGetMemHandle");
    const size_t n = static_cast<size_t>(c->size);
    uint8_t* buf = nullptr;
    Q38_CUDA(cudaMalloc(&buf, kH * (n + 1)), "cudaMalloc(handle exchange)");
    std::vector<uint8_t> all(kH * n);
    int rc = Q38_OK;
    if (cudaMemcpy(buf + kH * n, &h, kH, cudaMemcpyHostToDevice) != cudaSuccess)
        rc = fail(Q38_ERR_CUDA, "copy IPC handle");
    else if (int r = g_nccl.allGather(buf + kH * n, buf, kH, kNcclUint8, c->comm, nullptr))
        rc = nccl_fail(r, "ncclAllGather(IPC handles)");
    else if (cudaStreamSynchronize(nullptr) != cudaSuccess ||
             cudaMemcpy(all.data(), buf, kH * n, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = fail(Q38_ERR_CUDA, "gather IPC handles");
    cudaFree(buf);
    for (size_t r = 0; r < n && rc == Q38_OK; ++r) {
        peers[r] = nullptr;
        if (static_cast<int>(r) == c->rank) {
            peers[r] = base;
            continue;
        }
        cudaIpcMemHandle_t ph;
        memcpy(&ph, all.data() + kH * r, kH);
        const cudaError_t e = cudaIpcOpenMemHandle(&peers[r], ph, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            peers[r] = nullptr;
            rc = cuda_fail(e, "cudaIpcOpenMemHandle(peer exchange region)");
        }
    }
    return rc;
}

// Undo comm_map_peers (the peers' mappings only).
void comm_unmap_peers(int rank, int size, void** peers) {
    for (int r = 0; r < size; ++r) {
        if (r != rank && peers[r]) cudaIpcCloseMemHandle(peers[r]);
        peers[r] = nullptr;
    }
}

}  // namespace

extern "C" {

int q38_comm_unique_id(uint8_t* id) {
    if (!id) return fail(Q38_ERR_INVALID, "q38_comm_unique_id: id is null");
    NcclApi* n = nullptr;
    if (int rc = nccl_api(&n)) return rc;
    NcclUniqueId u{};
    if (int r = n->getUniqueId(&u)) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(id, u.internal, sizeof(u.internal));
    return Q38_OK;
}

int q38_comm_init(int nranks, int rank, const uint8_t* id, q38_comm** out) {
    if (!id || !out || nranks < 1 || rank < 0 || rank >= nranks) return fail(Q38_ERR_INVALID, "q38_comm_init: bad arguments");
    NcclApi* n = nullptr;
    if (int rc = nccl_api(&n)) return rc;
    int dev = 0;
    DeviceState* st = nullptr;
    if (int rc = current_device(&dev, &st)) return rc;
    NcclUniqueId u{};
    memcpy(u.internal, id, sizeof(u.internal));
    auto c = std::make_unique<q38_comm>();
    if (int r = n->commInitRank(&c->comm, nranks, u, rank)) return nccl_fail(r, "ncclCommInitRank");
    c->rank = rank;
    c->size = nranks;
    c->device = dev;
    *out = c.release();
    return Q38_OK;
}

int q38_comm_destroy(q38_comm* c) {
    if (!c) return Q38_OK;
    int rc = Q38_OK;
    if (c->comm && g_nccl.ok)
        if (int r = g_nccl.commDestroy(c->comm)) rc = nccl_fail(r, "ncclCommDestroy");
    delete c;
    return rc;
}

int q38_comm_allreduce_f32(q38_comm* c, q38_devptr buf, size_t count, q38_stream stream) {
    if (!c || !buf) return fail(Q38_ERR_INVALID, "q38_comm_allreduce_f32: bad arguments");
    if (int r = g_nccl.allReduce(dptr<void>(buf), dptr<void>(buf), count, kNcclFloat32, kNcclSum, c->comm,
                                 as_stream(stream)))
        return nccl_fail(r, "ncclAllReduce");
    return Q38_OK;
}

}  // extern "C"

#include "pack.cuh"
#include "engine.cuh"
