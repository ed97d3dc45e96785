/*
 * q38rt.h -- C ABI of the Q38RT B200 runtime (libq38rt_b200.so).
 *
 * Every entry point returns an int status (Q38_OK == 0) and takes only plain
 * C types: device addresses travel as q38_devptr (a CUdeviceptr-compatible
 * 64-bit integer), streams as q38_stream (a cudaStream_t / CUstream handle,
 * NULL = legacy default stream).  On failure q38_last_error() returns a
 * message for the calling thread.  Kernels are built for sm_100a only; a
 * call on any other device returns Q38_ERR_UNSUPPORTED.  There is no CPU
 * fallback.
 *
 * The entry points replace the reference's sm_86 PTX kernels and the
 * NvidiaDriver plumbing around them (rffanlab/qwen382743090, src/driver.cpp);
 * each declaration names the reference interface it replaces.
 */
#ifndef Q38RT_H
#define Q38RT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint64_t q38_devptr;
typedef void* q38_stream;

enum {
    Q38_OK = 0,
    Q38_ERR_INVALID = 1,     /* bad argument / shape / alignment */
    Q38_ERR_CUDA = 2,        /* CUDA runtime or driver error */
    Q38_ERR_UNSUPPORTED = 3, /* not an sm_100 device, or layout/type not handled */
    Q38_ERR_NOMEM = 4,
    Q38_ERR_NO_DEVICE = 5,
    Q38_ERR_FAULT = 6        /* a kernel gave up a bounded wait (see q38_fault_status) */
};

/* GGML type ids used by Q38PACK (src/plan.cpp:14-41). */
enum { Q38_TYPE_F32 = 0, Q38_TYPE_Q4_K = 12, Q38_TYPE_Q5_K = 13, Q38_TYPE_Q6_K = 14, Q38_TYPE_Q8_K = 15,
       Q38_TYPE_IQ4_XS = 23 };

/* Tensor execution layouts (include/q38/q38pack.hpp:30-33, plus the B200 one). */
enum { Q38_LAYOUT_GGUF_NATIVE = 0, Q38_LAYOUT_SM86_Q5K_SOA = 1, Q38_LAYOUT_B200_TILED = 2 };

/* ---------------------------------------------------------------- runtime */

/* Message of the last failing call on this thread ("" when none). */
const char* q38_last_error(void);

/* Library build string, e.g. "q38rt-b200 sm_100a". */
const char* q38_version(void);

typedef struct {
    int ordinal;
    int sm_major, sm_minor;
    int sm_count;
    size_t total_memory;
    size_t l2_bytes;
    size_t vmm_granularity;
    int vmm_supported;
    int driver_version;
    char name[128];
} q38_device_info;

/* Device probe; replaces NvidiaDriver::open's queries (src/driver.cpp:4305-4392). */
int q38_device_count(int* count);
int q38_device_query(int device, q38_device_info* info);

/* Opaque per-device context: current device, VMM allocations, workspaces. */
typedef struct q38_ctx q38_ctx;

/* Replaces NvidiaDriver::open / close (include/q38/driver.hpp:102-103). */
int q38_ctx_open(int device, q38_ctx** out);
int q38_ctx_close(q38_ctx* ctx);

/* Device memory through CUDA VMM (reserve + create + map + set access, sized
 * up to the allocation granularity); replaces ScopedVmm (src/driver.cpp:147-204). */
int q38_alloc(q38_ctx* ctx, size_t bytes, q38_devptr* out);
int q38_free(q38_ctx* ctx, q38_devptr ptr);

/* Copies; replace cuMemcpyHtoD_v2 / cuMemcpyDtoH_v2 in every run_* host. */
int q38_memcpy_h2d(q38_devptr dst, const void* src, size_t bytes, q38_stream stream);
int q38_memcpy_d2h(void* dst, q38_devptr src, size_t bytes, q38_stream stream);
int q38_memcpy_d2d(q38_devptr dst, q38_devptr src, size_t bytes, q38_stream stream);
int q38_memset_d8(q38_devptr dst, uint8_t value, size_t bytes, q38_stream stream);
int q38_stream_synchronize(q38_stream stream);

/* Device memory the library holds as lazily grown scratch on `device` (the
 * x-pack / x-fragment workspace of the f32 and Q8_K GEMV entries and the
 * staging of q38_gemv_f32_host), in bytes; 0 before the first such call.
 * Lets a caller with a fixed memory plan see what those entries allocated.
 * No reference counterpart (the reference's kernels take no scratch). */
int q38_scratch_bytes(int device, size_t* bytes);

/* Bounded-wait fault word of the kernels: 0 = none, else the site id. */
int q38_fault_status(uint32_t* site);
int q38_fault_clear(void);

/* ------------------------------------------------------------- activations */

/* Bytes of the x-pack (int8 limbs + group sums + scales) for `batch` rows of
 * `cols` activations; nl = 3 or 4 for F32 input (23- or 30-bit activations),
 * 1 for Q8_K input.  0 for an unsupported nl or cols not a multiple of 256. */
size_t q38_xpack_bytes(uint32_t nl, uint32_t cols, uint32_t batch);

/* x f32 [batch][cols] -> x-pack (nl = 3).  No reference counterpart: the
 * reference GEMVs read f32 x directly (src/driver.cpp:3897-3905). */
int q38_xpack_f32(q38_devptr x, uint32_t cols, uint32_t batch, q38_devptr xpack, q38_stream stream);

/* The same with nl = 3 or 4 limbs.  The library's own f32 entry points use
 * four limbs when cols > 6144: with three, the rounding of x alone reaches a
 * standard deviation of ~4e-5 of the FP64 dot at K = 17408 on the benchmark's
 * weights, close to the 1e-4 absolute tolerance. */
int q38_xpack_f32_limbs(q38_devptr x, uint32_t cols, uint32_t batch, uint32_t nl, q38_devptr xpack,
                        q38_stream stream);

/* Q8_K blocks [batch][cols/256][292 B] -> x-pack (nl = 1).  Consumes the
 * output of quantize_q8_k_cpu (src/quant.cpp:336-389). */
int q38_xpack_q8k(q38_devptr xq8, uint32_t cols, uint32_t batch, q38_devptr xpack, q38_stream stream);

/* Q8_K activations made on the device: quantize_q8_k_cpu (src/quant.cpp:336-389,
 * rounding of :253-259), which the reference runs on the CPU outside its timing
 * (src/q5k_q8k_gemv.cpp:91).  f32 x [cols] (cols % 256 == 0) -> 292-byte
 * blocks, bit-exact to the CPU for finite x.  q38_rmsnorm_q8k fuses it into the
 * RMSNorm producer: out = Q8_K(x * inv_rms * w) for one row of n <= 32768, and
 * y (f32, optional) gets the normalised values that were quantised. */
int q38_quantize_q8k(q38_devptr x, uint32_t cols, q38_devptr out, q38_stream stream);
int q38_rmsnorm_q8k(q38_devptr x, q38_devptr w, uint32_t n, float eps, q38_devptr y, q38_devptr out,
                    q38_stream stream);

/* ------------------------------------------------------------------- GEMV */

/* One quantised weight matrix as stored in Q38PACK: cols = dims[0] (K),
 * rows = dims[1] (N).  layout 0: `data` = row-major GGUF blocks.
 * layout 1 (Q5_K only): data = META plane (20 B/block), aux0 = QH plane
 * (32 B/block), aux1 = QS plane (128 B/block), all 16-byte aligned.
 * layout 2 (Q5_K and Q4_K, cols a multiple of 512): data = fragment tiles of
 * 8 rows x 2 super-blocks, row-octet major (Q5_K: QS 2048 | QH 512 | SC 256 |
 * DM 64 = 2880 B; Q4_K: QS 2048 | SC 256 | DM 64 = 2368 B), 16-byte aligned;
 * rows pad to a multiple of 8 with zero rows. */
typedef struct {
    uint32_t ggml_type;
    uint32_t layout;
    uint32_t rows;
    uint32_t cols;
    q38_devptr data;
    q38_devptr aux0;
    q38_devptr aux1;
} q38_weight_desc;

/* y[t][r] = sum_k W[r][k] x[t][k] for t < batch from a pre-packed x.
 * Dispatch by (ggml_type, layout) replaces select_projection_kernel
 * (src/runtime.cpp:42-64): layout 0 Q4_K / Q5_K / Q6_K / IQ4_XS and layout 1
 * Q5_K (layout 2 takes x-fragments: q38_gemv_xfrag).  The x-pack must be
 * 16-byte aligned.  y is written, not accumulated. */
int q38_gemv_packed(const q38_weight_desc* w, q38_devptr xpack, uint32_t nl, uint32_t batch, q38_devptr y,
                    q38_stream stream);

/* Q5_K SoA GEMV with f32 x, packing x into the calling device's internal
 * workspace first.  Replaces the PTX entry q38_q5k_sm86_soa_gemv_vec(meta, qh,
 * qs, x, y, cols, rows) (src/driver.cpp:3897-3905) launched by
 * run_q5k_sm86_gemv_smoke (src/driver.cpp:6931-6933). */
int q38_q5k_sm86_soa_gemv_vec(q38_devptr meta, q38_devptr qh, q38_devptr qs, q38_devptr x, q38_devptr y,
                              uint32_t cols, uint32_t rows, q38_stream stream);

/* q38_q5k_sm86_soa_gemv_vec without any device allocation.  No reference
 * counterpart: the reference launches its kernels with no scratch at all.
 * Same arguments, kernels and results (bit for bit) as
 * q38_q5k_sm86_soa_gemv_vec, but x is packed into a fixed scratch array that
 * is part of the library's device image (one per device, 135,680 bytes) instead
 * of a cudaMalloc'd workspace, so no call allocates or frees device memory.
 * cols above 32768 is rejected with Q38_ERR_INVALID.  Every call on a device
 * shares that device's one scratch: calls that can overlap (other streams,
 * other host threads) race on it and must be serialised by the caller. */
int q38_q5k_sm86_soa_gemv_vec_noalloc(q38_devptr meta, q38_devptr qh, q38_devptr qs, q38_devptr x, q38_devptr y,
                                      uint32_t cols, uint32_t rows, q38_stream stream);

/* Bytes of a matrix in the B200 tiled layout (Q38_LAYOUT_B200_TILED):
 * ceil(rows/8) row octets x cols/512 chunks x the type's tile (2880 B Q5_K,
 * 2368 B Q4_K, 3360 B Q6_K).  0 if the type is not Q5_K / Q4_K / Q6_K or cols
 * is not a positive multiple of 512.  No reference counterpart (new layout).
 * Q6_K tiles hold the GGUF block's 210 bytes per row and super-block,
 * rearranged for the tensor-core lanes; they take f32 or Q8_K activations
 * (q38_gemv_f32 / q38_gemv_q8k), not the Q5_K/Q4_K x-fragments. */
size_t q38_tiled_bytes(uint32_t ggml_type, uint32_t cols, uint32_t rows);
size_t q38_q5k_tiled_bytes(uint32_t cols, uint32_t rows); /* = q38_tiled_bytes(Q5_K, ...) */
/* Row-major GGUF blocks (Q5_K, Q4_K or Q6_K) already on the device -> layout-2
 * tiles (q38_tiled_bytes bytes, 16-byte aligned), on the stream. */
int q38_repack_tiled(uint32_t ggml_type, q38_devptr blocks, uint32_t cols, uint32_t rows, q38_devptr tiles,
                     q38_stream stream);

/* Activations for layout-2 weights ("x-fragments"): per 256-element block
 * 1088 bytes = four balanced int8 limbs of round(x / unit) (|x / unit| < 2^30,
 * unit a power of two per block) in mma fragment order, then per limb a record
 * {double unit * 256^limb / 8, float group sums}.  q38_xfrag_bytes gives the
 * size of batch rows; q38_xfrag_f32 packs f32 x [batch][cols] and
 * q38_xfrag_q8k Q8_K blocks (limb 0 = the Q8_K byte, unit = d).  No reference
 * counterpart (the reference packs x per kernel). */
size_t q38_xfrag_bytes(uint32_t cols, uint32_t batch);
int q38_xfrag_f32(q38_devptr x, uint32_t cols, uint32_t batch, q38_devptr xfrag, q38_stream stream);
int q38_xfrag_q8k(q38_devptr xq8, uint32_t cols, uint32_t batch, q38_devptr xfrag, q38_stream stream);

/* y = W x for layout-2 weights with pre-packed x-fragments (batch 1): the
 * tensor-core GEMV.  Same results as q38_gemv_f32 on the same x.  Both
 * buffers 16-byte aligned; y is written, not accumulated. */
int q38_gemv_xfrag(const q38_weight_desc* w, q38_devptr xfrag, q38_devptr y, q38_stream stream);

/* Two projections of the same input in one launch: ya = Wa x and yb = Wb x for
 * layout-2 matrices of the same cols, one Q5_K and one Q4_K in either order
 * (the decode layer's qkv+z with beta+alpha, ffn_gate with ffn_up), x as
 * x-fragments that fit in shared memory (cols <= 6144).  The CTAs split
 * between the matrices by their tiles; each output has the bits of its own
 * q38_gemv_xfrag.  No reference counterpart (the reference launches the
 * projections one by one). */
int q38_gemv_xfrag_pair(const q38_weight_desc* wa, const q38_weight_desc* wb, q38_devptr xfrag, q38_devptr ya,
                        q38_devptr yb, q38_stream stream);

/* Q5_K GEMV over the B200 tiled layout with f32 x (x-fragments into the
 * device workspace first).  Same contract as q38_q5k_sm86_soa_gemv_vec
 * (src/driver.cpp:3897-3905), the weights in layout 2 instead of the planes. */
int q38_q5k_tiled_gemv(q38_devptr w, q38_devptr x, q38_devptr y, uint32_t cols, uint32_t rows, q38_stream stream);

/* y = W x with f32 x for any (type, layout) this library runs: layout 0
 * Q4_K / Q5_K / Q6_K / IQ4_XS, layout 1 Q5_K, layout 2 Q5_K and Q4_K; batch 1.  The dispatch of
 * select_projection_kernel (src/runtime.cpp:42-64).  x is packed inside every
 * CTA when it fits in shared memory (cols <= 6144 for most types), else into the
 * device's workspace first: calls on different streams of one device must then
 * not overlap.  Layout-0 Q6_K and IQ4_XS tensors must be readable up to the
 * next 16-byte boundary past their end (true inside a Q38PACK mapping and for
 * q38_alloc'd buffers). */
int q38_gemv_f32(const q38_weight_desc* w, q38_devptr x, q38_devptr y, q38_stream stream);

/* q38_gemv_f32 with x and y in page-locked host memory (cudaHostAlloc or
 * cudaHostRegister; pageable memory is rejected), for callers that hold the
 * activations on the host as the reference's CPU path does.  The SMs
 * read x over the bus into a device staging buffer (a copy kernel chained to
 * the GEMV with PDL, no copy-engine transfer); layout-2 GEMVs store y into the
 * host buffer themselves, other layouts through a second copy kernel; y is
 * complete when the stream is.  Calls on different streams of one device must
 * not overlap (shared staging). */
int q38_gemv_f32_host(const q38_weight_desc* w, const float* x, float* y, q38_stream stream);

/* q38_gemv_f32_host for x that the host wrote before the call: the SMs read
 * and quantise x before the work queued earlier on the stream has finished
 * (only their stores into the staging buffer wait for it), so the bus read
 * overlaps the previous GEMV.  The caller promises that no device work queued
 * before this call writes x (for instance, x must not be the y of an earlier
 * host-buffer GEMV still in flight on the stream: use q38_gemv_f32_host for
 * that).  Same results as q38_gemv_f32_host.  No reference counterpart (the
 * reference copies x with a synchronous cuMemcpyHtoD before each launch). */
int q38_gemv_f32_host_fed(const q38_weight_desc* w, const float* x, float* y, q38_stream stream);

/* Reference rows for checks, computed plainly on the device (one thread per
 * weight, the block formats of src/quant.cpp:99-503 with their float
 * operation order, FP64 products summed in a fixed order): the check the
 * reference's smoke entries run on the CPU (src/driver.cpp:6946-6965).  For the
 * first nrows rows of a GGUF-native Q4_K/Q5_K/Q6_K/IQ4_XS or Q5_K SoA matrix:
 * y64 = FP64 dot with x (when x is given; double [nrows]) and deq = the
 * dequantised weights (when given; f32 [nrows][cols], bit-exact to the CPU
 * dequantisation). */
int q38_check_rows(const q38_weight_desc* w, uint32_t nrows, q38_devptr x, q38_devptr y64, q38_devptr deq,
                   q38_stream stream);

/* Reference values of the decoder-layer ops for checks, computed plainly on the
 * device: the reference's CPU check loops (src/driver.cpp:8090-8242, 8365-8393,
 * 11255-11301) restated for one thread per output, FP64 arithmetic in their
 * order and every stored value rounded to float where they store a float.
 * Used by the C++ facade's layer smokes in place of a CPU copy.
 *   q38_check_conv4: conv4 + SiLU + roll of the [3][C] state (weight [C][4]).
 *   q38_check_l2norm: per head x / sqrt(sum x^2 + eps).
 *   q38_check_beta_gate: sigmoid(b); softplus(a + dt_bias) * A.
 *   q38_check_gdn: one GDN step, state [Hv][D][D], q/k head h % Hq.
 *   q38_check_rmsnorm: per group of dim values x / sqrt(mean x^2 + eps) * w,
 *     times SiLU(z) when z is given (the gated norm; w has dim values).
 *   q38_check_silu_mul: SiLU(g) * u. */
int q38_check_conv4(q38_devptr qkv, q38_devptr weight, q38_devptr state_in, q38_devptr conv_out,
                    q38_devptr state_out, uint32_t channels, q38_stream stream);
int q38_check_l2norm(q38_devptr x, uint32_t heads, uint32_t dim, float eps, q38_devptr y, q38_stream stream);
int q38_check_beta_gate(q38_devptr beta_raw, q38_devptr alpha_raw, q38_devptr dt_bias, q38_devptr ssm_a, uint32_t n,
                        q38_devptr beta, q38_devptr gate, q38_stream stream);
int q38_check_gdn(q38_devptr q, q38_devptr k, q38_devptr v, q38_devptr gate, q38_devptr beta, q38_devptr state_in,
                  q38_devptr out, q38_devptr state_out, uint32_t qk_heads, uint32_t value_heads, uint32_t dim,
                  q38_stream stream);
int q38_check_rmsnorm(q38_devptr x, q38_devptr w, q38_devptr z, uint32_t groups, uint32_t dim, float eps, q38_devptr y,
                      q38_stream stream);
int q38_check_silu_mul(q38_devptr gate, q38_devptr up, uint32_t n, q38_devptr y, q38_stream stream);

/* y = W x with x given as Q8_K blocks (quantize_q8_k_cpu, src/quant.cpp:336-389),
 * packed into the device workspace first (same stream caveat as above). */
int q38_gemv_q8k(const q38_weight_desc* w, q38_devptr xq8, q38_devptr y, q38_stream stream);

/* Y[b] = W X[b] for batch activation rows (multi-token verify / prefill):
 * x f32 [batch][cols], y f32 [batch][rows].  Q5_K and Q4_K in layout 2 run on
 * the tensor cores eight rows at a time: each weight tile is streamed from
 * HBM once and decoded once per call for all rows (int8 mma.sync over the
 * fragment tiles, exact integer group scales, fp64 block scales); row b of Y
 * is bit-identical to the batch-1 GEMV of X[b] on the same CTA split.  Other
 * types and layouts run one GEMV per row.  No reference counterpart (the
 * reference decodes one token at a time).  Packs x into the device workspace
 * (same stream caveat as q38_gemv_f32). */
int q38_gemm_f32(const q38_weight_desc* w, q38_devptr x, uint32_t batch, q38_devptr y, q38_stream stream);

/* The same Y[b] = W X[b] on the fifth-generation tensor cores: tcgen05.mma
 * (kind::i8) with the accumulators in tensor memory.  Per super-block, 128
 * weight rows' codes are decoded from the layout-2 tiles into shared memory
 * once for all activation rows, and one MMA per 32-weight group gives the exact
 * int32 group dot products of up to 8 rows' four x limbs; group scales in
 * int32, block scales in fp64 as in the batch-1 kernels.  Q5_K and Q4_K in
 * layout 2 only; rows within the GEMV tolerance of the FP64 dot (not
 * bit-identical to the batch-1 GEMV: the K range may be split across CTAs and
 * the partial sums added in a fixed order).  Uses the device workspace like
 * q38_gemm_f32.  No reference counterpart. */
int q38_gemm_f32_tc(const q38_weight_desc* w, q38_devptr x, uint32_t batch, q38_devptr y, q38_stream stream);

/* Q8_1 activations: x f32 [cols] (cols % 32 == 0) -> cols / 32 blocks of 36 B
 * (d fp16 | s fp16 | int8 qs[32]), bit-exact to quantize_q8_1_cpu
 * (src/quant.cpp:264-313).  With q38_iq4xs_q8_1_gemv, the replacement of the
 * PTX entry q38_iq4xs_q81_gemv(weights, xq, y, cols, rows)
 * (src/driver.cpp:2641-2875): y = W x for IQ4_XS GGUF blocks and Q8_1 x,
 * exact integer group dots scaled in FP64.  The reference set this variant
 * aside (slower than F32 activations on its GPU); it is kept for
 * compatibility. */
int q38_quantize_q8_1(q38_devptr x, uint32_t cols, q38_devptr out, q38_stream stream);
int q38_iq4xs_q8_1_gemv(q38_devptr w, q38_devptr xq81, q38_devptr y, uint32_t cols, uint32_t rows,
                        q38_stream stream);

/* Drop-ins for the reference's layout-0 PTX entries (weights, x, y, cols,
 * rows): q38_q4k_gemv_f32 (src/driver.cpp:1857-1863), q38_q5k_gemv_f32
 * (:3253-3259), q38_q6k_gemv_f32_scalar (:1322-1328), q38_iq4xs_gemv_f32_prmt
 * (:2889-2895) and q38_q5k_q8k_dp4a_gemv (:3669-3675). */
int q38_q4k_gemv_f32(q38_devptr w, q38_devptr x, q38_devptr y, uint32_t cols, uint32_t rows, q38_stream stream);
int q38_q5k_gemv_f32(q38_devptr w, q38_devptr x, q38_devptr y, uint32_t cols, uint32_t rows, q38_stream stream);
int q38_q6k_gemv_f32(q38_devptr w, q38_devptr x, q38_devptr y, uint32_t cols, uint32_t rows, q38_stream stream);
int q38_iq4xs_gemv_f32(q38_devptr w, q38_devptr x, q38_devptr y, uint32_t cols, uint32_t rows, q38_stream stream);
int q38_q5k_q8k_dp4a_gemv(q38_devptr w, q38_devptr xq8, q38_devptr y, uint32_t cols, uint32_t rows,
                          q38_stream stream);

/* Q5_K SoA GEMV with Q8_K activations; replaces q38_q5k_q8k_dp4a_gemv
 * (src/driver.cpp:3660-3885), here over the SoA planes. */
int q38_q5k_sm86_soa_q8k_gemv(q38_devptr meta, q38_devptr qh, q38_devptr qs, q38_devptr xq8, q38_devptr y,
                              uint32_t cols, uint32_t rows, q38_stream stream);

/* -------------------------------------------------------------- layer ops
 * All f32, batch-1 decode, head dimension 128 for the GDN pieces.  Each
 * replaces one or two of the reference's PTX entries with the same argument
 * meaning (src/driver.cpp line ranges given per entry). */

/* y[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * w for `rows` rows of n;
 * q38_sumsq + q38_rmsnorm_apply (:240-324). */
int q38_rmsnorm(q38_devptr x, q38_devptr w, q38_devptr y, uint32_t n, uint32_t rows, float eps, q38_stream stream);

/* Causal depthwise conv (kernel 4, weight [C][4]) + SiLU of the new qkv
 * column and roll of the [3][C] state; q38_conv4_silu_roll (:759-837).
 * state_in may equal state_out. */
int q38_conv4_silu_roll(q38_devptr qkv, q38_devptr weight, q38_devptr state_in, q38_devptr conv_out,
                        q38_devptr state_out, uint32_t channels, q38_stream stream);

/* q = L2norm(conv[0, H*128)), k = L2norm(conv[H*128, 2H*128)) per 128-head,
 * x * rsqrt(sum x^2 + eps); q38_qk_l2norm_128 (:839-946). */
int q38_qk_l2norm(q38_devptr conv, q38_devptr q, q38_devptr k, uint32_t qk_heads, float eps, q38_stream stream);

/* beta = sigmoid(beta_raw), gate = softplus(alpha_raw + dt_bias) * ssm_a;
 * q38_beta_gate_48 (:948-1017). */
int q38_beta_gate(q38_devptr beta_raw, q38_devptr alpha_raw, q38_devptr dt_bias, q38_devptr ssm_a,
                  q38_devptr beta_out, q38_devptr gate_out, uint32_t heads, q38_stream stream);

/* One Gated DeltaNet decode step; state [Hv][128 col][128 row] f32, value head
 * h uses q/k head h % qk_heads, gate is the log-decay (applied as e^gate),
 * out = (S' q) * scale; q38_gdn_ar_128 (:555-752).  state_in may equal
 * state_out. */
int q38_gdn_step(q38_devptr q, q38_devptr k, q38_devptr v, q38_devptr gate, q38_devptr beta, q38_devptr state_in,
                 q38_devptr out, q38_devptr state_out, uint32_t qk_heads, uint32_t value_heads, float scale,
                 q38_stream stream);

/* Per 128-head: in * rsqrt(mean(in^2) + eps) * weight[128] * SiLU(z);
 * q38_gated_rmsnorm_silu_128 (:1025-1143). */
int q38_gated_rmsnorm_silu(q38_devptr input, q38_devptr weight, q38_devptr z, q38_devptr out, uint32_t heads,
                           float eps, q38_stream stream);

/* out = x + residual; q38_add_residual_f32 (:1145-1180). */
int q38_add_residual(q38_devptr x, q38_devptr residual, q38_devptr out, uint32_t n, q38_stream stream);

/* out = SiLU(gate) * up; q38_ffn_silu_mul_f32 (:1182-1228). */
int q38_ffn_silu_mul(q38_devptr gate, q38_devptr up, q38_devptr out, uint32_t n, q38_stream stream);

/* The recurrent core of one layer in one launch (one CTA per value head):
 * conv4+SiLU+roll of the q/k/v channels, q/k L2 norm, beta/gate, the GDN step
 * and the gated RMSNorm * SiLU(z).  Same results as the five entries above in
 * sequence (the reference's launch chain, src/driver.cpp:7803-7983).
 * conv_in and conv_out must be different buffers (value heads that share a
 * q/k head each read the old conv state); state_in may equal state_out. */
typedef struct {
    q38_devptr qkv;        /* f32 [2*qk_heads*128 + value_heads*128] */
    q38_devptr conv_w;     /* f32 [C][4] */
    q38_devptr conv_in;    /* f32 [3][C] */
    q38_devptr conv_out;   /* f32 [3][C] */
    q38_devptr beta_raw;   /* f32 [value_heads] */
    q38_devptr alpha_raw;  /* f32 [value_heads] */
    q38_devptr dt_bias;    /* f32 [value_heads] */
    q38_devptr ssm_a;      /* f32 [value_heads] */
    q38_devptr state_in;   /* f32 [value_heads][128][128] */
    q38_devptr state_out;  /* f32 [value_heads][128][128] */
    q38_devptr z;          /* f32 [value_heads*128] */
    q38_devptr norm_w;     /* f32 [128] */
    q38_devptr out;        /* f32 [value_heads*128] */
    uint32_t qk_heads;
    uint32_t value_heads;
    float eps;             /* rms_eps of the q/k L2 norm and the gated RMSNorm */
    float scale;           /* 1/sqrt(128) */
} q38_gdn_fused_args;

int q38_gdn_fused(const q38_gdn_fused_args* args, q38_stream stream);

/* ----------------------------------------------------------------- Q38PACK
 * mmap reader of the Q38PACK container (versions 1 and 2 as written by the
 * reference, 3 = + layout 2), the GPU placement plan and a resident upload.
 * Replace PackFile::open / tensors / find_tensor / tensor_data
 * (include/q38/q38pack.hpp:71-100, src/q38pack.cpp:56-190) and
 * PlacementPlan::build (include/q38/placement.hpp:27-38, src/placement.cpp:23-60). */
typedef struct q38_pack q38_pack;

typedef struct {
    uint32_t version, header_bytes, flags, tensor_count, alignment;
    uint64_t directory_offset, directory_bytes, manifest_offset, manifest_bytes;
    uint64_t raw_gguf_meta_offset, raw_gguf_meta_bytes, data_offset, data_bytes;
    uint64_t source_file_size, source_data_offset;
} q38_pack_header_info;

typedef struct {
    char name[164];          /* NUL-terminated, at most 160 characters */
    uint32_t ndim, ggml_type;
    uint64_t dims[4];        /* dims[0] = K (cols), dims[1] = N (rows) */
    uint64_t data_offset, stored_bytes, source_offset;   /* absolute file offsets */
    uint32_t role, flags, layout, layout_flags;
    uint64_t aux0_offset, aux1_offset;                   /* layout 1 planes (absolute) */
} q38_tensor_record;

typedef struct {
    uint64_t page_bytes, tensor_payload_bytes, reserved_va_bytes, page_padding_bytes, page_count;
} q38_plan_stats;

int q38_pack_open(const char* path, q38_pack** out);
int q38_pack_close(q38_pack* pack);
int q38_pack_header(const q38_pack* pack, q38_pack_header_info* out);
int q38_pack_tensor(const q38_pack* pack, uint32_t index, q38_tensor_record* out);
int q38_pack_find(const q38_pack* pack, const char* name, uint32_t* index);
int q38_pack_host_data(const q38_pack* pack, uint32_t index, const void** data);
/* Tensors in directory order at 256-byte aligned offsets of one virtual range
 * rounded up to page_bytes (a power of two); va_offsets (tensor_count entries)
 * may be NULL. */
int q38_pack_plan(const q38_pack* pack, uint64_t page_bytes, q38_plan_stats* stats, uint64_t* va_offsets);
/* Allocate the planned range through VMM (q38_alloc) and copy every payload to
 * its offset; *base is the range's device address (free with q38_free). */
int q38_pack_upload(const q38_pack* pack, q38_ctx* ctx, uint64_t page_bytes, q38_devptr* base);
/* GEMV descriptor of tensor `index` of a pack uploaded at base. */
int q38_pack_weight_desc(const q38_pack* pack, uint32_t index, q38_devptr base, q38_weight_desc* out);

/* ------------------------------------------------------------ communicator
 * NCCL over NVLink for tensor-parallel decode, one process per GPU: the
 * decode engine uses it to share the CUDA IPC handles of the exchange regions
 * and for the per-step argmax key; the row-parallel sums go through
 * q38_tp_exchange.  NCCL is loaded at run time (the process's libnccl.so.2, or
 * Q38_NCCL_LIB).  No reference counterpart: the reference has no multi-GPU
 * code. */
typedef struct q38_comm q38_comm;
/* 128-byte unique id, made on one rank and shared with the others. */
int q38_comm_unique_id(uint8_t* id);
/* Collective: every rank calls it with the same id, on its own device. */
int q38_comm_init(int nranks, int rank, const uint8_t* id, q38_comm** out);
int q38_comm_destroy(q38_comm* comm);
/* In-place sum all-reduce of count floats. */
int q38_comm_allreduce_f32(q38_comm* comm, q38_devptr buf, size_t count, q38_stream stream);

/* Tensor-parallel exchange fused with the next RMSNorm: the all-reduce the
 * decode engine runs after each row-parallel projection.  Every rank owns an
 * exchange region of q38_tp_exchange_bytes(n) that all ranks map (the engine
 * shares them through CUDA IPC); this rank stores its partial straight into
 * the peers' regions (16-byte units {x[2i], epoch, x[2i+1], epoch}) and
 * polls its own, then x_out = x_in + partial(rank 0) + partial(rank 1) + ...
 * in rank order (the same bits on every rank) and, with norm_w, writes the
 * x-fragments (q38_xfrag_f32 layout) of RMSNorm(x_out) * norm_w.  The epoch
 * of the call is (*step << 9) + instance + 1; consecutive calls alternate
 * the instance parity; every call on a region uses the same n (the region's
 * last bytes hold this rank's own scratch: each CTA's block sum of squares as
 * a unit tagged with the call's epoch).  Alignment: x_in, x_out and step
 * 4 bytes, part 8 bytes, region, norm_w and xfrag 16 bytes (Q38_ERR_INVALID
 * otherwise).  Every poll is bounded: a partial that never arrives
 * records fault site 5 (q38_fault_status) after about a second and the
 * kernel finishes; while the fault word is set, calls skip their waits. */
typedef struct {
    q38_devptr x_in, x_out, part; /* f32 [n]; x_out must not alias x_in */
    q38_devptr region[8];         /* every rank's region as mapped in this process */
    q38_devptr step;              /* uint32 step counter */
    q38_devptr norm_w;            /* f32 [n], or 0: x_out only */
    q38_devptr xfrag;             /* x-fragments out (q38_xfrag_bytes(n, 1)) when norm_w is set */
    uint32_t n;                   /* multiple of 256, at most 32768 */
    uint32_t rank, size;          /* size <= 8 */
    uint32_t instance;            /* <= 510 */
    float eps;
} q38_tp_exchange_desc;
size_t q38_tp_exchange_bytes(uint32_t n);
int q38_tp_exchange(const q38_tp_exchange_desc* d, q38_stream stream);

/* ----------------------------------------------------------- decode engine
 * Batch-1 greedy decode of a synthetic hybrid Qwen model with seeded random
 * weights generated on the current device.  No reference counterpart: the
 * reference runs one recurrent layer (run_qwen35_layer0_full,
 * src/driver.cpp:7025-8631) and has native decode disabled
 * (src/runtime.cpp:74-76).  Layer L is full attention when
 * L % attn_every == attn_every - 1 (layers 3, 7, ..., 63 of the real model,
 * src/layer_topology.cpp:152-173).  Weight types: qkv/z, ssm_out, ffn_up,
 * ffn_down, attn q/k/output Q5_K (layout 2), beta/alpha Q4_K (layout 2),
 * ffn_gate Q4_K (layout 2) or IQ4_XS (layout 0, cfg.ffn_gate_type), attn v,
 * token_embd and output Q6_K (layout 0). */
typedef struct {
    uint32_t n_layers;       /* 64 */
    uint32_t attn_every;     /* 4 */
    uint32_t hidden;         /* 5120 */
    uint32_t ffn;            /* 17408 */
    uint32_t vocab;          /* 151936 */
    uint32_t gdn_qk_heads;   /* 16 (head dim 128) */
    uint32_t gdn_v_heads;    /* 48 */
    uint32_t attn_q_heads;   /* 24 (head dim 256, each with a 256-wide output gate) */
    uint32_t attn_kv_heads;  /* 4 */
    uint32_t rope_dim;       /* rotary dims of each attention head (NeoX halves) */
    uint32_t ctx;            /* KV-cache capacity in tokens */
    float rope_theta;        /* 1e7 */
    float rms_eps;           /* 1e-6 */
    uint64_t seed;
    uint32_t tp_rank;        /* tensor-parallel rank of this process (0 for one GPU) */
    uint32_t tp_size;        /* 1, 2, 4 or 8; ranks > 1 need q38_model_set_comm */
    uint32_t ffn_gate_type;  /* 0 or Q38_TYPE_Q4_K: Q4_K tiles; Q38_TYPE_IQ4_XS: IQ4_XS GGUF blocks (the
                                reference model's ffn_gate, src/layer_topology.cpp:87) */
} q38_model_config;

typedef struct {
    uint64_t weight_bytes_per_step;  /* algorithmic (GGUF block size) weight bytes one step streams */
    uint64_t state_bytes_per_step;   /* GDN state bytes read + written per step */
    uint64_t arena_bytes;            /* device bytes held by the model */
} q38_model_stats;

typedef struct q38_model q38_model;

/* Allocates and generates this rank's shard.  Every rank's shard is a slice
 * of the same seeded model (weights depend only on the seed and global
 * indices), so results at any tp_size match tp_size 1 up to summation order.
 * Sharding: GDN heads by q/k head block (value heads h with h % 16 in the
 * block), ffn rows in 256-row units, attention by query heads (KV heads
 * replicated when tp_size > kv heads), lm_head by vocab rows; row-parallel
 * ssm_out, attn_output and ffn_down end in the peer-memory exchange of
 * q38_tp_exchange, fused with the RMSNorm that follows (the greedy argmax
 * keys still meet in one NCCL max all-reduce per step). */
int q38_model_create(const q38_model_config* cfg, q38_model** out);
/* The same model with its weights read from a Q38PACK instead of seeded:
 * every weight of this rank's shard comes from the pack tensor the reference
 * names (blk.L.attn_norm.weight, attn_qkv / attn_gate (fused as one qkvz
 * matrix), ssm_beta / ssm_alpha (fused), ssm_out, ssm_conv1d, ssm_dt.bias,
 * ssm_a, ssm_norm, post_attention_norm, ffn_gate / ffn_up / ffn_down; attn_q,
 * attn_k, attn_v, attn_output, attn_q_norm, attn_k_norm on full-attention
 * layers; token_embd, output, output_norm), checked against cfg's shapes and
 * types.  A matrix may be stored as GGUF blocks (layout 0), Q5_K SoA planes
 * (layout 1) or B200 tiles (layout 2).  Each rank uploads only the rows its
 * shard reads (row windows of the tensor), converts them to GGUF blocks on the
 * device, gathers its rows and super-blocks and tiles them; the arena it fills
 * is its placement plan (256-byte aligned tensors in one range, the rule of
 * PlacementPlan::build, src/placement.cpp:23-60).  Recurrent states and the KV
 * cache are synthetic context seeded from cfg->seed as in q38_model_create,
 * so a pack written from a seeded model reproduces it bit for bit.  The pack
 * is only read during the call. */
int q38_model_create_from_pack(const q38_model_config* cfg, const q38_pack* pack, q38_model** out);
/* Collective over the communicator (every rank calls it, in the same order):
 * allocates this rank's exchange region and maps every peer's through CUDA
 * IPC.  Once per model. */
int q38_model_set_comm(q38_model* model, q38_comm* comm);

/* The slice rank cfg->tp_rank holds (computed on the host, no device). */
typedef struct {
    uint32_t qk_head0, qk_heads;   /* GDN q/k heads [qk_head0, qk_head0 + qk_heads) */
    uint32_t v_heads;              /* GDN value heads, global ids in local order: */
    uint32_t v_head[64];
    uint32_t ffn_row0, ffn_row1;   /* ffn_gate / ffn_up rows, ffn_down K range */
    uint32_t q_head0, q_heads;     /* attention query heads */
    uint32_t kv_head0, kv_heads;   /* attention KV heads (replicated when tp_size > kv heads) */
    uint32_t vocab0, vocab1;       /* lm_head rows */
} q38_shard_info;
int q38_model_shard_info(const q38_model_config* cfg, q38_shard_info* out);
int q38_model_destroy(q38_model* model);
int q38_model_info(const q38_model* model, q38_model_stats* out);
/* Current token and position (the token is the input of the next step). */
int q38_model_set_position(q38_model* model, int32_t token, int32_t pos, uint64_t kv_seed);
int q38_model_get_position(q38_model* model, int32_t* token, int32_t* pos);
/* A fresh sequence: recurrent conv and GDN states zeroed, position 0, `token`
 * the input of the next step (the KV cache needs no clearing: a step reads
 * positions up to its own).  At tp_size > 1 every rank calls it. */
int q38_model_reset(q38_model* model, int32_t token);
/* The input token of the next step, keeping the position and the caches
 * (prompt tokens are fed this way, one step each).  Every rank at tp_size > 1. */
int q38_model_set_token(q38_model* model, int32_t token);
/* Enqueue one decode step: embed token, all layers, lm_head, argmax;
 * position += 1.  Everything stays on the device. */
int q38_model_step(q38_model* model, q38_stream stream);
/* x <- layer(x) in place for one layer (x f32 [hidden] on the device). */
int q38_model_layer(q38_model* model, uint32_t layer, q38_devptr x, q38_stream stream);
/* Capture `steps` decode steps into one CUDA graph on a non-default stream;
 * q38_model_replay launches it. */
int q38_model_capture(q38_model* model, uint32_t steps, q38_stream stream);
int q38_model_replay(q38_model* model, q38_stream stream);
/* Descriptor of a named tensor ("token_embd", "output", "output_norm", "x",
 * "logits", "blk.N.attn_norm", "blk.N.attn_qkvz", "blk.N.ssm_ba", ...); f32
 * vectors come back as type F32 with cols = element count. */
int q38_model_tensor(const q38_model* model, const char* name, q38_weight_desc* out);

#ifdef __cplusplus
}
#endif

#endif /* Q38RT_H */
