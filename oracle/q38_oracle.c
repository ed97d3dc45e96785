/*
 * q38_oracle.c -- CPU restatement of the Q38RT hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * runtime in qwen382743090_b200/: only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference legs may load it.  The product path
 * never links, calls or falls back to it.
 *
 * Every function restates one piece of the reference implementation
 * (rffanlab/qwen382743090) in plain C, citing the reference file:line it
 * follows.  The restatement is pinned in two ways by tests/test_oracle.py:
 *   - bit-exact agreement with the reference's own src/quant.cpp, compiled
 *     from the reference tree into oracle/_ref/ (see oracle/Makefile), on
 *     seeded random blocks of every quant type, and
 *   - the golden vectors of tests/golden/ (generated from oracle/_ref by
 *     tests/golden/make_golden.py) plus the one golden Q5_K block that the
 *     reference's tests/test_q38pack.py:70-79,128-158 holds.
 * GQA attention and RoPE have no reference code; their restatement here is
 * the textbook math and is marked "parity unpinned" where it appears.
 *
 * All reductions here accumulate in double (the reference checks GPU results
 * against FP64 dots, src/driver.cpp:6946-6965).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#include <pthread.h>

#define QK 256

/* ------------------------------------------------------------------ */
/* a1: IEEE half <-> float (src/quant.cpp:11-87).                       */
/* ------------------------------------------------------------------ */
static float bits_to_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float q38o_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 31u;
    uint32_t m = h & 1023u;
    if (e == 31u) return bits_to_f32(sign | 0x7f800000u | (m << 13));
    if (e == 0u) {
        if (m == 0u) return bits_to_f32(sign);
        /* subnormal half: value m * 2^-24, exactly representable in f32 */
        float v = (float)m * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    return bits_to_f32(sign | ((e + 112u) << 23) | (m << 13));
}

uint16_t q38o_fp32_to_fp16(float value) {
    uint32_t b = f32_to_bits(value);
    uint32_t sign = (b >> 16) & 0x8000u;
    int e = (int)((b >> 23) & 255u);
    uint32_t m = b & 0x7fffffu;
    if (e == 255) return (uint16_t)(sign | 0x7c00u | (m ? 0x200u : 0u));
    int he = e - 112; /* rebias 127 -> 15 */
    if (he >= 31) return (uint16_t)(sign | 0x7c00u);
    if (he <= 0) {
        if (he < -10) return (uint16_t)sign;
        uint32_t full = m | 0x800000u;
        int sh = 14 - he;
        uint32_t q = full >> sh;
        uint32_t rem = full & ((1u << sh) - 1u);
        uint32_t half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)he << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++; /* carry may roll into the exponent */
    if (q >= 0x7c00u) q = 0x7c00u;
    return (uint16_t)(sign | q);
}

static float ld_half(const uint8_t* p) { uint16_t h; memcpy(&h, p, 2); return q38o_fp16_to_fp32(h); }

/* ------------------------------------------------------------------ */
/* a2: 6-bit scale/min unpack of the 12-byte K-quant header             */
/* (src/quant.cpp:89-97).                                               */
/* ------------------------------------------------------------------ */
void q38o_scale_min_k4(int j, const uint8_t* s, uint8_t* sc, uint8_t* mn) {
    if (j < 4) {
        *sc = s[j] & 63u;
        *mn = s[j + 4] & 63u;
    } else {
        *sc = (uint8_t)((s[j + 4] & 15u) | ((s[j - 4] >> 6) << 4));
        *mn = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* a7: Q4_K, 144 B: d, dmin | scales[12] | qs[128] (src/quant.cpp:99-136). */
void q38o_dequant_q4k(const uint8_t* b, float* out) {
    float d = ld_half(b), dmin = ld_half(b + 2);
    const uint8_t* sc = b + 4;
    const uint8_t* qs = b + 16;
    for (int c = 0; c < 4; ++c) {          /* 64-weight chunks */
        uint8_t s0, m0, s1, m1;
        q38o_scale_min_k4(2 * c, sc, &s0, &m0);
        q38o_scale_min_k4(2 * c + 1, sc, &s1, &m1);
        float d0 = d * (float)s0, n0 = dmin * (float)m0;
        float d1 = d * (float)s1, n1 = dmin * (float)m1;
        for (int l = 0; l < 32; ++l) {
            out[64 * c + l] = d0 * (float)(qs[32 * c + l] & 15u) - n0;
            out[64 * c + 32 + l] = d1 * (float)(qs[32 * c + l] >> 4) - n1;
        }
    }
}

/* a3: Q5_K, 176 B: d, dmin | scales[12] | qh[32] | qs[128]
 * (src/quant.cpp:138-183).  Group g takes the low (g even) or high (g odd)
 * nibble of qs[(g/2)*32 + l] and bit g of qh[l]. */
void q38o_dequant_q5k(const uint8_t* b, float* out) {
    float d = ld_half(b), dmin = ld_half(b + 2);
    const uint8_t* sc = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    for (int g = 0; g < 8; ++g) {
        uint8_t s, m;
        q38o_scale_min_k4(g, sc, &s, &m);
        float ds = d * (float)s, dm = dmin * (float)m;
        for (int l = 0; l < 32; ++l) {
            uint8_t byte = qs[(g >> 1) * 32 + l];
            int q = (g & 1) ? (byte >> 4) : (byte & 15);
            if (qh[l] & (1u << g)) q += 16;
            out[32 * g + l] = ds * (float)q - dm;
        }
    }
}

/* a4: lossless SoA repack, 176 B -> 180 B logical record
 * d,dmin | 8 x {u8 scale, u8 min} | qh[32] | qs[128] (src/quant.cpp:401-423). */
void q38o_repack_q5k_soa(const uint8_t* src, uint8_t* dst) {
    memcpy(dst, src, 4);
    for (int g = 0; g < 8; ++g) {
        uint8_t s, m;
        q38o_scale_min_k4(g, src + 4, &s, &m);
        dst[4 + 2 * g] = s;
        dst[5 + 2 * g] = m;
    }
    memcpy(dst + 20, src + 16, 32);
    memcpy(dst + 52, src + 48, 128);
}

/* a5: dequant of the 180 B SoA record (src/quant.cpp:425-463). */
void q38o_dequant_q5k_soa(const uint8_t* b, float* out) {
    float d = ld_half(b), dmin = ld_half(b + 2);
    const uint8_t* qh = b + 20;
    const uint8_t* qs = b + 52;
    for (int g = 0; g < 8; ++g) {
        float ds = d * (float)b[4 + 2 * g];
        float dm = dmin * (float)b[5 + 2 * g];
        for (int l = 0; l < 32; ++l) {
            uint8_t byte = qs[(g >> 1) * 32 + l];
            int q = (g & 1) ? (byte >> 4) : (byte & 15);
            if (qh[l] & (1u << g)) q += 16;
            out[32 * g + l] = ds * (float)q - dm;
        }
    }
}

/* a8: Q6_K, 210 B: ql[128] | qh[64] | int8 scales[16] | fp16 d
 * (src/quant.cpp:186-249).  Weight n (0..255): half h = n/128, r = n%128,
 * quarter t = r/32, l = r%32; low nibble source ql[64h + l + 32(t&1)]
 * (low nibble for t<2, high for t>=2), 2 high bits (qh[32h+l] >> 2t) & 3,
 * scale sc[8h + 2t + l/16]. */
void q38o_dequant_q6k(const uint8_t* b, float* out) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    float d = ld_half(b + 208);
    for (int n = 0; n < 256; ++n) {
        int h = n >> 7, r = n & 127, t = r >> 5, l = r & 31;
        uint8_t lb = ql[64 * h + l + 32 * (t & 1)];
        int lo = (t < 2) ? (lb & 15) : (lb >> 4);
        int hi = (qh[32 * h + l] >> (2 * t)) & 3;
        int q = (lo | (hi << 4)) - 32;
        out[n] = d * (float)sc[8 * h + 2 * t + l / 16] * (float)q;
    }
}

/* a9: IQ4_XS, 136 B: d | scales_h u16 | scales_l[4] | qs[128]
 * (src/quant.cpp:465-503).  The 16-entry non-linear codebook is the one of
 * src/quant.cpp:468-471. */
static const int8_t kIQ4NL[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                  1,    13,   25,  38,  53,  69,  89,  113};

void q38o_dequant_iq4xs(const uint8_t* b, float* out) {
    float d = ld_half(b);
    uint16_t sh;
    memcpy(&sh, b + 2, 2);
    const uint8_t* sl = b + 4;
    const uint8_t* qs = b + 8;
    for (int g = 0; g < 8; ++g) {
        int ls = ((sl[g >> 1] >> (4 * (g & 1))) & 15) | (((sh >> (2 * g)) & 3) << 4);
        float dl = d * (float)(ls - 32);
        for (int j = 0; j < 16; ++j) {
            out[32 * g + j] = dl * (float)kIQ4NL[qs[16 * g + j] & 15];
            out[32 * g + 16 + j] = dl * (float)kIQ4NL[qs[16 * g + j] >> 4];
        }
    }
}

/* a10: Q8_K quantize, 292 B: f32 d | int8 qs[256] | int16 bsums[16]
 * (src/quant.cpp:336-389).  The scale carries the sign of the value of
 * largest magnitude (first one wins on ties); rounding is the 1.5*2^23
 * magic-add (src/quant.cpp:253-259). */
static int round_magic(float v) {
    float t = v + 12582912.0f;
    int32_t i;
    memcpy(&i, &t, 4);
    return (i & 0x007fffff) - 0x00400000;
}

int q38o_quantize_q8k(const float* x, size_t n, uint8_t* out) {
    if (!x || !out || n == 0 || n % QK) return -1;
    for (size_t ib = 0; ib < n / QK; ++ib) {
        const float* v = x + ib * QK;
        uint8_t* blk = out + ib * 292;
        float amax = 0.0f, vmax = 0.0f;
        for (int j = 0; j < QK; ++j) {
            float a = fabsf(v[j]);
            if (a > amax) { amax = a; vmax = v[j]; }
        }
        int8_t* qs = (int8_t*)(blk + 4);
        int16_t bs[16];
        float d = 0.0f;
        if (amax == 0.0f) {
            memcpy(blk, &d, 4);
            memset(qs, 0, QK);
            memset(blk + 260, 0, 32);
            continue;
        }
        float iscale = -127.0f / vmax;
        d = 1.0f / iscale;
        memcpy(blk, &d, 4);
        for (int j = 0; j < QK; ++j) {
            int q = round_magic(iscale * v[j]);
            qs[j] = (int8_t)(q > 127 ? 127 : q);
        }
        for (int k = 0; k < 16; ++k) {
            int s = 0;
            for (int j = 0; j < 16; ++j) s += qs[16 * k + j];
            bs[k] = (int16_t)s;
        }
        memcpy(blk + 260, bs, 32);
    }
    return 0;
}

void q38o_dequant_q8k(const uint8_t* b, float* out) {
    float d;
    memcpy(&d, b, 4);
    const int8_t* qs = (const int8_t*)(b + 4);
    for (int j = 0; j < QK; ++j) out[j] = d * (float)qs[j];
}

/* ------------------------------------------------------------------ */
/* GGML type ids and block sizes (src/plan.cpp:14-41, runtime.cpp:42-64) */
/* ------------------------------------------------------------------ */
enum { T_F32 = 0, T_Q4K = 12, T_Q5K = 13, T_Q6K = 14, T_Q8K = 15, T_IQ4XS = 23 };

size_t q38o_block_bytes(int type) {
    switch (type) {
    case T_Q4K: return 144;
    case T_Q5K: return 176;
    case T_Q6K: return 210;
    case T_Q8K: return 292;
    case T_IQ4XS: return 136;
    default: return 0;
    }
}

int q38o_dequant_block(int type, const uint8_t* b, float* out) {
    switch (type) {
    case T_Q4K: q38o_dequant_q4k(b, out); return 0;
    case T_Q5K: q38o_dequant_q5k(b, out); return 0;
    case T_Q6K: q38o_dequant_q6k(b, out); return 0;
    case T_Q8K: q38o_dequant_q8k(b, out); return 0;
    case T_IQ4XS: q38o_dequant_iq4xs(b, out); return 0;
    default: return -1;
    }
}

/* ------------------------------------------------------------------ */
/* GEMV references: FP64 accumulate of dequantised weights times x      */
/* (src/driver.cpp:6946-6965 SoA, :5338-5359 Q6_K, :6739-6755 Q8_K).     */
/* Rows are split over `threads` POSIX threads (1 = the reference's own */
/* single-threaded check).                                              */
/* ------------------------------------------------------------------ */
typedef struct {
    int type;              /* GGML type of the weights */
    int soa;               /* 1: META/QH/QS planes (Q5_K only) */
    const uint8_t* w;      /* row-major blocks (soa=0) */
    const uint8_t *meta, *qh, *qs; /* planes (soa=1) */
    const float* x;        /* f32 activations, batch rows of cols */
    const uint8_t* xq8;    /* Q8_K activations instead of x when non-null */
    size_t rows, cols, batch;
    double* y;             /* batch x rows */
    size_t r0, r1;
} gemv_job;

static void gemv_rows(const gemv_job* J) {
    size_t nb = J->cols / QK, bb = q38o_block_bytes(J->type);
    float wd[QK], xd[QK];
    uint8_t rec[180];
    for (size_t r = J->r0; r < J->r1; ++r) {
        for (size_t t = 0; t < J->batch; ++t) J->y[t * J->rows + r] = 0.0;
        for (size_t ib = 0; ib < nb; ++ib) {
            size_t bi = r * nb + ib;
            if (J->soa) {
                memcpy(rec, J->meta + bi * 20, 20);
                memcpy(rec + 20, J->qh + bi * 32, 32);
                memcpy(rec + 52, J->qs + bi * 128, 128);
                q38o_dequant_q5k_soa(rec, wd);
            } else {
                q38o_dequant_block(J->type, J->w + bi * bb, wd);
            }
            for (size_t t = 0; t < J->batch; ++t) {
                const float* xv;
                if (J->xq8) {
                    q38o_dequant_q8k(J->xq8 + (t * nb + ib) * 292, xd);
                    xv = xd;
                } else {
                    xv = J->x + t * J->cols + ib * QK;
                }
                double acc = 0.0;
                for (int j = 0; j < QK; ++j) acc += (double)wd[j] * (double)xv[j];
                J->y[t * J->rows + r] += acc;
            }
        }
    }
}

static void* gemv_thread(void* p) { gemv_rows((const gemv_job*)p); return NULL; }

static int run_gemv(gemv_job base, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if ((size_t)threads > base.rows) threads = (int)base.rows;
    if (threads <= 1) { base.r0 = 0; base.r1 = base.rows; gemv_rows(&base); return 0; }
    pthread_t tid[256];
    gemv_job jobs[256];
    for (int i = 0; i < threads; ++i) {
        jobs[i] = base;
        jobs[i].r0 = base.rows * (size_t)i / (size_t)threads;
        jobs[i].r1 = base.rows * (size_t)(i + 1) / (size_t)threads;
        if (pthread_create(&tid[i], NULL, gemv_thread, &jobs[i]) != 0) {
            gemv_rows(&jobs[i]);
            tid[i] = 0;
        }
    }
    for (int i = 0; i < threads; ++i) if (tid[i]) pthread_join(tid[i], NULL);
    return 0;
}

/* GGUF-native weights (type 12/13/14/23) times f32 x[batch][cols]. */
int q38o_gemv(int type, const uint8_t* w, const float* x, size_t rows, size_t cols,
              size_t batch, double* y, int threads) {
    if (!q38o_block_bytes(type) || type == T_Q8K || cols % QK || !w || !x || !y) return -1;
    gemv_job j = {type, 0, w, 0, 0, 0, x, 0, rows, cols, batch ? batch : 1, y, 0, 0};
    return run_gemv(j, threads);
}

/* GGUF-native weights times Q8_K-quantised activations: both dequantised,
 * FP64 dot (src/driver.cpp:6739-6755). */
int q38o_gemv_q8k(int type, const uint8_t* w, const uint8_t* xq8, size_t rows, size_t cols,
                  size_t batch, double* y, int threads) {
    if (!q38o_block_bytes(type) || type == T_Q8K || cols % QK || !w || !xq8 || !y) return -1;
    gemv_job j = {type, 0, w, 0, 0, 0, 0, xq8, rows, cols, batch ? batch : 1, y, 0, 0};
    return run_gemv(j, threads);
}

/* Q5_K SoA planes META20 / QH32 / QS128 times f32 x (the checker of
 * run_q5k_sm86_gemv_smoke, src/driver.cpp:6937-6987, over all rows). */
int q38o_gemv_q5k_soa(const uint8_t* meta, const uint8_t* qh, const uint8_t* qs, const float* x,
                      size_t rows, size_t cols, size_t batch, double* y, int threads) {
    if (cols % QK || !meta || !qh || !qs || !x || !y) return -1;
    gemv_job j = {T_Q5K, 1, 0, meta, qh, qs, x, 0, rows, cols, batch ? batch : 1, y, 0, 0};
    return run_gemv(j, threads);
}

/* ------------------------------------------------------------------ */
/* Decoder-layer pointwise math (FP64), restated from the reference's   */
/* composition check in run_qwen35_layer0_full.                          */
/* ------------------------------------------------------------------ */

/* a13: y = x * rsqrt(mean(x^2) + eps) * w (src/driver.cpp:8365-8381). */
void q38o_rmsnorm(const float* x, const float* w, size_t n, float eps, float* y) {
    double ss = 0.0;
    for (size_t i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
    double inv = 1.0 / sqrt(ss / (double)n + (double)eps);
    for (size_t i = 0; i < n; ++i) y[i] = (float)((double)x[i] * inv * (double)w[i]);
}

/* a14 conv: causal depthwise conv (kernel 4) + SiLU and state roll
 * (src/driver.cpp:8090-8110).  state is [3][C] oldest first, weight [C][4]. */
void q38o_conv4_silu_roll(const float* state_in, const float* x, const float* w, size_t C,
                          float* out, float* state_out) {
    for (size_t c = 0; c < C; ++c) {
        float x0 = state_in[c], x1 = state_in[C + c], x2 = state_in[2 * C + c], x3 = x[c];
        const float* wc = w + 4 * c;
        double raw = (double)x0 * wc[0] + (double)x1 * wc[1] + (double)x2 * wc[2] + (double)x3 * wc[3];
        out[c] = (float)(raw / (1.0 + exp(-raw)));
        state_out[c] = x1;
        state_out[C + c] = x2;
        state_out[2 * C + c] = x3;
    }
}

/* a14 qk-norm: per head x * rsqrt(sum x^2 + eps) (src/driver.cpp:8112-8140). */
void q38o_l2norm_heads(const float* x, size_t heads, size_t dim, float eps, float* y) {
    for (size_t h = 0; h < heads; ++h) {
        double ss = 0.0;
        for (size_t i = 0; i < dim; ++i) ss += (double)x[h * dim + i] * (double)x[h * dim + i];
        double inv = 1.0 / sqrt(ss + (double)eps);
        for (size_t i = 0; i < dim; ++i) y[h * dim + i] = (float)((double)x[h * dim + i] * inv);
    }
}

/* a14 gates: beta = sigmoid(b); g = softplus(a + dt_bias) * A, softplus
 * linear above 20 and exp below -20 (src/driver.cpp:8142-8159). */
static double softplus_ref(double v) {
    if (v > 20.0) return v;
    if (v < -20.0) return exp(v);
    return log1p(exp(v));
}

void q38o_beta_gate(const float* b, const float* a, const float* dt_bias, const float* A, size_t n,
                    float* beta, float* g) {
    for (size_t h = 0; h < n; ++h) {
        beta[h] = (float)(1.0 / (1.0 + exp(-(double)b[h])));
        g[h] = (float)(softplus_ref((double)a[h] + (double)dt_bias[h]) * (double)A[h]);
    }
}

/* a15: one Gated DeltaNet decode step (src/driver.cpp:11255-11301 and
 * :8161-8214).  State [H][col][row], value head h reads q/k head h % Hq,
 * g is the log-decay (applied as e^g), out scaled by 1/sqrt(D). */
void q38o_gdn_step(const float* q, const float* k, const float* v, const float* g,
                   const float* beta, const float* state_in, size_t Hq, size_t Hv, size_t D,
                   float* out, float* state_out) {
    double scale = 1.0 / sqrt((double)D);
    for (size_t h = 0; h < Hv; ++h) {
        const float* qh = q + (h % Hq) * D;
        const float* kh = k + (h % Hq) * D;
        double G = exp((double)g[h]), B = (double)beta[h];
        for (size_t c = 0; c < D; ++c) {
            const float* s = state_in + (h * D + c) * D;
            float* so = state_out + (h * D + c) * D;
            double kv = 0.0;
            for (size_t i = 0; i < D; ++i) kv += (double)s[i] * (double)kh[i];
            double delta = ((double)v[h * D + c] - G * kv) * B;
            double o = 0.0;
            for (size_t i = 0; i < D; ++i) {
                double u = G * (double)s[i] + (double)kh[i] * delta;
                so[i] = (float)u;
                o += u * (double)qh[i];
            }
            out[h * D + c] = (float)(o * scale);
        }
    }
}

/* a12: Q8_1 activations (src/quant.cpp:264-313): per 32 values d = amax /
 * 127, q = clamp(round(x * (1 / d)), -127, 127), then d and s = sum(q) * d
 * as fp16; 36-byte blocks d | s | int8 qs[32].  0 on success, -1 when n is not
 * a positive multiple of 32. */
int q38o_quantize_q8_1(const float* x, size_t n, uint8_t* out) {
    if (!x || !out || n == 0 || n % 32u) return -1;
    for (size_t b = 0; b < n / 32u; ++b) {
        const float* v = x + b * 32u;
        uint8_t* blk = out + b * 36u;
        float amax = 0.0f;
        for (size_t j = 0; j < 32u; ++j) {
            const float a = fabsf(v[j]);
            amax = amax < a ? a : amax;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        int sum = 0;
        for (size_t j = 0; j < 32u; ++j) {
            int q = (int)roundf(v[j] * id);
            q = q < -127 ? -127 : (q > 127 ? 127 : q);
            blk[4u + j] = (uint8_t)(int8_t)q;
            sum += q;
        }
        const uint16_t dh = q38o_fp32_to_fp16(d), sh = q38o_fp32_to_fp16((float)sum * d);
        memcpy(blk, &dh, 2);
        memcpy(blk + 2, &sh, 2);
    }
    return 0;
}

/* Inputs of the reference's GDN decode-core smoke (run_gdn_ar_smoke,
 * src/driver.cpp:11198-11244): q/k from a sin/cos pattern of (i, h),
 * L2-normalised per head with eps 1e-6f added to the sum of squares; per value
 * head a log-decay g and beta; v and the state from sin/cos patterns of their
 * flat index.  Float arithmetic as written there (sinf/cosf of floats). */
void q38o_gdn_smoke_inputs(size_t Hq, size_t Hv, size_t D, float* q, float* k, float* v, float* g,
                           float* beta, float* state) {
    const float eps = 1.0e-6f;
    for (size_t h = 0; h < Hq; ++h) {
        double q_ss = 0.0, k_ss = 0.0;
        for (size_t i = 0; i < D; ++i) {
            const float fi = (float)i, fh = (float)h;
            const float qv = sinf(fi * 0.037f + fh * 0.11f) * 0.8f + cosf(fi * 0.013f - fh * 0.07f) * 0.2f;
            const float kv = cosf(fi * 0.029f + fh * 0.09f) * 0.75f - sinf(fi * 0.017f + fh * 0.05f) * 0.25f;
            q[h * D + i] = qv;
            k[h * D + i] = kv;
            q_ss += (double)qv * qv;
            k_ss += (double)kv * kv;
        }
        const double q_inv = 1.0 / sqrt(q_ss + eps), k_inv = 1.0 / sqrt(k_ss + eps);
        for (size_t i = 0; i < D; ++i) {
            q[h * D + i] = (float)((double)q[h * D + i] * q_inv);
            k[h * D + i] = (float)((double)k[h * D + i] * k_inv);
        }
    }
    for (size_t h = 0; h < Hv; ++h) {
        g[h] = -0.025f - 0.0015f * (float)(h % 19);
        beta[h] = 0.20f + 0.012f * (float)(h % 37);
        for (size_t c = 0; c < D; ++c) {
            const size_t o = h * D + c;
            const float fidx = (float)o;
            v[o] = sinf(fidx * 0.009f) * 0.7f + cosf(fidx * 0.004f) * 0.3f;
            const size_t base = (h * D + c) * D;
            for (size_t i = 0; i < D; ++i) {
                const float fs = (float)(base + i);
                state[base + i] = 0.012f * sinf(fs * 0.0013f) + 0.006f * cosf(fs * 0.0007f);
            }
        }
    }
}

/* a16: per-head RMSNorm(o) * w[D] * SiLU(z) (src/driver.cpp:8216-8242). */
void q38o_gated_rmsnorm_silu(const float* o, const float* z, const float* w, size_t heads, size_t D,
                             float eps, float* y) {
    for (size_t h = 0; h < heads; ++h) {
        double ss = 0.0;
        for (size_t i = 0; i < D; ++i) ss += (double)o[h * D + i] * (double)o[h * D + i];
        double inv = 1.0 / sqrt(ss / (double)D + (double)eps);
        for (size_t i = 0; i < D; ++i) {
            double zv = (double)z[h * D + i];
            y[h * D + i] = (float)((double)o[h * D + i] * inv * (double)w[i] * (zv / (1.0 + exp(-zv))));
        }
    }
}

/* a17: SiLU(g) * u (src/driver.cpp:8383-8393) and residual add. */
void q38o_silu_mul(const float* g, const float* u, size_t n, float* y) {
    for (size_t i = 0; i < n; ++i) {
        double gv = (double)g[i];
        y[i] = (float)(gv / (1.0 + exp(-gv)) * (double)u[i]);
    }
}

void q38o_add(const float* a, const float* b, size_t n, float* y) {
    for (size_t i = 0; i < n; ++i) y[i] = (float)((double)a[i] + (double)b[i]);
}

/* ------------------------------------------------------------------ */
/* a19: GQA decode attention.  NOT in the reference (parity unpinned):  */
/* textbook softmax(q k^T / sqrt(D)) v over an fp16 KV cache with GQA    */
/* group Hq/Hkv, RoPE (rotate-half, NeoX style) on the first rope_dim    */
/* dims with base theta, and an optional sigmoid output gate.            */
/* ------------------------------------------------------------------ */
void q38o_rope(float* x, size_t heads, size_t D, size_t rope_dim, size_t pos, double theta) {
    size_t half = rope_dim / 2;
    for (size_t h = 0; h < heads; ++h) {
        float* v = x + h * D;
        for (size_t i = 0; i < half; ++i) {
            double inv = pow(theta, -2.0 * (double)i / (double)rope_dim);
            double ang = (double)pos * inv, c = cos(ang), s = sin(ang);
            double a = v[i], b = v[i + half];
            v[i] = (float)(a * c - b * s);
            v[i + half] = (float)(b * c + a * s);
        }
    }
}

/* q [Hq][D] f32; kcache/vcache [Hkv][T][D] fp16 bits; out [Hq][D]. */
void q38o_attn_decode(const float* q, const uint16_t* kc, const uint16_t* vc, size_t Hq, size_t Hkv,
                      size_t D, size_t T, size_t ldT, float* out) {
    size_t grp = Hq / Hkv;
    double scale = 1.0 / sqrt((double)D);
    for (size_t h = 0; h < Hq; ++h) {
        size_t kvh = h / grp;
        const uint16_t* K = kc + kvh * ldT * D;
        const uint16_t* V = vc + kvh * ldT * D;
        double mx = -1e300, den = 0.0;
        for (size_t t = 0; t < T; ++t) {
            double s = 0.0;
            for (size_t i = 0; i < D; ++i) s += (double)q[h * D + i] * (double)q38o_fp16_to_fp32(K[t * D + i]);
            s *= scale;
            if (s > mx) mx = s;
        }
        for (size_t i = 0; i < D; ++i) out[h * D + i] = 0.0f;
        double acc[1024];
        for (size_t i = 0; i < D && i < 1024; ++i) acc[i] = 0.0;
        for (size_t t = 0; t < T; ++t) {
            double s = 0.0;
            for (size_t i = 0; i < D; ++i) s += (double)q[h * D + i] * (double)q38o_fp16_to_fp32(K[t * D + i]);
            double p = exp(s * scale - mx);
            den += p;
            for (size_t i = 0; i < D; ++i) acc[i] += p * (double)q38o_fp16_to_fp32(V[t * D + i]);
        }
        for (size_t i = 0; i < D; ++i) out[h * D + i] = (float)(acc[i] / den);
    }
}
