/*
 * cw_oracle.c -- CPU restatement of EggerMarc/chat-wgpu's decode path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product).  See
 * cw_oracle.h for the contract and the reference citations.
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).
 */
#define _GNU_SOURCE
#include "cw_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* WGSL literal used as "minus infinity" by the reference's attention and
 * argmax shaders (src/kernels/attention.wgsl:27, src/kernels/argmax.wgsl:23). */
#define REF_NEG_INF (-3.402823e38f)

static int g_threads = 0;
void orc_set_threads(int n) { g_threads = n; }
int orc_get_threads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

static uint16_t rd16(const uint8_t* b) { return (uint16_t)(b[0] | (b[1] << 8)); }

/* ======================================================================== */
/* dequantisation: src/loader/dequant.rs                                     */
/* ======================================================================== */

/* src/loader/dequant.rs:9-21 -- exact decode incl. subnormals, inf, nan. */
float orc_f16_to_f32(uint16_t h) {
    int sign = (h >> 15) & 1;
    int e = (h >> 10) & 0x1f;
    float mant = (float)(h & 0x3ff);
    float mag;
    if (e == 0) {
        mag = mant * ldexpf(1.0f, -24);
    } else if (e == 0x1f) {
        mag = (mant == 0.0f) ? INFINITY : NAN;
    } else {
        mag = (1.0f + mant / 1024.0f) * ldexpf(1.0f, e - 15);
    }
    return sign ? -mag : mag;
}

/* src/loader/dequant.rs:23-25 */
float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* src/loader/dequant.rs:37-39 */
void orc_dequant_f16(const uint8_t* b, size_t n, float* out) {
    for (size_t i = 0; i < n; i++) out[i] = orc_f16_to_f32(rd16(b + 2 * i));
}

/* src/loader/dequant.rs:46-58 -- 34-byte blocks: f16 d, 32 x i8, v = d*q. */
void orc_dequant_q8_0(const uint8_t* b, size_t n, float* out) {
    for (size_t blk = 0; blk < n / 32; blk++) {
        const uint8_t* base = b + blk * 34;
        float d = orc_f16_to_f32(rd16(base));
        for (int j = 0; j < 32; j++) out[blk * 32 + j] = d * (float)(int8_t)base[2 + j];
    }
}

/* src/loader/dequant.rs:62-78 -- 18-byte blocks: f16 d, 16 bytes; low nibble
 * of byte j -> element j, high nibble -> element j+16, v = d*(q-8). */
void orc_dequant_q4_0(const uint8_t* b, size_t n, float* out) {
    for (size_t blk = 0; blk < n / 32; blk++) {
        const uint8_t* base = b + blk * 18;
        float d = orc_f16_to_f32(rd16(base));
        for (int j = 0; j < 16; j++) {
            uint8_t byte = base[2 + j];
            int lo = (byte & 0x0f) - 8;
            int hi = (byte >> 4) - 8;
            out[blk * 32 + j] = d * (float)lo;
            out[blk * 32 + j + 16] = d * (float)hi;
        }
    }
}

/* src/loader/dequant.rs:82-97 -- 20-byte blocks: f16 d, f16 m, v = d*q + m. */
void orc_dequant_q4_1(const uint8_t* b, size_t n, float* out) {
    for (size_t blk = 0; blk < n / 32; blk++) {
        const uint8_t* base = b + blk * 20;
        float d = orc_f16_to_f32(rd16(base));
        float m = orc_f16_to_f32(rd16(base + 2));
        for (int j = 0; j < 16; j++) {
            uint8_t byte = base[4 + j];
            out[blk * 32 + j] = d * (float)(byte & 0x0f) + m;
            out[blk * 32 + j + 16] = d * (float)(byte >> 4) + m;
        }
    }
}

/* src/loader/dequant.rs:102-131 -- 210-byte super-blocks of 256. */
void orc_dequant_q6_k(const uint8_t* b, size_t n, float* out) {
    for (size_t blk = 0; blk < n / 256; blk++) {
        const uint8_t* base = b + blk * 210;
        const uint8_t* ql = base;
        const uint8_t* qh = base + 128;
        const int8_t* sc = (const int8_t*)(base + 192);
        float d = orc_f16_to_f32(rd16(base + 208));
        float* y = out + blk * 256;
        for (int half = 0; half < 2; half++) {
            int qlo = half * 64, qho = half * 32, sco = half * 8, yo = half * 128;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int q1 = ((ql[qlo + l] & 0x0f) | (((qh[qho + l] >> 0) & 3) << 4)) - 32;
                int q2 = ((ql[qlo + l + 32] & 0x0f) | (((qh[qho + l] >> 2) & 3) << 4)) - 32;
                int q3 = ((ql[qlo + l] >> 4) | (((qh[qho + l] >> 4) & 3) << 4)) - 32;
                int q4 = ((ql[qlo + l + 32] >> 4) | (((qh[qho + l] >> 6) & 3) << 4)) - 32;
                y[yo + l] = d * (float)sc[sco + is] * (float)q1;
                y[yo + l + 32] = d * (float)sc[sco + is + 2] * (float)q2;
                y[yo + l + 64] = d * (float)sc[sco + is + 4] * (float)q3;
                y[yo + l + 96] = d * (float)sc[sco + is + 6] * (float)q4;
            }
        }
    }
}

/* GGUF Q4_K / Q5_K (ggml block_q4_K 144 B, block_q5_K 176 B per 256 weights).
 * The reference does not implement them (dequant.rs:6, ROADMAP.md:52-53);
 * this restates ggml's published layout: f16 d, f16 dmin, 12 bytes of eight
 * 6-bit (scale, min) pairs, [Q5_K: 32 bytes of fifth bits,] 128 bytes of
 * nibbles.  Chunk c (64 weights) uses pair 2c for its low nibbles (weights
 * 64c .. 64c+31) and 2c+1 for its high nibbles; w = (d*sc)*q - (dmin*m) in
 * f32, two roundings, no contraction. */
static void kq_scale_min(int j, const uint8_t* q, int* sc, int* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

static void dequant_qk_45(const uint8_t* b, size_t n, float* out, int five) {
    const size_t bs = five ? 176 : 144;
    for (size_t blk = 0; blk < n / 256; blk++) {
        const uint8_t* base = b + blk * bs;
        const float d = orc_f16_to_f32(rd16(base));
        const float dmin = orc_f16_to_f32(rd16(base + 2));
        const uint8_t* scales = base + 4;
        const uint8_t* qh = five ? base + 16 : NULL;
        const uint8_t* qs = base + (five ? 48 : 16);
        float* y = out + blk * 256;
        for (int c = 0; c < 4; c++) {
            int sc1, m1, sc2, m2;
            kq_scale_min(2 * c, scales, &sc1, &m1);
            kq_scale_min(2 * c + 1, scales, &sc2, &m2);
            const float d1 = d * (float)sc1, mm1 = dmin * (float)m1;
            const float d2 = d * (float)sc2, mm2 = dmin * (float)m2;
            for (int l = 0; l < 32; l++) {
                int lo = qs[32 * c + l] & 0x0f, hi = qs[32 * c + l] >> 4;
                if (five) {
                    lo += ((qh[l] >> (2 * c)) & 1) << 4;
                    hi += ((qh[l] >> (2 * c + 1)) & 1) << 4;
                }
                float t = d1 * (float)lo;
                y[64 * c + l] = t - mm1;
                t = d2 * (float)hi;
                y[64 * c + 32 + l] = t - mm2;
            }
        }
    }
}

void orc_dequant_q4_k(const uint8_t* b, size_t n, float* out) { dequant_qk_45(b, n, out, 0); }
void orc_dequant_q5_k(const uint8_t* b, size_t n, float* out) { dequant_qk_45(b, n, out, 1); }

/* ======================================================================== */
/* q4 re-quantiser and GEMVs                                                 */
/* ======================================================================== */

/* Rust `f32 as i32` (saturating, NaN -> 0). */
static int32_t rust_f32_as_i32(float v) {
    if (v != v) return 0;
    if (v >= 2147483648.0f) return INT32_MAX;
    if (v <= -2147483648.0f) return INT32_MIN;
    return (int32_t)v;
}

/* src/kernels/q4.rs:37-60.  absmax/8 scale, round half away from zero
 * (Rust f32::round == C roundf), +8, clamp to 0..15, sequential nibbles:
 * nibble n of word w of block b holds element b*32 + w*8 + n. */
void orc_quantize_q4_0(const float* data, size_t out_f, size_t in_f,
                       float* scales, uint32_t* quants) {
    size_t nblocks = in_f / 32;
    for (size_t o = 0; o < out_f; o++) {
        for (size_t b = 0; b < nblocks; b++) {
            size_t base = o * in_f + b * 32;
            float absmax = 0.0f;
            for (int j = 0; j < 32; j++) absmax = fmaxf(absmax, fabsf(data[base + j]));
            float d = absmax / 8.0f;
            float inv = (d != 0.0f) ? 1.0f / d : 0.0f;
            scales[o * nblocks + b] = d;
            for (int w = 0; w < 4; w++) {
                uint32_t word = 0;
                for (int n = 0; n < 8; n++) {
                    float v = data[base + w * 8 + n];
                    /* wrapping add, as Rust release builds do */
                    int32_t qi = (int32_t)((uint32_t)rust_f32_as_i32(roundf(v * inv)) + 8u);
                    if (qi < 0) qi = 0;
                    if (qi > 15) qi = 15;
                    word |= (uint32_t)qi << (n * 4);
                }
                quants[o * (in_f / 8) + b * 4 + w] = word;
            }
        }
    }
}

/* src/main.rs:133-150 -- sequential f32 dequant-and-dot of the crate layout. */
void orc_q4_gemv(const float* x, const float* scales, const uint32_t* quants,
                 size_t in_f, size_t out_f, float* y) {
    size_t nblocks = in_f / 32;
#pragma omp parallel for schedule(static) num_threads(orc_get_threads())
    for (long long oo = 0; oo < (long long)out_f; oo++) {
        size_t o = (size_t)oo;
        float sum = 0.0f;
        for (size_t b = 0; b < nblocks; b++) {
            float d = scales[o * nblocks + b];
            for (int w = 0; w < 4; w++) {
                uint32_t word = quants[o * (in_f / 8) + b * 4 + w];
                for (int n = 0; n < 8; n++) {
                    uint32_t q = (word >> (n * 4)) & 0xF;
                    size_t k = b * 32 + w * 8 + n;
                    sum += d * ((float)q - 8.0f) * x[k];
                }
            }
        }
        y[o] = sum;
    }
}

/* Dense-mode GEMV over a GGUF Q4_0 weight: each weight is dequantised exactly
 * as src/loader/dequant.rs:62-78 (d*(q-8), exact in f32) and the dot follows
 * src/kernels/matmul.wgsl:43-50 (sum = sum + A[k]*B[k], k ascending). */
void orc_q4_0_gemv(const float* x, const uint8_t* blocks, size_t in_f,
                   size_t out_f, float* y) {
    size_t nb = in_f / 32;
#pragma omp parallel for schedule(static) num_threads(orc_get_threads())
    for (long long oo = 0; oo < (long long)out_f; oo++) {
        size_t o = (size_t)oo;
        const uint8_t* row = blocks + o * nb * 18;
        float sum = 0.0f;
        for (size_t b = 0; b < nb; b++) {
            const uint8_t* blk = row + b * 18;
            float d = orc_f16_to_f32(rd16(blk));
            float w[32];
            for (int j = 0; j < 16; j++) {
                w[j] = d * (float)((blk[2 + j] & 0x0f) - 8);
                w[j + 16] = d * (float)((blk[2 + j] >> 4) - 8);
            }
            for (int j = 0; j < 32; j++) sum = sum + x[b * 32 + j] * w[j];
        }
        y[o] = sum;
    }
}

/* examples/bench/src/lib.rs:221-233 */
void orc_matmul(const float* a, const float* b, size_t m, size_t k, size_t n,
                float* c) {
#pragma omp parallel for schedule(static) num_threads(orc_get_threads())
    for (long long ii = 0; ii < (long long)m; ii++) {
        size_t i = (size_t)ii;
        for (size_t j = 0; j < n; j++) {
            float s = 0.0f;
            for (size_t kk = 0; kk < k; kk++) s += a[i * k + kk] * b[kk * n + j];
            c[i * n + j] = s;
        }
    }
}

/* ======================================================================== */
/* norm / rope / attention / glu / add / argmax                              */
/* ======================================================================== */

/* src/kernels/norm.wgsl:20-56.  32 lanes stride the row, their partial sums
 * are combined (lane order), inverseSqrt(ss/dim + eps), y = x*inv*w or
 * x*inv*(1+w). */
void orc_rmsnorm(const float* x, const float* w, size_t rows, size_t dim,
                 float eps, int unit, float* y) {
    for (size_t r = 0; r < rows; r++) {
        const float* xr = x + r * dim;
        float part[32];
        for (int l = 0; l < 32; l++) {
            float ss = 0.0f;
            for (size_t i = (size_t)l; i < dim; i += 32) ss = ss + xr[i] * xr[i];
            part[l] = ss;
        }
        float ss = 0.0f;
        for (int l = 0; l < 32; l++) ss += part[l];
        float inv = 1.0f / sqrtf(ss / (float)dim + eps);
        for (size_t i = 0; i < dim; i++)
            y[r * dim + i] = unit ? xr[i] * inv * (1.0f + w[i]) : xr[i] * inv * w[i];
    }
}

/* src/kernels/rope.wgsl:25-34 (rotate-half / NeoX layout). */
void orc_rope(const float* x, size_t rows, size_t head_dim, uint32_t pos,
              float theta, float* y) {
    size_t half = head_dim / 2;
    for (size_t r = 0; r < rows; r++) {
        size_t base = r * head_dim;
        for (size_t i = 0; i < half; i++) {
            float exponent = -2.0f * (float)i / (float)head_dim;
            float freq = (float)pos * powf(theta, exponent);
            float c = cosf(freq), s = sinf(freq);
            float lo = x[base + i], hi = x[base + i + half];
            y[base + i] = lo * c - hi * s;
            y[base + i + half] = hi * c + lo * s;
        }
    }
}

/* src/kernels/attention.wgsl:23-96 restated lane by lane: lane l owns keys
 * j = l, l+32, ... with its own online softmax (m, denom, acc[hd]); the 32
 * lane states are then merged (max, rescale, sum).  Scale = hd^-0.5
 * (src/kernels/attention.rs:18), GQA map kv = h / (n_heads/n_kv)
 * (attention.rs:25-27).  softcap/window are the Gemma-2 extensions. */
void orc_attention_ext(const float* q, const float* k, const float* v,
                       size_t n_heads, size_t n_kv, size_t seq,
                       size_t head_dim, float softcap, uint32_t window,
                       float* out) {
    const float scale = powf((float)head_dim, -0.5f);
    const size_t heads_per_kv = n_heads / n_kv;
    const size_t kvstride = n_kv * head_dim;
    const size_t hd4 = head_dim & ~(size_t)3;
    size_t j0 = 0;
    if (window > 0 && seq > window) j0 = seq - window;
#pragma omp parallel for schedule(static) num_threads(orc_get_threads())
    for (long long hh = 0; hh < (long long)n_heads; hh++) {
        size_t h = (size_t)hh;
        size_t kvh = h / heads_per_kv;
        const float* qh = q + h * head_dim;
        float m[32], den[32];
        float* acc = (float*)calloc(32 * head_dim, sizeof(float));
        for (int l = 0; l < 32; l++) { m[l] = REF_NEG_INF; den[l] = 0.0f; }
        for (int l = 0; l < 32; l++) {
            float* a = acc + (size_t)l * head_dim;
            for (size_t j = j0 + (size_t)l; j < seq; j += 32) {
                const float* kj = k + j * kvstride + kvh * head_dim;
                const float* vj = v + j * kvstride + kvh * head_dim;
                float s = 0.0f;
                for (size_t t = 0; t < hd4; t += 4) {
                    float d4 = qh[t] * kj[t] + qh[t + 1] * kj[t + 1] +
                               qh[t + 2] * kj[t + 2] + qh[t + 3] * kj[t + 3];
                    s += d4;
                }
                for (size_t t = hd4; t < head_dim; t++) s += qh[t] * kj[t];
                s *= scale;
                if (softcap > 0.0f) s = softcap * tanhf(s / softcap);
                float m_new = fmaxf(m[l], s);
                float corr = expf(m[l] - m_new);
                float p = expf(s - m_new);
                den[l] = den[l] * corr + p;
                for (size_t t = 0; t < head_dim; t++) a[t] = a[t] * corr + vj[t] * p;
                m[l] = m_new;
            }
        }
        float m_all = m[0];
        for (int l = 1; l < 32; l++) m_all = fmaxf(m_all, m[l]);
        float corr[32], dsum = 0.0f;
        for (int l = 0; l < 32; l++) { corr[l] = expf(m[l] - m_all); dsum += den[l] * corr[l]; }
        float inv = 1.0f / dsum;
        for (size_t t = 0; t < head_dim; t++) {
            float o = 0.0f;
            for (int l = 0; l < 32; l++) o += acc[(size_t)l * head_dim + t] * corr[l];
            out[h * head_dim + t] = o * inv;
        }
        free(acc);
    }
}

void orc_attention(const float* q, const float* k, const float* v,
                   size_t n_heads, size_t n_kv, size_t seq, size_t head_dim,
                   float* out) {
    orc_attention_ext(q, k, v, n_heads, n_kv, seq, head_dim, 0.0f, 0, out);
}

/* src/kernels/ewise.wgsl:9-13 */
void orc_add(const float* a, const float* b, size_t n, float* c) {
    for (size_t i = 0; i < n; i++) c[i] = a[i] + b[i];
}

/* src/kernels/glu.wgsl:25 and :33-36: silu(x) = x/(1+exp(-x)). */
void orc_swiglu(const float* g, const float* u, size_t n, float* out) {
    for (size_t i = 0; i < n; i++) {
        float x = g[i];
        out[i] = x / (1.0f + expf(-x)) * u[i];
    }
}

/* src/kernels/glu.wgsl:27-30 and :38-42: tanh-approximate GELU. */
void orc_geglu(const float* g, const float* u, size_t n, float* out) {
    const float c = 0.7978845608028654f;
    for (size_t i = 0; i < n; i++) {
        float x = g[i];
        float gl = 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
        out[i] = gl * u[i];
    }
}

/* src/kernels/argmax.wgsl:18-55: strict '>' scan from the shader's -3.402823e38
 * start value, ties to the lowest index, NaN never wins, result 0 when no value
 * beats the start value. */
uint32_t orc_argmax(const float* logits, size_t n) {
    float best = REF_NEG_INF;
    uint32_t bi = 0;
    for (size_t i = 0; i < n; i++) {
        if (logits[i] > best) { best = logits[i]; bi = (uint32_t)i; }
    }
    return bi;
}

/* ======================================================================== */
/* GGUF v3 parser: src/loader/gguf.rs:68-106                                  */
/* ======================================================================== */

enum { MT_U = 0, MT_F = 1, MT_STR = 2, MT_OTHER = 3 };
typedef struct { char* key; int kind; uint64_t u; double f; char* s; } orc_meta;
typedef struct {
    char* name; uint32_t dtype; uint32_t n_dims; uint64_t dims[4];
    uint64_t n_elems; uint64_t offset;
} orc_tinfo;

typedef struct {
    const uint8_t* map; size_t map_len;
    orc_meta* meta; size_t n_meta;
    orc_tinfo* t; size_t n_t;
    const uint8_t* data; size_t data_len;
} orc_gguf;

typedef struct { const uint8_t* b; size_t n, p; int bad; } cur_t;
static int need(cur_t* c, size_t k) { if (c->p + k > c->n) { c->bad = 1; return 0; } return 1; }
static uint64_t c_u64(cur_t* c) { if (!need(c, 8)) return 0; uint64_t v; memcpy(&v, c->b + c->p, 8); c->p += 8; return v; }
static uint32_t c_u32(cur_t* c) { if (!need(c, 4)) return 0; uint32_t v; memcpy(&v, c->b + c->p, 4); c->p += 4; return v; }
static const uint8_t* c_bytes(cur_t* c, size_t k) { if (!need(c, k)) return NULL; const uint8_t* r = c->b + c->p; c->p += k; return r; }
static char* c_str(cur_t* c) {
    uint64_t len = c_u64(c);
    if (c->bad || len > c->n) { c->bad = 1; return NULL; }
    const uint8_t* s = c_bytes(c, (size_t)len);
    if (!s) return NULL;
    char* r = (char*)malloc((size_t)len + 1);
    memcpy(r, s, (size_t)len); r[len] = 0; return r;
}
static void skip_scalar(cur_t* c, uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: c_bytes(c, 1); break;
        case 2: case 3: c_bytes(c, 2); break;
        case 4: case 5: case 6: c_bytes(c, 4); break;
        case 8: free(c_str(c)); break;
        case 10: case 11: case 12: c_bytes(c, 8); break;
        default: break;
    }
}

static void gguf_free(orc_gguf* g) {
    for (size_t i = 0; i < g->n_meta; i++) { free(g->meta[i].key); free(g->meta[i].s); }
    for (size_t i = 0; i < g->n_t; i++) free(g->t[i].name);
    free(g->meta); free(g->t);
    if (g->map) munmap((void*)g->map, g->map_len);
    memset(g, 0, sizeof(*g));
}

static int gguf_open(const char* path, orc_gguf* g, char* err, size_t errlen) {
    memset(g, 0, sizeof(*g));
    int fd = open(path, O_RDONLY);
    if (fd < 0) { snprintf(err, errlen, "cannot open %s", path); return -1; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) { close(fd); snprintf(err, errlen, "bad file %s", path); return -1; }
    void* p = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) { snprintf(err, errlen, "mmap failed"); return -1; }
    g->map = (const uint8_t*)p; g->map_len = (size_t)st.st_size;
    cur_t c = { g->map, g->map_len, 0, 0 };
    const uint8_t* magic = c_bytes(&c, 4);
    if (!magic || memcmp(magic, "GGUF", 4) != 0) { snprintf(err, errlen, "not a GGUF file"); gguf_free(g); return -1; }
    (void)c_u32(&c); /* version */
    uint64_t n_t = c_u64(&c), n_meta = c_u64(&c);
    if (n_t > (1u << 24) || n_meta > (1u << 24)) { snprintf(err, errlen, "implausible GGUF counts"); gguf_free(g); return -1; }
    g->meta = (orc_meta*)calloc(n_meta ? n_meta : 1, sizeof(orc_meta));
    for (uint64_t i = 0; i < n_meta && !c.bad; i++) {
        orc_meta* m = &g->meta[g->n_meta++];
        m->key = c_str(&c);
        uint32_t t = c_u32(&c);
        m->kind = MT_OTHER;
        switch (t) {
            case 0: { const uint8_t* b = c_bytes(&c, 1); if (b) { m->kind = MT_U; m->u = b[0]; } break; }
            case 1: { const uint8_t* b = c_bytes(&c, 1); if (b) { m->kind = MT_U; m->u = (uint64_t)(int64_t)(int8_t)b[0]; } break; }
            case 2: { const uint8_t* b = c_bytes(&c, 2); if (b) { m->kind = MT_U; m->u = rd16(b); } break; }
            case 3: { const uint8_t* b = c_bytes(&c, 2); if (b) { m->kind = MT_U; m->u = (uint64_t)(int64_t)(int16_t)rd16(b); } break; }
            case 4: m->kind = MT_U; m->u = c_u32(&c); break;
            case 5: m->kind = MT_U; m->u = (uint64_t)(int64_t)(int32_t)c_u32(&c); break;
            case 6: { const uint8_t* b = c_bytes(&c, 4); if (b) { float f; memcpy(&f, b, 4); m->kind = MT_F; m->f = f; } break; }
            case 7: { const uint8_t* b = c_bytes(&c, 1); if (b) { m->kind = MT_U; m->u = b[0]; } break; }
            case 8: m->kind = MT_STR; m->s = c_str(&c); break;
            case 9: { uint32_t et = c_u32(&c); uint64_t cnt = c_u64(&c);
                      for (uint64_t k = 0; k < cnt && !c.bad; k++) skip_scalar(&c, et);
                      break; }
            case 10: case 11: m->kind = MT_U; m->u = c_u64(&c); break;
            case 12: { const uint8_t* b = c_bytes(&c, 8); if (b) { double f; memcpy(&f, b, 8); m->kind = MT_F; m->f = f; } break; }
            default: break;
        }
    }
    g->t = (orc_tinfo*)calloc(n_t ? n_t : 1, sizeof(orc_tinfo));
    for (uint64_t i = 0; i < n_t && !c.bad; i++) {
        orc_tinfo* t = &g->t[g->n_t++];
        t->name = c_str(&c);
        t->n_dims = c_u32(&c);
        if (t->n_dims > 4) { c.bad = 1; break; }
        t->n_elems = 1;
        for (uint32_t d = 0; d < t->n_dims; d++) { t->dims[d] = c_u64(&c); t->n_elems *= t->dims[d]; }
        t->dtype = c_u32(&c);
        t->offset = c_u64(&c);
    }
    if (c.bad) { snprintf(err, errlen, "truncated GGUF header"); gguf_free(g); return -1; }
    uint64_t align = 32;
    for (size_t i = 0; i < g->n_meta; i++)
        if (g->meta[i].key && strcmp(g->meta[i].key, "general.alignment") == 0 && g->meta[i].kind == MT_U)
            align = g->meta[i].u;
    if (align == 0) align = 32;
    size_t ds = (size_t)((c.p + align - 1) / align * align);
    if (ds > g->map_len) { snprintf(err, errlen, "GGUF data section out of range"); gguf_free(g); return -1; }
    g->data = g->map + ds; g->data_len = g->map_len - ds;
    return 0;
}

static const orc_meta* gg_meta(const orc_gguf* g, const char* key) {
    for (size_t i = 0; i < g->n_meta; i++) if (g->meta[i].key && strcmp(g->meta[i].key, key) == 0) return &g->meta[i];
    return NULL;
}
static const orc_tinfo* gg_tensor(const orc_gguf* g, const char* name) {
    for (size_t i = 0; i < g->n_t; i++) if (g->t[i].name && strcmp(g->t[i].name, name) == 0) return &g->t[i];
    return NULL;
}
/* gguf.rs:165-186 */
static uint32_t gg_u32(const orc_gguf* g, const char* key) {
    const orc_meta* m = gg_meta(g, key);
    if (m && m->kind == MT_U) return (uint32_t)m->u;
    if (m && m->kind == MT_F) return (uint32_t)m->f;
    return 0;
}
static float gg_f32(const orc_gguf* g, const char* key) {
    const orc_meta* m = gg_meta(g, key);
    if (m && m->kind == MT_F) return (float)m->f;
    if (m && m->kind == MT_U) return (float)m->u;
    return 0.0f;
}

/* ======================================================================== */
/* Model: src/model/qwen3.rs (+ restated Gemma-2 variant)                     */
/* ======================================================================== */

typedef struct {
    uint32_t dtype; size_t in_f, out_f; size_t row_bytes; const uint8_t* data;
    const float* bias; /* optional (dense-path Linear bias, src/model/layers.rs:20-21,59-61) */
    float* bias_buf;
} orc_mat;

typedef struct {
    float *attn_norm, *q_norm, *k_norm, *ffn_norm, *post_attn_norm, *post_ffw_norm;
    orc_mat wq, wk, wv, wo, gate, up, down;
} orc_layer;

struct orc_model {
    orc_gguf g;
    int family; /* 0 qwen3, 1 qwen2/llama (no qk norm), 2 gemma2 */
    size_t dim, n_layers, n_heads, n_kv, hd, hidden, vocab;
    float eps, theta, attn_softcap, final_softcap, embed_scale;
    uint32_t window;
    int unit_norm, geglu, qk_norm, post_norms;
    orc_layer* L;
    float* final_norm;
    orc_mat embed, lm_head;
    /* state */
    size_t max_seq;
    float *kc, *vc; /* [n_layers][max_seq][kv_dim] */
    /* Hook::tap values of layer tap_layer from the last step (mod.rs:155-165) */
    long tap_layer;
    float *tap_q, *tap_post_attn, *tap_layer_out;
};

static size_t row_bytes_for(uint32_t dtype, size_t in_f) {
    switch (dtype) {
        case 0: return in_f * 4;
        case 1: return in_f * 2;
        case 2: return in_f / 32 * 18;
        case 3: return in_f / 32 * 20;
        case 8: return in_f / 32 * 34;
        case 12: return in_f / 256 * 144;
        case 13: return in_f / 256 * 176;
        case 14: return in_f / 256 * 210;
        case 30: return in_f * 2; /* BF16: dequant_bf16 (dequant.rs:41-43); tensor_f32 has no arm for it (gguf.rs:113-121) */
        default: return 0;
    }
}

/* gguf.rs:109-122 dtype dispatch */
static void dequant_row(const orc_mat* m, size_t row, float* out) {
    const uint8_t* b = m->data + row * m->row_bytes;
    switch (m->dtype) {
        case 0: memcpy(out, b, m->in_f * 4); break;
        case 1: orc_dequant_f16(b, m->in_f, out); break;
        case 2: orc_dequant_q4_0(b, m->in_f, out); break;
        case 3: orc_dequant_q4_1(b, m->in_f, out); break;
        case 8: orc_dequant_q8_0(b, m->in_f, out); break;
        case 12: orc_dequant_q4_k(b, m->in_f, out); break;
        case 13: orc_dequant_q5_k(b, m->in_f, out); break;
        case 14: orc_dequant_q6_k(b, m->in_f, out); break;
        case 30: for (size_t i = 0; i < m->in_f; i++) out[i] = orc_bf16_to_f32(rd16(b + 2 * i)); break;
    }
}

static int load_mat(orc_model* M, const char* name, size_t in_f, size_t out_f, orc_mat* m, char* err, size_t errlen) {
    const orc_tinfo* t = gg_tensor(&M->g, name);
    if (!t) { snprintf(err, errlen, "missing tensor %s", name); return -1; }
    if (t->n_elems != (uint64_t)in_f * out_f) { snprintf(err, errlen, "tensor %s has %llu elements, expected %zu", name, (unsigned long long)t->n_elems, in_f * out_f); return -1; }
    m->dtype = t->dtype; m->in_f = in_f; m->out_f = out_f;
    m->row_bytes = row_bytes_for(t->dtype, in_f);
    if (!m->row_bytes) { snprintf(err, errlen, "tensor %s: ggml dtype %u not supported", name, t->dtype); return -1; }
    if (t->offset + m->row_bytes * out_f > M->g.data_len) { snprintf(err, errlen, "tensor %s out of range", name); return -1; }
    m->data = M->g.data + t->offset;
    return 0;
}

static float* load_vec(orc_model* M, const char* name, size_t len, char* err, size_t errlen) {
    orc_mat m;
    if (load_mat(M, name, len, 1, &m, err, errlen)) return NULL;
    float* v = (float*)malloc(len * sizeof(float));
    dequant_row(&m, 0, v);
    return v;
}

/* y = W x (+ bias): per row, dequantise exactly, then the sequential dot of
 * src/kernels/matmul.wgsl:43-50; bias added as src/model/layers.rs:59-61. */
static void mat_vec(const orc_mat* m, const float* x, float* y) {
    size_t in_f = m->in_f;
#pragma omp parallel num_threads(orc_get_threads())
    {
        float* tmp = (float*)malloc(in_f * sizeof(float));
#pragma omp for schedule(static)
        for (long long oo = 0; oo < (long long)m->out_f; oo++) {
            dequant_row(m, (size_t)oo, tmp);
            float s = 0.0f;
            for (size_t k = 0; k < in_f; k++) s = s + x[k] * tmp[k];
            y[oo] = m->bias ? s + m->bias[oo] : s;
        }
        free(tmp);
    }
}

void orc_model_close(orc_model* M) {
    if (!M) return;
    if (M->L) {
        for (size_t i = 0; i < M->n_layers; i++) {
            orc_layer* l = &M->L[i];
            free(l->attn_norm); free(l->q_norm); free(l->k_norm); free(l->ffn_norm);
            free(l->post_attn_norm); free(l->post_ffw_norm);
            free(l->wq.bias_buf); free(l->wk.bias_buf); free(l->wv.bias_buf);
        }
        free(M->L);
    }
    free(M->final_norm); free(M->kc); free(M->vc);
    free(M->tap_q); free(M->tap_post_attn); free(M->tap_layer_out);
    gguf_free(&M->g);
    free(M);
}

static int opt_bias(orc_model* M, const char* name, size_t len, orc_mat* m, char* err, size_t errlen) {
    if (!gg_tensor(&M->g, name)) return 0;
    m->bias_buf = load_vec(M, name, len, err, errlen);
    if (!m->bias_buf) return -1;
    m->bias = m->bias_buf;
    return 0;
}

orc_model* orc_model_open(const char* path, char* err, size_t errlen) {
    orc_model* M = (orc_model*)calloc(1, sizeof(orc_model));
    if (gguf_open(path, &M->g, err, errlen)) { free(M); return NULL; }
    const orc_meta* am = gg_meta(&M->g, "general.architecture");
    const char* arch = (am && am->kind == MT_STR && am->s) ? am->s : "qwen3";
    if (strcmp(arch, "qwen3") == 0) M->family = 0;
    else if (strcmp(arch, "qwen2") == 0 || strcmp(arch, "llama") == 0) M->family = 1;
    else if (strcmp(arch, "gemma2") == 0) M->family = 2;
    else { snprintf(err, errlen, "unsupported architecture %s", arch); orc_model_close(M); return NULL; }
    char key[256];
#define K(s) (snprintf(key, sizeof key, "%s.%s", arch, s), key)
    M->n_layers = gg_u32(&M->g, K("block_count"));
    M->dim = gg_u32(&M->g, K("embedding_length"));
    M->n_heads = gg_u32(&M->g, K("attention.head_count"));
    M->n_kv = gg_u32(&M->g, K("attention.head_count_kv"));
    M->hd = gg_u32(&M->g, K("attention.key_length"));
    M->hidden = gg_u32(&M->g, K("feed_forward_length"));
    M->eps = gg_f32(&M->g, K("attention.layer_norm_rms_epsilon"));
    M->theta = gg_f32(&M->g, K("rope.freq_base"));
    M->vocab = gg_u32(&M->g, K("vocab_size"));
    if (M->n_kv == 0) M->n_kv = M->n_heads;
    if (M->hd == 0 && M->n_heads) M->hd = M->dim / M->n_heads;
    if (M->vocab == 0) { /* gguf.rs:171-177 */
        const orc_tinfo* te = gg_tensor(&M->g, "token_embd.weight");
        if (te) for (uint32_t d = 0; d < te->n_dims; d++) if (te->dims[d] > M->vocab) M->vocab = te->dims[d];
    }
    if (M->theta == 0.0f) M->theta = (M->family == 2) ? 10000.0f : 1000000.0f;
    M->qk_norm = (M->family == 0);
    if (M->family == 2) {
        M->unit_norm = 1; M->geglu = 1; M->post_norms = 1;
        M->window = gg_u32(&M->g, K("attention.sliding_window"));
        M->attn_softcap = gg_f32(&M->g, K("attn_logit_softcapping"));
        M->final_softcap = gg_f32(&M->g, K("final_logit_softcapping"));
        M->embed_scale = sqrtf((float)M->dim);
    }
#undef K
    if (!M->dim || !M->n_layers || !M->n_heads || !M->hd || !M->hidden || !M->vocab ||
        M->n_heads % M->n_kv || M->dim % 32 || M->hidden % 32 || (M->n_heads * M->hd) % 32) {
        snprintf(err, errlen, "bad model dimensions"); orc_model_close(M); return NULL;
    }
    size_t qd = M->n_heads * M->hd, kvd = M->n_kv * M->hd;
    M->L = (orc_layer*)calloc(M->n_layers, sizeof(orc_layer));
    char nm[256];
    for (size_t i = 0; i < M->n_layers; i++) {
        orc_layer* l = &M->L[i];
#define N(s) (snprintf(nm, sizeof nm, "blk.%zu.%s", i, s), nm)
        if (!(l->attn_norm = load_vec(M, N("attn_norm.weight"), M->dim, err, errlen))) goto fail;
        if (load_mat(M, N("attn_q.weight"), M->dim, qd, &l->wq, err, errlen)) goto fail;
        if (load_mat(M, N("attn_k.weight"), M->dim, kvd, &l->wk, err, errlen)) goto fail;
        if (load_mat(M, N("attn_v.weight"), M->dim, kvd, &l->wv, err, errlen)) goto fail;
        if (opt_bias(M, N("attn_q.bias"), qd, &l->wq, err, errlen)) goto fail;
        if (opt_bias(M, N("attn_k.bias"), kvd, &l->wk, err, errlen)) goto fail;
        if (opt_bias(M, N("attn_v.bias"), kvd, &l->wv, err, errlen)) goto fail;
        if (load_mat(M, N("attn_output.weight"), qd, M->dim, &l->wo, err, errlen)) goto fail;
        if (M->qk_norm) {
            if (!(l->q_norm = load_vec(M, N("attn_q_norm.weight"), M->hd, err, errlen))) goto fail;
            if (!(l->k_norm = load_vec(M, N("attn_k_norm.weight"), M->hd, err, errlen))) goto fail;
        }
        if (!(l->ffn_norm = load_vec(M, N("ffn_norm.weight"), M->dim, err, errlen))) goto fail;
        if (load_mat(M, N("ffn_gate.weight"), M->dim, M->hidden, &l->gate, err, errlen)) goto fail;
        if (load_mat(M, N("ffn_up.weight"), M->dim, M->hidden, &l->up, err, errlen)) goto fail;
        if (load_mat(M, N("ffn_down.weight"), M->hidden, M->dim, &l->down, err, errlen)) goto fail;
        if (M->post_norms) {
            if (!(l->post_attn_norm = load_vec(M, N("post_attention_norm.weight"), M->dim, err, errlen))) goto fail;
            if (!(l->post_ffw_norm = load_vec(M, N("post_ffw_norm.weight"), M->dim, err, errlen))) goto fail;
        }
#undef N
    }
    if (!(M->final_norm = load_vec(M, "output_norm.weight", M->dim, err, errlen))) goto fail;
    if (load_mat(M, "token_embd.weight", M->dim, M->vocab, &M->embed, err, errlen)) goto fail;
    /* tied head when output.weight is absent (src/model/qwen3.rs:93-98) */
    if (load_mat(M, gg_tensor(&M->g, "output.weight") ? "output.weight" : "token_embd.weight",
                 M->dim, M->vocab, &M->lm_head, err, errlen)) goto fail;
    return M;
fail:
    orc_model_close(M);
    return NULL;
}

void orc_model_dims(const orc_model* M, uint32_t* o) {
    o[0] = (uint32_t)M->dim; o[1] = (uint32_t)M->n_layers; o[2] = (uint32_t)M->n_heads;
    o[3] = (uint32_t)M->n_kv; o[4] = (uint32_t)M->hd; o[5] = (uint32_t)M->hidden; o[6] = (uint32_t)M->vocab;
}

int orc_model_reset(orc_model* M, size_t max_seq) {
    free(M->kc); free(M->vc);
    size_t n = M->n_layers * max_seq * M->n_kv * M->hd;
    M->kc = (float*)calloc(n ? n : 1, sizeof(float));
    M->vc = (float*)calloc(n ? n : 1, sizeof(float));
    M->max_seq = max_seq;
    return (M->kc && M->vc) ? 0 : -1;
}

/* src/model/qwen3.rs:128-133 (embed), :139-191 (forward), :135-137 (logits). */
int orc_model_step(orc_model* M, uint32_t token, size_t pos, float* hidden_out, float* logits) {
    if (pos >= M->max_seq || token >= M->vocab) return -1;
    size_t dim = M->dim, qd = M->n_heads * M->hd, kvd = M->n_kv * M->hd, hid = M->hidden;
    float* h = (float*)malloc(dim * sizeof(float));
    float* normed = (float*)malloc(dim * sizeof(float));
    float* q = (float*)malloc(qd * sizeof(float));
    float* k = (float*)malloc(kvd * sizeof(float));
    float* v = (float*)malloc(kvd * sizeof(float));
    float* tmpq = (float*)malloc(qd * sizeof(float));
    float* tmpk = (float*)malloc(kvd * sizeof(float));
    float* attn = (float*)malloc(qd * sizeof(float));
    float* ao = (float*)malloc(dim * sizeof(float));
    float* g = (float*)malloc(hid * sizeof(float));
    float* u = (float*)malloc(hid * sizeof(float));
    float* act = (float*)malloc(hid * sizeof(float));
    float* ff = (float*)malloc(dim * sizeof(float));

    dequant_row(&M->embed, token, h);
    if (M->embed_scale > 0.0f)
        for (size_t i = 0; i < dim; i++) h[i] = h[i] * M->embed_scale;
    for (size_t li = 0; li < M->n_layers; li++) {
        orc_layer* l = &M->L[li];
        orc_rmsnorm(h, l->attn_norm, 1, dim, M->eps, M->unit_norm, normed);
        mat_vec(&l->wq, normed, q);
        mat_vec(&l->wk, normed, k);
        mat_vec(&l->wv, normed, v);
        if (M->qk_norm) {
            orc_rmsnorm(q, l->q_norm, M->n_heads, M->hd, M->eps, 0, tmpq);
            orc_rmsnorm(k, l->k_norm, M->n_kv, M->hd, M->eps, 0, tmpk);
            memcpy(q, tmpq, qd * sizeof(float));
            memcpy(k, tmpk, kvd * sizeof(float));
        }
        orc_rope(q, M->n_heads, M->hd, (uint32_t)pos, M->theta, tmpq);
        orc_rope(k, M->n_kv, M->hd, (uint32_t)pos, M->theta, tmpk);
        const int tapped = M->tap_q && (long)li == M->tap_layer;
        if (tapped) memcpy(M->tap_q, tmpq, qd * sizeof(float));   /* qwen3.rs:165 */
        float* kc = M->kc + li * M->max_seq * kvd;
        float* vc = M->vc + li * M->max_seq * kvd;
        memcpy(kc + pos * kvd, tmpk, kvd * sizeof(float));   /* src/model/cache.rs:21-24 */
        memcpy(vc + pos * kvd, v, kvd * sizeof(float));
        uint32_t window = (M->window && (li % 2 == 0)) ? M->window : 0;
        orc_attention_ext(tmpq, kc, vc, M->n_heads, M->n_kv, pos + 1, M->hd,
                          M->attn_softcap, window, attn);
        mat_vec(&l->wo, attn, ao);
        if (M->post_norms) { orc_rmsnorm(ao, l->post_attn_norm, 1, dim, M->eps, 1, normed); memcpy(ao, normed, dim * sizeof(float)); }
        orc_add(h, ao, dim, h);
        if (tapped) memcpy(M->tap_post_attn, h, dim * sizeof(float));   /* qwen3.rs:180 */
        orc_rmsnorm(h, l->ffn_norm, 1, dim, M->eps, M->unit_norm, normed);
        mat_vec(&l->gate, normed, g);
        mat_vec(&l->up, normed, u);
        if (M->geglu) orc_geglu(g, u, hid, act); else orc_swiglu(g, u, hid, act);
        mat_vec(&l->down, act, ff);
        if (M->post_norms) { orc_rmsnorm(ff, l->post_ffw_norm, 1, dim, M->eps, 1, normed); memcpy(ff, normed, dim * sizeof(float)); }
        orc_add(h, ff, dim, h);
        if (tapped) memcpy(M->tap_layer_out, h, dim * sizeof(float));   /* qwen3.rs:188 */
    }
    orc_rmsnorm(h, M->final_norm, 1, dim, M->eps, M->unit_norm, normed);
    if (hidden_out) memcpy(hidden_out, normed, dim * sizeof(float));
    if (logits) {
        mat_vec(&M->lm_head, normed, logits);
        if (M->final_softcap > 0.0f)
            for (size_t i = 0; i < M->vocab; i++)
                logits[i] = M->final_softcap * tanhf(logits[i] / M->final_softcap);
    }
    free(h); free(normed); free(q); free(k); free(v); free(tmpq); free(tmpk);
    free(attn); free(ao); free(g); free(u); free(act); free(ff);
    return 0;
}

int orc_model_set_tap(orc_model* M, long layer) {
    free(M->tap_q); free(M->tap_post_attn); free(M->tap_layer_out);
    M->tap_q = M->tap_post_attn = M->tap_layer_out = NULL;
    M->tap_layer = layer;
    if (layer < 0) return 0;
    if ((size_t)layer >= M->n_layers) return -1;
    M->tap_q = (float*)calloc(M->n_heads * M->hd, sizeof(float));
    M->tap_post_attn = (float*)calloc(M->dim, sizeof(float));
    M->tap_layer_out = (float*)calloc(M->dim, sizeof(float));
    return (M->tap_q && M->tap_post_attn && M->tap_layer_out) ? 0 : -1;
}

int orc_model_get_tap(const orc_model* M, float* q, float* post_attn, float* layer_out) {
    if (!M->tap_q) return -1;
    memcpy(q, M->tap_q, M->n_heads * M->hd * sizeof(float));
    memcpy(post_attn, M->tap_post_attn, M->dim * sizeof(float));
    memcpy(layer_out, M->tap_layer_out, M->dim * sizeof(float));
    return 0;
}

/* src/model/mod.rs:57-125.  Note the reference's loop checks the count after
 * pushing, so max_new == 0 still yields one token; out_tokens must hold
 * max(max_new, 1) entries. */
int orc_generate(orc_model* M, const uint32_t* prompt, size_t n_prompt,
                 size_t max_new, uint32_t* out_tokens, float* logits_out) {
    if (n_prompt == 0) return -1;
    size_t total = n_prompt + max_new;
    if (orc_model_reset(M, total)) return -1;
    float* logits = (float*)malloc(M->vocab * sizeof(float));
    uint32_t next = prompt[0];
    size_t produced = 0;
    int rc = 0;
    for (size_t pos = 0; pos < total; pos++) {
        int need_logits = (pos + 1 >= n_prompt);
        if (orc_model_step(M, next, pos, NULL, need_logits ? logits : NULL)) { rc = -1; break; }
        if (pos + 1 < n_prompt) {
            next = prompt[pos + 1];
        } else {
            uint32_t tok = orc_argmax(logits, M->vocab);
            if (logits_out) memcpy(logits_out + produced * M->vocab, logits, M->vocab * sizeof(float));
            out_tokens[produced++] = tok;
            next = tok;
            if (produced >= max_new) break;
        }
    }
    free(logits);
    return rc;
}
