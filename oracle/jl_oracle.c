/*
 * jl_oracle.c -- CPU restatement of the reference engine's forward pass,
 * MXFP4 codec and quantizer.  TEST INFRASTRUCTURE ONLY (see jl_oracle.h).
 *
 * Citations are to the reference project (fawwaz46/jalapenos-at-home):
 *   engine/src/lib.rs, engine/src/model.rs, engine/src/mxfp4.rs,
 *   python/quantize_mxfp4.py.
 * Build flags: -O2 -ffp-contract=off (no fused multiply-add, as Rust).
 */
#include "jl_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define HEAD_DIM 128
#define HALF_DIM 64
static const float ROPE_THETA = 1000000.0f; /* lib.rs:25 */

/* ------------------------------------------------------------------ */
/* scalar formats                                                       */

float jlo_bf16_to_f32(uint16_t bits) {
    uint32_t u = (uint32_t)bits << 16; /* lib.rs:74-76 */
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t jlo_f32_to_bf16(float value) {
    uint32_t u;
    memcpy(&u, &value, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40); /* quiet NaN */
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

/* ------------------------------------------------------------------ */
/* MXFP4 codec                                                          */

static const float LEVELS[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f}; /* mxfp4.rs:3 */

int jlo_mxfp4_validate(size_t rows, size_t cols, size_t packed_len, size_t scales_len,
                       const uint8_t* scales) {
    /* mxfp4.rs:11-25 */
    if (rows == 0 || cols == 0 || cols % 32 != 0) return -1;
    if (rows > SIZE_MAX / cols) return -1;
    size_t elements = rows * cols;
    if (packed_len != elements / 2 || scales_len != elements / 32) return -2;
    for (size_t i = 0; i < scales_len; ++i)
        if (scales[i] == 255) return -3;
    return 0;
}

float jlo_mxfp4_value(const uint8_t* packed, const uint8_t* scales, size_t index) {
    /* mxfp4.rs:28-33 */
    unsigned code = (packed[index / 2] >> (4 * (index % 2))) & 15u;
    int exponent = (int)scales[index / 32] - 127;
    float magnitude = LEVELS[code & 7] * ldexpf(1.0f, exponent); /* powi is exact for these */
    return (code & 8) == 0 ? magnitude : -magnitude;
}

void jlo_mxfp4_values(const uint8_t* packed, const uint8_t* scales, size_t start, size_t end,
                      float* out) {
    /* mxfp4.rs:35-49: one scale per 32-block, applied to each level */
    size_t k = 0;
    for (size_t block = start / 32; block < (end + 31) / 32; ++block) {
        float scale = ldexpf(1.0f, (int)scales[block] - 127);
        size_t lo = start > block * 32 ? start : block * 32;
        size_t hi = end < (block + 1) * 32 ? end : (block + 1) * 32;
        for (size_t index = lo; index < hi; ++index) {
            unsigned code = (packed[index / 2] >> (4 * (index % 2))) & 15u;
            float magnitude = LEVELS[code & 7] * scale;
            out[k++] = (code & 8) == 0 ? magnitude : -magnitude;
        }
    }
}

int jlo_mxfp4_quantize(const float* values, size_t rows, size_t width, uint8_t* packed,
                       uint8_t* scales) {
    /* quantize_mxfp4.py:18-39 */
    static const float MIDPOINTS[7] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f};
    if (width % 32 != 0) return -1;                /* :21-22 */
    for (size_t i = 0; i < rows * width; ++i)      /* :23-24 */
        if (!isfinite(values[i])) return -2;
    size_t blocks = width / 32;
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
        for (size_t b = 0; b < blocks; ++b) {
            const float* v = values + r * width + b * 32;
            float maximum = 0.0f;                  /* :27 np.max(np.abs(blocks)) */
            for (int i = 0; i < 32; ++i) {
                float a = fabsf(v[i]);
                if (a > maximum) maximum = a;
            }
            int e = 0;
            frexpf(maximum, &e);                   /* :29 frexp -> floor(log2)+1 */
            int exponent = e - 3;
            if (exponent < -127) exponent = -127;
            if (exponent > 127) exponent = 127;
            if (maximum == 0.0f) exponent = -127;  /* :30 */
            uint8_t codes[32];
            for (int i = 0; i < 32; ++i) {
                float scaled = ldexpf(fabsf(v[i]), -exponent);      /* :31 */
                unsigned code = 0;                                   /* :32 searchsorted left */
                while (code < 7 && MIDPOINTS[code] < scaled) ++code;
                float midpoint = MIDPOINTS[code < 6 ? code : 6];    /* :33 */
                if ((code & 1u) && scaled == midpoint) code += 1;   /* :34 ties to even */
                if (signbit(v[i])) code |= 8u;                       /* :35 */
                codes[i] = (uint8_t)code;
            }
            uint8_t* p = packed + r * (width / 2) + b * 16;
            for (int j = 0; j < 16; ++j)                             /* :37 */
                p[j] = (uint8_t)(codes[2 * j] | (codes[2 * j + 1] << 4));
            scales[r * blocks + b] = (uint8_t)(exponent + 127);      /* :38 */
        }
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* seeded synthetic weights                                            */

static inline void philox_round(uint32_t c[4], uint32_t k0, uint32_t k1) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
}

void jlo_philox4x32_10(const uint32_t ctr[4], uint32_t k0, uint32_t k1, uint32_t out[4]) {
    uint32_t c[4] = {ctr[0], ctr[1], ctr[2], ctr[3]};
    for (int r = 0; r < 10; ++r) {
        if (r > 0) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        philox_round(c, k0, k1);
    }
    memcpy(out, c, sizeof c);
}

/* Fixed words that separate the weight stream from any other Philox use. */
#define SYNTH_CTR3 0x6a616c61u /* "jala" */
#define SYNTH_KEY1 0x70656e6fu /* "peno" */

void jlo_synth_bf16(uint64_t seed, uint32_t tensor_index, uint64_t first, size_t n, uint16_t* out) {
    const double two_pi = 6.283185307179586476925286766559;
    const double inv32 = 1.0 / 4294967296.0;
#pragma omp parallel for schedule(static)
    for (int64_t g = (int64_t)(first / 4); g < (int64_t)((first + n + 3) / 4); ++g) {
        uint32_t ctr[4] = {(uint32_t)g, (uint32_t)((uint64_t)g >> 32), tensor_index, SYNTH_CTR3};
        uint32_t r[4];
        uint32_t k0 = (uint32_t)seed ^ (uint32_t)(seed >> 32);
        jlo_philox4x32_10(ctr, k0, SYNTH_KEY1, r);
        double u0 = ((double)r[0] + 0.5) * inv32, u1 = ((double)r[1] + 0.5) * inv32;
        double u2 = ((double)r[2] + 0.5) * inv32, u3 = ((double)r[3] + 0.5) * inv32;
        double a = sqrt(-2.0 * log(u0)), b = sqrt(-2.0 * log(u2));
        double z[4] = {a * cos(two_pi * u1), a * sin(two_pi * u1), b * cos(two_pi * u3),
                       b * sin(two_pi * u3)};
        for (int j = 0; j < 4; ++j) {
            uint64_t e = (uint64_t)g * 4 + (uint64_t)j;
            if (e < first || e >= first + n) continue;
            out[e - first] = jlo_f32_to_bf16((float)(0.02 * z[j]));
        }
    }
}

/* ------------------------------------------------------------------ */
/* model                                                                */

typedef struct {
    int kind, rows, cols;
    const uint16_t* bf16;
    const uint8_t* packed;
    const uint8_t* scales;
} matrix_t;

typedef struct {
    matrix_t proj[7];
    const uint16_t* norm[4]; /* input_ln, post_ln, q_norm, k_norm */
} layer_t;

struct jlo_model {
    int layers, hidden, q_heads, kv_heads, inter, vocab, max_positions, eos;
    matrix_t embed, head;
    int has_head;
    const uint16_t* final_norm;
    layer_t* layer;
};

struct jlo_cache {
    int layers, width, round_bf16;
    size_t len, cap;
    float** keys;
    float** values;
};

jlo_model* jlo_model_new(int layers, int hidden, int q_heads, int kv_heads, int inter, int vocab,
                         int max_positions, int eos) {
    jlo_model* m = (jlo_model*)calloc(1, sizeof *m);
    if (!m) return NULL;
    m->layers = layers;
    m->hidden = hidden;
    m->q_heads = q_heads;
    m->kv_heads = kv_heads;
    m->inter = inter;
    m->vocab = vocab;
    m->max_positions = max_positions;
    m->eos = eos;
    m->layer = (layer_t*)calloc(layers > 0 ? (size_t)layers : 1, sizeof(layer_t));
    return m;
}

void jlo_model_free(jlo_model* m) {
    if (!m) return;
    free(m->layer);
    free(m);
}

static matrix_t* matrix_slot(jlo_model* m, int which, int layer) {
    if (which == JLO_EMBED) return &m->embed;
    if (which == JLO_HEAD) return &m->head;
    if (which >= JLO_Q && which <= JLO_DOWN && layer >= 0 && layer < m->layers)
        return &m->layer[layer].proj[which];
    return NULL;
}

static const matrix_t* matrix_get(const jlo_model* m, int which, int layer) {
    return matrix_slot((jlo_model*)m, which, layer);
}

int jlo_model_set_matrix(jlo_model* m, int which, int layer, int kind, int rows, int cols,
                         const uint16_t* bf16, const uint8_t* packed, const uint8_t* scales) {
    matrix_t* s = matrix_slot(m, which, layer);
    if (!s) return -1;
    if (kind == JLO_BF16 && !bf16) return -1;
    if (kind == JLO_MXFP4 && (!packed || !scales || cols % 32)) return -1;
    s->kind = kind;
    s->rows = rows;
    s->cols = cols;
    s->bf16 = bf16;
    s->packed = packed;
    s->scales = scales;
    if (which == JLO_HEAD) m->has_head = 1;
    return 0;
}

int jlo_model_set_norm(jlo_model* m, int which, int layer, const uint16_t* bf16) {
    if (which == JLO_FINAL_NORM) {
        m->final_norm = bf16;
        return 0;
    }
    if (which < JLO_INPUT_LN || which > JLO_K_NORM || layer < 0 || layer >= m->layers) return -1;
    m->layer[layer].norm[which - JLO_INPUT_LN] = bf16;
    return 0;
}

jlo_cache* jlo_cache_new(const jlo_model* m, int round_bf16) {
    jlo_cache* c = (jlo_cache*)calloc(1, sizeof *c);
    if (!c) return NULL;
    c->layers = m->layers;
    c->width = m->kv_heads * HEAD_DIM;
    c->round_bf16 = round_bf16;
    size_t n = m->layers > 0 ? (size_t)m->layers : 1;
    c->keys = (float**)calloc(n, sizeof(float*));
    c->values = (float**)calloc(n, sizeof(float*));
    return c;
}

void jlo_cache_free(jlo_cache* c) {
    if (!c) return;
    for (int l = 0; l < c->layers; ++l) {
        free(c->keys[l]);
        free(c->values[l]);
    }
    free(c->keys);
    free(c->values);
    free(c);
}

size_t jlo_cache_len(const jlo_cache* c) { return c->len; }

int jlo_cache_truncate(jlo_cache* c, size_t len) {
    if (len > c->len) return -1; /* model.rs:46 assert!(len <= self.len) */
    c->len = len;
    return 0;
}

static int cache_reserve(jlo_cache* c, size_t tokens) {
    if (tokens <= c->cap) return 0;
    size_t cap = c->cap ? c->cap : 64;
    while (cap < tokens) cap *= 2;
    for (int l = 0; l < c->layers; ++l) {
        float* k = (float*)realloc(c->keys[l], cap * (size_t)c->width * sizeof(float));
        if (!k) return -1;
        c->keys[l] = k;
        float* v = (float*)realloc(c->values[l], cap * (size_t)c->width * sizeof(float));
        if (!v) return -1;
        c->values[l] = v;
    }
    c->cap = cap;
    return 0;
}

/* ---- building blocks ----------------------------------------------- */

/* Signed E2M1 level of each nibble of a byte: [byte][0] the low nibble (the
 * even element), [byte][1] the high one. */
static float g_pair_levels[256][2];
static int g_pair_ready = 0;

static void pair_levels_init(void) {
    if (g_pair_ready) return;
#pragma omp critical(jlo_pair_levels)
    if (!g_pair_ready) {
        for (int b = 0; b < 256; ++b)
            for (int h = 0; h < 2; ++h) {
                unsigned code = (unsigned)(b >> (4 * h)) & 15u;
                g_pair_levels[b][h] = (code & 8) ? -LEVELS[code & 7] : LEVELS[code & 7];
            }
        g_pair_ready = 1;
    }
}

static void decode_row(const matrix_t* w, int r, float* wrow) {
    /* mxfp4.rs:35-49 for one row.  A level times a power-of-two scale is the
     * same number whichever sign is applied first (round to nearest even is
     * symmetric), so the signed table gives Mxfp4::values' exact values. */
    const int K = w->cols;
    if (w->kind == JLO_MXFP4) {
        const uint8_t* p = w->packed + (size_t)r * (K / 2);
        const uint8_t* sc = w->scales + (size_t)r * (K / 32);
        for (int b = 0; b < K / 32; ++b) {
            const float scale = ldexpf(1.0f, (int)sc[b] - 127);
            for (int j = 0; j < 16; ++j) {
                const uint8_t byte = p[b * 16 + j];
                wrow[b * 32 + 2 * j] = g_pair_levels[byte][0] * scale;
                wrow[b * 32 + 2 * j + 1] = g_pair_levels[byte][1] * scale;
            }
        }
    } else {
        const uint16_t* src = w->bf16 + (size_t)r * K;
        for (int i = 0; i < K; ++i) {
            uint32_t u = (uint32_t)src[i] << 16;
            memcpy(&wrow[i], &u, 4);
        }
    }
}

static void matmul_rows(const matrix_t* w, const float* x, size_t rows, float* y) {
    /* lib.rs:240-266: each sum starts at 0.0 and adds x*w in order of i.
     * A weight row is decoded once (Mxfp4::values gives the same exact
     * values as Mxfp4::value).  One token row: four weight rows are summed
     * side by side (their decoded values interleaved, so the four sums are
     * one vector operation).  Several token rows: eight token rows side by
     * side, from a transposed copy of x.  Every sum still accumulates in
     * index order with separately rounded products, so results are
     * identical to the one-row-at-a-time loop. */
    const int K = w->cols, O = w->rows;
    pair_levels_init();
    float* xt = NULL;
    const size_t groups = (rows + 7) / 8;
    if (rows > 1) {
        /* xt[g][i][j] = x[8g + j][i] (zero past the last row) */
        xt = (float*)calloc(groups * (size_t)K * 8, sizeof(float));
        if (!xt) abort();
        for (size_t t = 0; t < rows; ++t)
            for (int i = 0; i < K; ++i) xt[((t / 8) * (size_t)K + i) * 8 + t % 8] = x[t * (size_t)K + i];
    }
#pragma omp parallel
    {
        float* wrow = (float*)malloc((size_t)4 * K * sizeof(float));
        float* w4 = (float*)malloc((size_t)4 * K * sizeof(float));
        if (!wrow || !w4) abort();
        if (rows == 1) {
#pragma omp for schedule(static)
            for (int r0 = 0; r0 < O; r0 += 4) {
                const int nr = O - r0 < 4 ? O - r0 : 4;
                for (int j = 0; j < 4; ++j) decode_row(w, r0 + (j < nr ? j : 0), wrow + (size_t)j * K);
                for (int i = 0; i < K; ++i)
                    for (int j = 0; j < 4; ++j) w4[(size_t)i * 4 + j] = wrow[(size_t)j * K + i];
                float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                for (int i = 0; i < K; ++i) {
                    const float xi = x[i];
                    for (int j = 0; j < 4; ++j) s[j] += xi * w4[(size_t)i * 4 + j];
                }
                for (int j = 0; j < nr; ++j) y[r0 + j] = s[j];
            }
        } else {
#pragma omp for schedule(static)
            for (int r = 0; r < O; ++r) {
                decode_row(w, r, wrow);
                for (size_t g = 0; g < groups; ++g) {
                    const size_t t0 = g * 8;
                    const size_t nt = rows - t0 < 8 ? rows - t0 : 8;
                    const float* xg = xt + g * (size_t)K * 8;
                    float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                    for (int i = 0; i < K; ++i) {
                        const float wi = wrow[i];
                        for (int j = 0; j < 8; ++j) sum[j] += xg[(size_t)i * 8 + j] * wi;
                    }
                    for (size_t j = 0; j < nt; ++j) y[(t0 + j) * (size_t)O + r] = sum[j];
                }
            }
        }
        free(wrow);
        free(w4);
    }
    free(xt);
}

int jlo_matmul(const jlo_model* m, int which, int layer, const float* x, size_t rows, float* y) {
    const matrix_t* w = matrix_get(m, which, layer);
    if (!w || (!w->bf16 && !w->packed)) return -1;
    matmul_rows(w, x, rows, y);
    return 0;
}

int jlo_matmul_raw(int kind, int rows, int cols, const uint16_t* bf16, const uint8_t* packed,
                   const uint8_t* scales, const float* x, size_t n, float* y) {
    matrix_t w = {kind, rows, cols, bf16, packed, scales};
    if (kind == JLO_MXFP4 ? (!packed || !scales || cols % 32) : !bf16) return -1;
    matmul_rows(&w, x, n, y);
    return 0;
}

void jlo_rms_norm(const float* x, size_t rows, size_t width, const uint16_t* w, float* out) {
    /* lib.rs:268-290 */
    for (size_t t = 0; t < rows; ++t) {
        const float* xt = x + t * width;
        float sum = 0.0f;
        for (size_t i = 0; i < width; ++i) sum += xt[i] * xt[i];
        float average = sum / (float)width;
        float size = sqrtf(average + 1e-6f);
        for (size_t i = 0; i < width; ++i) out[t * width + i] = xt[i] / size * jlo_bf16_to_f32(w[i]);
    }
}

void jlo_rope(float* x, size_t rows, size_t heads, size_t offset) {
    /* lib.rs:291-321.  Reads the un-rotated input for every pair. */
    const size_t row_len = heads * HEAD_DIM;
    for (size_t t = 0; t < rows; ++t) {
        float position = (float)(offset + t);
        for (size_t h = 0; h < heads; ++h) {
            float* head = x + t * row_len + h * HEAD_DIM;
            for (int i = 0; i < HALF_DIM; ++i) {
                float freq = 1.0f / powf(ROPE_THETA, (float)i / (float)HALF_DIM);
                float angle = position * freq;
                float c = cosf(angle), s = sinf(angle);
                float a = head[i], b = head[i + HALF_DIM];
                head[i] = a * c - b * s;
                head[i + HALF_DIM] = b * c + a * s;
            }
        }
    }
}

uint32_t jlo_argmax(const float* values, size_t n) {
    /* model.rs:288-296 */
    size_t best = 0;
    for (size_t i = 1; i < n; ++i)
        if (values[i] > values[best]) best = i;
    return (uint32_t)best;
}

void jlo_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int jlo_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---- layers ----------------------------------------------------------- */

static float round_kv(float v, int round_bf16) {
    return round_bf16 ? jlo_bf16_to_f32(jlo_f32_to_bf16(v)) : v;
}

/* attention (lib.rs:337-450) for `rows` tokens starting at cache position
 * `offset`; appends keys/values to layer `l` of the cache. */
static int attention(const jlo_model* m, jlo_cache* cache, int l, const float* x, size_t rows,
                     size_t offset, float* out) {
    const layer_t* L = &m->layer[l];
    const size_t q_len = (size_t)m->q_heads * HEAD_DIM, kv_len = (size_t)m->kv_heads * HEAD_DIM;
    float* q = (float*)malloc(rows * q_len * sizeof(float));
    float* k = (float*)malloc(rows * kv_len * sizeof(float));
    float* v = (float*)malloc(rows * kv_len * sizeof(float));
    float* mixed = (float*)calloc(rows * q_len, sizeof(float));
    if (!q || !k || !v || !mixed) {
        free(q); free(k); free(v); free(mixed);
        return -2;
    }
    matmul_rows(&L->proj[JLO_Q], x, rows, q); /* :353-355 */
    matmul_rows(&L->proj[JLO_K], x, rows, k);
    matmul_rows(&L->proj[JLO_V], x, rows, v);
    /* :363-374 per-head RMSNorm, in place is safe (row read before write) */
    jlo_rms_norm(q, rows * m->q_heads, HEAD_DIM, L->norm[2], q);
    jlo_rms_norm(k, rows * m->kv_heads, HEAD_DIM, L->norm[3], k);
    jlo_rope(q, rows, m->q_heads, offset); /* :387-388 */
    jlo_rope(k, rows, m->kv_heads, offset);
    /* :393-396 append post-RoPE keys and values */
    float* K = cache->keys[l];
    float* V = cache->values[l];
    for (size_t i = 0; i < rows * kv_len; ++i) {
        K[offset * kv_len + i] = round_kv(k[i], cache->round_bf16);
        V[offset * kv_len + i] = round_kv(v[i], cache->round_bf16);
    }
    const int group = m->q_heads / m->kv_heads;           /* :397 */
    const float scale = sqrtf((float)HEAD_DIM);           /* :398 */
    /* every (row, head) pair is independent: threads take whole pairs, each
     * computed in the reference's order */
    const long pairs = (long)rows * m->q_heads;
    int fail = 0;
#pragma omp parallel
    {
        float* sc = (float*)malloc((offset + rows) * sizeof(float));
        if (!sc) {
#pragma omp atomic write
            fail = 1;
        }
#pragma omp for schedule(dynamic, 1)
        for (long p = 0; p < pairs; ++p) {
            if (!sc) continue;
            const size_t t = (size_t)(p / m->q_heads);
            const int h = (int)(p % m->q_heads);
            int kv_h = h / group;
            const float* qh = q + t * q_len + (size_t)h * HEAD_DIM;
            size_t visible = offset + t + 1;
            for (size_t s = 0; s < visible; ++s) {          /* :410-417 */
                const float* kh = K + s * kv_len + (size_t)kv_h * HEAD_DIM;
                float dot = 0.0f;
                for (int i = 0; i < HEAD_DIM; ++i) dot += qh[i] * kh[i];
                sc[s] = dot / scale;
            }
            float max = -INFINITY;                          /* :420-425 */
            for (size_t s = 0; s < visible; ++s)
                if (sc[s] > max) max = sc[s];
            float total = 0.0f;                             /* :426-430 */
            for (size_t s = 0; s < visible; ++s) {
                sc[s] = expf(sc[s] - max);
                total += sc[s];
            }
            float* o = mixed + t * q_len + (size_t)h * HEAD_DIM;
            for (size_t s = 0; s < visible; ++s) {          /* :433-439 */
                float share = sc[s] / total;
                const float* vh = V + s * kv_len + (size_t)kv_h * HEAD_DIM;
                for (int i = 0; i < HEAD_DIM; ++i) o[i] += share * vh[i];
            }
        }
        free(sc);
    }
    if (fail) {
        free(q); free(k); free(v); free(mixed);
        return -2;
    }
    matmul_rows(&L->proj[JLO_O], mixed, rows, out); /* :444-449 */
    free(q); free(k); free(v); free(mixed);
    return 0;
}

/* mlp (lib.rs:452-468) */
static int mlp(const jlo_model* m, int l, const float* x, size_t rows, float* out) {
    const layer_t* L = &m->layer[l];
    size_t n = rows * (size_t)m->inter;
    float* gate = (float*)malloc(n * sizeof(float));
    float* up = (float*)malloc(n * sizeof(float));
    if (!gate || !up) {
        free(gate); free(up);
        return -2;
    }
    matmul_rows(&L->proj[JLO_GATE], x, rows, gate);
    matmul_rows(&L->proj[JLO_UP], x, rows, up);
    for (size_t i = 0; i < n; ++i) gate[i] = (gate[i] / (1.0f + expf(-gate[i]))) * up[i];
    matmul_rows(&L->proj[JLO_DOWN], gate, rows, out);
    free(gate); free(up);
    return 0;
}

static void embed_rows(const jlo_model* m, const uint32_t* tokens, size_t n, float* x) {
    /* lib.rs:213-235 then model.rs:167-170 (bf16 -> f32) */
    const matrix_t* e = &m->embed;
    const size_t width = (size_t)e->cols;
    for (size_t t = 0; t < n; ++t) {
        size_t start = (size_t)tokens[t] * width;
        if (e->kind == JLO_MXFP4) {
            jlo_mxfp4_values(e->packed, e->scales, start, start + width, x + t * width);
            for (size_t i = 0; i < width; ++i) {
                uint32_t u;
                memcpy(&u, &x[t * width + i], 4);
                x[t * width + i] = jlo_bf16_to_f32((uint16_t)(u >> 16)); /* truncation, :227 */
            }
        } else {
            for (size_t i = 0; i < width; ++i) x[t * width + i] = jlo_bf16_to_f32(e->bf16[start + i]);
        }
    }
}

int jlo_append_hidden(const jlo_model* m, jlo_cache* c, const uint32_t* tokens, size_t n,
                      int layers, float* out) {
    /* model.rs:163-164 */
    if (n == 0 || c->len + n > (size_t)m->max_positions) return -1;
    if (layers < 0 || layers > m->layers) return -1;
    for (size_t t = 0; t < n; ++t)
        if (tokens[t] >= (uint32_t)m->embed.rows) return -1;
    if (cache_reserve(c, c->len + n)) return -2;
    const size_t H = (size_t)m->hidden;
    float* normalized = (float*)malloc(n * H * sizeof(float));
    float* delta = (float*)malloc(n * H * sizeof(float));
    if (!normalized || !delta) {
        free(normalized); free(delta);
        return -2;
    }
    embed_rows(m, tokens, n, out);
    int rc = 0;
    for (int l = 0; l < layers && rc == 0; ++l) {
        const layer_t* L = &m->layer[l];
        jlo_rms_norm(out, n, H, L->norm[0], normalized);            /* :174-177 */
        rc = attention(m, c, l, normalized, n, c->len, delta);      /* :178-185 */
        if (rc) break;
        for (size_t i = 0; i < n * H; ++i) out[i] += delta[i];      /* :186-188 */
        jlo_rms_norm(out, n, H, L->norm[1], normalized);            /* :190-193 */
        rc = mlp(m, l, normalized, n, delta);                       /* :194 */
        if (rc) break;
        for (size_t i = 0; i < n * H; ++i) out[i] += delta[i];      /* :195-197 */
    }
    free(normalized);
    free(delta);
    if (rc) return rc;
    c->len += n;                                                    /* :199 */
    return 0;
}

int jlo_predict(const jlo_model* m, jlo_cache* c, const uint32_t* tokens, size_t n, int all,
                uint32_t* out_ids, float* out_logits) {
    /* model.rs:209-240 */
    const size_t H = (size_t)m->hidden;
    float* hidden = (float*)malloc((n ? n : 1) * H * sizeof(float));
    if (!hidden) return -2;
    int rc = jlo_append_hidden(m, c, tokens, n, m->layers, hidden);
    if (rc) {
        free(hidden);
        return rc;
    }
    size_t rows = all ? n : 1;
    const float* src = all ? hidden : hidden + (n - 1) * H;  /* :222-227 last row only */
    float* normalized = (float*)malloc(rows * H * sizeof(float));
    const matrix_t* head = m->has_head ? &m->head : &m->embed; /* :229-233 */
    float* logits = (float*)malloc(rows * (size_t)head->rows * sizeof(float));
    if (!normalized || !logits) {
        free(hidden); free(normalized); free(logits);
        return -2;
    }
    jlo_rms_norm(src, rows, H, m->final_norm, normalized);      /* :228 */
    matmul_rows(head, normalized, rows, logits);                /* :234 */
    for (size_t r = 0; r < rows; ++r) {                         /* :235-239 */
        out_ids[r] = jlo_argmax(logits + r * (size_t)head->rows, (size_t)head->rows);
        if (out_logits)
            memcpy(out_logits + r * (size_t)head->rows, logits + r * (size_t)head->rows,
                   (size_t)head->rows * sizeof(float));
    }
    free(hidden); free(normalized); free(logits);
    return 0;
}
