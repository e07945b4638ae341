/*
 * Exact CPU statement of TurboQuant compress / decompress (test infrastructure).
 *
 * Not part of the product: only tests/, smoke() and bench.py's CPU baseline load
 * it. Follows the reference's CPU statement of the kernel
 * (crates/fracture-core/src/turboquant.rs:1225-1290 and :1056-1100) and the
 * kernels backends/fracture-cuda/kernels/turboquant_compress.cu:48-186 and
 * turboquant_decompress.cu:40-93:
 *
 *   sumsq  = sequential float sum of x_j*x_j        (separate mul/add roundings)
 *   norm   = sqrtf(sumsq), stored as fp16 (nearest-even)
 *   xn_j   = x_j / (norm + 1e-8f)                    (IEEE division)
 *   y_i    = sequential float sum_j Pi[i][j]*xn_j    (separate mul/add roundings)
 *   idx_i  = first k minimising fabsf(y_i - c_k)     (strict <)
 *   packed = MSB-first bit stream of idx (2/4/8-bit: the reference layout;
 *            3-bit: the same stream rule)
 *
 * Build with -ffp-contract=off (oracle/Makefile) so no multiply-add is fused.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400) == 0);
            man &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float bf16_to_f32(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* float -> fp16 bits, round to nearest even (also for subnormals and overflow). */
static uint16_t f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00 | (ax > 0x7f800000u ? 0x200 : 0));
    }
    if (ax >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7c00);
    }
    if (ax < 0x38800000u) { /* result is subnormal or zero in fp16 */
        if (ax < 0x33000000u) return (uint16_t)sign; /* < 2^-25: rounds to 0 */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7fffff) | 0x800000;
        int shift = 126 - (int)e; /* 14 - (e - 127) + 13 - 1 ... */
        /* value = m * 2^(e-150); fp16 subnormal unit = 2^-24 => q = m * 2^(e-126) */
        uint32_t q = m >> (shift);
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 127 + 15;
    uint32_t m = ax & 0x7fffff;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (q & 1))) q++;
    return (uint16_t)(sign | q);
}

typedef struct {
    const void* x;
    int kind; /* 0 fp16 bits, 1 bf16 bits, 2 float32 */
    const float* rot;
    const float* cen;
    int n_levels;
    uint8_t* packed;
    uint16_t* norms;
    uint8_t* idx_out;
    long n_vec;
    int d;
    int bits;
    long begin, end;
} compress_job;

static void compress_range(compress_job* j) {
    const int d = j->d;
    const int P = (d * j->bits + 7) / 8;
    float* x = (float*)malloc(sizeof(float) * (size_t)d);
    float* xn = (float*)malloc(sizeof(float) * (size_t)d);
    int* id = (int*)malloc(sizeof(int) * (size_t)d);
    for (long v = j->begin; v < j->end; ++v) {
        for (int t = 0; t < d; ++t) {
            long off = v * d + t;
            if (j->kind == 0) x[t] = f16_to_f32(((const uint16_t*)j->x)[off]);
            else if (j->kind == 1) x[t] = bf16_to_f32(((const uint16_t*)j->x)[off]);
            else x[t] = ((const float*)j->x)[off];
        }
        float s = 0.0f;
        for (int t = 0; t < d; ++t) {
            float sq = x[t] * x[t];
            s = s + sq;
        }
        float norm = sqrtf(s);
        j->norms[v] = f32_to_f16(norm);
        float den = norm + 1e-8f;
        for (int t = 0; t < d; ++t) xn[t] = x[t] / den;
        for (int i = 0; i < d; ++i) {
            const float* row = j->rot + (size_t)i * d;
            float acc = 0.0f;
            for (int t = 0; t < d; ++t) {
                float p = row[t] * xn[t];
                acc = acc + p;
            }
            float best = fabsf(acc - j->cen[0]);
            int bi = 0;
            for (int k = 1; k < j->n_levels; ++k) {
                float dist = fabsf(acc - j->cen[k]);
                if (dist < best) { best = dist; bi = k; }
            }
            id[i] = bi;
            if (j->idx_out) j->idx_out[v * d + i] = (uint8_t)bi;
        }
        uint8_t* out = j->packed + v * P;
        memset(out, 0, (size_t)P);
        for (int i = 0; i < d; ++i) {
            for (int b = 0; b < j->bits; ++b) {
                long bitpos = (long)i * j->bits + b;
                if ((id[i] >> (j->bits - 1 - b)) & 1) out[bitpos >> 3] |= (uint8_t)(0x80u >> (bitpos & 7));
            }
        }
    }
    free(x);
    free(xn);
    free(id);
}

static void* compress_thread(void* p) {
    compress_range((compress_job*)p);
    return NULL;
}

/* x: [n_tok, heads, d]; packed: [n_tok, heads*P]; norms: [n_tok, heads] fp16 bits. */
int tq_oracle_compress(const void* x, int kind, const float* rot, const float* cen, int n_levels,
                       uint8_t* packed, uint16_t* norms, uint8_t* idx_out, long n_tok, int heads,
                       int d, int bits, int num_threads) {
    if (bits < 1 || bits > 8 || d <= 0 || n_levels != (1 << bits)) return 1;
    long n_vec = n_tok * heads;
    if (num_threads < 1) num_threads = 1;
    if (num_threads > 256) num_threads = 256;
    compress_job jobs[256];
    pthread_t th[256];
    long per = (n_vec + num_threads - 1) / num_threads;
    int started = 0;
    for (int t = 0; t < num_threads; ++t) {
        compress_job* j = &jobs[t];
        j->x = x; j->kind = kind; j->rot = rot; j->cen = cen; j->n_levels = n_levels;
        j->packed = packed; j->norms = norms; j->idx_out = idx_out; j->n_vec = n_vec;
        j->d = d; j->bits = bits;
        j->begin = t * per;
        j->end = (t + 1) * per < n_vec ? (t + 1) * per : n_vec;
        if (j->begin >= j->end) break;
        if (num_threads == 1) {
            compress_range(j);
        } else {
            pthread_create(&th[t], NULL, compress_thread, j);
            started++;
        }
    }
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
    return 0;
}

typedef struct {
    const uint8_t* packed;
    const uint16_t* norms;
    const float* rot;
    const float* cen;
    float* out;
    int d, bits;
    long begin, end;
} decompress_job;

static void decompress_range(decompress_job* j) {
    const int d = j->d;
    const int P = (d * j->bits + 7) / 8;
    float* yh = (float*)malloc(sizeof(float) * (size_t)d);
    for (long v = j->begin; v < j->end; ++v) {
        const uint8_t* in = j->packed + v * P;
        for (int i = 0; i < d; ++i) {
            int code = 0;
            for (int b = 0; b < j->bits; ++b) {
                long bitpos = (long)i * j->bits + b;
                code = (code << 1) | ((in[bitpos >> 3] >> (7 - (bitpos & 7))) & 1);
            }
            yh[i] = j->cen[code];
        }
        float nrm = f16_to_f32(j->norms[v]);
        for (int i = 0; i < d; ++i) {
            float acc = 0.0f;
            for (int t = 0; t < d; ++t) {
                float p = j->rot[(size_t)t * d + i] * yh[t];
                acc = acc + p;
            }
            j->out[v * d + i] = acc * nrm;
        }
    }
    free(yh);
}

static void* decompress_thread(void* p) {
    decompress_range((decompress_job*)p);
    return NULL;
}

/* packed: [n_tok, heads*P]; norms fp16 bits [n_tok, heads]; out float32 [n_tok, heads, d]. */
int tq_oracle_decompress(const uint8_t* packed, const uint16_t* norms, const float* rot,
                         const float* cen, float* out, long n_tok, int heads, int d, int bits,
                         int num_threads) {
    if (bits < 1 || bits > 8 || d <= 0) return 1;
    long n_vec = n_tok * heads;
    if (num_threads < 1) num_threads = 1;
    if (num_threads > 256) num_threads = 256;
    decompress_job jobs[256];
    pthread_t th[256];
    long per = (n_vec + num_threads - 1) / num_threads;
    int started = 0;
    for (int t = 0; t < num_threads; ++t) {
        decompress_job* j = &jobs[t];
        j->packed = packed; j->norms = norms; j->rot = rot; j->cen = cen; j->out = out;
        j->d = d; j->bits = bits;
        j->begin = t * per;
        j->end = (t + 1) * per < n_vec ? (t + 1) * per : n_vec;
        if (j->begin >= j->end) break;
        if (num_threads == 1) {
            decompress_range(j);
        } else {
            pthread_create(&th[t], NULL, decompress_thread, j);
            started++;
        }
    }
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
    return 0;
}
