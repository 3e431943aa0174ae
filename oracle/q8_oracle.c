/* q8_oracle.c: TEST INFRASTRUCTURE ONLY (see q8_oracle.h for what it restates and from where).
 * Built with -ffp-contract=off so that every a*b+c here is two roundings unless written as fmaf,
 * the convention of the reference's host builds (scripts/lib.sh:34-37). */
#include "q8_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define QK 32
#define BLOCK_BYTES 34

/* ---------------------------------------------------------------- formats */

/* IEEE binary16 -> binary32, exact for every pattern; a NaN keeps its payload shifted into
 * place and its quiet bit as it was (the decode of src/card/knc.h:157-173, written from the
 * binary16 definition: subnormals are m * 2^-24). */
float q8o_half(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 31u, man = h & 1023u;
    uint32_t bits;
    float f;
    if (exp == 0) {
        f = ldexpf((float)man, -24); /* exact: man < 2^10 */
        return sign ? -f : f;
    }
    if (exp == 31)
        bits = sign | 0x7f800000u | man << 13;
    else
        bits = sign | (exp + 112u) << 23 | man << 13;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t q8o_to_half(float f)
{
    _Float16 h = (_Float16)f; /* the compiler's conversion: round to nearest even */
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

long q8o_gguf_bytes(long rows, long cols) { return rows * (cols / QK) * BLOCK_BYTES; }

long q8o_split_scale_stride(long cols) { return (cols / QK + 7) / 8 * 8; }

long q8o_split_row_bytes(long cols) { return cols + 2 * q8o_split_scale_stride(cols); }

long q8o_split_bytes(long rows, long cols) { return rows * q8o_split_row_bytes(cols); }

/* The row-split layout: row r at r * (cols + 2*S) holds its cols int8 quants, then its cols/32
 * fp16 scales padded with zeros to S = cols/32 rounded up to a multiple of 8 entries. */
void q8o_repack_split(const uint8_t *q8, long rows, long cols, uint8_t *out)
{
    const long nb = cols / QK, ss = q8o_split_scale_stride(cols), rb = q8o_split_row_bytes(cols);
    for (long r = 0; r < rows; r++) {
        uint8_t *row = out + r * rb;
        memset(row + cols, 0, (size_t)(ss * 2));
        for (long b = 0; b < nb; b++) {
            const uint8_t *blk = q8 + (r * nb + b) * BLOCK_BYTES;
            memcpy(row + cols + b * 2, blk, 2);
            memcpy(row + b * QK, blk + 2, QK);
        }
    }
}

void q8o_unpack_split(const uint8_t *split, long rows, long cols, uint8_t *q8)
{
    const long nb = cols / QK, rb = q8o_split_row_bytes(cols);
    for (long r = 0; r < rows; r++) {
        const uint8_t *row = split + r * rb;
        for (long b = 0; b < nb; b++) {
            uint8_t *blk = q8 + (r * nb + b) * BLOCK_BYTES;
            memcpy(blk, row + cols + b * 2, 2);
            memcpy(blk + 2, row + b * QK, QK);
        }
    }
}

/* ---------------------------------------------------------------- synthetic inputs */

/* splitmix64's output function (Steele, Lea, Flood 2014) */
static inline uint64_t mix64(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* An approximately normal N(0,1) value, exactly reproducible on any IEEE machine: the
 * Irwin-Hall sum of 12 uniform 16-bit integers, each centred by +1/2, scaled by 2^-16, minus 6.
 * Mean 0, variance 1; every step is exact in binary32. Element `index` of stream `stream`. */
float q8o_normal(uint64_t seed, uint64_t stream, uint64_t index)
{
    const uint64_t base = mix64(seed + 0x9E3779B97F4A7C15ull * (stream + 1));
    uint32_t s = 0;
    for (uint64_t k = 0; k < 3; k++) {
        const uint64_t z = mix64(base + (index * 3 + k + 1) * 0x9E3779B97F4A7C15ull);
        s += (uint32_t)(z & 0xffff) + (uint32_t)((z >> 16) & 0xffff) + (uint32_t)((z >> 32) & 0xffff) + (uint32_t)(z >> 48);
    }
    /* (2s + 12) * 2^-17 - 6: exact (2s + 12 < 2^21) */
    return (float)(2 * s + 12) * (1.0f / 131072.0f) - 6.0f;
}

void q8o_fill_f32(float *out, long n, uint64_t seed, uint64_t stream, float sigma)
{
    for (long i = 0; i < n; i++)
        out[i] = q8o_normal(seed, stream, (uint64_t)i) * sigma;
}

/* llama.cpp's Q8_0 convention: d = amax/127 in binary32, stored as fp16; q = round(w * (1/d)) */
void q8o_fill_q8_0(uint8_t *out, long row0, long rows, long cols, uint64_t seed, uint64_t stream, float sigma)
{
    const long nb = cols / QK;
    for (long r = 0; r < rows; r++)
        for (long b = 0; b < nb; b++) {
            float w[QK], amax = 0.0f;
            for (int i = 0; i < QK; i++) {
                w[i] = q8o_normal(seed, stream, (uint64_t)((row0 + r) * cols + b * QK + i)) * sigma;
                const float a = fabsf(w[i]);
                amax = a > amax ? a : amax;
            }
            const float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
            uint8_t *blk = out + (r * nb + b) * BLOCK_BYTES;
            const uint16_t dh = q8o_to_half(d);
            memcpy(blk, &dh, 2);
            for (int i = 0; i < QK; i++) {
                float v = roundf(w[i] * id);
                v = v > 127.0f ? 127.0f : v < -127.0f ? -127.0f : v;
                blk[2 + i] = (uint8_t)(int8_t)v;
            }
        }
}

/* ---------------------------------------------------------------- products */

/* One output row in the reference's order (src/card/gemv.c:93-111: per tile `t` from zero, 32
 * fmas in column order, then one fma by the block's fp16 scale into the running sum). */
static float row_dot(const uint8_t *row, long nb, const float *x)
{
    float acc = 0.0f;
    for (long b = 0; b < nb; b++) {
        const uint8_t *blk = row + b * BLOCK_BYTES;
        uint16_t h;
        memcpy(&h, blk, 2);
        float t = 0.0f;
        for (int i = 0; i < QK; i++)
            t = fmaf((float)(int8_t)blk[2 + i], x[b * QK + i], t);
        acc = fmaf(t, q8o_half(h), acc);
    }
    return acc;
}

static double row_dot_f64(const uint8_t *row, long nb, const float *x)
{
    double acc = 0.0;
    for (long b = 0; b < nb; b++) {
        const uint8_t *blk = row + b * BLOCK_BYTES;
        uint16_t h;
        memcpy(&h, blk, 2);
        const double d = (double)q8o_half(h);
        for (int i = 0; i < QK; i++)
            acc += d * (double)(int8_t)blk[2 + i] * (double)x[b * QK + i];
    }
    return acc;
}

struct job {
    const uint8_t *q8;
    long rows, cols, t;
    const int32_t *idx; /* NULL: rows 0..rows-1 */
    const float *x;
    float *y;
    double *y64;
    int tid, n;
};

static void *worker(void *arg)
{
    const struct job *j = arg;
    const long nb = j->cols / QK, rb = nb * BLOCK_BYTES;
    const long r0 = j->rows * j->tid / j->n, r1 = j->rows * (j->tid + 1) / j->n;
    for (long r = r0; r < r1; r++) {
        const uint8_t *row = j->q8 + (j->idx ? (long)j->idx[r] : r) * rb;
        for (long k = 0; k < j->t; k++) {
            if (j->y64)
                j->y64[k * j->rows + r] = row_dot_f64(row, nb, j->x + k * j->cols);
            else
                j->y[k * j->rows + r] = row_dot(row, nb, j->x + k * j->cols);
        }
    }
    return NULL;
}

static void run(struct job proto, int threads)
{
    if (threads < 1)
        threads = 1;
    if (threads > 256)
        threads = 256;
    pthread_t th[256];
    struct job jobs[256];
    for (int i = 0; i < threads; i++) {
        jobs[i] = proto;
        jobs[i].tid = i;
        jobs[i].n = threads;
    }
    int started = 0;
    for (int i = 1; i < threads; i++)
        started += pthread_create(&th[i], NULL, worker, &jobs[i]) == 0 ? 1 : 0;
    worker(&jobs[0]);
    if (started != threads - 1) { /* a thread failed to start: do its share here */
        for (int i = 1; i < threads; i++)
            worker(&jobs[i]);
        return;
    }
    for (int i = 1; i < threads; i++)
        pthread_join(th[i], NULL);
}

void q8o_gemv(const uint8_t *q8, long rows, long cols, const float *x, float *y, int threads)
{
    run((struct job){.q8 = q8, .rows = rows, .cols = cols, .t = 1, .x = x, .y = y}, threads);
}

void q8o_gemm(const uint8_t *q8, long rows, long cols, const float *x, long t, float *y, int threads)
{
    run((struct job){.q8 = q8, .rows = rows, .cols = cols, .t = t, .x = x, .y = y}, threads);
}

void q8o_gemv_rows(const uint8_t *q8, long cols, const int32_t *idx, long n, const float *x, float *y, int threads)
{
    run((struct job){.q8 = q8, .rows = n, .cols = cols, .t = 1, .idx = idx, .x = x, .y = y}, threads);
}

void q8o_gemm_f64(const uint8_t *q8, long rows, long cols, const float *x, long t, double *y, int threads)
{
    run((struct job){.q8 = q8, .rows = rows, .cols = cols, .t = t, .x = x, .y64 = y}, threads);
}

/* ---------------------------------------------------------------- the gate known answers */

/* xorshift32 (Marsaglia 2003, shifts 13, 17, 5) and the exact unit value built from its top 24
 * bits, as the reference's gate inputs are drawn (src/gate/gate_common.h:22-35). */
static uint32_t xs32(uint32_t *s)
{
    uint32_t v = *s;
    v ^= v << 13;
    v ^= v >> 17;
    v ^= v << 5;
    return *s = v;
}

static float unit(uint32_t *s) { return (float)((int32_t)(xs32(s) >> 8) - 8388608) * (1.0f / 8388608.0f); }

static uint32_t bits_of(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

/* FNV-1a over the 32-bit result words (src/gate/gate_common.h:354-363) */
static uint64_t fnv1a32(const float *c, long n)
{
    uint64_t h = 0xcbf29ce484222325ull;
    for (long i = 0; i < n; i++) {
        h ^= bits_of(c[i]);
        h *= 0x100000001b3ull;
    }
    return h;
}

static float pow2f(int e)
{
    const uint32_t b = (uint32_t)(127 + e) << 23;
    float f;
    memcpy(&f, &b, 4);
    return f;
}

/* The judge's half conversion (src/gate/upconv_cmp.c:26-31): the compiler's _Float16 */
static float half_judge(uint16_t h)
{
    _Float16 f;
    memcpy(&f, &h, 2);
    return (float)f;
}

enum { N8 = 512, NB = 4096, NF = 131072, NH = 4096 };

void q8o_gate21_hashes(uint64_t out[7])
{
    /* the inputs, drawn in the order of src/gate/upconv_common.h:246-273 */
    static float x8[N8], c8[N8], xb[NB], cb[NB], sc[NB / 16], xf[NF], cf[NF], xh[NH];
    static float r_s8[N8], r_u8fma[N8], r_u8mul[N8], r_b16[NB], r_f16[NF], r_hsum[NH / 16];
    uint32_t s = 0x2545F491u;
    for (int i = 0; i < N8; i++) {
        const int second = i >= 256;
        x8[i] = second ? unit(&s) : 1.0f;
        c8[i] = second ? unit(&s) : 0.0f;
    }
    for (int i = 0; i < NF; i++) {
        const int second = i >= 65536;
        xf[i] = second ? unit(&s) : 1.0f;
        cf[i] = second ? unit(&s) : 0.0f;
    }
    for (int i = 0; i < NB; i++) {
        xb[i] = unit(&s);
        cb[i] = unit(&s);
    }
    for (int i = 0; i < NB / 16; i++)
        sc[i] = unit(&s);
    for (int i = 0; i < NH; i++) {
        const float m = unit(&s);
        xh[i] = m * pow2f((int)(xs32(&s) % 41u) - 20);
    }
    /* the results, as src/gate/upconv_cmp.c:45-59 computes them */
    for (int i = 0; i < N8; i++) {
        const float q = (float)(int8_t)(uint8_t)i, u = (float)(uint8_t)i;
        r_s8[i] = fmaf(x8[i], q, c8[i]);
        r_u8fma[i] = fmaf(x8[i], u, c8[i]);
        volatile float p = x8[i] * u;
        r_u8mul[i] = p + c8[i];
    }
    for (int i = 0; i < NB; i++)
        r_b16[i] = fmaf(xb[i], sc[i / 16], cb[i]);
    for (int i = 0; i < NF; i++)
        r_f16[i] = fmaf(xf[i], half_judge((uint16_t)i), cf[i]);
    for (int b = 0; b < NH / 16; b++) {
        float v[16], t[16];
        memcpy(v, xh + 16 * b, sizeof v);
        for (int k = 1; k < 16; k <<= 1) { /* the tree: lane pairs i^1, i^2, i^4, i^8 */
            for (int i = 0; i < 16; i++)
                t[i] = v[i] + v[i ^ k];
            memcpy(v, t, sizeof v);
        }
        r_hsum[b] = v[0];
    }
    out[0] = fnv1a32(r_s8, N8);
    out[1] = fnv1a32(r_u8fma, N8);
    out[2] = fnv1a32(r_u8mul, N8);
    out[3] = fnv1a32(r_b16, NB);
    out[4] = fnv1a32(r_b16, NB); /* bcast: the same arithmetic through another load */
    out[5] = fnv1a32(r_f16, NF);
    out[6] = fnv1a32(r_hsum, NH / 16);
}

void q8o_gate_a(uint64_t *hash, uint32_t words[3])
{
    enum { N = 4096 };
    static float a[N], b[N], c[N];
    uint32_t s = 0x9E3779B9u; /* src/gate/gate_common.h:20, 337-345 */
    for (int i = 0; i < N; i++) {
        a[i] = unit(&s);
        b[i] = unit(&s);
        c[i] = unit(&s);
    }
    for (int i = 0; i < N; i++)
        c[i] = fmaf(a[i], b[i], c[i]);
    *hash = fnv1a32(c, N);
    words[0] = bits_of(c[0]);
    words[1] = bits_of(c[1]);
    words[2] = bits_of(c[N - 1]);
}
