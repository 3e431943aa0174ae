/* q8_oracle.h: TEST INFRASTRUCTURE ONLY. A CPU restatement of the reference's Q8_0 weight
 * products (Lasimeri/Intel-Phi-APL), used by tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg as the checker. Nothing on the product path links or calls it.
 *
 * What it restates, and from where (paths inside the reference project):
 *   - the GGUF Q8_0 block: an fp16 scale d, then 32 int8 q; w = d*q
 *     (src/host/gguf_reader.c:21, src/apl/gguf_read.apl:37-46);
 *   - the exact IEEE binary16 -> binary32 decode of d (src/card/knc.h:157-173);
 *   - the product's rounding order, per output row: for each 32-column block a sequential
 *     fmaf chain t = fma(q_i, x_i, t) from +0 over the 32 columns, then acc = fma(t, d, acc),
 *     block after block from acc = +0 (src/card/gemv.c:90-117, the whole-group path of
 *     gemv_i_thread at src/card/gemv.c:168-181);
 *   - gemm: every token follows gemv's order bit for bit (src/card/gemm.h:6-7,
 *     src/card/gemm.c:25-156); x is [t][cols], y is [t][rows] (src/card/gemm.h:28-31);
 *   - the F64 check: dequantise exactly to double, then a double dot product
 *     (tests/host/gguf_rows.c:51-58, src/apl/ref_harness.apl:94);
 *   - the gate 2.1 and gate A known answers: the up-convert, fma and tree-sum results over the
 *     reference's own generated inputs, hashed with FNV-1a (src/gate/upconv_common.h:246-307,
 *     src/gate/gate_common.h:14-63, src/gate/upconv_cmp.c:45-59, src/gate/fma_ref.c:50-66).
 *
 * Parity pin: tests/golden/ holds the reference's own golden hashes and y vectors produced by the
 * reference's host model compiled from its sources (oracle/Makefile, tests/golden/make_golden.py);
 * tests check this restatement against them bit for bit. */
#ifndef Q8_ORACLE_H
#define Q8_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- formats */
float q8o_half(uint16_t h);                 /* exact binary16 -> binary32 */
uint16_t q8o_to_half(float f);              /* binary32 -> binary16, round to nearest even */
long q8o_gguf_bytes(long rows, long cols);  /* rows * cols/32 * 34 */
long q8o_split_bytes(long rows, long cols); /* the row-split layout: per row, quants then padded scales */
long q8o_split_row_bytes(long cols);
long q8o_split_scale_stride(long cols);     /* scale entries per row: cols/32 rounded up to 8 */
/* GGUF Q8_0 rows -> the split layout (host restatement of the device repack) */
void q8o_repack_split(const uint8_t *q8, long rows, long cols, uint8_t *out);
/* the split layout -> GGUF Q8_0 rows */
void q8o_unpack_split(const uint8_t *split, long rows, long cols, uint8_t *q8);

/* ---- the seeded synthetic inputs (counter based: any element reproducible alone) */
float q8o_normal(uint64_t seed, uint64_t stream, uint64_t index);
void q8o_fill_f32(float *out, long n, uint64_t seed, uint64_t stream, float sigma);
/* rows [row0, row0+rows) of a Q8_0 matrix with cols columns, w ~ sigma * N(0,1), quantised as
 * d = max|w|/127 (stored fp16), q = round(w/d) clamped to [-127,127]; GGUF layout */
void q8o_fill_q8_0(uint8_t *out, long row0, long rows, long cols, uint64_t seed, uint64_t stream, float sigma);

/* ---- the products, in the reference's rounding order (see the header comment) */
void q8o_gemv(const uint8_t *q8, long rows, long cols, const float *x, float *y, int threads);
void q8o_gemm(const uint8_t *q8, long rows, long cols, const float *x, long t, float *y, int threads);
/* row-gathered gemv: y[i] = row idx[i] of W times x */
void q8o_gemv_rows(const uint8_t *q8, long cols, const int32_t *idx, long n, const float *x, float *y, int threads);
/* F64: exact dequant, double dot product, y in double */
void q8o_gemm_f64(const uint8_t *q8, long rows, long cols, const float *x, long t, double *y, int threads);

/* ---- the reference's gate known answers, recomputed here: hashes in the golden file's order
 * s8 u8fma u8mul b16 bcast f16 hsum (gate 2.1), then gate A's hash and words c0 c1 clast */
void q8o_gate21_hashes(uint64_t out[7]);
void q8o_gate_a(uint64_t *hash, uint32_t words[3]);

/* ---- the host-half primitives beside the products (prims_oracle.c; src/host/rt_host.c:128-279),
 * in the reference's rounding order. l: h entries, the kv head of each query head. c % 8 == 0. */
void q8o_ip21_kv(float *z, const float *kv, long n1, long c, const long *l, long h, long t, const float *b);
void q8o_ip12_kv(float *z, const float *a, const float *kv, long n1, long c, const long *l, long h, long t);
void q8o_ip21(float *z, const float *a, long h, long r, long c, const float *b);
void q8o_scale_outer(float *z, const float *s, float g, const float *a, const float *b, long m, long k);

#ifdef __cplusplus
}
#endif
#endif
